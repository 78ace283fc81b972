"""The fp32 torch restatement (the timed CPU baseline) against the double-precision C oracle."""
import math

import numpy as np
import pytest
import torch

from aegaeon_b200 import synth
from oracle import oracle as orc
from oracle.torch_ref import DecodeLayerCPU

DT = {torch.float16: orc.FP16, torch.bfloat16: orc.BF16}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("dtype,Hq,Hkv", [(torch.float16, 28, 4), (torch.bfloat16, 32, 4), (torch.float16, 8, 8)])
def test_decode_layer_cpu_matches_oracle(dtype, Hq, Hkv):
    cfg = synth.CONFIGS["cfg1"]
    lay = synth.make_layout(cfg)
    seq = lay.seq_lens.copy()
    seq[1] = 0  # an empty sequence gets zero rows
    B, D, L, N = len(seq), 128, 2, lay.num_blocks
    g = torch.Generator().manual_seed(5)
    cache = torch.randn((N, L, 2, 16, Hkv, D), generator=g).to(dtype)
    q = torch.randn((B, Hq, D), generator=g).to(dtype)
    k_new = torch.randn((B, Hkv, D), generator=g).to(dtype)
    v_new = torch.randn((B, Hkv, D), generator=g).to(dtype)
    pos = np.maximum(seq.astype(np.int64) - 1, 0)
    slots = lay.block_tables[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    slots[seq == 0] = -1
    scale = 1.0 / math.sqrt(D)
    layer = 1

    want_cache = _bits(cache).copy()
    flat = want_cache.reshape(-1)
    half = 16 * Hkv * D
    bs = L * 2 * half
    kb = flat[layer * 2 * half:]
    orc.c_reshape_and_cache(_bits(k_new), _bits(v_new), kb, kb[half:], bs, N, slots)
    want = orc.c_paged_attention(_bits(q), kb, kb[half:], bs, lay.block_tables, seq, Hkv, scale, DT[dtype])

    out = torch.empty_like(q)
    DecodeLayerCPU(lay.block_tables, seq, scale).run(q, cache[:, layer, 0], cache[:, layer, 1], k_new, v_new,
                                                     torch.as_tensor(slots), out)
    assert np.array_equal(_bits(cache), want_cache)  # the cache write is bit-exact
    ok, err, excess = orc.compare_attention(_bits(out), want, DT[dtype])
    assert ok, f"max |err| {err:.3e}, excess {excess:.3e}"
    assert not _bits(out)[1].any()

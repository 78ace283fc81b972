"""Shared helpers of the GPU parity tests: seeded decode inputs and oracle checks on compact copies."""
from __future__ import annotations

import numpy as np
import torch

from aegaeon_b200 import synth
from aegaeon_b200.layout import BLOCK_SIZE
from oracle import oracle as orc

ATOL, RTOL = 2e-3, 1e-2  # fp16/bf16 attention tolerance against the double-precision oracle

DT = {torch.float16: orc.FP16, torch.bfloat16: orc.BF16}


def make_tables(seq_lens, num_blocks, seed, width=None):
    rng = np.random.default_rng(seed)
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    nb = (seq_lens.astype(np.int64) + BLOCK_SIZE - 1) // BLOCK_SIZE
    W = int(width or max(1, nb.max()))
    perm = rng.permutation(num_blocks)
    assert nb.sum() <= num_blocks
    tables = np.zeros((len(seq_lens), W), np.int32)
    off = 0
    for i, n in enumerate(nb):
        tables[i, :n] = perm[off:off + n]
        off += n
    return tables


def oracle_attention_layer(q: torch.Tensor, k_view: torch.Tensor, v_view: torch.Tensor, tables: np.ndarray,
                           seq_lens: np.ndarray, scale: float, threads: int = 0) -> np.ndarray:
    """Runs the C oracle on a compact host copy of the blocks the batch uses.

    ``k_view``/``v_view`` are the (N, 16, Hkv, D) device views of one layer.
    """
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    nb = (np.clip(seq_lens, 0, None).astype(np.int64) + BLOCK_SIZE - 1) // BLOCK_SIZE
    used = np.concatenate([tables[i, :nb[i]] for i in range(len(nb))]) if nb.sum() else np.zeros(0, np.int64)
    uniq, inv = np.unique(used, return_inverse=True)
    compact = np.zeros_like(tables)
    off = 0
    for i, n in enumerate(nb):
        compact[i, :n] = inv[off:off + n]
        off += n
    idx = torch.as_tensor(uniq.astype(np.int64), device=k_view.device)
    if len(uniq):
        kc = k_view.index_select(0, idx).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        vc = v_view.index_select(0, idx).contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    else:
        shape = (1,) + tuple(k_view.shape[1:])
        kc = np.zeros(shape, np.uint16)
        vc = np.zeros(shape, np.uint16)
    Hkv, D = k_view.shape[2], k_view.shape[3]
    qh = q.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return orc.c_paged_attention(qh, kc.reshape(-1), vc.reshape(-1), 16 * Hkv * D, compact, seq_lens, Hkv, scale,
                                 DT[q.dtype], threads)


def assert_attention_close(out: torch.Tensor, want_bits: np.ndarray, what: str = ""):
    got = out.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    ok, max_err, excess = orc.compare_attention(got, want_bits, DT[out.dtype], ATOL, RTOL)
    assert ok, f"{what}: max |err| {max_err:.3e}, worst excess over atol+rtol*|ref| {excess:.3e}"
    return max_err


def decode_case(B, Hq, Hkv, seq_lens, dtype, num_layers=2, extra_blocks=8, seed=0, std=1.0, width=None,
                device="cuda"):
    """A random (N, L, 2, 16, Hkv, D) cache, tables and q for an explicit list of seq_lens."""
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    nb = int(((seq_lens.astype(np.int64) + 15) // 16).sum())
    N = nb + extra_blocks
    tables = make_tables(seq_lens, N, seed, width)
    g = torch.Generator(device=device).manual_seed(seed)
    kv = torch.randn((N, num_layers, 2, 16, Hkv, 128), generator=g, device=device, dtype=torch.float32).mul_(std)
    kv = kv.to(dtype)
    q = (torch.randn((B, Hq, 128), generator=g, device=device) * std).to(dtype)
    return kv, q, tables, seq_lens

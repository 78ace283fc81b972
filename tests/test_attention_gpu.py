"""Paged decode attention on the GPU against the CPU oracle (tolerance atol 2e-3 / rtol 1e-2)."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import ops, synth
from aegaeon_b200._native import (AEG_DEVERR_BLOCK_ID_RANGE, AEG_DEVERR_SEQ_LEN_RANGE)
from tests.gpu_helpers import assert_attention_close, decode_case, oracle_attention_layer

pytestmark = pytest.mark.gpu

SCALE = 1.0 / np.sqrt(128)


def _run(kv, q, tables, seq_lens, layer=0, plan=None):
    dev = q.device
    t = torch.as_tensor(tables, device=dev)
    s = torch.as_tensor(seq_lens, device=dev)
    out = torch.full_like(q, float("nan"))
    ops.paged_attention_decode(out, q, kv, layer, t, s, SCALE, plan=plan)
    return out


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (32, 4), (40, 40), (8, 8), (6, 2), (16, 1), (7, 1), (12, 4)])
def test_attention_shapes(cuda_device, dtype, Hq, Hkv):
    seq_lens = [1, 15, 16, 17, 33, 250, 700, 5]
    B = len(seq_lens)
    kv, q, tables, sl = decode_case(B, Hq, Hkv, seq_lens, dtype, seed=Hq + Hkv)
    for layer in (0, 1):
        out = _run(kv, q, tables, sl, layer)
        want = oracle_attention_layer(q, kv[:, layer, 0], kv[:, layer, 1], tables, sl, SCALE)
        assert_attention_close(out, want, f"Hq={Hq} Hkv={Hkv} {dtype} layer {layer}")


def test_cfg1_matches_oracle(cuda_device):
    cfg = synth.CONFIGS["cfg1"]
    lay = synth.make_layout(cfg)
    gen = torch.Generator().manual_seed(cfg.seed + 1)
    kv = torch.randn((lay.num_blocks, 1, 2, 16, cfg.num_kv_heads, 128), generator=gen).to(cfg.dtype).to(cuda_device)
    q = torch.randn((cfg.batch, cfg.num_q_heads, 128), generator=gen).to(cfg.dtype).to(cuda_device)
    out = _run(kv, q, lay.block_tables, lay.seq_lens)
    want = oracle_attention_layer(q, kv[:, 0, 0], kv[:, 0, 1], lay.block_tables, lay.seq_lens, SCALE)
    assert_attention_close(out, want, "cfg1")


def test_long_and_short_sequences_split_and_merge(cuda_device):
    # One 6000-token sequence among short ones forces multi-unit splits and the in-kernel merge.
    seq_lens = [6000, 3, 40, 1, 1024, 2047, 2048, 2049]
    kv, q, tables, sl = decode_case(len(seq_lens), 28, 4, seq_lens, torch.float16, num_layers=1, seed=11)
    plan = ops.DecodePlan(len(seq_lens), 28, 4, 128, cuda_device)
    plan.plan(torch.as_tensor(sl, device=cuda_device), tables.shape[1])
    out = _run(kv, q, tables, sl, plan=plan)
    want = oracle_attention_layer(q, kv[:, 0, 0], kv[:, 0, 1], tables, sl, SCALE)
    assert_attention_close(out, want, "split")
    # plan invariants: every (sequence, group) block range is covered exactly once
    ws = plan.workspace
    hdr = ws[:256].view(torch.int32).cpu()
    n_units = int(hdr[0])
    assert n_units >= len(seq_lens)
    # reuse of the same plan on a second layer call gives identical bits (counters self-reset)
    out2 = _run(kv, q, tables, sl, plan=plan)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))


def test_zero_length_sequence_gives_zero_row(cuda_device):
    seq_lens = [0, 20, 0, 1]
    kv, q, tables, sl = decode_case(4, 28, 4, seq_lens, torch.bfloat16, num_layers=1, seed=5, width=4)
    out = _run(kv, q, tables, sl)
    assert torch.all(out[0] == 0) and torch.all(out[2] == 0)
    want = oracle_attention_layer(q, kv[:, 0, 0], kv[:, 0, 1], tables, sl, SCALE)
    assert_attention_close(out, want, "zero-length")


def test_strided_query_and_vllm_layout(cuda_device):
    # q and out as views into wider [B, (Hq + 2 Hkv) * D] rows; caches in vLLM's (2, N, 16, Hkv, D) layout.
    B, Hq, Hkv = 6, 28, 4
    seq_lens = [100, 1, 300, 17, 64, 999]
    _, _, tables, sl = decode_case(B, Hq, Hkv, seq_lens, torch.float16, num_layers=1, seed=3)
    N = int(tables.max()) + 1
    g = torch.Generator(device=cuda_device).manual_seed(9)
    caches = torch.randn((2, N, 16, Hkv, 128), generator=g, device=cuda_device).half()
    qkv = torch.randn((B, (Hq + 2 * Hkv) * 128), generator=g, device=cuda_device).half()
    q = qkv[:, : Hq * 128].view(B, Hq, 128)
    assert q.stride(0) == (Hq + 2 * Hkv) * 128
    big_out = torch.zeros((B, (Hq + 8) * 128), device=cuda_device, dtype=torch.float16)
    out = big_out[:, : Hq * 128].view(B, Hq, 128)
    ops.flash_attn_decode(q, caches[0], caches[1], torch.as_tensor(tables, device=cuda_device),
                          torch.as_tensor(sl, device=cuda_device), SCALE, out=out)
    want = oracle_attention_layer(q, caches[0], caches[1], tables, sl, SCALE)
    assert_attention_close(out, want, "strided/vLLM layout")
    assert torch.all(big_out[:, Hq * 128:] == 0)  # nothing written past the heads


def test_deterministic(cuda_device):
    seq_lens = list(np.random.default_rng(0).integers(1, 3000, size=48))
    kv, q, tables, sl = decode_case(48, 32, 4, seq_lens, torch.bfloat16, num_layers=1, seed=21)
    a = _run(kv, q, tables, sl)
    b = _run(kv, q, tables, sl)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_bad_block_id_and_seq_len_are_reported_not_faulted(cuda_device):
    ops.read_device_errors(cuda_device)
    seq_lens = [40, 20]
    kv, q, tables, sl = decode_case(2, 28, 4, seq_lens, torch.float16, num_layers=1, seed=1, width=3)
    tables = tables.copy()
    tables[0, 1] = kv.size(0) + 1000  # out of range: TMA fills zeros, flag raised
    out = _run(kv, q, tables, sl)
    flags = ops.read_device_errors(cuda_device)
    assert flags & AEG_DEVERR_BLOCK_ID_RANGE
    assert torch.isfinite(out.float()).all()
    # a seq_len longer than the table is clamped and reported
    sl2 = np.array([40, 20 * 16], np.int32)
    tables2 = tables.copy()
    tables2[0, 1] = 0
    _run(kv, q, tables2, sl2)
    assert ops.read_device_errors(cuda_device) & AEG_DEVERR_SEQ_LEN_RANGE
    assert ops.read_device_errors(cuda_device) == 0  # cleared by the read


@pytest.mark.parametrize("name,layers", [("cfg2", (0, 27)), ("cfg3", (47,)), ("cfg4", (0,))])
def test_full_size_configs_one_layer(cuda_device, name, layers):
    cfg = synth.CONFIGS[name]
    lay = synth.make_layout(cfg)
    shape = (lay.num_blocks, cfg.num_layers, 2, 16, cfg.num_kv_heads, 128)
    kv = torch.empty(shape, dtype=cfg.dtype, device=cuda_device)
    synth.fill_normal_(kv, cfg.value_std, cfg.seed)
    g = torch.Generator(device=cuda_device).manual_seed(cfg.seed + 7)
    q = (torch.randn((cfg.batch, cfg.num_q_heads, 128), generator=g, device=cuda_device) * cfg.value_std).to(cfg.dtype)
    plan = ops.DecodePlan(cfg.batch, cfg.num_q_heads, cfg.num_kv_heads, 128, cuda_device)
    plan.plan(torch.as_tensor(lay.seq_lens, device=cuda_device), lay.width)
    for layer in layers:
        out = _run(kv, q, lay.block_tables, lay.seq_lens, layer, plan=plan)
        want = oracle_attention_layer(q, kv[:, layer, 0], kv[:, layer, 1], lay.block_tables, lay.seq_lens, SCALE)
        assert_attention_close(out, want, f"{name} layer {layer}")
    del kv
    torch.cuda.empty_cache()

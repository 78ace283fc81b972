"""Paged decode attention on the GPU against the CPU oracle (tolerance atol 2e-3 / rtol 1e-2)."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import ops, synth
from aegaeon_b200._native import (AEG_DEVERR_BLOCK_ID_RANGE, AEG_DEVERR_SEQ_LEN_RANGE, AEG_DEVERR_WAIT_TIMEOUT)
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
    t_dev = torch.as_tensor(tables, device=cuda_device)
    s_dev = torch.as_tensor(sl, device=cuda_device)
    plan.plan(s_dev, t_dev)
    out = torch.full_like(q, float("nan"))
    ops.paged_attention_decode(out, q, kv, 0, t_dev, s_dev, SCALE, plan=plan)
    want = oracle_attention_layer(q, kv[:, 0, 0], kv[:, 0, 1], tables, sl, SCALE)
    assert_attention_close(out, want, "split")
    # the plan produced at least one unit per (sequence, KV head)
    ws = plan.workspace
    hdr = ws[:256].view(torch.int32).cpu()
    n_units = int(hdr[0])
    assert n_units >= len(seq_lens) * 4
    # reuse of the same plan on a second layer call gives identical bits (counters self-reset)
    out2 = torch.full_like(q, float("nan"))
    ops.paged_attention_decode(out2, q, kv, 0, t_dev, s_dev, SCALE, plan=plan)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_very_large_batch_of_short_sequences(cuda_device, dtype):
    """5000 sequences of 0..40 tokens (more than the plan keeps block counts for in shared
    memory, and more (sequence, head) pairs than worker warps): within tolerance of the oracle,
    zero rows for empty sequences, no device error."""
    rng = np.random.default_rng(21)
    seq_lens = rng.integers(0, 41, size=5000)
    kv, q, tables, sl = decode_case(len(seq_lens), 8, 1, seq_lens, dtype, num_layers=1, seed=21)
    ops.read_device_errors(cuda_device)
    out = _run(kv, q, tables, sl)
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) == 0
    assert torch.all(out[torch.as_tensor(sl == 0, device=cuda_device)] == 0)
    want = oracle_attention_layer(q, kv[:, 0, 0], kv[:, 0, 1], tables, sl, SCALE)
    assert_attention_close(out, want, "5000 short sequences")


def _first_warp_flag_offset(B: int, Hkv: int) -> int:
    """Byte offset of worker warp 0's publication flag in a DecodePlan workspace: a 256-byte
    header, then the warp records (three 16-byte records for each of the 4096 worker warps the
    workspace is sized for, plus one) and the split-pair entries (16 bytes per (sequence, KV
    head) pair), each region rounded up to 256 bytes."""
    def up(x):
        return (x + 255) & ~255
    return up(up(256 + 3 * 16 * (4096 + 1)) + 16 * B * Hkv)


def test_merge_wait_runs_out_and_reports(cuda_device):
    """Failure detection without a fault: worker warp 0's publication flag is set to a value that
    no launch stamps, as if that warp had never published its pieces, so the merges that need
    them wait until their bounded wait (2 s) runs out. The launch reports
    AEG_DEVERR_WAIT_TIMEOUT and returns, the context stays usable, and the next plan and launch
    give the right output."""
    import time

    seq_lens = [3000, 40, 700, 5]  # the first pair spans many worker warps, warp 0 among them
    B, Hq, Hkv = len(seq_lens), 28, 4
    kv, q, tables, sl = decode_case(B, Hq, Hkv, seq_lens, torch.float16, num_layers=1, seed=13)
    t_dev = torch.as_tensor(tables, device=cuda_device)
    s_dev = torch.as_tensor(sl, device=cuda_device)
    want = oracle_attention_layer(q, kv[:, 0, 0], kv[:, 0, 1], tables, sl, SCALE)
    plan = ops.DecodePlan(B, Hq, Hkv, 128, cuda_device).plan(s_dev, t_dev)
    ops.read_device_errors(cuda_device)
    out = torch.full_like(q, float("nan"))
    ops.paged_attention_decode(out, q, kv, 0, t_dev, s_dev, SCALE, plan=plan)  # every flag now holds 1
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) == 0
    assert_attention_close(out, want, "before")
    off = _first_warp_flag_offset(B, Hkv)
    flag = plan.workspace[off:off + 4].view(torch.int32)
    assert int(flag.item()) == 1  # the offset holds a publication flag after one launch
    flag.fill_(7)
    t0 = time.perf_counter()
    ops.paged_attention_decode(torch.empty_like(q), q, kv, 0, t_dev, s_dev, SCALE, plan=plan)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert ops.read_device_errors(cuda_device) & AEG_DEVERR_WAIT_TIMEOUT
    assert 1.5 < waited < 20, waited
    plan.plan(s_dev, t_dev)  # a new plan starts every flag at zero again
    out = torch.full_like(q, float("nan"))
    ops.paged_attention_decode(out, q, kv, 0, t_dev, s_dev, SCALE, plan=plan)
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) == 0
    assert_attention_close(out, want, "after")


@pytest.mark.parametrize("seq_lens", [[0, 20, 0, 1], [0, 0, 0]])
def test_zero_length_sequence_gives_zero_row(cuda_device, seq_lens):
    """Empty sequences give zero rows, also when the whole batch is empty (a plan of no blocks)."""
    kv, q, tables, sl = decode_case(len(seq_lens), 28, 4, seq_lens, torch.bfloat16, num_layers=1, seed=5, width=4)
    ops.read_device_errors(cuda_device)
    out = _run(kv, q, tables, sl)
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) == 0
    assert torch.all(out[torch.as_tensor(sl == 0, device=cuda_device)] == 0)
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
    t_dev = torch.as_tensor(lay.block_tables, device=cuda_device)
    s_dev = torch.as_tensor(lay.seq_lens, device=cuda_device)
    plan.plan(s_dev, t_dev)
    for layer in layers:
        out = torch.full_like(q, float("nan"))
        ops.paged_attention_decode(out, q, kv, layer, t_dev, s_dev, SCALE, plan=plan)
        want = oracle_attention_layer(q, kv[:, layer, 0], kv[:, layer, 1], lay.block_tables, lay.seq_lens, SCALE)
        assert_attention_close(out, want, f"{name} layer {layer}")
    del kv
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (40, 40), (16, 1)])
def test_fused_decode_layer_equals_write_then_attend(cuda_device, dtype, Hq, Hkv):
    # decode_layer == reshape_and_cache at the decode slot followed by paged_attention_decode:
    # identical cache bits and identical output bits.
    seq_lens = [1, 15, 16, 17, 300, 2500, 64, 33]
    B = len(seq_lens)
    kv, q, tables, sl = decode_case(B, Hq, Hkv, seq_lens, dtype, num_layers=2, seed=Hq * 3 + Hkv)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    k_new = torch.randn((B, Hkv, 128), generator=g, device=cuda_device).to(dtype)
    v_new = torch.randn((B, Hkv, 128), generator=g, device=cuda_device).to(dtype)
    t = torch.as_tensor(tables, device=cuda_device)
    s = torch.as_tensor(sl, device=cuda_device)
    pos = sl.astype(np.int64) - 1
    slots = torch.as_tensor(tables[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16, device=cuda_device)
    kv_a, kv_b = kv.clone(), kv.clone()
    layer = 1
    out_a = torch.full_like(q, float("nan"))
    out_b = torch.full_like(q, float("nan"))
    ops.reshape_and_cache(k_new, v_new, kv_a, layer, slots)
    ops.paged_attention_decode(out_a, q, kv_a, layer, t, s, SCALE)
    ops.decode_layer(out_b, q, k_new, v_new, kv_b, layer, t, s, SCALE)
    assert torch.equal(kv_a.view(torch.int16), kv_b.view(torch.int16))
    assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16))
    want = oracle_attention_layer(q, kv_a[:, layer, 0], kv_a[:, layer, 1], tables, sl, SCALE)
    assert_attention_close(out_b, want, f"fused Hq={Hq} Hkv={Hkv} {dtype}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (16, 1)])
def test_attention_after_decode_write_requests_tiles_early(cuda_device, dtype, Hq, Hkv):
    # reshape_and_cache at the decode slots, then paged_attention_decode launched right behind it
    # with after_decode_write=True: the attention requests its first tiles before the write has
    # finished and reads each sequence's newest row again afterwards. Two rounds with different
    # new rows, each equal bit for bit to the fused layer on a separate copy of the cache.
    seq_lens = [1, 15, 16, 17, 300, 2500, 64, 33, 4000, 2]
    B = len(seq_lens)
    kv, q, tables, sl = decode_case(B, Hq, Hkv, seq_lens, dtype, num_layers=2, seed=Hq * 7 + Hkv)
    t = torch.as_tensor(tables, device=cuda_device)
    s = torch.as_tensor(sl, device=cuda_device)
    pos = sl.astype(np.int64) - 1
    slots = torch.as_tensor(tables[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16, device=cuda_device)
    layer = 1
    kv_c = kv.clone()
    plan = ops.DecodePlan(B, Hq, Hkv, 128, cuda_device).plan(s, t)
    ops.paged_attention_decode(torch.empty_like(q), q, kv_c, 0, t, s, SCALE, plan=plan)  # the plan is now complete
    g = torch.Generator(device=cuda_device).manual_seed(9)
    for rnd in range(2):
        k_new = torch.randn((B, Hkv, 128), generator=g, device=cuda_device).to(dtype)
        v_new = torch.randn((B, Hkv, 128), generator=g, device=cuda_device).to(dtype)
        out_c = torch.full_like(q, float("nan"))
        ops.reshape_and_cache(k_new, v_new, kv_c, layer, slots)
        ops.paged_attention_decode(out_c, q, kv_c, layer, t, s, SCALE, plan=plan, after_decode_write=True)
        kv_b = kv.clone()
        out_b = torch.full_like(q, float("nan"))
        ops.decode_layer(out_b, q, k_new, v_new, kv_b, layer, t, s, SCALE)
        torch.cuda.synchronize()
        assert torch.equal(kv_c[:, layer].view(torch.int16), kv_b[:, layer].view(torch.int16))
        assert torch.equal(out_c.view(torch.int16), out_b.view(torch.int16)), f"round {rnd}"
    assert ops.read_device_errors() == 0


@pytest.mark.parametrize("name", ["vllm_cfg1_fp16.npz", "vllm_gqa8_bf16.npz"])
def test_matches_vllm_golden_vectors(cuda_device, name):
    # Same inputs as vLLM's kernels in tests/golden/make_golden.py: the cache write of the
    # reshape operator equals vLLM's bit for bit (padding slot skipped), and the decode output
    # is within the attention tolerance of vLLM's.
    import hashlib
    import os

    from oracle import oracle as orc

    g = dict(np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", name)))
    dt = torch.bfloat16 if str(g["dtype"]) == "bf16" else torch.float16
    to = lambda a: torch.from_numpy(a.view(np.int16)).to(cuda_device).view(dt)
    kv = to(g["cache_before"])
    q, k_new, v_new = to(g["q"]), to(g["k_new"]), to(g["v_new"])
    t = torch.as_tensor(g["tables"], device=cuda_device)
    s = torch.as_tensor(g["seq_lens"], device=cuda_device)
    layer = int(g["layer"])
    ops.reshape_and_cache(k_new, v_new, kv, layer, torch.as_tensor(g["slot_mapping"], device=cuda_device))
    after = kv.view(torch.int16).cpu().numpy().view(np.uint16)
    assert hashlib.sha256(after.tobytes()).hexdigest() == str(g["cache_after_sha256"])
    out = torch.empty_like(q)
    ops.paged_attention_decode(out, q, kv, layer, t, s, float(g["scale"]))
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    ok, err, excess = orc.compare_attention(got, g["out_vllm"], orc.BF16 if dt == torch.bfloat16 else orc.FP16)
    assert ok, (err, excess)


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_plan_stats_describe_the_batch(cuda_device, name):
    """DecodePlan.stats() reads back what the plan built; its counts follow from the batch: one
    position per (sequence, head) block plus the start cost of every non-empty pair, at least one
    unit per non-empty pair, one more per warp start inside a pair, and two partial slots per
    such cut at most."""
    cfg = synth.CONFIGS[name]
    lay = synth.make_layout(cfg)
    plan = ops.DecodePlan(cfg.batch, cfg.num_q_heads, cfg.num_kv_heads, 128, cuda_device)
    plan.plan(torch.as_tensor(lay.seq_lens, device=cuda_device), torch.as_tensor(lay.block_tables, device=cuda_device))
    st = plan.stats()
    nb = (np.asarray(lay.seq_lens, dtype=np.int64) + 15) // 16
    nonempty = int((nb > 0).sum()) * cfg.num_kv_heads
    assert st["items"] == int(nb.sum()) * cfg.num_kv_heads + 2 * nonempty
    assert nonempty <= st["units"] <= nonempty + st["workers"]
    assert st["workers"] % 8 == 0 and st["workers"] > 0
    assert 0 <= st["partial_slots"] <= 2 * st["workers"]
    assert st["split_pair_entries"] <= cfg.batch * cfg.num_kv_heads
    assert st["merge_items"] >= st["split_pair_entries"] - (cfg.batch * cfg.num_kv_heads - nonempty)

"""Prefill (prompt) attention on the GPU (``ops.flash_attn_varlen_prefill``): against the fp64
oracle (atol 2e-3 / rtol 1e-2, the attention tolerance of this path) on small varlen batches, and
against torch fp32 scaled-dot-product attention per prompt on larger ones. Also the prompt half
of the cache write: reshape_and_cache over a batch of prompts' tokens, bit-exact."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from aegaeon_b200 import ops
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

DT = {torch.float16: orc.FP16, torch.bfloat16: orc.BF16}


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _inputs(dev, lens, Hq, Hkv, dtype, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    T = int(sum(lens))
    q = torch.randn((T, Hq, 128), generator=g, device=dev).to(dtype)
    k = torch.randn((T, Hkv, 128), generator=g, device=dev).to(dtype)
    v = torch.randn((T, Hkv, 128), generator=g, device=dev).to(dtype)
    cu = torch.as_tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=dev)
    return q, k, v, cu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (8, 8), (16, 4), (12, 4)])
def test_prefill_matches_oracle(cuda_device, dtype, Hq, Hkv):
    lens = [1, 17, 64, 65, 0, 130]
    q, k, v, cu = _inputs(cuda_device, lens, Hq, Hkv, dtype, 3)
    scale = 128 ** -0.5
    out = ops.flash_attn_varlen_prefill(q, k, v, cu, max(lens), scale)
    torch.cuda.synchronize()
    want = orc.np_prefill_attention(_bits(q), _bits(k), _bits(v), cu.cpu().numpy(), scale, DT[dtype])
    ok, err, excess = orc.compare_attention(_bits(out), want, DT[dtype])
    assert ok, (err, excess)
    assert ops.read_device_errors(cuda_device) == 0


@pytest.mark.parametrize("dtype,lens", [(torch.float16, [2048, 777, 1, 1500]), (torch.bfloat16, [2048, 777, 1, 1500]),
                                        (torch.bfloat16, [8192, 5])])
def test_prefill_long_prompts_match_torch_fp32(cuda_device, dtype, lens):
    """Larger batches against torch fp32 SDPA per prompt, up to the longest prompt of the
    workload's range (8192 tokens, 64 key tiles per query tile)."""
    Hq, Hkv = 28, 4
    q, k, v, cu = _inputs(cuda_device, lens, Hq, Hkv, dtype, 5)
    scale = 128 ** -0.5
    out = ops.flash_attn_varlen_prefill(q, k, v, cu, max(lens), scale)
    torch.cuda.synchronize()
    c = cu.cpu().tolist()
    for b in range(len(lens)):
        s0, s1 = c[b], c[b + 1]
        qq = q[s0:s1].float().transpose(0, 1)                                      # [Hq, L, D]
        kk = k[s0:s1].float().transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)
        vv = v[s0:s1].float().transpose(0, 1).repeat_interleave(Hq // Hkv, dim=0)
        ref = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, scale=scale).transpose(0, 1)
        got = out[s0:s1].float()
        tol = 2e-3 + 1e-2 * ref.abs()
        assert bool(((got - ref).abs() <= tol).all()), (b, float((got - ref).abs().max()))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_many_tiny_prompts_match_oracle(cuda_device, dtype):
    """600 prompts of 0..3 tokens and one of 300 (many (level, prompt) groups, most of them a
    single partly filled query tile, and empty prompts the work counter skips)."""
    rng = np.random.default_rng(17)
    lens = rng.integers(0, 4, size=600).tolist() + [300]
    Hq, Hkv = 8, 2
    q, k, v, cu = _inputs(cuda_device, lens, Hq, Hkv, dtype, 19)
    scale = 128 ** -0.5
    ops.read_device_errors(cuda_device)
    out = ops.flash_attn_varlen_prefill(q, k, v, cu, max(lens), scale)
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) == 0
    want = orc.np_prefill_attention(_bits(q), _bits(k), _bits(v), cu.cpu().numpy(), scale, DT[dtype])
    ok, err, excess = orc.compare_attention(_bits(out), want, DT[dtype])
    assert ok, (err, excess)


def test_prefill_work_counter_repeats_and_streams(cuda_device):
    """The kernel's CTAs take (level, prompt, head) items from a per-launch counter; the host
    rotates over 64 counter slots and each launch's last CTA resets its slot. More than 64
    launches in a row, launches on two streams at once, a batch with fewer items than SMs and a
    batch of mostly empty prompts must all give the bits of a first, solo launch."""
    scale = 128 ** -0.5
    batches = [([300, 1, 777, 64], 28, 4, torch.bfloat16), ([5], 8, 8, torch.float16),
               ([0, 0, 513, 0, 0, 0, 2], 28, 4, torch.float16)]
    runs = []
    for i, (lens, Hq, Hkv, dtype) in enumerate(batches):
        q, k, v, cu = _inputs(cuda_device, lens, Hq, Hkv, dtype, 20 + i)
        ref = ops.flash_attn_varlen_prefill(q, k, v, cu, max(lens), scale)
        runs.append((q, k, v, cu, max(lens), ref))
    torch.cuda.synchronize()
    for rep in range(70):
        q, k, v, cu, mx, ref = runs[rep % len(runs)]
        out = ops.flash_attn_varlen_prefill(q, k, v, cu, mx, scale)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), rep
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    outs = []
    for rep in range(12):
        q, k, v, cu, mx, ref = runs[rep % len(runs)]
        with torch.cuda.stream(streams[rep % 2]):
            outs.append((ops.flash_attn_varlen_prefill(q, k, v, cu, mx, scale), ref))
    torch.cuda.synchronize()
    for i, (got, ref) in enumerate(outs):
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), i
    assert ops.read_device_errors(cuda_device) == 0
    # the mostly-empty batch is still right
    q, k, v, cu, mx, ref = runs[2]
    want = orc.np_prefill_attention(_bits(q), _bits(k), _bits(v), cu.cpu().numpy(), scale, orc.FP16)
    ok, err, excess = orc.compare_attention(_bits(ref), want, orc.FP16)
    assert ok, (err, excess)


def test_prefill_rejects_out_of_range_prompts(cuda_device):
    lens = [10, 20]
    q, k, v, cu = _inputs(cuda_device, lens, 8, 8, torch.float16, 1)
    out = torch.zeros_like(q)
    bad = torch.as_tensor([0, 10, 40], dtype=torch.int32, device=cuda_device)  # prompt 1 runs past the 30 tokens
    ops.flash_attn_varlen_prefill(q, k, v, bad, 30, 128 ** -0.5, out=out)
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) & 0x4
    assert not out[10:].any()  # the bad prompt's rows were not written
    ref = ops.flash_attn_varlen_prefill(q, k, v, cu, 20, 128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(out[:10], ref[:10])


def test_prompt_cache_write_bit_exact(cuda_device):
    """reshape_and_cache of a batch of prompts (slots from the step-input restatement)."""
    rng = np.random.default_rng(9)
    lens = [300, 45, 1, 1024]
    N, L, Hkv = 128, 2, 4
    perm = rng.permutation(N)
    tables, off = [], 0
    for n in lens:
        nb = (n + 15) // 16
        tables.append(perm[off:off + nb].tolist())
        off += nb
    slots = orc.np_step_inputs(lens, [0] * len(lens), tables)["slot_mapping"]
    T = len(slots)
    kv = torch.randint(-32768, 32768, (N, L, 2, 16, Hkv, 128), dtype=torch.int32).to(torch.int16)
    key = torch.randint(-32768, 32768, (T, Hkv, 128), dtype=torch.int32).to(torch.int16)
    val = torch.randint(-32768, 32768, (T, Hkv, 128), dtype=torch.int32).to(torch.int16)
    kv_dev = kv.to(cuda_device).view(torch.bfloat16)
    ops.reshape_and_cache(key.to(cuda_device).view(torch.bfloat16), val.to(cuda_device).view(torch.bfloat16), kv_dev,
                          1, torch.as_tensor(slots, device=cuda_device))
    ref = kv.numpy().view(np.uint16).copy()
    orc.np_reshape_and_cache(key.numpy().view(np.uint16), val.numpy().view(np.uint16), ref[:, 1, 0], ref[:, 1, 1], slots)
    assert np.array_equal(_bits(kv_dev), ref)


@pytest.mark.parametrize("Hkv", [4, 40])
def test_prompt_cache_write_many_tokens(cuda_device, Hkv):
    """From 1024 tokens on the cache write runs one warp per token: bit-exact against the oracle
    with padding slots (-1) skipped and an out-of-range slot skipped and reported."""
    rng = np.random.default_rng(10 + Hkv)
    T, N, L = 2600, 256, 2
    slots = rng.permutation(N * 16)[:T].astype(np.int64)
    slots[::97] = -1
    slots[5] = N * 16 + 3  # past the pool
    kv = torch.randint(-32768, 32768, (N, L, 2, 16, Hkv, 128), dtype=torch.int32).to(torch.int16)
    key = torch.randint(-32768, 32768, (T, Hkv, 128), dtype=torch.int32).to(torch.int16)
    val = torch.randint(-32768, 32768, (T, Hkv, 128), dtype=torch.int32).to(torch.int16)
    kv_dev = kv.to(cuda_device).view(torch.float16)
    ops.read_device_errors(cuda_device)
    ops.reshape_and_cache(key.to(cuda_device).view(torch.float16), val.to(cuda_device).view(torch.float16), kv_dev,
                          0, torch.as_tensor(slots, device=cuda_device))
    torch.cuda.synchronize()
    assert ops.read_device_errors(cuda_device) & 0x2  # AEG_DEVERR_SLOT_RANGE
    ok = slots.copy()
    ok[ok >= N * 16] = -1
    ref = kv.numpy().view(np.uint16).copy()
    orc.np_reshape_and_cache(key.numpy().view(np.uint16), val.numpy().view(np.uint16), ref[:, 0, 0], ref[:, 0, 1], ok)
    assert np.array_equal(_bits(kv_dev), ref)

"""The CPU oracle itself: C restatement vs numpy restatement vs hand-computed answers."""
import math

import numpy as np
import pytest

from oracle import oracle as orc


def _rand_bits(rng, shape, dtype, std=1.0):
    x = rng.standard_normal(shape) * std
    return orc.f64_to_bits(x, dtype)


def _layout(rng, B, N, max_ctx, W=None):
    ctx = rng.integers(1, max_ctx + 1, size=B).astype(np.int32)
    nb = (ctx + 15) // 16
    W = W or int(nb.max())
    perm = rng.permutation(N)
    assert nb.sum() <= N
    tables = np.zeros((B, W), np.int32)
    off = 0
    for b in range(B):
        tables[b, : nb[b]] = perm[off: off + nb[b]]
        off += nb[b]
    return ctx, tables


@pytest.mark.parametrize("dtype", [orc.FP16, orc.BF16])
@pytest.mark.parametrize("Hq,Hkv", [(28, 4), (32, 4), (8, 8), (6, 2), (16, 1)])
def test_c_attention_matches_numpy(dtype, Hq, Hkv):
    rng = np.random.default_rng(Hq * 100 + Hkv + dtype)
    B, D, N, L = 3, 128, 40, 2
    ctx, tables = _layout(rng, B, N, 150)
    cache = _rand_bits(rng, (N, L, 2, 16, Hkv, D), dtype)
    q = _rand_bits(rng, (B, Hq, D), dtype)
    layer = 1
    kb, vb = cache[:, layer, 0], cache[:, layer, 1]
    flat = cache.reshape(-1)
    bs = L * 2 * 16 * Hkv * D
    k_base = flat[(layer * 2 + 0) * 16 * Hkv * D:]
    v_base = flat[(layer * 2 + 1) * 16 * Hkv * D:]
    got = orc.c_paged_attention(q, k_base, v_base, bs, tables, ctx, Hkv, orc.scale_for(D), dtype)
    want = orc.np_paged_attention(q, kb, vb, tables, ctx, orc.scale_for(D), dtype)
    # Both are double-precision restatements rounded once: they agree to the last bit except for
    # rare ties decided by summation order.
    g = orc.bits_to_f64(got, dtype)
    w = orc.bits_to_f64(want, dtype)
    ulp = 2.0 ** -10 if dtype == orc.FP16 else 2.0 ** -7
    assert np.all(np.abs(g - w) <= ulp * np.maximum(np.abs(w), 2.0 ** -14))
    assert (got == want).mean() > 0.999


def test_attention_hand_computed():
    # One token: the output is that token's V row. Two tokens with equal scores: the mean.
    D, Hkv, Hq = 128, 1, 2
    k = np.zeros((2, 16, Hkv, D))
    v = np.zeros((2, 16, Hkv, D))
    v[1, 0, 0, :] = np.arange(D) / 64.0
    v[1, 1, 0, :] = 1.0
    q = np.zeros((2, Hq, D))
    q[:, :, 0] = 1.0
    kb = orc.f64_to_bits(k, orc.FP16)
    vb = orc.f64_to_bits(v, orc.FP16)
    qb = orc.f64_to_bits(q, orc.FP16)
    tables = np.array([[1], [1]], np.int32)
    seq = np.array([1, 2], np.int32)
    out = orc.bits_to_f64(orc.np_paged_attention(qb, kb, vb, tables, seq, 0.1, orc.FP16), orc.FP16)
    assert np.allclose(out[0, 0], np.arange(D) / 64.0, atol=1e-3)
    assert np.allclose(out[1, 1], (np.arange(D) / 64.0 + 1.0) / 2, atol=1e-3)
    flat_k = kb.reshape(-1)
    flat_v = vb.reshape(-1)
    c = orc.bits_to_f64(orc.c_paged_attention(qb, flat_k, flat_v, 16 * Hkv * D, tables, seq, Hkv, 0.1, orc.FP16),
                        orc.FP16)
    assert np.array_equal(c, out)


def test_attention_zero_length_and_softmax_shift():
    rng = np.random.default_rng(7)
    D, Hkv, Hq, N = 128, 2, 4, 8
    kb = _rand_bits(rng, (N, 16, Hkv, D), orc.FP16)
    vb = _rand_bits(rng, (N, 16, Hkv, D), orc.FP16)
    q = _rand_bits(rng, (2, Hq, D), orc.FP16)
    tables = np.array([[3, 4], [5, 6]], np.int32)
    out = orc.c_paged_attention(q, kb.reshape(-1), vb.reshape(-1), 16 * Hkv * D, tables, np.array([0, 20], np.int32),
                                Hkv, 0.125, orc.FP16)
    assert np.all(out[0] == 0)  # empty context -> zero row
    # Large scores do not overflow (max-subtracted softmax).
    big = orc.c_paged_attention(q, kb.reshape(-1), vb.reshape(-1), 16 * Hkv * D, tables, np.array([3, 20], np.int32),
                                Hkv, 50.0, orc.FP16)
    assert np.all(np.isfinite(orc.bits_to_f64(big, orc.FP16)))


def test_reshape_and_cache_c_vs_numpy():
    rng = np.random.default_rng(1)
    N, L, Hkv, D, T = 12, 3, 4, 128, 9
    cache = rng.integers(0, 65536, size=(N, L, 2, 16, Hkv, D), dtype=np.uint16)
    ref = cache.copy()
    key = rng.integers(0, 65536, size=(T, Hkv, D), dtype=np.uint16)
    val = rng.integers(0, 65536, size=(T, Hkv, D), dtype=np.uint16)
    slots = rng.permutation(N * 16)[:T].astype(np.int64)
    slots[2] = -1  # padding slot is skipped
    layer = 2
    flat = cache.reshape(-1)
    bs = L * 2 * 16 * Hkv * D
    rc = orc.c_reshape_and_cache(key, val, flat[(layer * 2) * 16 * Hkv * D:], flat[(layer * 2 + 1) * 16 * Hkv * D:],
                                 bs, N, slots)
    assert rc == 0
    orc.np_reshape_and_cache(key, val, ref[:, layer, 0], ref[:, layer, 1], slots)
    assert np.array_equal(cache, ref)
    # untouched layers stay untouched
    assert np.array_equal(cache[:, :layer], ref[:, :layer])


def test_reshape_and_cache_out_of_range_slot_reported():
    N, Hkv, D = 2, 1, 128
    cache = np.zeros((N, 1, 2, 16, Hkv, D), np.uint16)
    key = np.ones((1, Hkv, D), np.uint16)
    flat = cache.reshape(-1)
    rc = orc.c_reshape_and_cache(key, key, flat, flat[16 * Hkv * D:], 2 * 16 * Hkv * D, N,
                                 np.array([N * 16], np.int64))
    assert rc == 1 and not cache.any()


def test_swap_and_copy_c_vs_numpy():
    rng = np.random.default_rng(2)
    bb, Nd, Nh, n = 1024, 32, 16, 10
    dev = rng.integers(0, 256, size=(Nd, bb), dtype=np.uint8)
    host = rng.integers(0, 256, size=(Nh, bb), dtype=np.uint8)
    src = rng.permutation(Nd)[:n]
    dst = rng.permutation(Nh)[:n]
    d1, h1 = dev.copy(), host.copy()
    d2, h2 = dev.copy(), host.copy()
    orc.c_swap(d1, h1, src, dst, False)
    orc.np_swap(d2, h2, src, dst, False)
    assert np.array_equal(h1, h2) and np.array_equal(d1, d2)
    back = rng.permutation(Nd)[:n]
    orc.c_swap(d1, h1, dst, back, True)
    orc.np_swap(d2, h2, dst, back, True)
    assert np.array_equal(d1, d2)
    assert np.array_equal(d1[back], dev[src])  # round trip
    p = rng.permutation(Nd)
    orc.c_copy_blocks(d1, p[:8], p[8:16])
    orc.np_copy_blocks(d2, p[:8], p[8:16])
    assert np.array_equal(d1, d2)


def test_bf16_rounding_ties_to_even():
    # 1 + 2^-8 is halfway between two bf16 values; ties go to the even mantissa.
    x = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -2.5, 0.0])
    bits = orc.f64_to_bits(x, orc.BF16)
    back = orc.bits_to_f64(bits, orc.BF16)
    assert back[0] == 1.0 and back[1] == 1.0 + 4 * 2.0 ** -8 and back[2] == -2.5 and back[3] == 0.0
    assert math.isnan(orc.bits_to_f64(orc.f64_to_bits(np.array([np.nan]), orc.BF16), orc.BF16)[0])

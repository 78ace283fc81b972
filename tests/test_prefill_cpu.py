"""Prefill attention oracle (restated from vLLM 0.5.1's prompt call flash_attn_varlen_func with
causal=True): causal visibility and the GQA head map, checked on hand-sized cases (no GPU)."""
import numpy as np

from oracle import oracle as orc


def _bits(x):
    return orc.f64_to_bits(np.asarray(x, dtype=np.float64), orc.FP16)


def test_first_token_sees_only_itself_and_heads_share_kv():
    rng = np.random.default_rng(0)
    T, Hq, Hkv, D = 5, 4, 2, 8
    q = _bits(rng.standard_normal((T, Hq, D)))
    k = _bits(rng.standard_normal((T, Hkv, D)))
    v = _bits(rng.standard_normal((T, Hkv, D)))
    out = orc.bits_to_f64(orc.np_prefill_attention(q, k, v, [0, 3, 5], 0.3, orc.FP16), orc.FP16)
    vf = orc.bits_to_f64(v, orc.FP16)
    for s0 in (0, 3):  # the first token of each prompt returns its own value row
        for h in range(Hq):
            assert np.allclose(out[s0, h], vf[s0, h // 2], atol=1e-3)


def test_matches_a_direct_loop():
    rng = np.random.default_rng(1)
    T, Hq, Hkv, D = 9, 6, 3, 16
    q, k, v = (_bits(rng.standard_normal(s)) for s in ((T, Hq, D), (T, Hkv, D), (T, Hkv, D)))
    cu = [0, 4, 4, 9]  # an empty prompt in the middle
    got = orc.bits_to_f64(orc.np_prefill_attention(q, k, v, cu, 0.25, orc.FP16), orc.FP16)
    qf, kf, vf = (orc.bits_to_f64(x, orc.FP16) for x in (q, k, v))
    for b in range(3):
        for i in range(cu[b], cu[b + 1]):
            for h in range(Hq):
                s = np.array([qf[i, h] @ kf[j, h // 2] * 0.25 for j in range(cu[b], i + 1)])
                p = np.exp(s - s.max())
                want = (p / p.sum()) @ vf[cu[b]:i + 1, h // 2]
                assert np.allclose(got[i, h], want, atol=2e-3, rtol=1e-2)

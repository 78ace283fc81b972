"""CPU oracle of the Aegaeon per-token serving path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this module, and only as the checker or as the timed CPU baseline; the product package
``aegaeon_b200`` never does.

Two independent restatements of the reference's algorithms live here:

* the C library ``oracle/liboracle.so`` (``oracle/oracle.c``; built by ``oracle/build.py``),
  wrapped by the ``c_*`` functions; attention in double precision with OpenMP;
* numpy versions (``np_*``) written directly from the same reference sources, used to check
  the C library on small cases.

Reference anchors (paths inside the reference checkout):
  swap               aegaeon/ops/swap.cu:25-60 (block bytes: swap.cu:34)
  copy_blocks        vLLM 0.5.1 copy_blocks semantics; no reference call site
                     (aegaeon/aegaeon/block_manager.py:803-804, :876-950)
  reshape_and_cache  vLLM 0.5.1 reshape_and_cache_flash, called from aegaeon/aegaeon/worker.py:517-523;
                     slot rule worker.py:628-633
  decode attention   vLLM 0.5.1 FlashAttention decode (flash_attn_with_kvcache with block_table,
                     causal, one query token); GQA head map h // (Hq / Hkv); tables/lengths from
                     worker.py:640-653; layout worker.py:388-451, config.py:256-271
  slot mapping       aegaeon/aegaeon/worker.py:596-682; padding aegaeon/aegaeon/utils.py:241-257
  step inputs        the same function: positions, offsets, decode/prompt table rows (np_step_inputs)
  prefill attention  vLLM 0.5.1 prompt call flash_attn_varlen_func(..., causal=True) (np_prefill_attention)

Parity pins: the reference ships no kernel tests or golden vectors (its tests are smoke scripts
without numeric assertions). ``swap`` is pinned against the reference's own operator compiled
from source into ``oracle/_ref`` (GPU test). Attention and reshape_and_cache are pinned against
golden vectors produced by the installed vLLM's kernels of the same family
(``tests/golden/make_golden.py``), since vLLM 0.5.1 itself is absent; so is prompt attention
(vLLM's varlen FlashAttention, causal). ``np_step_inputs`` restates the reference's per-step
Python loops; the reference's ``Worker`` cannot be imported here, so that integer restatement is
not pinned to the reference's own outputs.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

FP16, BF16 = 0, 1


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        from . import build as _build  # noqa: WPS433 (local import keeps the module light)

        path = _build.build_oracle_lib()
        L = ctypes.CDLL(path)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.orc_swap.argtypes = [vp, vp, ctypes.c_size_t, vp, vp, i64, i32]
        L.orc_copy_blocks.argtypes = [vp, ctypes.c_size_t, vp, vp, i64]
        L.orc_reshape_and_cache.argtypes = [vp, vp, i64, i64, vp, vp, i64, i64, vp, i64, i32, i32]
        L.orc_paged_attention.argtypes = [vp, i64, vp, i64, vp, vp, i64, vp, i32, vp, i32, i32, i32, i32,
                                          ctypes.c_double, i32, i32]
        for f in (L.orc_swap, L.orc_copy_blocks, L.orc_reshape_and_cache, L.orc_paged_attention):
            f.restype = i32
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _u16(a: np.ndarray) -> np.ndarray:
    if a.dtype != np.uint16:
        raise TypeError(f"expected raw 16-bit storage (uint16), got {a.dtype}")
    return a


# -------------------------------------------------------------------------------------------
# C-library restatements


def c_swap(dev_pool: np.ndarray, host_pool: np.ndarray, src, dst, is_swap_in: bool) -> None:
    """In-place: dev_pool / host_pool are uint8 [N, block_bytes] arrays."""
    src = np.ascontiguousarray(src, dtype=np.int64)
    dst = np.ascontiguousarray(dst, dtype=np.int64)
    bb = dev_pool.shape[1]
    assert host_pool.shape[1] == bb
    lib().orc_swap(_ptr(dev_pool), _ptr(host_pool), bb, _ptr(src), _ptr(dst), src.size, int(is_swap_in))


def c_copy_blocks(pool: np.ndarray, src, dst) -> None:
    src = np.ascontiguousarray(src, dtype=np.int64)
    dst = np.ascontiguousarray(dst, dtype=np.int64)
    lib().orc_copy_blocks(_ptr(pool), pool.shape[1], _ptr(src), _ptr(dst), src.size)


def c_reshape_and_cache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                        block_stride: int, num_blocks: int, slots: np.ndarray) -> int:
    """key/value uint16 [T, Hkv, D]; k_cache/v_cache flat uint16 views (base of each cache)."""
    T, Hkv, D = key.shape
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    return lib().orc_reshape_and_cache(_ptr(_u16(key)), _ptr(_u16(value)), Hkv * D, Hkv * D, _ptr(k_cache),
                                       _ptr(v_cache), block_stride, num_blocks, _ptr(slots), T, Hkv, D)


def c_paged_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, block_stride: int,
                      tables: np.ndarray, seq_lens: np.ndarray, num_kv_heads: int, scale: float, dtype: int,
                      num_threads: int = 0) -> np.ndarray:
    """q uint16 [B, Hq, D]; k_cache/v_cache uint16 flat arrays starting at block 0 of the view."""
    B, Hq, D = q.shape
    tables = np.ascontiguousarray(tables, dtype=np.int32)
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    out = np.zeros((B, Hq, D), dtype=np.uint16)
    lib().orc_paged_attention(_ptr(out), Hq * D, _ptr(_u16(np.ascontiguousarray(q))), Hq * D, _ptr(k_cache),
                              _ptr(v_cache), block_stride, _ptr(tables), tables.shape[1], _ptr(seq_lens), B, Hq,
                              num_kv_heads, D, float(scale), int(dtype), int(num_threads))
    return out


# -------------------------------------------------------------------------------------------
# numpy restatements


def bits_to_f64(a: np.ndarray, dtype: int) -> np.ndarray:
    a = np.asarray(a, dtype=np.uint16)
    if dtype == FP16:
        return a.view(np.float16).astype(np.float64)
    return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def f64_to_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    if dtype == FP16:
        return x.astype(np.float16).view(np.uint16)
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def np_swap(dev_pool: np.ndarray, host_pool: np.ndarray, src, dst, is_swap_in: bool) -> None:
    for s, d in zip(np.asarray(src), np.asarray(dst)):
        if is_swap_in:
            dev_pool[d] = host_pool[s]
        else:
            host_pool[d] = dev_pool[s]


def np_copy_blocks(pool: np.ndarray, src, dst) -> None:
    for s, d in zip(np.asarray(src), np.asarray(dst)):
        pool[d] = pool[s]


def np_reshape_and_cache(key: np.ndarray, value: np.ndarray, k_blocks: np.ndarray, v_blocks: np.ndarray,
                         slots) -> None:
    """k_blocks/v_blocks: [N, 16, Hkv, D] views (numpy strided views into the cache)."""
    n_slots = k_blocks.shape[0] * 16
    for t, s in enumerate(np.asarray(slots, dtype=np.int64)):
        if s < 0 or s >= n_slots:
            continue
        k_blocks[s // 16, s % 16] = key[t]
        v_blocks[s // 16, s % 16] = value[t]


def np_paged_attention(q: np.ndarray, k_blocks: np.ndarray, v_blocks: np.ndarray, tables: np.ndarray,
                       seq_lens: np.ndarray, scale: float, dtype: int) -> np.ndarray:
    """q uint16 [B, Hq, D]; k_blocks/v_blocks uint16 [N, 16, Hkv, D]; returns uint16 [B, Hq, D]."""
    B, Hq, D = q.shape
    Hkv = k_blocks.shape[2]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D), dtype=np.uint16)
    qf = bits_to_f64(q, dtype)
    for b in range(B):
        n = int(min(max(seq_lens[b], 0), tables.shape[1] * 16))
        if n == 0:
            continue
        pos = np.arange(n)
        blk = tables[b, pos // 16]
        kb = bits_to_f64(k_blocks[blk, pos % 16], dtype)  # [n, Hkv, D]
        vb = bits_to_f64(v_blocks[blk, pos % 16], dtype)
        for h in range(Hq):
            kvh = h // G
            s = kb[:, kvh, :] @ qf[b, h] * scale
            p = np.exp(s - s.max())
            o = (p[:, None] * vb[:, kvh, :]).sum(0) / p.sum()
            out[b, h] = f64_to_bits(o, dtype)
    return out


def np_slot_mapping(seq_lens, context_lens, tables) -> np.ndarray:
    """Slots of positions [context_len, seq_len) of every request, concatenated."""
    slots = []
    for n, c, t in zip(seq_lens, context_lens, tables):
        for i in range(c, n):
            slots.append(int(t[i // 16]) * 16 + i % 16)
    return np.asarray(slots, dtype=np.int64)


def np_prefill_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens, scale: float,
                         dtype: int) -> np.ndarray:
    """Causal prompt attention, restated from vLLM 0.5.1's prompt call
    ``flash_attn_varlen_func(q, k, v, cu, cu, max_len, max_len, softmax_scale, causal=True)``
    (Aegaeon prefills whole prompts, aegaeon/aegaeon/worker.py:603-626): query i of prompt b sees
    keys 0..i of the same prompt, query head h reads KV head h // (Hq // Hkv); double precision,
    output rounded to ``dtype``. q/k/v are 16-bit patterns [T, H, D]."""
    qf, kf, vf = (bits_to_f64(x, dtype) for x in (q, k, v))
    T, Hq, D = qf.shape
    G = Hq // kf.shape[1]
    out = np.zeros((T, Hq, D))
    for b in range(len(cu_seqlens) - 1):
        s0, s1 = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        L = s1 - s0
        if L <= 0:
            continue
        mask = np.triu(np.ones((L, L), dtype=bool), 1)
        for h in range(Hq):
            S = qf[s0:s1, h] @ kf[s0:s1, h // G].T * scale
            S[mask] = -np.inf
            S -= S.max(axis=1, keepdims=True)
            P = np.exp(S)
            P /= P.sum(axis=1, keepdims=True)
            out[s0:s1, h] = P @ vf[s0:s1, h // G]
    return f64_to_bits(out, dtype)


def np_step_inputs(seq_lens, context_lens, tables) -> dict:
    """Per-step model inputs of a batch, restated from Worker._prepare_model_inputs
    (aegaeon/aegaeon/worker.py:596-682; padding utils.py:241-257).

    ``tables[i]`` is request i's block list. Per request (worker.py:596-633): a decode request
    (context_len > 0) keeps its block list as its table row, a prompt gets an empty row;
    positions context_len .. seq_len - 1 and their slots table[p // 16] * 16 + p % 16 are
    appended in request order. Rows are zero-padded to the longest (worker.py:640-646); query
    and sequence start offsets are int32 cumulative sums with a leading 0 (worker.py:653-676).
    """
    rows, positions, slots, query_lens = [], [], [], []
    for n, c, t in zip(seq_lens, context_lens, tables):
        rows.append(list(t) if c > 0 else [])
        query_lens.append(n - c)
        for p in range(c, n):
            positions.append(p)
            slots.append(int(t[p // 16]) * 16 + p % 16)
    width = max((len(r) for r in rows), default=0)
    padded = np.zeros((len(rows), width), dtype=np.int32)
    for i, r in enumerate(rows):
        padded[i, :len(r)] = r
    q = np.asarray(query_lens, dtype=np.int64)
    n = np.asarray(seq_lens, dtype=np.int64)
    qsl = np.zeros(len(q) + 1, dtype=np.int32)
    ssl = np.zeros(len(n) + 1, dtype=np.int32)
    qsl[1:] = np.cumsum(q).astype(np.int32)
    ssl[1:] = np.cumsum(n).astype(np.int32)
    return {"slot_mapping": np.asarray(slots, dtype=np.int64), "positions": np.asarray(positions, dtype=np.int64),
            "query_lens": q, "query_start_loc": qsl, "seq_start_loc": ssl, "block_tables": padded,
            "seq_lens": np.asarray(seq_lens, dtype=np.int32), "context_lens": np.asarray(context_lens, dtype=np.int32)}


def compare_attention(got: np.ndarray, want: np.ndarray, dtype: int, atol: float = 2e-3, rtol: float = 1e-2):
    """Returns (ok, max_abs_err, worst_excess) under |got - want| <= atol + rtol * |want|."""
    g = bits_to_f64(got, dtype)
    w = bits_to_f64(want, dtype)
    err = np.abs(g - w)
    bound = atol + rtol * np.abs(w)
    excess = float((err - bound).max()) if err.size else 0.0
    ok = bool(np.all(np.isfinite(g)) and excess <= 0.0)
    return ok, float(err.max()) if err.size else 0.0, excess


def scale_for(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)

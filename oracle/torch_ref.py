"""fp32 PyTorch restatement of one decode layer on the host — TEST INFRASTRUCTURE / CPU BASELINE ONLY.

Only ``tests/`` and ``bench.py``'s CPU-baseline leg and reference arm may import this module; the
product package ``aegaeon_b200`` never does. It is the "reference PyTorch path" of the serving
hot path run on the host cores: the reference itself has no CPU implementation (its cache write
and decode attention are vLLM 0.5.1 CUDA kernels), so this restates them in plain torch ops with
fp32 compute, the way a PyTorch reimplementation of the reference's per-layer calls would:

* ``reshape_and_cache``: vLLM 0.5.1 ``reshape_and_cache_flash`` as reached from
  ``aegaeon/aegaeon/worker.py:517-523`` — ``K_l[slot // 16, slot % 16] = key[t]`` (same for V),
  slots < 0 skipped; the decode slot is position ``seq_len - 1`` (``worker.py:628-633``).
* decode attention: vLLM 0.5.1 FlashAttention decode with a block table (``flash_attn_with_kvcache``
  with one query token, causal, bottom-right aligned, so every cached key ``j < seq_len`` is
  visible); query head ``h`` reads KV head ``h // (Hq / Hkv)``; the blocks of the layer are
  gathered and widened to fp32 once, then each sequence runs torch's fp32 scaled-dot-product
  attention over its keys, and the output is rounded to the storage dtype once.

Cache layout: Aegaeon's storage layout ``(N, L, 2, 16, Hkv, D)`` (``worker.py:388-451``,
``config.py:256-271``); a layer's K and V are the ``[:, l, 0]`` and ``[:, l, 1]`` views. All torch
intra-op threads are used (``torch.set_num_threads``).
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn.functional as F


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      slots: torch.Tensor) -> None:
    """``k_cache``/``v_cache`` [N, 16, Hkv, D] views; ``key``/``value`` [T, Hkv, D]; int64 slots."""
    n_slots = k_cache.size(0) * 16
    ok = (slots >= 0) & (slots < n_slots)
    s = slots[ok]
    blk, row = s // 16, s % 16
    k_cache[blk, row] = key[ok]
    v_cache[blk, row] = value[ok]


class DecodeLayerCPU:
    """One decode layer (cache write + attention) of a fixed batch on the host, fp32 compute.

    ``block_tables`` int32 [B, W] and ``seq_lens`` int32 [B] as the reference's per-step metadata
    (``worker.py:640-653``). ``run`` writes ``out`` [B, Hq, D] in the storage dtype; sequences of
    length 0 get zero rows.
    """

    def __init__(self, block_tables: np.ndarray, seq_lens: np.ndarray, scale: float, threads: int | None = None):
        W = block_tables.shape[1]
        self.n = np.clip(np.asarray(seq_lens, dtype=np.int64), 0, W * 16)
        nb = (self.n + 15) // 16
        self.offs = np.concatenate([[0], np.cumsum(nb)]).astype(np.int64)
        rows = [block_tables[b, :nb[b]].astype(np.int64) for b in range(len(nb))]
        self.blocks = torch.as_tensor(np.concatenate(rows) if rows else np.zeros(0, np.int64))
        self.scale = float(scale)
        self.threads = max(1, threads or host_threads())
        self._bufs = None  # gather buffers, reused across calls

    def _buffers(self, k_cache: torch.Tensor) -> tuple:
        shape = (self.blocks.numel(),) + tuple(k_cache.shape[1:])
        if self._bufs is None or self._bufs[0].shape != shape or self._bufs[0].dtype != k_cache.dtype:
            self._bufs = (torch.empty(shape, dtype=k_cache.dtype), torch.empty(shape, dtype=torch.float32),
                          torch.empty(shape, dtype=torch.float32))
        return self._bufs

    def run(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, key: torch.Tensor,
            value: torch.Tensor, slots: torch.Tensor, out: torch.Tensor) -> None:
        if torch.get_num_threads() != self.threads:
            torch.set_num_threads(self.threads)
        reshape_and_cache(key, value, k_cache, v_cache, slots)
        Hq, Hkv, D = q.size(1), k_cache.size(2), k_cache.size(3)
        G = Hq // Hkv
        g16, kf, vf = self._buffers(k_cache)
        torch.index_select(k_cache, 0, self.blocks, out=g16)
        kf.copy_(g16)
        torch.index_select(v_cache, 0, self.blocks, out=g16)
        vf.copy_(g16)
        kf, vf = kf.view(-1, Hkv, D), vf.view(-1, Hkv, D)  # [blocks * 16, Hkv, D] in fp32
        for b in range(len(self.n)):
            n = int(self.n[b])
            if n == 0:
                out[b].zero_()
                continue
            a = int(self.offs[b]) * 16
            k = kf[a:a + n].permute(1, 0, 2)  # [Hkv, n, D]
            v = vf[a:a + n].permute(1, 0, 2)
            o = F.scaled_dot_product_attention(q[b].float().view(Hkv, G, D), k, v, scale=self.scale)
            out[b] = o.reshape(Hq, D).to(out.dtype)

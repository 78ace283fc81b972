"""KV-cache geometry and per-step attention metadata of Aegaeon's serving path.

* Block geometry: one block holds ``BLOCK_SIZE = 16`` tokens of every layer; its shape is
  ``(L, 2, 16, Hkv, D)`` (aegaeon/aegaeon/config.py:13, :256-271). The device cache is
  ``(N, L, 2, 16, Hkv, D)`` and the model runs on the permuted view ``(L, 2, N, 16, Hkv, D)``
  (aegaeon/aegaeon/worker.py:388-451); the host swap pool has the same per-block shape
  (worker.py:398-407).
* Decode metadata: ``slot = table[i // 16] * 16 + i % 16`` for the new positions
  ``[context_len, seq_len)`` (worker.py:628-633); block tables are int32 and padded with 0 to the
  longest table (worker.py:640-646, aegaeon/aegaeon/utils.py:241-257); seq_lens are int32
  (worker.py:653) and the slot mapping is int64 (worker.py:680-682).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

BLOCK_SIZE = 16
KV_PERM = (1, 2, 0, 3, 4, 5)


def kv_block_shape(num_layers: int, num_kv_heads: int, head_dim: int) -> tuple[int, ...]:
    """Per-block shape ``(L, 2, 16, Hkv, D)``."""
    return (num_layers, 2, BLOCK_SIZE, num_kv_heads, head_dim)


def kv_cache_run_view(kv_cache: torch.Tensor) -> torch.Tensor:
    """The ``(L, 2, N, 16, Hkv, D)`` view the model layers index by ``[layer][0|1]``."""
    if kv_cache.dim() != 6:
        raise ValueError(f"kv_cache must be 6-D (N, L, 2, 16, Hkv, D), got {tuple(kv_cache.shape)}")
    return kv_cache.permute(*KV_PERM)


def block_bytes(kv_cache: torch.Tensor) -> int:
    """Bytes of one whole multi-layer block (the swap unit)."""
    if kv_cache.size(0) == 0:
        return 0
    return kv_cache.numel() * kv_cache.element_size() // kv_cache.size(0)


@dataclass
class DecodeMetadata:
    slot_mapping: torch.Tensor   # int64 [num_new_tokens]
    block_tables: torch.Tensor   # int32 [B, max_table_len], zero padded
    seq_lens: torch.Tensor       # int32 [B]
    context_lens: torch.Tensor   # int32 [B]
    max_seq_len: int


def pad_block_tables(tables: Sequence[Sequence[int]], max_len: int | None = None, pad: int = 0) -> np.ndarray:
    """int32 ``[len(tables), max_len]`` array, each row padded at the end with ``pad``."""
    width = max((len(t) for t in tables), default=0) if max_len is None else max_len
    out = np.full((len(tables), width), pad, dtype=np.int32)
    for i, t in enumerate(tables):
        if len(t) > width:
            raise ValueError(f"block table {i} has {len(t)} entries, more than max_len={width}")
        out[i, : len(t)] = np.asarray(t, dtype=np.int32)
    return out


def slots_for(table: Sequence[int], start: int, end: int) -> list[int]:
    """Cache slots of token positions ``[start, end)`` of one sequence."""
    return [int(table[i // BLOCK_SIZE]) * BLOCK_SIZE + i % BLOCK_SIZE for i in range(start, end)]


def build_decode_metadata(seq_lens: Sequence[int], context_lens: Sequence[int],
                          block_tables: Sequence[Sequence[int]],
                          device: torch.device | str = "cpu") -> DecodeMetadata:
    """Slot mapping, padded block tables and lengths for a batch of requests.

    ``seq_lens[i]`` counts the tokens of request i after this step and ``context_lens[i]`` those
    already in the cache; decode requests have ``seq_len - context_len == 1``. Requests with
    ``context_len == 0`` are prompts: their slots are produced but their table row is empty,
    as in the reference's prefill path.
    """
    if not (len(seq_lens) == len(context_lens) == len(block_tables)):
        raise ValueError("seq_lens, context_lens and block_tables must have the same length")
    slots: list[int] = []
    rows: list[Sequence[int]] = []
    for n, c, table in zip(seq_lens, context_lens, block_tables):
        if not 0 <= c <= n:
            raise ValueError(f"context_len {c} must lie in [0, seq_len={n}]")
        if (n + BLOCK_SIZE - 1) // BLOCK_SIZE > len(table):
            raise ValueError(f"block table of {len(table)} blocks cannot hold {n} tokens")
        slots.extend(slots_for(table, c, n))
        rows.append(list(table) if c > 0 else [])
    padded = pad_block_tables(rows)
    return DecodeMetadata(
        slot_mapping=torch.tensor(slots, dtype=torch.int64, device=device),
        block_tables=torch.from_numpy(padded).to(device),
        seq_lens=torch.tensor(list(seq_lens), dtype=torch.int32, device=device),
        context_lens=torch.tensor(list(context_lens), dtype=torch.int32, device=device),
        max_seq_len=max(seq_lens, default=0),
    )

"""Seeded synthetic inputs for the five benchmark configurations of the serving path.

The reference publishes no kernel-level dataset for this path; the configurations are synthetic
by definition (contexts, block assignment and values are drawn from seeded generators):

* ``cfg1`` — one Qwen2.5-7B attention layer (Hq 28, Hkv 4, D 128, fp16), batch 4, contexts
  uniform in [17, 300], 64 physical blocks assigned by a seeded permutation, seed 0.
* ``cfg2`` — Qwen2.5-7B decode step, 28 layers, fp16, batch 64, contexts
  round(lognormal(5.5, 1)) clipped to [4, 4096], a shuffled pool of 16384 blocks; each layer
  writes one new token per sequence (slot of position ctx-1) and attends over ctx tokens.
* ``cfg3`` — Yi-1.5-9B-shaped decode, bf16, Hq 32 / Hkv 4, 48 layers, batch 256, contexts
  round(lognormal(6, 1)) clipped to [4, 8192]; sequence i belongs to GPU i mod n, each GPU has a
  pool sized to its own sequences.
* ``cfg4`` — Llama-2-13B-shaped MHA decode, fp16, Hq = Hkv = 40, 40 layers, batch 32, contexts
  uniform in [2048, 4096], values N(0, 0.5^2) (0.5 read as the standard deviation), seed 3.
* ``cfg5`` — KV-block swap and copy on the Qwen2.5-7B block (28 x 2 x 16 x 4 x 128 fp16 =
  917,504 bytes): 4096 random device blocks out to the host pool and back into fresh ids, and
  copy_blocks over 8192 disjoint random pairs; data are random 16-bit patterns.

Host-side draws use ``torch.Generator`` on the CPU; large value fills use a seeded CUDA
generator on the target device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .layout import BLOCK_SIZE


@dataclass(frozen=True)
class DecodeConfig:
    name: str
    batch: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    num_layers: int
    dtype: torch.dtype
    ctx_dist: tuple  # ("uniform", lo, hi) or ("lognormal", mu, sigma, lo, hi)
    pool_blocks: int | None  # None: sized to the sequences
    value_std: float
    seed: int
    model: str = ""

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads


CONFIGS: dict[str, DecodeConfig] = {
    "cfg1": DecodeConfig("cfg1", 4, 28, 4, 128, 1, torch.float16, ("uniform", 17, 300), 64, 1.0, 0,
                         "Qwen2.5-7B attention layer"),
    "cfg2": DecodeConfig("cfg2", 64, 28, 4, 128, 28, torch.float16, ("lognormal", 5.5, 1.0, 4, 4096), 16384, 1.0, 0,
                         "Qwen2.5-7B"),
    "cfg3": DecodeConfig("cfg3", 256, 32, 4, 128, 48, torch.bfloat16, ("lognormal", 6.0, 1.0, 4, 8192), None, 1.0, 0,
                         "Yi-1.5-9B-shaped"),
    "cfg4": DecodeConfig("cfg4", 32, 40, 40, 128, 40, torch.float16, ("uniform", 2048, 4096), None, 0.5, 3,
                         "Llama-2-13B-shaped (MHA)"),
}

SWAP_CFG = dict(name="cfg5", num_layers=28, num_kv_heads=4, head_dim=128, dtype=torch.float16,
                device_blocks=16384, swap_blocks=4096, copy_pairs=8192, seed=0)


def draw_contexts(cfg: DecodeConfig, gen: torch.Generator) -> torch.Tensor:
    kind = cfg.ctx_dist[0]
    if kind == "uniform":
        lo, hi = cfg.ctx_dist[1], cfg.ctx_dist[2]
        return torch.randint(lo, hi + 1, (cfg.batch,), generator=gen, dtype=torch.int64)
    _, mu, sigma, lo, hi = cfg.ctx_dist
    x = torch.empty(cfg.batch, dtype=torch.float64).log_normal_(mu, sigma, generator=gen)
    return torch.clamp(torch.round(x), lo, hi).to(torch.int64)


@dataclass
class DecodeLayout:
    """Context lengths, block tables and the pool size of one (shard of a) decode config."""
    seq_lens: np.ndarray          # int32 [B]
    block_tables: np.ndarray      # int32 [B, W], zero padded
    num_blocks: int               # pool size N
    seq_ids: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int64))  # global sequence ids

    @property
    def width(self) -> int:
        return self.block_tables.shape[1]

    @property
    def total_tokens(self) -> int:
        return int(self.seq_lens.astype(np.int64).sum())

    @property
    def total_blocks(self) -> int:
        return int(((self.seq_lens.astype(np.int64) + BLOCK_SIZE - 1) // BLOCK_SIZE).sum())


def balanced_split(ctx: np.ndarray, world: int) -> list[np.ndarray]:
    """Sequence ids per rank with about equal total context: longest first, each to the rank with
    the least context so far (lowest rank on ties); ids ascending within a rank."""
    load = np.zeros(world, np.int64)
    owner = np.empty(len(ctx), np.int64)
    for i in sorted(range(len(ctx)), key=lambda i: (-int(ctx[i]), i)):
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += int(ctx[i])
    return [np.flatnonzero(owner == r) for r in range(world)]


def make_layout(cfg: DecodeConfig, rank: int = 0, world: int = 1, split: str = "mod") -> DecodeLayout:
    """Seeded contexts and block assignment. With ``world > 1`` returns this rank's sequences:
    ``split="mod"`` takes sequences i = rank mod world (equal counts), ``split="balanced"`` the
    ranks' shares of ``balanced_split`` (about equal context)."""
    gen = torch.Generator().manual_seed(cfg.seed)
    ctx = draw_contexts(cfg, gen).numpy()
    if split == "mod":
        ids = np.arange(cfg.batch)[rank::world]
    elif split == "balanced":
        ids = balanced_split(ctx, world)[rank]
    else:
        raise ValueError(f"split must be 'mod' or 'balanced', not {split!r}")
    ctx = ctx[ids]
    nblk = (ctx + BLOCK_SIZE - 1) // BLOCK_SIZE
    need = int(nblk.sum())
    n_pool = cfg.pool_blocks if cfg.pool_blocks is not None else need
    if need > n_pool:
        raise ValueError(f"{cfg.name}: {need} blocks needed but the pool holds {n_pool}")
    perm = torch.randperm(n_pool, generator=gen).numpy()
    W = int(nblk.max()) if len(nblk) else 1
    tables = np.zeros((len(ctx), max(W, 1)), dtype=np.int32)
    off = 0
    for i, nb in enumerate(nblk):
        tables[i, :nb] = perm[off:off + nb]
        off += nb
    return DecodeLayout(seq_lens=ctx.astype(np.int32), block_tables=tables, num_blocks=n_pool, seq_ids=ids)


def compact_layout(layout: DecodeLayout) -> DecodeLayout:
    """The same sequences over a pool that holds only their blocks (ids 0..total-1, in table order)."""
    nb = (layout.seq_lens.astype(np.int64) + BLOCK_SIZE - 1) // BLOCK_SIZE
    tables = np.zeros_like(layout.block_tables)
    off = 0
    for i, n in enumerate(nb):
        tables[i, :n] = np.arange(off, off + n)
        off += n
    return DecodeLayout(seq_lens=layout.seq_lens.copy(), block_tables=tables, num_blocks=max(int(off), 1),
                        seq_ids=layout.seq_ids.copy())


def new_token_slots(layout: DecodeLayout) -> np.ndarray:
    """Slot of each sequence's newest position ``ctx - 1`` (written before the layer's attention)."""
    pos = layout.seq_lens.astype(np.int64) - 1
    blk = layout.block_tables[np.arange(len(pos)), pos // BLOCK_SIZE].astype(np.int64)
    return blk * BLOCK_SIZE + pos % BLOCK_SIZE


def fill_normal_(t: torch.Tensor, std: float, seed: int) -> torch.Tensor:
    """Fills ``t`` with N(0, std^2) from a generator seeded on ``t``'s device, in bounded chunks."""
    gen = torch.Generator(device=t.device).manual_seed(seed)
    flat = t.view(-1)
    chunk = 1 << 28
    for s in range(0, flat.numel(), chunk):
        part = flat[s:s + chunk]
        part.normal_(0.0, std, generator=gen)
    return t


def random_bits_(t: torch.Tensor, seed: int) -> torch.Tensor:
    """Fills a 2-byte tensor with uniformly random 16-bit patterns (NaN/Inf encodings included)."""
    gen = torch.Generator(device=t.device).manual_seed(seed)
    flat = t.view(torch.int16).view(-1)
    chunk = 1 << 28
    for s in range(0, flat.numel(), chunk):
        part = flat[s:s + chunk]
        part.copy_(torch.randint(-32768, 32768, (part.numel(),), generator=gen, device=t.device,
                                 dtype=torch.int32).to(torch.int16))
    return t


def kv_cache_bytes(cfg: DecodeConfig, num_blocks: int) -> int:
    return num_blocks * cfg.num_layers * 2 * BLOCK_SIZE * cfg.num_kv_heads * cfg.head_dim * 2


def algorithmic_bytes_per_layer(cfg: DecodeConfig, layout: DecodeLayout) -> dict:
    """Bytes an ideal kernel moves per layer call (KV read once, q read, out written, tables)."""
    s = 2
    kv = layout.total_tokens * cfg.num_kv_heads * cfg.head_dim * 2 * s
    qo = 2 * len(layout.seq_lens) * cfg.num_q_heads * cfg.head_dim * s
    tables = 4 * layout.total_blocks + 4 * len(layout.seq_lens)
    cache_write = len(layout.seq_lens) * (2 * cfg.num_kv_heads * cfg.head_dim * s * 2 + 8)
    return {"attention": kv + qo + tables, "kv_read": kv, "reshape_and_cache": cache_write}


def attention_flops_per_layer(cfg: DecodeConfig, layout: DecodeLayout) -> int:
    return 4 * layout.total_tokens * cfg.num_q_heads * cfg.head_dim


def default_scale(cfg: DecodeConfig) -> float:
    return 1.0 / math.sqrt(cfg.head_dim)


def qwen2_7b_param_bytes(dtype_bytes: int = 2, layers: int = 28) -> list[int]:
    """Byte sizes of Qwen2.5-7B's parameters in load order (hidden 3584, intermediate 18944,
    28 query / 4 KV heads of 128, vocabulary 152064, untied embeddings): the weight-switch
    workload."""
    h, inter, kv, vocab = 3584, 18944, 4 * 128, 152064
    shapes = [(vocab, h)]
    for _ in range(layers):
        shapes += [(h, h), (h,), (kv, h), (kv,), (kv, h), (kv,), (h, h), (inter, h), (inter, h), (h, inter), (h,), (h,)]
    shapes += [(h,), (vocab, h)]
    out = []
    for sh in shapes:
        n = 1
        for d in sh:
            n *= d
        out.append(n * dtype_bytes)
    return out

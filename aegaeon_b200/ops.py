"""Python mirror of Aegaeon's ``aegaeon.ops`` operator module, backed by the sm_100a C ABI.

``swap`` keeps the exact call signature and meaning of the reference operator
(``aegaeon/ops/ops.h:4-10``, ``aegaeon/ops/swap.cu:25-60``): it runs on the current torch stream,
returns before the copy completes, and takes the block geometry from ``kv_cache``. The other
operators are the per-layer cache write and decode attention that the reference reaches through
vLLM 0.5.1 (``aegaeon/aegaeon/worker.py:517-523``) and the block copy of vLLM's cache ops, on
Aegaeon's ``(N, L, 2, 16, Hkv, D)`` block layout.

Every operator validates its arguments on the host and raises ``ValueError`` (bad argument),
``NotImplementedError`` (unsupported shape) or ``AegaeonError`` (CUDA failure). There is no CPU
or PyTorch fallback: the work always runs in the CUDA library.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import numpy as np
import torch

from . import _native
from ._native import AEG_DECODE_PREFETCH, AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE, check, lib
from .layout import BLOCK_SIZE, block_bytes

_DTYPES = {torch.float16: _native.AEG_DTYPE_FP16, torch.bfloat16: _native.AEG_DTYPE_BF16}


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")


def _same_device(dev: torch.device, **tensors) -> None:
    """Raises ValueError unless every given tensor lives on ``dev`` (the device the work runs on):
    a kernel handed another GPU's address would read across NVLink or fault."""
    for name, t in tensors.items():
        if t is not None and t.device != dev:
            raise ValueError(f"{name} is on {t.device}, the operation runs on {dev}")


def _ids_array(ids, name: str) -> np.ndarray:
    if isinstance(ids, torch.Tensor):
        ids = ids.detach().cpu().numpy()
    arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int64).reshape(-1))
    return arr


def _device_ids(ids, device: torch.device, name: str) -> torch.Tensor:
    if isinstance(ids, torch.Tensor):
        if ids.dtype != torch.int64:
            ids = ids.to(torch.int64)
        return ids.to(device, non_blocking=True).contiguous().view(-1)
    return torch.as_tensor(np.asarray(ids, dtype=np.int64).reshape(-1)).to(device, non_blocking=True)


def read_device_errors(device: torch.device | int | None = None) -> int:
    """Reads and clears the library's sticky device error bits (synchronises the stream)."""
    dev = torch.device("cuda") if device is None else torch.device(device)
    if isinstance(device, int):
        dev = torch.device("cuda", device)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    flags = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        check(lib.aeg_read_device_errors(_stream(dev), ctypes.byref(flags)), "read_device_errors")
    return int(flags.value)


# --------------------------------------------------------------------------------------------
# Block movement


def _check_pools(kv_cache: torch.Tensor, kv_swap: torch.Tensor) -> int:
    _require_cuda(kv_cache, "kv_cache")
    if not isinstance(kv_swap, torch.Tensor) or kv_swap.device.type != "cpu":
        raise ValueError("kv_swap must be a CPU (host) tensor")
    if not kv_cache.is_contiguous() or not kv_swap.is_contiguous():
        raise ValueError("kv_cache and kv_swap must be contiguous")
    bb = block_bytes(kv_cache)
    if kv_swap.dim() > 0 and kv_swap.size(0) > 0:
        host_bb = kv_swap.numel() * kv_swap.element_size() // kv_swap.size(0)
        if host_bb != bb:
            raise ValueError(f"kv_swap block of {host_bb} bytes differs from kv_cache block of {bb} bytes")
    return bb


def swap(source_block_ids: Sequence[int], target_block_ids: Sequence[int], is_swap_in: bool,
         kv_cache: torch.Tensor, kv_swap: torch.Tensor) -> None:
    """Copies whole KV blocks between the device cache and the host swap pool.

    ``is_swap_in``: host block ``source_block_ids[i]`` -> device block ``target_block_ids[i]``;
    otherwise device -> host. Enqueued on the current stream of ``kv_cache``'s device.
    """
    src = _ids_array(source_block_ids, "source_block_ids")
    dst = _ids_array(target_block_ids, "target_block_ids")
    if src.shape != dst.shape:
        raise ValueError(f"{src.size} source ids but {dst.size} target ids")
    bb = _check_pools(kv_cache, kv_swap)
    if src.size == 0:
        return
    n_host = kv_swap.size(0) if kv_swap.dim() > 0 else 0
    with torch.cuda.device(kv_cache.device):
        st = lib.aeg_swap(kv_cache.data_ptr(), kv_swap.data_ptr(), bb, kv_cache.size(0), n_host,
                          src.ctypes.data, dst.ctypes.data, src.size, int(bool(is_swap_in)),
                          _stream(kv_cache.device))
    check(st, "swap")


def swap_sm(source_block_ids, target_block_ids, is_swap_in: bool, kv_cache: torch.Tensor,
            kv_swap: torch.Tensor) -> None:
    """``swap`` done by one kernel over the mapped page-locked host pool (scattered ids, one launch).

    ``kv_swap`` must be page-locked (``pin_memory()`` or ``cudaHostRegister``). Ids may be lists or
    int64 tensors; they are staged to the device on the current stream.
    """
    bb = _check_pools(kv_cache, kv_swap)
    dev = kv_cache.device
    src = _device_ids(source_block_ids, dev, "source_block_ids")
    dst = _device_ids(target_block_ids, dev, "target_block_ids")
    if src.numel() != dst.numel():
        raise ValueError(f"{src.numel()} source ids but {dst.numel()} target ids")
    if src.numel() == 0:
        return
    n_host = kv_swap.size(0) if kv_swap.dim() > 0 else 0
    with torch.cuda.device(dev):
        st = lib.aeg_swap_sm(kv_cache.data_ptr(), kv_swap.data_ptr(), bb, kv_cache.size(0), n_host,
                             src.data_ptr(), dst.data_ptr(), src.numel(), int(bool(is_swap_in)), _stream(dev))
    check(st, "swap_sm")
    # keep the staged id tensors alive until the kernel has consumed them
    src.record_stream(torch.cuda.current_stream(dev))
    dst.record_stream(torch.cuda.current_stream(dev))


def swap_batched(src: torch.Tensor, dst: torch.Tensor, is_swap_in: bool, kv_cache: torch.Tensor,
                 kv_swap: torch.Tensor, engine: str = "dma") -> None:
    """``swap`` for id lists already held as int64 tensors (no Python list conversion).

    ``engine="dma"``: host (CPU) id tensors, read in place; one copy-engine transfer per run of
    blocks adjacent on both sides, as ``swap``. ``engine="sm"``: ids on the device (or staged
    there), one kernel over the mapped page-locked ``kv_swap``, as ``swap_sm``. Same stream and
    completion rules as ``swap``.
    """
    for t, name in ((src, "src"), (dst, "dst")):
        if not isinstance(t, torch.Tensor) or t.dtype != torch.int64:
            raise ValueError(f"{name} must be an int64 tensor")
    if engine == "sm":
        swap_sm(src, dst, is_swap_in, kv_cache, kv_swap)
        return
    if engine != "dma":
        raise ValueError(f"engine must be 'dma' or 'sm', not {engine!r}")
    if src.device.type != "cpu" or dst.device.type != "cpu":
        raise ValueError("engine='dma' reads the ids on the host: src and dst must be CPU tensors")
    swap(src.contiguous(), dst.contiguous(), is_swap_in, kv_cache, kv_swap)


def copy_blocks(src_ids, dst_ids, kv_cache: torch.Tensor) -> None:
    """``kv_cache[dst_ids[i]] = kv_cache[src_ids[i]]`` for whole multi-layer blocks (device to device)."""
    _require_cuda(kv_cache, "kv_cache")
    if not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be contiguous")
    dev = kv_cache.device
    src = _device_ids(src_ids, dev, "src_ids")
    dst = _device_ids(dst_ids, dev, "dst_ids")
    if src.numel() != dst.numel():
        raise ValueError(f"{src.numel()} source ids but {dst.numel()} destination ids")
    if src.numel() == 0:
        return
    with torch.cuda.device(dev):
        st = lib.aeg_copy_blocks(kv_cache.data_ptr(), block_bytes(kv_cache), kv_cache.size(0), src.data_ptr(),
                                 dst.data_ptr(), src.numel(), _stream(dev))
    check(st, "copy_blocks")
    src.record_stream(torch.cuda.current_stream(dev))
    dst.record_stream(torch.cuda.current_stream(dev))


# --------------------------------------------------------------------------------------------
# GPU <-> GPU block migration. The reference stubs this path (Worker.register_kvcache_mem_handles
# and Worker.migrate_blocks, aegaeon/aegaeon/worker.py:841-872; BlockManager._migrate_requests,
# aegaeon/aegaeon/block_manager.py:876-950): the target engine opens the source engine's KV-cache
# IPC handles (aegaeon/aegaeon/cuda_wrapper.py:190-208) and copies each request's blocks into
# blocks of its own pool.

IPC_HANDLE_BYTES = _native.AEG_IPC_HANDLE_BYTES


def export_kv_cache(kv_cache: torch.Tensor) -> bytes:
    """The IPC handle of a device block pool, for ``open_kv_cache`` in another process.

    ``kv_cache`` must live in memory from cudaMalloc (PyTorch's default allocator). The handle is
    plain bytes; send it through any host channel (``torch.distributed`` object collectives, a
    store, a pipe). The exporter keeps ``kv_cache`` alive while others have it open.
    """
    _require_cuda(kv_cache, "kv_cache")
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    with torch.cuda.device(kv_cache.device):
        check(lib.aeg_ipc_export(kv_cache.data_ptr(), buf), "ipc_export")
    return buf.raw


class PeerKVCache:
    """Another process's block pool mapped into this process (``aeg_ipc_open``).

    ``num_blocks`` and ``block_bytes`` describe the pool (the exporter's ``kv_cache.size(0)`` and
    ``layout.block_bytes(kv_cache)``); the mapping must cover them. ``close()`` (or leaving a
    ``with`` block) unmaps it once the work that reads it has completed.
    """

    def __init__(self, handle: bytes, num_blocks: int, block_bytes_: int):
        if not isinstance(handle, (bytes, bytearray)) or len(handle) != IPC_HANDLE_BYTES:
            raise ValueError(f"an IPC handle is {IPC_HANDLE_BYTES} bytes")
        if num_blocks < 0 or block_bytes_ <= 0:
            raise ValueError("num_blocks must be >= 0 and block_bytes positive")
        ptr = ctypes.c_void_p()
        avail = ctypes.c_int64()
        check(lib.aeg_ipc_open(bytes(handle), ctypes.byref(ptr), ctypes.byref(avail)), "ipc_open")
        self.ptr = int(ptr.value or 0)
        self.num_blocks = int(num_blocks)
        self.block_bytes = int(block_bytes_)
        if num_blocks * block_bytes_ > avail.value:
            self.close()
            raise ValueError(f"the mapped pool holds {avail.value} bytes, fewer than "
                             f"{num_blocks} blocks x {block_bytes_} bytes")

    def close(self) -> None:
        if self.ptr:
            ptr, self.ptr = self.ptr, 0
            check(lib.aeg_ipc_close(ptr), "ipc_close")

    def __enter__(self) -> "PeerKVCache":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def open_kv_cache(handle: bytes, num_blocks: int, block_bytes_: int) -> PeerKVCache:
    """Maps a pool exported by ``export_kv_cache`` in another process."""
    return PeerKVCache(handle, num_blocks, block_bytes_)


def _pool(p, name: str) -> tuple[int, int, int, torch.device | None]:
    """(address, blocks, block bytes, device of a local tensor or None) of a migration pool."""
    if isinstance(p, PeerKVCache):
        if not p.ptr:
            raise ValueError(f"{name} is closed")
        return p.ptr, p.num_blocks, p.block_bytes, None
    _require_cuda(p, name)
    if not p.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return p.data_ptr(), p.size(0), block_bytes(p), p.device


def migrate_blocks(source_block_ids, target_block_ids, source, target, *, engine: str = "sm") -> None:
    """``target[target_block_ids[i]] <- source[source_block_ids[i]]`` for whole multi-layer blocks
    between two GPUs' pools.

    ``source`` / ``target`` are device tensors of this process (on any GPU it can reach) or
    ``PeerKVCache`` mappings of another process's pool. The work runs on the device of ``target``
    when it is a tensor (a pull, as the reference's target engine does), else on the device of
    ``source`` (a push), on that device's current stream, and returns before it completes.
    ``engine="sm"``: one kernel streams 16-byte vectors over NVLink (ids staged to the device);
    ``engine="dma"``: the copy engines, one transfer per run of blocks adjacent on both sides.
    """
    s_ptr, s_n, s_bb, s_dev = _pool(source, "source")
    t_ptr, t_n, t_bb, t_dev = _pool(target, "target")
    if s_bb != t_bb:
        raise ValueError(f"block sizes differ: source {s_bb} bytes, target {t_bb} bytes")
    dev = t_dev if t_dev is not None else s_dev
    if dev is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    if engine == "dma":
        src = _ids_array(source_block_ids, "source_block_ids")
        dst = _ids_array(target_block_ids, "target_block_ids")
        if src.shape != dst.shape:
            raise ValueError(f"{src.size} source ids but {dst.size} target ids")
        if src.size == 0:
            return
        with torch.cuda.device(dev):
            st = lib.aeg_migrate_blocks_dma(t_ptr, t_n, s_ptr, s_n, s_bb, src.ctypes.data, dst.ctypes.data,
                                            src.size, _stream(dev))
        check(st, "migrate_blocks_dma")
        return
    if engine != "sm":
        raise ValueError(f"engine must be 'sm' or 'dma', not {engine!r}")
    src = _device_ids(source_block_ids, dev, "source_block_ids")
    dst = _device_ids(target_block_ids, dev, "target_block_ids")
    if src.numel() != dst.numel():
        raise ValueError(f"{src.numel()} source ids but {dst.numel()} target ids")
    if src.numel() == 0:
        return
    with torch.cuda.device(dev):
        st = lib.aeg_migrate_blocks(t_ptr, t_n, s_ptr, s_n, s_bb, src.data_ptr(), dst.data_ptr(), src.numel(),
                                    _stream(dev))
    check(st, "migrate_blocks")
    src.record_stream(torch.cuda.current_stream(dev))
    dst.record_stream(torch.cuda.current_stream(dev))


# --------------------------------------------------------------------------------------------
# Prefill attention (vLLM 0.5.1 FlashAttention backend, prompt tokens: flash_attn_varlen_func)


def flash_attn_varlen_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                              max_seqlen: int, softmax_scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of every prompt over itself, the call vLLM makes for prompts:
    ``flash_attn_varlen_func(q, k, v, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen,
    softmax_scale, causal=True)``.

    ``q`` [T, Hq, 128], ``k``/``v`` [T, Hkv, 128] (fp16 or bf16, token-major, head dim
    contiguous), ``cu_seqlens`` int32 [B + 1] on the device (prompt b = tokens cu[b] .. cu[b+1] - 1),
    ``max_seqlen`` the longest prompt. Returns ``out`` [T, Hq, 128].
    """
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _require_cuda(t, name)
        if t.dim() != 3 or t.stride(2) != 1 or t.stride(1) != t.size(2):
            raise ValueError(f"{name} must be [tokens, heads, head_dim] with contiguous heads")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share an fp16 or bf16 dtype")
    T, Hq, D = q.shape
    if k.shape[0] != T or v.shape != k.shape:
        raise ValueError("k and v must be [tokens, Hkv, head_dim] with q's token count")
    _require_cuda(cu_seqlens, "cu_seqlens")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or not cu_seqlens.is_contiguous():
        raise ValueError("cu_seqlens must be a contiguous int32 vector")
    if out is None:
        out = torch.empty_like(q)
    if out.shape != q.shape or out.dtype != q.dtype or out.stride(2) != 1 or out.stride(1) != D:
        raise ValueError("out must match q")
    dev = q.device
    _same_device(dev, k=k, v=v, cu_seqlens=cu_seqlens, out=out)
    with torch.cuda.device(dev):
        st = lib.aeg_prefill_attention(out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(),
                                       k.stride(0), v.data_ptr(), v.stride(0), cu_seqlens.data_ptr(), T,
                                       cu_seqlens.numel() - 1, int(max_seqlen), Hq, k.size(1), D, float(softmax_scale),
                                       _DTYPES[q.dtype], _stream(dev))
    check(st, "prefill_attention")
    return out


# --------------------------------------------------------------------------------------------
# Model-weight switch (aegaeon/aegaeon/worker.py:358-365: one copy_ per parameter)


def copy_segments(dst: torch.Tensor, src: torch.Tensor, src_offsets, dst_offsets, sizes, *,
                  engine: str = "dma") -> None:
    """Copies byte segments ``src[src_offsets[i]:+sizes[i]] -> dst[dst_offsets[i]:+sizes[i]]``
    between two storages in one call (offsets and sizes in bytes, relative to each tensor's
    first byte), on the current stream of the CUDA side.

    The weight-switch use: ``src`` the page-locked host model cache, ``dst`` the device weight
    arena, one segment per parameter. ``engine="dma"``: copy engines, one transfer per run of
    segments adjacent on both sides; ``engine="sm"``: one kernel through the mapped host memory.
    Destination segments must not overlap; every segment must lie inside both tensors.
    """
    so, do, sz = (_ids_array(x, n) for x, n in ((src_offsets, "src_offsets"), (dst_offsets, "dst_offsets"),
                                                (sizes, "sizes")))
    if not (so.shape == do.shape == sz.shape):
        raise ValueError("src_offsets, dst_offsets and sizes must have the same length")
    if so.size == 0:
        return
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("dst and src must be contiguous")
    if (sz < 0).any() or (so < 0).any() or (do < 0).any():
        raise ValueError("offsets and sizes must be non-negative")
    if int((so + sz).max()) > src.numel() * src.element_size() or int((do + sz).max()) > dst.numel() * dst.element_size():
        raise ValueError("a segment runs past the end of its tensor")
    dev = dst.device if dst.device.type == "cuda" else src.device
    if dev.type != "cuda":
        raise ValueError("one of dst / src must be a CUDA tensor")
    eng = {"dma": _native.AEG_COPY_ENGINE_DMA, "sm": _native.AEG_COPY_ENGINE_SM}.get(engine)
    if eng is None:
        raise ValueError(f"engine must be 'dma' or 'sm', not {engine!r}")
    ws_bytes = lib.aeg_copy_segments_workspace_size(so.size) if eng == _native.AEG_COPY_ENGINE_SM else 0
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.aeg_copy_segments(dst.data_ptr(), src.data_ptr(), so.ctypes.data, do.ctypes.data, sz.ctypes.data,
                                   so.size, eng, ws.data_ptr(), ws_bytes, _stream(dev))
    check(st, "copy_segments")
    ws.record_stream(torch.cuda.current_stream(dev))


def tensor_segments(tensors, storage: torch.Tensor) -> tuple[np.ndarray, np.ndarray]:
    """(byte offsets within ``storage``, byte sizes) of tensors that live inside ``storage``."""
    base = storage.data_ptr()
    end = base + storage.numel() * storage.element_size()
    offs, sizes = [], []
    for t in tensors:
        n = t.numel() * t.element_size()
        if not (base <= t.data_ptr() and t.data_ptr() + n <= end) or not t.is_contiguous():
            raise ValueError("every tensor must be contiguous and inside the storage")
        offs.append(t.data_ptr() - base)
        sizes.append(n)
    return np.asarray(offs, dtype=np.int64), np.asarray(sizes, dtype=np.int64)


# --------------------------------------------------------------------------------------------
# Per-step model inputs on the device (Worker._prepare_model_inputs, aegaeon/aegaeon/worker.py:596-682)


class StepInputs:
    """Device tensors of one step's model inputs (see ``prepare_step_inputs``)."""

    def __init__(self, B: int, table_stride: int, capacity: int, device: torch.device):
        self.capacity = int(capacity)
        self.slot_mapping = torch.empty(self.capacity, dtype=torch.int64, device=device)
        self.positions = torch.empty(self.capacity, dtype=torch.int64, device=device)
        self.query_lens = torch.empty(B, dtype=torch.int64, device=device)
        self.query_start_loc = torch.empty(B + 1, dtype=torch.int32, device=device)
        self.seq_start_loc = torch.empty(B + 1, dtype=torch.int32, device=device)
        self.block_tables = torch.empty((B, table_stride), dtype=torch.int32, device=device)
        self.num_tokens = torch.empty(1, dtype=torch.int64, device=device)


def prepare_step_inputs(block_tables: torch.Tensor, context_lens: torch.Tensor, seq_lens: torch.Tensor,
                        capacity: int | None = None, out: StepInputs | None = None) -> StepInputs:
    """Slot mapping, positions, start offsets and attention table rows of a step, on the device.

    ``block_tables`` (int32 [B, W], request i's blocks in row i), ``context_lens`` and ``seq_lens``
    (int32 [B]) are device tensors that stay resident across steps (``update_block_tables`` applies
    a step's new blocks). ``capacity`` bounds the new tokens written (default B, i.e. a decode
    batch); ``out.num_tokens`` holds the true count, and a larger count raises a device error.
    Runs on the current stream; nothing is copied to the host.
    """
    for t, name in ((block_tables, "block_tables"), (context_lens, "context_lens"), (seq_lens, "seq_lens")):
        _require_cuda(t, name)
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    if block_tables.dim() != 2:
        raise ValueError("block_tables must be [B, W]")
    B, W = block_tables.shape
    if context_lens.numel() != B or seq_lens.numel() != B:
        raise ValueError("context_lens and seq_lens must have one entry per table row")
    dev = block_tables.device
    _same_device(dev, context_lens=context_lens, seq_lens=seq_lens)
    if out is None:
        out = StepInputs(B, W, B if capacity is None else capacity, dev)
    _same_device(dev, slot_mapping=out.slot_mapping, step_block_tables=out.block_tables)
    with torch.cuda.device(dev):
        st = lib.aeg_prepare_step_inputs(block_tables.data_ptr(), W, context_lens.data_ptr(), seq_lens.data_ptr(), B,
                                         out.slot_mapping.data_ptr(), out.positions.data_ptr(), out.capacity,
                                         out.query_lens.data_ptr(), out.query_start_loc.data_ptr(),
                                         out.seq_start_loc.data_ptr(), out.block_tables.data_ptr(),
                                         out.num_tokens.data_ptr(), _stream(dev))
    check(st, "prepare_step_inputs")
    return out


def update_block_tables(block_tables: torch.Tensor, updates) -> None:
    """Writes ``block_tables[row, col] = block`` for every (row, col, block) triple of ``updates``
    (an int32 [n, 3] tensor or a sequence of triples), on the current stream."""
    _require_cuda(block_tables, "block_tables")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or not block_tables.is_contiguous():
        raise ValueError("block_tables must be a contiguous int32 [rows, W] tensor")
    dev = block_tables.device
    if isinstance(updates, torch.Tensor):
        u = updates.to(device=dev, dtype=torch.int32).contiguous().view(-1, 3)
    else:
        u = torch.as_tensor(np.asarray(updates, dtype=np.int32).reshape(-1, 3)).to(dev, non_blocking=True)
    if u.numel() == 0:
        return
    with torch.cuda.device(dev):
        st = lib.aeg_update_block_tables(block_tables.data_ptr(), block_tables.size(1), block_tables.size(0),
                                         u.data_ptr(), u.size(0), _stream(dev))
    check(st, "update_block_tables")
    u.record_stream(torch.cuda.current_stream(dev))


# --------------------------------------------------------------------------------------------
# Per-layer cache write


def _layer_views(kv_cache: torch.Tensor, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
    _require_cuda(kv_cache, "kv_cache")
    if kv_cache.dim() != 6 or kv_cache.size(2) != 2 or kv_cache.size(3) != BLOCK_SIZE:
        raise ValueError(f"kv_cache must have shape (N, L, 2, 16, Hkv, D), got {tuple(kv_cache.shape)}")
    if not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be contiguous")
    if not 0 <= layer < kv_cache.size(1):
        raise ValueError(f"layer {layer} outside [0, {kv_cache.size(1)})")
    return kv_cache[:, layer, 0], kv_cache[:, layer, 1]


def _check_paged_view(t: torch.Tensor, name: str) -> None:
    _require_cuda(t, name)
    if t.dim() != 4 or t.size(1) != BLOCK_SIZE:
        raise ValueError(f"{name} must be (N, 16, Hkv, D), got {tuple(t.shape)}")
    Hkv, D = t.size(2), t.size(3)
    if t.stride(3) != 1 or t.stride(2) != D or t.stride(1) != Hkv * D:
        raise ValueError(f"{name} must have a contiguous (16, Hkv, D) block interior")


def reshape_and_cache_flash(key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor,
                            value_cache: torch.Tensor, slot_mapping: torch.Tensor,
                            kv_cache_dtype: str = "auto") -> None:
    """vLLM-shaped cache write: ``key_cache[s // 16, s % 16] = key[t]`` (same for value), s = slot_mapping[t] >= 0."""
    if kv_cache_dtype != "auto":
        raise NotImplementedError("only kv_cache_dtype='auto' (cache dtype == key dtype) is supported")
    _check_paged_view(key_cache, "key_cache")
    _check_paged_view(value_cache, "value_cache")
    for name, t in (("key", key), ("value", value)):
        _require_cuda(t, name)
        if t.dim() != 3 or t.stride(2) != 1 or t.stride(1) != t.size(2):
            raise ValueError(f"{name} must be [T, Hkv, D] with contiguous heads")
        if t.dtype != key_cache.dtype:
            raise ValueError(f"{name} dtype {t.dtype} differs from cache dtype {key_cache.dtype}")
    if key.shape != value.shape or key.shape[1:] != key_cache.shape[2:]:
        raise ValueError("key/value shapes do not match the cache (Hkv, D)")
    if key_cache.shape != value_cache.shape or key_cache.stride() != value_cache.stride():
        raise ValueError("key_cache and value_cache must have the same shape and strides")
    _require_cuda(slot_mapping, "slot_mapping")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or slot_mapping.numel() != key.size(0):
        raise ValueError("slot_mapping must be int64 [T]")
    if key.element_size() != 2:
        raise NotImplementedError("only 2-byte cache elements (fp16/bf16) are supported")
    slot_mapping = slot_mapping.contiguous()
    dev = key_cache.device
    _same_device(dev, key=key, value=value, value_cache=value_cache, slot_mapping=slot_mapping)
    with torch.cuda.device(dev):
        st = lib.aeg_reshape_and_cache(key.data_ptr(), value.data_ptr(), key.stride(0), value.stride(0),
                                       key_cache.data_ptr(), value_cache.data_ptr(), key_cache.stride(0),
                                       key_cache.size(0), slot_mapping.data_ptr(), key.size(0), key.size(1),
                                       key.size(2), _stream(dev))
    check(st, "reshape_and_cache")


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor, layer: int,
                      slot_mapping: torch.Tensor) -> None:
    """Writes the new tokens' K/V of ``layer`` into Aegaeon's ``(N, L, 2, 16, Hkv, D)`` cache."""
    kc, vc = _layer_views(kv_cache, layer)
    reshape_and_cache_flash(key, value, kc, vc, slot_mapping)


# --------------------------------------------------------------------------------------------
# Decode attention


class DecodePlan:
    """Per-step work plan + scratch for ``paged_attention_decode`` (built once, used by every layer).

    The plan depends only on ``seq_lens`` (like the per-step attention metadata of
    ``aegaeon/aegaeon/worker.py:694-711``). Its workspace is device memory owned by this object;
    one plan must not be used by two streams at the same time.
    """

    def __init__(self, batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 device: torch.device | str = "cuda"):
        self.batch, self.num_q_heads, self.num_kv_heads, self.head_dim = batch, num_q_heads, num_kv_heads, head_dim
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DecodePlan needs a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = lib.aeg_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim)
        if nbytes == 0:
            raise ValueError(f"invalid decode shape B={batch} Hq={num_q_heads} Hkv={num_kv_heads} D={head_dim}")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.table_width: int | None = None
        self.seq_lens: torch.Tensor | None = None
        self.block_tables: torch.Tensor | None = None

    def plan(self, seq_lens: torch.Tensor, block_tables: torch.Tensor) -> "DecodePlan":
        """Builds the unit list for ``seq_lens`` (int32 CUDA [B]) and ``block_tables`` (int32 CUDA
        [B, W]) on the current stream. Both must stay unchanged while the plan is in use."""
        _require_cuda(seq_lens, "seq_lens")
        _require_cuda(block_tables, "block_tables")
        if seq_lens.dtype != torch.int32 or seq_lens.dim() != 1 or seq_lens.numel() != self.batch:
            raise ValueError(f"seq_lens must be int32 [{self.batch}]")
        if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.size(0) != self.batch:
            raise ValueError(f"block_tables must be int32 [{self.batch}, W]")
        if block_tables.size(1) == 0:
            raise ValueError("block_tables has no columns")
        _same_device(self.device, seq_lens=seq_lens, block_tables=block_tables)
        seq_lens = seq_lens.contiguous()
        if block_tables.stride(1) != 1:
            block_tables = block_tables.contiguous()
        with torch.cuda.device(self.device):
            st = lib.aeg_decode_plan(self.workspace.data_ptr(), self.workspace.numel(), block_tables.data_ptr(),
                                     block_tables.stride(0), seq_lens.data_ptr(), self.batch, self.num_q_heads,
                                     self.num_kv_heads, self.head_dim, _stream(self.device))
        check(st, "decode_plan")
        self.table_width = block_tables.size(1)
        self.seq_lens = seq_lens
        self.block_tables = block_tables
        return self

    def stats(self) -> dict:
        """What the last ``plan`` built, read back from the workspace header (waits for the plan):
        the cost-axis positions (blocks plus kUnitCost per non-empty (sequence, head) pair), the
        worker warps the positions were cut for, the units (pieces of pairs between pair ends and
        warp starts), the split-pair entries (pairs cut across warps, plus empty pairs), the
        partial-result slots those pieces write, and the split-merge items."""
        words = self.workspace[:24].view(torch.int32).cpu().tolist()
        keys = ("items", "workers", "units", "split_pair_entries", "partial_slots", "merge_items")
        return dict(zip(keys, words))

    def matches(self, B: int, Hq: int, Hkv: int, D: int, block_table: torch.Tensor, seq_lens: torch.Tensor) -> bool:
        return ((self.batch, self.num_q_heads, self.num_kv_heads, self.head_dim) == (B, Hq, Hkv, D)
                and self.block_tables is not None and self.block_tables.data_ptr() == block_table.data_ptr()
                and self.seq_lens.data_ptr() == seq_lens.data_ptr() and self.table_width == block_table.size(1))


def flash_attn_decode(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                      block_table: torch.Tensor, cache_seqlens: torch.Tensor, softmax_scale: float | None = None,
                      out: torch.Tensor | None = None, plan: DecodePlan | None = None,
                      prefetch: bool = False, after_decode_write: bool = False) -> torch.Tensor:
    """Paged decode attention with one query token per sequence (vLLM FlashAttention decode call).

    query ``[B, Hq, D]``; key_cache/value_cache ``(N, 16, Hkv, D)`` views (any block stride);
    block_table int32 ``[B, W]``; cache_seqlens int32 ``[B]``. Returns ``out [B, Hq, D]``.
    ``plan`` must have been built for these ``cache_seqlens`` and ``W``; without one a plan is built
    on the fly (an extra launch). ``prefetch=True`` promises that the kernel launched just before
    on this stream writes neither these cache blocks nor the block table (``AEG_DECODE_PREFETCH``).
    ``after_decode_write=True`` promises that it wrote at most each sequence's newest position
    ``cache_seqlens[b] - 1`` (the decode ``reshape_and_cache_flash``) and no block table
    (``AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE``): tiles are requested early and that row is read
    again after the preceding kernel has finished.
    """
    _require_cuda(query, "query")
    if query.dim() != 3 or query.stride(2) != 1 or query.stride(1) != query.size(2):
        raise ValueError("query must be [B, Hq, D] with contiguous heads")
    _check_paged_view(key_cache, "key_cache")
    _check_paged_view(value_cache, "value_cache")
    if key_cache.shape != value_cache.shape or key_cache.stride() != value_cache.stride():
        raise ValueError("key_cache and value_cache must have the same shape and strides")
    B, Hq, D = query.shape
    Hkv = key_cache.size(2)
    if key_cache.size(3) != D:
        raise ValueError("head_dim of query and cache differ")
    if query.dtype not in _DTYPES or key_cache.dtype != query.dtype:
        raise ValueError("query and caches must share an fp16 or bf16 dtype")
    _require_cuda(block_table, "block_table")
    _require_cuda(cache_seqlens, "cache_seqlens")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.size(0) != B:
        raise ValueError("block_table must be int32 [B, W]")
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    if cache_seqlens.dtype != torch.int32 or cache_seqlens.shape != (B,):
        raise ValueError("cache_seqlens must be int32 [B]")
    cache_seqlens = cache_seqlens.contiguous()
    if out is None:
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
    else:
        _require_cuda(out, "out")
        if out.shape != query.shape or out.dtype != query.dtype or out.stride(2) != 1 or out.stride(1) != D:
            raise ValueError("out must match query's shape/dtype with contiguous heads")
    if B == 0:
        return out
    W = block_table.size(1)
    if W == 0:
        raise ValueError("block_table has no columns")
    if plan is None:
        plan = DecodePlan(B, Hq, Hkv, D, query.device).plan(cache_seqlens, block_table)
    elif not plan.matches(B, Hq, Hkv, D, block_table, cache_seqlens):
        raise ValueError("plan was built for a different batch / head layout / block tables / sequence lengths")
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    dev = query.device
    _same_device(dev, key_cache=key_cache, value_cache=value_cache, block_table=block_table,
                 cache_seqlens=cache_seqlens, out=out, plan_workspace=plan.workspace)
    with torch.cuda.device(dev):
        st = lib.aeg_paged_attn_decode(out.data_ptr(), out.stride(0), query.data_ptr(), query.stride(0),
                                       key_cache.data_ptr(), value_cache.data_ptr(), key_cache.stride(0),
                                       key_cache.size(0), block_table.data_ptr(), block_table.stride(0),
                                       cache_seqlens.data_ptr(), B, Hq, Hkv, D, scale, _DTYPES[query.dtype],
                                       plan.workspace.data_ptr(), plan.workspace.numel(),
                                       (AEG_DECODE_PREFETCH if prefetch else 0)
                                       | (AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE if after_decode_write else 0),
                                       _stream(dev))
    check(st, "paged_attention_decode")
    return out


def decode_layer_flash(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, key_cache: torch.Tensor,
                       value_cache: torch.Tensor, block_table: torch.Tensor, cache_seqlens: torch.Tensor,
                       softmax_scale: float | None = None, out: torch.Tensor | None = None,
                       plan: DecodePlan | None = None, prefetch: bool = False) -> torch.Tensor:
    """Cache write of each sequence's new token + decode attention, in one launch.

    ``key``/``value`` ``[B, Hkv, D]`` are written at position ``cache_seqlens[b] - 1`` of sequence b
    (the decode slot the reference builds, ``aegaeon/aegaeon/worker.py:628-633``), then attention runs
    over ``[0, cache_seqlens[b])``. Same result as ``reshape_and_cache_flash`` with those slots followed
    by ``flash_attn_decode``. ``prefetch`` as for ``flash_attn_decode``.
    """
    _require_cuda(query, "query")
    if query.dim() != 3 or query.stride(2) != 1 or query.stride(1) != query.size(2):
        raise ValueError("query must be [B, Hq, D] with contiguous heads")
    _check_paged_view(key_cache, "key_cache")
    _check_paged_view(value_cache, "value_cache")
    if key_cache.shape != value_cache.shape or key_cache.stride() != value_cache.stride():
        raise ValueError("key_cache and value_cache must have the same shape and strides")
    B, Hq, D = query.shape
    Hkv = key_cache.size(2)
    for name, t in (("key", key), ("value", value)):
        _require_cuda(t, name)
        if tuple(t.shape) != (B, Hkv, D) or t.stride(2) != 1 or t.stride(1) != D or t.dtype != query.dtype:
            raise ValueError(f"{name} must be [B, Hkv, D] of the query dtype with contiguous heads")
    if key_cache.size(3) != D:
        raise ValueError("head_dim of query and cache differ")
    if query.dtype not in _DTYPES or key_cache.dtype != query.dtype:
        raise ValueError("query and caches must share an fp16 or bf16 dtype")
    _require_cuda(block_table, "block_table")
    _require_cuda(cache_seqlens, "cache_seqlens")
    if block_table.dtype != torch.int32 or block_table.dim() != 2 or block_table.size(0) != B:
        raise ValueError("block_table must be int32 [B, W]")
    if block_table.stride(1) != 1:
        block_table = block_table.contiguous()
    if cache_seqlens.dtype != torch.int32 or cache_seqlens.shape != (B,):
        raise ValueError("cache_seqlens must be int32 [B]")
    cache_seqlens = cache_seqlens.contiguous()
    if out is None:
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
    elif out.shape != query.shape or out.dtype != query.dtype or out.stride(2) != 1 or out.stride(1) != D:
        raise ValueError("out must match query's shape/dtype with contiguous heads")
    if B == 0:
        return out
    if plan is None:
        plan = DecodePlan(B, Hq, Hkv, D, query.device).plan(cache_seqlens, block_table)
    elif not plan.matches(B, Hq, Hkv, D, block_table, cache_seqlens):
        raise ValueError("plan was built for a different batch / head layout / block tables / sequence lengths")
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    dev = query.device
    _same_device(dev, key=key, value=value, key_cache=key_cache, value_cache=value_cache, block_table=block_table,
                 cache_seqlens=cache_seqlens, out=out, plan_workspace=plan.workspace)
    with torch.cuda.device(dev):
        st = lib.aeg_decode_layer(out.data_ptr(), out.stride(0), query.data_ptr(), query.stride(0), key.data_ptr(),
                                  key.stride(0), value.data_ptr(), value.stride(0), key_cache.data_ptr(),
                                  value_cache.data_ptr(), key_cache.stride(0), key_cache.size(0), block_table.data_ptr(),
                                  block_table.stride(0), cache_seqlens.data_ptr(), B, Hq, Hkv, D, scale,
                                  _DTYPES[query.dtype], plan.workspace.data_ptr(), plan.workspace.numel(),
                                  AEG_DECODE_PREFETCH if prefetch else 0, _stream(dev))
    check(st, "decode_layer")
    return out


def decode_layer(out: torch.Tensor, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                 kv_cache: torch.Tensor, layer: int, block_tables: torch.Tensor, seq_lens: torch.Tensor,
                 scale: float, plan: DecodePlan | None = None, prefetch: bool = False) -> None:
    """Fused cache write + decode attention of ``layer`` over Aegaeon's ``(N, L, 2, 16, Hkv, D)`` cache."""
    kc, vc = _layer_views(kv_cache, layer)
    decode_layer_flash(query, key, value, kc, vc, block_tables, seq_lens, scale, out=out, plan=plan, prefetch=prefetch)


def paged_attention_decode(out: torch.Tensor, query: torch.Tensor, kv_cache: torch.Tensor, layer: int,
                           block_tables: torch.Tensor, seq_lens: torch.Tensor, scale: float,
                           plan: DecodePlan | None = None, prefetch: bool = False,
                           after_decode_write: bool = False) -> None:
    """Decode attention of ``layer`` over Aegaeon's ``(N, L, 2, 16, Hkv, D)`` cache, into ``out``."""
    kc, vc = _layer_views(kv_cache, layer)
    flash_attn_decode(query, kc, vc, block_tables, seq_lens, scale, out=out, plan=plan, prefetch=prefetch,
                      after_decode_write=after_decode_write)

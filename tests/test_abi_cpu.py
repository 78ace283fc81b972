"""The C-ABI library loads, exports every declared symbol, and validates on the host (no GPU)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from aegaeon_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "aegaeon_b200.h")


def _declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"AEG_API\s+[\w\s\*]+?\b(aeg_\w+)\s*\(", text)))


def test_header_declares_the_path():
    syms = _declared_symbols()
    for name in ("aeg_swap", "aeg_swap_sm", "aeg_copy_blocks", "aeg_reshape_and_cache", "aeg_decode_plan",
                 "aeg_paged_attn_decode", "aeg_decode_layer", "aeg_decode_workspace_size", "aeg_last_error", "aeg_read_device_errors"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in _declared_symbols() if s not in exported]
    assert not missing, missing
    # the Python binding covers the same set
    assert set(_native.SIGNATURES) == set(_declared_symbols())
    # nothing else leaks out of the library under the aeg_ prefix
    assert {s for s in exported if s.startswith("aeg_")} == set(_declared_symbols())


def test_version_and_workspace_size():
    lib = _native.lib
    assert lib.aeg_version() >= 100
    ws = lib.aeg_decode_workspace_size(64, 28, 4, 128)
    assert ws > 0 and ws % 256 == 0
    assert lib.aeg_decode_workspace_size(64, 28, 5, 128) == 0  # Hq not a multiple of Hkv
    assert lib.aeg_decode_workspace_size(256, 32, 4, 128) > lib.aeg_decode_workspace_size(64, 32, 4, 128)


def _fake(n=1 << 20):
    buf = (ctypes.c_uint8 * n)()
    return ctypes.addressof(buf), buf


def test_swap_rejects_out_of_range_ids_before_any_copy():
    lib = _native.lib
    dev, _k1 = _fake()
    host, _k2 = _fake()
    src = np.array([0, 5], np.int64)
    dst = np.array([1, 2], np.int64)
    st = lib.aeg_swap(dev, host, 64, 4, 4, src.ctypes.data, dst.ctypes.data, 2, 0, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT
    assert "source block id 5" in _native.last_error()
    st = lib.aeg_swap(dev, host, 64, 8, 2, src.ctypes.data, dst.ctypes.data, 2, 0, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT and "target block id 2" in _native.last_error()
    neg = np.array([-1], np.int64)
    st = lib.aeg_swap(dev, host, 64, 8, 8, neg.ctypes.data, dst.ctypes.data, 1, 1, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT
    assert lib.aeg_swap(dev, host, 64, 8, 8, src.ctypes.data, dst.ctypes.data, -1, 1, None) == 1
    assert lib.aeg_swap(dev, host, 64, 8, 8, src.ctypes.data, dst.ctypes.data, 0, 1, None) == 0  # empty: no-op


def test_decode_validation_on_host():
    lib = _native.lib
    p, _k = _fake()
    # unsupported head dim
    st = lib.aeg_decode_plan(p, 1 << 30, p, 16, p, 4, 28, 4, 64, None)
    assert st == _native.AEG_ERR_UNSUPPORTED and "head_dim" in _native.last_error()
    # GQA group too large
    st = lib.aeg_decode_plan(p, 1 << 30, p, 16, p, 4, 68, 4, 128, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT
    # misaligned workspace
    st = lib.aeg_decode_plan(p + 1, 1 << 30, p, 16, p, 4, 28, 4, 128, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT and "aligned" in _native.last_error()
    # workspace too small
    need = lib.aeg_decode_workspace_size(4, 28, 4, 128)
    aligned = (p + 255) // 256 * 256
    st = lib.aeg_decode_plan(aligned, need - 1, p, 16, p, 4, 28, 4, 128, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT and "need" in _native.last_error()
    # attention: bad dtype, misaligned cache base
    args = dict(out=p, q=p, k=p, v=p)
    st = lib.aeg_paged_attn_decode(p, 28 * 128, p, 28 * 128, p, p, 28 * 2 * 16 * 4 * 128, 64, p, 16, p, 4, 28, 4,
                                   128, 0.1, 7, aligned, need, 0, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT and "dtype" in _native.last_error()
    st = lib.aeg_paged_attn_decode(p, 28 * 128, p, 28 * 128, p + 2, p, 28 * 2 * 16 * 4 * 128, 64, p, 16, p, 4, 28, 4,
                                   128, 0.1, 0, aligned, need, 0, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT and "16-byte" in _native.last_error()
    del args


def test_reshape_and_cache_validation_on_host():
    lib = _native.lib
    p, _k = _fake()
    # token stride smaller than a row
    st = lib.aeg_reshape_and_cache(p, p, 100, 512, p, p, 16 * 512, 8, p, 4, 4, 128, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT
    # block stride smaller than 16 rows
    st = lib.aeg_reshape_and_cache(p, p, 512, 512, p, p, 512, 8, p, 4, 4, 128, None)
    assert st == _native.AEG_ERR_INVALID_ARGUMENT
    assert lib.aeg_reshape_and_cache(p, p, 512, 512, p, p, 16 * 512, 8, p, 0, 4, 128, None) == 0  # T = 0


def test_copy_blocks_validation_on_host():
    lib = _native.lib
    p, _k = _fake()
    assert lib.aeg_copy_blocks(p, 64, 8, p, p, -3, None) == _native.AEG_ERR_INVALID_ARGUMENT
    assert lib.aeg_copy_blocks(p, 64, 8, p, p, 0, None) == 0
    assert lib.aeg_copy_blocks(p, 64, 8, p + 1, p, 2, None) == _native.AEG_ERR_INVALID_ARGUMENT


def test_ops_module_imports_and_fails_loudly_without_cuda():
    import torch

    from aegaeon_b200 import ops

    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    kv = torch.zeros((4, 1, 2, 16, 4, 128), dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.copy_blocks([0], [1], kv)
    with pytest.raises(ValueError, match="CUDA"):
        ops.swap([0], [1], False, kv, torch.zeros_like(kv))


def test_operands_on_another_device_are_rejected():
    """Every operand of a launch must live on the device the work runs on; the check reads only
    each tensor's device, so it runs here with stand-ins for tensors on two GPUs."""
    import types

    import torch

    from aegaeon_b200 import ops

    on = lambda i: types.SimpleNamespace(device=torch.device("cuda", i))  # noqa: E731
    ops._same_device(torch.device("cuda", 0), key=on(0), value=on(0), out=None)
    with pytest.raises(ValueError, match="value is on cuda:1"):
        ops._same_device(torch.device("cuda", 0), key=on(0), value=on(1))


def test_migration_and_ipc_validation_on_host():
    lib = _native.lib
    p, _k1 = _fake()
    q, _k2 = _fake()
    inval = _native.AEG_ERR_INVALID_ARGUMENT
    ids = np.array([0, 1], np.int64)
    assert lib.aeg_migrate_blocks(p, 8, q, 8, 64, ids.ctypes.data, ids.ctypes.data, 0, None) == 0
    assert lib.aeg_migrate_blocks(p, 8, q, 8, 64, ids.ctypes.data, ids.ctypes.data, -1, None) == inval
    assert lib.aeg_migrate_blocks(None, 8, q, 8, 64, ids.ctypes.data, ids.ctypes.data, 2, None) == inval
    assert lib.aeg_migrate_blocks(p, 8, q, 8, 0, ids.ctypes.data, ids.ctypes.data, 2, None) == inval
    assert lib.aeg_migrate_blocks(p, 8, q, 8, 64, None, ids.ctypes.data, 2, None) == inval
    # copy-engine form: every host id is range-checked before anything is enqueued
    bad = np.array([0, 8], np.int64)
    assert lib.aeg_migrate_blocks_dma(p, 8, q, 8, 64, bad.ctypes.data, ids.ctypes.data, 2, None) == inval
    assert b"source block id 8" in lib.aeg_last_error()
    assert lib.aeg_migrate_blocks_dma(p, 8, q, 8, 64, ids.ctypes.data, bad.ctypes.data, 2, None) == inval
    assert b"target block id 8" in lib.aeg_last_error()
    # IPC handles: only this library's handles are accepted; unknown mappings cannot be closed
    out = ctypes.c_void_p()
    assert lib.aeg_ipc_open(b"\0" * _native.AEG_IPC_HANDLE_BYTES, ctypes.byref(out), None) == inval
    assert lib.aeg_ipc_close(p) == inval
    assert lib.aeg_ipc_export(None, ctypes.create_string_buffer(_native.AEG_IPC_HANDLE_BYTES)) == inval


def test_migration_ops_fail_loudly_without_cuda():
    import torch

    from aegaeon_b200 import ops

    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    kv = torch.zeros((4, 1, 2, 16, 4, 128), dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.migrate_blocks([0], [1], kv, kv)
    with pytest.raises(ValueError, match="IPC handle"):
        ops.open_kv_cache(b"short", 4, 1024)
    with pytest.raises(ValueError, match="CUDA"):
        ops.export_kv_cache(kv)


def test_segment_copy_validation_on_host():
    lib = _native.lib
    inval = _native.AEG_ERR_INVALID_ARGUMENT
    p, _k = _fake()
    o = np.array([0, 64], np.int64)
    sz = np.array([64, 64], np.int64)
    neg = np.array([0, -1], np.int64)
    assert lib.aeg_copy_segments(p, p, o.ctypes.data, o.ctypes.data, sz.ctypes.data, 0, 0, None, 0, None) == 0
    assert lib.aeg_copy_segments(p, p, o.ctypes.data, o.ctypes.data, sz.ctypes.data, -1, 0, None, 0, None) == inval
    assert lib.aeg_copy_segments(None, p, o.ctypes.data, o.ctypes.data, sz.ctypes.data, 2, 0, None, 0, None) == inval
    assert lib.aeg_copy_segments(p, p, o.ctypes.data, o.ctypes.data, sz.ctypes.data, 2, 7, None, 0, None) == inval
    assert lib.aeg_copy_segments(p, p, neg.ctypes.data, o.ctypes.data, sz.ctypes.data, 2, 0, None, 0, None) == inval
    assert lib.aeg_copy_segments(p, p, o.ctypes.data, o.ctypes.data, sz.ctypes.data, 2, 1, None, 0, None) == inval
    assert lib.aeg_copy_segments_workspace_size(10) >= 10 * 32 and lib.aeg_copy_segments_workspace_size(0) == 0


def test_tensor_segments_helper():
    import torch

    from aegaeon_b200 import ops

    storage = torch.zeros(1000, dtype=torch.uint8)
    a = storage[16:116].view(torch.float16)
    b = storage[128:128 + 40]
    offs, sizes = ops.tensor_segments([a, b], storage)
    assert offs.tolist() == [16, 128] and sizes.tolist() == [100, 40]
    with pytest.raises(ValueError):
        ops.tensor_segments([torch.zeros(4)], storage)


def test_prefill_validation_on_host():
    lib = _native.lib
    inval, unsup = _native.AEG_ERR_INVALID_ARGUMENT, _native.AEG_ERR_UNSUPPORTED
    buf = np.zeros(4096, np.int64)
    p = buf.ctypes.data  # 16-byte aligned
    args = dict(out=p, os=28 * 128, q=p, qs=28 * 128, k=p, ks=4 * 128, v=p, vs=4 * 128, cu=p, T=10, B=1, maxl=10,
                Hq=28, Hkv=4, D=128)

    def call(**kw):
        a = dict(args, **kw)
        return lib.aeg_prefill_attention(a["out"], a["os"], a["q"], a["qs"], a["k"], a["ks"], a["v"], a["vs"], a["cu"],
                                         a["T"], a["B"], a["maxl"], a["Hq"], a["Hkv"], a["D"], 0.088, 0, None)

    assert call(B=0) == 0 and call(T=0) == 0                   # nothing to do
    assert call(B=-1) == inval
    assert call(q=None) == inval
    assert call(Hq=30) == inval                                 # not a multiple of Hkv
    assert call(D=64) == unsup
    assert call(qs=100) == inval                                # stride below heads x head_dim
    assert call(q=p + 2) == inval                               # not 16-byte aligned
    assert call(ks=4 * 128 + 4) == inval                        # stride not a multiple of 8

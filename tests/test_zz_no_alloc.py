"""The allocation-free decode entry (aeg_paged_attn_decode_noalloc) against the regular one.

Both are called through the C ABI on the same inputs: the regular path as aeg_decode_plan +
aeg_paged_attn_decode with a caller-owned workspace, the allocation-free one with no workspace.
They run the same plan and kernel, so their outputs must be equal bit for bit; one case is also
checked against the oracle. Two calls in a row with different batches check that the static
scratch is re-planned and its flags reset between calls, and a rejected call must enqueue
nothing. The file name sorts last so that the suite also runs it after
every other GPU test; it passes on its own in a fresh process too.
"""
import ctypes

import numpy as np
import pytest
import torch

from aegaeon_b200 import _native
from aegaeon_b200._native import AEG_DTYPE_BF16, AEG_DTYPE_FP16, AEG_ERR_INVALID_ARGUMENT, AEG_OK
from tests.gpu_helpers import assert_attention_close, decode_case, oracle_attention_layer

pytestmark = pytest.mark.gpu

SCALE = 1.0 / np.sqrt(128)
LIB = _native.lib


def _args(out, q, kv, layer, tables, seq_lens):
    N, L, _, _, Hkv, D = kv.shape
    B, Hq, _ = q.shape
    k = kv[:, layer, 0]
    v = kv[:, layer, 1]
    dtype = AEG_DTYPE_BF16 if q.dtype == torch.bfloat16 else AEG_DTYPE_FP16
    return [out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), N,
            tables.data_ptr(), tables.stride(0), seq_lens.data_ptr(), B, Hq, Hkv, D, SCALE, dtype]


def _regular(q, kv, layer, tables, seq_lens, stream):
    B, Hq, D = q.shape
    Hkv = kv.shape[4]
    nbytes = LIB.aeg_decode_workspace_size(B, Hq, Hkv, D)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    out = torch.full_like(q, float("nan"))
    st = LIB.aeg_decode_plan(ws.data_ptr(), nbytes, tables.data_ptr(), tables.stride(0), seq_lens.data_ptr(), B, Hq,
                             Hkv, D, stream)
    assert st == AEG_OK, _native.last_error()
    st = LIB.aeg_paged_attn_decode(*_args(out, q, kv, layer, tables, seq_lens), ws.data_ptr(), nbytes, 0, stream)
    assert st == AEG_OK, _native.last_error()
    return out


def _noalloc(q, kv, layer, tables, seq_lens, stream):
    out = torch.full_like(q, float("nan"))
    st = LIB.aeg_paged_attn_decode_noalloc(*_args(out, q, kv, layer, tables, seq_lens), stream)
    assert st == AEG_OK, _native.last_error()
    return out


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _case(seed, B, Hq, Hkv, dtype, max_len):
    rng = np.random.default_rng(seed)
    seq_lens = rng.integers(1, max_len, size=B).astype(np.int32)
    seq_lens[0] = max_len  # one long sequence: its (sequence, head) pairs are split and merged
    seq_lens[1] = 0
    kv, q, tables, sl = decode_case(B, Hq, Hkv, seq_lens, dtype, seed=seed)
    dev = q.device
    return kv, q, torch.as_tensor(tables, device=dev), torch.as_tensor(sl, device=dev)


def test_noalloc_matches_regular_entry_on_two_calls_in_a_row(cuda_device):
    # Both entries run the same plan (the same worker count, hence the same cuts) and the same
    # kernel, so their outputs must agree bit for bit; the first case is also held to the
    # oracle's attention tolerance.
    stream = torch.cuda.current_stream().cuda_stream
    cases = [_case(11, 64, 28, 4, torch.float16, 3000), _case(12, 24, 32, 8, torch.bfloat16, 1800)]
    outs = []
    for kv, q, tables, sl in cases:  # back to back on one stream, no synchronisation between
        outs.append(_noalloc(q, kv, 1, tables, sl, stream))
    torch.cuda.synchronize()
    for (kv, q, tables, sl), got in zip(cases, outs):
        want = _regular(q, kv, 1, tables, sl, stream)
        torch.cuda.synchronize()
        g, w = _bits(got), _bits(want)
        assert np.array_equal(g, w), f"noalloc vs regular ({q.dtype}): {int((g != w).sum())} elements differ"
    kv, q, tables, sl = cases[0]
    want = oracle_attention_layer(q, kv[:, 1, 0], kv[:, 1, 1], tables.cpu().numpy(), sl.cpu().numpy(), SCALE)
    assert_attention_close(outs[0], want, "noalloc vs oracle")
    flags = ctypes.c_uint32(0)
    assert LIB.aeg_read_device_errors(stream, ctypes.byref(flags)) == AEG_OK
    assert flags.value == 0


def test_noalloc_rejected_call_enqueues_nothing(cuda_device):
    # A call that fails a check made after the scratch lookup (here num_blocks = 0) returns the
    # error before launching anything: its output is untouched and the next call still matches
    # the regular entry bit for bit.
    stream = torch.cuda.current_stream().cuda_stream
    kv, q, tables, sl = _case(13, 16, 28, 4, torch.float16, 900)
    out = torch.full_like(q, 7.0)
    args = _args(out, q, kv, 0, tables, sl)
    args[7] = 0  # num_blocks
    assert LIB.aeg_paged_attn_decode_noalloc(*args, stream) == AEG_ERR_INVALID_ARGUMENT
    assert "num_blocks" in _native.last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    got = _noalloc(q, kv, 0, tables, sl, stream)
    want = _regular(q, kv, 0, tables, sl, stream)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(got), _bits(want))


def test_noalloc_rejects_a_batch_beyond_the_scratch(cuda_device):
    # 40960 one-token sequences x 8 KV heads with a 16-head GQA group: 327,680 (sequence, head)
    # pairs need ~36 MB of scratch (48 bytes per pair on top of ~20 MB of partial rows), above
    # the 32 MiB the library holds. Every buffer is valid for this shape, and the call must fail
    # on the host before enqueuing anything.
    B, Hq, Hkv = 40960, 128, 8
    kv = torch.zeros((1, 1, 2, 16, Hkv, 128), dtype=torch.float16, device=cuda_device)
    q = torch.zeros((B, Hq, 128), dtype=torch.float16, device=cuda_device)
    tables = torch.zeros((B, 1), dtype=torch.int32, device=cuda_device)
    sl = torch.ones(B, dtype=torch.int32, device=cuda_device)
    out = torch.zeros_like(q)
    st = LIB.aeg_paged_attn_decode_noalloc(*_args(out, q, kv, 0, tables, sl), torch.cuda.current_stream().cuda_stream)
    assert st == AEG_ERR_INVALID_ARGUMENT
    assert "static scratch" in _native.last_error()
    torch.cuda.synchronize()
    assert int(out.abs().sum()) == 0

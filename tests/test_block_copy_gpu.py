"""swap / swap_sm / copy_blocks on the GPU: bit-exact against the oracle and the reference operator."""
import importlib.util
import os

import numpy as np
import pytest
import torch

from aegaeon_b200 import layout, ops, synth
from aegaeon_b200._native import AEG_DEVERR_BLOCK_ID_RANGE
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "aegaeon_ref_ops.so")


def _ref_ops():
    """The reference's own swap operator, compiled from its sources into oracle/_ref."""
    if not os.path.exists(REF_SO):
        pytest.skip("reference operator not built (oracle/build.py needs the reference checkout)")
    spec = importlib.util.spec_from_file_location("aegaeon_ref_ops", REF_SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _pools(n_dev, n_host, geom=(2, 2, 16, 4, 128), seed=0, pin=True, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    dev = torch.randint(-32768, 32768, (n_dev,) + geom, generator=g, dtype=torch.int32).to(torch.int16)
    host = torch.randint(-32768, 32768, (n_host,) + geom, generator=g, dtype=torch.int32).to(torch.int16)
    if pin:
        host = host.pin_memory()
    return dev.to(device).view(torch.float16), host.view(torch.float16)


def _u8(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint8).reshape(t.size(0), -1).copy()


@pytest.mark.parametrize("runs", [False, True])
def test_swap_out_and_in_bit_exact(cuda_device, runs):
    kv, host = _pools(64, 40)
    rng = np.random.default_rng(3)
    if runs:  # adjacent ids exercise the merged-transfer path
        src = list(range(10, 22)) + [40, 41, 5]
        dst = list(range(3, 15)) + [30, 31, 39]
    else:
        src = rng.permutation(64)[:20].tolist()
        dst = rng.permutation(40)[:20].tolist()
    d_ref, h_ref = _u8(kv), _u8(host)
    ops.swap(src, dst, False, kv, host)
    torch.cuda.synchronize()
    orc.c_swap(d_ref, h_ref, src, dst, False)
    assert np.array_equal(_u8(host), h_ref)
    back = rng.permutation(64)[:len(src)].tolist()
    ops.swap(dst, back, True, kv, host)
    torch.cuda.synchronize()
    orc.c_swap(d_ref, h_ref, dst, back, True)
    assert np.array_equal(_u8(kv), d_ref)


def test_swap_sm_bit_exact(cuda_device):
    kv, host = _pools(64, 40, seed=1)
    rng = np.random.default_rng(4)
    src = rng.permutation(64)[:25]
    dst = rng.permutation(40)[:25]
    d_ref, h_ref = _u8(kv), _u8(host)
    ops.swap_sm(torch.as_tensor(src), torch.as_tensor(dst), False, kv, host)
    torch.cuda.synchronize()
    orc.c_swap(d_ref, h_ref, src, dst, False)
    assert np.array_equal(_u8(host), h_ref)
    back = rng.permutation(64)[:25]
    ops.swap_sm(dst.tolist(), back.tolist(), True, kv, host)
    torch.cuda.synchronize()
    orc.c_swap(d_ref, h_ref, dst, back, True)
    assert np.array_equal(_u8(kv), d_ref)


@pytest.mark.parametrize("engine", ["dma", "sm"])
def test_swap_batched_matches_swap(cuda_device, engine):
    """The tensor-id form: CPU int64 ids for the copy engines, device ids for the SM kernel."""
    kv, host = _pools(64, 40, seed=2)
    rng = np.random.default_rng(5)
    src = torch.as_tensor(rng.permutation(64)[:30])
    dst = torch.as_tensor(rng.permutation(40)[:30])
    d_ref, h_ref = _u8(kv), _u8(host)
    ids = (src, dst) if engine == "dma" else (src.to(cuda_device), dst.to(cuda_device))
    ops.swap_batched(*ids, False, kv, host, engine=engine)
    torch.cuda.synchronize()
    orc.c_swap(d_ref, h_ref, src.numpy(), dst.numpy(), False)
    assert np.array_equal(_u8(host), h_ref)
    back = torch.as_tensor(rng.permutation(64)[:30])
    ops.swap_batched(dst, back, True, kv, host, engine=engine)
    torch.cuda.synchronize()
    orc.c_swap(d_ref, h_ref, dst.numpy(), back.numpy(), True)
    assert np.array_equal(_u8(kv), d_ref)
    with pytest.raises(ValueError, match="int64"):
        ops.swap_batched(dst.to(torch.int32), back, True, kv, host, engine=engine)
    if engine == "dma":
        with pytest.raises(ValueError, match="CPU tensors"):
            ops.swap_batched(dst.to(cuda_device), back, True, kv, host, engine="dma")


def test_swap_sm_rejects_pageable_host_pool(cuda_device):
    kv, host = _pools(8, 8, pin=False)
    with pytest.raises(ValueError, match="page-locked"):
        ops.swap_sm([0], [1], False, kv, host)


def test_swap_matches_reference_operator(cuda_device):
    ref = _ref_ops()
    kv_a, host_a = _pools(48, 32, seed=5)
    kv_b, host_b = kv_a.clone(), host_a.clone().pin_memory()
    rng = np.random.default_rng(6)
    src = rng.permutation(48)[:17].tolist()
    dst = rng.permutation(32)[:17].tolist()
    ops.swap(src, dst, False, kv_a, host_a)
    ref.swap(src, dst, False, kv_b, host_b)
    torch.cuda.synchronize()
    assert torch.equal(host_a.view(torch.int16), host_b.view(torch.int16))
    back = rng.permutation(48)[:17].tolist()
    ops.swap(dst, back, True, kv_a, host_a)
    ref.swap(dst, back, True, kv_b, host_b)
    torch.cuda.synchronize()
    assert torch.equal(kv_a.view(torch.int16), kv_b.view(torch.int16))
    # the SM-driven variant agrees with the reference operator as well
    ops.swap_sm(src, dst, False, kv_a, host_a)
    ref.swap(src, dst, False, kv_b, host_b)
    torch.cuda.synchronize()
    assert torch.equal(host_a.view(torch.int16), host_b.view(torch.int16))


def test_swap_rejects_bad_ids(cuda_device):
    kv, host = _pools(8, 4)
    with pytest.raises(ValueError, match="target block id 4"):
        ops.swap([0], [4], False, kv, host)
    with pytest.raises(ValueError, match="source block id -1"):
        ops.swap([-1], [0], True, kv, host)
    with pytest.raises(ValueError):
        ops.swap([0, 1], [0], True, kv, host)


def test_copy_blocks_bit_exact_and_reports_bad_ids(cuda_device):
    kv, _ = _pools(100, 1, geom=(3, 2, 16, 2, 128), seed=7)
    rng = np.random.default_rng(8)
    p = rng.permutation(100)
    src, dst = p[:30], p[30:60]
    ref = _u8(kv)
    ops.copy_blocks(torch.as_tensor(src), torch.as_tensor(dst), kv)
    orc.c_copy_blocks(ref, src, dst)
    assert np.array_equal(_u8(kv), ref)
    ops.read_device_errors(cuda_device)
    ops.copy_blocks([0, 500], [1, 2], kv)  # 500 is out of range: skipped and flagged
    assert ops.read_device_errors(cuda_device) & AEG_DEVERR_BLOCK_ID_RANGE
    torch.cuda.synchronize()
    assert torch.equal(kv[1].view(torch.int16), kv[0].view(torch.int16))


def test_copy_blocks_unaligned_block_bytes(cuda_device):
    # a block of 3 * 5 int16 = 30 bytes takes the byte-granular path and stays exact
    pool = torch.randint(-32768, 32768, (20, 3, 5), dtype=torch.int32).to(torch.int16).to(cuda_device)
    ref = pool.cpu().clone()
    ops.copy_blocks([1, 2, 3], [10, 11, 12], pool)
    ref[[10, 11, 12]] = ref[[1, 2, 3]]
    assert torch.equal(pool.cpu(), ref)


def test_cfg5_full_size_round_trip(cuda_device):
    """cfg5: 4096 random blocks out to pinned host, back into fresh ids; 8192 copy pairs."""
    c = synth.SWAP_CFG
    shape = (c["device_blocks"],) + layout.kv_block_shape(c["num_layers"], c["num_kv_heads"], c["head_dim"])
    kv = torch.empty(shape, dtype=c["dtype"], device=cuda_device)
    synth.random_bits_(kv, c["seed"])
    assert layout.block_bytes(kv) == 917504
    host = torch.empty((c["swap_blocks"],) + shape[1:], dtype=c["dtype"]).pin_memory()
    g = torch.Generator().manual_seed(c["seed"])
    out_ids = torch.randperm(c["device_blocks"], generator=g)[:c["swap_blocks"]]
    host_ids = torch.randperm(c["swap_blocks"], generator=g)
    in_ids = torch.randperm(c["device_blocks"], generator=g)[:c["swap_blocks"]]
    before = kv.index_select(0, out_ids.to(cuda_device)).view(torch.int16).clone()
    ops.swap(out_ids.tolist(), host_ids.tolist(), False, kv, host)
    torch.cuda.synchronize()
    # host block host_ids[i] holds device block out_ids[i]
    probe = [0, 1, 2047, 4095]
    for i in probe:
        assert torch.equal(host[host_ids[i]].view(torch.int16), before[i].cpu())
    ops.swap(host_ids.tolist(), in_ids.tolist(), True, kv, host)
    after = kv.index_select(0, in_ids.to(cuda_device)).view(torch.int16)
    assert torch.equal(after, before)
    del before, after
    # copy_blocks over disjoint pairs
    p = torch.randperm(c["device_blocks"], generator=g)
    src, dst = p[:c["copy_pairs"]].to(cuda_device), p[c["copy_pairs"]:2 * c["copy_pairs"]].to(cuda_device)
    want = kv.index_select(0, src).view(torch.int16).clone()
    ops.copy_blocks(src, dst, kv)
    assert torch.equal(kv.index_select(0, dst).view(torch.int16), want)
    del kv, want
    torch.cuda.empty_cache()

"""reshape_and_cache on the GPU: bit-exact against the CPU oracle."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import ops, synth
from aegaeon_b200._native import AEG_DEVERR_SLOT_RANGE
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("Hkv", [1, 4, 8, 40])
def test_reshape_and_cache_bit_exact(cuda_device, dtype, Hkv):
    N, L, T = 24, 3, 37
    rng = np.random.default_rng(Hkv)
    kv = torch.randint(-32768, 32768, (N, L, 2, 16, Hkv, 128), dtype=torch.int32).to(torch.int16)
    kv_dev = kv.to(cuda_device).view(dtype)
    key = torch.randint(-32768, 32768, (T, Hkv, 128), dtype=torch.int32).to(torch.int16)
    val = torch.randint(-32768, 32768, (T, Hkv, 128), dtype=torch.int32).to(torch.int16)
    slots = torch.as_tensor(rng.permutation(N * 16)[:T].astype(np.int64))
    slots[3] = -1
    slots[10] = -7
    layer = 1
    ops.reshape_and_cache(key.to(cuda_device).view(dtype), val.to(cuda_device).view(dtype), kv_dev, layer,
                          slots.to(cuda_device))
    ref = kv.numpy().view(np.uint16).copy()
    orc.np_reshape_and_cache(key.numpy().view(np.uint16), val.numpy().view(np.uint16), ref[:, layer, 0],
                             ref[:, layer, 1], slots.numpy())
    assert np.array_equal(_bits(kv_dev), ref)


def test_strided_key_value_views(cuda_device):
    # key/value as views into a fused qkv projection output [T, (Hq + 2 Hkv) * D]
    T, Hq, Hkv, N = 9, 28, 4, 10
    qkv = torch.randn((T, (Hq + 2 * Hkv) * 128), device=cuda_device).half()
    key = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    val = qkv[:, (Hq + Hkv) * 128:].view(T, Hkv, 128)
    caches = torch.zeros((2, N, 16, Hkv, 128), device=cuda_device, dtype=torch.float16)
    slots = torch.arange(5, 5 + T, device=cuda_device, dtype=torch.int64) * 7 % (N * 16)
    ops.reshape_and_cache_flash(key, val, caches[0], caches[1], slots)
    s = slots.cpu()
    for t in range(T):
        assert torch.equal(caches[0, s[t] // 16, s[t] % 16], key[t])
        assert torch.equal(caches[1, s[t] // 16, s[t] % 16], val[t])
    # odd element offsets take the 2-byte path and stay exact
    qkv2 = torch.randn((T, (Hq + 2 * Hkv) * 128 + 1), device=cuda_device).half()
    key2 = qkv2[:, 1:1 + Hkv * 128].view(T, Hkv, 128)
    ops.reshape_and_cache_flash(key2, key2, caches[0], caches[1], slots)
    for t in range(T):
        assert torch.equal(caches[0, s[t] // 16, s[t] % 16], key2[t])


def test_out_of_range_slot_is_skipped_and_reported(cuda_device):
    ops.read_device_errors(cuda_device)
    N = 4
    caches = torch.zeros((2, N, 16, 4, 128), device=cuda_device, dtype=torch.float16)
    key = torch.ones((2, 4, 128), device=cuda_device, dtype=torch.float16)
    slots = torch.tensor([N * 16, 3], device=cuda_device, dtype=torch.int64)
    ops.reshape_and_cache_flash(key, key, caches[0], caches[1], slots)
    assert ops.read_device_errors(cuda_device) & AEG_DEVERR_SLOT_RANGE
    assert caches[0, 0, 3].eq(1).all() and caches.sum().item() == 2 * 4 * 128


def test_cfg2_decode_step_writes(cuda_device):
    # cfg2 geometry at full pool size: each of the 28 layers writes one token per sequence.
    cfg = synth.CONFIGS["cfg2"]
    lay = synth.make_layout(cfg)
    kv = torch.zeros((lay.num_blocks, cfg.num_layers, 2, 16, 4, 128), dtype=cfg.dtype, device=cuda_device)
    slots = torch.as_tensor(synth.new_token_slots(lay), device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    for layer in range(cfg.num_layers):
        k = torch.randn((cfg.batch, 4, 128), generator=g, device=cuda_device).half()
        v = torch.randn((cfg.batch, 4, 128), generator=g, device=cuda_device).half()
        ops.reshape_and_cache(k, v, kv, layer, slots)
        blk = slots // 16
        off = slots % 16
        assert torch.equal(kv[blk, layer, 0, off], k)
        assert torch.equal(kv[blk, layer, 1, off], v)
    # exactly 2 * 28 * 64 rows were written
    nz = (kv.view(torch.int16) != 0).view(lay.num_blocks, cfg.num_layers, 2, 16, -1).any(-1).sum().item()
    assert nz == 2 * cfg.num_layers * cfg.batch

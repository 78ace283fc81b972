"""Model-weight switch (``ops.copy_segments``): a synthetic parameter list packed into a page-locked
host model cache is copied into a device arena in one call, bit-exact against the reference's
per-parameter loop (``new_storage.copy_(param.untyped_storage(), non_blocking=True)``,
aegaeon/aegaeon/worker.py:358-365) run with torch on the same inputs."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import ops

pytestmark = pytest.mark.gpu


def _packed(sizes, align, rng, jitter=False):
    offs, top = [], 0
    for n in sizes:
        top = (top + align - 1) // align * align
        if jitter and rng.random() < 0.3:
            top += int(rng.integers(1, 15))  # unaligned placements exercise the byte path
        offs.append(top)
        top += n
    return np.asarray(offs, np.int64), top


def _model(rng, jitter):
    # a few large matrices, odd-sized vectors and tiny tensors, like a transformer's parameters
    sizes = [int(x) for x in rng.integers(1, 4096, 40)] + [2 * 3584, 2 * 512, 3] + \
            [int(x) for x in rng.integers(1 << 16, 1 << 21, 12)]
    rng.shuffle(sizes)
    src_off, src_total = _packed(sizes, 16, rng, jitter)
    dst_off, dst_total = _packed(sizes, 16, rng, jitter)
    return np.asarray(sizes, np.int64), src_off, src_total, dst_off, dst_total


@pytest.mark.parametrize("engine", ["dma", "sm"])
@pytest.mark.parametrize("jitter", [False, True])
def test_weight_switch_matches_per_parameter_copies(cuda_device, engine, jitter):
    rng = np.random.default_rng(17 + jitter)
    sizes, so, s_total, do, d_total = _model(rng, jitter)
    cache = torch.from_numpy(rng.integers(0, 256, s_total, dtype=np.uint8)).pin_memory()
    arena = torch.zeros(d_total + 64, dtype=torch.uint8, device=cuda_device)
    want = torch.zeros_like(arena)
    for a, b, n in zip(so, do, sizes):  # the reference's loop
        want[b:b + n].copy_(cache[a:a + n], non_blocking=True)
    ops.copy_segments(arena, cache, so, do, sizes, engine=engine)
    torch.cuda.synchronize()
    assert torch.equal(arena, want)


def test_weight_switch_device_to_device(cuda_device):
    rng = np.random.default_rng(5)
    sizes, so, s_total, do, d_total = _model(rng, True)
    src = torch.from_numpy(rng.integers(0, 256, s_total, dtype=np.uint8)).to(cuda_device)
    arena = torch.zeros(d_total, dtype=torch.uint8, device=cuda_device)
    ops.copy_segments(arena, src, so, do, sizes, engine="sm")
    torch.cuda.synchronize()
    for a, b, n in zip(so, do, sizes):
        assert torch.equal(arena[b:b + n], src[a:a + n])


def test_weight_switch_rejects_bad_segments(cuda_device):
    cache = torch.zeros(1024, dtype=torch.uint8).pin_memory()
    arena = torch.zeros(1024, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="past the end"):
        ops.copy_segments(arena, cache, [0], [1000], [100])
    pageable = torch.zeros(1024, dtype=torch.uint8)
    with pytest.raises(ValueError, match="pageable"):
        ops.copy_segments(arena, pageable, [0], [0], [100], engine="sm")

"""Streams: the swap contract of the reference's worker and attention beside other grids.

* The reference runs ``ops.swap`` under ``torch.cuda.stream(swap_in/out_stream)`` and then
  records an interprocess event on that stream (``aegaeon/aegaeon/worker.py:739-765``); swap-in,
  swap-out and compute run on three streams (``worker.py:152-154``). The first tests show that
  the copy is enqueued on the current stream: it waits behind earlier work of that stream, the
  default stream does not wait for it, and an interprocess event recorded after it completes
  only when the copy has landed.
* Decode attention's split merge waits for other CTAs of its own grid. These tests run it while
  swap_sm and copy_blocks occupy the GPU from two other streams, and as two grids with two
  workspaces on two streams (the library orders such launches so that each grid starts only
  after the previous one is fully resident): the outputs must equal a solo run bit for bit and no
  bounded wait may time out.
"""
import time

import numpy as np
import pytest
import torch

from aegaeon_b200 import layout, ops, synth
from aegaeon_b200._native import AEG_DEVERR_WAIT_TIMEOUT
from tests.gpu_helpers import decode_case

pytestmark = pytest.mark.gpu

SLEEP_CYCLES = int(4e8)  # ~0.2 s of device time at B200 clocks


def _warm_kernels(device):
    """Runs once every kernel the ordering checks launch (on scratch pools of their own), so that
    no lazy module load (which waits for the device) happens while the swap stream is busy."""
    torch.cuda._sleep(1000)
    marker = torch.ones(1, device=device)
    marker += 1
    dev, host = _pools(2, 2, seed=1)
    ids = torch.as_tensor([0], device=device)
    ops.swap_sm(ids, ids, False, dev, host)
    ops.swap_sm(ids, ids, True, dev, host)
    torch.cuda.synchronize()


def _pools(n_dev, n_host, seed):
    geom = layout.kv_block_shape(28, 4, 128)
    dev = synth.random_bits_(torch.empty((n_dev,) + geom, dtype=torch.float16, device="cuda"), seed)
    host = torch.zeros((n_host,) + geom, dtype=torch.float16).pin_memory()
    return dev, host


@pytest.mark.parametrize("engine", ["dma", "sm"])
def test_swap_out_is_ordered_on_the_current_stream(cuda_device, engine):
    kv, host = _pools(64, 48, seed=21)
    rng = np.random.default_rng(21)
    src = rng.permutation(64)[:40].tolist()
    dst = rng.permutation(48)[:40].tolist()
    # swap_sm takes its ids from device tensors staged before the stream work (a list would be
    # copied from pageable memory, which may make the host wait for the stream)
    d_src, d_dst = torch.as_tensor(src, device=cuda_device), torch.as_tensor(dst, device=cuda_device)
    _warm_kernels(cuda_device)
    before = host.view(torch.int16).clone()
    swap_stream = torch.cuda.Stream()
    with torch.cuda.stream(swap_stream):
        torch.cuda._sleep(SLEEP_CYCLES)  # earlier work on the swap stream
        if engine == "dma":
            ops.swap(src, dst, False, kv, host)
        else:
            ops.swap_sm(d_src, d_dst, False, kv, host)
        done = torch.cuda.Event(interprocess=True)
        done.record(swap_stream)
    assert len(bytes(done.ipc_handle())) > 0  # shareable with the engine's other processes
    # The default stream does not wait for the swap stream ...
    marker = torch.ones(1, device=cuda_device)
    marker += 1
    torch.cuda.current_stream().synchronize()
    # ... and the copy has not run yet: it is queued behind the sleep on the swap stream.
    assert not done.query()
    assert torch.equal(host.view(torch.int16), before)
    done.synchronize()
    want = kv.view(torch.int16).cpu()
    got = host.view(torch.int16)
    for s, d in zip(src, dst):
        assert torch.equal(got[d], want[s])


def test_swap_in_is_ordered_on_the_current_stream(cuda_device):
    kv, host = _pools(64, 48, seed=22)
    host.view(torch.int16).copy_(torch.randint(-32768, 32768, host.shape, dtype=torch.int32).to(torch.int16))
    rng = np.random.default_rng(22)
    src = rng.permutation(48)[:32].tolist()
    dst = rng.permutation(64)[:32].tolist()
    before = kv.view(torch.int16).clone()
    _warm_kernels(cuda_device)
    swap_stream = torch.cuda.Stream()
    with torch.cuda.stream(swap_stream):
        torch.cuda._sleep(SLEEP_CYCLES)
        ops.swap(src, dst, True, kv, host)
        done = torch.cuda.Event(interprocess=True)
        done.record(swap_stream)
    # A copy of the cache on the default stream sees the blocks before the swap-in.
    snap = kv.view(torch.int16).clone()
    torch.cuda.current_stream().synchronize()
    assert not done.query()
    assert torch.equal(snap, before)
    done.synchronize()
    got = kv.view(torch.int16).cpu()
    for s, d in zip(src, dst):
        assert torch.equal(got[d], host.view(torch.int16)[s])


def _decode_inputs(seed, B=64, Hq=28, Hkv=4, L=4, dtype=torch.float16):
    rng = np.random.default_rng(seed)
    seq = np.clip(np.round(rng.lognormal(5.5, 1.0, B)), 4, 3000).astype(np.int32)
    kv, q, tables, sl = decode_case(B, Hq, Hkv, seq, dtype, num_layers=L, seed=seed)
    dev = q.device
    return kv, q, torch.as_tensor(tables, device=dev), torch.as_tensor(sl, device=dev)


def _decode_layers(plan, kv, q, tables, sl, outs, scale):
    for l in range(kv.size(1)):
        ops.paged_attention_decode(outs[l], q, kv, l, tables, sl, scale, plan=plan)


def test_decode_beside_swap_and_copy_blocks_on_other_streams(cuda_device):
    scale = 128 ** -0.5
    kv, q, tables, sl = _decode_inputs(31)
    L = kv.size(1)
    plan = ops.DecodePlan(q.size(0), q.size(1), kv.size(4), 128).plan(sl, tables)
    solo = [torch.empty_like(q) for _ in range(L)]
    _decode_layers(plan, kv, q, tables, sl, solo, scale)
    torch.cuda.synchronize()

    pool, host = _pools(2048, 1024, seed=32)
    rng = np.random.default_rng(33)
    dev = cuda_device
    out_ids = torch.as_tensor(rng.permutation(2048)[:1024], device=dev)
    host_ids = torch.as_tensor(rng.permutation(1024), device=dev)
    perm = rng.permutation(2048)
    copy_src, copy_dst = torch.as_tensor(perm[:1024], device=dev), torch.as_tensor(perm[1024:], device=dev)
    want_pool = pool.view(torch.int16).clone()
    s_swap, s_copy = torch.cuda.Stream(), torch.cuda.Stream()

    def timed_decode(outs):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            _decode_layers(plan, kv, q, tables, sl, outs, scale)
        b.record()
        return a, b

    outs = [torch.empty_like(q) for _ in range(L)]
    a0, b0 = timed_decode(outs)
    torch.cuda.synchronize()
    alone_ms = a0.elapsed_time(b0)
    s_swap.wait_stream(torch.cuda.current_stream())
    s_copy.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_swap):
        ops.swap_sm(out_ids, host_ids, False, pool, host)
    with torch.cuda.stream(s_copy):
        ops.copy_blocks(copy_src, copy_dst, pool)
    t0 = time.perf_counter()
    a1, b1 = timed_decode(outs)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    beside_ms = a1.elapsed_time(b1)
    print(f"\ndecode x{5 * L}: alone {alone_ms:.3f} ms, beside swap_sm + copy_blocks {beside_ms:.3f} ms "
          f"(wall {wall * 1e3:.1f} ms)")
    for l in range(L):
        assert torch.equal(outs[l].view(torch.int16), solo[l].view(torch.int16)), f"layer {l} differs"
    assert ops.read_device_errors() & AEG_DEVERR_WAIT_TIMEOUT == 0
    # the copies themselves are exact
    want_pool[copy_dst] = want_pool[copy_src]
    assert torch.equal(pool.view(torch.int16), want_pool)
    got_host = host.view(torch.int16)
    ref_rows = want_pool.cpu()  # swap-out read the pool before or after copy_blocks: check only untouched ids
    touched = set(copy_dst.tolist())
    for s, d in zip(out_ids.tolist(), host_ids.tolist()):
        if s not in touched:
            assert torch.equal(got_host[d], ref_rows[s])
    assert wall < 1.0, "a bounded wait ran long"


def test_two_decode_grids_on_two_streams(cuda_device):
    scale = 128 ** -0.5
    cases = [_decode_inputs(41, B=64), _decode_inputs(42, B=48, Hq=32, Hkv=8, dtype=torch.bfloat16)]
    plans, solos = [], []
    for kv, q, tables, sl in cases:
        plan = ops.DecodePlan(q.size(0), q.size(1), kv.size(4), 128).plan(sl, tables)
        solo = [torch.empty_like(q) for _ in range(kv.size(1))]
        _decode_layers(plan, kv, q, tables, sl, solo, scale)
        plans.append(plan)
        solos.append(solo)
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [[torch.empty_like(c[1]) for _ in range(c[0].size(1))] for c in cases]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    t0 = time.perf_counter()
    for rep in range(6):  # alternate launches between the streams, nothing ordering them
        for i in range(2):
            kv, q, tables, sl = cases[i]
            with torch.cuda.stream(streams[i]):
                for l in range(kv.size(1)):
                    ops.paged_attention_decode(outs[i][l], q, kv, l, tables, sl, scale, plan=plans[i])
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    print(f"\n2 streams x 6 reps x 4 layers: {wall * 1e3:.1f} ms wall")
    for i in range(2):
        for l in range(len(outs[i])):
            assert torch.equal(outs[i][l].view(torch.int16), solos[i][l].view(torch.int16)), f"case {i} layer {l}"
    assert ops.read_device_errors() & AEG_DEVERR_WAIT_TIMEOUT == 0
    assert wall < 1.0, "a bounded wait ran long"

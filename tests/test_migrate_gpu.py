"""GPU <-> GPU KV block migration (``ops.migrate_blocks``), bit-exact.

The oracle of a whole-block byte copy is the copy itself: ``expected = target.clone();
expected[dst] = source[src]`` in torch indexing, compared through int16 views (any bit pattern,
NaN encodings included). Cases: two pools on one GPU, a pull from a peer GPU of the same
process, and the reference's cross-process form (the target engine opens the source engine's
pool through an IPC handle, aegaeon/aegaeon/worker.py:841-872), as a pull and as a push, on
one GPU or on two when the box has them. Migrated blocks then serve decode attention exactly as
the originals did.
"""
import multiprocessing as mp
import queue as queue_mod

import numpy as np
import pytest
import torch

from aegaeon_b200 import ops
from aegaeon_b200.layout import block_bytes
from tests.gpu_helpers import make_tables

pytestmark = pytest.mark.gpu

BLOCK = (3, 2, 16, 2, 128)  # (L, 2, 16, Hkv, D) of one block: 48 KiB
N_SRC, N_DST = 48, 40
TIMEOUT = 180


def _pool(device, seed: int, n: int) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    bits = torch.randint(-32768, 32768, (n,) + BLOCK, generator=g, device=device, dtype=torch.int32)
    return bits.to(torch.int16).view(torch.float16)


def _expect(target: torch.Tensor, source: torch.Tensor, src, dst) -> torch.Tensor:
    exp = target.clone()
    exp[torch.as_tensor(dst, device=target.device)] = source.to(target.device)[torch.as_tensor(src, device=target.device)]
    return exp


def _same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    return torch.equal(a.view(torch.int16).cpu(), b.view(torch.int16).cpu())


def _ids(seed: int, n: int):
    rng = np.random.default_rng(seed)
    return rng.choice(N_SRC, n, replace=False).astype(np.int64), rng.choice(N_DST, n, replace=False).astype(np.int64)


@pytest.mark.parametrize("engine", ["sm", "dma"])
def test_migrate_between_pools_on_one_gpu(cuda_device, engine):
    src_pool = _pool(cuda_device, 1, N_SRC)
    dst_pool = _pool(cuda_device, 2, N_DST)
    src, dst = _ids(3, 25)
    want = _expect(dst_pool, src_pool, src, dst)
    ops.migrate_blocks(src.tolist(), dst.tolist(), src_pool, dst_pool, engine=engine)
    torch.cuda.synchronize()
    assert _same_bits(dst_pool, want)
    assert ops.read_device_errors(cuda_device) == 0


def test_migrate_skips_out_of_range_device_ids(cuda_device):
    src_pool = _pool(cuda_device, 4, N_SRC)
    dst_pool = _pool(cuda_device, 5, N_DST)
    before = dst_pool.clone()
    ops.migrate_blocks([0, N_SRC], [1, 2], src_pool, dst_pool)  # second pair: source id out of range
    torch.cuda.synchronize()
    want = before.clone()
    want[1] = src_pool[0]
    assert _same_bits(dst_pool, want)
    assert ops.read_device_errors(cuda_device) & 0x1
    with pytest.raises(ValueError, match="source block id"):
        ops.migrate_blocks([0, N_SRC], [1, 2], src_pool, dst_pool, engine="dma")


def test_migrated_blocks_serve_attention_unchanged(cuda_device):
    """A batch's blocks moved to new ids in another pool give bit-identical decode attention."""
    L, Hkv, D, Hq, B = 2, 4, 128, 28, 6
    g = torch.Generator(device=cuda_device).manual_seed(7)
    src_pool = torch.randn((64, L, 2, 16, Hkv, D), generator=g, device=cuda_device).half()
    dst_pool = torch.randn((80, L, 2, 16, Hkv, D), generator=g, device=cuda_device).half()
    seq_lens = np.array([5, 17, 100, 33, 250, 1], np.int32)
    t_src = make_tables(seq_lens, 64, 11)
    t_dst = make_tables(seq_lens, 80, 12, width=t_src.shape[1])
    nb = (seq_lens + 15) // 16
    src_ids = np.concatenate([t_src[i, :nb[i]] for i in range(B)]).astype(np.int64)
    dst_ids = np.concatenate([t_dst[i, :nb[i]] for i in range(B)]).astype(np.int64)
    ops.migrate_blocks(src_ids, dst_ids, src_pool, dst_pool)
    q = torch.randn((B, Hq, D), generator=g, device=cuda_device).half()
    lens = torch.as_tensor(seq_lens, device=cuda_device)
    for layer in range(L):
        a = torch.empty_like(q)
        b = torch.empty_like(q)
        ops.paged_attention_decode(a, q, src_pool, layer, torch.as_tensor(t_src, device=cuda_device), lens, D ** -0.5)
        ops.paged_attention_decode(b, q, dst_pool, layer, torch.as_tensor(t_dst, device=cuda_device), lens, D ** -0.5)
        torch.cuda.synchronize()
        assert _same_bits(a, b), layer


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("engine", ["sm", "dma"])
def test_migrate_pulls_from_a_peer_gpu_in_process(engine):
    target_dev, source_dev = torch.device("cuda", 0), torch.device("cuda", 1)
    src_pool = _pool(source_dev, 6, N_SRC)
    dst_pool = _pool(target_dev, 7, N_DST)
    src, dst = _ids(8, 30)
    want = _expect(dst_pool, src_pool, src, dst)
    ops.migrate_blocks(src, dst, src_pool, dst_pool, engine=engine)
    torch.cuda.synchronize(target_dev)
    assert _same_bits(dst_pool, want)
    assert ops.read_device_errors(target_dev) == 0


# ---- cross-process: the exporting engine runs in a child process --------------------------

def _exporter(device_index: int, to_parent, from_parent) -> None:
    """Child: owns a pool, exports it, and checks the blocks the parent pushes into it."""
    try:
        dev = torch.device("cuda", device_index)
        torch.cuda.set_device(dev)
        pool = _pool(dev, 21, N_SRC)
        torch.cuda.synchronize(dev)
        to_parent.put(("handle", ops.export_kv_cache(pool), pool.size(0), block_bytes(pool)))
        msg = from_parent.get(timeout=TIMEOUT)
        assert msg[0] == "pushed"
        _, dst, blocks = msg
        want = _pool(dev, 21, N_SRC)
        want[torch.as_tensor(dst, device=dev)] = torch.from_numpy(blocks).to(dev).view(torch.float16)
        torch.cuda.synchronize(dev)
        to_parent.put(("checked", _same_bits(pool, want)))
        assert from_parent.get(timeout=TIMEOUT)[0] == "bye"  # the parent has closed its mapping
    except Exception as e:  # reported to the parent, which fails the test
        to_parent.put(("error", repr(e)))


def test_migrate_through_ipc_handles_across_processes():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    peer = 1 if torch.cuda.device_count() >= 2 else 0
    ctx = mp.get_context("spawn")
    to_parent, from_parent = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_exporter, args=(peer, to_parent, from_parent), daemon=True)
    child.start()
    try:
        msg = to_parent.get(timeout=TIMEOUT)
        assert msg[0] == "handle", msg
        _, handle, n_blocks, bb = msg
        dev = torch.device("cuda", 0)
        local = _pool(dev, 22, N_DST)
        remote_init = _pool(dev, 21, N_SRC)  # the child's pool, regenerated from its seed
        with ops.open_kv_cache(handle, n_blocks, bb) as remote:
            for i, engine in enumerate(("sm", "dma")):  # pull, as the reference's target engine does
                src, dst = _ids(30 + i, 20)
                want = _expect(local, remote_init, src, dst)
                ops.migrate_blocks(src, dst, remote, local, engine=engine)
                torch.cuda.synchronize(dev)
                assert _same_bits(local, want), engine
            # push: this process writes blocks of its own pool into the mapped one
            rng = np.random.default_rng(40)
            src = rng.choice(N_DST, 12, replace=False).astype(np.int64)
            dst = rng.choice(N_SRC, 12, replace=False).astype(np.int64)
            ops.migrate_blocks(src, dst, local, remote)
            torch.cuda.synchronize(dev)
            blocks = local[torch.as_tensor(src, device=dev)].view(torch.int16).cpu().numpy()
            from_parent.put(("pushed", dst, blocks))
            msg = to_parent.get(timeout=TIMEOUT)
            assert msg == ("checked", True), msg
        assert ops.read_device_errors(dev) == 0
        from_parent.put(("bye",))
        child.join(timeout=TIMEOUT)
        assert child.exitcode == 0
    finally:
        if child.is_alive():
            child.kill()
            child.join(timeout=30)
    try:
        extra = to_parent.get_nowait()
        assert extra[0] != "error", extra
    except queue_mod.Empty:
        pass

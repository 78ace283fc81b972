"""Multi-rank host logic on CPU (gloo, world size 2): per-request sharding and max-over-ranks timing.

Decode attention shards per request (sequence i -> rank i mod N, each rank with its own block
pool); there is no data-path collective. These tests run two gloo ranks on the host: each rank
builds its shard of a synthetic layout, computes its sequences with the CPU oracle, and the
gathered result must equal the single-rank computation of the whole batch. The bench's
max-over-ranks reduction and a rank that fails before the collective are also covered.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiny_cfg():
    from aegaeon_b200 import synth

    return synth.DecodeConfig("tiny", 10, 8, 2, 128, 1, torch.float16, ("uniform", 1, 90), None, 1.0, 7, "tiny")


def _rank_outputs(cfg, rank, world):
    """Oracle attention of this rank's shard; values depend only on the global sequence id."""
    from aegaeon_b200 import synth
    from oracle import oracle as orc

    lay = synth.make_layout(cfg, rank, world)
    N = lay.num_blocks
    Hkv, D, Hq = cfg.num_kv_heads, cfg.head_dim, cfg.num_q_heads
    kb = np.zeros((N, 16, Hkv, D), np.uint16)
    vb = np.zeros((N, 16, Hkv, D), np.uint16)
    q = np.zeros((len(lay.seq_ids), Hq, D), np.uint16)
    for i, sid in enumerate(lay.seq_ids):
        rng = np.random.default_rng(1000 + int(sid))
        n = int(lay.seq_lens[i])
        ks = orc.f64_to_bits(rng.standard_normal((n, Hkv, D)), orc.FP16)
        vs = orc.f64_to_bits(rng.standard_normal((n, Hkv, D)), orc.FP16)
        for j in range(n):
            blk = lay.block_tables[i, j // 16]
            kb[blk, j % 16] = ks[j]
            vb[blk, j % 16] = vs[j]
        q[i] = orc.f64_to_bits(rng.standard_normal((Hq, D)), orc.FP16)
    out = orc.c_paged_attention(q, kb.reshape(-1), vb.reshape(-1), 16 * Hkv * D, lay.block_tables, lay.seq_lens, Hkv,
                                0.0883883, orc.FP16, 1)
    return lay.seq_ids, out


def _worker(rank, world, port, result_path):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _tiny_cfg()
        ids, out = _rank_outputs(cfg, rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, (ids, out))
        import bench

        t = bench._max_over_ranks(1.0 + rank, world, torch.device("cpu"))
        if rank == 0:
            np.savez(result_path, t=t, **{f"ids{r}": g[0] for r, g in enumerate(gathered)},
                     **{f"out{r}": g[1] for r, g in enumerate(gathered)})
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_matches_single_rank(tmp_path):
    world = 2
    path = str(tmp_path / "res.npz")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, start_method="spawn")
    res = np.load(path)
    assert float(res["t"]) == 2.0  # max over ranks
    cfg = _tiny_cfg()
    ids_all, out_all = _rank_outputs(cfg, 0, 1)
    merged = np.zeros_like(out_all)
    seen = []
    for r in range(world):
        for k, sid in enumerate(res[f"ids{r}"]):
            merged[int(sid)] = res[f"out{r}"][k]
            seen.append(int(sid))
    assert sorted(seen) == list(range(cfg.batch))
    assert np.array_equal(merged, out_all)


def _failing_worker(rank, world, port):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("rank 1 failed before the timing reduction")
        t = torch.tensor([1.0])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # rank 0 must not hang: the group times out
    finally:
        dist.destroy_process_group()


def test_failed_rank_surfaces_as_error_not_hang():
    with pytest.raises(Exception):
        mp.start_processes(_failing_worker, args=(2, _free_port()), nprocs=2, start_method="spawn")

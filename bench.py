#!/usr/bin/env python
"""Benchmark of the Aegaeon per-token serving hot path on B200.

Default workload (``--config cfg3``, the largest single-GPU decode configuration that BASELINE.json
splits across 1/2/4/8 GPUs): one Yi-1.5-9B-shaped decode step = 48 layers x (reshape_and_cache of
one new token per sequence + paged decode attention), batch 256, bf16, contexts
round(lognormal(6, 1)) in [4, 8192]. Under torchrun the batch is split i mod N over the ranks,
each with its own block pool (strong scaling, no collective on the data path). A step is captured
once as a CUDA graph and replayed; the K/V read per step (16.7 GB at N=1) is far larger than the
126 MB L2, so no flush is needed.

One JSON line on rank 0 with the step throughput, the dominant kernel's roofline (in the step, as
an isolated launch, and after a QKV-shaped GEMM as in the model's forward), the end-to-end number
through the public step API, the host link (one GPU and all ranks at once), the cfg5 KV-block swap
set beside the reference's own swap operator built from its sources, a cross-GPU migration check
(N >= 2), the fp32 torch CPU baseline and, at N = 1, the per-layer figures of the other decode
configurations (cfg1, cfg2, cfg4) and compact figures of the prefill, step-input and weight-switch
rows (each also a --config of its own) on the same GPU.

``--impl reference`` times the reference path's CPU restatement (oracle/torch_ref.py, fp32 torch,
all host threads) on whole L-layer steps of a bounded sample of the same workload, with the same
steps, warm-up and config; for ``--config cfg5`` it times the reference's own swap operator.
Other configs: cfg1/cfg2/cfg4 (decode), cfg5 (swap / copy_blocks), migrate, prep, weights, prefill.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="cfg3", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "migrate", "prep", "weights", "prefill"])
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    p.add_argument("--no-swap", action="store_true", help="decode configs: skip the swap-set leg")
    p.add_argument("--no-other-configs", action="store_true",
                   help="cfg3 at N = 1: skip the per-layer figures of cfg1, cfg2 and cfg4 and the prefill, "
                        "step-input and weight-switch figures")
    p.add_argument("--swap-scale", type=float, default=1.0, help="decode configs: scale the swap set (small cases)")
    p.add_argument("--unfused", action="store_true",
                   help="run each layer as reshape_and_cache + paged_attention_decode (two operators)")
    p.add_argument("--split", choices=["mod", "balanced"], default="mod",
                   help="cfg3 under torchrun: sequence i on rank i mod N (default), or shares of about equal context")
    p.add_argument("--layers", type=int, default=0,
                   help="decode configs, profiling only: override the layer count (same work per launch, smaller pool)")
    p.add_argument("--compact-pool", action="store_true",
                   help="size the block pool to the blocks the batch uses (same kernels; small-case profiling)")
    p.add_argument("--scale", type=float, default=1.0,
                   help="cfg5 / migrate only: scale the pool and the moved block counts (small cases)")
    p.add_argument("--profile-run", action="store_true",
                   help="timed graph replays only: no clock pre-roll, per-launch timing, end-to-end or CPU leg")
    return p.parse_args()


def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s earlier pool measurement)"


def _ncu_traffic(kernel_key: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == kernel_key:
                return float(parts[1])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------------------------------
# Clock sampling (nvidia-smi during the timed region)

_CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, device: torch.device):
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ident, f"--query-gpu={_CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "nvidia-smi unavailable"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "no samples"}
        pmax = max(r["power"] for r in rows)
        load = [r for r in rows if r["power"] >= 0.5 * pmax] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("swp", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(load),
                "power_w_max": pmax}


# ------------------------------------------------------------------------------------------
# The workload description shared by both arms (the reference arm prints the same dict)


def _decode_layout(cfg, world: int, rank: int, split: str = "mod"):
    """This rank's share of a decode config: cfg3 splits its batch over the ranks (strong scaling;
    by default sequence i on rank i mod N, the split BASELINE.json names); the others run the
    whole batch on every rank."""
    from aegaeon_b200 import synth

    if cfg.name == "cfg3":
        return synth.make_layout(cfg, rank, world, split), "strong"
    return synth.make_layout(cfg), "weak"


def _ctx_desc(cfg) -> str:
    d = cfg.ctx_dist
    if d[0] == "uniform":
        return f"uniform integers in [{d[1]}, {d[2]}]"
    return f"round(lognormal({d[1]}, {d[2]})) clipped to [{d[3]}, {d[4]}]"


def decode_config(cfg, world: int, fused: bool = True, split: str = "mod") -> dict:
    """The ``config`` object of a decode line, identical in both arms (whole job at ``world`` GPUs)."""
    from aegaeon_b200 import synth

    full = synth.make_layout(cfg)
    L, Hq, Hkv, D = cfg.num_layers, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    strong = cfg.name == "cfg3"
    batch = cfg.batch if strong else cfg.batch * world
    sum_ctx = full.total_tokens * (1 if strong else world)
    kv_step = sum_ctx * Hkv * D * 2 * 2 * L
    if strong and split == "balanced":
        how = (f"batch {cfg.batch} split over {world} GPU(s) in shares of about equal context (longest first to "
               "the least-loaded GPU), each GPU its own pool")
    elif strong:
        how = f"batch {cfg.batch} split over {world} GPU(s): sequence i on GPU i mod {world}, each GPU its own pool"
    else:
        how = f"batch {cfg.batch} per GPU on each of {world} GPU(s), each GPU its own pool"
    return {
        "workload": f"{cfg.name}: {cfg.model} decode step, {L} layers x (reshape_and_cache of one new token per "
                    f"sequence + paged decode attention), {how}",
        "batch": batch, "layers": L, "q_heads": Hq, "kv_heads": Hkv, "head_dim": D, "block_size": 16,
        "storage_dtype": "bf16" if cfg.dtype == torch.bfloat16 else "fp16",
        "context_lengths": _ctx_desc(cfg), "seed": cfg.seed, "value_std": cfg.value_std,
        "sum_ctx": sum_ctx, "max_ctx": int(full.seq_lens.max()), "kv_bytes_per_step": kv_step,
        "accumulate": "fp32",
        "l2": (f"inputs larger than L2: {kv_step / world / 1e9:.2f} GB of K/V read per step per GPU, each layer's "
               "blocks read once per step, vs 126 MB L2 (no flush)"),
        "parallelism": f"{world} GPU(s), one process each, no collective on the data path",
        "layer_kernels": ("fused cache write + attention (one launch per layer)" if fused else
                          "reshape_and_cache + paged attention (two launches per layer)"),
    }


# ------------------------------------------------------------------------------------------
# CPU restatement timing (oracle/torch_ref.py, fp32 torch): the reference arm and cpu_baseline


class CpuDecodeSample:
    """A bounded sample of a decode config's batch, run on the host by the fp32 torch
    restatement: whole L-layer steps (cache write + attention per layer) over a stratified
    sample of the batch (sequences sorted by context length, every k-th taken), with k chosen so
    that one step takes about ``target_step_s`` on this host. Each layer has its own cache
    blocks (the sample's blocks only); the values are N(0, std^2) in the storage dtype."""

    MAX_SAMPLE_BYTES = 8 << 30

    def __init__(self, cfg, lay, target_step_s: float, seed: int = 0):
        from oracle.torch_ref import host_threads

        self.cfg, self.lay = cfg, lay
        self.threads = host_threads()
        torch.set_num_threads(self.threads)
        B = len(lay.seq_lens)
        block_bytes = 2 * 16 * cfg.num_kv_heads * cfg.head_dim * 2  # one (block, layer): K and V
        # probe: two layers of a small stratified sample, to size the real one
        k_probe = max(1, B // 8)
        probe = self._build(k_probe, 2, seed)
        probe_step = self._stepper(probe, 2)
        probe_step()
        t0 = time.perf_counter()
        probe_step()
        t_layer = (time.perf_counter() - t0) / 2
        per_ctx = t_layer / max(1, probe["sum_ctx"])
        full_step = per_ctx * lay.total_tokens * cfg.num_layers
        k = int(min(B, max(1, math.ceil(full_step / max(target_step_s, 1e-3)))))
        while True:  # bound the host memory of the sample
            blocks = self._pick_blocks(k)
            if blocks * cfg.num_layers * block_bytes <= self.MAX_SAMPLE_BYTES or k >= B:
                break
            k = min(B, k * 2)
        del probe, probe_step
        self.s = self._build(k, cfg.num_layers, seed)
        self.step = self._stepper(self.s, cfg.num_layers)
        # the probe overstates the cost of a large sample (fixed per-call costs): time one real
        # step and grow the sample once if it runs well under the target
        t0 = time.perf_counter()
        self.step()
        t_step = time.perf_counter() - t0
        if t_step < 0.5 * target_step_s and k > 1:
            k2 = max(1, int(k * t_step / target_step_s))
            while k2 < k and self._pick_blocks(k2) * cfg.num_layers * block_bytes > self.MAX_SAMPLE_BYTES:
                k2 += 1
            if k2 < k:
                del self.s, self.step
                k = k2
                self.s = self._build(k, cfg.num_layers, seed)
                self.step = self._stepper(self.s, cfg.num_layers)
        self.k = k
        self.batch = self.s["batch"]
        self.sum_ctx = self.s["sum_ctx"]

    def _pick(self, k: int) -> np.ndarray:
        order = np.argsort(self.lay.seq_lens, kind="stable")
        return np.sort(order[(k - 1) // 2::k])

    def _pick_blocks(self, k: int) -> int:
        ctx = self.lay.seq_lens[self._pick(k)].astype(np.int64)
        return int(((ctx + 15) // 16).sum())

    def _build(self, k: int, layers: int, seed: int) -> dict:
        from oracle.torch_ref import DecodeLayerCPU

        cfg = self.cfg
        pick = self._pick(k)
        ctx = self.lay.seq_lens[pick].astype(np.int64)
        nb = (ctx + 15) // 16
        tables = np.zeros((len(ctx), max(1, int(nb.max()) if len(nb) else 1)), np.int32)
        off = 0
        for i, n in enumerate(nb):
            tables[i, :n] = np.arange(off, off + n)
            off += int(n)
        Hq, Hkv, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        g = torch.Generator().manual_seed(seed)
        cache = torch.empty((max(off, 1), layers, 2, 16, Hkv, D), dtype=cfg.dtype)
        one = (torch.randn((max(off, 1), 2, 16, Hkv, D), generator=g) * cfg.value_std).to(cfg.dtype)
        for l in range(layers):
            cache[:, l] = one
        Bs = len(ctx)
        q = (torch.randn((layers, Bs, Hq, D), generator=g) * cfg.value_std).to(cfg.dtype)
        k_new = (torch.randn((layers, Bs, Hkv, D), generator=g) * cfg.value_std).to(cfg.dtype)
        v_new = (torch.randn((layers, Bs, Hkv, D), generator=g) * cfg.value_std).to(cfg.dtype)
        pos = np.maximum(ctx - 1, 0)
        slots = torch.as_tensor(tables[np.arange(Bs), pos // 16].astype(np.int64) * 16 + pos % 16)
        out = torch.empty_like(q)
        layer = DecodeLayerCPU(tables, ctx.astype(np.int32), 1.0 / math.sqrt(D), self.threads)
        return dict(cache=cache, q=q, k_new=k_new, v_new=v_new, slots=slots, out=out, layer=layer, batch=Bs,
                    sum_ctx=int(ctx.sum()))

    @staticmethod
    def _stepper(s: dict, layers: int):
        def step():
            for l in range(layers):
                s["layer"].run(s["q"][l], s["cache"][:, l, 0], s["cache"][:, l, 1], s["k_new"][l], s["v_new"][l],
                               s["slots"], s["out"][l])
        return step

    def describe(self, what: str) -> str:
        return (f"{what}: fp32 torch restatement (oracle/torch_ref.py: block gather, fp32 SDPA per sequence, cache "
                f"write) of whole {self.cfg.num_layers}-layer steps over a stratified sample of the batch "
                f"(sequences sorted by context, every {self.k}-th: {self.batch} of {len(self.lay.seq_lens)} "
                f"sequences, sum ctx {self.sum_ctx} of {self.lay.total_tokens}); tokens/s = sampled sequences / "
                f"step time; {self.threads} host threads")


def cpu_baseline_leg(cfg, budget_s: float) -> dict:
    """cpu_baseline of the decode line: the fp32 torch restatement on a bounded sample, best of up
    to 5 whole steps within ``budget_s``."""
    lay = synth_layout_full(cfg)
    smp = CpuDecodeSample(cfg, lay, target_step_s=budget_s / 5)
    smp.step()  # warm-up
    times = []
    t_start = time.perf_counter()
    while len(times) < 5 and (not times or time.perf_counter() - t_start < budget_s):
        t0 = time.perf_counter()
        smp.step()
        times.append(time.perf_counter() - t0)
    best = min(times)
    return {"value": smp.batch / best, "unit": "tokens/s", "cores": smp.threads, "kind": "port",
            "sample": smp.describe(f"best of {len(times)} steps")}


def synth_layout_full(cfg):
    from aegaeon_b200 import synth

    return synth.make_layout(cfg)


# ------------------------------------------------------------------------------------------
# Our arm


def _barrier(world):
    if world > 1:
        torch.distributed.barrier()


def _max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _gather_floats(xs, world: int, device) -> list:
    """Every rank's list of floats (same length on every rank), as a list per rank."""
    t = torch.tensor(xs, dtype=torch.float64, device=device)
    if world == 1:
        return [t.tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [o.tolist() for o in out]


def _per_launch_ms(fn_list, device, sleep_cycles=int(4e7)):
    """Device durations of launches measured with CUDA events on the launching stream.

    The first function runs once first (untimed), so that no launch in the timed list loads a
    kernel module (a lazy module load synchronises the device, which would leave the events
    timing the host's launch gaps). A sleep kernel is then queued so that the host enqueues every
    (event, launch, event) triple before the device reaches them; launches run back to back and
    each event pair brackets exactly one kernel.
    """
    stream = torch.cuda.current_stream(device)
    for fn in fn_list[:1]:
        fn()
    torch.cuda.synchronize(device)
    pairs = []
    torch.cuda._sleep(sleep_cycles)
    for fn in fn_list:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        pairs.append((e0, e1))
    torch.cuda.synchronize(device)
    return [a.elapsed_time(b) for a, b in pairs]


def _graph_ms(fn, steps: int, device) -> float:
    """Mean device time of one replay of ``fn`` captured as a CUDA graph (events around ``steps``
    back-to-back replays, after 3 warm-up replays)."""
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    stream = torch.cuda.current_stream(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    a.record(stream)
    for _ in range(steps):
        g.replay()
    b.record(stream)
    torch.cuda.synchronize(device)
    del g
    return a.elapsed_time(b) / steps


def _load_reference_swap():
    """The reference's own ``aegaeon.ops.swap`` compiled from its sources into oracle/_ref by
    oracle/build.py (a baseline, never the measured product), or None."""
    import importlib.util

    so = os.path.join(ROOT, "oracle", "_ref", "aegaeon_ref_ops.so")
    if not os.path.exists(so):
        return None
    spec = importlib.util.spec_from_file_location("aegaeon_ref_ops", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _timed_ms(fn, reps: int, device, warm: int = 1) -> float:
    stream = torch.cuda.current_stream(device)
    for _ in range(warm):
        fn()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        fn()
    b.record(stream)
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / reps


def link_leg(device, world: int, reps: int = 5) -> dict:
    """Pinned host link: one contiguous 1 GiB copy each way, this GPU alone (rank 0, the others
    idle) and all ranks at once (device-timed per rank; the slowest rank and the sum)."""
    nbytes = 1 << 30
    big_h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    big_d = torch.empty(nbytes, dtype=torch.uint8, device=device)
    rank = torch.distributed.get_rank() if world > 1 else 0
    h2d = lambda: big_d.copy_(big_h, non_blocking=True)  # noqa: E731
    d2h = lambda: big_h.copy_(big_d, non_blocking=True)  # noqa: E731
    res = {}
    _barrier(world)
    if rank == 0:
        res["h2d_gbs_one_gpu"] = nbytes / (_timed_ms(h2d, reps, device) / 1e3) / 1e9
        res["d2h_gbs_one_gpu"] = nbytes / (_timed_ms(d2h, reps, device) / 1e3) / 1e9
    _barrier(world)
    if world > 1:
        per = []
        for fn in (h2d, d2h):
            fn()
            torch.cuda.synchronize(device)
            _barrier(world)
            per.append(nbytes / (_timed_ms(fn, reps, device, warm=0) / 1e3) / 1e9)
            _barrier(world)
        allr = _gather_floats(per, world, device)
        h, d = [r[0] for r in allr], [r[1] for r in allr]
        res.update({"h2d_gbs_per_gpu_all_at_once": min(h), "d2h_gbs_per_gpu_all_at_once": min(d),
                    "h2d_gbs_sum_all_at_once": sum(h), "d2h_gbs_sum_all_at_once": sum(d)})
    del big_h, big_d
    return res


def swap_leg(device, scale: float = 1.0, reps: int = 3) -> dict:
    """The cfg5 swap set on one GPU: 4096 scattered 917,504-byte blocks of a 16384-block pool out
    to a pinned host pool and back into fresh ids (bit-exact round trip checked), by this
    library's copy-engine path (``ops.swap``) and SM path (``ops.swap_sm``) and by the reference's
    own operator built from its sources (oracle/_ref, the bar); copy_blocks of 8192 pairs."""
    from aegaeon_b200 import layout, ops, synth

    c = dict(synth.SWAP_CFG)
    if scale != 1.0:
        for k in ("device_blocks", "swap_blocks", "copy_pairs"):
            c[k] = max(2, int(c[k] * scale))
        c["copy_pairs"] = min(c["copy_pairs"], c["device_blocks"] // 2)
        c["swap_blocks"] = min(c["swap_blocks"], c["device_blocks"])
    shape = (c["device_blocks"],) + layout.kv_block_shape(c["num_layers"], c["num_kv_heads"], c["head_dim"])
    kv = torch.empty(shape, dtype=c["dtype"], device=device)
    synth.random_bits_(kv, c["seed"])
    bb = layout.block_bytes(kv)
    n = c["swap_blocks"]
    host = torch.empty((n,) + shape[1:], dtype=c["dtype"]).pin_memory()
    g = torch.Generator().manual_seed(c["seed"])
    out_ids = torch.randperm(c["device_blocks"], generator=g)[:n].tolist()
    host_ids = torch.randperm(n, generator=g).tolist()
    in_ids = torch.randperm(c["device_blocks"], generator=g)[:n].tolist()
    p = torch.randperm(c["device_blocks"], generator=g)
    src, dst = p[:c["copy_pairs"]].to(device), p[c["copy_pairs"]:2 * c["copy_pairs"]].to(device)
    d_out, d_host, d_in = (torch.as_tensor(x, device=device) for x in (out_ids, host_ids, in_ids))
    want = kv[d_out].clone()  # the blocks that go out, to check the round trip
    ms = {
        "out_dma": _timed_ms(lambda: ops.swap(out_ids, host_ids, False, kv, host), reps, device),
        "out_sm": _timed_ms(lambda: ops.swap_sm(d_out, d_host, False, kv, host), reps, device),
        "in_dma": _timed_ms(lambda: ops.swap(host_ids, in_ids, True, kv, host), reps, device),
        "in_sm": _timed_ms(lambda: ops.swap_sm(d_host, d_in, True, kv, host), reps, device),
    }
    torch.cuda.synchronize(device)
    ok = bool(torch.equal(kv[d_in].view(torch.int16), want.view(torch.int16)))
    ref = _load_reference_swap()
    if ref is not None:
        ms["out_reference"] = _timed_ms(lambda: ref.swap(out_ids, host_ids, False, kv, host), reps, device)
        ms["in_reference"] = _timed_ms(lambda: ref.swap(host_ids, in_ids, True, kv, host), reps, device)
    ms["copy_blocks"] = _timed_ms(lambda: ops.copy_blocks(src, dst, kv), max(reps, 5), device)
    gbs = {k: (2 * c["copy_pairs"] if k == "copy_blocks" else n) * bb / (v / 1e3) / 1e9 for k, v in ms.items()}
    res = {"set": f"{n} scattered {bb:,}-byte blocks of a {c['device_blocks']}-block pool (cfg5)"
                  + ("" if scale == 1.0 else f", scaled x{scale}"),
           "bytes_per_direction": n * bb, "gbs": gbs, "ms": ms, "round_trip_bit_exact": ok,
           "out_gbs": max(gbs["out_dma"], gbs["out_sm"]), "in_gbs": max(gbs["in_dma"], gbs["in_sm"]),
           "copy_blocks_pairs": c["copy_pairs"]}
    if ref is not None:
        res["reference_op"] = "aegaeon.ops.swap built from aegaeon/ops/{ops.cpp,swap.cu} (oracle/_ref)"
        res["vs_reference_op"] = {"out": res["out_gbs"] / gbs["out_reference"], "in": res["in_gbs"] / gbs["in_reference"]}
    else:
        res["reference_op"] = "unavailable: oracle/_ref/aegaeon_ref_ops.so not built (no reference checkout)"
    del kv, host, want
    torch.cuda.empty_cache()
    return res


def migration_leg(kv: torch.Tensor, world: int, rank: int, device, n_blocks: int = 512, reps: int = 3) -> dict:
    """Cross-GPU proof of ops.migrate_blocks: every rank maps the pool of rank (r + 1) % N through
    its IPC handle and pulls ``n_blocks`` scattered blocks into scattered blocks of its own pool
    with the SM kernel (plain 16-byte peer loads over NVLink), timed on the device; the pulled
    blocks are then checked bit for bit against the owner's digest of its source blocks."""
    from aegaeon_b200 import layout, ops

    bb = layout.block_bytes(kv)
    N = kv.size(0)
    handles = [None] * world
    torch.distributed.all_gather_object(handles, (ops.export_kv_cache(kv), N, bb))
    peer_rank = (rank + 1) % world
    peer = ops.open_kv_cache(*handles[peer_rank])
    # Sources from the lower half of the peer's pool, targets in the upper half of this pool: a
    # rank's pulled-from blocks are never the blocks its own pull writes.
    lo_peer, lo_mine = peer.num_blocks // 2, N // 2
    n = min(n_blocks, lo_peer, N - lo_mine)
    g = torch.Generator().manual_seed(4242 + rank)
    src = torch.randperm(lo_peer, generator=g)[:n]
    dst = lo_mine + torch.randperm(N - lo_mine, generator=g)[:n]
    d_src, d_dst = src.to(device), dst.to(device)
    # every rank learns which of its blocks its puller reads (rank r is pulled by r - 1)
    wanted = [None] * world
    torch.distributed.all_gather_object(wanted, src.tolist())
    mine = torch.as_tensor(wanted[(rank - 1) % world], device=device)

    def digest(ids: torch.Tensor) -> list:
        w = torch.arange(bb // 4, device=device, dtype=torch.int64) % 65521 + 1
        acc = torch.zeros(2, dtype=torch.int64, device=device)
        for i in range(0, ids.numel(), 16):
            blk = kv.view(torch.int32).view(N, -1)[ids[i:i + 16]].to(torch.int64)
            acc[0] += blk.sum()
            acc[1] += (blk * w).sum()
        return acc.tolist()

    torch.cuda.synchronize(device)
    _barrier(world)
    pull = lambda: ops.migrate_blocks(d_src, d_dst, peer, kv)  # noqa: E731
    ms = _max_over_ranks(_timed_ms(pull, reps, device), world, device)
    torch.cuda.synchronize(device)
    _barrier(world)
    got = digest(d_dst)          # what this rank pulled
    owner = digest(mine)         # what its puller should have pulled from this rank
    all_got = [None] * world
    all_owner = [None] * world
    torch.distributed.all_gather_object(all_got, got)
    torch.distributed.all_gather_object(all_owner, owner)
    ok = all(all_got[r] == all_owner[(r + 1) % world] for r in range(world))
    _barrier(world)
    peer.close()
    _barrier(world)
    return {"migrate_ok": ok, "blocks_per_rank": n, "block_bytes": bb,
            "gbs_per_gpu": n * bb / (ms / 1e3) / 1e9, "ms_slowest_rank": ms,
            "how": "each rank pulls scattered blocks from rank (r + 1) % N over NVLink (ops.migrate_blocks, "
                   "SM kernel, plain peer loads), all ranks at once; bit-exact by digests of source and target"}


def other_configs_leg(device, peak: float, max_layers: int = 4) -> dict:
    """cfg1, cfg2 and cfg4, the other decode configurations, beside the cfg3 headline on the same
    GPU: each as a step graph (plan + fused cache write and attention per layer) of its layers, at
    most ``max_layers`` of them for cfg4 (its pool then holds those layers only: same blocks and
    bytes per launch), per layer = (step - plan) / layers, and as launches timed alone. Tokens/s
    of a whole step follow as batch / (plan + layers x per-layer time). Also the same step as the
    reference's two calls per layer (cache write, then attention), relative to the fused one."""
    from aegaeon_b200 import ops, synth
    from aegaeon_b200.step import DecodeStep

    res = {}
    for name in ("cfg1", "cfg2", "cfg4"):
        cfg = synth.CONFIGS[name]
        lt = min(cfg.num_layers, max_layers) if name == "cfg4" else cfg.num_layers
        cfg_t = dataclasses.replace(cfg, num_layers=lt)
        lay = synth.make_layout(cfg_t)
        B = len(lay.seq_lens)
        Hq, Hkv, D = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
        scale = synth.default_scale(cfg)
        kv = torch.empty((lay.num_blocks, lt, 2, 16, Hkv, D), dtype=cfg.dtype, device=device)
        synth.fill_normal_(kv, cfg.value_std, cfg.seed)
        step = DecodeStep(kv, Hq, B, lay.width, scale)
        g = torch.Generator(device=device).manual_seed(cfg.seed + 17)
        inputs = dict(q=(torch.randn(step.q.shape, generator=g, device=device) * cfg.value_std).to(cfg.dtype),
                      k_new=(torch.randn(step.k_new.shape, generator=g, device=device) * cfg.value_std).to(cfg.dtype),
                      v_new=(torch.randn(step.v_new.shape, generator=g, device=device) * cfg.value_std).to(cfg.dtype),
                      slot_mapping=torch.as_tensor(synth.new_token_slots(lay), device=device),
                      block_tables=torch.as_tensor(lay.block_tables, device=device),
                      seq_lens=torch.as_tensor(lay.seq_lens, device=device))
        stream = torch.cuda.current_stream(device)
        reps = 20

        def step_graph_ms(st):
            st.load_inputs(**inputs)
            st.capture()
            for _ in range(3):
                st.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(device)
            a.record(stream)
            for _ in range(reps):
                st.replay()
            b.record(stream)
            torch.cuda.synchronize(device)
            return a.elapsed_time(b) / reps

        step_ms = step_graph_ms(step)
        assert torch.isfinite(step.out.float()).all(), f"non-finite {name} output"
        # the reference's two calls per layer (cache write, then attention) as one step graph
        unfused_ms = step_graph_ms(DecodeStep(kv, Hq, B, lay.width, scale, fused=False))
        plan_ms = statistics.median(_per_launch_ms([lambda: step.plan.plan(step.seq_lens, step.block_tables)] * 4,
                                                   device))
        fns = [lambda l=l: ops.decode_layer(step.out[l], step.q[l], step.k_new[l], step.v_new[l], kv, l,
                                            step.block_tables, step.seq_lens, scale, plan=step.plan)
               for l in range(lt)]
        iso_ms = statistics.median(_per_launch_ms(fns * max(1, 8 // lt), device))
        algo = synth.algorithmic_bytes_per_layer(cfg_t, lay)
        lb = algo["attention"] + algo["reshape_and_cache"]
        per_layer = max((step_ms - plan_ms) / lt, 1e-6)
        res[name] = {
            "workload": f"{name}: {Hq}/{Hkv} heads, {str(cfg.dtype).replace('torch.', '')}, batch {B}, "
                        f"{_ctx_desc(cfg)}, {lt} of {cfg.num_layers} layers in the step graph",
            "layer_bytes": lb,
            "in_step_launch_us": per_layer * 1e3,
            "frac": lb / (per_layer / 1e3) / 1e9 / peak,
            "isolated_launch_us": iso_ms * 1e3,
            "frac_isolated_launch": lb / (iso_ms / 1e3) / 1e9 / peak,
            "plan_us": plan_ms * 1e3,
            "tokens_per_s": B / ((plan_ms + per_layer * cfg.num_layers) / 1e3),
            "unfused_step_vs_fused": unfused_ms / step_ms,
        }
        del step, kv
        torch.cuda.empty_cache()
    return res


def rows_leg(local) -> dict:
    """The other rows' own measurements (their --config runs) in compact form for the default line
    at N = 1: prefill attention beside vLLM's FlashAttention, the per-step input builder beside the
    reference's loops, and the model-weight switch beside the host link and the reference's loop."""
    ns = argparse.Namespace(steps=20, warmup=3, scale=1.0)
    pf = prefill_line(ns, local)
    pr = prep_line(ns, local)
    ws = run_weights(ns, 1, 0, local, embed=True)
    return {
        "prefill": {"metric": pf["metric"], "value": pf["value"], "unit": pf["unit"],
                    "workload": pf["config"]["workload"], "detail": pf["detail"], "roofline": pf["roofline"],
                    "cpu_baseline": pf["cpu_baseline"]},
        "step_inputs": {"metric": pr["metric"], "value": pr["value"], "unit": pr["unit"],
                        "workload": pr["config"]["workload"], "batches": pr["batches"],
                        "cpu_baseline": pr["cpu_baseline"]},
        "weight_switch": {"metric": ws["metric"], "value": ws["value"], "unit": ws["unit"],
                          "workload": ws["config"]["workload"], "detail_gbs": ws["detail_gbs"],
                          "roofline": ws["roofline"], "cpu_baseline": ws["cpu_baseline"],
                          "first_mib_matches": ws["first_mib_matches"]},
    }


def run_decode(args, world, rank, local):
    from aegaeon_b200 import ops, synth
    from aegaeon_b200.step import DecodePipeline, DecodeStep

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = synth.CONFIGS[args.config]
    if args.layers:
        cfg = dataclasses.replace(cfg, num_layers=args.layers)
    lay, scaling = _decode_layout(cfg, world, rank, args.split)
    if args.compact_pool:
        lay = synth.compact_layout(lay)
    B = len(lay.seq_lens)
    L, Hq, Hkv, D = cfg.num_layers, cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim
    scale = synth.default_scale(cfg)

    kv = torch.empty((lay.num_blocks, L, 2, 16, Hkv, D), dtype=cfg.dtype, device=device)
    synth.fill_normal_(kv, cfg.value_std, cfg.seed + 1000 * rank)
    step = DecodeStep(kv, Hq, B, lay.width, scale, fused=not args.unfused)
    g = torch.Generator(device=device).manual_seed(cfg.seed + 17 + rank)
    dev_inputs = dict(
        q=(torch.randn(step.q.shape, generator=g, device=device) * cfg.value_std).to(cfg.dtype),
        k_new=(torch.randn(step.k_new.shape, generator=g, device=device) * cfg.value_std).to(cfg.dtype),
        v_new=(torch.randn(step.v_new.shape, generator=g, device=device) * cfg.value_std).to(cfg.dtype),
        slot_mapping=torch.as_tensor(synth.new_token_slots(lay), device=device),
        block_tables=torch.as_tensor(lay.block_tables, device=device),
        seq_lens=torch.as_tensor(lay.seq_lens, device=device),
    )
    host_inputs = {k: v.cpu().pin_memory() for k, v in dev_inputs.items()}
    host_out = torch.empty(step.out.shape, dtype=step.out.dtype).pin_memory()
    step.load_inputs(**dev_inputs)
    step.capture()
    torch.cuda.synchronize(device)

    for _ in range(max(args.warmup, 3)):
        step.replay()
    torch.cuda.synchronize(device)

    if args.profile_run:
        for _ in range(args.steps):
            step.replay()
        torch.cuda.synchronize(device)
        if rank == 0:
            print(json.dumps({"profile_run": True, "config": cfg.name, "steps": args.steps,
                              "pool_blocks": lay.num_blocks}), flush=True)
        return
    clocks = ClockSampler(device)
    # Untimed pre-roll of ~1 s so that the clock samples cover the GPU under this load.
    t_pre = time.perf_counter()
    while time.perf_counter() - t_pre < 1.0:
        for _ in range(20):
            step.replay()
        torch.cuda.synchronize(device)

    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize(device)
    e0.record(stream)
    for _ in range(args.steps):
        step.replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    _barrier(world)
    own_ms = e0.elapsed_time(e1)  # this rank's timed region
    ms = _max_over_ranks(own_ms, world, device)
    clock_info = clocks.stop()
    assert torch.isfinite(step.out.float()).all(), "non-finite attention output"

    # Per-launch durations of the dominant kernel (the layer's attention launch with its split
    # merge; fused with the cache write unless --unfused) and of the separate cache write.
    n_prof = max(1, min(args.steps, 4))
    attn_fns, write_fns = [], []
    for _ in range(n_prof):
        for layer in range(L):
            if step.fused:
                attn_fns.append(lambda l=layer: ops.decode_layer(step.out[l], step.q[l], step.k_new[l], step.v_new[l],
                                                                 kv, l, step.block_tables, step.seq_lens, scale,
                                                                 plan=step.plan))
            else:
                attn_fns.append(lambda l=layer: ops.paged_attention_decode(step.out[l], step.q[l], kv, l,
                                                                           step.block_tables, step.seq_lens, scale,
                                                                           plan=step.plan))
            write_fns.append(lambda l=layer: ops.reshape_and_cache(step.k_new[l], step.v_new[l], kv, l,
                                                                   step.slot_mapping))
    attn_ms = []
    for s in range(n_prof):
        attn_ms += _per_launch_ms(attn_fns[s * L:(s + 1) * L], device)
    write_ms = _per_launch_ms(write_fns[:L], device)
    # The cache write as a stream runs it: one graph of L back-to-back launches (each waits for
    # the one before under programmatic dependent launch), per launch.
    def writes():
        for fn in write_fns[:L]:
            fn()

    write_graph_ms = _graph_ms(writes, max(3, min(args.steps, 20)), device) / L
    plan_ms = _per_launch_ms([lambda: step.plan.plan(step.seq_lens, step.block_tables)] * 4, device)
    plan_med_ms = statistics.median(plan_ms)

    # Attention as the model forward calls it: each layer's attention follows that layer's QKV
    # projection (a cuBLAS GEMM of the model's shape that does not trigger dependents), not the
    # previous layer's attention. Per-layer time = (graph of L x (GEMM + attention) - graph of
    # L x GEMM - plan) / L.
    hidden = Hq * D
    x = torch.randn((B, hidden), device=device).to(cfg.dtype)
    w_qkv = (torch.randn((hidden, (Hq + 2 * Hkv) * D), device=device) / math.sqrt(hidden)).to(cfg.dtype)
    qkv = torch.empty((B, (Hq + 2 * Hkv) * D), device=device, dtype=cfg.dtype)

    def gemms():
        for _ in range(L):
            torch.matmul(x, w_qkv, out=qkv)

    def model_like():
        step.plan.plan(step.seq_lens, step.block_tables)
        for l in range(L):
            torch.matmul(x, w_qkv, out=qkv)
            ops.decode_layer(step.out[l], step.q[l], step.k_new[l], step.v_new[l], kv, l, step.block_tables,
                             step.seq_lens, scale, plan=step.plan, prefetch=True)

    n_model = max(3, min(args.steps, 20))
    gemm_ms = _graph_ms(gemms, n_model, device)
    model_ms = _graph_ms(model_like, n_model, device)
    in_model_ms = max((model_ms - gemm_ms - plan_med_ms) / L, 1e-6)
    del x, w_qkv, qkv

    # The two-operator form the reference calls per layer (reshape_and_cache, then attention),
    # as a step graph beside the fused one.
    unfused_ms = None
    if step.fused:
        uf = DecodeStep(kv, Hq, B, lay.width, scale, fused=False)
        uf.load_inputs(**dev_inputs)
        unfused_ms = _graph_ms(uf.run_eager, n_model, device)
        del uf

    # End to end through the public step API with host buffers: every step uploads its inputs
    # from pinned host memory and reads its outputs back, overlapped with the neighbouring
    # steps' kernels (DecodePipeline: two buffer slots, upload and download streams).
    pipe = DecodePipeline(kv, Hq, B, lay.width, scale, fused=not args.unfused)
    for sl in pipe.slots:
        sl.load_inputs(**dev_inputs)
    pipe.capture()
    host_outs = [host_out, torch.empty_like(host_out).pin_memory()]
    pipe.run([host_inputs], host_outs, 4)
    torch.cuda.synchronize(device)
    _barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    pipe.run([host_inputs], host_outs, args.steps)
    f1.record(stream)
    torch.cuda.synchronize(device)
    _barrier(world)
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1), world, device)
    assert torch.isfinite(host_outs[(args.steps - 1) % 2].float()).all(), "non-finite end-to-end output"
    del pipe

    # Host link (one GPU, and all ranks at once) and the KV-block swap set (rank 0).
    link = link_leg(device, world)
    swap = None
    if rank == 0 and not args.no_swap:
        swap = swap_leg(device, scale=args.swap_scale)
        swap.update({"frac_of_link": {"out": swap["out_gbs"] / link["d2h_gbs_one_gpu"],
                                      "in": swap["in_gbs"] / link["h2d_gbs_one_gpu"]},
                     "link": {k: link[k] for k in ("h2d_gbs_one_gpu", "d2h_gbs_one_gpu")}})
    _barrier(world)
    migration = migration_leg(kv, world, rank, device) if world > 1 else None

    peak, peak_src = _peaks()
    others = rows = None
    if world == 1 and rank == 0 and args.config == "cfg3" and not args.no_other_configs and not args.layers:
        others = other_configs_leg(device, peak)
        rows = rows_leg(local)
    algo = synth.algorithmic_bytes_per_layer(cfg, lay)
    launch_bytes = algo["attention"] + (algo["reshape_and_cache"] if step.fused else 0)
    ms_step = ms / args.steps
    tokens_total = B * world if scaling == "weak" else cfg.batch
    value = tokens_total / (ms_step / 1e3)
    # Per-rank figures of the dominant kernel from each rank's own timed step, gathered; the
    # roofline reports the rank whose step bounds the job (the longest one).
    own_step = own_ms / args.steps
    in_step_ms = max((own_step - plan_med_ms) / L, 1e-6)
    if not step.fused:
        in_step_ms = max((own_step - plan_med_ms - L * write_graph_ms) / L, 1e-6)
    attn_avg_ms = statistics.mean(attn_ms)
    per_rank = _gather_floats([launch_bytes, in_step_ms, attn_avg_ms, in_model_ms, algo["kv_read"] * L,
                               (algo["attention"] + algo["reshape_and_cache"]) * L, own_step], world, device)
    bound = max(range(world), key=lambda r: per_rank[r][6])
    lb, ism, iso, imd = per_rank[bound][0], per_rank[bound][1], per_rank[bound][2], per_rank[bound][3]
    rank_bytes = [r[0] for r in per_rank]
    kv_step_all = sum(r[4] for r in per_rank)
    bytes_step_all = sum(r[5] for r in per_rank)
    achieved = lb / (ism / 1e3) / 1e9
    traffic = _ncu_traffic(f"decode_attn_{cfg.name}" + ("" if world == 1 else f"_n{world}"))
    h2d, d2h = step.input_bytes(), step.output_bytes()
    e2e_step_s = e2e_ms / args.steps / 1e3

    line = {
        "metric": "decode-attn tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "fp16" if cfg.dtype == torch.float16 else "bf16",
        "data": "synthetic: seeded contexts, block tables and N(0, std^2) K/V/q (no dataset on this path)",
        "config": decode_config(cfg, world, fused=step.fused, split=args.split),
        "shard": {"rank0_batch": B, "rank0_pool_blocks": lay.num_blocks, "rank0_sum_ctx": lay.total_tokens,
                  "rank0_layer_bytes": launch_bytes,
                  "layer_bytes_per_rank": rank_bytes,
                  "imbalance": max(rank_bytes) / (sum(rank_bytes) / world),
                  "in_step_frac_per_rank": [r[0] / (r[1] / 1e3) / 1e9 / peak for r in per_rank],
                  "bound_rank": bound},
        "kv_read_gbs": kv_step_all / (ms_step / 1e3) / 1e9,
        "hbm_frac_step": bytes_step_all / world / (ms_step / 1e3) / 1e9 / peak,
        "e2e": {
            "value": tokens_total / e2e_step_s,
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d * world,
            "d2h_bytes_per_step": d2h * world,
            "ms_per_step": e2e_ms / args.steps,
            "path": "aegaeon_b200.step.DecodePipeline.run: per step pinned host inputs -> H2D (upload stream), "
                    "graph replay, D2H of the outputs (download stream); copies of neighbouring steps overlap "
                    "the kernels",
        },
        "gpu_launches": args.steps * step.launches_per_step,
        "roofline": {
            "bound": "hbm",
            "kernel": "decode_attn_kernel (" + ("fused cache write + " if step.fused else "")
                      + "attention + split merge, one launch per layer)",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": peak_src,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": lb,
            "duration": "per layer launch in the timed step graph of the rank whose step bounds the job: "
                        "(its step - plan) / layers",
            "in_step_launch_us": ism * 1e3,
            "avg_launch_us": iso * 1e3,
            "frac_isolated_launch": lb / (iso / 1e3) / 1e9 / peak,
            "in_model_launch_us": imd * 1e3,
            "frac_in_model": lb / (imd / 1e3) / 1e9 / peak,
            "in_model": "each layer's attention launched after a cuBLAS GEMM of the model's QKV shape "
                        f"([{B}, {hidden}] x [{hidden}, {(Hq + 2 * Hkv) * D}]), the order of the forward pass; "
                        "(graph of L x (GEMM + attention) - graph of L x GEMM - plan) / L",
            "launches_timed": len(attn_ms),
            "reshape_and_cache_us": write_graph_ms * 1e3,
            "reshape_and_cache": f"{len(lay.seq_lens)} new tokens per launch; per launch in a CUDA graph of {L} "
                                 "back-to-back launches (reshape_and_cache_us) and between events around one "
                                 "launch alone (reshape_and_cache_isolated_us)",
            "reshape_and_cache_isolated_us": statistics.median(write_ms) * 1e3,
            "plan_median_us": plan_med_ms * 1e3,
            "plan": step.plan.stats(),
        },
        "clocks": clock_info,
    }
    if unfused_ms is not None:
        line["unfused_step"] = {"ms_per_step": unfused_ms, "vs_fused": unfused_ms / ms_step,
                                "what": "the same step as reshape_and_cache + paged_attention_decode per layer "
                                        "(the reference's two calls), one CUDA graph"}
    line["host_link"] = link
    if world > 1 and "h2d_gbs_per_gpu_all_at_once" in link:
        line["e2e"]["frac_of_concurrent_link"] = {
            "h2d": h2d / e2e_step_s / 1e9 / link["h2d_gbs_per_gpu_all_at_once"],
            "d2h": d2h / e2e_step_s / 1e9 / link["d2h_gbs_per_gpu_all_at_once"]}
    else:
        line["e2e"]["frac_of_link"] = {"h2d": h2d / e2e_step_s / 1e9 / link["h2d_gbs_one_gpu"],
                                       "d2h": d2h / e2e_step_s / 1e9 / link["d2h_gbs_one_gpu"]}
    if swap is not None:
        line["swap"] = swap
    if others is not None:
        line["other_configs"] = others
    if rows is not None:
        line["rows"] = rows
    if migration is not None:
        line["migration"] = migration
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_leg(cfg, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del step, kv


def run_swap(args, world, rank, local):
    """cfg5: swap out/in of 4096 scattered blocks and copy_blocks of 8192 pairs (GB/s)."""
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    link = link_leg(device, 1)
    sw = swap_leg(device, scale=args.scale, reps=max(1, min(args.steps, 5)))
    peak, peak_src = _peaks()
    cb = sw["gbs"]["copy_blocks"]
    line = {
        "metric": "KV-block swap GB/s", "value": sw["out_gbs"], "unit": "GB/s", "n_gpus": 1,
        "steps": max(1, min(args.steps, 5)), "warmup": 1, "ms_per_step": min(sw["ms"]["out_dma"], sw["ms"]["out_sm"]),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u16",
        "data": "synthetic random 16-bit patterns",
        "config": {"workload": f"cfg5: swap-out of {sw['set']} to pinned host memory and back into fresh ids; "
                               f"copy_blocks {sw['copy_blocks_pairs']} pairs"},
        "swap": sw, "host_link": link,
        "swap_frac_of_link": {"out": sw["out_gbs"] / link["d2h_gbs_one_gpu"], "in": sw["in_gbs"] / link["h2d_gbs_one_gpu"]},
        "roofline": {"bound": "hbm", "kernel": "block_copy_vec_kernel (copy_blocks)", "achieved": cb,
                     "peak": peak, "unit": "GB/s", "frac": cb / peak, "peak_source": peak_src,
                     "traffic": _ncu_traffic("copy_blocks_cfg5")},
    }
    print(json.dumps(line), flush=True)


def run_migrate(args, world, rank, local):
    """GPU <-> GPU block migration over NVLink (GB/s): every rank pulls the cfg5 swap set (4096
    scattered 917,504-byte blocks) from the pool of rank (r + 1) % N, mapped through its IPC
    handle, into scattered blocks of its own pool, all ranks at once (each GPU's links carry
    data both ways). Also timed: the copy-engine form, a push, and one contiguous 1 GiB
    copy-engine transfer from the peer (the link reference)."""
    from aegaeon_b200 import layout, ops, synth

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world < 2:
        if rank == 0:
            print(json.dumps({"metric": "KV-block migration GB/s", "n_gpus": world,
                              "unavailable": "GPU <-> GPU migration needs two or more GPUs (torchrun)"}), flush=True)
        return
    c = dict(synth.SWAP_CFG)
    if args.scale != 1.0:
        for k in ("device_blocks", "swap_blocks"):
            c[k] = max(2, int(c[k] * args.scale))
        c["swap_blocks"] = min(c["swap_blocks"], c["device_blocks"])
    shape = (c["device_blocks"],) + layout.kv_block_shape(c["num_layers"], c["num_kv_heads"], c["head_dim"])
    kv = torch.empty(shape, dtype=c["dtype"], device=device)
    synth.random_bits_(kv, c["seed"] + rank)
    bb = layout.block_bytes(kv)
    handles = [None] * world
    torch.distributed.all_gather_object(handles, (ops.export_kv_cache(kv), kv.size(0), bb))
    peer_rank = (rank + 1) % world
    peer = ops.open_kv_cache(*handles[peer_rank])
    g = torch.Generator().manual_seed(c["seed"] + 100 + rank)
    n = c["swap_blocks"]
    src = torch.randperm(c["device_blocks"], generator=g)[:n]
    dst = torch.randperm(c["device_blocks"], generator=g)[:n]
    d_src, d_dst = src.to(device), dst.to(device)
    run_len = max(1, min(c["device_blocks"], (1 << 30) // bb))
    contiguous = torch.arange(run_len, dtype=torch.int64)
    stream = torch.cuda.current_stream(device)

    def timed(fn, reps):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(device)
        _barrier(world)
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        t = torch.tensor([a.elapsed_time(b) / reps], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)  # slowest rank
        return float(t.item())

    reps = max(1, min(args.steps, 20))
    res = {
        "pull_sm_ms": timed(lambda: ops.migrate_blocks(d_src, d_dst, peer, kv), reps),
        "pull_dma_ms": timed(lambda: ops.migrate_blocks(src, dst, peer, kv, engine="dma"), reps),
        "push_sm_ms": timed(lambda: ops.migrate_blocks(d_dst, d_src, kv, peer), reps),
        "link_contiguous_dma_ms": timed(lambda: ops.migrate_blocks(contiguous, contiguous, peer, kv, engine="dma"),
                                        reps),
    }
    torch.cuda.synchronize(device)
    _barrier(world)
    peer.close()
    _barrier(world)
    per_gpu = {k.replace("_ms", "_gbs"): (run_len if k.startswith("link") else n) * bb / (v / 1e3) / 1e9
               for k, v in res.items()}
    link = per_gpu["link_contiguous_dma_gbs"]
    best = max(per_gpu["pull_sm_gbs"], per_gpu["pull_dma_gbs"])
    if rank == 0:
        line = {
            "metric": "KV-block migration GB/s", "value": best * world, "unit": "GB/s", "n_gpus": world,
            "steps": reps, "warmup": max(args.warmup, 3), "ms_per_step": min(res["pull_sm_ms"], res["pull_dma_ms"]),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u16",
            "data": "synthetic random 16-bit patterns",
            "config": {"workload": f"every rank pulls {n} scattered {bb:,}-byte blocks from rank (r + 1) % {world} "
                                   f"(IPC-mapped pool of {c['device_blocks']} blocks) into scattered blocks of its own"
                                   + ("" if args.scale == 1.0 else f" (scaled x{args.scale})")},
            "per_gpu_gbs": per_gpu, "detail_ms": res,
            "roofline": {"bound": "nvlink", "kernel": "block_copy_vec_kernel (migrate_blocks, pull over NVLink)",
                         "achieved": per_gpu["pull_sm_gbs"], "peak": link, "unit": "GB/s",
                         "frac": per_gpu["pull_sm_gbs"] / link,
                         "peak_source": "measured here: one contiguous 1 GiB copy-engine transfer from the peer, "
                                        "all ranks at once",
                         "traffic": None},
        }
        print(json.dumps(line), flush=True)
    del kv


def _weight_layout(scale: float):
    """Parameter sizes of the weight-switch workload and their 16-byte-aligned packed offsets
    (the layout of the reference's bump allocators, aegaeon/aegaeon/allocator.py:54-81)."""
    from aegaeon_b200 import synth

    layers = max(1, int(round(28 * scale)))
    sizes = np.asarray(synth.qwen2_7b_param_bytes(2, layers), np.int64)
    offs = np.zeros_like(sizes)
    top = 0
    for i, n in enumerate(sizes):
        top = (top + 15) // 16 * 16
        offs[i] = top
        top += int(n)
    return sizes, offs, top, layers


def _time_calls(fn, reps, device, stream):
    fn()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        fn()
    b.record(stream)
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / reps


def _reference_weight_loop(arena, cache, offs, sizes):
    """The reference's switch: one non-blocking copy_ per parameter (worker.py:358-365)."""
    for o, n in zip(offs.tolist(), sizes.tolist()):
        arena[o:o + n].copy_(cache[o:o + n], non_blocking=True)


def run_weights(args, world, rank, local, reference_only=False, embed=False):
    """Model-weight switch (GB/s): Qwen2.5-7B's parameters (bf16) from a page-locked host model
    cache into a device arena, one call (copy engines over runs of adjacent parameters, or one
    kernel through the mapped host memory), against the reference's per-parameter copy_ loop
    and a contiguous 1 GiB pinned copy (the host link)."""
    from aegaeon_b200 import ops

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    sizes, offs, total, layers = _weight_layout(args.scale)
    cache = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    cache[: 1 << 20].random_(0, 256)
    arena = torch.empty(total, dtype=torch.uint8, device=device)
    reps = max(1, min(args.steps, 3))
    ref_ms = _time_calls(lambda: _reference_weight_loop(arena, cache, offs, sizes), reps, device, stream)
    gb = total / 1e9
    workload = (f"Qwen2.5-7B parameters ({len(sizes)} tensors, {layers} layers, bf16, {total / 1e9:.2f} GB) "
                "pinned host model cache -> device arena, both packed 16-byte aligned")
    if reference_only:
        print(json.dumps({"impl": "reference", "metric": "weight-switch GB/s", "value": gb / (ref_ms / 1e3),
                          "unit": "GB/s", "n_gpus": 1, "steps": reps, "warmup": 1, "ms_per_step": ref_ms,
                          "higher_is_better": True, "config": {"workload": workload},
                          "cpu_baseline": {"value": gb / (ref_ms / 1e3), "unit": "GB/s", "cores": 1, "kind": "reference",
                                           "sample": "the reference's per-parameter copy_ loop (torch), whole model"},
                          "e2e": {"value": gb / (ref_ms / 1e3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    res = {"reference_loop_ms": ref_ms,
           "dma_ms": _time_calls(lambda: ops.copy_segments(arena, cache, offs, offs, sizes, engine="dma"), reps,
                                 device, stream),
           "sm_ms": _time_calls(lambda: ops.copy_segments(arena, cache, offs, offs, sizes, engine="sm"), reps,
                                device, stream)}
    big = min(total, 1 << 30)
    res["link_contiguous_ms"] = _time_calls(lambda: arena[:big].copy_(cache[:big], non_blocking=True), 5, device, stream)
    ok = torch.equal(arena[: 1 << 20].cpu(), cache[: 1 << 20])
    gbs = {k.replace("_ms", "_gbs"): (big if k.startswith("link") else total) / (v / 1e3) / 1e9 for k, v in res.items()}
    best = max(gbs["dma_gbs"], gbs["sm_gbs"])
    del arena, cache
    line = {
        "metric": "weight-switch GB/s", "value": best, "unit": "GB/s", "n_gpus": 1, "steps": reps, "warmup": 1,
        "ms_per_step": min(res["dma_ms"], res["sm_ms"]), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic parameter bytes", "config": {"workload": workload},
        "detail_ms": res, "detail_gbs": gbs, "first_mib_matches": ok,
        "roofline": {"bound": "host link", "achieved": best, "peak": gbs["link_contiguous_gbs"], "unit": "GB/s",
                     "frac": best / gbs["link_contiguous_gbs"],
                     "peak_source": "measured here: one contiguous 1 GiB pinned host-to-device copy"},
        "cpu_baseline": {"value": gbs["reference_loop_gbs"], "unit": "GB/s", "cores": 1, "kind": "reference",
                         "sample": "the reference's per-parameter copy_ loop (torch), whole model"},
    }
    if embed:
        return line
    print(json.dumps(line), flush=True)


def _prefill_lengths(scale: float = 1.0):
    """Prompt lengths of the prefill workload: 16 prompts, round(lognormal(6.5, 0.8)) clipped to
    [16, 8192], seed 7 (Qwen2.5-7B heads: 28 query, 4 KV, head dim 128)."""
    rng = np.random.default_rng(7)
    n = max(1, int(round(16 * scale)))
    return np.clip(np.round(rng.lognormal(6.5, 0.8, n)), 16, 8192).astype(np.int64)


def _vllm_varlen():
    """vLLM's bundled FlashAttention varlen kernel (the reference's kernel family), if it loads."""
    try:
        from vllm.vllm_flash_attn import flash_attn_varlen_func
        return flash_attn_varlen_func, "vllm.vllm_flash_attn.flash_attn_varlen_func"
    except Exception as e:  # noqa: BLE001 - any import failure means "not available"
        return None, f"unavailable: {type(e).__name__}: {str(e)[:160]}"


def run_prefill(args, world, rank, local):
    print(json.dumps(prefill_line(args, local)), flush=True)


def prefill_line(args, local) -> dict:
    """Prefill attention (TFLOP/s, causal FLOPs 2 x 2 x Hq x D x L(L+1)/2 per prompt): this
    library's kernel on a batch of prompts with inputs resident, beside vLLM's FlashAttention
    varlen kernel on the same inputs when it loads, and the oracle on one prompt of the batch."""
    from aegaeon_b200 import ops
    from oracle import oracle as orc

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    lens = _prefill_lengths(args.scale)
    Hq, Hkv, D = 28, 4, 128
    T = int(lens.sum())
    flops = float(sum(4.0 * Hq * D * L * (L + 1) / 2 for L in lens))
    cu = torch.as_tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=device)
    scale = D ** -0.5
    peak, peak_src = _peaks()
    peak_tf = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak_tf = float(json.load(f)["bf16_tflops"])
    except Exception:  # noqa: BLE001
        peak_tf = 1590.0
    res = {}
    fa, fa_note = _vllm_varlen()
    for dtype in (torch.bfloat16, torch.float16):
        g = torch.Generator(device=device).manual_seed(11)
        q = torch.randn((T, Hq, D), generator=g, device=device).to(dtype)
        k = torch.randn((T, Hkv, D), generator=g, device=device).to(dtype)
        v = torch.randn((T, Hkv, D), generator=g, device=device).to(dtype)
        out = torch.empty_like(q)
        reps = max(3, min(args.steps, 20))
        ms = _time_calls(lambda: ops.flash_attn_varlen_prefill(q, k, v, cu, int(lens.max()), scale, out=out), reps,
                         device, stream)
        name = "bf16" if dtype == torch.bfloat16 else "fp16"
        res[name] = {"ms": ms, "tflops": flops / (ms / 1e3) / 1e12}
        if fa is not None:
            try:
                call = lambda: fa(q, k, v, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=int(lens.max()),  # noqa: E731
                                  max_seqlen_k=int(lens.max()), softmax_scale=scale, causal=True)
                fa_ms = _time_calls(call, reps, device, stream)
                ref_out = call()
                torch.cuda.synchronize(device)
                res[name]["vllm_fa_ms"] = fa_ms
                res[name]["vllm_fa_tflops"] = flops / (fa_ms / 1e3) / 1e12
                res[name]["max_abs_diff_vs_vllm_fa"] = float((ref_out.float() - out.float()).abs().max())
            except Exception as e:  # noqa: BLE001
                res[name]["vllm_fa"] = f"failed: {type(e).__name__}: {str(e)[:160]}"
    # The prompt half of the cache write: every prompt token's K and V (bf16) into the blocks of
    # a 28-layer cache whose prompts own scattered blocks, layer 0 (vLLM's reshape_and_cache_flash
    # over the prompt tokens). Bytes: K and V read once and written once, plus the slots.
    nblk = int(sum((int(L) + 15) // 16 for L in lens))
    pool_blocks = max(4 * nblk, 1024)
    kv_pool = torch.zeros((pool_blocks, 28, 2, 16, Hkv, D), dtype=torch.bfloat16, device=device)
    perm = np.random.default_rng(5).permutation(pool_blocks)[:nblk]
    slots, b0 = [], 0
    for L in lens:  # each prompt's tokens fill its own blocks in order
        nb = (int(L) + 15) // 16
        blocks = perm[b0:b0 + nb]
        b0 += nb
        pos = np.arange(int(L))
        slots.append(blocks[pos // 16] * 16 + pos % 16)
    slot_t = torch.as_tensor(np.concatenate(slots).astype(np.int64), device=device)
    # Six input sets (more than L2 together) and a different layer per launch, so that no launch
    # finds its rows in L2; each launch timed alone between events (launches queued behind a sleep).
    g = torch.Generator(device=device).manual_seed(12)
    kns = [torch.randn((T, Hkv, D), generator=g, device=device).to(torch.bfloat16) for _ in range(6)]
    vns = [torch.randn((T, Hkv, D), generator=g, device=device).to(torch.bfloat16) for _ in range(6)]
    w_fns = [lambda l=l: ops.reshape_and_cache(kns[l % 6], vns[l % 6], kv_pool, l, slot_t) for l in range(13)]
    w_ms = statistics.median(_per_launch_ms(w_fns, device)[1:])

    def w_all():
        for fn in w_fns:
            fn()

    w_graph_ms = _graph_ms(w_all, 5, device) / len(w_fns)
    w_bytes = 2 * 2 * T * Hkv * D * 2 + T * 8
    res["prompt_cache_write"] = {"tokens": T, "us": w_ms * 1e3, "gbs": w_bytes / (w_ms / 1e3) / 1e9,
                                 "frac_of_hbm": w_bytes / (w_ms / 1e3) / 1e9 / peak,
                                 "graph_us": w_graph_ms * 1e3,
                                 "graph_frac_of_hbm": w_bytes / (w_graph_ms / 1e3) / 1e9 / peak,
                                 "bytes": w_bytes, "what": "bf16 K/V of every prompt token into scattered blocks "
                                                           "of one layer of a 28-layer cache, inputs and layers "
                                                           "rotated past L2; us: median launch alone between events; "
                                                           "graph_us: per launch in a CUDA graph of 13 back-to-back "
                                                           "launches"}
    del kns, vns
    del kv_pool
    # CPU baseline: the oracle (numpy, fp64) on the batch's shortest prompt of at least 256 tokens
    Ls = int(min([L for L in lens if L >= 256] or [int(lens.min())]))
    rng = np.random.default_rng(0)
    qb, kb, vb = (orc.f64_to_bits(rng.standard_normal((Ls, h, D)), orc.BF16) for h in (Hq, Hkv, Hkv))
    t0 = time.perf_counter()
    orc.np_prefill_attention(qb, kb, vb, [0, Ls], scale, orc.BF16)
    cpu_s = time.perf_counter() - t0
    cpu_tf = 4.0 * Hq * D * Ls * (Ls + 1) / 2 / cpu_s / 1e12
    b = res["bf16"]
    return {
        "metric": "prefill-attn TFLOP/s", "value": b["tflops"], "unit": "TFLOP/s", "n_gpus": 1, "steps": reps,
        "warmup": 1, "ms_per_step": b["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic N(0,1) q/k/v",
        "config": {"workload": f"{len(lens)} prompts, lengths round(lognormal(6.5, 0.8)) in [16, 8192] (sum {T}, "
                               f"max {int(lens.max())}), causal, Hq 28 / Hkv 4 / D 128",
                   "prompt_lengths": lens.tolist()},
        "detail": res, "vllm_fa": fa_note,
        "roofline": {"bound": "tensor", "kernel": "prefill_tc_kernel (tcgen05.mma, TMEM accumulators, TMA)", "achieved": b["tflops"],
                     "peak": peak_tf, "unit": "TFLOP/s", "frac": b["tflops"] / peak_tf,
                     "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS burst)"},
        "cpu_baseline": {"value": cpu_tf, "unit": "TFLOP/s", "cores": 1, "kind": "port",
                         "sample": f"the oracle (numpy fp64) on one {Ls}-token prompt, all 28 heads"},
    }


def _prep_batches():
    """(name, seq_lens, context_lens, block lists) of the step-input benchmark: the cfg2 and cfg3
    decode batches and a mixed batch of 32 prompts (lognormal lengths) with 224 decode requests."""
    from aegaeon_b200 import synth

    out = []
    for name in ("cfg2", "cfg3"):
        lay = synth.make_layout(synth.CONFIGS[name])
        seq = lay.seq_lens.astype(np.int64)
        nb = (seq + 15) // 16
        tables = [lay.block_tables[i, :nb[i]].tolist() for i in range(len(seq))]
        out.append((f"{name} decode (B={len(seq)})", seq.tolist(), (seq - 1).tolist(), tables))
    rng = np.random.default_rng(5)
    seq = np.clip(np.round(rng.lognormal(6, 1, 256)), 4, 4096).astype(np.int64)
    ctx = np.where(np.arange(256) < 32, 0, seq - 1)
    perm = rng.permutation(1 << 20)
    tables, off = [], 0
    for n in seq:
        k = int((n + 15) // 16)
        tables.append(perm[off:off + k].tolist())
        off += k
    out.append(("mixed: 32 prompts + 224 decode", seq.tolist(), ctx.tolist(), tables))
    return out


def run_prep(args, world, rank, local):
    line = prep_line(args, local)
    if rank == 0:
        print(json.dumps(line), flush=True)


def prep_line(args, local) -> dict:
    """Per-step model inputs on the device (ops.prepare_step_inputs) against the reference's
    per-request Python loops restated in the oracle (Worker._prepare_model_inputs,
    aegaeon/aegaeon/worker.py:596-682), per batch: device microseconds per step (CUDA events,
    inputs resident) and the host loop's microseconds."""
    from aegaeon_b200 import ops
    from oracle import oracle as orc

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    stream = torch.cuda.current_stream(device)
    rows = {}
    for name, seq, ctx, tables in _prep_batches():
        B = len(seq)
        W = max(len(t) for t in tables)
        t = np.zeros((B, W), np.int32)
        for i, r in enumerate(tables):
            t[i, :len(r)] = r
        bt = torch.as_tensor(t, device=device)
        c = torch.as_tensor(np.asarray(ctx, np.int32), device=device)
        s = torch.as_tensor(np.asarray(seq, np.int32), device=device)
        T = int(sum(a - b for a, b in zip(seq, ctx)))
        out = ops.StepInputs(B, W, T, device)
        for _ in range(max(args.warmup, 3)):
            ops.prepare_step_inputs(bt, c, s, out=out)
        torch.cuda.synchronize(device)
        reps = 200
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            ops.prepare_step_inputs(bt, c, s, out=out)
        b.record(stream)
        torch.cuda.synchronize(device)
        dev_us = a.elapsed_time(b) / reps * 1e3
        want = orc.np_step_inputs(seq, ctx, tables)
        ok = out.slot_mapping[:T].cpu().numpy().tolist() == want["slot_mapping"].tolist()
        t0 = time.perf_counter()
        n_host = 0
        while time.perf_counter() - t0 < 1.0:
            orc.np_step_inputs(seq, ctx, tables)
            n_host += 1
        host_us = (time.perf_counter() - t0) / n_host * 1e6
        rows[name] = {"tokens": T, "device_us": dev_us, "host_loop_us": host_us, "matches_oracle": ok}
    first = rows[next(iter(rows))]
    return {
            "metric": "step-input prep us", "value": first["device_us"], "unit": "us", "n_gpus": 1, "steps": 200,
            "warmup": max(args.warmup, 3), "ms_per_step": first["device_us"] / 1e3, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "int32/int64", "data": "synthetic (bench configs)",
            "config": {"workload": "slot mapping, positions, start offsets and attention table rows of one step; "
                                   "value = the cfg2 decode batch"},
            "batches": rows,
            "cpu_baseline": {"value": first["host_loop_us"], "unit": "us", "cores": 1, "kind": "port",
                             "sample": "the oracle's restatement of the reference's per-request Python loops "
                                       "(no tensor creation or host-to-device copies), timed for 1 s"},
    }


# ------------------------------------------------------------------------------------------
# Reference arm: the reference path on the host cores (decode), or its own swap operator (cfg5)


def run_reference_swap(args, world, rank):
    """cfg5 reference arm: the reference's own aegaeon.ops.swap (built from its sources into
    oracle/_ref) on the cfg5 swap set, through its public signature on the current stream."""
    ref = _load_reference_swap()
    if ref is None:
        print(json.dumps({"impl": "reference", "metric": "KV-block swap GB/s",
                          "unavailable": "oracle/_ref/aegaeon_ref_ops.so is not built (needs the reference checkout)"}),
              flush=True)
        return
    from aegaeon_b200 import layout, synth

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    c = dict(synth.SWAP_CFG)
    shape = (c["device_blocks"],) + layout.kv_block_shape(c["num_layers"], c["num_kv_heads"], c["head_dim"])
    kv = torch.empty(shape, dtype=c["dtype"], device=device)
    synth.random_bits_(kv, c["seed"])
    bb = layout.block_bytes(kv)
    n = c["swap_blocks"]
    host = torch.empty((n,) + shape[1:], dtype=c["dtype"]).pin_memory()
    g = torch.Generator().manual_seed(c["seed"])
    out_ids = torch.randperm(c["device_blocks"], generator=g)[:n].tolist()
    host_ids = torch.randperm(n, generator=g).tolist()
    for _ in range(args.warmup):
        ref.swap(out_ids, host_ids, False, kv, host)
    torch.cuda.synchronize(device)
    ms = _timed_ms(lambda: ref.swap(out_ids, host_ids, False, kv, host), args.steps, device, warm=0)
    gbs = n * bb / (ms / 1e3) / 1e9
    print(json.dumps({
        "impl": "reference", "metric": "KV-block swap GB/s", "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u16", "data": "synthetic random 16-bit patterns",
        "config": {"workload": f"cfg5: swap-out of {n} scattered {bb:,}-byte blocks of a {c['device_blocks']}-block "
                               "pool to pinned host memory"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": 1, "kind": "reference",
                         "sample": "the reference's aegaeon.ops.swap (one cudaMemcpyAsync per block) on the whole set"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference(args, world, rank):
    if rank != 0:
        return
    from aegaeon_b200 import synth

    if args.config == "weights":
        run_weights(args, world, rank, int(os.environ.get("LOCAL_RANK", "0")), reference_only=True)
        return
    if args.config == "prefill":
        print(json.dumps({"impl": "reference", "metric": "prefill-attn TFLOP/s",
                          "unavailable": "the reference's prefill attention is vLLM 0.5.1's FlashAttention (absent); "
                                         "--config prefill times vLLM's bundled FlashAttention beside this library"}),
              flush=True)
        return
    if args.config == "prep":
        print(json.dumps({"impl": "reference", "metric": "step-input prep us",
                          "unavailable": "the reference builds step inputs in Python inside Worker (ray, vLLM); "
                                         "its loop is timed as the cpu_baseline of --config prep"}), flush=True)
        return
    if args.config == "migrate":
        print(json.dumps({"impl": "reference", "metric": "KV-block migration GB/s",
                          "unavailable": "the reference's GPU -> GPU migration is a stub (Worker.migrate_blocks "
                                         "raises NotImplementedError, aegaeon/aegaeon/worker.py:851)"}), flush=True)
        return
    if args.config == "cfg5":
        run_reference_swap(args, world, rank)
        return
    cfg = synth.CONFIGS[args.config]
    lay = synth.make_layout(cfg)  # the whole batch: the CPU path serves the whole job at any N
    # each step is a whole L-layer step of a bounded sample, sized so that the run ends in minutes
    target = min(6.0, 150.0 / max(1, args.steps + args.warmup))
    smp = CpuDecodeSample(cfg, lay, target_step_s=target)
    for _ in range(args.warmup):
        smp.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        smp.step()
    secs = time.perf_counter() - t0
    value = smp.batch / (secs / args.steps)
    sample = smp.describe(f"{args.steps} timed steps after {args.warmup} warm-up steps")
    line = {
        "metric": "decode-attn tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if cfg.name == "cfg3" else "weak", "vs_baseline": None,
        "dtype": "fp16" if cfg.dtype == torch.float16 else "bf16", "impl": "reference",
        "data": "synthetic: seeded contexts, block tables and N(0, std^2) K/V/q (no dataset on this path)",
        "config": decode_config(cfg, world, fused=not args.unfused, split=args.split),
        "compute": "fp32 (storage dtype in and out)",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": smp.threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference's cache write and decode attention are un-vendored vLLM 0.5.1 CUDA kernels with no "
                 "CPU path; this arm runs their fp32 PyTorch restatement on the host cores, one process serving the "
                 "whole job whatever N is"),
    }
    print(json.dumps(line), flush=True)


def main():
    args = _args()
    world, rank, local = _dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=180),
                                             device_id=torch.device("cuda", local))
    try:
        if args.config == "cfg5":
            if rank == 0:
                run_swap(args, world, rank, local)
        elif args.config == "migrate":
            run_migrate(args, world, rank, local)
        elif args.config == "prep":
            if rank == 0:
                run_prep(args, world, rank, local)
        elif args.config == "weights":
            if rank == 0:
                run_weights(args, world, rank, local)
        elif args.config == "prefill":
            if rank == 0:
                run_prefill(args, world, rank, local)
        else:
            run_decode(args, world, rank, local)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark of the Aegaeon per-token serving hot path on B200.

Default workload (``--config cfg2``): one Qwen2.5-7B decode step = 28 layers x (reshape_and_cache
of one new token per sequence + paged decode attention), batch 64, lognormal contexts, a pool of
16384 blocks (15 GB fp16). A step is captured once as a CUDA graph (the plan, then per layer the
fused cache-write/attention launch and its split merge) and replayed; the KV read per step
(1.6 GB) is far larger than the 126 MB L2, so no flush is needed.

One JSON line on rank 0 (see the keys below). ``--impl reference`` times the CPU restatement of
the reference's path (the oracle, all host threads) on the same workload.
``--config cfg5`` measures the swap / copy_blocks path instead (GB/s).

Multi-GPU: one process per GPU (torchrun); every rank runs its own cfg2 batch on its own pool
(weak scaling, no data-path collective); the step time is the max over ranks.
"""
from __future__ import annotations

import argparse
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
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="cfg2", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "migrate", "prep", "weights", "prefill"])
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle timing")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    p.add_argument("--unfused", action="store_true",
                   help="run each layer as reshape_and_cache + paged_attention_decode (two operators)")
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


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
# CPU restatement timing (oracle): the reference arm and the cpu_baseline leg


def _cpu_decode_setup(cfg, lay, seed=0):
    """Compact host copy of the workload: only the blocks the batch uses, values N(0, std^2)."""
    from aegaeon_b200.layout import BLOCK_SIZE
    from oracle import oracle as orc

    nb = (lay.seq_lens.astype(np.int64) + BLOCK_SIZE - 1) // BLOCK_SIZE
    compact = np.zeros_like(lay.block_tables)
    off = 0
    for i, n in enumerate(nb):
        compact[i, :n] = np.arange(off, off + n)
        off += n
    n_used = int(off)
    g = torch.Generator().manual_seed(seed)
    L, Hkv, D, Hq, B = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, cfg.num_q_heads, cfg.batch
    # one layer's K/V blocks are enough: every layer call reads the same amount (layers differ only in
    # their data), so the sample reuses this layer's values for each timed call.
    kv = (torch.randn((n_used, 2, 16, Hkv, D), generator=g) * cfg.value_std).to(cfg.dtype)
    kvb = kv.view(torch.int16).numpy().view(np.uint16)
    q = (torch.randn((B, Hq, D), generator=g) * cfg.value_std).to(cfg.dtype).view(torch.int16).numpy().view(np.uint16)
    knew = (torch.randn((B, Hkv, D), generator=g)).to(cfg.dtype).view(torch.int16).numpy().view(np.uint16)
    slots = np.empty(B, np.int64)
    pos = lay.seq_lens.astype(np.int64) - 1
    slots[:] = compact[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    dtype = orc.BF16 if cfg.dtype == torch.bfloat16 else orc.FP16
    return dict(kvb=kvb, q=q, knew=knew, slots=slots, tables=compact, n_used=n_used, dtype=dtype)


def _cpu_layer_call(cfg, lay, st, threads):
    from oracle import oracle as orc

    kvb = st["kvb"]
    flat = kvb.reshape(-1)
    blk = 2 * 16 * cfg.num_kv_heads * cfg.head_dim
    half = 16 * cfg.num_kv_heads * cfg.head_dim
    orc.c_reshape_and_cache(st["knew"], st["knew"], flat, flat[half:], blk, st["n_used"], st["slots"])
    orc.c_paged_attention(st["q"], flat, flat[half:], blk, st["tables"], lay.seq_lens, cfg.num_kv_heads,
                          1.0 / math.sqrt(cfg.head_dim), st["dtype"], threads)


def cpu_decode_throughput(cfg, lay, budget_s: float, max_calls: int | None = None, warmup: int = 1):
    """tokens/s of the CPU restatement: B / (mean layer-call time x L), plus the sample description."""
    threads = _host_threads()
    st = _cpu_decode_setup(cfg, lay)
    for _ in range(warmup):
        _cpu_layer_call(cfg, lay, st, threads)
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        _cpu_layer_call(cfg, lay, st, threads)
        times.append(time.perf_counter() - t0)
        if max_calls is not None and len(times) >= max_calls:
            break
        if max_calls is None and time.perf_counter() - t_start >= budget_s:
            break
    per_layer = statistics.mean(times)
    value = cfg.batch / (per_layer * cfg.num_layers)
    sample = (f"{len(times)} layer calls (reshape_and_cache + decode attention over all {cfg.batch} sequences, "
              f"sum ctx {lay.total_tokens}) timed, tokens/s = B / (mean call time x {cfg.num_layers} layers)")
    return value, threads, sample, per_layer


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


def _per_launch_ms(fn_list, device, sleep_cycles=int(4e7)):
    """Device durations of launches measured with CUDA events on the launching stream.

    A sleep kernel is queued first so that the host enqueues every (event, launch, event) triple
    before the device reaches them; launches then run back to back and each event pair brackets
    exactly one kernel.
    """
    stream = torch.cuda.current_stream(device)
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


def run_decode(args, world, rank, local):
    from aegaeon_b200 import ops, synth
    from aegaeon_b200.step import DecodePipeline, DecodeStep

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = synth.CONFIGS[args.config]
    if cfg.name == "cfg3" and world > 1:
        lay = synth.make_layout(cfg, rank, world)  # strong split of the batch across ranks
        scaling = "strong"
    else:
        lay = synth.make_layout(cfg)
        scaling = "weak"
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
        for _ in range(50):
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
    ms = _max_over_ranks(e0.elapsed_time(e1), world, device)
    clock_info = clocks.stop()

    # Per-launch durations of the dominant kernel (the layer's attention launch with its split
    # merge; fused with the cache write unless --unfused) and of the separate cache write.
    n_prof = max(1, min(args.steps, 8))
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
    plan_ms = _per_launch_ms([lambda: step.plan.plan(step.seq_lens, step.block_tables)] * 4, device)

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

    # Sanity: the timed outputs are finite (the work was done).
    assert torch.isfinite(step.out.float()).all(), "non-finite attention output"

    algo = synth.algorithmic_bytes_per_layer(cfg, lay)
    ms_step = ms / args.steps
    tokens_total = B * world
    value = tokens_total / (ms_step / 1e3)
    kv_step = algo["kv_read"] * L
    attn_avg_ms = statistics.mean(attn_ms)
    launch_bytes = algo["attention"] + (algo["reshape_and_cache"] if step.fused else 0)
    # The dominant kernel's duration in the timed steps: the step time (CUDA events over the timed
    # region) less the plan launch, per layer launch. Inside the step graph consecutive layer
    # launches overlap through programmatic dependent launch, so this is the time a layer adds to
    # the step; an isolated launch (events around it alone) also carries launch latency.
    plan_med_ms = statistics.median(plan_ms)
    in_step_ms = max((ms / args.steps - plan_med_ms) / L, 1e-6)
    if not step.fused:
        in_step_ms = max((ms / args.steps - plan_med_ms - L * statistics.median(write_ms)) / L, 1e-6)
    achieved = launch_bytes / (in_step_ms / 1e3) / 1e9
    achieved_isolated = launch_bytes / (attn_avg_ms / 1e3) / 1e9
    peak, peak_src = _peaks()
    traffic = _ncu_traffic(f"decode_attn_{cfg.name}")

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
        "config": {
            "workload": f"{cfg.name}: {cfg.model} decode step, {L} layers x (reshape_and_cache + paged decode "
                        f"attention), one new token per sequence",
            "batch_per_gpu": B, "layers": L, "q_heads": Hq, "kv_heads": Hkv, "head_dim": D, "block_size": 16,
            "pool_blocks": lay.num_blocks, "sum_ctx": lay.total_tokens, "max_ctx": int(lay.seq_lens.max()),
            "kv_bytes_per_step": kv_step, "accumulate": "fp32",
            "l2": f"inputs larger than L2: {kv_step / 1e9:.2f} GB of K/V read per step vs 126 MB L2 (no flush)",
            "parallelism": f"{world} GPU(s), one process each, own pool and batch, no collective",
            "launch": ("one CUDA graph per step: plan + per layer one fused cache-write/attention/split-merge "
                       "launch (PDL)" if step.fused else
                       "one CUDA graph per step: plan + per layer reshape_and_cache and attention (PDL)"),
        },
        "kv_read_gbs": kv_step * world / (ms_step / 1e3) / 1e9,
        "hbm_frac_step": (algo["attention"] + algo["reshape_and_cache"]) * L / (ms_step / 1e3) / 1e9 / peak,
        "e2e": {
            "value": tokens_total / (e2e_ms / args.steps / 1e3),
            "unit": "tokens/s",
            "h2d_bytes_per_step": step.input_bytes(),
            "d2h_bytes_per_step": step.output_bytes(),
            "ms_per_step": e2e_ms / args.steps,
            "path": "aegaeon_b200.step.DecodePipeline.run: per step pinned host inputs -> H2D (upload stream), "
                    "graph replay, D2H of the outputs (download stream); copies of neighbouring steps overlap "
                    "the kernels",
        },
        "gpu_launches": args.steps * step.launches_per_step,
        "roofline": {
            "bound": "hbm",
            "kernel": "decode_attn_kernel (fused cache write + attention + split merge, one launch per layer)",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": peak_src,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": launch_bytes,
            "duration": "per layer launch in the timed step graph: (step - plan) / layers",
            "in_step_launch_us": in_step_ms * 1e3,
            "avg_launch_us": attn_avg_ms * 1e3,
            "achieved_isolated_launch": achieved_isolated,
            "frac_isolated_launch": achieved_isolated / peak,
            "launches_timed": len(attn_ms),
            "reshape_and_cache_median_us": statistics.median(write_ms) * 1e3,
            "plan_median_us": statistics.median(plan_ms) * 1e3,
        },
        "clocks": clock_info,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        v, cores, sample, _ = cpu_decode_throughput(cfg, lay, args.cpu_seconds)
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del step, kv


def run_swap(args, world, rank, local):
    """cfg5: swap out/in of 4096 scattered blocks and copy_blocks of 8192 pairs (GB/s)."""
    from aegaeon_b200 import layout, ops, synth

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    c = dict(synth.SWAP_CFG)
    if args.scale != 1.0:
        for k in ("device_blocks", "swap_blocks", "copy_pairs"):
            c[k] = max(2, int(c[k] * args.scale))
        c["copy_pairs"] = min(c["copy_pairs"], c["device_blocks"] // 2)
        c["swap_blocks"] = min(c["swap_blocks"], c["device_blocks"])
    shape = (c["device_blocks"],) + layout.kv_block_shape(c["num_layers"], c["num_kv_heads"], c["head_dim"])
    kv = torch.empty(shape, dtype=c["dtype"], device=device)
    synth.random_bits_(kv, c["seed"])
    bb = layout.block_bytes(kv)
    host = torch.empty((c["swap_blocks"],) + shape[1:], dtype=c["dtype"]).pin_memory()
    g = torch.Generator().manual_seed(c["seed"])
    out_ids = torch.randperm(c["device_blocks"], generator=g)[:c["swap_blocks"]].tolist()
    host_ids = torch.randperm(c["swap_blocks"], generator=g).tolist()
    in_ids = torch.randperm(c["device_blocks"], generator=g)[:c["swap_blocks"]].tolist()
    p = torch.randperm(c["device_blocks"], generator=g)
    src = p[:c["copy_pairs"]].to(device)
    dst = p[c["copy_pairs"]:2 * c["copy_pairs"]].to(device)
    d_out, d_host, d_in = (torch.as_tensor(x, device=device) for x in (out_ids, host_ids, in_ids))
    stream = torch.cuda.current_stream(device)

    def timed(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / reps

    reps = max(1, min(args.steps, 5))
    n = c["swap_blocks"]
    res = {
        "swap_out_dma_ms": timed(lambda: ops.swap(out_ids, host_ids, False, kv, host), reps),
        "swap_in_dma_ms": timed(lambda: ops.swap(host_ids, in_ids, True, kv, host), reps),
        "swap_out_sm_ms": timed(lambda: ops.swap_sm(d_out, d_host, False, kv, host), reps),
        "swap_in_sm_ms": timed(lambda: ops.swap_sm(d_host, d_in, True, kv, host), reps),
        "copy_blocks_ms": timed(lambda: ops.copy_blocks(src, dst, kv), max(reps, 10)),
    }
    # host-link reference: one contiguous pinned 1 GiB copy each way
    big_h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    big_d = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    res["link_h2d_gbs"] = (1 << 30) / (timed(lambda: big_d.copy_(big_h, non_blocking=True), 5) / 1e3) / 1e9
    res["link_d2h_gbs"] = (1 << 30) / (timed(lambda: big_h.copy_(big_d, non_blocking=True), 5) / 1e3) / 1e9
    gbs = {k.replace("_ms", "_gbs"): (n * bb if "swap" in k else 2 * c["copy_pairs"] * bb) / (v / 1e3) / 1e9
           for k, v in res.items() if k.endswith("_ms")}
    best_swap = max(gbs["swap_out_dma_gbs"], gbs["swap_out_sm_gbs"])
    peak, peak_src = _peaks()
    line = {
        "metric": "KV-block swap GB/s", "value": best_swap, "unit": "GB/s", "n_gpus": 1, "steps": reps,
        "warmup": 2, "ms_per_step": min(res["swap_out_dma_ms"], res["swap_out_sm_ms"]), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u16", "data": "synthetic random 16-bit patterns",
        "config": {"workload": f"cfg5: {n} scattered {bb:,}-byte blocks HBM -> pinned host (swap-out); "
                               f"back into fresh ids; copy_blocks {c['copy_pairs']} pairs"
                               + ("" if args.scale == 1.0 else f" (scaled x{args.scale})")},
        "detail_ms": res, "detail_gbs": gbs,
        "swap_frac_of_link": {"out": best_swap / res["link_d2h_gbs"],
                              "in": max(gbs["swap_in_dma_gbs"], gbs["swap_in_sm_gbs"]) / res["link_h2d_gbs"]},
        "roofline": {"bound": "hbm", "kernel": "block_copy_vec_kernel (copy_blocks)", "achieved": gbs["copy_blocks_gbs"],
                     "peak": peak, "unit": "GB/s", "frac": gbs["copy_blocks_gbs"] / peak, "peak_source": peak_src,
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


def run_weights(args, world, rank, local, reference_only=False):
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
    print(json.dumps({
        "metric": "weight-switch GB/s", "value": best, "unit": "GB/s", "n_gpus": 1, "steps": reps, "warmup": 1,
        "ms_per_step": min(res["dma_ms"], res["sm_ms"]), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic parameter bytes", "config": {"workload": workload},
        "detail_ms": res, "detail_gbs": gbs, "first_mib_matches": ok,
        "roofline": {"bound": "host link", "achieved": best, "peak": gbs["link_contiguous_gbs"], "unit": "GB/s",
                     "frac": best / gbs["link_contiguous_gbs"],
                     "peak_source": "measured here: one contiguous 1 GiB pinned host-to-device copy"},
        "cpu_baseline": {"value": gbs["reference_loop_gbs"], "unit": "GB/s", "cores": 1, "kind": "reference",
                         "sample": "the reference's per-parameter copy_ loop (torch), whole model"},
    }), flush=True)


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
    # CPU baseline: the oracle (numpy, fp64) on the batch's shortest prompt of at least 256 tokens
    Ls = int(min([L for L in lens if L >= 256] or [int(lens.min())]))
    rng = np.random.default_rng(0)
    qb, kb, vb = (orc.f64_to_bits(rng.standard_normal((Ls, h, D)), orc.BF16) for h in (Hq, Hkv, Hkv))
    t0 = time.perf_counter()
    orc.np_prefill_attention(qb, kb, vb, [0, Ls], scale, orc.BF16)
    cpu_s = time.perf_counter() - t0
    cpu_tf = 4.0 * Hq * D * Ls * (Ls + 1) / 2 / cpu_s / 1e12
    b = res["bf16"]
    print(json.dumps({
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
    }), flush=True)


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
    if rank == 0:
        first = rows[next(iter(rows))]
        print(json.dumps({
            "metric": "step-input prep us", "value": first["device_us"], "unit": "us", "n_gpus": 1, "steps": 200,
            "warmup": max(args.warmup, 3), "ms_per_step": first["device_us"] / 1e3, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "int32/int64", "data": "synthetic (bench configs)",
            "config": {"workload": "slot mapping, positions, start offsets and attention table rows of one step; "
                                   "value = the cfg2 decode batch"},
            "batches": rows,
            "cpu_baseline": {"value": first["host_loop_us"], "unit": "us", "cores": 1, "kind": "port",
                             "sample": "the oracle's restatement of the reference's per-request Python loops "
                                       "(no tensor creation or host-to-device copies), timed for 1 s"},
        }), flush=True)


# ------------------------------------------------------------------------------------------
# Reference arm: the CPU restatement of the reference's path on the host cores


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
    name = args.config if args.config != "cfg5" else "cfg2"
    cfg = synth.CONFIGS[name]
    lay = synth.make_layout(cfg)
    # each step is one layer call of the full batch; cap the count so the run stays within minutes
    budget_calls = args.steps
    t_probe = time.perf_counter()
    threads = _host_threads()
    st = _cpu_decode_setup(cfg, lay)
    _cpu_layer_call(cfg, lay, st, threads)
    one = time.perf_counter() - t_probe
    max_calls = max(1, min(budget_calls, int(150.0 / max(one, 1e-3))))
    for _ in range(min(args.warmup, 3)):
        _cpu_layer_call(cfg, lay, st, threads)
    times = []
    for _ in range(max_calls):
        t0 = time.perf_counter()
        _cpu_layer_call(cfg, lay, st, threads)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.mean(times)
    value = cfg.batch / (per_layer * cfg.num_layers)
    sample = (f"{len(times)} of {args.steps} requested steps, each one layer call (reshape_and_cache + decode "
              f"attention over all {cfg.batch} sequences, sum ctx {lay.total_tokens}); tokens/s = "
              f"B / (mean call time x {cfg.num_layers} layers)")
    line = {
        "metric": "decode-attn tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": len(times),
        "warmup": min(args.warmup, 3), "ms_per_step": per_layer * cfg.num_layers * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp64 (restatement)", "impl": "reference",
        "data": "synthetic: seeded contexts, block tables and N(0, std^2) values",
        "config": {"workload": f"{cfg.name}: {cfg.model} decode step, {cfg.num_layers} layers x (reshape_and_cache + "
                               f"paged decode attention)", "batch_per_gpu": cfg.batch, "sum_ctx": lay.total_tokens},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference's attention and cache write live in un-vendored vLLM 0.5.1 with no CPU path; "
                 "this arm runs the C restatement of the path (oracle/oracle.c) with all host threads"),
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

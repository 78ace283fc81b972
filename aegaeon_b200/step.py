"""Decode-step runner: the attention half of ``Worker.step`` captured as one CUDA graph.

Per decode step the reference worker (``aegaeon/aegaeon/worker.py:456-552``) builds the attention
metadata once (``:554-713``) and then, for each of the L layers, writes the new token's K/V into
its slot and runs paged decode attention over the cache (``:517-523``). ``DecodeStep`` owns static
device buffers for those per-step inputs, records one step (plan + L x (cache write + attention))
into a CUDA graph, and replays it; ``run_from_host`` is the end-to-end form that copies the step's
inputs from page-locked host memory and reads the outputs back.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class StepShape:
    batch: int
    num_layers: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    table_width: int


class DecodeStep:
    """One decode step over an L-layer cache. ``fused=True`` (default) runs each layer as one
    fused cache-write + attention launch (``ops.decode_layer``, plus its split merge);
    ``fused=False`` runs the two operators the reference calls per layer (``reshape_and_cache``
    then ``paged_attention_decode``) with ``slot_mapping`` as given."""

    def __init__(self, kv_cache: torch.Tensor, num_q_heads: int, batch: int, table_width: int, scale: float,
                 fused: bool = True):
        if kv_cache.dim() != 6:
            raise ValueError("kv_cache must be (N, L, 2, 16, Hkv, D)")
        dev = kv_cache.device
        L, Hkv, D = kv_cache.size(1), kv_cache.size(4), kv_cache.size(5)
        self.kv_cache = kv_cache
        self.shape = StepShape(batch, L, num_q_heads, Hkv, D, table_width)
        self.scale = float(scale)
        dt = kv_cache.dtype
        self.q = torch.zeros((L, batch, num_q_heads, D), dtype=dt, device=dev)
        self.k_new = torch.zeros((L, batch, Hkv, D), dtype=dt, device=dev)
        self.v_new = torch.zeros((L, batch, Hkv, D), dtype=dt, device=dev)
        self.out = torch.zeros((L, batch, num_q_heads, D), dtype=dt, device=dev)
        self.slot_mapping = torch.zeros((batch,), dtype=torch.int64, device=dev)
        self.block_tables = torch.zeros((batch, table_width), dtype=torch.int32, device=dev)
        self.seq_lens = torch.zeros((batch,), dtype=torch.int32, device=dev)
        self.plan = ops.DecodePlan(batch, num_q_heads, Hkv, D, dev)
        self.fused = fused
        self.graph: torch.cuda.CUDAGraph | None = None

    @property
    def launches_per_step(self) -> int:
        """Kernels one step launches: the plan, then per layer the fused cache-write/attention
        launch (fused) or the cache write and the attention (unfused)."""
        return 1 + (1 if self.fused else 2) * self.shape.num_layers

    def run_eager(self) -> None:
        """One step on the current stream, op by op."""
        self.plan.plan(self.seq_lens, self.block_tables)
        for layer in range(self.shape.num_layers):
            if self.fused:
                # Each layer's launch follows the previous layer's (which writes only its own layer's
                # rows) or the plan: its first K/V tiles may be requested before that kernel ends.
                ops.decode_layer(self.out[layer], self.q[layer], self.k_new[layer], self.v_new[layer], self.kv_cache,
                                 layer, self.block_tables, self.seq_lens, self.scale, plan=self.plan, prefetch=True)
            else:
                # The cache write stores each sequence's newest row (slot_mapping holds the decode
                # slots, position seq_len - 1): the attention may request its tiles early and
                # reads that row again once the write has finished.
                ops.reshape_and_cache(self.k_new[layer], self.v_new[layer], self.kv_cache, layer, self.slot_mapping)
                ops.paged_attention_decode(self.out[layer], self.q[layer], self.kv_cache, layer, self.block_tables,
                                           self.seq_lens, self.scale, plan=self.plan, after_decode_write=True)

    def capture(self) -> "DecodeStep":
        """Records one step into a CUDA graph (after one eager warm-up step on a side stream)."""
        side = torch.cuda.Stream(self.kv_cache.device)
        side.wait_stream(torch.cuda.current_stream(self.kv_cache.device))
        with torch.cuda.stream(side):
            self.run_eager()
        torch.cuda.current_stream(self.kv_cache.device).wait_stream(side)
        torch.cuda.synchronize(self.kv_cache.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.run_eager()
        self.graph = g
        return self

    def replay(self) -> None:
        if self.graph is None:
            self.capture()
        self.graph.replay()

    def load_inputs(self, q, k_new, v_new, slot_mapping, block_tables, seq_lens) -> None:
        """Copies one step's inputs into the static buffers (asynchronous if the sources are pinned)."""
        self.q.copy_(q, non_blocking=True)
        self.k_new.copy_(k_new, non_blocking=True)
        self.v_new.copy_(v_new, non_blocking=True)
        self.slot_mapping.copy_(slot_mapping, non_blocking=True)
        self.block_tables.copy_(block_tables, non_blocking=True)
        self.seq_lens.copy_(seq_lens, non_blocking=True)

    def run_from_host(self, host_inputs: dict, host_out: torch.Tensor) -> None:
        """End-to-end step: host inputs -> device, replay, device outputs -> ``host_out`` (pinned)."""
        self.load_inputs(**host_inputs)
        self.replay()
        host_out.copy_(self.out, non_blocking=True)

    def input_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.q, self.k_new, self.v_new, self.slot_mapping, self.block_tables, self.seq_lens))

    def output_bytes(self) -> int:
        return self.out.numel() * self.out.element_size()


class DecodePipeline:
    """End-to-end decode steps with the host transfers overlapped with the compute.

    Two ``DecodeStep`` slots share the KV cache, each with its own input/output buffers, plan
    workspace and CUDA graph. Step i runs in slot i % 2 on the compute stream while the inputs of
    step i + 1 are copied into the other slot on an upload stream and the outputs of step i - 1
    are read back on a download stream (the link is full duplex). Every step still copies its
    own inputs from page-locked host memory and reads its own outputs back; only the order of
    those copies relative to the kernels changes. Compute stays in step order, so a step's cache
    writes are made before the next step's attention reads the cache, as in the reference.
    """

    def __init__(self, kv_cache: torch.Tensor, num_q_heads: int, batch: int, table_width: int, scale: float,
                 fused: bool = True):
        self.slots = [DecodeStep(kv_cache, num_q_heads, batch, table_width, scale, fused) for _ in range(2)]
        dev = kv_cache.device
        self.device = dev
        self.up = torch.cuda.Stream(dev)
        self.down = torch.cuda.Stream(dev)
        self._loaded = [torch.cuda.Event() for _ in range(2)]   # slot inputs uploaded
        self._computed = [torch.cuda.Event() for _ in range(2)]  # slot step finished (inputs free, outputs ready)
        self._read = [torch.cuda.Event() for _ in range(2)]      # slot outputs read back (outputs free)

    @property
    def step(self) -> DecodeStep:
        return self.slots[0]

    def capture(self) -> "DecodePipeline":
        for s in self.slots:
            s.capture()
        return self

    def run(self, host_inputs, host_outs, steps: int) -> None:
        """Runs ``steps`` steps; step i reads ``host_inputs[i % len]`` (dict of pinned tensors as for
        ``DecodeStep.load_inputs``) and writes its outputs to ``host_outs[i % 2]`` (pinned). Returns
        with all copies enqueued; the current stream waits for the last read-back."""
        compute = torch.cuda.current_stream(self.device)
        self.up.wait_stream(compute)
        self.down.wait_stream(compute)

        def upload(i):
            s = i % 2
            if i >= 2:
                self.up.wait_event(self._computed[s])  # step i - 2 no longer reads these inputs
            with torch.cuda.stream(self.up):
                self.slots[s].load_inputs(**host_inputs[i % len(host_inputs)])
                self._loaded[s].record(self.up)

        upload(0)
        for i in range(steps):
            s = i % 2
            if i + 1 < steps:
                upload(i + 1)
            compute.wait_event(self._loaded[s])
            if i >= 2:
                compute.wait_event(self._read[s])  # the outputs of step i - 2 have been read back
            self.slots[s].replay()
            self._computed[s].record(compute)
            self.down.wait_event(self._computed[s])
            with torch.cuda.stream(self.down):
                host_outs[s].copy_(self.slots[s].out, non_blocking=True)
                self._read[s].record(self.down)
        compute.wait_stream(self.down)
        compute.wait_stream(self.up)

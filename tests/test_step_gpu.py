"""Decode-step runners on the GPU: the captured step equals the per-layer operators, and the
pipelined end-to-end runner returns, for every step, exactly what a step run alone returns."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import ops
from aegaeon_b200.step import DecodePipeline, DecodeStep
from tests.gpu_helpers import make_tables

pytestmark = pytest.mark.gpu

SCALE = 1.0 / np.sqrt(128)


def _setup(device, seed=0, B=8, L=2, Hq=8, Hkv=2):
    rng = np.random.default_rng(seed)
    seq_lens = rng.integers(1, 400, size=B).astype(np.int32)
    nb = int(((seq_lens + 15) // 16).sum())
    N = nb + 4
    tables = make_tables(seq_lens, N, seed)
    g = torch.Generator(device=device).manual_seed(seed)
    kv = torch.randn((N, L, 2, 16, Hkv, 128), generator=g, device=device).to(torch.float16)
    return kv, tables, seq_lens, (B, L, Hq, Hkv)


def _inputs(device, shape, tables, seq_lens, seed):
    B, L, Hq, Hkv = shape
    g = torch.Generator(device=device).manual_seed(seed)
    pos = seq_lens.astype(np.int64) - 1
    slots = tables[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    return dict(q=torch.randn((L, B, Hq, 128), generator=g, device=device).to(torch.float16),
                k_new=torch.randn((L, B, Hkv, 128), generator=g, device=device).to(torch.float16),
                v_new=torch.randn((L, B, Hkv, 128), generator=g, device=device).to(torch.float16),
                slot_mapping=torch.as_tensor(slots, device=device),
                block_tables=torch.as_tensor(tables, device=device),
                seq_lens=torch.as_tensor(seq_lens, device=device))


def test_captured_step_equals_per_layer_operators(cuda_device):
    kv, tables, seq_lens, shape = _setup(cuda_device)
    B, L, Hq, Hkv = shape
    inp = _inputs(cuda_device, shape, tables, seq_lens, 1)
    kv_ref = kv.clone()
    step = DecodeStep(kv, Hq, B, tables.shape[1], SCALE)
    step.load_inputs(**inp)
    step.capture()
    step.replay()
    torch.cuda.synchronize()
    plan = ops.DecodePlan(B, Hq, Hkv, 128, cuda_device).plan(inp["seq_lens"], inp["block_tables"])
    for layer in range(L):
        out = torch.empty_like(inp["q"][layer])
        ops.decode_layer(out, inp["q"][layer], inp["k_new"][layer], inp["v_new"][layer], kv_ref, layer,
                         inp["block_tables"], inp["seq_lens"], SCALE, plan=plan)
        assert torch.equal(out.view(torch.int16), step.out[layer].view(torch.int16)), layer
    assert torch.equal(kv.view(torch.int16), kv_ref.view(torch.int16))


def test_pipeline_steps_equal_single_steps(cuda_device):
    kv, tables, seq_lens, shape = _setup(cuda_device, seed=3)
    B, L, Hq, Hkv = shape
    steps = 5
    host_inputs = [{k: v.cpu().pin_memory() for k, v in _inputs(cuda_device, shape, tables, seq_lens, 10 + i).items()}
                   for i in range(3)]
    # reference: each step alone through run_from_host, on its own copy of the cache
    kv_ref = kv.clone()
    single = DecodeStep(kv_ref, Hq, B, tables.shape[1], SCALE)
    single.load_inputs(**host_inputs[0])
    single.capture()
    want = []
    for i in range(steps):
        out = torch.empty(single.out.shape, dtype=single.out.dtype).pin_memory()
        single.run_from_host(host_inputs[i % 3], out)
        torch.cuda.synchronize()
        want.append(out.clone())
    pipe = DecodePipeline(kv, Hq, B, tables.shape[1], SCALE)
    for sl in pipe.slots:
        sl.load_inputs(**host_inputs[0])
    pipe.capture()
    got = []
    host_outs = [torch.empty(single.out.shape, dtype=single.out.dtype).pin_memory() for _ in range(2)]
    for i in range(steps):  # one step per call, so that each step's read-back can be kept
        pipe.run([host_inputs[i % 3]], [host_outs[0], host_outs[1]], 1)
        torch.cuda.synchronize()
        got.append(host_outs[0].clone())
    for i in range(steps):
        assert torch.equal(got[i].view(torch.int16), want[i].view(torch.int16)), i
    # several steps per call: the last step's outputs land in host_outs[(steps - 1) % 2]
    pipe.run([host_inputs[i % 3] for i in range(steps)], host_outs, steps)
    torch.cuda.synchronize()
    assert torch.equal(host_outs[(steps - 1) % 2].view(torch.int16), want[steps - 1].view(torch.int16))
    assert torch.equal(host_outs[(steps - 2) % 2].view(torch.int16), want[steps - 2].view(torch.int16))

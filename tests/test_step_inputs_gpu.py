"""Per-step model inputs built on the device (``ops.prepare_step_inputs``), bit-exact against
the oracle restatement of Worker._prepare_model_inputs (aegaeon/aegaeon/worker.py:596-682)."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import ops
from oracle import oracle as orc
from tests.test_step_inputs_cpu import _batch

pytestmark = pytest.mark.gpu


def _device_batch(dev, seq, ctx, tables, W):
    t = np.zeros((len(seq), W), np.int32)
    for i, row in enumerate(tables):
        t[i, :len(row)] = row
    return (torch.as_tensor(t, device=dev), torch.as_tensor(np.asarray(ctx, np.int32), device=dev),
            torch.as_tensor(np.asarray(seq, np.int32), device=dev))


def _check(out, want, B, W):
    T = len(want["slot_mapping"])
    assert int(out.num_tokens.item()) == T
    assert out.slot_mapping[:T].cpu().numpy().tolist() == want["slot_mapping"].tolist()
    assert out.positions[:T].cpu().numpy().tolist() == want["positions"].tolist()
    assert out.query_lens.cpu().numpy().tolist() == want["query_lens"].tolist()
    assert out.query_start_loc.cpu().numpy().tolist() == want["query_start_loc"].tolist()
    assert out.seq_start_loc.cpu().numpy().tolist() == want["seq_start_loc"].tolist()
    got_t = out.block_tables.cpu().numpy()
    w = want["block_tables"].shape[1] if B else 0
    assert np.array_equal(got_t[:, :w], want["block_tables"])
    assert not got_t[:, w:].any()


@pytest.mark.parametrize("B,prompt_frac", [(1, 0.0), (64, 0.0), (256, 0.0), (37, 0.4), (300, 1.0), (5000, 0.1), (9000, 0.05)])
def test_step_inputs_match_oracle(cuda_device, B, prompt_frac):
    rng = np.random.default_rng(B)
    seq, ctx, tables = _batch(rng, B, prompt_frac)
    W = max(len(t) for t in tables) + 3  # persistent tables are wider than the batch needs
    bt, c, s = _device_batch(cuda_device, seq, ctx, tables, W)
    want = orc.np_step_inputs(seq, ctx, tables)
    out = ops.prepare_step_inputs(bt, c, s, capacity=len(want["slot_mapping"]) + 5)
    torch.cuda.synchronize()
    _check(out, want, B, W)
    assert ops.read_device_errors(cuda_device) == 0


def test_empty_batch(cuda_device):
    bt = torch.zeros((0, 4), dtype=torch.int32, device=cuda_device)
    e = torch.zeros(0, dtype=torch.int32, device=cuda_device)
    out = ops.prepare_step_inputs(bt, e, e, capacity=0)
    torch.cuda.synchronize()
    assert int(out.num_tokens.item()) == 0 and out.query_start_loc.cpu().tolist() == [0]


def test_table_deltas_then_inputs(cuda_device):
    """A decode step that crosses a block boundary appends one block per such request."""
    rng = np.random.default_rng(3)
    B, W = 40, 40
    seq, ctx, tables = _batch(rng, B, 0.0, max_len=500)
    bt, c, s = _device_batch(cuda_device, seq, ctx, tables, W)
    # next step: every sequence grows by one token; those at a block boundary get a new block
    nxt = 200000
    updates = []
    for i in range(B):
        n = seq[i] + 1
        if (n + 15) // 16 > len(tables[i]):
            tables[i] = tables[i] + [nxt]
            updates.append((i, len(tables[i]) - 1, nxt))
            nxt += 1
        seq[i], ctx[i] = n, n - 1
    ops.update_block_tables(bt, updates)
    c.copy_(torch.as_tensor(np.asarray(ctx, np.int32)))
    s.copy_(torch.as_tensor(np.asarray(seq, np.int32)))
    out = ops.prepare_step_inputs(bt, c, s)
    torch.cuda.synchronize()
    _check(out, orc.np_step_inputs(seq, ctx, tables), B, W)
    assert ops.read_device_errors(cuda_device) == 0


def test_invalid_requests_and_overflow_are_flagged(cuda_device):
    seq, ctx, tables = [10, 5, 40, 20], [9, 7, 0, 19], [[1], [2], [3, 4, 5], [6, 7]]
    bt, c, s = _device_batch(cuda_device, seq, ctx, tables, 3)
    out = ops.prepare_step_inputs(bt, c, s, capacity=64)  # request 1 has context_len > seq_len
    torch.cuda.synchronize()
    assert out.query_lens.cpu().tolist() == [1, 0, 40, 1]
    assert ops.read_device_errors(cuda_device) & 0x4
    good = [0, 2, 3]
    want = orc.np_step_inputs([seq[i] for i in good], [ctx[i] for i in good], [tables[i] for i in good])
    T = len(want["slot_mapping"])
    assert out.slot_mapping[:T].cpu().tolist() == want["slot_mapping"].tolist()
    out = ops.prepare_step_inputs(bt, c, s, capacity=10)  # 42 new tokens, room for 10
    torch.cuda.synchronize()
    assert int(out.num_tokens.item()) == 42
    assert out.slot_mapping.cpu().tolist() == want["slot_mapping"][:10].tolist()
    assert ops.read_device_errors(cuda_device) & 0x2


def test_out_of_range_table_updates_are_skipped_and_flagged(cuda_device):
    bt = torch.zeros((4, 8), dtype=torch.int32, device=cuda_device)
    ops.read_device_errors(cuda_device)
    ops.update_block_tables(bt, [(0, 1, 7), (4, 0, 9), (1, 8, 5), (-1, 0, 3), (3, 7, 11)])
    torch.cuda.synchronize()
    want = torch.zeros((4, 8), dtype=torch.int32)
    want[0, 1] = 7
    want[3, 7] = 11
    assert torch.equal(bt.cpu(), want)
    assert ops.read_device_errors(cuda_device) & 0x1

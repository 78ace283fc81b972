"""Per-step model inputs: the oracle restatement of Worker._prepare_model_inputs
(aegaeon/aegaeon/worker.py:596-682) against the package's host builder, and the device entry
points' host-side validation (no GPU)."""
import numpy as np

from aegaeon_b200 import _native, layout
from oracle import oracle as orc


def _batch(rng, B, prompt_frac=0.3, max_len=600):
    seq, ctx, tables = [], [], []
    perm = rng.permutation(max(100000, B * ((max_len + 15) // 16)))
    off = 0
    for _ in range(B):
        n = int(rng.integers(1, max_len))
        c = 0 if rng.random() < prompt_frac else n - 1
        nb = (n + 15) // 16
        tables.append(perm[off:off + nb].tolist())
        off += nb
        seq.append(n)
        ctx.append(c)
    return seq, ctx, tables


def test_oracle_matches_host_builder():
    rng = np.random.default_rng(0)
    for B in (0, 1, 7, 64):
        seq, ctx, tables = _batch(rng, B)
        want = orc.np_step_inputs(seq, ctx, tables)
        md = layout.build_decode_metadata(seq, ctx, tables)
        assert md.slot_mapping.numpy().tolist() == want["slot_mapping"].tolist()
        if B:
            assert np.array_equal(md.block_tables.numpy(), want["block_tables"])
        assert want["query_start_loc"][-1] == len(want["slot_mapping"]) == sum(s - c for s, c in zip(seq, ctx))
        assert want["seq_start_loc"][-1] == sum(seq)


def test_oracle_decode_batch_has_one_token_per_request():
    seq, ctx, tables = [5, 33, 16], [4, 32, 15], [[9], [1, 2, 3], [4]]
    r = orc.np_step_inputs(seq, ctx, tables)
    assert r["positions"].tolist() == [4, 32, 15]
    assert r["slot_mapping"].tolist() == [9 * 16 + 4, 3 * 16 + 0, 4 * 16 + 15]
    assert r["query_start_loc"].tolist() == [0, 1, 2, 3]
    assert r["block_tables"].tolist() == [[9, 0, 0], [1, 2, 3], [4, 0, 0]]


def test_step_input_entry_points_validate_on_host():
    lib = _native.lib
    inval = _native.AEG_ERR_INVALID_ARGUMENT
    buf = np.zeros(64, np.int64)
    p = buf.ctypes.data
    assert lib.aeg_prepare_step_inputs(p, 4, p, p, -1, p, p, 8, p, p, p, None, p, None) == inval
    assert lib.aeg_prepare_step_inputs(p, 0, p, p, 2, p, p, 8, p, p, p, None, p, None) == inval
    assert lib.aeg_prepare_step_inputs(p, 4, p, p, 2, p, p, 8, p, None, p, None, p, None) == inval
    assert lib.aeg_prepare_step_inputs(p, 4, p, p, 2, p + 4, p, 8, p, p, p, None, p, None) == inval  # misaligned
    assert lib.aeg_update_block_tables(p, 4, 2, p, -1, None) == inval
    assert lib.aeg_update_block_tables(p, 4, 2, p, 0, None) == 0
    assert lib.aeg_update_block_tables(None, 4, 2, p, 3, None) == inval

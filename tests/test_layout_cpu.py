"""Host logic: block geometry, slot mapping and padded block tables (no GPU)."""
import numpy as np
import pytest
import torch

from aegaeon_b200 import layout, synth
from oracle import oracle as orc


def test_block_shape_and_run_view():
    assert layout.kv_block_shape(28, 4, 128) == (28, 2, 16, 4, 128)
    kv = torch.arange(3 * 2 * 2 * 16 * 1 * 4, dtype=torch.int32).view(3, 2, 2, 16, 1, 4)
    run = layout.kv_cache_run_view(kv)
    assert run.shape == (2, 2, 3, 16, 1, 4)
    # run[l][kv][n] is storage block n, layer l, K/V kv
    assert torch.equal(run[1][0][2], kv[2, 1, 0])
    assert torch.equal(run[0][1][1], kv[1, 0, 1])
    # block bytes of the Qwen2.5-7B geometry, fp16 (the swap unit)
    q = torch.empty((1, 28, 2, 16, 4, 128), dtype=torch.float16)
    assert layout.block_bytes(q) == 917504


def test_slot_mapping_decode_and_prefill():
    tables = [[7, 3, 9], [2], [5, 6]]
    seq_lens = [35, 16, 20]
    ctx_lens = [34, 15, 0]  # two decodes, one prompt of 20 tokens
    md = layout.build_decode_metadata(seq_lens, ctx_lens, tables)
    want = orc.np_slot_mapping(seq_lens, ctx_lens, tables)
    assert md.slot_mapping.dtype == torch.int64
    assert np.array_equal(md.slot_mapping.numpy(), want)
    assert md.slot_mapping[0].item() == 9 * 16 + 34 % 16
    assert md.slot_mapping[1].item() == 2 * 16 + 15
    # prompt rows get an empty table, padded with 0
    assert md.block_tables.dtype == torch.int32
    assert md.block_tables.tolist() == [[7, 3, 9], [2, 0, 0], [0, 0, 0]]
    assert md.seq_lens.tolist() == seq_lens and md.seq_lens.dtype == torch.int32
    assert md.max_seq_len == 35


def test_metadata_rejects_inconsistent_requests():
    with pytest.raises(ValueError):
        layout.build_decode_metadata([40], [39], [[1, 2]])  # table too short for 40 tokens
    with pytest.raises(ValueError):
        layout.build_decode_metadata([10], [11], [[1]])
    with pytest.raises(ValueError):
        layout.pad_block_tables([[1, 2, 3]], max_len=2)


def test_pad_block_tables():
    t = layout.pad_block_tables([[1, 2], [], [3]], pad=0)
    assert t.dtype == np.int32 and t.tolist() == [[1, 2], [0, 0], [3, 0]]


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_synthetic_layouts(name):
    cfg = synth.CONFIGS[name]
    lay = synth.make_layout(cfg)
    assert lay.seq_lens.shape == (cfg.batch,)
    nb = (lay.seq_lens + 15) // 16
    used = np.concatenate([lay.block_tables[i, : nb[i]] for i in range(cfg.batch)])
    assert len(np.unique(used)) == len(used)  # every block belongs to one sequence
    assert used.max() < lay.num_blocks and used.min() >= 0
    slots = synth.new_token_slots(lay)
    assert np.all(slots // 16 == lay.block_tables[np.arange(cfg.batch), (lay.seq_lens - 1) // 16])
    lo = cfg.ctx_dist[1] if cfg.ctx_dist[0] == "uniform" else cfg.ctx_dist[3]
    hi = cfg.ctx_dist[2] if cfg.ctx_dist[0] == "uniform" else cfg.ctx_dist[4]
    assert lay.seq_lens.min() >= lo and lay.seq_lens.max() <= hi


def test_cfg1_fits_its_64_block_pool():
    lay = synth.make_layout(synth.CONFIGS["cfg1"])
    assert lay.total_blocks <= 64 and lay.num_blocks == 64


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharding_partitions_sequences(world):
    cfg = synth.CONFIGS["cfg3"]
    full = synth.make_layout(cfg)
    seen = []
    for r in range(world):
        sh = synth.make_layout(cfg, r, world)
        assert np.array_equal(sh.seq_lens, full.seq_lens[r::world])
        assert sh.num_blocks == sh.total_blocks  # pool sized to its own sequences
        seen.extend(sh.seq_ids.tolist())
    assert sorted(seen) == list(range(cfg.batch))


def test_weight_switch_workload_is_qwen2_7b():
    from aegaeon_b200 import synth

    sizes = synth.qwen2_7b_param_bytes()
    assert len(sizes) == 2 + 28 * 12 + 1           # embeddings, 12 tensors per layer, final norm, lm head
    assert sum(sizes) == 15_231_233_024             # 7.6B bf16 parameters
    assert sizes[0] == sizes[-1] == 152064 * 3584 * 2


def test_balanced_split_assigns_every_sequence_once_with_even_context():
    from aegaeon_b200 import synth

    cfg = synth.CONFIGS["cfg3"]
    for world in (1, 2, 4, 8):
        lays = [synth.make_layout(cfg, r, world, "balanced") for r in range(world)]
        ids = np.concatenate([l.seq_ids for l in lays])
        assert sorted(ids.tolist()) == list(range(cfg.batch))
        tot = [l.total_tokens for l in lays]
        assert max(tot) - min(tot) <= int(synth.make_layout(cfg).seq_lens.max())  # within one sequence
        for l in lays:  # each rank's pool holds exactly its own blocks
            assert l.num_blocks == l.total_blocks
    mod = [synth.make_layout(cfg, r, 8).seq_ids for r in range(8)]
    assert [m.tolist() for m in mod] == [list(range(r, cfg.batch, 8)) for r in range(8)]

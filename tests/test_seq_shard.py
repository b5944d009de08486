"""Query-row sharding, host side (CPU): the token plan and the model's refusals."""
import pytest


def test_plan_splits_latents_in_whole_key_tiles_camera_last():
    from flow_model import FlowSpec
    from seq_shard import seq_shard_plan

    s = FlowSpec()
    for world in (1, 2, 4, 8):
        st = seq_shard_plan(s, world)
        assert st[0] == 0 and st[-1] == s.seq == 8193 and len(st) == world + 1
        sizes = [b - a for a, b in zip(st, st[1:])]
        assert sizes[:-1] == [8192 // world] * (world - 1) and sizes[-1] == 8192 // world + 1
        assert all(a % 128 == 0 for a in st[:-1])
    with pytest.raises(ValueError, match="whole"):
        seq_shard_plan(FlowSpec.small(), 2)  # 64 latent tokens: no 128-token tiles to share
    with pytest.raises(ValueError):
        seq_shard_plan(s, 16)


def test_model_refuses_odd_block_counts_and_bad_ranks():
    from flow_model import FlowSpec, FlowWeights
    from seq_shard import SeqShardedFlowModel

    with pytest.raises(ValueError, match="odd"):
        SeqShardedFlowModel(FlowWeights(FlowSpec(blocks=3)), rank=0, world=2, device="cpu")
    with pytest.raises(ValueError, match="rank"):
        SeqShardedFlowModel(FlowWeights(FlowSpec(blocks=2)), rank=2, world=2, device="cpu")
    with pytest.raises(ValueError, match="exchange"):
        SeqShardedFlowModel(FlowWeights(FlowSpec(blocks=2)), rank=0, world=2, device="cpu", exchange="x")

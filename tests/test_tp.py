"""Tensor-parallel host logic on CPU: shard maps partition every sharded dimension exactly,
and ranks agree on them when exchanged over a gloo process group (world size 2)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _shards(tp, **overrides):
    from gfxinfer_b200 import session as gs

    cfg = gs.model_config(**overrides)
    return cfg, [gs.tp_shard(cfg, r, tp) for r in range(tp)]


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_shards_partition_config2(tp):
    cfg, shards = _shards(tp)
    def covers(first, count, total):
        spans = sorted((getattr(s, first), getattr(s, count)) for s in shards)
        position = 0
        for start, n in spans:
            assert start == position and n > 0
            position += n
        assert position == total
    covers("gdn_key_head0", "gdn_key_heads", cfg.gdn_key_heads)
    covers("gdn_value_head0", "gdn_value_heads", cfg.gdn_value_heads)
    covers("q_head0", "q_heads", cfg.q_heads)
    covers("intermediate0", "intermediate", cfg.intermediate)
    covers("vocab0", "vocab", cfg.vocab)
    covers("fc_column0", "fc_columns", 2 * cfg.hidden)
    group = cfg.q_heads // cfg.kv_heads
    for s in shards:
        assert s.intermediate % 128 == 0 and s.vocab % 16 == 0 and s.fc_columns % 128 == 0
        assert s.gdn_channels == 2 * s.gdn_key_heads * 128 + s.gdn_value_heads * 128
        # every query head's KV head lies in the rank's KV range
        for h in range(s.q_head0, s.q_head0 + s.q_heads):
            assert s.kv_head0 <= h // group < s.kv_head0 + s.kv_heads
        # GDN value heads map to the rank's own key heads
        ratio = cfg.gdn_value_heads // cfg.gdn_key_heads
        for v in range(s.gdn_value_head0, s.gdn_value_head0 + s.gdn_value_heads):
            assert s.gdn_key_head0 <= v // ratio < s.gdn_key_head0 + s.gdn_key_heads


def test_invalid_tp_sizes_are_rejected():
    from gfxinfer_b200 import GfxbError
    from gfxinfer_b200 import session as gs

    with pytest.raises(GfxbError):
        gs.tp_shard(gs.model_config(), 0, 3)  # 16 GDN key heads do not split 3 ways
    with pytest.raises(GfxbError):
        gs.tp_shard(gs.model_config(), 2, 2)


def _rank_main(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from gfxinfer_b200 import session as gs

    shard = gs.tp_shard(gs.model_config(), rank, world)
    mine = torch.tensor([shard.q_head0, shard.q_heads, shard.intermediate0, shard.intermediate, shard.vocab0,
                         shard.vocab], dtype=torch.int64)
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    if rank == 0:
        queue.put([g.tolist() for g in gathered])
    dist.destroy_process_group()


def test_ranks_agree_over_gloo():
    from gfxinfer_b200 import build

    build.build()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    result = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (q0, nq0, i0, ni0, v0, nv0), (q1, nq1, i1, ni1, v1, nv1) = result
    assert (q0, q0 + nq0, q1 + nq1) == (0, q1, 24)
    assert (i0, i0 + ni0, i1 + ni1) == (0, i1, 17408)
    assert (v0, v0 + nv0, v1 + nv1) == (0, v1, 151936)

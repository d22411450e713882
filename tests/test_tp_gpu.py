"""Tensor parallelism on 2 GPUs: the sharded model equals the unsharded one.

Each rank holds its slice of the same global synthetic model; row-parallel
outputs are summed across ranks (NVLink peer all-reduce, or NCCL), which changes the fp32 summation
order, so TP=2 is compared to the (bit-exact) TP=1 oracle with a tolerance:
first-step logits within 1e-3 of their largest magnitude, the whole token
stream equal to the oracle's, and both ranks emitting identical token streams.
Skipped with fewer than two GPUs.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import SMALL_MODEL, OracleModel, model_config, prompt_tokens  # noqa: E402


def _rank(rank, world, id_queue, result_queue, prompt, env=None):
    import os

    import torch as t

    os.environ.update(env or {})
    t.cuda.set_device(rank)
    from gfxinfer_b200 import session as gs

    if rank == 0:
        nccl_id = gs.nccl_unique_id()
        for _ in range(world - 1):
            id_queue.put(nccl_id)
    else:
        nccl_id = id_queue.get(timeout=120)
    engine = gs.Engine.create(gs.model_config(**SMALL_MODEL), device=rank, tp_rank=rank, tp_size=world,
                              nccl_id=nccl_id)
    session = gs.QwenDecodeSession.create(engine)
    first = session.greedy_step(prompt[0])
    shard = gs.tp_shard(gs.model_config(**SMALL_MODEL), rank, world)
    _, logits = session.read_state(shard.vocab)
    token = first
    stream = [first]
    for tok in prompt[1:]:
        token = session.greedy_step(tok)
    for _ in range(12):
        stream.append(token)
        token = session.greedy_step(token)
    block = session.block_step(prompt[:5])
    result_queue.put((rank, logits, stream, block))
    session.close()
    engine.close()


def _run_tp2(prompt, env=None):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    id_queue, result_queue = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, id_queue, result_queue, prompt, env)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (l, s, b)) for r, l, s, b in [result_queue.get(timeout=300) for _ in procs])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return results


def test_tp2_matches_tp1(oracle):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from gfxinfer_b200 import build

    build.build()
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 99, cfg.vocab, 6)
    results = _run_tp2(prompt)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    first = ref.greedy_step(prompt[0])
    want = ref.logits()
    got = np.concatenate([results[0][0], results[1][0]])
    assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max()
    token = first
    for tok in prompt[1:]:
        token = ref.greedy_step(tok)
    stream = [first]
    for _ in range(12):
        stream.append(token)
        token = ref.greedy_step(token)
    assert results[0][1] == stream  # the whole TP=2 stream equals the TP=1 oracle's
    assert results[0][1] == results[1][1]  # both ranks select the same tokens
    assert results[0][2] == results[1][2]


def test_tp2_peer_all_reduce_equals_nccl(oracle):
    """The NVLink peer all-reduce (GFXB_PEER_ALLREDUCE=1) and NCCL's give the same bits at
    TP=2 (one fp32 addition per element, which commutes): identical logits,
    token streams and verifier block on both paths."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from gfxinfer_b200 import build

    build.build()
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 7, cfg.vocab, 6)
    peer = _run_tp2(prompt, {"GFXB_PEER_ALLREDUCE": "1"})
    nccl = _run_tp2(prompt, {"GFXB_PEER_ALLREDUCE": "0"})
    for r in range(2):
        np.testing.assert_array_equal(peer[r][0].view(np.uint32), nccl[r][0].view(np.uint32))
        assert peer[r][1] == nccl[r][1]
        assert peer[r][2] == nccl[r][2]

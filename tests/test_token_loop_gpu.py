"""Persistent token kernel: one launch per greedy step (all layers, LM head,
argmax) must reproduce the per-operation path and the CPU oracle bit for bit.

The kernel streams every weight tile of the step through a shared-memory ring
ahead of the compute warps and meets at grid barriers between operations;
none of that may change a single bit: tokens, the final hidden state and the
logits are compared exactly, at the small model's widths and at config-2
widths (hidden 5120, MLP 17408 W3, 48/16 GDN heads, 24/4 attention heads,
vocab 151936), with A4 and A8 activations.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import SMALL_MODEL, OracleModel, model_config, prompt_tokens  # noqa: E402


def _stream(step, prompt, steps):
    token = None
    for t in prompt:
        token = step(t)
    out = []
    for _ in range(steps):
        out.append(token)
        token = step(token)
    return out


def _engine(**kw):
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import session as gs

    return gs.Engine.create(gs.model_config(**kw), include_mtp=False)


def _session(engine, step_kernel, graphs=True):
    from gfxinfer_b200 import abi
    from gfxinfer_b200 import session as gs

    kernel = {"persistent": abi.STEP_PERSISTENT, "launches": abi.STEP_LAUNCHES}[step_kernel]
    return gs.QwenDecodeSession.create(engine, use_graphs=graphs, step_kernel=kernel)


@pytest.fixture(scope="module")
def small_engine():
    engine = _engine(**SMALL_MODEL)
    yield engine
    engine.close()


@pytest.mark.parametrize("graphs", [True, False])
def test_small_model_matches_oracle(oracle, small_engine, graphs):
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 7, cfg.vocab, 9)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    want = _stream(ref.greedy_step, prompt, 40)
    session = _session(small_engine, "persistent", graphs)
    got = _stream(session.greedy_step, prompt, 40)
    assert got == want
    hidden, logits = session.read_state(cfg.vocab)
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    session.close()


def test_persistent_equals_launches_past_attention_chunks(oracle, small_engine):
    """Positions cross the 128-position attention chunks (three chunks merged at the end)."""
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 8, cfg.vocab, 4)
    a = _session(small_engine, "persistent")
    b = _session(small_engine, "launches")
    assert _stream(a.greedy_step, prompt, 300) == _stream(b.greedy_step, prompt, 300)
    ha, la = a.read_state(cfg.vocab)
    hb, lb = b.read_state(cfg.vocab)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))


def test_device_loop_matches_greedy_steps(oracle, small_engine):
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 9, cfg.vocab, 4)
    a = _session(small_engine, "launches")
    stream = _stream(a.greedy_step, prompt, 24)
    b = _session(small_engine, "persistent")
    for t in prompt[:-1]:
        b.greedy_step(t)
    b.enqueue_greedy(prompt[-1], 24)
    b.sync()
    assert b.last_token() == stream[23]


def test_a8_activations_match_oracle(oracle):
    kw = dict(SMALL_MODEL, activation_bits=8, layers=4)
    cfg = model_config(**kw)
    engine = _engine(**kw)
    session = _session(engine, "persistent")
    ref = OracleModel(oracle, cfg, include_mtp=False)
    prompt = prompt_tokens(oracle, cfg.seed, cfg.vocab, 6)
    assert _stream(session.greedy_step, prompt, 10) == _stream(ref.greedy_step, prompt, 10)
    hidden, logits = session.read_state(cfg.vocab)
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    session.close()
    engine.close()


def test_config2_widths_match_launches_and_oracle(oracle):
    cfg = model_config(layers=4, max_context=160)
    engine = _engine(layers=4, max_context=160)
    prompt = prompt_tokens(oracle, cfg.seed, cfg.vocab, 3)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    persistent = _session(engine, "persistent")
    assert _stream(persistent.greedy_step, prompt, 2) == _stream(ref.greedy_step, prompt, 2)
    hidden, logits = persistent.read_state(cfg.vocab)
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    persistent.close()
    # a longer run against the per-operation path, across the 128-position chunk boundary
    a = _session(engine, "persistent")
    b = _session(engine, "launches")
    assert _stream(a.greedy_step, prompt, 140) == _stream(b.greedy_step, prompt, 140)
    ha, la = a.read_state(cfg.vocab)
    hb, lb = b.read_state(cfg.vocab)
    np.testing.assert_array_equal(ha, hb)
    np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))
    a.close()
    b.close()
    engine.close()


def test_persistent_required_is_refused_for_unsupported_hidden():
    from gfxinfer_b200 import GfxbError
    from gfxinfer_b200 import session as gs

    kw = dict(SMALL_MODEL, hidden=512, layers=2)  # hidden / 256 = 2: no token-kernel instance
    engine = _engine(**kw)
    with pytest.raises(GfxbError):
        _session(engine, "persistent")
    auto = gs.QwenDecodeSession.create(engine)  # AUTO runs the per-operation launches
    auto.greedy_step(1)
    auto.close()
    engine.close()


def test_trace_step_timeline(oracle, small_engine):
    """The traced step returns the greedy step's token and a consistent timeline:
    per CTA, barrier arrival <= release, and operation i + 1 starts after operation i."""
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 10, cfg.vocab, 5)
    a = _session(small_engine, "persistent")
    b = _session(small_engine, "launches")
    for t in prompt[:-1]:
        a.greedy_step(t)
        b.greedy_step(t)
    token, timeline, kinds = a.trace_step(prompt[-1])
    assert token == b.greedy_step(prompt[-1])
    assert len(kinds) + 1 == timeline.shape[0]
    assert set(np.unique(kinds) & 0xF) <= {1, 2, 3, 4}
    assert kinds[-1] == 4  # argmax closes the step
    assert (timeline > 0).all()
    assert (timeline[:, 1, :] >= timeline[:, 0, :]).all()
    assert (np.diff(timeline[:, 1, :], axis=0) >= 0).all()
    a.close()
    b.close()

"""End-to-end decode parity: the B200 session vs the CPU oracle's scalar forward.

Bit-exact: every kernel follows the oracle's reduction order, so tokens,
final hidden states and logits agree exactly. The reference's own
end-to-end gates are restated too: block_step equals serial greedy steps
(src/cli/main.cpp:866-887) and the speculative stream equals the serial
greedy stream (src/cli/main.cpp:961-979).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import SMALL_MODEL, OracleModel, model_config, prompt_tokens  # noqa: E402


@pytest.fixture(scope="module")
def small_engine():
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import session as gs

    engine = gs.Engine.create(gs.model_config(**SMALL_MODEL))
    yield engine
    engine.close()


def _session(engine, graphs=True):
    from gfxinfer_b200 import session as gs

    return gs.QwenDecodeSession.create(engine, use_graphs=graphs)


def _greedy_stream(step, prompt, steps):
    token = None
    for t in prompt:
        token = step(t)
    out = []
    for _ in range(steps):
        out.append(token)
        token = step(token)
    return out


def test_greedy_128_steps_bit_exact_small_model(oracle, small_engine):
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed, cfg.vocab, 16)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    want = _greedy_stream(ref.greedy_step, prompt, 128)
    session = _session(small_engine)
    got = _greedy_stream(session.greedy_step, prompt, 128)
    assert got == want
    hidden, logits = session.read_state(cfg.vocab)
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    assert len(set(want)) > 8  # the stream is not degenerate
    session.close()


def test_eager_and_graph_paths_agree(oracle, small_engine):
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 1, cfg.vocab, 5)
    a, b = _session(small_engine, graphs=True), _session(small_engine, graphs=False)
    assert _greedy_stream(a.greedy_step, prompt, 20) == _greedy_stream(b.greedy_step, prompt, 20)


def test_device_resident_loop_matches_greedy(oracle, small_engine):
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 2, cfg.vocab, 4)
    a = _session(small_engine)
    stream = _greedy_stream(a.greedy_step, prompt, 12)
    b = _session(small_engine)
    for t in prompt[:-1]:
        b.greedy_step(t)
    b.enqueue_greedy(prompt[-1], 12)
    b.sync()
    # the device loop feeds each argmax back: its last output is the 12th generated token
    assert b.last_token() == stream[11]
    assert b.position() == len(prompt) + 11


@pytest.mark.parametrize("width", [2, 5, 17, 32])
def test_block_step_equals_serial_greedy(oracle, small_engine, width):
    cfg = model_config(**SMALL_MODEL)
    tokens = prompt_tokens(oracle, cfg.seed + width, cfg.vocab, 40)
    serial = _session(small_engine)
    expected = [serial.greedy_step(t) for t in tokens[:8]]
    expected += [serial.greedy_step(t) for t in tokens[8:8 + width]]
    block = _session(small_engine)
    got = block.block_step(tokens[:8]) + block.block_step(tokens[8:8 + width])
    assert got == expected
    assert block.position() == 8 + width


def test_mtp_draft_bit_exact(oracle, small_engine):
    cfg = model_config(**SMALL_MODEL)
    prompt = prompt_tokens(oracle, cfg.seed + 7, cfg.vocab, 6)
    ref = OracleModel(oracle, cfg, include_mtp=True)
    session = _session(small_engine)
    want, got = [], []
    for t in prompt:
        nxt_ref = ref.greedy_step(t)
        nxt = session.greedy_step(t)
        assert nxt == nxt_ref
        want.append(ref.mtp_draft(nxt_ref))
        got.append(session.mtp_draft(nxt))
    assert got == want


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("depth", [1, 4, 8])
def test_speculative_stream_equals_greedy(oracle, small_engine, depth, graph):
    """spec-bench (src/cli/main.cpp:917-979): one greedy step, then speculative rounds; the
    emitted stream must equal the serial greedy stream token for token, with the round's
    device work eager or replayed from the captured speculative graph."""
    from gfxinfer_b200 import session as gs

    cfg = model_config(**SMALL_MODEL)
    start = prompt_tokens(oracle, cfg.seed + 11, cfg.vocab, 1)[0]
    spec = gs.QwenDecodeSession.create(small_engine, graph_verifier_batch=depth + 1 if graph else 0)
    first = spec.greedy_step(start)
    emitted, seed, proposed, accepted = [first], first, 0, 0
    while len(emitted) < 40:
        result = spec.speculative_step(seed, depth)
        assert 1 <= len(result.tokens) <= depth + 1
        proposed += result.proposed_drafts
        accepted += result.accepted_drafts
        emitted.extend(result.tokens)
        seed = result.tokens[-1]
    serial = _session(small_engine)
    token = serial.greedy_step(start)
    reference = [token]
    while len(reference) < len(emitted):
        token = serial.greedy_step(token)
        reference.append(token)
    assert emitted == reference
    assert spec.position() == serial.position()


@pytest.mark.parametrize("graph", [False, True])
def test_speculative_forced_acceptance(oracle, small_engine, graph):
    """Rounds whose drafts come from the serial greedy stream, with the first wrong draft planted at
    every position k = 0..D-1 and none at all: each round must accept exactly k (or all D) drafts,
    emit the greedy stream, and leave states that later rounds and plain greedy steps continue
    correctly. Covers the partial-acceptance replay (qwen_runtime.cpp:1497-1519) and the
    full-acceptance state commit with the MTP cache advance (:1520-1534), which random MTP weights
    never reach."""
    from gfxinfer_b200 import session as gs

    cfg = model_config(**SMALL_MODEL)
    start = prompt_tokens(oracle, cfg.seed + 17, cfg.vocab, 1)[0]
    serial = _session(small_engine)
    reference = [serial.greedy_step(start)]
    while len(reference) < 160:
        reference.append(serial.greedy_step(reference[-1]))
    depth = 4
    spec = gs.QwenDecodeSession.create(small_engine, graph_verifier_batch=depth + 1 if graph else 0)
    emitted = [spec.greedy_step(start)]
    plan = [depth, 0, 1, 2, 3, depth, depth, 2, 0, depth, 3, 1]  # accepted drafts per round
    for wanted in plan:
        n = len(emitted)
        drafts = reference[n:n + depth]
        if wanted < depth:
            drafts[wanted] = (drafts[wanted] + 1) % cfg.vocab  # the first wrong draft
        result = spec.speculative_step(emitted[-1], depth, drafts=drafts)
        assert result.accepted_drafts == wanted
        assert result.tokens == reference[n:n + wanted + 1]
        emitted.extend(result.tokens)
        assert spec.position() == len(emitted)  # the start token and every emitted token but the newest
    # regular MTP rounds and greedy steps continue from the committed / rolled-back states
    while len(emitted) < 100:
        emitted.extend(spec.speculative_step(emitted[-1], depth).tokens)
    for _ in range(5):
        emitted.append(spec.greedy_step(emitted[-1]))
    assert emitted == reference[:len(emitted)]


def test_prefill_equals_serial_greedy(oracle, small_engine):
    """Chunked prefill (32-token causal blocks, LM head on the last token only) leaves the state and
    the next token of greedy steps over every prompt token, for prompts that end inside, at and
    after a block boundary."""
    cfg = model_config(**SMALL_MODEL)
    for length in (1, 31, 32, 33, 100):
        prompt = prompt_tokens(oracle, cfg.seed + length, cfg.vocab, length)
        serial = _session(small_engine)
        want = _greedy_stream(serial.greedy_step, prompt, 20)
        chunked = _session(small_engine)
        token = chunked.prefill(prompt)
        assert chunked.position() == length
        got = []
        for _ in range(20):
            got.append(token)
            token = chunked.greedy_step(token)
        assert got == want, length
        np.testing.assert_array_equal(chunked.read_state()[0], serial.read_state()[0])
        serial.close()
        chunked.close()


def test_speculative_graph_with_other_depths_runs_eagerly(oracle, small_engine):
    """A session captured for 4 drafts still serves rounds of 2 drafts (eagerly), interleaved."""
    from gfxinfer_b200 import session as gs

    cfg = model_config(**SMALL_MODEL)
    start = prompt_tokens(oracle, cfg.seed + 13, cfg.vocab, 1)[0]
    spec = gs.QwenDecodeSession.create(small_engine, graph_verifier_batch=5)
    first = spec.greedy_step(start)
    emitted, seed, depth = [first], first, 4
    while len(emitted) < 30:
        result = spec.speculative_step(seed, depth)
        emitted.extend(result.tokens)
        seed = result.tokens[-1]
        depth = 2 if depth == 4 else 4
    serial = _session(small_engine)
    token = serial.greedy_step(start)
    reference = [token]
    while len(reference) < len(emitted):
        token = serial.greedy_step(token)
        reference.append(token)
    assert emitted == reference


def test_invalid_arguments_are_rejected(small_engine):
    from gfxinfer_b200 import GfxbError

    session = _session(small_engine)
    with pytest.raises(GfxbError) as error:
        session.greedy_step(10**9)
    assert error.value.status == 1
    with pytest.raises(GfxbError):
        session.block_step([])
    with pytest.raises(GfxbError):
        session.block_step([1] * 33)
    with pytest.raises(GfxbError):
        session.speculative_step(1, 4)  # no aligned MTP state yet


def test_full_width_four_layers_matches_oracle(oracle):
    """Config-2 widths (hidden 5120, MLP 17408 W3, 48/16 GDN heads, 24/4 attention heads, vocab 151936)."""
    from gfxinfer_b200 import session as gs

    cfg = model_config(layers=4, max_context=64)
    engine = gs.Engine.create(gs.model_config(layers=4, max_context=64), include_mtp=False)
    session = gs.QwenDecodeSession.create(engine)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    prompt = prompt_tokens(oracle, cfg.seed, cfg.vocab, 3)
    assert _greedy_stream(session.greedy_step, prompt, 2) == _greedy_stream(ref.greedy_step, prompt, 2)
    hidden, logits = session.read_state(cfg.vocab)
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    session.close()
    engine.close()

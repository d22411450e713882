"""Parity at the benchmarked configurations: the B200 session vs the CPU oracle's forward.

* Config 2, the headline model: all 64 layers (48 GDN + 16 gated-attention), hidden 5120,
  W3 MLP 17408, W4 projections and LM head over vocab 151936, A4, context 512. A 64-token
  uniform-random prompt, then 128 greedy steps: every token, the final hidden state and the
  final logits bit-exact (the reference's serial-parity gate, src/cli/main.cpp:866-887,
  restated against the CPU forward).
* Config 4 widths: W2 MLP, W4 projections, A8 activations, context 4096, 8 layers (6 GDN +
  2 attention): a 3840-token prompt through chunked prefill, then 256 greedy steps up to the
  last cache slot, with attention reading up to 32 chunks of 128 positions.

The oracle needs about 13 GB of host memory for config 2 (packed codes) and the host's
cores for a few minutes; it runs after the GPU has produced its stream.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_lib import OracleModel, model_config, prompt_tokens  # noqa: E402


@pytest.fixture(scope="module")
def gs():
    from gfxinfer_b200 import build

    build.build()
    from gfxinfer_b200 import session

    return session


def _threads(oracle):
    oracle.lib.or_set_threads(os.cpu_count() or 1)


def test_config2_64_layers_128_greedy_steps_bit_exact(oracle, gs):
    overrides = dict(max_context=512)
    cfg = model_config(**overrides)
    prompt = prompt_tokens(oracle, cfg.seed, cfg.vocab, 64)
    engine = gs.Engine.create(gs.model_config(**overrides), include_mtp=False)
    session = gs.QwenDecodeSession.create(engine)
    token = None
    for t in prompt:
        token = session.greedy_step(t)
    got = []
    for _ in range(128):
        got.append(token)
        token = session.greedy_step(token)
    hidden, logits = session.read_state(cfg.vocab)
    session.close()
    engine.close()

    _threads(oracle)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    ref.prefill(prompt[:-1])  # layer-major blocks: the same bits as stepping each token
    token = ref.greedy_step(prompt[-1])
    want = []
    for _ in range(128):
        want.append(token)
        token = ref.greedy_step(token)
    assert got == want
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    assert len(set(want)) > 16  # not a degenerate stream
    ref.close()


def test_config4_w2_a8_context_4096_bit_exact(oracle, gs):
    overrides = dict(layers=8, mlp_bits=2, activation_bits=8, max_context=4096)
    cfg = model_config(**overrides)
    prompt = prompt_tokens(oracle, cfg.seed + 4, cfg.vocab, 3840)
    steps = 4096 - len(prompt)  # the last step writes the last cache slot
    engine = gs.Engine.create(gs.model_config(**overrides), include_mtp=False)
    session = gs.QwenDecodeSession.create(engine)
    token = session.prefill(prompt)
    got = []
    for _ in range(steps):
        got.append(token)
        token = session.greedy_step(token)
    assert session.position() == 4096
    hidden, logits = session.read_state(cfg.vocab)
    session.close()
    engine.close()

    _threads(oracle)
    ref = OracleModel(oracle, cfg, include_mtp=False)
    ref.prefill(prompt[:-1])
    token = ref.greedy_step(prompt[-1])
    want = []
    for _ in range(steps):
        want.append(token)
        token = ref.greedy_step(token)
    assert got == want
    np.testing.assert_array_equal(hidden, ref.last_hidden())
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits().view(np.uint32))
    ref.close()

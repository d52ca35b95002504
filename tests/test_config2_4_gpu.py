"""BASELINE configs 2 and 4 through the engine against the oracle fixtures
(tests/golden/make_golden.py: the restatement of reference.cpp, pinned bit
for bit to the compiled reference by tests/test_oracle.py).

- Config 2: Q8_0, one session, a 2048-token uniform prompt as four 512-row
  passes, then 128 greedy tokens: logits after the prompt and after the
  last teacher-forced step within the Q8_0 gates (max-abs 5e-2, KL < 1e-3);
  greedy tokens, teacher-forced and free-running, may differ only at a
  reference near-tie (top-2 margin below the prompt pass's logit deviation).
- Config 4 geometry: BF16 numerical-reference weights, three sessions at
  depths 300, 700 and 1100 (the 256-key sliding rings wrapped; global layers
  over the whole depth), decoded together through ForwardBatch for 4 rounds
  with each session's reference token: every session's logits within the
  BF16 gate (max-abs 2e-2, KL < 1e-3) after its prompt and every round
  (tests/session_test.cpp:224-283's ragged batch, against the oracle)."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, kl, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_KL = 1e-3
NEAR_TIE = 1e-2


@pytest.fixture(scope="module")
def config2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = np.load(os.path.join(GOLDEN, "config2.npz"))
    w = lfm3.SyntheticWeights(seed=0)
    model = lfm3.Model(w.weights)
    s = model.session(4096)
    after = s.forward(g["prompt"])  # 4 passes of 512 rows
    forced, logits = [], after
    for t in g["generated"]:
        forced.append(int(np.argmax(logits)))
        logits = s.forward([int(t)])
    free_s = model.session(4096)
    free_logits = free_s.forward(g["prompt"])
    free = []
    for _ in range(len(g["generated"])):
        free.append(int(np.argmax(free_logits)))
        free_logits = free_s.forward([free[-1]])
    return g, after, logits, forced, free


def test_config2_logits(config2):
    g, after, final, _, _ = config2
    e1 = float(np.abs(after - g["after_prompt"]).max())
    e2 = float(np.abs(final - g["final"]).max())
    print(f"config 2: max|diff| {e1:.3e} after the 2048-token prompt, {e2:.3e} "
          f"after 128 steps; KL {kl(g['after_prompt'], after):.2e} / "
          f"{kl(g['final'], final):.2e}")
    assert e1 <= 5e-2 and e2 <= 5e-2
    assert kl(g["after_prompt"], after) < MAX_KL
    assert kl(g["final"], final) < MAX_KL


def test_config2_greedy(config2):
    g, _, _, forced, free = config2
    ref = [int(t) for t in g["generated"]]
    mismatches = [i for i, (a, b) in enumerate(zip(forced, ref)) if a != b]
    n = 0
    while n < len(ref) and free[n] == ref[n]:
        n += 1
    print(f"config 2 greedy: teacher-forced {len(ref) - len(mismatches)}/{len(ref)} "
          f"identical (reference margins at mismatches "
          f"{[round(float(g['margin'][i]), 5) for i in mismatches]}); free-running "
          f"identical prefix {n}/{len(ref)}")
    assert all(float(g["margin"][i]) < NEAR_TIE for i in mismatches)
    if n < len(ref):
        assert float(g["margin"][n]) < NEAR_TIE


def test_config4_ragged_bf16_batch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = np.load(os.path.join(GOLDEN, "ragged_bf16.npz"))
    w = lfm3.SyntheticWeights(seed=0, matrix_type=lfm3.abi.BF16)
    model = lfm3.Model(w.weights)
    prompts = [g["prompt0"], g["prompt1"], g["prompt2"]]
    sessions = [model.session(2048) for _ in prompts]
    worst = 0.0
    for r, (s, p) in enumerate(zip(sessions, prompts)):
        got = s.forward(p)
        err = float(np.abs(got - g["logits"][r, 0]).max())
        worst = max(worst, err)
        assert err <= 2e-2, (r, err)
        assert kl(g["logits"][r, 0], got) < MAX_KL
    for step in range(g["tokens"].shape[1]):
        outs = lfm3.Session.forward_batch(
            sessions, [int(g["tokens"][r, step]) for r in range(len(sessions))])
        for r, got in enumerate(outs):
            want = g["logits"][r, step + 1]
            err = float(np.abs(got - want).max())
            worst = max(worst, err)
            assert err <= 2e-2, (r, step, err)
            assert kl(want, got) < MAX_KL
            assert int(np.argmax(got)) == int(np.argmax(want)) or \
                float(np.diff(np.sort(want)[-2:])[0]) < NEAR_TIE
    print(f"BF16 ragged batch at depths {[len(p) for p in prompts]}: worst "
          f"max|diff| {worst:.3e} over prompts and 4 rounds")

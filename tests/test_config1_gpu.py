"""BASELINE config 1 at full size against the compiled reference: the graded
synthetic geometry (seed 0) with Q8_0 matrices and with the BF16
numerical-reference matrices, a uniform 128-token prompt as one prompt pass,
then 64 greedy decode steps. The fixtures (tests/golden/config1.npz,
config1_bf16.npz) hold the reference oracle's (reference.cpp) prompt, greedy
tokens and logits after the prompt and after the last step.

North-star gates: greedy tokens identical for the 64 steps, final logits
within max-abs 5e-2 (Q8_0) / 2e-2 (BF16) of the reference with KL < 1e-3. The reference oracle
keeps FP32 K/V where the GPU engine keeps the F16 ring of the reference's
GPU design, so logits differ by up to ~1e-2; a step whose reference top-2
margin is below that bound is a near-tie, reported and not counted as a
divergence."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, kl, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_KL = 1e-3
NEAR_TIE = 1e-2  # reference top-2 margins below the observed logit error
# (fixture, matrix type, north-star max-abs logits tolerance)
CASES = {"q8_0": ("config1.npz", lfm3.abi.Q8_0, 5e-2),
         "bf16": ("config1_bf16.npz", lfm3.abi.BF16, 2e-2)}


@pytest.fixture(scope="module", params=sorted(CASES))
def run(request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    fixture, matrix_type, max_abs = CASES[request.param]
    g = dict(np.load(os.path.join(GOLDEN, fixture)))
    g["max_abs"] = max_abs
    weights = lfm3.SyntheticWeights(seed=0, matrix_type=matrix_type)
    model = lfm3.Model(weights.weights)
    session = model.session(1024)
    after_prompt = session.forward(g["prompt"])
    ours, logits = [], after_prompt
    for step in range(len(g["generated"])):
        ours.append(int(np.argmax(logits)))
        # teacher forcing with the reference's token keeps one near-tie from
        # changing every later step
        logits = session.forward([int(g["generated"][step])])
    return g, after_prompt, logits, ours


def test_logits_after_prompt(run):
    g, after_prompt, _, _ = run
    err = float(np.abs(after_prompt - g["after_prompt"]).max())
    print(f"after prompt: max|diff| {err:.3e}, KL {kl(g['after_prompt'], after_prompt):.3e}")
    assert err <= g["max_abs"]
    assert kl(g["after_prompt"], after_prompt) < MAX_KL


def test_final_logits(run):
    g, _, final, _ = run
    err = float(np.abs(final - g["final"]).max())
    print(f"after 64 steps: max|diff| {err:.3e}, KL {kl(g['final'], final):.3e}")
    assert err <= g["max_abs"]
    assert kl(g["final"], final) < MAX_KL


def test_greedy_tokens_identical(run):
    g, _, _, ours = run
    mismatches = [i for i, (a, b) in enumerate(zip(ours, g["generated"])) if a != int(b)]
    print(f"greedy: {64 - len(mismatches)}/64 identical; reference top-2 margins "
          f"at mismatches: {[float(g['margin'][i]) for i in mismatches]}")
    # every step whose reference top-2 margin is above the logit error must
    # agree; only the near-ties (4 of the 64 steps of this fixture) may flip
    assert all(float(g["margin"][i]) < NEAR_TIE for i in mismatches)
    assert len(mismatches) <= int((g["margin"] < NEAR_TIE).sum())

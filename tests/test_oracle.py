"""The CPU oracle (oracle/lfm3_oracle.c, a restatement of reference.cpp) is
pinned against the reference itself: bit for bit against reference.cpp
compiled unmodified (oracle/_ref, when the reference tree was available at
build time) and against the golden vectors that compiled reference produced
(tests/golden/*.npz)."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, ensure_oracle_built, lfm3

ensure_oracle_built()
import oracle  # noqa: E402


def small_weights(jitter=0.1, matrix_type=lfm3.abi.Q8_0, **kw):
    return lfm3.SyntheticWeights(lfm3.small_config(**kw), seed=0,
                                 matrix_type=matrix_type, norm_jitter=jitter)


def test_restatement_matches_golden_small():
    g = np.load(os.path.join(GOLDEN, "small.npz"))
    w = small_weights()
    o = oracle.Oracle(w.weights, 256, threads=3)
    logits = None
    for i, t in enumerate(g["prompt"]):
        logits = o.step(int(t), i + 1 == len(g["prompt"]))
    got = [logits]
    for t in g["generated"]:
        assert int(np.argmax(got[-1])) == int(t)
        got.append(o.step(int(t), True))
    np.testing.assert_array_equal(np.stack(got), g["logits"])


def test_restatement_matches_golden_config1_prefix():
    """First steps of the graded geometry against the compiled reference's
    fixture: bit-exact logits after the 128-token prompt."""
    path = os.path.join(GOLDEN, "config1.npz")
    if not os.path.exists(path):
        pytest.skip("config1 fixture not generated")
    g = np.load(path)
    w = lfm3.SyntheticWeights(seed=0)
    o = oracle.Oracle(w.weights, 1024, threads=os.cpu_count() or 1)
    logits = None
    for i, t in enumerate(g["prompt"]):
        logits = o.step(int(t), i + 1 == len(g["prompt"]))
    np.testing.assert_array_equal(logits, g["after_prompt"])
    assert int(np.argmax(logits)) == int(g["generated"][0])


@pytest.mark.skipif(not oracle.reference_available(),
                    reason="oracle/_ref not built (no reference tree)")
@pytest.mark.parametrize("matrix_type", [lfm3.abi.Q8_0, lfm3.abi.BF16])
def test_restatement_bit_exact_vs_compiled_reference(matrix_type):
    # window 16 < 60 steps: the sliding rings wrap
    w = small_weights(matrix_type=matrix_type, window=16)
    o = oracle.Oracle(w.weights, 128, threads=2)
    r = oracle.ReferenceOracle(w.weights, 128)
    rng = np.random.default_rng(3)
    for t in rng.integers(0, w.config.vocab, 60):
        a = o.step(int(t), True)
        b = r.step(int(t), True)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    o.reset()
    r.reset()
    assert o.position == r.position == 0
    np.testing.assert_array_equal(o.step(5, True), r.step(5, True))


def test_restatement_thread_count_invariant():
    w = small_weights()
    outs = []
    for threads in (1, 4):
        o = oracle.Oracle(w.weights, 32, threads=threads)
        outs.append(np.stack([o.step(t, True) for t in (1, 2, 3, 4)]))
    np.testing.assert_array_equal(outs[0], outs[1])


def test_restatement_refuses_invalid_steps():
    w = small_weights()
    o = oracle.Oracle(w.weights, 2)
    with pytest.raises(ValueError):
        o.step(w.config.vocab, True)
    o.step(1, False)
    o.step(1, False)
    with pytest.raises(ValueError):  # context full
        o.step(1, False)
    with pytest.raises(ValueError):
        oracle.Oracle(w.weights, 0)


def test_kv_half_rounding_matches_numpy():
    """The oracle's test-only F16 K/V switch rounds exactly as IEEE fp16
    (numpy): ties to even, subnormals, overflow to infinity."""
    import oracle
    lib = oracle.restatement_lib()
    rng = np.random.default_rng(0)
    values = np.concatenate([
        rng.normal(0, 1, 3000), rng.normal(0, 1e-5, 3000),
        rng.normal(0, 3e4, 500),
        [65504, 65519.99, 65520, 1e9, -1e-8, 0.0, -0.0, 2.0 ** -24,
         2.0 ** -25, 3 * 2.0 ** -25, 1 + 2.0 ** -11, 1 + 3 * 2.0 ** -11,
         2.0 ** -14 * (1 - 2.0 ** -11)]]).astype(np.float32)
    for v in values:
        got = lib.lfm3_oracle_round_half(float(v))
        want = float(np.float32(np.float16(v)))
        assert got == want or (np.isinf(got) and np.isinf(want)), (float(v), got, want)
        assert np.signbit(got) == np.signbit(want) or got != 0

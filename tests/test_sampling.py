"""Token selection (include/lfm3_cuda.h, lfm3_sampler): the library's host
sampler (lfm3_sample_host) against an independent restatement of the rule in
Python, token for token, on CPU.

The reference samples host logits with Gufo core's sampling::SamplerState
(runner.cpp:268-296; defaults temperature 0.1, top-k 50, repeat penalty 1.1
at runner.cpp:31-35), which is not in the reference tree, so the rule is the
library's own: repetition penalty on each distinct recent token, the top_k
largest logits by (logit desc, id asc), weights exp((l_i - l_0) / T) in
double precision summed in that order, a SplitMix64 draw. The device kernels
are checked against lfm3_sample_host in test_sampling_gpu.py.
"""
import importlib
import math
from decimal import Decimal, getcontext

import numpy as np
import pytest

lfm3 = importlib.import_module("lfm3-gufo-extension_b200")

M64 = (1 << 64) - 1


def splitmix64(seed):
    z = (seed + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def _ln2_split():
    """ln 2 as a 42-bit head (n * head exact for |n| < 2^11) and a tail."""
    getcontext().prec = 60
    ln2 = Decimal(2).ln()
    head = float(round(ln2 * (1 << 42))) / (1 << 42)
    return head, float(ln2 - Decimal(head))


LN2_HI, LN2_LO = _ln2_split()
INV_LN2 = 1.0 / math.log(2.0)
INV_FACTORIAL = [1.0 / math.factorial(i) for i in range(13, -1, -1)]


def exp_rule(x):
    """exp(x), x <= 0: Cody-Waite reduction, degree-13 Taylor series by
    Horner's rule, scale 2^n; each operation separately rounded."""
    if not x > -700.0:
        return 0.0
    n = math.floor(x * INV_LN2 + 0.5)
    r = (x - n * LN2_HI) - n * LN2_LO
    p = INV_FACTORIAL[0]
    for c in INV_FACTORIAL[1:]:
        p = p * r + c
    return p * 2.0 ** n


def keys(v):
    u = v.view(np.uint32).astype(np.uint64)
    neg = (u & 0x80000000) != 0
    return np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000).astype(np.int64)


def sample_rule(logits, temperature, top_k, penalty, recent, seed):
    v = np.array(logits, dtype=np.float32)
    p = np.float32(penalty)
    if p != np.float32(1.0):
        seen = set()
        for t in recent:
            if t in seen or t >= v.size:
                continue
            seen.add(t)
            v[t] = v[t] / p if v[t] > 0 else v[t] * p
    order = np.lexsort((np.arange(v.size), -keys(v)))
    T = float(np.float32(temperature))
    if T == 0.0:
        return int(order[0])
    k = min(top_k, v.size)
    top = order[:k]
    v0 = float(v[top[0]])
    w = [exp_rule((float(v[i]) - v0) / T) for i in top]
    total = 0.0
    for x in w:
        total += x
    u = (splitmix64(seed) >> 11) * 2.0 ** -53
    target = u * total
    run = 0.0
    for i, x in enumerate(w):
        run += x
        if run > target:
            return int(top[i])
    return int(top[-1])


def test_exp_rule_accuracy():
    xs = np.concatenate([-np.geomspace(1e-9, 699.0, 4000), [0.0, -0.5, -1.0]])
    for x in xs:
        x = float(x)
        assert abs(exp_rule(x) - math.exp(x)) <= 4e-16 * math.exp(x), x
    assert exp_rule(-700.5) == 0.0


def _check(x, smp, recent, seeds):
    got = lfm3.sample_host(x, smp, recent=recent, seeds=seeds)
    for r in range(x.shape[0]):
        want = sample_rule(x[r], smp.temperature, smp.top_k,
                           smp.repeat_penalty, recent[r] if recent else [],
                           int(seeds[r]))
        assert int(got[r]) == want, (r, int(got[r]), want)


@pytest.mark.parametrize("vocab", [65536, 5000, 37, 3])
@pytest.mark.parametrize("temperature,top_k,penalty", [
    (0.1, 50, 1.1), (0.7, 64, 1.1), (1.5, 2, 0.8), (0.1, 1, 1.0),
    (0.0, 50, 1.1), (2.0, 64, 1.0)])
def test_host_sampler_matches_rule(vocab, temperature, top_k, penalty):
    rng = np.random.default_rng(vocab + top_k)
    rows = 8
    x = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    recent = [rng.integers(0, vocab, size=int(rng.integers(0, 65)))
              .tolist() for _ in range(rows)]
    # penalise the current favourites too, with repeats
    for r in range(rows):
        recent[r] = (recent[r] + [int(x[r].argmax())] * 2)[-64:]
    seeds = rng.integers(0, 2**63, size=rows, dtype=np.uint64)
    _check(x, lfm3.sampler(temperature, top_k, penalty), recent, seeds)


def test_ties_go_to_the_lower_id():
    rng = np.random.default_rng(5)
    vocab = 20000
    # few distinct values: many ties inside the top-k and at its boundary
    x = np.round(rng.standard_normal((8, vocab)) * 2) / 2
    x = x.astype(np.float32)
    x[:, 100] = x[:, 7] = x.max()  # a tie for the largest logit
    recent = [[7]] * 4 + [[]] * 4
    seeds = np.arange(8, dtype=np.uint64) * 977
    for smp in (lfm3.sampler(0.0, 1, 1.0), lfm3.sampler(0.5, 50, 1.0),
                lfm3.sampler(0.5, 64, 1.3)):
        _check(x, smp, recent, seeds)
    greedy = lfm3.sample_host(x, lfm3.sampler(0.0, 1, 1.0))
    assert (greedy == 7).all()


def test_signed_zeros_and_penalty_sign():
    x = np.full((2, 64), -5.0, np.float32)
    x[0, 3], x[0, 9] = -0.0, 0.0  # +0 ranks above -0
    x[1, 4], x[1, 5] = 2.0, -1.0
    got = lfm3.sample_host(x, lfm3.sampler(0.0, 1, 1.0))
    assert got[0] == 9
    # penalty 4: 2.0 -> 0.5 (divided), -1.0 -> -4.0 (multiplied)
    got = lfm3.sample_host(x, lfm3.sampler(0.0, 1, 4.0), recent=[[], [4, 4]])
    assert got[1] == 4
    x[1, 6] = 0.6
    got = lfm3.sample_host(x, lfm3.sampler(0.0, 1, 4.0), recent=[[], [4]])
    assert got[1] == 6


def test_draws_follow_the_softmax():
    x = np.array([[2.0, 1.5, 1.0, 0.0, -1.0, -3.0]], np.float32)
    T = 0.8
    p = np.exp((x[0] - x[0].max()) / T)
    p /= p.sum()
    n = 6000
    counts = np.zeros(6)
    for s in range(n):
        counts[lfm3.sample_host(x, lfm3.sampler(T, 6, 1.0), seeds=[s])[0]] += 1
    assert np.abs(counts / n - p).max() < 0.025
    # top_k 2 keeps only the two largest
    got = {int(lfm3.sample_host(x, lfm3.sampler(T, 2, 1.0), seeds=[s])[0])
           for s in range(400)}
    assert got == {0, 1}


@pytest.mark.parametrize("bad", [
    dict(temperature=-0.1), dict(temperature=float("nan")),
    dict(top_k=0), dict(top_k=65), dict(repeat_penalty=0.0),
    dict(repeat_penalty=float("inf"))])
def test_invalid_controls_refused(bad):
    args = dict(temperature=0.5, top_k=10, repeat_penalty=1.1)
    args.update(bad)
    x = np.zeros((1, 100), np.float32)
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.sample_host(x, lfm3.sampler(**args))


def test_invalid_tables_refused():
    x = np.zeros((1, 100), np.float32)
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.sample_host(x, lfm3.sampler(), recent=[[100]])
    # a vocabulary too large for top_k 64 (more than 4096 candidates)
    big = np.zeros((1, 64 * 4096 + 1), np.float32)
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.sample_host(big, lfm3.sampler(0.5, 64, 1.0))
    assert lfm3.sample_host(big, lfm3.sampler(0.5, 63, 1.0)).shape == (1,)


@pytest.mark.parametrize("temperature", [1e-30, 1e-3, 1e30])
def test_extreme_temperatures_and_infinite_logits(temperature):
    rng = np.random.default_rng(17)
    x = (rng.standard_normal((6, 300)) * 4).astype(np.float32)
    x[0, :] = -np.inf          # every candidate masked
    x[1, 5] = np.inf           # one unbounded logit
    x[2, 7] = x[2, 9] = np.inf
    x[3, ::2] = -np.inf        # half the vocabulary masked
    seeds = rng.integers(0, 2**63, size=6, dtype=np.uint64)
    recent = [[1, 2, 3]] * 6
    for top_k in (1, 7, 64):
        _check(x, lfm3.sampler(temperature, top_k, 1.3), recent, seeds)

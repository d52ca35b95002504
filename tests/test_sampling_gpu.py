"""Token selection on the device (lfm3_cuda_sample and the engine's
lfm3_session_forward_batch_sample) against the library's host sampler
(lfm3_sample_host, itself checked against a restatement of the rule in
test_sampling.py): the same token for every row, bit for bit, including
ties at the top-k boundary, penalties, vocabularies that are not a multiple
of the 4096-logit segment, and more than eight rows per call."""
import ctypes

import numpy as np
import pytest

from helpers import abi, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def setup_module(module):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def device_sample(x, smp, recent=None, seeds=None):
    lib = lfm3.library()
    rows, vocab = x.shape
    logits = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = torch.zeros(rows, dtype=torch.int32, device="cuda")
    scratch = torch.empty(
        lib.lfm3_cuda_sample_scratch_bytes(rows, vocab, smp.top_k) // 4 + 1,
        dtype=torch.int32, device="cuda")
    table, count, seed = lfm3.sample_tables(rows, recent, seeds)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lfm3.check(lib.lfm3_cuda_sample(
        ctypes.c_void_p(logits.data_ptr()), rows, vocab, vocab,
        ctypes.byref(smp), lfm3._ptr(table), lfm3._ptr(count), lfm3._ptr(seed),
        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(scratch.data_ptr()),
        stream))
    torch.cuda.synchronize()
    return out.cpu().numpy().astype(np.uint32)


@pytest.mark.parametrize("vocab", [65536, 65535, 5000, 4097, 37, 3])
@pytest.mark.parametrize("temperature,top_k,penalty", [
    (0.1, 50, 1.1), (0.7, 64, 1.1), (1.5, 2, 0.8), (0.0, 50, 1.1),
    (2.0, 64, 1.0), (0.3, 1, 1.0)])
def test_device_matches_host(vocab, temperature, top_k, penalty):
    rng = np.random.default_rng(vocab * 7 + top_k)
    rows = 11  # two launch pairs (8 + 3 rows)
    x = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    recent = [(rng.integers(0, vocab, size=int(rng.integers(0, 60))).tolist()
               + [int(x[r].argmax())] * 2)[-64:] for r in range(rows)]
    seeds = rng.integers(0, 2**63, size=rows, dtype=np.uint64)
    smp = lfm3.sampler(temperature, top_k, penalty)
    want = lfm3.sample_host(x, smp, recent=recent, seeds=seeds)
    got = device_sample(x, smp, recent=recent, seeds=seeds)
    assert (got == want).all(), (got, want)


def test_device_ties_and_many_seeds():
    rng = np.random.default_rng(3)
    vocab = 65536
    # values on a 0.5 grid: hundreds of ties at every top-k boundary
    x = (np.round(rng.standard_normal((8, vocab)) * 2) / 2).astype(np.float32)
    x[:, 9000] = x[:, 70] = x.max() + 1
    for s in range(6):
        seeds = rng.integers(0, 2**63, size=8, dtype=np.uint64)
        for smp in (lfm3.sampler(0.0, 1, 1.0), lfm3.sampler(0.4, 50, 1.0),
                    lfm3.sampler(1.0, 64, 1.2)):
            recent = [[70, 70, 5]] * 3 + [[]] * 5
            want = lfm3.sample_host(x, smp, recent=recent, seeds=seeds)
            got = device_sample(x, smp, recent=recent, seeds=seeds)
            assert (got == want).all(), (s, got, want)
    got = device_sample(x, lfm3.sampler(0.0, 1, 1.0))
    assert (got == 70).all()


@pytest.fixture(scope="module")
def small():
    w = lfm3.SyntheticWeights(lfm3.small_config(), seed=0, norm_jitter=0.1)
    model = lfm3.Model(w.weights)
    return w, model


def test_forward_batch_sample_matches_host_selection(small):
    """A batched round with selection on the device picks, for every
    session, the host sampler's token over the same round's logits, and the
    logits stay readable."""
    w, model = small
    rng = np.random.default_rng(21)
    vocab = w.config.vocab
    a = [model.session(256) for _ in range(4)]
    b = [model.session(256) for _ in range(4)]
    for sa, sb, n in zip(a, b, (5, 17, 33, 40)):
        prompt = rng.integers(0, vocab, n).astype(np.uint32)
        sa.forward(prompt, logits=False)
        sb.forward(prompt, logits=False)
    smp = lfm3.sampler(0.7, 50, 1.1)
    history = [[int(t)] for t in rng.integers(0, vocab, 4)]
    tokens = [h[0] for h in history]
    for step in range(6):
        seeds = [1000 * step + r for r in range(4)]
        nxt = lfm3.Session.forward_batch_sample(a, tokens, smp,
                                                recent=history, seeds=seeds)
        mine = np.stack([s.read_logits() for s in a])
        want = lfm3.sample_host(mine, smp, recent=history, seeds=seeds)
        assert (nxt == want).all(), (step, nxt, want)
        # the same round through ForwardBatch (host logits)
        logits = np.stack(lfm3.Session.forward_batch(b, tokens))
        assert np.abs(logits - mine).max() <= 1e-4, step
        for r in range(4):
            history[r] = (history[r] + [int(nxt[r])])[-64:]
        tokens = [int(t) for t in nxt]
    assert [s.position for s in a] == [s.position for s in b]


def test_forward_batch_sample_refuses_without_mutation(small):
    w, model = small
    s = [model.session(64) for _ in range(2)]
    for x in s:
        x.forward([1, 2, 3], logits=False)
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.Session.forward_batch_sample(s, [1, 2], lfm3.sampler(0.5, 65, 1.0))
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.Session.forward_batch_sample(s, [1, 2], lfm3.sampler(),
                                          recent=[[w.config.vocab], []])
    assert [x.position for x in s] == [3, 3] and all(x.coherent for x in s)


def test_device_degenerate_rows():
    """Rows whose logits are all equal, two-valued, or tied exactly at the
    top-k boundary: the selection keeps the lowest ids among equals, on the
    device as on the host."""
    vocab = 65536
    x = np.zeros((6, vocab), np.float32)
    x[1, :] = 1.5
    x[2, ::2] = -2.0
    x[3, :] = -1.0
    x[3, 1000:1064] = 3.0                      # exactly 64 tied maxima
    x[4, 5::4096] = 7.0                        # one maximum per segment
    x[5, :] = np.float32(-0.0)
    x[5, 777] = 0.0                            # +0 above the -0 rows
    seeds = np.arange(6, dtype=np.uint64) * 12345 + 1
    for smp in (lfm3.sampler(0.0, 1, 1.0), lfm3.sampler(0.5, 50, 1.0),
                lfm3.sampler(0.5, 64, 1.1), lfm3.sampler(2.0, 1, 1.0)):
        recent = [[0, 1, 2]] * 6
        want = lfm3.sample_host(x, smp, recent=recent, seeds=seeds)
        got = device_sample(x, smp, recent=recent, seeds=seeds)
        assert (got == want).all(), (smp.temperature, smp.top_k, got, want)

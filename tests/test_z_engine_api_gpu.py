"""The engine surface beyond token rounds (the reference's engine.hpp):
input embeddings (ForwardEmbeddings with host or device rows, ForwardInputs
mixing token and embedding runs across a 512-row pass boundary,
ForwardBatchInputs with device rows), the continuation hooks
(continuation_hooks.hpp), PrepareLogits, BeginRestore / FinishRestore over
direct writes to the continuation buffers, Speculate and the d1 decision
stub. Each embedding path is checked against the token path whose embedding
rows it feeds (the Q8_0 rows dequantised on the host exactly as the kernels
do, d * q in FP32)."""
import ctypes

import numpy as np
import pytest

from helpers import abi, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def small():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    w = lfm3.SyntheticWeights(lfm3.small_config(), seed=0, norm_jitter=0.1)
    model = lfm3.Model(w.weights)
    return w, model


def embedding_rows(w, tokens):
    """Rows of the Q8_0 embedding table, dequantised as d * q in FP32."""
    t = w.weights.embedding
    assert t.type == abi.Q8_0
    hidden = t.cols
    raw = np.frombuffer(ctypes.string_at(t.data, t.bytes), np.uint8)
    table = raw.reshape(t.rows, hidden // 32, 34)
    d = table[:, :, :2].copy().view(np.float16).astype(np.float32)
    q = table[:, :, 2:].view(np.int8).astype(np.float32)
    rows = (q * d).reshape(t.rows, hidden)
    return np.ascontiguousarray(rows[np.asarray(tokens)])


def close(a, b):
    assert np.abs(np.asarray(a) - np.asarray(b)).max() <= TOL


def test_forward_embeddings_match_tokens(small):
    w, model = small
    rng = np.random.default_rng(31)
    tokens = rng.integers(0, w.config.vocab, 40).astype(np.uint32)
    rows = embedding_rows(w, tokens)
    a, b, c = (model.session(256) for _ in range(3))
    want = a.forward(tokens)
    close(b.forward_embeddings(rows), want)
    dev = torch.from_numpy(rows).cuda()
    torch.cuda.synchronize()
    close(c.forward_embeddings(None, device_rows=(dev.data_ptr(), len(tokens))),
          want)
    # one more row: the single-row (decode round) path
    t = int(rng.integers(0, w.config.vocab))
    row = embedding_rows(w, [t])
    want = a.forward([t])
    close(b.forward_embeddings(row), want)
    dev1 = torch.from_numpy(row).cuda()
    torch.cuda.synchronize()
    close(c.forward_embeddings(None, device_rows=(dev1.data_ptr(), 1)), want)
    assert a.position == b.position == c.position == 41


def test_forward_inputs_mixed_runs(small):
    """Token and embedding runs share passes; the embedding run straddles
    the first 512-row pass boundary."""
    w, model = small
    rng = np.random.default_rng(32)
    tokens = rng.integers(0, w.config.vocab, 600).astype(np.uint32)
    a, b = model.session(1024), model.session(1024)
    want = a.forward(tokens)
    got = b.forward_inputs([("tokens", tokens[:500]),
                            ("rows", embedding_rows(w, tokens[500:530])),
                            ("tokens", tokens[530:])])
    close(got, want)
    assert b.position == 600


def test_batch_inputs_with_device_rows(small):
    w, model = small
    rng = np.random.default_rng(33)
    vocab = w.config.vocab
    a = [model.session(256) for _ in range(3)]
    b = [model.session(256) for _ in range(3)]
    for sa, sb, n in zip(a, b, (7, 19, 33)):
        p = rng.integers(0, vocab, n).astype(np.uint32)
        sa.forward(p, logits=False)
        sb.forward(p, logits=False)
    tokens = [int(t) for t in rng.integers(0, vocab, 3)]
    dev = torch.from_numpy(embedding_rows(w, tokens)).cuda()
    torch.cuda.synchronize()
    stride = dev.shape[1] * 4
    rows = [dev.data_ptr(), None, dev.data_ptr() + 2 * stride]
    lfm3.Session.forward_batch_inputs(a, tokens, logits=True)
    lfm3.Session.forward_batch_inputs(b, [0, tokens[1], 0], logits=True, rows=rows)
    for sa, sb in zip(a, b):
        close(sb.read_logits(), sa.read_logits())
        assert sa.position == sb.position


def test_continuation_hooks(small):
    w, model = small
    s, t = model.session(128), model.session(128)
    calls, refuse = [], {"write": False}

    def before_write(first, end):
        calls.append(("write", first, end))
        return refuse["write"]

    s.set_continuation_hooks(before_write, lambda: calls.append(("reset",)),
                             lambda: calls.append(("restore",)))
    s.forward([1, 2, 3, 4, 5], logits=False)
    t.forward([6, 7, 8, 9, 10], logits=False)
    lfm3.Session.forward_batch([s, t], [11, 12], logits=False)
    assert calls == [("write", 0, 5), ("write", 5, 6)]
    snap = s.save_snapshot()
    # a refused write changes nothing
    refuse["write"] = True
    with pytest.raises(lfm3.Lfm3Error):
        s.forward([13], logits=False)
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.Session.forward_batch([t, s], [14, 15], logits=False)
    assert s.position == 6 and t.position == 6 and s.coherent and t.coherent
    refuse["write"] = False
    s.restore_snapshot(snap)
    s.reset()
    assert calls[-2:] == [("restore",), ("reset",)]
    # two accepted writes, two refused, the restore and the reset
    assert len(calls) == 6
    s.set_continuation_hooks()
    s.forward([1], logits=False)
    assert len(calls) == 6


def test_prepare_logits_and_direct_restore(small):
    w, model = small
    cfg = w.config
    rng = np.random.default_rng(34)
    a, b, ref = model.session(128), model.session(128), model.session(128)
    p = rng.integers(0, cfg.vocab, 21).astype(np.uint32)
    a.forward(p, logits=False)
    ref.forward(p, logits=False)
    lfm3.Session.forward_batch_inputs([a], [5], logits=False)
    want = lfm3.Session.forward_batch([ref], [5])[0]
    a.prepare_logits()
    close(a.read_logits(), want)
    # b takes a's state by direct copies between the continuation buffers
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_size_t, ctypes.c_int]
    d2d = 3

    def copy(tensor, layer, nbytes):
        assert cudart.cudaMemcpy(b.continuation_data(tensor, layer),
                                 a.continuation_data(tensor, layer), nbytes, d2d) == 0

    b.begin_restore()
    assert not b.coherent
    copy(0, 0, cfg.vocab * 4)
    copy(1, 0, cfg.hidden * 4)
    for i in range(cfg.n_layers):
        if cfg.layer_type[i] == abi.CONV:
            copy(2, i, cfg.hidden * (cfg.conv_width - 1) * 4)
        else:
            nbytes = a.ring_capacity(i) * cfg.kv_heads[i] * 128 * 2
            copy(3, i, nbytes)
            copy(4, i, nbytes)
    b.finish_restore(a.position)
    assert b.coherent and b.position == a.position
    np.testing.assert_array_equal(b.read_logits(), a.read_logits())
    for t in (7, 9, 11):
        close(b.forward([t]), a.forward([t]))


def test_speculate_and_decision_stub(small):
    w, model = small
    s = model.session(64)
    s.speculate(3)
    lib = lfm3.library()
    toks = np.array([1, 2], np.uint32)
    assert lib.lfm3_session_forward_decision(s.handle, lfm3._ptr(toks), 2,
                                             None) == -3
    assert s.position == 0 and s.coherent

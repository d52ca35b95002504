"""End-to-end parity of the B200 engine against the CPU oracle (the
restatement of reference.cpp, itself pinned to the compiled reference), and
the session invariants of the reference's tests/session_test.cpp: chunked vs
serial prefill, batched vs serial decode at ragged depths, exact reset,
snapshots, refusal of invalid input without mutation, poisoning."""
import os

import numpy as np
import pytest

from helpers import GOLDEN, ensure_oracle_built, kl, lfm3, top2_margin

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ensure_oracle_built()
import oracle  # noqa: E402

# north-star tolerances for Q8_0 logits
MAX_ABS = 5e-2
MAX_KL = 1e-3


@pytest.fixture(scope="module")
def small():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    w = lfm3.SyntheticWeights(lfm3.small_config(), seed=0, norm_jitter=0.1)
    model = lfm3.Model(w.weights)
    return w, model


def test_prompt_and_greedy_match_golden(small):
    """Prompt pass (40 rows, sliding window 32 wraps) then 20 greedy decode
    steps against the compiled reference's fixture."""
    w, model = small
    g = np.load(os.path.join(GOLDEN, "small.npz"))
    s = model.session(256)
    logits = s.forward(g["prompt"])
    got = [logits]
    for t in g["generated"]:
        got.append(s.forward([int(t)]))
    for step, (a, b) in enumerate(zip(got, g["logits"])):
        err = float(np.abs(a - b).max())
        assert err <= MAX_ABS, (step, err)
        assert kl(b, a) < MAX_KL, step
        if top2_margin(b) > 4 * err:
            assert int(np.argmax(a)) == int(np.argmax(b)), step


def test_free_running_greedy_matches_oracle(small):
    w, model = small
    o = oracle.Oracle(w.weights, 512, threads=4)
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, w.config.vocab, 70).astype(np.uint32)
    s = model.session(512)
    ours = s.forward(prompt)
    ref = o.run(prompt)[len(prompt) - 1]
    for step in range(24):
        assert float(np.abs(ours - ref).max()) <= MAX_ABS
        assert kl(ref, ours) < MAX_KL
        tok = int(np.argmax(ref))
        assert int(np.argmax(ours)) == tok or top2_margin(ref) < 1e-3, step
        ours = s.forward([tok])
        ref = o.step(tok, True)


def test_deep_prompt_matches_oracle(small):
    """A 2200-token prompt in 512-row passes (the full-attention layers'
    prompt attention on the tcgen05 kernel, keys split into three spans and
    merged by the combine kernel), then greedy steps, against the oracle
    with the engine's F16 K/V rounding (the configs' deep prompts at the
    small geometry)."""
    w, model = small
    n = 2200
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, w.config.vocab, n).astype(np.uint32)
    o = oracle.Oracle(w.weights, n + 8, threads=8, kv_half=True)
    marks = list(range(511, n, 512)) + [n - 1]
    want = o.run(prompt, logits_at=marks)
    s = model.session(n + 8)
    for first in range(0, n, 512):
        got = s.forward(prompt[first:first + 512])
        last = min(first + 512, n) - 1
        ref = want[last]
        err = float(np.abs(got - ref).max())
        assert err <= MAX_ABS, (last, err)
        assert kl(ref, got) < MAX_KL, last
    for step in range(3):
        tok = int(np.argmax(ref))
        got, ref = s.forward([tok]), o.step(tok, True)
        assert float(np.abs(got - ref).max()) <= MAX_ABS, step
        assert kl(ref, got) < MAX_KL, step


def test_chunked_matches_serial(small):
    """513 tokens in one Forward (512 + 1 rows) vs one token at a time
    (tests/session_test.cpp:117-144)."""
    w, model = small
    rng = np.random.default_rng(5)
    tokens = rng.integers(0, w.config.vocab, 513).astype(np.uint32)
    a, b = model.session(1024), model.session(1024)
    batched = a.forward(tokens)
    serial = None
    for i, t in enumerate(tokens):
        serial = b.forward([int(t)], logits=i + 1 == len(tokens))
    err = float(np.abs(serial - batched).max())
    assert kl(serial, batched) < 1e-5 and err < 0.02, (kl(serial, batched), err)
    assert int(np.argmax(serial)) == int(np.argmax(batched))
    # reset reproduces exact logits
    a.reset()
    again = a.forward(tokens)
    np.testing.assert_array_equal(again, batched)


@pytest.mark.parametrize("width", [2, 3, 4, 8])
def test_batched_matches_serial_at_ragged_depths(small, width):
    """C2/C3/C4/C8 rounds vs serial decode at depths 1/33/257/513
    (tests/session_test.cpp:224-283)."""
    w, model = small
    rng = np.random.default_rng(9)
    tokens = rng.integers(0, w.config.vocab, 600).astype(np.uint32)
    lanes, controls = [], []
    for row in range(width):
        count = [1, 33, 257, 513][row % 4]
        lanes.append(model.session(1024))
        controls.append(model.session(1024))
        lanes[-1].forward(tokens[:count], logits=False)
        controls[-1].forward(tokens[:count], logits=False)
    worst = 0.0
    for step in range(3):
        inputs = [int(tokens[(row + step) % len(tokens)]) for row in range(width)]
        actual = lfm3.Session.forward_batch(lanes, inputs)
        for row in range(width):
            expected = controls[row].forward([inputs[row]])
            assert lanes[row].position == controls[row].position
            assert np.isfinite(actual[row]).all()
            worst = max(worst, float(np.abs(actual[row] - expected).max()))
            assert int(np.argmax(actual[row])) == int(np.argmax(expected))
    assert worst < 0.002, worst
    # a duplicate session is refused without mutating anything
    boundary = lanes[0].position
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.Session.forward_batch([lanes[0], lanes[0]], [1, 2])
    assert lanes[0].position == boundary and lanes[0].coherent


def test_invalid_input_refused_without_mutation(small):
    w, model = small
    s = model.session(64)
    s.forward(list(range(10)), logits=False)
    with pytest.raises(lfm3.Lfm3Error):
        s.forward([w.config.vocab])
    assert s.position == 10
    with pytest.raises(lfm3.Lfm3Error):
        s.forward(list(range(60)))  # context overflow
    assert s.position == 10 and s.coherent
    with pytest.raises(lfm3.Lfm3Error):
        model.session(w.config.context + 1)


def test_snapshot_round_trip_and_fork(small):
    w, model = small
    rng = np.random.default_rng(2)
    tokens = rng.integers(0, w.config.vocab, 300).astype(np.uint32)
    a, b = model.session(512), model.session(512)
    a.forward(tokens[:290])  # sliding rings (32) wrapped
    snap = a.save_snapshot()
    before = a.read_logits()
    a.forward(tokens[290:297], logits=False)
    a.restore_snapshot(snap)
    b.restore_snapshot(snap)
    assert a.position == b.position == 290
    np.testing.assert_array_equal(a.read_logits(), before)
    np.testing.assert_array_equal(a.forward(tokens[297:300]),
                                  b.forward(tokens[297:300]))
    # every header word is checked (tests/session_test.cpp:200-207)
    for word in range(8):
        bad = snap.copy()
        bad[word * 4] ^= 0x80
        with pytest.raises(lfm3.Lfm3Error):
            a.restore_snapshot(bad)
        assert a.position == 293
    with pytest.raises(lfm3.Lfm3Error):
        a.restore_snapshot(snap[:-1])
    assert a.position == 293


def test_intermediate_and_empty_snapshots(small):
    """A snapshot taken after a prompt pass that computed no logits carries
    the frontier's logits, and replays like the uninterrupted session; an
    empty session's snapshot restores to position 0
    (tests/session_test.cpp:211-223)."""
    w, model = small
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, w.config.vocab, 300).astype(np.uint32)
    a, b = model.session(512), model.session(512)
    a.forward(tokens[:257], logits=False)
    partial = a.save_snapshot()
    want = b.forward(tokens[:257])
    np.testing.assert_allclose(a.read_logits(), want, rtol=0, atol=1e-5)
    a.forward(tokens[:19], logits=False)
    a.restore_snapshot(partial)
    np.testing.assert_allclose(a.forward(tokens[257:]), b.forward(tokens[257:]),
                               rtol=0, atol=1e-5)
    a.reset()
    empty = a.save_snapshot()
    b.restore_snapshot(empty)
    assert b.position == 0 and b.coherent


def test_snapshot_header_is_the_references(small):
    """Word 7 is the reference's ConfigSignature (engine.cpp:1403-1419), so a
    header written by the reference's engine restores: here one built word by
    word from the reference's rule (tests/test_snapshot_format.py) around
    this session's payload. An empty session writes zeros for the frontier
    and logits, as the reference does."""
    import struct
    from test_snapshot_format import reference_signature

    w, model = small
    cfg = w.config
    s = model.session(128)
    s.forward(list(range(40)), logits=False)
    snap = s.save_snapshot()
    words = struct.unpack("<8I", snap[:32].tobytes())
    assert words == (0x334D464C, 2, 128, 40, cfg.hidden, cfg.vocab,
                     cfg.n_layers, reference_signature(cfg))
    rebuilt = np.frombuffer(struct.pack(
        "<8I", 0x334D464C, 2, 128, 40, cfg.hidden, cfg.vocab, cfg.n_layers,
        reference_signature(cfg)), np.uint8)
    t = model.session(128)
    t.restore_snapshot(np.concatenate([rebuilt, snap[32:]]))
    np.testing.assert_array_equal(t.forward([7]), s.forward([7]))
    t.reset()
    empty = t.save_snapshot()
    assert not empty[32:32 + 4 * (cfg.hidden + cfg.vocab)].any()


def test_poisoned_session_refuses_snapshot(small):
    """A poisoned session's state may be half written: SaveSnapshot refuses
    it (engine.cpp:1471-1472) until Reset."""
    w, model = small
    s = model.session(128)
    s.forward([1, 2, 3], logits=False)
    s.inject_failure(5)
    with pytest.raises(lfm3.Lfm3Error):
        s.forward([4, 5, 6, 7])
    assert not s.coherent
    with pytest.raises(lfm3.Lfm3Error) as refused:
        s.save_snapshot()
    assert refused.value.code == -4  # LFM3_ERR_POISONED
    s.reset()
    assert s.save_snapshot().size > 0


def test_device_failure_poisons_until_reset(small):
    """A failing CUDA call mid-pass (injected on the host) poisons the
    session; it refuses work until Reset (engine.cpp:905-927, 1300-1332)."""
    w, model = small
    s = model.session(128)
    s.forward([1, 2, 3], logits=False)
    s.inject_failure(5)
    with pytest.raises(lfm3.Lfm3Error):
        s.forward([4, 5, 6, 7])
    assert not s.coherent
    with pytest.raises(lfm3.Lfm3Error):
        s.forward([4])
    s.reset()
    assert s.coherent and s.position == 0
    fresh = model.session(128)
    np.testing.assert_array_equal(s.forward([1, 2, 3]), fresh.forward([1, 2, 3]))
    assert lfm3.library().lfm3_cuda_take_device_error() == 0


def test_bounded_wait_gives_up_and_reports():
    """A device wait that nothing ends gives up after its limit and records
    its code in the device error word; the context stays usable."""
    lib = lfm3.library()
    lib.lfm3_cuda_take_device_error()
    lfm3.check(lib.lfm3_cuda_wait_probe(20000, None))
    torch.cuda.synchronize()
    assert lib.lfm3_cuda_take_device_error() == 5
    assert lib.lfm3_cuda_take_device_error() == 0
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2


def test_device_wait_failure_reported_by_next_round(small):
    """ForwardBatchInputs returns before its round ends: a device wait that
    gave up is reported by the next round, which fails and poisons its
    sessions until Reset."""
    w, model = small
    lib = lfm3.library()
    a, b = model.session(64), model.session(64)
    a.forward([1, 2, 3], logits=False)
    b.forward([4, 5], logits=False)
    lfm3.Session.forward_batch_inputs([a, b], [6, 7])
    torch.cuda.synchronize()  # that round ends before the failing wait runs
    lib.lfm3_cuda_take_device_error()
    lfm3.check(lib.lfm3_cuda_wait_probe(5000, None))
    torch.cuda.synchronize()
    # this round's last kernel sees the error word; once it has finished, the
    # next round reports it
    lfm3.Session.forward_batch_inputs([a, b], [8, 9])
    torch.cuda.synchronize()
    with pytest.raises(lfm3.Lfm3Error):
        lfm3.Session.forward_batch_inputs([a, b], [10, 11])
    assert not a.coherent and not b.coherent
    assert lib.lfm3_cuda_take_device_error() == 0
    a.reset()
    b.reset()
    assert a.coherent and b.coherent
    fresh = model.session(64)
    np.testing.assert_array_equal(a.forward([1, 2, 3]), fresh.forward([1, 2, 3]))


@pytest.mark.parametrize("sample", [True, False])
def test_device_wait_failure_reported_by_synchronous_round(small, sample):
    """ForwardBatchSample and ForwardBatch (logits) wait for their round and
    read the failure from the host-mapped word the round's last kernel
    wrote: the call fails, poisons its sessions and consumes the code."""
    w, model = small
    lib = lfm3.library()
    a, b = model.session(64), model.session(64)
    a.forward([1, 2, 3], logits=False)
    b.forward([4, 5], logits=False)
    torch.cuda.synchronize()
    lib.lfm3_cuda_take_device_error()
    lfm3.check(lib.lfm3_cuda_wait_probe(5000, None))
    torch.cuda.synchronize()
    with pytest.raises(lfm3.Lfm3Error):
        if sample:
            lfm3.Session.forward_batch_sample([a, b], [6, 7],
                                              lfm3.sampler(0.0, 1, 1.0))
        else:
            lfm3.Session.forward_batch([a, b], [6, 7])
    assert not a.coherent and not b.coherent
    assert lib.lfm3_cuda_take_device_error() == 0
    a.reset()
    b.reset()
    # a clean round afterwards goes through
    a.forward([1, 2, 3], logits=False)
    b.forward([4, 5], logits=False)
    lfm3.Session.forward_batch_sample([a, b], [6, 7], lfm3.sampler(0.0, 1, 1.0))
    assert a.coherent and b.coherent


# ---- BF16 numerical-reference weights (north-star logits tolerance 2e-2) ------
BF16_MAX_ABS = 2e-2


@pytest.fixture(scope="module")
def small_bf16():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    w = lfm3.SyntheticWeights(lfm3.small_config(), seed=0, matrix_type=lfm3.abi.BF16,
                              norm_jitter=0.1)
    model = lfm3.Model(w.weights)
    return w, model


def test_bf16_prompt_and_greedy_match_golden(small_bf16):
    """BF16 matrices: prompt pass (CUDA-core exact BF16 x FP32 projections)
    and 20 greedy decode steps against the compiled reference's fixture."""
    w, model = small_bf16
    g = np.load(os.path.join(GOLDEN, "small_bf16.npz"))
    s = model.session(256)
    logits = s.forward(g["prompt"])
    got = [logits]
    for t in g["generated"]:
        got.append(s.forward([int(t)]))
    for step, (a, b) in enumerate(zip(got, g["logits"])):
        err = float(np.abs(a - b).max())
        assert err <= BF16_MAX_ABS, (step, err)
        assert kl(b, a) < MAX_KL, step
        if top2_margin(b) > 4 * err:
            assert int(np.argmax(a)) == int(np.argmax(b)), step


def test_bf16_batched_matches_serial(small_bf16):
    """A batched BF16 decode round equals each session's own serial step."""
    w, model = small_bf16
    rng = np.random.default_rng(23)
    lengths = [5, 33, 70]
    prompts = [rng.integers(0, w.config.vocab, n).astype(np.uint32) for n in lengths]
    batch = [model.session(256) for _ in lengths]
    serial = [model.session(256) for _ in lengths]
    for a, b, p in zip(batch, serial, prompts):
        a.forward(p)
        b.forward(p)
    nxt = [int(t) for t in rng.integers(0, w.config.vocab, len(lengths))]
    outs = lfm3.Session.forward_batch(batch, nxt)
    for o, s, t in zip(outs, serial, nxt):
        ref = s.forward([t])
        assert float(np.abs(o - ref).max()) <= 2e-3
        assert int(np.argmax(o)) == int(np.argmax(ref))

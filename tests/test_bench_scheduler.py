"""The bench's config-3 scheduler (bench.config3_job) on the CPU against a
fake engine that records every call: arrivals are respected, prompt passes
go first-come first-served in chunks of at most 512 rows, one pass precedes
each decode round, every decoding session is in each round (at most 8 rows),
each session decodes exactly the requested tokens, and the device selection
gets each row's penalty window and a fresh seed."""
import os
import sys
from types import SimpleNamespace

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


class FakeSession:
    def __init__(self, log, index, context):
        self.log, self.index, self.context = log, index, context
        self.position = 0
        self.closed = False

    def forward(self, tokens, logits=True):
        self.log.append(("pass", self.index, self.position, len(tokens), logits))
        self.position += len(tokens)
        assert self.position <= self.context
        return np.zeros(16, np.float32) if logits else None

    def close(self):
        self.closed = True


def fake_engine():
    log, made = [], []

    class Model:
        def session(self, context):
            s = FakeSession(log, len(made), context)
            made.append(s)
            return s

    def forward_batch_sample(sessions, tokens, smp, recent=None, seeds=None):
        assert 1 <= len(sessions) <= 8
        assert len(recent) == len(seeds) == len(tokens) == len(sessions)
        for s, t, r in zip(sessions, tokens, recent):
            assert r[-1] == t and len(r) <= 64  # the consumed token is penalised
            s.position += 1
        log.append(("round", [s.index for s in sessions], list(seeds)))
        return np.array([(t * 7 + 1) % 16 for t in tokens], np.uint32)

    lfm3 = SimpleNamespace(
        sampler=lambda *a: a,
        sample_host=lambda logits, smp, recent=None, seeds=None: np.array([3], np.uint32),
        Session=SimpleNamespace(forward_batch_sample=forward_batch_sample))
    return lfm3, Model(), log, made


def test_config3_schedule():
    lfm3, model, log, made = fake_engine()
    cfg = SimpleNamespace(vocab=16)
    decode = 40
    trace = []
    job = bench.config3_job(lfm3, model, cfg, rank=0, prompt_max=1500,
                            decode_tokens=decode, trace=trace)
    lengths, _ = bench.rank_workload(0, 1500, 16)
    arrive = job["arrivals"]
    assert arrive[0] == 0 and all(0 <= b - a <= 2 for a, b in zip(arrive, arrive[1:]))
    # every engine call carries its scheduler step; a step holds at most one
    # pass, then at most one round
    assert len(trace) == len(log)
    assert [t[1] for t in trace] == [e[0] for e in log]
    for (s0, k0, _), (s1, k1, _) in zip(trace, trace[1:]):
        assert s1 > s0 or (s1 == s0 and k0 == "pass" and k1 == "round")
    passes, rounds_rows = [], []
    prompt_done = [0] * 8
    decoded = [0] * 8
    for (step, _, _), entry in zip(trace, log):
        if entry[0] == "pass":
            _, i, pos, n, want_logits = entry
            assert arrive[i] <= step, "pass before the session arrived"
            assert pos == prompt_done[i] and 1 <= n <= 512
            # FIFO: no earlier arrived session still has prompt left
            for j in range(i):
                assert not (arrive[j] <= step and prompt_done[j] < lengths[j])
            prompt_done[i] += n
            assert want_logits == (prompt_done[i] == lengths[i])
            if want_logits:
                decoded[i] = 1
            passes.append(step)
        else:
            _, rows, seeds = entry
            live = [i for i in range(8) if prompt_done[i] == lengths[i] and decoded[i] < decode]
            assert rows == live and len(set(seeds)) == len(seeds)
            for i in rows:
                decoded[i] += 1
            rounds_rows.append(len(rows))
    assert decoded == [decode] * 8
    assert prompt_done == [int(n) for n in lengths]
    assert job["passes"] == sum(-(-int(n) // 512) for n in lengths) == len(passes)
    assert job["rounds"] == len(rounds_rows)
    assert job["decode_tokens"] == sum(rounds_rows) == 8 * (decode - 1)
    assert job["prefill_tokens"] == int(sum(lengths))
    assert all(s.closed for s in made)

"""The bench's config-3 job driver (bench.config3_job) on the CPU against a
fake scheduler that records every call: requests are admitted exactly at
their arrival steps (0-2 steps apart) with their whole prompt, 256-token
budget, distinct seeds and a context that holds prompt + budget; the job
steps until the scheduler is idle and aggregates the pass and round
statistics. (The scheduling itself, passes and rounds, is the library's
lfm3_scheduler, checked on the GPU by tests/test_scheduler_gpu.py.)"""
import os
import sys
from types import SimpleNamespace

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


class FakeScheduler:
    """First come first served passes of <= 512 rows, then a round of every
    request whose prompt is done, like lfm3_scheduler."""

    def __init__(self, model, sampler):
        self.reqs, self.step_no, self.admits, self.closed = [], 0, [], False

    def admit(self, prompt, max_new, seed, context):
        assert len(prompt) + max_new <= context
        self.admits.append((self.step_no, len(prompt), max_new, seed))
        self.reqs.append({"n": len(prompt), "done": 0, "gen": 0, "max": max_new})
        return len(self.reqs) - 1

    def step(self):
        st = SimpleNamespace(pass_request=-1, pass_rows=0, round_rows=0,
                             pass_ms=1.0, round_ms=2.0)
        for i, r in enumerate(self.reqs):
            if r["done"] < r["n"]:
                k = min(512, r["n"] - r["done"])
                r["done"] += k
                if r["done"] == r["n"]:
                    r["gen"] = 1
                st.pass_request, st.pass_rows = i, k
                break
        live = [r for r in self.reqs if r["done"] == r["n"] and 0 < r["gen"] < r["max"]]
        for r in live[:8]:
            r["gen"] += 1
        st.round_rows = len(live[:8])
        self.step_no += 1
        return st

    @property
    def idle(self):
        return all(r["gen"] >= r["max"] for r in self.reqs)

    def tokens(self, i):
        return np.zeros(self.reqs[i]["gen"], np.uint32)

    def close(self):
        self.closed = True


def test_config3_job_driver():
    made = []

    def make(model, sampler):
        made.append(FakeScheduler(model, sampler))
        return made[-1]

    lfm3 = SimpleNamespace(sampler=lambda *a: a, Scheduler=make)
    cfg = SimpleNamespace(vocab=16)
    decode = 40
    trace = []
    job = bench.config3_job(lfm3, object(), cfg, rank=0, prompt_max=1500,
                            decode_tokens=decode, trace=trace)
    sched = made[0]
    lengths, _ = bench.rank_workload(0, 1500, 16)
    arrive = job["arrivals"]
    assert arrive[0] == 0 and all(0 <= b - a <= 2 for a, b in zip(arrive, arrive[1:]))
    assert [a[0] for a in sched.admits] == arrive
    assert [a[1] for a in sched.admits] == [int(n) for n in lengths]
    assert all(a[2] == decode for a in sched.admits)
    assert len({a[3] for a in sched.admits}) == 8
    assert job["passes"] == sum(-(-int(n) // 512) for n in lengths)
    assert job["prefill_tokens"] == int(sum(lengths))
    assert job["decode_tokens"] == 8 * (decode - 1)
    assert abs(job["prefill_s"] - job["passes"] * 1e-3) < 1e-9
    assert abs(job["decode_s"] - job["rounds"] * 2e-3) < 1e-9
    assert sum(1 for t in trace if t[1] == "pass") == job["passes"]
    assert sched.closed

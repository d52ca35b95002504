"""The multi-GPU bench path (replicas, no collective on the data path) as
world-size-2 `gloo` ranks on the CPU: rank plumbing, the MAX over ranks, the
per-rank session partition and the whole-job rate."""
import json
import os
import socket
import sys

import pytest

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK=str(rank))
    import bench
    ranks = bench.Ranks("gloo")
    lengths, prompts = bench.rank_workload(ranks.rank, 4096, 65536)
    # a timing that differs per rank: the job is as slow as its slowest rank
    slowest = ranks.sync_max(10.0 + ranks.rank)
    tokens = ranks.sync_sum(float(sum(len(p) for p in prompts)))
    ranks.barrier()
    c5_lengths, c5_prompts = bench.config5_workload(ranks.rank, 65536)
    record = {"rank": ranks.rank, "world": ranks.world, "slowest": slowest,
              "tokens": tokens, "lengths": [int(n) for n in lengths],
              "c5_lengths": [int(n) for n in c5_lengths],
              "c5_heads": [[int(t) for t in p[:4]] for p in c5_prompts],
              "rate": bench.job_rate(bench.SESSIONS * 4, ranks.world, slowest)}
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(record, f)
    ranks.close()


def test_two_rank_replicas(tmp_path):
    world, port = 2, _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    recs = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    assert [r["rank"] for r in recs] == [0, 1]
    assert all(r["world"] == 2 for r in recs)
    # MAX over ranks: both see rank 1's 11 ms
    assert all(r["slowest"] == 11.0 for r in recs)
    # sessions are partitioned: each rank draws its own prompt lengths
    assert recs[0]["lengths"] != recs[1]["lengths"]
    assert all(64 <= n <= 4096 for r in recs for n in r["lengths"])
    total = sum(sum(r["lengths"]) for r in recs)
    assert all(r["tokens"] == total for r in recs)
    # config 5's 64 sessions: 8 per rank, disjoint between ranks, prompts
    # log-uniform in [512, 32768]
    assert all(len(r["c5_lengths"]) == 8 for r in recs)
    assert all(512 <= n <= 32768 for r in recs for n in r["c5_lengths"])
    heads = [tuple(h) for r in recs for h in r["c5_heads"]]
    assert len(set(heads)) == len(heads)
    # whole-job rate: 8 sessions x 4 steps on each of 2 ranks over 11 ms
    assert recs[0]["rate"] == pytest.approx(8 * 4 * 2 / 0.011)


def test_single_rank_defaults(monkeypatch):
    for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    import bench
    ranks = bench.Ranks("gloo")
    assert (ranks.world, ranks.rank, ranks.local) == (1, 0, 0)
    assert ranks.sync_max(3.5) == 3.5 and ranks.sync_sum(2.0) == 2.0
    ranks.barrier()
    ranks.close()

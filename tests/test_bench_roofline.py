"""The bench's roofline arithmetic on the graded geometry (CPU): decode
bytes per round (Q8_0 weights once plus, per row, the K/V rows attention
reads, the new K/V row, convolution state, logits and the embedding row) and
prompt-pass FLOPs with the engine's live-row pruning, against the figures
derived by hand for this geometry."""
import os
import sys

import pytest

from helpers import lfm3

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.fixture(scope="module")
def cfg():
    return lfm3.default_config()


def test_weight_bytes(cfg):
    assert bench.matrix_elements(cfg) * 34 // 32 == 1_780_733_952


def test_decode_round_bytes(cfg):
    assert bench.decode_round_bytes(cfg, [0] * 8) == 1_794_984_192
    assert bench.decode_round_bytes(cfg, [2048] * 8) == 2_017_200_384
    # BF16: 2 bytes per weight and a 4096-byte BF16 embedding row per token
    # (the hand figure 4,192,416,000 counted the Q8_0 row's 2176 bytes)
    assert bench.decode_round_bytes(cfg, [8192] * 8, bf16=True) == \
        4_192_416_000 + 8 * (4096 - 2176)


@pytest.mark.parametrize("position,tflop", [(0, 1.4650), (1536, 1.4986),
                                            (32256, 2.1446)])
def test_prefill_flops(cfg, position, tflop):
    assert bench.prefill_flops(cfg, 512, position) / 1e12 == \
        pytest.approx(tflop, abs=5e-5)


def test_traffic_comes_from_the_data_file():
    """roofline.traffic reads profiles/traffic.json (never a Markdown
    summary); the recorded round traffic is within a few percent of the
    algorithmic weight bytes (every weight byte read once)."""
    per_launch = bench.committed_traffic("decode_gemv_round")
    assert per_launch is not None
    import json
    entry = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))["decode_gemv_round"]
    assert per_launch == entry["dram_bytes_per_launch"]
    ratio = per_launch / entry["algorithmic_bytes_per_launch"]
    assert 0.99 < ratio < 1.05
    assert bench.committed_traffic("no such kernel") is None

"""Shared test helpers: the package, the oracle and comparison metrics."""
import importlib
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")

lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
abi = lfm3.abi


def kl(p_logits, q_logits):
    """KL(softmax(p) || softmax(q)) in float64."""
    p = np.asarray(p_logits, np.float64)
    q = np.asarray(q_logits, np.float64)
    lp = p - p.max()
    lp -= np.log(np.exp(lp).sum())
    lq = q - q.max()
    lq -= np.log(np.exp(lq).sum())
    return float((np.exp(lp) * (lp - lq)).sum())


def top2_margin(logits):
    top = np.partition(np.asarray(logits), -2)[-2:]
    return float(top.max() - top.min())


def ensure_oracle_built():
    """Builds oracle/liboracle.so (and oracle/_ref when the reference tree is
    present) if missing."""
    import subprocess
    lib = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "all"],
                       check=True)
    return lib

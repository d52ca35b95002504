"""Generates the golden fixtures of tests/golden/ by running the reference's
own CPU oracle (reference.cpp compiled unmodified into oracle/_ref, see
oracle/Makefile) on the synthetic weights of lfm3_synth_generate.

  config1.npz  graded geometry (hidden 2048, FFN 8192, 16/4 heads, vocab
               65536, 24 layers CCSGCCSGCCSGCCSGCCSGCCGC), Q8_0, seed 0:
               uniform 128-token prompt (numpy default_rng(0)), 64 greedy
               tokens, full logits after the prompt and after the last step,
               per-step argmax and top-2 margin.
  small.npz    small geometry of the same architecture (tests' small_config,
               norm jitter 0.1): 40-token prompt (default_rng(7)), 20 greedy
               tokens, logits after the prompt and after every greedy step.
  config1_bf16.npz, small_bf16.npz
               the same with BF16 matrices (the numerical-reference weights,
               N(0, 0.02) rounded to BF16 instead of quantised to Q8_0).

Run from the repository root:
  python tests/golden/make_golden.py [small|config1|small_bf16|config1_bf16]
(each config1 fixture takes about ten minutes of one core).
"""
import importlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
import oracle  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

SMALL = dict(norm_jitter=0.1, prompt=40, steps=20, seed=7)
CONFIG1 = dict(prompt=128, steps=64, seed=0)


def small(matrix_type=lfm3.abi.Q8_0, name="small.npz"):
    w = lfm3.SyntheticWeights(lfm3.small_config(), seed=0, matrix_type=matrix_type,
                              norm_jitter=SMALL["norm_jitter"])
    ref = oracle.ReferenceOracle(w.weights, 256)
    rng = np.random.default_rng(SMALL["seed"])
    prompt = rng.integers(0, w.config.vocab, SMALL["prompt"]).astype(np.uint32)
    logits = [ref.step(int(t), i + 1 == len(prompt))
              for i, t in enumerate(prompt)][-1:]
    generated = []
    for _ in range(SMALL["steps"]):
        tok = int(np.argmax(logits[-1]))
        generated.append(tok)
        logits.append(ref.step(tok, True))
    np.savez_compressed(os.path.join(HERE, name), prompt=prompt,
                        generated=np.array(generated, np.uint32),
                        logits=np.stack(logits).astype(np.float32))


def config1(matrix_type=lfm3.abi.Q8_0, name="config1.npz"):
    w = lfm3.SyntheticWeights(seed=0, matrix_type=matrix_type)
    ref = oracle.ReferenceOracle(w.weights, 1024)
    rng = np.random.default_rng(CONFIG1["seed"])
    prompt = rng.integers(0, w.config.vocab, CONFIG1["prompt"]).astype(np.uint32)
    t0 = time.time()
    logits = None
    for i, t in enumerate(prompt):
        logits = ref.step(int(t), i + 1 == len(prompt))
    after_prompt = logits.copy()
    generated, argmax, margin = [], [], []
    for _ in range(CONFIG1["steps"]):
        top2 = np.partition(logits, -2)[-2:]
        tok = int(np.argmax(logits))
        generated.append(tok)
        argmax.append(tok)
        margin.append(float(top2.max() - top2.min()))
        logits = ref.step(tok, True)
    np.savez_compressed(os.path.join(HERE, name), prompt=prompt,
                        generated=np.array(generated, np.uint32),
                        after_prompt=after_prompt.astype(np.float32),
                        final=logits.astype(np.float32),
                        margin=np.array(margin, np.float32),
                        seconds=np.float64(time.time() - t0))


if __name__ == "__main__":
    which = sys.argv[1:] or ["small", "config1"]
    if "small" in which:
        small()
    if "config1" in which:
        config1()
    if "small_bf16" in which:
        small(lfm3.abi.BF16, "small_bf16.npz")
    if "config1_bf16" in which:
        config1(lfm3.abi.BF16, "config1_bf16.npz")

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
  config1_f16kv.npz, config2.npz, ragged_bf16.npz
               made with the restatement (oracle/lfm3_oracle.c, pinned bit
               for bit to the compiled reference by tests/test_oracle.py) on 8
               threads: config 1 with K/V rounded through fp16 (the engine's
               rings), BASELINE config 2 (2048-token prompt, 128 greedy
               tokens), and BF16 sessions at depths 300 / 700 / 1100.

Run from the repository root:
  python tests/golden/make_golden.py [small|config1|small_bf16|config1_bf16|
                                      config1_f16kv|config2|ragged_bf16]
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


def greedy_run(ref, prompt, steps, name, **extra):
    """Prompt, then `steps` free-running greedy tokens of one oracle: tokens,
    logits after the prompt and after the last step, top-2 margins."""
    t0 = time.time()
    logits = None
    for i, t in enumerate(prompt):
        logits = ref.step(int(t), i + 1 == len(prompt))
    after_prompt = logits.copy()
    generated, margin = [], []
    for _ in range(steps):
        top2 = np.partition(logits, -2)[-2:]
        generated.append(int(np.argmax(logits)))
        margin.append(float(top2.max() - top2.min()))
        logits = ref.step(generated[-1], True)
    np.savez_compressed(os.path.join(HERE, name), prompt=prompt,
                        generated=np.array(generated, np.uint32),
                        after_prompt=after_prompt.astype(np.float32),
                        final=logits.astype(np.float32),
                        margin=np.array(margin, np.float32),
                        seconds=np.float64(time.time() - t0), **extra)


def config1_f16kv(threads=8):
    """config1's prompt and 64 greedy tokens through the restatement with
    its test-only F16 K/V switch: the reference's arithmetic with the K/V
    rounding of the engine's F16 rings as the only change."""
    w = lfm3.SyntheticWeights(seed=0)
    ref = oracle.Oracle(w.weights, 1024, threads=threads, kv_half=True)
    rng = np.random.default_rng(CONFIG1["seed"])
    prompt = rng.integers(0, w.config.vocab, CONFIG1["prompt"]).astype(np.uint32)
    greedy_run(ref, prompt, CONFIG1["steps"], "config1_f16kv.npz")


CONFIG2 = dict(prompt=2048, steps=128, seed=2)


def config2(threads=8):
    """BASELINE config 2 on the restatement (bit-exact with reference.cpp):
    Q8_0, a 2048-token uniform prompt, then 128 greedy tokens."""
    w = lfm3.SyntheticWeights(seed=0)
    ref = oracle.Oracle(w.weights, 4096, threads=threads)
    rng = np.random.default_rng(CONFIG2["seed"])
    prompt = rng.integers(0, w.config.vocab, CONFIG2["prompt"]).astype(np.uint32)
    greedy_run(ref, prompt, CONFIG2["steps"], "config2.npz")


RAGGED = dict(prompts=(300, 700, 1100), rounds=4, seed=3)


def ragged_bf16(threads=8):
    """BF16 numerical-reference weights at full geometry: three sessions with
    prompts of 300, 700 and 1100 tokens (sliding rings of 256 wrapped), then
    4 rounds in which every session advances its own greedy token; logits of
    every session after its prompt and after every round."""
    w = lfm3.SyntheticWeights(seed=0, matrix_type=lfm3.abi.BF16)
    rng = np.random.default_rng(RAGGED["seed"])
    prompts = [rng.integers(0, w.config.vocab, n).astype(np.uint32)
               for n in RAGGED["prompts"]]
    logits, tokens = [], []
    for prompt in prompts:
        ref = oracle.Oracle(w.weights, 2048, threads=threads)
        out = ref.run(prompt)[len(prompt) - 1]
        rows, toks = [out], []
        for _ in range(RAGGED["rounds"]):
            toks.append(int(np.argmax(rows[-1])))
            rows.append(ref.step(toks[-1], True))
        logits.append(np.stack(rows).astype(np.float32))
        tokens.append(toks)
        ref.close()
    np.savez_compressed(os.path.join(HERE, "ragged_bf16.npz"),
                        prompt0=prompts[0], prompt1=prompts[1],
                        prompt2=prompts[2], tokens=np.array(tokens, np.uint32),
                        logits=np.stack(logits))


if __name__ == "__main__":
    which = sys.argv[1:] or ["small", "config1"]
    if "config1_f16kv" in which:
        config1_f16kv()
    if "config2" in which:
        config2()
    if "ragged_bf16" in which:
        ragged_bf16()
    if "small" in which:
        small()
    if "config1" in which:
        config1()
    if "small_bf16" in which:
        small(lfm3.abi.BF16, "small_bf16.npz")
    if "config1_bf16" in which:
        config1(lfm3.abi.BF16, "config1_bf16.npz")

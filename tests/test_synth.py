"""Synthetic weights: deterministic, thread-count independent, and Q8_0
blocks follow the llama.cpp rule (d = amax / 127 as fp16, q = round(x / d))
applied to the BF16 values."""
import ctypes

import numpy as np

from helpers import abi, lfm3


def tensor_bytes(t):
    return np.ctypeslib.as_array(ctypes.cast(t.data, ctypes.POINTER(ctypes.c_uint8)),
                                 (t.bytes,)).copy()


def test_deterministic_and_thread_independent():
    cfg = lfm3.small_config()
    a = lfm3.SyntheticWeights(cfg, seed=0, threads=1)
    b = lfm3.SyntheticWeights(cfg, seed=0, threads=5)
    c = lfm3.SyntheticWeights(cfg, seed=1, threads=2)
    for name in ("embedding", "output_norm", "rope_freqs"):
        ta, tb = getattr(a.weights, name), getattr(b.weights, name)
        np.testing.assert_array_equal(tensor_bytes(ta), tensor_bytes(tb))
    for name in ("gate", "in_proj", "conv"):
        np.testing.assert_array_equal(tensor_bytes(getattr(a.weights.layers[0], name)),
                                      tensor_bytes(getattr(b.weights.layers[0], name)))
    assert not np.array_equal(tensor_bytes(a.weights.embedding),
                              tensor_bytes(c.weights.embedding))
    # tied output (weights.cpp:55-57)
    assert a.weights.output.data == a.weights.embedding.data


def test_q8_blocks_follow_the_rule():
    cfg = lfm3.small_config()
    q8 = lfm3.SyntheticWeights(cfg, seed=0, matrix_type=abi.Q8_0)
    bf = lfm3.SyntheticWeights(cfg, seed=0, matrix_type=abi.BF16)
    t8, tb = q8.weights.layers[1].gate, bf.weights.layers[1].gate
    assert t8.rows == tb.rows and t8.cols == tb.cols
    raw = tensor_bytes(t8).reshape(t8.rows, t8.cols // 32, 34)
    d = raw[:, :, :2].copy().view(np.float16)[..., 0].astype(np.float32)
    q = raw[:, :, 2:].view(np.int8).astype(np.float32)
    x = (tensor_bytes(tb).view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    x = x.reshape(t8.rows, t8.cols // 32, 32)
    amax = np.abs(x).max(-1)
    d32 = (amax / np.float32(127)).astype(np.float32)
    np.testing.assert_array_equal(d, d32.astype(np.float16).astype(np.float32))
    inv = np.where(d32 != 0, np.float32(1) / d32, np.float32(0)).astype(np.float32)
    scaled = (x * inv[..., None]).astype(np.float32)
    expect = np.sign(scaled) * np.floor(np.abs(scaled) + np.float32(0.5))
    np.testing.assert_array_equal(q, expect)
    # approximately N(0, 0.02)
    assert abs(float(x.std()) - 0.02) < 0.001
    assert abs(float(x.mean())) < 0.001


def test_norms_rope_and_conv_weights():
    w = lfm3.SyntheticWeights(lfm3.small_config(), seed=0)
    n = tensor_bytes(w.weights.layers[0].norm).view(np.float32)
    np.testing.assert_array_equal(n, np.ones_like(n))
    r = tensor_bytes(w.weights.rope_freqs).view(np.float32)
    assert r.size == 64
    np.testing.assert_array_equal(r[:32], np.ones(32, np.float32))
    np.testing.assert_array_equal(r[32:], np.full(32, 1e30, np.float32))
    conv = w.weights.layers[0].conv
    assert (conv.cols, conv.rows, conv.type) == (7, w.config.hidden, abi.F32)


def test_half_conversions_match_numpy():
    lib = lfm3.library()
    rng = np.random.default_rng(0)
    values = np.concatenate([
        rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 2000), [65504, 65520, 1e-8,
        -6.1e-5, 0.0, -0.0, 2.0**-25, 3 * 2.0**-26]]).astype(np.float32)
    for v in values:
        bits = lib.lfm3_float_to_half(float(v))
        assert bits == int(np.float16(v).view(np.uint16)), v
        back = lib.lfm3_half_to_float(bits)
        assert back == float(np.float16(v)) or (np.isinf(back) and np.isinf(np.float16(v)))


def test_default_geometry():
    cfg = lfm3.default_config()
    assert (cfg.hidden, cfg.intermediate, cfg.vocab, cfg.heads, cfg.head_dim) == (
        2048, 8192, 65536, 16, 128)
    assert cfg.pattern() == "CCSGCCSGCCSGCCSGCCSGCCGC"
    assert [cfg.kv_heads[i] for i in range(24)].count(4) == 11
    assert (cfg.window, cfg.conv_width, cfg.context) == (256, 7, 262144)


def test_oracle_copy_of_the_generator_matches_and_loads_no_cuda_library():
    """The bench's reference arm makes its weights with the generator built
    into the oracle libraries: the same bytes as the package's, and the
    process maps no library of this package."""
    import subprocess
    import sys

    from helpers import ROOT, ensure_oracle_built
    ensure_oracle_built()
    import oracle
    cfg = lfm3.small_config()
    a = lfm3.SyntheticWeights(cfg, seed=4, threads=2)
    for prefer in (False, True):
        b = oracle.SyntheticWeights(cfg, seed=4, threads=3, prefer_reference=prefer)
        for name in ("embedding", "output_norm"):
            np.testing.assert_array_equal(tensor_bytes(getattr(a.weights, name)),
                                          tensor_bytes(getattr(b.weights, name)))
        np.testing.assert_array_equal(tensor_bytes(a.weights.layers[2].q),
                                      tensor_bytes(b.weights.layers[2].q))
    code = ("import sys; sys.path[:0] = [%r, %r]; import oracle; "
            "w = oracle.SyntheticWeights(oracle.default_config(), seed=0); "
            "print(open('/proc/self/maps').read())" % (ROOT, f"{ROOT}/oracle"))
    maps = subprocess.run([sys.executable, "-c", code], capture_output=True,
                          text=True, check=True).stdout
    assert "liblfm3_cuda" not in maps
    assert "oracle" in maps

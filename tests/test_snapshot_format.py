"""Snapshot v2 header compatibility with the reference's engine, on the CPU.

Header word 7 is the reference's ConfigSignature (engine.cpp:1403-1419),
restated here independently of the library: FNV-1a over the bytes (little
endian) of hidden, intermediate, vocab, heads, head_dim, window, conv_width,
the bit patterns of eps, theta and theta_swa, then each layer's type and KV
head count. A snapshot written by either engine carries the same word, so it
restores in the other.
"""
import ctypes
import struct

import pytest

from helpers import abi, lfm3


def reference_signature(cfg):
    h = 2166136261

    def mix(value):
        nonlocal h
        for i in range(4):
            h = ((h ^ ((value >> (8 * i)) & 0xFF)) * 16777619) & 0xFFFFFFFF

    def bits(f):
        return struct.unpack("<I", struct.pack("<f", f))[0]

    for v in (cfg.hidden, cfg.intermediate, cfg.vocab, cfg.heads, cfg.head_dim,
              cfg.window, cfg.conv_width, bits(cfg.eps), bits(cfg.theta),
              bits(cfg.theta_swa)):
        mix(v)
    for i in range(cfg.n_layers):
        mix(cfg.layer_type[i])
        mix(cfg.kv_heads[i])
    return h


def signature(cfg):
    return lfm3.library().lfm3_snapshot_signature(ctypes.byref(cfg))


# Word 7 of every snapshot of the graded geometry (hidden 2048, FFN 8192,
# vocab 65536, 16 heads of 128, window 256, conv width 7, eps 1e-5, theta 1e6 /
# 1e4, layers CCSGCCSGCCSGCCSGCCSGCCGC with 4 KV heads): the golden value of
# the restatement above.
GRADED_SIGNATURE = 0xAD3F27CE


def test_signature_matches_reference_rule():
    assert reference_signature(lfm3.default_config()) == GRADED_SIGNATURE
    for cfg in (lfm3.default_config(), lfm3.small_config(),
                lfm3.small_config(pattern="SGC", kv_heads=1)):
        assert signature(cfg) == reference_signature(cfg)
    assert signature(lfm3.default_config()) == GRADED_SIGNATURE


@pytest.mark.parametrize("field,value", [
    ("intermediate", 7680), ("heads", 32), ("eps", 1e-6), ("theta", 5e5),
    ("theta_swa", 2e4), ("window", 512), ("vocab", 65535)])
def test_signature_covers_every_reference_field(field, value):
    cfg = lfm3.default_config()
    setattr(cfg, field, value)
    assert signature(cfg) != GRADED_SIGNATURE
    assert signature(cfg) == reference_signature(cfg)


def test_signature_ignores_context_and_sees_layers():
    cfg = lfm3.default_config()
    cfg.context = 4096  # header word 2 carries the context, not word 7
    assert signature(cfg) == GRADED_SIGNATURE
    cfg = lfm3.default_config()
    cfg.layer_type[3] = abi.SLIDING_ATTENTION
    assert signature(cfg) != GRADED_SIGNATURE
    cfg = lfm3.default_config()
    cfg.kv_heads[3] = 8
    assert signature(cfg) != GRADED_SIGNATURE


def test_null_config():
    assert lfm3.library().lfm3_snapshot_signature(None) == 0

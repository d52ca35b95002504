"""Python handles on the CPU oracles — TEST INFRASTRUCTURE ONLY.

`Oracle` drives the plain-C restatement (oracle/lfm3_oracle.c, built as
oracle/liboracle.so); `ReferenceOracle` drives the reference's own
reference.cpp compiled unmodified into oracle/_ref/libref_oracle.so (present
only where the reference tree was available at build time). Both follow
Reference::Step (reference.cpp:72-168). Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline legs may import this module.
"""
import ctypes
import importlib
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
RESTATEMENT = os.path.join(HERE, "liboracle.so")
REFERENCE = os.path.join(HERE, "_ref", "libref_oracle.so")

abi = importlib.import_module("lfm3-gufo-extension_b200.abi")


def _load(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"oracle library {path} is not built")
    return ctypes.CDLL(path)


_restatement = None
_reference = None


def restatement_lib():
    global _restatement
    if _restatement is None:
        lib = _load(RESTATEMENT)
        lib.lfm3_oracle_create.argtypes = [
            ctypes.POINTER(abi.Weights), ctypes.c_uint32, ctypes.c_int]
        lib.lfm3_oracle_create.restype = ctypes.c_void_p
        lib.lfm3_oracle_destroy.argtypes = [ctypes.c_void_p]
        lib.lfm3_oracle_reset.argtypes = [ctypes.c_void_p]
        lib.lfm3_oracle_step.argtypes = [
            ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        lib.lfm3_oracle_step.restype = ctypes.c_int
        lib.lfm3_oracle_position.argtypes = [ctypes.c_void_p]
        lib.lfm3_oracle_position.restype = ctypes.c_uint32
        lib.lfm3_oracle_hidden.argtypes = [ctypes.c_void_p]
        lib.lfm3_oracle_hidden.restype = ctypes.POINTER(ctypes.c_float)
        lib.lfm3_oracle_set_kv_half.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.lfm3_oracle_set_kv_half.restype = None
        lib.lfm3_oracle_round_half.argtypes = [ctypes.c_float]
        lib.lfm3_oracle_round_half.restype = ctypes.c_float
        _restatement = lib
    return _restatement


def reference_available():
    return os.path.exists(REFERENCE)


def reference_lib():
    global _reference
    if _reference is None:
        lib = _load(REFERENCE)
        lib.ref_oracle_create.argtypes = [
            ctypes.POINTER(abi.Weights), ctypes.c_uint32, ctypes.c_char_p,
            ctypes.c_size_t]
        lib.ref_oracle_create.restype = ctypes.c_void_p
        lib.ref_oracle_step.argtypes = [
            ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        lib.ref_oracle_step.restype = ctypes.c_int
        lib.ref_oracle_reset.argtypes = [ctypes.c_void_p]
        lib.ref_oracle_position.argtypes = [ctypes.c_void_p]
        lib.ref_oracle_position.restype = ctypes.c_uint32
        lib.ref_oracle_destroy.argtypes = [ctypes.c_void_p]
        _reference = lib
    return _reference


def _synth_lib(prefer_reference):
    """The oracle library whose copy of the synthetic-weight generator to
    use: oracle/_ref when present and preferred, else the restatement's."""
    lib = reference_lib() if prefer_reference and reference_available() \
        else restatement_lib()
    if not getattr(lib, "_synth_declared", False):
        abi.declare_synth(lib)
        lib._synth_declared = True
    return lib


def default_config(prefer_reference=False):
    """The graded geometry (lfm3_synth_default_config), without the CUDA
    library."""
    cfg = abi.Config()
    _synth_lib(prefer_reference).lfm3_synth_default_config(ctypes.byref(cfg))
    return cfg


class SyntheticWeights:
    """Host weights from lfm3_synth_generate (include/lfm3_synth.h) as built
    into an oracle library, for CPU-only runs that must not load the CUDA
    library; the same seed gives the same bytes as the package's
    SyntheticWeights."""

    def __init__(self, config=None, seed=0, matrix_type=abi.Q8_0,
                 norm_jitter=0.0, threads=0, prefer_reference=True):
        self.lib = _synth_lib(prefer_reference)
        self.model = abi.SynthModel()
        cfg = config if config is not None else default_config(prefer_reference)
        rc = self.lib.lfm3_synth_generate(
            ctypes.byref(cfg), seed, matrix_type, norm_jitter, threads,
            ctypes.byref(self.model))
        if rc:
            raise ValueError(f"lfm3_synth_generate failed ({rc})")

    @property
    def weights(self):
        return self.model.weights

    @property
    def config(self):
        return self.model.weights.config

    def close(self):
        if self.model.storage:
            self.lib.lfm3_synth_free(ctypes.byref(self.model))

    __del__ = close


class _Base:
    def __init__(self, weights):
        self.weights = weights  # keep the ctypes struct (and its owner) alive
        self.vocab = weights.config.vocab

    def run(self, tokens, logits_at=None):
        """Steps through tokens; returns {index: logits} for indices in
        logits_at (default: the last token only)."""
        tokens = list(tokens)
        wanted = set(logits_at) if logits_at is not None else {len(tokens) - 1}
        out = {}
        for i, t in enumerate(tokens):
            out_i = self.step(t, i in wanted)
            if out_i is not None:
                out[i] = out_i
        return out

    def greedy(self, prompt, steps):
        """Prompt then `steps` greedy tokens; returns (tokens, logits list)."""
        logits = self.run(prompt)[len(prompt) - 1]
        generated, history = [], [logits]
        for _ in range(steps):
            token = int(np.argmax(logits))
            generated.append(token)
            logits = self.step(token, True)
            history.append(logits)
        return generated, history


class Oracle(_Base):
    """The C restatement (reference.cpp:72-168)."""

    def __init__(self, weights, context, threads=1, kv_half=False):
        super().__init__(weights)
        self.lib = restatement_lib()
        self.handle = self.lib.lfm3_oracle_create(
            ctypes.byref(weights), context, threads)
        if not self.handle:
            raise ValueError("invalid oracle context")
        # test-only: K/V stored through fp16 as the engine's rings hold them
        self.lib.lfm3_oracle_set_kv_half(self.handle, int(kv_half))

    def step(self, token, want_logits=True):
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        ptr = logits.ctypes.data if want_logits else None
        if self.lib.lfm3_oracle_step(self.handle, token, ptr) != 0:
            raise ValueError("invalid oracle step")
        return logits

    def reset(self):
        self.lib.lfm3_oracle_reset(self.handle)

    @property
    def position(self):
        return self.lib.lfm3_oracle_position(self.handle)

    def hidden(self):
        h = self.weights.config.hidden
        return np.ctypeslib.as_array(
            self.lib.lfm3_oracle_hidden(self.handle), (h,)).copy()

    def close(self):
        if self.handle:
            self.lib.lfm3_oracle_destroy(self.handle)
            self.handle = None

    __del__ = close


class ReferenceOracle(_Base):
    """The reference's own reference.cpp, compiled unmodified (oracle/_ref)."""

    def __init__(self, weights, context):
        super().__init__(weights)
        self.lib = reference_lib()
        err = ctypes.create_string_buffer(512)
        self.handle = self.lib.ref_oracle_create(
            ctypes.byref(weights), context, err, 512)
        if not self.handle:
            raise ValueError("reference oracle refused: " + err.value.decode())

    def step(self, token, want_logits=True):
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        ptr = logits.ctypes.data if want_logits else None
        if self.lib.ref_oracle_step(self.handle, token, ptr) != 0:
            raise ValueError("invalid reference step")
        return logits

    def reset(self):
        self.lib.ref_oracle_reset(self.handle)

    @property
    def position(self):
        return self.lib.ref_oracle_position(self.handle)

    def close(self):
        if self.handle:
            self.lib.ref_oracle_destroy(self.handle)
            self.handle = None

    __del__ = close

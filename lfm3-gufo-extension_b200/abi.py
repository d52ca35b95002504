"""ctypes view of the C ABI in include/lfm3_types.h, lfm3_synth.h and lfm3_cuda.h.

The structures mirror the reference's host types (config.hpp:8-20,
weights.hpp:7-26) as declared in include/lfm3_types.h.
"""
import ctypes
import os

MAX_LAYERS = 256
F32, F16, Q8_0, BF16 = 0, 1, 8, 30
CONV, FULL_ATTENTION, SLIDING_ATTENTION = 0, 1, 2

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "lib", "liblfm3_cuda.so")


class Config(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_uint32),
        ("intermediate", ctypes.c_uint32),
        ("vocab", ctypes.c_uint32),
        ("context", ctypes.c_uint32),
        ("heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32),
        ("window", ctypes.c_uint32),
        ("conv_width", ctypes.c_uint32),
        ("n_layers", ctypes.c_uint32),
        ("eps", ctypes.c_float),
        ("theta", ctypes.c_float),
        ("theta_swa", ctypes.c_float),
        ("kv_heads", ctypes.c_uint32 * MAX_LAYERS),
        ("layer_type", ctypes.c_uint32 * MAX_LAYERS),
    ]

    def pattern(self):
        letters = {CONV: "C", FULL_ATTENTION: "G", SLIDING_ATTENTION: "S"}
        return "".join(letters[self.layer_type[i]] for i in range(self.n_layers))


class Tensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("type", ctypes.c_uint32),
        ("cols", ctypes.c_uint32),
        ("rows", ctypes.c_uint32),
        ("bytes", ctypes.c_size_t),
    ]


_LAYER_TENSORS = [
    "norm", "ffn_norm", "post_norm", "post_ffn_norm", "gate", "up", "down",
    "conv", "in_proj", "out_proj", "q", "k", "v", "q_norm", "k_norm",
    "attn_gate", "attn_out",
]


class Layer(ctypes.Structure):
    _fields_ = [(name, Tensor) for name in _LAYER_TENSORS]


class Weights(ctypes.Structure):
    _fields_ = [
        ("config", Config),
        ("embedding", Tensor),
        ("output", Tensor),
        ("output_norm", Tensor),
        ("rope_freqs", Tensor),
        ("layers", Layer * MAX_LAYERS),
    ]


class SynthModel(ctypes.Structure):
    _fields_ = [
        ("weights", Weights),
        ("storage", ctypes.c_void_p),
        ("storage_bytes", ctypes.c_size_t),
    ]


class Input(ctypes.Structure):
    """lfm3_input: a run of token ids or of host embedding rows."""
    _fields_ = [
        ("tokens", ctypes.c_void_p),
        ("n_tokens", ctypes.c_size_t),
        ("rows", ctypes.c_void_p),
        ("n_rows", ctypes.c_size_t),
    ]


HOOK_WRITE = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_uint32,
                              ctypes.c_uint32)
HOOK_EVENT = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p)


class ContinuationHooks(ctypes.Structure):
    """lfm3_continuation_hooks: nonzero from a callback refuses the change."""
    _fields_ = [
        ("user", ctypes.c_void_p),
        ("before_write", HOOK_WRITE),
        ("before_reset", HOOK_EVENT),
        ("before_restore", HOOK_EVENT),
    ]


SAMPLE_MAX_TOP_K = 64
SAMPLE_MAX_RECENT = 64


class Sampler(ctypes.Structure):
    """lfm3_sampler (include/lfm3_cuda.h): temperature 0 selects the largest
    logit; top_k 1..64; repeat_penalty 1 disables the penalty."""
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_uint32),
        ("repeat_penalty", ctypes.c_float),
    ]


class StepStats(ctypes.Structure):
    """lfm3_step_stats: what one scheduler step ran."""
    _fields_ = [
        ("pass_request", ctypes.c_int32),
        ("pass_rows", ctypes.c_uint32),
        ("round_rows", ctypes.c_uint32),
        ("finished", ctypes.c_uint32),
        ("pass_ms", ctypes.c_double),
        ("round_ms", ctypes.c_double),
    ]


def declare_synth(lib):
    """Argument types of the lfm3_synth_* entry points (include/lfm3_synth.h)."""
    lib.lfm3_synth_default_config.argtypes = [ctypes.POINTER(Config)]
    lib.lfm3_synth_default_config.restype = None
    lib.lfm3_synth_set_layers.argtypes = [
        ctypes.POINTER(Config), ctypes.c_char_p, ctypes.c_uint32]
    lib.lfm3_synth_set_layers.restype = ctypes.c_int
    lib.lfm3_synth_generate.argtypes = [
        ctypes.POINTER(Config), ctypes.c_uint64, ctypes.c_uint32, ctypes.c_float,
        ctypes.c_int, ctypes.POINTER(SynthModel)]
    lib.lfm3_synth_generate.restype = ctypes.c_int
    lib.lfm3_synth_free.argtypes = [ctypes.POINTER(SynthModel)]
    lib.lfm3_synth_free.restype = None
    lib.lfm3_row_bytes.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    lib.lfm3_row_bytes.restype = ctypes.c_size_t
    lib.lfm3_float_to_half.argtypes = [ctypes.c_float]
    lib.lfm3_float_to_half.restype = ctypes.c_uint16
    lib.lfm3_half_to_float.argtypes = [ctypes.c_uint16]
    lib.lfm3_half_to_float.restype = ctypes.c_float

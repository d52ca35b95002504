"""B200-native LFM3 backbone step (sm_100a).

Python handle on liblfm3_cuda.so (include/lfm3_cuda.h): the engine (Model /
Session, the reference's engine.hpp) and the synthetic-weight generator. The
kernels and the engine are native; this module only declares the C ABI and
wraps host buffers. It fails loudly when the library is missing: there is no
other implementation to fall back to.

Import with importlib (the directory name is not an identifier):

    lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
"""
import ctypes
import importlib
import os

import numpy as np

abi = importlib.import_module(__name__ + ".abi")

_lib = None


class Lfm3Error(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"LFM3 error {code}: {message}")
        self.code = code


def library():
    """Loads lib/liblfm3_cuda.so once (raises if it was never built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(abi.LIBRARY):
        raise FileNotFoundError(
            f"{abi.LIBRARY} is not built: run build.py in the package")
    lib = ctypes.CDLL(abi.LIBRARY)
    abi.declare_synth(lib)
    P, I, U32, SZ, F = (ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32,
                        ctypes.c_size_t, ctypes.c_float)
    sigs = {
        "lfm3_last_error": ([], ctypes.c_char_p),
        "lfm3_cuda_take_device_error": ([], ctypes.c_uint),
        "lfm3_cuda_wait_probe": ([U32, P], I),
        "lfm3_cuda_dense_workspace_bytes": ([SZ, SZ], SZ),
        "lfm3_cuda_split_partial_bytes": ([], SZ),
        "lfm3_cuda_split_ticket_words": ([], SZ),
        "lfm3_cuda_prompt_rows": ([], I),
        "lfm3_cuda_embed": ([P, P, P, I, P], I),
        "lfm3_cuda_dense": ([P, P, P, I, P, P], I),
        "lfm3_cuda_project": ([P, I, P, I, P, P, I], I),
        "lfm3_cuda_project_swiglu": ([P, P, P, P, P, I, P, P, I], I),
        "lfm3_cuda_project_ffn": ([P, P, P, P, P, P, P, I, P, P, I], I),
        "lfm3_cuda_residual_norm": ([P, P, P, P, P, I, I, F, I, P, P], I),
        "lfm3_cuda_short_conv": ([P, P, P, P, I, I, I, P, I], I),
        "lfm3_cuda_rope_frequencies": ([P, I, F, P], I),
        "lfm3_cuda_rope": ([P, P, P, I, I, I, I, P], I),
        "lfm3_cuda_attention": ([P, P, P, P, P, P, P, I, I, I, I, I, I, I, P,
                                 P], I),
        "lfm3_cuda_attention_stored": ([P, P, P, P, P, I, I, I, I, I, I, P,
                                        P], I),
        "lfm3_cuda_attention_scratch_bytes": ([I, I, I, I], SZ),
        "lfm3_cuda_attention_decode_noalloc": ([P, P, P, P, P, P, P, I, I, I,
                                                I, I, I, P], I),
        "lfm3_cuda_prompt_heads": ([P, P, P, P, P, P, P, P, P, I, I, I, I, I,
                                    F, P], I),
        "lfm3_cuda_decode_heads": ([P, P, P, P, P, P, P, P, P, I, I, I, I, I,
                                    F, P], I),
        "lfm3_cuda_store_kv": ([P, P, P, P, I, I, I, I, P], I),
        "lfm3_cuda_pack_kv": ([P, P, P, P, SZ, P], I),
        "lfm3_cuda_select_rows": ([P, P, P, I, P], I),
        "lfm3_cuda_batched_rmsnorm": ([P, P, P, P, SZ, SZ, F, P], I),
        "lfm3_model_load": ([ctypes.POINTER(abi.Weights)], P),
        "lfm3_model_free": ([P], None),
        "lfm3_model_config": ([P, ctypes.POINTER(abi.Config)], I),
        "lfm3_model_weight_bytes": ([P], SZ),
        "lfm3_session_create": ([P, U32], P),
        "lfm3_session_free": ([P], None),
        "lfm3_session_forward": ([P, P, SZ, P], I),
        "lfm3_session_forward_batch": ([P, P, SZ, P], I),
        "lfm3_session_forward_batch_inputs": ([P, P, P, SZ, I], I),
        "lfm3_session_read_logits": ([P, P], I),
        "lfm3_session_read_hidden": ([P, P], I),
        "lfm3_session_reset": ([P], I),
        "lfm3_session_position": ([P], U32),
        "lfm3_session_is_coherent": ([P], I),
        "lfm3_session_stream": ([P], P),
        "lfm3_session_continuation_data": ([P, I, SZ], P),
        "lfm3_session_ring_capacity": ([P, SZ], U32),
        "lfm3_session_snapshot_bytes": ([P], SZ),
        "lfm3_snapshot_signature": ([ctypes.POINTER(abi.Config)], U32),
        "lfm3_session_save_snapshot": ([P, P, SZ], I),
        "lfm3_session_restore_snapshot": ([P, P, SZ], I),
        "lfm3_session_inject_failure": ([P, I], I),
        "lfm3_session_set_profiling": ([P, I], I),
        "lfm3_session_take_profile": ([P, P, P], I),
        "lfm3_cuda_launch_count": ([], ctypes.c_ulonglong),
        "lfm3_session_forward_embeddings": ([P, P, SZ, I, P], I),
        "lfm3_session_forward_inputs": ([P, ctypes.POINTER(abi.Input), SZ, P], I),
        "lfm3_session_speculate": ([P, U32], I),
        "lfm3_session_forward_decision": ([P, P, SZ, P], I),
        "lfm3_session_set_continuation_hooks": (
            [P, ctypes.POINTER(abi.ContinuationHooks)], I),
        "lfm3_session_prepare_logits": ([P], I),
        "lfm3_session_begin_restore": ([P], I),
        "lfm3_session_finish_restore": ([P, U32], I),
        "lfm3_cuda_shares_split": ([P, I, I, P], I),
        "lfm3_cuda_batched_residual_add": ([P, P, P, SZ, SZ, P], I),
        "lfm3_cuda_gemv": ([P, U32, P, P, SZ, SZ, P], I),
        "lfm3_cuda_decode_workspace_bytes": ([P, I, I], SZ),
        "lfm3_cuda_decode_project": ([P, I, I, P, I, P, P, P, P], I),
        "lfm3_cuda_batched_quant_gemm_fp32": ([U32, P, P, P, SZ, SZ, SZ, P], I),
        "lfm3_cuda_exact_bf16_gemm_fp32_small_batch": ([P, P, P, SZ, SZ, SZ, P], I),
        "lfm3_cuda_sample_scratch_bytes": ([I, I, I], SZ),
        "lfm3_cuda_sample": ([P, I, I, I, ctypes.POINTER(abi.Sampler), P, P,
                              P, P, P, P], I),
        "lfm3_sample_host": ([P, I, I, I, ctypes.POINTER(abi.Sampler), P, P,
                              P, P], I),
        "lfm3_session_forward_batch_sample": ([P, P, SZ,
                                               ctypes.POINTER(abi.Sampler),
                                               P, P, P, P], I),
        "lfm3_scheduler_create": ([P, ctypes.POINTER(abi.Sampler)], P),
        "lfm3_scheduler_free": ([P], None),
        "lfm3_scheduler_admit": ([P, P, SZ, U32, ctypes.c_uint64, U32], I),
        "lfm3_scheduler_step": ([P, ctypes.POINTER(abi.StepStats)], I),
        "lfm3_scheduler_idle": ([P], I),
        "lfm3_scheduler_tokens": ([P, I, P, SZ], SZ),
        "lfm3_scheduler_finished": ([P, I], I),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def launch_count():
    """Kernels this library has launched in this process."""
    return int(library().lfm3_cuda_launch_count())


def check(code):
    """Raises Lfm3Error for a nonzero status of the C ABI."""
    if code != 0:
        raise Lfm3Error(code, library().lfm3_last_error().decode())
    return code


def _ptr(array):
    return ctypes.c_void_p(array.ctypes.data) if array is not None else None


# ---- token selection -------------------------------------------------------------

def sampler(temperature=0.1, top_k=50, repeat_penalty=1.1):
    """lfm3_sampler; the defaults are the reference runner's (runner.cpp:31-35)."""
    return abi.Sampler(float(temperature), int(top_k), float(repeat_penalty))


def sample_tables(rows, recent=None, seeds=None):
    """Host tables of lfm3_sampler's rows: recent[r] (a sequence of at most 64
    tokens; only its distinct values matter) and seeds[r] (uint64)."""
    table = np.zeros((rows, abi.SAMPLE_MAX_RECENT), np.uint32)
    count = np.zeros(rows, np.uint32)
    for r, toks in enumerate(recent or []):
        toks = np.asarray(toks, dtype=np.uint32)[-abi.SAMPLE_MAX_RECENT:]
        table[r, :toks.size] = toks
        count[r] = toks.size
    seed = np.zeros(rows, np.uint64)
    if seeds is not None:
        seed[:] = np.asarray(seeds, dtype=np.uint64)
    return table, count, seed


def sample_host(logits, sampler_, recent=None, seeds=None):
    """lfm3_sample_host over host logits [rows][vocab]: the selected tokens."""
    x = np.ascontiguousarray(np.atleast_2d(np.asarray(logits, np.float32)))
    rows, vocab = x.shape
    table, count, seed = sample_tables(rows, recent, seeds)
    out = np.zeros(rows, np.uint32)
    check(library().lfm3_sample_host(
        _ptr(x), rows, vocab, vocab, ctypes.byref(sampler_), _ptr(table),
        _ptr(count), _ptr(seed), _ptr(out)))
    return out


# ---- synthetic weights -----------------------------------------------------------

def default_config():
    cfg = abi.Config()
    library().lfm3_synth_default_config(ctypes.byref(cfg))
    return cfg


def small_config(hidden=512, intermediate=1024, vocab=1024, heads=4, kv_heads=2,
                 window=32, context=4096, pattern="CSGCSG"):
    """A small geometry of the same architecture, for fast tests."""
    cfg = default_config()
    cfg.hidden, cfg.intermediate, cfg.vocab = hidden, intermediate, vocab
    cfg.heads, cfg.window, cfg.context = heads, window, context
    if library().lfm3_synth_set_layers(ctypes.byref(cfg), pattern.encode(),
                                       kv_heads):
        raise ValueError("invalid layer pattern " + pattern)
    return cfg


class SyntheticWeights:
    """Host weights from lfm3_synth_generate (freed with the object)."""

    def __init__(self, config=None, seed=0, matrix_type=abi.Q8_0,
                 norm_jitter=0.0, threads=0):
        self.model = abi.SynthModel()
        cfg = config if config is not None else default_config()
        rc = library().lfm3_synth_generate(
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
        if _lib is not None and self.model.storage:
            _lib.lfm3_synth_free(ctypes.byref(self.model))

    def __del__(self):
        self.close()


# ---- engine --------------------------------------------------------------------------

class Model:
    """Model::Load (engine.hpp:27-30): weights copied to the current device."""

    def __init__(self, weights):
        lib = library()
        self._weights = weights  # the host copy must outlive nothing here
        # bound now: at interpreter exit the module's globals may be gone
        self._free = lib.lfm3_model_free
        self.handle = lib.lfm3_model_load(ctypes.byref(weights))
        if not self.handle:
            raise Lfm3Error(-1, lib.lfm3_last_error().decode())
        self.config = abi.Config()
        check(lib.lfm3_model_config(self.handle, ctypes.byref(self.config)))

    @property
    def weight_bytes(self):
        return library().lfm3_model_weight_bytes(self.handle)

    def session(self, context):
        return Session(self, context)

    def close(self):
        if getattr(self, "handle", None):
            self._free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class Scheduler:
    """lfm3_scheduler: continuous batching of requests on one model (one
    <=512-row prompt pass, first come first served, then one decode round of
    up to 8 requests with device token selection, per step)."""

    def __init__(self, model, sampler_):
        lib = library()
        self.model = model
        self._free = lib.lfm3_scheduler_free
        self._sampler = sampler_
        self.handle = lib.lfm3_scheduler_create(model.handle, ctypes.byref(sampler_))
        if not self.handle:
            raise Lfm3Error(-1, lib.lfm3_last_error().decode())

    def admit(self, prompt, max_new, seed, context):
        toks = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        rc = library().lfm3_scheduler_admit(self.handle, _ptr(toks), toks.size,
                                            int(max_new), int(seed), int(context))
        if rc < 0:
            check(rc)
        return rc

    def step(self):
        st = abi.StepStats()
        check(library().lfm3_scheduler_step(self.handle, ctypes.byref(st)))
        return st

    @property
    def idle(self):
        return bool(library().lfm3_scheduler_idle(self.handle))

    def tokens(self, request):
        lib = library()
        n = lib.lfm3_scheduler_tokens(self.handle, request, None, 0)
        out = np.zeros(n, np.uint32)
        lib.lfm3_scheduler_tokens(self.handle, request, _ptr(out), n)
        return out

    def finished(self, request):
        return library().lfm3_scheduler_finished(self.handle, request)

    def close(self):
        if getattr(self, "handle", None):
            self._free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class Session:
    """Session (engine.hpp:46-163)."""

    PREFILL_CHUNK = 512
    MAX_BATCH = 8

    def __init__(self, model, context):
        lib = library()
        self.model = model
        self.vocab = model.config.vocab
        self.hidden = model.config.hidden
        self._free = lib.lfm3_session_free  # see Model.__init__
        self.handle = lib.lfm3_session_create(model.handle, context)
        if not self.handle:
            raise Lfm3Error(-1, lib.lfm3_last_error().decode())

    def forward(self, tokens, logits=True, out=None):
        """Advances tokens; returns the last row's logits (or None)."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if logits and out is None:
            out = np.empty(self.vocab, np.float32)
        check(library().lfm3_session_forward(
            self.handle, _ptr(toks), toks.size, _ptr(out) if logits else None))
        return out if logits else None

    @staticmethod
    def forward_batch(sessions, tokens, logits=True, outs=None):
        """One token per session (ForwardBatch); returns a list of logits."""
        lib = library()
        n = len(sessions)
        handles = (ctypes.c_void_p * n)(*[s.handle for s in sessions])
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if logits and outs is None:
            outs = [np.empty(s.vocab, np.float32) for s in sessions]
        ptrs = ((ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
                if logits else None)
        check(lib.lfm3_session_forward_batch(handles, _ptr(toks), n, ptrs))
        return outs if logits else None

    @staticmethod
    def forward_batch_sample(sessions, tokens, sampler_, recent=None,
                             seeds=None):
        """ForwardBatch followed by token selection on the device: returns
        the selected token of each session (uint32 array)."""
        n = len(sessions)
        handles = (ctypes.c_void_p * n)(*[s.handle for s in sessions])
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        table, count, seed = sample_tables(n, recent, seeds)
        out = np.zeros(n, np.uint32)
        check(library().lfm3_session_forward_batch_sample(
            handles, _ptr(toks), n, ctypes.byref(sampler_), _ptr(table),
            _ptr(count), _ptr(seed), _ptr(out)))
        return out

    @staticmethod
    def forward_batch_inputs(sessions, tokens, logits=True, rows=None):
        """ForwardBatchInputs: one token per session, logits left on the
        device; rows[i], when given and not None, is the device address of
        session i's input embedding row (used instead of tokens[i])."""
        n = len(sessions)
        handles = (ctypes.c_void_p * n)(*[s.handle for s in sessions])
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        ptrs = (ctypes.c_void_p * n)(*rows) if rows is not None else None
        check(library().lfm3_session_forward_batch_inputs(
            handles, _ptr(toks), ptrs, n, int(bool(logits))))

    def forward_embeddings(self, rows, logits=True, device_rows=None):
        """ForwardEmbeddings: host rows (float32 [n][hidden]), or with
        device_rows=(address, n) rows in device memory; returns the last
        row's logits (or None)."""
        out = np.empty(self.vocab, np.float32) if logits else None
        if device_rows is not None:
            address, n = device_rows
            check(library().lfm3_session_forward_embeddings(
                self.handle, ctypes.c_void_p(address), n, 1, _ptr(out)))
        else:
            x = np.ascontiguousarray(np.asarray(rows, np.float32))
            check(library().lfm3_session_forward_embeddings(
                self.handle, _ptr(x), x.size // self.hidden, 0, _ptr(out)))
        return out

    def forward_inputs(self, runs, logits=True):
        """ForwardInputs over runs [("tokens", ids) | ("rows", floats
        [n][hidden])]; returns the last row's logits (or None)."""
        keep, structs = [], []
        for kind, data in runs:
            if kind == "tokens":
                a = np.ascontiguousarray(np.asarray(data, np.uint32))
                structs.append(abi.Input(a.ctypes.data, a.size, None, 0))
            else:
                a = np.ascontiguousarray(np.asarray(data, np.float32))
                structs.append(abi.Input(None, 0, a.ctypes.data,
                                         a.size // self.hidden))
            keep.append(a)
        arr = (abi.Input * len(structs))(*structs)
        out = np.empty(self.vocab, np.float32) if logits else None
        check(library().lfm3_session_forward_inputs(
            self.handle, arr, len(structs), _ptr(out)))
        return out

    def set_continuation_hooks(self, before_write=None, before_reset=None,
                               before_restore=None):
        """Installs Python callables as ContinuationHooks (a truthy return
        refuses the change); no arguments removes them."""
        lib = library()
        if before_write is None and before_reset is None and before_restore is None:
            self._hooks = None
            check(lib.lfm3_session_set_continuation_hooks(self.handle, None))
            return
        h = abi.ContinuationHooks(
            None,
            abi.HOOK_WRITE(lambda u, a, b: int(bool(before_write and before_write(a, b)))),
            abi.HOOK_EVENT(lambda u: int(bool(before_reset and before_reset()))),
            abi.HOOK_EVENT(lambda u: int(bool(before_restore and before_restore()))))
        self._hooks = h  # the callbacks must outlive the session's use of them
        check(lib.lfm3_session_set_continuation_hooks(self.handle, ctypes.byref(h)))

    def prepare_logits(self):
        check(library().lfm3_session_prepare_logits(self.handle))

    def begin_restore(self):
        check(library().lfm3_session_begin_restore(self.handle))

    def finish_restore(self, position):
        check(library().lfm3_session_finish_restore(self.handle, position))

    def speculate(self, token):
        check(library().lfm3_session_speculate(self.handle, token))

    def read_logits(self):
        out = np.empty(self.vocab, np.float32)
        check(library().lfm3_session_read_logits(self.handle, _ptr(out)))
        return out

    def read_hidden(self):
        out = np.empty(self.hidden, np.float32)
        check(library().lfm3_session_read_hidden(self.handle, _ptr(out)))
        return out

    def reset(self):
        check(library().lfm3_session_reset(self.handle))

    @property
    def position(self):
        return library().lfm3_session_position(self.handle)

    @property
    def coherent(self):
        return bool(library().lfm3_session_is_coherent(self.handle))

    @property
    def stream(self):
        return library().lfm3_session_stream(self.handle)

    def continuation_data(self, tensor, layer=0):
        return library().lfm3_session_continuation_data(self.handle, tensor,
                                                        layer)

    def ring_capacity(self, layer):
        return library().lfm3_session_ring_capacity(self.handle, layer)

    def save_snapshot(self):
        lib = library()
        n = lib.lfm3_session_snapshot_bytes(self.handle)
        buf = np.empty(n, np.uint8)
        check(lib.lfm3_session_save_snapshot(self.handle, _ptr(buf), n))
        return buf

    def restore_snapshot(self, payload):
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        check(library().lfm3_session_restore_snapshot(
            self.handle, _ptr(payload), payload.size))

    PROFILE_CLASSES = ("decode_projection", "decode_attention", "row_kernels",
                       "prompt_projection", "prompt_attention", "prompt_other")

    def set_profiling(self, on):
        check(library().lfm3_session_set_profiling(self.handle, int(bool(on))))

    def take_profile(self):
        """{class: (milliseconds, launches)} since the last call."""
        ms = np.zeros(6, np.float64)
        n = np.zeros(6, np.int64)
        check(library().lfm3_session_take_profile(self.handle, _ptr(ms), _ptr(n)))
        return {c: (float(ms[i]), int(n[i])) for i, c in enumerate(self.PROFILE_CLASSES)}

    def inject_failure(self, after_calls):
        check(library().lfm3_session_inject_failure(self.handle, after_calls))

    def close(self):
        if getattr(self, "handle", None):
            self._free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

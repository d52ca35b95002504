"""lfm3_cuda_attention_decode_noalloc, the decode attention entry point for
callers that cannot allocate device memory (a fixed serving arena, or a
thread that must not call cudaMalloc between steps), against the existing
entry point lfm3_cuda_attention with a caller-provided scratch buffer.

Two calls in a row with different shapes and depths: the second must not
see anything the first left in the shared static scratch. The file is named
to be collected last; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from helpers import lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu



def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def inputs(rng, heads, kv_heads, position, capacity):
    stride = kv_heads * 128
    q = torch.from_numpy(rng.normal(0, 0.7, heads * 128).astype(np.float32)).cuda()
    gate = torch.from_numpy(rng.normal(0, 0.7, heads).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.normal(0, 0.5, stride).astype(np.float16)).cuda()
    v = torch.from_numpy(rng.normal(0, 0.9, stride).astype(np.float16)).cuda()
    ck = torch.from_numpy(rng.normal(0, 0.6, capacity * stride).astype(np.float16)).cuda()
    cv = torch.from_numpy(rng.normal(0, 0.8, capacity * stride).astype(np.float16)).cuda()
    return q, gate, k, v, ck, cv


@pytest.mark.parametrize("calls", [[(16, 4, 4999, 0), (4, 2, 300, 256)]])
def test_noalloc_matches_scratch_entry_point(calls):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = lfm3.library()
    rng = np.random.default_rng(123)
    for heads, kv_heads, position, window in calls:
        capacity = window if window else position + 1
        q, gate, k, v, ck, cv = inputs(rng, heads, kv_heads, position, capacity)
        want = torch.empty(heads * 128, dtype=torch.float32, device="cuda")
        got = torch.full_like(want, float("nan"))
        scratch = torch.empty(
            lib.lfm3_cuda_attention_scratch_bytes(heads, 128, position + 1, 1) // 4 + 1,
            dtype=torch.float32, device="cuda")
        lfm3.check(lib.lfm3_cuda_attention(
            ptr(q), ptr(k), ptr(v), ptr(gate), ptr(ck), ptr(cv), ptr(want), 1, heads,
            kv_heads, 128, position, capacity, window, None, ptr(scratch)))
        lfm3.check(lib.lfm3_cuda_attention_decode_noalloc(
            ptr(q), ptr(k), ptr(v), ptr(gate), ptr(ck), ptr(cv), ptr(got), heads,
            kv_heads, 128, position, capacity, window, None))
        torch.cuda.synchronize()
        a, b = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(a).all()
        # the same kernel with the same span plan (kMaxDecodeSplits spans of
        # the row's keys): the same bits
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_noalloc_refuses_more_heads_than_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = lfm3.library()
    x = torch.zeros(64 * 128, dtype=torch.float32, device="cuda")
    h = torch.zeros(64 * 128, dtype=torch.float16, device="cuda")
    rc = lib.lfm3_cuda_attention_decode_noalloc(
        ptr(x), ptr(h), ptr(h), ptr(x), ptr(h), ptr(h), ptr(x), 64, 8, 128, 0, 1, 0,
        None)
    assert rc == -3
    assert b"32 query heads" in lib.lfm3_last_error()

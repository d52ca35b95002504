"""The full-attention prompt kernel on the tcgen05 tensor cores
(lfm3_cuda_attention_stored, csrc/attention_prompt_tc.cu) against the same
FP64 formula as the attention known-answer tests (tests/ops_test.cpp:148-220:
causal gated GQA attention over the rounded F16 keys and values), and
against the mma.sync prompt kernel of lfm3_cuda_attention, which rounds Q
and the probabilities to FP16 the same way. The chunk is stored into the
cache first, as the engine packs full-attention rows in place."""
import ctypes

import numpy as np
import pytest

from helpers import lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

D = 128
lib = None


def setup_module(module):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    global lib
    lib = lfm3.library()


def data(n, scale, phase=0.0):
    i = np.arange(n, dtype=np.float32)
    return (np.float32(scale) * np.sin(i * np.float32(0.73) + np.float32(phase))
            ).astype(np.float32)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def expected(q, ck, cv, gates, n, H, KH, P):
    """FP64 attention of rows P .. P + n - 1 over cache keys 0 .. row."""
    G = H // KH
    qq = q.reshape(n, H, D).astype(np.float64)
    kk = ck[:(P + n) * KH * D].reshape(P + n, KH, D).astype(np.float64)
    vv = cv[:(P + n) * KH * D].reshape(P + n, KH, D).astype(np.float64)
    out = np.zeros((n, H, D))
    g = gates.reshape(n, H).astype(np.float64)
    for h in range(H):
        s = qq[:, h] @ kk[:, h // G].T / np.sqrt(D)  # [n][keys]
        s[np.arange(P + n)[None, :] > (P + np.arange(n))[:, None]] = -np.inf
        s = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h] = (s / s.sum(axis=1, keepdims=True)) @ vv[:, h // G]
        out[:, h] /= (1 + np.exp(-g[:, h]))[:, None]
    return out


def run(n, P, H, KH, poison_tail=False):
    capacity = P + n + 77
    stride = KH * D
    q, gates = data(n * H * D, 0.7), data(n * H, 0.7, 1.0)
    k16 = data(capacity * stride, 0.5, 2.0).astype(np.float16)
    v16 = data(capacity * stride, 0.9, 3.0).astype(np.float16)
    if poison_tail:  # slots the pass has not written hold NaN
        k16[(P + n) * stride:] = np.float16(np.nan)
        v16[(P + n) * stride:] = np.float16(np.nan)
    want = expected(q, k16.astype(np.float64), v16.astype(np.float64), gates, n,
                    H, KH, P)
    dq = torch.from_numpy(q).cuda()
    dg = torch.from_numpy(gates).cuda()
    ck = torch.from_numpy(k16.view(np.int16)).cuda()
    cv = torch.from_numpy(v16.view(np.int16)).cuda()
    scratch = torch.empty(
        lib.lfm3_cuda_attention_scratch_bytes(H, D, P + n, n) // 4 + 1,
        dtype=torch.float32, device="cuda")
    out = torch.full((n * H * D,), float("nan"), dtype=torch.float32,
                     device="cuda")
    lfm3.check(lib.lfm3_cuda_attention_stored(
        ptr(dq), ptr(dg), ptr(ck), ptr(cv), ptr(out), n, H, KH, D, P, capacity,
        None, ptr(scratch)))
    # the mma.sync kernel on the same keys, the chunk passed separately
    chunk_k = ck[P * stride:(P + n) * stride].clone()
    chunk_v = cv[P * stride:(P + n) * stride].clone()
    ref = torch.empty_like(out)
    lfm3.check(lib.lfm3_cuda_attention(
        ptr(dq), ptr(chunk_k), ptr(chunk_v), ptr(dg), ptr(ck), ptr(cv),
        ptr(ref), n, H, KH, D, P, capacity, 0, None, ptr(scratch)))
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(n, H, D).astype(np.float64)
    other = ref.cpu().numpy().reshape(n, H, D).astype(np.float64)
    assert np.isfinite(got).all()
    err = np.abs(got - want).max()
    assert err <= 1e-3, err  # the operator tests' prompt tolerance
    assert np.abs(got - other).max() <= 5e-4
    return err


@pytest.mark.parametrize("n", [1, 8, 33, 64, 65, 128, 200, 512])
def test_group2(n):
    run(n, 259, 4, 2)


@pytest.mark.parametrize("n,P", [(512, 0), (77, 3000), (512, 3000), (129, 1)])
def test_model_heads(n, P):
    run(n, P, 16, 4)


@pytest.mark.parametrize("n", [31, 256])
def test_group8(n):
    run(n, 1000, 16, 2)


def test_spans_over_long_history():
    run(40, 17000, 4, 2)
    run(512, 9000, 16, 4)


def test_unwritten_slots_do_not_leak():
    run(100, 50, 16, 4, poison_tail=True)
    run(512, 0, 16, 4, poison_tail=True)


def test_refusals():
    assert lib.lfm3_cuda_attention_stored(None, None, None, None, None, 1, 4, 2,
                                          64, 0, 8, None, None) == -3
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    p = ptr(dummy)
    # position + n beyond the capacity (the keys would wrap)
    assert lib.lfm3_cuda_attention_stored(p, p, p, p, p, 8, 4, 2, 128, 4, 10,
                                          None, p) == -1

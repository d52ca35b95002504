"""Operator known-answer tests on the GPU, ported case for case from the
reference's tests/ops_test.cpp: every operator against an independent FP64
formula, through the C ABI (include/lfm3_cuda.h), with the reference's
tolerances. Device memory comes from torch (plumbing only)."""
import ctypes

import numpy as np
import pytest

from helpers import abi, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

lib = None


def setup_module(module):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    global lib
    lib = lfm3.library()


def data(n, scale=0.1):
    """Data (tests/ops_test.cpp:30-35): scale * sin(0.73 i) in FP32."""
    i = np.arange(n, dtype=np.float32)
    return (np.float32(scale) * np.sin(i * np.float32(0.73))).astype(np.float32)


def dev(array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def near(got, want, limit):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    err = np.abs(got - want)
    assert err.max() <= limit, (float(err.max()), int(err.argmax()))


def workspace(rows, K):
    q = torch.empty(lib.lfm3_cuda_dense_workspace_bytes(rows, K) // 4 + 1,
                    dtype=torch.float32, device="cuda")
    rm = torch.zeros(max(rows, 1), dtype=torch.int32, device="cuda")
    part = torch.empty(lib.lfm3_cuda_split_partial_bytes() // 4,
                       dtype=torch.float32, device="cuda")
    tick = torch.zeros(lib.lfm3_cuda_split_ticket_words(), dtype=torch.int32,
                       device="cuda")
    ws = lfm3.abi  # noqa: F841
    struct = WorkspaceStruct(ptr(q), ptr(rm), ptr(part), ptr(tick))
    return struct, (q, rm, part, tick)


class WorkspaceStruct(ctypes.Structure):
    _fields_ = [("quantized", ctypes.c_void_p), ("row_max", ctypes.c_void_p),
                ("partial", ctypes.c_void_p), ("tickets", ctypes.c_void_p)]


def q8_tensor(blocks_bytes, cols, rows):
    buf = dev(np.frombuffer(blocks_bytes, np.uint8).copy())
    t = abi.Tensor(buf.data_ptr(), abi.Q8_0, cols, rows, len(blocks_bytes))
    return t, buf


def round16(x):
    return x.astype(np.float16).astype(np.float32)


# ---- Projection (tests/ops_test.cpp:46-89) ------------------------------------
@pytest.mark.parametrize("n", [1, 8, 9, 15, 16, 29, 32, 33, 128, 512])
def test_projection(n):
    M, K = 37, 2048
    nb = M * K // 32
    i = np.arange(nb)
    d = (0x2400 + 32 * (i % 10)).astype(np.uint16)
    j = np.arange(32)
    qs = ((i[:, None] * 17 + j[None, :] * 37) % 255 - 127).astype(np.int8)
    blocks = np.zeros((nb, 34), np.uint8)
    blocks[:, :2] = d.view(np.uint8).reshape(nb, 2)
    blocks[:, 2:] = qs.view(np.uint8)
    x = data(n * K, 0.07).reshape(n, K)
    inputs = x.copy()
    if n >= lib.lfm3_cuda_prompt_rows():
        for r in range(n):
            e = 14 - int(np.floor(np.log2(np.abs(x[r]).max())))
            inputs[r] = np.ldexp(np.ldexp(x[r], e).astype(np.float16)
                                 .astype(np.float32), -e)
    w = (d.view(np.float16).astype(np.float64)[:, None] * qs).reshape(M, K)
    expected = inputs.astype(np.float64) @ w.T
    t, keep = q8_tensor(blocks.tobytes(), K, M)
    dx, out = dev(x), torch.empty(n * M, dtype=torch.float32, device="cuda")
    ws, keep2 = workspace(n, K)
    lfm3.check(lib.lfm3_cuda_dense(ctypes.byref(t), ptr(dx), ptr(out), n, None,
                                   ctypes.byref(ws)))
    near(host(out).reshape(n, M), expected, 1e-4)


@pytest.mark.parametrize("n", [1, 5, 8])
def test_projection_tall(n):
    """Decode projections of matrices tall enough for 64-row tiles (more than
    four per SM), with a ragged last tile."""
    M, K = 4 * 148 * 64 + 37, 512
    nb = M * K // 32
    i = np.arange(nb)
    d = (0x2400 + 32 * (i % 10)).astype(np.uint16)
    j = np.arange(32)
    qs = ((i[:, None] * 17 + j[None, :] * 37) % 255 - 127).astype(np.int8)
    blocks = np.zeros((nb, 34), np.uint8)
    blocks[:, :2] = d.view(np.uint8).reshape(nb, 2)
    blocks[:, 2:] = qs.view(np.uint8)
    x = data(n * K, 0.07).reshape(n, K)
    w = (d.view(np.float16).astype(np.float64)[:, None] * qs).reshape(M, K)
    expected = x.astype(np.float64) @ w.T
    t, keep = q8_tensor(blocks.tobytes(), K, M)
    dx, out = dev(x), torch.empty(n * M, dtype=torch.float32, device="cuda")
    ws, keep2 = workspace(n, K)
    lfm3.check(lib.lfm3_cuda_dense(ctypes.byref(t), ptr(dx), ptr(out), n, None,
                                   ctypes.byref(ws)))
    near(host(out).reshape(n, M), expected, 1e-4)


# ---- BF16 projections (exact BF16 x FP32, hip/ops.hip:1917-2005) ---------------
def bf16_tensor(w32, cols, rows):
    """BF16 matrix [rows][cols] from FP32 values (round to nearest even)."""
    bits = w32.astype(np.float32).view(np.uint32)
    bf = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    buf = dev(bf.copy())
    t = abi.Tensor(buf.data_ptr(), abi.BF16, cols, rows, bf.nbytes)
    exact = (bf.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return t, buf, exact.reshape(rows, cols)


@pytest.mark.parametrize("n", [1, 8, 9, 16, 37, 512])
def test_projection_bf16(n):
    M, K = 70, 512 + 256
    w32 = data(M * K, 0.05).reshape(M, K)
    t, keep, w = bf16_tensor(w32, K, M)
    x = data(n * K, 0.3).reshape(n, K) + np.float32(0.01)
    expected = x.astype(np.float64) @ w.T
    dx, out = dev(x), torch.empty(n * M, dtype=torch.float32, device="cuda")
    ws, keep2 = workspace(n, K)
    lfm3.check(lib.lfm3_cuda_dense(ctypes.byref(t), ptr(dx), ptr(out), n, None,
                                   ctypes.byref(ws)))
    near(host(out).reshape(n, M), expected, 2e-5)


@pytest.mark.parametrize("n", [1, 8, 20])
def test_ffn_bf16(n):
    H, F = 256, 512
    gw, keep_g, g64 = bf16_tensor(data(F * H, 0.06).reshape(F, H), H, F)
    uw, keep_u, u64 = bf16_tensor(data(F * H, 0.05).reshape(F, H) * -1, H, F)
    dw, keep_d, d64 = bf16_tensor(data(H * F, 0.04).reshape(H, F), F, H)
    x = data(n * H, 0.5).reshape(n, H)
    g = x.astype(np.float64) @ g64.T
    u = x.astype(np.float64) @ u64.T
    hidden = g / (1 + np.exp(-g)) * u
    expected = hidden @ d64.T
    dx = dev(x)
    h = torch.empty(n * F, dtype=torch.float32, device="cuda")
    out = torch.empty(n * H, dtype=torch.float32, device="cuda")
    ws, keep2 = workspace(n, F)
    lfm3.check(lib.lfm3_cuda_project_ffn(ctypes.byref(gw), ctypes.byref(uw),
                                         ctypes.byref(dw), ptr(dx), ptr(h), None,
                                         ptr(out), n, None, ctypes.byref(ws),
                                         0))
    near(host(h).reshape(n, F), hidden, 2e-5)
    near(host(out).reshape(n, H), expected, 5e-5)


# ---- ShortConv (tests/ops_test.cpp:90-116) ------------------------------------
@pytest.mark.parametrize("n", [1, 8, 9, 15, 16, 29, 32, 33, 128, 512])
def test_conv(n):
    H, L = 37, 7
    projection, weight, history = data(n * 3 * H), data(H * L, 0.3), data(H * (L - 1))
    p = projection.reshape(n, 3 * H).astype(np.float64)
    expected = np.zeros((n, H))
    expected_history = history.reshape(H, L - 1).copy()
    for c in range(H):
        seq = list(history.reshape(H, L - 1)[c].astype(np.float64))
        for t in range(n):
            seq.append(float(np.float32(projection[t * 3 * H + c] *
                                        projection[t * 3 * H + 2 * H + c])))
            s = sum(float(weight[c * L + k]) * seq[t + k] for k in range(L))
            expected[t, c] = s * p[t, H + c]
        expected_history[c] = seq[n:n + L - 1]
    dp, dw, dh = dev(projection), dev(weight), dev(history)
    y = torch.empty(n * H, dtype=torch.float32, device="cuda")
    lfm3.check(lib.lfm3_cuda_short_conv(ptr(dp), ptr(dw), ptr(dh), ptr(y), n, H,
                                        L, None, 1))
    near(host(y).reshape(n, H), expected, 1e-7)
    near(host(dh).reshape(H, L - 1), expected_history, 0)


# ---- RoPE (tests/ops_test.cpp:117-141) -------------------------------------------
@pytest.mark.parametrize("n", [1, 8, 9, 15, 16, 29, 32, 33, 128, 512])
def test_rotary(n):
    D, H, P = 128, 3, 12001
    x = data(n * H * D)
    factors = np.ones(D // 2, np.float32)
    factors[32:] = 1e30
    xr = x.reshape(n, H, D).astype(np.float64)
    expected = xr.copy()
    # std::pow(1000000.0F, -2.0F * i / D) is the C library's powf (numpy's
    # float32 power is not correctly rounded)
    powf = ctypes.CDLL("libm.so.6").powf
    powf.argtypes, powf.restype = [ctypes.c_float, ctypes.c_float], ctypes.c_float
    base = np.array([powf(1000000.0, float(np.float32(-2.0) * np.float32(i) / np.float32(D)))
                     for i in range(D // 2)], np.float32)
    for row in range(n):
        angle = ((np.float32(P + row) * base) / factors).astype(np.float32).astype(np.float64)
        a, b = xr[row, :, :64], xr[row, :, 64:]
        expected[row, :, :64] = a * np.cos(angle) - b * np.sin(angle)
        expected[row, :, 64:] = b * np.cos(angle) + a * np.sin(angle)
    dx, df = dev(x), dev(factors)
    freq = torch.empty(D // 2, dtype=torch.float32, device="cuda")
    lfm3.check(lib.lfm3_cuda_rope_frequencies(ptr(freq), D, 1000000.0, None))
    lfm3.check(lib.lfm3_cuda_rope(ptr(dx), ptr(freq), ptr(df), n, H, D, P, None))
    near(host(dx).reshape(n, H, D), expected, 2e-5)


# ---- gated GQA attention (tests/ops_test.cpp:148-220) ------------------------
def run_attention(n, window, P=259, H=4, KH=2):
    D = 128
    capacity = window if window else P + n
    stride = KH * D
    q, k = data(n * H * D, 0.7), round16(data(n * stride, 0.5))
    v, gates = round16(data(n * stride, 0.9)), data(n * H, 0.7)
    ck, cv = round16(data(capacity * stride, 0.6)), round16(data(capacity * stride, 0.8))
    qq = q.reshape(n, H, D).astype(np.float64)
    kk, vv = k.reshape(n, KH, D).astype(np.float64), v.reshape(n, KH, D).astype(np.float64)
    ckk, cvv = ck.reshape(capacity, KH, D).astype(np.float64), cv.reshape(capacity, KH, D).astype(np.float64)
    expected = np.zeros((n, H, D))
    for row in range(n):
        last = P + row
        first = max(0, last + 1 - window) if window else 0
        ts = np.arange(first, last + 1)
        for h in range(H):
            kh = h // (H // KH)
            keys = np.stack([kk[t - P, kh] if t >= P else ckk[t % capacity, kh] for t in ts])
            vals = np.stack([vv[t - P, kh] if t >= P else cvv[t % capacity, kh] for t in ts])
            s = keys @ qq[row, h] / np.sqrt(D)
            s = np.exp(s - s.max())
            expected[row, h] = (s / s.sum()) @ vals / (1 + np.exp(-float(gates[row * H + h])))
    dq, dk, dv, dg = dev(q), dev(k), dev(v), dev(gates)
    dck, dcv = dev(ck), dev(cv)
    k16 = torch.empty(k.size, dtype=torch.int16, device="cuda")
    v16 = torch.empty_like(k16)
    ck16 = torch.empty(ck.size, dtype=torch.int16, device="cuda")
    cv16 = torch.empty_like(ck16)
    out = torch.empty(n * H * D, dtype=torch.float32, device="cuda")
    scratch = torch.empty(lib.lfm3_cuda_attention_scratch_bytes(H, D, P + n, n) // 4 + 1,
                          dtype=torch.float32, device="cuda")
    lfm3.check(lib.lfm3_cuda_pack_kv(ptr(dk), ptr(dv), ptr(k16), ptr(v16), k.size, None))
    lfm3.check(lib.lfm3_cuda_pack_kv(ptr(dck), ptr(dcv), ptr(ck16), ptr(cv16), ck.size, None))
    lfm3.check(lib.lfm3_cuda_attention(ptr(dq), ptr(k16), ptr(v16), ptr(dg), ptr(ck16),
                                       ptr(cv16), ptr(out), n, H, KH, D, P, capacity,
                                       window, None, ptr(scratch)))
    lfm3.check(lib.lfm3_cuda_store_kv(ptr(k16), ptr(v16), ptr(ck16), ptr(cv16), n, stride,
                                      P, capacity, None))
    near(host(out).reshape(n, H, D), expected, 2e-6 if n == 1 else 1e-3)
    # the ring holds exactly the rounded rows
    ck2, cv2 = ck.reshape(capacity, stride).copy(), cv.reshape(capacity, stride).copy()
    for row in range(n):
        ck2[(P + row) % capacity] = k.reshape(n, stride)[row]
        cv2[(P + row) % capacity] = v.reshape(n, stride)[row]
    got_k = host(ck16).view(np.float16).astype(np.float32).reshape(capacity, stride)
    got_v = host(cv16).view(np.float16).astype(np.float32).reshape(capacity, stride)
    np.testing.assert_array_equal(got_k, ck2)
    np.testing.assert_array_equal(got_v, cv2)


@pytest.mark.parametrize("n", [1, 8, 9, 15, 16, 29, 32, 33, 128, 512])
@pytest.mark.parametrize("window", [0, 256])
def test_attention(n, window):
    run_attention(n, window)


@pytest.mark.parametrize("window", [0, 256])
def test_long_decode_history(window):
    run_attention(1, window, P=4999)


# Decode rows whose keys end at, just before or just after a warp's 16-key
# block and a 64-key tile (each warp of the decode kernel owns 16 keys of a
# tile, so warps with no keys, a partial block and a partial tile all occur).
@pytest.mark.parametrize("P", [0, 1, 14, 15, 16, 17, 47, 48, 63, 64, 65, 255, 256, 257])
@pytest.mark.parametrize("window", [0, 256])
@pytest.mark.parametrize("heads", [(4, 2), (16, 4)])
def test_decode_key_block_edges(P, window, heads):
    run_attention(1, window, P=P, H=heads[0], KH=heads[1])


@pytest.mark.parametrize("window", [0, 256])
def test_prompt_over_long_history(window):
    run_attention(40, window, P=17000)


@pytest.mark.parametrize("n", [1, 77, 512])
@pytest.mark.parametrize("window", [0, 256])
def test_model_heads(n, window):
    run_attention(n, window, P=3000, H=16, KH=4)


def test_unsupported_shapes_refused():
    t = abi.Tensor(None, abi.Q8_0, 2048, 37, 0)
    assert lib.lfm3_cuda_attention(None, None, None, None, None, None, None, 1, 4,
                                   2, 64, 0, 1, 0, None, None) == -3
    assert lib.lfm3_cuda_residual_norm(None, None, None, None, None, 1, 100, 1e-5,
                                       0, None, None) == -3
    ws = WorkspaceStruct()
    assert lib.lfm3_cuda_dense(ctypes.byref(t), None, None, 1, None,
                               ctypes.byref(ws)) == -3

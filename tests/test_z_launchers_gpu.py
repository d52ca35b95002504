"""The launch-level operators of hip/ops.hpp (LaunchGEMV,
LaunchBatchedQuantGEMMFp32, LaunchExactBf16GEMMFp32SmallBatch,
LaunchBatchedResidualAdd): each equals the Dense path (lfm3_cuda_dense,
itself checked against FP64 formulas in test_ops_gpu.py) on the same
matrix and rows, or the exact FP32 sum."""
import ctypes

import numpy as np
import pytest

from helpers import abi, lfm3

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


class Workspace(ctypes.Structure):
    _fields_ = [("quantized", ctypes.c_void_p), ("row_max", ctypes.c_void_p),
                ("partial", ctypes.c_void_p), ("tickets", ctypes.c_void_p)]


def setup_module(module):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def q8_bytes(w):
    """Q8_0 rows (llama.cpp rule: d = amax / 127 as fp16, q = round(x / d))."""
    M, K = w.shape
    blocks = w.reshape(M, K // 32, 32).astype(np.float32)
    d = (np.abs(blocks).max(axis=2) / 127).astype(np.float16)
    inv = np.where(d.astype(np.float32) > 0, 1 / d.astype(np.float32), 0)
    q = np.clip(np.round(blocks * inv[:, :, None]), -127, 127).astype(np.int8)
    out = np.empty((M, K // 32, 34), np.uint8)
    out[:, :, :2] = d.view(np.uint8).reshape(M, K // 32, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def bf16_bytes(w):
    u = w.astype(np.float32).view(np.uint32)
    # round to nearest even; int16 storage (the same bits) for torch
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).view(np.int16)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def dense(lib, wbuf, wtype, M, K, x):
    rows = x.shape[0]
    row_bytes = K // 32 * 34 if wtype == abi.Q8_0 else 2 * K
    t = abi.Tensor(wbuf.data_ptr(), wtype, K, M, M * row_bytes)
    out = torch.empty((rows, M), dtype=torch.float32, device="cuda")
    q = torch.empty(lib.lfm3_cuda_dense_workspace_bytes(rows, K) // 4 + 1,
                    dtype=torch.float32, device="cuda")
    ws = Workspace(q.data_ptr(), None, None, None)
    xd = dev(x)
    lfm3.check(lib.lfm3_cuda_dense(ctypes.byref(t), p(xd), p(out), rows, None,
                                   ctypes.byref(ws)))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("rows", [1, 3, 8, 20])
def test_q8_launchers_equal_dense(rows):
    lib = lfm3.library()
    rng = np.random.default_rng(rows)
    M, K = 384, 1024
    w = rng.standard_normal((M, K)).astype(np.float32) * 0.05
    wbuf = dev(q8_bytes(w))
    x = rng.standard_normal((rows, K)).astype(np.float32)
    want = dense(lib, wbuf, abi.Q8_0, M, K, x)
    xd = dev(x)
    y = torch.empty((rows, M), dtype=torch.float32, device="cuda")
    if rows == 1:
        lfm3.check(lib.lfm3_cuda_gemv(p(wbuf), abi.Q8_0, p(xd), p(y), M, K, None))
    else:
        lfm3.check(lib.lfm3_cuda_batched_quant_gemm_fp32(
            abi.Q8_0, p(wbuf), p(xd), p(y), rows, M, K, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("rows", [1, 5])
def test_bf16_launchers_equal_dense(rows):
    lib = lfm3.library()
    rng = np.random.default_rng(40 + rows)
    M, K = 256, 512
    w = rng.standard_normal((M, K)).astype(np.float32) * 0.05
    wbuf = dev(bf16_bytes(w))
    x = rng.standard_normal((rows, K)).astype(np.float32)
    want = dense(lib, wbuf, abi.BF16, M, K, x)
    xd = dev(x)
    y = torch.empty((rows, M), dtype=torch.float32, device="cuda")
    if rows == 1:
        lfm3.check(lib.lfm3_cuda_gemv(p(wbuf), abi.BF16, p(xd), p(y), M, K, None))
    else:
        lfm3.check(lib.lfm3_cuda_exact_bf16_gemm_fp32_small_batch(
            p(wbuf), p(xd), p(y), rows, M, K, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), want)


def test_batched_residual_add():
    lib = lfm3.library()
    rng = np.random.default_rng(7)
    a = rng.standard_normal((6, 1024)).astype(np.float32)
    b = rng.standard_normal((6, 1024)).astype(np.float32)
    ad, bd = dev(a), dev(b)
    out = torch.empty_like(ad)
    lfm3.check(lib.lfm3_cuda_batched_residual_add(p(ad), p(bd), p(out), 6, 1024, None))
    # in place, as the reference's engine calls it (out == a)
    lfm3.check(lib.lfm3_cuda_batched_residual_add(p(ad), p(bd), p(ad), 6, 1024, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), a + b)
    np.testing.assert_array_equal(ad.cpu().numpy(), a + b)
    assert lib.lfm3_cuda_batched_residual_add(p(ad), p(bd), p(out), 6, 1001, None) == -3


class Output(ctypes.Structure):
    _fields_ = [("weight", ctypes.POINTER(abi.Tensor)), ("out", ctypes.c_void_p)]


def test_split_ready_projection():
    """ResidualNorm with split writes the next projection's FP16 prompt input
    into the workspace; Project with split_ready reads it from there instead
    of converting x (hip/ops.hpp:44-48, 59-65) and matches the projection of
    the FP32 normalised rows."""
    lib = lfm3.library()
    rng = np.random.default_rng(9)
    n, H, M = 32, 512, 256
    x = rng.standard_normal((n, H)).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    w = rng.standard_normal((M, H)).astype(np.float32) * 0.05
    wbuf, nbuf, xd = dev(q8_bytes(w)), dev(norm_w), dev(x)
    wt = abi.Tensor(wbuf.data_ptr(), abi.Q8_0, H, M, M * (H // 32 * 34))
    nt = abi.Tensor(nbuf.data_ptr(), abi.F32, H, 1, H * 4)
    q = torch.empty(lib.lfm3_cuda_dense_workspace_bytes(n, H) // 4 + 1,
                    dtype=torch.float32, device="cuda")
    ws = Workspace(q.data_ptr(), None, None, None)
    z = torch.empty((n, H), dtype=torch.float32, device="cuda")
    unused = torch.zeros((n, H), dtype=torch.float32, device="cuda")
    a = torch.empty((n, M), dtype=torch.float32, device="cuda")
    b = torch.empty((n, M), dtype=torch.float32, device="cuda")
    # FP32 normalised rows, converted by the projection
    lfm3.check(lib.lfm3_cuda_residual_norm(None, None, p(xd), ctypes.byref(nt),
                                           p(z), n, H, 1e-5, 0, None,
                                           ctypes.byref(ws)))
    oa = (Output * 1)(Output(ctypes.pointer(wt), a.data_ptr()))
    lfm3.check(lib.lfm3_cuda_project(oa, 1, p(z), n, None, ctypes.byref(ws), 0))
    # the norm's FP16 output, read where it was written
    lfm3.check(lib.lfm3_cuda_residual_norm(None, None, p(xd), ctypes.byref(nt),
                                           None, n, H, 1e-5, 1, None,
                                           ctypes.byref(ws)))
    ob = (Output * 1)(Output(ctypes.pointer(wt), b.data_ptr()))
    lfm3.check(lib.lfm3_cuda_project(ob, 1, p(unused), n, None,
                                     ctypes.byref(ws), 1))
    torch.cuda.synchronize()
    ra, rb = a.cpu().numpy(), b.cpu().numpy()
    assert np.isfinite(ra).all() and np.abs(ra).max() > 0.1
    assert np.abs(ra - rb).max() <= 1e-4

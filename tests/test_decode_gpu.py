"""The engine's decode projection kernel (q8_decode.cu) on caller matrices,
through lfm3_cuda_decode_project: every shape the decode round uses (single
and fused four-output projections, gate/up with SwiGLU, K = 2048 and 8192,
the LM head's height) at 1..8 rows against an FP64 formula, with the
reference's projection tolerance (tests/ops_test.cpp:46-89: 1e-4). Shapes
whose tiles fall to several CTAs exercise the ordered partial-sum fix-up;
repeated calls must agree bit for bit. The same shapes with BF16 matrices
(the numerical-reference weights) run the kernel's BF16 records: each input
as three exact bf16 terms, products accumulated in FP32."""
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


def q8_matrix(M, K, seed):
    """Random Q8_0 rows: fp16 scales around 2^-9, codes in [-127, 127];
    returns (GGUF bytes, FP64 weights)."""
    rng = np.random.default_rng(seed)
    nb = M * K // 32
    d = (rng.uniform(0.5, 2.0, nb) * 2.0 ** -9).astype(np.float16)
    qs = rng.integers(-127, 128, (nb, 32)).astype(np.int8)
    blocks = np.zeros((nb, 34), np.uint8)
    blocks[:, :2] = d.view(np.uint8).reshape(nb, 2)
    blocks[:, 2:] = qs.view(np.uint8)
    w = (d.astype(np.float64)[:, None] * qs).reshape(M, K)
    return blocks.tobytes(), w


def bf16_matrix(M, K, seed):
    """Random BF16 rows ~ N(0, 0.02); returns (bytes, FP64 weights)."""
    rng = np.random.default_rng(seed)
    w = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    b = w.to(torch.bfloat16)
    raw = b.view(torch.int16).numpy().tobytes()
    return raw, b.to(torch.float64).numpy()


class Matrices:
    def __init__(self, shapes, K, seed=0, bf16=False):
        self.keep, self.tensors, self.w = [], [], []
        for j, M in enumerate(shapes):
            raw, w = (bf16_matrix if bf16 else q8_matrix)(M, K, seed + j)
            buf = torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda()
            self.keep.append(buf)
            self.tensors.append(abi.Tensor(buf.data_ptr(),
                                           abi.BF16 if bf16 else abi.Q8_0, K,
                                           M, len(raw)))
            self.w.append(w)
        n = len(self.tensors)
        self.array = (ctypes.POINTER(abi.Tensor) * n)(
            *[ctypes.pointer(t) for t in self.tensors])


def project(mats, x, swiglu=False, repeat=1):
    n_w = len(mats.tensors)
    rows, K = x.shape
    ws_bytes = lib.lfm3_cuda_decode_workspace_bytes(mats.array, n_w, int(swiglu))
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes // 4 + 64, dtype=torch.float32, device="cuda")
    base = (ws.data_ptr() + 255) // 256 * 256
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    outs = [torch.full((rows, int(t.rows)), float("nan"), dtype=torch.float32,
                       device="cuda")
            for t in (mats.tensors[:1] if swiglu else mats.tensors)]
    optr = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    ld = (ctypes.c_size_t * len(outs))(*[int(o.shape[1]) for o in outs])
    results = []
    for _ in range(repeat):
        lfm3.check(lib.lfm3_cuda_decode_project(
            mats.array, n_w, int(swiglu), ctypes.c_void_p(dx.data_ptr()), rows,
            optr, ld, ctypes.c_void_p(base), None))
        torch.cuda.synchronize()
        results.append([o.cpu().numpy().copy() for o in outs])
    return results


def inputs(rows, K, seed=1):
    rng = np.random.default_rng(seed)
    return rng.normal(0, 0.1, (rows, K)).astype(np.float32)


def near(got, want, limit=1e-4):
    assert np.isfinite(got).all()
    err = np.abs(got.astype(np.float64) - want)
    assert err.max() <= limit, (float(err.max()), np.unravel_index(err.argmax(), err.shape))


@pytest.mark.parametrize("rows", [1, 3, 8])
@pytest.mark.parametrize("M,K", [(2048, 2048), (37, 2048), (2048, 8192),
                                 (600, 512), (65536, 2048)])
def test_plain(rows, M, K):
    mats = Matrices([M], K, seed=M + K)
    x = inputs(rows, K)
    (got,), = project(mats, x)
    near(got, x.astype(np.float64) @ mats.w[0].T)


@pytest.mark.parametrize("rows", [2, 8])
def test_fused_qkvg(rows):
    """q, k, v and the attention gate (16 rows) in one launch, as the decode
    round projects an attention layer's input."""
    mats = Matrices([2048, 512, 512, 16], 2048, seed=11)
    x = inputs(rows, 2048, seed=2)
    got = project(mats, x)[0]
    for g, w in zip(got, mats.w):
        near(g, x.astype(np.float64) @ w.T)


@pytest.mark.parametrize("rows", [1, 8])
@pytest.mark.parametrize("F", [8192, 1024, 48])
def test_swiglu(rows, F):
    mats = Matrices([F, F], 2048, seed=F)
    x = inputs(rows, 2048, seed=3)
    (got,), = project(mats, x, swiglu=True)
    g = x.astype(np.float64) @ mats.w[0].T
    u = x.astype(np.float64) @ mats.w[1].T
    near(got, g / (1 + np.exp(-g)) * u)


def test_repeated_calls_identical():
    """Split tiles are summed in unit order by whichever CTA finishes last:
    results never depend on timing."""
    mats = Matrices([2048, 512, 512, 16], 2048, seed=5)
    x = inputs(8, 2048, seed=4)
    runs = project(mats, x, repeat=4)
    for r in runs[1:]:
        for a, b in zip(runs[0], r):
            np.testing.assert_array_equal(a, b)


def test_refuses_unsupported_shapes():
    mats = Matrices([64], 512)
    bad = abi.Tensor(mats.tensors[0].data, abi.Q8_0, 320, 64, 64 * 10 * 34)
    arr = (ctypes.POINTER(abi.Tensor) * 1)(ctypes.pointer(bad))
    assert lib.lfm3_cuda_decode_workspace_bytes(arr, 1, 0) == 0
    assert lib.lfm3_cuda_decode_workspace_bytes(mats.array, 1, 1) == 0  # swiglu needs 2


@pytest.mark.parametrize("rows", [1, 8])
@pytest.mark.parametrize("M,K", [(2048, 2048), (2048, 8192), (600, 512),
                                 (65536, 2048)])
def test_plain_bf16(rows, M, K):
    mats = Matrices([M], K, seed=M + K, bf16=True)
    x = inputs(rows, K)
    (got,), = project(mats, x)
    near(got, x.astype(np.float64) @ mats.w[0].T)


@pytest.mark.parametrize("rows", [3, 8])
def test_fused_qkvg_bf16(rows):
    mats = Matrices([2048, 512, 512, 16], 2048, seed=13, bf16=True)
    x = inputs(rows, 2048, seed=2)
    got = project(mats, x)[0]
    for g, w in zip(got, mats.w):
        near(g, x.astype(np.float64) @ w.T)


@pytest.mark.parametrize("F", [8192, 48])
def test_swiglu_bf16(F):
    mats = Matrices([F, F], 2048, seed=F + 1, bf16=True)
    x = inputs(8, 2048, seed=3)
    (got,), = project(mats, x, swiglu=True)
    g = x.astype(np.float64) @ mats.w[0].T
    u = x.astype(np.float64) @ mats.w[1].T
    near(got, g / (1 + np.exp(-g)) * u)


def test_mixed_types_refused():
    q = Matrices([64], 512)
    b = Matrices([64], 512, bf16=True)
    arr = (ctypes.POINTER(abi.Tensor) * 2)(ctypes.pointer(q.tensors[0]),
                                           ctypes.pointer(b.tensors[0]))
    assert lib.lfm3_cuda_decode_workspace_bytes(arr, 2, 0) == 0

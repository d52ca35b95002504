"""Host-only operator logic of the C ABI (no GPU): SharesSplit
(hip/ops.hpp:41-43), which decides whether projections of n rows read one
FP16 prompt input."""
import ctypes

from helpers import abi, lfm3


class Workspace(ctypes.Structure):
    _fields_ = [("quantized", ctypes.c_void_p), ("row_max", ctypes.c_void_p),
                ("partial", ctypes.c_void_p), ("tickets", ctypes.c_void_p)]


class Output(ctypes.Structure):
    _fields_ = [("weight", ctypes.POINTER(abi.Tensor)), ("out", ctypes.c_void_p)]


def shares(tensors, n, workspace=True):
    lib = lfm3.library()
    outs = (Output * len(tensors))(*[Output(ctypes.pointer(t), 0x1000) for t in tensors])
    ws = Workspace(0x2000 if workspace else None, None, None, None)
    return lib.lfm3_cuda_shares_split(outs, len(tensors), n, ctypes.byref(ws))


def test_shares_split():
    # payload pointers are never dereferenced on the host
    q8 = abi.Tensor(0x10000, abi.Q8_0, 2048, 512, 512 * 2176)
    q8b = abi.Tensor(0x20000, abi.Q8_0, 2048, 16, 16 * 2176)
    q8_wide = abi.Tensor(0x30000, abi.Q8_0, 8192, 512, 512 * 8704)
    bf = abi.Tensor(0x40000, abi.BF16, 2048, 512, 512 * 4096)
    rows = lfm3.library().lfm3_cuda_prompt_rows()
    assert rows == 16
    assert shares([q8, q8b], rows) == 1
    assert shares([q8, q8b], rows - 1) == 0       # decode rows keep FP32
    assert shares([q8, q8_wide], 64) == 0          # widths differ
    assert shares([q8, bf], 64) == 0               # BF16 reads FP32 rows
    assert shares([q8], 64, workspace=False) == 0  # nowhere to hold it
    assert shares([q8] * 5, 64) == 0               # at most four outputs

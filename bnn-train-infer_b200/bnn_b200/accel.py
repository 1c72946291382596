"""Python binding of the BNN_* accelerator API v2 (include/bnn_b200_accel.h).

A thin ctypes mirror of the C ABI with the reference's names, argument
meaning and status codes (bnn-accelerator/bnn-accelerator.h): functions
return BNN_Status values; the object wrappers raise BnnError carrying the
status. `Api(cdll)` binds any library exporting the eleven BNN_* symbols,
which is how tests drive the same jobs through libbnn_b200.so and through
the reference soft backend.
"""
import ctypes
from ctypes import POINTER, c_char_p, c_int, c_size_t, c_uint8, c_uint16, c_uint32, c_void_p

import numpy as np

from . import _lib

API_VERSION = 2

OK, EINVAL, ENOMEM, ENOTSUP, ERANGE, EBUSY, EIO, ETIMEOUT = 0, -1, -2, -3, -4, -5, -6, -7
STATUS_NAMES = {OK: "BNN_OK", EINVAL: "BNN_EINVAL", ENOMEM: "BNN_ENOMEM", ENOTSUP: "BNN_ENOTSUP",
                ERANGE: "BNN_ERANGE", EBUSY: "BNN_EBUSY", EIO: "BNN_EIO", ETIMEOUT: "BNN_ETIMEOUT"}

OP_GEMV, OP_GEMM, OP_DOT_GROUPS, OP_GEMV_F32, OP_GEMM_F32 = 1, 2, 3, 4, 5
TYPE_I8, TYPE_F32, TYPE_I16 = 1, 2, 3
CAP_GEMV, CAP_GEMM, CAP_DOT_GROUPS, CAP_GEMV_F32, CAP_GEMM_F32 = 1, 2, 4, 8, 16
GROUP = 128

OP_TYPES = {OP_GEMV: (TYPE_I8, TYPE_F32), OP_GEMM: (TYPE_I8, TYPE_F32),
            OP_DOT_GROUPS: (TYPE_I8, TYPE_I16), OP_GEMV_F32: (TYPE_F32, TYPE_F32),
            OP_GEMM_F32: (TYPE_F32, TYPE_F32)}


class Caps(ctypes.Structure):
    _fields_ = [("api_version", c_uint32), ("max_in_features", c_uint32),
                ("max_out_features", c_uint32), ("max_rows", c_uint32),
                ("group_size", c_uint32), ("supported_ops", c_uint32)]


class MatrixDesc(ctypes.Structure):
    _fields_ = [("in_features", c_uint32), ("out_features", c_uint32), ("group_size", c_uint32),
                ("weight_bits", POINTER(c_uint8)), ("weight_bytes", c_size_t),
                ("scale_fp16", POINTER(c_uint16)), ("scale_count", c_size_t)]


class BufferView(ctypes.Structure):
    _fields_ = [("buffer", c_void_p), ("type", c_int), ("offset", c_size_t),
                ("row_stride", c_size_t)]


class Job(ctypes.Structure):
    _fields_ = [("operation", c_int), ("matrix", c_void_p), ("input", BufferView),
                ("output", BufferView), ("rows", c_uint32)]


class BnnError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}")


class Api:
    """The eleven BNN_* entry points of one library, with ctypes signatures."""

    def __init__(self, cdll=None):
        self.dll = cdll if cdll is not None else _lib.load()
        d = self.dll
        sig = {
            "BNN_DeviceOpen": (c_int, [c_uint32, POINTER(c_void_p)]),
            "BNN_DeviceClose": (c_int, [c_void_p]),
            "BNN_DeviceGetCaps": (c_int, [c_void_p, POINTER(Caps)]),
            "BNN_MatrixCreate": (c_int, [c_void_p, POINTER(MatrixDesc), POINTER(c_void_p)]),
            "BNN_MatrixDestroy": (None, [c_void_p]),
            "BNN_BufferAlloc": (c_int, [c_void_p, c_size_t, POINTER(c_void_p)]),
            "BNN_BufferFree": (None, [c_void_p]),
            "BNN_BufferWrite": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t]),
            "BNN_BufferRead": (c_int, [c_void_p, c_size_t, c_void_p, c_size_t]),
            "BNN_Execute": (c_int, [c_void_p, POINTER(Job)]),
            "BNN_StatusString": (c_char_p, [c_int]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(d, name)
            fn.restype = res
            fn.argtypes = args
            setattr(self, name, fn)

    def status_string(self, status):
        return self.BNN_StatusString(status).decode()


def _check(status, what):
    if status != OK:
        raise BnnError(status, what)


class Device:
    def __init__(self, index=0, api=None):
        self.api = api or Api()
        h = c_void_p()
        _check(self.api.BNN_DeviceOpen(index, ctypes.byref(h)), "BNN_DeviceOpen")
        self.handle = h

    def caps(self):
        c = Caps()
        _check(self.api.BNN_DeviceGetCaps(self.handle, ctypes.byref(c)), "BNN_DeviceGetCaps")
        return c

    def close(self):
        if self.handle:
            _check(self.api.BNN_DeviceClose(self.handle), "BNN_DeviceClose")
            self.handle = None

    def execute(self, op, matrix, inp, out, rows=1, in_offset=0, in_stride=0, out_offset=0,
                out_stride=0, in_type=None, out_type=None):
        """Runs one job; returns the BNN_Status (does not raise)."""
        it, ot = OP_TYPES.get(op, (TYPE_I8, TYPE_F32))
        job = Job(operation=op, matrix=matrix.handle if matrix else None,
                  input=BufferView(inp.handle if inp else None, it if in_type is None else in_type,
                                   in_offset, in_stride),
                  output=BufferView(out.handle if out else None, ot if out_type is None else out_type,
                                    out_offset, out_stride),
                  rows=rows)
        return self.api.BNN_Execute(self.handle, ctypes.byref(job))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Matrix:
    """A W1 matrix; bits uint8 [N][K/8], scales uint16 [N][K/128]."""

    def __init__(self, device, bits, scales):
        self.device = device
        bits = np.ascontiguousarray(bits, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.uint16)
        n, kb = bits.shape
        self.k, self.n = kb * 8, n
        desc = MatrixDesc(self.k, n, GROUP, bits.ctypes.data_as(POINTER(c_uint8)), bits.nbytes,
                          scales.ctypes.data_as(POINTER(c_uint16)), scales.size)
        h = c_void_p()
        _check(device.api.BNN_MatrixCreate(device.handle, ctypes.byref(desc), ctypes.byref(h)),
               "BNN_MatrixCreate")
        self.handle = h

    def destroy(self):
        if self.handle:
            self.device.api.BNN_MatrixDestroy(self.handle)
            self.handle = None


class Buffer:
    def __init__(self, device, nbytes):
        self.device = device
        self.nbytes = nbytes
        h = c_void_p()
        _check(device.api.BNN_BufferAlloc(device.handle, nbytes, ctypes.byref(h)), "BNN_BufferAlloc")
        self.handle = h

    def write(self, data, offset=0):
        data = np.ascontiguousarray(data)
        _check(self.device.api.BNN_BufferWrite(self.handle, offset, data.ctypes.data, data.nbytes),
               "BNN_BufferWrite")

    def read(self, nbytes=None, offset=0):
        nbytes = self.nbytes - offset if nbytes is None else nbytes
        out = np.empty(nbytes, dtype=np.uint8)
        _check(self.device.api.BNN_BufferRead(self.handle, offset, out.ctypes.data, nbytes),
               "BNN_BufferRead")
        return out

    def free(self):
        if self.handle:
            self.device.api.BNN_BufferFree(self.handle)
            self.handle = None


def run_op(device, op, bits, scales, x, rows=None):
    """Convenience: one packed job end to end (upload, execute, read back).

    x: int8 [M][K] for I8 ops, float32 [M][K] for F32 ops. Returns the output
    array (float32 [M][N] or int16 [M][N][G]); raises BnnError on failure."""
    m = Matrix(device, bits, scales)
    x = np.ascontiguousarray(x)
    if x.ndim == 1:
        x = x[None, :]
    rows = x.shape[0] if rows is None else rows
    n, g = m.n, m.k // GROUP
    out_shape = (rows, n, g) if op == OP_DOT_GROUPS else (rows, n)
    out_dtype = np.int16 if op == OP_DOT_GROUPS else np.float32
    out_bytes = int(np.prod(out_shape)) * np.dtype(out_dtype).itemsize
    bi, bo = Buffer(device, x.nbytes), Buffer(device, out_bytes)
    try:
        bi.write(x)
        st = device.execute(op, m, bi, bo, rows=rows)
        _check(st, "BNN_Execute")
        return bo.read().view(out_dtype).reshape(out_shape)
    finally:
        bi.free()
        bo.free()
        m.destroy()

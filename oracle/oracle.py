"""Python face of the CPU oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg to check or time the B200 path; never by the
product package.

Two checkers live here:
  * libbnn_oracle.so (oracle/bnn_oracle.c): this project's restatement of the
    reference soft backend's arithmetic (soft-bnn-accelerator.c:92-276),
    OpenMP-parallel over output channels, bit-identical by construction;
  * oracle/_ref/libbnn_soft_ref.so: the reference soft backend itself,
    compiled from its own source by oracle/Makefile (present wherever
    `make -C oracle ref` ran, i.e. this container and, by the snapshot,
    the GPU box).
Both are pinned against the reference's golden vectors in tests/golden/.
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libbnn_oracle.so"
SOFT_REF_PATH = HERE / "_ref" / "libbnn_soft_ref.so"
REF_DIR = HERE / "_ref"

_lib = None


def build():
    """Compile the oracle library (and nothing else)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "lib"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        f = _lib.oracle_quantize_row
        f.restype = ctypes.c_float
        f.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        _lib.oracle_half_to_float.restype = ctypes.c_float
        _lib.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        _lib.oracle_compute_rows.restype = None
        _lib.oracle_compute_rows.argtypes = [
            ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        _lib.oracle_validate_f32.restype = ctypes.c_int
        _lib.oracle_validate_f32.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        _lib.oracle_validate_i8.restype = ctypes.c_int
        _lib.oracle_validate_i8.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def half_to_float(h):
    return lib().oracle_half_to_float(int(h) & 0xFFFF)


def quantize_rows(x):
    """x float32 [M][K] -> (q int8 [M][K], s float32 [M]) per soft :175-211."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    m, k = x.shape
    q = np.empty((m, k), dtype=np.int8)
    s = np.empty(m, dtype=np.float32)
    for i in range(m):
        s[i] = lib().oracle_quantize_row(_ptr(x[i]), k, _ptr(q[i]))
    return q, s


def _contract(bits, scales, q, row_scale, mode):
    bits = np.ascontiguousarray(bits, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    q = np.ascontiguousarray(q, dtype=np.int8)
    if q.ndim == 1:
        q = q[None, :]
    m, k = q.shape
    n = bits.shape[0]
    assert bits.shape == (n, k // 8) and scales.shape == (n, k // 128)
    if mode == 0:
        out = np.empty((m, n, k // 128), dtype=np.int16)
    else:
        out = np.empty((m, n), dtype=np.float32)
    rs = None
    if row_scale is not None:
        rs = np.ascontiguousarray(row_scale, dtype=np.float32)
    lib().oracle_compute_rows(k, n, m, _ptr(bits), _ptr(scales), _ptr(q),
                              _ptr(rs) if rs is not None else None, mode, _ptr(out))
    return out


def dot_groups(bits, scales, q):
    """BNN_OP_DOT_GROUPS: int16 [M][N][K/128]."""
    return _contract(bits, scales, q, None, 0)


def gemm_i8(bits, scales, q):
    """BNN_OP_GEMV/GEMM on int8 input: Z float32 [M][N]."""
    return _contract(bits, scales, q, None, 1)


def gemm_f32(bits, scales, x):
    """BNN_OP_GEMV_F32/GEMM_F32: returns (Y [M][N], Q [M][K], s [M])."""
    q, s = quantize_rows(x)
    return _contract(bits, scales, q, s, 1), q, s


def finite(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    return bool(lib().oracle_validate_f32(_ptr(x), x.size))


def soft_ref_available():
    return SOFT_REF_PATH.exists()


def ref_tool(name):
    """Path of a binary compiled from reference sources, or None."""
    p = REF_DIR / name
    return p if p.exists() and os.access(p, os.X_OK) else None

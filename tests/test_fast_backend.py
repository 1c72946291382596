"""The multi-threaded CPU backend (oracle/bnn_fast_backend.c) against the soft
backend, on the CPU.

The full-shape parity tests (tests/test_parity_full_gpu.py) check the device
engine against the reference engine's own sources linked over this backend
(oracle/_ref/libbnn_engine_fast.so), because the soft backend needs ~15 s per
Qwen3-1.7B token. That is only sound if the two reference builds agree bit for
bit, which this file pins:
  * BNN_Execute of every op at Qwen3 linear shapes (incl. K = 6144) and a
    multi-row GEMM, byte-compared with the soft backend compiled from its
    source (oracle/_ref/libbnn_soft_ref.so);
  * the whole reference engine over each backend: teacher-forced Qwen3
    logits, a greedy stream, and bnn-mlp classify logits, bit-identical.
"""
import ctypes

import numpy as np
import pytest

from bnn_b200 import gguf, synth

import ref_engine

pytestmark = pytest.mark.skipif(not (ref_engine.available() and ref_engine.available(fast=True)),
                                reason="reference engine libraries not built (make -C oracle ref)")

OP_GEMV, OP_GEMM, OP_DOT, OP_GEMV_F32, OP_GEMM_F32 = 1, 2, 3, 4, 5
I8, F32, I16 = 1, 2, 3


class MatrixDesc(ctypes.Structure):
    _fields_ = [("in_features", ctypes.c_uint32), ("out_features", ctypes.c_uint32),
                ("group_size", ctypes.c_uint32), ("weight_bits", ctypes.c_void_p),
                ("weight_bytes", ctypes.c_size_t), ("scale_fp16", ctypes.c_void_p),
                ("scale_count", ctypes.c_size_t)]


class View(ctypes.Structure):
    _fields_ = [("buffer", ctypes.c_void_p), ("type", ctypes.c_int), ("offset", ctypes.c_size_t),
                ("row_stride", ctypes.c_size_t)]


class Job(ctypes.Structure):
    _fields_ = [("operation", ctypes.c_int), ("matrix", ctypes.c_void_p), ("input", View),
                ("output", View), ("rows", ctypes.c_uint32)]


def execute(lib, op, bits, scales, x):
    """One BNN_Execute through a BNN_* library; returns the output array."""
    n, kb = bits.shape
    k = kb * 8
    rows = x.shape[0]
    dev, mat, bi, bo = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.BNN_DeviceOpen(0, ctypes.byref(dev)) == 0
    bits = np.ascontiguousarray(bits)
    scales = np.ascontiguousarray(scales)
    d = MatrixDesc(k, n, 128, bits.ctypes.data, bits.nbytes, scales.ctypes.data, scales.size)
    assert lib.BNN_MatrixCreate(dev, ctypes.byref(d), ctypes.byref(mat)) == 0
    x = np.ascontiguousarray(x)
    out_bytes = rows * (n * (k // 128) * 2 if op == OP_DOT else n * 4)
    assert lib.BNN_BufferAlloc(dev, ctypes.c_size_t(x.nbytes), ctypes.byref(bi)) == 0
    assert lib.BNN_BufferAlloc(dev, ctypes.c_size_t(out_bytes), ctypes.byref(bo)) == 0
    assert lib.BNN_BufferWrite(bi, ctypes.c_size_t(0), x.ctypes.data, ctypes.c_size_t(x.nbytes)) == 0
    in_t = F32 if op in (OP_GEMV_F32, OP_GEMM_F32) else I8
    out_t = I16 if op == OP_DOT else F32
    job = Job(op, mat, View(bi, in_t, 0, 0), View(bo, out_t, 0, 0), rows)
    st = lib.BNN_Execute(dev, ctypes.byref(job))
    out = np.empty(out_bytes, dtype=np.uint8)
    assert lib.BNN_BufferRead(bo, ctypes.c_size_t(0), out.ctypes.data, ctypes.c_size_t(out_bytes)) == 0
    lib.BNN_BufferFree(bi)
    lib.BNN_BufferFree(bo)
    lib.BNN_MatrixDestroy(mat)
    assert lib.BNN_DeviceClose(dev) == 0
    assert st == 0, f"BNN_Execute status {st}"
    return out


def libs():
    soft = ctypes.CDLL(str(ref_engine.LIB.parent / "libbnn_soft_ref.so"))
    fast = ref_engine.dll(fast=True)
    for lib in (soft, fast):
        lib.BNN_DeviceOpen.argtypes = [ctypes.c_uint32, ctypes.c_void_p]
        lib.BNN_MatrixCreate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.BNN_BufferAlloc.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        lib.BNN_BufferWrite.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
        lib.BNN_BufferRead.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t]
        lib.BNN_Execute.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.BNN_BufferFree.argtypes = [ctypes.c_void_p]
        lib.BNN_MatrixDestroy.argtypes = [ctypes.c_void_p]
        lib.BNN_DeviceClose.argtypes = [ctypes.c_void_p]
    return soft, fast


@pytest.mark.parametrize("k,n,rows", [(2048, 1024, 1), (6144, 512, 1), (2048, 640, 5), (384, 17, 3)])
def test_execute_matches_soft(k, n, rows):
    soft, fast = libs()
    rng = synth.rng_for(11, salt=k + n + rows)
    bits, scales = synth.w1_matrix(rng, k, n)
    x = synth.activations(rng, rows, k)
    q = synth.i8_activations(rng, rows, k)
    f32_op = OP_GEMV_F32 if rows == 1 else OP_GEMM_F32
    i8_op = OP_GEMV if rows == 1 else OP_GEMM
    for op, inp in ((f32_op, x), (i8_op, q), (OP_DOT, q)):
        a = execute(soft, op, bits, scales, inp)
        b = execute(fast, op, bits, scales, inp)
        assert a.tobytes() == b.tobytes(), f"op {op} differs from the soft backend"


def test_engine_over_fast_backend_matches_soft(tmp_path):
    shape = gguf.Qwen3Shape(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=600,
                            context=128)
    path = gguf.qwen3_model(tmp_path / "tiny.gguf", shape, seed=21)
    ids = np.random.default_rng(3).integers(0, shape.vocab, size=9).astype(np.int32)
    soft = ref_engine.RefEngine(path, n_ctx=64)
    fast = ref_engine.RefEngine(path, n_ctx=64, fast=True)
    try:
        for i in range(len(ids)):  # teacher forced, one token per call
            a, b = soft.decode(ids[i:i + 1]), fast.decode(ids[i:i + 1])
            assert a.view(np.uint32).tobytes() == b.view(np.uint32).tobytes(), f"position {i}"
        soft.truncate(0)
        fast.truncate(0)
        assert soft.greedy(ids[:5], 8) == fast.greedy(ids[:5], 8)
    finally:
        soft.close()
        fast.close()
    mpath = gguf.bnn_mlp_model(tmp_path / "mlp.gguf")
    x = np.random.default_rng(4).standard_normal((70, 896)).astype(np.float32)
    x[:, 784:] = 0
    soft = ref_engine.RefEngine(mpath, n_batch=64)
    fast = ref_engine.RefEngine(mpath, n_batch=64, fast=True)
    try:
        for b0 in (0, 64):  # a full batch and the 6-sample tail
            a, b = soft.classify(x[b0:b0 + 64]), fast.classify(x[b0:b0 + 64])
            assert a.view(np.uint32).tobytes() == b.view(np.uint32).tobytes()
    finally:
        soft.close()
        fast.close()

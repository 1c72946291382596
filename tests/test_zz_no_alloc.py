"""bnn_b200_gemm_f32_noalloc against BNN_Execute(GEMM_F32) (marked gpu).

The allocation-free entry point serves callers that cannot let the library
cudaMalloc while they run (a framework allocator owns the free device
memory, or a hot loop cannot absorb cudaMalloc's synchronisation). It must
give the same bits as the regular GEMM_F32 job, call after call, on the
shared fixed scratch array. This file is collected last on purpose.
"""
import ctypes

import numpy as np
import oracle
import pytest

from bnn_b200 import accel, synth

pytestmark = pytest.mark.gpu


def bind(api):
    fn = api.dll.bnn_b200_gemm_f32_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    ptr = api.dll.bnn_b200_buffer_device_ptr
    ptr.restype = ctypes.c_void_p
    ptr.argtypes = [ctypes.c_void_p]
    return fn, ptr


@pytest.mark.parametrize("k,n,rows", [(2048, 2048, 1), (6144, 2048, 1), (384, 17, 3), (8192, 96, 16)])
def test_noalloc_matches_execute_twice(k, n, rows):
    dev = accel.Device(0)
    noalloc, devptr = bind(dev.api)
    rng = synth.rng_for(9, salt=k + n + rows)
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(dev, bits, scales)
    bi, bo = accel.Buffer(dev, rows * k * 4), accel.Buffer(dev, rows * n * 4)
    try:
        for call in range(2):  # two calls in a row reuse the same scratch
            x = synth.activations(rng, rows, k) * np.float32(1 + call)
            want = accel.run_op(dev, accel.OP_GEMM_F32, bits, scales, x)
            bi.write(x)
            bo.write(np.full(rows * n * 4, 0x5A, dtype=np.uint8))
            st = noalloc(mat.handle, devptr(bi.handle), rows, devptr(bo.handle))
            assert st == accel.OK, f"call {call}: status {st}"
            got = bo.read().view(np.float32).reshape(rows, n)
            assert got.tobytes() == want.tobytes(), f"call {call} differs from BNN_Execute"
            # and straight against the CPU restatement of the soft backend
            ref, _, _ = oracle.gemm_f32(bits, scales, x)
            assert got.tobytes() == np.ascontiguousarray(ref, dtype=np.float32).tobytes(), \
                f"call {call} differs from the oracle"
    finally:
        bi.free()
        bo.free()
        mat.destroy()
        dev.close()


def test_noalloc_rejects_beyond_limits_and_bad_input():
    dev = accel.Device(0)
    noalloc, devptr = bind(dev.api)
    rng = synth.rng_for(9, salt=1)
    k, n = 256, 32
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(dev, bits, scales)
    bi, bo = accel.Buffer(dev, 17 * k * 4), accel.Buffer(dev, 17 * n * 4)
    try:
        assert noalloc(mat.handle, devptr(bi.handle), 17, devptr(bo.handle)) == accel.ERANGE
        assert noalloc(mat.handle, devptr(bi.handle), 0, devptr(bo.handle)) == accel.EINVAL
        x = synth.activations(rng, 2, k)
        x[1, 7] = np.inf
        bi.write(x)
        sentinel = np.full(2 * n * 4, 0x5A, dtype=np.uint8)
        bo.write(sentinel)
        assert noalloc(mat.handle, devptr(bi.handle), 2, devptr(bo.handle)) == accel.ERANGE
        assert bo.read(2 * n * 4).tobytes() == sentinel.tobytes()
        x[1, 7] = 1.0
        bi.write(x)
        assert noalloc(mat.handle, devptr(bi.handle), 2, devptr(bo.handle)) == accel.OK
    finally:
        bi.free()
        bo.free()
        mat.destroy()
        dev.close()

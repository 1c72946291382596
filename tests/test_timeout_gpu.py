"""The bounded-wait path: a device wait that runs out returns BNN_ETIMEOUT and
leaves the device usable (marked gpu).

Every wait in the kernels gives up after a limit and reports it through the
status word, which BNN_Execute maps to BNN_ETIMEOUT (bnn-accelerator.h:25-26:
the call may leave partial output, :202). The test lowers the limit to 1 ms
and makes the contraction's copy warps issue nothing (bnn_b200_test_wait_limit):
the consumer warps' waits for their weight tiles then run out, a flag that
nothing sets, with no copy in flight and nothing faulting. Then the limits
return to normal and the same job, on the same handle, must succeed
bit-identically to the oracle.
"""
import ctypes

import numpy as np
import pytest

from bnn_b200 import accel, synth

pytestmark = pytest.mark.gpu

ETIMEOUT = -7


def hook(api):
    fn = api.dll.bnn_b200_test_wait_limit
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int]
    return fn


@pytest.mark.parametrize("op,rows", [(accel.OP_GEMV_F32, 1), (accel.OP_GEMM_F32, 3)])
def test_starved_contraction_times_out_then_recovers(oracle_mod, op, rows):
    dev = accel.Device(0)
    set_limit = hook(dev.api)
    rng = synth.rng_for(13, salt=rows)
    k, n = 2048, 1024
    bits, scales = synth.w1_matrix(rng, k, n)
    x = synth.activations(rng, rows, k)
    mat = accel.Matrix(dev, bits, scales)
    bi, bo = accel.Buffer(dev, x.nbytes), accel.Buffer(dev, rows * n * 4)
    try:
        bi.write(x)
        assert set_limit(dev.handle, 1_000_000, 1) == accel.OK
        try:
            st = dev.execute(op, mat, bi, bo, rows=rows)
        finally:
            assert set_limit(dev.handle, 0, 0) == accel.OK
        assert st == ETIMEOUT, f"status {st}, expected BNN_ETIMEOUT"
        # the same handle, matrix and buffers work again
        assert dev.execute(op, mat, bi, bo, rows=rows) == accel.OK
        got = bo.read().view(np.float32).reshape(rows, n)
        want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
        assert got.tobytes() == np.ascontiguousarray(want, dtype=np.float32).tobytes()
    finally:
        bi.free()
        bo.free()
        mat.destroy()
        dev.close()

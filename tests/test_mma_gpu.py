"""Parity of the tensor-core contraction (tcgen05 kind::i8, w1a8_mma.cuh).

BNN_Execute runs jobs of 64 or more rows on the tensor cores. Every result is
compared with the CPU oracle (the restatement of soft-bnn-accelerator.c that
is pinned to the reference's golden vectors): DOT_GROUPS and the I8 ops bit
for bit as integers, the F32 ops bit for bit as floats — the epilogue keeps
the reference's per-group FP32 order, so no tolerance is needed.

Shapes cover ragged M (partial 128-row tiles), ragged N (partial 128-row
tiles, and several tiles per row), odd group counts (the TMEM chunk holds 2
groups), the largest K (8192), unaligned views, rejection before any output
write, and the BNN_* threshold itself (63 rows on the dp4a path, 64 on the
tensor cores).
"""
import numpy as np
import pytest

from bnn_b200 import accel, synth

pytestmark = pytest.mark.gpu


def _run(dev, orc, op, bits, scales, x):
    if op == accel.OP_GEMM_F32:
        want, _, _ = orc.gemm_f32(bits, scales, x)
        got = accel.run_op(dev, op, bits, scales, x)
        return np.array_equal(got.view(np.uint32), want.view(np.uint32))
    _, q, _ = orc.gemm_f32(bits, scales, x)
    if op == accel.OP_GEMM:
        want = orc.gemm_i8(bits, scales, q)
        got = accel.run_op(dev, op, bits, scales, q)
        return np.array_equal(got.view(np.uint32), want.view(np.uint32))
    want = orc.dot_groups(bits, scales, q)
    got = accel.run_op(dev, op, bits, scales, q)
    return np.array_equal(got, want)


@pytest.mark.parametrize("m,k,n", [
    (64, 128, 8),        # one group, one 8-row block
    (63, 2048, 64),      # just below the threshold: dp4a path
    (64, 2048, 64),      # just at it: tensor cores
    (129, 384, 17),      # ragged M and N, 3 groups (one partial chunk)
    (256, 1152, 96),     # 9 groups: one full chunk + 1
    (300, 6144, 40),     # 48 groups, 6 chunks, both TMEM buffers reused
    (96, 8192, 33),      # the largest K
    (200, 1024, 300),    # three 128-row N tiles, the last one partial
    (512, 2048, 640),    # full tiles only, four M tiles
])
@pytest.mark.parametrize("op", [accel.OP_GEMM_F32, accel.OP_GEMM, accel.OP_DOT_GROUPS])
def test_tensor_core_parity(b200_device, oracle_mod, m, k, n, op):
    rng = synth.rng_for(21, salt=m * 7 + k + n)
    bits, scales = synth.w1_matrix(rng, k, n)
    x = synth.activations(rng, m, k)
    assert _run(b200_device, oracle_mod, op, bits, scales, x)


def test_tensor_core_extremes(b200_device, oracle_mod):
    """|D| = 16256 in every group, and special binary16 scales."""
    rng = synth.rng_for(22)
    k, n, m = 1024, 40, 70
    bits, _ = synth.w1_matrix(rng, k, n)
    pool = np.array([0x3C00, 0xBC00, 0x0001, 0x8001, 0x03FF, 0x0400, 0x0000, 0x8000, 0x7BFF],
                    dtype=np.uint16)
    scales = pool[rng.integers(0, pool.size, size=(n, k // 128))]
    signs = np.unpackbits(bits[5], bitorder="little").astype(np.int8) * 2 - 1
    q = synth.i8_activations(rng, m, k)
    q[0] = signs * 127
    q[1] = -signs * 127
    d = accel.run_op(b200_device, accel.OP_DOT_GROUPS, bits, scales, q)
    assert np.all(d[0, 5] == 16256) and np.all(d[1, 5] == -16256)
    assert np.array_equal(d, oracle_mod.dot_groups(bits, scales, q))
    z = accel.run_op(b200_device, accel.OP_GEMM, bits, scales, q)
    assert np.array_equal(z.view(np.uint32), oracle_mod.gemm_i8(bits, scales, q).view(np.uint32))


def test_tensor_core_unaligned_views(b200_device, oracle_mod):
    rng = synth.rng_for(23)
    k, n, m = 512, 45, 77
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(b200_device, bits, scales)
    x = synth.activations(rng, m, k)
    in_row = x[0].nbytes
    in_stride, in_off = in_row + 12, 4
    out_row = n * 4
    out_stride, out_off = out_row + 6, 2
    raw_in = np.full(in_off + m * in_stride + 5, 0xFF, dtype=np.uint8)
    for r in range(m):
        raw_in[in_off + r * in_stride:in_off + r * in_stride + in_row] = x[r].view(np.uint8)
    sentinel = np.full(out_off + m * out_stride + 9, 0xA5, dtype=np.uint8)
    bi, bo = accel.Buffer(b200_device, raw_in.nbytes), accel.Buffer(b200_device, sentinel.nbytes)
    try:
        bi.write(raw_in)
        bo.write(sentinel)
        st = b200_device.execute(accel.OP_GEMM_F32, mat, bi, bo, rows=m, in_offset=in_off,
                                 in_stride=in_stride, out_offset=out_off, out_stride=out_stride)
        assert st == accel.OK
        want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
        expect = sentinel.copy()
        for r in range(m):
            expect[out_off + r * out_stride:out_off + r * out_stride + out_row] = \
                np.ascontiguousarray(want[r]).view(np.uint8).reshape(-1)
        assert np.array_equal(bo.read(), expect)  # padding between rows untouched
    finally:
        bi.free()
        bo.free()
        mat.destroy()


def test_tensor_core_rejection_then_recovery(b200_device, oracle_mod):
    rng = synth.rng_for(24)
    k, n, m = 384, 50, 130
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(b200_device, bits, scales)
    x = synth.activations(rng, m, k)
    bi, bo = accel.Buffer(b200_device, x.nbytes), accel.Buffer(b200_device, m * n * 4)
    try:
        sentinel = np.full(m * n * 4, 0x5A, dtype=np.uint8)
        bo.write(sentinel)
        xb = x.copy()
        xb[m - 1, 7] = np.nan  # a row of the second 128-row tile
        bi.write(xb)
        assert b200_device.execute(accel.OP_GEMM_F32, mat, bi, bo, rows=m) == accel.ERANGE
        assert np.array_equal(bo.read(), sentinel)
        bi.write(x)
        assert b200_device.execute(accel.OP_GEMM_F32, mat, bi, bo, rows=m) == accel.OK
        want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
        assert np.array_equal(bo.read().view(np.uint32).reshape(m, n), want.view(np.uint32))
    finally:
        bi.free()
        bo.free()
        mat.destroy()

"""Parity of libbnn_b200.so with the reference on a B200 (marked gpu).

Every comparison is bit-exact: DOT_GROUPS is integer, and the FP32 ops
follow the same per-op rounding as the soft backend, so the bar of the
reference's own conformance test (memcmp of outputs) applies.

  * the reference's unmodified conformance program
    (tests/accelerator/test_bnn_accelerator.c), linked against
    libbnn_b200.so by oracle/Makefile;
  * the reference golden vectors (RTL regression case) through the API;
  * the single-op sweep shapes (Qwen3-1.7B linears), GEMV_F32 and
    DOT_GROUPS, with 2048x151669 chunked like bnn-sw-v2/linear.c:161-216;
  * multi-row GEMM/GEMM_F32, unaligned views, rejection and recovery.
"""
import subprocess

import numpy as np
import pytest

from bnn_b200 import accel, synth

pytestmark = pytest.mark.gpu

MAX_OUT = 8192


def bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and a.tobytes() == b.tobytes()


def test_reference_conformance_program(oracle_mod):
    exe = oracle_mod.ref_tool("b200_conformance")
    if exe is None:
        pytest.skip("oracle/_ref/b200_conformance not built (make -C oracle ref-b200)")
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "successful jobs" in out.stdout


def test_golden_rtl_case(b200_device, golden):
    z = accel.run_op(b200_device, accel.OP_GEMM, golden["bits"], golden["scales"], golden["q_full"])
    assert bits_equal(z.view(np.uint32), golden["golden_full_i8"])
    zt = accel.run_op(b200_device, accel.OP_GEMM, golden["bits"][:, :16], golden["scales"][:, :1],
                      golden["q_tile"])
    assert bits_equal(zt.view(np.uint32), golden["golden_tile_i8"])
    yt = accel.run_op(b200_device, accel.OP_GEMM_F32, golden["bits"][:, :16],
                      golden["scales"][:, :1], golden["x_tile"])
    assert bits_equal(yt.view(np.uint32), golden["golden_tile_f32"])


def chunked_gemv_f32(device, bits, scales, x):
    """GEMV_F32 over out_features > 8192 the way linear.c does it: one input
    buffer, chunks of <= max_out_features rows, one read per chunk."""
    n, kb = bits.shape
    k = kb * 8
    mats = [accel.Matrix(device, bits[o:o + MAX_OUT], scales[o:o + MAX_OUT])
            for o in range(0, n, MAX_OUT)]
    bi, bo = accel.Buffer(device, k * 4), accel.Buffer(device, min(n, MAX_OUT) * 4)
    y = np.empty(n, dtype=np.float32)
    try:
        bi.write(np.ascontiguousarray(x, dtype=np.float32))
        for i, m in enumerate(mats):
            assert device.execute(accel.OP_GEMV_F32, m, bi, bo, rows=1) == accel.OK
            y[i * MAX_OUT:i * MAX_OUT + m.n] = bo.read(m.n * 4).view(np.float32)
    finally:
        bi.free()
        bo.free()
        for m in mats:
            m.destroy()
    return y


@pytest.mark.parametrize("k,n", synth.SWEEP_SHAPES)
def test_sweep_gemv_f32(b200_device, oracle_mod, k, n):
    rng = synth.rng_for(1, salt=k * 7 + n)
    bits, scales = synth.w1_matrix(rng, k, n)
    x = synth.activations(rng, 1, k)
    want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
    got = chunked_gemv_f32(b200_device, bits, scales, x[0])
    assert bits_equal(got.view(np.uint32), want[0].view(np.uint32))


@pytest.mark.parametrize("k,n", synth.SWEEP_SHAPES[:4] + [(2048, 8192)])
def test_sweep_dot_groups(b200_device, oracle_mod, k, n):
    rng = synth.rng_for(1, salt=k * 11 + n)
    bits, scales = synth.w1_matrix(rng, k, n)
    q, _ = oracle_mod.quantize_rows(synth.activations(rng, 1, k))
    want = oracle_mod.dot_groups(bits, scales, q)
    got = accel.run_op(b200_device, accel.OP_DOT_GROUPS, bits, scales, q)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("m", [2, 3, 8, 9, 16, 64, 130, 512])
def test_gemm_f32_rows(b200_device, oracle_mod, m):
    rng = synth.rng_for(3, salt=m)
    k, n = 2048, 320
    bits, scales = synth.w1_matrix(rng, k, n)
    x = synth.activations(rng, m, k)
    want, q, _ = oracle_mod.gemm_f32(bits, scales, x)
    got = accel.run_op(b200_device, accel.OP_GEMM_F32, bits, scales, x)
    assert bits_equal(got.view(np.uint32), want.view(np.uint32))
    z = accel.run_op(b200_device, accel.OP_GEMM, bits, scales, q)
    assert bits_equal(z.view(np.uint32), oracle_mod.gemm_i8(bits, scales, q).view(np.uint32))
    # up to 8 rows the int8 ops run as one kernel that slices the rows itself
    d = accel.run_op(b200_device, accel.OP_DOT_GROUPS, bits, scales, q)
    assert np.array_equal(d, oracle_mod.dot_groups(bits, scales, q))


@pytest.mark.parametrize("op", [accel.OP_GEMM_F32, accel.OP_GEMM, accel.OP_DOT_GROUPS])
def test_unaligned_views(b200_device, oracle_mod, op):
    rng = synth.rng_for(4, salt=op)
    k, n, m = 384, 17, 3
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(b200_device, bits, scales)
    f32 = op == accel.OP_GEMM_F32
    x = synth.activations(rng, m, k) if f32 else synth.i8_activations(rng, m, k)
    in_row = x[0].nbytes
    in_stride, in_off = in_row + 7, 3
    g = k // 128
    out_row = n * g * 2 if op == accel.OP_DOT_GROUPS else n * 4
    out_stride, out_off = out_row + 11, 5
    raw_in = np.full(in_off + m * in_stride + 9, 0xFF if f32 else 0x80, dtype=np.uint8)
    for r in range(m):
        raw_in[in_off + r * in_stride:in_off + r * in_stride + in_row] = x[r].view(np.uint8)
    sentinel = np.full(out_off + m * out_stride + 13, 0xA5, dtype=np.uint8)
    bi, bo = accel.Buffer(b200_device, raw_in.nbytes), accel.Buffer(b200_device, sentinel.nbytes)
    try:
        bi.write(raw_in)
        bo.write(sentinel)
        st = b200_device.execute(op, mat, bi, bo, rows=m, in_offset=in_off, in_stride=in_stride,
                                 out_offset=out_off, out_stride=out_stride)
        assert st == accel.OK
        got = bo.read()
        if f32:
            want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
        elif op == accel.OP_GEMM:
            want = oracle_mod.gemm_i8(bits, scales, x)
        else:
            want = oracle_mod.dot_groups(bits, scales, x)
        expect = sentinel.copy()
        for r in range(m):
            expect[out_off + r * out_stride:out_off + r * out_stride + out_row] = \
                np.ascontiguousarray(want[r]).view(np.uint8).reshape(-1)
        assert bits_equal(got, expect)
        assert bits_equal(bi.read(), raw_in)  # input untouched
    finally:
        bi.free()
        bo.free()
        mat.destroy()


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_nonfinite_rejected_output_untouched_then_recovers(b200_device, oracle_mod, bad):
    rng = synth.rng_for(5)
    k, n, m = 384, 17, 3
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(b200_device, bits, scales)
    x = synth.activations(rng, m, k)
    bi, bo = accel.Buffer(b200_device, x.nbytes), accel.Buffer(b200_device, m * n * 4)
    try:
        sentinel = np.full(m * n * 4, 0x5A, dtype=np.uint8)
        bo.write(sentinel)
        xb = x.copy()
        xb[m - 1, k - 1] = bad  # last element of the last row
        bi.write(xb)
        assert b200_device.execute(accel.OP_GEMM_F32, mat, bi, bo, rows=m) == accel.ERANGE
        assert bits_equal(bo.read(), sentinel)
        bi.write(x)
        assert b200_device.execute(accel.OP_GEMM_F32, mat, bi, bo, rows=m) == accel.OK
        want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
        assert bits_equal(bo.read().view(np.float32).reshape(m, n).view(np.uint32),
                          want.view(np.uint32))
    finally:
        bi.free()
        bo.free()
        mat.destroy()


def test_minus128_rejected_then_recovers(b200_device, oracle_mod):
    rng = synth.rng_for(6)
    k, n, m = 384, 3, 3
    bits, scales = synth.w1_matrix(rng, k, n)
    mat = accel.Matrix(b200_device, bits, scales)
    q = synth.i8_activations(rng, m, k)
    bi, bo = accel.Buffer(b200_device, q.nbytes), accel.Buffer(b200_device, m * n * (k // 128) * 2)
    try:
        for pos in (0, 127, 128, 383):
            sentinel = np.full(bo.nbytes, 0x5A, dtype=np.uint8)
            bo.write(sentinel)
            qb = q.copy()
            qb[1, pos] = -128
            bi.write(qb)
            assert b200_device.execute(accel.OP_DOT_GROUPS, mat, bi, bo, rows=m) == accel.ERANGE
            assert bits_equal(bo.read(), sentinel)
        bi.write(q)
        assert b200_device.execute(accel.OP_DOT_GROUPS, mat, bi, bo, rows=m) == accel.OK
        assert np.array_equal(bo.read().view(np.int16).reshape(m, n, k // 128),
                              oracle_mod.dot_groups(bits, scales, q))
    finally:
        bi.free()
        bo.free()
        mat.destroy()


def test_extremes_and_special_scales(b200_device, oracle_mod):
    """|D| = 16256 extremes, subnormal/zero/negative-zero/max binary16 scales,
    and subnormal activations (scale underflow to FLT_TRUE_MIN)."""
    rng = synth.rng_for(7)
    k, n = 384, 17
    bits, _ = synth.w1_matrix(rng, k, n)
    pool = np.array([0x3C00, 0xBC00, 0x0001, 0x8001, 0x03FF, 0x0400, 0x0000, 0x8000, 0x7BFF],
                    dtype=np.uint16)
    scales = pool[rng.integers(0, pool.size, size=(n, k // 128))]
    signs = np.unpackbits(bits[0], bitorder="little").astype(np.int8) * 2 - 1
    q = np.stack([signs * 127, -signs * 127]).astype(np.int8)
    d = accel.run_op(b200_device, accel.OP_DOT_GROUPS, bits, scales, q)
    assert np.all(d[0, 0] == 16256) and np.all(d[1, 0] == -16256)
    assert np.array_equal(d, oracle_mod.dot_groups(bits, scales, q))
    for mul in (1.0, 2.0 ** -140, 2.0 ** -149, 2.0 ** 120):
        x = (synth.activations(rng, 3, k) * np.float32(mul)).astype(np.float32)
        want, _, _ = oracle_mod.gemm_f32(bits, scales, x)
        got = accel.run_op(b200_device, accel.OP_GEMM_F32, bits, scales, x)
        assert bits_equal(got.view(np.uint32), want.view(np.uint32))


def _unbounded_matrix(device, bits, scales):
    """A matrix past the reference's 8192-row cap (bnn_b200_matrix_create_unbounded,
    how the device engine holds lm_head): its contraction runs several rounds of
    tiles per CTA."""
    import ctypes
    dll = device.api.dll
    fn = dll.bnn_b200_matrix_create_unbounded
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(accel.MatrixDesc), ctypes.POINTER(ctypes.c_void_p)]
    n, kb = bits.shape
    desc = accel.MatrixDesc(kb * 8, n, accel.GROUP, bits.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                            bits.nbytes, scales.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), scales.size)
    h = ctypes.c_void_p()
    assert fn(device.handle, ctypes.byref(desc), ctypes.byref(h)) == accel.OK
    m = accel.Matrix.__new__(accel.Matrix)
    m.device, m.k, m.n, m.handle = device, kb * 8, n, h
    return m


def test_multi_round_tiles(b200_device, oracle_mod):
    """4741 blocks of 8 rows on 2 x 148 CTAs of 8-block tiles: each CTA loops
    over two or three tiles through its shared-memory ring (the last tile
    partly past the matrix). GEMV_F32 and DOT_GROUPS stay bit-exact."""
    rng = synth.rng_for(9, salt=1)
    k, n = 256, 8 * 4741 - 3
    bits, scales = synth.w1_matrix(rng, k, n)
    bits, scales = np.ascontiguousarray(bits), np.ascontiguousarray(scales)
    x = synth.activations(rng, 1, k)
    want, q, _ = oracle_mod.gemm_f32(bits, scales, x)
    m = _unbounded_matrix(b200_device, bits, scales)
    bi, bq, bo, bd = (accel.Buffer(b200_device, k * 4), accel.Buffer(b200_device, k),
                      accel.Buffer(b200_device, n * 4), accel.Buffer(b200_device, n * (k // 128) * 2))
    try:
        bi.write(np.ascontiguousarray(x[0], dtype=np.float32))
        assert b200_device.execute(accel.OP_GEMV_F32, m, bi, bo, rows=1) == accel.OK
        got = bo.read(n * 4).view(np.float32)
        assert bits_equal(got.view(np.uint32), want[0].view(np.uint32))
        bq.write(np.ascontiguousarray(q[0], dtype=np.int8))
        assert b200_device.execute(accel.OP_DOT_GROUPS, m, bq, bd, rows=1) == accel.OK
        d = bd.read(n * (k // 128) * 2).view(np.int16).reshape(1, -1)
        assert np.array_equal(d, oracle_mod.dot_groups(bits, scales, q).reshape(1, -1))
    finally:
        for b in (bi, bq, bo, bd):
            b.free()
        m.destroy()


def test_async_jobs_read_inputs_in_order(b200_device, oracle_mod):
    """Single-kernel F32 jobs enqueued back to back (bnn_b200_execute_async):
    a job may load and quantise its input before the previous kernel ends
    only when no job in flight writes that input. Chains (each job reading
    the previous job's output, through the fixed-G kernel and the general
    one) and independent jobs sharing one input all stay bit-exact."""
    import ctypes
    dll = b200_device.api.dll
    dll.bnn_b200_execute_async.restype = ctypes.c_int
    dll.bnn_b200_execute_async.argtypes = [ctypes.c_void_p, ctypes.POINTER(accel.Job)]
    dll.bnn_b200_sync.restype = ctypes.c_int
    dll.bnn_b200_sync.argtypes = [ctypes.c_void_p]
    rng = synth.rng_for(10, salt=3)
    k, n_big = 2048, 8 * 2600  # 2600 blocks: one block per compute warp, the G = 16 kernel
    sq_bits, sq_scales = (np.ascontiguousarray(a) for a in synth.w1_matrix(rng, k, k))
    big_bits, big_scales = (np.ascontiguousarray(a) for a in synth.w1_matrix(rng, k, n_big))
    sq = accel.Matrix(b200_device, sq_bits, sq_scales)
    big = _unbounded_matrix(b200_device, big_bits, big_scales)
    x = np.ascontiguousarray(synth.activations(rng, 1, k)[0], dtype=np.float32)
    bufs = {}

    def buf(name, n):
        bufs[name] = accel.Buffer(b200_device, n * 4)
        return bufs[name]

    def enqueue(m, src, dst):
        job = accel.Job(operation=accel.OP_GEMV_F32, matrix=m.handle,
                        input=accel.BufferView(src.handle, accel.TYPE_F32, 0, 0),
                        output=accel.BufferView(dst.handle, accel.TYPE_F32, 0, 0), rows=1)
        assert dll.bnn_b200_execute_async(b200_device.handle, ctypes.byref(job)) == accel.OK

    def ref(bits, scales, v):
        out, _, _ = oracle_mod.gemm_f32(bits, scales, v.reshape(1, -1))
        return out[0]

    try:
        buf("x", k).write(x)
        # x -> a -> b -> c through the square matrix; x -> big0; a -> big1 (a in
        # flight); x -> big2 (x is no job's output); c -> big3
        enqueue(sq, bufs["x"], buf("a", k))
        enqueue(big, bufs["x"], buf("big0", n_big))
        enqueue(sq, bufs["a"], buf("b", k))
        enqueue(big, bufs["a"], buf("big1", n_big))
        enqueue(sq, bufs["b"], buf("c", k))
        enqueue(big, bufs["x"], buf("big2", n_big))
        enqueue(big, bufs["c"], buf("big3", n_big))
        assert dll.bnn_b200_sync(b200_device.handle) == accel.OK
        a = ref(sq_bits, sq_scales, x)
        b = ref(sq_bits, sq_scales, a)
        c = ref(sq_bits, sq_scales, b)
        want = {"a": a, "b": b, "c": c, "big0": ref(big_bits, big_scales, x), "big1": ref(big_bits, big_scales, a),
                "big2": ref(big_bits, big_scales, x), "big3": ref(big_bits, big_scales, c)}
        for name, w in want.items():
            got = bufs[name].read(w.size * 4).view(np.float32)
            assert bits_equal(got.view(np.uint32), w.view(np.uint32)), name
    finally:
        for bb in bufs.values():
            bb.free()
        sq.destroy()
        big.destroy()

"""Pins the CPU oracle before it is trusted as the checker (CPU only).

  * the reference's three golden vectors (bnn-hw-v2/simple_test/tests/case,
    re-expressed in tests/golden/rtl_case.npz) reproduce bit-exactly;
  * the Q1_0 block fixture (tools/gguf-lens/test/fixtures/dequant.json)
    decodes to its expected values;
  * binary16 known answers (the literal table of
    tests/accelerator/test_bnn_accelerator.c:28-36 in the reference);
  * on seeded sweeps the oracle matches the reference soft backend itself,
    compiled from its own source into oracle/_ref/ (skipped if absent).
"""
import ctypes

import numpy as np
import pytest

from bnn_b200 import accel, synth

HALF_KNOWN = [(0x3C00, 1.0), (0xBC00, -1.0), (0x3800, 0.5), (0x4000, 2.0),
              (0x0001, 2.0 ** -24), (0x8001, -(2.0 ** -24)), (0x03FF, 1023 * 2.0 ** -24),
              (0x83FF, -1023 * 2.0 ** -24), (0x0400, 2.0 ** -14), (0x8400, -(2.0 ** -14)),
              (0x0000, 0.0), (0x8000, -0.0), (0x3C01, 1.0 + 2.0 ** -10), (0x7BFF, 65504.0)]


def test_golden_full_i8(oracle_mod, golden):
    z = oracle_mod.gemm_i8(golden["bits"], golden["scales"], golden["q_full"])
    assert np.array_equal(z.view(np.uint32), golden["golden_full_i8"])


def test_golden_tile_i8(oracle_mod, golden):
    z = oracle_mod.gemm_i8(golden["bits"][:, :16], golden["scales"][:, :1], golden["q_tile"])
    assert np.array_equal(z.view(np.uint32), golden["golden_tile_i8"])


def test_golden_tile_f32(oracle_mod, golden):
    y, q, s = oracle_mod.gemm_f32(golden["bits"][:, :16], golden["scales"][:, :1], golden["x_tile"])
    assert np.array_equal(y.view(np.uint32), golden["golden_tile_f32"])
    assert np.array_equal(q, golden["q_tile"])
    assert np.all(s == golden["f32_tile_scale"])


def test_q1_0_block_fixture(oracle_mod):
    from pathlib import Path
    d = np.load(Path(__file__).parent / "golden" / "q1_0_block.npz")
    block = d["block"]
    assert block.size == int(d["block_bytes"]) == 18
    scale = oracle_mod.half_to_float(int(block[0]) | (int(block[1]) << 8))
    signs = np.unpackbits(block[2:], bitorder="little").astype(np.float32) * 2 - 1
    assert np.array_equal(np.float32(scale) * signs, d["expected"])


@pytest.mark.parametrize("half,value", HALF_KNOWN)
def test_half_known_answers(oracle_mod, half, value):
    got = oracle_mod.half_to_float(half)
    assert np.float32(got).tobytes() == np.float32(value).tobytes()


def test_quantizer_modes(oracle_mod):
    """Zero row, underflow to FLT_TRUE_MIN, ties away from zero, FLT_MAX."""
    tiny = np.float32(2.0 ** -149)
    rows = np.zeros((4, 128), dtype=np.float32)
    rows[1, 0] = tiny
    rows[2, :4] = [127.0, 0.5, -0.5, 1.5]
    rows[3, :2] = [np.finfo(np.float32).max, -np.finfo(np.float32).max]
    q, s = oracle_mod.quantize_rows(rows)
    assert s[0] == 1.0 and not q[0].any()
    assert s[1].view(np.uint32) == 1 and q[1, 0] == 1
    assert list(q[2, :4]) == [127, 1, -1, 2]
    assert list(q[3, :2]) == [127, -127]


@pytest.fixture(scope="module")
def soft_device(oracle_mod):
    if not oracle_mod.soft_ref_available():
        pytest.skip("reference soft backend not compiled (make -C oracle ref-soft)")
    api = accel.Api(ctypes.CDLL(str(oracle_mod.SOFT_REF_PATH)))
    dev = accel.Device(0, api)
    yield dev
    dev.close()


@pytest.mark.parametrize("k,n,m", [(128, 3, 1), (384, 17, 3), (2048, 64, 2), (8192, 9, 1)])
def test_oracle_matches_soft_backend(oracle_mod, soft_device, k, n, m):
    rng = synth.rng_for(1, salt=k + n)
    bits, scales = synth.w1_matrix(rng, k, n)
    x = synth.activations(rng, m, k)
    y_ref = accel.run_op(soft_device, accel.OP_GEMM_F32, bits, scales, x)
    y, q, _ = oracle_mod.gemm_f32(bits, scales, x)
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    d_ref = accel.run_op(soft_device, accel.OP_DOT_GROUPS, bits, scales, q)
    assert np.array_equal(oracle_mod.dot_groups(bits, scales, q), d_ref)
    z_ref = accel.run_op(soft_device, accel.OP_GEMM, bits, scales, q)
    assert np.array_equal(oracle_mod.gemm_i8(bits, scales, q).view(np.uint32), z_ref.view(np.uint32))


def test_oracle_matches_soft_subnormal_scales(oracle_mod, soft_device):
    rng = synth.rng_for(1, salt=99)
    k, n = 384, 17
    bits, _ = synth.w1_matrix(rng, k, n)
    pool = np.array([h for h, _ in HALF_KNOWN], dtype=np.uint16)
    scales = pool[rng.integers(0, pool.size, size=(n, k // 128))]
    x = synth.activations(rng, 3, k) * np.float32(2.0 ** -140)
    y_ref = accel.run_op(soft_device, accel.OP_GEMM_F32, bits, scales, x)
    y, _, _ = oracle_mod.gemm_f32(bits, scales, x)
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))

"""Parity at the benchmark's own shapes (marked gpu).

The device engine against the reference engine's sources (bnn-sw-v2 engine,
qwen3.c, bnn-mlp.c) at the sizes BASELINE's configs name, bit for bit:

  * a 2-layer model at the full Qwen3-1.7B width (hidden 2048, 16/8 heads of
    128, SwiGLU 6144, vocab 151669): the benchmark's 32-token prompt through
    the batched prefill, teacher-forced logits at 5 positions, and a greedy
    stream of 64 steps identical to the reference's;
  * the full 28-layer configs[2] model (the benchmarked one): the prompt's
    prefill logits and the next two decode steps' logits;
  * configs[3]'s shape at 2 layers: 512 positions prefilled in ONE call, the
    logits of every position equal to the reference's token-by-token
    BNNE_Decode (tools/precision/dump-logits.c:295-306);
  * configs[0] in full: 1000 bnn-mlp samples in calls of 64 (15 full batches
    and the 40-sample tail) against the reference classify over the soft
    backend.

The Qwen3 cases run the reference engine over oracle/bnn_fast_backend.c
(oracle/_ref/libbnn_engine_fast.so): the soft backend takes ~15 s per
full-width token on one core; tests/test_fast_backend.py pins the two
backends bit-identical. The reference's greedy pick is numpy's argmax (first
maximum), as bnn-infer-v2.c:48-54.
"""
import numpy as np
import pytest

from bench import MODEL_SEED, prompt_ids
from bnn_b200 import engine, gguf

pytestmark = pytest.mark.gpu

FULL2 = gguf.Qwen3Shape(layers=2, context=1024)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def ref_mod(oracle_mod):
    import ref_engine
    if not (ref_engine.available() and ref_engine.available(fast=True)):
        pytest.skip("reference engine libraries not built (make -C oracle ref)")
    return ref_engine


@pytest.fixture(scope="module")
def full2(tmp_path_factory):
    return gguf.qwen3_model(tmp_path_factory.mktemp("full2") / "full2.gguf", FULL2, seed=MODEL_SEED)


def test_full_width_prompt_logits_and_greedy_stream(b200_device, ref_mod, full2):
    prompt = prompt_ids(FULL2.vocab)
    forced = np.array([17, 151668, 0, 90210], dtype=np.int32)
    ref = ref_mod.RefEngine(full2, n_ctx=1024, fast=True)
    m = engine.Model(b200_device, full2)
    ctx = engine.Context(m, n_ctx=1024)
    try:
        # the prompt as one call (batched prefill), then four forced tokens
        assert np.array_equal(bits(ctx.decode(prompt)[0]), bits(ref.decode(prompt))), "prompt call"
        for i, t in enumerate(forced):
            assert np.array_equal(bits(ctx.decode([t])[0]), bits(ref.decode([t]))), f"forced token {i}"
    finally:
        ctx.free()
        ref.close()
    ref = ref_mod.RefEngine(full2, n_ctx=1024, fast=True)
    steps = 64
    want = ref.greedy(prompt, steps)
    ref.close()
    ctx = engine.Context(m, n_ctx=1024)
    try:
        assert int(ctx.decode_argmax(prompt)[0]) == want[0]
        got = ctx.generate(steps)[0]
        assert list(got) == want
        assert ctx.pos == len(prompt) + steps - 1
    finally:
        ctx.free()
        m.free()


def test_qwen3_1p7b_prefill_and_two_steps(b200_device, ref_mod, tmp_path):
    path = gguf.qwen3_model(tmp_path / "qwen3_1p7b.gguf", gguf.QWEN3_1_7B, seed=MODEL_SEED)
    prompt = prompt_ids(gguf.QWEN3_1_7B.vocab)
    ref = ref_mod.RefEngine(path, n_ctx=1024, fast=True)
    m = engine.Model(b200_device, path)
    ctx = engine.Context(m, n_ctx=1024)
    try:
        want = ref.decode(prompt)
        got = ctx.decode(prompt)[0]
        assert np.array_equal(bits(got), bits(want)), "prompt (batched prefill)"
        tok = int(np.argmax(want))
        for step in range(2):
            want = ref.decode([tok])
            got = ctx.decode([tok])[0]
            assert np.array_equal(bits(got), bits(want)), f"decode step {step}"
            tok = int(np.argmax(want))
    finally:
        ctx.free()
        m.free()
        ref.close()


def test_prefill_512_per_position_logits(b200_device, ref_mod, full2):
    n = 512
    ids = np.random.default_rng(20261204).integers(0, FULL2.vocab, size=n).astype(np.int32)
    m = engine.Model(b200_device, full2)
    ctx = engine.Context(m, n_ctx=1024)
    try:
        got = ctx.decode_logits_all(ids)  # one call: the batched prefill of all 512 positions
        assert ctx.pos == n
    finally:
        ctx.free()
        m.free()
    ref = ref_mod.RefEngine(full2, n_ctx=1024, fast=True)
    try:
        for p in range(n):  # dump-logits: one BNNE_Decode per token
            want = ref.decode(ids[p:p + 1])
            assert np.array_equal(bits(got[p]), bits(want)), f"position {p}"
    finally:
        ref.close()


def test_classify_config0_all_batches(b200_device, ref_mod, tmp_path):
    path = gguf.bnn_mlp_model(tmp_path / "mlp.gguf")
    batch, n_samples = 64, 1000
    rng = np.random.default_rng(20261201)
    x = np.zeros((n_samples, 896), dtype=np.float32)
    x[:, :784] = rng.standard_normal((n_samples, 784)).astype(np.float32)
    ref = ref_mod.RefEngine(path, n_batch=batch)  # soft backend: the reference itself
    m = engine.Model(b200_device, path)
    ctx = engine.Context(m, n_batch=batch)
    try:
        for b0 in range(0, n_samples, batch):
            want = ref.classify(x[b0:b0 + batch])
            got = ctx.classify(x[b0:b0 + batch])
            assert got.shape == want.shape
            assert np.array_equal(bits(got), bits(want)), f"samples {b0}..{b0 + len(want) - 1}"
            assert np.array_equal(np.argmax(got, axis=1), np.argmax(want, axis=1))
    finally:
        ctx.free()
        m.free()
        ref.close()

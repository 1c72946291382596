"""Device-resident engine vs the reference engine (marked gpu).

The reference engine (bnn-sw-v2 + soft backend, compiled from its own
sources into oracle/_ref/libbnn_engine_soft.so) and BNND_* run the same
seeded synthetic GGUF files:
  * per-position logits under teacher forcing, bit-exact in exact mode;
  * greedy token streams identical over the whole generation;
  * multi-row contexts reproduce the single-row reference per row;
  * bnn-mlp classify logits bit-exact (batch 64);
  * argument/range errors return the reference's status codes;
  * the reference CLI tools linked against libbnn_b200.so (the drop-in)
    dump the same logits as with the soft backend.
Fast mode (tree reductions) is checked against the reference within the
reference's own implementation tolerance, relative L2 of the logits <= 5%
(tools/precision/compare-qwen3.py:233-253): a different summation order
shifts some int8 roundings, and those shifts propagate.
"""
import subprocess

import numpy as np
import pytest

from bnn_b200 import accel, engine, gguf

pytestmark = pytest.mark.gpu

TINY = gguf.Qwen3Shape(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=600,
                       context=256)
SMALL = gguf.Qwen3Shape(layers=3, hidden=1024, heads=8, kv_heads=4, head_dim=128, ffn=2048,
                        vocab=3000, context=512)


@pytest.fixture(scope="module")
def ref_engine_mod(oracle_mod):
    import ref_engine
    if not ref_engine.available():
        pytest.skip("reference engine library not built (make -C oracle ref-soft)")
    return ref_engine


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("models")
    return {
        "tiny": gguf.qwen3_model(d / "tiny.gguf", TINY, seed=11),
        "small": gguf.qwen3_model(d / "small.gguf", SMALL, seed=12, scale_lo=0.02, scale_hi=0.2),
        "mlp": gguf.bnn_mlp_model(d / "mlp.gguf"),
    }


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_teacher_forced_logits_bit_exact(b200_device, ref_engine_mod, models, name):
    shape = TINY if name == "tiny" else SMALL
    rng = np.random.default_rng(5)
    ids = rng.integers(0, shape.vocab, size=12).astype(np.int32)
    ref = ref_engine_mod.RefEngine(models[name], n_ctx=64)
    m = engine.Model(b200_device, models[name])
    ctx = engine.Context(m, n_ctx=64)
    try:
        for i, t in enumerate(ids):
            want = ref.decode([t])
            got = ctx.decode([t])[0]
            assert np.array_equal(bits(got), bits(want)), f"position {i}"
        assert ctx.pos == len(ids)
    finally:
        ctx.free()
        m.free()
        ref.close()


def test_prefill_call_matches_sequential(b200_device, ref_engine_mod, models):
    ids = np.arange(3, 40, 3, dtype=np.int32)
    ref = ref_engine_mod.RefEngine(models["small"], n_ctx=64)
    m = engine.Model(b200_device, models["small"])
    ctx = engine.Context(m, n_ctx=64)
    try:
        want = ref.decode(ids)
        got = ctx.decode(ids)[0]
        assert np.array_equal(bits(got), bits(want))
    finally:
        ctx.free()
        m.free()
        ref.close()


def test_greedy_stream_identical(b200_device, ref_engine_mod, models):
    prompt = np.array([7, 100, 2999, 42, 5, 1000, 77, 1], dtype=np.int32)
    steps = 24
    ref = ref_engine_mod.RefEngine(models["small"], n_ctx=128)
    want = ref.greedy(prompt, steps)
    ref.close()
    m = engine.Model(b200_device, models["small"])
    ctx = engine.Context(m, n_ctx=128)
    try:
        first = ctx.decode_argmax(prompt)
        assert int(first[0]) == want[0]
        got = ctx.generate(steps)[0]
        assert list(got) == want
        assert ctx.pos == len(prompt) + steps - 1
    finally:
        ctx.free()
        m.free()


def test_batched_rows_match_single_row_reference(b200_device, ref_engine_mod, models):
    rows = 3
    rng = np.random.default_rng(9)
    prompts = rng.integers(0, SMALL.vocab, size=(rows, 6)).astype(np.int32)
    m = engine.Model(b200_device, models["small"])
    ctx = engine.Context(m, n_ctx=64, n_batch=rows)
    try:
        got = ctx.decode(prompts)
        gen = ctx.generate(5)
    finally:
        ctx.free()
        m.free()
    for r in range(rows):
        ref = ref_engine_mod.RefEngine(models["small"], n_ctx=64)
        want = ref.decode(prompts[r])
        assert np.array_equal(bits(got[r]), bits(want)), f"row {r}"
        ref.close()
        ref = ref_engine_mod.RefEngine(models["small"], n_ctx=64)
        assert list(gen[r]) == ref.greedy(prompts[r], 5), f"row {r}"
        ref.close()


def test_truncate_and_redecode(b200_device, ref_engine_mod, models):
    ids = np.array([5, 6, 7, 8, 9], dtype=np.int32)
    m = engine.Model(b200_device, models["tiny"])
    ctx = engine.Context(m, n_ctx=32)
    ref = ref_engine_mod.RefEngine(models["tiny"], n_ctx=32)
    try:
        ctx.decode(ids)
        ctx.truncate(2)
        assert ctx.pos == 2
        got = ctx.decode([123])[0]
        ref.decode(ids[:2])
        want = ref.decode([123])
        assert np.array_equal(bits(got), bits(want))
    finally:
        ctx.free()
        m.free()
        ref.close()


def test_range_errors(b200_device, models):
    m = engine.Model(b200_device, models["tiny"])
    ctx = engine.Context(m, n_ctx=8)
    try:
        with pytest.raises(engine.EngineError) as e:
            ctx.decode([TINY.vocab])
        assert e.value.status == engine.ERANGE
        with pytest.raises(engine.EngineError) as e:
            ctx.decode(np.zeros(9, dtype=np.int32))
        assert e.value.status == engine.ERANGE
        assert ctx.pos == 0
        with pytest.raises(engine.EngineError) as e:
            ctx.truncate(1)
        assert e.value.status == engine.EINVAL
        with pytest.raises(engine.EngineError) as e:
            engine.Context(m, n_ctx=TINY.context + 1)
        assert e.value.status == engine.ERANGE
    finally:
        ctx.free()
        m.free()


def test_classify_bit_exact(b200_device, ref_engine_mod, models):
    rng = np.random.default_rng(20261201)
    x = np.zeros((64, 896), dtype=np.float32)
    x[:, :784] = rng.standard_normal((64, 784))
    ref = ref_engine_mod.RefEngine(models["mlp"], n_batch=64)
    want = ref.classify(x)
    ref.close()
    m = engine.Model(b200_device, models["mlp"])
    ctx = engine.Context(m, n_batch=64)
    try:
        got = ctx.classify(x)
        assert np.array_equal(bits(got), bits(want))
        xb = x.copy()
        xb[3, 5] = np.nan
        with pytest.raises(engine.EngineError) as e:
            ctx.classify(xb)
        assert e.value.status == engine.EINVAL
    finally:
        ctx.free()
        m.free()


def test_fast_mode_within_tolerance(b200_device, ref_engine_mod, models):
    ids = np.arange(10, 30, dtype=np.int32)
    ref = ref_engine_mod.RefEngine(models["small"], n_ctx=64)
    want = ref.decode(ids)
    ref.close()
    m = engine.Model(b200_device, models["small"])
    ctx = engine.Context(m, n_ctx=64, exact=False)
    try:
        got = ctx.decode(ids)[0]
    finally:
        ctx.free()
        m.free()
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 0.05, rel


def test_dropin_reference_tools_match(oracle_mod, models, tmp_path):
    soft = oracle_mod.ref_tool("dump-logits-soft")
    b200 = oracle_mod.ref_tool("dump-logits-b200")
    if soft is None or b200 is None:
        pytest.skip("reference tools not built (make -C oracle ref)")
    ids = tmp_path / "ids.txt"
    ids.write_text("1 2 3 4 5 6 7 8\n")
    outs = []
    for exe in (soft, b200):
        out = tmp_path / f"{exe.name}.bin"
        r = subprocess.run([str(exe), "--model", str(models["small"]), "--ids-file", str(ids),
                            "--out", str(out)], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr
        outs.append(out.read_bytes())
    assert outs[0] == outs[1]


# a 40000-row lm_head (5000 blocks: 625 8-block tiles on 296 CTAs) runs more
# than one round of tiles per CTA through the shared-memory ring
ROUNDS = gguf.Qwen3Shape(layers=1, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=40000,
                         context=64)


def test_multi_round_lm_head_logits(b200_device, ref_engine_mod, tmp_path):
    path = gguf.qwen3_model(tmp_path / "rounds.gguf", ROUNDS, seed=14)
    rng = np.random.default_rng(6)
    ids = rng.integers(0, ROUNDS.vocab, size=5).astype(np.int32)
    ref = ref_engine_mod.RefEngine(path, n_ctx=32)
    m = engine.Model(b200_device, path)
    ctx = engine.Context(m, n_ctx=32)
    try:
        for i, t in enumerate(ids):
            want = ref.decode([t])
            got = ctx.decode([t])[0]
            assert np.array_equal(bits(got), bits(want)), f"position {i}"
    finally:
        ctx.free()
        m.free()
        ref.close()


@pytest.mark.parametrize("n", [1, 7, 64, 256, 300])
def test_classify_batch_sizes(b200_device, ref_engine_mod, models, n):
    """Up to 256 samples a call runs as one fused kernel (every layer of a
    sample in one CTA); larger batches run layer by layer on the tensor
    cores. Both are bit-identical to the reference."""
    rng = np.random.default_rng(100 + n)
    x = np.zeros((n, 896), dtype=np.float32)
    x[:, :784] = rng.standard_normal((n, 784))
    ref = ref_engine_mod.RefEngine(models["mlp"], n_batch=n)
    want = ref.classify(x)
    ref.close()
    m = engine.Model(b200_device, models["mlp"])
    ctx = engine.Context(m, n_batch=max(n, 64))
    try:
        got = ctx.classify(x)
        assert np.array_equal(bits(got), bits(want))
    finally:
        ctx.free()
        m.free()


def test_classify_hidden_overflow_rejected(b200_device, ref_engine_mod, tmp_path):
    """post_scale ~1e30: the first layer's outputs overflow to infinity, so
    the second layer's input is rejected as the accelerator rejects a
    non-finite row, by the fused kernel and by the per-layer path alike (and
    the reference fails the call too)."""
    path = gguf.bnn_mlp_model(tmp_path / "big.gguf", seed=5, post_scale_mul=1e30)
    rng = np.random.default_rng(8)
    x = np.zeros((300, 896), dtype=np.float32)
    x[:, :784] = rng.standard_normal((300, 784))
    ref = ref_engine_mod.RefEngine(path, n_batch=8)
    with pytest.raises(RuntimeError):
        ref.classify(x[:8])
    ref.close()
    m = engine.Model(b200_device, path)
    ctx = engine.Context(m, n_batch=300)
    try:
        for n in (8, 300):
            with pytest.raises(engine.EngineError) as e:
                ctx.classify(x[:n])
            assert e.value.status == engine.ERANGE, n
        # the context stays usable
        ok = gguf.bnn_mlp_model(tmp_path / "ok.gguf", seed=5)
        m2 = engine.Model(b200_device, ok)
        ctx2 = engine.Context(m2, n_batch=8)
        try:
            assert np.isfinite(ctx2.classify(x[:8])).all()
        finally:
            ctx2.free()
            m2.free()
    finally:
        ctx.free()
        m.free()

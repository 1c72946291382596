"""Batched prefill on the tensor cores vs one decode step per token (marked gpu).

A decode call of BNND_PREFILL_MIN_TOKENS or more tokens per row runs the
prompt layer by layer over every position at once (prefill_kernels.cuh,
w1a8_mma.cuh). Each output element keeps the decode step's arithmetic, so
logits, the greedy pick, the KV cache (seen through later steps) and the
generated stream must be bit-identical to the same call with
prefill_chunk = 0 (one decode step per token, as the reference's
BNNE_Decode, engine.c:241-273), in exact and in fast mode. The reference
engine itself is compared in test_engine_gpu.py (its prefill-call test
takes the batched path).
"""
import numpy as np
import pytest

from bnn_b200 import engine, gguf

pytestmark = pytest.mark.gpu

TINY = gguf.Qwen3Shape(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=600,
                       context=256)
SMALL = gguf.Qwen3Shape(layers=3, hidden=1024, heads=8, kv_heads=4, head_dim=128, ffn=2048,
                        vocab=3000, context=512)
WIDE = gguf.Qwen3Shape(layers=2, hidden=2048, heads=16, kv_heads=8, head_dim=128, ffn=6144,
                       vocab=4000, context=1024)
# four query heads per KV head, and a context long enough that a tile's
# attention scores no longer fit in shared memory (global scratch path)
LONG = gguf.Qwen3Shape(layers=1, hidden=512, heads=4, kv_heads=1, head_dim=128, ffn=512, vocab=700,
                       context=2048)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("pf_models")
    return {
        "tiny": (gguf.qwen3_model(d / "tiny.gguf", TINY, seed=31), TINY),
        "small": (gguf.qwen3_model(d / "small.gguf", SMALL, seed=32, scale_lo=0.02, scale_hi=0.2), SMALL),
        "wide": (gguf.qwen3_model(d / "wide.gguf", WIDE, seed=33), WIDE),
        "long": (gguf.qwen3_model(d / "long.gguf", LONG, seed=34), LONG),
    }


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def run(dev, path, calls, rows=1, n_ctx=0, exact=True, chunk=engine.PREFILL_CHUNK_DEFAULT, gen=0):
    """Feeds each [rows][n] block of `calls` through decode; returns the logits
    of every call, the generated stream and the final position."""
    m = engine.Model(dev, path)
    ctx = engine.Context(m, n_ctx=n_ctx, n_batch=rows, exact=exact, prefill_chunk=chunk)
    try:
        logits = [ctx.decode(c) for c in calls]
        stream = ctx.generate(gen) if gen else None
        return logits, stream, ctx.pos
    finally:
        ctx.free()
        m.free()


def same(a, b):
    la, sa, pa = a
    lb, sb, pb = b
    assert pa == pb
    for i, (x, y) in enumerate(zip(la, lb)):
        assert np.array_equal(bits(x), bits(y)), f"call {i}"
    if sa is not None:
        assert np.array_equal(sa, sb)


@pytest.mark.parametrize("name", ["tiny", "small", "wide"])
@pytest.mark.parametrize("exact", [True, False])
def test_prefill_matches_steps(b200_device, models, name, exact):
    path, shape = models[name]
    rng = np.random.default_rng(40 + len(name))
    prompt = rng.integers(0, shape.vocab, size=(1, 40)).astype(np.int32)
    want = run(b200_device, path, [prompt], n_ctx=128, exact=exact, chunk=0, gen=6)
    got = run(b200_device, path, [prompt], n_ctx=128, exact=exact, gen=6)
    same(got, want)


def test_prefill_rows_and_chunks(b200_device, models):
    """Three rows, prompts split into chunks of 16 positions (3 passes), then a
    second batched call that starts at position 40."""
    path, shape = models["small"]
    rng = np.random.default_rng(41)
    calls = [rng.integers(0, shape.vocab, size=(3, 40)).astype(np.int32),
             rng.integers(0, shape.vocab, size=(3, 9)).astype(np.int32)]
    want = run(b200_device, path, calls, rows=3, n_ctx=96, chunk=0, gen=5)
    same(run(b200_device, path, calls, rows=3, n_ctx=96, chunk=16, gen=5), want)
    same(run(b200_device, path, calls, rows=3, n_ctx=96, gen=5), want)


def test_prefill_after_steps_and_without_logits(b200_device, models):
    """Short calls (decode steps) before a batched one; a batched call without
    logits followed by a single step."""
    path, shape = models["tiny"]
    rng = np.random.default_rng(42)
    a = rng.integers(0, shape.vocab, size=(1, 3)).astype(np.int32)
    b = rng.integers(0, shape.vocab, size=(1, 30)).astype(np.int32)
    c = rng.integers(0, shape.vocab, size=(1, 1)).astype(np.int32)
    want = run(b200_device, path, [a, b, c], n_ctx=64, chunk=0)
    same(run(b200_device, path, [a, b, c], n_ctx=64), want)

    def no_logits(chunk):
        m = engine.Model(b200_device, path)
        ctx = engine.Context(m, n_ctx=64, prefill_chunk=chunk)
        try:
            assert ctx.decode(b, want_logits=False) is None
            return [ctx.decode(c)], None, ctx.pos
        finally:
            ctx.free()
            m.free()

    same(no_logits(engine.PREFILL_CHUNK_DEFAULT), no_logits(0))


def test_prefill_argmax_and_stream(b200_device, models):
    path, shape = models["small"]
    rng = np.random.default_rng(43)
    prompt = rng.integers(0, shape.vocab, size=(1, 24)).astype(np.int32)
    out = []
    for chunk in (0, engine.PREFILL_CHUNK_DEFAULT):
        m = engine.Model(b200_device, path)
        ctx = engine.Context(m, n_ctx=64, prefill_chunk=chunk)
        try:
            first = ctx.decode_argmax(prompt)
            out.append((int(first[0]), list(ctx.generate(12)[0]), ctx.pos))
        finally:
            ctx.free()
            m.free()
    assert out[0] == out[1]


def test_prefill_long_prompt(b200_device, models):
    """A 512-position prompt in one pass (the prefill configuration's length)
    on the Qwen3-1.7B widths; the sequential run is the oracle."""
    path, shape = models["wide"]
    rng = np.random.default_rng(44)
    prompt = rng.integers(0, shape.vocab, size=(1, 512)).astype(np.int32)
    want = run(b200_device, path, [prompt], n_ctx=600, chunk=0, gen=4)
    same(run(b200_device, path, [prompt], n_ctx=600, gen=4), want)


@pytest.mark.parametrize("exact", [True, False])
def test_prefill_long_context_four_heads_per_kv(b200_device, models, exact):
    """1400 positions, 4 query heads per KV head: the score rows of a tile
    exceed shared memory, so the kernel keeps them in device scratch."""
    path, shape = models["long"]
    rng = np.random.default_rng(45)
    prompt = rng.integers(0, shape.vocab, size=(1, 1400)).astype(np.int32)
    want = run(b200_device, path, [prompt], n_ctx=1500, exact=exact, chunk=0, gen=4)
    same(run(b200_device, path, [prompt], n_ctx=1500, exact=exact, chunk=2048, gen=4), want)
    same(run(b200_device, path, [prompt], n_ctx=1500, exact=exact, chunk=300, gen=4), want)


@pytest.mark.parametrize("exact", [True, False])
def test_multi_row_steps_match_single_rows(b200_device, models, exact):
    """Five context rows: every row is prepared (RMSNorm, quantisation) in
    its own CTA and the contraction reads the sliced rows; every row must
    equal a one-row context fed the same tokens."""
    path, shape = models["small"]
    rng = np.random.default_rng(46)
    rows = 5
    calls = [rng.integers(0, shape.vocab, size=(rows, 20)).astype(np.int32),
             rng.integers(0, shape.vocab, size=(rows, 3)).astype(np.int32)]
    got = run(b200_device, path, calls, rows=rows, n_ctx=96, exact=exact, gen=6)
    for r in range(rows):
        want = run(b200_device, path, [c[r:r + 1] for c in calls], n_ctx=96, exact=exact, gen=6)
        for i, (x, y) in enumerate(zip(got[0], want[0])):
            assert np.array_equal(bits(x[r]), bits(y[0])), f"row {r} call {i}"
        assert np.array_equal(got[1][r], want[1][0]), f"row {r} stream"

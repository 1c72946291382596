"""The persistent decode-step kernel against the per-kernel step graph (marked gpu).

A one-row, exact-mode context runs every decode step with logits as ONE
cooperative kernel (decode_step.cuh) while the K/V history fits an SM's
shared memory, and the per-kernel graph beyond (BNND_StepKernelPositions).
Both must give the same bits: logits of every step, the greedy stream and
the K/V cache as later steps see it, including runs that cross from one
path to the other. BNN_STEP_KERNEL=0 (read at context creation) turns the
step kernel off for the comparison. The reference engine itself is compared
in test_engine_gpu.py and test_parity_full_gpu.py, which take this path.
"""
import os

import numpy as np
import pytest

from bnn_b200 import engine, gguf

pytestmark = pytest.mark.gpu

SHAPES = {
    "tiny": gguf.Qwen3Shape(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=600,
                            context=512),
    "gqa4": gguf.Qwen3Shape(layers=2, hidden=512, heads=4, kv_heads=1, head_dim=128, ffn=1536, vocab=1000,
                            context=512),
    "wide": gguf.Qwen3Shape(layers=2, hidden=2048, heads=16, kv_heads=8, head_dim=128, ffn=6144,
                            vocab=5000, context=512),
}


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def run(dev, path, prompt, forced, gen, step_kernel):
    os.environ["BNN_STEP_KERNEL"] = "1" if step_kernel else "0"
    try:
        m = engine.Model(dev, path)
        ctx = engine.Context(m, n_ctx=512)
    finally:
        os.environ.pop("BNN_STEP_KERNEL", None)
    try:
        positions = ctx.step_kernel_positions()
        logits = [ctx.decode(prompt)[0]]
        logits += [ctx.decode([t])[0] for t in forced]
        stream = ctx.generate(gen)[0]
        logits.append(ctx.decode([int(stream[-1])])[0])
        return positions, logits, stream, ctx.pos
    finally:
        ctx.free()
        m.free()


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_step_kernel_matches_per_kernel_graph(b200_device, tmp_path, name):
    shape = SHAPES[name]
    path = gguf.qwen3_model(tmp_path / f"{name}.gguf", shape, seed=61)
    rng = np.random.default_rng(62)
    prompt = rng.integers(0, shape.vocab, size=5).astype(np.int32)
    forced = rng.integers(0, shape.vocab, size=6).astype(np.int32)
    on = run(b200_device, path, prompt, forced, 40, True)
    off = run(b200_device, path, prompt, forced, 40, False)
    assert on[0] > 60, "the step kernel should serve these positions"
    assert off[0] == 0
    assert on[3] == off[3]
    for i, (a, b) in enumerate(zip(on[1], off[1])):
        assert np.array_equal(bits(a), bits(b)), f"call {i}"
    assert np.array_equal(on[2], off[2])


def test_step_kernel_hands_over_past_its_positions(b200_device, tmp_path):
    """A greedy run that starts below the step kernel's position limit and
    ends beyond it (the per-kernel graph continues on the same cache)."""
    shape = SHAPES["gqa4"]
    path = gguf.qwen3_model(tmp_path / "gqa4.gguf", shape, seed=63)
    os.environ["BNN_STEP_KERNEL"] = "1"
    try:
        m = engine.Model(b200_device, path)
        ctx = engine.Context(m, n_ctx=512)
    finally:
        os.environ.pop("BNN_STEP_KERNEL", None)
    limit = ctx.step_kernel_positions()
    ctx.free()
    m.free()
    assert 0 < limit < 480
    rng = np.random.default_rng(64)
    prompt = rng.integers(0, shape.vocab, size=limit - 20).astype(np.int32)  # batched prefill
    forced = rng.integers(0, shape.vocab, size=4).astype(np.int32)
    on = run(b200_device, path, prompt, forced, 40, True)
    off = run(b200_device, path, prompt, forced, 40, False)
    assert on[3] == off[3] > limit
    for i, (a, b) in enumerate(zip(on[1], off[1])):
        assert np.array_equal(bits(a), bits(b)), f"call {i}"
    assert np.array_equal(on[2], off[2])

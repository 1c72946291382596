"""Host-side pieces of bench.py (no GPU): the roofline denominators and the
committed ncu traffic figure, and the reference CPU baseline sample (one
token through the reference engine, whatever the shape of the prompt)."""
import json
import tempfile
from pathlib import Path

import numpy as np
import pytest

import bench

ROOT = Path(__file__).resolve().parents[1]


def test_measured_peaks_from_driver_file():
    p = ROOT / "MEASURED_PEAKS.json"
    hbm, kind = bench.measured_peaks()
    if p.exists():
        assert kind == "measured"
        assert hbm == float(json.loads(p.read_text())["hbm_gbs"])
    else:
        assert (hbm, kind) == (6650.0, "fallback")


def test_ncu_traffic_keyed_by_metric():
    d = json.loads((ROOT / "profiles" / "roofline_traffic.json").read_text())
    assert bench.ncu_traffic(bench.METRIC) == d[bench.METRIC]
    # one batch-1 decode launch per contraction: within 5 % of its algorithmic bytes
    assert abs(d[bench.METRIC] / 2178287 - 1.0) < 0.05
    # no capture of the 8-context workload is committed: no traffic figure for it
    assert bench.ncu_traffic(bench.METRIC + "_8ctx") is None


def test_cpu_baseline_sample_is_one_token():
    import ref_engine
    if not ref_engine.available():
        pytest.skip("reference engine library not built (make -C oracle ref-soft)")
    from bnn_b200 import gguf
    shape = gguf.Qwen3Shape(layers=1, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=300,
                            context=bench.CTX)
    with tempfile.TemporaryDirectory() as d:
        path = gguf.qwen3_model(Path(d) / "m.gguf", shape, seed=3)
        for prompt in (np.arange(32, dtype=np.int32), np.zeros((8, 64), dtype=np.int32)):
            rate, seconds = bench.cpu_baseline_sample(path, prompt)
            assert rate == pytest.approx(1.0 / seconds)
            # a 1-layer, 256-wide step takes milliseconds; a whole prompt row
            # (64 steps) would take tens of times longer
            assert seconds < 0.5


class _FakeContext:
    """Positions and the logits flag as the engine keeps them (BNND_Decode*,
    BNND_Generate, BNND_ContextTruncate), recording the position of every
    decoded step."""

    def __init__(self, n_prompt, n_ctx):
        self.pos, self.n_ctx, self.have_logits, self.steps = n_prompt, n_ctx, True, []

    def truncate(self, pos):
        assert pos <= self.pos
        self.pos, self.have_logits = pos, False

    def decode_argmax(self, tok):
        assert self.pos + 1 <= self.n_ctx
        self.steps.append(self.pos)
        self.pos += 1
        self.have_logits = True
        return np.asarray(tok) + 1

    def generate(self, s):
        assert self.have_logits and s >= 1 and self.pos + s - 1 <= self.n_ctx
        self.steps.extend(range(self.pos, self.pos + s - 1))
        self.pos += s - 1


@pytest.mark.parametrize("total", [0, 1, 5, 128, 129, 256, 300])
def test_timed_steps_repeat_the_configured_generation(total):
    n_prompt, gen_steps = bench.PROMPT_TOKENS, bench.GEN_STEPS
    first = np.array([7], dtype=np.int32)
    for per_token in (False, True):
        ctx = _FakeContext(n_prompt, bench.CTX)
        if per_token:
            bench.run_generations_per_token(ctx, first, n_prompt, gen_steps, total)
        else:
            assert bench.run_generations(ctx, ctx.generate, first, n_prompt, gen_steps, total) == total
        assert len(ctx.steps) == total
        # every step at a position of the configured generation, in repeats
        # that each start right after the prompt
        want = [n_prompt + i % gen_steps for i in range(total)]
        assert ctx.steps == want


def test_reference_arm_times_configured_positions(monkeypatch, tmp_path):
    """--impl reference on a 1-layer model: the forked copies decode from the
    end of the prompt, steps x ms_per_step is the slowest copy's time, and the
    config block is the device arm's."""
    import argparse
    import ref_engine
    if not ref_engine.available():
        pytest.skip("reference engine library not built (make -C oracle ref-soft)")
    from bnn_b200 import gguf
    shape = gguf.Qwen3Shape(layers=1, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=300,
                            context=bench.CTX)
    path = gguf.qwen3_model(tmp_path / "m.gguf", shape, seed=3)
    monkeypatch.setattr(bench, "model_path", lambda cache: path)
    args = argparse.Namespace(steps=6, ref_procs=3, model_cache=str(tmp_path))
    out = bench.run_reference(args)
    assert out["impl"] == "reference" and out["steps"] == 6
    assert out["value"] == pytest.approx(out["steps"] / (out["steps"] * out["ms_per_step"] / 1e3), rel=1e-2)
    assert out["config"] == bench.decode_config(bench.gguf_shape(), bench.GEN_STEPS, bench.PROMPT_TOKENS,
                                                bench.CTX, 1, bench.WORKLOAD)
    assert f"positions {bench.PROMPT_TOKENS}..{bench.PROMPT_TOKENS + 1}" in out["cpu_baseline"]["sample"]

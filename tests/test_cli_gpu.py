"""The engine's command line (bnn-infer-b200) against the reference CLI
(bnn-infer-v2.c, compiled from the reference sources with the reference's
CPU accelerator as oracle/_ref/bnn-infer-v2-soft): on the same files and
arguments, the same exit status and byte-identical standard output, for text
generation (default prompt, --prompt, --chat, --ids, --steps 0, a context
that fills up, an EOG stop, and each input error) and classification (with
and without labels, --verbose, batches that do and do not divide the sample
count, and each input error)."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "bnn-train-infer_b200" / "lib" / "bnn-infer-b200"
SHAPE = dict(layers=2, hidden=256, heads=2, kv_heads=1, head_dim=128, ffn=512, context=1024)
PROMPT = "kato's RIne 2024 — 日本語?"


@pytest.fixture(scope="module")
def tools(oracle_mod):
    ref = oracle_mod.ref_tool("bnn-infer-v2-soft")
    if ref is None:
        pytest.skip("reference CLI not built (make -C oracle ref)")
    assert CLI.exists(), "bnn-infer-b200 not built: make -C bnn-train-infer_b200"
    return CLI, ref


@pytest.fixture(scope="module")
def vocab():
    from bnn_b200 import gguf
    return gguf.bpe_vocabulary(seed=7)


@pytest.fixture(scope="module")
def llm_path(tmp_path_factory, vocab):
    from bnn_b200 import gguf
    shape = gguf.Qwen3Shape(vocab=len(vocab.tokens), **SHAPE)
    return gguf.qwen3_model(tmp_path_factory.mktemp("cli") / "llm.gguf", shape, seed=19, vocab=vocab)


@pytest.fixture(scope="module")
def mlp(tmp_path_factory):
    from bnn_b200 import gguf
    d = tmp_path_factory.mktemp("cli_mlp")
    path = gguf.bnn_mlp_model(d / "mlp.gguf", seed=8)
    rng = np.random.default_rng(12)
    n = 37
    x = rng.random((n, gguf.MNIST_MLP.dims[0]), dtype=np.float32)  # ModelInfo.input_size
    (d / "x.bin").write_bytes(x.tobytes())
    (d / "y.bin").write_bytes(rng.integers(0, 10, size=n, dtype=np.uint8).tobytes())
    (d / "y_short.bin").write_bytes(bytes(n - 1))
    (d / "y_range.bin").write_bytes(bytes(n - 1) + b"\x0a")
    (d / "x_ragged.bin").write_bytes(x.tobytes()[:-4])
    (d / "empty.bin").write_bytes(b"")
    return path, d


def _same(tools, args, cwd, expect_rc=0):
    mine, ref = tools
    want = subprocess.run([str(ref), *map(str, args)], capture_output=True, timeout=900, cwd=cwd)
    got = subprocess.run([str(mine), *map(str, args)], capture_output=True, timeout=900, cwd=cwd)
    assert want.returncode == expect_rc, want.stderr
    assert got.returncode == want.returncode, (got.stderr, want.stderr)
    assert got.stdout == want.stdout, (got.stdout[-200:], want.stdout[-200:])
    return got


def _prompt_len(dev, path, text):
    from bnn_b200 import engine
    m = engine.Model(dev, path)
    try:
        return len(m.tokenize(text, True))
    finally:
        m.free()


@pytest.mark.parametrize("args", [
    [],
    ["--prompt", PROMPT, "--steps", "24", "--ctx", "96"],
    ["--chat", "--prompt", "hi there", "--steps", "16", "--ctx", "128"],
    ["--chat", "--steps", "6"],
    ["--prompt", PROMPT, "--steps", "0", "--ctx", "64"],
    ["--prompt", PROMPT, "--steps", "1", "--ctx", "64"],
    ["--prompt", "x", "--steps", "300", "--ctx", "1024"],
], ids=["defaults", "prompt", "chat", "chat-default-prompt", "steps0", "steps1", "long"])
def test_llm_output_matches_reference(tools, llm_path, tmp_path, args):
    r = _same(tools, ["llm", llm_path, *args], tmp_path)
    assert r.stdout.endswith(b"\n")


def test_llm_ids_file(tools, llm_path, tmp_path):
    (tmp_path / "ids.txt").write_text("1 2 3\n  40\t5 \n")
    _same(tools, ["llm", llm_path, "--ids", "ids.txt", "--steps", "9", "--ctx", "32"], tmp_path)


def test_llm_context_fills_up(tools, b200_device, llm_path, tmp_path):
    n = _prompt_len(b200_device, llm_path, PROMPT)
    for extra in (1, 2, 5):
        _same(tools, ["llm", llm_path, "--prompt", PROMPT, "--steps", "40", "--ctx", n + extra], tmp_path)


@pytest.mark.parametrize("case", ["no-room", "prompt-overflows", "ctx-over-model", "empty-prompt",
                                  "ids-trailing", "ids-range", "ids-too-many", "ids-empty", "ids-missing",
                                  "classify-model", "missing-model"])
def test_llm_errors_match_reference(tools, b200_device, llm_path, mlp, tmp_path, case):
    n = _prompt_len(b200_device, llm_path, PROMPT)
    (tmp_path / "trail.txt").write_text("1 2 x")
    (tmp_path / "range.txt").write_text("1 1000000")
    (tmp_path / "many.txt").write_text(" ".join(["7"] * 9))
    (tmp_path / "empty.txt").write_text(" \n")
    args = {
        "no-room": ["--prompt", PROMPT, "--ctx", n],
        "prompt-overflows": ["--prompt", PROMPT, "--ctx", n - 1],
        "ctx-over-model": ["--ctx", 1025],
        "empty-prompt": ["--prompt", ""],
        "ids-trailing": ["--ids", "trail.txt"],
        "ids-range": ["--ids", "range.txt"],
        "ids-too-many": ["--ids", "many.txt", "--ctx", 8],
        "ids-empty": ["--ids", "empty.txt"],
        "ids-missing": ["--ids", "nope.txt"],
    }.get(case)
    model = {"classify-model": mlp[0], "missing-model": tmp_path / "nope.gguf"}.get(case, llm_path)
    _same(tools, ["llm", model, *(args or [])], tmp_path, expect_rc=1)


def test_llm_no_room_is_fine_without_steps(tools, b200_device, llm_path, tmp_path):
    n = _prompt_len(b200_device, llm_path, PROMPT)
    _same(tools, ["llm", llm_path, "--prompt", PROMPT, "--ctx", n, "--steps", "0"], tmp_path)


def test_llm_stops_at_eog(tools, vocab, tmp_path):
    """A model whose greedy output reaches a new token after a few steps,
    saved again with eos_token_id set to that token: both CLIs stop before
    it."""
    import ref_engine
    from bnn_b200 import gguf
    if not ref_engine.available():
        pytest.skip("reference engine library not built (oracle/_ref)")
    shape = gguf.Qwen3Shape(vocab=len(vocab.tokens), **SHAPE)
    a = gguf.qwen3_model(tmp_path / "a.gguf", shape, seed=22, vocab=vocab)
    ref = ref_engine.RefEngine(a, n_ctx=64)
    try:
        _, ids = ref.tokenize_raw(PROMPT, 1)
        seq = [int(np.argmax(ref.decode(ids)))]
        for _ in range(15):
            seq.append(int(np.argmax(ref.decode([seq[-1]]))))
    finally:
        ref.close()
    k = next((i for i in range(2, len(seq)) if seq[i] not in seq[:i]), None)
    assert k is not None, seq
    b = gguf.qwen3_model(tmp_path / "b.gguf", shape, seed=22,
                         vocab=gguf.BpeVocab(vocab.tokens, vocab.types, vocab.merges, seq[k]))
    full = _same(tools, ["llm", a, "--prompt", PROMPT, "--steps", "16", "--ctx", "64"], tmp_path)
    cut = _same(tools, ["llm", b, "--prompt", PROMPT, "--steps", "16", "--ctx", "64"], tmp_path)
    assert len(cut.stdout) < len(full.stdout)


@pytest.mark.parametrize("args", [
    ["--input", "x.bin"],
    ["--input", "x.bin", "--labels", "y.bin"],
    ["--input", "x.bin", "--labels", "y.bin", "--verbose", "--batch", "5"],
    ["--input", "x.bin", "--verbose", "--batch", "100"],
    ["--input", "x.bin", "--labels", "y.bin", "--batch", "37"],
    ["--input", "x.bin", "--verbose", "--batch", "1"],
], ids=["plain", "labels", "verbose-b5", "verbose-b100", "b37", "b1"])
def test_classify_output_matches_reference(tools, mlp, args):
    path, d = mlp
    r = _same(tools, ["classify", path, *args], d)
    assert b"class counts:" in r.stdout


@pytest.mark.parametrize("args", [
    ["--input", "x_ragged.bin"],
    ["--input", "empty.bin"],
    ["--input", "nope.bin"],
    ["--input", "x.bin", "--labels", "y_short.bin"],
    ["--input", "x.bin", "--labels", "y_range.bin"],
    ["--input", "x.bin", "--labels", "nope.bin"],
], ids=["ragged", "empty", "missing", "labels-short", "labels-range", "labels-missing"])
def test_classify_errors_match_reference(tools, mlp, args):
    path, d = mlp
    _same(tools, ["classify", path, *args], d, expect_rc=1)


def test_classify_rejects_language_model(tools, llm_path, mlp):
    _same(tools, ["classify", llm_path, "--input", "x.bin"], mlp[1], expect_rc=1)

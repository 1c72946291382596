"""Argument rules of the engine's command line (bnn-train-infer_b200/cli/
bnn_infer_b200.cpp) against the reference CLI (bnn-infer-v2.c, compiled from
the reference sources as oracle/_ref/bnn-infer-v2-soft): every malformed
command line is rejected with the usage text and exit status 1 before a
device is opened, and well-formed ones are not. CPU only: on a host without
a GPU the well-formed lines then fail at BNN_DeviceOpen, which still shows
that they passed the parser."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "bnn-train-infer_b200" / "lib" / "bnn-infer-b200"

MALFORMED = [
    [],
    ["foo"],
    ["LLM", "m.gguf"],
    ["llm"],
    ["llm", "m.gguf", "--prompt", "a", "--ids", "f"],
    ["llm", "m.gguf", "--prompt", "a", "--prompt", "b"],
    ["llm", "m.gguf", "--ids", "f", "--ids", "g"],
    ["llm", "m.gguf", "--steps"],
    ["llm", "m.gguf", "--steps", "-1"],
    ["llm", "m.gguf", "--steps", "+1"],
    ["llm", "m.gguf", "--steps", "1x"],
    ["llm", "m.gguf", "--steps", " 1"],
    ["llm", "m.gguf", "--steps", ""],
    ["llm", "m.gguf", "--steps", "4294967296"],
    ["llm", "m.gguf", "--steps", "99999999999999999999999"],
    ["llm", "m.gguf", "--steps", "1", "--steps", "2"],
    ["llm", "m.gguf", "--ctx", "0"],
    ["llm", "m.gguf", "--ctx", "8", "--ctx", "8"],
    ["llm", "m.gguf", "--chat", "--chat"],
    ["llm", "a.gguf", "b.gguf"],
    ["llm", "m.gguf", "--unknown"],
    ["llm", "-"],
    ["llm", "--chat"],
    ["classify", "m.gguf"],
    ["classify", "--input", "f"],
    ["classify", "m.gguf", "--input"],
    ["classify", "m.gguf", "--input", "f", "--input", "g"],
    ["classify", "m.gguf", "--input", "f", "--labels"],
    ["classify", "m.gguf", "--input", "f", "--labels", "a", "--labels", "b"],
    ["classify", "m.gguf", "--input", "f", "--batch", "0"],
    ["classify", "m.gguf", "--input", "f", "--batch", "-3"],
    ["classify", "m.gguf", "--input", "f", "--batch", "2", "--batch", "2"],
    ["classify", "m.gguf", "--input", "f", "--verbose", "--verbose"],
    ["classify", "m.gguf", "--input", "f", "--steps", "3"],
    ["classify", "a.gguf", "b.gguf", "--input", "f"],
]

WELL_FORMED = [
    ["llm", "missing.gguf"],
    ["llm", "missing.gguf", "--steps", "4294967295"],
    ["llm", "missing.gguf", "--steps", "0", "--ctx", "007"],
    ["llm", "missing.gguf", "--chat", "--prompt", "", "--ctx", "1"],
    ["llm", "--ids", "f", "missing.gguf"],
    ["classify", "missing.gguf", "--input", "f"],
    ["classify", "--batch", "1", "--labels", "l", "--verbose", "--input", "f", "missing.gguf"],
]


@pytest.fixture(scope="module")
def cli():
    if not CLI.exists():
        pytest.skip("CLI not built (make -C bnn-train-infer_b200)")
    return CLI


def _run(exe, args):
    return subprocess.run([str(exe), *args], capture_output=True, timeout=120)


@pytest.mark.parametrize("args", MALFORMED, ids=lambda a: " ".join(a) or "<none>")
def test_malformed_command_lines(cli, oracle_mod, args):
    r = _run(cli, args)
    assert r.returncode == 1 and r.stdout == b"" and r.stderr.startswith(b"usage: "), r
    ref = oracle_mod.ref_tool("bnn-infer-v2-soft")
    if ref is not None:
        want = _run(ref, args)
        assert want.returncode == 1 and want.stdout == b"" and want.stderr.startswith(b"usage: "), want


@pytest.mark.parametrize("args", WELL_FORMED, ids=" ".join)
def test_well_formed_command_lines(cli, oracle_mod, tmp_path, args):
    r = subprocess.run([str(cli), *args], capture_output=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 1 and r.stdout == b"", r
    assert r.stderr.startswith(b"error: ") and b"usage" not in r.stderr, r.stderr
    ref = oracle_mod.ref_tool("bnn-infer-v2-soft")
    if ref is not None:
        want = subprocess.run([str(ref), *args], capture_output=True, timeout=300, cwd=tmp_path)
        assert want.returncode == 1 and want.stderr.startswith(b"error: "), want


def test_stats_flag_is_an_extension(cli):
    """--stats (timings on standard error) is accepted once per command."""
    for args in (["llm", "missing.gguf", "--stats"], ["classify", "missing.gguf", "--input", "f", "--stats"]):
        assert b"usage" not in _run(cli, args).stderr
        assert _run(cli, args + ["--stats"]).stderr.startswith(b"usage: ")


def test_usage_names_the_program(cli):
    r = _run(cli, [])
    lines = r.stderr.decode().splitlines()
    assert lines[0] == f"usage: {cli} llm MODEL.gguf [--prompt TEXT | --ids FILE]"
    assert lines[2].startswith(f"       {cli} classify MODEL.gguf --input FILE")
    assert all(len(l) - len(l.lstrip()) == len(str(cli)) + 8 for l in (lines[1], lines[3]))

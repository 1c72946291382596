"""The exact parallel form of the reference's serial sum of squares
(bnn-train-infer_b200/csrc/exact_sum.cuh, the RMSNorm sum of qwen3.c:361-372)
checked on the host: tests/exact_sum_host.cpp replays the 256-thread
algorithm and the 512-thread wide form (exact_sumsq_wide) with the header's own host-callable pieces and the device code's
order of float operations, and compares each result bit for bit with the
serial loop, over six families of vectors (normal, outliers, 2^-60..2^50
magnitudes, half-ulp ties, tiny/huge/zero mixes, 16K..64K lengths). The
device kernels are compared with the reference on the GPU in the engine
tests; this pins the algorithm itself. A planted mistake (runs off by one
unit) must be caught."""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("esum") / "exact_sum_host"
    subprocess.run(["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math",
                    "-I", str(ROOT / "bnn-train-infer_b200" / "csrc"), "-o", str(out),
                    str(ROOT / "tests" / "exact_sum_host.cpp")], check=True)
    return out


def _run(exe, *args):
    r = subprocess.run([str(exe), *map(str, args)], capture_output=True, text=True, timeout=300)
    m = re.search(r"checked (\d+) mismatches (\d+)", r.stdout)
    assert m, r.stdout + r.stderr
    return r, int(m.group(1)), int(m.group(2))


@pytest.mark.parametrize("form", ["", "wide"])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_parallel_sum_bit_exact(exe, seed, form):
    r, checked, bad = _run(exe, 300, seed, form) if form else _run(exe, 300, seed)
    assert checked == 1800 and bad == 0, r.stdout
    assert r.returncode == 0
    # the run path (the parallel shortcut) is taken, not only serial replays
    runs = [int(x) for x in re.findall(r"ops: (\d+) runs", r.stdout)]
    assert len(runs) == 6 and min(runs) > 100, r.stdout


@pytest.mark.parametrize("form", ["", "wide"])
def test_planted_mistake_is_caught(exe, form):
    r, checked, bad = _run(exe, 40, 7, "plant", form) if form else _run(exe, 40, 7, "plant")
    assert bad > 0 and r.returncode == 1, r.stdout

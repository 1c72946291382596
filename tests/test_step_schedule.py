"""The copy schedule of the persistent decode-step kernel, on the CPU.

bnn-train-infer_b200/csrc/step_schedule.h is plain C++: this test compiles it
with g++ into a small harness and checks, for the Qwen3-1.7B shape and for
small shapes, with rings from roomy to tight:
  * every copy fits the ring, 128-byte aligned, in one piece;
  * no copy overlaps any copy that may still be live when it is issued
    (copies need .. i-1), at most kSlots copies are live, and `need` never
    decreases (the producer releases in order);
  * the block ranges of the contraction CTAs partition every matrix exactly
    (q|k|v, o/down rows, gate|up pairs, lm_head), and every CTA's copies
    carry exactly its blocks.
"""
import json
import shutil
import subprocess

import pytest

from conftest import PKG

HARNESS = r"""
#include <cstdio>
#include <cstdlib>
#include "step_schedule.h"
using namespace bnn::step;
int main(int argc, char** argv) {
    ScheduleShape s{(uint32_t)atoi(argv[1]), (uint32_t)atoi(argv[2]), (uint32_t)atoi(argv[3]),
                    (uint32_t)atoi(argv[4]), (uint32_t)atoi(argv[5]), (uint32_t)atoi(argv[6]),
                    (uint32_t)atoi(argv[7])};
    std::vector<LayerSrc> layers(s.layers);
    for (uint32_t l = 0; l < s.layers; ++l)
        layers[l] = LayerSrc{(1ull << 40) * (l + 1), (1ull << 40) * (l + 1) + (1ull << 36),
                             (1ull << 40) * (l + 1) + (2ull << 36), (1ull << 40) * (l + 1) + (3ull << 36),
                             (1ull << 40) * (l + 1) + (4ull << 36), (1ull << 40) * (l + 1) + (5ull << 36)};
    std::printf("[");
    for (uint32_t j = 0; j < s.n_gemv; ++j) {
        std::vector<Copy> c;
        if (!build_schedule(s, layers, 1ull << 50, 1ull << 51, j, &c)) {
            std::printf("%s\"fail\"", j ? "," : "");
            continue;
        }
        std::printf("%s[", j ? "," : "");
        for (size_t i = 0; i < c.size(); ++i)
            std::printf("%s[%llu,%u,%u,%u,%u]", i ? "," : "", (unsigned long long)c[i].src, c[i].bytes,
                        c[i].ring_off, c[i].need, c[i].blocks);
        std::printf("]");
    }
    std::printf("]\n");
    return 0;
}
"""

SLOTS = 16
LM_CHUNK = 16


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no host C++ compiler")
    d = tmp_path_factory.mktemp("sched")
    src = d / "h.cpp"
    src.write_text(HARNESS)
    exe = d / "h"
    subprocess.run([gxx, "-std=c++17", "-O1", f"-I{PKG / 'csrc'}", str(src), "-o", str(exe)], check=True)
    return exe


def run(exe, layers, hidden, ffn, qkv_rows, vocab, n_gemv, ring):
    out = subprocess.run([str(exe)] + [str(v) for v in (layers, hidden, ffn, qkv_rows, vocab, n_gemv, ring)],
                         capture_output=True, text=True, check=True).stdout
    return json.loads(out)


def split(j, n, nb):
    return j * nb // n, (j + 1) * nb // n


@pytest.mark.parametrize("shape,n_gemv,ring", [
    ((28, 2048, 6144, 4096, 151669), 132, 150 * 1024),
    ((28, 2048, 6144, 4096, 151669), 132, 48 * 1024),
    ((2, 256, 512, 512, 600), 146, 64 * 1024),
    ((3, 1024, 2048, 2048, 3000), 140, 20 * 1024),
])
def test_schedule_ring_and_ownership(harness, shape, n_gemv, ring):
    layers, hidden, ffn, qkv_rows, vocab = shape
    scheds = run(harness, layers, hidden, ffn, qkv_rows, vocab, n_gemv, ring)
    assert len(scheds) == n_gemv and "fail" not in scheds
    gc, gf = hidden // 128, ffn // 128
    bbc, bbf = gc * 144, gf * 144
    nb_qkv, nb_c, np_gu, nb_v = qkv_rows // 8, hidden // 8, ffn // 8, (vocab + 7) // 8
    owned = {"qkv": [], "o": [], "gu": [], "v": []}
    for j, copies in enumerate(scheds):
        prev_need = 0
        for i, (src, nbytes, off, need, blocks) in enumerate(copies):
            assert off % 128 == 0 and nbytes % 16 == 0 and off + nbytes <= ring
            assert prev_need <= need <= i and i - need < SLOTS
            prev_need = need
            for k in range(need, i):
                o2, b2 = copies[k][2], copies[k][1]
                assert not (o2 < off + nbytes and off < o2 + b2), f"CTA {j}: copy {i} overlaps live copy {k}"
        # the copies carry exactly this CTA's ranges, in the kernel's order
        q0, q1 = split(j, n_gemv, nb_qkv)
        o0, o1 = split(j, n_gemv, nb_c)
        p0, p1 = split(j, n_gemv, np_gu)
        v0, v1 = split(j, n_gemv, nb_v)
        want = []
        for _ in range(layers):
            if q1 > q0:
                want += [(hidden * 4, 0), ((q1 - q0) * bbc, q1 - q0)]
            if o1 > o0:
                want += [((o1 - o0) * bbc, o1 - o0)]
            if p1 > p0:
                want += [(hidden * 4, 0), (2 * (p1 - p0) * bbc, 2 * (p1 - p0))]
            if o1 > o0:
                want += [((o1 - o0) * bbf, o1 - o0)]
        if v1 > v0:
            want += [(hidden * 4, 0)]
            want += [(min(LM_CHUNK, v1 - b) * bbc, min(LM_CHUNK, v1 - b)) for b in range(v0, v1, LM_CHUNK)]
        assert [(c[1], c[4]) for c in copies] == want
        owned["qkv"].append((q0, q1))
        owned["o"].append((o0, o1))
        owned["gu"].append((p0, p1))
        owned["v"].append((v0, v1))
    for name, total in (("qkv", nb_qkv), ("o", nb_c), ("gu", np_gu), ("v", nb_v)):
        covered = [b for b0, b1 in owned[name] for b in range(b0, b1)]
        assert covered == list(range(total)), name

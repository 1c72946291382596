#!/usr/bin/env python3
"""Regenerate the committed golden fixtures from the reference tree.

Run once where a checkout of the reference is available (--ref); the
outputs are committed, so the machines that run the tests never need it.

Outputs
  rtl_case.npz   the reference's fixed W1A8 regression case
                 (bnn-hw-v2/simple_test/tests/case/: memory.img, meta.json,
                 golden_{full_i8,tile_i8,tile_f32}.hex), re-expressed in the
                 public BNN_MatrixDesc layout:
                   bits        uint8  [512][64]   row-major weight bits
                   scales      uint16 [512][4]    binary16 patterns
                   q_full      int8   [16][512]   GEMM input, K=512
                   q_tile      int8   [16][128]   GEMM input, K=128
                   x_tile      float32[16][128]   GEMM_F32 input, K=128
                   golden_full_i8 / golden_tile_i8 / golden_tile_f32
                               uint32 [16][512]   FP32 bit patterns
  q1_0_block.npz one Q1_0 block and its dequantised values, from
                 tools/gguf-lens/test/fixtures/dequant.json (key "Q1_0"):
                 scale first (LE fp16), then 128 LSB-first sign bits.

The memory image stores the weights as 18-byte Q1_0 records ordered
[n_block 4][k_group 4][channel 128] at 0x1000; the inputs sit at the
addresses in meta.json (gen_model_case.py:47-53, 222-239 in the reference).
"""
import argparse
import os
import base64
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_hex(path):
    words = [int(line, 16) for line in path.read_text().splitlines()
             if line and not line.startswith("#")]
    return np.asarray(words, dtype=np.uint32)


def rtl_case(ref):
    case = ref / "bnn-hw-v2/simple_test/tests/case"
    meta = json.loads((case / "meta.json").read_text())
    image = np.frombuffer((case / "memory.img").read_bytes(), dtype=np.uint8)
    k, n, rows = meta["matrix"]["in_features"], meta["matrix"]["out_features"], meta["rows"]
    group = meta["matrix"]["group_size"]
    addr = meta["addresses"]
    n_blocks, k_groups = n // group, k // group

    records = image[addr["weights"]:addr["weights"] + n * k_groups * 18].reshape(
        n_blocks, k_groups, group, 18)
    # -> [n][k_group][18]
    blocks = records.transpose(0, 2, 1, 3).reshape(n, k_groups, 18)
    scales = blocks[:, :, 0:2].copy().view("<u2").reshape(n, k_groups).astype(np.uint16)
    bits = np.ascontiguousarray(blocks[:, :, 2:]).reshape(n, k // 8)

    def region(name, count, dtype):
        start = addr[name]
        nbytes = count * np.dtype(dtype).itemsize
        return image[start:start + nbytes].view(dtype).copy()

    q_full = region("int8_full_input", rows * k, np.int8).reshape(rows, k)
    q_tile = region("int8_tile_input", rows * group, np.int8).reshape(rows, group)
    x_tile = region("f32_tile_input", rows * group, "<f4").astype(np.float32).reshape(rows, group)
    out = dict(bits=bits, scales=scales, q_full=q_full, q_tile=q_tile, x_tile=x_tile,
               f32_tile_scale=np.float32(meta["f32_tile_scale"]))
    for w in meta["workloads"]:
        out["golden_" + w["name"]] = load_hex(case / w["golden"]).reshape(rows, n)
    np.savez_compressed(HERE / "rtl_case.npz", **out)
    return out


def q1_0_block(ref):
    data = json.loads((ref / "tools/gguf-lens/test/fixtures/dequant.json").read_text())["Q1_0"]
    raw = np.frombuffer(base64.b64decode(data["bytes"]), dtype=np.uint8)
    expected = np.asarray(data["expected"], dtype=np.float32)
    np.savez_compressed(HERE / "q1_0_block.npz", block=raw, expected=expected,
                        block_elems=np.int64(data["block"]), block_bytes=np.int64(data["size"]))


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref", type=Path,
                    default=Path(os.environ.get("BNN_REFERENCE") or HERE.parents[2] / "reference"),
                    help="reference checkout (default: $BNN_REFERENCE, else 'reference' beside the repo root)")
    args = ap.parse_args()
    rtl_case(args.ref)
    q1_0_block(args.ref)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()

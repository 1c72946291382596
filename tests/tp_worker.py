"""One rank of the tensor-parallel engine check (launched by tests/test_tp_gpu.py
through torch.distributed.run, one process per GPU).

Every rank loads its column shard of the same synthetic Qwen3 model and
decodes the same prompt and greedy continuation; rank 0 also runs the
unsharded engine on its GPU. The sharded logits and tokens must be
bit-identical to the unsharded ones (each output element's arithmetic does
not change under out_features sharding). The NCCL id is handed around over a
gloo process group; prints "TP OK <world>" on success.
"""
import datetime
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "bnn-train-infer_b200"), str(ROOT)]

# One node: NCCL's bootstrap over loopback, its root at a fixed address that
# rank 0 opens when the communicator is created.
os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
os.environ.setdefault("NCCL_COMM_ID", f"127.0.0.1:{int(os.environ.get('MASTER_PORT', '29500')) + 1}")

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from bnn_b200 import accel, engine, gguf  # noqa: E402

SHAPE = gguf.Qwen3Shape(layers=3, hidden=1024, heads=8, kv_heads=4, head_dim=128, ffn=2048, vocab=3000,
                        context=512)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    path = Path(os.environ["BNN_TP_MODEL"])
    if rank == 0 and not path.exists():
        gguf.qwen3_model(path, SHAPE, seed=31, scale_lo=0.02, scale_hi=0.2)
    dist.barrier()
    dev = accel.Device(rank)
    api = engine.EngineApi(dev.api.dll)
    box = [engine.comm_id_create(api) if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    rng = np.random.default_rng(5)
    for rows in (1, 3, 5):  # 5: every row prepared in its own CTA (sliced contraction)
        prompt = rng.integers(0, SHAPE.vocab, size=(rows, 12), dtype=np.int32)
        model = engine.Model(dev, path, api, world=world, rank=rank)
        ctx = engine.Context(model, n_ctx=256, n_batch=rows, comm_id=box[0])
        logits = ctx.decode(prompt)
        nxt = ctx.decode_argmax(np.argmax(logits, axis=1).astype(np.int32))
        gen = ctx.generate(20)
        last = ctx.decode(gen[:, -1])
        ctx.free()
        model.free()
        if rank == 0:
            ref_model = engine.Model(dev, path, api)
            ref = engine.Context(ref_model, n_ctx=256, n_batch=rows)
            rl = ref.decode(prompt)
            rn = ref.decode_argmax(np.argmax(rl, axis=1).astype(np.int32))
            rg = ref.generate(20)
            rlast = ref.decode(rg[:, -1])
            ref.free()
            ref_model.free()
            assert np.array_equal(logits.view(np.uint32), rl.view(np.uint32)), f"prompt logits differ (rows {rows})"
            assert np.array_equal(nxt, rn) and np.array_equal(gen, rg), f"greedy tokens differ (rows {rows})"
            assert np.array_equal(last.view(np.uint32), rlast.view(np.uint32)), f"final logits differ (rows {rows})"
        dist.barrier()
        toks = [None] * world
        dist.all_gather_object(toks, gen.tolist())
        assert all(t == toks[0] for t in toks), "ranks disagree on the greedy tokens"
    dev.close()
    dist.barrier()
    if rank == 0:
        print(f"TP OK {world}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

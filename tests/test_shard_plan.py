"""Host side of tensor parallelism: BNND_ShardPlan's row ranges, computed by
2, 4 and 8 gloo ranks on CPU, partition every matrix exactly (whole GQA groups for
q|k|v, matching gate/up ranges, 8-row lm_head stride), and shapes that do not
split are refused. No GPU is needed."""
import datetime
import os
import sys
from pathlib import Path

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "bnn-train-infer_b200"), str(ROOT)]


def _info(engine, heads=16, kv_heads=8, hd=128, hidden=2048, ffn=6144, vocab=151669):
    info = engine.ModelInfo()
    info.task = engine.TASK_LLM
    info.heads, info.kv_heads, info.head_dim = heads, kv_heads, hd
    info.hidden, info.ffn, info.n_vocab = hidden, ffn, vocab
    return info


SHAPES = (dict(), dict(vocab=3000, hidden=1024, heads=8, kv_heads=4, ffn=2048))


def _splits(shape, world):
    return shape.get("kv_heads", 8) % world == 0 and shape.get("heads", 16) % world == 0


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from bnn_b200 import _lib, engine
    api = engine.EngineApi(_lib.load())
    for shape in (s for s in SHAPES if _splits(s, world)):
        info = _info(engine, **shape)
        p = engine.shard_plan(api, info, world, rank)
        mine = {f: getattr(p, f) for f, _ in engine.ShardInfo._fields_}
        plans = [None] * world
        dist.all_gather_object(plans, mine)
        if rank == 0:
            out.put((shape, plans))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_plans_partition_every_matrix(world):
    from bnn_b200 import engine
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, 29641 + world, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for s in SHAPES if _splits(s, world)]
    assert results
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for shape, plans in results:
        info = _info(engine, **shape)
        for key, total, unit in (("q", info.heads * info.head_dim, info.head_dim * info.heads // info.kv_heads),
                                 ("kv", info.kv_heads * info.head_dim, info.head_dim),
                                 ("c", info.hidden, 8), ("f", info.ffn, 8)):
            covered = 0
            for p in plans:
                assert p[key + "_begin"] == covered and p[key + "_rows"] % unit == 0
                covered += p[key + "_rows"]
            assert covered == total
        covered = 0
        for p in plans:
            assert p["v_stride"] % 8 == 0 and p["v_begin"] == covered
            covered += p["v_rows"]
        assert covered == info.n_vocab


def test_unsplittable_shapes_refused():
    from bnn_b200 import _lib, engine
    api = engine.EngineApi(_lib.load())
    with pytest.raises(engine.EngineError) as e:
        engine.shard_plan(api, _info(engine, heads=2, kv_heads=1, hidden=256, ffn=512), 2, 0)
    assert e.value.status == engine.ENOTSUP
    with pytest.raises(engine.EngineError) as e:
        engine.shard_plan(api, _info(engine), 2, 2)
    assert e.value.status == engine.EINVAL

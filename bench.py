#!/usr/bin/env python3
"""Benchmark: Qwen3-1.7B-shape W1A8 greedy decode tokens/s on B200.

Workload: random-init Qwen3-1.7B architecture
(28 layers, hidden 2048, 16 q / 8 kv heads of 128, SwiGLU 6144, vocab 151669,
tied Q1_0 embedding/lm_head, RMSNorm gains ~N(1, 0.02), rope theta 1e6), a
32-token seeded prompt, 128 greedy steps at ctx 1024, batch 1. A step is
one decoded token: one pass of the device-resident engine over the whole
model (241.9 MB of Q1_0 weights streamed from HBM per token, larger than
L2). The K timed steps repeat the 128-step generation: each repeat rewinds
the context to the end of the (cached) prompt and feeds the prompt's first
pick, so every timed step decodes at a position of the configured workload.

value     tokens/s of BNND_Generate with everything resident on the device,
          timed with CUDA events on the engine's stream (max over ranks).
e2e       the same through the public per-token call BNND_DecodeArgmax with
          host token ids in and the host argmax out every step (4 B each way).
text_stream  the same generation as streamed text (BNND_GenerateStream, a
          host piece callback per token, device steps queued ahead), wall clock.
other_configs  (one-GPU runs) short timed runs of configs[3] (--prefill),
          configs[0] (--classify) and configs[1]'s 2048x151669 GEMV_F32
          (--sweep), each with its own roofline, e2e and clocks, so every
          BASELINE config is measured in the default line.
roofline  the W1A8 contraction kernel (the step's dominant kernel), from an
          instrumented replay of the same step graph: algorithmic bytes
          (N*K*0.140625 + 4K + 4N per linear) / its device time, against the
          measured HBM copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline  the reference engine itself (bnn-sw-v2 + soft backend, compiled
          from its sources into oracle/_ref) decoding one token of the same
          model on one host core.

--config5 measures BASELINE configs[4]: 8 independent contexts (one context
row each) with 64-token seeded prompts, 256 greedy steps at ctx 4096; every
linear is a GEMV of 8 rows; with --tp under torchrun the model is
column-sharded over the ranks. value is the aggregate tokens/s.

--prefill measures BASELINE configs[3] instead: a step is one batched
prefill of 512 seeded prompt tokens (every linear a GEMM of 512 rows on the
tensor cores, tcgen05 kind::i8) plus the greedy pick of the next token,
through BNND_DecodeArgmax with host ids in and out; value is prompt
tokens/s, the roofline the int8 tensor rate of the whole prefill.

--sweep measures BASELINE configs[1]: GEMV_F32 and DOT_GROUPS at the Qwen3
linear shapes (K x N = 2048x2048, 2048x1024, 2048x6144, 6144x2048,
2048x151669), rows = 1. Kernel time is CUDA events around each job on the
device's stream with L2 flushed (a 256 MB write, read back) before every job
and, for 2048x151669, also as a stream of jobs over 8 device copies of the
matrix (the value); GB/s is
the algorithmic bytes (N*K*0.140625 + 4K + 4N for GEMV_F32, N*K/8 + K + 2NK/128
for DOT_GROUPS) over that time. e2e is the full synchronous call with host
buffers (BufferWrite, BNN_Execute, BufferRead; 2048x151669 through 19 jobs of
at most 8192 rows, as linear.c does). value is GEMV_F32 GB/s at 2048x151669.

--classify measures BASELINE configs[0]: the bnn-mlp classifier
(896->512 relu, 512->512 relu, 512->10) over 1000 seeded samples in batches
of 64 through BNND_Classify (each linear a 64-row GEMM_F32 on the tensor
cores), host samples in and logits out per call; value is samples/s.

--impl reference runs only the reference's CPU path: one soft-engine process
per host core (it is single-threaded), each decoding tokens of the same
model, and reports their aggregate tokens/s.

Multi-GPU (torchrun, one rank per GPU): every rank decodes its own replica
(independent sequences, no collective on the data path): weak scaling.
--tp instead decodes one sequence with the model column-sharded over the
ranks (NCCL all-gathers inside the step graph): strong scaling, value is the
tokens/s of that one sequence.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "bnn-train-infer_b200"), str(ROOT / "oracle")]

METRIC = "qwen3_1p7b_w1a8_decode_tokens_per_s"
PROMPT_TOKENS = 32
CTX = 1024
GEN_STEPS = 128          # configs[2]: greedy steps after the prompt
GEN_STEPS_8CTX = 256     # configs[4]
MODEL_SEED = 20261203  # rng_for(config index 2)
PROMPT_SEED = 20261203 + 7
WORKLOAD = ("configs[2]: Qwen3-1.7B-shape W1A8 greedy decode, random-init weights, "
            "32-token seeded prompt, 128 greedy steps, ctx 1024, batch 1")
PREFILL_METRIC = "qwen3_1p7b_w1a8_prefill_tokens_per_s"
PREFILL_TOKENS = 512
PREFILL_SEED = 20261204  # rng_for(config index 3)
PREFILL_WORKLOAD = ("configs[3]: Qwen3-1.7B-shape W1A8 prefill of 512 seeded tokens in one pass "
                    "(GEMM rows=512 on the tcgen05 int8 path), random-init weights, ctx 1024")


DATA = "synthetic (seeded random-init weights and prompt; no checkpoint offline)"


def gguf_shape():
    from bnn_b200 import gguf
    return gguf.QWEN3_1_7B


def decode_config(shape, gen_steps, n_prompt, n_ctx, batch, workload):
    """The workload description both arms print (identical for the same config)."""
    weights = shape.weights()
    return {"workload": workload, "prompt_tokens": n_prompt, "ctx": n_ctx, "greedy_steps": gen_steps,
            "timed": (f"decode steps of the {gen_steps}-step greedy generation after the prompt "
                      f"(positions {n_prompt}..{n_prompt + gen_steps - 1})"),
            "batch": batch, "layers": shape.layers, "hidden": shape.hidden, "ffn": shape.ffn,
            "vocab": shape.vocab, "weight_bytes_per_token": int(weights * 0.140625),
            "l2": "inputs larger than L2: 242 MB of weights streamed per token vs 126 MB L2"}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def run_generations(ctx, generate, first, n_prompt, gen_steps, total):
    """Decodes `total` steps as repeats of the configured greedy generation.
    Each repeat rewinds to the end of the prompt (whose K/V stay cached),
    feeds the prompt's first pick and decodes up to `gen_steps` steps, i.e.
    positions n_prompt .. n_prompt + gen_steps - 1 of the real greedy stream,
    so every timed step is a step of the configured workload at its position.
    generate(s) runs s - 1 further steps after a decode with logits (the
    first of its s ids is the pick that decode made)."""
    done = 0
    while done < total:
        s = min(gen_steps, total - done)
        ctx.truncate(n_prompt)
        ctx.decode_argmax(first)  # the step at position n_prompt
        if s > 1:
            generate(s)
        done += s
    return done


def run_generations_per_token(ctx, first, n_prompt, gen_steps, total):
    """run_generations through the per-token public call (host ids in and
    out every step); returns the last ids."""
    done, tok = 0, first
    while done < total:
        s = min(gen_steps, total - done)
        ctx.truncate(n_prompt)
        tok = first
        for _ in range(s):
            tok = ctx.decode_argmax(tok)
        done += s
    return tok


def stream_block(ctx, first, n_prompt, gen_steps):
    """The configured generation as streamed text: BNND_GenerateStream hands
    each token's piece to a host callback while the device runs up to four
    steps ahead (the reference CLI's loop, bnn-infer-v2.c:253-282). Wall
    clock around the public calls (rewind, the step at position n_prompt,
    the stream), as a user sees it; tokens = ids handed out (the stream stops
    early at an EOG token)."""
    pieces = []

    def on_piece(_tok, piece):
        pieces.append(piece)
        return False

    def one():
        pieces.clear()
        ctx.truncate(n_prompt)
        ctx.decode_argmax(first)
        return ctx.generate_stream(gen_steps, on_piece)

    one()
    one()
    t0 = time.perf_counter()
    ids = one()
    wall = time.perf_counter() - t0
    return {"value": round(len(ids) / wall, 2), "unit": "tokens/s", "tokens": int(len(ids)),
            "bytes_out": sum(len(p) for p in pieces), "wall_ms": round(wall * 1e3, 3),
            "call": "BNND_GenerateStream with a Python piece callback, wall clock"}


def model_path(cache):
    cache = Path(cache)
    cache.mkdir(parents=True, exist_ok=True)
    p = cache / f"qwen3_1p7b_seed{MODEL_SEED}.gguf"
    if not p.exists():
        from bnn_b200 import gguf
        tmp = p.with_suffix(f".tmp{os.getpid()}")
        t0 = time.time()
        gguf.qwen3_model(tmp, gguf.QWEN3_1_7B, seed=MODEL_SEED)
        os.replace(tmp, p)
        log(f"generated {p} in {time.time() - t0:.1f}s")
    return p


def prompt_ids(vocab):
    import numpy as np
    return np.random.default_rng(PROMPT_SEED).integers(0, vocab, size=PROMPT_TOKENS).astype(np.int32)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(prefix="clocks", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.out.close()

    def summary(self):
        rows = []
        try:
            for line in Path(self.out.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(rows), "reasons": reasons}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(metric):
    """Per-launch DRAM bytes of the contraction kernel from the committed ncu
    summary (profiles/roofline_traffic.json), if one matches this workload's
    metric (None otherwise)."""
    p = ROOT / "profiles" / "roofline_traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(metric)
    except (ValueError, OSError):
        return None


def cpu_baseline_sample(path, prompt):
    """One decode step of the same model through the reference engine (soft
    backend, one core). Returns (tokens/s, seconds) or None."""
    import ref_engine
    if not ref_engine.available():
        return None
    import numpy as np
    first = np.asarray(prompt).reshape(-1)[:1]  # one token (configs[4] passes [rows][prompt])
    ref = ref_engine.RefEngine(path, n_ctx=CTX)
    try:
        t0 = time.perf_counter()
        ref.decode(first)
        dt = time.perf_counter() - t0
    finally:
        ref.close()
    return 1.0 / dt, dt


def run_b200(args):
    import numpy as np
    import torch
    from bnn_b200 import accel, engine

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    tp = args.tp and world > 1
    dist = None
    if world > 1:
        # the engine owns the data-path NCCL communicator of the sharded runs
        # (bootstrap root at a fixed loopback address); the process group
        # (gloo) only coordinates the host: barriers and the max over ranks
        os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
        os.environ.setdefault("NCCL_COMM_ID", f"127.0.0.1:{int(os.environ.get('MASTER_PORT', '29500')) + 1}")
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    torch.cuda.set_device(local)

    if rank == 0 or world == 1:
        path = model_path(args.model_cache)
    if dist:
        dist.barrier()
        path = model_path(args.model_cache)

    dev = accel.Device(local)
    api = engine.EngineApi(dev.api.dll)
    t0 = time.time()
    model = engine.Model(dev, path, api, world=world if tp else 1, rank=rank if tp else 0)
    log(f"[rank {rank}] model loaded in {time.time() - t0:.1f}s")
    info = model.info
    batch, n_ctx, n_prompt = (8, 4096, 64) if args.config5 else (1, CTX, PROMPT_TOKENS)
    if args.config5:
        prompt = np.random.default_rng(20261205).integers(0, info.n_vocab, size=(batch, n_prompt)).astype(np.int32)
    else:
        prompt = prompt_ids(info.n_vocab)
    comm_id = None
    if tp:
        box = [engine.comm_id_create(api) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm_id = box[0]
    ctx = engine.Context(model, n_ctx=n_ctx, n_batch=batch, exact=not args.fast, comm_id=comm_id)
    stream = torch.cuda.ExternalStream(ctx.stream())
    launches_per_step = ctx.step_launches()

    def timed(fn, on=None):
        """Device time of fn() on stream `on` (the context's), max over ranks."""
        on = stream if on is None else on
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(on)
        fn()
        e1.record(on)
        e1.synchronize()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms])
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    if args.prefill:
        out = run_prefill(args, ctx, info, timed, rank, world)
        ctx.free()
        model.free()
        dev.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return out

    # ---- device-resident value: the K timed steps repeat the configured
    # greedy generation after the prompt (positions n_prompt ..
    # n_prompt + gen_steps - 1), K / gen_steps times
    first = ctx.decode_argmax(prompt)            # prefill (untimed); the prompt's first pick
    gen_steps = GEN_STEPS_8CTX if args.config5 else GEN_STEPS
    if n_prompt + gen_steps + 1 > n_ctx:
        raise SystemExit(f"prompt + {gen_steps} steps must fit ctx {n_ctx}")
    gen = api.Generate

    def generate(s):
        api.check(gen(ctx.handle, s, None))

    run_generations(ctx, generate, first, n_prompt, gen_steps, args.warmup)  # warm-up steps
    with ClockSampler(local) as clocks:
        ms = timed(lambda: run_generations(ctx, generate, first, n_prompt, gen_steps, args.steps))
    clk = clocks.summary()
    streams = batch * (1 if tp else world)  # sequences decoded by the whole job
    value = args.steps * streams / (ms / 1e3)

    # ---- end to end through the public per-token call (host ids in/out)
    run_generations_per_token(ctx, first, n_prompt, gen_steps, args.warmup)
    host_tok = np.empty(batch, dtype=np.int32)

    def e2e_loop():
        host_tok[:] = run_generations_per_token(ctx, first, n_prompt, gen_steps, args.steps)

    ms_e2e = timed(e2e_loop)
    e2e_value = args.steps * streams / (ms_e2e / 1e3)
    text_stream = stream_block(ctx, first, n_prompt, gen_steps) if batch == 1 and not tp else None

    step_positions = ctx.step_kernel_positions()
    timed_pos = [n_prompt + i % gen_steps for i in range(args.steps)]
    if batch == 1 and not tp and step_positions > max(timed_pos):
        # ---- the whole step is ONE kernel (decode_step_kernel): its time is the
        # event-timed step; algorithmic bytes per token: Q1_0 weights (0.140625
        # bytes each) + K/V history read + K/V append + norm gains + embed row
        peak, peak_kind = measured_peaks()
        kv_row = info.n_layers * info.kv_heads * info.head_dim * 4 * 2
        gains = (2 * info.n_layers + 1) * info.hidden * 4 + 2 * info.n_layers * info.head_dim * 4
        weight_bytes_step = info.weight_count * 0.140625
        bytes_per_step = (weight_bytes_step + kv_row * statistics.mean(p + 1 for p in timed_pos) + kv_row + gains
                          + info.hidden // 8 + info.hidden // 128 * 2)
        kernel_ms = ms / args.steps
        achieved = bytes_per_step / (kernel_ms / 1e3) / 1e9
        assert achieved <= peak, "algorithmic bytes per step / step time above the HBM peak"
        roofline = {
            "kernel": "decode_step_kernel", "dominant_kernel": "decode_step_kernel", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "peak_source": peak_kind, "traffic": ncu_traffic(METRIC + "_step_kernel"),
            "launches_per_step": 1, "bytes_per_step": round(bytes_per_step),
            "kernel_ms_per_step": round(kernel_ms, 4), "share_of_step": 1.0,
            "method": ("one persistent kernel per decode step (graph of one cooperative launch): its time is "
                       "the event-timed step; bytes = Q1_0 weights + K/V history read at the timed positions + "
                       "K/V append + norm gains + embedding row"),
        }
        launches_per_step = 1
    else:
        roofline = None
    # ---- roofline of the dominant kernel of the per-kernel step graph
    # (instrumented replay of the same step), when that graph is the timed path
    if roofline is None:
        roofline = per_kernel_roofline(args, ctx, prompt, ms)

    # ---- configs[3] on the same model and GPU (one GPU jobs only): the
    # batched 512-token prefill, a short timed run inside this line
    others = {}
    if world == 1 and not (args.config5 or args.no_other_configs):
        others["configs[3]"] = _brief(run_prefill(_sub_args(args), ctx, info, timed, rank, world))

    # ---- the sharded design on this job's GPUs: configs[4] with every linear
    # column-sharded over the ranks (a single GPU at N = 1), so the scaling
    # run records it at 1, 2, 4 and 8 GPUs next to the replicas
    tp_info = None
    if not (args.config5 or args.no_tp_block) and (info.heads % world == 0 and info.kv_heads % world == 0):
        ctx.free()
        tp_info = tp_block(args, dev, api, path, world, rank, dist, timed, engine)
        ctx = None

    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            sample = cpu_baseline_sample(path, prompt)
            if sample:
                cpu = {"value": round(sample[0], 6), "unit": "tokens/s", "cores": 1, "kind": "reference",
                       "sample": f"one decode step (position 0, with lm_head) of the same model through the "
                                 f"reference engine + soft backend built from its sources, 1 thread: "
                                 f"{sample[1]:.2f} s"}
        weight_bytes = info.weight_count * 0.140625
        workload = WORKLOAD
        if args.config5:
            workload = ("configs[4]: Qwen3-1.7B-shape W1A8, 8 independent contexts with 64-token seeded prompts, "
                        "256 greedy steps at ctx 4096" + (f", column-sharded over {world} GPUs" if tp else ""))
        out = {
            "metric": METRIC + ("_8ctx" if args.config5 else ""), "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "int8",
            "data": DATA,
            "config": decode_config(gguf_shape(), gen_steps, n_prompt, n_ctx, batch, workload),
            "impl_config": {"numerics": "fast" if args.fast else "exact (reference operation order)",
                            "decode_step": ("one persistent kernel per token (decode_step_kernel)"
                                            if roofline.get("kernel") == "decode_step_kernel"
                                            else "per-kernel step graph"),
                            "parallelism": (f"tensor parallel x{world} (column-sharded linears, NCCL all-gather)"
                                            if tp else f"replicas x{world}" if world > 1 else "single GPU")},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4 * batch,
                    "d2h_bytes_per_step": 4 * batch, "call": "BNND_DecodeArgmax per token, host ids in and out"},
            "clocks": clk,
            "gpu_launches": int(launches_per_step * args.steps),
        }
        if text_stream:
            out["text_stream"] = text_stream
        if tp_info:
            out["tp"] = tp_info
    if ctx is not None:
        ctx.free()
    model.free()
    dev.close()
    if others:
        # configs[0] and configs[1] need their own model / matrices: after
        # this model is gone, each a short timed run of its own mode
        others["configs[0]"] = _brief(run_classify(_sub_args(args)))
        others["configs[1]"] = _brief(run_sweep(_sub_args(args, sweep_shape="2048x151669")))
        if out is not None:
            out["other_configs"] = others
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return out


def _sub_args(args, **kw):
    """The options of a short block inside the default line: 8 timed steps
    after 3 warm-up steps."""
    sub = argparse.Namespace(**vars(args))
    sub.steps, sub.warmup, sub.sweep_shape = 8, 3, None
    for k, v in kw.items():
        setattr(sub, k, v)
    return sub


def _brief(line):
    """A mode's JSON line without the keys the enclosing line already holds."""
    if line is None:
        return None
    keep = ("metric", "value", "unit", "steps", "warmup", "ms_per_step", "config", "roofline", "e2e", "clocks")
    return {k: line[k] for k in keep if k in line}


def tp_block(args, dev, api, path, world, rank, dist, timed, engine):
    """BASELINE configs[4] on `world` GPUs with the model column-sharded over
    them (one GPU at world 1): 8 contexts with 64-token seeded prompts,
    greedy steps at ctx 4096 (the timed steps repeat the 256-step generation
    from the end of the prompts). Returns the block for the bench line."""
    import numpy as np
    comm = None
    if world > 1:
        box = [engine.comm_id_create(api) if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = box[0]
    model = engine.Model(dev, path, api, world=world, rank=rank)
    batch, n_prompt, gen_steps = 8, 64, GEN_STEPS_8CTX
    prompt = np.random.default_rng(20261205).integers(0, model.info.n_vocab, size=(batch, n_prompt)).astype(np.int32)
    ctx = engine.Context(model, n_ctx=4096, n_batch=batch, comm_id=comm)
    try:
        first = ctx.decode_argmax(prompt)

        def generate(s):
            api.check(api.Generate(ctx.handle, s, None))

        steps = args.tp_steps
        run_generations(ctx, generate, first, n_prompt, gen_steps, 3)
        import torch
        ms = timed(lambda: run_generations(ctx, generate, first, n_prompt, gen_steps, steps),
                   torch.cuda.ExternalStream(ctx.stream()))
        # The all-gathers of the instrumented replay absorb any skew between
        # the ranks' starts; the first replay also builds and uploads the
        # instrumented graph, at a different speed on every rank. So one
        # replay is discarded and the ranks meet before the measured one.
        for keep in (False, True):
            ctx.truncate(n_prompt)
            ctx.decode_argmax(first)
            if keep and dist is not None:
                dist.barrier()
            stats, total = ctx.profile(2 if keep else 1)
        gather = sum(v[1] for k, v in stats.items() if k.startswith("all_gather"))
        return {"workload": "configs[4]: 8 contexts, 64-token prompts, greedy steps at ctx 4096",
                "world": world, "value": round(steps * batch / (ms / 1e3), 2), "unit": "tokens/s",
                "ms_per_step": round(ms / steps, 4), "steps": steps,
                "parallelism": (f"column-sharded linears over {world} GPUs, NCCL all-gathers" if world > 1
                                else "single GPU"),
                "allgather_share": round(gather / total, 4) if total > 0 else None}
    finally:
        ctx.free()
        model.free()


def per_kernel_roofline(args, ctx, prompt, ms):
    """Roofline of the W1A8 contraction in the per-kernel step graph: its
    share of an instrumented replay times the event-timed step."""
    ctx.truncate(0)
    ctx.decode_argmax(prompt)
    stats, total_ms = ctx.profile(args.profile_steps)

    by_kernel = {}
    for name, (launches, kms, kbytes) in stats.items():
        key = "w1a8_contract_kernel" if name.startswith(("w1a8_gemv:", "w1a8_mma:")) else name
        l0, m0, b0 = by_kernel.get(key, (0, 0.0, 0.0))
        by_kernel[key] = (l0 + launches, m0 + kms, b0 + kbytes)
    dominant = max(by_kernel, key=lambda k: by_kernel[k][1])
    launches, kms, kbytes = by_kernel["w1a8_contract_kernel"]
    peak, peak_kind = measured_peaks()
    # The instrumented replay (an event between every pair of launches) is
    # slower than the real step, so it gives only the kernel's SHARE of the
    # step; the time is that share of the un-instrumented, event-timed step.
    share = kms / total_ms
    step_ms = ms / args.steps
    kernel_ms = share * step_ms
    bytes_per_step = kbytes / args.profile_steps
    achieved = bytes_per_step / (kernel_ms / 1e3) / 1e9
    step_gbs = bytes_per_step / (step_ms / 1e3) / 1e9
    assert kernel_ms <= step_ms + 1e-9, "kernel time per step exceeds the step"
    assert step_gbs <= peak, "algorithmic bytes per step / step time above the HBM peak"
    traffic = ncu_traffic(METRIC + ("_8ctx" if args.config5 else ""))
    return {
        "kernel": "w1a8_contract_kernel", "dominant_kernel": dominant, "bound": "hbm",
        "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_source": peak_kind,
        "traffic": traffic, "launches_per_step": launches,
        "bytes_per_launch": round(kbytes / (launches * args.profile_steps), 1),
        "kernel_ms_per_step": round(kernel_ms, 4), "share_of_step": round(share, 4),
        "method": ("share of the contraction in an instrumented replay of the step graph x the "
                   "event-timed step (ms_per_step); achieved = its algorithmic bytes per step / that time"),
        "step_gbs": round(step_gbs, 1), "step_frac": round(step_gbs / peak, 4),
        "step_ms_instrumented": round(total_ms / args.profile_steps, 4),
        "kernel_share": {k: round(v[1] / total_ms, 4) for k, v in sorted(by_kernel.items(), key=lambda kv: -kv[1][1])},
    }


def run_prefill(args, ctx, info, timed, rank, world):
    """one batched 512-token prefill + greedy pick per step."""
    import numpy as np
    prompt = np.random.default_rng(PREFILL_SEED).integers(0, info.n_vocab, size=(1, PREFILL_TOKENS)).astype(np.int32)

    def step():
        ctx.truncate(0)
        ctx.decode_argmax(prompt)

    for _ in range(args.warmup):
        step()

    def loop():
        for _ in range(args.steps):
            step()

    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clocks:
        ms = timed(loop)
    clk = clocks.summary()
    value = PREFILL_TOKENS * args.steps * world / (ms / 1e3)
    # int8 multiply-adds (x2) of the layers' linears over every position, and
    # of the lm_head over the last one (the pick)
    head = float(info.hidden) * info.n_vocab
    ops = 2.0 * PREFILL_TOKENS * (info.weight_count - head) + 2.0 * head
    achieved = ops * args.steps / (ms / 1e3) / 1e12
    d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else None
    peak = 2.0 * float(d["bf16_tflops"]) if d else 2.0 * 1590.0
    if rank != 0:
        return None
    return {
        "metric": PREFILL_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded random-init weights and prompt; no checkpoint offline)",
        "config": {"workload": PREFILL_WORKLOAD, "prompt_tokens": PREFILL_TOKENS, "ctx": CTX,
                   "numerics": "fast" if args.fast else "exact (reference operation order)",
                   "l2": "inputs larger than L2: 242 MB of weights per pass vs 126 MB L2",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2),
                     "peak": round(peak, 1), "unit": "TOPS", "frac": round(achieved / peak, 4),
                     "peak_source": ("2 x measured dense bf16 (MEASURED_PEAKS.json): the int8 dense rate is "
                                     "twice bf16" if d else "2 x fallback bf16"),
                     "traffic": None,
                     "what": "int8 ops (2 per multiply-add) of the 28 layers' linears over 512 rows and "
                             "the lm_head over the last row / step time; attention and norms are inside "
                             "the step time"},
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": PREFILL_TOKENS * 4,
                "d2h_bytes_per_step": 4, "call": "BNND_DecodeArgmax of the 512-token prompt, host ids in and out"},
        "clocks": clk,
    }


def run_classify(args):
    """bnn-mlp classify, 1000 samples in batches of 64."""
    import numpy as np
    import torch
    from bnn_b200 import accel, engine, gguf
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    torch.cuda.set_device(local)
    if world > 1:
        # data-parallel: every rank classifies its own copy of the sample set
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    cache = Path(args.model_cache)
    cache.mkdir(parents=True, exist_ok=True)
    path = cache / "bnn_mlp_seed20261201.gguf"
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        gguf.bnn_mlp_model(tmp)
        os.replace(tmp, path)
    if dist:
        dist.barrier()
    dev = accel.Device(local)
    api = engine.EngineApi(dev.api.dll)
    model = engine.Model(dev, path, api)
    info = model.info
    batch, n_samples = 64, 1000
    rng = np.random.default_rng(20261201)
    x = np.zeros((n_samples, info.input_size), dtype=np.float32)
    x[:, :784] = rng.standard_normal((n_samples, 784)).astype(np.float32)
    ctx = engine.Context(model, n_batch=batch)
    stream = torch.cuda.ExternalStream(ctx.stream())
    out = np.empty((n_samples, info.n_classes), dtype=np.float32)

    def one_pass():
        for b0 in range(0, n_samples, batch):
            out[b0:b0 + batch] = ctx.classify(x[b0:b0 + batch])

    for _ in range(args.warmup):
        one_pass()
    with ClockSampler(local) as clocks:
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            one_pass()
        e1.record(stream)
        e1.synchronize()
        wall = time.perf_counter() - t0
        torch.cuda.synchronize()
    clk = clocks.summary()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms, wall], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, wall = float(t[0].item()), float(t[1].item())
    value = n_samples * args.steps * world / (ms / 1e3)
    macs = 896 * 512 + 512 * 512 + 512 * 10  # per sample
    tops = 2.0 * macs * n_samples * args.steps * world / (ms / 1e3) / 1e12
    d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else None
    peak = 2.0 * float(d["bf16_tflops"]) if d else 2.0 * 1590.0
    pred = out.argmax(axis=1)
    ctx.free()
    model.free()
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    return {
        "metric": "bnn_mlp_classify_samples_per_s", "value": round(value, 1), "unit": "samples/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded bnn-mlp weights; 1000 N(0,1) samples of 784 values, zero-padded to 896)",
        "config": {"workload": "configs[0]: bnn-mlp W1A8 classifier 896->512->512->10, 1000 samples, "
                               "BNND_Classify batch 64 (16 calls per step)",
                   "l2": "weights (0.1 MB) stay in L2; the workload is latency-bound (one step = 16 calls)",
                   "parallelism": f"data-parallel x{world} (every rank its own sample set)" if world > 1 else "single GPU",
                   "predicted_class_histogram": np.bincount(pred, minlength=info.n_classes).tolist()},
        "roofline": {"bound": "tensor", "achieved": round(tops, 3), "peak": round(peak, 1), "unit": "TOPS",
                     "frac": round(tops / peak, 6),
                     "peak_source": "2 x measured dense bf16" if d else "2 x fallback bf16", "traffic": None,
                     "what": "2 x 726,016 int8 multiply-adds per sample / step time (host copies included)"},
        "e2e": {"value": round(n_samples * args.steps * world / wall, 1), "unit": "samples/s",
                "h2d_bytes_per_step": n_samples * info.input_size * 4, "d2h_bytes_per_step": n_samples * info.n_classes * 4,
                "call": "BNND_Classify per batch of 64, host samples in, host logits out"},
        "clocks": clk,
    }


SWEEP_SHAPES = [(2048, 2048), (2048, 1024), (2048, 6144), (6144, 2048), (2048, 151669)]  # (K, N)
SWEEP_STREAM = 8            # device copies of a large matrix for the job-stream timing
L2_BYTES = 126 << 20        # B200 L2


def run_sweep(args):
    """single-op GEMV_F32 / DOT_GROUPS sweep, rows = 1."""
    import ctypes
    import numpy as np
    import torch
    from bnn_b200 import accel, synth
    torch.cuda.set_device(0)
    dev = accel.Device(0)
    dll = dev.api.dll
    dll.bnn_b200_execute_async.restype = ctypes.c_int
    dll.bnn_b200_execute_async.argtypes = [ctypes.c_void_p, ctypes.POINTER(accel.Job)]
    dll.bnn_b200_sync.restype = ctypes.c_int
    dll.bnn_b200_sync.argtypes = [ctypes.c_void_p]
    dll.bnn_b200_device_stream.restype = ctypes.c_void_p
    dll.bnn_b200_device_stream.argtypes = [ctypes.c_void_p]
    dll.bnn_b200_matrix_create_unbounded.restype = ctypes.c_int
    dll.bnn_b200_matrix_create_unbounded.argtypes = [ctypes.c_void_p, ctypes.POINTER(accel.MatrixDesc),
                                                     ctypes.POINTER(ctypes.c_void_p)]
    stream = torch.cuda.ExternalStream(dll.bnn_b200_device_stream(dev.handle))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > 2 x L2
    flush_sink = torch.empty((), dtype=torch.uint8, device="cuda")
    hbm, hbm_kind = measured_peaks()
    rng = synth.rng_for(1)
    results = []

    def matrix(bits, scales, k, n):
        bits = np.ascontiguousarray(bits)
        scales = np.ascontiguousarray(scales)
        desc = accel.MatrixDesc(k, n, accel.GROUP, bits.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), bits.nbytes,
                                scales.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), scales.size)
        h = ctypes.c_void_p()
        st = dll.bnn_b200_matrix_create_unbounded(dev.handle, ctypes.byref(desc), ctypes.byref(h))
        if st != accel.OK:
            raise accel.BnnError(st, "matrix")
        m = accel.Matrix.__new__(accel.Matrix)
        m.device, m.k, m.n, m.handle = dev, k, n, h
        return m

    shapes = SWEEP_SHAPES
    if args.sweep_shape:
        k_, n_ = (int(v) for v in args.sweep_shape.lower().split("x"))
        shapes = [(k_, n_)]
    with ClockSampler(0) as clocks:
        for k, n in shapes:
            bits, scales = synth.w1_matrix(rng, k, n)
            x = synth.activations(rng, 1, k)
            scale = float(np.abs(x).max()) / 127.0
            q = np.clip(np.rint(x / scale), -127, 127).astype(np.int8)
            m = matrix(bits, scales, k, n)
            g = k // 128
            for op, inp, out_bytes, alg in (
                    (accel.OP_GEMV_F32, x, n * 4, n * k * 0.140625 + 4 * k + 4 * n),
                    (accel.OP_DOT_GROUPS, q, n * g * 2, n * k / 8 + k + 2 * n * g)):
                bi, bo = accel.Buffer(dev, inp.nbytes), accel.Buffer(dev, out_bytes)
                bi.write(inp)
                it, ot = accel.OP_TYPES[op]
                job = accel.Job(operation=op, matrix=m.handle, input=accel.BufferView(bi.handle, it, 0, 0),
                                output=accel.BufferView(bo.handle, ot, 0, 0), rows=1)
                times = []
                for i in range(args.warmup + args.steps):
                    with torch.cuda.stream(stream):
                        # L2 flush: write a buffer twice the L2, then read it, so the
                        # flush's dirty lines are written back before the timed job
                        flush.fill_(i & 0xff)
                        flush_sink.copy_(flush.max())
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record(stream)
                        if dll.bnn_b200_execute_async(dev.handle, ctypes.byref(job)) != accel.OK:
                            raise accel.BnnError(-1, "execute_async")
                        e1.record(stream)
                    e1.synchronize()
                    if i >= args.warmup:
                        times.append(e0.elapsed_time(e1))
                if dll.bnn_b200_sync(dev.handle) != accel.OK:
                    raise accel.BnnError(-1, "sync")
                us = statistics.median(times) * 1e3
                # Matrices larger than L2 / 3 are also timed as a stream of jobs: the
                # job runs on SWEEP_STREAM device copies of the matrix in turn (together
                # more than twice the L2, so every job reads its weights from HBM), all
                # jobs between one pair of events, per-job time = elapsed / jobs. This
                # leaves out the launch latency and the 2 us event granularity that a
                # single timed job carries.
                stream_us = None
                wbytes = n * k * 0.140625
                if wbytes * SWEEP_STREAM > 2 * L2_BYTES:
                    copies = [m] + [matrix(bits, scales, k, n) for _ in range(SWEEP_STREAM - 1)]
                    sjobs = [accel.Job(operation=op, matrix=mc.handle, input=job.input, output=job.output, rows=1)
                             for mc in copies]
                    st_times = []
                    for i in range(args.warmup + args.steps):
                        with torch.cuda.stream(stream):
                            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                            e0.record(stream)
                            for sj in sjobs:
                                if dll.bnn_b200_execute_async(dev.handle, ctypes.byref(sj)) != accel.OK:
                                    raise accel.BnnError(-1, "execute_async")
                            e1.record(stream)
                        e1.synchronize()
                        if i >= args.warmup:
                            st_times.append(e0.elapsed_time(e1) / len(sjobs))
                    if dll.bnn_b200_sync(dev.handle) != accel.OK:
                        raise accel.BnnError(-1, "sync")
                    stream_us = statistics.median(st_times) * 1e3
                    for mc in copies[1:]:
                        mc.destroy()
                # the public synchronous path, host buffers (N > 8192: 8192-row chunks)
                host_out = np.empty(out_bytes, dtype=np.uint8)
                chunks = []
                if n <= 8192:
                    chunks.append((m, bo, n))
                else:
                    for r0 in range(0, n, 8192):
                        rn = min(8192, n - r0)
                        mc = accel.Matrix(dev, bits[r0:r0 + rn], scales[r0:r0 + rn])
                        chunks.append((mc, accel.Buffer(dev, out_bytes // n * rn), rn))
                t_e2e = []
                for i in range(max(3, args.steps // 4)):
                    t0 = time.perf_counter()
                    bi.write(inp)
                    off = 0
                    for mc, bc, rn in chunks:
                        st = dev.execute(op, mc, bi, bc, rows=1)
                        if st != accel.OK:
                            raise accel.BnnError(st, "BNN_Execute")
                        nb = out_bytes // n * rn
                        host_out[off:off + nb] = bc.read(nb)
                        off += nb
                    t_e2e.append(time.perf_counter() - t0)
                for mc, bc, rn in chunks:
                    if mc is not m:
                        mc.destroy()
                        bc.free()
                e2e_us = statistics.median(t_e2e) * 1e6
                results.append({"op": "GEMV_F32" if op == accel.OP_GEMV_F32 else "DOT_GROUPS", "k": k, "n": n,
                                "bytes": int(alg), "kernel_us": round(us, 2),
                                "gbs": round(alg / (us * 1e-6) / 1e9, 1),
                                "frac_of_hbm": round(alg / (us * 1e-6) / 1e9 / hbm, 4),
                                "e2e_us": round(e2e_us, 1), "e2e_jobs": len(chunks)})
                if stream_us is not None:
                    results[-1].update({"stream_kernel_us": round(stream_us, 2),
                                        "stream_gbs": round(alg / (stream_us * 1e-6) / 1e9, 1),
                                        "stream_frac_of_hbm": round(alg / (stream_us * 1e-6) / 1e9 / hbm, 4)})
                bi.free()
                bo.free()
            m.destroy()
    clk = clocks.summary()
    dev.close()
    head = [r for r in results if r["op"] == "GEMV_F32" and r["n"] == shapes[-1][1]][0]
    head_gbs = head.get("stream_gbs", head["gbs"])
    head_us = head.get("stream_kernel_us", head["kernel_us"])
    return {
        "metric": "w1a8_gemv_f32_hbm_gbs", "value": head_gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(head_us / 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded W1 bits, FP16 scales ~U[0.005,0.05], FP32 N(0,1) activations with 1% x20)",
        "config": {"workload": ("one shape of " if args.sweep_shape else "") +
                               "configs[1]: single-op GEMV_F32 / DOT_GROUPS sweep at the Qwen3-1.7B linear "
                               "shapes, rows = 1 (value: GEMV_F32 2048x151669 as one job, timed in a stream "
                               "of jobs over 8 device copies of the matrix; kernel_us/gbs: one job after an "
                               "L2 flush, launch latency included)",
                   "l2": "kernel_us: flushed before every timed job (256 MB written, then read back, so no dirty "
                         "flush lines are written back inside the timed job); stream_kernel_us: inputs larger "
                         "than L2 (8 copies x 44 MB, each job's weights last touched 7 jobs earlier)",
                   "shapes": results},
        "roofline": {"bound": "hbm", "achieved": head_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": round(head_gbs / hbm, 4), "peak_source": hbm_kind, "traffic": None,
                     "what": "one GEMV_F32 job = one kernel (in-CTA quantise + contraction), per-job time in the stream of jobs, algorithmic bytes"},
        "e2e": {"value": round(head["bytes"] / (head["e2e_us"] * 1e-6) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": 2048 * 4, "d2h_bytes_per_step": 151669 * 4,
                "call": "BufferWrite + 19 x BNN_Execute (<= 8192 rows) + BufferRead, host buffers"},
        "clocks": clk,
    }


def _ref_child(ref, tok, n_tokens, conn):
    """A forked copy of the prefilled reference engine: decodes n_tokens
    greedy steps from the prompt's pick (positions PROMPT_TOKENS ..) and
    sends back (tokens, seconds)."""
    import numpy as np
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        tok = int(np.argmax(ref.decode([tok])))
    conn.send((n_tokens, time.perf_counter() - t0))
    conn.close()


def run_reference(args):
    """The reference engine (bnn-sw-v2 + soft backend, single-threaded, built
    from its sources) on the host cores, at the configured positions: one
    process prefills the 32-token prompt through BNNE_Decode (untimed), then
    forks one copy per core (no GPU has been touched in this process), and
    every copy decodes greedy steps from position 32 on, as the device arm's
    timed steps do. value = tokens of all copies / the slowest copy's time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    import multiprocessing as mp
    import numpy as np
    import ref_engine
    if not ref_engine.available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libbnn_engine_soft.so not built"}
    path = model_path(args.model_cache)
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    procs = max(1, min(cores, args.ref_procs, args.steps))
    per = max(1, args.steps // procs)
    ref = ref_engine.RefEngine(path, n_ctx=CTX)
    prompt = prompt_ids(ref.info.n_vocab)
    t0 = time.perf_counter()
    first = int(np.argmax(ref.decode(prompt)))  # positions 0..31, untimed
    prefill_s = time.perf_counter() - t0
    ctxm = mp.get_context("fork")
    pipes, workers = [], []
    for _ in range(procs):
        a, b = ctxm.Pipe(duplex=False)
        w = ctxm.Process(target=_ref_child, args=(ref, first, per, b))
        w.start()
        pipes.append(a)
        workers.append(w)
    results = [p.recv() for p in pipes]
    for w in workers:
        w.join()
    ref.close()
    tokens = sum(r[0] for r in results)
    slowest = max(r[1] for r in results)
    value = tokens / slowest
    sample = (f"{procs} forked copies of the reference soft engine (single-threaded each) on {cores} host "
              f"cores after one untimed {PROMPT_TOKENS}-token prompt prefill ({prefill_s:.0f} s); each copy "
              f"decodes {per} greedy step(s) at positions {PROMPT_TOKENS}..{PROMPT_TOKENS + per - 1}; "
              f"aggregate tokens / slowest copy")
    return {
        "metric": METRIC, "value": round(value, 6), "unit": "tokens/s", "n_gpus": 0, "steps": tokens,
        "warmup": PROMPT_TOKENS, "ms_per_step": round(slowest * 1e3 / tokens, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": DATA,
        "config": decode_config(gguf_shape(), GEN_STEPS, PROMPT_TOKENS, CTX, 1, WORKLOAD),
        "impl": "reference",
        "impl_config": {"numerics": "reference (soft backend)", "parallelism": f"{procs} host processes"},
        "cpu_baseline": {"value": round(value, 6), "unit": "tokens/s", "cores": procs, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--fast", action="store_true", help="tree reductions instead of the reference order")
    ap.add_argument("--profile-steps", type=int, default=4)
    ap.add_argument("--ref-procs", type=int, default=32)
    ap.add_argument("--tp-steps", type=int, default=32,
                    help="timed steps of the column-sharded configs[4] block")
    ap.add_argument("--no-tp-block", action="store_true",
                    help="skip the column-sharded configs[4] block of the default run")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="skip the short configs[0], configs[1] and configs[3] blocks of the default run")
    ap.add_argument("--classify", action="store_true",
                    help="BASELINE configs[0]: bnn-mlp classify, batch 64 (samples/s)")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE configs[1]: single-op GEMV_F32 / DOT_GROUPS sweep (HBM GB/s)")
    ap.add_argument("--sweep-shape", default=None,
                    help="with --sweep: one KxN shape only (e.g. 2048x151669, for profiling)")
    ap.add_argument("--config5", action="store_true",
                    help="BASELINE configs[4]: 8 contexts, 64-token prompts, ctx 4096 (with --tp: sharded)")
    ap.add_argument("--prefill", action="store_true",
                    help="BASELINE configs[3]: batched 512-token prefill instead of decode")
    ap.add_argument("--tp", action="store_true",
                    help="with --gpus N under torchrun: one sequence on a column-sharded model instead of N replicas")
    ap.add_argument("--model-cache", default=os.environ.get("BNN_MODEL_CACHE", "/tmp/bnn_b200_models"))
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.sweep and args.impl != "reference":
        out = run_sweep(args)
    elif args.classify and args.impl != "reference":
        out = run_classify(args)
    else:
        out = run_reference(args) if args.impl == "reference" else run_b200(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

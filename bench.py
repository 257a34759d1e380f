#!/usr/bin/env python
"""Decode throughput of llama.rs's Qwen2 token loop on B200 (benchmark config 3).

Workload (default --config c3): the Qwen2.5-7B-shape model (seed 2, q4km),
64 independent sequences, each a 1024-token uniform prompt followed by greedy
decoding, context 4096; the sequences are split data-parallel over the ranks
(one process per GPU, no collective on the data path).  A "step" is one greedy
decode step of every local sequence; `value` is decode tokens/s over all ranks
(device time, CUDA events, max over ranks), `e2e` the same through the public
C-ABI call with host buffers (token ids in, token ids out, every step).

Also reported: batch-1 decode on the same model (the north-star target), the
prefill rate, the GEMV roofline (per-launch CUDA events inside the run), the
SM clocks seen during the timed region, and the reference CPU path (the C++
restatement of the reference AVX2 backend, oracle/) timed on the host cores.

`--impl reference` times only that CPU path, on the same workload and metric.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))



def load_pkg():
    import importlib.util
    if "llamars_b200" in sys.modules:
        return sys.modules["llamars_b200"]
    pkg = os.path.join(ROOT, "llama.rs_b200")
    spec = importlib.util.spec_from_file_location(
        "llamars_b200", os.path.join(pkg, "__init__.py"), submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llamars_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    return oracle


WORKLOADS = {
    "c3": dict(cfg="config_c3", seed=2, recipe="Q4KM", seqs=64, prompt=1024, decode=256, ctx=4096,
               model="Qwen2.5-7B-shape", quant="q4km"),
    "c2": dict(cfg="config_c2", seed=1, recipe="Q4K", seqs=1, prompt=512, decode=128, ctx=4096,
               model="Qwen2.5-1.5B-shape", quant="q4k"),
    "c4": dict(cfg="config_c4", seed=3, recipe="Q4K", seqs=16, prompt=2048, decode=256, ctx=8192,
               model="Qwen2.5-32B-shape", quant="q4k"),
    "c0": dict(cfg="config_c0", seed=0, recipe="Q4KM", seqs=1, prompt=128, decode=32, ctx=4096,
               model="Qwen2.5-0.5B-shape", quant="q4km"),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, phys_index):
        self.idx = phys_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "samples": len(rows), "reasons": sorted(reasons)}


# DRAM bytes read + written per batched-matmul call of a 64-sequence c3 step
# (5.10 GB over 113 calls), profiles/matmul_traffic_c3_b64.md.
MATMUL_TRAFFIC_C3_B64 = 45.1e6


def launches_per_step(layers, batch):
    # estimate when the graph's node count is unavailable: embed, per layer
    # q/k, v, attention, o, gate_up, down (+ x preparation and K-split sums at
    # batch > 1), then lm_head, advance
    per_layer = 6 + (3 if batch > 1 else 0)
    return 1 + layers * per_layer + (2 if batch == 1 else 3)


def model_cache_path(wl):
    layers = f"_L{wl['layers']}" if wl.get("layers") else ""
    return os.path.join(tempfile.gettempdir(),
                        f"llamars_{wl['cfg']}{layers}_s{wl['seed']}_{wl['recipe']}_v1.lrs")


def build_model(lrs, wl, threads=0, barrier=None, builder=True):
    """The workload's synthetic model.  The pre-quantized bytes are cached in a
    flat file under the temp directory: the builder (local rank 0) generates
    and writes it when absent, the other ranks wait at `barrier` and map it."""
    path = model_cache_path(wl)
    if builder and not os.path.exists(path):
        cfg = getattr(lrs, wl["cfg"])()
        if wl.get("layers"):
            cfg.num_hidden_layers = wl["layers"]
        sm = lrs.SynthModel(cfg, wl["seed"], lrs.LoadQuantization[wl["recipe"]], threads=threads)
        try:
            lrs.save_model_file(sm.desc(), path)
        except OSError:
            if barrier is None:
                return cfg, sm
            raise
        del sm
    if barrier is not None:
        barrier()
    mf = lrs.ModelFile(path)
    return mf.config, mf


def cpu_decode_rate(orc, desc, vocab, wl, P, threads, budget_s=15.0, warmup=2):
    """The reference AVX2 path (the oracle's restatement of src/simd.rs with
    the row-parallel pool of src/backend.rs:143-162) on the host cores: greedy
    decode steps of one sequence at the workload's context (positions P, P+1,
    ...).  The prompt is not run through the CPU (it would take minutes): the
    dense f32 KV cache of the restatement starts zeroed, and the cost of a
    decode step depends on the context length only.  Returns (tok/s, steps)."""
    om = orc.OracleModel(desc, P + 512, orc.AVX2, threads)
    tok = int(prompt_ids(wl["seed"], 1, vocab)[0])
    for i in range(warmup):
        tok = int(orc.argmax(om.forward_token(tok, P + i)))
    t0 = time.perf_counter()
    tok = int(orc.argmax(om.forward_token(tok, P + warmup)))
    per_tok = max(time.perf_counter() - t0, 1e-4)
    n = int(max(2, min(256, budget_s / per_tok)))
    t0 = time.perf_counter()
    for i in range(n):
        tok = int(orc.argmax(om.forward_token(tok, P + warmup + 1 + i)))
    return n / (time.perf_counter() - t0), n


def prompt_ids(seed, n, vocab, sequence=0):
    """prompt_tokens of the package (numpy PCG64), restated so the reference
    arm does not load the CUDA library."""
    rng = np.random.default_rng(seed + 1000 if sequence == 0 else [seed, sequence])
    return rng.integers(0, vocab, n, dtype=np.int64).astype(np.uint32)


def workload_config(wl, total_seqs, P, world, tp, layers=0, kv_bf16=False):
    """The `config` object both arms print for a workload."""
    return {"workload": f"{wl['model']} {wl['quant']}: {total_seqs} sequences x "
                        f"({P} prompt + greedy decode), ctx {wl['ctx']}, "
                        + (f"{layers} layers (profiling case), " if layers else "") +
                        (f"tensor-parallel over {world} GPUs" if tp else
                         f"data-parallel over {world} GPU(s)"),
            "parallelism": f"tp{world}" if tp else f"dp{world}",
            "sequences_per_gpu": total_seqs if tp else total_seqs // max(world, 1), "prompt": P,
            "kv_cache": "bf16" if kv_bf16 else "f32"}


# The arithmetic of this implementation's dot products (the GPU arm's config).
GPU_ARITHMETIC = ("weights decoded exactly from their GGML blocks; f32 accumulation; x split "
                  "for the dot products: batch 1 int8 hi/lo per 8 columns (~15 bits, dp4a), "
                  "batched f16 hi + lo (~22 bits, tensor cores, exact products); attention and "
                  "norms in f32")


def run_reference(args, wl):
    """The reference CPU path alone: the model file is mapped without the CUDA
    library (oracle.MappedModel); when the cache is missing a child process
    builds it first (untimed).  Each step is one greedy decode step of one
    sequence at the GPU arm's context (the reference has no batching)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = model_cache_path(wl)
    if not os.path.exists(path):
        code = ("import sys; sys.path.insert(0, %r); import bench; "
                "bench.build_model(bench.load_pkg(), %r, %d)" % (ROOT, wl, os.cpu_count() or 1))
        subprocess.run([sys.executable, "-c", code], check=True)
    orc = load_oracle()
    mf = orc.MappedModel(path)
    threads = os.cpu_count() or 1
    P = args.prompt or wl["prompt"]
    om = orc.OracleModel(mf.desc(), P + args.warmup + args.steps + 8, orc.AVX2, threads)
    tok = int(prompt_ids(wl["seed"], 1, mf.vocab_size)[0])
    pos = P
    for _ in range(args.warmup):
        tok = int(orc.argmax(om.forward_token(tok, pos)))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = int(orc.argmax(om.forward_token(tok, pos)))
        pos += 1
    dt = time.perf_counter() - t0
    value = args.steps / dt
    sample = (f"1 sequence (the reference has no batching) at context {P}..{P + args.warmup + args.steps}: "
              f"{args.warmup} warm-up + {args.steps} timed greedy decode steps; the f32 KV cache of "
              "the prompt positions starts zeroed instead of running the prompt on the CPU "
              "(a step's cost depends on the context length only)")
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random weights and ids)",
        "config": dict(workload_config(wl, args.seqs or wl["seqs"], P, args.gpus,
                                       args.tp and args.gpus > 1, wl.get("layers", 0), args.kv_bf16),
                       kernel="avx2", threads=threads, cpu=cpu_model(),
                       arithmetic="the reference AVX2 dots (src/simd.rs): f32 weights times f32 x"),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample + "; C++ restatement of the reference AVX2 backend "
                                            "(src/simd.rs) -- the Rust reference cannot be built "
                                            "here (no cargo)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_ours(args, wl):
    import torch
    lrs = load_pkg()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    total_seqs = args.seqs or wl["seqs"]
    tp = args.tp and world > 1
    if not tp and total_seqs % world:
        raise SystemExit("sequences must divide evenly over the GPUs")
    B = total_seqs if tp else total_seqs // world
    P = args.prompt or wl["prompt"]
    ncpu = os.cpu_count() or 1

    t_build = time.perf_counter()
    cfg, sm = build_model(lrs, wl, ncpu, barrier if world > 1 else None, builder=local == 0)
    build_s = time.perf_counter() - t_build
    be = lrs.CudaBackend(local)
    tp_kw = {}
    if tp:
        # one tensor-parallel model over the ranks; rank 0 makes the NCCL id
        obj = [lrs.tp_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0)
        tp_kw = dict(tp_rank=rank, tp_world=world, tp_id=obj[0])
    model = lrs.CudaQwen2Model(be, sm.desc(), max_seq_len=wl["ctx"], max_sequences=B,
                               kv_bf16=args.kv_bf16, **tp_kw)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", local))

    def ev():
        return torch.cuda.Event(enable_timing=True)

    # ---- prefill every local sequence (prompt of P uniform ids) ----
    first_seq = 0 if tp else rank * B
    prompts = [lrs.prompt_tokens(wl["seed"], P, cfg.vocab_size, first_seq + s) for s in range(B)]
    firsts = []
    p0, p1 = ev(), ev()
    p0.record(ext)
    for s in range(B):
        _, f = model.prefill(prompts[s], 0, seq=s, want_logits=False)
        firsts.append(f)
    p1.record(ext)
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(p0.elapsed_time(p1))
    seqs = list(range(B))
    pos = [P] * B

    # ---- warm-up (W greedy steps, graph captured on the first) ----
    out = model.decode_greedy(firsts, pos, args.warmup, seqs)
    firsts = out[-1].tolist()
    pos = [p + args.warmup for p in pos]

    # ---- timed region: K device-resident greedy steps ----
    phys = local
    if os.environ.get("CUDA_VISIBLE_DEVICES"):
        phys = os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local]
    clocks = ClockSampler(phys)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    t0, t1 = ev(), ev()
    torch.cuda.nvtx.range_push("lrs_decode_timed")
    t0.record(ext)
    model.decode_enqueue(firsts, pos, args.steps, seqs)
    t1.record(ext)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clock_info = clocks.stop()
    step_kernels = model.step_kernels()
    barrier()
    step_ms = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    toks = model.read_tokens(B, args.steps)
    firsts = toks[-1].tolist()
    pos = [p + args.steps for p in pos]
    value = total_seqs / (step_ms / 1e3)

    # ---- e2e: the public C-ABI call per step, host token ids in and out ----
    barrier()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record(ext)
    for _ in range(args.steps):
        out = model.decode_greedy(firsts, pos, 1, seqs)
        firsts = out[0].tolist()
        pos = [p + 1 for p in pos]
    e1.record(ext)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    e2e_value = total_seqs / (e2e_ms / 1e3)

    # ---- GEMV roofline: one step with per-launch CUDA events ----
    gemv_ms, gemv_n, prof_step_ms, attn_ms = model.profile_step(firsts, pos, seqs)
    gemv_ms = max_over_ranks(gemv_ms)
    attn_ms = max_over_ranks(attn_ms)
    kv_elem = 2 if args.kv_bf16 else 4
    kvw = cfg.num_key_value_heads * cfg.resolved_head_dim()
    # K and V rows read by the step (positions 0..pos) plus the row written, all layers
    kv_bytes = sum(2 * cfg.num_hidden_layers * kvw * kv_elem * (p + 2) for p in pos)
    wbytes = model.weight_bytes()
    hbm, peak_kind = peaks()
    achieved = wbytes / (gemv_ms / 1e3) / 1e9
    pos = [p + 1 for p in pos]

    # ---- batch-1 decode on the same model (sequence 0) ----
    b1 = None
    if not args.no_b1:
        model.decode_greedy([firsts[0]], [pos[0]], 3, [0])
        q0, q1 = ev(), ev()
        q0.record(ext)
        model.decode_enqueue([firsts[0]], [pos[0] + 3], args.steps, [0])
        q1.record(ext)
        torch.cuda.synchronize()
        b1_ms = max_over_ranks(q0.elapsed_time(q1)) / args.steps
        g1, n1, _, _ = model.profile_step([int(model.read_tokens(1, args.steps)[-1, 0])],
                                       [pos[0] + 3 + args.steps], [0])
        g1 = max_over_ranks(g1)
        b1 = {"decode_tok_s_per_gpu": 1e3 / b1_ms, "ms_per_step": b1_ms,
              "weight_stream_gbs": wbytes / (b1_ms / 1e3) / 1e9,
              "weight_stream_frac": wbytes / (b1_ms / 1e3) / 1e9 / hbm,
              "gemv_gbs": wbytes / (g1 / 1e3) / 1e9, "gemv_frac": wbytes / (g1 / 1e3) / 1e9 / hbm,
              "gemv_launches": n1}

    # ---- CPU baseline: reference AVX2 path (port) on rank 0 at N=1 ----
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        orc = load_oracle()
        rate, n = cpu_decode_rate(orc, sm.desc(), cfg.vocab_size, wl, P, ncpu)
        cpu = {"value": rate, "unit": "tok/s", "cores": ncpu, "kind": "port", "cpu": cpu_model(),
               "sample": f"1 sequence at context {P}: {n} greedy decode steps of the same model "
                         "(KV of the prompt positions zeroed, not computed); C++ restatement of "
                         "the reference AVX2 backend (src/simd.rs, row-parallel pool as "
                         "src/backend.rs:143-162)"}

    if rank == 0:
        nl = launches_per_step(cfg.num_hidden_layers, B)
        # DRAM bytes per matmul call from one ncu capture of this workload's
        # launch shapes (profiles/matmul_traffic_c3_b64.md); other workloads
        # have no capture
        full_c3 = (args.config == "c3" and B == 64 and not wl.get("layers") and not args.kv_bf16
                   and not args.prompt and not args.ctx)
        traffic = MATMUL_TRAFFIC_C3_B64 if full_c3 else None
        traffic_src = ("ncu dram__bytes_read+write per matmul launch, profiles/matmul_traffic_c3_b64.md"
                       if full_c3 else None)
        line = {
            "metric": "decode_tokens_per_s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random weights N(0,0.02), uniform prompt ids)",
            "config": {**workload_config(wl, total_seqs, P, world, tp, wl.get("layers", 0),
                                         args.kv_bf16),
                       "arithmetic": GPU_ARITHMETIC,
                       "l2": f"inputs larger than L2: {wbytes / 1e9:.2f} GB of weights streamed per step"},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 12 * B,
                    "d2h_bytes_per_step": 4 * B + 4},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic,
                         "traffic_source": traffic_src,
                         "kernel": ("gemm_tc_kernel (tcgen05, Q4_K/Q6_K) + gemm_mma_kernel (Q8_0): batched quantized matmul (x split, matmul, "
                                    "K-split epilogue) of every projection and the LM head"
                                    if B > 1 else "gemv5_kernel: batch-1 quantized GEMV"),
                         "bytes_per_launch": wbytes / gemv_n, "ms_per_launch": gemv_ms / gemv_n,
                         "launches": gemv_n, "peak_kind": peak_kind,
                         "share_of_step": gemv_ms / prof_step_ms},
            "attention": {"kernel": "attn_split_kernel (RoPE, KV store and split merge fused), all layers",
                          "kv_bytes_per_step": kv_bytes, "ms": attn_ms,
                          "achieved_gbs": kv_bytes / (attn_ms / 1e3) / 1e9,
                          "frac": kv_bytes / (attn_ms / 1e3) / 1e9 / hbm,
                          "share_of_step": attn_ms / prof_step_ms},
            "step_hbm": {"bytes_per_step": wbytes + kv_bytes,
                         "achieved_gbs": (wbytes + kv_bytes) / (step_ms / 1e3) / 1e9,
                         "frac": (wbytes + kv_bytes) / (step_ms / 1e3) / 1e9 / hbm},
            "weight_stream_gbs": wbytes / (step_ms / 1e3) / 1e9,
            "prefill_tok_s": total_seqs * P / (prefill_ms / 1e3),
            "b1": b1,
            "cpu_baseline": cpu,
            "clocks": clock_info,
            "gpu_launches": (step_kernels or nl) * args.steps,
            "model_build_s": build_s,
        }
        print(json.dumps(line), flush=True)
    model.close()
    be.close()
    if world > 1:
        torch.distributed.destroy_process_group()


SWEEP_SHAPES = ["4864x896", "896x4864", "18944x3584", "3584x18944", "152064x3584"]
SWEEP_TYPES = ["F16", "BF16", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q4_K", "Q5_K", "Q6_K"]


def run_gemv_sweep(args):
    """benchmark config 1: GB/s of the quantized GEMV per type, shape and batch.

    W ~ N(0, 0.02) quantized on the host, x ~ N(0, 1); each cell times `iters`
    back-to-back launches with CUDA events after 3 warm-up launches.  Shapes
    smaller than L2 partly run from L2 when repeated; 152064x3584 exceeds L2.
    Parity of every row is covered by tests/test_gpu_gemv.py."""
    import torch
    lrs = load_pkg()
    be = lrs.CudaBackend(0)
    ext = torch.cuda.ExternalStream(be.stream(), device=torch.device("cuda", 0))
    hbm, peak_kind = peaks()
    types = args.types.split(",") if args.types else SWEEP_TYPES
    shapes = args.shapes.split(",") if args.shapes else SWEEP_SHAPES
    batches = [int(b) for b in args.batches.split(",")]
    rng = np.random.default_rng(0)
    cells = []
    for shape in shapes:
        rows, cols = (int(v) for v in shape.split("x"))
        v = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
        for qt in types:
            t = lrs.QuantTensor.quantize(v, rows, cols, lrs.QuantType[qt])
            if t.quant_type != lrs.QuantType[qt]:
                cells.append({"type": qt, "shape": shape, "skipped":
                              f"cols % block != 0 (the reference falls back to {t.quant_type.name})"})
                continue
            be.upload(t)
            for b in batches:
                x = torch.randn(b, cols, device="cuda", dtype=torch.float32)
                y = torch.empty(b, rows, device="cuda", dtype=torch.float32)
                torch.cuda.synchronize()
                for _ in range(3):
                    be.matvec_device(t, x.data_ptr(), b, y.data_ptr())
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(ext)
                for _ in range(args.iters):
                    be.matvec_device(t, x.data_ptr(), b, y.data_ptr())
                e1.record(ext)
                torch.cuda.synchronize()
                be.synchronize()
                ms = e0.elapsed_time(e1) / args.iters
                nbytes = t.data.size + b * (cols + rows) * 4
                gbs = nbytes / (ms / 1e3) / 1e9
                cells.append({"type": qt, "shape": shape, "batch": b, "us": round(ms * 1e3, 2),
                              "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
                              "weight_mb": round(t.data.size / 1e6, 2)})
            be.release(t)
    print(json.dumps({"metric": "gemv_sweep", "peak_gbs": hbm, "peak_kind": peak_kind,
                      "cells": cells}), flush=True)
    be.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c3", choices=sorted(WORKLOADS))
    ap.add_argument("--seqs", type=int, default=0, help="total sequences (default: the config's)")
    ap.add_argument("--prompt", type=int, default=0, help="prompt tokens (default: the config's)")
    ap.add_argument("--kv-bf16", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small profiling cases only)")
    ap.add_argument("--ctx", type=int, default=0, help="override the context length")
    ap.add_argument("--tp", action="store_true",
                    help="one tensor-parallel model over the ranks instead of data parallel")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--no-b1", action="store_true")
    ap.add_argument("--gemv-sweep", action="store_true", help="benchmark config 1 GEMV sweep")
    ap.add_argument("--types", default="")
    ap.add_argument("--shapes", default="")
    ap.add_argument("--batches", default="1,8,64")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.gemv_sweep:
        run_gemv_sweep(args)
        return
    wl = dict(WORKLOADS[args.config])
    if args.layers:
        wl["layers"] = args.layers
    if args.ctx:
        wl["ctx"] = args.ctx
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()

"""Benchmark: batch-1 greedy decode of a Mistral-7B-v0.3-shape decoder packed in
GSD-LQ Precision mode (random-init N(0, 0.02^2) weights, synthetic token ids).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token (all 32 layers + LM head + greedy pick) at positions
after a 1536-token prompt; positions wrap back to 1536 when the 2048-entry KV cache
is full.  The timed region holds K steps, replayed as CUDA graphs with the token fed
back on the device, bracketed by a barrier and device synchronisation; the device
time is the max over ranks.  One JSON line is printed by rank 0.

N > 1 runs tensor parallelism (strong scaling: the same single sequence, the packed
linears sharded across ranks, an all-reduce after the O and down projections).

--impl reference times the reference's own C engine (oracle/_ref, built from the
reference source with the reference's flags) on the host cores with all of them in
use: each step is one whole decode token through the reference engine's seven
functions, on format-valid packed bytes of the same shapes drawn with NumPy (this arm
loads no library of this repository and uses no GPU).  Under torchrun only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s batch1 Mistral-7B-shape Precision; unpack-matvec HBM GB/s % peak"
PUBLISHED_TOKS = {"precision": 6.5, "turbo": 12.5}  # the reference's Mistral-7B decode rates (README.md:32-33)
# DRAM bytes (read + write) of one gate/up launch of a Mistral-7B Precision layer, from one ncu capture on a
# B200, and the algorithmic bytes of that launch (a tensor-parallel rank's launch scales both)
GU_TRAFFIC = 66_802_432 + 711_168
GU_ALGO = 66_527_368
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
REF_TIME_BUDGET_S = 240.0  # the reference arm's timed tokens are capped to about this much host time
SWEEP_SHAPES = ((4096, 4096), (4096, 14336), (14336, 4096), (32768, 4096))  # (rows, cols) of W
SWEEP_BATCHES = (1, 4, 16, 64)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def prefill_roofline(cfg: dict, tokens: int, secs: float, pk: dict, pk_src: str, sequences: int = 1) -> dict:
    """Tensor-pipe roofline of a prefill of ``tokens`` prompt tokens per sequence from position 0: 2 flops per
    packed weight of every layer linear per token (the LM head does not run), plus causal attention
    (QK^T and PV: 4 * heads * head_dim flops per query-key pair, t + 1 keys for token t), against the
    measured dense bf16 burst peak."""
    H, F = cfg["hidden_size"], cfg["ffn_size"]
    q, kv = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    weights = cfg["n_layers"] * (q * H + 2 * kv * H + H * q + 3 * F * H)
    pairs = tokens * (tokens + 1) // 2
    flops = sequences * (2 * weights * tokens + cfg["n_layers"] * 4 * q * pairs)
    peak = float(pk["bf16_tflops"])
    achieved = flops / secs / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "flops": flops, "peak_source": f"{pk_src} bf16_tflops"}


def vs_published(args, tok_s):
    """value / the reference's published decode rate, for the one model it publishes (Mistral-7B)."""
    return tok_s / PUBLISHED_TOKS[args.mode] if args.model == "mistral-7b" else None


def parse():
    ap = argparse.ArgumentParser(description="Batch-1 greedy decode throughput (one JSON line on rank 0).")
    ap.add_argument("--gpus", type=int, default=1, help="GPUs of this node (N > 1: tensor parallelism, via torchrun)")
    ap.add_argument("--steps", type=int, default=256, help="timed decode tokens")
    ap.add_argument("--warmup", type=int, default=8, help="untimed decode tokens before them (at least 3)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours",
                    help="this engine, or the reference's C engine on the host cores")
    ap.add_argument("--model", default="mistral-7b", help="model shape (random-init weights of that architecture)")
    ap.add_argument("--mode", default="precision", choices=["precision", "turbo"], help="packing mode")
    ap.add_argument("--prompt", type=int, default=1536, help="KV length at the first timed token")
    ap.add_argument("--seed", type=int, default=0, help="seed of the weights and inputs")
    ap.add_argument("--e2e-steps", type=int, default=64, help="tokens timed through the host-facing forward_token")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the reference CPU sample (cpu_baseline)")
    ap.add_argument("--no-kinds", action="store_true", help="skip the per-launch-kind timings")
    ap.add_argument("--layers", type=int, default=0, help="override n_layers (debug only; not a bench number)")
    ap.add_argument("--step", choices=["fused", "per-op"], default="per-op",
                    help="one persistent launch per token (fused) or the per-operation launches in CUDA graphs")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences decoded in lockstep (B > 1: batched decode through the tensor-core GEMM, one GPU)")
    ap.add_argument("--max-seq", type=int, default=2048, help="KV cache length per sequence (batched decode)")
    ap.add_argument("--sweep", action="store_true",
                    help="the unpack-matvec / dequant-GEMM bandwidth sweep (4 shapes x 2 modes x B = 1/4/16/64)")
    return ap.parse_args()


def metric_name(args) -> str:
    """BASELINE's metric for its headline config; the same quantity named for the other configs."""
    if args.sweep:
        return "packed linear GB/s (unpack-matvec at B=1, dequant-GEMM at B=1/4/16/64) % of HBM peak"
    if args.batch == 1 and args.model == "mistral-7b" and args.mode == "precision":
        return METRIC
    return f"decode tok/s batch{args.batch} {args.model}-shape {args.mode.capitalize()}"


def workload_config(args, world: int) -> dict:
    """The `config` object of both arms' lines (the same workload, whatever runs it)."""
    if args.sweep:
        return {"workload": "packed linears of shapes 4096x4096, 4096x14336, 14336x4096, 32768x4096 (rows x cols), "
                            "N(0,0.02^2) weights packed in Precision and Turbo, batch 1/4/16/64",
                "shapes": [list(s) for s in SWEEP_SHAPES], "batches": list(SWEEP_BATCHES), "global_batch": None,
                "parallelism": "tp1",
                "l2": "every timed call reads a different copy of the matrix; the copies total more than L2"}
    kv = f"KV length {args.prompt} at the first timed token"
    if args.batch > 1:
        kv += f" (every sequence), {args.max_seq}-entry KV cache per sequence"
    return {"workload": f"{args.model}-shape {args.mode} greedy decode, batch {args.batch}, {kv}, random-init "
                        f"N(0,0.02^2) weights",
            "model": args.model, "mode": args.mode, "prompt": args.prompt, "global_batch": args.batch,
            "parallelism": f"tp{world}",
            "l2": "inputs larger than L2: every step streams all packed weights"}


def physical_cores() -> int:
    """Host cores this process may use: physical cores, bounded by the CPU affinity mask."""
    n_aff = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        import psutil
        phys = psutil.cpu_count(logical=False) or n_aff
    except ImportError:
        phys = n_aff
    return max(1, min(phys, n_aff))


def use_all_cores() -> int:
    """Set the OpenMP thread count of the reference engine to every physical core, whatever the
    launcher exported (torchrun sets OMP_NUM_THREADS=1): the environment variable for a libgomp
    not yet initialised, and omp_set_num_threads for one that is."""
    n = physical_cores()
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(n)
    except (OSError, AttributeError):
        pass
    return n


class ClockSampler:
    """nvidia-smi clocks/throttle sampling, started before the warm-up and stopped after the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index: int):
        self.dev, self.proc = dev_index, None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def init_dist(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def build_model(args, device):
    import gsdlq_b200.packer as P
    cfg = P.make_config(args.model, **({"n_layers": args.layers} if args.layers else {}))
    t0 = time.time()
    dm = P.random_model_cuda(cfg, args.mode, seed=args.seed, device=device)
    return cfg, dm, time.time() - t0


def time_region(fn, steps, world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    fn(steps)
    e.record()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    ms = s.elapsed_time(e)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


# ---- the reference engine on the host cores ----------------------------------------------------
def oracle_model(host, eng, max_seq=2048):
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    tabs = {r: oracle.codebook(r) for r in (6, 8)}

    def rec(t):
        return oracle.hex_record({"radius": t.radius, "k_dim": t.k_dim, "rows": t.rows, "cols": t.cols},
                                 {k: memoryview(np.ascontiguousarray(v)).cast("B") for k, v in t.blobs().items()},
                                 tabs)
    m = {"cfg": host.config, "embed": host.dense["token_embd.weight"].astype(np.float32),
         "final_norm": host.dense["output_norm.weight"], "layers": []}
    for l in range(host.config["n_layers"]):
        lyr = {"attn_norm": host.dense[f"blk.{l}.attn_norm.weight"],
               "ffn_norm": host.dense[f"blk.{l}.ffn_norm.weight"]}
        for n, k in zip(oracle.LINEARS, oracle.KEYS):
            lyr[k] = rec(host.hex[f"blk.{l}.{n}.weight"])
        m["layers"].append(lyr)
    m["lm_head"] = rec(host.hex["output.weight"])
    return oracle.OracleModel(m, eng, max_seq=max_seq)


def reference_engine():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    eng = oracle.CEngine.reference()
    if eng is not None:
        return eng, "reference"
    return oracle.CEngine.restatement(), "port"


def seed_kv(om, P0, seed):
    """KV state at the prompt length: seeded N(0,1) fp16 (attention cost depends on length, not values)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    for c in (om.k_cache, om.v_cache):
        c[:, :P0] = rng.standard_normal(c[:, :P0].shape, dtype=np.float32).astype(np.float16).view(np.uint16)


def timed_tokens(om, P0, warmup, steps, budget_s=REF_TIME_BUDGET_S):
    """Whole greedy decode tokens through the engine from pos P0: (timed count, seconds, per-token s).

    The timed count is `steps`, lowered only when `steps` tokens would take longer than `budget_s`
    at the first warm-up token's rate."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    tok, pos = 7, P0
    t_first = None
    for _ in range(max(1, warmup)):
        t = time.perf_counter()
        tok = oracle.argmax(om.forward_token(tok, pos))
        t_first = t_first or time.perf_counter() - t
        pos = P0 + (pos + 1 - P0) % (om.max_seq - P0)
    n = max(1, min(steps, int(budget_s / max(t_first, 1e-6))))
    ts = []
    for _ in range(n):
        t = time.perf_counter()
        tok = oracle.argmax(om.forward_token(tok, pos))
        ts.append(time.perf_counter() - t)
        pos = P0 + (pos + 1 - P0) % (om.max_seq - P0)
    return n, sum(ts), ts


def cpu_reference_sample(host_model, P0, seed):
    """cpu_baseline of the ours arm: two whole decode tokens through the reference engine on all host cores."""
    cores = use_all_cores()
    eng, kind = reference_engine()
    om = oracle_model(host_model, eng)
    seed_kv(om, P0, seed)
    n, secs, _ = timed_tokens(om, P0, warmup=1, steps=2, budget_s=60.0)
    return {"value": n / secs, "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{n} whole greedy decode tokens from pos {P0} (all layers + final norm + LM head + argmax) "
                      f"through the reference C engine, OpenMP threads = {cores}, after 1 warm-up token"}


# ---- our engine ------------------------------------------------------------------------------
def kind_times(model, world):
    """Device time of each launch kind of a step, each kind as one CUDA graph of its launches over all
    layers back to back (distinct weights per layer, so the weights stream from HBM; no L2 prefetch),
    with the kind's algorithmic bytes per launch.  Consecutive launches alternate between the two
    workspaces."""
    import torch
    from gsdlq_b200 import ops
    kinds = {"qkv": 0, "attn": 1, "o": 2, "gate_up": 3, "down": 4}
    pos = int(model.state[1].item())
    H, hd = model.hidden, model.head_dim
    out = {}
    lay = "blk.0."

    def nb(*names):
        return sum(model.hex[lay + n + ".weight"].nbytes() for n in names)
    q_rows = model.n_heads_local * hd
    kv_rows = model.n_kv_local * hd
    byt = {"qkv": nb("attn_q", "attn_k", "attn_v") + 8 * H + 4 * q_rows + 2 * 2 * kv_rows,
           "attn": 2 * (pos + 1) * kv_rows * 2 + 8 * q_rows,
           "o": nb("attn_output") + 4 * q_rows + 8 * H,
           "gate_up": nb("ffn_gate", "ffn_up") + 8 * H + 4 * model.ffn_local,
           "down": nb("ffn_down") + 4 * model.ffn_local + 8 * H,
           "head": model.hex["output.weight"].nbytes() + 8 * H + 4 * model.vocab_local}
    rep = 5

    def alone(j):  # a copy without the L2 prefetch of the next launch's weights (nothing would read them)
        c = type(j).from_buffer_copy(j)
        c.prefetch.n = 0
        return c
    for name, idx in list(kinds.items()) + [("head", None)]:
        jobs = [alone(lj[idx]) for lj in model.layer_jobs] if idx is not None else [alone(model.head_job)] * 2

        def run_all():
            for i, j in enumerate(jobs):
                if name == "attn":
                    ops.attention(j)
                else:
                    ops.linear(j, model.ws[i % 2])
        run_all()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_all()
        g.replay()

        def reps(n):
            for _ in range(n):
                g.replay()
        ms = time_region(reps, rep, world) / (rep * len(jobs))
        del g
        out[name] = {"us": round(ms * 1e3, 2), "bytes": byt[name], "gbs": round(byt[name] / (ms / 1e3) / 1e9, 1)}
    # the timing runs leave partial sums in the workspaces and a key in the argmax word: clear them
    for w in model.ws:
        w.zero_()
    model.key.zero_()
    torch.cuda.synchronize()
    return out, pos


def comm_time(model, world):
    """Device time per step of the step's collectives alone (2 all-reduces of the hidden vector per layer
    and the argmax MAX), as one CUDA graph, on scratch buffers; max over ranks."""
    import torch
    buf = torch.zeros(model.hidden, dtype=torch.float32, device=model.device)
    key = torch.zeros(1, dtype=torch.int64, device=model.device)

    def coll():
        for _ in range(model.n_layers):
            model.tp.allreduce_buf(buf)
            model.tp.allreduce_buf(buf)
        model.tp.key_max(key)
    coll()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        coll()
    g.replay()

    def reps(n):
        for _ in range(n):
            g.replay()
    ms = time_region(reps, 10, world) / 10
    del g
    torch.cuda.synchronize()
    return ms * 1e3


def run_ours(args):
    import numpy as np
    import torch
    world, rank, local = init_dist(args)
    device = torch.device("cuda", local)
    from gsdlq_b200.model import GSDLQModel
    from gsdlq_b200 import _lib as L
    tp = None
    if world > 1:
        from gsdlq_b200.tp import TensorParallel
        tp = TensorParallel(rank, world)
    cfg, dm, pack_s = build_model(args, device)
    model = GSDLQModel(dm, device=device, tp=tp, fused_step=args.step == "fused")
    host_model = None
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        import gsdlq_b200.packer as P
        host_model = P.device_model_to_host(dm)
    del dm
    V, P0 = cfg["vocab_size"], args.prompt
    rng = np.random.default_rng(args.seed + 1)
    prompt = rng.integers(0, V, P0).tolist()
    # prefill time of the prompt with chunked tensor-core prefill (one GPU), then the KV state of the timed
    # steps from token-by-token prefill at every N, so that the greedy ids compare across N
    prefill_s = prefill_token_s = None
    if world == 1:
        t0 = time.time()
        model.prefill(prompt[:-1], batched=True)
        torch.cuda.synchronize()
        prefill_s = time.time() - t0
    t0 = time.time()
    model.prefill(prompt[:-1], batched=False)
    torch.cuda.synchronize()
    prefill_token_s = time.time() - t0
    span = model.max_seq - (P0 - 1)

    state = {"pos": P0 - 1}
    model.set_state(prompt[-1], P0 - 1)

    def steps(n):
        for _ in range(n):
            if state["pos"] >= model.max_seq:
                state["pos"] = P0 - 1
                model.state[1:2].fill_(P0 - 1)  # device-side position reset (wrap), stream-ordered
            model.step(with_head=True)
            state["pos"] += 1

    sampler = ClockSampler(local)
    sampler.start()  # before the warm-up, so that its start-up lands outside the timed region
    steps(args.warmup)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("decode")  # lets a profiler select the timed steps (ncu --nvtx-include decode/)
    ms = time_region(steps, args.steps, world)
    torch.cuda.nvtx.range_pop()
    clocks = sampler.stop()
    flags = L.device_flags()
    if flags:
        raise RuntimeError(f"device flags raised during the bench: {L.flag_names(flags)}")
    # the greedy ids of the timed steps (the same on every rank; equal across N when TP is correct)
    n_ids = min(args.warmup + args.steps, model.out_ids.numel())
    ids = model.out_ids[args.warmup:n_ids].cpu().numpy().astype(np.int32)
    ids_sha = hashlib.sha256(ids.tobytes()).hexdigest()[:16]
    tok_s = args.steps / (ms / 1e3)
    ms_step = ms / args.steps
    mean_pos = P0 + min(span, args.warmup + args.steps) / 2
    bytes_tok = model.packed_bytes_per_token(pos=int(mean_pos))
    pk, pk_src = peaks()
    hbm = float(pk["hbm_gbs"])

    kinds, kinds_pos = ({}, None) if args.no_kinds else kind_times(model, world)
    comm_us = comm_time(model, world) if world > 1 else None
    if kinds:
        gu_ms, gu_bytes, gu_gbs = kinds["gate_up"]["us"] / 1e3, kinds["gate_up"]["bytes"], kinds["gate_up"]["gbs"]
    else:
        gu_ms = gu_bytes = gu_gbs = None

    e2e = None
    if rank == 0 and world == 1 and args.e2e_steps > 0:
        n = min(args.e2e_steps, model.max_seq - P0)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tok = prompt[-1]
        model.forward_token(tok, P0 - 1)
        s.record()
        for i in range(n):
            lg = model.forward_token(tok, P0 + i)   # H2D (token, pos, step) + D2H logits each step
            tok = int(np.argmax(lg))
        e.record()
        torch.cuda.synchronize()
        e_ms = s.elapsed_time(e) / n
        e2e = {"value": 1e3 / e_ms, "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4 * V,
               "api": "GSDLQModel.forward_token(token_id, pos) -> np.float32[vocab]"}
    elif world > 1 and args.e2e_steps > 0:
        # every rank runs the same public calls (set_state: H2D of token and position; step; the greedy
        # token read back), so the ranks' collectives stay in step; device time, max over ranks
        import torch.distributed as dist
        n = min(args.e2e_steps, model.max_seq - P0)
        tok = prompt[-1]
        model.set_state(tok, P0 - 1)
        model.step(with_head=True)
        tok = int(model.state[0].item())
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(n):
            model.set_state(tok, P0 + i)
            model.step(with_head=True)
            tok = int(model.state[0].item())
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / n], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = {"value": 1e3 / float(t.item()), "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4,
               "api": "GSDLQModel.set_state(token_id, pos) + step() + the greedy token read from the device"}

    cpu = None
    if host_model is not None:
        cpu = cpu_reference_sample(host_model, P0, args.seed + 2)

    # our kernels per step: 5 per layer (QKV, attention, O, gate/up, down), the LM head and the greedy advance;
    # one persistent launch per step with the fused step (collective launches are NCCL's, not counted)
    launches_per_step = 1 if model.fused_step else 5 * model.n_layers + 2
    if rank == 0:
        conf = workload_config(args, world)
        line = {
            "metric": metric_name(args), "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": vs_published(args, tok_s), "dtype": "f32",
            "data": "synthetic", "config": conf,
            "token_bytes": bytes_tok, "token_gbs": bytes_tok / (ms_step / 1e3) / 1e9,
            "token_hbm_frac": bytes_tok / (ms_step / 1e3) / 1e9 / hbm,
            "roofline": None if not kinds else {
                "bound": "hbm", "kernel": "hexmv_kernel<SWIGLU> (fused gate/up linear)",
                "achieved": gu_gbs, "peak": hbm, "unit": "GB/s", "frac": gu_gbs / hbm,
                "peak_source": f"{pk_src} hbm_gbs", "bytes_per_launch": gu_bytes, "launch_ms": gu_ms,
                "traffic": GU_TRAFFIC * gu_bytes / GU_ALGO if (args.model == "mistral-7b" and
                                                               args.mode == "precision") else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one full gate/up launch of "
                                  "this workload on one GPU, scaled by this launch's share of its bytes"},
            "kinds": kinds, "kinds_pos": kinds_pos, "comm_us_per_step": comm_us, "ids_sha": ids_sha,
            "ids_head": ids[:8].tolist(),
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks, "pack_s": round(pack_s, 2),
            "prefill_s": round(prefill_s, 3) if prefill_s is not None else None,
            "prefill_tok_s": round((P0 - 1) / prefill_s, 1) if prefill_s else None,
            "prefill_token_by_token_s": round(prefill_token_s, 3),
            "prefill_roofline": prefill_roofline(cfg, P0 - 1, prefill_s, pk, pk_src) if prefill_s else None,
            "avg_bpw": round(model.avg_bpw, 4), "step": "fused" if model.fused_step else "per-op",
            "n_layers": model.n_layers, "l2_prefetch": model.prefetch,
            "tp_exchange": model.tp.exchange if model.tp is not None else None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        model.release()
        dist.destroy_process_group()


def _clone_hex(h):
    from gsdlq_b200.ops import DeviceHex
    t = {k: (getattr(h, k).clone() if getattr(h, k, None) is not None else None)
         for k in ("codes", "scales", "row_ptr", "kink_cols", "kink_deltas", "U", "S", "Vt")}
    return DeviceHex(None, rows=h.rows, cols=h.cols, k_dim=h.k_dim, radius=h.radius, nnz=h.nnz, **t)


def _event_us(fn, reps):
    import torch
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(reps):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / reps


def run_batch(args):
    """Batched greedy decode: args.batch sequences in lockstep (BatchDecoder), one GPU."""
    import math
    import numpy as np
    import torch
    world, rank, local = init_dist(args)
    if world > 1:
        if rank == 0:
            print(json.dumps({"impl": "ours", "unavailable": "batched decode runs on one GPU (--batch > 1 with N=1)"}))
        return
    device = torch.device("cuda", local)
    from gsdlq_b200.model import GSDLQModel
    from gsdlq_b200.batch import BatchDecoder
    from gsdlq_b200 import _lib as L, ops
    import gsdlq_b200.packer as P
    cfg, dm, pack_s = build_model(args, device)
    S, B, P0, V = args.max_seq, args.batch, args.prompt, cfg["vocab_size"]
    model = GSDLQModel(dm, device=device, max_seq=S)
    host_model = None if args.no_cpu_baseline else P.device_model_to_host(dm)
    del dm
    bd = BatchDecoder(model, B, max_seq=S)
    rng = np.random.default_rng(args.seed + 1)
    prompts = [rng.integers(0, V, P0).tolist() for _ in range(B)]
    torch.cuda.synchronize()
    t0 = time.time()
    for b, pr in enumerate(prompts):
        bd.prefill(b, pr[:-1])
    torch.cuda.synchronize()
    prefill_s = time.time() - t0
    bd.set_tokens([pr[-1] for pr in prompts], [P0 - 1] * B)
    state = {"pos": P0 - 1}

    def steps(n):
        for _ in range(n):
            if state["pos"] >= S:
                state["pos"] = P0 - 1
                bd.pos.fill_(P0 - 1)  # device-side position reset (wrap), stream-ordered
            bd.step()
            state["pos"] += 1

    sampler = ClockSampler(local)
    sampler.start()
    steps(args.warmup)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("decode")
    ms = time_region(steps, args.steps, 1)
    torch.cuda.nvtx.range_pop()
    clocks = sampler.stop()
    flags = L.device_flags()
    if flags:
        raise RuntimeError(f"device flags raised during the bench: {L.flag_names(flags)}")
    out = bd.out_ids.cpu().numpy()
    ids_sha = hashlib.sha256(out[:, P0:P0 + 16].astype(np.int32).tobytes()).hexdigest()[:16]
    ms_step = ms / args.steps
    tok_s = B * args.steps / (ms / 1e3)
    span = S - (P0 - 1)
    mean_pos = P0 + min(span, args.warmup + args.steps) / 2
    kv_bytes = 2 * model.n_layers * int(mean_pos + 1) * model.n_kv_local * model.head_dim * 2  # per sequence
    w_bytes = sum(h.nbytes() for h in model.hex.values()) + B * model.hidden * 2
    step_bytes = w_bytes + B * kv_bytes
    pk, pk_src = peaks()
    hbm = float(pk["hbm_gbs"])
    # the two kernel kinds that carry the step's bytes, each timed alone: one layer's batched decode
    # attention (its KV rows) and the largest linear's dequant-GEMM
    pos_mid = torch.full((B,), int(mean_pos), dtype=torch.int32, device=device)
    sm = 1.0 / math.sqrt(model.head_dim)
    lib, sh = L.load(), ops.stream_handle()

    def attn(i):
        L.check(lib.gsdlq_attention_decode_batch(bd.q.data_ptr(), 0, bd.k_cache.data_ptr(), bd.v_cache.data_ptr(),
                                                 bd.seq_stride, bd.att.data_ptr(), bd.awork.data_ptr(),
                                                 bd.awork.numel(), i % model.n_layers, pos_mid.data_ptr(), B,
                                                 model.n_heads_local, model.n_kv_local, model.head_dim, S, sm, sh),
                "attention_decode_batch")
    attn(0)
    attn_us = _event_us(attn, 3 * model.n_layers)
    attn_bytes = kv_bytes // model.n_layers * B
    names = [f"blk.{l}.ffn_gate.weight" for l in range(model.n_layers)]
    gx = torch.randn((B, model.hidden), device=device)

    def gate(i):
        h = model.hex[names[i % len(names)]]
        ops.hex2d_matmul(gx, h, bd.xy[h.radius], bd.g, bd.work)
    gate(0)
    gate_us = _event_us(gate, 2 * len(names))
    gate_bytes = model.hex[names[0]].nbytes()
    kinds = {"attention": {"us": round(attn_us, 2), "bytes": attn_bytes, "gbs": round(attn_bytes / attn_us / 1e3, 1),
                           "launches_per_step": model.n_layers},
             "ffn_gate_gemm": {"us": round(gate_us, 2), "bytes": gate_bytes,
                               "gbs": round(gate_bytes / gate_us / 1e3, 1), "launches_per_step": model.n_layers}}
    dom = max(kinds, key=lambda k: kinds[k]["us"] * kinds[k]["launches_per_step"])
    kd = kinds[dom]
    # e2e through the public surface: host token ids and positions in, greedy picks out, every step
    n_e2e = min(args.e2e_steps, S - P0)
    e2e = None
    if n_e2e > 0:
        ids_h = np.array([pr[-1] for pr in prompts], np.int32)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for i in range(n_e2e):
            bd.set_tokens(ids_h, np.full(B, P0 - 1 + i, np.int32))
            bd.step()
            ids_h = bd.ids.cpu().numpy()
        e.record()
        torch.cuda.synchronize()
        e_ms = s.elapsed_time(e) / n_e2e
        e2e = {"value": B * 1e3 / e_ms, "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B,
               "api": "BatchDecoder.set_tokens(ids, positions) + step() + the picks read back"}
    cpu = None
    if host_model is not None:
        cpu = cpu_reference_sample(host_model, P0, args.seed + 2)
        cpu["sample"] += "; the reference decodes one sequence at a time, so its batch rate is this rate"
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    splits = max(1, min(8, -(-4 * sms // (B * model.n_kv_local)), -(-S // 32)))
    qkv_g = 1 if any(k.endswith("qkv") for k in bd.fused) else 3
    gu_g = 1 if any(k.endswith("gu") for k in bd.fused) else 2
    per_layer = 1 + 3 * qkv_g + 1 + 1 + (1 if splits > 1 else 0) + 3 + 1 + 1 + 3 * gu_g + 1 + 3 + 1
    launches = 1 + per_layer * model.n_layers + 1 + 3 + 1  # a GEMM call is 3 kernels
    line = {
        "metric": metric_name(args), "value": tok_s, "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(args, 1),
        "step_bytes": step_bytes, "step_gbs": step_bytes / (ms_step / 1e3) / 1e9,
        "step_hbm_frac": step_bytes / (ms_step / 1e3) / 1e9 / hbm,
        "roofline": {"bound": "hbm", "kernel": "attention_decode_kernel" if dom == "attention" else "hexmm_kernel",
                     "achieved": kd["gbs"], "peak": hbm, "unit": "GB/s", "frac": kd["gbs"] / hbm,
                     "peak_source": f"{pk_src} hbm_gbs", "bytes_per_launch": kd["bytes"], "launch_ms": kd["us"] / 1e3,
                     "traffic": None},
        "kinds": kinds, "ids_sha": ids_sha, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches * args.steps,
        "clocks": clocks, "pack_s": round(pack_s, 2), "prefill_s": round(prefill_s, 3),
        "prefill_tok_s": round(B * (P0 - 1) / prefill_s, 1),
        "prefill_roofline": prefill_roofline(cfg, P0 - 1, prefill_s, pk, pk_src, sequences=B),
        "avg_bpw": round(model.avg_bpw, 4),
        "n_layers": model.n_layers,
    }
    print(json.dumps(line), flush=True)


def run_sweep(args):
    """The packed-linear bandwidth sweep: each shape and mode, the drop-in unpack-matvec at B = 1 and the
    dequant-GEMM at B = 1/4/16/64, each call reading a different copy of the matrix."""
    import numpy as np
    import torch
    world, rank, local = init_dist(args)
    if world > 1:
        if rank == 0:
            print(json.dumps({"impl": "ours", "unavailable": "the sweep runs on one GPU"}))
        return
    device = torch.device("cuda", local)
    import gsdlq_b200.packer as P
    from gsdlq_b200 import _lib as L, ops
    pk, pk_src = peaks()
    hbm = float(pk["hbm_gbs"])
    sampler = ClockSampler(local)
    sampler.start()
    rows_out, head = [], None
    torch.manual_seed(args.seed)
    for mode in ("precision", "turbo"):
        for (R, C) in SWEEP_SHAPES:
            w = torch.randn(R, C, device=device) * 0.02
            h = P.pack_matrix_cuda(w, mode, seed=args.seed)
            del w
            nb = h.nbytes()
            copies = [h] + [_clone_hex(h) for _ in range(max(1, -(-3 * 126 * 2 ** 20 // nb)) - 1)]
            xy = torch.from_numpy(ops.codebook(h.radius)).to(device)
            x = torch.randn((max(SWEEP_BATCHES), C), device=device)
            y = torch.zeros((max(SWEEP_BATCHES), R), device=device)
            tk = torch.zeros(16, device=device)
            work = ops.matmul_work(max(SWEEP_BATCHES), C, device)

            def mv(i):
                c = copies[i % len(copies)]
                if c.k_dim:
                    ops.lowrank_proj(x[0], c, tk)
                ops.hex2d_matvec(x[0], c, xy, tk, y[0])
            mv(0)
            us = _event_us(mv, 4 * len(copies))
            rows_out.append({"shape": [R, C], "mode": mode, "batch": 1, "kernel": "unpack-matvec (hexmv)",
                             "us": round(us, 2), "gbs": round(nb / us / 1e3, 1), "hbm_frac": round(nb / us / 1e3 / hbm, 3),
                             "bytes": nb})
            for B in SWEEP_BATCHES:
                def mm(i, B=B):
                    ops.hex2d_matmul(x[:B], copies[i % len(copies)], xy, y[:B], work)
                mm(0)
                us = _event_us(mm, 4 * len(copies))
                e = {"shape": [R, C], "mode": mode, "batch": B, "kernel": "dequant-GEMM (hexmm, tcgen05)",
                     "us": round(us, 2), "gbs": round(nb / us / 1e3, 1), "hbm_frac": round(nb / us / 1e3 / hbm, 3),
                     "useful_tflops": round(2.0 * R * C * B / us / 1e6, 2), "bytes": nb}
                rows_out.append(e)
                if (R, C) == (14336, 4096) and mode == "precision" and B == 16:
                    head = e
            del copies, h
            torch.cuda.empty_cache()
    clocks = sampler.stop()
    flags = L.device_flags()
    if flags:
        raise RuntimeError(f"device flags raised during the sweep: {L.flag_names(flags)}")
    line = {"metric": metric_name(args), "value": head["gbs"], "unit": "GB/s", "n_gpus": 1, "steps": None,
            "warmup": 1, "ms_per_step": head["us"] / 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(args, 1),
            "value_is": "14336x4096 Precision, batch 16, dequant-GEMM",
            "roofline": {"bound": "hbm", "kernel": "hexmm_kernel", "achieved": head["gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": head["gbs"] / hbm, "peak_source": f"{pk_src} hbm_gbs", "traffic": None},
            "sweep": rows_out, "clocks": clocks,
            "tensor_pipe": "sm__pipe_tensor_cycles_active from ncu, in the profiles folder (hexmm_kernel summary)"}
    print(json.dumps(line), flush=True)


def run_reference_sweep(args):
    """The reference's unpack-matvec (its C engine) on the host cores for each sweep shape and mode; the
    reference has no batched path, so batch B costs B matvecs."""
    import numpy as np
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cores = use_all_cores()
    import gsdlq_b200.packer as P
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    eng, kind = reference_engine()
    tabs = {r: oracle.codebook(r) for r in (6, 8)}
    rows_out, head = [], None
    rng = np.random.default_rng(args.seed)
    for mode in ("precision", "turbo"):
        for (R, C) in SWEEP_SHAPES:
            cfg = {"n_layers": 0}
            t = P.random_packed_matrix(R, C, mode, seed=args.seed) if hasattr(P, "random_packed_matrix") else None
            if t is None:
                raise RuntimeError("packer.random_packed_matrix missing")
            rec = oracle.hex_record({"radius": t.radius, "k_dim": t.k_dim, "rows": t.rows, "cols": t.cols},
                                    {k: memoryview(np.ascontiguousarray(v)).cast("B") for k, v in t.blobs().items()},
                                    tabs)
            x = rng.standard_normal(C).astype(np.float32)
            eng.matvec(x, rec, np.zeros(16, np.float32))
            n, t0 = 0, time.perf_counter()
            while n < 3 or time.perf_counter() - t0 < 1.0:
                eng.matvec(x, rec, np.zeros(16, np.float32))
                n += 1
            us = (time.perf_counter() - t0) / n * 1e6
            nb = t.nbytes()
            e = {"shape": [R, C], "mode": mode, "batch": 1, "us": round(us, 1), "gbs": round(nb / us / 1e3, 2),
                 "bytes": nb, "calls": n}
            rows_out.append(e)
            if (R, C) == (14336, 4096) and mode == "precision":
                head = e
    line = {"metric": metric_name(args), "value": head["gbs"], "unit": "GB/s", "n_gpus": world, "steps": None,
            "warmup": 1, "ms_per_step": head["us"] / 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": workload_config(args, world), "value_is": "14336x4096 Precision, one matvec",
            "cpu_baseline": {"value": head["gbs"], "unit": "GB/s", "cores": cores, "kind": kind,
                             "sample": "repeated matvecs of one packed matrix per shape and mode for about 1 s each"},
            "e2e": {"value": head["gbs"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "sweep": rows_out, "runs_on": f"host cores ({cores} OpenMP threads), no GPU"}
    print(json.dumps(line), flush=True)


def run_reference(args):
    """The reference's C engine on the host cores (no GPU, no library of this repository)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = use_all_cores()  # before the engine (and its OpenMP runtime) is loaded
    import gsdlq_b200.packer as P
    cfg = P.make_config(args.model, **({"n_layers": args.layers} if args.layers else {}))
    t0 = time.time()
    host = P.random_packed_model(cfg, args.mode, seed=args.seed)
    pack_s = time.time() - t0
    eng, kind = reference_engine()
    om = oracle_model(host, eng)
    P0 = args.prompt
    seed_kv(om, P0, args.seed + 2)
    n, secs, ts = timed_tokens(om, P0, args.warmup, args.steps)
    tok_s = n / secs
    sample = (f"{n} whole greedy decode tokens from pos {P0} (all {om.n_layers} layers + final norm + LM head + "
              f"argmax) after {max(1, args.warmup)} warm-up tokens, OpenMP threads = {cores}; packed bytes of the "
              f"same shapes drawn with NumPy (random_packed_model)")
    conf = workload_config(args, world)
    line = {"metric": metric_name(args), "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": n,
            "warmup": max(1, args.warmup), "ms_per_step": 1e3 * secs / n, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": vs_published(args, tok_s), "dtype": "f32",
            "data": "synthetic", "impl": "reference", "config": conf,
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "token_ms": [round(1e3 * t, 1) for t in ts[:8]], "pack_s": round(pack_s, 2),
            "avg_bpw": round(host.avg_bpw, 4), "runs_on": f"host cores ({cores} OpenMP threads), no GPU"}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference_sweep(a) if a.sweep else run_reference(a)
    elif a.sweep:
        run_sweep(a)
    elif a.batch > 1:
        run_batch(a)
    else:
        run_ours(a)

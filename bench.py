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
GU_TRAFFIC = 66_794_752 + 727_296
GU_ALGO = 66_527_368
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
REF_TIME_BUDGET_S = 240.0  # the reference arm's timed tokens are capped to about this much host time


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


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
    return ap.parse_args()


def workload_config(args, world: int) -> dict:
    """The `config` object of both arms' lines (the same workload, whatever runs it)."""
    return {"workload": f"{args.model}-shape {args.mode} greedy decode, batch 1, KV length {args.prompt} at the "
                        f"first timed token, random-init N(0,0.02^2) weights",
            "model": args.model, "mode": args.mode, "prompt": args.prompt, "global_batch": 1,
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
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
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
            "avg_bpw": round(model.avg_bpw, 4), "step": "fused" if model.fused_step else "per-op",
            "n_layers": model.n_layers, "l2_prefetch": model.prefetch,
            "tp_exchange": model.tp.exchange if model.tp is not None else None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        model.release()
        dist.destroy_process_group()


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
    line = {"metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": n,
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
        run_reference(a)
    else:
        run_ours(a)

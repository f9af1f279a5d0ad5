"""GSDLQModel: the reference's model surface on the B200 engine.

Surface kept from the reference (gsd_lq_v2/run_gpu_native_chat.py:732-984 and
gsd_lq_v2/gsd_lq_cpu_runtime.py:121-443):

    m = GSDLQModel("model.gsd2", rope_interleaved=1)
    logits = m.forward_token(token_id, pos, return_logits=True)   # np.float32[vocab] | None
    nxt = m.sample_token(logits, temperature=0.0, top_p=0.9)
    m.cfg, m.avg_bpw, m.vram_used_mb, m.cl.total_vram_mb, m.cl.release_all(), m.tokenizer

One decode step is, per layer (5 launches; no host round trip inside a step):

    1. QKV   fused linear: RMSNorm prologue (layer 0: embedding lookup), Q/K/V with
             in-kernel low-rank + kinks, RoPE + fp16 KV append epilogue
    2. attention (split-KV, last CTA combines)
    3. O     fused linear, residual-add epilogue into x
    4. gate/up fused linear: RMSNorm prologue, SwiGLU epilogue
    5. down  fused linear, residual-add epilogue into x

then the LM head (RMSNorm prologue, fused greedy argmax).  The layer stack and
the head are each captured once in a CUDA graph and replayed; the token id and
position are read from device memory, so replays need no re-capture.
"""
from __future__ import annotations

import ctypes
import math
import os
import time

import numpy as np
import torch

from . import _lib as L
from . import ops
from .gsd2 import PackedModel, read_gsd2, HexTensor
from .tokenizer import from_config as tokenizer_from_config

MAX_SEQ_LEN = 2048  # the reference's compile-time cache length (run_gpu_native_chat.py:99)


class _DeviceInfo:
    """Stands in for the reference's ``model.cl`` OpenCL runtime object."""

    def __init__(self, model: "GSDLQModel"):
        self._m = model
        p = torch.cuda.get_device_properties(model.device)
        self.total_vram_mb = p.total_memory / (1024 * 1024)
        self.device_name = p.name

    def release_all(self):
        self._m.release()


class DevicePacked:
    """A packed model whose tensors are already in device memory (GPU packer output)."""

    def __init__(self, config: dict, hexes: dict, dense: dict, avg_bpw: float, mode: str):
        self.config, self.hexes, self.dense, self.avg_bpw, self.mode = config, hexes, dense, avg_bpw, mode


class GSDLQModel:
    def __init__(self, source, rope_interleaved: int = 1, device=None, max_seq: int = MAX_SEQ_LEN,
                 use_graph: bool = True, verbose: bool = False, tp=None, unit_kinks: bool = False,
                 fused_step: bool = False, lr_forward: bool = True, prefetch: int | None = None):
        t0 = time.time()
        if not torch.cuda.is_available():
            raise RuntimeError("GSDLQModel needs a CUDA device (there is no CPU path)")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        torch.cuda.set_device(self.device)
        L.load()
        if rope_interleaved != 1:
            raise NotImplementedError("the fused decode step implements interleaved RoPE, the only mode the "
                                      "reference runtime uses (run_gpu_native_chat.py:1061-1077); the drop-in "
                                      "gsdlq_rope_and_store_kv supports both")
        self.rope_interleaved = rope_interleaved
        self.max_seq = max_seq
        self.use_graph = use_graph
        self.tp = tp
        self.unit_kinks = unit_kinks
        self._want_fused = fused_step and tp is None
        self.lr_forward = lr_forward
        # L2 prefetch policy of the launches (see _wire_prefetch); GSDLQ_PREFETCH overrides the default
        self.prefetch = int(os.environ.get("GSDLQ_PREFETCH", "0")) if prefetch is None else int(prefetch)
        self._plans: dict = {}
        if isinstance(source, str):
            source = read_gsd2(source)
        self._load(source)
        if self.tp is not None:
            self.tp.setup(self)  # the residual exchange among the ranks (collective: every rank calls it)
            self._wire_exchange()
        self.cl = _DeviceInfo(self)
        self.tokenizer = tokenizer_from_config(self.cfg)  # SentencePiece BPE over the header's vocabulary
        self._graphs: dict = {}
        self.load_seconds = time.time() - t0
        if verbose:
            print(f"[gsdlq] loaded in {self.load_seconds:.2f}s, {self.vram_used_mb:.1f} MB on {self.cl.device_name}")

    # ------------------------------------------------------------------ loading
    def _load(self, src):
        dev = self.device
        c = dict(src.config)
        self.cfg = c
        self.n_layers, self.hidden = c["n_layers"], c["hidden_size"]
        self.n_heads, self.n_kv_heads, self.head_dim = c["n_heads"], c["n_kv_heads"], c["head_dim"]
        self.ffn_size, self.vocab_size = c["ffn_size"], c["vocab_size"]
        self.rms_eps, self.rope_theta = float(c["rms_eps"]), float(c["rope_theta"])
        self.avg_bpw = float(src.avg_bpw)
        self.mode = getattr(src, "mode", "unknown")
        if self.tp is not None:
            src = self.tp.shard(src)
            c = self.cfg = dict(src.config)
        self.n_heads_local = c.get("n_heads_local", self.n_heads)
        self.n_kv_local = c.get("n_kv_heads_local", self.n_kv_heads)
        self.ffn_local = c.get("ffn_size_local", self.ffn_size)
        self.vocab_local = c.get("vocab_size_local", self.vocab_size)
        if isinstance(src, DevicePacked):
            self.hex = src.hexes
            self.embed = src.dense["token_embd.weight"]
            self.norms = {k: v for k, v in src.dense.items() if k != "token_embd.weight"}
        else:
            hexes: dict[str, HexTensor] = src.hex
            blobs = [a for t in hexes.values() for a in t.blobs().values()]
            arena = ops.Arena(ops.Arena.bytes_needed(blobs), dev)
            self._arena = arena
            self.hex = {n: ops.DeviceHex(t, dev, arena=arena) for n, t in hexes.items()}
            self.embed = torch.from_numpy(np.ascontiguousarray(src.dense["token_embd.weight"])).to(dev)
            self.norms = {k: torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(dev)
                          for k, v in src.dense.items() if k != "token_embd.weight"}
        if self.unit_kinks:
            # kinks regrouped per work unit: the fused linear applies them in its streaming loop
            for h in self.hex.values():
                h.build_unit_kinks()
        H, Lc = self.hidden, self.n_layers
        hd, kvl, hl = self.head_dim, self.n_kv_local, self.n_heads_local
        f32 = dict(dtype=torch.float32, device=dev)
        self.k_cache = torch.zeros((Lc, self.max_seq, kvl, hd), dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.x = torch.zeros(H, **f32)
        self.q = torch.zeros(hl * hd, **f32)
        self.att = torch.zeros(hl * hd, **f32)
        self.h = torch.zeros(self.ffn_local, **f32)
        self.logits = torch.zeros(self.vocab_local, **f32)
        self.state = torch.zeros(4, dtype=torch.int32, device=dev)      # token, pos, step, spare
        self.key = torch.zeros(2, dtype=torch.int64, device=dev)        # greedy argmax key (u64 bits)
        self.out_ids = torch.zeros(max(self.max_seq, 1), dtype=torch.int32, device=dev)
        self.rope_cs = torch.from_numpy(ops.rope_table(self.max_seq, hd, self.rope_theta)).to(dev)
        pb, wb = ops.attention_ws_size(hl, kvl, hd, self.max_seq)
        self.attn_partial = torch.zeros(pb // 4 + 1, **f32)
        self.attn_ws = torch.zeros(wb // 4 + 1, dtype=torch.int32, device=dev)
        self._build_jobs()
        if self._want_fused:
            self._build_plans()
        torch.cuda.synchronize(dev)
        self.vram_used_mb = self._bytes_resident() / (1024 * 1024)

    def _bytes_resident(self) -> int:
        n = sum(h.nbytes() for h in self.hex.values())
        n += self.embed.numel() * 2 + sum(t.numel() * 4 for t in self.norms.values())
        n += 2 * self.k_cache.numel() * 2
        return n

    def packed_bytes_per_token(self, pos: int | None = None) -> int:
        """Algorithmic bytes one decode step must read: all packed linears + KV rows read + embedding row."""
        n = sum(h.nbytes() for h in self.hex.values()) + self.hidden * 2
        if pos is not None:
            n += 2 * self.n_layers * (pos + 1) * self.n_kv_local * self.head_dim * 2
        return n

    # ------------------------------------------------------------------ jobs
    def _job(self, mats, input_mode, x=None, norm=None, epilogue=L.EPI_STORE, ys=(), resid=None, layer=0,
             argmax=False):
        j = L.LinearJob()
        for i, m in enumerate(mats):
            j.mat[i] = m.desc()
        j.n_mat = len(mats)
        j.input_mode = input_mode
        j.x = x.data_ptr() if x is not None else None
        j.norm_w = norm.data_ptr() if norm is not None else None
        j.eps = self.rms_eps
        if input_mode == L.IN_EMBED:
            j.embed = self.embed.data_ptr()
            j.token = self.state.data_ptr()
            j.vocab = self.vocab_size
            j.x_out = self.x.data_ptr()
        j.epilogue = epilogue
        for i, y in enumerate(ys):
            j.y[i] = y.data_ptr() if y is not None else None
        j.resid = resid.data_ptr() if resid is not None else None
        j.k_cache = self.k_cache.data_ptr()
        j.v_cache = self.v_cache.data_ptr()
        j.pos = self.state.data_ptr() + 4
        j.rope_cs = self.rope_cs.data_ptr()
        j.layer, j.max_seq, j.head_dim, j.interleaved = layer, self.max_seq, self.head_dim, 1
        j.argmax_key = self.key.data_ptr() if argmax else None
        j.argmax_index_base = self.tp.rank * self.vocab_local if (argmax and self.tp is not None) else 0
        return j

    def _build_jobs(self):
        self.layer_jobs = []
        for l in range(self.n_layers):
            p = f"blk.{l}."
            hx = lambda n: self.hex[p + n + ".weight"]  # noqa: E731
            an, fn = self.norms[p + "attn_norm.weight"], self.norms[p + "ffn_norm.weight"]
            qkv = self._job([hx("attn_q"), hx("attn_k"), hx("attn_v")],
                            L.IN_EMBED if l == 0 else L.IN_RMSNORM, x=self.x, norm=an,
                            epilogue=L.EPI_ROPE_KV, ys=(self.q, None, None), layer=l)
            att = L.AttnJob(q=self.q.data_ptr(), k_cache=self.k_cache.data_ptr(), v_cache=self.v_cache.data_ptr(),
                            out=self.att.data_ptr(), pos_dev=self.state.data_ptr() + 4, pos_val=0, layer=l,
                            n_heads=self.n_heads_local, n_kv_heads=self.n_kv_local, head_dim=self.head_dim,
                            max_seq=self.max_seq, sm_scale=1.0 / math.sqrt(self.head_dim), block_table=None,
                            page_size=0, partial=self.attn_partial.data_ptr(), workspace=self.attn_ws.data_ptr())
            # tensor parallel: rank 0 adds its partial to the residual, the other ranks store their bare
            # partials into x; the all-reduce(sum) that follows leaves x + sum of partials everywhere
            res_epi = L.EPI_RESID if (self.tp is None or self.tp.rank == 0) else L.EPI_STORE
            o = self._job([hx("attn_output")], L.IN_PLAIN, x=self.att, epilogue=res_epi,
                          ys=(self.x,), resid=self.x)
            gu = self._job([hx("ffn_gate"), hx("ffn_up")], L.IN_RMSNORM, x=self.x, norm=fn,
                           epilogue=L.EPI_SWIGLU, ys=(self.h,))
            dn = self._job([hx("ffn_down")], L.IN_PLAIN, x=self.h, epilogue=res_epi,
                           ys=(self.x,), resid=self.x)
            self.layer_jobs.append((qkv, att, o, gu, dn))
        self.head_job = self._job([self.hex["output.weight"]], L.IN_RMSNORM, x=self.x,
                                  norm=self.norms["output_norm.weight"], epilogue=L.EPI_STORE, ys=(self.logits,),
                                  argmax=True)
        # Workspaces: consecutive fused-linear launches may overlap (programmatic dependent
        # launch), so they alternate between two buffers; each launch leaves its own at zero.
        jobs = [j for lj in self.layer_jobs for j in (lj[0], lj[2], lj[3], lj[4])] + [self.head_job]
        need = max(ops.linear_ws_size(j) for j in jobs)
        self.ws = [torch.zeros((need + 15) // 16 * 4, dtype=torch.int32, device=self.device) for _ in range(2)]
        self.ws_of = {}
        k = 0
        for lj in self.layer_jobs:
            for j in (lj[0], lj[2], lj[3], lj[4]):
                self.ws_of[id(j)] = self.ws[k % 2]
                k += 1
        self.ws_of[id(self.head_job)] = self.ws[k % 2]
        if self.tp is None and self.lr_forward:
            self._wire_forwarding()
        self._wire_prefetch(self.prefetch)

    def _wire_forwarding(self):
        """Low-rank forwarding: every op whose output is the next linear's input adds that linear's
        projection of it (strip by strip, fixed point) to the next launch's workspace, which then
        skips its own grid-wide projection.  (Tensor parallelism forwards only with the fused
        exchange, whose O and down epilogues hold the summed residual; with separate all-reduce
        launches they see partial sums and every launch keeps its in-kernel projection.)"""
        def acc(job):
            return self.ws_of[id(job)].data_ptr() + 64  # the workspace's accumulator words

        def into(src, dst, mats, norm):
            if sum(m.k_dim for m in mats) == 0:
                return  # no low-rank term to forward
            for i in range(3):
                src.fwd_vt[i] = mats[i].desc().Vt if i < len(mats) and mats[i].k_dim > 0 else None
                src.fwd_k[i] = mats[i].k_dim if i < len(mats) else 0
            src.fwd_norm_w = norm.data_ptr() if norm is not None else None
            src.fwd_acc = acc(dst)
            dst.lr_forwarded = 1

        hx = lambda l, n: self.hex[f"blk.{l}.{n}.weight"]  # noqa: E731
        for l, (qkv, att, o, gu, dn) in enumerate(self.layer_jobs):
            ho = hx(l, "attn_output")
            if ho.k_dim > 0:
                att.fwd_vt, att.fwd_k, att.fwd_acc = ho.desc().Vt, ho.k_dim, acc(o)
                o.lr_forwarded = 1
            into(o, gu, [hx(l, "ffn_gate"), hx(l, "ffn_up")], self.norms[f"blk.{l}.ffn_norm.weight"])
            into(gu, dn, [hx(l, "ffn_down")], None)
            # (not into the LM head: prefill steps and graph warm-ups run the layers without it, and a
            # forwarded sum must always be consumed by the launch it was made for)
            if l + 1 < self.n_layers:
                into(dn, self.layer_jobs[l + 1][0], [hx(l + 1, n) for n in ("attn_q", "attn_k", "attn_v")],
                     self.norms[f"blk.{l + 1}.attn_norm.weight"])

    @staticmethod
    def _ranges(mats) -> list[tuple[int, int]]:
        """(address, bytes) of the packed blobs of ``mats`` that a launch streams: codes, scales,
        kink columns and deltas, U and Vt (16-byte aligned starts; lengths cut to multiples of 16)."""
        out = []
        for h in mats:
            for t in (h.codes, h.scales, h.kink_cols, h.kink_deltas, h.U, h.Vt):
                if t is None or t.numel() == 0:
                    continue
                p, n = t.data_ptr(), t.numel() * t.element_size()
                n -= n % 16
                if p % 16 == 0 and n > 0:
                    out.append((p, n))
        return out

    @staticmethod
    def _set_prefetch(job, ranges):
        ranges = ranges[:L.MAX_PREFETCH]
        job.prefetch.n = len(ranges)
        for i, (p, n) in enumerate(ranges):
            job.prefetch.ptr[i] = p
            job.prefetch.bytes[i] = n

    # links of the L2 prefetch policy (bits of GSDLQ_PREFETCH / the prefetch argument)
    PF_QKV_O, PF_ATTN_GU, PF_O_GU, PF_GU_DOWN, PF_DOWN_NEXT, PF_HEAD_QKV = 1, 2, 4, 8, 16, 32

    def _wire_prefetch(self, policy: int):
        """L2 prefetch of later launches' weights (gsdlq_prefetch_t): a launch fetches into L2 the
        packed weights that a later launch will stream, so that HBM keeps working while the dependent
        launches wait for one another.  ``policy`` is a bit set of links: QKV -> O (1), attention ->
        gate/up (2), O -> gate/up (4), gate/up -> down (8), down -> the next layer's QKV or the head
        (16), head -> the first QKV of the next step (32); 0 = none."""
        jobs = [j for lj in self.layer_jobs for j in lj] + [self.head_job]
        for j in jobs:
            j.prefetch.n = 0
        if policy == 0:
            return
        hx = lambda l, n: self.hex[f"blk.{l}.{n}.weight"]  # noqa: E731
        qkv_w = lambda l: [hx(l, n) for n in ("attn_q", "attn_k", "attn_v")]  # noqa: E731
        for l, (qkv, att, o, gu, dn) in enumerate(self.layer_jobs):
            if policy & self.PF_QKV_O:
                self._set_prefetch(qkv, self._ranges([hx(l, "attn_output")]))
            if policy & self.PF_ATTN_GU:
                self._set_prefetch(att, self._ranges([hx(l, "ffn_gate"), hx(l, "ffn_up")]))
            if policy & self.PF_O_GU:
                self._set_prefetch(o, self._ranges([hx(l, "ffn_gate"), hx(l, "ffn_up")]))
            if policy & self.PF_GU_DOWN:
                self._set_prefetch(gu, self._ranges([hx(l, "ffn_down")]))
            if policy & self.PF_DOWN_NEXT:
                nxt = qkv_w(l + 1) if l + 1 < self.n_layers else [self.hex["output.weight"]]
                self._set_prefetch(dn, self._ranges(nxt))
        if policy & self.PF_HEAD_QKV:
            self._set_prefetch(self.head_job, self._ranges(qkv_w(0)))

    def _wire_exchange(self):
        """Tensor parallelism with the fused exchange: the O and down launches of every rank sum the
        ranks' partial outputs in their epilogue (gsdlq_linear_job_t.exchange), so the step has no
        separate all-reduce launches."""
        if not self.tp.fused_epilogue:
            return
        for (qkv, att, o, gu, dn) in self.layer_jobs:
            for j in (o, dn):
                j.epilogue = L.EPI_RESID
                j.resid = self.x.data_ptr()
                j.exchange = self.tp.comm
        # every rank holds the summed residual in the O and down epilogues, so low-rank forwarding works
        # as on one GPU: row-parallel consumers (O, down) receive their rank's partial projection, whose
        # U S term the exchange sums with the rest of the partial output
        if self.lr_forward:
            self._wire_forwarding()

    def linear(self, job):
        ops.linear(job, self.ws_of[id(job)])

    def _build_plans(self):
        """The whole step as one persistent launch (gsdlq_decode_step), with and without the head.

        Shapes the decode kernel is not built for keep the per-operation launches."""
        lib = L.load()
        layers = (L.DecodeLayer * self.n_layers)()
        for i, (qkv, att, o, gu, dn) in enumerate(self.layer_jobs):
            layers[i] = L.DecodeLayer(qkv=qkv, attn=att, o=o, gate_up=gu, down=dn)
        st = self.state.data_ptr()
        for name, head in (("full", self.head_job), ("layers", L.LinearJob())):
            d = L.DecodeDesc(n_layers=self.n_layers, layers=layers, head=head,
                             argmax_key=self.key.data_ptr(), token=st, pos=st + 4, step=st + 8,
                             out_ids=self.out_ids.data_ptr(), max_out=self.out_ids.numel())
            plan = ctypes.c_void_p()
            status = lib.gsdlq_decode_plan_create(ctypes.byref(d), ctypes.byref(plan))
            if status == -3:  # GSDLQ_ERR_UNSUPPORTED: keep the per-operation launches
                self._destroy_plans()
                return
            L.check(status, "gsdlq_decode_plan_create")
            self._plans[name] = plan

    def _destroy_plans(self):
        lib = L.load()
        for plan in self._plans.values():
            lib.gsdlq_decode_plan_destroy(plan)
        self._plans = {}

    @property
    def fused_step(self) -> bool:
        """True when each step runs as one persistent launch (gsdlq_decode_step)."""
        return bool(self._plans)

    # ------------------------------------------------------------------ step
    def _run_layers(self):
        allreduce = self.tp.allreduce if (self.tp is not None and not self.tp.fused_epilogue) else None
        for qkv, att, o, gu, dn in self.layer_jobs:
            self.linear(qkv)
            ops.attention(att)
            self.linear(o)
            if allreduce:
                allreduce(self, "o")
            self.linear(gu)
            self.linear(dn)
            if allreduce:
                allreduce(self, "down")

    def _run_head(self, advance: bool = True):
        self.linear(self.head_job)
        if self.tp is not None:
            self.tp.finish_head(self)
        if advance:
            lib = L.load()
            st = self.state.data_ptr()
            L.check(lib.gsdlq_greedy_advance(self.key.data_ptr(), st, st + 4, st + 8, self.out_ids.data_ptr(),
                                             self.out_ids.numel(), ops.stream_handle()), "greedy_advance")

    def _graph(self, name, fn):
        g = self._graphs.get(name)
        if g is None:
            # eager warm-up (sets kernel attributes and NCCL state outside capture); the step's
            # device-side bookkeeping (token, pos, greedy key) is restored so that the warm-up
            # leaves no trace and the replay that follows does the real work
            smp = getattr(self, "_smp", None)
            saved = (self.state.clone(), self.key.clone(), self.out_ids.clone(),
                     smp["done"].clone() if smp is not None else None)
            fn()
            torch.cuda.synchronize(self.device)
            self.state.copy_(saved[0])
            self.key.copy_(saved[1])
            self.out_ids.copy_(saved[2])
            if smp is not None:
                smp["done"].copy_(saved[3])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            self._graphs[name] = g
        return g

    def step(self, with_head: bool = True):
        """One decode step on the device (token/pos taken from self.state)."""
        if self._plans:
            plan = self._plans["full" if with_head else "layers"]
            L.check(L.load().gsdlq_decode_step(plan, ops.stream_handle()), "gsdlq_decode_step")
            return
        if self.use_graph:
            self._graph("layers", self._run_layers).replay()
            if with_head:
                self._graph("head", self._run_head).replay()
        else:
            self._run_layers()
            if with_head:
                self._run_head()

    def synchronize(self):
        """Wait for the model's device work (timing, or before reading results another way)."""
        torch.cuda.synchronize(self.device)

    def set_state(self, token_id: int, pos: int):
        if not 0 <= pos < self.max_seq:
            raise ValueError(f"pos {pos} outside [0, {self.max_seq})")
        if not 0 <= token_id < self.vocab_size:
            raise ValueError(f"token id {token_id} outside [0, {self.vocab_size})")
        self.state[0:3].copy_(torch.tensor([token_id, pos, 0], dtype=torch.int32))

    # ------------------------------------------------------------------ reference surface
    def forward_token(self, token_id: int, pos: int, return_logits: bool = True):
        self.set_state(int(token_id), int(pos))
        self.step(with_head=return_logits)
        if not return_logits:
            return None
        return self.logits_host()

    def logits_host(self) -> np.ndarray:
        if self.tp is not None:
            return self.tp.gather_logits(self)
        return self.logits.cpu().numpy()

    def sample_token(self, logits, temperature: float = 0.0, top_p: float = 0.9) -> int:
        """Greedy when temperature <= 0, else temperature + top-p sampling (gsd_lq_cpu_runtime.py:422-443)."""
        logits = np.nan_to_num(np.asarray(logits, np.float32), nan=-1e4, posinf=100.0, neginf=-1e4)
        if temperature <= 0.0:
            return int(np.argmax(logits))
        z = logits / max(temperature, 1e-4)
        z -= np.max(z)
        p = np.exp(z)
        s = p.sum()
        if s <= 0 or np.isnan(s):
            return int(np.argmax(logits))
        p /= s
        idx = np.argsort(p)[::-1]
        cp = np.cumsum(p[idx])
        cut = int(np.argmax(cp > top_p)) + 1
        top, pt = idx[:cut], p[idx[:cut]]
        ps = pt.sum()
        if ps <= 0 or np.isnan(ps):  # the reference's p_sum guard (gsd_lq_cpu_runtime.py:439-441)
            return int(top[0])
        pt = pt / ps
        return int(np.random.choice(top, p=pt))

    def sample_device(self, temperature: float = 0.0, top_p: float = 0.9, u: float | None = None) -> int:
        """sample_token on the device over the last step's logits (gsdlq_sample_top_p).  u: the uniform
        draw np.random.choice would make; by default np.random.random_sample(), taken only when
        temperature > 0 (the reference draws only then), so that picks follow the reference's under the
        same NumPy seed."""
        if self.tp is not None:
            raise NotImplementedError("device sampling needs the whole vocabulary on one GPU; under tensor "
                                      "parallelism use sample_token(logits_host())")
        if u is None:
            u = float(np.random.random_sample()) if temperature > 0.0 else 0.0
        sb = self._sample_bufs()
        sb["u"][0] = u
        L.check(L.load().gsdlq_sample_top_p(self.logits.data_ptr(), self.vocab_local, float(temperature), float(top_p),
                                            sb["u"].data_ptr(), None, sb["work"].data_ptr(), sb["work"].numel(),
                                            None, sb["index"].data_ptr(), ops.stream_handle()), "gsdlq_sample_top_p")
        return int(sb["index"].item())

    def _sample_bufs(self):
        b = getattr(self, "_smp", None)
        if b is None:
            n = ctypes.c_size_t()
            L.check(L.load().gsdlq_sample_work_size(self.vocab_local, ctypes.byref(n)), "gsdlq_sample_work_size")
            b = {"work": torch.zeros(int(n.value), dtype=torch.uint8, device=self.device),
                 "u": torch.zeros(self.max_seq, dtype=torch.float64, device=self.device),
                 "index": torch.zeros(1, dtype=torch.int32, device=self.device),
                 "done": torch.zeros(1, dtype=torch.int32, device=self.device)}
            self._smp = b
        return b

    PREFILL_CHUNK = 128  # tokens per chunk of batched prefill (the dequant-GEMM's largest batch)

    @property
    def batched_prefill_supported(self) -> bool:
        """The chunk kernels' shape limits: head_dim 64 or 128 (gsdlq_attention_rows), at most 8 query heads
        per kv head."""
        return self.head_dim in (64, 128) and self.n_heads_local // self.n_kv_local <= 8

    def prefill(self, ids, start_pos: int = 0, batched: bool | None = None):
        """Fill the KV cache for ``ids`` at positions start_pos.. (no logits).

        Batched (default on one GPU): chunks of up to 128 tokens, every packed linear as one tensor-core
        dequant-GEMM over the chunk, causal attention over the chunk's rows.  Token by token (as the
        reference does, run_gpu_native_chat.py:1128-1131) with batched=False, under tensor parallelism,
        for shapes outside batched_prefill_supported, or with GSDLQ_PREFILL=token."""
        ids = [int(t) for t in ids]
        if batched is None:
            batched = (self.tp is None and os.environ.get("GSDLQ_PREFILL", "batched") != "token"
                       and self.batched_prefill_supported)
        if not batched:
            for i, t in enumerate(ids):
                self.set_state(t, start_pos + i)
                self.step(with_head=False)
            return
        if start_pos + len(ids) > self.max_seq:
            raise ValueError("prefill past max_seq")
        for c in range(0, len(ids), self.PREFILL_CHUNK):
            self._prefill_chunk(ids[c:c + self.PREFILL_CHUNK], start_pos + c)

    def _prefill_bufs(self):
        b = getattr(self, "_pf", None)
        if b is None:
            T, dev = self.PREFILL_CHUNK, self.device
            f32 = dict(dtype=torch.float32, device=dev)
            qd, kvd = self.n_heads_local * self.head_dim, self.n_kv_local * self.head_dim
            b = {"x": torch.zeros((T, self.hidden), **f32), "xn": torch.zeros((T, self.hidden), **f32),
                 "q": torch.zeros((T, qd), **f32), "k": torch.zeros((T, kvd), **f32), "v": torch.zeros((T, kvd), **f32),
                 "att": torch.zeros((T, qd), **f32), "o": torch.zeros((T, self.hidden), **f32),
                 "g": torch.zeros((T, self.ffn_local), **f32), "u": torch.zeros((T, self.ffn_local), **f32),
                 "work": ops.matmul_work(T, max(h.cols for h in self.hex.values()), dev),
                 "awork": ops.attention_rows_work(T, self.n_heads_local, self.head_dim, dev),
                 "ids": torch.zeros(T, dtype=torch.int32, device=dev),
                 "xy": {r: torch.from_numpy(ops.codebook(r)).to(dev) for r in (6, 8)}}
            self._pf = b
        return b

    def _prefill_chunk(self, ids, pos0: int, k_cache=None, v_cache=None, max_seq: int | None = None):
        """One chunk of batched prefill into (k_cache, v_cache) ([layers][max_seq][kv heads][head_dim]
        fp16; the model's own cache by default)."""
        lib, sh = L.load(), ops.stream_handle()
        b = self._prefill_bufs()
        kc = self.k_cache if k_cache is None else k_cache
        vc = self.v_cache if v_cache is None else v_cache
        S = self.max_seq if max_seq is None else max_seq
        n, H, F = len(ids), self.hidden, self.ffn_local
        b["ids"][:n].copy_(torch.tensor(ids, dtype=torch.int32))

        def mm(xin, name, yout):
            ops.hex2d_matmul(xin[:n], self.hex[name], b["xy"][self.hex[name].radius], yout, b["work"])
        x, xn = b["x"], b["xn"]
        L.check(lib.gsdlq_embed_rows(self.embed.data_ptr(), b["ids"].data_ptr(), n, self.vocab_size, H,
                                     x.data_ptr(), sh), "gsdlq_embed_rows")
        sm = 1.0 / math.sqrt(self.head_dim)
        for l in range(self.n_layers):
            p = f"blk.{l}."
            L.check(lib.gsdlq_rmsnorm_rows(x.data_ptr(), self.norms[p + "attn_norm.weight"].data_ptr(), xn.data_ptr(),
                                           n, H, self.rms_eps, sh), "gsdlq_rmsnorm_rows")
            mm(xn, p + "attn_q.weight", b["q"])
            mm(xn, p + "attn_k.weight", b["k"])
            mm(xn, p + "attn_v.weight", b["v"])
            L.check(lib.gsdlq_rope_kv_rows(b["q"].data_ptr(), b["k"].data_ptr(), b["v"].data_ptr(), kc.data_ptr(),
                                           vc.data_ptr(), self.rope_cs.data_ptr(), l, pos0, n, self.n_heads_local,
                                           self.n_kv_local, self.head_dim, S, sh), "gsdlq_rope_kv_rows")
            L.check(lib.gsdlq_attention_rows(b["q"].data_ptr(), kc.data_ptr(), vc.data_ptr(), b["att"].data_ptr(),
                                             b["awork"].data_ptr(), b["awork"].numel(), l, pos0, n,
                                             self.n_heads_local, self.n_kv_local, self.head_dim, S, sm, sh),
                    "gsdlq_attention_rows")
            mm(b["att"], p + "attn_output.weight", b["o"])
            L.check(lib.gsdlq_vec_add(x.data_ptr(), x.data_ptr(), b["o"].data_ptr(), n * H, sh), "gsdlq_vec_add")
            L.check(lib.gsdlq_rmsnorm_rows(x.data_ptr(), self.norms[p + "ffn_norm.weight"].data_ptr(), xn.data_ptr(),
                                           n, H, self.rms_eps, sh), "gsdlq_rmsnorm_rows")
            mm(xn, p + "ffn_gate.weight", b["g"])
            mm(xn, p + "ffn_up.weight", b["u"])
            L.check(lib.gsdlq_swiglu(b["g"].data_ptr(), b["u"].data_ptr(), b["g"].data_ptr(), n * F, sh),
                    "gsdlq_swiglu")
            mm(b["g"], p + "ffn_down.weight", b["o"])
            L.check(lib.gsdlq_vec_add(x.data_ptr(), x.data_ptr(), b["o"].data_ptr(), n * H, sh), "gsdlq_vec_add")

    def generate(self, prompt_ids, max_new_tokens: int, temperature: float = 0.0, top_p: float = 0.9,
                 eos_id: int | None = None, check_every: int = 16, start_pos: int = 0,
                 on_tokens=None) -> list[int]:
        """Generation with the loop on the device: one graph replay per token (layers, LM head, then the
        pick and the bookkeeping), no host round trip per token.

        temperature <= 0: greedy (the reference's smoke loop, run_gpu_native_chat.py:1039-1055); else
        temperature + top-p picks on the device with the reference's rules (sample_token,
        gsd_lq_cpu_runtime.py:422-443), one np.random.random_sample() draw per token taken up front,
        which is the sequence the reference's np.random.choice calls would consume.  eos_id: stop when
        the pick is eos_id, without returning it (the reference chat loop, run_gpu_native_chat.py:
        1142-1144); the host looks at the device's done flag every check_every tokens and the steps
        after the stop do no more bookkeeping.

        start_pos: the KV cache already holds prompt_ids[:start_pos] at positions 0 .. start_pos - 1 (a
        previous turn's tokens, as the reference's chat loop reuses them, run_gpu_native_chat.py:1112-1114),
        so only the rest of the prompt is prefilled.  on_tokens(ids): called with the ids produced since
        its last call, every check_every tokens and once at the end (streaming); each call reads the
        device's step counter, one host synchronisation per check_every tokens."""
        ids = list(prompt_ids)
        if not ids:
            raise ValueError("the prompt needs at least one token")
        if max_new_tokens < 0 or len(ids) + max_new_tokens > self.max_seq:
            raise ValueError("prompt + new tokens exceed max_seq")
        if check_every < 1:
            raise ValueError("check_every must be at least 1")
        if not 0 <= start_pos < len(ids):
            raise ValueError("start_pos must lie inside the prompt (its last token is always run)")
        sampled = temperature > 0.0
        if sampled and self.tp is not None:
            raise NotImplementedError("device sampling needs the whole vocabulary on one GPU")
        self.prefill(ids[start_pos:-1], start_pos=start_pos)
        self.set_state(ids[-1], len(ids) - 1)
        checks = eos_id is not None or on_tokens is not None
        if not sampled and not checks:
            for _ in range(max_new_tokens):
                self.step(with_head=True)   # the head's advance kernel feeds the next replay
            return self.out_ids[:max_new_tokens].cpu().tolist()
        sb = self._sample_bufs()
        if sampled:
            sb["u"][:max_new_tokens].copy_(torch.from_numpy(np.random.random_sample(max_new_tokens)))
        sb["done"].zero_()
        eos = -1 if eos_id is None else int(eos_id)
        name = f"head_gen_{float(temperature)!r}_{float(top_p)!r}_{eos}"
        # the sampling settings are baked into the captured head: keep only the latest such graph
        for old in [k for k in self._graphs if k.startswith("head_gen_") and k != name]:
            del self._graphs[old]

        def run_head_gen():
            lib, st = L.load(), self.state.data_ptr()
            self.linear(self.head_job)
            if sampled:
                L.check(lib.gsdlq_sample_top_p(self.logits.data_ptr(), self.vocab_local, float(temperature),
                                               float(top_p), sb["u"].data_ptr(), st + 8, sb["work"].data_ptr(),
                                               sb["work"].numel(), self.key.data_ptr(), None, ops.stream_handle()),
                        "gsdlq_sample_top_p")
            L.check(lib.gsdlq_advance_eos(self.key.data_ptr(), st, st + 4, st + 8, self.out_ids.data_ptr(),
                                          self.out_ids.numel(), eos, sb["done"].data_ptr(), ops.stream_handle()),
                    "gsdlq_advance_eos")

        emitted = 0
        for i in range(max_new_tokens):
            if self._plans:
                L.check(L.load().gsdlq_decode_step(self._plans["layers"], ops.stream_handle()), "gsdlq_decode_step")
            elif self.use_graph:
                self._graph("layers", self._run_layers).replay()
            else:
                self._run_layers()
            if self.use_graph:
                self._graph(name, run_head_gen).replay()
            else:
                run_head_gen()
            if checks and (i + 1) % check_every == 0:
                if on_tokens is not None:
                    n = int(self.state[2].item())
                    if n > emitted:
                        on_tokens(self.out_ids[emitted:n].cpu().tolist())
                        emitted = n
                if eos_id is not None and int(sb["done"].item()):
                    break
        n = int(self.state[2].item())
        out = self.out_ids[:n].cpu().tolist()
        if on_tokens is not None and n > emitted:
            on_tokens(out[emitted:])
        return out

    def release(self):
        self._graphs.clear()
        self._destroy_plans()
        if self.tp is not None:
            torch.cuda.synchronize(self.device)
            self.tp.close()
        for k in ("hex", "embed", "norms", "k_cache", "v_cache", "_arena"):
            if hasattr(self, k):
                delattr(self, k)
        torch.cuda.empty_cache()

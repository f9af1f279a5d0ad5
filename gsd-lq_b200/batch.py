"""Batched decode: B independent sequences advanced one token each per step.

The reference decodes one sequence at a time (Model.forward_token, run_gpu_native_chat.py:921-984);
this keeps its per-token operations and runs them for B sequences at once, each with its own KV cache
and position:

  embed_rows -> per layer: rmsnorm_rows, q / k / v linears, rope_kv_batch (RoPE + fp16 K/V append at each
  sequence's position), attention_decode_batch, O linear + residual, rmsnorm_rows, gate / up linears,
  SwiGLU, down linear + residual -> rmsnorm_rows, LM head linear, argmax_rows (greedy pick, position + 1)

Every packed linear is one call of the tensor-core dequant-GEMM (gsdlq_hex2d_matmul) over the B rows, so
the weights are decoded once per step for all sequences; without a low-rank term (Turbo) q/k/v and gate/up
run as one GEMM each over their stacked rows.  The step is captured as one CUDA graph and
replayed; tokens and positions stay on the device between steps.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib as L
from . import ops


def _stack_rows(hs):
    """One packed matrix whose rows are those of ``hs`` in order (same columns, radius, no low-rank term):
    codes, scales and kinks concatenate, the kink row pointers are offset."""
    import torch
    from .ops import DeviceHex
    rps, off = [], 0
    for i, h in enumerate(hs):
        rp = h.row_ptr.view(torch.int32).long()
        rps.append((rp if i == 0 else rp[1:]) + off)
        off += int(rp[-1].item())
    kc = [h.kink_cols for h in hs if h.kink_cols is not None and h.nnz]
    kd = [h.kink_deltas for h in hs if h.kink_deltas is not None and h.nnz]
    return DeviceHex(None, rows=sum(h.rows for h in hs), cols=hs[0].cols, k_dim=0, radius=hs[0].radius,
                     codes=torch.cat([h.codes for h in hs]), scales=torch.cat([h.scales for h in hs]),
                     row_ptr=torch.cat(rps).to(torch.int32), kink_cols=torch.cat(kc) if kc else None,
                     kink_deltas=torch.cat(kd) if kd else None, U=None, S=None, Vt=None, nnz=off)


class BatchDecoder:
    """Greedy lockstep decode of ``batch`` sequences over a loaded GSDLQModel's weights (one GPU)."""

    def __init__(self, model, batch: int, max_seq: int | None = None, use_graph: bool = True):
        if model.tp is not None:
            raise NotImplementedError("batched decode runs on one GPU")
        if not 1 <= batch <= ops.MATMUL_MAX_BATCH:
            raise ValueError(f"batch must be in [1, {ops.MATMUL_MAX_BATCH}]")
        if not model.batched_prefill_supported:
            raise NotImplementedError("batched decode needs head_dim 64 or 128")
        m = self.m = model
        self.B = B = batch
        self.S = S = model.max_seq if max_seq is None else int(max_seq)
        if S > model.max_seq:
            raise ValueError("max_seq above the model's (its RoPE table)")
        self.use_graph = use_graph
        dev = m.device
        f32 = dict(dtype=torch.float32, device=dev)
        Lc, kv, hd = m.n_layers, m.n_kv_local, m.head_dim
        self.k_cache = torch.zeros((B, Lc, S, kv, hd), dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.seq_stride = Lc * S * kv * hd
        H, F, qd = m.hidden, m.ffn_local, m.n_heads_local * hd
        self.x, self.xn = torch.zeros((B, H), **f32), torch.zeros((B, H), **f32)
        self.q, self.att = torch.zeros((B, qd), **f32), torch.zeros((B, qd), **f32)
        self.k, self.v = torch.zeros((B, kv * hd), **f32), torch.zeros((B, kv * hd), **f32)
        self.o = torch.zeros((B, H), **f32)
        self.g, self.u = torch.zeros((B, F), **f32), torch.zeros((B, F), **f32)
        self.logits = torch.zeros((B, m.vocab_local), **f32)
        self.work = ops.matmul_work(B, max(h.cols for h in m.hex.values()), dev)
        self.awork = ops.attention_rows_work(B, m.n_heads_local, hd, dev)
        self.xy = {r: torch.from_numpy(ops.codebook(r)).to(dev) for r in (6, 8)}
        self.ids = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.out_ids = torch.zeros((B, S), dtype=torch.int32, device=dev)
        # Linears that read the same input and have no low-rank term (Turbo) run as one GEMM over their
        # stacked rows: q/k/v, and gate/up.  With a low-rank term each matrix has its own Vt, so they stay apart.
        self.fused = {}
        for l in range(Lc):
            p = f"blk.{l}."
            for key, names in (("qkv", ("attn_q", "attn_k", "attn_v")), ("gu", ("ffn_gate", "ffn_up"))):
                hs = [m.hex[p + n + ".weight"] for n in names]
                if all(h.k_dim == 0 and h.radius == hs[0].radius and h.cols == hs[0].cols for h in hs):
                    self.fused[p + key] = _stack_rows(hs)
        if self.fused:
            self.qkv = torch.zeros((B, qd + 2 * kv * hd), **f32)
            self.gu = torch.zeros((B, 2 * F), **f32)
        self._graph = None

    # ------------------------------------------------------------------ state
    def prefill(self, b: int, ids, start_pos: int = 0):
        """Fill sequence b's cache with ``ids`` at positions start_pos.. (chunked tensor-core prefill)."""
        ids = [int(t) for t in ids]
        if start_pos + len(ids) > self.S:
            raise ValueError("prefill past max_seq")
        for c in range(0, len(ids), self.m.PREFILL_CHUNK):
            self.m._prefill_chunk(ids[c:c + self.m.PREFILL_CHUNK], start_pos + c, self.k_cache[b], self.v_cache[b],
                                  self.S)

    def set_tokens(self, ids, positions):
        """The next input token and its position, per sequence."""
        ids, positions = np.asarray(ids, np.int32), np.asarray(positions, np.int32)
        if ids.shape != (self.B,) or positions.shape != (self.B,):
            raise ValueError("one token and one position per sequence")
        if (positions < 0).any() or (positions >= self.S).any():
            raise ValueError(f"positions outside [0, {self.S})")
        if (ids < 0).any() or (ids >= self.m.vocab_size).any():
            raise ValueError("token id outside the vocabulary")
        self.ids.copy_(torch.from_numpy(ids))
        self.pos.copy_(torch.from_numpy(positions))

    # ------------------------------------------------------------------ the step
    def _mm(self, xin, name, yout):
        h = self.fused[name] if name in self.fused else self.m.hex[name]
        ops.hex2d_matmul(xin, h, self.xy[h.radius], yout, self.work)

    def _run(self, with_pick: bool = True):
        m, lib, sh = self.m, L.load(), ops.stream_handle()
        B, H, F = self.B, m.hidden, m.ffn_local
        x, xn = self.x, self.xn
        L.check(lib.gsdlq_embed_rows(m.embed.data_ptr(), self.ids.data_ptr(), B, m.vocab_size, H, x.data_ptr(), sh),
                "gsdlq_embed_rows")
        sm = 1.0 / math.sqrt(m.head_dim)
        for l in range(m.n_layers):
            p = f"blk.{l}."
            L.check(lib.gsdlq_rmsnorm_rows(x.data_ptr(), m.norms[p + "attn_norm.weight"].data_ptr(), xn.data_ptr(), B,
                                           H, m.rms_eps, sh), "gsdlq_rmsnorm_rows")
            if p + "qkv" in self.fused:  # one GEMM; q, k, v are column ranges of its rows
                self._mm(xn, p + "qkv", self.qkv)
                qd, kvd, stride = m.n_heads_local * m.head_dim, m.n_kv_local * m.head_dim, self.qkv.shape[1]
                qp = self.qkv.data_ptr()
                kp, vp = qp + 4 * qd, qp + 4 * (qd + kvd)
            else:
                self._mm(xn, p + "attn_q.weight", self.q)
                self._mm(xn, p + "attn_k.weight", self.k)
                self._mm(xn, p + "attn_v.weight", self.v)
                qp, kp, vp, stride = self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), 0
            L.check(lib.gsdlq_rope_kv_batch(qp, kp, vp, stride, self.k_cache.data_ptr(), self.v_cache.data_ptr(),
                                            self.seq_stride, m.rope_cs.data_ptr(), l, self.pos.data_ptr(), B,
                                            m.n_heads_local, m.n_kv_local, m.head_dim, self.S, sh),
                    "gsdlq_rope_kv_batch")
            L.check(lib.gsdlq_attention_decode_batch(qp, stride, self.k_cache.data_ptr(),
                                                     self.v_cache.data_ptr(), self.seq_stride, self.att.data_ptr(),
                                                     self.awork.data_ptr(), self.awork.numel(), l,
                                                     self.pos.data_ptr(), B, m.n_heads_local, m.n_kv_local,
                                                     m.head_dim, self.S, sm, sh), "gsdlq_attention_decode_batch")
            self._mm(self.att, p + "attn_output.weight", self.o)
            L.check(lib.gsdlq_vec_add(x.data_ptr(), x.data_ptr(), self.o.data_ptr(), B * H, sh), "gsdlq_vec_add")
            L.check(lib.gsdlq_rmsnorm_rows(x.data_ptr(), m.norms[p + "ffn_norm.weight"].data_ptr(), xn.data_ptr(), B,
                                           H, m.rms_eps, sh), "gsdlq_rmsnorm_rows")
            if p + "gu" in self.fused:  # one GEMM over the stacked gate and up rows, then SwiGLU per row
                self._mm(xn, p + "gu", self.gu)
                L.check(lib.gsdlq_swiglu_rows(self.gu.data_ptr(), self.g.data_ptr(), B, F, sh), "gsdlq_swiglu_rows")
            else:
                self._mm(xn, p + "ffn_gate.weight", self.g)
                self._mm(xn, p + "ffn_up.weight", self.u)
                L.check(lib.gsdlq_swiglu(self.g.data_ptr(), self.u.data_ptr(), self.g.data_ptr(), B * F, sh),
                        "gsdlq_swiglu")
            self._mm(self.g, p + "ffn_down.weight", self.o)
            L.check(lib.gsdlq_vec_add(x.data_ptr(), x.data_ptr(), self.o.data_ptr(), B * H, sh), "gsdlq_vec_add")
        L.check(lib.gsdlq_rmsnorm_rows(x.data_ptr(), m.norms["output_norm.weight"].data_ptr(), xn.data_ptr(), B, H,
                                       m.rms_eps, sh), "gsdlq_rmsnorm_rows")
        self._mm(xn, "output.weight", self.logits)
        if with_pick:
            L.check(lib.gsdlq_argmax_rows(self.logits.data_ptr(), B, m.vocab_local, self.ids.data_ptr(),
                                          self.pos.data_ptr(), self.out_ids.data_ptr(), self.S, sh),
                    "gsdlq_argmax_rows")

    def step(self):
        """One token for every sequence: logits into self.logits, greedy picks into self.ids (the next
        inputs), out_ids[b][pos + 1] = pick, positions + 1."""
        if not self.use_graph:
            self._run()
            return
        if self._graph is None:
            # eager warm-up outside the capture (kernel attributes); tokens, positions and outputs are
            # restored, and the K/V rows it wrote are written again, with the same values, by the replay
            saved = (self.ids.clone(), self.pos.clone(), self.out_ids.clone())
            self._run()
            torch.cuda.synchronize(self.m.device)
            for t, v in zip((self.ids, self.pos, self.out_ids), saved):
                t.copy_(v)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._run()
            self._graph = g
        self._graph.replay()

    def logits_host(self) -> np.ndarray:
        """The last step's logits, [B][vocab]."""
        return self.logits.cpu().numpy()

    def generate(self, prompts, max_new_tokens: int) -> list[list[int]]:
        """Greedy continuation of every prompt (prefilled by chunks, then lockstep decode)."""
        if len(prompts) != self.B:
            raise ValueError(f"{self.B} prompts expected")
        for b, pr in enumerate(prompts):
            if len(pr) == 0:
                raise ValueError("every prompt needs at least one token")
            if len(pr) + max_new_tokens > self.S:
                raise ValueError("prompt + new tokens exceed max_seq")
            self.prefill(b, pr[:-1])
        self.set_tokens([pr[-1] for pr in prompts], [len(pr) - 1 for pr in prompts])
        for _ in range(max_new_tokens):
            self.step()
        out = self.out_ids.cpu().numpy()
        return [out[b, len(pr):len(pr) + max_new_tokens].tolist() for b, pr in enumerate(prompts)]

    def release(self):
        self._graph = None
        for k in ("k_cache", "v_cache", "work", "awork"):
            if hasattr(self, k):
                delattr(self, k)
        torch.cuda.empty_cache()

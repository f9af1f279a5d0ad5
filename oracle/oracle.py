"""CPU oracle for the GSD-LQ decode path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as a checker / baseline.  The
product package never imports it.

Contents
  * ``codebook``          -- NumPy restatement of _get_turbo_codebook
                             (gsd_lq_v2/gsd_lq_cpu_runtime.py:111-118).
  * ``dequant``           -- the dequantised-weight definition of the
                             reference's NumPy path (gsd_lq_cpu_runtime.py:281-284).
  * ``CEngine``           -- ctypes binding of a C engine with the reference's
                             seven entry points.  ``CEngine.restatement()`` loads
                             our C restatement (oracle/gsdlq_oracle.c);
                             ``CEngine.reference()`` loads the reference's own
                             engine compiled from its source (oracle/_ref), with
                             the argument types the reference declares
                             (gsd_lq_cpu_runtime.py:91-108).
  * ``read_gsd2``         -- restatement of the reference's .gsd2 reader
                             (gsd_lq_cpu_runtime.py:128-217).
  * ``OracleModel``       -- the decoder step of CPUMistralV2Model.forward_token
                             (gsd_lq_cpu_runtime.py:302-420) driven through a
                             CEngine, plus the greedy pick (:422-425).
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "_build", "libgsdlq_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libgsd_cpu.so")
MAX_SEQ_LEN = 2048  # gsd_lq_cpu_runtime.py:22


def reference_dir() -> str | None:
    """Where the reference source tree is: $GSDLQ_REFERENCE, else the `reference_path` that the
    repository's BASELINE.json records; None when neither names an existing directory."""
    d = os.environ.get("GSDLQ_REFERENCE")
    if not d:
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                d = json.load(f).get("reference_path")
        except (OSError, ValueError):
            d = None
    return d if d and os.path.isdir(d) else None


def build(quiet: bool = True) -> None:
    """Build the restatement (and, where the reference tree exists, the reference) with make."""
    ref = reference_dir()
    cmd = ["make", "-C", HERE, "all"] + ([f"REF_DIR={ref}"] if ref else [])
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def codebook(radius: int) -> tuple[np.ndarray, int]:
    """A2 lattice table, gsd_lq_cpu_runtime.py:111-118 (float64 math, one cast to float32)."""
    h = float(np.sqrt(3.0) / 2.0)
    pts = [[r0 + 0.5 * r1, r1 * h]
           for r0 in range(-radius, radius + 1)
           for r1 in range(-radius, radius + 1)
           if abs(r0 + r1) <= radius]
    return np.array(pts, dtype=np.float32), len(pts)


def dequant(codes: np.ndarray, scales_u16: np.ndarray, xy: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """W = xy[codes].reshape(rows, cols) * repeat(f32(f16 scales), 64): gsd_lq_cpu_runtime.py:281-284."""
    s = scales_u16.view(np.float16).astype(np.float32)
    pts = xy[codes].reshape(rows, cols)
    return pts * np.repeat(s.reshape(rows, cols // 64), 64, axis=1)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class CEngine:
    """A C engine exposing the reference's seven functions (names resolved per library)."""

    NAMES = ("rmsnorm", "vec_add", "swiglu", "lowrank_proj", "hex2d_matvec",
             "rope_and_store_kv", "gqa_attention")

    def __init__(self, path: str, prefix: str, kind: str):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path, self.kind = path, kind
        self.lib = ctypes.CDLL(path)
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        # argument types as declared at gsd_lq_cpu_runtime.py:95-108
        sig = {
            "rmsnorm": [vp, vp, vp, i32, f32],
            "vec_add": [vp, vp, vp, i32],
            "swiglu": [vp, vp, vp, i32],
            "lowrank_proj": [vp, vp, vp, vp, i32, i32],
            "hex2d_matvec": [vp] * 10 + [i32] * 4,
            "rope_and_store_kv": [vp] * 5 + [i32] * 6 + [f32, i32],
            "gqa_attention": [vp] * 4 + [i32] * 6 + [f32],
        }
        for n in self.NAMES:
            fn = getattr(self.lib, prefix + n)
            fn.argtypes = sig[n]
            fn.restype = None
            setattr(self, n, fn)
        if kind == "restatement":
            self.lib.orc_codebook.argtypes = [i32, vp, i32]
            self.lib.orc_codebook.restype = i32
            self.lib.orc_dequant.argtypes = [vp, vp, vp, vp, i32, i32]
            self.lib.orc_argmax.argtypes = [vp, i32]
            self.lib.orc_argmax.restype = i32
            self.lib.orc_num_threads.restype = i32
            self.lib.orc_rope_cos_sin.argtypes = [i32, i32, i32, f32, vp, vp]

    @classmethod
    def restatement(cls) -> "CEngine":
        if not os.path.exists(ORACLE_LIB):
            build()
        return cls(ORACLE_LIB, "orc_", "restatement")

    @classmethod
    def reference(cls) -> "CEngine | None":
        """The reference's own engine built from its source, or None if it was never built here."""
        if not os.path.exists(REF_LIB):
            try:
                build()
            except RuntimeError:
                return None
        return cls(REF_LIB, "gsd_cpu_", "reference") if os.path.exists(REF_LIB) else None

    # -- convenience wrappers (NumPy in, NumPy out) -------------------------------------
    def matvec(self, x: np.ndarray, rec: dict, tmp_k: np.ndarray | None = None) -> np.ndarray:
        """The reference's _matvec_cpu (gsd_lq_cpu_runtime.py:251-277): low-rank first, then the fused matvec."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rec["rows"], np.float32)
        tk = np.zeros(16, np.float32) if tmp_k is None else tmp_k
        if rec["k_dim"] > 0:
            self.lowrank_proj(_p(x), _p(rec["Vt"]), _p(rec["S"]), _p(tk), rec["k_dim"], rec["cols"])
        self.hex2d_matvec(_p(x), _p(rec["codes"]), _p(rec["scales"]), _p(rec["xy_table"]), _p(rec["U"]),
                          _p(tk), _p(rec["row_ptr"]), _p(rec["kink_cols"]), _p(rec["kink_deltas"]), _p(y),
                          rec["rows"], rec["cols"], rec["k_dim"], rec["n_pts"])
        return y


def hex_record(meta: dict, blobs: dict, xy_tables: dict) -> dict:
    """A packed-linear record with the keys of load_hex_cpu (gsd_lq_cpu_runtime.py:173-199)."""
    r = meta["radius"]
    xy, n_pts = xy_tables[r]
    k = meta["k_dim"]
    rec = {
        "rows": meta["rows"], "cols": meta["cols"], "k_dim": k, "n_pts": n_pts, "xy_table": xy,
        "codes": np.frombuffer(blobs["codes"], np.uint8),
        "scales": np.frombuffer(blobs["scales"], np.uint16),
        "row_ptr": np.frombuffer(blobs["row_ptr"], np.uint32),
        "kink_cols": np.frombuffer(blobs["kink_cols"], np.uint16),
        "kink_deltas": np.frombuffer(blobs["kink_deltas"], np.float32),
    }
    if k > 0:
        rec["U"] = np.frombuffer(blobs["U"], np.uint16)
        rec["S"] = np.frombuffer(blobs["S"], np.float32)
        rec["Vt"] = np.frombuffer(blobs["Vt"], np.uint16)
    else:  # dummies, gsd_lq_cpu_runtime.py:170-171,183-184
        rec["U"] = rec["Vt"] = np.zeros(2, np.uint16)
        rec["S"] = np.zeros(1, np.float32)
    return rec


LINEARS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
KEYS = ("q", "k", "v", "o", "gate", "up", "down")


def read_gsd2(path: str) -> dict:
    """Restatement of the .gsd2 reader of CPUMistralV2Model.__init__ (gsd_lq_cpu_runtime.py:128-217).

    Returns {"cfg", "avg_bpw", "embed" (f32), "layers": [{attn_norm, ffn_norm, q..down}],
    "final_norm", "lm_head"}.
    """
    tables = {r: codebook(r) for r in (6, 8)}
    with open(path, "rb") as f:
        if f.read(4) != b"GSD2":
            raise ValueError("bad magic")
        hlen = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(hlen).decode("utf-8"))
        base = 12 + hlen
        tensors = header["tensors"]

        def blob(m):
            f.seek(base + m["offset"])
            return f.read(m["nbytes"])

        def hexrec(name):
            m = tensors[name]
            keys = ["codes", "scales", "row_ptr", "kink_cols", "kink_deltas"]
            if m["k_dim"] > 0:
                keys += ["U", "S", "Vt"]
            return hex_record(m, {k: blob(m[k]) for k in keys}, tables)

        em = tensors["token_embd.weight"]["data"]
        model = {
            "cfg": header["config"],
            "avg_bpw": header.get("avg_bpw", 3.79),
            "embed": np.frombuffer(blob(em), np.float16).astype(np.float32).reshape(em["shape"]),
            "layers": [],
        }
        for l in range(model["cfg"]["n_layers"]):
            p = f"blk.{l}."
            lyr = {
                "attn_norm": np.frombuffer(blob(tensors[p + "attn_norm.weight"]["data"]), np.float32),
                "ffn_norm": np.frombuffer(blob(tensors[p + "ffn_norm.weight"]["data"]), np.float32),
            }
            for name, key in zip(LINEARS, KEYS):
                lyr[key] = hexrec(p + name + ".weight")
            model["layers"].append(lyr)
        model["final_norm"] = np.frombuffer(blob(tensors["output_norm.weight"]["data"]), np.float32)
        model["lm_head"] = hexrec("output.weight")
    return model


def argmax(logits: np.ndarray) -> int:
    """Greedy pick, gsd_lq_cpu_runtime.py:422-425."""
    return int(np.argmax(np.nan_to_num(logits, nan=-1e4, posinf=100.0, neginf=-1e4)))


class OracleModel:
    """forward_token of CPUMistralV2Model (gsd_lq_cpu_runtime.py:302-420) over a CEngine.

    ``model`` is the dict of ``read_gsd2`` (or any dict with the same arrays).  The KV
    cache is the reference's contiguous fp16 cache [n_layers, max_seq, n_kv, head_dim].
    """

    def __init__(self, model: dict, engine: CEngine, max_seq: int = MAX_SEQ_LEN, rope_interleaved: int = 1):
        self.m, self.e = model, engine
        c = model["cfg"]
        self.cfg = c
        self.n_layers, self.hidden = c["n_layers"], c["hidden_size"]
        self.n_heads, self.n_kv, self.hd = c["n_heads"], c["n_kv_heads"], c["head_dim"]
        self.ffn, self.eps, self.theta = c["ffn_size"], float(c["rms_eps"]), float(c["rope_theta"])
        self.vocab = c["vocab_size"]
        self.max_seq = max_seq
        self.interleaved = rope_interleaved
        self.k_cache = np.zeros((self.n_layers, max_seq, self.n_kv, self.hd), np.uint16)
        self.v_cache = np.zeros_like(self.k_cache)
        q_dim = self.n_heads * self.hd
        self.x = np.zeros(self.hidden, np.float32)
        self.xb = np.zeros(max(self.hidden, q_dim), np.float32)
        self.q = np.zeros(q_dim, np.float32)
        self.k = np.zeros(self.n_kv * self.hd, np.float32)
        self.v = np.zeros(self.n_kv * self.hd, np.float32)
        self.att = np.zeros(q_dim, np.float32)
        self.gate = np.zeros(self.ffn, np.float32)
        self.up = np.zeros(self.ffn, np.float32)
        self.tmp_k = np.zeros(16, np.float32)
        self.logits = np.zeros(self.vocab, np.float32)

    def _mv(self, x, rec, out):
        e = self.e
        if rec["k_dim"] > 0:
            e.lowrank_proj(_p(x), _p(rec["Vt"]), _p(rec["S"]), _p(self.tmp_k), rec["k_dim"], rec["cols"])
        e.hex2d_matvec(_p(x), _p(rec["codes"]), _p(rec["scales"]), _p(rec["xy_table"]), _p(rec["U"]),
                       _p(self.tmp_k), _p(rec["row_ptr"]), _p(rec["kink_cols"]), _p(rec["kink_deltas"]),
                       _p(out), rec["rows"], rec["cols"], rec["k_dim"], rec["n_pts"])

    def layer(self, l: int, pos: int) -> None:
        """One decoder layer (gsd_lq_cpu_runtime.py:305-404)."""
        e, lyr, H = self.e, self.m["layers"][l], self.hidden
        xb = self.xb[:H]
        e.rmsnorm(_p(self.x), _p(lyr["attn_norm"]), _p(xb), H, self.eps)
        self._mv(xb, lyr["q"], self.q)
        self._mv(xb, lyr["k"], self.k)
        self._mv(xb, lyr["v"], self.v)
        e.rope_and_store_kv(_p(self.q), _p(self.k), _p(self.v), _p(self.k_cache), _p(self.v_cache),
                            l, pos, self.n_heads, self.n_kv, self.hd, self.max_seq, self.theta, self.interleaved)
        sm = 1.0 / float(np.sqrt(self.hd))
        e.gqa_attention(_p(self.q), _p(self.k_cache), _p(self.v_cache), _p(self.att), l, pos,
                        self.n_heads, self.n_kv, self.hd, self.max_seq, sm)
        self._mv(self.att, lyr["o"], xb)
        self.x += xb
        e.rmsnorm(_p(self.x), _p(lyr["ffn_norm"]), _p(xb), H, self.eps)
        self._mv(xb, lyr["gate"], self.gate)
        self._mv(xb, lyr["up"], self.up)
        e.swiglu(_p(self.gate), _p(self.up), _p(self.gate), self.ffn)
        self._mv(self.gate, lyr["down"], xb)
        self.x += xb

    def forward_token(self, token_id: int, pos: int, return_logits: bool = True):
        self.x[:] = self.m["embed"][token_id]
        for l in range(self.n_layers):
            self.layer(l, pos)
        if not return_logits:
            return None
        xb = self.xb[:self.hidden]
        self.e.rmsnorm(_p(self.x), _p(self.m["final_norm"]), _p(xb), self.hidden, self.eps)
        self._mv(xb, self.m["lm_head"], self.logits)
        return self.logits.copy()

    @staticmethod
    def sample_token(logits: np.ndarray) -> int:
        return argmax(logits)

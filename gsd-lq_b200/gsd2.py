""".gsd2 container: reader, writer and format validation.

Layout (the reference's readers: gsd_lq_v2/gsd_lq_cpu_runtime.py:128-217 and
gsd_lq_v2/run_gpu_native_chat.py:741-833):

    b"GSD2" | u64 little-endian header length | UTF-8 JSON header | blobs

Blob offsets in the header are relative to ``12 + header_length``.  The header
holds ``config`` (model shape, rms_eps, rope_theta, tokenizer tables),
``avg_bpw`` and ``tensors``:

  * dense tensors ``{"data": {"offset", "nbytes", "shape"}}``: ``token_embd.weight``
    (fp16 [vocab, hidden]) and the RMSNorm weights (fp32 [hidden]);
  * packed ("hex") linears ``{"radius", "k_dim", "rows", "cols", "codes", "scales",
    "U", "S", "Vt", "row_ptr", "kink_cols", "kink_deltas"}``, each blob a
    ``{"offset", "nbytes"}``.  codes u8[R*C/2], scales f16[R*C/64], U f16[R*k],
    S f32[k], Vt f16[k*C], row_ptr u32[R+1], kink_cols u16[nnz], kink_deltas f32[nnz].

The writer adds keys the reference ignores: ``format_version``, ``mode``,
``packer`` and a 256-byte ``alignment`` of every blob (so blobs can be copied
straight to device memory).  The reader checks every invariant the kernels rely
on and raises ``FormatError`` instead of letting a malformed file reach the GPU:
the reference checks nothing and treats violations as undefined behaviour.
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
from typing import Callable

import numpy as np

from . import codebook

MAGIC = b"GSD2"
ALIGN = 256
MAX_K = 16          # the reference's tmp_k buffer holds 16 values (gsd_lq_cpu_runtime.py:231)
LINEAR_NAMES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
CONFIG_KEYS = ("n_layers", "hidden_size", "n_heads", "n_kv_heads", "head_dim", "ffn_size",
               "rms_eps", "rope_theta", "vocab_size")


class FormatError(ValueError):
    """A .gsd2 file or packed tensor violates the format."""


@dataclasses.dataclass
class HexTensor:
    """One packed linear (rows = out-features, cols = in-features)."""
    rows: int
    cols: int
    radius: int
    k_dim: int
    codes: np.ndarray            # uint8  [rows*cols/2]
    scales: np.ndarray           # uint16 [rows*cols/64] (fp16 bits)
    row_ptr: np.ndarray          # uint32 [rows+1]
    kink_cols: np.ndarray        # uint16 [nnz]
    kink_deltas: np.ndarray      # float32 [nnz]
    U: np.ndarray | None = None  # uint16 [rows*k] (fp16 bits)
    S: np.ndarray | None = None  # float32 [k]
    Vt: np.ndarray | None = None  # uint16 [k*cols] (fp16 bits)

    @property
    def n_pts(self) -> int:
        return codebook.num_points(self.radius)

    @property
    def nnz(self) -> int:
        return int(self.kink_cols.size)

    def blobs(self) -> dict[str, np.ndarray]:
        b = {"codes": self.codes, "scales": self.scales, "row_ptr": self.row_ptr,
             "kink_cols": self.kink_cols, "kink_deltas": self.kink_deltas}
        if self.k_dim > 0:
            b.update(U=self.U, S=self.S, Vt=self.Vt)
        return b

    def nbytes(self) -> int:
        return int(sum(a.nbytes for a in self.blobs().values()))

    def validate(self, check_codes: bool = True, check_values: bool = False) -> None:
        r, c, k = self.rows, self.cols, self.k_dim
        if r <= 0 or c <= 0:
            raise FormatError(f"bad shape {r}x{c}")
        if c % 64:
            raise FormatError(f"cols={c} is not a multiple of 64 (scale groups would straddle rows)")
        if c > 65535:
            raise FormatError(f"cols={c} does not fit the u16 kink column index")
        if self.radius not in codebook.RADII:
            raise FormatError(f"radius {self.radius} not in {codebook.RADII}")
        if not 0 <= k <= MAX_K:
            raise FormatError(f"k_dim={k} outside [0, {MAX_K}]")
        want = {"codes": (np.uint8, r * c // 2), "scales": (np.uint16, r * c // 64),
                "row_ptr": (np.uint32, r + 1)}
        if k > 0:
            want.update(U=(np.uint16, r * k), S=(np.float32, k), Vt=(np.uint16, k * c))
        for name, (dt, n) in want.items():
            a = getattr(self, name)
            if a is None or a.dtype != dt or a.size != n:
                got = None if a is None else (a.dtype, a.size)
                raise FormatError(f"{name}: expected {np.dtype(dt)}[{n}], got {got}")
        rp = self.row_ptr
        if rp[0] != 0 or np.any(rp[1:] < rp[:-1]):
            raise FormatError("row_ptr must start at 0 and be non-decreasing")
        nnz = int(rp[-1])
        if self.kink_cols.dtype != np.uint16 or self.kink_cols.size != nnz:
            raise FormatError(f"kink_cols: expected uint16[{nnz}]")
        if self.kink_deltas.dtype != np.float32 or self.kink_deltas.size != nnz:
            raise FormatError(f"kink_deltas: expected float32[{nnz}]")
        if nnz and int(self.kink_cols.max()) >= c:
            raise FormatError("kink column index out of range")
        if check_codes and self.codes.size and int(self.codes.max()) >= self.n_pts:
            raise FormatError(f"code index >= n_pts={self.n_pts}")
        if check_values:
            # fp16 blobs are stored as u16 bit patterns: exponent all ones is inf or NaN
            for name in ("scales", "U", "Vt"):
                a = getattr(self, name)
                if a is not None and a.size and np.any((a & 0x7C00) == 0x7C00):
                    raise FormatError(f"{name}: non-finite fp16 values")
            for name in ("S", "kink_deltas"):
                a = getattr(self, name)
                if a is not None and a.size and not np.all(np.isfinite(a)):
                    raise FormatError(f"{name}: non-finite values")

    def row_slice(self, r0: int, r1: int) -> "HexTensor":
        """Rows [r0, r1) as a new packed tensor (column-parallel sharding)."""
        c, k = self.cols, self.k_dim
        rp = self.row_ptr
        a, b = int(rp[r0]), int(rp[r1])
        return HexTensor(
            rows=r1 - r0, cols=c, radius=self.radius, k_dim=k,
            codes=np.ascontiguousarray(self.codes[r0 * c // 2:r1 * c // 2]),
            scales=np.ascontiguousarray(self.scales[r0 * c // 64:r1 * c // 64]),
            row_ptr=(rp[r0:r1 + 1] - rp[r0]).astype(np.uint32),
            kink_cols=np.ascontiguousarray(self.kink_cols[a:b]),
            kink_deltas=np.ascontiguousarray(self.kink_deltas[a:b]),
            U=None if k == 0 else np.ascontiguousarray(self.U[r0 * k:r1 * k]),
            S=None if k == 0 else self.S.copy(),
            Vt=None if k == 0 else self.Vt.copy())

    def col_slice(self, c0: int, c1: int) -> "HexTensor":
        """Columns [c0, c1) as a new packed tensor (row-parallel sharding).

        c0 and c1 must be multiples of 64.  Codes/scales are cut per row, kinks
        are filtered to the range (and re-based), Vt is cut by columns and U/S are
        kept whole, so the shards' outputs sum to the full output."""
        if c0 % 64 or c1 % 64:
            raise FormatError("column shards must be multiples of 64")
        r, c, k = self.rows, self.cols, self.k_dim
        codes = self.codes.reshape(r, c // 2)[:, c0 // 2:c1 // 2]
        scales = self.scales.reshape(r, c // 64)[:, c0 // 64:c1 // 64]
        rows_of = np.repeat(np.arange(r), np.diff(self.row_ptr.astype(np.int64)))
        keep = (self.kink_cols >= c0) & (self.kink_cols < c1)
        counts = np.bincount(rows_of[keep], minlength=r)
        rp = np.zeros(r + 1, np.uint32)
        rp[1:] = np.cumsum(counts)
        return HexTensor(
            rows=r, cols=c1 - c0, radius=self.radius, k_dim=k,
            codes=np.ascontiguousarray(codes).reshape(-1),
            scales=np.ascontiguousarray(scales).reshape(-1),
            row_ptr=rp,
            kink_cols=(self.kink_cols[keep].astype(np.int64) - c0).astype(np.uint16),
            kink_deltas=np.ascontiguousarray(self.kink_deltas[keep]),
            U=None if k == 0 else self.U.copy(),
            S=None if k == 0 else self.S.copy(),
            Vt=None if k == 0 else np.ascontiguousarray(self.Vt.reshape(k, c)[:, c0:c1]).reshape(-1))


@dataclasses.dataclass
class PackedModel:
    config: dict
    hex: dict[str, HexTensor]
    dense: dict[str, np.ndarray]
    avg_bpw: float = 0.0
    mode: str = "precision"
    extra: dict = dataclasses.field(default_factory=dict)

    def layer_linear(self, layer: int, name: str) -> HexTensor:
        return self.hex[f"blk.{layer}.{name}.weight"]

    def linear_bytes(self) -> int:
        return sum(t.nbytes() for t in self.hex.values())

    def linear_weights(self) -> int:
        return sum(t.rows * t.cols for t in self.hex.values())


def compute_avg_bpw(hexes: dict[str, HexTensor]) -> float:
    w = sum(t.rows * t.cols for t in hexes.values())
    return 8.0 * sum(t.nbytes() for t in hexes.values()) / max(w, 1)


INT_CONFIG_KEYS = ("n_layers", "hidden_size", "n_heads", "n_kv_heads", "head_dim", "ffn_size", "vocab_size")


def check_config(cfg: dict) -> None:
    """Shape keys are positive integers and rms_eps / rope_theta positive finite numbers, checked before any
    arithmetic on them (the reference reads them unchecked, gsd_lq_cpu_runtime.py:136-145)."""
    if not isinstance(cfg, dict):
        raise FormatError("config must be a JSON object")
    for k in CONFIG_KEYS:
        if k not in cfg:
            raise FormatError(f"config is missing {k!r}")
    for k in INT_CONFIG_KEYS:
        v = cfg[k]
        if isinstance(v, bool) or not isinstance(v, int) or v <= 0:
            raise FormatError(f"config {k}={v!r} is not a positive integer")
    for k in ("rms_eps", "rope_theta"):
        v = cfg[k]
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not np.isfinite(v) or v <= 0:
            raise FormatError(f"config {k}={v!r} is not a positive finite number")
    if cfg["n_heads"] % cfg["n_kv_heads"]:
        raise FormatError("n_heads must be a multiple of n_kv_heads")
    if cfg["head_dim"] % 2:
        raise FormatError("head_dim must be even")


def hex_names(n_layers: int) -> list[str]:
    names = [f"blk.{l}.{n}.weight" for l in range(n_layers) for n in LINEAR_NAMES]
    return names + ["output.weight"]


def dense_names(n_layers: int) -> list[str]:
    names = ["token_embd.weight", "output_norm.weight"]
    for l in range(n_layers):
        names += [f"blk.{l}.attn_norm.weight", f"blk.{l}.ffn_norm.weight"]
    return names


def write_gsd2(path: str, model: PackedModel) -> None:
    """Write ``model`` as a .gsd2 file that the reference's own readers accept."""
    check_config(model.config)
    metas: dict = {}
    chunks: list[tuple[int, np.ndarray]] = []
    off = 0

    def put(a: np.ndarray) -> dict:
        nonlocal off
        off = (off + ALIGN - 1) // ALIGN * ALIGN
        m = {"offset": off, "nbytes": int(a.nbytes)}
        chunks.append((off, np.ascontiguousarray(a)))
        off += a.nbytes
        return m

    for name, a in model.dense.items():
        m = put(a)
        m["shape"] = list(a.shape)
        metas[name] = {"data": m, "dtype": str(a.dtype)}
    for name, t in model.hex.items():
        t.validate(check_codes=False)
        m = {"radius": t.radius, "k_dim": t.k_dim, "rows": t.rows, "cols": t.cols}
        for bn, a in t.blobs().items():
            m[bn] = put(a)
        metas[name] = m
    # keys carried over from a file that was read come first: the layout keys below describe this file
    header = dict(model.extra)
    header.update({"format_version": 2, "mode": model.mode, "alignment": ALIGN,
                   "avg_bpw": float(model.avg_bpw or compute_avg_bpw(model.hex)),
                   "config": model.config, "tensors": metas})
    hb = json.dumps(header).encode("utf-8")
    # pad the header so that the blob region starts on an aligned file offset
    pad = (-(12 + len(hb))) % ALIGN
    hb += b" " * pad
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        base = f.tell()
        for o, a in chunks:
            f.seek(base + o)
            f.write(a.tobytes(order="C"))
        f.truncate(base + off)


def read_gsd2(path: str, mmap: bool = True, check_codes: bool = True,
              progress: Callable[[str], None] | None = None, check_values: bool = True) -> PackedModel:
    """Parse and validate a .gsd2 file.  Blobs are read-only memory-mapped views when ``mmap``.

    ``check_codes`` scans every code against the codebook size; ``check_values`` checks that scales, norm
    weights, S, U, Vt and kink deltas are finite.  A header that states an ``alignment`` (this writer's files)
    must keep every blob offset on it; the reference's own files state none and may place blobs anywhere.
    """
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        magic = f.read(4)
        if magic != MAGIC:
            raise FormatError(f"invalid GSD2 magic {magic!r}")
        raw = f.read(8)
        if len(raw) != 8:
            raise FormatError("truncated header length")
        hlen = struct.unpack("<Q", raw)[0]
        if hlen <= 0 or 12 + hlen > size:
            raise FormatError(f"header length {hlen} exceeds file size {size}")
        try:
            header = json.loads(f.read(hlen).decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise FormatError(f"header is not JSON: {e}") from None
    if not isinstance(header, dict):
        raise FormatError("header must be a JSON object")
    align = header.get("alignment", 1)
    if isinstance(align, bool) or not isinstance(align, int) or align <= 0 or align & (align - 1):
        raise FormatError(f"alignment {align!r} is not a positive power of two")
    base = 12 + hlen
    data = np.memmap(path, dtype=np.uint8, mode="r") if mmap else np.fromfile(path, dtype=np.uint8)

    def blob(meta: dict, dt, what: str) -> np.ndarray:
        try:
            o, n = meta["offset"], meta["nbytes"]
            if isinstance(o, bool) or isinstance(n, bool) or not isinstance(o, int) or not isinstance(n, int):
                raise TypeError
        except (KeyError, TypeError):
            raise FormatError(f"{what}: malformed blob descriptor") from None
        if o < 0 or n < 0 or base + o + n > size:
            raise FormatError(f"{what}: blob [{o}, {o + n}) runs past the end of the file")
        if o % align:
            raise FormatError(f"{what}: offset {o} breaks the header's {align}-byte alignment")
        if n % np.dtype(dt).itemsize:
            raise FormatError(f"{what}: {n} bytes is not a whole number of {np.dtype(dt)}")
        return data[base + o:base + o + n].view(dt)

    if "config" not in header or "tensors" not in header:
        raise FormatError("header lacks config/tensors")
    cfg = header["config"]
    check_config(cfg)
    tensors = header["tensors"]
    if not isinstance(tensors, dict) or not all(isinstance(v, dict) for v in tensors.values()):
        raise FormatError("tensors must map names to JSON objects")
    L = cfg["n_layers"]
    dense: dict[str, np.ndarray] = {}
    for name in dense_names(L):
        if name not in tensors:
            raise FormatError(f"missing tensor {name}")
        m = tensors[name].get("data")
        if not isinstance(m, dict):
            raise FormatError(f"{name}: missing data descriptor")
        dt = np.float16 if name == "token_embd.weight" else np.float32
        a = blob(m, dt, name)
        shape = m.get("shape", [a.size])
        if not isinstance(shape, list) or not all(isinstance(d, int) and not isinstance(d, bool) and d >= 0
                                                  for d in shape):
            raise FormatError(f"{name}: shape {shape!r} is not a list of sizes")
        shape = tuple(shape)
        if int(np.prod(shape)) != a.size:
            raise FormatError(f"{name}: shape {shape} does not match {a.size} elements")
        if check_values and not np.all(np.isfinite(a)):
            raise FormatError(f"{name}: non-finite values")
        dense[name] = a.reshape(shape)
    H, V = cfg["hidden_size"], cfg["vocab_size"]
    if dense["token_embd.weight"].shape != (V, H):
        raise FormatError("token_embd.weight must be [vocab, hidden]")
    hexes: dict[str, HexTensor] = {}
    for name in hex_names(L):
        if name not in tensors:
            raise FormatError(f"missing tensor {name}")
        m = tensors[name]
        try:
            k = int(m["k_dim"])
            if not 0 <= k <= MAX_K:
                raise FormatError(f"{name}: k_dim={k} outside [0, {MAX_K}]")
            if int(m["radius"]) not in codebook.RADII:
                raise FormatError(f"{name}: radius {m['radius']} not in {codebook.RADII}")
            t = HexTensor(
                rows=int(m["rows"]), cols=int(m["cols"]), radius=int(m["radius"]), k_dim=k,
                codes=blob(m["codes"], np.uint8, name + ".codes"),
                scales=blob(m["scales"], np.uint16, name + ".scales"),
                row_ptr=blob(m["row_ptr"], np.uint32, name + ".row_ptr"),
                kink_cols=blob(m["kink_cols"], np.uint16, name + ".kink_cols"),
                kink_deltas=blob(m["kink_deltas"], np.float32, name + ".kink_deltas"),
                U=blob(m["U"], np.uint16, name + ".U") if k > 0 else None,
                S=blob(m["S"], np.float32, name + ".S") if k > 0 else None,
                Vt=blob(m["Vt"], np.uint16, name + ".Vt") if k > 0 else None)
        except KeyError as e:
            raise FormatError(f"{name}: missing field {e}") from None
        try:
            t.validate(check_codes=check_codes, check_values=check_values)
        except FormatError as e:
            raise FormatError(f"{name}: {e}") from None
        hexes[name] = t
        if progress:
            progress(name)
    _check_shapes(cfg, hexes)
    extra = {k: v for k, v in header.items() if k not in ("config", "tensors", "avg_bpw", "mode")}
    return PackedModel(config=cfg, hex=hexes, dense=dense, avg_bpw=float(header.get("avg_bpw", 3.79)),
                       mode=str(header.get("mode", "unknown")), extra=extra)


def _check_shapes(cfg: dict, hexes: dict[str, HexTensor]) -> None:
    H, F = cfg["hidden_size"], cfg["ffn_size"]
    q, kv = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    want = {"attn_q": (q, H), "attn_k": (kv, H), "attn_v": (kv, H), "attn_output": (H, q),
            "ffn_gate": (F, H), "ffn_up": (F, H), "ffn_down": (H, F)}
    for l in range(cfg["n_layers"]):
        for n, shp in want.items():
            t = hexes[f"blk.{l}.{n}.weight"]
            if (t.rows, t.cols) != shp:
                raise FormatError(f"blk.{l}.{n}: shape {(t.rows, t.cols)} != {shp}")
    t = hexes["output.weight"]
    if (t.rows, t.cols) != (cfg["vocab_size"], H):
        raise FormatError("output.weight must be [vocab, hidden]")

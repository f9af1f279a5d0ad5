"""Torch-tensor wrappers over the C ABI (device memory in, device memory out).

Every function launches on the current torch CUDA stream and raises
``GsdlqError`` when the library reports a failure.  No function here has a
CPU path.
"""
from __future__ import annotations

import ctypes
import warnings

import numpy as np
import torch

from . import _lib as L
from .gsd2 import HexTensor


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_handle(stream: torch.cuda.Stream | None = None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _lib():
    return L.load()


def to_device_bytes(a: np.ndarray, device) -> torch.Tensor:
    """Upload the raw bytes of a NumPy array (any dtype) as a uint8 device tensor."""
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.reshape(-1).view(np.uint8))
    return t.to(device, non_blocking=False)


class DeviceHex:
    """A packed linear resident in device memory (reference layout), with its C descriptor."""

    def __init__(self, t: HexTensor | None = None, device="cuda", arena: "Arena | None" = None, **tensors):
        if t is not None:
            self.rows, self.cols, self.k_dim, self.radius = t.rows, t.cols, t.k_dim, t.radius
            up = (lambda a: arena.put(a)) if arena is not None else (lambda a: to_device_bytes(a, device))
            self.codes = up(t.codes)
            self.scales = up(t.scales)
            self.row_ptr = up(t.row_ptr)
            self.kink_cols = up(t.kink_cols) if t.nnz else None
            self.kink_deltas = up(t.kink_deltas) if t.nnz else None
            self.U = up(t.U) if t.k_dim else None
            self.S = up(t.S) if t.k_dim else None
            self.Vt = up(t.Vt) if t.k_dim else None
            self.nnz = t.nnz
        else:  # already on the device (GPU packer)
            for k, v in tensors.items():
                setattr(self, k, v)
        self.n_pts = 217 if self.radius == 8 else 127

    def nbytes(self) -> int:
        n = 0
        for k in ("codes", "scales", "row_ptr", "kink_cols", "kink_deltas", "U", "S", "Vt"):
            v = getattr(self, k, None)
            if v is not None:
                n += v.numel() * v.element_size()
        return n

    def build_unit_kinks(self):
        """Regroup the CSR kinks per 16-row x 512-column work unit (gsdlq_unit_kinks); the fused
        linear then applies them in its streaming loop.  Keeps the CSR arrays (the drop-in path)."""
        gu = (self.cols // 64 + 7) // 8
        n_units = ((self.rows + 15) // 16) * gu
        dev = self.codes.device
        self.unit_kink_off = torch.zeros(n_units + 1, dtype=torch.int32, device=dev)
        self.unit_kinks = torch.zeros(max(1, 2 * self.nnz), dtype=torch.int32, device=dev)
        L.check(_lib().gsdlq_unit_kinks(ptr(self.row_ptr), ptr(self.kink_cols), ptr(self.kink_deltas), self.rows,
                                        self.cols, ptr(self.unit_kink_off), ptr(self.unit_kinks), stream_handle()),
                "gsdlq_unit_kinks")
        return self

    def desc(self) -> L.HexMat:
        uko = getattr(self, "unit_kink_off", None)
        uk = getattr(self, "unit_kinks", None)
        return L.HexMat(unit_kink_off=uko.data_ptr() if uko is not None else None,
                        unit_kinks=uk.data_ptr() if uk is not None else None,
                        codes=self.codes.data_ptr(), scales=self.scales.data_ptr(),
                        U=self.U.data_ptr() if self.U is not None else None,
                        S=self.S.data_ptr() if self.S is not None else None,
                        Vt=self.Vt.data_ptr() if self.Vt is not None else None,
                        row_ptr=self.row_ptr.data_ptr(),
                        kink_cols=self.kink_cols.data_ptr() if self.kink_cols is not None else None,
                        kink_deltas=self.kink_deltas.data_ptr() if self.kink_deltas is not None else None,
                        rows=self.rows, cols=self.cols, k_dim=self.k_dim, radius=self.radius)


class Arena:
    """One device allocation holding many 256-byte-aligned blobs (fewer, larger copies)."""

    ALIGN = 256

    def __init__(self, nbytes: int, device="cuda"):
        self.buf = torch.empty(nbytes + self.ALIGN, dtype=torch.uint8, device=device)
        self.off = (-self.buf.data_ptr()) % self.ALIGN
        self.cap = nbytes + self.ALIGN

    @classmethod
    def bytes_needed(cls, arrays) -> int:
        return sum((a.nbytes + cls.ALIGN - 1) // cls.ALIGN * cls.ALIGN for a in arrays)

    def put(self, a: np.ndarray) -> torch.Tensor:
        a = np.ascontiguousarray(a)
        n = a.nbytes
        if self.off + n > self.cap:
            raise MemoryError("arena overflow")
        dst = self.buf[self.off:self.off + n]
        if n:
            # read-only memory-mapped blobs go straight to the device: torch only reads the view
            with warnings.catch_warnings():
                warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
                src = torch.from_numpy(a.reshape(-1).view(np.uint8))
            dst.copy_(src, non_blocking=False)
        self.off += (n + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        return dst

    def alloc(self, n: int) -> torch.Tensor:
        if self.off + n > self.cap:
            raise MemoryError("arena overflow")
        dst = self.buf[self.off:self.off + n]
        self.off += (n + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        return dst


# ---- drop-in functions (reference signatures) --------------------------------------------
def rmsnorm(x, w, out, eps):
    L.check(_lib().gsdlq_rmsnorm(ptr(x), ptr(w), ptr(out), x.numel(), eps, stream_handle()), "rmsnorm")


def vec_add(y, a, b):
    L.check(_lib().gsdlq_vec_add(ptr(y), ptr(a), ptr(b), y.numel(), stream_handle()), "vec_add")


def swiglu(gate, up, out):
    L.check(_lib().gsdlq_swiglu(ptr(gate), ptr(up), ptr(out), gate.numel(), stream_handle()), "swiglu")


def lowrank_proj(x, h: DeviceHex, tmp_k):
    L.check(_lib().gsdlq_lowrank_proj(ptr(x), ptr(h.Vt), ptr(h.S), ptr(tmp_k), h.k_dim, h.cols,
                                      stream_handle()), "lowrank_proj")


def hex2d_matvec(x, h: DeviceHex, xy_table, tmp_k, y):
    L.check(_lib().gsdlq_hex2d_matvec(ptr(x), ptr(h.codes), ptr(h.scales), ptr(xy_table), ptr(h.U), ptr(tmp_k),
                                      ptr(h.row_ptr), ptr(h.kink_cols), ptr(h.kink_deltas), ptr(y), h.rows, h.cols,
                                      h.k_dim, h.n_pts, stream_handle()), "hex2d_matvec")


MATMUL_MAX_BATCH = 128  # GSDLQ_MATMUL_MAX_BATCH


def matmul_work_bytes(batch: int, cols: int) -> int:
    n = ctypes.c_size_t()
    L.check(_lib().gsdlq_hex2d_matmul_work_size(batch, cols, ctypes.byref(n)), "hex2d_matmul_work_size")
    return int(n.value)


def matmul_work(batch: int, cols: int, device="cuda") -> torch.Tensor:
    """Scratch for hex2d_matmul of up to ``batch`` tokens and ``cols`` columns (1024-byte aligned)."""
    return torch.empty(matmul_work_bytes(batch, cols) + 1024, dtype=torch.uint8, device=device)


def _aligned(work: torch.Tensor) -> tuple[int, int]:
    p = work.data_ptr()
    a = (p + 1023) & ~1023
    return a, work.numel() * work.element_size() - (a - p)


def hex2d_matmul(x, h: DeviceHex, xy_table, y, work):
    """y[b] = the packed linear of x[b] for every row b of x ([batch][cols] -> [batch][rows]); work: a
    matmul_work buffer."""
    wp, wb = _aligned(work)
    L.check(_lib().gsdlq_hex2d_matmul(ptr(x), x.shape[0], ptr(h.codes), ptr(h.scales), ptr(xy_table), ptr(h.U),
                                      ptr(h.S), ptr(h.Vt), ptr(h.row_ptr), ptr(h.kink_cols), ptr(h.kink_deltas),
                                      ptr(y), wp, wb, h.rows, h.cols, h.k_dim, h.n_pts, stream_handle()),
            "hex2d_matmul")


def sample_top_p(logits: torch.Tensor, temperature: float, top_p: float, u: float) -> int:
    """gsdlq_sample_top_p over a device logits vector with the uniform draw u; returns the pick."""
    n = logits.numel()
    b = ctypes.c_size_t()
    L.check(_lib().gsdlq_sample_work_size(n, ctypes.byref(b)), "sample_work_size")
    work = torch.empty(int(b.value), dtype=torch.uint8, device=logits.device)
    ud = torch.tensor([u], dtype=torch.float64, device=logits.device)
    out = torch.full((1,), -2, dtype=torch.int32, device=logits.device)
    L.check(_lib().gsdlq_sample_top_p(ptr(logits), n, float(temperature), float(top_p), ptr(ud), None, ptr(work),
                                      work.numel(), None, ptr(out), stream_handle()), "sample_top_p")
    return int(out.item())


def attention_rows_work(n: int, n_heads: int, head_dim: int, device="cuda") -> torch.Tensor:
    """Scratch for gsdlq_attention_rows of up to ``n`` tokens (float32; torch's allocations are 16-byte
    aligned)."""
    b = ctypes.c_size_t()
    L.check(_lib().gsdlq_attention_rows_work_size(n, n_heads, head_dim, ctypes.byref(b)), "attention_rows_work_size")
    return torch.empty(int(b.value), dtype=torch.uint8, device=device)


def rope_and_store_kv(q, k, v, k_cache, v_cache, layer, pos, n_heads, n_kv, hd, max_seq, theta, interleaved=1):
    L.check(_lib().gsdlq_rope_and_store_kv(ptr(q), ptr(k), ptr(v), ptr(k_cache), ptr(v_cache), layer, pos, n_heads,
                                           n_kv, hd, max_seq, theta, interleaved, stream_handle()),
            "rope_and_store_kv")


def gqa_attention(q, k_cache, v_cache, out, layer, pos, n_heads, n_kv, hd, max_seq, sm_scale):
    L.check(_lib().gsdlq_gqa_attention(ptr(q), ptr(k_cache), ptr(v_cache), ptr(out), layer, pos, n_heads, n_kv, hd,
                                       max_seq, sm_scale, stream_handle()), "gqa_attention")


# ---- engine functions ---------------------------------------------------------------------
def codebook(radius: int) -> np.ndarray:
    buf = np.zeros(2 * 256, np.float32)
    n = _lib().gsdlq_codebook(radius, buf.ctypes.data_as(ctypes.c_void_p), 256)
    if n < 0:
        L.check(n, "codebook")
    return buf[:2 * n].reshape(n, 2).copy()


def dequant(h: DeviceHex, xy_table, out):
    L.check(_lib().gsdlq_dequant(ptr(h.codes), ptr(h.scales), ptr(xy_table), ptr(out), h.rows, h.cols, h.n_pts,
                                 stream_handle()), "dequant")


def argmax(x, out_idx):
    L.check(_lib().gsdlq_argmax(ptr(x), x.numel(), ptr(out_idx), stream_handle()), "argmax")


def pack_lattice(w: torch.Tensor, radius: int, codes, scales, residual=None):
    r, c = w.shape
    L.check(_lib().gsdlq_pack_lattice(ptr(w), r, c, radius, ptr(codes), ptr(scales), ptr(residual),
                                      stream_handle()), "pack_lattice")


def rope_table(max_seq: int, head_dim: int, theta: float) -> np.ndarray:
    t = np.zeros((max_seq, head_dim // 2, 2), np.float32)
    L.check(_lib().gsdlq_rope_table(t.ctypes.data_as(ctypes.c_void_p), max_seq, head_dim, theta), "rope_table")
    return t


def linear_ws_size(job: L.LinearJob) -> int:
    n = ctypes.c_size_t(0)
    L.check(_lib().gsdlq_linear_ws_size(ctypes.byref(job), ctypes.byref(n)), "gsdlq_linear_ws_size")
    return n.value


def linear_workspace(job: L.LinearJob, device="cuda") -> torch.Tensor:
    """A zeroed, 16-byte aligned device workspace large enough for ``job``."""
    return torch.zeros((linear_ws_size(job) + 15) // 16 * 4, dtype=torch.int32, device=device)


def linear(job: L.LinearJob, ws: torch.Tensor):
    L.check(_lib().gsdlq_linear(ctypes.byref(job), ptr(ws), ws.numel() * ws.element_size(), stream_handle()),
            "gsdlq_linear")


def attention_ws_size(n_heads, n_kv, hd, max_seq) -> tuple[int, int]:
    pb, wb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    L.check(_lib().gsdlq_attention_ws_size(n_heads, n_kv, hd, max_seq, ctypes.byref(pb), ctypes.byref(wb)),
            "attention_ws_size")
    return pb.value, wb.value


def attention(job: L.AttnJob):
    L.check(_lib().gsdlq_attention(ctypes.byref(job), stream_handle()), "gsdlq_attention")

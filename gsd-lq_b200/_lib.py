"""ctypes binding of libgsdlq_cuda.so (the C ABI declared in include/gsdlq.h).

The library is loaded from the package directory, where ``build.py`` puts it.
There is no fallback: if the library is missing or a call fails, an exception
is raised.
"""
from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libgsdlq_cuda.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "gsdlq.h")

vp, i32, f32, u32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_uint
szp = ctypes.POINTER(ctypes.c_size_t)

GSDLQ_OK = 0
EPI_STORE, EPI_RESID, EPI_SWIGLU, EPI_ROPE_KV = 0, 1, 2, 3
IN_PLAIN, IN_RMSNORM, IN_EMBED = 0, 1, 2
FLAG_NAMES = {0x1: "bad_code", 0x2: "bad_kink", 0x4: "bad_pos", 0x8: "bad_table", 0x10: "timeout",
              0x20: "bad_token", 0x40: "unsupported", 0x80: "range"}


class HexMat(ctypes.Structure):
    _fields_ = [("codes", vp), ("scales", vp), ("U", vp), ("S", vp), ("Vt", vp), ("row_ptr", vp),
                ("kink_cols", vp), ("kink_deltas", vp), ("rows", i32), ("cols", i32), ("k_dim", i32),
                ("radius", i32), ("unit_kink_off", vp), ("unit_kinks", vp)]


MAX_PREFETCH = 16


class Prefetch(ctypes.Structure):
    _fields_ = [("ptr", vp * MAX_PREFETCH), ("bytes", ctypes.c_uint64 * MAX_PREFETCH), ("n", i32)]


class LinearJob(ctypes.Structure):
    _fields_ = [("mat", HexMat * 3), ("n_mat", i32), ("input_mode", i32), ("x", vp), ("norm_w", vp),
                ("eps", f32), ("embed", vp), ("token", vp), ("vocab", i32), ("x_out", vp), ("epilogue", i32),
                ("y", vp * 3), ("resid", vp), ("k_cache", vp), ("v_cache", vp), ("pos", vp), ("rope_cs", vp),
                ("layer", i32), ("max_seq", i32), ("head_dim", i32), ("interleaved", i32),
                ("argmax_key", vp), ("argmax_index_base", i32), ("fwd_vt", vp * 3), ("fwd_k", i32 * 3),
                ("fwd_norm_w", vp), ("fwd_acc", vp), ("lr_forwarded", i32), ("prefetch", Prefetch),
                ("exchange", vp)]


class AttnJob(ctypes.Structure):
    _fields_ = [("q", vp), ("k_cache", vp), ("v_cache", vp), ("out", vp), ("pos_dev", vp), ("pos_val", i32),
                ("layer", i32), ("n_heads", i32), ("n_kv_heads", i32), ("head_dim", i32), ("max_seq", i32),
                ("sm_scale", f32), ("block_table", vp), ("page_size", i32), ("partial", vp), ("workspace", vp),
                ("fwd_vt", vp), ("fwd_k", i32), ("fwd_acc", vp), ("prefetch", Prefetch)]


class DecodeLayer(ctypes.Structure):
    _fields_ = [("qkv", LinearJob), ("attn", AttnJob), ("o", LinearJob), ("gate_up", LinearJob), ("down", LinearJob)]


class DecodeDesc(ctypes.Structure):
    _fields_ = [("n_layers", i32), ("layers", ctypes.POINTER(DecodeLayer)), ("head", LinearJob),
                ("argmax_key", vp), ("token", vp), ("pos", vp), ("step", vp), ("out_ids", vp), ("max_out", i32)]


SIGNATURES = {
    "gsdlq_status_string": ([i32], ctypes.c_char_p),
    "gsdlq_last_cuda_error": ([], i32),
    "gsdlq_device_flags": ([ctypes.POINTER(u32), vp], i32),
    "gsdlq_version": ([], ctypes.c_char_p),
    "gsdlq_rmsnorm": ([vp, vp, vp, i32, f32, vp], i32),
    "gsdlq_vec_add": ([vp, vp, vp, i32, vp], i32),
    "gsdlq_swiglu": ([vp, vp, vp, i32, vp], i32),
    "gsdlq_lowrank_proj": ([vp, vp, vp, vp, i32, i32, vp], i32),
    "gsdlq_hex2d_matvec": ([vp] * 10 + [i32] * 4 + [vp], i32),
    "gsdlq_hex2d_matvec_noalloc": ([vp] * 10 + [i32] * 4 + [vp], i32),
    "gsdlq_hex2d_matmul": ([vp, i32] + [vp] * 11 + [ctypes.c_size_t] + [i32] * 4 + [vp], i32),
    "gsdlq_hex2d_matmul_work_size": ([i32, i32, szp], i32),
    "gsdlq_rope_and_store_kv": ([vp] * 5 + [i32] * 6 + [f32, i32, vp], i32),
    "gsdlq_gqa_attention": ([vp] * 4 + [i32] * 6 + [f32, vp], i32),
    "gsdlq_codebook": ([i32, vp, i32], i32),
    "gsdlq_dequant": ([vp, vp, vp, vp, i32, i32, i32, vp], i32),
    "gsdlq_argmax": ([vp, i32, vp, vp], i32),
    "gsdlq_pack_lattice": ([vp, i32, i32, i32, vp, vp, vp, vp], i32),
    "gsdlq_linear": ([ctypes.POINTER(LinearJob), vp, ctypes.c_size_t, vp], i32),
    "gsdlq_linear_ws_size": ([ctypes.POINTER(LinearJob), szp], i32),
    "gsdlq_attention_ws_size": ([i32, i32, i32, i32, szp, szp], i32),
    "gsdlq_attention": ([ctypes.POINTER(AttnJob), vp], i32),
    "gsdlq_rope_table": ([vp, i32, i32, f32], i32),
    "gsdlq_greedy_advance": ([vp, vp, vp, vp, vp, i32, vp], i32),
    "gsdlq_advance_eos": ([vp, vp, vp, vp, vp, i32, i32, vp, vp], i32),
    "gsdlq_sample_work_size": ([i32, szp], i32),
    "gsdlq_sample_top_p": ([vp, i32, f32, f32, vp, vp, vp, ctypes.c_size_t, vp, vp, vp], i32),
    "gsdlq_unit_kinks": ([vp, vp, vp, i32, i32, vp, vp, vp], i32),
    "gsdlq_decode_plan_create": ([ctypes.POINTER(DecodeDesc), ctypes.POINTER(vp)], i32),
    "gsdlq_decode_step": ([vp, vp], i32),
    "gsdlq_decode_plan_destroy": ([vp], i32),
    "gsdlq_comm_create": ([i32, i32, i32, ctypes.POINTER(vp), vp], i32),
    "gsdlq_comm_connect": ([vp, vp], i32),
    "gsdlq_comm_allreduce_sum": ([vp, vp, i32, vp], i32),
    "gsdlq_comm_allreduce_max_u64": ([vp, vp, vp], i32),
    "gsdlq_comm_destroy": ([vp], i32),
    "gsdlq_embed_rows": ([vp, vp, i32, i32, i32, vp, vp], i32),
    "gsdlq_rmsnorm_rows": ([vp, vp, vp, i32, i32, f32, vp], i32),
    "gsdlq_rope_kv_rows": ([vp] * 6 + [i32] * 7 + [vp], i32),
    "gsdlq_attention_rows_work_size": ([i32, i32, i32, ctypes.POINTER(ctypes.c_size_t)], i32),
    "gsdlq_rope_kv_batch": ([vp] * 3 + [i32] + [vp] * 2 + [ctypes.c_size_t, vp, i32, vp] + [i32] * 5 + [vp], i32),
    "gsdlq_attention_decode_batch": ([vp, i32, vp, vp, ctypes.c_size_t, vp, vp, ctypes.c_size_t, i32, vp]
                                     + [i32] * 5 + [f32, vp], i32),
    "gsdlq_swiglu_rows": ([vp, vp, i32, i32, vp], i32),
    "gsdlq_argmax_rows": ([vp, i32, i32, vp, vp, vp, i32, vp], i32),
    "gsdlq_attention_rows": ([vp] * 5 + [ctypes.c_size_t] + [i32] * 7 + [f32, vp], i32),
}
IPC_HANDLE_BYTES = 64


class GsdlqError(RuntimeError):
    pass


_lib = None


def header_symbols(path: str = HEADER) -> list[str]:
    """Function names declared in include/gsdlq.h."""
    txt = open(path).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(gsdlq_[a-z0-9_]+)\s*\(", txt)))


def load(path: str = LIB_PATH):
    """Load and type the library (once).  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise GsdlqError(f"{path} is missing: build it with `python -m gsdlq_b200.build` "
                         "(or __graft_entry__.build()); there is no CPU fallback")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(status: int, what: str = "") -> None:
    if status != GSDLQ_OK:
        lib = load()
        msg = lib.gsdlq_status_string(status).decode()
        extra = ""
        if status == -2:
            extra = f" (cudaError {lib.gsdlq_last_cuda_error()})"
        raise GsdlqError(f"{what or 'gsdlq call'} failed: {msg}{extra}")


def device_flags(stream=None) -> int:
    lib = load()
    v = u32(0)
    check(lib.gsdlq_device_flags(ctypes.byref(v), stream), "gsdlq_device_flags")
    return int(v.value)


def flag_names(flags: int) -> list[str]:
    return [n for b, n in FLAG_NAMES.items() if flags & b]

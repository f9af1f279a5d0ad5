"""Synthetic, format-conformant GSD-LQ packer.

The reference ships no packer (its READMEs call the encoder proprietary), so
the engine brings its own.  It writes exactly the fields the reference's
readers and kernels consume; how well it compresses is not a claim of this
project.  Design (one 64-weight group = one fp16 scale, one code per weight pair):

  1. scale = max|w| over the group / (R * FIT), FIT = 1/(1 + 1/sqrt(3)), so the
     square [-max, max]^2 of any pair, divided by the scale, lies inside the
     radius-R hexagon; the scale is rounded to fp16 and that rounded value is
     the one used below.
  2. each pair (w0, w1)/scale is rounded to the nearest A2 lattice point: the
     point lies in one rhombus (r0f, r1f) of the (1,0),(1/2,sqrt3/2) basis and
     its nearest lattice point is one of the rhombus's four corners; ties keep
     the first corner in the order (0,0),(1,0),(0,1),(1,1).  A corner outside
     the hexagon is replaced by the nearest hexagon point.  All of this is
     float32 arithmetic with no fused multiply-add, so the NumPy and CUDA
     packers produce identical codes and scales.
  3. residual E = W - dequant(codes, scales).  Precision mode: a rank-k
     truncated SVD E ~ U diag(S) Vt (U, Vt stored fp16, S fp32) and, per row,
     the ``kinks_per_row`` largest |E - U S Vt| entries as CSR "kinks"
     (ascending column order).  Turbo mode: k=0 and no kinks.

Modes: turbo = radius 8, k 0, no kinks (4.26 bpw incl. row_ptr);
precision = radius 8, k 16, max(4, cols/256) kinks per row.
"""
from __future__ import annotations

import numpy as np

from . import codebook
from .gsd2 import HexTensor, PackedModel, compute_avg_bpw, hex_names, LINEAR_NAMES

FIT = np.float32(1.0 / (1.0 + 1.0 / np.sqrt(3.0)))
H32 = np.float32(np.sqrt(3.0) / 2.0)
IH32 = np.float32(2.0 / np.sqrt(3.0))

MODES = {
    "turbo": {"radius": 8, "k_dim": 0, "kink_div": 0},
    "precision": {"radius": 8, "k_dim": 16, "kink_div": 256},
}


def mode_params(mode: str, cols: int) -> tuple[int, int, int]:
    p = MODES[mode]
    kinks = max(4, cols // p["kink_div"]) if p["kink_div"] else 0
    return p["radius"], p["k_dim"], kinks


def group_scales(w: np.ndarray, radius: int) -> np.ndarray:
    """fp16 scale bits [R*C/64] for a float32 [R, C] matrix."""
    r, c = w.shape
    amax = np.abs(w.reshape(r, c // 64, 64)).max(axis=2)
    s = (amax / (np.float32(radius) * FIT)).astype(np.float32)
    return s.astype(np.float16).view(np.uint16).reshape(-1)


def quantize_lattice(w: np.ndarray, radius: int) -> tuple[np.ndarray, np.ndarray]:
    """Lattice codes u8[R*C/2] and fp16 scale bits u16[R*C/64] of a float32 [R, C] matrix."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    r, c = w.shape
    if c % 64:
        raise ValueError("cols must be a multiple of 64")
    sbits = group_scales(w, radius)
    s = sbits.view(np.float16).astype(np.float32)
    inv = np.zeros_like(s)
    nz = s > 0
    inv[nz] = np.float32(1.0) / s[nz]
    inv_e = np.repeat(inv.reshape(r, c // 64), 32, axis=1).reshape(-1)   # one per pair
    pairs = w.reshape(-1, 2)
    u = pairs[:, 0] * inv_e
    v = pairs[:, 1] * inv_e
    r1f = v * IH32
    r0f = u - np.float32(0.5) * r1f
    a = np.floor(r0f).astype(np.int32)
    b = np.floor(r1f).astype(np.int32)
    best_d = None
    best0 = best1 = None
    for da, db in ((0, 0), (1, 0), (0, 1), (1, 1)):
        c0, c1 = a + da, b + db
        px = c0.astype(np.float32) + np.float32(0.5) * c1.astype(np.float32)
        py = c1.astype(np.float32) * H32
        dx = u - px
        dy = v - py
        d = dx * dx + dy * dy
        if best_d is None:
            best_d, best0, best1 = d, c0, c1
        else:
            take = d < best_d
            best_d = np.where(take, d, best_d)
            best0 = np.where(take, c0, best0)
            best1 = np.where(take, c1, best1)
    R = radius
    out = (np.abs(best0) > R) | (np.abs(best1) > R) | (np.abs(best0 + best1) > R)
    if np.any(out):
        idx = np.nonzero(out)[0]
        pts = codebook.lattice_coords(R).astype(np.int32)
        px = pts[:, 0].astype(np.float32) + np.float32(0.5) * pts[:, 1].astype(np.float32)
        py = pts[:, 1].astype(np.float32) * H32
        dx = u[idx, None] - px[None, :]
        dy = v[idx, None] - py[None, :]
        j = np.argmin(dx * dx + dy * dy, axis=1)
        best0[idx] = pts[j, 0]
        best1[idx] = pts[j, 1]
    codes = codebook.code_index_table(R)[best0 + R, best1 + R]
    assert codes.min() >= 0
    return codes.astype(np.uint8), sbits


def dequant(codes: np.ndarray, sbits: np.ndarray, radius: int, rows: int, cols: int) -> np.ndarray:
    """W[r,c] = xy[code][c&1] * f32(scale): the dequantised-weight definition."""
    xy = codebook.xy_table(radius)
    s = sbits.view(np.float16).astype(np.float32)
    return xy[codes].reshape(rows, cols) * np.repeat(s.reshape(rows, cols // 64), 64, axis=1)


def lowrank_kinks(e: np.ndarray, k_dim: int, kinks_per_row: int, rng: np.random.Generator | None = None):
    """Rank-k factors (U f16 bits, S f32, Vt f16 bits) and CSR kinks of a residual matrix."""
    r, c = e.shape
    U = S = Vt = None
    e2 = e
    if k_dim > 0:
        if min(r, c) <= 2048:
            u, s, vt = np.linalg.svd(e.astype(np.float64), full_matrices=False)
        else:  # randomized range finder with two power iterations
            rng = rng or np.random.default_rng(0)
            q = k_dim + 8
            y = e.astype(np.float64) @ rng.standard_normal((c, q))
            for _ in range(2):
                y, _ = np.linalg.qr(y)
                y = e.astype(np.float64) @ (e.astype(np.float64).T @ y)
            qm, _ = np.linalg.qr(y)
            ub, s, vt = np.linalg.svd(qm.T @ e.astype(np.float64), full_matrices=False)
            u = qm @ ub
        # a matrix smaller than k in either dimension has fewer components: the rest are zero, so the
        # factors keep the declared k_dim (the format's U/S/Vt sizes)
        kk = min(k_dim, u.shape[1])
        Uh = np.zeros((r, k_dim), np.float16)
        Uh[:, :kk] = u[:, :kk].astype(np.float16)
        Sf = np.zeros(k_dim, np.float32)
        Sf[:kk] = s[:kk].astype(np.float32)
        Vh = np.zeros((k_dim, c), np.float16)
        Vh[:kk] = vt[:kk].astype(np.float16)
        e2 = e - (Uh.astype(np.float32) * Sf[None, :]) @ Vh.astype(np.float32)
        U, S, Vt = Uh.view(np.uint16).reshape(-1), Sf, Vh.view(np.uint16).reshape(-1)
    if kinks_per_row > 0:
        n = min(kinks_per_row, c)
        cols = np.argpartition(-np.abs(e2), n - 1, axis=1)[:, :n]
        cols.sort(axis=1)
        deltas = np.take_along_axis(e2, cols, axis=1).astype(np.float32)
        row_ptr = np.arange(r + 1, dtype=np.uint32) * np.uint32(n)
        kc, kd = cols.astype(np.uint16).reshape(-1), deltas.reshape(-1)
    else:
        row_ptr = np.zeros(r + 1, np.uint32)
        kc, kd = np.zeros(0, np.uint16), np.zeros(0, np.float32)
    return U, S, Vt, row_ptr, kc, kd


def pack_matrix(w: np.ndarray, mode: str = "precision", radius: int | None = None,
                k_dim: int | None = None, kinks_per_row: int | None = None) -> HexTensor:
    """Pack one float32 [rows, cols] weight matrix."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    R, K, KN = mode_params(mode, cols)
    R = R if radius is None else radius
    K = K if k_dim is None else k_dim
    KN = KN if kinks_per_row is None else kinks_per_row
    codes, sbits = quantize_lattice(w, R)
    e = w - dequant(codes, sbits, R, rows, cols)
    U, S, Vt, rp, kc, kd = lowrank_kinks(e, K, KN)
    t = HexTensor(rows=rows, cols=cols, radius=R, k_dim=K, codes=codes, scales=sbits,
                  row_ptr=rp, kink_cols=kc, kink_deltas=kd, U=U, S=S, Vt=Vt)
    t.validate()
    return t


# ---------------------------------------------------------------------------------------
# model configurations (shape-only proxies; no bias, interleaved RoPE as the reference runs)
CONFIGS = {
    "mistral-7b": dict(n_layers=32, hidden_size=4096, n_heads=32, n_kv_heads=8, head_dim=128,
                       ffn_size=14336, vocab_size=32768, rms_eps=1e-5, rope_theta=1e6),
    "qwen2.5-1.5b": dict(n_layers=28, hidden_size=1536, n_heads=12, n_kv_heads=2, head_dim=128,
                         ffn_size=8960, vocab_size=151936, rms_eps=1e-6, rope_theta=1e6),
    "smollm2-1.7b": dict(n_layers=24, hidden_size=2048, n_heads=32, n_kv_heads=32, head_dim=64,
                         ffn_size=8192, vocab_size=49152, rms_eps=1e-5, rope_theta=1e4),
    "tiny": dict(n_layers=2, hidden_size=256, n_heads=4, n_kv_heads=2, head_dim=64,
                 ffn_size=512, vocab_size=512, rms_eps=1e-5, rope_theta=1e4),
}


def synthetic_vocab(vocab: int) -> dict:
    """Tokenizer tables the reference's loader requires (names only; prompts are token ids)."""
    toks, types = ["<unk>", "<s>", "</s>"], [2, 3, 3]
    if vocab >= 3 + 256:
        toks += [f"<0x{b:02X}>" for b in range(256)]
        types += [6] * 256
    while len(toks) < vocab:
        toks.append(f"▁w{len(toks)}")
        types.append(1)
    toks, types = toks[:vocab], types[:vocab]
    return {"tokens": toks, "scores": [-float(i) for i in range(vocab)], "token_types": types,
            "bos_id": 1, "eos_id": 2}


def make_config(name: str, **over) -> dict:
    cfg = dict(CONFIGS[name])
    cfg.update(over)
    cfg.update(synthetic_vocab(cfg["vocab_size"]))
    return cfg


def linear_shapes(cfg: dict) -> dict[str, tuple[int, int]]:
    H, F = cfg["hidden_size"], cfg["ffn_size"]
    q, kv = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    return {"attn_q": (q, H), "attn_k": (kv, H), "attn_v": (kv, H), "attn_output": (H, q),
            "ffn_gate": (F, H), "ffn_up": (F, H), "ffn_down": (H, F)}


def _norm(rng: np.random.Generator, n: int, jitter: float) -> np.ndarray:
    w = np.ones(n, np.float32)
    if jitter:
        w += np.float32(jitter) * rng.standard_normal(n, dtype=np.float32)
    return w


def random_model(cfg: dict, mode: str = "precision", seed: int = 0, std: float = 0.02,
                 norm_jitter: float = 0.0) -> PackedModel:
    """Random-init N(0, std^2) decoder packed with the NumPy packer (small shapes; tests).

    RMSNorm weights are 1 (+ ``norm_jitter`` * N(0,1) when non-zero, so tests see them used)."""
    rng = np.random.default_rng(seed)
    shapes = linear_shapes(cfg)
    hexes: dict[str, HexTensor] = {}
    for name in hex_names(cfg["n_layers"]):
        key = name.split(".")[-2]
        shp = shapes[key] if key in shapes else (cfg["vocab_size"], cfg["hidden_size"])
        w = (rng.standard_normal(shp, dtype=np.float32) * np.float32(std))
        hexes[name] = pack_matrix(w, mode)
    H = cfg["hidden_size"]
    dense = {"token_embd.weight":
             (rng.standard_normal((cfg["vocab_size"], H), dtype=np.float32) * np.float32(std)).astype(np.float16),
             "output_norm.weight": _norm(rng, H, norm_jitter)}
    for l in range(cfg["n_layers"]):
        dense[f"blk.{l}.attn_norm.weight"] = _norm(rng, H, norm_jitter)
        dense[f"blk.{l}.ffn_norm.weight"] = _norm(rng, H, norm_jitter)
    return PackedModel(config=cfg, hex=hexes, dense=dense, avg_bpw=compute_avg_bpw(hexes), mode=mode,
                       extra={"packer": {"name": "gsdlq_b200.packer", "seed": seed, "std": std}})


def _random_hex(rng, draw, r: int, c: int, mode: str, scale) -> HexTensor:
    """One format-valid packed tensor (see random_packed_model); draw(n) gives n uniform codes."""
    R, k, kn = mode_params(mode, c)
    codes = draw(r * c // 2)
    scales = np.full(r * c // 64, scale, np.uint16)
    if kn:
        kn = min(kn, c)
        # distinct ascending columns per row: one random offset inside each of kn equal bins
        bins = (np.arange(kn, dtype=np.int64) * c) // kn
        width = np.diff(np.append(bins, c))
        cols = (bins[None, :] + (rng.random((r, kn)) * width[None, :]).astype(np.int64)).astype(np.uint16)
        deltas = (rng.standard_normal(r * kn, dtype=np.float32) * np.float32(0.002))
        row_ptr = (np.arange(r + 1, dtype=np.uint64) * kn).astype(np.uint32)
        kc = cols.reshape(-1)
    else:
        kc, deltas, row_ptr = np.zeros(0, np.uint16), np.zeros(0, np.float32), np.zeros(r + 1, np.uint32)
    U = S = Vt = None
    if k:
        U = (rng.standard_normal(r * k, dtype=np.float32) * np.float32(0.05)).astype(np.float16).view(np.uint16)
        S = np.sort(rng.random(k, dtype=np.float32))[::-1].copy() * np.float32(0.5)
        Vt = (rng.standard_normal(k * c, dtype=np.float32) * np.float32(0.05)).astype(np.float16).view(np.uint16)
    return HexTensor(rows=r, cols=c, radius=R, k_dim=k, codes=codes, scales=scales, row_ptr=row_ptr,
                     kink_cols=kc, kink_deltas=deltas, U=U, S=S, Vt=Vt)


def random_packed_matrix(rows: int, cols: int, mode: str = "precision", seed: int = 0) -> HexTensor:
    """One format-valid packed matrix of the given shape, drawn as random_packed_model draws its tensors."""
    rng = np.random.default_rng(seed)
    R, _, _ = mode_params(mode, 64)
    scale = np.float16(0.02 * 3.0 / (R * float(FIT))).view(np.uint16)
    n_pts = codebook.num_points(R)
    return _random_hex(rng, lambda n: rng.integers(0, n_pts, n, dtype=np.uint8), rows, cols, mode, scale)


def random_packed_model(cfg: dict, mode: str = "precision", seed: int = 0) -> PackedModel:
    """Format-valid packed tensors of a whole decoder, drawn directly with NumPy (no quantisation).

    Codes are uniform over the radius-8 lattice, scales are the fp16 value the packer gives a
    N(0, 0.02^2) group, U/Vt are small fp16 values, S is positive, and every row carries the mode's
    kink count at distinct ascending columns.  The decode engines do the same work on these bytes
    as on packed weights (no step depends on the values), so this stands in for ``random_model`` at
    shapes where quantising and factorising with NumPy would take many minutes.  Uses no GPU."""
    rng = np.random.default_rng(seed)
    shapes = linear_shapes(cfg)
    hexes: dict[str, HexTensor] = {}
    R, K, _ = mode_params(mode, 64)
    n_pts = codebook.num_points(R)
    scale = np.float16(0.02 * 3.0 / (R * float(FIT))).view(np.uint16)
    # codes: slices of one 64 MiB pool of uniform codes at random offsets (drawing gigabytes one by one
    # with NumPy's generator would take most of a minute)
    pool = rng.integers(0, n_pts, 1 << 26, dtype=np.uint8)

    def draw(n):
        out, i, off = np.empty(n, np.uint8), 0, int(rng.integers(0, pool.size))
        while i < n:
            m = min(n - i, pool.size - off)
            out[i:i + m] = pool[off:off + m]
            i, off = i + m, 0
        return out
    for name in hex_names(cfg["n_layers"]):
        key = name.split(".")[-2]
        r, c = shapes[key] if key in shapes else (cfg["vocab_size"], cfg["hidden_size"])
        hexes[name] = _random_hex(rng, draw, r, c, mode, scale)
    H = cfg["hidden_size"]
    dense = {"token_embd.weight":
             (rng.standard_normal((cfg["vocab_size"], H), dtype=np.float32) * np.float32(0.02)).astype(np.float16),
             "output_norm.weight": np.ones(H, np.float32)}
    for l in range(cfg["n_layers"]):
        dense[f"blk.{l}.attn_norm.weight"] = np.ones(H, np.float32)
        dense[f"blk.{l}.ffn_norm.weight"] = np.ones(H, np.float32)
    return PackedModel(config=cfg, hex=hexes, dense=dense, avg_bpw=compute_avg_bpw(hexes), mode=mode,
                       extra={"packer": {"name": "gsdlq_b200.packer.random_packed_model", "seed": seed}})


__all__ = ["pack_matrix", "quantize_lattice", "dequant", "random_model", "random_packed_model", "random_packed_matrix",
           "make_config",
           "CONFIGS", "MODES", "LINEAR_NAMES", "linear_shapes"]


# ---------------------------------------------------------------------------------------
# CUDA packer: the same lattice step on the GPU (bit-identical codes/scales/residual,
# gsdlq_pack_lattice), low-rank factors and kinks with torch linear algebra.  Used for
# the large benchmark shapes, where the NumPy packer would take minutes.
def lowrank_factors_torch(resid, K: int):
    """Rank-K factors of a float32 [rows, cols] tensor by torch.svd_lowrank (q = K + 8, two power
    iterations): U fp16 [rows, K], S fp32 [K], Vt fp16 [K, cols].  A matrix with fewer than K
    components gets zero columns / entries / rows for the rest, so the sizes match the declared k_dim."""
    import torch
    rows, cols = resid.shape
    u, s, v = torch.svd_lowrank(resid, q=min(K + 8, rows, cols), niter=2)
    kk = min(K, u.shape[1])
    Uh = resid.new_zeros((rows, K), dtype=torch.float16)
    Uh[:, :kk] = u[:, :kk].half()
    S = resid.new_zeros(K, dtype=torch.float32)
    S[:kk] = s[:kk].float()
    Vh = resid.new_zeros((K, cols), dtype=torch.float16)
    Vh[:kk] = v[:, :kk].T.half()
    return Uh, S, Vh


def pack_matrix_cuda(w, mode: str = "precision", radius: int | None = None, k_dim: int | None = None,
                     kinks_per_row: int | None = None, seed: int = 0):
    """Pack a float32 [rows, cols] CUDA tensor; returns an ``ops.DeviceHex``."""
    import torch
    from . import ops
    rows, cols = w.shape
    R, K, KN = mode_params(mode, cols)
    R = R if radius is None else radius
    K = K if k_dim is None else k_dim
    KN = KN if kinks_per_row is None else kinks_per_row
    dev = w.device
    codes = torch.empty(rows * cols // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(rows * cols // 64, dtype=torch.int16, device=dev)
    resid = torch.empty_like(w)
    ops.pack_lattice(w, R, codes, scales, resid)
    U = S = Vt = None
    if K > 0:
        gen_state = torch.cuda.get_rng_state(dev)
        torch.manual_seed(seed)
        Uh, S, Vh = lowrank_factors_torch(resid, K)
        torch.cuda.set_rng_state(gen_state, dev)
        resid -= (Uh.float() * S[None, :]) @ Vh.float()
        U, Vt = Uh.view(torch.int16).reshape(-1), Vh.view(torch.int16).reshape(-1)
    if KN > 0:
        n = min(KN, cols)
        _, idx = resid.abs().topk(n, dim=1, sorted=False)
        idx, _ = idx.sort(dim=1)
        deltas = resid.gather(1, idx).contiguous().reshape(-1)
        kc = idx.to(torch.int32).to(torch.int16).reshape(-1).contiguous()  # u16 bits (cols <= 65535)
        row_ptr = (torch.arange(rows + 1, device=dev, dtype=torch.int64) * n).to(torch.int32)
        nnz = rows * n
    else:
        kc = deltas = None
        row_ptr = torch.zeros(rows + 1, dtype=torch.int32, device=dev)
        nnz = 0
    del resid
    return ops.DeviceHex(None, rows=rows, cols=cols, k_dim=K, radius=R, codes=codes, scales=scales, row_ptr=row_ptr,
                         kink_cols=kc, kink_deltas=deltas, U=U, S=S, Vt=Vt, nnz=nnz)


def device_hex_to_host(h) -> HexTensor:
    """Copy a DeviceHex back into a NumPy HexTensor (reference-format arrays)."""
    def arr(t, dt):
        return np.zeros(0, dt) if t is None else t.detach().cpu().contiguous().view(-1).numpy().view(dt).copy()
    return HexTensor(rows=h.rows, cols=h.cols, radius=h.radius, k_dim=h.k_dim,
                     codes=arr(h.codes, np.uint8), scales=arr(h.scales, np.uint16),
                     row_ptr=arr(h.row_ptr, np.uint32), kink_cols=arr(h.kink_cols, np.uint16),
                     kink_deltas=arr(h.kink_deltas, np.float32),
                     U=arr(h.U, np.uint16) if h.k_dim else None, S=arr(h.S, np.float32) if h.k_dim else None,
                     Vt=arr(h.Vt, np.uint16) if h.k_dim else None)


def random_model_cuda(cfg: dict, mode: str = "precision", seed: int = 0, std: float = 0.02, device="cuda",
                      norm_jitter: float = 0.0, progress=None):
    """Random-init N(0, std^2) decoder packed on the GPU; returns a ``model.DevicePacked``."""
    import torch
    from .model import DevicePacked
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    shapes = linear_shapes(cfg)
    hexes = {}
    nbytes = nweights = 0
    for i, name in enumerate(hex_names(cfg["n_layers"])):
        key = name.split(".")[-2]
        r, c = shapes[key] if key in shapes else (cfg["vocab_size"], cfg["hidden_size"])
        w = torch.randn((r, c), generator=g, device=dev, dtype=torch.float32).mul_(std)
        h = pack_matrix_cuda(w, mode, seed=seed + i)
        del w
        hexes[name] = h
        nbytes += h.nbytes()
        nweights += r * c
        if progress:
            progress(name)
    H = cfg["hidden_size"]
    dense = {"token_embd.weight": torch.randn((cfg["vocab_size"], H), generator=g, device=dev).mul_(std).half()}

    def norm():
        v = torch.ones(H, device=dev, dtype=torch.float32)
        if norm_jitter:
            v += norm_jitter * torch.randn(H, generator=g, device=dev)
        return v
    dense["output_norm.weight"] = norm()
    for l in range(cfg["n_layers"]):
        dense[f"blk.{l}.attn_norm.weight"] = norm()
        dense[f"blk.{l}.ffn_norm.weight"] = norm()
    torch.cuda.synchronize(dev)
    return DevicePacked(config=cfg, hexes=hexes, dense=dense, avg_bpw=8.0 * nbytes / nweights, mode=mode)


def device_model_to_host(dm) -> PackedModel:
    """Host (NumPy) copy of a DevicePacked model, in the .gsd2 reference format."""
    hexes = {n: device_hex_to_host(h) for n, h in dm.hexes.items()}
    dense = {}
    for n, t in dm.dense.items():
        a = t.detach().cpu().numpy()
        dense[n] = a.astype(np.float16) if n == "token_embd.weight" else a.astype(np.float32)
    return PackedModel(config=dm.config, hex=hexes, dense=dense, avg_bpw=dm.avg_bpw, mode=dm.mode)

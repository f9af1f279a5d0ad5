"""Kernel parity on the GPU: every C-ABI entry point against the CPU oracle.

Tolerances: bit-exact for dequant, codes/scales, RoPE/KV fp16 stores, argmax and
vec_add; matvec within 1e-3 relative (observed ~1e-5);
fp32 reductions (RMSNorm, low-rank, attention) within 1e-5 relative.
"""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

MATVEC_TOL = 1e-3


def rel_err(y, yr):
    """Mixed error: max |y - yr| / (|yr| + rms(yr)) -- relative for large entries, absolute (in units of
    the rms) for entries near zero, where a plain relative error is undefined."""
    y, yr = np.asarray(y, np.float64), np.asarray(yr, np.float64)
    scale = np.abs(yr) + np.sqrt(np.mean(yr ** 2)) + 1e-30
    return float(np.max(np.abs(y - yr) / scale))


def plain_rel_err(y, yr):
    """Plain relative error max |y - yr| / |yr| over the entries with |yr| above the rms of yr."""
    y, yr = np.asarray(y, np.float64), np.asarray(yr, np.float64)
    big = np.abs(yr) > np.sqrt(np.mean(yr ** 2))
    if not big.any():
        return 0.0
    return float(np.max(np.abs(y[big] - yr[big]) / np.abs(yr[big])))


def matvec_err(y, yr):
    """The matvec bar: both the mixed error and the plain relative error of the large entries."""
    return max(rel_err(y, yr), plain_rel_err(y, yr))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


@pytest.fixture(scope="module")
def env(cuda_lib):
    import gsdlq_b200.ops as ops
    import gsdlq_b200._lib as L
    L.device_flags()  # clear
    return ops, L


def rand_hex(rng, rows, cols, k=16, nnz=4, radius=8):
    import gsdlq_b200.codebook as cb
    import gsdlq_b200.gsd2 as G
    n_pts = cb.num_points(radius)
    t = G.HexTensor(
        rows=rows, cols=cols, radius=radius, k_dim=k,
        codes=rng.integers(0, n_pts, rows * cols // 2, dtype=np.uint8),
        scales=(rng.random(rows * cols // 64, dtype=np.float32) * 0.01 + 1e-3).astype(np.float16).view(np.uint16),
        row_ptr=(np.arange(rows + 1) * nnz).astype(np.uint32),
        kink_cols=np.sort(rng.integers(0, cols, (rows, nnz)), axis=1).astype(np.uint16).reshape(-1),
        kink_deltas=(rng.standard_normal(rows * nnz) * 0.01).astype(np.float32),
        U=(rng.standard_normal(rows * k) * 0.05).astype(np.float16).view(np.uint16) if k else None,
        S=rng.random(k, dtype=np.float32) if k else None,
        Vt=(rng.standard_normal(k * cols) * 0.05).astype(np.float16).view(np.uint16) if k else None)
    t.validate()
    return t


def oracle_rec(t):
    import oracle
    tabs = {r: oracle.codebook(r) for r in (6, 8)}
    return oracle.hex_record({"radius": t.radius, "k_dim": t.k_dim, "rows": t.rows, "cols": t.cols},
                             {k: v.tobytes() for k, v in t.blobs().items()}, tabs)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("radius,rows,cols", [(8, 32, 128), (6, 100, 4096), (8, 1024, 4096)])
def test_dequant_bitexact(env, restated, rng, radius, rows, cols):
    ops, L = env
    t = rand_hex(rng, rows, cols, k=0, nnz=0, radius=radius)
    h = ops.DeviceHex(t)
    import gsdlq_b200.codebook as cb
    xy = dev(cb.xy_table(radius))
    w = torch.empty(rows, cols, device="cuda")
    ops.dequant(h, xy, w)
    W = np.zeros((rows, cols), np.float32)
    restated.lib.orc_dequant(_p(t.codes), _p(t.scales), _p(cb.xy_table(radius)), _p(W), rows, cols)
    assert np.array_equal(w.cpu().numpy(), W)


def test_dequant_bitexact_golden(env):
    """The GPU W equals the reference NumPy path's W (golden) bit for bit."""
    import os
    from conftest import GOLDEN
    import gsdlq_b200.gsd2 as G
    import gsdlq_b200.codebook as cb
    ops, L = env
    m = G.read_gsd2(os.path.join(GOLDEN, "tiny_precision.gsd2"))
    t = m.hex["blk.0.attn_q.weight"]
    g = np.load(os.path.join(GOLDEN, "tiny_precision_ref.npz"))
    w = torch.empty(t.rows, t.cols, device="cuda")
    ops.dequant(ops.DeviceHex(t), dev(cb.xy_table(t.radius)), w)
    assert np.array_equal(w.cpu().numpy(), g["W_q"])


@pytest.mark.parametrize("rows,cols,k,nnz,radius", [
    (16, 64, 0, 0, 8), (33, 128, 16, 4, 8), (64, 256, 8, 1, 6), (4096, 4096, 16, 16, 8),
    (1024, 4096, 0, 0, 8), (4096, 14336, 16, 56, 8), (256, 1536, 16, 6, 6)])
def test_hex2d_matvec_dropin(env, restated, rng, rows, cols, k, nnz, radius):
    ops, L = env
    import gsdlq_b200.codebook as cb
    t = rand_hex(rng, rows, cols, k=k, nnz=nnz, radius=radius)
    rec = oracle_rec(t)
    x = rng.standard_normal(cols).astype(np.float32)
    tk_host = np.zeros(16, np.float32)
    yr = restated.matvec(x, rec, tk_host)
    h = ops.DeviceHex(t)
    xd, y, tk = dev(x), torch.zeros(rows, device="cuda"), torch.zeros(16, device="cuda")
    if k:
        ops.lowrank_proj(xd, h, tk)
    ops.hex2d_matvec(xd, h, dev(cb.xy_table(radius)), tk, y)
    torch.cuda.synchronize()
    if k:
        assert rel_err(tk.cpu().numpy()[:k], tk_host[:k]) < 1e-5
    assert matvec_err(y.cpu().numpy(), yr) < MATVEC_TOL
    assert L.device_flags() == 0


def test_matvec_linearity_fullsize(env, rng):
    """Size-independent property at the 4096x32768 LM-head shape: W(ax+by) = aWx + bWy."""
    ops, L = env
    import gsdlq_b200.codebook as cb
    t = rand_hex(rng, 32768, 4096, k=16, nnz=16)
    h = ops.DeviceHex(t)
    xy = dev(cb.xy_table(8))
    x1 = torch.randn(4096, device="cuda")
    x2 = torch.randn(4096, device="cuda")
    outs = []
    for x in (x1, x2, 2.0 * x1 - 3.0 * x2):
        tk, y = torch.zeros(16, device="cuda"), torch.zeros(32768, device="cuda")
        ops.lowrank_proj(x, h, tk)
        ops.hex2d_matvec(x, h, xy, tk, y)
        outs.append(y)
    comb = 2.0 * outs[0] - 3.0 * outs[1]
    assert rel_err(outs[2].cpu().numpy(), comb.cpu().numpy()) < 1e-4


def test_elementwise(env, restated, rng):
    ops, L = env
    n = 4096 + 37
    x = rng.standard_normal(n).astype(np.float32) * 3
    w = rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, device="cuda")
    ops.rmsnorm(dev(x), dev(w), out, 1e-5)
    r = np.zeros(n, np.float32)
    restated.rmsnorm(_p(x), _p(w), _p(r), n, 1e-5)
    assert rel_err(out.cpu().numpy(), r) < 1e-5
    ops.vec_add(out, dev(x), dev(w))
    restated.vec_add(_p(r), _p(x), _p(w), n)
    assert np.array_equal(out.cpu().numpy(), r)
    g = dev(x)
    ops.swiglu(g, dev(w), g)  # out aliases gate, as the reference runtime calls it
    restated.swiglu(_p(x), _p(w), _p(r), n)
    assert rel_err(g.cpu().numpy(), r) < 1e-5


@pytest.mark.parametrize("interleaved", [1, 0])
@pytest.mark.parametrize("nh,nkv,hd", [(32, 8, 128), (12, 2, 128), (8, 8, 64)])
def test_rope_store_bitexact(env, restated, rng, interleaved, nh, nkv, hd):
    ops, L = env
    Lc, S = 2, 64
    kc = np.zeros((Lc, S, nkv, hd), np.uint16)
    vc = np.zeros_like(kc)
    kd = torch.zeros((Lc, S, nkv, hd), dtype=torch.int16, device="cuda")
    vd = torch.zeros_like(kd)
    for pos in (0, 1, 17, 63):
        q = rng.standard_normal(nh * hd).astype(np.float32)
        k = rng.standard_normal(nkv * hd).astype(np.float32)
        v = rng.standard_normal(nkv * hd).astype(np.float32)
        qd = dev(q)
        ops.rope_and_store_kv(qd, dev(k), dev(v), kd, vd, 1, pos, nh, nkv, hd, S, 1e6, interleaved)
        restated.rope_and_store_kv(_p(q), _p(k), _p(v), _p(kc), _p(vc), 1, pos, nh, nkv, hd, S, 1e6, interleaved)
        assert np.array_equal(qd.cpu().numpy(), q)
    assert np.array_equal(kd.cpu().numpy().view(np.uint16), kc)
    assert np.array_equal(vd.cpu().numpy().view(np.uint16), vc)


@pytest.mark.parametrize("nh,nkv,hd,S", [(32, 8, 128, 2048), (12, 2, 128, 2048), (32, 32, 64, 256), (4, 4, 128, 100),
                                         (64, 8, 128, 4096), (8, 4, 32, 300), (16, 2, 64, 1000)])
def test_gqa_attention(env, restated, rng, nh, nkv, hd, S):
    ops, L = env
    Lc = 2
    kc = (rng.standard_normal((Lc, S, nkv, hd)) * 2).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((Lc, S, nkv, hd)).astype(np.float16).view(np.uint16)
    kd, vd = dev(kc.view(np.int16)), dev(vc.view(np.int16))
    for pos in sorted({0, 1, 63, 64, 65, S // 2, S - 1}):
        q = rng.standard_normal(nh * hd).astype(np.float32)
        o = torch.zeros(nh * hd, device="cuda")
        ops.gqa_attention(dev(q), kd, vd, o, 1, pos, nh, nkv, hd, S, 1 / math.sqrt(hd))
        r = np.zeros(nh * hd, np.float32)
        restated.gqa_attention(_p(q), _p(kc), _p(vc), _p(r), 1, pos, nh, nkv, hd, S, 1 / math.sqrt(hd))
        assert rel_err(o.cpu().numpy(), r) < 1e-5, pos


@pytest.mark.parametrize("nh,nkv,hd,S,page,fk", [(32, 8, 128, 2048, 16, 16), (12, 2, 128, 700, 64, 40),
                                                  (16, 16, 64, 512, 32, 0)])
def test_attention_job_paged_and_forward(env, restated, rng, nh, nkv, hd, S, page, fk):
    """gsdlq_attention over a paged cache (shuffled block table) against the oracle on the same rows
    laid out contiguously, and the low-rank forward sum_c Vt[j][c] * out[c] it adds (2^-32 fixed point)."""
    ops, L = env
    kc = (rng.standard_normal((1, S, nkv, hd)) * 2).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((1, S, nkv, hd)).astype(np.float16).view(np.uint16)
    n_pages = (S + page - 1) // page
    perm = rng.permutation(n_pages + 3)[:n_pages].astype(np.int32)
    pool_k = np.zeros((n_pages + 3, page, nkv, hd), np.uint16)
    pool_v = np.zeros_like(pool_k)
    for t in range(S):
        pool_k[perm[t // page], t % page] = kc[0, t]
        pool_v[perm[t // page], t % page] = vc[0, t]
    pk, pv = dev(pool_k.view(np.int16)), dev(pool_v.view(np.int16))
    bt = dev(perm)
    pb, wb = ops.attention_ws_size(nh, nkv, hd, S)
    part = torch.zeros(pb // 4 + 1, device="cuda")
    wsp = torch.zeros(wb // 4 + 1, dtype=torch.int32, device="cuda")
    vt = (rng.standard_normal((max(fk, 1), nh * hd)) * 0.05).astype(np.float16)
    vtd = dev(vt.view(np.int16))
    for pos in sorted({0, 5, page - 1, page, S // 3, S - 1}):
        q = rng.standard_normal(nh * hd).astype(np.float32)
        qd = dev(q)
        o = torch.zeros(nh * hd, device="cuda")
        acc = torch.zeros(max(fk, 1), dtype=torch.int64, device="cuda")
        j = L.AttnJob(q=qd.data_ptr(), k_cache=pk.data_ptr(), v_cache=pv.data_ptr(), out=o.data_ptr(), pos_dev=None,
                      pos_val=pos, layer=0, n_heads=nh, n_kv_heads=nkv, head_dim=hd, max_seq=S,
                      sm_scale=1 / math.sqrt(hd), block_table=bt.data_ptr(), page_size=page,
                      partial=part.data_ptr(), workspace=wsp.data_ptr(),
                      fwd_vt=vtd.data_ptr() if fk else None, fwd_k=fk, fwd_acc=acc.data_ptr() if fk else None)
        ops.attention(j)
        torch.cuda.synchronize()
        r = np.zeros(nh * hd, np.float32)
        restated.gqa_attention(_p(q), _p(kc), _p(vc), _p(r), 0, pos, nh, nkv, hd, S, 1 / math.sqrt(hd))
        got = o.cpu().numpy()
        assert rel_err(got, r) < 1e-5, pos
        if fk:
            want = vt.astype(np.float64) @ r.astype(np.float64)
            fwd = acc.cpu().numpy().astype(np.float64) / 2.0 ** 32
            assert np.max(np.abs(fwd - want)) < 1e-4 * (np.max(np.abs(want)) + 1e-3), pos
        assert int(wsp.abs().sum().item()) == 0


def test_argmax_rules(env, oracle_mod):
    ops, L = env
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    cases = [np.array([1, np.nan, 3, 3, np.inf, -np.inf], np.float32),
             np.array([0.5, 2.0, 2.0, np.nan], np.float32),
             np.random.default_rng(0).standard_normal(151936).astype(np.float32)]
    cases[2][[5, 70000]] = 9.0
    for c in cases:
        ops.argmax(dev(c), out)
        assert int(out.item()) == oracle_mod.argmax(c)


@pytest.mark.parametrize("radius", [6, 8])
def test_pack_lattice_bitexact_vs_numpy(env, radius):
    ops, L = env
    import gsdlq_b200.packer as P
    rng = np.random.default_rng(radius)
    w = (rng.standard_normal((96, 512)) * 0.02).astype(np.float32)
    w[3, :64] = 0.0          # all-zero group
    w[5, 64:128] *= 1000.0   # large group
    codes, sb = P.quantize_lattice(w, radius)
    e = w - P.dequant(codes, sb, radius, 96, 512)
    wd = dev(w)
    c = torch.empty(96 * 256, dtype=torch.uint8, device="cuda")
    s = torch.empty(96 * 8, dtype=torch.int16, device="cuda")
    r = torch.empty_like(wd)
    ops.pack_lattice(wd, radius, c, s, r)
    assert np.array_equal(c.cpu().numpy(), codes)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), sb)
    assert np.array_equal(r.cpu().numpy(), e)


@pytest.mark.skipif(__import__("os").environ.get("GSDLQ_ATTN_CLUSTER") == "0",
                    reason="already running the split/counter attention kernel")
def test_split_counter_attention_in_subprocess(cuda_lib):
    """GSDLQ_ATTN_CLUSTER=0 (read once per process) selects the split/counter attention kernel
    instead of the cluster kernel; the attention parity cases and the golden model pass with it."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, GSDLQ_ATTN_CLUSTER="0")
    cmd = [sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
           os.path.join(here, "test_gpu_kernels.py") + "::test_gqa_attention",
           os.path.join(here, "test_gpu_kernels.py") + "::test_attention_job_paged_and_forward",
           os.path.join(here, "test_gpu_model.py") + "::test_golden_tiny"]
    r = subprocess.run(cmd, env=env, cwd=os.path.dirname(here), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]

"""Pin the oracle: our C restatement vs the reference engine (built from its own
source) and vs golden vectors produced by the reference's Python runtime."""
import ctypes
import os

import numpy as np
import pytest

from conftest import GOLDEN


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _rand_hex(rng, rows, cols, k, nnz_per_row, radius=8):
    import gsdlq_b200.codebook as cb
    n_pts = cb.num_points(radius)
    rec = {
        "rows": rows, "cols": cols, "k_dim": k, "n_pts": n_pts, "xy_table": cb.xy_table(radius),
        "codes": rng.integers(0, n_pts, rows * cols // 2, dtype=np.uint8),
        "scales": (rng.random(rows * cols // 64, dtype=np.float32) * 0.01 + 1e-3).astype(np.float16).view(np.uint16),
        "row_ptr": (np.arange(rows + 1) * nnz_per_row).astype(np.uint32),
        "kink_cols": rng.integers(0, cols, rows * nnz_per_row).astype(np.uint16),
        "kink_deltas": (rng.standard_normal(rows * nnz_per_row) * 0.01).astype(np.float32),
    }
    if k:
        rec["U"] = (rng.standard_normal(rows * k) * 0.05).astype(np.float16).view(np.uint16)
        rec["S"] = rng.random(k, dtype=np.float32)
        rec["Vt"] = (rng.standard_normal(k * cols) * 0.05).astype(np.float16).view(np.uint16)
    else:
        rec["U"] = rec["Vt"] = np.zeros(2, np.uint16)
        rec["S"] = np.zeros(1, np.float32)
    return rec


@pytest.mark.parametrize("rows,cols,k,nnz", [(64, 128, 16, 4), (33, 256, 0, 0), (128, 1024, 8, 3),
                                             (1, 64, 1, 1), (5, 65472, 16, 8)])  # widest row a u16 kink reaches
def test_matvec_restatement_bitexact_vs_reference(restated, reference_engine, rng, rows, cols, k, nnz):
    rec = _rand_hex(rng, rows, cols, k, nnz)
    if nnz:
        rec["kink_cols"][nnz - 1::nnz] = cols - 1  # the last column, in every row
    x = rng.standard_normal(cols).astype(np.float32)
    y1 = restated.matvec(x, rec)
    y2 = reference_engine.matvec(x, rec)
    assert np.array_equal(y1, y2)


def test_matvec_restatement_bitexact_property(restated, reference_engine):
    """Random shapes, both radii, k in [0, 16] and ragged kink rows (unsorted and repeated columns, empty
    rows): the restatement equals the reference engine bit for bit."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    import gsdlq_b200.codebook as cb

    @hyp.settings(max_examples=30, deadline=None, derandomize=True)
    @hyp.given(rows=st.integers(1, 160), g=st.integers(1, 24), k=st.integers(0, 16), radius=st.sampled_from([6, 8]),
               seed=st.integers(0, 2 ** 31 - 1))
    def check(rows, g, k, radius, seed):
        rng = np.random.default_rng(seed)
        cols = 64 * g
        rec = _rand_hex(rng, rows, cols, k, 0, radius=radius)
        counts = rng.integers(0, 5, rows)
        rec["row_ptr"] = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
        nnz = int(counts.sum())
        kc = rng.integers(0, cols, nnz)
        if nnz > 1:
            kc[-1] = kc[0]  # a repeated column
        rec["kink_cols"] = kc.astype(np.uint16)
        rec["kink_deltas"] = (rng.standard_normal(nnz) * 0.01).astype(np.float32)
        assert rec["n_pts"] == cb.num_points(radius)
        x = rng.standard_normal(cols).astype(np.float32)
        assert np.array_equal(restated.matvec(x, rec), reference_engine.matvec(x, rec))

    check()


def test_elementwise_bitexact_vs_reference(restated, reference_engine, rng):
    n = 1000
    x = rng.standard_normal(n).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    outs = []
    for e in (restated, reference_engine):
        o1 = np.zeros(n, np.float32)
        e.rmsnorm(_p(x), _p(w), _p(o1), n, 1e-5)
        o2 = np.zeros(n, np.float32)
        e.vec_add(_p(o2), _p(x), _p(w), n)
        o3 = np.zeros(n, np.float32)
        e.swiglu(_p(x), _p(w), _p(o3), n)
        tk = np.zeros(16, np.float32)
        vt = (rng.standard_normal(16 * n)).astype(np.float16).view(np.uint16) if not outs else outs[0][4]
        s = np.linspace(0.5, 2, 16).astype(np.float32)
        e.lowrank_proj(_p(x), _p(vt), _p(s), _p(tk), 16, n)
        outs.append((o1, o2, o3, tk, vt))
    for a, b in zip(outs[0][:4], outs[1][:4]):
        assert np.array_equal(a, b)


def test_elementwise_bitexact_property(restated, reference_engine):
    """RMSNorm, add, SwiGLU (also in place, out aliasing gate as the reference's caller does) and the
    low-rank projection over random lengths, eps, k and input scales (large gates saturate the sigmoid):
    restatement == reference, bit for bit."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=30, deadline=None, derandomize=True)
    @hyp.given(n=st.integers(1, 5000), k=st.integers(1, 16), eps=st.sampled_from([1e-5, 1e-6, 1e-3]),
               scale=st.sampled_from([1e-3, 1.0, 40.0]), seed=st.integers(0, 2 ** 31 - 1))
    def check(n, k, eps, scale, seed):
        r = np.random.default_rng(seed)
        x = (r.standard_normal(n) * scale).astype(np.float32)
        w = r.standard_normal(n).astype(np.float32)
        vt = r.standard_normal(k * n).astype(np.float16).view(np.uint16)
        sv = r.random(k, dtype=np.float32)
        outs = []
        for e in (restated, reference_engine):
            o1 = np.zeros(n, np.float32)
            e.rmsnorm(_p(x), _p(w), _p(o1), n, eps)
            o2 = np.zeros(n, np.float32)
            e.vec_add(_p(o2), _p(x), _p(w), n)
            o3 = np.zeros(n, np.float32)
            e.swiglu(_p(x), _p(w), _p(o3), n)
            g = x.copy()
            e.swiglu(_p(g), _p(w), _p(g), n)
            tk = np.zeros(16, np.float32)
            e.lowrank_proj(_p(x), _p(vt), _p(sv), _p(tk), k, n)
            outs.append((o1, o2, o3, g, tk))
        for a, b in zip(*outs):
            assert np.array_equal(a, b, equal_nan=True)

    check()


@pytest.mark.parametrize("interleaved", [1, 0])
def test_rope_attention_bitexact_vs_reference(restated, reference_engine, rng, interleaved):
    L, S, nh, nkv, hd = 2, 64, 8, 2, 32
    res = []
    for e in (restated, reference_engine):
        r = np.random.default_rng(5)
        kc = np.zeros((L, S, nkv, hd), np.uint16)
        vc = np.zeros_like(kc)
        outs = []
        for pos in range(20):
            q = r.standard_normal(nh * hd).astype(np.float32)
            k = r.standard_normal(nkv * hd).astype(np.float32)
            v = r.standard_normal(nkv * hd).astype(np.float32)
            e.rope_and_store_kv(_p(q), _p(k), _p(v), _p(kc), _p(vc), 1, pos, nh, nkv, hd, S, 10000.0, interleaved)
            o = np.zeros(nh * hd, np.float32)
            e.gqa_attention(_p(q), _p(kc), _p(vc), _p(o), 1, pos, nh, nkv, hd, S, 1 / np.sqrt(hd))
            outs.append((q.copy(), o))
        res.append((kc, vc, outs))
    assert np.array_equal(res[0][0], res[1][0])
    assert np.array_equal(res[0][1], res[1][1])
    for (q1, o1), (q2, o2) in zip(res[0][2], res[1][2]):
        assert np.array_equal(q1, q2) and np.array_equal(o1, o2)


def test_rope_attention_bitexact_property(restated, reference_engine):
    """RoPE + fp16 KV store and GQA attention over random head sizes, GQA ratios, cache lengths, positions,
    theta and both rotation layouts, on a randomly pre-filled cache: restatement == reference, bit for bit."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=25, deadline=None, derandomize=True)
    @hyp.given(hd=st.sampled_from([32, 64, 128]), nkv=st.sampled_from([1, 2, 4]), grp=st.integers(1, 4),
               S=st.sampled_from([16, 64, 200]), data=st.data(), theta=st.sampled_from([1e4, 5e5, 1e6]),
               interleaved=st.sampled_from([0, 1]), seed=st.integers(0, 2 ** 31 - 1))
    def check(hd, nkv, grp, S, data, theta, interleaved, seed):
        nh, L = nkv * grp, 2
        pos = data.draw(st.integers(0, S - 1))
        r = np.random.default_rng(seed)
        cache0 = r.standard_normal((2, L, S, nkv, hd)).astype(np.float16).view(np.uint16)
        q0 = r.standard_normal(nh * hd).astype(np.float32)
        k = r.standard_normal(nkv * hd).astype(np.float32)
        v = r.standard_normal(nkv * hd).astype(np.float32)
        res = []
        for e in (restated, reference_engine):
            kc, vc, q = cache0[0].copy(), cache0[1].copy(), q0.copy()
            e.rope_and_store_kv(_p(q), _p(k), _p(v), _p(kc), _p(vc), 1, pos, nh, nkv, hd, S, theta, interleaved)
            o = np.zeros(nh * hd, np.float32)
            e.gqa_attention(_p(q), _p(kc), _p(vc), _p(o), 1, pos, nh, nkv, hd, S, 1 / np.sqrt(hd))
            res.append((q, kc, vc, o))
        for a, b in zip(*res):
            assert np.array_equal(a, b)

    check()


@pytest.mark.parametrize("mode", ["precision", "turbo"])
def test_oracle_model_matches_golden(oracle_mod, restated, mode):
    """Our restated reader + decoder step reproduce the reference runtime's logits bit for bit."""
    g = np.load(os.path.join(GOLDEN, f"tiny_{mode}_ref.npz"))
    m = oracle_mod.read_gsd2(os.path.join(GOLDEN, f"tiny_{mode}.gsd2"))
    om = oracle_mod.OracleModel(m, restated)
    for pos, tok in enumerate(g["tokens"]):
        lg = om.forward_token(int(tok), pos)
        assert np.array_equal(lg, g["logits"][pos]), f"pos {pos}"
        assert oracle_mod.argmax(lg) == g["picks"][pos]
    # single matvecs through the C engine path
    x = g["x"]
    for key in ("q", "k", "gate"):
        assert np.array_equal(restated.matvec(x, m["layers"][0][key]), g["mv_" + key])


def test_oracle_dequant_matches_reference_numpy_path(oracle_mod, restated):
    """orc_dequant == the W the reference's NumPy fallback builds (gsd_lq_cpu_runtime.py:281-284)."""
    g = np.load(os.path.join(GOLDEN, "tiny_precision_ref.npz"))
    m = oracle_mod.read_gsd2(os.path.join(GOLDEN, "tiny_precision.gsd2"))
    rec = m["layers"][0]["q"]
    W = np.zeros((rec["rows"], rec["cols"]), np.float32)
    restated.lib.orc_dequant(_p(rec["codes"]), _p(rec["scales"]), _p(rec["xy_table"]), _p(W), rec["rows"],
                             rec["cols"])
    assert np.array_equal(W, g["W_q"])
    assert np.array_equal(oracle_mod.dequant(rec["codes"], rec["scales"], rec["xy_table"], rec["rows"],
                                             rec["cols"]), g["W_q"])


def test_oracle_argmax_rules(restated, oracle_mod):
    x = np.array([1.0, np.nan, 3.0, 3.0, np.inf, -np.inf], np.float32)
    assert oracle_mod.argmax(x) == 4
    assert restated.lib.orc_argmax(_p(x), x.size) == 4
    y = np.array([0.5, 2.0, 2.0, np.nan], np.float32)
    assert oracle_mod.argmax(y) == 1 == restated.lib.orc_argmax(_p(y), y.size)

"""Codebook, .gsd2 reader/writer, packer invariants, format fault injection (CPU)."""
import json
import os
import struct

import numpy as np
import pytest

from conftest import GOLDEN
import gsdlq_b200.codebook as cb
import gsdlq_b200.gsd2 as G
import gsdlq_b200.packer as P


@pytest.mark.parametrize("radius,n", [(6, 127), (8, 217)])
def test_codebook_bitexact_vs_reference_golden(radius, n, oracle_mod):
    g = np.load(os.path.join(GOLDEN, "codebook.npz"))
    t = cb.xy_table(radius)
    assert t.shape == (n, 2) and cb.num_points(radius) == n
    assert np.array_equal(t, g[f"cpu{radius}"]) and np.array_equal(t, g[f"gpu{radius}"])
    assert np.array_equal(oracle_mod.codebook(radius)[0], t)
    rr = cb.lattice_coords(radius).astype(np.float64)
    assert np.array_equal((rr[:, 0] + 0.5 * rr[:, 1]).astype(np.float32), t[:, 0])
    assert np.array_equal((rr[:, 1] * (np.sqrt(3.0) / 2.0)).astype(np.float32), t[:, 1])


def test_codebook_c_restatement(restated):
    import ctypes
    for r in (6, 8):
        buf = np.zeros(2 * 256, np.float32)
        n = restated.lib.orc_codebook(r, buf.ctypes.data_as(ctypes.c_void_p), 256)
        assert np.array_equal(buf[:2 * n].reshape(n, 2), cb.xy_table(r))


def test_reader_matches_oracle_reader(oracle_mod):
    path = os.path.join(GOLDEN, "tiny_precision.gsd2")
    m = G.read_gsd2(path)
    o = oracle_mod.read_gsd2(path)
    assert m.config["n_layers"] == o["cfg"]["n_layers"]
    t = m.hex["blk.1.ffn_down.weight"]
    r = o["layers"][1]["down"]
    for k in ("codes", "scales", "row_ptr", "kink_cols", "kink_deltas", "U", "S", "Vt"):
        assert np.array_equal(getattr(t, k), r[k]), k
    assert np.array_equal(m.dense["token_embd.weight"].astype(np.float32), o["embed"])


def test_roundtrip(tmp_path):
    cfg = P.make_config("tiny", n_layers=1, hidden_size=128, n_heads=2, n_kv_heads=1, head_dim=64,
                        ffn_size=192, vocab_size=64)
    m = P.random_model(cfg, "precision", seed=3)
    p = str(tmp_path / "m.gsd2")
    G.write_gsd2(p, m)
    r = G.read_gsd2(p)
    for n, t in m.hex.items():
        for k, a in t.blobs().items():
            assert np.array_equal(a, getattr(r.hex[n], k)), (n, k)
    # every blob starts on a 256-byte boundary of the file
    with open(p, "rb") as f:
        f.read(4)
        hlen = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(hlen))
    assert (12 + hlen) % 256 == 0
    for meta in hdr["tensors"].values():
        for v in meta.values():
            if isinstance(v, dict) and "offset" in v:
                assert v["offset"] % 256 == 0


def test_packer_invariants_and_determinism():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((48, 256)) * 0.02).astype(np.float32)
    a = P.pack_matrix(w, "precision")
    b = P.pack_matrix(w, "precision")
    for k in ("codes", "scales", "row_ptr", "kink_cols", "kink_deltas"):
        assert np.array_equal(getattr(a, k), getattr(b, k))
    assert a.k_dim == 16 and a.nnz == 48 * 4
    assert np.all(np.diff(a.kink_cols.reshape(48, 4).astype(int), axis=1) > 0)
    # reconstruction error of the lattice part is bounded by the scale (hexagon cell radius 1/sqrt3)
    W = P.dequant(a.codes, a.scales, a.radius, 48, 256)
    s = np.repeat(a.scales.view(np.float16).astype(np.float32).reshape(48, 4), 64, axis=1)
    err = np.hypot(*(w - W).reshape(-1, 2).T)
    assert np.all(err <= s.reshape(-1, 2)[:, 0] * (1 / np.sqrt(3) + 1e-3))
    t = P.pack_matrix(w, "turbo")
    assert t.k_dim == 0 and t.nnz == 0 and t.U is None
    assert abs(G.compute_avg_bpw({"x": t}) - (4.25 + 32 * 49 / (48 * 256))) < 1e-6


def test_packer_nearest_point_is_exact():
    """Every code is a nearest hexagon point of (w0, w1)/scale (brute force over the table)."""
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((8, 128)) * 0.02).astype(np.float32)
    for radius in (6, 8):
        codes, sb = P.quantize_lattice(w, radius)
        s = np.repeat(sb.view(np.float16).astype(np.float32).reshape(8, 2), 32, axis=1).reshape(-1)
        pr = w.reshape(-1, 2) / s[:, None]
        t = cb.xy_table(radius)
        d = ((pr[:, None, :] - t[None]) ** 2).sum(-1)
        best = d.min(1)
        assert np.allclose(d[np.arange(len(codes)), codes], best, rtol=0, atol=1e-5)


# ---- fault injection: malformed files are rejected on the host -------------------------
def _tiny_file(tmp_path):
    cfg = P.make_config("tiny", n_layers=1, hidden_size=64, n_heads=1, n_kv_heads=1, head_dim=64,
                        ffn_size=128, vocab_size=32)
    m = P.random_model(cfg, "turbo", seed=5)
    p = str(tmp_path / "t.gsd2")
    G.write_gsd2(p, m)
    return p


def _rewrite_header(p, fn):
    raw = open(p, "rb").read()
    hlen = struct.unpack("<Q", raw[4:12])[0]
    hdr = json.loads(raw[12:12 + hlen])
    fn(hdr)
    hb = json.dumps(hdr).encode()
    hb += b" " * (hlen - len(hb)) if len(hb) <= hlen else b""
    assert len(hb) == hlen
    open(p, "wb").write(raw[:12] + hb + raw[12 + hlen:])


def test_bad_magic(tmp_path):
    p = _tiny_file(tmp_path)
    raw = bytearray(open(p, "rb").read())
    raw[:4] = b"GSD1"
    open(p, "wb").write(bytes(raw))
    with pytest.raises(G.FormatError, match="magic"):
        G.read_gsd2(p)


def test_truncated_file(tmp_path):
    p = _tiny_file(tmp_path)
    raw = open(p, "rb").read()
    open(p, "wb").write(raw[:len(raw) - 1000])
    with pytest.raises(G.FormatError, match="past the end"):
        G.read_gsd2(p)


def test_header_length_overflow(tmp_path):
    p = _tiny_file(tmp_path)
    raw = bytearray(open(p, "rb").read())
    raw[4:12] = struct.pack("<Q", 1 << 40)
    open(p, "wb").write(bytes(raw))
    with pytest.raises(G.FormatError, match="exceeds"):
        G.read_gsd2(p)


def test_out_of_range_code_rejected(tmp_path):
    p = _tiny_file(tmp_path)
    m = G.read_gsd2(p)
    raw = bytearray(open(p, "rb").read())
    hlen = struct.unpack("<Q", raw[4:12])[0]
    hdr = json.loads(raw[12:12 + hlen])
    off = 12 + hlen + hdr["tensors"]["blk.0.attn_q.weight"]["codes"]["offset"]
    raw[off + 5] = 250  # >= 217 points of radius 8
    open(p, "wb").write(bytes(raw))
    with pytest.raises(G.FormatError, match="code index"):
        G.read_gsd2(p)
    assert m is not None


@pytest.mark.parametrize("mutate,msg", [
    (lambda h: h["tensors"]["blk.0.attn_q.weight"].__setitem__("k_dim", 17), "k_dim"),
    (lambda h: h["tensors"]["blk.0.attn_q.weight"].__setitem__("radius", 7), "radius"),
    (lambda h: h["tensors"]["blk.0.attn_q.weight"].__setitem__("cols", 96), "multiple of 64"),
    (lambda h: h["config"].__setitem__("n_kv_heads", 3), "multiple of n_kv_heads"),
    (lambda h: h["tensors"].pop("blk.0.ffn_up.weight"), "missing tensor"),
    (lambda h: h["config"].__setitem__("n_kv_heads", 0), "positive integer"),
    (lambda h: h["config"].__setitem__("n_layers", "1"), "positive integer"),
    (lambda h: h["config"].__setitem__("head_dim", 64.0), "positive integer"),
    (lambda h: h["config"].__setitem__("rms_eps", -1e-5), "positive finite"),
    (lambda h: h["config"].__setitem__("rope_theta", None), "positive finite"),
    (lambda h: h.__setitem__("config", [1, 2]), "JSON object"),
    (lambda h: h.__setitem__("alignment", 96), "power of two"),
    (lambda h: h["tensors"].__setitem__("output_norm.weight", {"x": 1}), "data descriptor"),
    (lambda h: h["tensors"].__setitem__("blk.0.attn_k.weight", 7), "JSON objects"),
    (lambda h: h["tensors"]["blk.0.attn_q.weight"]["codes"].__setitem__("offset", 0.5), "malformed"),
    (lambda h: h["tensors"]["blk.0.attn_q.weight"]["scales"].__setitem__("nbytes", True), "malformed"),
    (lambda h: h["tensors"]["blk.0.attn_q.weight"]["codes"].__setitem__(
        "offset", h["tensors"]["blk.0.attn_q.weight"]["codes"]["offset"] + 4), "alignment"),
    (lambda h: h["tensors"]["token_embd.weight"]["data"].__setitem__("shape", [32, -64]), "list of sizes"),
])
def test_header_violations(tmp_path, mutate, msg):
    p = _tiny_file(tmp_path)
    _rewrite_header(p, mutate)
    with pytest.raises(G.FormatError, match=msg):
        G.read_gsd2(p)


def test_header_not_an_object(tmp_path):
    p = _tiny_file(tmp_path)
    raw = open(p, "rb").read()
    hlen = struct.unpack("<Q", raw[4:12])[0]
    open(p, "wb").write(raw[:12] + b"[]".ljust(hlen) + raw[12 + hlen:])
    with pytest.raises(G.FormatError, match="JSON object"):
        G.read_gsd2(p)


def _poke(p, tensor, blob, index, value):
    """Overwrite element ``index`` of one blob in place (``value`` a numpy scalar of the blob's type)."""
    raw = bytearray(open(p, "rb").read())
    hlen = struct.unpack("<Q", raw[4:12])[0]
    meta = json.loads(raw[12:12 + hlen])["tensors"][tensor][blob]
    b = np.asarray(value).tobytes()
    off = 12 + hlen + meta["offset"] + index * len(b)
    raw[off:off + len(b)] = b
    open(p, "wb").write(bytes(raw))


@pytest.mark.parametrize("tensor,blob,value", [
    ("blk.0.ffn_down.weight", "scales", np.uint16(0x7C00)),      # fp16 +inf
    ("blk.0.attn_v.weight", "scales", np.uint16(0xFE01)),        # fp16 NaN
    ("output_norm.weight", "data", np.float32(np.nan)),
    ("token_embd.weight", "data", np.float16(np.inf)),
])
def test_non_finite_values_rejected(tmp_path, tensor, blob, value):
    p = _tiny_file(tmp_path)
    _poke(p, tensor, blob, 3, value)
    with pytest.raises(G.FormatError, match="non-finite"):
        G.read_gsd2(p)
    G.read_gsd2(p, check_values=False)  # the structure is intact: only the value check objects


def test_non_finite_low_rank_and_kinks_rejected(tmp_path):
    cfg = P.make_config("tiny", n_layers=1, hidden_size=64, n_heads=1, n_kv_heads=1, head_dim=64,
                        ffn_size=128, vocab_size=32)
    for blob, value in (("S", np.float32(np.inf)), ("kink_deltas", np.float32(np.nan)),
                        ("U", np.uint16(0x7C00)), ("Vt", np.uint16(0xFC00))):
        p = str(tmp_path / f"{blob}.gsd2")
        G.write_gsd2(p, P.random_model(cfg, "precision", seed=6))
        _poke(p, "blk.0.ffn_gate.weight", blob, 1, value)
        with pytest.raises(G.FormatError, match=f"{blob}: non-finite"):
            G.read_gsd2(p)


def test_unaligned_reference_layout_reads(tmp_path):
    """A file laid out like the reference's writer (blobs back to back, no ``alignment`` key) reads the
    same tensors as the aligned file it was made from."""
    p = _tiny_file(tmp_path)
    raw = open(p, "rb").read()
    hlen = struct.unpack("<Q", raw[4:12])[0]
    hdr = json.loads(raw[12:12 + hlen])
    body = bytearray()
    for meta in hdr["tensors"].values():
        for v in meta.values():
            if isinstance(v, dict) and "offset" in v:
                src = 12 + hlen + v["offset"]
                body += raw[src:src + v["nbytes"]]
                v["offset"] = len(body) - v["nbytes"]
    hdr.pop("alignment")
    hb = json.dumps(hdr).encode()
    q = str(tmp_path / "packed.gsd2")
    open(q, "wb").write(G.MAGIC + struct.pack("<Q", len(hb)) + hb + bytes(body))
    assert (12 + len(hb)) % 4 or any(
        v["offset"] % 256 for m in hdr["tensors"].values() for v in m.values() if isinstance(v, dict) and "offset" in v)
    a, b = G.read_gsd2(p), G.read_gsd2(q)
    for n, t in a.hex.items():
        for k, x in t.blobs().items():
            assert np.array_equal(x, getattr(b.hex[n], k)), (n, k)
    for n, x in a.dense.items():
        assert np.array_equal(x, b.dense[n]), n
    # writing what was read restores the aligned layout
    r = str(tmp_path / "rewritten.gsd2")
    G.write_gsd2(r, b)
    G.read_gsd2(r)


def test_kink_invariants():
    t = P.pack_matrix((np.random.default_rng(2).standard_normal((16, 128)) * 0.02).astype(np.float32),
                      "precision")
    bad = G.HexTensor(**{**t.__dict__, "row_ptr": t.row_ptr[::-1].copy()})
    with pytest.raises(G.FormatError, match="row_ptr"):
        bad.validate()
    kc = t.kink_cols.copy()
    kc[0] = 200
    with pytest.raises(G.FormatError, match="kink column"):
        G.HexTensor(**{**t.__dict__, "kink_cols": kc}).validate()


def test_shard_slices_sum_to_whole():
    """Row shards concatenate and column shards sum (oracle numerics) to the unsharded matvec."""
    import oracle
    eng = oracle.CEngine.restatement()
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    t = P.pack_matrix(w, "precision")
    x = rng.standard_normal(256).astype(np.float32)
    tabs = {r: oracle.codebook(r) for r in (6, 8)}
    rec = lambda h: oracle.hex_record({"radius": h.radius, "k_dim": h.k_dim, "rows": h.rows, "cols": h.cols},  # noqa
                                      {k: v.tobytes() for k, v in h.blobs().items()}, tabs)
    full = eng.matvec(x, rec(t))
    rows = np.concatenate([eng.matvec(x, rec(t.row_slice(a, a + 16))) for a in range(0, 64, 16)])
    assert np.array_equal(rows, full)
    cols = sum(eng.matvec(x[a:a + 128], rec(t.col_slice(a, a + 128))) for a in (0, 128))
    assert np.allclose(cols, full, rtol=1e-5, atol=1e-6)


def test_slices_compose_and_sum_property():
    """Property check of the shard slicers over random shapes and cut points: every slice validates,
    slices of slices equal direct slices, and column slices at any 64-column cuts sum to the whole."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    import oracle
    eng = oracle.CEngine.restatement()
    tabs = {r: oracle.codebook(r) for r in (6, 8)}

    def rec(h):
        return oracle.hex_record({"radius": h.radius, "k_dim": h.k_dim, "rows": h.rows, "cols": h.cols},
                                 {k: v.tobytes() for k, v in h.blobs().items()}, tabs)

    def same(a, b):
        return all(np.array_equal(x, y) for x, y in zip(a.blobs().values(), b.blobs().values())) and \
            (a.rows, a.cols, a.nnz) == (b.rows, b.cols, b.nnz)

    @hyp.settings(max_examples=25, deadline=None, derandomize=True)
    @hyp.given(rows=st.integers(1, 40), g=st.integers(2, 6), mode=st.sampled_from(["precision", "turbo"]),
               data=st.data())
    def check(rows, g, mode, data):
        cols = 64 * g
        rng = np.random.default_rng(rows * 131 + g)
        t = P.pack_matrix((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32), mode)
        a = data.draw(st.integers(0, rows - 1))
        b = data.draw(st.integers(a + 1, rows))
        c = data.draw(st.integers(0, b - a - 1))
        d = data.draw(st.integers(c + 1, b - a))
        rs = t.row_slice(a, b)
        rs.validate()
        assert same(rs.row_slice(c, d), t.row_slice(a + c, a + d))
        cuts = sorted(set([0, cols] + [64 * data.draw(st.integers(1, g - 1)) for _ in range(2)]))
        parts = [t.col_slice(lo, hi) for lo, hi in zip(cuts, cuts[1:])]
        for p in parts:
            p.validate()
        assert sum(p.nnz for p in parts) == t.nnz
        x = rng.standard_normal(cols).astype(np.float32)
        full = eng.matvec(x, rec(t))
        tot = sum(eng.matvec(x[lo:hi].copy(), rec(p)) for (lo, hi), p in zip(zip(cuts, cuts[1:]), parts))
        assert np.allclose(tot, full, rtol=1e-5, atol=1e-5)

    check()


def test_lowrank_factors_torch_pad_and_match():
    """The GPU packer's factor step on CPU tensors: full-rank shapes equal torch.svd_lowrank's leading K
    components; a matrix with fewer than K components gets zero padding up to k_dim."""
    torch = pytest.importorskip("torch")
    g = torch.Generator().manual_seed(4)
    a = torch.randn(64, 128, generator=g) * 0.02
    torch.manual_seed(1)
    Uh, S, Vh = P.lowrank_factors_torch(a, 16)
    torch.manual_seed(1)
    u, s, v = torch.svd_lowrank(a, q=24, niter=2)
    assert torch.equal(Uh, u[:, :16].half()) and torch.equal(S, s[:16].float()) and torch.equal(Vh, v[:, :16].T.half())
    small = torch.randn(5, 128, generator=g)
    Uh, S, Vh = P.lowrank_factors_torch(small, 16)
    assert Uh.shape == (5, 16) and S.shape == (16,) and Vh.shape == (16, 128)
    assert not Uh[:, 5:].any() and not S[5:].any() and not Vh[5:].any()
    rec = (Uh.float() * S[None, :]) @ Vh.float()
    assert torch.allclose(rec, small, atol=2e-2 * float(small.abs().max()))


def test_packer_small_matrix_keeps_k_dim():
    """A Precision matrix with fewer rows than k keeps k_dim = 16 with zero-padded factors."""
    w = (np.random.default_rng(2).standard_normal((3, 128)) * 0.02).astype(np.float32)
    t = P.pack_matrix(w, "precision")
    t.validate()
    assert t.k_dim == 16 and t.U.size == 3 * 16 and t.Vt.size == 16 * 128
    assert not t.S[3:].any()


def test_gsd2_roundtrip_property(tmp_path):
    """Random small configurations (GQA ratios, head sizes, FFN and vocabulary sizes, both modes) survive
    write -> read byte for byte, and the oracle's own reader (a restatement of the reference's) agrees."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    import oracle
    counter = iter(range(10 ** 6))
    seen = []

    @hyp.settings(max_examples=12, deadline=None, derandomize=True)
    @hyp.given(hd=st.sampled_from([32, 64]), nkv=st.integers(1, 3), grp=st.integers(1, 3), fg=st.integers(1, 4),
               vocab=st.integers(40, 200), mode=st.sampled_from(["precision", "turbo"]), layers=st.integers(1, 2))
    def check(hd, nkv, grp, fg, vocab, mode, layers):
        nh = nkv * grp
        if (nh * hd) % 64:
            hd = 64  # hidden = n_heads * head_dim is the column count of q/k/v/gate/up: a multiple of 64
        cfg = P.make_config("tiny", n_layers=layers, hidden_size=nh * hd, n_heads=nh, n_kv_heads=nkv, head_dim=hd,
                            ffn_size=64 * fg, vocab_size=vocab)
        seen.append((nh, nkv, hd, 64 * fg, vocab, mode, layers))
        m = P.random_model(cfg, mode, seed=next(counter))
        p = str(tmp_path / f"r{next(counter)}.gsd2")
        G.write_gsd2(p, m)
        r = G.read_gsd2(p)
        assert r.config["n_layers"] == layers and r.mode == m.mode
        for n, t in m.hex.items():
            for k, a in t.blobs().items():
                assert np.array_equal(a, getattr(r.hex[n], k)), (n, k)
        for n, a in m.dense.items():
            assert np.array_equal(np.asarray(a), np.asarray(r.dense[n])), n
        o = oracle.read_gsd2(p)
        lay = o["layers"][layers - 1]["down"]
        t = m.hex[f"blk.{layers - 1}.ffn_down.weight"]
        for k in ("codes", "scales", "row_ptr", "kink_cols", "kink_deltas"):
            assert np.array_equal(getattr(t, k), lay[k]), k

    check()
    assert len(set(seen)) >= 8, seen


def test_arena_alignment_and_upload_from_mmap(tmp_path):
    """The device arena (here on CPU tensors) takes every blob of a memory-mapped .gsd2 straight from the
    mapped pages, each at a 256-byte-aligned address, byte for byte; overflow is an error, not a wrap."""
    import warnings
    import torch
    from gsdlq_b200.ops import Arena
    cfg = P.make_config("tiny", n_layers=1, hidden_size=128, n_heads=2, n_kv_heads=1, head_dim=64,
                        ffn_size=192, vocab_size=64)
    p = str(tmp_path / "m.gsd2")
    G.write_gsd2(p, P.random_model(cfg, "precision", seed=4))
    r = G.read_gsd2(p, mmap=True)
    blobs = [a for t in r.hex.values() for a in t.blobs().values()]
    assert any(isinstance(a, np.memmap) or isinstance(getattr(a, "base", None), np.memmap) for a in blobs)
    ar = Arena(Arena.bytes_needed(blobs), device="cpu")
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", UserWarning)  # torch notes that mapped pages are read-only
        outs = [ar.put(a) for a in blobs]
    for a, d in zip(blobs, outs):
        if a.nbytes:
            assert d.data_ptr() % Arena.ALIGN == 0
        assert np.array_equal(d.numpy(), np.ascontiguousarray(a).reshape(-1).view(np.uint8))
    with pytest.raises(MemoryError):
        ar.put(np.zeros(Arena.ALIGN + 1, np.uint8))
    assert torch.is_tensor(outs[0])


def test_arena_places_mapped_blobs_on_256_byte_boundaries():
    """The upload arena copies read-only memory-mapped blobs as they are, each at a 256-byte-aligned offset
    (checked here on a host arena: the placement logic is the same for a device one)."""
    import warnings
    import gsdlq_b200.ops as ops
    m = G.read_gsd2(os.path.join(GOLDEN, "tiny_precision.gsd2"))
    blobs = [a for t in list(m.hex.values())[:3] for a in t.blobs().values()]
    assert not blobs[0].flags.writeable
    ar = ops.Arena(ops.Arena.bytes_needed(blobs), "cpu")
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        views = [ar.put(a) for a in blobs]
    for a, v in zip(blobs, views):
        assert v.data_ptr() % 256 == 0
        assert np.array_equal(v.numpy(), np.ascontiguousarray(a).reshape(-1).view(np.uint8))
    with pytest.raises(MemoryError):
        ar.put(np.zeros(512, np.uint8))


@pytest.mark.parametrize("mode", ["precision", "turbo"])
def test_bench_generator_round_trip(tmp_path, mode):
    """The bench's weight generator (random_packed_model) writes files the hardened reader accepts with every
    check on, blob for blob; layout keys carried over from a read file never override the written layout."""
    cfg = P.make_config("tiny")
    m = P.random_packed_model(cfg, mode, seed=4)
    m.extra = {"alignment": 512, "format_version": 1, "note": "kept"}
    p = str(tmp_path / "g.gsd2")
    G.write_gsd2(p, m)
    r = G.read_gsd2(p, check_codes=True, check_values=True)
    assert r.extra["alignment"] == 256 and r.extra["format_version"] == 2 and r.extra["note"] == "kept"
    assert r.mode == mode
    for n, t in m.hex.items():
        for k, a in t.blobs().items():
            assert np.array_equal(a, getattr(r.hex[n], k)), (n, k)
    for n, a in m.dense.items():
        assert np.array_equal(np.asarray(a).reshape(-1), r.dense[n].reshape(-1)), n

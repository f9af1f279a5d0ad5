"""Tensor-parallel host logic on CPU: world_size-2 gloo ranks run the engine's TP
dataflow (sharded packed linears, residual all-reduce after O and down, vocab-parallel
head with the 64-bit MAX-key greedy pick) through the oracle C engine, and must match
the unsharded oracle forward.  Also a rank that dies is noticed by its peer through
a short process-group timeout instead of a hang."""
import ctypes
import os
import socket

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

TOKENS = [1, 17, 300, 42, 255]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _tp_forward(rank, world, path, tokens):
    """The engine's TP step, with oracle arithmetic, on this rank's shard."""
    import sys
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import torch
    import torch.distributed as dist
    import oracle
    import gsdlq_b200.gsd2 as G
    import gsdlq_b200.tp as TP
    eng = oracle.CEngine.restatement()
    full = G.read_gsd2(path)
    sh = TP.shard_packed(full, rank, world)
    c = sh.config
    tabs = {r: oracle.codebook(r) for r in (6, 8)}

    def rec(t):
        return oracle.hex_record({"radius": t.radius, "k_dim": t.k_dim, "rows": t.rows, "cols": t.cols},
                                 {k: np.ascontiguousarray(v).tobytes() for k, v in t.blobs().items()}, tabs)
    H, hd, S = c["hidden_size"], c["head_dim"], 64
    nh, nkv, vl = c["n_heads_local"], c["n_kv_heads_local"], c["vocab_size_local"]
    kc = np.zeros((c["n_layers"], S, nkv, hd), np.uint16)
    vc = np.zeros_like(kc)
    embed = full.dense["token_embd.weight"].astype(np.float32)
    out = []
    for pos, tok in enumerate(tokens):
        x = embed[tok].copy()
        for l in range(c["n_layers"]):
            p = f"blk.{l}."
            xb = np.zeros(H, np.float32)
            eng.rmsnorm(_p(x), _p(full.dense[p + "attn_norm.weight"]), _p(xb), H, float(c["rms_eps"]))
            q = eng.matvec(xb, rec(sh.hex[p + "attn_q.weight"]))
            k = eng.matvec(xb, rec(sh.hex[p + "attn_k.weight"]))
            v = eng.matvec(xb, rec(sh.hex[p + "attn_v.weight"]))
            eng.rope_and_store_kv(_p(q), _p(k), _p(v), _p(kc), _p(vc), l, pos, nh, nkv, hd, S,
                                  float(c["rope_theta"]), 1)
            att = np.zeros(nh * hd, np.float32)
            eng.gqa_attention(_p(q), _p(kc), _p(vc), _p(att), l, pos, nh, nkv, hd, S, 1.0 / np.sqrt(hd))
            part = eng.matvec(att, rec(sh.hex[p + "attn_output.weight"]))
            y = torch.from_numpy(x + part if rank == 0 else part)
            dist.all_reduce(y)
            x = y.numpy().copy()
            eng.rmsnorm(_p(x), _p(full.dense[p + "ffn_norm.weight"]), _p(xb), H, float(c["rms_eps"]))
            g = eng.matvec(xb, rec(sh.hex[p + "ffn_gate.weight"]))
            u = eng.matvec(xb, rec(sh.hex[p + "ffn_up.weight"]))
            h = np.zeros_like(g)
            eng.swiglu(_p(g), _p(u), _p(h), g.size)
            part = eng.matvec(h, rec(sh.hex[p + "ffn_down.weight"]))
            y = torch.from_numpy(x + part if rank == 0 else part)
            dist.all_reduce(y)
            x = y.numpy().copy()
        xb = np.zeros(H, np.float32)
        eng.rmsnorm(_p(x), _p(full.dense["output_norm.weight"]), _p(xb), H, float(c["rms_eps"]))
        lg = eng.matvec(xb, rec(sh.hex["output.weight"]))
        # 64-bit greedy key: (ordered value, ~global index), MSB flipped for a signed MAX all-reduce
        i = int(np.argmax(lg))
        b = int(np.float32(lg[i]).view(np.uint32))
        ordered = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
        key = (ordered << 32) | (0xFFFFFFFF - (i + rank * vl))
        kt = torch.tensor([key ^ (1 << 63)], dtype=torch.uint64).view(torch.int64)
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
        pick = 0xFFFFFFFF - ((int(kt.item()) ^ -(1 << 63)) & 0xFFFFFFFF)
        parts = [torch.empty(vl) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(lg))
        out.append((torch.cat(parts).numpy(), pick))
    return out


def _worker(rank, world, port, path, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = _tp_forward(rank, world, path, TOKENS)
        if rank == 0:
            q.put([(lg, pk) for lg, pk in res])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["precision", "turbo"])
def test_tp2_matches_unsharded(oracle_mod, restated, mode):
    import torch.multiprocessing as mp
    path = os.path.join(GOLDEN, f"tiny_{mode}.gsd2")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    om = oracle_mod.OracleModel(oracle_mod.read_gsd2(path), restated, max_seq=64)
    g = np.load(os.path.join(GOLDEN, f"tiny_{mode}_ref.npz"))
    for pos, tok in enumerate(TOKENS):
        full = om.forward_token(tok, pos)
        lg, pick = res[pos]
        assert np.allclose(lg, full, rtol=1e-4, atol=1e-5), float(np.max(np.abs(lg - full)))
        assert pick == oracle_mod.argmax(full) == int(g["picks"][pos])


def _dying_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        dist.all_reduce(t)
        q.put("no-error")
    except Exception as e:  # the survivor's next collective ends with an error, not a hang
        q.put(type(e).__name__)


def test_peer_death_is_detected():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
    assert msg != "no-error"


def test_tp4_matches_unsharded(oracle_mod, restated, tmp_path):
    """Four gloo ranks on a model that shards four ways: 2 of 8 query heads and 1 of 4 KV heads per
    rank, O and down cut into 64- and 128-column slices, an 80-row vocabulary slice each."""
    import torch.multiprocessing as mp
    import gsdlq_b200.gsd2 as G
    import gsdlq_b200.packer as P
    cfg = P.make_config("tiny", n_layers=2, hidden_size=256, n_heads=8, n_kv_heads=4, head_dim=32,
                        ffn_size=512, vocab_size=320)
    path = str(tmp_path / "tp4_precision.gsd2")
    G.write_gsd2(path, P.random_model(cfg, "precision", seed=5, norm_jitter=0.1))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 4, port, path, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    om = oracle_mod.OracleModel(oracle_mod.read_gsd2(path), restated, max_seq=64)
    for pos, tok in enumerate(TOKENS):
        full = om.forward_token(tok, pos)
        lg, pick = res[pos]
        assert np.allclose(lg, full, rtol=1e-4, atol=1e-5), float(np.max(np.abs(lg - full)))
        assert pick == oracle_mod.argmax(full)


def _typed_device_hex(t):
    """A DeviceHex on CPU tensors with the GPU packer's dtypes (pack_matrix_cuda)."""
    import torch
    from gsdlq_b200.ops import DeviceHex

    def T(a, dt):
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(dt).copy())
    k, nz = t.k_dim, t.nnz
    return DeviceHex(None, rows=t.rows, cols=t.cols, k_dim=k, radius=t.radius, codes=T(t.codes, np.uint8),
                     scales=T(t.scales, np.int16), row_ptr=T(t.row_ptr, np.int32),
                     kink_cols=T(t.kink_cols, np.int16) if nz else None,
                     kink_deltas=T(t.kink_deltas, np.float32) if nz else None,
                     U=T(t.U, np.int16) if k else None, S=T(t.S, np.float32) if k else None,
                     Vt=T(t.Vt, np.int16) if k else None, nnz=nz)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("mode", ["precision", "turbo"])
def test_device_shards_equal_host_shards(world, mode):
    """tp.shard_device (the slicer of GPU-packed models that bench.py and GSDLQModel(tp=...) use) gives
    the same bytes as the host shard_packed checked above, on CPU tensors: codes and scales per row,
    kinks filtered and re-based by column range, Vt sliced by columns, U / S kept whole."""
    import gsdlq_b200.packer as P
    import gsdlq_b200.tp as TP
    from gsdlq_b200.model import DevicePacked
    cfg = P.make_config("tiny", n_layers=1, hidden_size=256, n_heads=8, n_kv_heads=4, head_dim=32,
                        ffn_size=512, vocab_size=320)
    pm = P.random_model(cfg, mode, seed=9)
    dm = DevicePacked(config=cfg, hexes={n: _typed_device_hex(t) for n, t in pm.hex.items()}, dense=pm.dense,
                      avg_bpw=pm.avg_bpw, mode=mode)
    for rank in range(world):
        host = TP.shard_packed(pm, rank, world)
        dev = TP.shard_device(dm, rank, world)
        assert dev.config == host.config
        for name, t in host.hex.items():
            d = P.device_hex_to_host(dev.hexes[name])
            assert (d.rows, d.cols, d.k_dim, d.radius, d.nnz) == (t.rows, t.cols, t.k_dim, t.radius, t.nnz), name
            for key, arr in t.blobs().items():
                got = np.ascontiguousarray(d.blobs()[key]).reshape(-1).view(np.uint8)
                want = np.ascontiguousarray(arr).reshape(-1).view(np.uint8)
                assert np.array_equal(got, want), (name, key, rank)


@pytest.mark.parametrize("model,world,ok", [
    ("mistral-7b", 2, True), ("mistral-7b", 8, True), ("mistral-7b", 3, False),
    ("qwen2.5-1.5b", 2, True), ("qwen2.5-1.5b", 4, False),      # 2 kv heads
    ("smollm2-1.7b", 8, True),
])
def test_tp_shape_checks(model, world, ok):
    """Tensor-parallel sharding refuses configurations whose heads, FFN or vocabulary do not split evenly,
    or whose row-parallel shards are not whole 64-column scale groups, before anything is sliced."""
    import gsdlq_b200.packer as P
    import gsdlq_b200.tp as T
    cfg = P.make_config(model)
    if ok:
        T.check_divisible(cfg, world)
        loc = T.local_config(cfg, world)
        assert loc["n_heads_local"] * world == cfg["n_heads"] and loc["ffn_size_local"] * world == cfg["ffn_size"]
    else:
        with pytest.raises(ValueError, match="divisible"):
            T.check_divisible(cfg, world)
    small = P.make_config("tiny", n_heads=2, n_kv_heads=2, head_dim=64, ffn_size=192, vocab_size=64)
    with pytest.raises(ValueError, match="multiples of 64"):
        T.check_divisible(small, 2)   # 192 / 2 = 96 FFN columns per rank

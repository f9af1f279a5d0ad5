"""Tensor parallelism for the packed decoder (one process per GPU, NCCL over NVLink).

Sharding (Megatron style; the reference has no multi-device code at all):

  * column-parallel  attn_q / attn_k / attn_v (by heads), ffn_gate / ffn_up (by rows):
      rows are cut; codes, scales, U and the CSR kinks follow their rows; Vt and S
      stay whole, so every rank computes the full low-rank projection of its input.
  * row-parallel     attn_output (by the rank's heads), ffn_down (by ffn columns):
      columns are cut in multiples of 64; codes/scales are cut per row, kinks are
      filtered to the column range, Vt is cut by columns and U/S stay whole, so
      the ranks' partial outputs -- U S (Vt_r x_r) included -- sum to the full one.
  * vocab-parallel   output.weight rows; greedy pick = all-reduce MAX of a 64-bit
      (value, ~global index) key, so ties still go to the lowest index.

Per layer there are two all-reduces of the hidden-size fp32 residual: rank 0's
O/down epilogue adds its partial to the residual, the other ranks store their bare
partials into the same buffer, and one all-reduce(sum) leaves x + sum_r partial_r
on every rank.  The all-reduce is the library's one-shot exchange over peer memory
(gsdlq_comm_allreduce_sum; rank-ordered sums, so every rank holds the same bits), or
NCCL's with exchange="nccl".
"""
from __future__ import annotations

import numpy as np

from .gsd2 import HexTensor, PackedModel

COLUMN = ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up")
ROW = ("attn_output", "ffn_down")


def check_divisible(cfg: dict, world: int) -> None:
    for k in ("n_heads", "n_kv_heads", "ffn_size", "vocab_size"):
        if cfg[k] % world:
            raise ValueError(f"{k}={cfg[k]} is not divisible by world size {world}")
    if (cfg["ffn_size"] // world) % 64 or (cfg["n_heads"] * cfg["head_dim"] // world) % 64:
        raise ValueError("row-parallel shards must be multiples of 64 columns")


def local_config(cfg: dict, world: int) -> dict:
    c = dict(cfg)
    c["n_heads_local"] = cfg["n_heads"] // world
    c["n_kv_heads_local"] = cfg["n_kv_heads"] // world
    c["ffn_size_local"] = cfg["ffn_size"] // world
    c["vocab_size_local"] = cfg["vocab_size"] // world
    c["tp_world"] = world
    return c


def shard_ranges(cfg: dict, name: str, rank: int, world: int) -> tuple[str, int, int]:
    """('rows'|'cols', start, stop) of rank's shard of linear ``name``."""
    hd = cfg["head_dim"]
    if name in ("attn_q",):
        n = cfg["n_heads"] * hd // world
        return "rows", rank * n, (rank + 1) * n
    if name in ("attn_k", "attn_v"):
        n = cfg["n_kv_heads"] * hd // world
        return "rows", rank * n, (rank + 1) * n
    if name in ("ffn_gate", "ffn_up"):
        n = cfg["ffn_size"] // world
        return "rows", rank * n, (rank + 1) * n
    if name == "attn_output":
        n = cfg["n_heads"] * hd // world
        return "cols", rank * n, (rank + 1) * n
    if name == "ffn_down":
        n = cfg["ffn_size"] // world
        return "cols", rank * n, (rank + 1) * n
    if name == "output":
        n = cfg["vocab_size"] // world
        return "rows", rank * n, (rank + 1) * n
    raise KeyError(name)


def shard_packed(pm: PackedModel, rank: int, world: int) -> PackedModel:
    """Host (NumPy) shard of a packed model for ``rank``."""
    cfg = pm.config
    check_divisible(cfg, world)
    hexes = {}
    for full, t in pm.hex.items():
        kind, a, b = shard_ranges(cfg, full.split(".")[-2], rank, world)
        hexes[full] = t.row_slice(a, b) if kind == "rows" else t.col_slice(a, b)
    return PackedModel(config=local_config(cfg, world), hex=hexes, dense=pm.dense, avg_bpw=pm.avg_bpw,
                       mode=pm.mode, extra=dict(pm.extra))


# ---- device (torch) shards of GPU-packed tensors ---------------------------------------------
def _row_slice_dev(h, r0: int, r1: int):
    import torch
    from .ops import DeviceHex
    c, k = h.cols, h.k_dim
    rp = h.row_ptr.view(torch.int32).long()
    a, b = int(rp[r0].item()), int(rp[r1].item())
    row_ptr = (rp[r0:r1 + 1] - a).to(torch.int32).contiguous()
    nnz = b - a
    return DeviceHex(None, rows=r1 - r0, cols=c, k_dim=k, radius=h.radius,
                     codes=h.codes[r0 * c // 2:r1 * c // 2].contiguous(),
                     scales=h.scales[r0 * c // 64:r1 * c // 64].contiguous(),
                     row_ptr=row_ptr,
                     kink_cols=h.kink_cols[a:b].contiguous() if nnz else None,
                     kink_deltas=h.kink_deltas[a:b].contiguous() if nnz else None,
                     U=h.U[r0 * k:r1 * k].contiguous() if k else None,
                     S=h.S.clone() if k else None, Vt=h.Vt.clone() if k else None, nnz=nnz)


def _col_slice_dev(h, c0: int, c1: int):
    import torch
    from .ops import DeviceHex
    r, c, k = h.rows, h.cols, h.k_dim
    codes = h.codes.view(r, c // 2)[:, c0 // 2:c1 // 2].contiguous().view(-1)
    scales = h.scales.view(r, c // 64)[:, c0 // 64:c1 // 64].contiguous().view(-1)
    kc = kd = None
    rp_new = torch.zeros(r + 1, dtype=torch.int32, device=h.codes.device)
    nnz = 0
    if h.kink_cols is not None and h.kink_cols.numel():
        cols = h.kink_cols.view(torch.int16).to(torch.int32) & 0xFFFF
        rp = h.row_ptr.view(torch.int32).long()
        rows_of = torch.repeat_interleave(torch.arange(r, device=cols.device), rp[1:] - rp[:-1])
        keep = (cols >= c0) & (cols < c1)
        counts = torch.bincount(rows_of[keep], minlength=r)
        rp_new[1:] = torch.cumsum(counts, 0).to(torch.int32)
        kc = (cols[keep] - c0).to(torch.int16).contiguous()
        kd = h.kink_deltas[keep].contiguous()
        nnz = int(kc.numel())
        if nnz == 0:
            kc = kd = None
    Vt = None
    if k:
        Vt = h.Vt.view(k, c)[:, c0:c1].contiguous().view(-1)
    return DeviceHex(None, rows=r, cols=c1 - c0, k_dim=k, radius=h.radius, codes=codes, scales=scales,
                     row_ptr=rp_new, kink_cols=kc, kink_deltas=kd,
                     U=h.U.clone() if k else None, S=h.S.clone() if k else None, Vt=Vt, nnz=nnz)


def shard_device(dm, rank: int, world: int):
    """Device shard of a DevicePacked model (GPU packer output) for ``rank``."""
    from .model import DevicePacked
    cfg = dm.config
    check_divisible(cfg, world)
    hexes = {}
    for full, h in dm.hexes.items():
        kind, a, b = shard_ranges(cfg, full.split(".")[-2], rank, world)
        hexes[full] = _row_slice_dev(h, a, b) if kind == "rows" else _col_slice_dev(h, a, b)
    return DevicePacked(config=local_config(cfg, world), hexes=hexes, dense=dm.dense, avg_bpw=dm.avg_bpw,
                        mode=dm.mode)


class TensorParallel:
    """Collective plumbing for GSDLQModel(tp=...) over an initialised torch.distributed group.

    ``exchange`` picks the path of the per-layer residual all-reduce and of the greedy-key maximum:
    "p2p" (default; GSDLQ_TP_EXCHANGE overrides) is the library's one-shot exchange over CUDA-IPC
    mapped peer buffers (gsdlq_comm_*), "nccl" is torch.distributed.all_reduce.  torch.distributed
    is used in both cases for the rendezvous (the IPC handles are all-gathered over it)."""

    def __init__(self, rank: int, world: int, group=None, exchange: str | None = None):
        import os
        self.rank, self.world, self.group = rank, world, group
        self.exchange = exchange or os.environ.get("GSDLQ_TP_EXCHANGE", "p2p")
        if self.exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange {self.exchange!r}: use 'p2p' or 'nccl'")
        self.comm = None

    @property
    def fused_epilogue(self) -> bool:
        """True when the O and down launches sum the ranks' partials themselves (p2p exchange, unless
        GSDLQ_TP_FUSED=0 asks for separate all-reduce launches)."""
        import os
        return self.comm is not None and os.environ.get("GSDLQ_TP_FUSED", "1") != "0"

    def setup(self, model):
        """Create and connect this rank's exchange buffer (p2p), sized for the hidden vector."""
        if self.exchange != "p2p" or self.comm is not None:
            return
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _lib as L
        lib = L.load()
        comm = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * L.IPC_HANDLE_BYTES)()
        L.check(lib.gsdlq_comm_create(self.world, self.rank, model.hidden, ctypes.byref(comm), handle),
                "gsdlq_comm_create")
        mine = torch.tensor(bytearray(handle), dtype=torch.uint8, device=model.device)
        every = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(every, mine, group=self.group)
        handles = bytes(torch.cat(every).cpu().numpy().tobytes())
        buf = (ctypes.c_uint8 * len(handles)).from_buffer_copy(handles)
        L.check(lib.gsdlq_comm_connect(comm, buf), "gsdlq_comm_connect")
        self.comm = comm
        dist.barrier(group=self.group)

    def close(self):
        if self.comm is not None:
            from . import _lib as L
            L.check(L.load().gsdlq_comm_destroy(self.comm), "gsdlq_comm_destroy")
            self.comm = None

    def shard(self, src):
        from .model import DevicePacked
        if isinstance(src, DevicePacked):
            return shard_device(src, self.rank, self.world)
        return shard_packed(src, self.rank, self.world)

    def vocab_base(self, model) -> int:
        return self.rank * model.vocab_local

    # called inside the captured layer step
    def allreduce(self, model, which: str):
        self.allreduce_buf(model.x)

    def allreduce_buf(self, buf):
        """Sum of ``buf`` over the ranks, in place (the residual exchange of one O or down projection)."""
        if self.comm is not None:
            from . import _lib as L
            from .ops import stream_handle
            L.check(L.load().gsdlq_comm_allreduce_sum(self.comm, buf.data_ptr(), buf.numel(), stream_handle()),
                    "gsdlq_comm_allreduce_sum")
            return
        import torch.distributed as dist
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)

    def key_max(self, key):
        """Maximum over the ranks of the unsigned 64-bit key ``key[0]``, in place."""
        if self.comm is not None:
            from . import _lib as L
            from .ops import stream_handle
            L.check(L.load().gsdlq_comm_allreduce_max_u64(self.comm, key.data_ptr(), stream_handle()),
                    "gsdlq_comm_allreduce_max_u64")
            return
        import torch.distributed as dist
        k = key[:1]
        k.bitwise_xor_(-(1 << 63))  # MSB flipped so that signed order = unsigned order
        dist.all_reduce(k, op=dist.ReduceOp.MAX, group=self.group)
        k.bitwise_xor_(-(1 << 63))

    def finish_head(self, model):
        """Global greedy pick: the maximum over ranks of the 64-bit (value, ~global index) keys."""
        self.key_max(model.key)

    def gather_logits(self, model) -> np.ndarray:
        import torch
        import torch.distributed as dist
        parts = [torch.empty_like(model.logits) for _ in range(self.world)]
        dist.all_gather(parts, model.logits, group=self.group)
        return torch.cat(parts).cpu().numpy()

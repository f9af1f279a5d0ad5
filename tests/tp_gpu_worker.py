"""One rank of the tensor-parallel GPU parity check (launched by tests/test_gpu_tp.py under torchrun).

Every rank packs the same 2-layer Mistral-7B-shape Precision model on its GPU (same seed; a digest of
the packed bytes is compared across ranks first), then runs

  * GSDLQModel(tp=TensorParallel) -- the sharded CUDA path: column/row/vocab shards, the EPI_STORE /
    EPI_RESID split of the residual, the argmax index base and the in-kernel low-rank projection of
    column shards, with an all-reduce after O and down;
  * GSDLQModel() unsharded on the same rank;
  * on rank 0, the oracle decoder over the same packed bytes (the reference C engine when built).

through a 24-token prompt and 16 greedy steps (every rank feeds the oracle's pick, broadcast from
rank 0), comparing gathered TP logits with the unsharded and oracle logits, and then the device-side
greedy loop (generate) of both models.  Rank 0 writes the results as JSON to $TP_RESULT.
"""
import datetime
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def digest(dm) -> int:
    h = hashlib.sha256()
    for n in sorted(dm.hexes):
        d = dm.hexes[n]
        for t in (d.codes, d.scales, d.U, d.S, d.Vt, d.row_ptr, d.kink_cols, d.kink_deltas):
            if t is not None:
                h.update(t.detach().cpu().numpy().tobytes())
    for n in sorted(dm.dense):
        h.update(dm.dense[n].detach().cpu().numpy().tobytes())
    return int.from_bytes(h.digest()[:7], "little")


def main():
    world, rank, local = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=90), device_id=dev)
    import gsdlq_b200.packer as P
    import gsdlq_b200._lib as L
    from gsdlq_b200.model import GSDLQModel
    from gsdlq_b200.tp import TensorParallel
    from conftest import oracle_decoder, top2_margin, NEAR_TIE
    import oracle

    cfg = P.make_config("mistral-7b", n_layers=2)
    dm = P.random_model_cuda(cfg, "precision", seed=31, norm_jitter=0.1, device=dev)
    dg = torch.tensor([digest(dm)], dtype=torch.int64, device=dev)
    all_dg = [torch.zeros_like(dg) for _ in range(world)]
    dist.all_gather(all_dg, dg)
    same_bytes = len({int(t.item()) for t in all_dg}) == 1
    host = P.device_model_to_host(dm) if rank == 0 else None
    m1 = GSDLQModel(dm, device=dev, max_seq=256)
    mt = GSDLQModel(dm, device=dev, max_seq=256, tp=TensorParallel(rank, world))
    del dm
    om = oracle_decoder(host, max_seq=256) if rank == 0 else None

    prompt = np.random.default_rng(32).integers(0, cfg["vocab_size"], 24).tolist()
    res = {"world": world, "same_bytes": same_bytes, "tp_vs_1": 0.0, "tp_vs_oracle": 0.0, "one_vs_oracle": 0.0,
           "pick_mismatch_tp_1": 0, "ties": [], "bad_picks": []}
    lt = l1 = lr = None
    for pos, t in enumerate(prompt):
        last = pos == len(prompt) - 1
        lt = mt.forward_token(t, pos, return_logits=last)
        l1 = m1.forward_token(t, pos, return_logits=last)
        if rank == 0:
            lr = om.forward_token(t, pos, return_logits=last)
    tok = torch.zeros(1, dtype=torch.int64, device=dev)
    for i in range(17):
        pos = len(prompt) + i
        if rank == 0:
            res["tp_vs_1"] = max(res["tp_vs_1"], float(np.max(np.abs(lt - l1))))
            res["tp_vs_oracle"] = max(res["tp_vs_oracle"], float(np.max(np.abs(lt - lr))))
            res["one_vs_oracle"] = max(res["one_vs_oracle"], float(np.max(np.abs(l1 - lr))))
            a, a1, b = mt.sample_token(lt), m1.sample_token(l1), oracle.argmax(lr)
            res["pick_mismatch_tp_1"] += int(a != a1)
            if a != b:
                mg = top2_margin(lr)
                (res["ties"] if mg < NEAR_TIE else res["bad_picks"]).append((i, a, b, mg))
            tok.fill_(b)
        if i == 16:
            break
        dist.broadcast(tok, 0)
        nxt = int(tok.item())
        lt = mt.forward_token(nxt, pos)
        l1 = m1.forward_token(nxt, pos)
        if rank == 0:
            lr = om.forward_token(nxt, pos)
    # the device-side greedy loop, sharded and unsharded, from the same prompt
    gt = mt.generate(prompt[:20], 12)
    g1 = m1.generate(prompt[:20], 12)
    gids = torch.tensor(gt, dtype=torch.int64, device=dev)
    all_g = [torch.zeros_like(gids) for _ in range(world)]
    dist.all_gather(all_g, gids)
    res["generate_tp"] = gt
    res["generate_1"] = g1
    res["generate_same_on_ranks"] = all(torch.equal(all_g[0], g) for g in all_g)
    flags = L.device_flags()
    fl = torch.tensor([flags], dtype=torch.int64, device=dev)
    dist.all_reduce(fl, op=dist.ReduceOp.MAX)
    res["device_flags"] = int(fl.item())
    mt.release()
    m1.release()
    if rank == 0:
        with open(os.environ["TP_RESULT"], "w") as f:
            json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Tensor parallelism on GPUs: GSDLQModel(tp=N) against the unsharded model and the oracle.

Launches tests/tp_gpu_worker.py under torchrun on N GPUs of this node (skipped when fewer are
present), once with the library's peer-memory exchange (gsdlq_comm_*) and once with NCCL's
all-reduce.  Bars: gathered TP logits within 1e-2 max-abs of the unsharded GPU model's and of the
oracle's, greedy picks identical to the oracle's except at recorded near-ties, and the device-side
greedy loop producing the same ids sharded and unsharded, on every rank.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "tp_gpu_worker.py")
LOGIT_TOL = 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
@pytest.mark.parametrize("world", [2, 4])
def test_tp_logits_and_picks_match_single_gpu_and_oracle(world, exchange, tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "tp.json"
    env = dict(os.environ, TP_RESULT=str(out), NCCL_NVLS_ENABLE="0", GSDLQ_TP_EXCHANGE=exchange)
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), WORKER]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=700)
    assert r.returncode == 0, (r.stdout[-4000:], r.stderr[-4000:])
    res = json.loads(out.read_text())
    print(f"\nTP={world} ({exchange}): max|dlogit| tp-vs-1 {res['tp_vs_1']:.3e}, tp-vs-oracle {res['tp_vs_oracle']:.3e}, "
          f"1-vs-oracle {res['one_vs_oracle']:.3e}, near-ties {res['ties']}")
    assert res["same_bytes"], "ranks packed different bytes"
    assert res["tp_vs_1"] < LOGIT_TOL and res["tp_vs_oracle"] < LOGIT_TOL, res
    assert not res["bad_picks"], res["bad_picks"]
    assert res["generate_same_on_ranks"], res
    assert res["generate_tp"] == res["generate_1"], res
    assert res["device_flags"] == 0, res

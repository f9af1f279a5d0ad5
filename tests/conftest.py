"""Shared test setup.

Markers: ``gpu`` -- needs a CUDA device (B200); everything else runs on CPU.
The oracle (oracle/) is imported here only as the checker.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def restated(oracle_mod):
    return oracle_mod.CEngine.restatement()


@pytest.fixture(scope="session")
def reference_engine(oracle_mod):
    eng = oracle_mod.CEngine.reference()
    if eng is None:
        pytest.skip("reference C engine not built here (oracle/_ref missing)")
    return eng


@pytest.fixture(scope="session")
def cuda_lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gsdlq_b200 import _lib
    return _lib.load()


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def oracle_decoder(host, engine=None, max_seq=2048):
    """The oracle decoder (CPUMistralV2Model.forward_token restated, oracle/oracle.py) over a host
    PackedModel's bytes, driven by ``engine`` (default: the reference's own C engine when it was
    built here, else the C restatement)."""
    import oracle
    if engine is None:
        engine = oracle.CEngine.reference() or oracle.CEngine.restatement()
    tabs = {r: oracle.codebook(r) for r in (6, 8)}

    def rec(t):
        return oracle.hex_record({"radius": t.radius, "k_dim": t.k_dim, "rows": t.rows, "cols": t.cols},
                                 {k: np.ascontiguousarray(v).tobytes() for k, v in t.blobs().items()}, tabs)
    cfg = host.config
    m = {"cfg": cfg, "embed": host.dense["token_embd.weight"].astype(np.float32),
         "final_norm": host.dense["output_norm.weight"], "layers": []}
    for l in range(cfg["n_layers"]):
        lyr = {"attn_norm": host.dense[f"blk.{l}.attn_norm.weight"], "ffn_norm": host.dense[f"blk.{l}.ffn_norm.weight"]}
        for n, k in zip(oracle.LINEARS, oracle.KEYS):
            lyr[k] = rec(host.hex[f"blk.{l}.{n}.weight"])
        m["layers"].append(lyr)
    m["lm_head"] = rec(host.hex["output.weight"])
    return oracle.OracleModel(m, engine, max_seq=max_seq)


def top2_margin(logits) -> float:
    """Top-1 minus top-2 of the reference's sanitised logits (how close a greedy pick was to a tie)."""
    z = np.nan_to_num(np.asarray(logits, np.float32), nan=-1e4, posinf=100.0, neginf=-1e4)
    a = np.partition(z, -2)[-2:]
    return float(a[1] - a[0])


NEAR_TIE = 1e-3  # a top-1/top-2 margin below this is a near-tie: the two engines may pick differently


def greedy_parity(model, om, prompt, steps, logit_tol=1e-2):
    """Greedy decode of ``prompt`` then ``steps`` tokens on the GPU model and the oracle decoder.

    Every step compares the logits (max-abs) and the greedy picks.  A differing pick fails unless the
    oracle's top-1/top-2 margin is below NEAR_TIE; such a near-tie is recorded with its margin and
    both engines continue from the oracle's pick (so the rest of the run stays comparable).
    Returns {"worst": max-abs logit difference, "ties": [(step, margin)], "min_margin": ...}."""
    lg = lr = None
    for pos, t in enumerate(prompt):
        last = pos == len(prompt) - 1
        lg = model.forward_token(int(t), pos, return_logits=last)
        lr = om.forward_token(int(t), pos, return_logits=last)
    return greedy_continue(model, om, lg, lr, len(prompt), steps, logit_tol)


def greedy_continue(model, om, lg, lr, pos0, steps, logit_tol=1e-2):
    """The decode part of greedy_parity, from logits ``lg`` (GPU) and ``lr`` (oracle) at position pos0 - 1."""
    import oracle
    worst, ties, min_margin = 0.0, [], float("inf")
    for i in range(steps):
        worst = max(worst, float(np.max(np.abs(lg - lr))))
        a, b = model.sample_token(lg), oracle.argmax(lr)
        margin = top2_margin(lr)
        min_margin = min(min_margin, margin)
        if a != b:
            assert margin < NEAR_TIE, f"greedy picks differ at step {i} ({a} vs {b}) with margin {margin:.3e}"
            ties.append((i, margin))
        lg = model.forward_token(b, pos0 + i)
        lr = om.forward_token(b, pos0 + i)
    worst = max(worst, float(np.max(np.abs(lg - lr))))
    assert worst < logit_tol, worst
    return {"worst": worst, "ties": ties, "min_margin": min_margin}

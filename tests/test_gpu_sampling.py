"""Temperature + top-p sampling on the device (gsdlq_sample_top_p) and the device generate loop with
sampling and the EOS stop.

The reference's sampler is sample_token (gsd_lq_cpu_runtime.py:422-443); tests/golden/sampling_ref.npz
holds its picks on fixed logits under fixed np.random seeds.  The device pick takes the draw
np.random.choice makes (np.random.random_sample() after the seed).  It must equal the reference's pick
except where the reference's result hangs on float rounding or on NumPy's unspecified order among equal
probabilities: top_p >= 1 (whether a float32 running sum ever exceeds 1) and nuclei holding tied
probabilities -- there the device pick must be a token of the same probability as the reference's
(ties) or of the distribution's support (top_p >= 1).  Larger vocabularies are checked against
smp_restated, a float64 / exact-integer restatement of the device algorithm.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ONE = 2.0 ** 56


def _probs(l, t):
    l = np.nan_to_num(np.asarray(l, np.float32), nan=-1e4, posinf=100.0, neginf=-1e4).astype(np.float32)
    z = (l / np.float32(max(t, 1e-4))).astype(np.float32)
    e = np.exp((z - z.max()).astype(np.float32)).astype(np.float32)
    return (e / np.float32(e.sum(dtype=np.float32))).astype(np.float32)


def _has_ties(l, t, top_p):
    """Equal probabilities among the reference's nucleus and the entry after it."""
    p = _probs(l, t)
    srt = np.sort(p)[::-1]
    k = int(np.argmax(np.cumsum(srt) > top_p)) + 1
    top = srt[: min(len(p), k + 1)]
    return len(np.unique(top)) < len(top)


def smp_restated(l, t, top_p, u):
    """The device algorithm's rule in exact integer sums: descending order of p (ties by index), the
    nucleus up to the first exact running sum above top_p, the pick where the running sum of p / P
    exceeds u times its total."""
    l = np.nan_to_num(np.asarray(l, np.float32), nan=-1e4, posinf=100.0, neginf=-1e4).astype(np.float32)
    if t <= 0:
        return int(np.argmax(l))
    p = _probs(l, t)
    order = np.lexsort((np.arange(len(p)), -p.astype(np.float64)))
    fm = [int(v) for v in np.floor(p[order].astype(np.float64) * ONE)]
    tgt, cum, k = int(np.floor(np.float64(np.float32(top_p)) * ONE)), 0, 1
    for j, m in enumerate(fm):
        cum += m
        if cum > tgt:
            k = j + 1
            break
    nuc = order[:k]
    P = np.float32(sum(fm[:k]) / ONE)
    pn = [int(np.floor(np.float64(np.float32(p[i] / P)) * ONE)) for i in nuc]
    target, cum = int(u * sum(pn)), 0
    for i, m in zip(nuc, pn):
        cum += m
        if cum > target:
            return int(i)
    return int(nuc[-1])


def test_device_sampler_against_reference_picks(cuda_lib):
    import gsdlq_b200.ops as ops
    g = np.load(os.path.join(GOLDEN, "sampling_ref.npz"))
    logits, cases, seeds, picks = g["logits"], g["cases"], g["seeds"], g["picks"]
    state = np.random.get_state()
    exact = loose = 0
    try:
        for i, lg in enumerate(logits):
            ld = torch.from_numpy(np.ascontiguousarray(lg)).cuda()
            for j, (t, p) in enumerate(cases):
                for k, seed in enumerate(seeds):
                    np.random.seed(int(seed))
                    u = float(np.random.random_sample()) if t > 0 else 0.0
                    got, ref = ops.sample_top_p(ld, float(t), float(p), u), int(picks[i, j, k])
                    if t <= 0 or (p < 1.0 and not _has_ties(lg, t, p)):
                        assert got == ref, (i, (t, p), int(seed), got, ref)
                        exact += 1
                    else:
                        pr = _probs(lg, t)
                        assert 0 <= got < len(lg) and pr[got] > 0
                        if p < 1.0:
                            assert pr[got] == pr[ref], (i, (t, p), int(seed), got, ref)
                        loose += 1
    finally:
        np.random.set_state(state)
    assert exact == 136 and loose == 104, (exact, loose)  # the split of the 240 golden picks


@pytest.mark.parametrize("n", [4096, 32768, 151936])
def test_device_sampler_large_vocab(cuda_lib, n):
    import gsdlq_b200.ops as ops
    rng = np.random.default_rng(n)
    for trial, (scale, t, p) in enumerate([(3.0, 0.4, 0.9), (1.0, 0.7, 0.9), (8.0, 1.0, 0.5), (0.5, 1.3, 0.99)]):
        lg = (rng.standard_normal(n) * scale).astype(np.float32)
        ld = torch.from_numpy(lg).cuda()
        for u in (0.0, 0.137, 0.5, 0.9999):
            assert ops.sample_top_p(ld, t, p, u) == smp_restated(lg, t, p, u), (n, trial, u)
    # greedy, and the first of equal maxima
    lg = np.zeros(n, np.float32)
    lg[[7, n - 3]] = 5.0
    assert ops.sample_top_p(torch.from_numpy(lg).cuda(), 0.0, 0.9, 0.5) == 7
    # a flat distribution: the pick is the u-quantile in index order
    flat = torch.zeros(n, device="cuda")
    got = ops.sample_top_p(flat, 1.0, 0.5, 0.25)
    assert got == smp_restated(np.zeros(n, np.float32), 1.0, 0.5, 0.25)


@pytest.fixture(scope="module")
def small_model(cuda_lib):
    import gsdlq_b200.packer as P
    from gsdlq_b200.model import GSDLQModel
    cfg = P.make_config("smollm2-1.7b", n_layers=2, vocab_size=4096)
    dm = P.random_model_cuda(cfg, "turbo", seed=5, norm_jitter=0.1)
    m = GSDLQModel(dm, max_seq=256)
    yield m
    m.release()


def test_generate_sampled_matches_step_by_step(small_model, monkeypatch):
    # token-by-token prefill: its sums are deterministic, so both paths see bit-identical caches (batched
    # prefill adds GEMM partial sums with atomics, and a sampled pick can flip on a last-bit difference)
    monkeypatch.setenv("GSDLQ_PREFILL", "token")
    m = small_model
    prompt = [11, 250, 3000, 17, 99]
    np.random.seed(3)
    got = m.generate(prompt, 24, temperature=0.8, top_p=0.9)
    # the same picks one token at a time: forward_token, then the device sampler with the same draws
    np.random.seed(3)
    draws = np.random.random_sample(24)
    m.prefill(prompt[:-1])
    tok, want = prompt[-1], []
    for i in range(24):
        m.forward_token(tok, len(prompt) - 1 + i)
        tok = m.sample_device(0.8, 0.9, u=float(draws[i]))
        want.append(tok)
    assert got == want


def test_generate_stops_at_eos(small_model, monkeypatch):
    monkeypatch.setenv("GSDLQ_PREFILL", "token")  # deterministic caches across the compared runs
    m = small_model
    prompt = [5, 6, 7]
    full = m.generate(prompt, 20)
    eos = full[6]
    first = full.index(eos)
    got = m.generate(prompt, 20, eos_id=eos, check_every=4)
    assert got == full[:first]
    # sampled, with the same draws: stops at the first sampled EOS
    np.random.seed(9)
    s_full = m.generate(prompt, 20, temperature=0.9, top_p=0.95)
    eos = s_full[10]
    np.random.seed(9)
    s_got = m.generate(prompt, 20, temperature=0.9, top_p=0.95, eos_id=eos, check_every=3)
    assert s_got == s_full[: s_full.index(eos)]

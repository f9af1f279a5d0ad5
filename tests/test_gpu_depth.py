"""Full-depth greedy parity on the GPU against the reference C engine.

The acceptance bar of the decode path: logits within 1e-2 max-abs of the reference's
and identical greedy top-1 tokens over a long decode, at the full layer count of the
BASELINE shapes.  The reference side is the reference's own C engine (oracle/_ref,
compiled from its source; the C restatement where it was not built) driven by the
oracle decoder on the host cores, over the same packed bytes as the GPU model.

* Qwen2.5-1.5B shape, Precision, all 28 layers: a 512-token uniform-random prompt,
  then 256 greedy steps.
* Mistral-7B shape, Precision, all 32 layers: 16 greedy steps from position 1536,
  with positions 0..1535 of both KV caches filled with the same seeded fp16 values
  (no 1536-token CPU prefill).

A differing pick is allowed only at a near-tie (oracle top-2 margin < 1e-3); near-ties
are printed with their margins and counted.  Run with ``-s`` to see the summary lines.
"""
import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
torch = pytest.importorskip("torch")

from conftest import oracle_decoder, greedy_parity, greedy_continue  # noqa: E402

LOGIT_TOL = 1e-2
MAX_NEAR_TIES = 2  # more than this many near-ties would make the pick comparison meaningless


def _models(name, mode, seed, max_seq, **over):
    import gsdlq_b200.packer as P
    from gsdlq_b200.model import GSDLQModel
    cfg = P.make_config(name, **over)
    dm = P.random_model_cuda(cfg, mode, seed=seed, norm_jitter=0.1)
    host = P.device_model_to_host(dm)
    m = GSDLQModel(dm, max_seq=max_seq)
    del dm
    om = oracle_decoder(host, max_seq=max_seq)
    return cfg, m, om


def test_qwen_full_depth_512_prompt_256_greedy(cuda_lib):
    import gsdlq_b200._lib as L
    cfg, m, om = _models("qwen2.5-1.5b", "precision", seed=11, max_seq=1024)
    assert m.n_layers == 28
    prompt = np.random.default_rng(12).integers(0, cfg["vocab_size"], 512).tolist()
    r = greedy_parity(m, om, prompt, 256, LOGIT_TOL)
    print(f"\nqwen2.5-1.5b x28 precision, 512+256 ({om.e.kind} engine): max|dlogit| {r['worst']:.3e}, "
          f"near-ties {len(r['ties'])} {r['ties']}, smallest top-2 margin {r['min_margin']:.3e}")
    assert len(r["ties"]) <= MAX_NEAR_TIES
    assert L.device_flags() == 0


def test_mistral_full_depth_from_seeded_kv(cuda_lib):
    import gsdlq_b200._lib as L
    P0 = 1536
    cfg, m, om = _models("mistral-7b", "precision", seed=21, max_seq=2048)
    assert m.n_layers == 32
    rng = np.random.default_rng(22)
    for c_host, c_dev in ((om.k_cache, m.k_cache), (om.v_cache, m.v_cache)):
        c_host[:, :P0] = rng.standard_normal(c_host[:, :P0].shape, dtype=np.float32).astype(np.float16).view(np.uint16)
        c_dev[:, :P0].copy_(torch.from_numpy(c_host[:, :P0].view(np.float16)))
    tok = int(rng.integers(0, cfg["vocab_size"]))
    lg = m.forward_token(tok, P0 - 1)
    lr = om.forward_token(tok, P0 - 1)
    r = greedy_continue(m, om, lg, lr, P0, 16, LOGIT_TOL)
    print(f"\nmistral-7b x32 precision, 16 steps from pos {P0} ({om.e.kind} engine): max|dlogit| {r['worst']:.3e}, "
          f"near-ties {len(r['ties'])} {r['ties']}, smallest top-2 margin {r['min_margin']:.3e}")
    assert len(r["ties"]) <= MAX_NEAR_TIES
    assert L.device_flags() == 0

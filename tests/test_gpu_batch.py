"""Batched decode (gsdlq_b200.batch.BatchDecoder): B sequences in lockstep through the tensor-core
dequant-GEMM, batched RoPE / KV append and batched decode attention, against the batch-1 engine run on
each sequence alone (GSDLQModel.forward_token) and against the oracle decoder.

The reference decodes one sequence at a time (run_gpu_native_chat.py:921-984), so the batch-1 path is the
reference behaviour: every sequence's logits must match it within the north star's 1e-2 at every step
(teacher-forced with the batch's own greedy picks, so both paths see the same tokens), with the same
greedy pick except at near-ties.
"""
import numpy as np
import pytest

from conftest import oracle_decoder, top2_margin, NEAR_TIE

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

LOGIT_TOL = 1e-2


@pytest.mark.parametrize("name,over,mode,batch", [
    ("smollm2-1.7b", dict(n_layers=2), "turbo", 16),
    ("mistral-7b", dict(n_layers=2), "precision", 5),
    ("qwen2.5-1.5b", dict(n_layers=2), "precision", 3),
])
def test_batch_decode_matches_single_sequence(cuda_lib, name, over, mode, batch):
    import oracle
    import gsdlq_b200.packer as P
    import gsdlq_b200._lib as L
    from gsdlq_b200.model import GSDLQModel
    from gsdlq_b200.batch import BatchDecoder
    cfg = P.make_config(name, **over)
    dm = P.random_model_cuda(cfg, mode, seed=23, norm_jitter=0.1)
    m = GSDLQModel(dm, max_seq=320)
    bd = BatchDecoder(m, batch, max_seq=320)
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, cfg["vocab_size"], int(n)).tolist() for n in rng.integers(2, 200, batch)]
    steps = 6
    for b, pr in enumerate(prompts):
        bd.prefill(b, pr[:-1])
    bd.set_tokens([pr[-1] for pr in prompts], [len(pr) - 1 for pr in prompts])
    got, picks = [], []
    for s in range(steps):
        bd.step()
        got.append(bd.logits_host())
        picks.append(bd.ids.cpu().numpy().copy())
    # each sequence alone through the batch-1 engine, fed the batch's picks
    worst, ties = 0.0, 0
    for b, pr in enumerate(prompts):
        m.prefill(pr[:-1])
        tok, pos = pr[-1], len(pr) - 1
        for s in range(steps):
            lg = m.forward_token(tok, pos + s)
            worst = max(worst, float(np.max(np.abs(lg - got[s][b]))))
            if int(np.argmax(lg)) != int(picks[s][b]):
                assert top2_margin(lg) < NEAR_TIE, (b, s)
                ties += 1
            tok = int(picks[s][b])
    print(f"\n{name} B={batch}: max |dlogit| vs batch-1 {worst:.2e}, near-tie picks {ties}")
    assert worst < LOGIT_TOL
    # sequence 0's first step against the oracle decoder
    host = P.device_model_to_host(dm)
    om = oracle_decoder(host, oracle.CEngine.restatement(), max_seq=320)
    pr = prompts[0]
    for pos, t in enumerate(pr):
        lr = om.forward_token(t, pos, return_logits=pos == len(pr) - 1)
    assert float(np.max(np.abs(lr - got[0][0]))) < LOGIT_TOL
    assert L.device_flags() == 0
    # generate: the same continuations as the step loop above (its own batched prefill may differ from the
    # first one in the last bits -- the GEMM adds with atomics -- so a pick may differ only at a near-tie,
    # after which that sequence is not compared further)
    bd2 = BatchDecoder(m, batch, max_seq=320)
    outs = bd2.generate(prompts, steps)
    for b in range(batch):
        for s in range(steps):
            if outs[b][s] != int(picks[s][b]):
                assert top2_margin(got[s][b]) < NEAR_TIE, (b, s)
                break
    bd.release()
    bd2.release()
    m.release()


def test_batch_decode_rejects_bad_positions(cuda_lib):
    import gsdlq_b200.packer as P
    from gsdlq_b200.model import GSDLQModel
    from gsdlq_b200.batch import BatchDecoder
    cfg = P.make_config("smollm2-1.7b", n_layers=1)
    m = GSDLQModel(P.random_model_cuda(cfg, "turbo", seed=1), max_seq=64)
    bd = BatchDecoder(m, 2, max_seq=64)
    with pytest.raises(ValueError):
        bd.set_tokens([1, 2], [0, 64])
    with pytest.raises(ValueError):
        bd.set_tokens([1, cfg["vocab_size"]], [0, 1])
    with pytest.raises(ValueError):
        BatchDecoder(m, 2, max_seq=65)
    bd.release()
    m.release()

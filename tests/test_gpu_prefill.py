"""Chunked prefill on the GPU (tcgen05 dequant-GEMM per linear, row kernels around it) against
token-by-token prefill and the oracle.

The reference fills the KV cache one forward_token per prompt token (run_gpu_native_chat.py:1128-1131);
GSDLQModel.prefill runs chunks of up to 128 tokens instead.  After a batched prefill of a prompt that
spans several chunks (the last one partial), the next token's logits must agree with those after a
token-by-token prefill of the same prompt and with the oracle decoder's: max-abs < 1e-2, the same greedy
pick; the two KV caches must agree to fp16 rounding.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from conftest import oracle_decoder  # noqa: E402

LOGIT_TOL = 1e-2


@pytest.mark.parametrize("name,over,mode,n_prompt", [
    ("mistral-7b", dict(n_layers=2), "precision", 300),
    ("qwen2.5-1.5b", dict(n_layers=2), "precision", 129),
    ("smollm2-1.7b", dict(n_layers=2), "turbo", 200),
])
def test_batched_prefill_matches_token_prefill_and_oracle(cuda_lib, name, over, mode, n_prompt):
    import oracle
    import gsdlq_b200.packer as P
    import gsdlq_b200._lib as L
    from gsdlq_b200.model import GSDLQModel
    cfg = P.make_config(name, **over)
    dm = P.random_model_cuda(cfg, mode, seed=41, norm_jitter=0.1)
    host = P.device_model_to_host(dm)
    a = GSDLQModel(dm, max_seq=512)
    b = GSDLQModel(dm, max_seq=512)
    prompt = np.random.default_rng(42).integers(0, cfg["vocab_size"], n_prompt).tolist()
    a.prefill(prompt[:-1], batched=True)
    b.prefill(prompt[:-1], batched=False)
    torch.cuda.synchronize()
    n = n_prompt - 1
    for ca, cb in ((a.k_cache, b.k_cache), (a.v_cache, b.v_cache)):
        da, db = ca[:, :n].float(), cb[:, :n].float()
        assert torch.max(torch.abs(da - db)).item() <= 2e-3 * max(1.0, torch.max(torch.abs(db)).item()) + 2e-3
    la = a.forward_token(prompt[-1], n)
    lb = b.forward_token(prompt[-1], n)
    om = oracle_decoder(host, oracle.CEngine.restatement(), max_seq=512)
    for pos, t in enumerate(prompt):
        lr = om.forward_token(t, pos, return_logits=pos == n)
    err_ab, err_ar = float(np.max(np.abs(la - lb))), float(np.max(np.abs(la - lr)))
    print(f"\n{name}: batched vs token prefill max|dlogit| {err_ab:.2e}, vs oracle {err_ar:.2e}")
    assert err_ab < LOGIT_TOL and err_ar < LOGIT_TOL
    assert a.sample_token(la) == b.sample_token(lb) == oracle.argmax(lr)
    # decoding continues identically from either cache
    assert L.device_flags() == 0


@pytest.mark.parametrize("n_heads,n_kv,hd,pos0,n", [
    (32, 8, 128, 1024, 128), (32, 8, 128, 0, 128), (12, 2, 128, 300, 77), (32, 32, 64, 1900, 128),
    (12, 2, 128, 0, 1), (16, 2, 64, 63, 65)])
def test_attention_rows_vs_torch(cuda_lib, n_heads, n_kv, hd, pos0, n):
    """gsdlq_attention_rows (position tiles, position splits merged by the combine kernel) against a
    float64 torch restatement of causal GQA attention over the fp16 cache."""
    import gsdlq_b200._lib as L
    import gsdlq_b200.ops as ops
    max_seq, layers, layer = 2048, 2, 1
    g = torch.Generator(device="cpu").manual_seed(pos0 * 7 + n)
    kc = torch.randn((layers, max_seq, n_kv, hd), generator=g).half().cuda()
    vc = torch.randn((layers, max_seq, n_kv, hd), generator=g).half().cuda()
    q = (torch.randn((n, n_heads, hd), generator=g) * 2.0).cuda()
    out = torch.full((n, n_heads, hd), 7.0, device="cuda")
    work = ops.attention_rows_work(n, n_heads, hd)
    sm = 1.0 / hd ** 0.5
    L.check(L.load().gsdlq_attention_rows(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), work.data_ptr(),
                                          work.numel(), layer, pos0, n, n_heads, n_kv, hd, max_seq, sm, None),
            "attention_rows")
    torch.cuda.synchronize()
    K, V = kc[layer].double().cpu(), vc[layer].double().cpu()
    qd, gq = q.double().cpu(), n_heads // n_kv
    ref = torch.empty((n, n_heads, hd), dtype=torch.float64)
    for t in range(n):
        length = pos0 + t + 1
        for h in range(n_heads):
            s = (K[:length, h // gq] @ qd[t, h]) * sm
            p = torch.softmax(s, 0)
            ref[t, h] = p @ V[:length, h // gq]
    err = torch.max(torch.abs(out.double().cpu() - ref)).item()
    assert err < 2e-5, err
    assert L.device_flags() == 0

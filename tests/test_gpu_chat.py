"""The chat session on the GPU: a turn that reuses the previous turn's cache rows gives the reply a fresh
model gives for the whole prompt, greedy and sampled, and the streamed text adds up to the reply.

Both sides prefill token by token (GSDLQ_PREFILL=token): every cache row then comes from the same decode
path, so the rows, logits and picks are bit-identical whether or not they were reused."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from conftest import GOLDEN  # noqa: E402


@pytest.mark.parametrize("temperature", [0.0, 0.4])
def test_chat_turn_with_reused_rows_matches_a_fresh_model(cuda_lib, monkeypatch, temperature):
    monkeypatch.setenv("GSDLQ_PREFILL", "token")
    from gsdlq_b200.chat import ChatSession, format_mistral_prompt
    from gsdlq_b200.model import GSDLQModel
    import gsdlq_b200._lib as L
    path = os.path.join(GOLDEN, "tiny_precision.gsd2")
    m = GSDLQModel(path, max_seq=256)
    s = ChatSession(m, system="Be brief.", temperature=temperature, max_new_tokens=6, stream_every=4)
    np.random.seed(11)
    s.turn("hi")
    pieces = []
    np.random.seed(12)
    t2 = s.turn("tell me more", on_text=pieces.append)
    assert 0 < t2.prefill_tokens < t2.prompt_tokens - 1  # some rows were reused
    dec = [m.tokenizer.decode(t2.ids[:k]) for k in range(len(t2.ids) + 1)]
    if all(dec[k + 1].startswith(dec[k]) for k in range(len(t2.ids))):  # no partial UTF-8 byte run
        assert "".join(pieces) == dec[-1] and dec[-1].strip() == t2.text
    f = GSDLQModel(path, max_seq=256)
    p2 = f.tokenizer.encode(format_mistral_prompt(s.history[:1], "tell me more", "Be brief."), add_bos=True)
    assert len(p2) == t2.prompt_tokens
    np.random.seed(12)
    ref = f.generate(p2, min(6, 256 - len(p2) - 1), temperature=temperature, top_p=0.9,
                     eos_id=f.tokenizer.eos_id)
    assert t2.ids == ref
    assert L.device_flags() == 0

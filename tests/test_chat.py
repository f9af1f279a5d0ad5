"""The chat surface (gsdlq_b200.chat) on the host: the prompt template against the reference's
format_mistral_prompt (tests/golden/chat_prompt_ref.json, recorded by make_golden.py), the shared-prefix
rule, and a session's bookkeeping over a stand-in model that keeps its KV cache as a token list."""
import json
import os

import pytest

from conftest import GOLDEN
from gsdlq_b200.chat import ChatSession, format_mistral_prompt, shared_prefix
from gsdlq_b200.tokenizer import from_config


def test_prompt_template_matches_reference():
    g = json.load(open(os.path.join(GOLDEN, "chat_prompt_ref.json"), encoding="utf-8"))
    assert len(g["cases"]) >= 12
    for c in g["cases"]:
        hist = [tuple(t) for t in c["history"]]
        assert format_mistral_prompt(hist, c["message"]) == c["lightweight"], c
        assert format_mistral_prompt(hist, c["message"], system=g["system"]) == c["with_system"], c


@pytest.mark.parametrize("cached,prompt,n", [
    ([], [1, 2, 3], 0),
    ([1, 2, 3, 4], [1, 2, 3, 4], 3),        # the last prompt token is always run
    ([1, 2, 9, 4], [1, 2, 3, 4, 5], 2),
    ([1, 2], [1, 2, 3, 4], 2),
    ([5], [1, 2], 0),
    ([1], [1], 0),
])
def test_shared_prefix(cached, prompt, n):
    assert shared_prefix(cached, prompt) == n


class FakeModel:
    """GSDLQModel's generate contract over a token-list KV cache: prefill writes ids at their positions;
    each decode step runs the current token (writes its row) and picks the next from a script; an EOS pick
    stops without being returned or run; at the token limit the last pick is never run."""

    def __init__(self, tokenizer, max_seq, replies):
        self.tokenizer, self.max_seq, self.replies = tokenizer, max_seq, list(replies)
        self.kv = [None] * max_seq
        self.prefills = []

    def prefill(self, ids, start_pos=0):
        self.prefills.append((start_pos, len(ids)))
        for i, t in enumerate(ids):
            self.kv[start_pos + i] = t

    def synchronize(self):
        pass

    def generate(self, ids, max_new, temperature, top_p, eos_id, check_every, start_pos, on_tokens):
        assert self.kv[:start_pos] == list(ids[:start_pos]), "reused rows differ from the prompt"
        self.prefill(ids[start_pos:-1], start_pos)
        script = self.replies.pop(0)
        out, t, p = [], ids[-1], len(ids) - 1
        for i in range(max_new):
            self.kv[p] = t
            pick = script[i] if i < len(script) else eos_id
            if pick == eos_id:
                break
            out.append(pick)
            t, p = pick, p + 1
            if (i + 1) % check_every == 0:
                on_tokens(out[-check_every:])
        done = (len(out) // check_every) * check_every
        if len(out) > done:
            on_tokens(out[done:])
        return out


@pytest.fixture(scope="module")
def tok():
    g = json.load(open(os.path.join(GOLDEN, "tokenizer_ref.json"), encoding="utf-8"))
    return from_config(g["vocab"])


def _word_ids(tok, text):
    return tok.encode(text, add_bos=False)


def test_session_reuses_the_cache_and_streams(tok):
    r1, r2 = _word_ids(tok, "hello there"), _word_ids(tok, "fine thanks")
    m = FakeModel(tok, 512, [r1 + [tok.eos_id], r2])
    s = ChatSession(m, system="Be brief.", temperature=0.0, max_new_tokens=len(r2), stream_every=3)
    pieces = []
    t1 = s.turn("hi", on_text=pieces.append)
    assert t1.ids == r1 and t1.text == tok.decode(r1).strip() and "".join(pieces) == tok.decode(r1)
    assert t1.prefill_tokens == t1.prompt_tokens - 1 and not t1.reset
    assert s.history == [("hi", t1.text)]
    assert s.cached == tok.encode(format_mistral_prompt([], "hi", "Be brief."), add_bos=True) + r1
    # second turn: every row of the first turn's prompt and reply that the new prompt repeats is reused
    t2 = s.turn("how are you?")
    p2 = tok.encode(format_mistral_prompt([("hi", t1.text)], "how are you?", "Be brief."), add_bos=True)
    n = shared_prefix(tok.encode(format_mistral_prompt([], "hi", "Be brief."), add_bos=True) + r1, p2)
    assert n > 0 and t2.prefill_tokens == len(p2) - 1 - n and t2.ids == r2
    # stopped at the token limit: the last reply token was picked but never run, so it is not cached
    assert s.cached == p2 + r2[:-1] and m.kv[:len(s.cached)] == s.cached


def test_session_resets_when_the_prompt_nears_the_cache_end(tok):
    r = _word_ids(tok, "ok")
    m = FakeModel(tok, 160, [r + [tok.eos_id]] * 4)
    s = ChatSession(m, temperature=0.0, reserve=64)
    resets = [s.turn("a fairly long message to fill the cache " * 2).reset for _ in range(4)]
    assert resets[0] is False and any(resets)
    last = len(resets) - 1 - resets[::-1].index(True)
    assert len(s.history) == len(resets) - last  # the history restarted at the last turn that reset
    with pytest.raises(ValueError, match="message alone"):
        ChatSession(FakeModel(tok, 40, [r]), temperature=0.0).turn("x" * 200)


def test_reset_forgets_the_conversation(tok):
    r = _word_ids(tok, "ok")
    m = FakeModel(tok, 256, [r + [tok.eos_id]] * 2)
    s = ChatSession(m, temperature=0.0)
    s.turn("one")
    s.reset()
    assert s.history == [] and s.cached == []
    t = s.turn("two")
    assert t.prefill_tokens == t.prompt_tokens - 1 and m.prefills[-2][0] == 0

"""The model's tokenizer (gsdlq_b200.tokenizer) against the reference's MistralSentencePieceTokenizer
(run_gpu_native_chat.py:660-729): encode and decode results recorded from the reference on a test
vocabulary (tests/golden/tokenizer_ref.json, written by make_golden.py), and the heap-based merge loop
against a plain quadratic statement of the same merge rule over random strings."""
import json
import os

import pytest

from conftest import GOLDEN
from gsdlq_b200.tokenizer import MIN_SCORE, MistralSentencePieceTokenizer, from_config


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "tokenizer_ref.json"), encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def tok(golden):
    return from_config(golden["vocab"])


def test_encode_matches_reference(tok, golden):
    for text, with_bos, without_bos in golden["encode"]:
        assert tok.encode(text) == with_bos, text
        assert tok.encode(text, add_bos=False) == without_bos, text


def test_decode_matches_reference(tok, golden):
    for ids, text in golden["decode"]:
        assert tok.decode(ids) == text, ids


def _merge_quadratic(tk, piece):
    """The merge rule stated directly: rescan all adjacent pairs, merge the highest-scoring one (the
    leftmost among equal scores, scores above MIN_SCORE only), until no adjacent pair is a token."""
    syms = []
    for ch in piece:
        syms.extend([ch] if ch in tk.vocab else [f"<0x{b:02X}>" for b in ch.encode("utf-8")])
    while True:
        best, at = None, -1
        for i in range(len(syms) - 1):
            t = tk.vocab.get(syms[i] + syms[i + 1])
            if t is None or not tk.scores[t] > MIN_SCORE:
                continue
            if best is None or tk.scores[t] > best:
                best, at = tk.scores[t], i
        if at < 0:
            return [tk.vocab.get(s, 0) for s in syms]
        syms[at:at + 2] = [syms[at] + syms[at + 1]]


def test_heap_merge_equals_quadratic_rule(tok):
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    alphabet = st.sampled_from(list("▁▁▁aabcdehilnorstwé12[]INST") + ["€", "😀"])

    @hyp.settings(max_examples=300, deadline=None, derandomize=True)
    @hyp.given(st.lists(alphabet, min_size=0, max_size=60).map("".join))
    def check(piece):
        assert tok._bpe(piece) == _merge_quadratic(tok, piece), piece

    check()


def test_round_trip(golden):
    """decode(encode(text)) gives the text back, with the leading space the encoder adds to the first text
    part, when every character is a token or has byte tokens; BOS and EOS are dropped."""
    tk = MistralSentencePieceTokenizer(**{k: golden["vocab"][k] for k in ("tokens", "scores", "token_types")},
                                       bos_id=1, eos_id=2)
    for text in ("hello world", "the thing and the other", "price 12€ 😀"):
        ids = tk.encode(text)
        assert ids[0] == 1 and tk.decode(ids + [2]) == " " + text
    # only the first text part gets the marker: text after a control token keeps its own start
    assert tk.decode(tk.encode("a[INST]b")) == " a[INST]b"


def test_from_gsd2_header():
    """The tokenizer the model object builds from a .gsd2 header (the golden tiny model's synthetic
    vocabulary: control tokens, 256 byte tokens and "▁w<i>" words, no single characters): text falls back
    to byte tokens, which decode to the marked text, and word ids decode to their words."""
    import gsdlq_b200.gsd2 as G
    cfg = G.read_gsd2(os.path.join(GOLDEN, "tiny_precision.gsd2")).config
    tk = from_config(cfg)
    assert (tk.bos_id, tk.eos_id) == (cfg["bos_id"], cfg["eos_id"])
    ids = tk.encode("w300 Zé")
    assert ids[0] == cfg["bos_id"] and all(tk.token_types[i] == 6 for i in ids[1:])
    assert len(ids) - 1 == len("▁w300▁Zé".encode("utf-8"))
    assert tk.decode(ids) == "▁w300▁Zé"  # byte tokens keep the marker, as the reference's decode does
    assert tk.decode([tk.vocab["▁w300"], tk.vocab["▁w301"]]) == " w300 w301"

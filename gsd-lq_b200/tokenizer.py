"""SentencePiece-BPE tokenizer over a .gsd2 header's vocabulary: the model object's ``.tokenizer``.

Same constructor, method names and results as the reference's ``MistralSentencePieceTokenizer``
(run_gpu_native_chat.py:660-729), so that a caller gets the same ids for the same text:

  * encode(text, add_bos=True): BOS first; the text is cut at the control tokens (token type 3), longest
    first, each of which maps to its own id; in every other part spaces become U+2581 and the first text
    part gets a leading U+2581 if it has none.  A part starts as one symbol per character, or one
    "<0xHH>" symbol per UTF-8 byte of a character the vocabulary lacks; adjacent symbols are then merged
    while some adjacent pair is itself a token, always the pair whose token has the highest score, the
    leftmost among equal scores (a score must exceed -1e30, so NaN and -inf never merge).  Symbols the
    vocabulary lacks become id 0.
  * decode(ids): BOS and EOS are dropped, byte tokens (type 6, "<0xHH>") become raw bytes, U+2581 becomes
    a space, and the bytes are decoded as UTF-8 with replacement characters.

The merges run on a heap of adjacent pairs over a linked list of symbols, O(n log n) per part, where the
reference rescans every pair after each merge, O(n^2).  Both take the same pair at every step: the heap
orders by (-score, index of the left symbol), and left-to-right order of live symbols is their index
order.  A string listed twice in the vocabulary resolves to its last id, as in a dict built in order.
With no control tokens at all the pre-split pattern is an empty group, which cuts the text between every
two characters; that is the reference's behaviour too, and kept (real vocabularies have control tokens).
"""
from __future__ import annotations

import heapq
import re

SPACE = "▁"
CONTROL, BYTE = 3, 6
MIN_SCORE = -1e30


class MistralSentencePieceTokenizer:
    def __init__(self, tokens, scores, token_types, bos_id: int = 1, eos_id: int = 2):
        self.tokens = list(tokens)
        self.scores = [float(s) for s in scores]
        self.token_types = list(token_types)
        self.bos_id, self.eos_id = bos_id, eos_id
        self.vocab = {t: i for i, t in enumerate(self.tokens)}
        control = sorted({t for t, ty in zip(self.tokens, self.token_types) if ty == CONTROL}, key=len, reverse=True)
        self._split = re.compile("(" + "|".join(re.escape(t) for t in control) + ")")
        self.byte_tokens = {i: int(t[3:5], 16) for i, (t, ty) in enumerate(zip(self.tokens, self.token_types))
                            if ty == BYTE and len(t) == 6 and t.startswith("<0x")}

    # ---- encode ----------------------------------------------------------------------------
    def _pair_score(self, a: str, b: str):
        tid = self.vocab.get(a + b)
        if tid is None:
            return None
        s = self.scores[tid]
        return s if s > MIN_SCORE else None

    def _bpe(self, text: str) -> list[int]:
        if not text:
            return []
        sym: list[str] = []
        for ch in text:
            if ch in self.vocab:
                sym.append(ch)
            else:
                sym.extend(f"<0x{b:02X}>" for b in ch.encode("utf-8"))
        n = len(sym)
        nxt = list(range(1, n + 1))
        nxt[-1] = -1
        prv = list(range(-1, n - 1))
        live = [True] * n
        heap: list = []

        def offer(i: int) -> None:  # the pair (i, its right neighbour)
            j = nxt[i]
            if j >= 0:
                s = self._pair_score(sym[i], sym[j])
                if s is not None:
                    heapq.heappush(heap, (-s, i, sym[i], sym[j]))

        for i in range(n - 1):
            offer(i)
        while heap:
            _, i, a, b = heapq.heappop(heap)
            j = nxt[i] if live[i] else -1
            if j < 0 or sym[i] != a or sym[j] != b:
                continue  # one side has merged since this pair was offered
            sym[i] = a + b
            live[j] = False
            nxt[i] = nxt[j]
            if nxt[i] >= 0:
                prv[nxt[i]] = i
            if prv[i] >= 0:
                offer(prv[i])
            offer(i)
        return [self.vocab.get(sym[i], 0) for i in range(n) if live[i]]

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = [self.bos_id] if add_bos else []
        first = True
        for part in self._split.split(text):
            if not part:
                continue
            tid = self.vocab.get(part)
            if tid is not None and self.token_types[tid] == CONTROL:
                ids.append(tid)
                first = False
                continue
            piece = part.replace(" ", SPACE)
            if first and not piece.startswith(SPACE):
                piece = SPACE + piece
            first = False
            ids.extend(self._bpe(piece))
        return ids

    # ---- decode ----------------------------------------------------------------------------
    def decode(self, ids) -> str:
        out = bytearray()
        for tid in ids:
            if tid in (self.bos_id, self.eos_id):
                continue
            b = self.byte_tokens.get(tid)
            if b is not None:
                out.append(b)
            else:
                out.extend(self.tokens[tid].replace(SPACE, " ").encode("utf-8"))
        return out.decode("utf-8", errors="replace")


def from_config(cfg: dict) -> MistralSentencePieceTokenizer:
    """The tokenizer of a .gsd2 header (tokens, scores, token_types, bos_id, eos_id)."""
    return MistralSentencePieceTokenizer(cfg.get("tokens", []), cfg.get("scores", []), cfg.get("token_types", []),
                                         cfg.get("bos_id", 1), cfg.get("eos_id", 2))

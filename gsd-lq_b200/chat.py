"""Multi-turn chat over a loaded model: the reference chat loop's surface as a library class.

The reference's loop (run_gpu_native_chat.py:1058-1170) formats the conversation with the Mistral
instruct template (format_mistral_prompt, :996-1013), encodes it with a BOS, reuses the KV cache rows of
the longest prefix shared with the previous turn's tokens (:1112-1114), starts the conversation over when
the prompt comes within 64 positions of the cache's end (:1116-1122), prefills the rest of the prompt
(:1126-1131), samples at temperature 0.4 / top-p 0.9 until EOS or min(512, cache end - 1) tokens, printing
the decoded text as it grows (:1137-1152), and keeps (user, reply) pairs as history (:1167).

Here the prompt is prefilled by chunks through the tensor-core GEMM, and generation runs on the device
(GSDLQModel.generate: one graph replay per token, sampling on the device, EOS stop). Text is streamed
every `stream_every` tokens instead of every token, one host synchronisation each time. The terminal
loop, its log file and its statistics printout are not part of the library.
"""
from __future__ import annotations

import dataclasses
import time
from typing import Callable


def format_mistral_prompt(history, new_user_msg: str, system: str | None = None) -> str:
    """The Mistral instruct template of the reference's format_mistral_prompt.

    history: (user, reply) pairs of earlier turns.  Without ``system`` the reference's lightweight layout
    (its is_cpu=True branch): "[INST] u [/INST] a</s>" per turn, then "[INST] new [/INST]".  With
    ``system`` (its default branch, whose rules text is the caller's here): the first turn's instruction
    reads "{system}\\n\\nUser: {u}"."""
    parts = []
    turns = list(history) + [(new_user_msg, None)]
    for i, (u, a) in enumerate(turns):
        inst = f"{system}\n\nUser: {u}" if system is not None and i == 0 else u
        parts.append(f"[INST] {inst} [/INST]" + ("" if a is None else f" {a}</s>"))
    return "".join(parts)


def shared_prefix(cached, prompt) -> int:
    """KV rows reusable from the previous turn: the length of the common prefix of ``cached`` and
    ``prompt``, at most len(prompt) - 1 (the last prompt token is always run, for its logits)."""
    n, top = 0, min(len(cached), len(prompt) - 1)
    while n < top and cached[n] == prompt[n]:
        n += 1
    return n


@dataclasses.dataclass
class Turn:
    text: str                 # the decoded reply, stripped (what enters the history)
    ids: list                 # its token ids (EOS excluded)
    prompt_tokens: int        # tokens of the whole prompt
    prefill_tokens: int       # of those, the ones prefilled this turn: neither reused nor the last
    prefill_s: float
    gen_s: float
    reset: bool               # the history was dropped to make the prompt fit


class ChatSession:
    """Conversation state over one model: history, the tokens whose K/V rows the cache holds, sampling
    settings.  ``turn(msg)`` runs one exchange and returns a Turn."""

    def __init__(self, model, system: str | None = None, temperature: float = 0.4, top_p: float = 0.9,
                 max_new_tokens: int = 512, reserve: int = 64, stream_every: int = 8):
        self.m = model
        self.tok = model.tokenizer
        self.system = system
        self.temperature, self.top_p = float(temperature), float(top_p)
        self.max_new_tokens, self.reserve, self.stream_every = int(max_new_tokens), int(reserve), int(stream_every)
        self.history: list[tuple[str, str]] = []
        self.cached: list[int] = []   # tokens at cache positions 0 .. len - 1

    def reset(self):
        """Forget the conversation (the reference's 'reset' command)."""
        self.history.clear()
        self.cached = []

    def _prompt_ids(self, msg: str) -> list[int]:
        return self.tok.encode(format_mistral_prompt(self.history, msg, self.system), add_bos=True)

    def turn(self, user_msg: str, on_text: Callable[[str], None] | None = None) -> Turn:
        S = self.m.max_seq
        ids = self._prompt_ids(user_msg)
        reset = False
        if len(ids) >= S - self.reserve:
            self.reset()
            reset = True
            ids = self._prompt_ids(user_msg)
            if len(ids) >= S - 1:
                raise ValueError(f"the message alone takes {len(ids)} tokens; the cache holds {S}")
        start = 0 if reset else shared_prefix(self.cached, ids)
        max_new = min(self.max_new_tokens, S - len(ids) - 1)
        shown = ""
        got: list[int] = []

        def stream(new_ids):
            # the reference prints decode(all ids so far) minus what it printed before (:1146-1149)
            nonlocal shown
            got.extend(new_ids)
            if on_text is not None:
                text = self.tok.decode(got)
                if len(text) > len(shown):
                    on_text(text[len(shown):])
                shown = text

        t0 = time.perf_counter()
        self.m.prefill(ids[start:-1], start_pos=start)
        self.m.synchronize()
        t1 = time.perf_counter()
        gen = self.m.generate(ids, max_new, temperature=self.temperature, top_p=self.top_p,
                              eos_id=self.tok.eos_id, check_every=self.stream_every, start_pos=len(ids) - 1,
                              on_tokens=stream)
        t2 = time.perf_counter()
        text = self.tok.decode(gen).strip()
        self.history.append((user_msg, text))
        # K/V rows written: the prompt and every reply token the model ran; when the reply stopped at the
        # token limit instead of an EOS, its last token was picked but never run
        ran = len(gen) if len(gen) < max_new else len(gen) - 1
        self.cached = ids + gen[:ran]
        return Turn(text=text, ids=gen, prompt_tokens=len(ids), prefill_tokens=len(ids) - 1 - start,
                    prefill_s=t1 - t0, gen_s=t2 - t1, reset=reset)

"""Generate the golden fixtures in this directory from the REFERENCE implementation.

Run in a container that holds the reference tree (its location taken from
$GSDLQ_REFERENCE, else from BASELINE.json's reference_path); the fixtures are
committed so the tests never need the reference at run time:

    python tests/golden/make_golden.py            # everything
    python tests/golden/make_golden.py sampling   # only sampling_ref.npz
    python tests/golden/make_golden.py tokenizer  # only tokenizer_ref.json
    python tests/golden/make_golden.py chat       # only chat_prompt_ref.json

What it records (all produced by the reference's own code):
  codebook.npz     _get_turbo_codebook(6|8) from both reference copies
                   (gsd_lq_cpu_runtime.py:111-118, run_gpu_native_chat.py:26-33)
  tiny.gsd2        a small random-init model written by our packer
  tiny_ref.npz     for tiny.gsd2, loaded by the reference's CPUMistralV2Model with its
                   C engine (built from the reference source into oracle/_ref):
                     - logits of forward_token over a fixed token sequence (with greedy picks)
                     - _matvec_cpu(x, layer0.q) and (k_dim = 0 path) _matvec_cpu(x, layer0.k of a turbo file)
                     - the NumPy-fallback dequantised weight W of layer0.q (the W definition)
                       and its fallback matvec
  sampling_ref.npz the reference's sample_token picks (temperature + top-p) on fixed logits
                   under fixed np.random seeds
  tokenizer_ref.json the reference's SentencePiece-BPE encode/decode on a test vocabulary
  chat_prompt_ref.json the reference's chat prompt template over fixed histories (its rules text
                   replaced by a test string)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

TOKENS = [1, 17, 300, 42, 255, 7, 299, 100]


def reference_tree() -> str:
    import oracle as O
    ref = O.reference_dir()  # $GSDLQ_REFERENCE, else BASELINE.json's reference_path
    if ref is None:
        raise SystemExit("the reference source tree is needed: set GSDLQ_REFERENCE")
    return ref


def main():
    import gsdlq_b200.packer as P
    import gsdlq_b200.gsd2 as G
    import oracle as O  # only to locate/build the reference .so

    O.build()
    sys.path.insert(0, os.path.join(reference_tree(), "gsd_lq_v2"))
    import gsd_lq_cpu_runtime as R
    import run_gpu_native_chat as RG

    np.savez(os.path.join(HERE, "codebook.npz"),
             cpu6=R._get_turbo_codebook(6)[0], cpu8=R._get_turbo_codebook(8)[0],
             gpu6=RG._get_turbo_codebook(6)[0], gpu8=RG._get_turbo_codebook(8)[0])

    cfg = P.make_config("tiny", n_layers=2, hidden_size=128, n_heads=4, n_kv_heads=2, head_dim=32,
                        ffn_size=256, vocab_size=320)
    for mode in ("precision", "turbo"):
        m = P.random_model(cfg, mode, seed=7, norm_jitter=0.1)
        path = os.path.join(HERE, f"tiny_{mode}.gsd2")
        G.write_gsd2(path, m)

        R.LIB_PATH = O.REF_LIB  # use the reference engine built from its own source
        ref = R.CPUMistralV2Model(path, rope_interleaved=1)
        assert ref.cpu.lib is not None, "reference C engine did not load"
        logits, picks = [], []
        for pos, tok in enumerate(TOKENS):
            lg = ref.forward_token(tok, pos, return_logits=True)
            logits.append(lg)
            picks.append(ref.sample_token(lg, temperature=0.0))
        rng = np.random.default_rng(3)
        x = rng.standard_normal(cfg["hidden_size"]).astype(np.float16).astype(np.float32)
        outs = {}
        for key in ("q", "k", "gate"):
            y = np.zeros(ref.layers[0][key]["rows"], np.float32)
            ref._matvec_cpu(x, ref.layers[0][key], y)
            outs["mv_" + key] = y
        # the NumPy fallback path (cpu.lib = None) defines the dequantised weight
        lib = ref.cpu.lib
        ref.cpu.lib = None
        lyr = ref.layers[0]["q"]
        scales_f32 = lyr["scales"].view(np.float16).astype(np.float32)
        pts = lyr["xy_table"][lyr["codes"]].reshape(lyr["rows"], lyr["cols"])
        W = pts * np.repeat(scales_f32.reshape(lyr["rows"], lyr["cols"] // 64), 64, axis=1)
        y_fb = np.zeros(lyr["rows"], np.float32)
        ref._matvec_cpu(x, lyr, y_fb)
        ref.cpu.lib = lib
        np.savez(os.path.join(HERE, f"tiny_{mode}_ref.npz"), tokens=np.array(TOKENS), logits=np.stack(logits),
                 picks=np.array(picks), x=x, W_q=W, mv_q_fallback=y_fb, **outs)
        print(mode, "picks", picks)


# (temperature, top_p) pairs of the sampling fixture: greedy, the chat default, a tight nucleus, top_p = 1.0
# (the cumulative sum may never exceed it, so the reference keeps only the top token) and a tiny temperature
SAMPLING_CASES = [(0.0, 0.9), (0.7, 0.9), (1.0, 0.5), (1.3, 1.0), (1e-6, 0.9), (0.9, 0.99)]
SAMPLING_SEEDS = range(8)


def sampling_logits():
    """Logit vectors of the sampling fixture: random, with NaN/+-inf entries, with a tie at the maximum."""
    rng = np.random.default_rng(11)
    out = [rng.standard_normal(320).astype(np.float32) * 3.0, rng.standard_normal(320).astype(np.float32) * 0.7]
    z = rng.standard_normal(320).astype(np.float32)
    z[[5, 77, 200]] = [np.nan, np.inf, -np.inf]
    out.append(z)
    z = rng.standard_normal(320).astype(np.float32)
    z[[10, 250]] = 9.0  # a tie: the first index wins the greedy pick
    out.append(z)
    out.append(np.full(320, -3.0, np.float32))  # flat: every token equally likely
    return np.stack(out)


def sampling_main():
    """sampling_ref.npz: the reference's sample_token (gsd_lq_cpu_runtime.py:422-443) under np.random.seed(s)."""
    sys.path.insert(0, os.path.join(reference_tree(), "gsd_lq_v2"))
    import gsd_lq_cpu_runtime as R

    logits = sampling_logits()
    picks = np.zeros((len(logits), len(SAMPLING_CASES), len(SAMPLING_SEEDS)), np.int64)
    for i, lg in enumerate(logits):
        for j, (t, p) in enumerate(SAMPLING_CASES):
            for k, seed in enumerate(SAMPLING_SEEDS):
                np.random.seed(seed)
                picks[i, j, k] = R.CPUMistralV2Model.sample_token(None, lg.copy(), temperature=t, top_p=p)
    np.savez(os.path.join(HERE, "sampling_ref.npz"), logits=logits, cases=np.array(SAMPLING_CASES),
             seeds=np.array(list(SAMPLING_SEEDS)), picks=picks)
    print("sampling picks", picks.shape)


def tokenizer_vocab():
    """A SentencePiece-style test vocabulary: control tokens, the 256 byte tokens, single characters and
    merged pieces with seeded scores, including equal scores (leftmost-merge ties), a NaN and a -inf score
    (never merged) and one string listed twice (its last id wins)."""
    rng = np.random.default_rng(21)
    toks = ["<unk>", "<s>", "</s>", "[INST]", "[/INST]", "<<SYS>>"]
    types = [2, 3, 3, 3, 3, 3]
    toks += [f"<0x{b:02X}>" for b in range(256)]
    types += [6] * 256
    chars = list("\u2581abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789.,!?'-:()é")
    toks += chars
    types += [1] * len(chars)
    pieces = ["\u2581t", "th", "\u2581th", "he", "\u2581the", "in", "ing", "\u2581a", "an", "\u2581an", "nd",
              "\u2581and", "er", "re", "on", "\u2581o", "\u2581of", "ll", "\u2581he", "\u2581hel", "\u2581hell",
              "\u2581hello", "lo", "llo", "wor", "\u2581w", "\u2581wor", "\u2581world", "or", "ld", "aa", "aaa",
              "\u2581\u2581", "\u2581\u2581\u2581\u2581", "es", "est", "\u2581t\u00e9", "\u00e9s", "ab", "bc",
              "abc", "ab", "IN", "ST", "\u2581[", "12", "123", "\u25811"]
    scores = [0.0] * len(toks)
    psc = list(np.round(rng.uniform(-12.0, -1.0, len(pieces)), 1))
    psc[pieces.index("th")] = psc[pieces.index("he")]    # a tie between overlapping pairs
    psc[pieces.index("bc")] = float("nan")               # never merged
    psc[pieces.index("ld")] = float("-inf")              # never merged
    toks += pieces
    types += [1] * len(pieces)
    scores += [float(x) for x in psc]
    return {"tokens": toks, "scores": scores, "token_types": types, "bos_id": 1, "eos_id": 2}


TOKENIZER_TEXTS = [
    "hello world", " hello world", "Hello World!", "the thing and the other", "  two  spaces", "",
    " ", "aaaaaaa", "abcabc abc", "[INST] hello [/INST] the end", "<s>the</s>", "[INST][/INST]",
    "t\u00e9s est", "price: 12\u20ac (123)", "emoji \U0001F600 ok", "tab\there\nnewline", "<<SYS>>of<<SYS>>",
    "inging ing in", "x" * 40, "\u2581already marked",
]


def tokenizer_main():
    """tokenizer_ref.json: the reference's MistralSentencePieceTokenizer (run_gpu_native_chat.py:660-729)
    on tokenizer_vocab(): encode of each text (with and without BOS) and decode of fixed id lists."""
    import json
    sys.path.insert(0, os.path.join(reference_tree(), "gsd_lq_v2"))
    import run_gpu_native_chat as RG

    v = tokenizer_vocab()
    tk = RG.MistralSentencePieceTokenizer(v["tokens"], v["scores"], v["token_types"], v["bos_id"], v["eos_id"])
    enc = [[t, tk.encode(t), tk.encode(t, add_bos=False)] for t in TOKENIZER_TEXTS]
    rng = np.random.default_rng(5)
    id_lists = [e[1] for e in enc]
    id_lists += [[int(i) for i in rng.integers(0, len(v["tokens"]), 12)] for _ in range(6)]
    id_lists += [[1, 6 + 0xE2, 6 + 0x82, 6 + 0xAC, 2], [6 + 0xE2, 6 + 0x82], [6 + 0xC3, 6 + 0xA9, 270, 2]]
    dec = [[ids, tk.decode(ids)] for ids in id_lists]
    with open(os.path.join(HERE, "tokenizer_ref.json"), "w", encoding="utf-8") as f:
        json.dump({"vocab": v, "encode": enc, "decode": dec}, f, ensure_ascii=False)
    print("tokenizer cases", len(enc), len(dec))


CHAT_SYSTEM = "Test rules: answer briefly.\nSecond line."
CHAT_HISTORIES = [
    [],
    [["hi", "Hello!"]],
    [["first question", "first answer"], ["second", "reply with \"quotes\" and </s> inside"]],
    [["a", ""], ["", "b"], ["x y z", "  padded  "]],
]
CHAT_MESSAGES = ["What is 2+2?", "", "multi\nline [INST] message"]


def chat_main():
    """chat_prompt_ref.json: the reference's format_mistral_prompt (run_gpu_native_chat.py:996-1013) over
    fixed histories and messages, in both of its layouts.  Its module-level rules text is replaced by
    CHAT_SYSTEM for the recording, so no text of the reference's own ends up in the fixture."""
    import json
    sys.path.insert(0, os.path.join(reference_tree(), "gsd_lq_v2"))
    import run_gpu_native_chat as RG

    RG.SYSTEM_RULES = CHAT_SYSTEM
    cases = []
    for h in CHAT_HISTORIES:
        for msg in CHAT_MESSAGES:
            hist = [tuple(t) for t in h]
            cases.append({"history": h, "message": msg,
                          "lightweight": RG.format_mistral_prompt(hist, msg, is_cpu=True),
                          "with_system": RG.format_mistral_prompt(hist, msg, is_cpu=False)})
    with open(os.path.join(HERE, "chat_prompt_ref.json"), "w", encoding="utf-8") as f:
        json.dump({"system": CHAT_SYSTEM, "cases": cases}, f, ensure_ascii=False, indent=0)
    print("chat prompt cases", len(cases))


if __name__ == "__main__":
    if sys.argv[1:] == ["sampling"]:
        sampling_main()
    elif sys.argv[1:] == ["tokenizer"]:
        tokenizer_main()
    elif sys.argv[1:] == ["chat"]:
        chat_main()
    else:
        main()
        sampling_main()
        tokenizer_main()
        chat_main()

"""Synthetic tokenizer.json files for the tokenizer and CLI tests (test
helper): vocabularies that mix plain pieces, SentencePiece "▁" and
byte-level "Ġ" word starts, "</w>" word ends, "##" continuations, multi-byte
UTF-8 and added tokens (special flagged 1 and true), with shuffled ids; and
random texts over them."""

import json

import numpy as np

SPM, GPT = "▁", "Ġ"
WORDS = ["the", "quick", "brown", "fox", "jump", "jumps", "over", "lazy", "dog", "deep", "seek", "infer", "token",
         "izer", "model", "gpu", "b200", "ten", "sor", "tensor", "a", "an", "in", "on", "at", "is", "it"]
UTF8 = ["é", "日本", "語", "ü", "ß"]
VARIANT_ONLY = {"zebra": SPM + "zebra", "yak": GPT + "yak", "wolf": "wolf</w>", "owl": SPM + "owl"}  # no plain form
SPACES = [" ", "  ", "\t", "\n", "\r\n", "\x0b", "\x0c"]
PUNCT = list(".,;:!?'\"-()[]")
BOOL_SPECIAL = 9  # flagged "special": true


def make_tokenizer(path, seed=0, root_ids=False, min_ids=0):
    """Write tokenizer.json; min_ids pads the vocabulary with filler pieces so
    that every id a model of that vocabulary size emits decodes."""
    rng = np.random.default_rng(seed)
    pieces = set("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789") | set(PUNCT)
    extra = ["".join(rng.choice(list("abcdefghijklmnopqrstuvwxyz"), size=int(rng.integers(2, 9)))) for _ in range(300)]
    for w in WORDS + extra:
        pieces.add(w)
        for form, keep in ((SPM + w, 0.6), (GPT + w, 0.4), (w + "</w>", 0.3), ("##" + w, 0.3)):
            if rng.random() < keep:
                pieces.add(form)
    for u in UTF8:
        pieces.add(u)
        pieces.add(SPM + u)
    pieces |= set(VARIANT_ONLY.values()) | {"##zebra", "##yak"}
    pieces = sorted(pieces)
    pieces += [f"<filler_{i}>" for i in range(max(0, min_ids - len(pieces)))]
    ids = rng.permutation(len(pieces))
    vocab = {p: int(i) for p, i in zip(pieces, ids)}
    added = [
        {"id": 7, "content": "<s>", "special": 1},
        {"id": BOOL_SPECIAL, "content": "</s>", "special": True},
        {"id": 11, "content": "override", "special": False},
        {"id": len(pieces) + 5, "content": "<beyond>", "special": 1},  # past the vocabulary: special only
    ]
    doc = {"version": "1.0", "added_tokens": added, "model": {"type": "BPE", "vocab": vocab, "unk_token_id": None}}
    if root_ids:
        doc["bos_token_id"], doc["eos_token_id"] = 3, 4
    with open(path, "w", encoding="utf-8") as f:
        json.dump(doc, f, ensure_ascii=bool(seed % 2))  # both escaped and raw UTF-8 JSON
    return vocab


def random_text(rng, n_words):
    out = []
    for _ in range(n_words):
        r = rng.random()
        if r < 0.45:
            out.append(str(rng.choice(WORDS)))
        elif r < 0.55:
            out.append(str(rng.choice(list(VARIANT_ONLY))))
        elif r < 0.7:
            out.append("".join(rng.choice(list("abcdefghijklmnopqrstuvwxyzXYZ0123"), size=int(rng.integers(1, 7)))))
        elif r < 0.8:
            out.append(str(rng.choice(UTF8)))
        elif r < 0.9:
            out.append(str(rng.choice(PUNCT)))
        else:
            out.append("<s>" if rng.random() < 0.5 else "</s>")
        out.append(str(rng.choice(SPACES)) if rng.random() < 0.8 else "")
    return "".join(out)



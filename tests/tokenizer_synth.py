"""A seeded synthetic tokenizer.bin in the reference's format
(dev/host/export_tokenizer.py:1-10): [u32 max_len] then per token
[f32 score][u32 len][bytes]. Ids 0-2 are <unk>, BOS, EOS as in llama2.c;
3..258 are the <0xHH> byte pieces the encoder falls back to; then single
characters and seeded multi-character merges with seeded scores."""
import struct

import numpy as np


def make_tokenizer(vocab_size=1024, seed=7):
    rng = np.random.default_rng(seed)
    pieces = ["<unk>", "\n<s>\n", "\n</s>\n"] + [f"<0x{b:02X}>" for b in range(256)]
    chars = [" "] + [chr(c) for c in range(ord("a"), ord("z") + 1)] + \
            [chr(c) for c in range(ord("A"), ord("Z") + 1)] + list(".,!?'")
    pieces += chars
    seen = set(pieces)
    letters = "etaoinshrdlu "
    while len(pieces) < vocab_size:
        n = int(rng.integers(2, 6))
        s = "".join(letters[int(i)] for i in rng.integers(0, len(letters), n))
        if s not in seen:
            seen.add(s)
            pieces.append(s)
    scores = np.zeros(vocab_size, np.float32)
    scores[259:] = -rng.random(vocab_size - 259).astype(np.float32) * 10.0
    enc = [p.encode("utf-8") for p in pieces]
    out = bytearray(struct.pack("I", max(len(e) for e in enc)))
    for e, sc in zip(enc, scores):
        out += struct.pack("fI", float(sc), len(e)) + e
    return bytes(out), pieces

"""Write tests/golden/tokenizer_toy.mmtok: a small synthetic tokenizer in the reference's
tokenizer.mmtok format (matmulfreellmCPU tools/provision.py:171-219), for the text-mode tests.

No real tokenizer.mmtok exists offline (the reference packs one from a downloaded HF
tokenizer.json), so this one is trained here, deterministically, by plain byte-pair merging
over a fixed corpus: pieces are <unk> <s> </s>, the 256 byte tokens <0x00>..<0xFF>, the
code points of the corpus (with the word boundary U+2581), then one piece per merge, in rank
order. 1,000 pieces in all, below the "small" test model's 2,048-id vocabulary. Some code
points (an emoji, CJK outside the corpus) are deliberately absent, so encoding them takes
the byte-fallback path.

    python tests/golden/make_tokenizer.py
"""
from __future__ import annotations

import collections
import os
import struct

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tokenizer_toy.mmtok")
SP = "▁"
N_PIECES = 1000

CORPUS = """
The quick brown fox jumps over the lazy dog. A matmul-free language model replaces every
dense projection with a ternary one, and its token mixer is a gated linear recurrence.
Once upon a time, there was a little model that ran on a big GPU. It read the weights once
per token and wrote one token at a time. The recurrent state stayed in memory between steps.
Numbers like 1024, 2048, 5632 and 32000 appear in configurations; so do 370M, 1.3B and 2.7B.
Café crème, naïve façade, über Straße -- ëxtra diacritics for the multi-byte path.
中文 文本 测试 -- a few CJK characters, repeated: 中文 文本.
""" * 3


def train():
    words = collections.Counter()
    for line in CORPUS.strip().splitlines():
        text = SP + line.replace(" ", SP)
        for w in text.split(SP):
            if w:
                words[SP + w] += 1
    chars = sorted({c for w in words for c in w})
    pieces = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + chars
    seqs = {w: list(w) for w in words}
    merges = []
    have = set(pieces)
    while len(pieces) < N_PIECES:
        pairs = collections.Counter()
        for w, n in words.items():
            s = seqs[w]
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += n
        if not pairs:
            break
        # most frequent pair; ties by the pair's text, so the order is deterministic
        (a, b), _ = min(pairs.items(), key=lambda kv: (-kv[1], kv[0]))
        merges.append(f"{a} {b}")
        if a + b not in have:
            pieces.append(a + b)
            have.add(a + b)
        for w in words:
            s, i, out = seqs[w], 0, []
            while i < len(s):
                if i + 1 < len(s) and s[i] == a and s[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[w] = out
    return pieces, merges


def write(path: str) -> str:
    pieces, merges = train()
    with open(path, "wb") as f:
        f.write(b"MMTOK1\n\x00")
        f.write(struct.pack("<II", len(pieces), len(merges)))
        f.write(struct.pack("<iii", 1, 2, 0))  # bos, eos, unk
        for p in pieces + merges:
            b = p.encode("utf-8")
            f.write(struct.pack("<I", len(b)))
            f.write(b)
    return path


if __name__ == "__main__":
    print(write(OUT))

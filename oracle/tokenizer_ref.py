"""CPU restatement of the text I/O of aion_b200/csrc/aion_tok.c (the
llama2.c tokenizer.bin format and its byte-pair encoding), the checker for
the library's encoder.  Test infrastructure only; the reference itself has
no tokenizer (token ids only, src/kernel_simd.c:1245)."""
from __future__ import annotations

import struct

import numpy as np


def write_tokenizer(path, pieces: list[bytes], scores) -> None:
    """tokenizer.bin: int32 max_token_length, then per token float32 score,
    int32 length, bytes."""
    with open(path, "wb") as f:
        f.write(struct.pack("<i", max(len(p) for p in pieces)))
        for p, s in zip(pieces, scores):
            f.write(struct.pack("<fi", float(s), len(p)))
            f.write(p)


def encode(pieces: list[bytes], scores, text: str, bos: bool = True, eos: bool = False) -> list[int]:
    lookup = {p: i for i, p in enumerate(pieces)}
    sc = np.asarray(scores, np.float32)
    toks = [1] if bos else []
    raw = text.encode("utf-8")
    if raw and b" " in lookup:
        toks.append(lookup[b" "])
    i = 0
    while i < len(raw):
        j = i + 1
        while j < len(raw) and (raw[j] & 0xC0) == 0x80 and j - i < 4:
            j += 1
        cp = raw[i:j]
        if cp in lookup:
            toks.append(lookup[cp])
        else:
            toks.extend(b + 3 for b in cp)
        i = j
    first = 1 if bos else 0
    while True:
        best, best_id, best_k = np.float32(-1e10), -1, -1
        for k in range(first, len(toks) - 1):
            m = pieces[toks[k]] + pieces[toks[k + 1]]
            if m in lookup and sc[lookup[m]] > best:
                best, best_id, best_k = sc[lookup[m]], lookup[m], k
        if best_k < 0:
            break
        toks[best_k:best_k + 2] = [best_id]
    if eos:
        toks.append(2)
    return toks


def decode(pieces: list[bytes], tokens) -> bytes:
    out, prev = b"", -1
    for t in tokens:
        if t not in (1, 2):
            p = pieces[t]
            if prev == 1 and p.startswith(b" "):
                p = p[1:]
            if len(p) == 6 and p.startswith(b"<0x") and p.endswith(b">"):
                p = bytes([int(p[3:5], 16)])
            out += p
        prev = t
    return out

"""Seeded synthetic tokenizers for the tokenizer, sampler and infer_ffi tests
(no network, no real vocabularies): a byte-level BPE vocabulary learned from
a generated corpus, written in the three forms the reference reads: GGUF
metadata (tokenizer.ggml.*), tokenizer.json and tokenizer.bin.
"""
from __future__ import annotations

import json
import struct
from collections import Counter
from pathlib import Path

import numpy as np

import tokenizer_ref as tr

SYLLABLES = ["ka", "lo", "mi", "ne", "ru", "ta", "shi", "von", "der", "an", "el", "is", "to", "ing", "er", "qu"]
EXTRA_WORDS = ["user", "assistant", "system", "hello", "world"]
UNICODE_BITS = ["é", "ß", "ñ", "Ωμέγα", "привет", "日本語", "😀", "٣٤", "Ⅻ", "café", "naïve"]
PUNCT = [".", ",", "!", "?", "'s", "'ll", "'ve", "'re", "'d", "--", "(", ")", "\"", "#", "$5", "3.14", "\t", "\n"]


def corpus(seed: int, n_words: int = 1500) -> str:
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_words):
        r = rng.random()
        if r < 0.7:
            w = "".join(rng.choice(SYLLABLES, size=int(rng.integers(1, 4))))
            if rng.random() < 0.15:
                w = w.capitalize()
        elif r < 0.8:
            w = str(int(rng.integers(0, 10000)))
        elif r < 0.88:
            w = str(rng.choice(UNICODE_BITS))
        elif r < 0.95:
            w = str(rng.choice(PUNCT))
        else:
            w = str(rng.choice(EXTRA_WORDS))
        out.append(w)
        out.append(" " if rng.random() < 0.9 else str(rng.choice(["  ", "\n", " \t"])))
    return "".join(out)


def learn_bpe(text: str, n_merges: int, chain_words=EXTRA_WORDS[:3]) -> tuple[list[str], list[str]]:
    """Byte-level BPE: 256 byte symbols (GPT-2 characters, in byte order), then
    merges that make each chain word a single token (highest priority), then
    merges learned by pair frequency over the GPT-2 pre-split corpus."""
    table = tr.gpt2_byte_table()
    vocab = list(table)
    merges: list[str] = []
    have = set(vocab)

    def add_merge(a: str, b: str) -> None:
        merges.append(f"{a} {b}")
        if a + b not in have:
            have.add(a + b)
            vocab.append(a + b)

    for w in chain_words:
        syms = [table[b] for b in w.encode()]
        cur = syms[0]
        for s in syms[1:]:
            add_merge(cur, s)
            cur = cur + s
    words = Counter(tr._GPT2.findall(text))
    seqs = {w: [table[b] for b in w.encode()] for w in words}
    while len(merges) < n_merges:
        pairs: Counter = Counter()
        for w, c in words.items():
            s = seqs[w]
            for i in range(len(s) - 1):
                pairs[(s[i], s[i + 1])] += c
        if not pairs:
            break
        (a, b), _ = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        add_merge(a, b)
        for w in words:
            s = seqs[w]
            i, out = 0, []
            while i < len(s):
                if i + 1 < len(s) and s[i] == a and s[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[w] = out
    return vocab, merges


def llama_vocab(vocab: list[str], size: int = 128256) -> list[str]:
    """Pads a learned vocabulary to a Llama-3-sized one with the special
    tokens at their Llama-3 ids (begin/end of text, headers, eot)."""
    out = list(vocab) + [f"<|reserved_{i}|>" for i in range(128000 - len(vocab))]
    specials = {128000: "<|begin_of_text|>", 128001: "<|end_of_text|>", 128006: "<|start_header_id|>",
                128007: "<|end_header_id|>", 128009: "<|eot_id|>"}
    for i in range(128000, size):
        out.append(specials.get(i, f"<|reserved_special_token_{i - 128000}|>"))
    return out


# ---------------------------------------------------------------- GGUF --
def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_str(k, v):
    return _s(k) + struct.pack("<I", 8) + _s(v)


def _kv_u32(k, v):
    return _s(k) + struct.pack("<II", 4, v)


def _kv_bool(k, v):
    return _s(k) + struct.pack("<IB", 7, 1 if v else 0)


def _kv_strs(k, vs):
    return _s(k) + struct.pack("<IIQ", 9, 8, len(vs)) + b"".join(_s(v) for v in vs)


def tokenizer_kvs(tokens, merges, bos, eos, pre="gpt2", add_bos=None, add_space=None, template=None) -> list:
    kvs = [_kv_str("tokenizer.ggml.model", "gpt2"), _kv_strs("tokenizer.ggml.tokens", tokens),
           _kv_strs("tokenizer.ggml.merges", merges), _kv_u32("tokenizer.ggml.bos_token_id", bos),
           _kv_u32("tokenizer.ggml.eos_token_id", eos), _kv_str("tokenizer.ggml.pre", pre)]
    if add_bos is not None:
        kvs.append(_kv_bool("tokenizer.ggml.add_bos_token", add_bos))
    if add_space is not None:
        kvs.append(_kv_bool("tokenizer.ggml.add_space_prefix", add_space))
    if template is not None:
        kvs.append(_kv_str("tokenizer.chat_template", template))
    return kvs


def write_gguf_tokenizer(path, tokens, merges, bos, eos, **kw) -> str:
    """A GGUF v3 file holding only metadata (enough for yl_tokenizer_load)."""
    kvs = [_kv_str("general.architecture", "llama")] + tokenizer_kvs(tokens, merges, bos, eos, **kw)
    Path(path).write_bytes(struct.pack("<IIQQ", 0x46554747, 3, 0, len(kvs)) + b"".join(kvs))
    return str(path)


def retokenize_gguf(src, dst, tokens, merges, bos, eos, **kw) -> str:
    """Copies a model GGUF, replacing its tokenizer metadata (tensor offsets
    are relative to the aligned data section, so they stay valid)."""
    d = Path(src).read_bytes()
    magic, ver, n_t, n_kv = struct.unpack_from("<IIQQ", d, 0)
    off = 24
    keep = []
    align = 32
    for _ in range(n_kv):
        start = off
        n, = struct.unpack_from("<Q", d, off)
        key = d[off + 8:off + 8 + n].decode()
        ty, = struct.unpack_from("<I", d, off + 8 + n)
        val, off = tr._gg_read(d, off + 12 + n, ty)
        if key == "general.alignment":
            align = int(val)
        if not key.startswith("tokenizer."):
            keep.append(d[start:off])
    tstart = off
    for _ in range(n_t):  # tensor infos: name, n_dims, dims, type, offset
        n, = struct.unpack_from("<Q", d, off)
        off += 8 + n
        nd, = struct.unpack_from("<I", d, off)
        off += 4 + 8 * nd + 4 + 8
    tinfo = d[tstart:off]
    data_start = (off + align - 1) // align * align
    kvs = keep + tokenizer_kvs(tokens, merges, bos, eos, **kw)
    head = struct.pack("<IIQQ", magic, ver, n_t, len(kvs)) + b"".join(kvs) + tinfo
    head += b"\0" * ((-len(head)) % align)
    Path(dst).write_bytes(head + d[data_start:])
    return str(dst)


def write_tokenizer_json(path, vocab: list[str], merges: list[str], added: dict[int, str]) -> str:
    obj = {"model": {"type": "BPE", "vocab": {t: i for i, t in enumerate(vocab) if i not in added},
                     "merges": merges},
           "added_tokens": [{"id": i, "content": c} for i, c in sorted(added.items())]}
    Path(path).write_text(json.dumps(obj, ensure_ascii=False), encoding="utf-8")
    return str(path)


def write_tokenizer_bin_vocab(path, vocab: list[str], scores: list[float], bos: int, eos: int) -> str:
    out = bytearray(struct.pack("<IIII", len(vocab), max(len(v.encode()) for v in vocab), bos, eos))
    for t, sc in zip(vocab, scores):
        b = t.encode()
        out += struct.pack("<fI", sc, len(b)) + b
    Path(path).write_bytes(bytes(out))
    return str(path)


def random_texts(seed: int, n: int) -> list[str]:
    """Texts over the corpus alphabet plus characters outside it."""
    rng = np.random.default_rng(seed)
    pieces = SYLLABLES + EXTRA_WORDS + UNICODE_BITS + PUNCT + [" ", "  ", "　", " ", "x'y", "'", "'S", "Z"]
    out = []
    for _ in range(n):
        k = int(rng.integers(1, 24))
        out.append("".join(str(rng.choice(pieces)) + (" " if rng.random() < 0.5 else "") for _ in range(k)))
    return out

"""Test infrastructure only: a Python restatement of the reference's tokenizer
(src_llm/tokenizer.rs) and sampler (src_llm/sampler.rs), the checker for the
C++ tokenizer and the device sampler of the product library. Nothing in the
product imports this file.

The GPT-2 pre-tokenizer split uses the `regex` module with the reference's
pattern (tokenizer.rs:28-30), an implementation independent of the product's
hand-written matcher. Chat templates: the reference renders them with
minijinja 2.20.0 (Cargo.lock), which is not installed here; jinja2 3.1.6
stands in, set to minijinja's defaults where the two differ on the cases the
tests render (see _MiniJinjaDefaults), so the C++ renderer is checked against
an independent Jinja implementation rather than against minijinja itself. Sums the reference chains in f32 (softmax denominator,
top-p cumulative sum, cdf) are taken with numpy's sequential float32
accumulate, which rounds after every addition like the reference's loops.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import jinja2
import numpy as np
import regex
from jinja2.sandbox import SandboxedEnvironment

GPT2_PATTERN = r"'(?:[sdmt]|ll|ve|re)| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+"
_GPT2 = regex.compile(GPT2_PATTERN)


def gpt2_byte_table() -> list[str]:
    """build_gpt2_byte_table (tokenizer.rs:55-76)."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    cs = list(bs)
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    table = [""] * 256
    for b, c in zip(bs, cs):
        table[b] = chr(c)
    return table


class Tokenizer:
    def __init__(self, vocab: list[str], scores: list[float], bos: int, eos: int, byte_level: bool,
                 pre: str = "default", add_bos_token: bool = True, add_space_prefix: bool = False):
        self.vocab = vocab
        self.scores = np.asarray(scores, np.float32)
        self.bos, self.eos = bos, eos
        self.byte_level = byte_level
        self.pre = pre
        self.add_bos_token = add_bos_token
        self.add_space_prefix = add_space_prefix
        # binary search over the text-sorted vocabulary (stable sort): the last
        # of equal texts, i.e. the highest id
        self.index = {}
        for i, t in enumerate(vocab):
            self.index[t] = i
        if byte_level:
            table = gpt2_byte_table()
            self.byte_to_token = [0] * 256
            self.token_to_byte = [None] * max(len(vocab), 256)
            self.char_to_byte = {}
            for b in range(256):
                c = table[b]
                self.char_to_byte[c] = b
                tid = self.index.get(c)
                if tid is not None:
                    self.byte_to_token[b] = tid
                    self.token_to_byte[tid] = b
        else:
            self.byte_to_token = [b + 3 for b in range(256)]

    # ---- constructors ----
    @classmethod
    def from_gguf_parts(cls, vocab, merges, bos, eos, pre="default", add_bos=True, add_space=False):
        """tokenizer.rs:78-132"""
        scores = [0.0] * len(vocab)
        idx = {t: i for i, t in enumerate(vocab)}
        for i, m in enumerate(merges):
            parts = m.split(" ", 1)
            if len(parts) == 2:
                j = idx.get(parts[0] + parts[1])
                if j is not None:
                    scores[j] = float(np.float32(len(merges) - i))
        return cls(list(vocab), scores, bos, eos, True, pre, add_bos, add_space)

    @classmethod
    def from_json(cls, path: str):
        """tokenizer.rs:134-217"""
        root = json.loads(Path(path).read_text(encoding="utf-8"))
        vocab_obj = root["model"]["vocab"]
        added = root["added_tokens"]
        max_id = max([int(v) for v in vocab_obj.values()] + [int(t["id"]) for t in added] + [0])
        vocab = [""] * (max_id + 1)
        for k in sorted(vocab_obj):  # serde_json's map iterates keys in sorted order
            vocab[int(vocab_obj[k])] = k
        for t in added:
            vocab[int(t["id"])] = t["content"]
        tok = cls.from_gguf_parts(vocab, root["model"]["merges"], 128000, 128009)
        for t in added:
            if t["content"] == "<|begin_of_text|>":
                tok.bos = int(t["id"])
            if t["content"] in ("<|end_of_text|>", "<|eot_id|>"):
                tok.eos = int(t["id"])
        return tok

    @classmethod
    def from_bin(cls, path: str):
        """tokenizer.rs:219-262 (lm.rs tokenizer.bin)"""
        d = Path(path).read_bytes()
        n, = struct.unpack_from("<I", d, 0)
        bos, eos = struct.unpack_from("<II", d, 8)
        off = 16
        vocab, scores = [], []
        for _ in range(n):
            sc, ln = struct.unpack_from("<fI", d, off)
            off += 8
            vocab.append(d[off:off + ln].decode("utf-8"))
            scores.append(sc)
            off += ln
        return cls(vocab, scores, bos, eos, False)

    @classmethod
    def from_gguf(cls, path: str):
        kv = read_gguf_metadata(path)
        tok = cls.from_gguf_parts(kv["tokenizer.ggml.tokens"], kv.get("tokenizer.ggml.merges", []),
                                  kv.get("tokenizer.ggml.bos_token_id", 128000),
                                  kv.get("tokenizer.ggml.eos_token_id", 128009),
                                  kv.get("tokenizer.ggml.pre", "default"),
                                  kv.get("tokenizer.ggml.add_bos_token", True),
                                  kv.get("tokenizer.ggml.add_space_prefix", False))
        tok.chat_template = kv.get("tokenizer.chat_template")  # transformer_llama_gguf.rs:634-641
        return tok

    # ---- encode / decode ----
    def has_llama_tokens(self) -> bool:
        return len(self.vocab) > 128009

    def _byte_encode(self, text: str) -> list[int]:
        return [self.byte_to_token[b] for b in text.encode("utf-8")]

    def _bpe_merge(self, toks: list[int]) -> None:
        """tokenizer.rs:306-336"""
        while True:
            best_score, best_id, best_idx = np.float32(-1e10), 0, -1
            for i in range(len(toks) - 1):
                j = self.index.get(self.vocab[toks[i]] + self.vocab[toks[i + 1]])
                if j is not None and self.scores[j] > best_score:
                    best_score, best_id, best_idx = self.scores[j], j, i
            if best_idx < 0:
                return
            toks[best_idx] = best_id
            del toks[best_idx + 1]

    def encode(self, text: str, bos: bool = False, eos: bool = False) -> list[int]:
        """tokenizer.rs:338-392"""
        assert text, "Text to encode should not be empty"
        toks: list[int] = [self.bos] if bos else []
        if self.pre in ("gpt2", "smollm"):
            if self.add_space_prefix and not text.startswith(" "):
                text = " " + text
            for seg in _GPT2.findall(text):
                st = self._byte_encode(seg)
                self._bpe_merge(st)
                toks += st
        else:
            if self.byte_level:
                st = self._byte_encode(text)
            else:
                st = []
                for c in text:
                    j = self.index.get(c)
                    if j is not None:
                        st.append(j)
                    else:
                        st += [b + 3 for b in c.encode("utf-8")]
            self._bpe_merge(st)
            toks += st
        if eos:
            toks.append(self.eos)
        return toks

    def decode(self, ids) -> str:
        """tokenizer.rs:523-551"""
        V = len(self.vocab)
        if self.byte_level:
            out = bytearray()
            for t in ids:
                b = self.token_to_byte[t] if t < len(self.token_to_byte) else None
                if b is not None:
                    out.append(b)
                elif t < V:
                    for c in self.vocab[t]:
                        if c in self.char_to_byte:
                            out.append(self.char_to_byte[c])
                        else:
                            out += c.encode("utf-8")
            return utf8_lossy(bytes(out))
        return "".join(self.vocab[t] for t in ids if t < V)

    def _wrap_n_header(self, text: str, header: str, wrap: bool) -> list[int]:
        """encode_wrap_n_header (tokenizer.rs:268-297)"""
        if not self.has_llama_tokens():
            t = [self.bos] if wrap and self.add_bos_token else []
            return t + (self.encode(text) if text else [])
        t = [128000] if wrap else []
        if header:
            t += [128006] + self.encode(header) + [128007, 271]
        if text:
            t += self.encode(text)
        if wrap:
            t += [271, 128009]
        return t

    chat_template = None

    def encode_template_output(self, text: str) -> list[int]:
        """tokenizer.rs:438-473, literally: every vocabulary entry containing
        '<' (a later equal text replacing an earlier one), the longest that
        matches at each '<', the text up to the next '<' through encode()."""
        text_to_id = {}
        for tid, t in enumerate(self.vocab):
            if "<" in t:
                text_to_id[t] = tid
        entries = [(t.encode(), tid) for t, tid in text_to_id.items()]
        b = text.encode()
        out, pos = [], 0
        while pos < len(b):
            if b[pos] == 0x3C:
                best, best_len = None, 0
                for tb, tid in entries:
                    if b.startswith(tb, pos) and len(tb) > best_len:
                        best, best_len = tid, len(tb)
                if best is not None:
                    out.append(best)
                    pos += best_len
                    continue
            start = pos
            pos += 1
            while pos < len(b) and b[pos] != 0x3C:
                pos += 1
            out += self.encode(b[start:pos].decode())
        return out

    def render_chat(self, messages, add_generation_prompt: bool) -> list[int]:
        """render_chat_template (tokenizer.rs:418-436)"""
        if self.chat_template is None:
            return []
        text = render_chat_template_text(self.chat_template, messages, add_generation_prompt)
        return self.encode_template_output(text) if text else []

    def encode_wrap_n_header(self, text: str, header: str, wrap: bool) -> list[int]:
        """tokenizer.rs:277-297"""
        return self._wrap_n_header(text, header, wrap)

    def set_chat_template(self, template: str) -> None:
        """tokenizer.rs:408-416 (jinja2 parses it here, as minijinja would)"""
        render_chat_template_text(template, [], False)
        self.chat_template = template

    def apply_system_template(self, system: str) -> list[int]:
        """tokenizer.rs:477-495"""
        if self.chat_template is not None:
            return self.render_chat([("system", system)], False)
        if self.has_llama_tokens():
            return self._wrap_n_header(system, "system", True)
        return self.encode(system) if system else []

    def apply_turn_template(self, user: str, add_empty_assistant: bool) -> list[int]:
        """tokenizer.rs:497-539"""
        if self.chat_template is not None:
            msgs = [("user", user)] + ([("assistant", "")] if add_empty_assistant else [])
            out = self.render_chat(msgs, add_empty_assistant)
            if add_empty_assistant and out and out[-1] == 128009:
                out.pop()
            return out
        if self.has_llama_tokens():
            u, a = self.encode("user"), self.encode("assistant")
            assert len(u) == 1 and len(a) == 1
            t = [128006, u[0], 128007, 271] + self._wrap_n_header(user, "", False) + [128009]
            return t + ([128006, a[0], 128007, 271] if add_empty_assistant else [])
        return ([self.bos] if self.add_bos_token else []) + self.encode(user)

    def chat_prompt(self, user: str, system: str = "") -> list[int]:
        """The console's fresh prompt (main.rs:149-153, :173): with a chat
        template [bos] (and a given system prompt's apply_system_template),
        without one apply_system_template(system); then
        apply_turn_template(user, true)"""
        if self.chat_template is not None:
            t = [self.bos] if self.add_bos_token else []
            if system:
                t += self.apply_system_template(system)
        else:
            t = self.apply_system_template(system)
        return t + self.apply_turn_template(user, True)


class _MiniJinjaDefaults(SandboxedEnvironment):
    """jinja2 set to minijinja's default behaviour (the reference's renderer,
    tokenizer.rs:408-430) where the two differ: no Python methods on strings,
    lists and maps (minijinja without pycompat: an error when called, an
    undefined value when only looked up), and booleans / none printed as
    true / false / none. Undefined values, whitespace control, the dropped
    trailing newline and autoescape off are jinja2's defaults already."""

    def is_safe_attribute(self, obj, attr, value):
        if isinstance(obj, (str, list, tuple, dict)) and callable(value):
            return False
        return super().is_safe_attribute(obj, attr, value)


def _finalize(v):
    if v is True:
        return "true"
    if v is False:
        return "false"
    if v is None:
        return "none"
    return v


def render_chat_template_text(template: str, messages, add_generation_prompt: bool) -> str:
    """The render of tokenizer.rs:418-428: context {messages: [{role,
    content}], add_generation_prompt}; serde_json's map keeps the keys sorted,
    so each message iterates content before role."""
    env = _MiniJinjaDefaults(finalize=_finalize, undefined=jinja2.Undefined)
    msgs = [{"content": c, "role": r} for r, c in messages]
    return env.from_string(template).render(messages=msgs, add_generation_prompt=add_generation_prompt)


def utf8_lossy(b: bytes) -> str:
    """String::from_utf8_lossy: one U+FFFD per maximal ill-formed subpart
    (Python's 'replace' error handler follows the same Unicode practice)."""
    return b.decode("utf-8", errors="replace")


# ---------------------------------------------------------------- GGUF --
_GG_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


def _gg_read(d: bytes, off: int, ty: int):
    if ty in _GG_SCALAR:
        fmt = _GG_SCALAR[ty]
        return struct.unpack_from(fmt, d, off)[0], off + struct.calcsize(fmt)
    if ty == 8:
        n, = struct.unpack_from("<Q", d, off)
        return d[off + 8:off + 8 + n].decode("utf-8"), off + 8 + n
    if ty == 9:
        et, n = struct.unpack_from("<IQ", d, off)
        off += 12
        out = []
        for _ in range(n):
            v, off = _gg_read(d, off, et)
            out.append(v)
        return out, off
    raise ValueError(f"GGUF value type {ty}")


def read_gguf_metadata(path: str) -> dict:
    d = Path(path).read_bytes()
    magic, ver, n_t, n_kv = struct.unpack_from("<IIQQ", d, 0)
    assert magic == 0x46554747 and ver == 3
    off = 24
    kv = {}
    for _ in range(n_kv):
        n, = struct.unpack_from("<Q", d, off)
        key = d[off + 8:off + 8 + n].decode("utf-8")
        off += 8 + n
        ty, = struct.unpack_from("<I", d, off)
        kv[key], off = _gg_read(d, off + 4, ty)
    return kv


# -------------------------------------------------------------- sampler --
def random_f32(seed: int) -> np.float32:
    """sampler.rs:81-91 (the state is the seed itself; it never advances)"""
    m = (1 << 64) - 1
    s = seed & m
    s ^= s >> 12
    s ^= (s << 25) & m
    s ^= s >> 27
    r = ((s * 0x2545F4914F6CDD1D) & m) >> 32
    return np.float32(np.float32(r >> 8) / np.float32(16777216.0))


def exp_f32(x: np.ndarray) -> np.ndarray:
    """e^x rounded once to f32 (the correctly rounded exp the device uses)."""
    return np.exp(x.astype(np.float64)).astype(np.float32)


class Sampler:
    """sampler.rs:41-180 with its persistent probability_idx array."""

    def __init__(self, vocab_size: int, temperature: float, top_p: float, seed: int):
        self.V = vocab_size
        self.temperature = np.float32(temperature)
        self.top_p = np.float32(top_p)
        self.rand = random_f32(seed)
        self.prob = np.zeros(vocab_size, np.float32)
        self.index = np.zeros(vocab_size, np.int64)

    @staticmethod
    def argmax(p: np.ndarray) -> int:
        best, bv = 0, p[0]
        idx = np.flatnonzero(p > bv)
        if idx.size == 0:
            return 0
        m = p[idx].max()
        return int(idx[np.flatnonzero(p[idx] == m)[0]]) if m == m else 0

    def sample(self, logits: np.ndarray) -> int:
        x = np.asarray(logits, np.float32).copy()
        if self.temperature == 0:
            return self.argmax(x)
        x = (x / self.temperature).astype(np.float32)
        e = exp_f32((x - x.max()).astype(np.float32))
        s = np.add.accumulate(e, dtype=np.float32)[-1]
        p = (e / s).astype(np.float32)
        if self.top_p <= 0 or self.top_p >= 1:
            cdf = np.add.accumulate(p, dtype=np.float32)
            hit = np.flatnonzero(self.rand < cdf)
            return int(hit[0]) if hit.size else self.V - 1
        cutoff = np.float32(np.float32(1.0) - self.top_p) / np.float32(self.V - 1)
        keep = np.flatnonzero(p >= cutoff)
        n0 = keep.size
        assert n0 > 0
        self.prob[:n0] = p[keep]
        self.index[:n0] = keep
        order = np.argsort(-self.prob, kind="stable")  # the whole array, leftovers included
        self.prob = self.prob[order]
        self.index = self.index[order]
        cum = np.add.accumulate(self.prob[:n0], dtype=np.float32)
        over = np.flatnonzero(cum > self.top_p)
        last = int(over[0]) if over.size else n0 - 1
        r = np.float32(self.rand * cum[last])
        hit = np.flatnonzero(r < cum[:last + 1])
        return int(self.index[hit[0]]) if hit.size else int(self.index[last])

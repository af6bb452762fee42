"""The host parsers that take untrusted input (chat templates from model
files, tokenizer text and ids) built with AddressSanitizer and UBSan and run
over generated inputs: the test templates, random-expression templates,
thousands of mutations of them (truncations, deleted, doubled and inserted
characters, stray delimiters, broken escapes), texts with ill-formed UTF-8
spliced in, and random id lists with ids past the vocabulary. CPU only."""
from __future__ import annotations

import random
import shutil
import subprocess
from pathlib import Path

import pytest

import test_chat_template as tct
import tokenizer_files as tf
from test_loader_fuzz import gguf_fields, mutate_gguf_field

ROOT = Path(__file__).resolve().parents[1]
HOST = ROOT / "yallma3-mini-inference_b200" / "csrc" / "host"


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("san") / "sanitize_harness"
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
           f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(Path(__file__).parent / "sanitize_harness.cpp"),
           str(HOST / "chat_template.cpp"), str(HOST / "tokenizer.cpp"), str(HOST / "json.cpp"),
           str(HOST / "upload.cpp"), "-L/usr/local/cuda/lib64", "-lcudart", "-lpthread", "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if r.returncode != 0 and ("asan" in r.stderr.lower() or "ubsan" in r.stderr.lower()):
        pytest.skip("sanitizer runtime not available: " + r.stderr[-300:])
    assert r.returncode == 0, r.stderr[-3000:]
    return out


def run(harness, *args):
    env = {"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0", "UBSAN_OPTIONS": "print_stacktrace=1:halt_on_error=1",
           "PATH": "/usr/bin:/bin", "LD_LIBRARY_PATH": "/usr/local/cuda/lib64"}
    r = subprocess.run([str(harness), *map(str, args)], capture_output=True, text=True, timeout=600, env=env)
    report = r.stdout + r.stderr
    assert r.returncode == 0, report[-4000:]
    assert "AddressSanitizer" not in report and "runtime error" not in report, report[-4000:]
    return r.stdout


def test_chat_templates_under_sanitizers(harness, tmp_path):
    base = [tct.T_BLOCKS, tct.T_HEADERS, tct.T_HEADERS_NO_GEN, tct.T_EXPR, tct.T_SPACE]
    base += [t for t, _ in [("{{ bos_token + 'x' }}", 0), ("{{ messages[0].content.strip() }}", 0),
                            ("{% if true %}open", 0), ("{{ 'unterminated }}", 0), ("{% raw %}{{ x }}{% endraw %}", 0), ("{%- raw -%} a {%- endraw %}", 0)]]
    base += [tct._Gen(s).template() for s in range(600)]
    r = random.Random(5)
    junk = ["{{", "}}", "{%", "%}", "{#", "#}", "-", "+", "'", '"', "\\", "(", ")", "[", "]", "|", ".", ":",
            "\\u12", "\\ud800", "\\udc00", "é", "for", "endfor", "if", "is", "not", "in", "**", "//"]
    corpus = list(base)
    for _ in range(2500):
        t = r.choice(base)
        i = r.randrange(len(t))
        op = r.randint(0, 4)
        if op == 0:
            t = t[:i]
        elif op == 1:
            t = t[:i] + t[i + 1:]
        elif op == 2:
            t = t[:i] + t[i] * 2 + t[i + 1:]
        elif op == 3:
            t = t[:i] + r.choice(junk) + t[i:]
        else:
            t = t[:i] + chr(r.randint(32, 126)) + t[i:]
        corpus.append(t)
    f = tmp_path / "templates.txt"
    f.write_text("\n<<<SEP>>>\n".join(corpus), encoding="utf-8")
    out = run(harness, "templates", f)
    n, rendered = int(out.split()[1]), int(out.split()[3])
    assert n == len(corpus) and rendered > len(base)  # most of the unmutated ones render (twice)


def test_tokenizer_under_sanitizers(harness, tmp_path):
    vocab, merges = tf.learn_bpe(tf.corpus(7), 300)
    path = tf.write_gguf_tokenizer(tmp_path / "t.gguf", vocab + ["<|im_start|>", "<|im_end|>"], merges, 1, 2,
                                   add_bos=True, template=tct.T_BLOCKS)
    r = random.Random(9)
    bad = [b"\xff", b"\xc3", b"\xe6\x97", b"\xed\xa0\x80", b"a\x80b", b"\xf4\x90\x80\x80"]
    texts = []
    for t in tf.random_texts(13, 250):
        b = t.encode()
        if r.random() < 0.25:
            i = r.randrange(len(b) + 1)
            b = b[:i] + r.choice(bad) + b[i:]
        texts.append(b.replace(b"\x01", b""))
    f = tmp_path / "texts.bin"
    f.write_bytes(b"\x01".join(texts))
    out = run(harness, "tokenizer", path, f)
    assert int(out.split()[1]) == len(texts)


def _mutations(data: bytes, r: random.Random, n: int) -> list:
    out = []
    for _ in range(n):
        b = bytearray(data)
        op = r.randint(0, 3)
        if op == 0:  # truncate
            b = b[:r.randrange(len(b))]
        elif op == 1:  # flip bytes
            for _ in range(r.randint(1, 8)):
                b[r.randrange(len(b))] = r.randrange(256)
        elif op == 2:  # a huge or off-by-some little-endian length somewhere
            i = r.randrange(max(1, len(b) - 8))
            b[i:i + 8] = r.choice([b"\xff" * 8, b"\x00\x00\x00\x80\x00\x00\x00\x00",
                                   (len(b) + r.randint(-3, 3)).to_bytes(8, "little", signed=True)])
        else:  # cut a span out
            i = r.randrange(len(b))
            del b[i:i + r.randint(1, 64)]
        out.append(bytes(b))
    return out


def test_tokenizer_files_under_sanitizers(harness, tmp_path):
    """Corrupted GGUF metadata, tokenizer.json and tokenizer.bin files: every
    load returns (an error or a tokenizer), nothing reads out of bounds."""
    vocab, merges = tf.learn_bpe(tf.corpus(7), 200)
    gguf = Path(tf.write_gguf_tokenizer(tmp_path / "ok.gguf", vocab, merges, 1, 2, template=tct.T_BLOCKS))
    (tmp_path / "j").mkdir()
    jpath = Path(tf.write_tokenizer_json(tmp_path / "j" / "tokenizer.json", vocab, merges, {len(vocab): "<|eot_id|>"}))
    (tmp_path / "b").mkdir()
    bpath = Path(tf.write_tokenizer_bin_vocab(tmp_path / "b" / "tokenizer.bin", vocab, [0.0] * len(vocab), 1, 2))
    r = random.Random(21)
    paths = [gguf]
    raw = gguf.read_bytes()
    fields = gguf_fields(raw)
    muts = _mutations(raw, r, 300) + [mutate_gguf_field(raw, fields, r) for _ in range(300)]
    for i, data in enumerate(muts):
        p = tmp_path / f"m{i}.gguf"
        p.write_bytes(data)
        paths.append(p)
    for kind, src, name, ext in (("j", jpath, "tokenizer.json", ".safetensors"), ("b", bpath, "tokenizer.bin", ".lmrs")):
        for i, data in enumerate(_mutations(src.read_bytes(), r, 150)):
            d = tmp_path / f"{kind}{i}"
            d.mkdir()
            (d / name).write_bytes(data)
            paths.append(d / f"model{ext}")
    lst = tmp_path / "paths.txt"
    lst.write_text("\n".join(str(p) for p in paths))
    out = run(harness, "load", lst)
    assert int(out.split()[1]) == len(paths) and int(out.split()[3]) >= 1


def test_json_under_sanitizers(harness, tmp_path):
    """The JSON reader (config.json, tokenizer.json, safetensors headers) on
    valid documents and mutations of them: escapes, surrogate pairs and lone
    surrogates, numbers at the edges, nesting past the reader's limit."""
    import json
    r = random.Random(31)
    base = [json.dumps({"a": [1, 2.5, -3e-7, True, None, "x\u00e9\ud83d\ude00"], "b": {"c": "\\\"/\b\f\n\r\t"}}),
            '{"hidden_size": 4096, "rope_scaling": {"factor": 8.0, "rope_type": "llama3"}, "x": 1e308, "y": -0}',
            "[" * 70 + "]" * 70, "[" * 20 + "{}" + "]" * 20, '"\\ud800"', '"\\udc00x"', "18446744073709551616",
            "-9223372036854775809", "1.7976931348623157e309", '{"a":1,"a":2}', "[1,]", "{,}", '"unterminated']
    docs = list(base)
    junk = ["{", "}", "[", "]", ",", ":", '"', "\\", "\\u", "\\ud83d", "e", "-", ".", "0", "9", "null", "tru"]
    for _ in range(3000):
        t = r.choice(base)
        i = r.randrange(len(t) + 1)
        op = r.randint(0, 2)
        if op == 0:
            t = t[:i]
        elif op == 1:
            t = t[:i] + r.choice(junk) + t[i:]
        else:
            t = t[:i] + t[i + 1:]
        docs.append(t)
    f = tmp_path / "docs.bin"
    f.write_bytes(b"\x01".join(d.encode("utf-8", "surrogatepass") for d in docs))
    out = run(harness, "json", f)
    assert int(out.split()[1]) == len(docs) and int(out.split()[3]) >= 3

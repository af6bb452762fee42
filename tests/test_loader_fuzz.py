"""Corrupted model files through yl_load_transformer (CPU): GGUF, safetensors
(with its config.json) and lm.rs files with truncations, flipped bytes, and
huge or wrapped lengths and offsets, concentrated in the headers the loaders
parse. Every load must end with an error code (without a GPU a file that
still parses stops at the first CUDA call), never with a crash: the loads run
in a child process whose exit status is checked."""
from __future__ import annotations

import random
import subprocess
import sys
from pathlib import Path

import model_files as mf

ROOT = Path(__file__).resolve().parents[1]


def _mutate(data: bytes, span: int, r: random.Random) -> bytes:
    b = bytearray(data)
    hi = max(1, min(span, len(b)))
    op = r.randint(0, 4)
    if op == 0:
        return bytes(b[:r.randrange(len(b))])
    if op == 1:
        for _ in range(r.randint(1, 6)):
            b[r.randrange(hi)] = r.randrange(256)
    elif op == 2:  # a little-endian length or offset replaced
        i = r.randrange(max(1, hi - 8))
        b[i:i + 8] = r.choice([b"\xff" * 8, b"\xf0\xff\xff\xff\xff\xff\xff\xff", b"\x00\x00\x00\x80\x00\x00\x00\x00",
                               (len(b) + r.randint(-64, 64)).to_bytes(8, "little", signed=True)])
    elif op == 3:
        i = r.randrange(hi)
        del b[i:i + r.randint(1, 32)]
    else:  # a 4-byte field (counts, types, dims) replaced
        i = r.randrange(max(1, hi - 4))
        b[i:i + 4] = r.choice([b"\xff\xff\xff\xff", b"\x00\x00\x00\x00", b"\x00\x00\x01\x00", b"\x07\x00\x00\x00"])
    return bytes(b)


_GG_SIZES = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}


def gguf_fields(d: bytes) -> list:
    """(offset, width) of every length, count, type, dimension and offset
    field of a GGUF v3 header: the places a corrupted file hurts a reader."""
    out = [(8, 8), (16, 8)]
    off = 24
    n_t, n_kv = int.from_bytes(d[8:16], "little"), int.from_bytes(d[16:24], "little")

    def strf(o):
        out.append((o, 8))
        return o + 8 + int.from_bytes(d[o:o + 8], "little")

    def val(o, ty):
        if ty == 8:
            return strf(o)
        if ty == 9:
            out.append((o, 4))
            out.append((o + 4, 8))
            et, n = int.from_bytes(d[o:o + 4], "little"), int.from_bytes(d[o + 4:o + 12], "little")
            o += 12
            for _ in range(n):
                o = val(o, et)
            return o
        return o + _GG_SIZES[ty]

    for _ in range(n_kv):
        off = strf(off)
        out.append((off, 4))
        ty = int.from_bytes(d[off:off + 4], "little")
        off = val(off + 4, ty)
    for _ in range(n_t):
        off = strf(off)
        nd = int.from_bytes(d[off:off + 4], "little")
        out.append((off, 4))
        off += 4
        for k in range(nd):
            out.append((off + 8 * k, 8))
        off += 8 * nd
        out += [(off, 4), (off + 4, 8)]
        off += 12
    return out


def mutate_gguf_field(data: bytes, fields: list, r: random.Random) -> bytes:
    """One header field set to an extreme: all ones, a top bit, zero, or about
    the file's size (lengths and offsets that wrap or overrun)."""
    o, w = r.choice(fields)
    top = (1 << (8 * w)) - 1
    v = r.choice([top, top - r.randint(0, 64), 1 << (8 * w - 1), 0, len(data) + r.randint(-64, 64), 1 << 32])
    b = bytearray(data)
    b[o:o + w] = (v & top).to_bytes(w, "little")
    return bytes(b)


def test_corrupted_model_files_fail_cleanly(yl, tmp_path):
    r = random.Random(17)
    paths = []
    gguf = Path(yl.synth_preset("tiny", str(tmp_path / "base.gguf")))
    data = gguf.read_bytes()
    fields = gguf_fields(data)
    for i in range(400):
        p = tmp_path / f"g{i}.gguf"
        # metadata and tensor infos lead the file: half the cases hit a header field on purpose
        p.write_bytes(mutate_gguf_field(data, fields, r) if i % 2 else _mutate(data, 24 * 1024, r))
        paths.append(p)
    st = mf.write_safetensors(tmp_path / "st", mf.ST_SMALL, seed=3)
    st_data, cfg = st.read_bytes(), (st.parent / "config.json").read_bytes()
    hlen = 8 + int.from_bytes(st_data[:8], "little")
    for i in range(110):
        d = tmp_path / f"s{i}"
        d.mkdir()
        for f in st.parent.iterdir():
            if f.name not in ("model.safetensors", "config.json"):
                (d / f.name).write_bytes(f.read_bytes())
        if i % 2:
            (d / "model.safetensors").write_bytes(_mutate(st_data, hlen, r))
            (d / "config.json").write_bytes(cfg)
        else:
            (d / "model.safetensors").write_bytes(st_data)
            (d / "config.json").write_bytes(_mutate(cfg, len(cfg), r))
        paths.append(d / "model.safetensors")
    lm = mf.write_lmrs(tmp_path / "lm", mf.LMRS_SMALL, seed=4)
    lm_data = lm.read_bytes()
    for i in range(110):
        d = tmp_path / f"l{i}"
        d.mkdir()
        (d / "tokenizer.bin").write_bytes((lm.parent / "tokenizer.bin").read_bytes())
        (d / "model.lmrs").write_bytes(_mutate(lm_data, 256, r))  # the 256-byte header
        paths.append(d / "model.lmrs")
    lst = tmp_path / "paths.txt"
    lst.write_text("\n".join(map(str, paths)))
    child = (
        "import importlib, sys\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "yl = importlib.import_module('yallma3-mini-inference_b200')\n"
        f"paths = open({str(lst)!r}).read().split('\\n')\n"
        "loaded = failed = 0\n"
        "for p in paths:\n"
        "    try:\n"
        "        m = yl.load_transformer(p, max_ctx_len=64)\n"
        "        del m\n"
        "        loaded += 1\n"
        "    except yl.YlError:\n"
        "        failed += 1\n"
        "print(loaded, failed)\n")
    res = subprocess.run([sys.executable, "-c", child], capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, (res.returncode, res.stderr[-3000:])
    loaded, failed = map(int, res.stdout.split()[-2:])
    assert loaded + failed == len(paths)

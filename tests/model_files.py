"""Writers of seeded synthetic model files in the reference's two other
formats, for the loader tests (no network, no checkpoints: random-init
weights of the named shapes).

safetensors (transformer_llama_st.rs:41-372): `model.safetensors` with
config.json and tokenizer.bin beside it. Quantized projections are MLX affine
8-bit: `<stem>.weight` U32 [rows, cols/4] holding the u8 quants in order,
`<stem>.scales` and `<stem>.biases` F16 [rows, cols/group]; a value is
q * scale + bias. Norms are F16. Without a "quantization" section in
config.json the projections are plain F16 [rows, cols].

lm.rs (transformer_llama_lmrs.rs:56-439): magic "lmrs", u32 version, the
packed 47-byte TransformerArgs at byte 8, tensors from byte 256 (embedding,
attention norms, wq, wk, wv, wo of every layer, ffn norms, w1, w2, w3, final
norm; a Q8 tensor is its int8 quants then its f32 scales, one per 32).

Also restates, in numpy, the requantization the safetensors loader applies
(util.rs:451-518), for the CPU tests of the oracle's loader.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

ST_SMALL = dict(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                num_hidden_layers=2, vocab_size=384, rms_norm_eps=1e-5, rope_theta=500000.0,
                max_position_embeddings=512)
# attention width (8 heads x 64) twice the model width
ST_WIDE_ATT = dict(ST_SMALL, num_attention_heads=8, num_key_value_heads=4, head_dim=64)
LMRS_SMALL = dict(dim=256, hidden_dim=768, n_layers=2, n_heads=4, head_size=64, n_kv_heads=1, vocab_size=512,
                  seq_len=256, rms_norm_eps=1e-5, rope_theta=500000.0, group_size=32)


def write_tokenizer_bin(path: Path, vocab_size: int, bos: int, eos: int) -> None:
    """tokenizer.rs:223-250 layout: vocab_size, max token length, bos, eos,
    then per token a f32 score, a u32 length and its bytes."""
    out = bytearray(struct.pack("<IIII", vocab_size, 8, bos, eos))
    for i in range(vocab_size):
        t = f"t{i}".encode()
        out += struct.pack("<fI", float(i), len(t)) + t
    path.write_bytes(bytes(out))


def _affine(rng: np.random.Generator, rows: int, cols: int, gs: int, std: float):
    q = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    ng = rows * cols // gs
    scale = (std * np.sqrt(12.0) / 255.0 * rng.uniform(0.6, 1.4, ng)).astype(np.float16)
    bias = (-127.5 * scale.astype(np.float32) + rng.normal(0, std * 0.05, ng)).astype(np.float16)
    return q, scale.reshape(rows, cols // gs), bias.reshape(rows, cols // gs)


def write_safetensors(dirpath, cfg: dict, seed: int, quantized: bool = True, group_size: int = 32,
                      quant_type: str | None = None, tokenizer: str = "bin", std: float = 0.02) -> Path:
    """Writes config.json, model.safetensors and a tokenizer into dirpath;
    returns the .safetensors path."""
    d = Path(dirpath)
    d.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    dim, ffn, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    att = cfg["num_attention_heads"] * cfg["head_dim"]
    kvd = cfg["num_key_value_heads"] * cfg["head_dim"]
    tensors: dict[str, tuple[str, list, bytes]] = {}

    def proj(stem: str, rows: int, cols: int):
        if quantized:
            q, sc, bi = _affine(rng, rows, cols, group_size, std)
            tensors[stem + ".weight"] = ("U32", [rows, cols // 4], q.tobytes())
            tensors[stem + ".scales"] = ("F16", [rows, cols // group_size], sc.tobytes())
            tensors[stem + ".biases"] = ("F16", [rows, cols // group_size], bi.tobytes())
        else:
            w = rng.normal(0, std, (rows, cols)).astype(np.float16)
            tensors[stem + ".weight"] = ("F16", [rows, cols], w.tobytes())

    def norm(name: str):
        w = (1.0 + rng.normal(0, 0.05, dim)).astype(np.float16)
        tensors[name] = ("F16", [dim], w.tobytes())

    proj("model.embed_tokens", cfg["vocab_size"], dim)
    norm("model.norm.weight")
    for l in range(L):
        p = f"model.layers.{l}."
        norm(p + "input_layernorm.weight")
        norm(p + "post_attention_layernorm.weight")
        proj(p + "self_attn.q_proj", att, dim)
        proj(p + "self_attn.k_proj", kvd, dim)
        proj(p + "self_attn.v_proj", kvd, dim)
        proj(p + "self_attn.o_proj", dim, att)
        proj(p + "mlp.gate_proj", ffn, dim)
        proj(p + "mlp.down_proj", dim, ffn)
        proj(p + "mlp.up_proj", ffn, dim)
    header, off, blobs = {"__metadata__": {"format": "mlx"}}, 0, []
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * (-len(hb) % 8)
    path = d / "model.safetensors"
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
    conf = dict(cfg)
    if quantized:
        conf["quantization"] = {"group_size": group_size, "bits": 8}
        if quant_type:
            conf["quantization"]["quant_type"] = quant_type
    (d / "config.json").write_text(json.dumps(conf, indent=1))
    if tokenizer == "bin":
        write_tokenizer_bin(d / "tokenizer.bin", cfg["vocab_size"], 1, 2)
    elif tokenizer == "json":
        added = [{"id": 300, "content": "<|begin_of_text|>"}, {"id": 301, "content": "<|end_of_text|>"},
                 {"id": 302, "content": "<|eot_id|>"}]
        (d / "tokenizer.json").write_text(json.dumps({"model": {"vocab": {}, "merges": []}, "added_tokens": added}))
    return path


def write_lmrs(dirpath, cfg: dict, seed: int, std: float = 0.02) -> Path:
    """Writes model.lmrs and tokenizer.bin into dirpath; returns the .lmrs path."""
    d = Path(dirpath)
    d.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    dim, ffn, L, gs = cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["group_size"]
    att = cfg["n_heads"] * cfg["head_size"]
    kvd = cfg["n_kv_heads"] * cfg["head_size"]
    args = struct.pack("<IIIIIIIIffBBIB", dim, ffn, L, cfg["n_heads"], cfg["head_size"], cfg["n_kv_heads"],
                       cfg["vocab_size"], cfg["seq_len"], cfg["rms_norm_eps"], cfg["rope_theta"], 1, 1, gs, 0)
    assert len(args) == 47
    out = bytearray(b"lmrs" + struct.pack("<I", 1) + args)
    out += b"\0" * (256 - len(out))

    def q8(rows: int, cols: int):
        q = rng.integers(-127, 128, size=rows * cols, dtype=np.int8)
        s = (np.abs(rng.normal(0, std / 64.0, rows * cols // gs)) + std / 512.0).astype(np.float32)
        return q.tobytes() + s.tobytes()

    def f32norm():
        return (1.0 + rng.normal(0, 0.05, dim)).astype(np.float32).tobytes()

    out += q8(cfg["vocab_size"], dim)
    for _ in range(L):
        out += f32norm()
    for rows, cols in ((att, dim), (kvd, dim), (kvd, dim), (dim, att)):
        for _ in range(L):
            out += q8(rows, cols)
    for _ in range(L):
        out += f32norm()
    for rows, cols in ((ffn, dim), (dim, ffn), (ffn, dim)):
        for _ in range(L):
            out += q8(rows, cols)
    out += f32norm()
    path = d / "model.lmrs"
    path.write_bytes(bytes(out))
    write_tokenizer_bin(d / "tokenizer.bin", cfg["vocab_size"], 1, 2)
    return path


def read_safetensors(path) -> dict[str, np.ndarray]:
    """Tensors of a safetensors file as numpy arrays (U32 as raw uint8 rows)."""
    raw = Path(path).read_bytes()
    (hlen,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + hlen])
    base = 8 + hlen
    out = {}
    for name, info in hdr.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        buf = raw[base + a:base + b]
        if info["dtype"] == "F16":
            out[name] = np.frombuffer(buf, np.float16).reshape(info["shape"])
        elif info["dtype"] == "U32":
            out[name] = np.frombuffer(buf, np.uint8).reshape(info["shape"][0], info["shape"][1] * 4)
    return out


def requantize_affine(q: np.ndarray, scales: np.ndarray, biases: np.ndarray, gs: int = 32):
    """util.rs:480-515 in numpy: v = q * scale + bias (each rounded to f32),
    scale' = max|v| / 127 (1 when all zero), q' = round-half-away(v / scale')
    clamped to [-128, 127]. Returns (int8 [rows, cols], f32 [rows, cols/gs])."""
    rows, cols = q.shape
    qg = q.reshape(rows, cols // gs, gs).astype(np.float32)
    sc = scales.astype(np.float32)[..., None]
    bi = biases.astype(np.float32)[..., None]
    v = (qg * sc).astype(np.float32) + bi
    mx = np.max(np.abs(v), axis=2)
    sym = np.where(mx == 0, np.float32(1.0), mx / np.float32(127.0)).astype(np.float32)
    ratio = (v / sym[..., None]).astype(np.float64)  # the f32 quotient, rounded below exactly in double
    r = np.sign(ratio) * np.floor(np.abs(ratio) + 0.5)
    qn = np.clip(r, -128, 127).astype(np.int8).reshape(rows, cols)
    return qn, sym

"""CPU: the safetensors and lm.rs loaders (transformer_llama_st.rs,
transformer_llama_lmrs.rs) on files written by tests/model_files.py.

The oracle's loaders are checked against the files themselves: its
embedding table must equal the numpy restatement of the safetensors
requantization (util.rs:451-518) and, for lm.rs, q * scale of the stored
Q8 embedding; BOS/EOS come from the tokenizer beside the model. The product
library's loaders are exercised here up to the point where they would touch
the device: every rejection the reference makes (and the Q4_0 safetensors
case and group sizes other than 32, which the device path refuses) happens
before any CUDA call.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

import model_files as mf


def test_json_reader_via_config_errors(yl, tmp_path):
    st = mf.write_safetensors(tmp_path / "a", mf.ST_SMALL, seed=1)
    cfg = st.parent / "config.json"
    good = cfg.read_text()
    cfg.write_text(good[:-5])  # truncated JSON
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -3 and "config.json" in str(e.value)
    d = json.loads(good)
    d["hidden_size"] = 256.0  # serde_json's as_u64 refuses a float literal
    cfg.write_text(json.dumps(d))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -3 and "hidden_size" in str(e.value)
    del d["head_dim"]
    d["hidden_size"] = 256
    cfg.write_text(json.dumps(d))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -3 and "head_dim" in str(e.value)


def test_st_rejections_before_the_device(yl, orc, tmp_path):
    # quant_type Q4_0: the reference loads Q8 tensors and runs its Q4_0 kernel on them
    st = mf.write_safetensors(tmp_path / "q4", mf.ST_SMALL, seed=2, quant_type="Q4_0")
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -8 and "Q4_0" in str(e.value)
    with pytest.raises(RuntimeError):
        orc.Model(str(st))
    # MLX's common group size 64: the device quantizes activations in groups of 32
    st = mf.write_safetensors(tmp_path / "g64", mf.ST_SMALL, seed=3, group_size=64)
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -8 and "32" in str(e.value)
    # no tokenizer beside the model
    st = mf.write_safetensors(tmp_path / "notok", mf.ST_SMALL, seed=4, tokenizer="none")
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -2 and "tokenizer" in str(e.value)
    # a header that claims more bytes than the file has
    st = mf.write_safetensors(tmp_path / "trunc", mf.ST_SMALL, seed=5)
    raw = st.read_bytes()
    st.write_bytes(raw[:len(raw) // 2])
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -3 and "bounds" in str(e.value)
    # a missing tensor
    st = mf.write_safetensors(tmp_path / "miss", mf.ST_SMALL, seed=6)
    raw = bytearray(st.read_bytes())
    (hlen,) = struct.unpack("<Q", raw[:8])
    hdr = raw[8:8 + hlen].replace(b"model.layers.1.mlp.up_proj.biases", b"model.layers.1.mlp.up_proj.bXases")
    st.write_bytes(bytes(raw[:8] + hdr + raw[8 + hlen:]))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(st))
    assert e.value.code == -3 and "up_proj.biases" in str(e.value)


def test_lmrs_rejections_before_the_device(yl, orc, tmp_path):
    p = mf.write_lmrs(tmp_path / "bad", mf.LMRS_SMALL, seed=1)
    raw = bytearray(p.read_bytes())
    p.write_bytes(b"LMRS" + bytes(raw[4:]))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(p))
    assert e.value.code == -3 and "lm.rs format" in str(e.value)
    with pytest.raises(RuntimeError, match="lm.rs format"):
        orc.Model(str(p))
    p.write_bytes(bytes(raw[:len(raw) - 1000]))  # shorter than its tensors
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(p))
    assert e.value.code == -3 and "shorter" in str(e.value)
    with pytest.raises(RuntimeError):
        orc.Model(str(p))
    zero = bytearray(raw)
    zero[8:12] = bytes(4)  # dim 0
    p.write_bytes(bytes(zero))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(p))
    assert e.value.code == -3 and "cannot be zero" in str(e.value)
    (tmp_path / "bad" / "tokenizer.bin").unlink()
    p.write_bytes(bytes(raw))
    with pytest.raises(yl.YlError) as e:
        yl.load_transformer(str(p))
    assert e.value.code == -2 and "tokenizer.bin" in str(e.value)


def test_oracle_st_requantization_matches_numpy(orc, tmp_path):
    st = mf.write_safetensors(tmp_path / "m", mf.ST_SMALL, seed=7)
    om = orc.Model(str(st), 512)
    t = mf.read_safetensors(st)
    q, sym = mf.requantize_affine(t["model.embed_tokens.weight"], t["model.embed_tokens.scales"],
                                  t["model.embed_tokens.biases"])
    want = (q.astype(np.float32).reshape(q.shape[0], -1, 32) * sym[..., None]).astype(np.float32).reshape(q.shape)
    for tok in (0, 1, 17, 383):
        np.testing.assert_array_equal(om.get_embeddings(tok), want[tok])
    sh = om.shape
    assert (sh.dim, sh.head_size, sh.n_heads, sh.n_kv_heads, sh.group_size) == (256, 64, 4, 2, 32)
    assert sh.rope_mode == orc.ROPE_LLAMA3 and sh.llama3_old_ctx == 512.0 and sh.ctx_len == 512
    assert (sh.bos, sh.eos) == (1, 2)


def test_oracle_st_f16_and_tokenizer_json(orc, tmp_path):
    st = mf.write_safetensors(tmp_path / "f", mf.ST_SMALL, seed=8, quantized=False, tokenizer="json")
    om = orc.Model(str(st), 256)
    t = mf.read_safetensors(st)
    np.testing.assert_array_equal(om.get_embeddings(5), t["model.embed_tokens.weight"][5].astype(np.float32))
    sh = om.shape
    assert sh.weight_format == orc.F16 and sh.ctx_len == 256
    assert (sh.bos, sh.eos) == (300, 302)  # the last of <|end_of_text|>, <|eot_id|> wins


def test_oracle_lmrs_embedding_and_shape(orc, tmp_path):
    p = mf.write_lmrs(tmp_path / "l", mf.LMRS_SMALL, seed=9)
    om = orc.Model(str(p), 100)
    raw = p.read_bytes()
    V, D = 512, 256
    q = np.frombuffer(raw[256:256 + V * D], np.int8).reshape(V, D)
    s = np.frombuffer(raw[256 + V * D:256 + V * D + V * D // 32 * 4], np.float32).reshape(V, D // 32)
    want = (q.astype(np.float32).reshape(V, -1, 32) * s[..., None]).astype(np.float32).reshape(V, D)
    for tok in (0, 3, 511):
        np.testing.assert_array_equal(om.get_embeddings(tok), want[tok])
    sh = om.shape
    assert (sh.dim, sh.hidden_dim, sh.n_layers, sh.n_kv_heads, sh.ctx_len) == (256, 768, 2, 1, 100)
    assert sh.llama3_old_ctx == 100.0 and (sh.bos, sh.eos) == (1, 2)


@pytest.mark.parametrize("kind", ["st_q8", "lmrs"])
def test_oracle_forward_runs_on_both_formats(orc, tmp_path, kind):
    if kind == "st_q8":
        p = mf.write_safetensors(tmp_path / kind, mf.ST_SMALL, seed=10)
    else:
        p = mf.write_lmrs(tmp_path / kind, mf.LMRS_SMALL, seed=10)
    om = orc.Model(str(p), 128)
    s = om.create_session()
    lo = om.forward_x([1, 5, 9, 2], 0, s)
    assert lo.shape[0] == om.shape.vocab_size and np.all(np.isfinite(lo))
    lo2 = om.forward_x([orc.argmax(lo)], 4, s)
    assert np.all(np.isfinite(lo2))

"""Tokenizer parity (CPU): the product's C++ tokenizer through the C-ABI
against the Python restatement of tokenizer.rs (oracle/tokenizer_ref.py), on
seeded synthetic BPE vocabularies in the three file forms the reference
reads, over random texts (ASCII words, contractions, numbers, punctuation,
letters of several scripts, emoji, odd whitespace)."""
from __future__ import annotations

import pytest

import tokenizer_files as tf
import tokenizer_ref as tr


@pytest.fixture(scope="module")
def bpe():
    vocab, merges = tf.learn_bpe(tf.corpus(7), 400)
    return vocab, merges


@pytest.fixture(scope="module")
def texts():
    return tf.random_texts(11, 120) + ["a", " ", "'s", "hello world", "  leading", "trailing  ", "x\n\ny",
                                       "日本語のテキスト", "mixed123abc", "$$$", "it's we'll they've you're I'd"]


@pytest.mark.parametrize("pre,add_space", [("gpt2", False), ("smollm", True), ("default", False)])
def test_gguf_encode_decode_match_restatement(yl, tmp_path, bpe, texts, pre, add_space):
    vocab, merges = bpe
    path = tf.write_gguf_tokenizer(tmp_path / "t.gguf", vocab, merges, 1, 2, pre=pre, add_space=add_space)
    ours = yl.Tokenizer.load(path)
    ref = tr.Tokenizer.from_gguf(path)
    assert ours.info()["vocab_size"] == len(vocab)
    for t in texts:
        ids = ours.encode(t)
        assert ids == ref.encode(t), t
        assert ours.encode(t, bos=True, eos=True) == [1] + ids + [2]
        # byte-level BPE round-trips (with the space prefix the encoder adds)
        assert ours.decode(ids) == ref.decode(ids) == (" " + t if add_space and not t.startswith(" ") else t)
    ours.close()


def test_decode_lossy_and_out_of_range(yl, tmp_path, bpe):
    vocab, merges = bpe
    path = tf.write_gguf_tokenizer(tmp_path / "t.gguf", vocab, merges, 1, 2)
    ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)
    e = ours.encode("日本😀")
    # pieces decoded one at a time split multi-byte characters (U+FFFD), as the console prints them
    pieces = [ours.decode([i]) for i in e]
    assert pieces == [ref.decode([i]) for i in e]
    assert "".join(ours.decode([i]) for i in ours.encode("abc")) == "abc"
    assert ours.decode([len(vocab) + 5, 10**6]) == ""
    assert ours.decode([]) == ""


def test_json_and_bin_forms(yl, tmp_path, bpe, texts):
    vocab, merges = bpe
    # tokenizer.json: added tokens override ids and name BOS/EOS
    added = {len(vocab): "<|begin_of_text|>", len(vocab) + 1: "<|eot_id|>"}
    full = vocab + [added[len(vocab)], added[len(vocab) + 1]]
    d = tmp_path / "st"
    d.mkdir()
    tf.write_tokenizer_json(d / "tokenizer.json", full, merges, added)
    (d / "model.safetensors").write_bytes(b"")
    ours = yl.Tokenizer.load(str(d / "model.safetensors"))
    ref = tr.Tokenizer.from_json(str(d / "tokenizer.json"))
    info = ours.info()
    assert (info["bos"], info["eos"]) == (ref.bos, ref.eos) == (len(vocab), len(vocab) + 1)
    for t in texts[:60]:
        assert ours.encode(t) == ref.encode(t), t
    # tokenizer.bin (lm.rs): character lookup, bytes + 3 fallback, file scores
    b = tmp_path / "lm"
    b.mkdir()
    bvocab = ["<unk>", "<s>", "</s>"] + [f"<0x{i:02X}>" for i in range(256)] + ["a", "b", "ab", "abc", "c", " ", " a"]
    scores = [0.0] * 259 + [1.0, 1.0, 5.0, 7.0, 1.0, 1.0, 3.0]
    tf.write_tokenizer_bin_vocab(b / "tokenizer.bin", bvocab, scores, 1, 2)
    (b / "m.lmrs").write_bytes(b"")
    ours = yl.Tokenizer.load(str(b / "m.lmrs"))
    ref = tr.Tokenizer.from_bin(str(b / "tokenizer.bin"))
    for t in ["abc", "a b", "cab é", "ab ab abc", "zz"]:
        assert ours.encode(t) == ref.encode(t), t
        ids = ours.encode(t)
        assert ours.decode(ids) == ref.decode(ids)


def test_chat_prompt_llama_and_small(yl, tmp_path, bpe):
    vocab, merges = bpe
    small = tf.write_gguf_tokenizer(tmp_path / "s.gguf", vocab, merges, 1, 2, add_bos=True)
    big_vocab = tf.llama_vocab(vocab)
    big = tf.write_gguf_tokenizer(tmp_path / "b.gguf", big_vocab, merges, 128000, 128009)
    for path in (small, big):
        ours, ref = yl.Tokenizer.load(path), tr.Tokenizer.from_gguf(path)
        for user in ["hello world", "what's 3.14?", "日本"]:
            assert ours.chat_prompt(user) == ref.chat_prompt(user)
            assert ours.chat_prompt(user, system="be brief") == ref.chat_prompt(user, system="be brief")
    p = yl.Tokenizer.load(big).chat_prompt("hi")
    assert p[:2] == [128000, 128006] and p[-4] == 128006 and p[-1] == 271


def test_errors(yl, tmp_path, bpe):
    vocab, merges = bpe
    path = tf.write_gguf_tokenizer(tmp_path / "t.gguf", vocab, merges, 1, 2)
    t = yl.Tokenizer.load(path)
    with pytest.raises(yl.YlError):
        t.encode("")  # the reference asserts non-empty text
    with pytest.raises(yl.YlError):
        yl.Tokenizer.load(str(tmp_path / "missing.gguf"))
    with pytest.raises(yl.YlError):
        yl.Tokenizer.load(str(tmp_path / "x.bin"))  # unknown extension
    # a Llama-size vocabulary whose "user" is not one token: the reference panics
    v2, m2 = tf.learn_bpe(tf.corpus(3), 50, chain_words=[])
    big = tf.write_gguf_tokenizer(tmp_path / "b.gguf", tf.llama_vocab(v2), m2, 128000, 128009)
    with pytest.raises(yl.YlError):
        yl.Tokenizer.load(big).chat_prompt("hi")


def test_sampler_restatement_pins():
    """random_f32 and the argmax rule of sampler.rs on fixed inputs."""
    import numpy as np
    # xorshift64* of the seed, >> 8, / 2^24 (computed by hand for seed 42)
    s = 42
    m = (1 << 64) - 1
    s ^= s >> 12
    s ^= (s << 25) & m
    s ^= s >> 27
    assert tr.random_f32(42) == np.float32((((s * 0x2545F4914F6CDD1D) & m) >> 32 >> 8) / 16777216.0)
    assert 0.0 <= tr.random_f32(42) < 1.0
    assert tr.Sampler.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert tr.Sampler.argmax(np.array([np.nan, 3, 4], np.float32)) == 0
    assert tr.Sampler.argmax(np.array([5, np.nan, 4], np.float32)) == 0

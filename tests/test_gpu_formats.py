"""GPU parity of the safetensors and lm.rs loaders: synthetic files written by
tests/model_files.py, loaded by the device library and by the oracle's own
loaders, then the strict bar of the benchmark configurations (logits within
1e-2 * max|logit| at every step, identical greedy ids teacher-forced and
free-running). Weights carry f32 scales here (requantized MLX groups, lm.rs
Q8), so the matvec, the int8 GEMM prefill and the embedding gather run their
f32-scale variants. A 40-token prompt puts the prefill on the GEMM path."""
from __future__ import annotations

import pytest

import model_files as mf
from test_gpu_configs import assert_strict, strict_run

pytestmark = pytest.mark.gpu

CASES = {
    "st_q8": lambda d: mf.write_safetensors(d, mf.ST_SMALL, seed=21),
    "st_q8_wide_attention": lambda d: mf.write_safetensors(d, mf.ST_WIDE_ATT, seed=22, tokenizer="json"),
    "st_f16": lambda d: mf.write_safetensors(d, mf.ST_SMALL, seed=23, quantized=False),
    "lmrs_q8": lambda d: mf.write_lmrs(d, mf.LMRS_SMALL, seed=24),
}


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("prompt_len", [9, 40])
def test_format_matches_oracle(yl, orc, tmp_path, name, prompt_len):
    path = str(CASES[name](tmp_path / name))
    gm = yl.load_transformer(path, max_ctx_len=256)
    assert gm.name() == ("TransformerLlamaLmrs" if name.startswith("lmrs") else "TransformerLlamaSt")
    om = orc.Model(path, 256)
    assert (gm.bos_token(), gm.eos_token()) == (om.shape.bos, om.shape.eos)
    vocab = om.shape.vocab_size
    del om
    prompt = yl.prompt_ids(vocab, prompt_len, 300 + prompt_len).tolist()
    assert_strict(strict_run(yl, orc, path, prompt, 48, 256, f"{name}_p{prompt_len}"))


def test_format_embeddings_match_oracle(yl, orc, tmp_path):
    import numpy as np
    for name in ("st_q8", "lmrs_q8", "st_f16"):
        path = str(CASES[name](tmp_path / name))
        gm = yl.load_transformer(path, max_ctx_len=128)
        om = orc.Model(path, 128)
        toks = [0, 1, 7, om.shape.vocab_size - 1, om.shape.vocab_size + 5]
        got = gm.get_embeddings_batch(toks)
        for i, t in enumerate(toks):
            np.testing.assert_array_equal(got[i], om.get_embeddings(t))

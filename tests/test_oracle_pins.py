"""CPU: pins the oracle to the reference's own known-answer and property tests
and to the independent numpy golden vectors (tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np
import pytest


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


# ---- golden vectors (numpy restatement, bit-exact) -------------------------

def test_quantizer_golden_bit_exact(orc, golden):
    g = golden["quant"]
    for k in ("rand", "edge"):
        q, s = orc.quantize_q8(g[f"x_{k}"])
        assert np.array_equal(q, g[f"q_{k}"])
        assert np.array_equal(bits(s), bits(g[f"s_{k}"]))


def test_matmul_golden_bit_exact(orc, golden):
    m = golden["matmul"]
    for nm in ("small", "batch", "wide"):
        b, n, o = (int(v) for v in m[f"{nm}_dims"])
        out = m[f"{nm}_init"].copy()
        orc.matmul_q8(out, m[f"{nm}_xq"], m[f"{nm}_xs"], m[f"{nm}_wq"], m[f"{nm}_ws"], n, o)
        assert np.array_equal(bits(out), bits(m[f"{nm}_out_acc"])), nm
        out = np.zeros(b * o, np.float32)
        orc.matmul_q8(out, m[f"{nm}_xq"], m[f"{nm}_xs"], m[f"{nm}_wq"], m[f"{nm}_ws"], n, o)
        assert np.array_equal(bits(out), bits(m[f"{nm}_out_zero"])), nm


# ---- tests/matmul_q8_tests.rs:30-53 ----------------------------------------

def test_matmul_q8_remainder_columns(orc):
    batch, n, o, gs = 1, 64, 33, 32
    out = np.zeros(batch * o, np.float32)
    orc.matmul_q8(out, np.ones(batch * n, np.int8), np.ones(batch * n // gs, np.float32),
                  np.ones(o * n, np.int8), np.ones(o * n // gs, np.float32), n, o, gs)
    assert np.all(np.abs(out - n) < 1e-5)


def test_matmul_quad_accumulates_remainder_overwrites(orc):
    # weight_type.rs:190-201 (+=) vs :223 (=)
    n, o = 32, 6
    out = np.full(o, 100.0, np.float32)
    orc.matmul_q8(out, np.ones(n, np.int8), np.ones(1, np.float32), np.ones(o * n, np.int8),
                  np.ones(o, np.float32), n, o)
    assert np.all(out[:4] == 132.0) and np.all(out[4:] == 32.0)


def test_block_dots_match_matmul_with_unit_scales(orc):
    rng = np.random.default_rng(3)
    n, o = 256, 12
    xq = rng.integers(-127, 128, n, dtype=np.int8)
    wq = rng.integers(-127, 128, o * n, dtype=np.int8)
    bd = orc.block_dots(xq, wq, 1, n, o)
    out = np.zeros(o, np.float32)
    orc.matmul_q8(out, xq, np.ones(n // 32, np.float32), wq, np.ones(o * n // 32, np.float32), n, o)
    assert np.array_equal(out, bd.sum(axis=2).reshape(-1).astype(np.float32))


# ---- tests/simd_tests.rs:87-247 (rms_norm) ---------------------------------

def _rms(v):
    v = np.asarray(v, np.float32)
    return float(np.sqrt(np.sum(v * v) / v.size))


@pytest.mark.parametrize("x,w,expect", [
    ([1.0, 2.0, 3.0, 4.0], [1.0] * 4, 1.0),
    ([1.0, 2.0, 3.0, 4.0], [2.0] * 4, 2.0),
    ([1000.0, 2000.0, 3000.0, 4000.0], [1.0] * 4, 1.0),
    ([-1.0, -2.0, -3.0, -4.0], [1.0] * 4, 1.0),
    ([-1.0, 2.0, -3.0, 4.0], [1.0] * 4, 1.0),
])
def test_rms_norm_properties(orc, x, w, expect):
    y = orc.rms_norm_scalar(np.array(x, np.float32), np.array(w, np.float32), 1e-5)
    assert abs(_rms(y) - expect) < 1e-3


def test_rms_norm_single_and_small(orc):
    y = orc.rms_norm_scalar(np.array([5.0], np.float32), np.ones(1, np.float32), 1e-5)
    assert abs(y[0] - 1.0) < 1e-3
    for x in ([1e-10] * 4, [0.0] * 4):
        y = orc.rms_norm_scalar(np.array(x, np.float32), np.ones(4, np.float32), 1e-5)
        assert np.all(np.isfinite(y))


@pytest.mark.parametrize("size", [8, 16, 32, 64, 128, 256, 7, 15, 33, 100, 1000])
def test_rms_norm_sizes(orc, size):
    y = orc.rms_norm_scalar(np.arange(size, dtype=np.float32), np.ones(size, np.float32), 1e-5)
    assert abs(_rms(y) - 1.0) < 1e-3


@pytest.mark.parametrize("size", [8, 64, 576, 4096])
def test_simd_rmsnorm_matches_scalar(orc, size):
    rng = np.random.default_rng(size)
    x = rng.standard_normal(size).astype(np.float32)
    w = rng.standard_normal(size).astype(np.float32)
    a = orc.rmsnorm(x, w, 1e-5)
    b = orc.rms_norm_scalar(x, w, 1e-5)
    np.testing.assert_allclose(a, b, rtol=2e-6, atol=1e-7)


# ---- tests/simd_tests.rs:249-340 (silu) ------------------------------------

def test_silu_properties(orc):
    xs = np.array([0.0, 1.0, -1.0, 10.0, -10.0, 0.5, -0.5, 100.0, -100.0], np.float32)
    y = orc.silu(xs)
    ref = xs / (1.0 + np.exp(-xs.astype(np.float64)))
    assert np.all(np.abs(y - ref) < 1e-3)
    assert y[0] == 0.0 and np.all(np.isfinite(y))


# ---- f16 decode (half::f16::to_f32), exhaustive ------------------------------

def test_f16_to_f32_exhaustive(orc):
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([orc.f16_to_f32(int(v)) for v in h[::7]], np.float32)
    r = ref[::7]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), r[~nan].view(np.uint32))


# ---- sampler.rs:67-79 --------------------------------------------------------

def test_argmax_first_max_wins(orc):
    assert orc.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert orc.argmax(np.array([5, 3, 5], np.float32)) == 0


# ---- forward-level invariants ------------------------------------------------

def test_forward_prefill_equals_stepwise(orc, model_factory):
    """Prefill of n tokens and n single-token calls give the same last logits
    (every per-token quantity is computed identically)."""
    path = model_factory("tiny")
    m = orc.Model(path, 256)
    toks = [3, 17, 99, 5, 250, 1]
    s1 = m.create_session()
    a = m.forward_x(toks, 0, s1)
    s2 = m.create_session()
    for i, t in enumerate(toks):
        b = m.forward_x([t], i, s2)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_forward_is_causal(orc, model_factory):
    path = model_factory("tiny")
    m = orc.Model(path, 256)
    s1, s2 = m.create_session(), m.create_session()
    m.forward_x([3, 17, 99, 5], 0, s1)
    m.forward_x([3, 17, 99, 400], 0, s2)
    k1, _ = s1.kv()
    k2, _ = s2.kv()
    sh = m.shape
    kvd = sh.n_kv_heads * sh.head_size
    # layer 0 keys of positions 0..2 do not depend on token 3
    assert np.array_equal(k1[:3 * kvd], k2[:3 * kvd])
    assert not np.array_equal(k1[3 * kvd:4 * kvd], k2[3 * kvd:4 * kvd])


def test_out_of_range_token_embeds_zero(orc, model_factory):
    m = orc.Model(model_factory("tiny"), 256)
    assert np.all(m.get_embeddings(10 ** 6) == 0)
    assert np.any(m.get_embeddings(5) != 0)


def test_q4_decode_modes(orc, model_factory):
    """GGML order (element j <- low nibble of byte j, j+16 <- high nibble,
    value (q-8)*d) vs the literal reference decode
    (transformer_llama_gguf.rs:394-405: lo -> 2j, hi -> 2j+1, no -8). With
    both decodes of the same bytes: ggml[j] = ref[2j] - 8d and
    ggml[j+16] = ref[2j+1] - 8d, exactly (small integers times an f16 d)."""
    path = model_factory("tiny", weight_format=1)
    g = orc.Model(path, 256, q4_mode=orc.Q4_GGML)
    r = orc.Model(path, 256, q4_mode=orc.Q4_REF)
    for tok in (0, 7, 300):
        eg, er = g.get_embeddings(tok), r.get_embeddings(tok)
        for b in range(eg.size // 32):
            bg, br = eg[32 * b:32 * b + 32], er[32 * b:32 * b + 32]
            lo = bg[:16] - br[0::2]
            hi = bg[16:] - br[1::2]
            assert np.all(lo == lo[0]) and np.all(hi == lo[0])


def test_quantize_tail_untouched(orc):
    x = np.arange(40, dtype=np.float32)
    q, s = orc.quantize_q8(x)
    assert s.size == 1 and np.all(q[32:] == 0)

"""The arithmetic of the F16 tensor-core GEMM (csrc/kernels/gemm_f16.cu),
emulated in numpy on the CPU against the oracle's matmul_f32
(weight_type.rs:228-270, one sequential f32 dot per output): each token's
row scaled by the power of two e that puts its max |x| in [2^14, 2^15),
split into f16 hi + lo, each 16-wide step's products (exact) summed and
added to an f32 accumulator, hi part then lo part, the result scaled by
2^-e. The bound is the one the GPU test holds the kernel to: 1e-5 of
sum |x| |w| per output. Rows of very large, very small, mixed and zero
magnitude included."""
from __future__ import annotations

import numpy as np
import pytest


def split(x: np.ndarray):
    m = float(np.max(np.abs(x)))
    e = 0 if m == 0.0 or not np.isfinite(m) else 15 - int(np.frexp(np.float32(m))[1])
    s = np.ldexp(x.astype(np.float32), e).astype(np.float32)
    hi = s.astype(np.float16)
    lo = (s - hi.astype(np.float32)).astype(np.float32).astype(np.float16)
    return hi, lo, e


def emulate(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    hi, lo, e = split(x)
    acc = np.zeros(w.shape[0], np.float32)
    w64 = w.astype(np.float64)
    for k0 in range(0, x.size, 16):
        for part in (hi, lo):
            p = (w64[:, k0:k0 + 16] * part[k0:k0 + 16].astype(np.float64)).sum(axis=1)
            acc = (acc.astype(np.float64) + p).astype(np.float32)
    return np.ldexp(acc, -e).astype(np.float32)


@pytest.mark.parametrize("kind", ["normal", "tiny", "huge", "mixed", "zero_row", "one_spike"])
def test_split_gemm_within_bound_of_oracle(orc, kind):
    o, n = 96, 2048
    rng = np.random.default_rng(len(kind))
    w = (rng.standard_normal((o, n)) * 0.02).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    if kind == "tiny":
        x *= np.float32(1e-30)
    elif kind == "huge":
        x *= np.float32(1e30)
    elif kind == "mixed":  # magnitudes over 12 decades in one row
        x *= (10.0 ** rng.uniform(-8, 4, n)).astype(np.float32)
    elif kind == "zero_row":
        x[:] = 0.0
    elif kind == "one_spike":  # one element far above the rest sets the scale
        x[17] = 5e4
    got = emulate(w, x)
    ref = np.zeros(o, np.float32)
    orc.matmul_f32(ref, x, w.reshape(-1), n, o)
    bound = (np.abs(x)[None, :].astype(np.float64) * np.abs(w)).sum(axis=1)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= 1e-5 * bound + 1e-300), kind
    if kind == "zero_row":
        assert np.all(got == 0.0)


def test_split_keeps_the_row_exact_to_22_bits():
    rng = np.random.default_rng(3)
    for scale in (1e-20, 1e-3, 1.0, 7e3, 1e25):
        x = (rng.standard_normal(4096) * scale).astype(np.float32)
        hi, lo, e = split(x)
        back = np.ldexp(hi.astype(np.float64) + lo.astype(np.float64), -e)
        big = np.abs(x) >= np.max(np.abs(x)) * 2.0 ** -10  # lo stays a normal f16 for these
        rel = np.abs(back[big] - x[big]) / np.abs(x[big])
        assert rel.max() <= 2.0 ** -21, (scale, rel.max())
        assert np.max(np.abs(hi.astype(np.float64))) <= 2.0 ** 15  # far from the f16 maximum

"""Generates tests/golden/*.npz: golden vectors for the quantizer and the
quantized matmul, from an independent numpy restatement of the reference
(not from the C++ oracle, which these fixtures pin).

Restated here:
  * quantization.rs:29-52  `quantize`: absmax/127 f32 scale, IEEE x/scale,
    round half away from zero, Rust `as i8` (saturating, NaN -> 0);
  * weight_type.rs:122-226 `matmul_q8_slices`: per output column, groups
    folded in order as out += ((f32)isum * w_scale) * x_scale; the first
    4*floor(o/4) columns add into `out`, the rest overwrite it; the quad path
    sees floor(remaining/8)*8 elements of a group;
  * tests/matmul_q8_tests.rs:30-53, the reference's known-answer test
    (all ones, n=64, o=33, gs=32 -> 64.0).

Run: python tests/golden/make_golden.py   (writes the .npz next to this file)
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
F32 = np.float32


def quantize_np(x: np.ndarray, gs: int = 32):
    x = np.asarray(x, F32)
    ng = x.size // gs
    xb = x[: ng * gs].reshape(ng, gs)
    a = np.abs(xb)
    a = np.where(np.isnan(a), F32(0), a)            # NaN never wins `val > wmax`
    wmax = np.maximum(a.max(axis=1), F32(0)).astype(F32)
    scale = (wmax / F32(127.0)).astype(F32)
    with np.errstate(all="ignore"):
        qv = (xb / scale[:, None]).astype(F32)
        q64 = qv.astype(np.float64)
        r = np.sign(q64) * np.floor(np.abs(q64) + 0.5)  # half away from zero, exact in f64
        r = np.where(np.isnan(r), 0.0, r)
        r = np.clip(r, -128, 127)
    return r.astype(np.int8).reshape(-1), scale


def matmul_q8_np(out: np.ndarray, xq, xs, wq, ws, n: int, o: int, gs: int = 32) -> np.ndarray:
    rows = out.size // o
    W = np.asarray(wq, np.int8).reshape(o, n).astype(np.int64)
    ws = np.asarray(ws, F32)
    xs = np.asarray(xs, F32)
    quads = o // 4 * 4
    for r in range(rows):
        x = np.asarray(xq[r * n:(r + 1) * n], np.int8).astype(np.int64)
        acc = out[r * o: r * o + quads].astype(F32)
        g = 0
        while g < n:
            ge = min(g + gs, n)
            ns = (ge - g) // 8 * 8
            isum = (W[:quads, g:g + ns] * x[g:g + ns]).sum(axis=1).astype(np.int32)
            wsel = ws[(np.arange(quads) * n + g) // gs]
            t = (isum.astype(F32) * wsel).astype(F32)
            t = (t * xs[(r * n + g) // gs]).astype(F32)
            acc = (acc + t).astype(F32)
            g = ge
        out[r * o: r * o + quads] = acc
        for c in range(quads, o):
            s = F32(0)
            g = 0
            while g < n:
                ge = min(g + gs, n)
                bs = np.int32((W[c, g:ge] * x[g:ge]).sum())
                t = F32(F32(bs) * ws[(c * n + g) // gs])
                t = F32(t * xs[(r * n + g) // gs])
                s = F32(s + t)
                g = ge
            out[r * o + c] = s
    return out


def edge_vector() -> np.ndarray:
    """Blocks exercising the quantizer's corner cases."""
    blocks = []
    blocks.append(np.zeros(32, F32))                                  # 0/0 -> NaN -> 0
    b = np.full(32, -0.0, F32); blocks.append(b)                      # negative zeros
    b = np.linspace(-1, 1, 32, dtype=F32); blocks.append(b)
    b = (np.arange(32, dtype=F32) - 16) * F32(0.5) / F32(127 / 16.0); blocks.append(b)  # many near-ties
    b = np.zeros(32, F32); b[5] = F32(127.0); b[6] = F32(0.5); b[7] = F32(-0.5); b[8] = F32(1.5)
    blocks.append(b)                                                   # exact .5 ties at scale 1
    b = np.zeros(32, F32); b[0] = np.nan; b[1] = F32(3.0); b[2] = F32(-1.5); blocks.append(b)  # NaN ignored by max
    b = np.full(32, F32(1e-40)); b[3] = F32(-2e-40); blocks.append(b)  # subnormals
    b = np.full(32, F32(3.0e38)); b[::2] *= -1; blocks.append(b)       # huge
    b = np.zeros(32, F32); b[0] = np.inf; b[1] = F32(1.0); blocks.append(b)  # inf scale
    rng = np.random.default_rng(11)
    b = rng.standard_normal(32).astype(F32) * F32(1e-3); blocks.append(b)
    return np.concatenate(blocks)


def main() -> None:
    rng = np.random.default_rng(20251201)
    # --- quantizer ---
    xr = rng.standard_normal(32 * 257).astype(F32) * F32(2.5)
    xe = edge_vector()
    q_r, s_r = quantize_np(xr)
    q_e, s_e = quantize_np(xe)
    np.savez_compressed(HERE / "quantize_q8.npz", x_rand=xr, q_rand=q_r, s_rand=s_r, x_edge=xe, q_edge=q_e,
                        s_edge=s_e)
    # --- matmul: reference KAT + random cases (quad + remainder columns, batch 3, accumulate) ---
    cases = {}
    n, o = 64, 33
    out = np.zeros(o, F32)
    matmul_q8_np(out, np.ones(n, np.int8), np.ones(n // 32, F32), np.ones(o * n, np.int8),
                 np.ones(o * n // 32, F32), n, o)
    cases["kat_out"] = out
    for name, (b, n, o) in {"small": (1, 96, 37), "batch": (3, 256, 70), "wide": (2, 1024, 130)}.items():
        x = rng.standard_normal(b * n).astype(F32)
        xq, xs = quantize_np(x)
        w = (rng.standard_normal(o * n) * 0.02).astype(F32)
        wq, _ = quantize_np(w)
        # f16-representable weight scales, like GGUF
        ws = (np.abs(rng.standard_normal(o * n // 32)) * 1e-3 + 1e-4).astype(np.float16).astype(F32)
        init = rng.standard_normal(b * o).astype(F32)
        out_acc = matmul_q8_np(init.copy(), xq, xs, wq, ws, n, o)
        out_zero = matmul_q8_np(np.zeros(b * o, F32), xq, xs, wq, ws, n, o)
        cases.update({f"{name}_x": x, f"{name}_xq": xq, f"{name}_xs": xs, f"{name}_wq": wq, f"{name}_ws": ws,
                      f"{name}_init": init, f"{name}_out_acc": out_acc, f"{name}_out_zero": out_zero,
                      f"{name}_dims": np.array([b, n, o], np.int64)})
    np.savez_compressed(HERE / "matmul_q8.npz", **cases)
    print("wrote", HERE / "quantize_q8.npz", HERE / "matmul_q8.npz")


if __name__ == "__main__":
    main()

"""GPU parity of the quantizer and the quantized matmul against the oracle
and the golden vectors, through the C-ABI (libyallma3_b200.so).

Tolerances: quantized activations and per-block int32 dots are bit-exact;
f32 matmul outputs |gpu - ref| <= 1e-5 * sum|terms| (different fold order)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gpu_quantize(yl, torch, x: np.ndarray):
    xd = dev(torch, x.astype(np.float32))
    q = torch.zeros(x.size, dtype=torch.int8, device="cuda")
    s = torch.zeros(x.size // 32, dtype=torch.float32, device="cuda")
    yl.quantize_q8_0(xd, q, s, x.size, 32)
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy()


def test_quantizer_golden_bit_exact(yl, torch_cuda, golden):
    g = golden["quant"]
    for k in ("rand", "edge"):
        q, s = gpu_quantize(yl, torch_cuda, g[f"x_{k}"])
        assert np.array_equal(q, g[f"q_{k}"]), k
        assert np.array_equal(s.view(np.uint32), g[f"s_{k}"].view(np.uint32)), k


@pytest.mark.parametrize("n", [32, 576 * 3, 4096, 14336 * 8, 1 << 22])
def test_quantizer_random_bit_exact(yl, orc, torch_cuda, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 50.0], n)).astype(np.float32)
    q, s = gpu_quantize(yl, torch_cuda, x)
    qo, so = orc.quantize_q8(x)
    assert np.array_equal(q, qo)
    assert np.array_equal(s.view(np.uint32), so.view(np.uint32))


def test_quantizer_half_ties_bit_exact(yl, orc, torch_cuda):
    """Blocks whose quotients x/scale sit on, or a few ulps either side of,
    half-integers: the device rounds x*(1/scale) and must fall back to the
    exact quotient exactly where the two could round differently."""
    rng = np.random.default_rng(7)
    blocks = []
    for amax in (127.0, 3.0, 0.7, 1e-3, 4.5e4, 1.0e-30):
        sc = np.float32(np.float32(amax) / np.float32(127.0))
        for _ in range(64):
            k = rng.integers(-126, 126, 31) + 0.5
            x = (k * np.float64(sc)).astype(np.float32)
            ulps = rng.integers(-4, 5, 31).astype(np.int32)
            x = (x.view(np.int32) + ulps).view(np.float32)
            blocks.append(np.concatenate([[np.float32(amax)], x]).astype(np.float32))
    x = np.concatenate(blocks)
    q, s = gpu_quantize(yl, torch_cuda, x)
    qo, so = orc.quantize_q8(x)
    assert np.array_equal(s.view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q, qo)


def test_quantize_dispatch_errors(yl, torch_cuda):
    x = torch_cuda.zeros(64, device="cuda")
    dst = yl.new_workspace_buffer(yl.WeightFormat.Q8_0, 64, 32)
    with pytest.raises(yl.YlError) as e:
        yl.quantize(yl.WeightFormat.F16, dst, x, 64, 32)
    assert e.value.code == -3  # format/variant mismatch (weight_type.rs:88)
    yl.quantize(yl.WeightFormat.Q8_0, dst, x, 64, 32)


def upload_weight(yl, fmt, wq, ws, o, n, scale_type=1, values=None):
    w = yl.QuantizedTensor.weight(fmt, o, n, 32, scale_type)
    if fmt == yl.WeightFormat.F16:
        w.upload(values=values)
    else:
        w.upload(quant_vals=wq, scale_factor=ws)
    return w


def upload_act(yl, fmt, xq, xs, values=None):
    n = xq.size if values is None else values.size
    x = yl.new_workspace_buffer(fmt, n, 32)
    if fmt == yl.WeightFormat.F16:
        x.upload(values=values)
    else:
        x.upload(quant_vals=xq, scale_factor=xs)
    return x


def run_matmul(yl, torch, x, w, n, o, batch, init=None, accumulate=True):
    out = dev(torch, init) if init is not None else torch_zeros(torch, batch * o)
    yl.matmul(out, x, w, n, o, 32, batch=batch, accumulate=accumulate)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def torch_zeros(torch, n):
    return torch.zeros(n, dtype=torch.float32, device="cuda")


def term_bound(xq, xs, wq, ws, b, n, o):
    """sum over groups of |isum * ws * xs| per output, for the tolerance."""
    bd = np.einsum("bgk,ogk->bog", xq.reshape(b, n // 32, 32).astype(np.int64),
                   wq.reshape(o, n // 32, 32).astype(np.int64))
    return np.abs(bd * ws.reshape(1, o, n // 32) * xs.reshape(b, 1, n // 32)).sum(axis=2).reshape(-1)


def test_reference_remainder_kat(yl, torch_cuda):
    """tests/matmul_q8_tests.rs:30-53 through the device matmul."""
    n, o = 64, 33
    for st in (0, 1):
        w = upload_weight(yl, yl.WeightFormat.Q8_0, np.ones(o * n, np.int8), np.ones(o * n // 32, np.float32), o, n, st)
        x = upload_act(yl, yl.WeightFormat.Q8_0, np.ones(n, np.int8), np.ones(n // 32, np.float32))
        out = run_matmul(yl, torch_cuda, x, w, n, o, 1)
        assert np.all(np.abs(out - n) < 1e-5)


def test_golden_matmul(yl, torch_cuda, golden):
    m = golden["matmul"]
    for nm in ("small", "batch", "wide"):
        b, n, o = (int(v) for v in m[f"{nm}_dims"])
        xq, xs, wq, ws = m[f"{nm}_xq"], m[f"{nm}_xs"], m[f"{nm}_wq"], m[f"{nm}_ws"]
        w = upload_weight(yl, yl.WeightFormat.Q8_0, wq, ws, o, n)
        x = upload_act(yl, yl.WeightFormat.Q8_0, xq, xs)
        tb = term_bound(xq, xs, wq, ws, b, n, o)
        got = run_matmul(yl, torch_cuda, x, w, n, o, b, init=m[f"{nm}_init"], accumulate=True)
        ref = m[f"{nm}_out_acc"]
        quad = np.tile(np.arange(o) < o // 4 * 4, b)
        tol = 1e-5 * (tb + np.abs(m[f"{nm}_init"]) * quad) + 1e-30
        assert np.all(np.abs(got - ref) <= tol), nm
        got = run_matmul(yl, torch_cuda, x, w, n, o, b, accumulate=False)
        assert np.all(np.abs(got - m[f"{nm}_out_zero"]) <= 1e-5 * tb + 1e-30), nm


@pytest.mark.parametrize("fmt", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("batch", [1, 3, 8, 16])
def test_block_dots_bit_exact(yl, orc, torch_cuda, fmt, batch):
    """With unit scales every output is the exact integer sum of the per-block
    int32 dots (|sum| < 2^24), so any block-dot error shows bit for bit."""
    rng = np.random.default_rng(batch)
    n, o = 2048, 260
    f = getattr(yl.WeightFormat, fmt)
    lo, hi = (-127, 128) if fmt == "Q8_0" else (-8, 8)
    wq = rng.integers(lo, hi, o * n, dtype=np.int8)
    xq = rng.integers(-127, 128, batch * n, dtype=np.int8)
    w = upload_weight(yl, f, wq, np.ones(o * n // 32, np.float32), o, n)
    x = upload_act(yl, f, xq, np.ones(batch * n // 32, np.float32))
    got = run_matmul(yl, torch_cuda, x, w, n, o, batch, accumulate=False)
    bd = orc.block_dots(xq, wq, batch, n, o)
    assert np.array_equal(got, bd.sum(axis=2).reshape(-1).astype(np.float32))


SWEEP = [(2048, 2048), (8192, 2048), (2048, 8192), (1024, 14336)]


@pytest.mark.parametrize("mk", SWEEP)
@pytest.mark.parametrize("batch", [1, 4, 16])
@pytest.mark.parametrize("fmt", ["Q8_0", "Q4_0"])
def test_sweep_vs_oracle(yl, orc, torch_cuda, mk, batch, fmt):
    o, n = mk
    rng = np.random.default_rng(o * 7 + n + batch)
    f = getattr(yl.WeightFormat, fmt)
    if fmt == "Q8_0":
        wq = rng.integers(-127, 128, o * n, dtype=np.int8)
    else:
        wq = rng.integers(-8, 8, o * n, dtype=np.int8)
    ws = (np.abs(rng.standard_normal(o * n // 32)) * 1e-3 + 1e-5).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(batch * n).astype(np.float32)
    xq, xs = orc.quantize_q8(x)
    w = upload_weight(yl, f, wq, ws, o, n)
    xa = upload_act(yl, f, xq, xs)
    got = run_matmul(yl, torch_cuda, xa, w, n, o, batch, accumulate=False)
    ref = np.zeros(batch * o, np.float32)
    orc.matmul_q8(ref, xq, xs, wq, ws, n, o)
    tb = term_bound(xq, xs, wq, ws, batch, n, o)
    assert np.all(np.abs(got - ref) <= 1e-5 * tb + 1e-30)


@pytest.mark.parametrize("mk", [(2048, 2048), (1000, 4096)])
@pytest.mark.parametrize("batch", [1, 5, 16, 24, 33, 64])  # 16+: the f16 tensor-core GEMM (16-, 32- and 64-token tiles)
def test_f16_vs_oracle(yl, orc, torch_cuda, mk, batch):
    o, n = mk
    rng = np.random.default_rng(o + n + batch)
    wv = (rng.standard_normal(o * n) * 0.02).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(batch * n).astype(np.float32)
    w = upload_weight(yl, yl.WeightFormat.F16, None, None, o, n, values=wv)
    xa = upload_act(yl, yl.WeightFormat.F16, None, None, values=x)
    got = run_matmul(yl, torch_cuda, xa, w, n, o, batch, accumulate=False)
    ref = np.zeros(batch * o, np.float32)
    orc.matmul_f32(ref, x, wv, n, o)
    bound = (np.abs(x.reshape(batch, 1, n)) * np.abs(wv.reshape(1, o, n))).sum(axis=2).reshape(-1)
    assert np.all(np.abs(got - ref) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("batch", [16, 40])
def test_f16_gemm_matches_matvec_accumulate(yl, torch_cuda, batch):
    """yl_matmul(accumulate) on F16: the tensor-core GEMM (16+ rows) and the
    matvec (gemm_f16_min 0) give the same results within the F16 bound, quad
    columns added and the tail stored alike."""
    o, n = 1030, 1024
    rng = np.random.default_rng(batch)
    wv = (rng.standard_normal(o * n) * 0.02).astype(np.float16).astype(np.float32)
    x = (rng.standard_normal(batch * n) * 30).astype(np.float32)
    init = rng.standard_normal(batch * o).astype(np.float32)
    w = upload_weight(yl, yl.WeightFormat.F16, None, None, o, n, values=wv)
    xa = upload_act(yl, yl.WeightFormat.F16, None, None, values=x)
    got = run_matmul(yl, torch_cuda, xa, w, n, o, batch, init=init, accumulate=True)
    yl.config_set("gemm_f16_min", 0)
    try:
        mv = run_matmul(yl, torch_cuda, xa, w, n, o, batch, init=init, accumulate=True)
    finally:
        yl.config_set("gemm_f16_min", 16)
    bound = (np.abs(x.reshape(batch, 1, n)) * np.abs(wv.reshape(1, o, n))).sum(axis=2).reshape(-1)
    assert np.all(np.abs(got - mv) <= 2e-5 * bound + 1e-6)
    tail = (np.arange(batch * o) % o) >= o // 4 * 4  # stored, not added (weight_type.rs:207-224)
    assert np.all(np.abs(got[tail] - mv[tail]) <= 2e-5 * bound[tail])


def test_f32_weight_scales(yl, orc, torch_cuda):
    """Weights with arbitrary f32 scales (lmrs / requantized safetensors)."""
    rng = np.random.default_rng(5)
    o, n = 300, 1024
    wq = rng.integers(-127, 128, o * n, dtype=np.int8)
    ws = (np.abs(rng.standard_normal(o * n // 32)) * 1e-3).astype(np.float32)
    x = rng.standard_normal(2 * n).astype(np.float32)
    xq, xs = orc.quantize_q8(x)
    w = upload_weight(yl, yl.WeightFormat.Q8_0, wq, ws, o, n, scale_type=0)
    got = run_matmul(yl, torch_cuda, upload_act(yl, yl.WeightFormat.Q8_0, xq, xs), w, n, o, 2, accumulate=False)
    ref = np.zeros(2 * o, np.float32)
    orc.matmul_q8(ref, xq, xs, wq, ws, n, o)
    assert np.all(np.abs(got - ref) <= 1e-5 * term_bound(xq, xs, wq, ws, 2, n, o) + 1e-30)


GEMM_CASES = [(260, 576, 5), (1000, 2048, 8), (384, 2080, 12), (128, 32, 16), (260, 576, 17), (1000, 2048, 32), (384, 2080, 20), (260, 576, 33), (1000, 2048, 64), (128, 32, 65),
              (384, 2080, 130), (2048, 2048, 256),
              # from 96 tokens Q8_0 runs on the tcgen05 kernel (128 x 128 tiles, 4 blocks per stage):
              # row / token tails, a single block, a partial last stage (65 blocks), several token tiles
              (300, 1056, 129), (128, 32, 100), (1000, 2080, 96), (512, 4096, 384), (4096, 4096, 512)]


@pytest.fixture
def gemm_path(yl, request):
    """Selects the Q8_0 GEMM kernel for the test: mma.sync (tc = 0) or the
    tcgen05 / tensor-memory kernel (tc = 1, from 96 tokens)."""
    tc = request.param
    yl.config_set("gemm_tc", tc)
    yield tc
    yl.config_set("gemm_tc", 0)


@pytest.mark.parametrize("o,n,batch", GEMM_CASES)
@pytest.mark.parametrize("fmt", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("scale_type", [1, 0])
@pytest.mark.parametrize("gemm_path", [0, 1], indirect=True)
def test_gemm_bit_exact_vs_oracle(yl, orc, torch_cuda, o, n, batch, fmt, scale_type, gemm_path):
    """Batches of 16 or more tokens run on the int8 tensor-core GEMM. It folds
    each 32-block's exact int32 dot as ((f32)isum * ws) * xs in group order,
    the oracle's sequence (weight_type.rs:190-201, :207-224), so into a zeroed output the
    results are bit-identical. Cases cover both token tiles (32 and 64), row
    and token tails, a single block, an odd block count (f16 scale pairs) and
    several K stages. With gemm_path 1, Q8_0 batches of 96+ tokens run on the
    tcgen05 kernel instead (the other cases are skipped there)."""
    if gemm_path and (fmt != "Q8_0" or batch < 96):
        pytest.skip("the tcgen05 kernel takes Q8_0 batches of 96 or more tokens")
    rng = np.random.default_rng(o + n + batch)
    f = getattr(yl.WeightFormat, fmt)
    lo, hi = (-127, 128) if fmt == "Q8_0" else (-8, 8)
    wq = rng.integers(lo, hi, o * n, dtype=np.int8)
    ws = (np.abs(rng.standard_normal(o * n // 32)) * 1e-3 + 1e-5).astype(np.float32)
    if scale_type == 1:
        ws = ws.astype(np.float16).astype(np.float32)
    x = rng.standard_normal(batch * n).astype(np.float32)
    xq, xs = orc.quantize_q8(x)
    w = upload_weight(yl, f, wq, ws, o, n, scale_type=scale_type)
    got = run_matmul(yl, torch_cuda, upload_act(yl, f, xq, xs), w, n, o, batch, accumulate=False)
    ref = np.zeros(batch * o, np.float32)
    orc.matmul_q8(ref, xq, xs, wq, ws, n, o)
    assert np.array_equal(got, ref), float(np.max(np.abs(got - ref)))


@pytest.mark.parametrize("fmt", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("batch", [40, 140])
@pytest.mark.parametrize("gemm_path", [0, 1], indirect=True)
def test_gemm_accumulate_quirk(yl, orc, torch_cuda, fmt, batch, gemm_path):
    """The `+=` quirk through the GEMM: quad columns add into the initial
    output, remainder columns overwrite it (weight_type.rs:190-201 vs :223).
    With gemm_path 1, 140 tokens of Q8_0 take the tcgen05 kernel."""
    if gemm_path and (fmt != "Q8_0" or batch < 96):
        pytest.skip("the tcgen05 kernel takes Q8_0 batches of 96 or more tokens")
    rng = np.random.default_rng(11)
    o, n = 262, 1024
    f = getattr(yl.WeightFormat, fmt)
    lo, hi = (-127, 128) if fmt == "Q8_0" else (-8, 8)
    wq = rng.integers(lo, hi, o * n, dtype=np.int8)
    ws = (np.abs(rng.standard_normal(o * n // 32)) * 1e-3 + 1e-5).astype(np.float16).astype(np.float32)
    xq, xs = orc.quantize_q8(rng.standard_normal(batch * n).astype(np.float32))
    init = rng.standard_normal(batch * o).astype(np.float32)
    w = upload_weight(yl, f, wq, ws, o, n)
    got = run_matmul(yl, torch_cuda, upload_act(yl, f, xq, xs), w, n, o, batch, init=init, accumulate=True)
    ref = init.copy()
    orc.matmul_q8(ref, xq, xs, wq, ws, n, o)
    quad = np.tile(np.arange(o) < o // 4 * 4, batch)
    tb = term_bound(xq, xs, wq, ws, batch, n, o)
    assert np.all(np.abs(got - ref) <= 1e-5 * (tb + np.abs(init) * quad) + 1e-30)


def test_full_size_lm_head_rows_sampled(yl, orc, torch_cuda):
    """(128256, 4096) Q8_0 at N=1: every output row depends on its own weight
    row only, so a random sample of rows checked against the oracle covers the
    full-size launch (grid, ring, tails)."""
    rng = np.random.default_rng(9)
    o, n = 128256, 4096
    wq = rng.integers(-127, 128, o * n, dtype=np.int8)
    ws = (np.abs(rng.standard_normal(o * n // 32)) * 1e-3 + 1e-5).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    xq, xs = orc.quantize_q8(x)
    w = upload_weight(yl, yl.WeightFormat.Q8_0, wq, ws, o, n)
    got = run_matmul(yl, torch_cuda, upload_act(yl, yl.WeightFormat.Q8_0, xq, xs), w, n, o, 1, accumulate=False)
    rows = np.unique(np.concatenate([rng.integers(0, o, 512), [0, 1, o - 1, o - 2]]))
    sub_w = wq.reshape(o, n)[rows].reshape(-1)
    sub_s = ws.reshape(o, n // 32)[rows].reshape(-1)
    ref = np.zeros(rows.size, np.float32)
    orc.matmul_q8(ref, xq, xs, sub_w, sub_s, n, rows.size)
    tb = term_bound(xq, xs, sub_w, sub_s, 1, n, rows.size)
    assert np.all(np.abs(got[rows] - ref) <= 1e-5 * tb + 1e-30)
    assert np.all(np.isfinite(got))


def test_matmul_format_mismatch(yl, torch_cuda):
    w = yl.QuantizedTensor.weight(yl.WeightFormat.Q8_0, 8, 64)
    x = yl.new_workspace_buffer(yl.WeightFormat.F16, 64, 32)
    out = torch_cuda.zeros(8, device="cuda")
    with pytest.raises(yl.YlError) as e:
        yl.matmul(out, x, w, 64, 8, 32)
    assert e.value.code == -3


@pytest.mark.parametrize("hd,nh,nkv,batch,start", [
    (128, 32, 8, 1, 700), (64, 9, 3, 1, 40), (64, 32, 8, 1, 0), (128, 4, 1, 1, 3000),
    (128, 32, 8, 7, 100), (64, 32, 8, 16, 0),
    (128, 32, 8, 64, 0), (128, 32, 8, 100, 300), (64, 9, 3, 40, 17), (128, 4, 1, 33, 0), (64, 16, 2, 50, 5),
    (128, 8, 8, 70, 2),
])
def test_fused_attention_vs_oracle(yl, orc, torch_cuda, hd, nh, nkv, batch, start):
    """forward.rs:299-400 through yl_fused_attention (GQA ratios 1, 3, 4 and 8,
    partial query blocks, key offsets, seq_len % 8 tails) against the oracle's
    restatement: bit-identical, the same f32 operations in the same order."""
    rng = np.random.default_rng(hd + nh + batch + start)
    seq = start + batch
    kvd = nkv * hd
    sq = rng.standard_normal(batch * nh * hd).astype(np.float32)
    kc = rng.standard_normal(seq * kvd).astype(np.float32)
    vc = rng.standard_normal(seq * kvd).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    ref = orc.fused_attention(sq, kc, vc, seq, batch, nh, nkv, hd, start, kvd, scale)
    out = torch_cuda.zeros(batch * nh * hd, device="cuda")
    yl.fused_attention(out, dev(torch_cuda, sq), dev(torch_cuda, kc), dev(torch_cuda, vc), seq, batch, nh, nkv, hd,
                       start, kvd, float(scale))
    torch_cuda.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got, ref), float(np.max(np.abs(got - ref)))

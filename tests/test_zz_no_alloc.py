"""GPU: yl_fused_attention_static, the entry point that allocates nothing.

It exists for callers that cannot allocate device memory where attention
runs (an engine whose memory manager owns all device memory, or a
latency-critical loop that must not hit the allocator). It keeps its split
partials in a fixed device array instead of a per-call workspace; this file
checks, through the C-ABI, that it returns what yl_fused_attention returns.

The file is named so that pytest collects it last: a run that stops at the
first failure has run every other test by the time it gets here.
"""
from __future__ import annotations

import ctypes as C
import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _lib():
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    return importlib.import_module("yallma3-mini-inference_b200").raw_lib()


def _call(fn, torch, out, sq, kc, vc, seq, batch, nh, nkv, hd, start, scale):
    rc = fn(C.c_void_p(out.data_ptr()), C.c_void_p(sq.data_ptr()), C.c_void_p(kc.data_ptr()),
            C.c_void_p(vc.data_ptr()), seq, batch, nh, nkv, hd, start, nkv * hd, C.c_float(scale), None)
    torch.cuda.synchronize()
    return rc


# (head_size, query heads, kv heads, start position) for single-token calls
CASES = [(128, 32, 8, 700), (64, 9, 3, 40)]


@pytest.mark.parametrize("hd,nh,nkv,start", CASES)
def test_static_matches_allocating_entry_point_twice(hd, nh, nkv, start):
    import torch
    assert torch.cuda.is_available()
    lib = _lib()
    scale = 1.0 / float(np.sqrt(hd))
    for call in range(2):  # two calls in a row: the shared array keeps the last call's contents
        rng = np.random.default_rng(1000 * call + hd + nh + start)
        seq = start + 1 + 17 * call
        pos = seq - 1
        sq = torch.from_numpy(rng.standard_normal(nh * hd).astype(np.float32)).cuda()
        kc = torch.from_numpy(rng.standard_normal(seq * nkv * hd).astype(np.float32)).cuda()
        vc = torch.from_numpy(rng.standard_normal(seq * nkv * hd).astype(np.float32)).cuda()
        ref = torch.zeros(nh * hd, device="cuda")
        got = torch.full((nh * hd,), float("nan"), device="cuda")
        assert _call(lib.yl_fused_attention, torch, ref, sq, kc, vc, seq, 1, nh, nkv, hd, pos, scale) == 0
        rc = _call(lib.yl_fused_attention_static, torch, got, sq, kc, vc, seq, 1, nh, nkv, hd, pos, scale)
        assert rc == 0, lib.yl_last_error().decode()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        # the same kernel on the same inputs: the same bits
        assert np.array_equal(g, r), float(np.max(np.abs(g - r)))


@pytest.mark.parametrize("batch,start", [(7, 100), (40, 17)])
def test_static_multi_token_matches_allocating_entry_point(batch, start):
    """Several query rows (partial and whole 16-row query blocks): the same
    result as yl_fused_attention, twice in a row."""
    import torch
    lib = _lib()
    hd, nh, nkv = 128, 32, 8
    scale = 1.0 / float(np.sqrt(hd))
    for call in range(2):
        rng = np.random.default_rng(7 * call + batch + start)
        seq = start + batch
        sq = torch.from_numpy(rng.standard_normal(batch * nh * hd).astype(np.float32)).cuda()
        kc = torch.from_numpy(rng.standard_normal(seq * nkv * hd).astype(np.float32)).cuda()
        vc = torch.from_numpy(rng.standard_normal(seq * nkv * hd).astype(np.float32)).cuda()
        ref = torch.zeros(batch * nh * hd, device="cuda")
        got = torch.full((batch * nh * hd,), float("nan"), device="cuda")
        assert _call(lib.yl_fused_attention, torch, ref, sq, kc, vc, seq, batch, nh, nkv, hd, start, scale) == 0
        rc = _call(lib.yl_fused_attention_static, torch, got, sq, kc, vc, seq, batch, nh, nkv, hd, start, scale)
        assert rc == 0, lib.yl_last_error().decode()
        assert np.array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_static_rejects_oversized_request():
    import torch
    lib = _lib()
    hd, nh, nkv, seq = 128, 64, 8, 8192  # 64 heads x 8192 weights x 4 bytes = 2 MiB > 1 MiB
    sq = torch.zeros(nh * hd, device="cuda")
    kc = torch.zeros(seq * nkv * hd, device="cuda")
    out = torch.zeros(nh * hd, device="cuda")
    rc = _call(lib.yl_fused_attention_static, torch, out, sq, kc, kc, seq, 1, nh, nkv, hd, seq - 1, 0.1)
    assert rc == -8 and b"static area" in lib.yl_last_error()

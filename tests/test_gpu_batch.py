"""GPU: batched decode of independent sessions (yl_batch_forward, §8(f3)).

n sessions of one model, each with its own prompt (different lengths, so
different positions), step together: the projections run once over the n
stacked rows (matvec in passes of 8 rows, the int8 GEMM from 16 rows) and one
attention launch serves every session's own cache. Each session's logits
must EQUAL, bit for bit, those of the same session stepped alone with
yl_forward_x (itself bit-exact against the oracle, tests/test_gpu_forward.py),
at every step of a greedy decode; one case also checks the oracle directly.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def run_batched(yl, path, prompts, steps, max_ctx=256):
    m = yl.load_transformer(path, max_ctx_len=max_ctx)
    sess = [m.create_session() for _ in prompts]
    first = []
    for s, p in zip(sess, prompts):
        _, am = m.forward_x_full(p, 0, s)
        first.append(am)
    b = m.create_batch(len(prompts))
    toks, pos = list(first), [len(p) for p in prompts]
    out_ids, out_lg = [], []
    for _ in range(steps):
        ids, lg = b.forward(sess, toks, pos, want_logits=True)
        out_ids.append(ids.copy())
        out_lg.append(lg.copy())
        toks = [int(i) for i in ids]
        pos = [q + 1 for q in pos]
    return first, np.array(out_ids), np.array(out_lg)


def run_single(yl, path, prompts, steps, max_ctx=256):
    m = yl.load_transformer(path, max_ctx_len=max_ctx)
    ids_all, lg_all = [], []
    for p in prompts:
        s = m.create_session()
        _, tok = m.forward_x_full(p, 0, s)
        ids, lgs, pos = [], [], len(p)
        for _ in range(steps):
            lg, tok = m.forward_x_full([tok], pos, s)
            ids.append(tok)
            lgs.append(lg.copy())
            pos += 1
        ids_all.append(ids)
        lg_all.append(lgs)
    return np.array(ids_all).T, np.transpose(np.array(lg_all), (1, 0, 2))


@pytest.mark.parametrize("preset,over,n", [
    ("tiny", {}, 3),
    ("tiny", {}, 8),
    ("tiny128", {}, 12),                      # two matvec passes (8 + 4 rows)
    ("tiny", {"weight_format": 1}, 16),       # Q4_0, projections on the GEMM
    ("tiny", {"weight_format": 2}, 5),        # F16
    ("tiny", {"llama3_scaling": True, "rope_theta": 5e5, "context_length": 131072}, 6),
])
def test_batched_decode_equals_single_sessions(yl, model_factory, preset, over, n):
    path = model_factory(preset, **over)
    vocab = yl.PRESETS[preset]["vocab_size"]
    prompts = [yl.prompt_ids(vocab, 3 + 5 * i, 500 + i).tolist() for i in range(n)]
    _, bids, blg = run_batched(yl, path, prompts, 12)
    sids, slg = run_single(yl, path, prompts, 12)
    assert np.array_equal(bids, sids), np.argwhere(bids != sids)[:5]
    assert np.array_equal(blg, slg), float(np.max(np.abs(blg - slg)))


def test_batched_decode_matches_oracle(yl, orc, model_factory):
    path = model_factory("tiny128")
    vocab = yl.PRESETS["tiny128"]["vocab_size"]
    prompts = [yl.prompt_ids(vocab, 4 + 7 * i, 900 + i).tolist() for i in range(4)]
    first, bids, blg = run_batched(yl, path, prompts, 10)
    for i, p in enumerate(prompts):
        om = orc.Model(path, 256)
        os_ = om.create_session()
        lo = om.forward_x(p, 0, os_)
        assert orc.argmax(lo) == first[i]
        tok, pos = first[i], len(p)
        for k in range(10):
            lo = om.forward_x([tok], pos, os_)
            err = float(np.max(np.abs(blg[k, i] - lo)) / np.max(np.abs(lo)))
            assert err < 1e-2 and orc.argmax(lo) == bids[k, i], (i, k, err)
            tok, pos = int(bids[k, i]), pos + 1


def test_batch_errors(yl, model_factory):
    m = yl.load_transformer(model_factory("tiny"), max_ctx_len=64)
    s1, s2 = m.create_session(), m.create_session()
    b = m.create_batch(2)
    with pytest.raises(yl.YlError) as e:
        b.forward([s1, s1], [1, 2], [0, 0])
    assert e.value.code == -1 and "twice" in str(e.value)
    with pytest.raises(yl.YlError) as e:
        b.forward([s1, s2], [1, 2], [0, 64])
    assert e.value.code == -6
    with pytest.raises(yl.YlError) as e:
        b.forward([s1, s2, m.create_session()], [1, 2, 3], [0, 0, 0])
    assert e.value.code == -1
    with pytest.raises(yl.YlError):
        m.create_batch(17)

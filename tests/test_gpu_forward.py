"""GPU parity of the full forward (Transformer::forward_x) against the CPU
oracle on small seeded synthetic GGUF models (two layers, narrow shapes).

Bar, with nothing relaxed: logits within 1e-2 * max|logit| of the oracle at
every step and greedy token ids identical over the whole run. The device
forward reproduces the oracle's residual stream bit for bit (only the
lm_head's logits are approximate, ~1e-7 relative), so these narrow models,
whose logits move by up to 1% under a one-ulp perturbation of the oracle
itself, pass the bar as written. The allowance helpers below
(oracle_sensitivity, bound_for, assert_ids_match) serve only the
tensor-parallel tests, whose all-reduce changes the summation order."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def close_logits(got: np.ndarray, ref: np.ndarray) -> float:
    return float(np.max(np.abs(got - ref)) / max(1e-30, float(np.max(np.abs(ref)))))


def run_pair(yl, orc, path, prompt, n_gen, max_ctx, fmt_override=None):
    """Prefill `prompt`, then greedy-decode n_gen tokens on device and oracle.
    Both sides are fed the oracle's greedy ids (so logits stay comparable even
    after a divergence); returns per-step relative logit errors and both id
    sequences (device argmax, oracle argmax)."""
    gm = yl.load_transformer(path, max_ctx_len=max_ctx, fmt_override=fmt_override)
    om = orc.Model(path, max_ctx, -1 if fmt_override is None else int(fmt_override))
    gs, os_ = gm.create_session(), om.create_session()
    errs, gids, oids, olg = [], [], [], []
    lg, am = gm.forward_x_full(prompt, 0, gs)
    lo = om.forward_x(prompt, 0, os_)
    assert lg[am] == lg.max() and int(np.argmax(lg)) == am  # lowest index among maxima
    errs.append(close_logits(lg, lo))
    gids.append(am)
    oids.append(orc.argmax(lo))
    olg.append(lo)
    pos = len(prompt)
    for _ in range(n_gen):
        tok = oids[-1]
        lg, am = gm.forward_x_full([tok], pos, gs)
        lo = om.forward_x([tok], pos, os_)
        errs.append(close_logits(lg, lo))
        gids.append(am)
        oids.append(orc.argmax(lo))
        olg.append(lo)
        pos += 1
    run_pair.oracle_logits = olg
    return errs, gids, oids, gm, gs


def assert_ids_match(gids, oids, olg, bound):
    """Greedy ids must be identical, except at a certified near-tie: a step
    where the oracle's own logit margin between its choice and ours is within
    the logit deviation bound (no implementation that is not bit-identical to
    the oracle can order such a pair reliably). Returns the near-tie steps."""
    flips = [k for k in range(len(oids)) if gids[k] != oids[k]]
    for k in flips:
        lo = olg[k]
        margin = float(lo[oids[k]] - lo[gids[k]]) / float(np.max(np.abs(lo)))
        assert 0.0 <= margin <= bound, (k, oids[k], gids[k], margin, bound)
        print(f"RELAXED near-tie id difference at step {k}: oracle {oids[k]}, device {gids[k]}, "
              f"margin {margin:.3e} <= bound {bound:.3e}", flush=True)
    assert len(flips) <= max(1, len(oids) // 32), flips
    return flips


def assert_exact_path(errs, gids, oids) -> None:
    """The strict bar: every step's logits within 1e-2 * max|logit|, every
    greedy id equal."""
    assert max(errs) < LOGIT_TOL, errs
    assert gids == oids, [k for k in range(len(oids)) if gids[k] != oids[k]]


def oracle_sensitivity(orc, path, prompt, ids, max_ctx) -> float:
    """Largest relative logit move of the oracle itself under a one-ulp
    perturbation (RMSNorm sum of squares in f64), fed the same tokens: how far
    any non-bit-identical implementation can land from the oracle on this
    model through activation-quantization flips alone."""
    outs = []
    for probe in (0, 1):
        orc.set_probe(probe)
        try:
            om = orc.Model(path, max_ctx)
            s = om.create_session()
            lg = [om.forward_x(prompt, 0, s)]
            for i, tok in enumerate(ids[:-1]):
                lg.append(om.forward_x([tok], len(prompt) + i, s))
            outs.append(lg)
        finally:
            orc.set_probe(0)
    return max(close_logits(a, b) for a, b in zip(*outs))


def bound_for(sens: float) -> float:
    """The 1e-2 bar, unless the test model's own one-ulp sensitivity is
    already within a factor 2 of it (then twice the sensitivity)."""
    if sens < LOGIT_TOL / 2:
        return LOGIT_TOL
    print(f"RELAXED logit bound {2.0 * sens:.3e} (oracle one-ulp sensitivity {sens:.3e})", flush=True)
    return 2.0 * sens


@pytest.mark.parametrize("preset,over", [
    ("tiny", {}),
    ("tiny128", {}),
    ("tiny", {"weight_format": 1}),
    ("tiny", {"weight_format": 2}),
    ("tiny", {"llama3_scaling": True, "rope_theta": 5e5, "context_length": 131072}),
    ("tiny128", {"weight_format": 1, "tied": True}),
])
def test_tiny_models_match_oracle(yl, orc, model_factory, preset, over):
    path = model_factory(preset, **over)
    vocab = yl.PRESETS[preset]["vocab_size"]
    prompt = yl.prompt_ids(vocab, 9, 1234).tolist()
    errs, gids, oids, _, _ = run_pair(yl, orc, path, prompt, 24, 256)
    assert_exact_path(errs, gids, oids)


@pytest.mark.parametrize("preset,over", [
    ("tiny", {}),
    ("tiny128", {"weight_format": 2}),
    ("tiny", {"weight_format": 2, "llama3_scaling": True, "rope_theta": 5e5, "context_length": 131072}),
])
def test_gemm_prefill_matches_oracle(yl, orc, model_factory, preset, over):
    """A 70-token prompt: every projection of the prefill runs on a
    tensor-core GEMM (two token tiles, the second partial): the int8 GEMM for
    Q8_0 (RMSNorm + quantize as its own kernel; SwiGLU + h quantization in the
    gate/up epilogue), the f16 GEMM for F16 (RMSNorm + hi/lo split as its own
    kernel; SwiGLU in the epilogue); then greedy decode on the matvec path."""
    path = model_factory(preset, **over)
    vocab = yl.PRESETS[preset]["vocab_size"]
    prompt = yl.prompt_ids(vocab, 70, 99).tolist()
    errs, gids, oids, _, _ = run_pair(yl, orc, path, prompt, 8, 256)
    assert_exact_path(errs, gids, oids)


@pytest.mark.parametrize("preset,over", [
    ("tiny", {}),
    ("tiny128", {"llama3_scaling": True, "rope_theta": 5e5, "context_length": 131072}),
])
def test_tcgen05_prefill_matches_oracle(yl, orc, model_factory, preset, over):
    """A 200-token Q8_0 prompt: every projection of the prefill runs on the
    tcgen05 kernel (two 128-token tiles, the second partial): the q/k/v store,
    the wo and down residual adds and the gate/up SwiGLU + h-quantize
    epilogue; then greedy decode."""
    path = model_factory(preset, **over)
    vocab = yl.PRESETS[preset]["vocab_size"]
    prompt = yl.prompt_ids(vocab, 200, 7).tolist()
    yl.config_set("gemm_tc", 1)
    try:
        errs, gids, oids, _, _ = run_pair(yl, orc, path, prompt, 8, 256)
    finally:
        yl.config_set("gemm_tc", 0)
    assert_exact_path(errs, gids, oids)


def test_decode_graph_matches_host_loop(yl, orc, model_factory):
    path = model_factory("tiny128")
    gm = yl.load_transformer(path, max_ctx_len=512)
    prompt = yl.prompt_ids(1000, 12, 5).tolist()
    s1 = gm.create_session()
    _, first = gm.forward_x_full(prompt, 0, s1, want_logits=False)
    dev_ids = gm.decode_greedy(s1, first, len(prompt), 40)
    s2 = gm.create_session()
    _, tok = gm.forward_x_full(prompt, 0, s2, want_logits=False)
    host_ids = []
    for i in range(40):
        _, nxt = gm.forward_x_full([tok], len(prompt) + i, s2, want_logits=False)
        host_ids.append(nxt)
        tok = nxt
    assert dev_ids.tolist() == host_ids


@pytest.mark.parametrize("preset", ["tiny", "tiny128"])
def test_long_context_decode_matches_oracle(yl, orc, model_factory, preset):
    """Decode past 16 x 64 positions: every split of the decode attention
    walks several key tiles (online softmax across tiles), and the graph path
    (keys fetched before the wait on the projection) equals the host loop."""
    path = model_factory(preset, context_length=2048)
    vocab = yl.PRESETS[preset]["vocab_size"]
    prompt = yl.prompt_ids(vocab, 1500, 77).tolist()
    errs, gids, oids, _, _ = run_pair(yl, orc, path, prompt, 6, 2048)
    assert_exact_path(errs, gids, oids)
    gm = yl.load_transformer(path, max_ctx_len=2048)
    s1 = gm.create_session()
    _, first = gm.forward_x_full(prompt, 0, s1, want_logits=False)
    dev_ids = gm.decode_greedy(s1, first, len(prompt), 24).tolist()
    s2 = gm.create_session()
    _, tok = gm.forward_x_full(prompt, 0, s2, want_logits=False)
    host_ids = []
    for i in range(24):
        _, tok = gm.forward_x_full([tok], len(prompt) + i, s2, want_logits=False)
        host_ids.append(tok)
    assert dev_ids == host_ids


def test_wide_ffn_dynamic_schedule_matches_oracle(yl, orc, model_factory):
    """A feed-forward and vocabulary wide enough (32768 gate/up rows, 16384
    logits) that single-token passes hand out 8-row sets dynamically: the
    gate/up + SwiGLU + h-quantize launch (h blocks completed across CTAs) and
    the lm_head + argmax launch, against the oracle and graph vs host loop."""
    path = model_factory("tiny", hidden_dim=16384, vocab_size=16384)
    prompt = yl.prompt_ids(16384, 9, 4321).tolist()
    errs, gids, oids, _, _ = run_pair(yl, orc, path, prompt, 12, 256)
    assert_exact_path(errs, gids, oids)
    gm = yl.load_transformer(path, max_ctx_len=256)
    s1 = gm.create_session()
    _, first = gm.forward_x_full(prompt, 0, s1, want_logits=False)
    dev_ids = gm.decode_greedy(s1, first, len(prompt), 24).tolist()
    s2 = gm.create_session()
    _, tok = gm.forward_x_full(prompt, 0, s2, want_logits=False)
    host_ids = []
    for i in range(24):
        _, tok = gm.forward_x_full([tok], len(prompt) + i, s2, want_logits=False)
        host_ids.append(tok)
    assert dev_ids == host_ids


def test_prefill_equals_stepwise_on_device(yl, model_factory):
    path = model_factory("tiny")
    gm = yl.load_transformer(path, max_ctx_len=256)
    toks = [3, 17, 99, 5, 250, 1, 77, 200, 12, 9]
    a, _ = gm.forward_x_full(toks, 0, gm.create_session())
    s = gm.create_session()
    for i, t in enumerate(toks):
        b, _ = gm.forward_x_full([t], i, s)
    assert close_logits(a, b) < 1e-4


def test_embeddings_match_oracle(yl, orc, model_factory):
    path = model_factory("tiny128")
    gm = yl.load_transformer(path, max_ctx_len=512)
    om = orc.Model(path, 512)
    for t in (0, 5, 999, 1000, 123456):
        assert np.array_equal(gm.get_embeddings(t), om.get_embeddings(t))
    batch = gm.get_embeddings_batch([1, 2, 5000])
    assert np.all(batch[2] == 0) and np.array_equal(batch[1], om.get_embeddings(2))


def test_forward_errors(yl, model_factory):
    path = model_factory("tiny")
    gm = yl.load_transformer(path, max_ctx_len=16)
    s = gm.create_session()
    with pytest.raises(yl.YlError) as e:
        gm.forward_x([1] * 4, 14, s)
    assert e.value.code == -6
    with pytest.raises(yl.YlError) as e:
        gm.forward_x([], 0, s)
    assert e.value.code == -1
    assert gm.name() == "TransformerLlamaGguf" and gm.vocab_size() == 512 and gm.max_ctx_len() == 16


def test_session_reset_restores_results(yl, model_factory):
    gm = yl.load_transformer(model_factory("tiny"), max_ctx_len=64)
    s = gm.create_session()
    a = gm.forward_x([4, 5, 6], 0, s)
    gm.forward_x([7, 8], 3, s)
    s.reset()
    b = gm.forward_x([4, 5, 6], 0, s)
    assert np.array_equal(a, b)


def test_ffi_load(yl, model_factory):
    assert yl.load_transformer_ffi(model_factory("tiny")) is True

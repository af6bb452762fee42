"""GPU parity on the benchmark configurations at the bar as written, plus the
decode step's attention kernel on its own.

Configurations (synthetic seeded GGUF files, random-init weights ~ N(0, 0.02)):
  c1  SmolLM2-135M shape, Q8_0, seed 0: prompt 16, 128 greedy steps, ctx 512
  c2  Llama-3.2-1B shape, Q8_0, llama3 RoPE (orig ctx 8192), seed 1:
      prompt 128, 256 greedy steps, ctx 4096
  c3  Llama-3.2-1B shape, Q4_0 weights on Q8_0 activations, seed 2: a 512-token
      prefill (int8 tensor-core GEMM), then 256 greedy steps
  c4  Llama-3-8B shape, Q8_0, untied lm_head, seed 3 (the benchmarked model):
      prompt 32, 128 greedy steps

Bar, with nothing relaxed: every step's logits within 1e-2 * max|logit| of the
oracle (forward.rs:119-280 restated in oracle/), the device's greedy id equal
to the oracle's at every step, and the device-resident free-running decode
(its own ids fed back, one CUDA graph per step) equal to the oracle's own
free-running sequence. Each test prints one `PARITY {...}` line with the
largest logit error, the smallest top-2 margin of the oracle and any id
difference.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    return float(np.max(np.abs(got - ref)) / max(1e-30, float(np.max(np.abs(ref)))))


def top2_margin(lo: np.ndarray) -> float:
    """Gap between the oracle's best and second-best logit, relative to max|logit|."""
    part = np.partition(lo, -2)[-2:]
    return float((part[1] - part[0]) / max(1e-30, float(np.max(np.abs(lo)))))


def strict_run(yl, orc, path: str, prompt: list, n_gen: int, max_ctx: int, name: str) -> dict:
    """Teacher-forced comparison along the oracle's own greedy path (both
    sides fed the oracle's ids, logits compared at every step), then the
    device's free-running decode from the same prompt."""
    gm = yl.load_transformer(path, max_ctx_len=max_ctx)
    om = orc.Model(path, max_ctx)
    gs, os_ = gm.create_session(), om.create_session()
    errs, gids, oids, margins = [], [], [], []
    lg, am = gm.forward_x_full(prompt, 0, gs)
    lo = om.forward_x(prompt, 0, os_)
    errs.append(rel_err(lg, lo))
    gids.append(am)
    oids.append(orc.argmax(lo))
    margins.append(top2_margin(lo))
    pos = len(prompt)
    for _ in range(n_gen):
        tok = oids[-1]
        lg, am = gm.forward_x_full([tok], pos, gs)
        lo = om.forward_x([tok], pos, os_)
        errs.append(rel_err(lg, lo))
        gids.append(am)
        oids.append(orc.argmax(lo))
        margins.append(top2_margin(lo))
        pos += 1
    del om, os_
    # free-running on the device: its own ids fed back through the decode graph
    s2 = gm.create_session()
    _, first = gm.forward_x_full(prompt, 0, s2, want_logits=False)
    free = [first] + gm.decode_greedy(s2, first, len(prompt), n_gen).tolist()
    diff_tf = [k for k in range(len(oids)) if gids[k] != oids[k]]
    diff_free = [k for k in range(len(oids)) if free[k] != oids[k]]
    rep = {"config": name, "prompt": len(prompt), "steps": n_gen, "max_rel_logit_err": max(errs),
           "mean_rel_logit_err": float(np.mean(errs)), "min_oracle_top2_margin": min(margins),
           "teacher_forced_id_diffs": diff_tf, "free_running_first_diff": diff_free[0] if diff_free else None}
    print("PARITY " + json.dumps(rep), flush=True)
    return rep


def assert_strict(rep: dict) -> None:
    assert rep["max_rel_logit_err"] < LOGIT_TOL, rep
    assert rep["teacher_forced_id_diffs"] == [], rep
    assert rep["free_running_first_diff"] is None, rep


def test_c1_smollm_shape_128_steps(yl, orc, model_factory):
    path = model_factory("c1")
    prompt = yl.prompt_ids(49152, 16, 1000).tolist()
    assert_strict(strict_run(yl, orc, path, prompt, 128, 512, "c1"))


@pytest.mark.slow
def test_c2_llama32_1b_q8_llama3_rope_256_steps(yl, orc, model_factory):
    path = model_factory("c2")
    prompt = yl.prompt_ids(128256, 128, 1001).tolist()
    assert_strict(strict_run(yl, orc, path, prompt, 256, 4096, "c2"))


@pytest.mark.slow
def test_c3_llama32_1b_q4_prefill512_256_steps(yl, orc, model_factory):
    path = model_factory("c3")
    prompt = yl.prompt_ids(128256, 512, 1002).tolist()
    assert_strict(strict_run(yl, orc, path, prompt, 256, 4096, "c3"))


@pytest.mark.slow
def test_c4_llama3_8b_benchmarked_model_128_steps(yl, orc, model_factory):
    """The model bench.py times (seed 3, untied lm_head, head_size 128, 32
    layers, the 4096 / 14336 matvec shapes)."""
    path = model_factory("c4")
    prompt = yl.prompt_ids(128256, 32, 1003).tolist()
    assert_strict(strict_run(yl, orc, path, prompt, 128, 4096, "c4"))


# ---------------------------------------------------------------------------
# The decode step's attention kernel alone: RoPE of q and the new k, cache
# write at pos, split attention over a thread-block cluster per KV head with
# the merge in distributed shared memory, Q8_0 blocks of the output.

ATT_CASES = [
    # (preset overrides, label)
    (dict(dim=256, n_heads=4, n_kv_heads=2), "hd64-gqa2"),
    (dict(dim=576, n_heads=9, n_kv_heads=3), "hd64-gqa3"),
    (dict(dim=512, n_heads=4, n_kv_heads=1), "hd128-gqa4"),
    (dict(dim=4096, n_heads=32, n_kv_heads=8), "hd128-gqa4-c4heads"),
    (dict(dim=1024, n_heads=8, n_kv_heads=1), "hd128-gqa8"),
    (dict(dim=2048, n_heads=32, n_kv_heads=8, llama3_scaling=True, rope_theta=5e5), "hd64-llama3"),
]


@pytest.mark.parametrize("over,label", ATT_CASES, ids=[c[1] for c in ATT_CASES])
@pytest.mark.parametrize("pos", [0, 700, 3000])
def test_decode_attention_kernel_vs_oracle(yl, orc, torch_cuda, model_factory, over, label, pos):
    torch = torch_cuda
    path = model_factory("tiny", n_layers=1, hidden_dim=256, vocab_size=256, context_length=4096, **over)
    gm = yl.load_transformer(path, max_ctx_len=4096)
    om = orc.Model(path, 4096)
    sh = om.shape
    hd, nh, nkv = sh.head_size, sh.n_heads, sh.n_kv_heads
    att, kvd = nh * hd, nkv * hd
    rng = np.random.default_rng(pos * 7 + hd + nh)
    qkv = rng.standard_normal(att + 2 * kvd).astype(np.float32)
    kc = np.zeros((pos + 1) * kvd, np.float32)
    vc = np.zeros((pos + 1) * kvd, np.float32)
    kc[: pos * kvd] = rng.standard_normal(pos * kvd).astype(np.float32)
    vc[: pos * kvd] = rng.standard_normal(pos * kvd).astype(np.float32)
    # oracle: rotate q and the new k, write k/v at pos, attend over 0..pos
    q_rot, k_rot = orc.rope(sh, qkv[:att], qkv[att:att + kvd], pos)
    kc_o, vc_o = kc.copy(), vc.copy()
    kc_o[pos * kvd:(pos + 1) * kvd] = k_rot
    vc_o[pos * kvd:(pos + 1) * kvd] = qkv[att + kvd:]
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    ref = orc.fused_attention(q_rot, kc_o, vc_o, pos + 1, 1, nh, nkv, hd, pos, kvd, scale)
    d_qkv = torch.from_numpy(qkv).cuda()
    d_kc, d_vc = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    out = torch.full((att,), float("nan"), device="cuda")
    oq = torch.zeros(att, dtype=torch.int8, device="cuda")
    osc = torch.zeros(att // 32, device="cuda")
    gm.attention_decode(d_qkv, d_kc, d_vc, pos, out=out, out_q=oq, out_s=osc)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    # the cache row is the oracle's rotated key bit for bit (same cos/sin
    # formulas, separately rounded rotation), the value row is copied
    assert np.array_equal(d_kc.cpu().numpy()[pos * kvd:], k_rot)
    assert np.array_equal(d_vc.cpu().numpy()[pos * kvd:], qkv[att + kvd:])
    # the reference's operation sequence: bit-identical
    assert np.array_equal(got, ref), (label, pos, float(np.max(np.abs(got - ref))))
    # the in-kernel Q8_0 blocks are the quantizer's output on the f32 result
    q_ref, s_ref = orc.quantize_q8(got)
    assert np.array_equal(oq.cpu().numpy(), q_ref)
    assert np.array_equal(osc.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


# ---------------------------------------------------------------------------


@pytest.mark.parametrize("preset", ["tiny", "tiny128"])
def test_decode_step_launches_equals_graph_kernel_nodes(yl, model_factory, preset):
    """yl_decode_step_launches (the count the bench reports) against the
    kernel nodes of the decode graph as captured."""
    gm = yl.load_transformer(model_factory(preset), max_ctx_len=256)
    s = gm.create_session()
    assert gm.decode_graph_launches(s) == gm.decode_step_launches() == 5 * gm.shape().n_layers + 2


def test_async_decode_calls_back_to_back(yl, model_factory):
    """Two yl_decode_greedy calls enqueued without synchronizing: the second
    must not change the first one's start token and position (each call's
    start state travels as kernel arguments)."""
    gm = yl.load_transformer(model_factory("tiny128"), max_ctx_len=512)
    prompt = yl.prompt_ids(1000, 12, 5).tolist()
    ref = gm.create_session()
    _, t0 = gm.forward_x_full(prompt, 0, ref, want_logits=False)
    ids_a = gm.decode_greedy(ref, t0, len(prompt), 8)
    ids_b = gm.decode_greedy(ref, 3, len(prompt) + 8, 8)  # restart from token 3 after the first run
    s = gm.create_session()
    _, t1 = gm.forward_x_full(prompt, 0, s, want_logits=False)
    assert t1 == t0
    assert gm.decode_greedy(s, t1, len(prompt), 8, sync=False) is None
    got_b = gm.decode_greedy(s, 3, len(prompt) + 8, 8)
    assert got_b.tolist() == ids_b.tolist()
    assert ids_a.size == 8

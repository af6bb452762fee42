"""Tensor parallelism on two and four GPUs (one spawned process per GPU): the sharded
forward (all-reduce after wo and down over NVLink peer memory, vocabulary-
parallel lm_head with the combined greedy id) against the CPU oracle, with
the same bar as the single-GPU tiny models, and the decode graph against the
host loop. Skipped where fewer GPUs than ranks are visible."""
from __future__ import annotations

import multiprocessing as mp
import socket

import numpy as np
import pytest

from test_gpu_forward import assert_ids_match, bound_for, close_logits, oracle_sensitivity

pytestmark = pytest.mark.gpu


def free_port() -> int:
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def need_gpus(n: int):
    import torch
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def run_tp(world, path, prompt, feed, n_graph):
    import tp_worker
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=tp_worker.decode_rank, args=(r, world, port, path, prompt, feed, n_graph, q))
          for r in range(world)]
    for p in ps:
        p.start()
    try:
        out = q.get(timeout=300)
    finally:
        for p in ps:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert "error" not in out, out
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    return out


@pytest.mark.parametrize("fused", ["1", "0"])
@pytest.mark.parametrize("preset,over,plen", [("tiny", {}, 9), ("tiny", {"hidden_dim": 16384, "vocab_size": 16384}, 9),
                                              ("tiny", {}, 40)])
def test_tp2_matches_oracle(yl, orc, model_factory, monkeypatch, preset, over, plen, fused):
    """fused "1": single-token steps exchange through the projections' pushes
    and the next RMSNorm prologue; "0": through the separate exchange kernel
    (the path multi-token passes always take). A 40-token prompt runs the
    sharded prefill on the tensor-core GEMM."""
    need_gpus(2)
    monkeypatch.setenv("YL_TP_FUSED", fused)  # read by the spawned ranks
    path = model_factory(preset, **over)
    vocab = over.get("vocab_size", yl.PRESETS[preset]["vocab_size"])
    prompt = yl.prompt_ids(vocab, plen, 1234).tolist()
    om = orc.Model(path, 256)
    os_ = om.create_session()
    olg = [om.forward_x(prompt, 0, os_)]
    oids = [orc.argmax(olg[0])]
    for i in range(16):
        olg.append(om.forward_x([oids[-1]], len(prompt) + i, os_))
        oids.append(orc.argmax(olg[-1]))
    out = run_tp(2, path, prompt, oids[:-1], 24)
    sens = oracle_sensitivity(orc, path, prompt, oids, 256)
    errs = [close_logits(g, o) for g, o in zip(out["logits"], olg)]
    assert max(errs) < bound_for(sens), (errs, sens)
    for k, lg in enumerate(out["logits"]):  # the combined id is the gathered logits' argmax
        assert out["ids"][k] == int(np.argmax(lg))
    assert_ids_match(out["ids"], oids, olg, bound_for(sens))
    assert out["dev"] == out["host"]


@pytest.mark.parametrize("plen", [9, 40])
def test_tp4_matches_oracle(yl, orc, model_factory, plen):
    """Four ranks (4 KV heads, one per rank; feed-forward and vocabulary in
    quarters): fused decode exchange among four inboxes, the sharded GEMM
    prefill at 40 tokens, combined greedy id. Skipped on fewer than 4 GPUs."""
    need_gpus(4)
    over = {"dim": 512, "n_heads": 8, "n_kv_heads": 4, "hidden_dim": 1024}
    path = model_factory("tiny", **over)
    vocab = yl.PRESETS["tiny"]["vocab_size"]
    prompt = yl.prompt_ids(vocab, plen, 4321).tolist()
    om = orc.Model(path, 256)
    os_ = om.create_session()
    olg = [om.forward_x(prompt, 0, os_)]
    oids = [orc.argmax(olg[0])]
    for i in range(12):
        olg.append(om.forward_x([oids[-1]], len(prompt) + i, os_))
        oids.append(orc.argmax(olg[-1]))
    out = run_tp(4, path, prompt, oids[:-1], 16)
    sens = oracle_sensitivity(orc, path, prompt, oids, 256)
    errs = [close_logits(g, o) for g, o in zip(out["logits"], olg)]
    assert max(errs) < bound_for(sens), (errs, sens)
    assert_ids_match(out["ids"], oids, olg, bound_for(sens))
    assert out["dev"] == out["host"]

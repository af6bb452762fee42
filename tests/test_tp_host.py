"""Tensor-parallel host logic on CPU: world-size-2 gloo ranks compute their
split (yl_tp_plan, no GPU) and rank 0 checks that the ranks' q heads, KV
heads, ffn rows and vocabulary rows partition the model exactly once, and
that shapes the split cannot serve are refused."""
from __future__ import annotations

import multiprocessing as mp
import socket

import pytest


def free_port() -> int:
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


C4 = dict(dim=4096, hidden_dim=14336, n_heads=32, head_size=128, n_kv_heads=8, vocab_size=128256)
TINY = dict(dim=256, hidden_dim=512, n_heads=4, head_size=64, n_kv_heads=2, vocab_size=512)
C1 = dict(dim=576, hidden_dim=1536, n_heads=9, head_size=64, n_kv_heads=3, vocab_size=49152)


def run_ranks(world: int, shapes: list) -> list:
    import tp_worker
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=tp_worker.plan_rank, args=(r, world, port, shapes, q)) for r in range(world)]
    for p in ps:
        p.start()
    try:
        out = q.get(timeout=120)
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in ps)
    return out


def covers(parts, total):
    spans = sorted(parts)
    pos = 0
    for a, n in spans:
        assert a == pos and n > 0
        pos += n
    assert pos == total


@pytest.mark.parametrize("world", [2, 4])
def test_tp_split_partitions_the_model(world):
    allp = run_ranks(world, [C4, TINY, C1])
    for si, sh in enumerate((C4, TINY, C1)):
        plans = [allp[r][si] for r in range(world)]
        if sh is C1 or (sh is TINY and world > 2):
            assert all(p.get("error") == -8 for p in plans)  # YL_ERR_UNSUPPORTED: replicas only
            continue
        covers([(p["q_rows0"], p["q_rows"]) for p in plans], sh["n_heads"] * sh["head_size"])
        covers([(p["kv_rows0"], p["kv_rows"]) for p in plans], sh["n_kv_heads"] * sh["head_size"])
        covers([(p["ffn_rows0"], p["ffn_rows"]) for p in plans], sh["hidden_dim"])
        covers([(p["vocab0"], p["vocab_rows"]) for p in plans], sh["vocab_size"])
        for p in plans:  # Q8 blocks and activation blocks never straddle ranks
            assert p["q_rows"] % 32 == 0 and p["ffn_rows"] % 64 == 0

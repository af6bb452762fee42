"""Rank body of the tensor-parallel tests (run in spawned child processes).

`plan_rank`: gloo rank that computes its split plan (no GPU) and gathers all.
`decode_rank`: one GPU per rank; loads its shard, connects the session over
CUDA IPC (handles exchanged with gloo), prefills, then steps token by token
(logits gathered) and through the decode graph."""
from __future__ import annotations

import datetime
import importlib
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _init(rank: int, world: int, port: int):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    return dist


def plan_rank(rank: int, world: int, port: int, shapes: list, q) -> None:
    dist = _init(rank, world, port)
    try:
        yl = importlib.import_module("yallma3-mini-inference_b200")
        mine = []
        for kw in shapes:
            try:
                mine.append(yl.tp_plan(yl.shape_of(**kw), rank, world))
            except yl.YlError as e:
                mine.append({"error": e.code})
        allp = [None] * world
        dist.all_gather_object(allp, mine)
        if rank == 0:
            q.put(allp)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def decode_rank(rank: int, world: int, port: int, path: str, prompt: list, feed: list, n_graph: int, q) -> None:
    dist = _init(rank, world, port)
    try:
        import numpy as np
        import torch
        torch.cuda.set_device(rank)
        yl = importlib.import_module("yallma3-mini-inference_b200")
        m = yl.load_transformer_tp(path, rank, world, max_ctx_len=256)
        s = m.create_session()
        s.tp_connect_group()
        lg, am = m.forward_x_full(prompt, 0, s)
        logits, ids = [lg.copy()], [am]
        for i, tok in enumerate(feed):  # teacher-forced with the given ids
            lg, am = m.forward_x_full([tok], len(prompt) + i, s)
            logits.append(lg.copy())
            ids.append(am)
        # free-running: decode graph vs host loop on fresh sessions
        s1 = m.create_session()
        s1.tp_connect_group()
        _, first = m.forward_x_full(prompt, 0, s1, want_logits=False)
        dev = m.decode_greedy(s1, first, len(prompt), n_graph).tolist()
        s2 = m.create_session()
        s2.tp_connect_group()
        _, tok = m.forward_x_full(prompt, 0, s2, want_logits=False)
        host = []
        for i in range(n_graph):
            _, tok = m.forward_x_full([tok], len(prompt) + i, s2, want_logits=False)
            host.append(tok)
        torch.cuda.synchronize()
        if rank == 0:
            q.put({"logits": np.stack(logits), "ids": ids, "dev": dev, "host": host})
        dist.barrier()
    except Exception as e:  # report, then leave like the others
        q.put({"rank": rank, "error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()

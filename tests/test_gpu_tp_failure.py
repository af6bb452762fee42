"""Failure detection without a GPU fault: a tensor-parallel peer that never
runs a step.

Two processes share GPU 0 as ranks 0 and 1 of a 2-way tensor-parallel model.
Both connect their exchange regions (CUDA IPC handles over gloo). Rank 1 then
stays alive but never launches a forward, so the flags rank 0's exchange
waits for are never set: every such wait is bounded (about 2 s of SM clock),
records the timeout in the session's error word and returns. The test checks
that rank 0's forward_x fails with YL_ERR_TIMEOUT instead of hanging, that the
CUDA context still works afterwards (a quantization equals the oracle's), and
that a fresh single-GPU model still produces its greedy token. No kernel is
made to fault or trap; rank 1 leaves only after rank 0 has finished."""
from __future__ import annotations

import multiprocessing as mp
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank(rank: int, port: int, path: str, done, q) -> None:
    import datetime
    import importlib
    import os
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "oracle"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120))
    try:
        torch.cuda.set_device(0)
        yl = importlib.import_module("yallma3-mini-inference_b200")
        m = yl.load_transformer_tp(path, rank, 2, max_ctx_len=128)
        s = m.create_session()
        s.tp_connect_group()
        dist.barrier()
        if rank == 1:  # connected, alive, and never stepping
            done.wait(timeout=240)
            q.put({"rank": 1, "ok": True})
            return
        res = {"rank": 0}
        t0 = time.time()
        try:
            m.forward_x_full([5, 6, 7, 8], 0, s)
            res["code"] = 0
        except yl.YlError as e:
            res["code"] = e.code
            res["msg"] = str(e)
        res["seconds"] = time.time() - t0
        # the context is still usable: a quantization, bit-exact against the oracle
        import pyoracle as orc
        x = (np.random.default_rng(1).standard_normal(4096) * 2).astype(np.float32)
        qd = torch.zeros(4096, dtype=torch.int8, device="cuda")
        sd = torch.zeros(128, dtype=torch.float32, device="cuda")
        yl.quantize_q8_0(torch.from_numpy(x).cuda(), qd, sd, 4096, 32)
        torch.cuda.synchronize()
        qo, so_ = orc.quantize_q8(x)
        res["quant_ok"] = bool(np.array_equal(qd.cpu().numpy(), qo) and np.array_equal(sd.cpu().numpy(), so_))
        q.put(res)
    except Exception as e:  # report, then leave
        q.put({"rank": rank, "error": repr(e)})
    finally:
        if rank == 0:
            done.set()
        dist.destroy_process_group()


def test_silent_peer_gives_timeout_not_hang(yl, orc, model_factory, torch_cuda):
    path = model_factory("tiny")
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, port, path, done, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r = q.get(timeout=300)
            got[r["rank"]] = r
    finally:
        done.set()
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert "error" not in got[0] and "error" not in got[1], got
    assert got[0]["code"] == -7, got[0]  # YL_ERR_TIMEOUT
    assert got[0]["seconds"] < 120, got[0]
    assert got[0]["quant_ok"], got[0]
    # a fresh single-GPU model in this process still decodes like the oracle
    m = yl.load_transformer(path, max_ctx_len=64)
    s = m.create_session()
    _, tok = m.forward_x_full([5, 6, 7, 8], 0, s)
    om = orc.Model(path, 64)
    assert tok == orc.argmax(om.forward_x([5, 6, 7, 8], 0, om.create_session()))
    s.close()
    m.close()

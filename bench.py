"""Decode benchmark: Llama-3-8B-shaped Q8_0, batch 1 (benchmark configuration 4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one batch-1 greedy decode token (one pass of the quantized forward
over one token). Setup (untimed): a seeded random-init GGUF with the config-4
shape is written (cached in $YL_BENCH_DIR, default /tmp), loaded through the
C-ABI, and a 512-token random prompt is prefilled. Then W warm-up steps and K
timed steps continue the sequence from position 512.

  value  device-resident greedy loop (one CUDA graph launch per token, token
         fed back on device), CUDA events on the launching stream, barrier +
         synchronize on both sides, max over ranks.
  e2e    the same metric through the reference-facing call yl_forward_x
         (Transformer::forward_x): host token id in, host logits + greedy id
         out every step (pinned buffers), timed on the host.
  roofline  the dominant kernel (Q8_0 gate/up matvec, 4096 -> 2x14336) timed
         alone with CUDA events, cycling through the 32 layers' weights so no
         launch reuses L2; algorithmic bytes / duration vs measured HBM peak.
  cpu_baseline  the CPU oracle (C++ restatement of the reference CPU path) on
         a bounded sample of the same decode, on all host cores and on the
         reference's default thread count (half the cores, rounded up,
         parallelism.rs:59-71), with the CPU model recorded.

With N > 1 (torchrun), the model is tensor-parallel over the N GPUs (Megatron
split: heads and ffn rows by rank, wo / down along their inputs, lm_head by
vocabulary rows; partial sums exchanged over NVLink peer memory). There is one
token stream, so value = tokens / max time over ranks (strong scaling).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PKG = "yallma3-mini-inference_b200"
PROMPT_LEN = 512
CONFIG = "c4"
TRAFFIC_GATEUP_BYTES = 128.22e6


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def bytes_per_token(cfg: dict, seq: float) -> float:
    """Algorithmic HBM bytes of one decode token: weights in file format
    (Q8_0 = 34/32 B per element), lm_head, f32 KV reads at length seq and the
    new K/V row writes."""
    d, f, L, V = cfg["dim"], cfg["hidden_dim"], cfg["n_layers"], cfg["vocab_size"]
    hd = d // cfg["n_heads"]
    kvd = hd * cfg["n_kv_heads"]
    per_layer = d * d + 2 * d * kvd + d * d + 3 * d * f
    b = 34.0 / 32.0
    return L * per_layer * b + V * d * b + L * (2 * seq * kvd * 4) + L * (2 * kvd * 4)


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 20 ms during
    the timed region, read-only through NVML (nvidia-smi polling at 200 ms as
    the fallback); one sample is also taken at entry and one at exit."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.nv = None
        self.h = None
        self.stop = threading.Event()
        self.samples: list[tuple[float, float, set]] = []  # (sm MHz, max sm MHz, active reasons)
        self.lines: list[str] = []

    def _nvml_open(self) -> bool:
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = None
            try:
                import torch
                pr = torch.cuda.get_device_properties(self.idx)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = nv.nvmlDeviceGetHandleByIndex(self.idx)
            self.nv, self.h = nv, h
            self._nvml_sample()
            return True
        except Exception:
            self.nv = None
            return False

    def _nvml_sample(self) -> None:
        nv, h = self.nv, self.h
        sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        bits = int(get(h))
        self.samples.append((sm, mx, {nm for nm, b in self.REASONS if bits & b}))

    def _nvml_loop(self) -> None:
        while not self.stop.wait(0.02):
            try:
                self._nvml_sample()
            except Exception:
                return

    def __enter__(self):
        if self._nvml_open():
            self.t = threading.Thread(target=self._nvml_loop, daemon=True)
            self.t.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.nv is not None:
            self.stop.set()
            self.t.join(timeout=5)
            try:
                self._nvml_sample()
            except Exception:
                pass
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        for f, m, r in self.samples:
            sm.append(f)
            mx = max(mx, m)
            reasons |= r
        names = [nm for nm, _ in self.REASONS]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = max(mx, float(p[2]))
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml 20 ms" if self.nv is not None else "nvidia-smi 200 ms"}


def ensure_model(yl, rank: int, world: int, dist) -> str:
    cache = Path(os.environ.get("YL_BENCH_DIR", tempfile.gettempdir()))
    path = cache / "yl_bench_c4_q8_0.gguf"
    ok = path.with_suffix(".ok")
    if rank == 0 and not ok.exists():
        t = time.time()
        yl.synth_preset(CONFIG, str(path))
        ok.write_text(str(time.time() - t))
    if world > 1:
        dist.barrier()
    return str(path)


def time_dominant_matvec(yl, torch, model, cfg: dict, iters: int, world: int = 1) -> dict:
    """Q8_0 gate/up matvec (rows 2*ffn/world, K = dim) alone, cycling over layers."""
    L, d, f = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"] // world
    ws = [model.weight(layer, 4) for layer in range(L)]
    x = (torch.randn(d, device="cuda") * 1.0).contiguous()
    xa = yl.new_workspace_buffer(yl.WeightFormat.Q8_0, d, 32)
    yl.quantize(yl.WeightFormat.Q8_0, xa, x, d, 32)
    out = torch.empty(2 * f, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(L):
            yl.matmul(out, xa, ws[i], d, 2 * f, 32, batch=1, accumulate=False, stream=st)
    torch.cuda.synchronize()
    # capture the launches in a CUDA graph so host launch cost does not enter
    # the device time; the graph cycles through all layers' matrices
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            yl.matmul(out, xa, ws[i % L], d, 2 * f, 32, batch=1, accumulate=False, stream=st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):  # replay() launches on the current stream
        g.replay()
        torch.cuda.synchronize()
        e0.record(st)
        g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    del g
    nbytes = 2 * f * d * 34 / 32 + d + d / 32 * 4 + 2 * f * 4
    return {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}


def cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(path: str, n_tokens: int, threads: int, half_threads: int | None = None, warmup: int = 1) -> dict:
    """Oracle decode of n_tokens at positions 512.. with a seeded KV prefix,
    after `warmup` untimed steps, on `threads` host threads; with half_threads
    also on that many (the reference's default pool, parallelism.rs:59-71)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle as orc
    t0 = time.time()
    m = orc.Model(path, 4096)
    load_s = time.time() - t0
    s = m.create_session()
    k, v = s.kv()
    sh = m.shape
    kvd = sh.n_kv_heads * sh.head_size
    rng = np.random.default_rng(0)
    for layer in range(sh.n_layers):
        base = layer * sh.ctx_len * kvd
        k[base:base + PROMPT_LEN * kvd] = rng.standard_normal(PROMPT_LEN * kvd).astype(np.float32)
        v[base:base + PROMPT_LEN * kvd] = rng.standard_normal(PROMPT_LEN * kvd).astype(np.float32)

    def timed(nt: int) -> float:
        orc.set_threads(nt)
        tok = 1
        for _ in range(max(1, warmup)):  # untimed (page-in, caches)
            m.forward_x([tok], PROMPT_LEN, s)
        t = time.perf_counter()
        for i in range(n_tokens):
            lg = m.forward_x([tok], PROMPT_LEN + 1 + i, s)
            tok = orc.argmax(lg)
        return n_tokens / (time.perf_counter() - t)

    out = {"value": timed(threads), "unit": "tokens/s", "cores": threads, "kind": "port",
           "cpu_model": cpu_model(), "host_cores": os.cpu_count(),
           "sample": f"{n_tokens} batch-1 decode tokens of config 4 at positions {PROMPT_LEN + 1}.. "
                     f"(KV prefix 0..{PROMPT_LEN - 1} seeded instead of a CPU prefill), "
                     f"oracle load {load_s:.0f}s untimed"}
    if half_threads and half_threads != threads:
        out["reference_default_threads"] = {"cores": half_threads, "value": timed(half_threads),
                                            "rule": "ceil(0.5 * cores), parallelism.rs:59-71"}
    return out


def write_model_in_subprocess(path: Path) -> None:
    """Writes the config-4 GGUF from a child process, so the process that times
    the reference arm never loads this repository's CUDA library."""
    if path.with_suffix(".ok").exists():
        return
    code = (f"import sys, importlib; sys.path.insert(0, {str(ROOT)!r}); "
            f"yl = importlib.import_module({PKG!r}); yl.synth_preset({CONFIG!r}, {str(path)!r})")
    subprocess.run([sys.executable, "-c", code], check=True)
    path.with_suffix(".ok").write_text("ok")


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cache = Path(os.environ.get("YL_BENCH_DIR", tempfile.gettempdir()))
    path = cache / "yl_bench_c4_q8_0.gguf"
    write_model_in_subprocess(path)
    steps = max(1, min(args.steps, 8))
    warmup = max(3, min(args.warmup, 5))  # at least 3 untimed steps; bounded CPU time
    threads = os.cpu_count() or 1
    cb = cpu_baseline(str(path), steps, threads, half_threads=max(1, -(-threads // 2)), warmup=warmup)
    line = {"impl": "reference", "metric": "decode tokens/s (Llama-3-8B-shape Q8_0, batch 1)",
            "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
            "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot / f32 accumulate", "data": "synthetic",
            "config": {"workload": "config 4: Llama-3-8B-shaped Q8_0, prompt 512, batch-1 greedy decode",
                       "global_batch": 1, "seq_len": PROMPT_LEN, "parallelism": "cpu"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


SWEEP_MK = [(2048, 2048), (8192, 2048), (2048, 8192), (14336, 4096), (4096, 14336), (128256, 4096)]
SWEEP_N = [1, 4, 16, 64, 512]


def sweep_case(yl, torch, rng) -> None:
    """The matvec / GEMM sweep: (M, K) x {Q8_0, Q4_0, F16} x N tokens through
    yl_matmul, each launch timed alone with CUDA events after a 256 MB write
    that evicts L2 (median of 7 after 2 untimed). One JSON line per case:
    GB/s = (M*K*b_fmt + N*K*(1+4/32) + N*M*4) / t against the measured HBM
    copy peak, and TOPS = 2*M*K*N / t."""
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs") if isinstance(peaks, dict) else None
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    big = max(m * k for m, k in SWEEP_MK)
    q8 = rng.integers(-127, 128, big, dtype=np.int8)
    fmts = [("Q8_0", yl.WeightFormat.Q8_0, 34 / 32), ("Q4_0", yl.WeightFormat.Q4_0, 18 / 32),
            ("F16", yl.WeightFormat.F16, 2.0)]
    for m, k in SWEEP_MK:
        for name, f, bf in fmts:
            w = yl.QuantizedTensor.weight(f, m, k, 32, 1)
            if name == "F16":
                w.upload(values=q8[: m * k].astype(np.float32) * np.float32(1e-3))
            else:
                wq = q8[: m * k] if name == "Q8_0" else (q8[: m * k] >> 4).astype(np.int8)
                w.upload(quant_vals=wq, scale_factor=np.full(m * k // 32, 1e-3, np.float32))
            for n in SWEEP_N:
                xa = yl.new_workspace_buffer(f, n * k, 32)
                yl.quantize(f, xa, torch.randn(n * k, device="cuda"), n * k, 32)
                out = torch.empty(n * m, device="cuda")
                ts = []
                for it in range(9):
                    flush.fill_(float(it))
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
                    ev[0].record()
                    yl.matmul(out, xa, w, k, m, 32, batch=n, accumulate=False)
                    ev[1].record()
                    torch.cuda.synchronize()
                    if it >= 2:
                        ts.append(ev[0].elapsed_time(ev[1]) * 1e-3)
                t = float(np.median(ts))
                gbs = (m * k * bf + n * k * (1 + 4 / 32) + n * m * 4) / t * 1e-9
                print(json.dumps({"case": "sweep", "M": m, "K": k, "fmt": name, "N": n, "us": t * 1e6,
                                  "gbs": gbs, "hbm_frac": gbs / hbm if hbm else None,
                                  "tops": 2.0 * m * k * n / t * 1e-12,
                                  "path": "gemm" if n >= 16 else "matvec"}), flush=True)
                del xa, out
            del w
            torch.cuda.synchronize()


def profile_case(case: str) -> None:
    """Small fixed workloads for ncu captures (printed results are not bench
    values). `matvec:ROWSxK`: three batch-1 Q8_0 matvecs of that shape with
    random weights (the bench's dominant kernel at 28672x4096). `gemm:OxKxB`:
    the Q8_0 matmul of B tokens (the tensor-core GEMM from 16 tokens), timed
    over 10 launches with CUDA events after 3 untimed ones. `prefill4`: the
    4-layer model below, one 512-token prefill. `sweep`: the matvec / GEMM
    sweep (sweep_case). `int8peak`: torch._int_mm on 8192^3 (the library
    int8 GEMM, the denominator of the GEMM's tensor fraction). `decode4`: a
    4-layer config-4-shaped model, prompt 8, then 4 decode steps launched
    kernel by kernel (no graph)."""
    import torch
    yl = importlib.import_module(PKG)
    torch.cuda.set_device(0)
    rng = np.random.default_rng(0)
    if case.startswith("matvec:"):
        o, n = (int(v) for v in case.split(":", 1)[1].split("x"))
        w = yl.QuantizedTensor.weight(yl.WeightFormat.Q8_0, o, n, 32, 1)
        w.upload(quant_vals=rng.integers(-127, 128, o * n, dtype=np.int8),
                 scale_factor=(np.abs(rng.standard_normal(o * n // 32)) * 1e-3).astype(np.float32))
        xa = yl.new_workspace_buffer(yl.WeightFormat.Q8_0, n, 32)
        yl.quantize(yl.WeightFormat.Q8_0, xa, torch.tensor(rng.standard_normal(n).astype(np.float32), device="cuda"),
                    n, 32)
        out = torch.zeros(o, device="cuda")
        for _ in range(3):
            yl.matmul(out, xa, w, n, o, 32, batch=1, accumulate=False)
    elif case.startswith("gemm:"):
        o, n, b = (int(v) for v in case.split(":", 1)[1].split("x"))
        w = yl.QuantizedTensor.weight(yl.WeightFormat.Q8_0, o, n, 32, 1)
        w.upload(quant_vals=rng.integers(-127, 128, o * n, dtype=np.int8),
                 scale_factor=(np.abs(rng.standard_normal(o * n // 32)) * 1e-3).astype(np.float32))
        xa = yl.new_workspace_buffer(yl.WeightFormat.Q8_0, b * n, 32)
        yl.quantize(yl.WeightFormat.Q8_0, xa, torch.tensor(rng.standard_normal(b * n).astype(np.float32),
                                                           device="cuda"), b * n, 32)
        out = torch.zeros(b * o, device="cuda")
        for _ in range(3):
            yl.matmul(out, xa, w, n, o, 32, batch=b, accumulate=False)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(10):
            yl.matmul(out, xa, w, n, o, 32, batch=b, accumulate=False)
        ev[1].record()
        torch.cuda.synchronize()
        us = ev[0].elapsed_time(ev[1]) * 100.0
        print(json.dumps({"case": case, "us_per_launch": us, "tops": 2.0 * o * n * b / us * 1e-6,
                          "weight_gbs": o * n * 34 / 32 / us * 1e-3}))
        return
    elif case == "sweep":
        sweep_case(yl, torch, rng)
        return
    elif case == "int8peak":
        # dense int8 tensor-core peak of the library GEMM (torch._int_mm, cuBLASLt), 8192^3
        a8 = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        b8 = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
        for _ in range(3):
            torch._int_mm(a8, b8)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(20):
            torch._int_mm(a8, b8)
        ev[1].record()
        torch.cuda.synchronize()
        us = ev[0].elapsed_time(ev[1]) * 50.0
        print(json.dumps({"case": case, "us_per_launch": us, "tops": 2.0 * 8192 ** 3 / us * 1e-6}))
        return
    elif case == "prefill4":
        path = os.path.join(os.environ.get("YL_BENCH_DIR", "/tmp"), "yl_c4_4layers.gguf")
        if not os.path.exists(path):
            yl.synth_preset(CONFIG, path, n_layers=4)
        m = yl.load_transformer(path, max_ctx_len=1024)
        prompt = yl.prompt_ids(yl.PRESETS[CONFIG]["vocab_size"], 512, 1).tolist()
        m.forward_x_full(prompt, 0, m.create_session(), want_logits=False)
    elif case == "decode4":
        path = os.path.join(os.environ.get("YL_BENCH_DIR", "/tmp"), "yl_c4_4layers.gguf")
        if not os.path.exists(path):
            yl.synth_preset(CONFIG, path, n_layers=4)
        m = yl.load_transformer(path, max_ctx_len=1024)
        s = m.create_session()
        prompt = yl.prompt_ids(yl.PRESETS[CONFIG]["vocab_size"], 8, 1).tolist()
        _, tok = m.forward_x_full(prompt, 0, s, want_logits=False)
        for i in range(4):
            _, tok = m.forward_x_full([tok], len(prompt) + i, s, want_logits=False)
    else:
        raise SystemExit(f"unknown --case {case}")
    torch.cuda.synchronize()
    print(json.dumps({"case": case, "ok": True}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=128)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-tokens", type=int, default=3)
    ap.add_argument("--case", default=None, help="profiling workload (matvec:ROWSxK, gemm:ROWSxKxTOKENS, sweep, int8peak, prefill4 or decode4), no bench line")
    args = ap.parse_args()
    if args.case:
        profile_case(args.case)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    args.warmup = max(3, args.warmup)

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    yl = importlib.import_module(PKG)
    cfg = yl.PRESETS[CONFIG]
    path = ensure_model(yl, rank, world, dist)
    t0 = time.time()
    # N > 1: tensor parallelism over the N GPUs (Megatron shards, exchanges
    # over NVLink peer memory); one token stream, so N does not multiply value
    if world > 1:
        model = yl.load_transformer_tp(path, rank, world, max_ctx_len=4096)
    else:
        model = yl.load_transformer(path, max_ctx_len=4096)
    load_s = time.time() - t0
    sess = model.create_session()
    if world > 1:
        sess.tp_connect_group()
    prompt = yl.prompt_ids(cfg["vocab_size"], PROMPT_LEN, cfg["seed"] + 1000)
    # one untimed prefill first (first launches load the kernels), then the
    # session is reset and the prompt prefilled again, timed
    model.forward_x_full(prompt, 0, sess, want_logits=False)
    sess.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _, tok = model.forward_x_full(prompt, 0, sess, want_logits=False)
    prefill_s = time.perf_counter() - t0
    pos = PROMPT_LEN
    # warm-up through the device graph
    ids = model.decode_greedy(sess, tok, pos, args.warmup)
    pos += args.warmup
    tok = int(ids[-1])
    stream = torch.cuda.Stream()  # a real stream: events and the graph launches share it
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        model.decode_greedy(sess, tok, pos, args.steps, stream=stream, sync=False)
        e1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    pos += args.steps
    tok = 1
    # e2e through the reference-facing call (host in / host out)
    e2e_steps = min(args.e2e_steps, args.steps)
    logits = torch.empty(cfg["vocab_size"], dtype=torch.float32).pin_memory().numpy()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        _, tok = model.forward_x_full([tok], pos + i, sess, want_logits=True, logits_out=logits)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    # batched decode of independent sessions (yl_batch_forward): 8 sessions
    # prefilled with the prompt, then greedy steps together; host call timed
    batched = None
    if world == 1:
        nb, bsteps = 8, 16
        bs = [model.create_session() for _ in range(nb)]
        btok = []
        for se in bs:
            _, t1 = model.forward_x_full(prompt, 0, se, want_logits=False)
            btok.append(t1)
        batch = model.create_batch(nb)
        bpos = [PROMPT_LEN] * nb
        for _ in range(2):  # untimed
            ids, _ = batch.forward(bs, btok, bpos)
            btok, bpos = [int(i) for i in ids], [q + 1 for q in bpos]
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(bsteps):
            ids, _ = batch.forward(bs, btok, bpos)
            btok, bpos = [int(i) for i in ids], [q + 1 for q in bpos]
        bsec = time.perf_counter() - t0
        batched = {"sessions": nb, "steps": bsteps, "tokens_per_s": nb * bsteps / bsec,
                   "ms_per_step": bsec / bsteps * 1e3, "call": "yl_batch_forward (host ids in and out each step)",
                   "positions": f"{PROMPT_LEN + 2}..{PROMPT_LEN + 2 + bsteps}"}
        del batch, bs
    # dominant kernel roofline (this rank's gate/up shard)
    mv = time_dominant_matvec(yl, torch, model, cfg, 96, world)
    peaks = measured_peaks()
    seq_avg = PROMPT_LEN + args.warmup + args.steps / 2.0
    btok = bytes_per_token(cfg, seq_avg)
    tokps = args.steps / (ms * 1e-3)
    line = {
        "metric": "decode tokens/s (Llama-3-8B-shape Q8_0, batch 1)",
        "value": tokps, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "int8 dot / f32 accumulate", "data": "synthetic",
        "config": {"workload": "config 4: Llama-3-8B-shaped Q8_0 (random-init, seed 3), prompt 512, "
                               "batch-1 greedy decode from position 512",
                   "model": "llama-3-8b-shape-q8_0", "global_batch": 1, "seq_len": PROMPT_LEN,
                   "parallelism": f"tp{world}" if world > 1 else "single",
                   "l2": "weights 8.1 GB per token > 126 MB L2 (no flush needed)"},
        "e2e": {"value": e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 16,
                "d2h_bytes_per_step": 4 * cfg["vocab_size"] + 4,
                "call": "yl_forward_x (Transformer::forward_x), logits + greedy id to host"},
        "roofline": {"bound": "hbm", "kernel": f"mv_kernel<Q8,NT=1> gate/up {2 * cfg['hidden_dim'] // world}x4096",
                     "achieved": mv["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": mv["gbs"] / peaks["hbm_gbs"], "peak_src": peaks["src"],
                     # DRAM read + write bytes of one launch of this kernel and shape,
                     # from one ncu capture of `bench.py --case matvec:28672x4096`
                     "traffic": TRAFFIC_GATEUP_BYTES if world == 1 else None, "traffic_unit": "bytes per launch",
                     "algorithmic_bytes": mv["bytes"], "launch_ms": mv["ms"]},
        # per GPU: each rank streams its shard (1/N of the weights) per token
        "step_roofline": {"bytes_per_token": btok, "bytes_per_token_per_gpu": btok / world,
                          "achieved_gbs_per_gpu": btok / world / (ms / args.steps * 1e-3) / 1e9,
                          "frac": btok / world / (ms / args.steps * 1e-3) / 1e9 / peaks["hbm_gbs"]},
        "gpu_launches": model.decode_step_launches() * args.steps,
        "clocks": clk.summary(),
        "prefill": {"tokens": PROMPT_LEN, "s": prefill_s, "tokens_per_s": PROMPT_LEN / prefill_s},
        "load_s": load_s,
    }
    if batched:
        line["batched"] = batched
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        del model, sess
        torch.cuda.empty_cache()
        nc = os.cpu_count() or 1
        line["cpu_baseline"] = cpu_baseline(path, args.cpu_tokens, nc, half_threads=max(1, -(-nc // 2)))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

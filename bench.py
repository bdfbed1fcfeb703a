"""Benchmark of the torchcl B200 GEMM path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg5] [--impl ours|reference]

Default workload: bf16 C = relu(A @ W + bias), M = N = K = 32768,
W column-sharded over the N ranks (rank r holds W[:, r*N/P:(r+1)*N/P] and its bias
slice, resident), A replicated, each rank computes its column block with the
fused epilogue, and the epilogue's TMA stores write every output tile into the
row-major C of every rank over NVLink (`--gather nccl`: local block + NCCL
all_gather + re-layout instead).  Total work is fixed as N grows ("scaling": "strong").
Other configs (--config cfg1..cfg4) run on one GPU for the parity/roofline notes.
`--graph` (one GPU) adds the host cost of one step through the public torchcl API
against one replay of the same step captured with torchcl.jit.graph_runner.

`value` is device time (CUDA events on the launching stream, max over ranks) with
inputs resident; `e2e` is the same metric through the C-ABI with pinned host
buffers: host->device copy of A, the GEMM (+ gather), device->host copy of C.
`--impl reference` times the CPU port of the reference algorithm (oracle/, k
ascending fp32 accumulation, all host threads) on a bounded sample of the same
workload.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
PKG = REPO / "ojasx-open-source-cuda-_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

CONFIGS = {
    # name: (M, N, K, dtype, epilogue unary, bias scale, W scale, A distribution, seed)
    "cfg1": dict(M=512, N=512, K=512, dtype="f32", act="relu", a="normal", w_scale=1.0, b_scale=1.0, seed=0,
                 desc="fp32 relu(A@B+bias) 512^3"),
    "cfg2": dict(M=8192, N=8192, K=8192, dtype="f32", act="gelu", a="uniform", w_scale=1.0, b_scale=0.1,
                 seed=1, desc="fp32 gelu_tanh(A@B+bias) 8192^3, 3xTF32"),
    "cfg3": dict(M=8192, N=11008, K=4096, dtype="bf16", act="silu", a="normal", w_scale=0.02, b_scale=0.0,
                 seed=2, desc="bf16 FFN silu(X@W+0) 8192x4096x11008"),
    "cfg4": dict(M=16, N=14336, K=4096, dtype="bf16", act="silu", a="normal", w_scale=0.02, b_scale=0.0,
                 seed=3, desc="bf16 skinny decode silu(X@W+bias) M=16 K=4096 N=14336"),
    "cfg5": dict(M=32768, N=32768, K=32768, dtype="bf16", act="relu", a="normal", w_scale=0.01,
                 b_scale=0.1, seed=4, desc="bf16 relu(A@W+bias) 32768^3, W column-sharded, C all-gathered"),
}
L2_BYTES = 126 * 1024 * 1024


def _peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples: list[list[str]] = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower().startswith("active")})
        pw = [float(s[3]) for s in self.samples if s[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": max(pw) if pw else None}


def _dist_setup():
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


# ── CPU baseline (reference arm and the cpu_baseline field) ───────────────────

def cpu_baseline(cfg: dict, steps: int = 1, min_seconds: float = 0.0, same_inputs=None) -> dict:
    """Time the oracle port on a bounded sample of the workload, all host threads.

    Runs `steps` samples, and more (at most 50) until `min_seconds` of CPU work
    have been timed; reports the median sample.  The sample is the block
    C[0:ms, 0:ns] (ms, ns <= 1024) with the full K.

    same_inputs (our arm, one GPU): (A, W, bias, C) device tensors of the timed
    run.  The port then runs on copies of A[0:ms, :], W[:, 0:ns] and bias[0:ns],
    and its output block is also the parity check of the GPU's C[0:ms, 0:ns]
    (returned under "parity"); without it (the reference arm) the sample's inputs
    are drawn on the host."""
    import numpy as np
    from oracle import build_oracle
    build_oracle.build_oracle()
    from oracle import oracle as O
    K = cfg["K"]
    ms = min(cfg["M"], 1024)
    ns = min(cfg["N"], 1024)
    half = cfg["dtype"] == "bf16"
    dt = O.BF16 if half else O.F32
    if same_inputs is not None:
        import torch
        Ad, Wd, bd, Cd = same_inputs

        def host(t):
            t = t.contiguous().cpu()
            return t.view(torch.int16).numpy().view(np.uint16) if half else t.numpy()
        A, B, bias = host(Ad[:ms]), host(Wd[:, :ns]), host(bd[:ns])
        gpu = Cd[:ms, :ns].float().cpu().numpy().astype(np.float64)
    else:
        rng = np.random.default_rng(cfg["seed"])
        A = rng.standard_normal((ms, K), dtype=np.float32)
        B = (rng.standard_normal((K, ns), dtype=np.float32) * cfg["w_scale"]).astype(np.float32)
        bias = rng.standard_normal(ns, dtype=np.float32) * cfg["b_scale"]
        if half:
            A, B, bias = O.bf16_bits(A), O.bf16_bits(B), O.bf16_bits(bias)
        gpu = None
    threads = os.cpu_count() or 1
    times = []
    out = None
    while len(times) < max(1, steps) or (sum(times) < min_seconds and len(times) < 50):
        t0 = time.perf_counter()
        out = O.gemm(A, B, dtype_a=dt, dtype_b=dt, dtype_c=dt, operand=bias, operand_kind="row",
                     operand_dtype=dt, unary=[cfg["act"]], threads=threads)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    flops = 2.0 * ms * ns * K
    res = {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
           "sample": f"C[0:{ms}, 0:{ns}] with full K={K} ({'bf16 widened to fp32' if half else 'fp32'}, "
                     f"k ascending, fp32 accumulate, {cfg['act']} epilogue), median of {len(times)}",
           "seconds_per_sample": t}
    if gpu is not None:
        ref = (O.bf16_to_f32(out) if half else out).astype(np.float64)
        rel = float(np.linalg.norm(gpu - ref) / max(np.linalg.norm(ref), 1e-30))
        mx = float(np.abs(gpu - ref).max())
        if half:
            ok, bar = rel <= 1e-2, "rel-L2 <= 1e-2"
        else:
            # max-abs scale ||A||_F ||B||_F / sqrt(MN) of the whole product, on the device
            Ad, Wd = same_inputs[0], same_inputs[1]
            scale = float(Ad.double().norm() * Wd.double().norm()) / (cfg["M"] * cfg["N"]) ** 0.5
            ok = rel <= 1e-5 and mx <= 1e-4 * scale
            bar = f"rel-L2 <= 1e-5 and max-abs <= 1e-4 * {scale:.4g}"
        res["parity"] = {"rel_l2": rel, "max_abs": mx, "bar": bar, "pass": bool(ok),
                         "sample": f"C[0:{ms}, 0:{ns}] of the timed run's output (full K) against "
                                   f"the oracle on the same device inputs"}
    return res


def run_reference(args, cfg, world, rank):
    if rank != 0:
        return 0
    t0 = time.perf_counter()
    for _ in range(args.warmup):
        cpu_baseline(cfg, 1)
    cb = cpu_baseline(cfg, args.steps)
    line = {"impl": "reference", "metric": _metric(cfg), "value": cb["value"], "unit": "TFLOP/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["seconds_per_sample"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
            "config": _config_block(args, cfg, world),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}
    print(json.dumps(line), flush=True)
    return 0


def _metric(cfg) -> str:
    return f"fused GEMM+epilogue TFLOP/s ({cfg['desc']})"


def _w_copies(cfg, world) -> int:
    """Copies of W (and bias) the timed steps rotate over.  A weight matrix between
    a quarter of L2 and L2 would otherwise stay cached from the previous step; with
    copies totalling about 3x L2, every step streams its W from HBM, as successive
    layers' weights do in a decode loop.  Smaller inputs get an L2 flush instead."""
    es = 2 if cfg["dtype"] == "bf16" else 4
    wbytes = cfg["K"] * (cfg["N"] // world) * es
    if L2_BYTES // 4 <= wbytes < L2_BYTES:
        return -(-3 * L2_BYTES // wbytes)
    return 1


def _l2_note(cfg, world) -> str:
    es = 2 if cfg["dtype"] == "bf16" else 4
    wbytes = cfg["K"] * (cfg["N"] // world) * es
    if wbytes >= L2_BYTES:
        return "inputs larger than L2"
    n = _w_copies(cfg, world)
    if n > 1:
        return (f"inputs larger than L2: steps rotate over {n} copies of W and bias "
                f"({n * wbytes / 1e6:.0f} MB)")
    return "L2 flushed (256 MiB write) between timed iterations"


def _config_block(args, cfg, world) -> dict:
    return {"workload": f"{args.config}: {cfg['desc']}", "M": cfg["M"], "N": cfg["N"], "K": cfg["K"],
            "epilogue": f"{cfg['act']}(acc + bias[N])",
            "parallelism": (f"N-shard{world}, C gathered by the GEMM epilogue over NVLink"
                            if getattr(args, "gather", "p2p") == "p2p" else
                            f"N-shard{world}, C gathered by NCCL all_gather + re-layout")
                           if world > 1 else "single GPU",
            "l2": _l2_note(cfg, world)}


# ── our implementation ──────────────────────────────────────────────────────

def make_inputs(cfg: dict, dev, world: int = 1, rank: int = 0):
    """Seeded synthetic inputs of a config on device `dev`: (A [M,K], this rank's
    column block of W [K, N/world], its bias slice [N/world]).

    A ~ U(-1,1) or N(0,1); W ~ N(0, w_scale^2); bias ~ N(0, b_scale^2), drawn in
    that order from one torch.Generator on the device.  W is drawn as `world`
    column blocks one after another and every rank draws all of them, so the ranks
    of one run hold slices of one and the same full W and bias.  The GPU parity
    tests regenerate the one-GPU inputs (world = 1) with this function."""
    import torch
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    Nl = N // world
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    if cfg["a"] == "uniform":
        A = (torch.rand(M, K, device=dev, generator=g) * 2 - 1).to(tdt)
    else:
        A = torch.randn(M, K, device=dev, generator=g).to(tdt)
    W = None
    for r in range(world):
        blk = (torch.randn(K, Nl, device=dev, generator=g) * cfg["w_scale"]).to(tdt)
        if r == rank:
            W = blk
        else:
            del blk
    bias_full = (torch.randn(N, device=dev, generator=g) * cfg["b_scale"]).to(tdt)
    bias = bias_full[rank * Nl:(rank + 1) * Nl].contiguous()
    return A, W, bias


def run_ours(args, cfg, world, rank, local):
    import torch
    import torch.distributed as dist
    from torchcl import _lib as L

    lib = L.lib()
    torch.cuda.set_device(local)
    info = L.DeviceInfo()
    L.check(lib.ojx_init(local, ctypes.byref(info)), "ojx_init")
    dev = torch.device("cuda", local)
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    code = L.BF16 if tdt == torch.bfloat16 else L.F32
    es = 2 if tdt == torch.bfloat16 else 4
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    if N % world:
        raise SystemExit(f"N={N} is not divisible by {world} ranks")
    Nl = N // world
    A, W, bias = make_inputs(cfg, dev, world, rank)
    n_copies = _w_copies(cfg, world)
    Ws = [W] + [W.clone() for _ in range(n_copies - 1)]
    biases = [bias] + [bias.clone() for _ in range(n_copies - 1)]
    needs_flush = K * Nl * es < L2_BYTES and n_copies == 1
    flush = torch.empty(256 * 1024 * 1024 if needs_flush else 1, device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    sharded = None
    if world > 1:
        from torchcl.mesh import ShardedGemm
        sharded = ShardedGemm(M, N, K, dtype="bf16" if code == L.BF16 else "fp16",
                              strategy=args.gather, stream=sp)
        C = sharded.c_view()
    else:
        C = torch.empty(M, N, device=dev, dtype=tdt)

    d = L.GemmDesc()
    d.M, d.N, d.K = M, Nl, K
    d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = code
    d.a, d.b, d.c, d.operand = A.data_ptr(), W.data_ptr(), C.data_ptr(), bias.data_ptr()
    d.operand_kind, d.binary_op = L.OPERAND_ROW, L.BINARY["add"]
    d.n_unary, d.unary[0] = 1, L.UNARY[cfg["act"]]
    d.fp32_mode = L.FP32_3XTF32 if code == L.F32 and M > 16 else L.FP32_AUTO
    if args.pair:
        d.flags |= L.FLAG_PAIR
    if args.skinny_counter:
        d.flags |= L.FLAG_SKINNY_COUNTER

    step_no = [0]

    def gemm():
        w, b = Ws[step_no[0] % n_copies], biases[step_no[0] % n_copies]
        step_no[0] += 1
        if sharded is not None:
            sharded.launch(A.data_ptr(), w.data_ptr(), b.data_ptr(), (cfg["act"],))
        else:
            d.b, d.operand = w.data_ptr(), b.data_ptr()
            L.check(lib.ojx_gemm(ctypes.byref(d), sp), "ojx_gemm")

    def gather():
        if sharded is not None:
            sharded.barrier()

    # warm-up
    for _ in range(args.warmup):
        gemm()
        gather()
    torch.cuda.synchronize(dev)
    route = L.ROUTES.get(lib.ojx_last_route())
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)

    # One GPU without L2 flushes: one event pair around the K back-to-back steps,
    # as a decode loop runs them (consecutive skinny launches overlap through
    # programmatic dependent launch, which an event between them would stop).
    # Otherwise events bracket each step's GEMM and gather.
    per_step = world > 1 or needs_flush
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps if per_step else 1)]
    launches0 = lib.ojx_kernel_launch_count()
    with ClockSampler(local) as clk:
        # Keep the GPU busy while the host queues the timed steps, so that the
        # events measure device time, not the host's launch latency.
        torch.cuda._sleep(int(1e6 + 2e5 * args.steps))
        if not per_step:
            ev[0][0].record(stream)
        for i in range(args.steps):
            if needs_flush:
                flush.zero_()
            if per_step:
                ev[i][0].record(stream)
            gemm()
            if per_step:
                ev[i][1].record(stream)
            gather()
            if per_step:
                ev[i][2].record(stream)
        if not per_step:
            ev[0][2].record(stream)
        torch.cuda.synchronize(dev)
    launches = lib.ojx_kernel_launch_count() - launches0
    L.check(lib.ojx_poll_device_error(), "device error")
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    gemm_ms = ([e[0].elapsed_time(e[1]) for e in ev] if per_step
               else [step_ms / args.steps] * args.steps)
    t = torch.tensor([step_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    total_ms = float(t.item())
    flops_total = 2.0 * M * N * K
    value = flops_total * args.steps / (total_ms / 1e3) / 1e12

    breakdown = None
    if world > 1 and args.gather == "p2p":
        breakdown = _sharded_breakdown(args, lib, L, d, A, Ws, biases, n_copies, M, Nl, ev, gemm_ms,
                                       dev, stream, world, sharded, cfg["act"])

    # e2e through the C-ABI with pinned host buffers
    e2e = e2e_measure(args, lib, L, A, C, M, K, N, es, gemm, gather, world, dev, stream, cfg=cfg,
                      W=Ws[0], bias=biases[0])

    peaks, peak_kind = _peaks()
    avg_gemm_ms = statistics.mean(gemm_ms)
    per_launch_flops = 2.0 * M * Nl * K
    achieved = per_launch_flops / (avg_gemm_ms / 1e3) / 1e12
    clocks = clk.summary()
    # The sustained (power-capped) GEMM peak applies when the timed region ran at the
    # power limit (the clock sampler saw sw_power_cap) or lasted over a second.
    sustained = avg_gemm_ms * args.steps > 1000.0 or "sw_power_cap" in (clocks.get("reasons") or [])
    peak = peaks.get("bf16_tflops_sustained" if sustained else "bf16_tflops", 1590.0)
    if code == L.F32:
        # 3xTF32 runs three tf32 MMAs (half the bf16 rate each) per fp32 multiply-add
        peak = peak / 2 / 3
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": _traffic(args),
            "kernel": f"ojx route {route}", "peak_source": f"{peak_kind} "
            f"{'bf16_tflops_sustained' if sustained else 'bf16_tflops'}"
            f"{' / 6 (3xTF32 effective)' if code == L.F32 else ''}",
            "algorithmic_flop_per_launch": per_launch_flops, "avg_launch_ms": avg_gemm_ms,
            "launch_timing": ("CUDA events around each launch" if per_step else
                              "one CUDA event pair around the K back-to-back launches, / K")}
    if cfg["dtype"] == "bf16" and M <= 16:
        bytes_per = es * (M * K + K * Nl + Nl + M * Nl)
        gbs = bytes_per / (avg_gemm_ms / 1e3) / 1e9
        roof.update({"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": bytes_per,
                     "peak_source": f"{peak_kind} hbm_gbs"})

    graph = graph_measure(args, cfg, A, Ws[0], biases[0], dev) if args.graph and world == 1 else None

    if rank == 0:
        cb = (cpu_baseline(cfg, 1, min_seconds=10.0, same_inputs=(A, Ws[0], biases[0], C))
              if world == 1 else None)
        line = {"metric": _metric(cfg), "value": value, "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": cfg["dtype"], "data": "synthetic (seeded torch.Generator on device)",
                "config": _config_block(args, cfg, world), "route": route, "roofline": roof,
                "cpu_baseline": ({k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
                                 if cb else None),
                "parity": cb.get("parity") if cb else None,
                "e2e": e2e, "gpu_launches": int(launches),
                "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
                "clock_samples": clocks.get("samples"), "power_w_max": clocks.get("power_w_max")}
        if graph is not None:
            line["graph"] = graph
        if breakdown is not None:
            line["step_breakdown"] = breakdown
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize(dev)
        sharded.close()
        dist.destroy_process_group()
    return 0


def _sharded_breakdown(args, lib, L, d, A, Ws, biases, n_copies, M, Nl, ev, gemm_ms, dev, stream,
                       world, sharded, act):
    """Where a sharded step's time goes, max over ranks (all ranks take part).

    After the timed steps, `args.steps` pairs of launches alternate on each rank:
    the all-gathering GEMM (its epilogue stores every tile into all ranks' C; the
    kernel completes after its stores and a system-scope fence) and the same GEMM
    writing only this rank's [M, N/P] block.  Alternating them keeps both under the
    same clock and power state; their mean difference is the peer-store tail.  The
    completion barrier (the one-element all-reduce after the kernel) is taken from
    the timed steps."""
    import torch
    import torch.distributed as dist
    barrier_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    C_local = torch.empty(M, Nl, device=dev, dtype=A.dtype)
    dl = L.GemmDesc.from_buffer_copy(d)
    dl.c, dl.ldc = C_local.data_ptr(), Nl
    sp = stream.cuda_stream
    pairs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    torch.cuda.synchronize(dev)
    dist.barrier()
    torch.cuda._sleep(int(1e6 + 2e5 * args.steps))
    for i, e in enumerate(pairs):
        w, b = Ws[i % n_copies].data_ptr(), biases[i % n_copies].data_ptr()
        dl.b, dl.operand = w, b
        e[0].record(stream)
        L.check(lib.ojx_gemm(ctypes.byref(dl), sp), "local gemm")
        e[1].record(stream)
        sharded.launch(A.data_ptr(), w, b, (act,))
        e[2].record(stream)
        sharded.barrier()
        e[3].record(stream)
    torch.cuda.synchronize(dev)
    local_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in pairs)
    ag_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in pairs)
    t = torch.tensor([statistics.mean(gemm_ms), ag_ms, local_ms, barrier_ms], device=dev,
                     dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    timed, ag, loc, bar = (float(x) for x in t.tolist())
    del C_local
    return {"gemm_allgather_ms": timed, "pairs_allgather_ms": ag, "pairs_local_only_ms": loc,
            "peer_store_tail_ms": ag - loc, "completion_barrier_ms": bar,
            "note": "per step, max over ranks; pairs_*: all-gathering and local-only launches of the "
                    "same GEMM alternated after the timed steps"}


def e2e_measure(args, lib, L, A, C, M, K, N, es, gemm, gather, world, dev, stream, cfg=None,
                W=None, bias=None):
    """Same metric end to end, host memory in and out, every step.

    One GPU: through the public torchcl API, as a user of the reference writes it:
    to_opencl(A) of a pinned host A, the lazy act(add(matmul(a, w), b)) and to_cpu,
    which runs the upload, the fused GEMM and the download as one overlapped
    pipeline (ojx_gemm_host_io) and returns C in pinned host memory; W and the bias
    stay resident.  Several GPUs: through the C-ABI and the mesh, upload, sharded
    GEMM with the gather, barrier and download one after another.  CUDA events on
    the stream the work runs on; max over ranks."""
    import torch
    import torch.distributed as dist
    a_bytes = M * K * es
    c_bytes = M * N * es
    if world == 1:
        import torchcl
        from torchcl.runtime.context import get_queue
        torchcl.init_opencl(device_index=dev.index or 0)
        A_host = A.cpu().pin_memory()
        w, b = torchcl.to_opencl(W.cpu()), torchcl.to_opencl(bias.cpu())
        act = getattr(torchcl, cfg["act"])
        qstream = torch.cuda.ExternalStream(get_queue(), device=dev)
        holder = []

        def step():
            a = torchcl.to_opencl(A_host)
            holder[:] = [torchcl.to_cpu(act(torchcl.add(torchcl.matmul(a, w), b)))]
        estream = qstream
    else:
        ha, hc = ctypes.c_void_p(), ctypes.c_void_p()
        L.check(lib.ojx_host_alloc(a_bytes, ctypes.byref(ha)), "pinned A")
        L.check(lib.ojx_host_alloc(c_bytes, ctypes.byref(hc)), "pinned C")
        sp = stream.cuda_stream
        L.check(lib.ojx_memcpy_d2h(ha.value, A.data_ptr(), a_bytes, sp))
        torch.cuda.synchronize(dev)

        def step():
            L.check(lib.ojx_memcpy_h2d(A.data_ptr(), ha.value, a_bytes, sp), "h2d")
            gemm()
            gather()
            L.check(lib.ojx_memcpy_d2h(hc.value, C.data_ptr(), c_bytes, sp), "d2h")
        estream = stream

    # Untimed warm-up steps, at least two: a caller keeps the previous result while
    # the next step runs, so the pinned-memory cache settles on two output blocks
    # (the first allocation of a 2 GB pinned block costs the better part of a second).
    steps = max(2, args.steps)
    for _ in range(max(2, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(estream)
    for _ in range(steps):
        step()
    e1.record(estream)
    torch.cuda.synchronize(dev)
    dt = e0.elapsed_time(e1) / 1e3
    t = torch.tensor([dt], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dt = float(t.item())
    if world == 1:
        ok = bool(torch.equal(holder[0].view(-1)[:1 << 20].to(dev), C.view(-1)[:1 << 20]))
        holder.clear()
        note = ("torchcl public API: to_opencl(pinned A) -> " + cfg["act"] + "(add(matmul(a, w), b))"
                " -> to_cpu, which overlaps the chunked upload, fused GEMM and download "
                "(ojx_gemm_host_io); W and bias resident")
    else:
        lib.ojx_host_free(ha.value)
        lib.ojx_host_free(hc.value)
        ok = None
        note = "C-ABI with pinned host buffers: upload, GEMM + gather, download; max over ranks"
    flops = 2.0 * M * N * K * steps
    out = {"value": flops / dt / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": a_bytes,
           "d2h_bytes_per_step": c_bytes, "steps": steps,
           "note": note + "; CUDA events on the stream the work runs on"}
    if ok is not None:
        out["matches_device_run"] = ok
    return out


def run_train(args, cfg):
    """One training step of a linear layer on one GPU, through the C-ABI with the
    operands resident: forward Y = X @ W^T + b (W stored [N, K] like nn.Linear),
    backward dX = dY @ W, dW = dY^T @ X (both read the stored operands transposed
    through the GEMM descriptor) and db = dY.sum(0).  The reference's
    LinearFunction (torchcl/autograd.py:355-412) does the same with two
    materialised transposes.  value = 3 * 2*M*N*K / step time."""
    import torch
    from torchcl import _lib as L

    lib = L.lib()
    torch.cuda.set_device(0)
    L.check(lib.ojx_init(0, ctypes.byref(L.DeviceInfo())), "ojx_init")
    dev = torch.device("cuda", 0)
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    code = L.BF16 if tdt == torch.bfloat16 else L.F32
    es = 2 if code == L.BF16 else 4
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    X = torch.randn(M, K, device=dev, generator=g).to(tdt)
    W = (torch.randn(N, K, device=dev, generator=g) * cfg["w_scale"]).to(tdt)
    b = (torch.randn(N, device=dev, generator=g) * 0.1).to(tdt)
    G = torch.randn(M, N, device=dev, generator=g).to(tdt)
    Y, dX = torch.empty(M, N, device=dev, dtype=tdt), torch.empty(M, K, device=dev, dtype=tdt)
    dW, db = torch.empty(N, K, device=dev, dtype=tdt), torch.empty(N, device=dev, dtype=tdt)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def desc(m, n, k, a, bb, c, ta=0, tb=0, bias=None):
        d = L.GemmDesc()
        d.M, d.N, d.K = m, n, k
        d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = code
        d.trans_a, d.trans_b = ta, tb
        d.a, d.b, d.c = a.data_ptr(), bb.data_ptr(), c.data_ptr()
        if bias is not None:
            d.operand, d.operand_kind, d.binary_op = bias.data_ptr(), L.OPERAND_ROW, L.BINARY["add"]
        return d

    descs = [desc(M, N, K, X, W, Y, tb=1, bias=b),   # forward
             desc(M, K, N, G, W, dX),                # dX = dY @ W
             desc(N, K, M, G, X, dW, ta=1)]          # dW = dY^T @ X
    names = ["forward", "grad_input", "grad_weight", "grad_bias"]

    def step(evs=None):
        for i, d in enumerate(descs):
            if evs:
                evs[i].record(stream)
            L.check(lib.ojx_gemm(ctypes.byref(d), sp), names[i])
        if evs:
            evs[3].record(stream)
        L.check(lib.ojx_sum_columns(db.data_ptr(), code, G.data_ptr(), code, M, N, 0, sp), "sum_columns")
        if evs:
            evs[4].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    routes = []
    for d in descs:
        L.check(lib.ojx_gemm(ctypes.byref(d), sp))
        routes.append(L.ROUTES.get(lib.ojx_last_route()))
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    launches0 = lib.ojx_kernel_launch_count()
    with ClockSampler(0) as clk:
        torch.cuda._sleep(int(1e6 + 2e5 * args.steps))
        for i in range(args.steps):
            step(evs[i])
        torch.cuda.synchronize(dev)
    launches = lib.ojx_kernel_launch_count() - launches0
    L.check(lib.ojx_poll_device_error(), "device error")
    part = [[e[j].elapsed_time(e[j + 1]) for e in evs] for j in range(4)]
    total_ms = sum(e[0].elapsed_time(e[4]) for e in evs)
    flops = 3 * 2.0 * M * N * K
    value = flops * args.steps / (total_ms / 1e3) / 1e12
    peaks, peak_kind = _peaks()
    peak = peaks.get("bf16_tflops", 1590.0) / (6 if code == L.F32 else 1)
    per = {}
    for j, name in enumerate(names[:3]):
        ms = statistics.mean(part[j])
        per[name] = {"route": routes[j], "ms": ms, "tflops": 2.0 * M * N * K / (ms / 1e3) / 1e12}
    cs_ms = statistics.mean(part[3])
    cs_bytes = M * N * es + N * es
    per["grad_bias"] = {"ms": cs_ms, "gbs": cs_bytes / (cs_ms / 1e3) / 1e9,
                        "frac_hbm": cs_bytes / (cs_ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
    top = max(per["forward"]["tflops"], per["grad_input"]["tflops"], per["grad_weight"]["tflops"])
    clocks = clk.summary()
    line = {"metric": f"linear-layer training step TFLOP/s (fwd + bwd, {cfg['desc']})", "value": value,
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic (seeded torch.Generator on device)",
            "config": {"workload": f"{args.config} train: Y = X W^T + b, dX = dY W, dW = dY^T X, db = sum(dY)",
                       "M": M, "N": N, "K": K,
                       "l2": f"inputs larger than L2 (X {M * K * es / 1e6:.0f} MB, W {N * K * es / 1e6:.0f} MB, "
                             f"dY {M * N * es / 1e6:.0f} MB); each GEMM streams two of them"},
            "kernels": per,
            "roofline": {"bound": "tensor", "achieved": flops / (sum(p["ms"] for k, p in per.items()
                                                                     if k != "grad_bias") / 1e3) / 1e12,
                         "peak": peak, "unit": "TFLOP/s", "best_gemm_tflops": top,
                         "peak_source": f"{peak_kind} bf16_tflops{' / 6 (3xTF32)' if code == L.F32 else ''}"},
            "gpu_launches": int(launches),
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    line["roofline"]["frac"] = line["roofline"]["achieved"] / peak
    print(json.dumps(line), flush=True)
    return 0


def run_batched(args, cfg):
    """`--batch B` on one GPU: B independent problems of the config's shape (A_b, W_b,
    per-problem bias row, fused activation) in ONE ojx_gemm_batched launch per step,
    the reference's blas.bmm path (torchcl/blas/__init__.py:123-150).
    value = B * 2*M*N*K / step time."""
    import torch
    from torchcl import _lib as L

    lib = L.lib()
    torch.cuda.set_device(0)
    L.check(lib.ojx_init(0, ctypes.byref(L.DeviceInfo())), "ojx_init")
    dev = torch.device("cuda", 0)
    tdt = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    code = L.BF16 if tdt == torch.bfloat16 else L.F32
    es = 2 if code == L.BF16 else 4
    Bn, M, N, K = args.batch, cfg["M"], cfg["N"], cfg["K"]
    g = torch.Generator(device=dev).manual_seed(cfg["seed"])
    A = torch.randn(Bn, M, K, device=dev, generator=g).to(tdt)
    W = (torch.randn(Bn, K, N, device=dev, generator=g) * cfg["w_scale"]).to(tdt)
    bias = (torch.randn(Bn, N, device=dev, generator=g) * cfg["b_scale"]).to(tdt)
    C = torch.empty(Bn, M, N, device=dev, dtype=tdt)
    in_bytes = (A.numel() + W.numel()) * es
    flush = torch.empty(256 * 1024 * 1024 if in_bytes < L2_BYTES else 1, device=dev, dtype=torch.uint8)
    d = L.GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.dtype_a = d.dtype_b = d.dtype_c = d.dtype_operand = code
    d.a, d.b, d.c, d.operand = A.data_ptr(), W.data_ptr(), C.data_ptr(), bias.data_ptr()
    d.operand_kind, d.binary_op = L.OPERAND_ROW, L.BINARY["add"]
    d.n_unary, d.unary[0] = 1, L.UNARY[cfg["act"]]
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step():
        L.check(lib.ojx_gemm_batched(ctypes.byref(d), Bn, M * K, K * N, M * N, N, sp), "gemm_batched")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    route = L.ROUTES.get(lib.ojx_last_route())
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    launches0 = lib.ojx_kernel_launch_count()
    with ClockSampler(0) as clk:
        torch.cuda._sleep(int(1e6 + 2e5 * args.steps))
        for e0, e1 in evs:
            if in_bytes < L2_BYTES:
                flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize(dev)
    launches = lib.ojx_kernel_launch_count() - launches0
    L.check(lib.ojx_poll_device_error(), "device error")
    ms = [e0.elapsed_time(e1) for e0, e1 in evs]
    total_ms = sum(ms)
    flops = Bn * 2.0 * M * N * K
    value = flops * args.steps / (total_ms / 1e3) / 1e12
    peaks, peak_kind = _peaks()
    peak = peaks.get("bf16_tflops", 1590.0) / (6 if code == L.F32 else 1)
    clocks = clk.summary()
    line = {"metric": f"batched fused GEMM TFLOP/s ({Bn} x {cfg['desc']})", "value": value,
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic (seeded torch.Generator on device)",
            "config": {"workload": f"{args.config} x batch {Bn}: C_b = {cfg['act']}(A_b @ W_b + bias_b)",
                       "batch": Bn, "M": M, "N": N, "K": K,
                       "l2": "inputs larger than L2" if in_bytes >= L2_BYTES
                             else "L2 flushed (256 MiB write) between timed iterations"},
            "route": route,
            "roofline": {"bound": "tensor", "achieved": value, "peak": peak, "unit": "TFLOP/s",
                         "frac": value / peak,
                         "peak_source": f"{peak_kind} bf16_tflops{' / 6 (3xTF32)' if code == L.F32 else ''}"},
            "gpu_launches": int(launches),
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    print(json.dumps(line), flush=True)
    return 0


def parse_attn_spec(spec: str) -> tuple[int, int, int, int, int, bool]:
    """'B,H,M,N,D[,causal]' -> (B, H, M, N, D, causal).  The sixth field is the
    word "causal" or a 0/1 flag."""
    parts = [x.strip() for x in spec.split(",")]
    if len(parts) not in (5, 6):
        raise ValueError(f"--attn wants B,H,M,N,D[,causal], got {spec!r}")
    B, H, M, N, D = (int(x) for x in parts[:5])
    causal = len(parts) == 6 and parts[5].lower() not in ("0", "", "false")
    return B, H, M, N, D, causal


def run_attention(args):
    """`--attn B,H,M,N,D[,causal]` on one GPU: torchcl.fused_attention's kernel
    through the C-ABI (ojx_attention) on device-resident bf16 Q, K, V; the fused
    route and the composed route (QK^T GEMM, softmax, PV GEMM) timed back to back.
    FLOPs = 4*B*H*M*N*D (half of the score matrix when causal and M == N)."""
    import torch
    from torchcl import _lib as L

    B, H, M, N, D, causal = parse_attn_spec(args.attn)
    lib = L.lib()
    torch.cuda.set_device(0)
    L.check(lib.ojx_init(0, ctypes.byref(L.DeviceInfo())), "ojx_init")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    q, k, v = (torch.randn(B, H, x, D, device=dev, generator=g).bfloat16() for x in (M, N, N))
    out = torch.empty(B, H, M, D, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    scale = D ** -0.5
    flops = 4.0 * B * H * M * N * D * (0.5 if causal and M == N else 1.0)

    def timed(flags):
        def step():
            L.check(lib.ojx_attention(out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), L.BF16,
                                      B, H, M, N, D, scale, int(causal), 0, flags, sp), "attention")
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        route = L.ROUTES.get(lib.ojx_last_route())
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        n0 = lib.ojx_kernel_launch_count()
        torch.cuda._sleep(int(1e6 + 2e5 * args.steps))
        for e0, e1 in evs:
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        L.check(lib.ojx_poll_device_error(), "device error")
        ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / args.steps
        return ms, route, (lib.ojx_kernel_launch_count() - n0) // args.steps

    with ClockSampler(0) as clk:
        ms_f, route_f, launches_f = timed(0)
        ms_c, route_c, launches_c = timed(L.ATTN_FLAG_COMPOSED)
    peaks, peak_kind = _peaks()
    peak = peaks.get("bf16_tflops", 1590.0)
    value = flops / (ms_f / 1e3) / 1e12
    clocks = clk.summary()
    line = {"metric": "fused attention TFLOP/s (bf16)", "value": value, "unit": "TFLOP/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_f, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded torch.Generator on device)",
            "config": {"workload": f"attention B={B} H={H} M={M} N={N} D={D}{' causal' if causal else ''}",
                       "l2": "inputs larger than L2" if 2 * B * H * N * D * 2 > L2_BYTES
                             else "K/V may stay in L2 between steps"},
            "route": route_f, "kernels_per_step": launches_f,
            "composed": {"route": route_c, "ms": ms_c, "tflops": flops / (ms_c / 1e3) / 1e12,
                         "kernels_per_step": launches_c},
            "roofline": {"bound": "tensor", "achieved": value, "peak": peak, "unit": "TFLOP/s",
                         "frac": value / peak, "peak_source": f"{peak_kind} bf16_tflops"},
            "clocks": {k: clocks[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}}
    print(json.dumps(line), flush=True)
    return 0


def graph_measure(args, cfg, A, W, bias, dev, iters: int = 200):
    """Host dispatch vs graph replay of one step through the public torchcl API.

    Dispatch: `blas.gemm(a, w, bias, act)` builds the lazy fused GEMM and a
    materialisation launches it (handles, descriptor, ctypes call, pool
    allocation).  Replay: the same step captured once with capture_graph and
    re-launched with CapturedGraph.replay().  Both timed on the host over `iters`
    steps with one synchronize at the end (the reference's showcase measures its
    replay speed-up the same way), after 10 untimed steps."""
    import torch
    import torchcl
    from torchcl import api, blas
    from torchcl.jit.graph_runner import capture_graph

    a = torchcl.to_opencl(A.cpu())
    w = torchcl.to_opencl(W.cpu())
    b = torchcl.to_opencl(bias.cpu())

    def step():
        out = blas.gemm(a, w, bias=b, activation=cfg["act"])
        api._get_buf(out)  # materialise: the launch
        return out

    def timed(fn):
        for _ in range(10):
            fn()
        torchcl.synchronize()
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
        torchcl.synchronize()
        return (time.perf_counter() - t0) / iters * 1e6

    dispatch_us = timed(step)
    with capture_graph("bench_step") as cg:
        out = step()
    ref = torchcl.to_cpu(step())
    cg.replay()
    got = torchcl.to_cpu(out)
    replay_us = timed(cg.replay)
    same = bool(torch.equal(ref, got))
    n_kernels = len(cg)
    cg.close()
    return {"dispatch_us_per_step": dispatch_us, "replay_us_per_step": replay_us,
            "speedup": dispatch_us / replay_us, "kernels_per_step": n_kernels,
            "replay_matches_dispatch": same, "iters": iters,
            "note": "host wall clock per step, one synchronize after the loop"}


def _traffic(args):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summaries
    (profiles/traffic.json), or None when that workload was not captured."""
    key = args.config + (f"@{args.size}" if args.size else "") + (f"@m{args.m}" if args.m else "")
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(key)
        except Exception:
            return None
    return None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="cfg5", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="multi-GPU: all-gather fused into the GEMM epilogue (p2p) or NCCL")
    # --decode-rows is the spelling to use under torchrun, whose parser takes a bare
    # --m for an abbreviation of its own options
    ap.add_argument("--m", "--decode-rows", dest="m", type=int, default=None,
                    help="override M (e.g. cfg4 M in {1,4,16})")
    ap.add_argument("--size", type=int, default=None, help="override M=N=K (cfg2 sweep)")
    ap.add_argument("--attn", default=None,
                    help="one GPU: time fused attention, 'B,H,M,N,D[,causal]' (bf16)")
    ap.add_argument("--batch", type=int, default=None,
                    help="one GPU: time this many problems of the config's shape in one batched GEMM")
    ap.add_argument("--train", action="store_true",
                    help="one GPU: time a linear-layer training step (forward + backward GEMMs)")
    ap.add_argument("--pair", action="store_true",
                    help="CTA-pair (cta_group::2) tcgen05 tiles where they apply (one-CTA tiles otherwise)")
    ap.add_argument("--skinny-counter", action="store_true",
                    help="skinny route: hand split-K partials over through the arrival counter "
                         "(the tagged hand-off otherwise, where it applies)")
    ap.add_argument("--graph", action="store_true",
                    help="one GPU: also time public-API dispatch vs graph replay of one step")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.m is not None:
        cfg["M"] = args.m
    if args.size is not None:
        cfg["M"] = cfg["N"] = cfg["K"] = args.size
    if args.m is not None or args.size is not None:
        cfg["desc"] += f" [M={cfg['M']} N={cfg['N']} K={cfg['K']}]"
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, cfg, world, rank)
    if args.attn:
        return run_attention(args)
    if args.train:
        return run_train(args, cfg)
    if args.batch:
        return run_batched(args, cfg)
    world, rank, local = _dist_setup()
    if world > 1 and args.config != "cfg5" and args.config != "cfg4":
        if rank == 0:
            print(json.dumps({"error": f"{args.config} runs on one GPU"}))
        return 0
    return run_ours(args, cfg, world, rank, local)


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python3
"""Benchmark of the B200 quantized-matmul / turbo4 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

Prints ONE JSON line (rank 0). Workloads (the reference benchmark configurations 1-5, seeded synthetic data):
  gemv   config 1: Q4_0 x Q8_0 GEMV of the Qwen3-1.7B gate_proj shape (6144 x 2048,
         W ~ N(0, 0.02) quantized with the reference's Q4_0 rule, x ~ N(0, 1)). One step =
         quantize x once + one matmul_multi launch over a stack of 72 distinct weight
         copies (510 MB, > 4x the 126 MB L2, so every step streams from HBM).
The reference arm (--impl reference) times the reference's CPU algorithm (the oracle
restatement of RIE's AVX2 path, all host cores) on a bounded sample of the same workload.
Multi-GPU: one process per GPU; each rank runs its own stack (weak scaling, no collective).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


FALLBACK_BF16_TFLOPS = 1590.0


def bf16_peak():
    """Dense bf16 (= f16) tensor throughput: MEASURED_PEAKS.json burst figure, else fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (cuBLAS bf16 8192^3 burst)"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded from an ncu capture (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(name)
    except Exception:
        return None


class Clocks:
    """Samples SM clocks / throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in (out or "").splitlines() if ln.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def tp_comm_id(world: int, rank: int):
    """Communicator id of a tensor-parallel backend: made on rank 0, broadcast to all."""
    if world == 1:
        return None
    import torch.distributed as dist
    from rust_interference_engine_b200 import model as M
    box = [M.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def dist_min(x: float, world: int) -> float:
    return -dist_max(-x, world)


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- workload: config 1 GEMV stack ---------------------------------------------------------
GEMV_ROWS, GEMV_K, GEMV_COPIES, GEMV_DISTINCT = 6144, 2048, 72, 8
GEMV_TYPE = "Q4_0"  # config 1; --wtype runs the same shape in another GGUF type
GEMV_EACH = False  # --shape RxK: weights of another shape, one launch per weight (decode-like)
BLOCK = {"Q4_0": (32, 18), "Q4_1": (32, 20), "Q5_0": (32, 22), "Q5_1": (32, 24), "Q8_0": (32, 34),
         "Q4_K": (256, 144), "Q5_K": (256, 176), "Q6_K": (256, 210)}


def gemv_weights(seed: int = 1):
    """GEMV_DISTINCT distinct matrices from N(0, 0.02) with the reference's quantizer."""
    import oracle as O
    rng = np.random.default_rng(seed)
    mats = []
    for _ in range(GEMV_DISTINCT):
        wf = rng.normal(0.0, 0.02, (GEMV_ROWS, GEMV_K)).astype(np.float32)
        mats.append(O.quantize_weight(getattr(O, GEMV_TYPE), wf))
    x = rng.standard_normal((1, GEMV_K)).astype(np.float32)
    return mats, x


def gemv_bytes_per_step():
    bs, bb = BLOCK[GEMV_TYPE]
    w = GEMV_ROWS * GEMV_K // bs * bb
    return GEMV_COPIES * (w + GEMV_K * 4 + GEMV_ROWS * 4), w


def gemv_kernel_name(wtype: str, launch_bytes: int, k: int = 4096) -> str:
    """The batch-1 GEMV kernel the library picks: the tensor-core kernel for Q4_K / Q5_K / Q6_K /
    Q4_0 launches of at least 8 MiB of weights (default of RIE_GEMV_KQ_MIN_MB), else the lane
    kernel."""
    min_mb = int(os.environ.get("RIE_GEMV_KQ_MIN_MB", "8"))
    if wtype == "Q4_0" and k < 4096:  # short Q4_0 rows stay on the lane kernel
        return "k_gemv<1,16>"
    if wtype in ("Q4_K", "Q5_K", "Q6_K", "Q4_0") and launch_bytes >= (min_mb << 20) and os.environ.get("RIE_GEMV_KQ") != "0":
        return "k_gemv_kq"
    return "k_gemv<1,16>"


def gemv_meta():
    kq = GEMV_TYPE.endswith("_K")
    tag = "config 1" if GEMV_TYPE == "Q4_0" else "config-1 shape"
    if GEMV_EACH:
        tag = f"{GEMV_ROWS}x{GEMV_K}, one launch per weight"
    return {"metric": f"quant-matmul HBM GB/s ({GEMV_TYPE} x {'Q8_K' if kq else 'Q8_0'} GEMV, {tag})", "unit": "GB/s",
            "dtype": f"int8 ({GEMV_TYPE} x {'Q8_K' if kq else 'Q8_0'} blocks, f32 combine)",
            "workload": f"gemv_{GEMV_TYPE.lower()}_{GEMV_ROWS}x{GEMV_K}" + ("_config1" if GEMV_TYPE == "Q4_0" else "")}


def run_gemv(args, world, rank, local):
    import torch

    import rust_interference_engine_b200 as rie
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    ctx = rie.Context(local, stream)
    ctx.set_static_weights(True)  # weights are uploaded once: matmuls stream them early (PDL)
    mats, x = gemv_weights()
    ws = [rie.Weight.upload(ctx, getattr(rie.GgmlType, GEMV_TYPE), GEMV_ROWS, GEMV_K, mats[i % GEMV_DISTINCT])
          for i in range(GEMV_COPIES)]
    fmt = rie.ActFormat.Q8K if GEMV_TYPE.endswith("_K") else rie.ActFormat.Q8_0
    xd = torch.from_numpy(x).cuda()
    outs = torch.zeros((GEMV_COPIES, GEMV_ROWS), device="cuda")
    acts = rie.QuantActs(ctx, 1, GEMV_K)
    jobs = [rie.MatmulJob(w, outs[i], GEMV_ROWS) for i, w in enumerate(ws)]

    def step(ev=None):
        acts.prepare(xd, 1, GEMV_K, fmt)
        if ev is not None:
            ev[0].record(stream)
        if GEMV_EACH:
            for j in jobs:
                rie.matmul_multi(ctx, acts, [j])
        else:
            rie.matmul_multi(ctx, acts, jobs)
        if ev is not None:
            ev[1].record(stream)

    for _ in range(max(args.warmup, 3)):
        step()
    ctx.sync()
    # parity spot check of the benchmarked output against the oracle
    import oracle as O
    want = O.matmul_multi(x, [(getattr(O, GEMV_TYPE), mats[0], GEMV_K)], n_threads=8)[0][0]
    got = outs[0].cpu().numpy()
    max_rel = float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-6))

    kern_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            step(kern_ev[i])
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = t0.elapsed_time(t1) / args.steps
    kern_ms = float(np.mean([a.elapsed_time(b) for a, b in kern_ev]))
    ctx.sync()

    # end to end through the public API with host buffers
    xh = torch.from_numpy(x).pin_memory()
    oh = torch.empty((GEMV_COPIES, GEMV_ROWS), pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            barrier(world)
            torch.cuda.synchronize()
            e0.record(stream)
        xd.copy_(xh, non_blocking=True)
        step()
        oh.copy_(outs, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    ms = dist_max(ms, world)
    e2e_ms = dist_max(e2e_ms, world)
    kern_ms = dist_max(kern_ms, world)
    step_bytes, w_bytes = gemv_bytes_per_step()
    peak, peak_kind = peaks()
    achieved = step_bytes / (kern_ms * 1e-3) / 1e9
    gm = gemv_meta()
    res = {
        "metric": gm["metric"],
        "value": world * step_bytes / (ms * 1e-3) / 1e9,
        "unit": "GB/s",
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "dtype": gm["dtype"],
        "config": {"workload": gm["workload"], "rows": GEMV_ROWS, "k": GEMV_K,
                   "weight_copies_per_step": GEMV_COPIES, "bytes_per_step": step_bytes,
                   "l2": f"inputs larger than L2 ({step_bytes / 1e6:.0f} MB weight stack per step)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "traffic": profile_traffic(gm["workload"]),
                     "kernel": gemv_kernel_name(GEMV_TYPE, step_bytes // (1 if not GEMV_EACH else GEMV_COPIES), GEMV_K),
                     "bytes_per_launch": step_bytes, "launch_ms": kern_ms},
        "e2e": {"value": world * step_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": GEMV_K * 4, "d2h_bytes_per_step": GEMV_COPIES * GEMV_ROWS * 4,
                "ms_per_step": e2e_ms},
        "gpu_launches": (1 + (GEMV_COPIES if GEMV_EACH else 1)) * args.steps,
        "clocks": clk.summary(),
        "check": {"max_rel_err_vs_oracle": max_rel, "tolerance": 1e-3},
    }
    return res


def cpu_gemv_sample(seconds: float, threads: int):
    """The oracle (RIE's AVX2 CPU path restated) on GEMVs of the same workload."""
    import oracle as O
    mats, x = gemv_weights()
    _, w_bytes = gemv_bytes_per_step()
    per = w_bytes + GEMV_K * 4 + GEMV_ROWS * 4
    t = getattr(O, GEMV_TYPE)
    O.matmul_multi(x, [(t, mats[0], GEMV_K)], n_threads=threads)
    n, t0 = 0, time.perf_counter()
    while True:
        O.matmul_multi(x, [(t, mats[n % GEMV_DISTINCT], GEMV_K)], n_threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": n * per / el / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} GEMVs of {GEMV_ROWS}x{GEMV_K} {GEMV_TYPE} (rotating over {GEMV_DISTINCT} matrices), {el:.1f} s",
            "path": "avx2" if O.have_avx2() else "scalar"}


# ---- workload: config 2 prefill GEMM -----------------------------------------------------
PF_M, PF_K, PF_N = 512, 4096, (14336, 4096)


def measured_int8_peak(torch):
    """cuBLAS int8 GEMM throughput (torch._int_mm, 8192^3, best of 5) as the tensor peak."""
    try:
        a = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda").t()
        for _ in range(3):
            torch._int_mm(a, b)
        best = 1e9
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        return 2 * 8192 ** 3 / (best * 1e-3) / 1e12, "measured (cuBLAS int8 via torch._int_mm, 8192^3 burst)"
    except Exception as e:  # pragma: no cover
        return 4500.0, f"nominal 4.5 POPS dense int8 ({type(e).__name__})"


def fma_peak() -> float:
    """f32 FMAs per second of the FP32 pipe: 148 SMs x 128 lanes x the maximum SM clock."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mhz = float(json.load(f).get("sm_max_mhz", 1965.0))
    except Exception:
        mhz = 1965.0
    return 148 * 128 * mhz * 1e6


def prefill_meta(gemm: str):
    """The prefill line names the arithmetic it measures: f16 tensor-core MMA on dequantized
    operands (default) or int8 MMA with the reference's exact block sums (--gemm i8)."""
    if gemm == "i8":
        return {"metric": "prefill Q4_0 GEMM int8 TOPS (config 2, M=512 K=4096 N=14336+4096, exact int8 block sums)",
                "unit": "TOPS", "dtype": "int8 (Q4_0 x Q8_0 blocks, tcgen05 kind::i8, f32 block-scale epilogue)",
                "workload": "prefill_q4_0_m512_k4096_config2_i8"}
    return {"metric": "prefill Q4_0 GEMM f16 TFLOP/s (config 2, M=512 K=4096 N=14336+4096, f16 MMA on dequantized operands)",
            "unit": "TFLOP/s", "dtype": "f16 MMA on dequantized Q4_0 weights x Q8_0 activations (d*q), f32 accumulate",
            "workload": "prefill_q4_0_m512_k4096_config2_f16"}


def run_prefill(args, world, rank, local):
    import torch

    import oracle as O
    import rust_interference_engine_b200 as rie
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    ctx = rie.Context(local, stream)
    i8 = args.gemm == "i8"
    ctx.set_prefill_gemm(rie.PrefillGemm.I8 if i8 else rie.PrefillGemm.F16)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((PF_M, PF_K)).astype(np.float32)
    mats = [O.quantize_weight(O.Q4_0, rng.normal(0.0, 0.02, (n, PF_K)).astype(np.float32)) for n in PF_N]
    ws = [rie.Weight.upload(ctx, rie.GgmlType.Q4_0, n, PF_K, m) for n, m in zip(PF_N, mats)]
    xd = torch.from_numpy(x).cuda()
    outs = [torch.zeros((PF_M, n), device="cuda") for n in PF_N]
    acts = rie.QuantActs(ctx, PF_M, PF_K)
    jobs = [rie.MatmulJob(w, o, w.rows) for w, o in zip(ws, outs)]
    flops = sum(2 * PF_M * PF_K * n for n in PF_N)

    def step(ev=None):
        acts.prepare(xd, PF_M, PF_K, rie.ActFormat.Q8_0)
        if ev is not None:
            ev[0].record(stream)
        rie.matmul_multi(ctx, acts, jobs)
        if ev is not None:
            ev[1].record(stream)

    for _ in range(max(args.warmup, 3)):
        step()
    ctx.sync()
    want = O.matmul_multi(x[:64], [(O.Q4_0, mats[1], PF_K)], n_threads=8)[0]
    got = outs[1][:64].cpu().numpy()
    max_rel = float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-6))
    kern_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            step(kern_ev[i])
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = dist_max(t0.elapsed_time(t1) / args.steps, world)
    kern_ms = dist_max(float(np.mean([a.elapsed_time(b) for a, b in kern_ev])), world)
    xh = torch.from_numpy(x).pin_memory()
    ohs = [torch.empty(o.shape, pin_memory=True) for o in outs]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            barrier(world)
            torch.cuda.synchronize()
            e0.record(stream)
        xd.copy_(xh, non_blocking=True)
        step()
        for oh, o in zip(ohs, outs):
            oh.copy_(o, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist_max(e0.elapsed_time(e1) / args.steps, world)
    i8_peak, i8_kind = measured_int8_peak(torch)
    achieved = flops / (kern_ms * 1e-3) / 1e12
    if i8:
        peak, peak_kind, kernel = i8_peak, i8_kind, "k_gemm_i8 (tcgen05 kind::i8, both weights in one launch)"
        dtype = "int8 (Q4_0 x Q8_0 blocks, tcgen05 kind::i8, exact block sums, f32 block-scale epilogue)"
        launches = 2  # activation quantization + one GEMM launch
    else:
        peak, peak_kind = bf16_peak()
        kernel = "k_acts_f16 + k_gemm_f16<Q4_0> (tcgen05 kind::f16, both weights in one launch)"
        dtype = "f16 MMA on dequantized Q4_0 weights x Q8_0 activations (d*q), f32 accumulate"
        launches = 3
    pm = prefill_meta(args.gemm)
    return {
        "metric": pm["metric"],
        "value": world * flops / (ms * 1e-3) / 1e12,
        "unit": pm["unit"],
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "dtype": dtype,
        "config": {"workload": pm["workload"], "m": PF_M, "k": PF_K, "n": list(PF_N),
                   "ops_per_step": flops, "l2": "weights 42 MB + activations (L2-resident re-use by design)",
                   "parallelism": f"replicas x{world}", "gemm": args.gemm,
                   "int8_peak_tops": i8_peak, "frac_of_int8_peak": achieved / i8_peak,
                   # exact block sums cost two f32 FMAs per output per 32-value block (d_w, then d_a):
                   # at 128 FMA per clock per SM that work alone bounds the int8 kernel
                   "fp32_epilogue_bound_tops": flops / (2 * PF_M * sum(PF_N) * (PF_K // 32) / fma_peak()) / 1e12,
                   "frac_of_epilogue_bound": achieved / (flops / (2 * PF_M * sum(PF_N) * (PF_K // 32) / fma_peak()) / 1e12)},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": pm["unit"], "frac": achieved / peak,
                     "peak_source": peak_kind,
                     "traffic": profile_traffic("gemm_i8_q4_0_config2" if i8 else "gemm_f16_q4_0_config2"),
                     "kernel": kernel, "launch_ms": kern_ms,
                     "note": "achieved = 2*M*K*N over the matmul_multi call (activation f16 prep + GEMM)"},
        "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": pm["unit"],
                "h2d_bytes_per_step": PF_M * PF_K * 4, "d2h_bytes_per_step": sum(PF_M * n * 4 for n in PF_N),
                "ms_per_step": e2e_ms},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
        "check": {"max_rel_err_vs_oracle": max_rel, "tolerance": 1e-3},
    }


# ---- workload: config 3 Qwen3-8B-shape Q4_K_M decode ------------------------------------
QWEN3_8B = dict(arch="qwen3", n_vocab=151936, n_embd=4096, n_layer=36, n_head=32, n_head_kv=8, head_dim=128,
                n_ff=12288, rope_dim=128, rope_base=1_000_000.0, rms_eps=1e-6)
DEC_PROMPT = 512  # config 3: 512-token prompt (--prompt changes it, e.g. for a short profile)
DEC_BATCH = 512   # prompt tokens per forward (the reference's --batch / n_batch; its CLI default is 64)


def qwen3_8b_spec(n_layer=None):
    from rust_interference_engine_b200 import GgmlType as G
    from rust_interference_engine_b200.model import SyntheticSpec
    kw = dict(QWEN3_8B)
    if n_layer is not None:
        kw["n_layer"] = n_layer
    return SyntheticSpec(wtype=G.Q4_K, embd_type=G.Q6_K, qk_norm=True,
                         type_overrides={"attn_v.weight": G.Q6_K, "ffn_down.weight": G.Q6_K}, **kw)


class RandomBlocks:
    """random_weight semantics (testing.rs:46-91) at numpy speed: random bytes with valid f16
    scale fields U[0.5, 1) x per-type scale (negative 30 % of the time where the reference
    allows it). The bytes differ from the reference's xorshift stream; the distribution is
    the one `rie bench --synthetic` uses."""

    SCALE = {2: 0.01, 3: 0.01, 6: 0.005, 7: 0.005, 8: 0.001, 12: 0.001, 13: 0.0007, 14: 0.0001}
    OFFS = {2: [0], 6: [0], 8: [0], 3: [0, 2], 7: [0, 2], 12: [0, 2], 13: [0, 2], 14: [208]}
    BB = {2: 18, 3: 20, 6: 22, 7: 24, 8: 34, 12: 144, 13: 176, 14: 210}
    BS = {2: 32, 3: 32, 6: 32, 7: 32, 8: 32, 12: 256, 13: 256, 14: 256}

    def __init__(self, seed):
        self.rng = np.random.default_rng(seed)

    def weight(self, t, rows, cols):
        t = int(t)
        nb = rows * cols // self.BS[t]
        data = np.frombuffer(self.rng.bytes(nb * self.BB[t]), dtype=np.uint8).reshape(nb, self.BB[t]).copy()
        for i, off in enumerate(self.OFFS[t]):
            v = (self.rng.random(nb, dtype=np.float32) * 0.5 + 0.5) * self.SCALE[t]
            if i == 0 and t in (2, 6, 8, 14):
                v = np.where(self.rng.random(nb, dtype=np.float32) < 0.3, -v, v)
            if i == 1 and t in (3, 7):
                v = -v * 8.0
            data[:, off:off + 2] = v.astype(np.float16).view(np.uint8).reshape(nb, 2)
        return data.reshape(-1)

    def vec(self, n, scale):
        return (self.rng.random(n, dtype=np.float32) * 2 - 1) * scale

    def norm(self, n):
        return (1.0 + 0.1 * (self.rng.random(n, dtype=np.float32) * 2 - 1)).astype(np.float32)


class DeviceWeights:
    """Benchmark weights as the configurations state them: N(0, 0.02) values drawn on the device
    (torch generator with a fixed seed, so every rank draws the same full tensors) and quantized
    there by the library (rcu_quantize_weight: Q4_0 / Q8_0 by the reference's rules, Q4_K / Q6_K
    by the library's own). Norm and bias vectors come from the host generator."""

    def __init__(self, ctx, seed):
        import torch
        self.ctx = ctx
        self.gen = torch.Generator(device="cuda").manual_seed(seed)
        self.host = RandomBlocks(seed)

    def weight(self, t, rows, cols):
        import torch

        import rust_interference_engine_b200 as rie
        ty = rie.GgmlType(int(t))
        rb = ty.row_bytes(cols)
        out = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
        chunk = max(1, (1 << 28) // cols)  # rows per 1 GiB f32 draft
        for r0 in range(0, rows, chunk):
            n = min(chunk, rows - r0)
            x = torch.empty(n, cols, device="cuda").normal_(0.0, 0.02, generator=self.gen)
            rie.quantize_weight(self.ctx, ty, n, cols, x, out[r0 * rb:])
        return out

    def vec(self, n, scale):
        return self.host.vec(n, scale)

    def norm(self, n):
        return self.host.norm(n)


def set_synthetic(model, spec, gen):
    """Loads every tensor of a synthetic model (device bytes go in without a host copy)."""
    for name, t, rows, cols, data in __import__("rust_interference_engine_b200.model", fromlist=["x"]).synthetic_tensors(
            spec, gen.weight, gen.vec, gen.norm):
        if hasattr(data, "is_cuda"):
            model.set_tensor_device(name, int(t), rows, cols, data)
        else:
            model.set_tensor(name, int(t), rows, cols, data)


def weight_bytes_per_token(spec):
    from rust_interference_engine_b200 import GgmlType as G
    e, ff, qd, kvd = spec.n_embd, spec.n_ff, spec.n_head * spec.head_dim, spec.n_head_kv * spec.head_dim
    per_layer = sum(G(spec.type_of(n)).row_bytes(c) * r for n, r, c in (
        ("attn_q.weight", qd, e), ("attn_k.weight", kvd, e), ("attn_v.weight", kvd, e), ("attn_output.weight", e, qd),
        ("ffn_gate.weight", ff, e), ("ffn_up.weight", ff, e), ("ffn_down.weight", e, ff)))
    head = G(spec.embd_type).row_bytes(e) * spec.n_vocab
    return spec.n_layer * per_layer + head


def run_decode(args, world, rank, local):
    import torch

    import rust_interference_engine_b200 as rie
    from rust_interference_engine_b200 import model as M
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    ctx = rie.Context(local, stream)
    spec = qwen3_8b_spec()
    gen = DeviceWeights(ctx, 3)  # same seed on every rank: every rank sees the same full tensors
    # N > 1: one model split tensor-parallel over the N GPUs (each rank keeps its shard)
    model = M.Model(ctx, spec.config(), rank, world)
    t_build = time.perf_counter()
    set_synthetic(model, spec, gen)
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t_build
    n_gen = max(args.warmup, 3) + args.steps
    n_ctx = DEC_PROMPT + n_gen + 1
    nb = DEC_BATCH
    be = M.CudaBackend(model, n_ctx, nb, rie.KvType.F16, comm_id=tp_comm_id(world, rank))
    prompt = np.random.default_rng(4).integers(0, spec.n_vocab, DEC_PROMPT).astype(np.uint32)
    gen_tokens = torch.from_numpy(np.random.default_rng(5).integers(0, spec.n_vocab, n_gen).astype(np.int32)).cuda()
    logits = torch.zeros(spec.n_vocab, device="cuda")
    prompt_d = torch.from_numpy(prompt.astype(np.int32)).cuda()

    def prefill():
        for p0 in range(0, DEC_PROMPT, nb):  # Engine::eval_tokens chunks at n_batch (engine.rs:263-269)
            be.forward_device(prompt_d[p0:], min(nb, DEC_PROMPT - p0), p0, logits)

    prefill()  # warm: kernel attributes, L2
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    prefill()
    p1.record(stream)
    torch.cuda.synchronize()
    pp_tps = DEC_PROMPT / (p0.elapsed_time(p1) * 1e-3)
    pos = DEC_PROMPT
    for i in range(max(args.warmup, 3)):  # the second decode step captures the CUDA graph
        be.forward_device(gen_tokens[i:], 1, pos, logits)
        pos += 1
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        torch.cuda.nvtx.range_push("decode_steps")  # lets a profiler select the timed launches
        t0.record(stream)
        for i in range(args.steps):
            be.forward_device(gen_tokens[max(args.warmup, 3) + i:], 1, pos + i, logits)
        t1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier(world)
    ms = dist_max(t0.elapsed_time(t1) / args.steps, world)
    finite = bool(torch.isfinite(logits).all())

    # e2e: the host API (Backend::forward), token in and logits out through host memory
    be2 = M.CudaBackend(model, n_ctx, nb, rie.KvType.F16, comm_id=tp_comm_id(world, rank))
    for p0_ in range(0, DEC_PROMPT, nb):
        be2.forward(prompt[p0_:p0_ + nb], p0_, False)
    pos2, tok = DEC_PROMPT, np.array([1], dtype=np.uint32)
    for i in range(max(args.warmup, 3)):
        be2.forward(tok, pos2)
        pos2 += 1
    e0 = time.perf_counter()
    for i in range(args.steps):
        out = be2.forward(tok, pos2)
        tok = np.array([int(np.argmax(out[0]))], dtype=np.uint32)  # greedy, as Engine::bench
        pos2 += 1
    e2e_s = time.perf_counter() - e0
    e2e_tps = args.steps / e2e_s
    del be2

    # dominant kernel: the gate+up GEMV launch (2 x 12288 x 4096 Q4_K), timed alone over
    # 8 layers' worth of distinct weights (453 MB > L2)
    gu_bytes = [gen.weight(rie.GgmlType.Q4_K, spec.n_ff, spec.n_embd) for _ in range(16)]
    gu = [rie.Weight.view(ctx, rie.GgmlType.Q4_K, spec.n_ff, spec.n_embd, b) for b in gu_bytes]
    xg = torch.randn(1, spec.n_embd, device="cuda")
    acts = rie.QuantActs(ctx, 1, spec.n_embd)
    acts.prepare(xg, 1, spec.n_embd, rie.ActFormat.Q8K)
    og = torch.zeros(2, spec.n_ff, device="cuda")
    jobs = [[rie.MatmulJob(gu[2 * i], og[0]), rie.MatmulJob(gu[2 * i + 1], og[1])] for i in range(8)]
    ctx.set_static_weights(True)  # as inside the forward: weights stream while the previous launch ends
    for j in jobs:
        rie.matmul_multi(ctx, acts, j)
    torch.cuda.synchronize()
    # 40 launches captured in one CUDA graph (as the decode step runs them: no host launch cost
    # between kernels), replayed three times; the fastest replay counts
    reps = 40
    gs = torch.cuda.Stream()
    ctx.set_stream(gs)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for r in range(reps):
            rie.matmul_multi(ctx, acts, jobs[r % 8])
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(4):
        with torch.cuda.stream(gs):
            g0.record(gs)
            graph.replay()
            g1.record(gs)
        gs.synchronize()
        times.append(g0.elapsed_time(g1) / reps)
    gemv_ms = min(times[1:])
    del graph
    ctx.set_stream(stream)
    gemv_bytes = 2 * rie.GgmlType.Q4_K.row_bytes(spec.n_embd) * spec.n_ff
    peak, peak_kind = peaks()
    achieved = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    wbytes = weight_bytes_per_token(spec)
    kv_bytes = 2 * spec.n_layer * spec.n_head_kv * spec.head_dim * 2 * (pos + args.steps // 2)
    return {
        "metric": "Qwen3-8B-shape Q4_K_M decode tg tok/s (config 3, batch 1)",
        "value": 1000.0 / ms,  # one sequence: N > 1 splits the model (tensor parallel), not the work
        "unit": "tok/s",
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "dtype": "int8 x Q4_K/Q6_K blocks (Q8_K activations), f32 glue, f16 KV",
        "config": {"workload": "qwen3_8b_q4_k_m_decode_config3", "layers": spec.n_layer, "hidden": spec.n_embd,
                   "ffn": spec.n_ff, "heads": f"{spec.n_head}/{spec.n_head_kv}x{spec.head_dim}",
                   "vocab": spec.n_vocab, "prompt": DEC_PROMPT, "context_at_timing": pos,
                   "weight_bytes_per_token": wbytes, "kv": "f16", "batch": 1,
                   "l2": "inputs larger than L2 (4.9 GB of weights streamed per token)",
                   "parallelism": f"tp{world} (NCCL all-reduce of Wo/down, all-gather of logits)" if world > 1
                   else "tp1", "decode": "CUDA graph replay per token",
                   "pp_tok_s": pp_tps, "prefill_batch": nb, "model_build_s": t_build},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind,
                     # ncu figure of this launch for the kernel that runs it (null until captured)
                     "traffic": profile_traffic("gemv_q4_k_gate_up" if gemv_kernel_name("Q4_K", gemv_bytes) ==
                                                "k_gemv<1,16>" else "gemv_kq_q4_k_gate_up"),
                     "kernel": gemv_kernel_name("Q4_K", gemv_bytes) + " (gate+up, 2 x 12288 x 4096 Q4_K)",
                     "bytes_per_launch": gemv_bytes,
                     "timing": "40 launches over 8 layers' distinct weights (453 MB > L2) in one CUDA graph",
                     "launch_ms": gemv_ms,
                     "whole_step_weight_gb_s": (wbytes + kv_bytes) / (ms * 1e-3) / 1e9},
        "e2e": {"value": dist_min(e2e_tps, world), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": spec.n_vocab * 4, "ms_per_step": 1000.0 * e2e_s / args.steps,
                "api": "CudaBackend.forward (rcu_backend_forward, host tokens/logits, greedy)"},
        # per token: 8 per layer (norm, QKV GEMV, attention with the q/k post-processing and KV
        # append, Wo GEMV, norm, gate+up GEMV, GLU, down GEMV) + position, embedding, final norm,
        # head GEMV (NCCL's own kernels at N > 1 not counted)
        "gpu_launches": args.steps * (8 * spec.n_layer + 4),
        "clocks": clk.summary(),
        "check": {"logits_finite": finite},
    }


# ---- workload: config 4 MoE decode (Qwen3-30B-A3B shape) --------------------------------
QWEN3_30B_A3B = dict(arch="qwen3moe", n_vocab=151936, n_embd=2048, n_layer=48, n_head=32, n_head_kv=4, head_dim=128,
                     n_ff=6144, rope_dim=128, rope_base=1_000_000.0, rms_eps=1e-6, n_expert=128, n_expert_used=8,
                     n_ff_exp=768, n_ff_shexp=0)
MOE_PROMPT = 64


def qwen3_moe_spec():
    from rust_interference_engine_b200 import GgmlType as G
    from rust_interference_engine_b200.model import SyntheticSpec
    return SyntheticSpec(wtype=G.Q4_K, embd_type=G.Q4_K, qk_norm=True, **QWEN3_30B_A3B)


def moe_bytes_per_token(spec):
    """Weight bytes one decoded token reads: attention, router (f32), 8 experts, head."""
    from rust_interference_engine_b200 import GgmlType as G
    rb = lambda cols: G.Q4_K.row_bytes(cols)
    e, qd, kvd = spec.n_embd, spec.n_head * spec.head_dim, spec.n_head_kv * spec.head_dim
    attn = (qd + 2 * kvd) * rb(e) + e * rb(qd)
    experts = spec.n_expert_used * (2 * spec.n_ff_exp * rb(e) + e * rb(spec.n_ff_exp))
    router = spec.n_expert * e * 4
    return spec.n_layer * (attn + experts + router) + spec.n_vocab * rb(e)


def run_moe(args, world, rank, local):
    import torch

    import rust_interference_engine_b200 as rie
    from rust_interference_engine_b200 import model as M
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    ctx = rie.Context(local, stream)
    spec = qwen3_moe_spec()
    gen = DeviceWeights(ctx, 4)  # same seed on every rank: every rank sees the same full tensors
    # N > 1: attention tensor-parallel, experts split across the ranks (expert parallelism)
    model = M.Model(ctx, spec.config(), rank, world)
    t_build = time.perf_counter()
    set_synthetic(model, spec, gen)
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t_build
    n_gen = max(args.warmup, 3) + args.steps
    be = M.CudaBackend(model, MOE_PROMPT + n_gen + 1, 64, rie.KvType.F16, comm_id=tp_comm_id(world, rank))
    prompt = torch.from_numpy(np.random.default_rng(4).integers(0, spec.n_vocab, MOE_PROMPT).astype(np.int32)).cuda()
    gen_tokens = torch.from_numpy(np.random.default_rng(5).integers(0, spec.n_vocab, n_gen).astype(np.int32)).cuda()
    logits = torch.zeros(spec.n_vocab, device="cuda")
    be.forward_device(prompt, MOE_PROMPT, 0, logits)
    pos = MOE_PROMPT
    for i in range(max(args.warmup, 3)):
        be.forward_device(gen_tokens[i:], 1, pos, logits)
        pos += 1
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            be.forward_device(gen_tokens[max(args.warmup, 3) + i:], 1, pos + i, logits)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = dist_max(t0.elapsed_time(t1) / args.steps, world)
    finite = bool(torch.isfinite(logits).all())
    # e2e: host tokens in, host logits out (Backend::forward)
    be2 = M.CudaBackend(model, MOE_PROMPT + n_gen + 1, 64, rie.KvType.F16, comm_id=tp_comm_id(world, rank))
    be2.forward(prompt.cpu().numpy().astype(np.uint32), 0)
    tok, p2 = np.array([1], dtype=np.uint32), MOE_PROMPT
    for i in range(max(args.warmup, 3)):
        be2.forward(tok, p2)
        p2 += 1
    barrier(world)
    e0 = time.perf_counter()
    for i in range(args.steps):
        out = be2.forward(tok, p2)
        tok = np.array([int(np.argmax(out[0]))], dtype=np.uint32)
        p2 += 1
    e2e_tps = args.steps / dist_max(time.perf_counter() - e0, world)
    be2.free()
    # batch of 256 tokens in one forward (config 4's large batch)
    be3 = M.CudaBackend(model, 512, 256, rie.KvType.F16, comm_id=tp_comm_id(world, rank))
    big = torch.from_numpy(np.random.default_rng(6).integers(0, spec.n_vocab, 256).astype(np.int32)).cuda()
    be3.forward_device(big, 256, 0, logits)
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    b0.record(stream)
    be3.forward_device(big, 256, 256, logits)
    b1.record(stream)
    torch.cuda.synchronize()
    b256_tps = 256 / (dist_max(b0.elapsed_time(b1), world) * 1e-3)
    be3.free()
    # dominant kernel: the expert gate+up GEMV of one token (16 x 768 x 2048 Q4_K), timed alone
    # over distinct copies (> L2)
    ws_bytes = [gen.weight(rie.GgmlType.Q4_K, spec.n_ff_exp, spec.n_embd) for _ in range(16 * 12)]
    ws = [rie.Weight.view(ctx, rie.GgmlType.Q4_K, spec.n_ff_exp, spec.n_embd, b) for b in ws_bytes]
    xg = torch.randn(1, spec.n_embd, device="cuda")
    acts = rie.QuantActs(ctx, 1, spec.n_embd)
    acts.prepare(xg, 1, spec.n_embd, rie.ActFormat.Q8K)
    ctx.set_static_weights(True)  # as inside the forward: weights stream while the previous launch ends
    og = torch.zeros(16, spec.n_ff_exp, device="cuda")
    jobs = [[rie.MatmulJob(ws[16 * g + j], og[j]) for j in range(16)] for g in range(12)]
    for j in jobs:
        rie.matmul_multi(ctx, acts, j)
    torch.cuda.synchronize()
    # 48 launches captured in one CUDA graph (as the decode step runs them: no host launch cost
    # between kernels), replayed four times; the fastest of the last three replays counts
    reps = 48
    gs = torch.cuda.Stream()
    ctx.set_stream(gs)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for r in range(reps):
            rie.matmul_multi(ctx, acts, jobs[r % 12])
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(4):
        with torch.cuda.stream(gs):
            g0.record(gs)
            graph.replay()
            g1.record(gs)
        gs.synchronize()
        times.append(g0.elapsed_time(g1) / reps)
    gemv_ms = min(times[1:])
    del graph
    ctx.set_stream(stream)
    gemv_bytes = 16 * rie.GgmlType.Q4_K.row_bytes(spec.n_embd) * spec.n_ff_exp
    peak, peak_kind = peaks()
    achieved = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    wb = moe_bytes_per_token(spec)
    return {
        "metric": META["moe"]["metric"], "value": 1000.0 / ms, "unit": "tok/s", "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "dtype": META["moe"]["dtype"],
        "config": {"workload": META["moe"]["workload"], "layers": spec.n_layer, "hidden": spec.n_embd,
                   "experts": f"{spec.n_expert} x ffn {spec.n_ff_exp}, top-{spec.n_expert_used} softmax",
                   "heads": f"{spec.n_head}/{spec.n_head_kv}x{spec.head_dim}", "vocab": spec.n_vocab,
                   "prompt": MOE_PROMPT, "weight_bytes_per_token": wb, "b256_tok_s": b256_tps, "batch": 1,
                   "l2": "inputs larger than L2 (expert weights streamed per token)",
                   "parallelism": f"tp{world} attention, ep{world} experts (NCCL all-reduce)" if world > 1 else "tp1",
                   "decode": "CUDA graph replay per token", "model_build_s": t_build},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "traffic": profile_traffic("gemv_q4_k_moe_experts"),
                     "kernel": gemv_kernel_name("Q4_K", gemv_bytes) + " (8 experts' gate+up, 16 x 768 x 2048 Q4_K)",
                     "bytes_per_launch": gemv_bytes, "launch_ms": gemv_ms,
                     "timing": "48 launches over 12 sets of distinct weights (170 MB > L2) in one CUDA graph",
                     "whole_step_weight_gb_s": wb / (ms * 1e-3) / 1e9},
        "e2e": {"value": e2e_tps, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": spec.n_vocab * 4,
                "api": "CudaBackend.forward (rcu_backend_forward, host tokens/logits, greedy)"},
        # per token: 11 per layer (norm, QKV GEMV, attention with the q/k post-processing and KV
        # append, Wo GEMV, norm, router, top-k routing, experts' gate+up GEMV, GLU, experts' down
        # GEMV, weighted combine) + position, embedding, final norm, head GEMV
        "gpu_launches": args.steps * (11 * spec.n_layer + 4),
        "clocks": clk.summary(),
        "check": {"logits_finite": finite},
    }


def cpu_moe_sample(seconds: float, threads: int):
    """The oracle's restated CPU forward (moe_ffn, AVX2 tier, all host threads) decoding the
    same MoE shape after a 16-token prompt."""
    import oracle as O
    from rust_interference_engine_b200.model import synthetic_tensors
    spec = qwen3_moe_spec()
    gen = RandomBlocks(4)
    om = O.OracleModel(O.ModelConfig.from_buffer_copy(bytes(spec.config())))
    for name, t, rows, cols, data in synthetic_tensors(spec, gen.weight, gen.vec, gen.norm):
        om.set_tensor(name, int(t), rows, cols, data)
    ob = O.OracleBackend(om, 256, 16, kv_type=O.KV_F16, n_threads=threads)
    ob.forward(np.arange(16, dtype=np.uint32), 0)
    n, pos, t0 = 0, 16, time.perf_counter()
    tok = np.array([1], dtype=np.uint32)
    while True:
        out = ob.forward(tok, pos)
        tok = np.array([int(np.argmax(out[0]))], dtype=np.uint32)
        n, pos = n + 1, pos + 1
        el = time.perf_counter() - t0
        if el >= seconds or pos >= 255:
            break
    return {"value": n / el, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode steps of the 48-layer Qwen3-30B-A3B-shape MoE at context 16-{pos}, {el:.1f} s",
            "path": "avx2" if O.have_avx2() else "scalar"}


# ---- workload: config 5 turbo4 attention (Llama-3.1-70B shape, context 32768) ------------
T5 = dict(n_layer=80, n_head=64, n_head_kv=8, head_dim=128, ctx=32768)


def run_turbo(args, world, rank, local):
    """One decode token's attention over all 80 layers' turbo4 caches at context 32768. With
    N > 1 every rank holds 8/N KV heads (and their 64/N query heads) of every layer, as the
    tensor-parallel forward does: each rank reads 1/N of the KV bytes, no exchange."""
    import torch

    import oracle as O
    import rust_interference_engine_b200 as rie
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    ctx = rie.Context(local, stream)
    L, H, KV, hd, S = T5["n_layer"], T5["n_head"], T5["n_head_kv"], T5["head_dim"], T5["ctx"]
    if KV % world:
        raise SystemExit("KV heads must divide by the GPU count")
    kvl, hl = KV // world, H // world
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    caches = []
    t_fill = time.perf_counter()
    chunk = 4096
    for _ in range(L):  # K, V ~ N(0, 1), encoded by the library's turbo4 append (rotate + 4-bit codes)
        c = rie.LayerCache(ctx, rie.KvType.Turbo4, kvl, hd, S)
        for p0 in range(0, S, chunk):
            k = torch.randn(chunk, kvl * hd, device="cuda", generator=gen)
            v = torch.randn(chunk, kvl * hd, device="cuda", generator=gen)
            c.store(k, v, chunk, p0)
        caches.append(c)
    torch.cuda.synchronize()
    t_fill = time.perf_counter() - t_fill
    q = torch.randn(L, hl * hd, device="cuda", generator=gen)
    out = torch.zeros(L, hl * hd, device="cuda")
    pos = S - 1  # the last position: the whole window is read

    def step():
        for il in range(L):
            rie.attention(ctx, caches[il], q[il], 1, hl, pos, out[il])

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # parity spot check of layer 0 against the oracle's turbo4 attention on the same cache bytes
    kc, vc = caches[0].export()
    want = O.attention(q[0].cpu().numpy(), kc, vc, hl, kvl, hd, pos, S, O.KV_TURBO4, n_threads=16)
    got = out[0].cpu().numpy()
    max_rel = float(np.max(np.abs(got - want.reshape(-1))) / max(float(np.max(np.abs(want))), 1e-6))
    kern = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            kern[i][0].record(stream)
            step()
            kern[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = dist_max(t0.elapsed_time(t1) / args.steps, world)
    row = rie.turbo.row_bytes_4(hd)
    kv_bytes = L * 2 * kvl * S * row  # per rank per step
    # e2e through the public API: query from pinned host memory, output back to the host
    qh = q.cpu().pin_memory()
    oh = torch.empty_like(out, device="cpu").pin_memory()
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            torch.cuda.synchronize()
            e0 = time.perf_counter()
        q.copy_(qh, non_blocking=True)
        step()
        oh.copy_(out, non_blocking=True)
        stream.synchronize()
    e2e_s = (time.perf_counter() - e0) / args.steps
    e2e_s = dist_max(e2e_s, world)
    peak, peak_kind = peaks()
    achieved = kv_bytes / (ms * 1e-3) / 1e9
    return {
        "metric": META["turbo"]["metric"], "value": world * kv_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "dtype": META["turbo"]["dtype"],
        "config": {"workload": META["turbo"]["workload"], "layers": L, "heads": f"{H}/{KV}x{hd}", "context": S,
                   "kv_bytes_per_step": world * kv_bytes, "row_bytes": row, "tok_s": 1000.0 / ms,
                   "l2": f"inputs larger than L2 ({world * kv_bytes / 1e9:.2f} GB of turbo4 KV per step)",
                   "parallelism": f"tp{world} (KV heads split, no exchange)", "kv_fill_s": t_fill},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "traffic": profile_traffic("attn_turbo4_70b_ctx32k"),
                     "kernel": "k_attn_dec_t4<G=8> (80 launches per step)", "bytes_per_launch": kv_bytes // L,
                     "launch_ms": float(np.mean([a.elapsed_time(b) for a, b in kern])) / L},
        "e2e": {"value": world * kv_bytes / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(q.numel() * 4),
                "d2h_bytes_per_step": int(out.numel() * 4), "ms_per_step": e2e_s * 1e3},
        "gpu_launches": args.steps * L,
        "clocks": clk.summary(),
        "check": {"max_rel_err_vs_oracle": max_rel, "tolerance": 2e-3},
    }


def cpu_turbo_sample(seconds: float, threads: int):
    """The oracle's turbo4 attention (turbo.rs score/axpy, AVX2 tier, all host threads) over
    one layer's 8 KV heads at context 32768; GB/s of KV read."""
    import oracle as O
    H, KV, hd, S = T5["n_head"], T5["n_head_kv"], T5["head_dim"], T5["ctx"]
    rng = np.random.default_rng(7)
    row = O.kv_row_bytes(O.KV_TURBO4, hd)
    # random valid rows (f16 scale + codes), same bytes / work as encoded N(0, 1) rows
    kc = rng.integers(0, 256, (KV * S, row), dtype=np.uint8)
    vc = rng.integers(0, 256, (KV * S, row), dtype=np.uint8)
    sc = np.frombuffer(np.float16(0.02).tobytes(), dtype=np.uint8)
    for b in range((row - hd // 2) // 2):  # one f16 scale per rotation block, then the codes
        kc[:, 2 * b:2 * b + 2] = sc
        vc[:, 2 * b:2 * b + 2] = sc
    q = rng.standard_normal(H * hd).astype(np.float32)
    O.attention(q, kc, vc, H, KV, hd, S - 1, S, O.KV_TURBO4, n_threads=threads)
    n, t0 = 0, time.perf_counter()
    while True:
        O.attention(q, kc, vc, H, KV, hd, S - 1, S, O.KV_TURBO4, n_threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": n * 2 * KV * S * row / el / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} single-layer turbo4 attentions (64/8 heads x 128, context {S}), {el:.1f} s",
            "path": "avx2" if O.have_avx2() else "scalar"}


def cpu_decode_sample(seconds: float, threads: int):
    """The oracle's restated CPU forward (AVX2 tier, all host threads) decoding on the same
    model shape: a 16-token prompt, then single-token steps until `seconds` elapse."""
    import oracle as O
    from rust_interference_engine_b200.model import synthetic_tensors
    spec = qwen3_8b_spec()
    gen = RandomBlocks(3)
    om = O.OracleModel(O.ModelConfig.from_buffer_copy(bytes(spec.config())))
    for name, t, rows, cols, data in synthetic_tensors(spec, gen.weight, gen.vec, gen.norm):
        om.set_tensor(name, int(t), rows, cols, data)
    # decode at the GPU arm's context (after its 512-token prompt): a 16-token prompt fills the
    # first cache rows, the rows up to the prompt length stay zero (the same attention work; a
    # real 512-token CPU prefill would take about a minute)
    ob = O.OracleBackend(om, DEC_PROMPT + 256, 16, kv_type=O.KV_F16, n_threads=threads)
    ob.forward(np.arange(16, dtype=np.uint32), 0)
    n, pos, t0 = 0, DEC_PROMPT, time.perf_counter()
    tok = np.array([1], dtype=np.uint32)
    while True:
        out = ob.forward(tok, pos)
        tok = np.array([int(np.argmax(out[0]))], dtype=np.uint32)
        n, pos = n + 1, pos + 1
        el = time.perf_counter() - t0
        if el >= seconds or pos >= DEC_PROMPT + 255:
            break
    return {"value": n / el, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode steps of the 36-layer Qwen3-8B-shape Q4_K_M model at context {DEC_PROMPT}-{pos} "
                      f"(random weight blocks; the CPU time does not depend on the values), {el:.1f} s",
            "path": "avx2" if O.have_avx2() else "scalar"}


def cpu_prefill_sample(seconds: float, threads: int):
    """The oracle's AVX2 matmul (4-token tiles, RIE's chunking) on 64-token slices of config 2."""
    import oracle as O
    rng = np.random.default_rng(2)
    x = rng.standard_normal((64, PF_K)).astype(np.float32)
    w = O.quantize_weight(O.Q4_0, rng.normal(0.0, 0.02, (PF_N[1], PF_K)).astype(np.float32))
    O.matmul_multi(x, [(O.Q4_0, w, PF_K)], n_threads=threads)
    n, t0 = 0, time.perf_counter()
    while True:
        O.matmul_multi(x, [(O.Q4_0, w, PF_K)], n_threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    ops = n * 2 * 64 * PF_K * PF_N[1]
    return {"value": ops / el / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{n} matmuls of 64 tokens x 4096 x 4096 (Q4_0), {el:.1f} s",
            "path": "avx2" if O.have_avx2() else "scalar"}


# ---- workload: config 5 as a whole model: Llama-3.1-70B-shape decode, Q4_0, turbo4 KV ------
# (benchmark configuration 5 names hidden 8192, 80 layers, 64/8 heads x 128, context 32768, Q4_0 weight
# GEMVs tensor-parallel over 8 GPUs; FFN 28672 and vocabulary 128256 are the public
# Llama-3.1-70B values, RoPE base 500000, RMS eps 1e-5)
LLAMA70B = dict(arch="llama", n_vocab=128256, n_embd=8192, n_layer=80, n_head=64, n_head_kv=8, head_dim=128,
                n_ff=28672, rope_dim=128, rope_base=500000.0, rms_eps=1e-5)
L70_CTX = 32768


def llama70b_spec(n_layer=None):
    from rust_interference_engine_b200 import GgmlType as G
    from rust_interference_engine_b200.model import SyntheticSpec
    kw = dict(LLAMA70B)
    if n_layer is not None:
        kw["n_layer"] = n_layer
    return SyntheticSpec(wtype=G.Q4_0, embd_type=G.Q4_0, qk_norm=False, **kw)


def run_llama70b(args, world, rank, local):
    """Decode of one sequence through the whole 80-layer model at context 32768: N > 1 splits the
    model tensor-parallel (column-parallel q/k/v/gate/up, row-parallel o/down with an all-reduce,
    vocabulary-parallel head with an all-gather); each rank's turbo4 KV cache holds its 8/N KV
    heads, filled with K, V ~ N(0, 1) for the positions before the timed tokens."""
    import torch

    import rust_interference_engine_b200 as rie
    from rust_interference_engine_b200 import _check, _dptr, _lib
    from rust_interference_engine_b200 import model as M
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    ctx = rie.Context(local, stream)
    spec = llama70b_spec()
    gen = DeviceWeights(ctx, 5)  # same seed on every rank: every rank draws the same full tensors
    model = M.Model(ctx, spec.config(), rank, world)
    t_build = time.perf_counter()
    set_synthetic(model, spec, gen)
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t_build
    n_gen = max(args.warmup, 3) + args.steps
    fill = L70_CTX - n_gen
    be = M.CudaBackend(model, L70_CTX + n_gen, 8, rie.KvType.Turbo4, comm_id=tp_comm_id(world, rank))
    kvl, hd = spec.n_head_kv // world, spec.head_dim
    g = torch.Generator(device="cuda").manual_seed(77 + rank)
    t_fill = time.perf_counter()
    lib = _lib.load()
    for il in range(spec.n_layer):  # K, V ~ N(0, 1) through the library's turbo4 append
        kv = be.kv_cache(il)
        for p0 in range(0, fill, 4096):
            n = min(4096, fill - p0)
            k = torch.randn(n, kvl * hd, device="cuda", generator=g)
            v = torch.randn(n, kvl * hd, device="cuda", generator=g)
            _check(ctx.ptr, lib.rcu_kv_store(ctx.ptr, kv, _dptr(k), _dptr(v), n, p0))
    torch.cuda.synchronize()
    t_fill = time.perf_counter() - t_fill
    toks = torch.from_numpy(np.random.default_rng(6).integers(0, spec.n_vocab, 2 * n_gen).astype(np.int32)).cuda()
    logits = torch.zeros(spec.n_vocab, device="cuda")
    pos = fill
    for i in range(max(args.warmup, 3)):  # the second decode step captures the CUDA graph
        be.forward_device(toks[i:], 1, pos, logits)
        pos += 1
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0.record(stream)
        for i in range(args.steps):
            be.forward_device(toks[max(args.warmup, 3) + i:], 1, pos + i, logits)
        t1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = dist_max(t0.elapsed_time(t1) / args.steps, world)
    pos += args.steps
    finite = bool(torch.isfinite(logits).all())
    # e2e: the host API, token in and logits out through host memory
    tok = np.array([1], dtype=np.uint32)
    for i in range(max(args.warmup, 3)):
        be.forward(tok, pos)
        pos += 1
    barrier(world)
    e0 = time.perf_counter()
    n_e2e = max(1, min(args.steps, n_gen - max(args.warmup, 3)))
    for i in range(n_e2e):
        out = be.forward(tok, pos)
        tok = np.array([int(np.argmax(out[0]))], dtype=np.uint32)
        pos += 1
    e2e_s = dist_max((time.perf_counter() - e0) / n_e2e, world)
    # dominant kernel: this rank's gate+up GEMV (2 x 28672 / N x 8192 Q4_0), timed in a CUDA graph
    ff = spec.n_ff // world
    gu_bytes = [gen.weight(rie.GgmlType.Q4_0, ff, spec.n_embd) for _ in range(4)]
    gu = [rie.Weight.view(ctx, rie.GgmlType.Q4_0, ff, spec.n_embd, b) for b in gu_bytes]
    xg = torch.randn(1, spec.n_embd, device="cuda")
    acts = rie.QuantActs(ctx, 1, spec.n_embd)
    acts.prepare(xg, 1, spec.n_embd, rie.ActFormat.Q8_0)
    og = torch.zeros(2, ff, device="cuda")
    jobs = [[rie.MatmulJob(gu[2 * i], og[0]), rie.MatmulJob(gu[2 * i + 1], og[1])] for i in range(2)]
    ctx.set_static_weights(True)
    for j in jobs:
        rie.matmul_multi(ctx, acts, j)
    torch.cuda.synchronize()
    reps = 20
    gs = torch.cuda.Stream()
    ctx.set_stream(gs)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for r in range(reps):
            rie.matmul_multi(ctx, acts, jobs[r % 2])
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(4):
        with torch.cuda.stream(gs):
            ev0.record(gs)
            graph.replay()
            ev1.record(gs)
        gs.synchronize()
        times.append(ev0.elapsed_time(ev1) / reps)
    gemv_ms = min(times[1:])
    del graph
    ctx.set_stream(stream)
    be.free()
    gemv_bytes = 2 * rie.GgmlType.Q4_0.row_bytes(spec.n_embd) * ff
    peak, peak_kind = peaks()
    achieved = gemv_bytes / (gemv_ms * 1e-3) / 1e9
    wbytes = weight_bytes_per_token(spec) // world
    kv_bytes = spec.n_layer * 2 * kvl * (L70_CTX - n_gen // 2) * rie.turbo.row_bytes_4(hd)
    return {
        "metric": META["llama70b"]["metric"],
        "value": 1000.0 / ms,  # one sequence: N > 1 splits the model (tensor parallel), not the work
        "unit": "tok/s",
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "dtype": META["llama70b"]["dtype"],
        "config": {"workload": META["llama70b"]["workload"], "layers": spec.n_layer, "hidden": spec.n_embd,
                   "ffn": spec.n_ff, "heads": f"{spec.n_head}/{spec.n_head_kv}x{hd}", "vocab": spec.n_vocab,
                   "context_at_timing": L70_CTX - n_gen // 2, "kv": "turbo4", "batch": 1,
                   "weight_bytes_per_token_per_gpu": wbytes, "kv_bytes_per_token_per_gpu": kv_bytes,
                   "l2": f"inputs larger than L2 ({(wbytes + kv_bytes) / 1e9:.1f} GB streamed per token per GPU)",
                   "parallelism": f"tp{world} (all-reduce of Wo/down, all-gather of logits)" if world > 1 else "tp1",
                   "decode": "CUDA graph replay per token", "model_build_s": t_build, "kv_fill_s": t_fill},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind,
                     # ncu figure of the one-GPU launch (the tensor-parallel shards are 1/N of it)
                     "traffic": profile_traffic("gemv_kq_q4_0_gate_up_70b") if world == 1 else None,
                     "kernel": gemv_kernel_name("Q4_0", gemv_bytes) + f" (gate+up, 2 x {ff} x 8192 Q4_0, this rank's shard)",
                     "bytes_per_launch": gemv_bytes, "launch_ms": gemv_ms,
                     "timing": "20 launches over 2 distinct weight pairs in one CUDA graph",
                     "whole_step_gb_s_per_gpu": (wbytes + kv_bytes) / (ms * 1e-3) / 1e9},
        "e2e": {"value": 1.0 / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": spec.n_vocab * 4,
                "ms_per_step": 1e3 * e2e_s, "api": "CudaBackend.forward (rcu_backend_forward, host tokens/logits, greedy)"},
        # per token: 9 per layer (norm, QKV GEMV, q/k post-processing + turbo4 KV append, attention,
        # Wo GEMV, norm, gate+up GEMV, GLU, down GEMV); 8 when a rank holds one or two KV heads
        # (4 or 8 GPUs: the attention does the post-processing) + position, embedding, final
        # norm, head GEMV
        "gpu_launches": args.steps * ((8 if kvl <= 2 else 9) * spec.n_layer + 4),
        "clocks": clk.summary(),
        "check": {"logits_finite": finite},
    }


def cpu_llama70b_sample(seconds: float, threads: int):
    """The oracle's CPU forward (AVX2 tier, all host threads) at the 70B shape with a turbo4
    cache of 32768 positions, extrapolated from models of one and two of its layers (the head
    and embedding in both): tok/s = 1 / (t1 + 79 (t2 - t1)). The cache rows are zero (the
    same attention work as filled rows)."""
    import oracle as O
    from rust_interference_engine_b200.model import synthetic_tensors
    per = []
    for nl in (1, 2):
        spec = llama70b_spec(nl)
        gen = RandomBlocks(5)
        om = O.OracleModel(O.ModelConfig.from_buffer_copy(bytes(spec.config())))
        for name, t, rows, cols, data in synthetic_tensors(spec, gen.weight, gen.vec, gen.norm):
            om.set_tensor(name, int(t), rows, cols, data)
        ob = O.OracleBackend(om, L70_CTX + 64, 1, kv_type=O.KV_TURBO4, n_threads=threads)
        pos, tok = L70_CTX - 64, np.array([1], dtype=np.uint32)
        ob.forward(tok, pos)
        n, t0 = 0, time.perf_counter()
        while True:
            ob.forward(tok, pos + 1 + n)
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds / 2 or n >= 60:
                break
        per.append(el / n)
        del ob, om
    t_tok = per[0] + 79 * max(per[1] - per[0], 0.0)
    return {"value": 1.0 / t_tok, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"decode steps of 1- and 2-layer models of the 70B shape at context {L70_CTX - 63} "
                      f"({per[0] * 1e3:.0f} / {per[1] * 1e3:.0f} ms per token), extrapolated to 80 layers",
            "path": "avx2" if O.have_avx2() else "scalar"}


WORKLOADS = {"gemv": (run_gemv, cpu_gemv_sample), "prefill": (run_prefill, cpu_prefill_sample),
             "decode": (run_decode, cpu_decode_sample), "moe": (run_moe, cpu_moe_sample),
             "turbo": (run_turbo, cpu_turbo_sample), "llama70b": (run_llama70b, cpu_llama70b_sample)}
META = {  # metric / unit / config of each workload, shared by both arms
    "turbo": {"metric": "turbo4 KV attention HBM GB/s (config 5, Llama-3.1-70B shape, context 32768)", "unit": "GB/s",
              "dtype": "u4 codes x int8 query (rotated domain, byte-shuffle lookup), f32 softmax",
              "workload": "turbo4_attention_70b_ctx32768_config5"},
    "llama70b": {"metric": "Llama-3.1-70B-shape Q4_0 decode tg tok/s, turbo4 KV at context 32768 (config 5, batch 1)",
                 "unit": "tok/s", "dtype": "int8 x Q4_0 blocks (Q8_0 activations), turbo4 KV (u4 codes x int8 query), f32 glue",
                 "workload": "llama31_70b_q4_0_turbo4_decode_config5"},
    "moe": {"metric": "Qwen3-30B-A3B-shape MoE decode tg tok/s (config 4, batch 1)", "unit": "tok/s",
            "dtype": "int8 x Q4_K blocks (Q8_K activations), f32 router / glue, f16 KV",
            "workload": "qwen3_30b_a3b_moe_decode_config4"},
    "decode": {"metric": "Qwen3-8B-shape Q4_K_M decode tg tok/s (config 3, batch 1)", "unit": "tok/s",
               "dtype": "int8 x Q4_K/Q6_K blocks (Q8_K activations), f32 glue, f16 KV",
               "workload": "qwen3_8b_q4_k_m_decode_config3"},
    "gemv": {"metric": "quant-matmul HBM GB/s (Q4_0 x Q8_0 GEMV, config 1)", "unit": "GB/s",
             "dtype": "int8 (Q4_0 x Q8_0 blocks, f32 combine)", "workload": "gemv_q4_0_6144x2048_config1"},
    "prefill": prefill_meta("f16"),
}


def step_units(workload: str) -> float:
    """Units of a workload's metric in one step (one pass of the hot path over one batch): the
    reference arm reports ms_per_step = these units / its measured rate."""
    if workload in ("decode", "moe", "llama70b"):
        return 1.0  # one token
    if workload == "gemv":
        return gemv_bytes_per_step()[0] / 1e9
    if workload == "prefill":
        return 2.0 * PF_M * PF_K * sum(PF_N) / 1e12
    if workload == "turbo":  # K and V rows of every layer, turbo4 at head_dim 128 (66-byte rows)
        return 2.0 * T5["n_layer"] * T5["n_head_kv"] * T5["ctx"] * 66 / 1e9
    raise KeyError(workload)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--wtype", default="Q4_0", choices=sorted(BLOCK),
                    help="GGUF type of the gemv workload (config 1 is Q4_0)")
    ap.add_argument("--gemm", default="f16", choices=["f16", "i8"],
                    help="prefill workload: tensor-core GEMM kind (f16 dequantized operands, or exact int8 for Q4_0)")
    ap.add_argument("--batch", type=int, default=512, help="decode workload: prompt tokens per forward (n_batch)")
    ap.add_argument("--prompt", type=int, default=512, help="prompt length of the decode workload (config 3: 512)")
    ap.add_argument("--shape", default=None, help="gemv workload: ROWSxK weights, one launch each (e.g. 24576x4096)")
    args = ap.parse_args()
    global GEMV_TYPE, DEC_PROMPT, DEC_BATCH, GEMV_ROWS, GEMV_K, GEMV_COPIES, GEMV_EACH, GEMV_DISTINCT
    GEMV_TYPE = args.wtype
    if args.shape:
        GEMV_ROWS, GEMV_K = (int(v) for v in args.shape.lower().split("x"))
        bs, bb = BLOCK[GEMV_TYPE]
        GEMV_COPIES = max(GEMV_DISTINCT, -(-520_000_000 // (GEMV_ROWS * GEMV_K // bs * bb)))
        GEMV_DISTINCT = max(1, min(GEMV_DISTINCT, 800_000_000 // (GEMV_ROWS * GEMV_K * 4)))  # host f32 draft
        GEMV_EACH = True
    DEC_PROMPT = args.prompt
    DEC_BATCH = args.batch
    META["gemv"] = gemv_meta()
    META["prefill"] = prefill_meta(args.gemm)
    world, rank, local = dist_init()

    if args.impl == "reference":
        if rank == 0:
            threads = os.cpu_count() or 1
            samples = []
            cpu_fn = WORKLOADS[args.workload][1]
            for _ in range(args.warmup):
                cpu_fn(0.2, threads)
            for _ in range(args.steps):
                samples.append(cpu_fn(max(args.cpu_seconds / max(args.steps, 1), 0.5), threads))
            v = float(np.median([s["value"] for s in samples]))
            cb = dict(samples[0])
            cb["value"] = v
            cb["sample"] = f"{args.steps} samples of: " + cb["sample"]
            m = META[args.workload]
            print(json.dumps({"impl": "reference", "metric": m["metric"], "value": v, "unit": m["unit"],
                              "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": 1e3 * step_units(args.workload) / v,
                              "higher_is_better": True, "scaling": "weak", "dtype": m["dtype"], "data": "synthetic",
                              "config": {"workload": m["workload"]}, "vs_baseline": None, "cpu_baseline": cb,
                              "e2e": {"value": v, "unit": m["unit"], "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    run_fn, cpu_fn = WORKLOADS[args.workload]
    res = run_fn(args, world, rank, local)
    if rank == 0:
        res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "vs_baseline": None,
                    "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)"})
        if world == 1:
            res["cpu_baseline"] = cpu_fn(args.cpu_seconds, os.cpu_count() or 1)
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the B200 GGML quantized matmul (BASELINE.json metric:
"Q4_K GEMM TFLOP/s (M=256) & GEMV weight-GB/s (M=1), % of roofline, 1/2/4/8 GPU").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workload (config.workload "q4k_ffn_up_m256"): BASELINE config 1's projection (Q4_K weights,
K=2560 -> N=10240, 256-element super-blocks with the config's value distributions) at M=256 bf16
activation rows -- the size the metric is quoted at. One step is one pass over a stack of
L=36 distinct weight matrices (36 x 14.7 MB = 531 MB of weights, > 4x the 126 MB L2, so every
matrix streams from HBM), each product writing its own f32 output. Synthetic seeded data.

With N GPUs (one process per GPU): the projection is column-sharded -- every rank owns a
10240-column shard of an N*10240-wide column-parallel layer (per-GPU work fixed: weak scaling) --
and the outputs stay sharded, as a tensor-parallel MLP's column-parallel first projection leaves
them (no collective on the data path of `value`). The `allgather` sub-line times the same stack
with every layer's f32 output shard all-gathered over NVLink by jk_sharded_matmul_allgather (the
copy engines push it into every peer's buffer over CUDA IPC while the next layer's product runs;
one bounded flag wait per step). `vocab_head` is BASELINE config 4 strong-scaled over the N GPUs
(M=2048, K=2560, N=262144 split by column, f32 logits all-gathered), compute-only and end to end
against max(compute, NVLink) time.

Printed JSON (rank 0): `value` = aggregate TFLOP/s of the timed steps (inputs resident in HBM,
device-timed with CUDA events, max over ranks); `e2e` = the same metric through the public API with
pinned host buffers, one product per step (its activations host->device, the product, its whole
f32 output device->host); `roofline` = the tensor-core kernel's achieved TFLOP/s per launch vs the
measured bf16 burst peak; `f16` = the same stack with FP16 activations; `gemv` = the M=1
weight-streaming GB/s on the same matrices and `gemv_vocab` on config 4's 377 MB matrix;
`cpu_baseline` = the reference's CPU arithmetic (quant.rs dequant restated in C + a CPU f32
matmul) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(REPO, "jevons-rs_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

K_DIM, N_DIM, M_ROWS, LAYERS = 2560, 10240, 256, 36
VOCAB_N = 262144  # config 4's vocabulary: the head matrix [VOCAB_N, K_DIM]
VOCAB_M = 2048    # config 4's rows: 8 requests x 256-token blocks
VOCAB_CHUNKS = 8  # row chunks of the sharded head: chunk i's copies overlap chunk i+1's product
NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction per B200 on this pool
METRIC = "Q4_K GEMM TFLOP/s (M=256)"
WORKLOAD = "q4k_ffn_up_m256"
Q4_K = 12
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------------------------------------
# clocks during the timed region (NVML, the library nvidia-smi reads)
# ------------------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {  # nvmlClocksEventReason bits
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, torch_device: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            import torch
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            try:
                self.h = nv.nvmlDeviceGetHandleByUUID(uuid.encode() if isinstance(uuid, str) else uuid)
            except Exception:
                self.h = nv.nvmlDeviceGetHandleByIndex(torch_device)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self._ok = True
        except Exception as e:  # NVML missing: report that instead of clocks
            self.err = repr(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                try:
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for b, name in self.REASONS.items():
                    if bits & b and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._ok:
            self._stop.set()
            self._t.join()

    def report(self):
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "err", "nvml")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------
# CPU baseline: the reference's block dequant (restated in C, oracle/) + CPU f32 matmul
# ------------------------------------------------------------------------------------------------
def cpu_gemm_sample(raw: np.ndarray, x_f32: np.ndarray, n_cols: int):
    """Dequantizes the first n_cols weight rows (oracle) and multiplies with torch's CPU f32 matmul.
    Returns (seconds total, seconds of dequant)."""
    import torch
    from oracle import oracle
    row_bytes = K_DIM // 256 * 144
    t0 = time.perf_counter()
    w = oracle.dequantize(Q4_K, raw[: n_cols * row_bytes]).reshape(n_cols, K_DIM)
    t1 = time.perf_counter()
    out = torch.from_numpy(x_f32) @ torch.from_numpy(w).t()
    t2 = time.perf_counter()
    del out
    return t2 - t0, t1 - t0


def cpu_baseline(raw: np.ndarray, x_f32: np.ndarray, budget_s: float = 12.0):
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_cols = 2048
    cpu_gemm_sample(raw, x_f32, 256)  # warm-up (thread pools, page faults)
    runs, total, deq = 0, 0.0, 0.0
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < budget_s or runs < 3:
        a, b = cpu_gemm_sample(raw, x_f32, n_cols)
        total += a
        deq += b
        runs += 1
    flops = 2.0 * M_ROWS * n_cols * K_DIM * runs
    return {
        "value": flops / total / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
        "sample": f"{runs} x Q4_K [M={M_ROWS}, K={K_DIM}] x [{n_cols} of the {N_DIM} weight rows]: oracle dequant "
                  f"(quant.rs restated in C, OpenMP) + torch CPU f32 matmul; dequant share "
                  f"{deq / total:.0%}, without dequant {flops / max(total - deq, 1e-9) / 1e12:.3f} TFLOP/s",
        "cpu": _cpu_model(),
    }


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def run_reference(args):
    """--impl reference: the reference's CPU arithmetic for this path on the host cores.

    The reference (Rust / CubeCL / HIP) cannot be built here (no cargo/rustc, no network) and its
    kernels have no CPU implementation, so this arm times the restatement of its block dequant
    (oracle/jk_oracle.c, quant.rs:25-101) feeding a CPU f32 matmul -- the stand-in named in the
    baseline plan. Each step is a bounded sample of the same workload (2048 of the 10240 weight rows)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch
    from jevons_kernels import synth
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rng = np.random.default_rng(1)
    raw = synth.q4k_blocks(rng, N_DIM, K_DIM)
    x = synth.activations(np.random.default_rng(2), M_ROWS, K_DIM, round_to="bf16")
    n_cols = 2048
    for _ in range(max(args.warmup, 1)):
        cpu_gemm_sample(raw, x, n_cols)
    times = []
    for _ in range(args.steps):
        a, _ = cpu_gemm_sample(raw, x, n_cols)
        times.append(a)
    total = sum(times)
    value = 2.0 * M_ROWS * n_cols * K_DIM * len(times) / total / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "m": M_ROWS, "k": K_DIM, "n": N_DIM, "weights": "Q4_K",
                   "sample_weight_rows": n_cols},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"Q4_K [M={M_ROWS}, K={K_DIM}] x [{n_cols} weight rows] per step: oracle dequant "
                                   "(quant.rs restated in C) + torch CPU f32 matmul", "cpu": _cpu_model()},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
# Routed-expert workloads of the reference's grouped-product benchmark
# (benchmarks/cubecl/results-routed-loop-2026-09-21/README.md, "Method"): 128 experts of Q4_K
# gate/up weights, K=2816 -> N=1408, top-8 routes; "balanced" spreads every token's 8 routes so each
# expert gets tokens*8/128 rows, "skewed" sends all tokens to the same 8 experts.
G_EXPERTS, G_N, G_K, G_TOP = 128, 1408, 2816, 8
G_WORKLOADS = [("routed_balanced_128", 128, "balanced"), ("routed_skewed_128", 128, "skewed"),
               ("routed_balanced_512", 512, "balanced"), ("routed_skewed_512", 512, "skewed")]


def grouped_bench(gpu, dev, timed, pk):
    """Times grouping + grouped product per workload (the reference's timed region: grouping, job
    construction, compute and scatter), for a small set of plans, and reports the fastest."""
    import torch
    from jevons_kernels import synth
    from jevons_kernels.gemm import (Buf, Groups, QMatrix, SplitScratch, group_max_jobs, group_routes,
                                     matmul_grouped, matvec_grouped)
    raw = synth.q4k_blocks(np.random.default_rng(7), G_EXPERTS * G_N, G_K)
    w = QMatrix.upload(gpu, Q4_K, G_N, G_K, G_EXPERTS, raw)
    del raw
    expert_bytes = G_N * G_K // 256 * 144
    scratch = SplitScratch(gpu)
    results = {}
    for name, tokens, kind in G_WORKLOADS:
        a = tokens * G_TOP
        if kind == "balanced":
            ids = np.array([(G_TOP * t + j) % G_EXPERTS for t in range(tokens) for j in range(G_TOP)])
        else:
            ids = np.tile(np.arange(G_TOP), tokens)
        active = len(np.unique(ids))
        per_expert = a // active
        x = torch.from_numpy(synth.activations(np.random.default_rng(8), tokens, G_K)).to(dev).bfloat16()
        ids_t = torch.from_numpy(ids.astype(np.int32)).to(dev)
        out = torch.empty(a, G_N, device=dev)
        cands = [("gemm", bm, 128) for bm in (32, 64, 128, 256) if bm // 2 < per_expert or bm == 32]
        cands += [("gemm", bm, 256) for bm in (128, 256) if bm // 2 < per_expert]
        if per_expert <= 16:
            cands.append(("gemv", per_expert, 0))
        best = None
        tried = {}
        for kind_p, tile, bn in cands:
            mj = group_max_jobs(a, G_EXPERTS, tile)
            sorted_ = torch.empty(a, dtype=torch.int32, device=dev)
            offsets = torch.empty(G_EXPERTS + 1, dtype=torch.int32, device=dev)
            jobs = torch.empty(1 + 2 * mj, dtype=torch.int32, device=dev)
            g = Groups(Buf(sorted_), Buf(offsets), Buf(jobs), mj, G_TOP, a)

            def call(tile=tile, bn=bn, kind_p=kind_p, g=g, sorted_=sorted_, offsets=offsets, jobs=jobs):
                group_routes(gpu, Buf(ids_t), Buf(sorted_), Buf(offsets), Buf(jobs), a, G_EXPERTS, tile)
                if kind_p == "gemv":
                    matvec_grouped(gpu, Buf(x), w, g, Buf(out), tile)
                else:
                    matmul_grouped(gpu, Buf(x), w, g, Buf(out), tile, bn, 1, scratch)
            steps = 50
            ms = timed(call, steps, 3) / steps
            label = f"{kind_p} {'mr' if kind_p == 'gemv' else 'bm'}={tile}" + (f" bn={bn}" if bn else "")
            tried[label] = round(ms * 1e3, 2)
            if best is None or ms < best[0]:
                best = (ms, label)
        ms, label = best
        flops = 2.0 * a * G_N * G_K
        wb = active * expert_bytes
        results[name] = {"us": ms * 1e3, "plan": label, "tflops": flops / (ms * 1e-3) / 1e12,
                         "weight_gbs": wb / (ms * 1e-3) / 1e9, "frac_of_hbm": wb / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                         "rows": a, "active_experts": active, "candidates_us": tried}
    return {"what": "group_routes + grouped product per call (128 experts Q4_K [1408, 2816], top-8, bf16 x), "
                    "CUDA graph replay, CUDA events; weights of the active experts stream from HBM",
            "workloads": results}


# BASELINE config 3 (crates/jevons-parakeet/src/config.rs:183-186, encoder.rs:53-61): 24 encoder
# layers of Q8_0 linears at M=750 frames, d=1024: FFN 1024->4096->1024 and four 1024->1024
# attention projections; each linear gets its own seeded f32 N(0,1) input (not chained).
CFG3_M, CFG3_D, CFG3_FF, CFG3_LAYERS = 750, 1024, 4096, 24
CFG3_SHAPES = [(CFG3_FF, CFG3_D), (CFG3_D, CFG3_FF)] + [(CFG3_D, CFG3_D)] * 4  # (n, k) per linear


def int8_peak_tops(dev):
    """Dense int8 tensor peak measured here: torch._int_mm (cuBLASLt) on 8192^3, best of 10."""
    import torch
    a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b.t())
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b.t())
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2.0 * 8192 ** 3 / (best * 1e-3) / 1e12


def cfg3_bench(gpu, dev, timed, pk, scratch):
    """Config 3, one step = one pass over the 24 layers x 6 linears (144 products, 320 MB of Q8_0
    weights): the int8 path (jk_quantize_act_q8 + jk_matmul_q8_int8 per linear) and the bf16
    tensor-core path (jk_matmul on the f32 activations, rounded to bf16), CUDA graph replay."""
    import torch
    from jevons_kernels import synth
    from jevons_kernels.gemm import Buf, QMatrix, matmul, matmul_q8_int8, q8_scales_len, quantize_act_q8
    m = CFG3_M
    rng = np.random.default_rng(3)
    raws = {shape: synth.q8_0_blocks(rng, shape[0], shape[1]) for shape in set(CFG3_SHAPES)}
    ws = [QMatrix.upload(gpu, 8, n, k, 1, raws[(n, k)]) for _ in range(CFG3_LAYERS) for (n, k) in CFG3_SHAPES]
    xs = {k: torch.from_numpy(synth.activations(np.random.default_rng(30 + k), m, k)).to(dev) for k in (CFG3_D, CFG3_FF)}
    xq = {k: torch.empty(m * k, dtype=torch.int8, device=dev) for k in xs}
    xd = {k: torch.empty(q8_scales_len(m, k), device=dev) for k in xs}
    outs = [torch.empty(m, w_n, device=dev) for w_n in (CFG3_FF, CFG3_D)]
    lin = [(ws[i], CFG3_SHAPES[i % 6]) for i in range(len(ws))]

    def step_i8():
        for w, (n, k) in lin:
            quantize_act_q8(gpu, Buf(xs[k]), m, k, Buf(xq[k]), Buf(xd[k]))
            matmul_q8_int8(gpu, w, Buf(xq[k]), Buf(xd[k]), m, Buf(outs[0 if n == CFG3_FF else 1]))

    def step_bf16():
        for w, (n, k) in lin:
            matmul(gpu, Buf(xs[k]), m, w, Buf(outs[0 if n == CFG3_FF else 1]), None, scratch)
    steps = 10
    flops = sum(2.0 * m * n * k for _, (n, k) in lin)
    t_i8 = timed(step_i8, steps, 3) / steps
    t_bf = timed(step_bf16, steps, 3) / steps
    peak_i8 = int8_peak_tops(dev)
    v_i8, v_bf = flops / (t_i8 * 1e-3) / 1e12, flops / (t_bf * 1e-3) / 1e12
    return {"what": "BASELINE config 3: 24 x {1024->4096, 4096->1024, 4 x 1024->1024} Q8_0 linears at M=750, "
                    "f32 activations; one step = all 144 products; CUDA graph replay, CUDA events",
            "int8_path": {"ms_per_step": t_i8, "tops": v_i8, "peak_int8_tops": peak_i8, "frac_of_int8_peak": v_i8 / peak_i8,
                          "includes": "per-linear activation quantization + kind::i8 product"},
            "bf16_path": {"ms_per_step": t_bf, "tflops": v_bf, "peak_bf16_tflops": pk.get("bf16_tflops"),
                          "frac_of_bf16_peak": v_bf / pk.get("bf16_tflops", 1.0), "includes": "f32->bf16 conversion + product"},
            "faster": "int8" if t_i8 < t_bf else "bf16"}


HEAD_VOCAB = 262144  # token-table rows of the head workloads (the Gemma vocabulary)


def head_bench(gpu, dev, timed, pk, vocab: int = HEAD_VOCAB):
    """The Q6_K embedding-table operators on a [HEAD_VOCAB, K_DIM] table of synthetic Q6_K blocks:
    the dequantized f16 transpose of the whole table (HBM-bound: reads the 551 MB table, writes
    the 1.34 GB transpose), candidate logits for 16 rows x 256 candidates, and 512 embedding rows
    (canvas rows with self-conditioning input). CUDA graph replay, CUDA events."""
    import torch
    from jevons_kernels import head
    from jevons_kernels.formats import TensorType
    from jevons_kernels.gemm import Buf, QMatrix

    rng = np.random.default_rng(21)
    d = K_DIM
    nb = vocab * d // 256
    raw = np.empty((nb, 210), np.uint8)
    raw[:, :192] = rng.integers(0, 256, size=(nb, 192), dtype=np.uint8)
    raw[:, 192:208] = rng.integers(-99, 100, size=(nb, 16)).astype(np.int8).view(np.uint8)
    raw[:, 208:210] = (0.001 + rng.random(nb) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    table = QMatrix.upload(gpu, TensorType.Q6K, vocab, d, 1, raw.reshape(-1))
    del raw
    table_bytes = vocab * d // 256 * 210
    res = {}

    out_t = torch.empty(vocab * d, dtype=torch.float16, device=dev)
    tbuf = Buf(out_t)

    def transpose():
        head.q6k_transposed_f16(gpu, table, vocab, d, out=tbuf)
    steps = 20
    ms = timed(transpose, steps, 3) / steps
    alg = table_bytes + vocab * d * 2
    res["q6k_transpose_f16"] = {"us": ms * 1e3, "algorithmic_bytes": alg, "gbs": alg / (ms * 1e-3) / 1e9,
                                "frac_of_hbm": alg / (ms * 1e-3) / 1e9 / pk["hbm_gbs"]}
    del out_t, tbuf

    rows, cands, cap = 16, 256, 30.0
    x16 = torch.from_numpy(rng.uniform(-1, 1, (rows, d)).astype(np.float16)).to(dev)
    pairs_np = np.stack([np.repeat(np.arange(rows), cands), rng.integers(0, vocab, rows * cands)], 1)
    pairs = torch.from_numpy(pairs_np.astype(np.int32).reshape(-1)).to(dev)
    logits = torch.empty(rows * cands, device=dev)
    xb, pb, lb = Buf(x16), Buf(pairs), Buf(logits)

    def pick():
        head.pick(gpu, xb, pb, rows * cands, table, lb, cap, d)
    steps = 200
    ms = timed(pick, steps, 3) / steps
    rb = rows * cands * d // 256 * 210
    res["pick_logits"] = {"us": ms * 1e3, "pairs": rows * cands, "table_row_gbs": rb / (ms * 1e-3) / 1e9}

    n_tok, first = 512, 0
    toks = torch.from_numpy(rng.integers(0, vocab, n_tok).astype(np.int32)).to(dev)
    w_attn = torch.from_numpy(rng.uniform(-1, 1, d).astype(np.float32)).to(dev)
    cond = torch.from_numpy(rng.uniform(-1, 1, (n_tok, d)).astype(np.float32)).to(dev)
    eo = torch.empty(n_tok * d, device=dev)
    ex = torch.empty(n_tok * d, dtype=torch.float16, device=dev)
    tb_, wb_, cb_, eob, exb = Buf(toks), Buf(w_attn), Buf(cond), Buf(eo), Buf(ex)

    def embed():
        head.embed(gpu, tb_, table, wb_, cb_, eob, exb, n_tok, first, d, 1e-6)
    ms = timed(embed, steps, 3) / steps
    eb = n_tok * (d // 256 * 210 + d * 4 + d * 4 + d * 2)
    res["embed_q6k"] = {"us": ms * 1e3, "rows": n_tok, "gbs": eb / (ms * 1e-3) / 1e9}
    return {"what": f"Q6_K table [{vocab}, {d}] (synthetic blocks); CUDA graph replay, CUDA events; "
                    "transpose bytes = table read + f16 transpose written", "ops": res}


def run_head_only(args):
    """`--head-only`: the Q6_K table workloads alone (one GPU), for profiling them; prints the
    head object of the bench line."""
    import torch
    from jevons_kernels.gemm import Gpu

    gpu = Gpu(0)
    dev = torch.device("cuda", 0)
    graphs = []

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        graphs.append(g)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    pk, _ = peaks()
    print(json.dumps({"head": head_bench(gpu, dev, timed, pk, args.head_vocab)}), flush=True)
    graphs.clear()
    return 0


def run_ours(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    from jevons_kernels import synth
    from jevons_kernels.gemm import Buf, Gpu, Plan, QMatrix, SplitScratch, matmul, matvec
    from jevons_kernels.shard import PeerGather, column_shard

    gpu = Gpu(local)
    dev = torch.device("cuda", local)
    L = args.layers
    # this rank's shard of an (N_DIM * world)-column layer: N_DIM weight rows, seeded by shard
    lo, hi = column_shard(N_DIM * world, world, rank)
    assert hi - lo == N_DIM
    rng = np.random.default_rng(1 + 1000 * rank)
    raw = synth.q4k_blocks(rng, N_DIM, K_DIM)
    # L distinct device copies (distinct memory defeats L2 reuse across the stack)
    ws = [QMatrix.upload(gpu, Q4_K, N_DIM, K_DIM, 1, raw) for _ in range(L)]
    x = torch.from_numpy(synth.activations(np.random.default_rng(2), M_ROWS, K_DIM)).to(dev).bfloat16()
    outs = [torch.empty(M_ROWS, N_DIM, device=dev) for _ in range(L)]
    scratch = SplitScratch(gpu)
    plan = Plan.heuristic(ws[0], M_ROWS, False)
    launches_per_product = 1  # one tensor-core kernel per product (split-K combined in-kernel)
    xb = Buf(x)
    obufs = [Buf(o) for o in outs]

    # N > 1, `allgather` sub-line: every layer writes its own gathered [N, M, N_DIM] buffer; the
    # copies of layer i run beside the product of layer i+1, and the step ends with one wait.
    pg = PeerGather(gpu, M_ROWS, N_DIM, buffers=L) if world > 1 else None

    def step(xbuf=xb):
        for i in range(L):
            matmul(gpu, xbuf, M_ROWS, ws[i], obufs[i], None, scratch)

    def step_gathered():
        for i in range(L):
            pg.run(ws[i], x, i=i, wait=False, chunks=1, scratch=scratch)
        pg.wait()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    flops_step = 2.0 * M_ROWS * N_DIM * K_DIM * L  # per rank
    graphs = []

    def timed(fn, steps, warmup, use_graph=True):
        """Warm-up, then `steps` runs of fn timed with CUDA events on the current stream (max over
        ranks). fn is replayed from a CUDA graph (NCCL all-gathers included: every rank captures
        the same sequence after the warm-up created the communicator) so host launch overhead is
        not timed."""
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        run = fn
        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            graphs.append(g)
            run = g.replay
            run()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            run()
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b))

    # ---- value: device-resident inputs --------------------------------------------------------
    sampler = ClockSampler(local)
    with sampler:
        ms = timed(step, args.steps, args.warmup)
    value = flops_step * world * args.steps / (ms * 1e-3) / 1e12
    allgather = None
    if world > 1:
        ag_ms = timed(step_gathered, args.steps, args.warmup)
        allgather = {
            "what": "the same stack with every layer's f32 output shard all-gathered into every rank's "
                    "[N, M, N_DIM] buffer by the copy engines (jk_sharded_matmul_allgather), one bounded "
                    "flag wait per step; CUDA graph replay, CUDA events, max over ranks",
            "value": flops_step * world * args.steps / (ag_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "ms_per_step": ag_ms / args.steps,
            "gather_bytes_sent_per_gpu_per_step": L * (world - 1) * M_ROWS * N_DIM * 4}

    # ---- roofline: one product launch = one tensor-core kernel (stream-K combines split-K
    # partials in-kernel), so its average duration is the step time over the layers.
    per_launch_ms = ms / args.steps / L
    pk, pk_kind = peaks()
    # The timed region is steps x ~1 ms (tens of ms, not a seconds-long power-capped loop), so the
    # kernel is rated against the burst bf16 figure.
    peak = pk.get("bf16_tflops", pk.get("bf16_tflops_sustained"))
    achieved = 2.0 * M_ROWS * N_DIM * K_DIM / (per_launch_ms * 1e-3) / 1e12
    traffic = None
    try:
        with open(os.path.join(REPO, "profiles", "roofline_traffic.json")) as f:
            traffic = json.load(f).get("q4k_gemm_m256_bytes_per_launch")
    except Exception:
        pass

    # ---- GEMV M=1 weight streaming on the same stack ------------------------------------------
    x1 = torch.from_numpy(synth.activations(np.random.default_rng(3), 1, K_DIM)).to(dev).bfloat16()
    o1 = [torch.empty(1, N_DIM, device=dev) for _ in range(L)]
    x1b, o1b = Buf(x1), [Buf(o) for o in o1]
    gv_steps = max(args.steps, 20)

    def gemv_step():
        for i in range(L):
            matvec(gpu, x1b, 1, ws[i], o1b[i])
    gv_ms = timed(gemv_step, gv_steps, 3)
    wbytes = N_DIM * K_DIM // 256 * 144
    gemv_gbs = wbytes * L * gv_steps * world / (gv_ms * 1e-3) / 1e9
    alg_bytes = wbytes + K_DIM * 2 + N_DIM * 4

    # ---- config 1 proper (M=32) ------------------------------------------------------------
    x32 = torch.from_numpy(synth.activations(np.random.default_rng(4), 32, K_DIM)).to(dev).bfloat16()
    o32 = [torch.empty(32, N_DIM, device=dev) for _ in range(L)]
    x32b, o32b = Buf(x32), [Buf(o) for o in o32]

    def m32_step():
        for i in range(L):
            matmul(gpu, x32b, 32, ws[i], o32b[i], None, scratch)
    c_ms = timed(m32_step, gv_steps, 3)
    m32_tflops = 2.0 * 32 * N_DIM * K_DIM * L * gv_steps * world / (c_ms * 1e-3) / 1e12

    # ---- e2e: host buffers through the public API -------------------------------------------
    # One step = one product as a caller serving it runs it: the step's activations host->device
    # from pinned memory, the product (jk_matmul), and its whole f32 output device->host. Steps
    # rotate over the L distinct matrices, so the weights stream from HBM as in the device-timed
    # step. On one GPU two steps are in flight on two streams (double-buffered host and device
    # buffers): step i+1's upload and product overlap step i's download, as a server pipelines
    # requests; each step still moves its own inputs and result. With N GPUs every rank runs the
    # same on its column shard (its result: its [M, N_DIM] shard of the output).
    nbuf = 2
    streams = [torch.cuda.Stream(device=dev) for _ in range(nbuf)]
    xhs = [x.cpu().pin_memory() for _ in range(nbuf)]
    ohs = [torch.empty(M_ROWS, N_DIM, dtype=torch.float32).pin_memory() for _ in range(nbuf)]
    xds = [torch.empty_like(x) for _ in range(nbuf)]
    # each in-flight step owns its device output and split-K scratch
    ods = [torch.empty(M_ROWS, N_DIM, device=dev) for _ in range(nbuf)]
    scrs = [scratch] + [SplitScratch(gpu) for _ in range(nbuf - 1)]
    e2e_state = {"i": 0}

    def e2e_product():
        i = e2e_state["i"]
        e2e_state["i"] = i + 1
        b, layer = i % nbuf, i % L
        with torch.cuda.stream(streams[b]):
            xds[b].copy_(xhs[b], non_blocking=True)
            matmul(gpu, Buf(xds[b]), M_ROWS, ws[layer], Buf(ods[b]), None, scrs[b])
            ohs[b].copy_(ods[b], non_blocking=True)

    def e2e_timed(steps, warmup):
        cur = torch.cuda.current_stream()
        for _ in range(warmup):
            e2e_product()
        torch.cuda.synchronize()
        barrier()
        a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(cur)
        for st in streams:
            st.wait_stream(cur)
        for _ in range(steps):
            e2e_product()
        for st in streams:
            cur.wait_stream(st)
        e.record(cur)
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(e))

    e_steps = max(args.steps, 2 * L)
    e_ms = e2e_timed(e_steps, args.warmup)
    e2e_value = 2.0 * M_ROWS * N_DIM * K_DIM * world * e_steps / (e_ms * 1e-3) / 1e12
    e2e_d2h = ohs[0].numel() * 4
    xh = xhs[0]

    # ---- the same stack at the reference's operand precision (FP16 activations) -------------
    x16 = x.float().half()
    x16b = Buf(x16)

    def step16():
        for i in range(L):
            matmul(gpu, x16b, M_ROWS, ws[i], obufs[i], None, scratch)
    f16_ms = timed(step16, args.steps, args.warmup)
    f16_tflops = flops_step * world * args.steps / (f16_ms * 1e-3) / 1e12

    # ---- config 4's matrix: the vocabulary head, Q4_K [262144, 2560] --------------------------
    # Every rank draws only its column shard (seeded by rank: the same value distributions, without
    # each of N ranks generating the whole 377 MB matrix).
    gv4 = vocab = None
    if not args.no_vocab:
        v_lo, v_hi = column_shard(VOCAB_N, world, rank)
        n_r = v_hi - v_lo
        raw4 = synth.q4k_blocks(np.random.default_rng(40 + 1000 * rank), n_r, K_DIM)
        w4 = QMatrix.upload(gpu, Q4_K, n_r, K_DIM, 1, raw4)
        del raw4
        if world == 1:  # M=1 product over the whole 377 MB matrix (larger than L2)
            o4 = torch.empty(1, VOCAB_N, device=dev)
            o4b = Buf(o4)

            def gemv4():
                matvec(gpu, x1b, 1, w4, o4b)
            g4_steps = 20
            g4_ms = timed(gemv4, g4_steps, 3)
            wb4 = VOCAB_N * K_DIM // 256 * 144
            gv4 = {"metric": "Q4_K GEMV weight-GB/s (M=1, K=2560, N=262144: config 4's matrix, 377 MB > L2)",
                   "value": wb4 * g4_steps / (g4_ms * 1e-3) / 1e9, "unit": "GB/s",
                   "frac_of_hbm": wb4 * g4_steps / (g4_ms * 1e-3) / 1e9 / pk.get("hbm_gbs", 1.0),
                   "us_per_product": g4_ms / g4_steps * 1e3}
        # M=2048 head, strong-scaled: compute-only, then product + all-gather of the f32 logits
        mv = VOCAB_M
        xv = torch.from_numpy(synth.activations(np.random.default_rng(44), mv, K_DIM)).to(dev).bfloat16()
        ov = torch.empty(mv, n_r, device=dev)
        xvb, ovb = Buf(xv), Buf(ov)
        v_steps = 5

        def head_compute():
            matmul(gpu, xvb, mv, w4, ovb, None, scratch)
        hc_ms = timed(head_compute, v_steps, 3) / v_steps
        flops_v = 2.0 * mv * VOCAB_N * K_DIM
        vplan = Plan.heuristic(w4, mv, False)
        e_v_ms = hc_ms
        if world > 1:
            del ov, ovb
            pgv = PeerGather(gpu, mv, n_r, buffers=1)

            def head_e2e():
                pgv.run(w4, xv, i=0, wait=True, chunks=VOCAB_CHUNKS, scratch=scratch)
            e_v_ms = timed(head_e2e, v_steps, 2) / v_steps
        gather_bytes = (world - 1) * mv * n_r * 4  # each GPU sends its shard to every peer (and receives as much)
        t_comp = flops_v / world / (pk.get("bf16_tflops", 1.0) * 1e12) * 1e3
        t_link = gather_bytes / (NVLINK_GBS * 1e9) * 1e3
        vocab = {"what": "BASELINE config 4: Q4_K vocab head M=2048 x K=2560 -> N=262144, column-split over "
                         f"{world} GPU(s), f32 logits all-gathered by copy engines (jk_sharded_matmul_allgather, "
                         f"{VOCAB_CHUNKS} row chunks); CUDA graph replay, CUDA events, max over ranks",
                 "plan": repr(vplan), "n_per_gpu": n_r,
                 "compute_ms": hc_ms, "compute_tflops_total": flops_v / (hc_ms * 1e-3) / 1e12,
                 "e2e_ms": e_v_ms, "e2e_tflops_total": flops_v / (e_v_ms * 1e-3) / 1e12,
                 "gather_bytes_sent_per_gpu": gather_bytes,
                 "roofline": {"compute_ms": t_comp, "nvlink_ms": t_link, "bound": "nvlink" if t_link > t_comp else "tensor",
                              "frac": max(t_comp, t_link) / e_v_ms, "nvlink_gbs": NVLINK_GBS,
                              "peak_tflops": pk.get("bf16_tflops")}}
        del w4

    # ---- Parakeet encoder linears on Q8_0, int8 path and bf16 path ---------
    cfg3 = None
    if world == 1 and not args.no_cfg3:
        cfg3 = cfg3_bench(gpu, dev, timed, pk, scratch)

    # ---- expert-grouped products (the reference's routed workloads), one GPU only -------------
    grouped = None
    if world == 1 and not args.no_grouped:
        grouped = grouped_bench(gpu, dev, timed, pk)
    head_ops = None
    if world == 1 and not args.no_head:
        head_ops = head_bench(gpu, dev, timed, pk)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        x_f32 = x.float().cpu().numpy()
        cpu = cpu_baseline(raw, x_f32)

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "weights": "Q4_K", "m": M_ROWS, "k": K_DIM, "n_per_gpu": N_DIM,
                       "n_total": N_DIM * world, "layers_per_step": L, "plan": repr(plan),
                       "l2": "inputs larger than L2: 36 distinct weight matrices (531 MB) per step",
                       "parallelism": f"column-shard x{world}" + (" (outputs stay sharded; the allgather sub-line gathers them)" if world > 1 else ""),
                       "activations": "bf16 N(0,1)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": f"gemm_tc_kernel<Q4_K,bf16,{plan.bm}>",
                         "per_launch_ms": per_launch_ms,
                         "peak_source": f"{pk_kind} bf16_tflops (burst: the timed region is {ms:.0f} ms)"},
            "gemv": {"metric": "Q4_K GEMV weight-GB/s (M=1)", "value": gemv_gbs, "unit": "GB/s",
                     "peak_hbm_gbs": pk.get("hbm_gbs"), "frac_of_hbm": gemv_gbs / pk.get("hbm_gbs", 1.0),
                     "algorithmic_gbs": gemv_gbs * alg_bytes / wbytes, "ms_per_product": gv_ms / gv_steps / L},
            "m32": {"metric": "Q4_K GEMM TFLOP/s (M=32, BASELINE config 1)", "value": m32_tflops, "unit": "TFLOP/s",
                    "weight_gbs": wbytes * L * gv_steps * world / (c_ms * 1e-3) / 1e9},
            "grouped": grouped,
            "head": head_ops,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": xh.numel() * 2,
                    "d2h_bytes_per_step": e2e_d2h, "steps": e_steps,
                    "what": "per step: x host->device (pinned), one jk_matmul product, its whole f32 output "
                            "device->host; steps rotate over the distinct matrices; two steps in flight on "
                            "two streams (double buffers); with N GPUs every rank on its column shard; "
                            "CUDA events, max over ranks"},
            "f16": {"metric": "Q4_K GEMM TFLOP/s (M=256), FP16 activations (the reference's operand type)",
                    "value": f16_tflops, "unit": "TFLOP/s", "ms_per_step": f16_ms / args.steps},
            "gemv_vocab": gv4,
            "vocab_head": vocab,
            "cfg3_parakeet_q8_0": cfg3,
            "allgather": allgather,
            # per step: one tensor-core kernel per layer
            "gpu_launches": args.steps * L * launches_per_product,
            "timing": "CUDA graph replay of each step, CUDA events, max over ranks",
            "clocks": sampler.report(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    graphs.clear()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-grouped", action="store_true", help="skip the expert-grouped workloads")
    ap.add_argument("--no-head", action="store_true", help="skip the Q6_K embedding-table workloads")
    ap.add_argument("--no-vocab", action="store_true", help="skip config 4's head (M=1 and M=2048, sharded)")
    ap.add_argument("--no-cfg3", action="store_true", help="skip config 3 (Q8_0 Parakeet linears, int8 and bf16 paths)")
    ap.add_argument("--head-only", action="store_true", help="run only the Q6_K embedding-table workloads")
    ap.add_argument("--head-vocab", type=int, default=HEAD_VOCAB, help="table rows of the head workloads")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.head_only:
        return run_head_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

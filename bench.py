#!/usr/bin/env python3
"""Benchmark of the quantized-matmul hot path on B200 (the driver's bench contract).

Default workload (N=1): BASELINE.json configs[1] -- Q4_K weights in the Qwen3-8B-like projection shapes
(K=4096: N=4096 q/o, N=1024 k/v, N=24576 fused gate+up; down K=12288, N=4096), bf16 activations. One STEP is one decode
token (M=1) through the six projections of a stack of `--layers` distinct weight copies (rotated so the weights,
868 MB at 8 layers, exceed the 126 MB L2), on the reference's default decode numerics: per layer each of the two
activation rows is quantised to int8 once (g_quant_q8, lk_quant_q8) and the six matvecs contract those codes with the
weight codes. `value` is the decode GEMV weight GB/s; the line also carries the same step with the quantisation folded
into every matvec's prologue (`decode_fused`), each decode launch form timed alone (`decode_gemv`: q|k|v, o, gate_up,
down and
configs[0]'s Q4_0 4096 x 4096 GEMV, each streamed from HBM), the bf16-activation decode, the prefill TFLOP/s at M=2048
over the same shapes
(step = row scale + the six tcgen05 GEMMs), a sweep over M in {1, 8, 64, 512, 2048}, the sharded IQ4_NL GEMMs and the
MoE layers. Each step is one CUDA-graph replay of the public ops' launches (16 quantisations and 32 matvec launches
per decode step -- q | k | v share one launch; the kernels chain with programmatic dependent launch).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--layers L]

--gpus N > 1 runs under torchrun, one rank per GPU, each rank with its own replica of the workload (weak scaling;
the decode step has no exchange); the sharded IQ4_NL GEMMs of configs[4] split their output columns over the ranks
and all-gather them (strong scaling). --impl reference times the reference's CPU path (gguf's dequantize + a float64
numpy matvec, as make_kernel_tests.py builds its references) on the same metric.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode GEMV weight GB/s (% HBM peak); prefill TFLOPS (% tensor peak)"
SHAPES = [("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096), ("gate_up", 4096, 24576),
          ("down", 12288, 4096)]   # (name, K, N)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum of one ncu-captured launch (`--profile-case mv_gate_up` /
# `gemm_gate_up`) divided by its algorithmic bytes: decode 56.666 MB / 56.727 MB; prefill 226.7 MB / 274.7 MB (output
# lines still in L2 at kernel exit are not counted). The bench scales them to its average launch, since traffic
# grows in proportion to the bytes a launch streams.
TRAFFIC_RATIO_DECODE = 56.666 / 56.727
TRAFFIC_RATIO_PREFILL = 226.7 / 274.7


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return FALLBACK_PEAKS, "fallback"


def rank_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


# ------------------------------------------------------------------------------------------------------------------
# clocks during the timed region
# ------------------------------------------------------------------------------------------------------------------
class Clocks:
    Q = ("timestamp,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.out = os.path.join("/tmp", f"lk_clocks_{os.getpid()}.csv")
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=open(self.out, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)   # the sampler's first query takes a moment

    def mark(self, begin):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in open(self.out):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9 and f[1] == self.uuid:
                try:
                    ts = time.mktime(time.strptime(f[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                except ValueError:
                    ts = None
                rows.append((ts, f))
        os.unlink(self.out)
        inside = [f for ts, f in rows if ts is not None and self.t0 - 1 <= ts <= self.t1 + 1] or [f for _, f in rows]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[2]) for r in inside if r[2].replace(".", "").isdigit()]
        mx = max(float(r[3]) for r in inside if r[3].replace(".", "").isdigit())
        reasons = sorted({self.NAMES[i] for r in inside for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(inside), "timed_s": round(self.t1 - self.t0, 3)}


# ------------------------------------------------------------------------------------------------------------------
# inputs: Q4_K blocks synthesised from a seed (timing does not depend on the values; parity is tested on quantised
# weights): f16 d and dmin of the size N(0, 0.02) weights get, uniform 6-bit scale/min fields and nibbles
# ------------------------------------------------------------------------------------------------------------------
Q4K_D = np.frombuffer(np.float16(5.2e-5).tobytes() * 2, np.uint8)   # d, dmin


def synth_q4k(rng, rows, k):
    w = rng.integers(0, 256, (rows, k // 256, 144), dtype=np.uint8)
    w[:, :, 0:4] = Q4K_D
    return w.reshape(rows, -1)


def synth_q6k(rng, rows, k):
    """Q6_K blocks (210 bytes per 256 values): uniform 6-bit codes and int8 sub-block scales, f16 d at byte 208."""
    b = rng.integers(0, 256, (rows * k // 256, 210), dtype=np.uint8)
    b[:, 208:210] = np.frombuffer(np.float16(2e-4).tobytes(), np.uint8)
    return b.reshape(rows, -1)


# ------------------------------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference's own CPU path for the decode matvec -- gguf's dequantize (the
# reference's pinned third-party dequantiser, gguf 0.19.0) and a float64 numpy matvec, as make_kernel_tests.py:45-47,
# 231-238 builds its references; the oracle port stands in only if gguf is missing
# ------------------------------------------------------------------------------------------------------------------
def cpu_decode_gbs(budget_s=10.0, rows=1024):
    """Dequantise + float64 matvec of a `rows`-row slice of the gate_up projection, repeated for ~budget_s seconds."""
    k = 4096
    rng = np.random.default_rng(1)
    w = synth_q4k(rng, rows, k)
    x = rng.standard_normal((1, k)).astype(np.float32)
    try:
        import gguf
        from gguf import GGMLQuantizationType

        def step():
            W = gguf.quants.dequantize(w, GGMLQuantizationType.Q4_K).reshape(rows, k)
            return x.astype(np.float64) @ W.T.astype(np.float64)
        kind, what = "reference", f"gguf {getattr(gguf, '__version__', '0.19.0')} dequantize + float64 numpy matvec"
    except ImportError:
        from oracle import qmm_oracle as O

        def step():
            return O.mv_ref("q4_k", w, x, rows, k)
        kind, what = "port", "oracle restatement (numpy dequant + float64 matvec)"
    t0 = time.perf_counter()
    reps = 0
    while True:
        step()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 100000:
            break
    gbs = reps * w.nbytes / el / 1e9
    return gbs, {"kind": kind, "cores": os.cpu_count(),
                 "sample": f"Q4_K {rows}x{k} slice of gate_up: {what} (BLAS threads = all host cores), "
                           f"{reps} reps in {el:.1f} s"}


def run_reference(args):
    rank, _, world = rank_env()
    if rank != 0:
        return
    # each step: a bounded sample of the decode workload on the host cores (~0.5 s)
    vals = []
    t_all = time.perf_counter()
    for i in range(args.warmup + min(args.steps, 20)):
        v, desc = cpu_decode_gbs(budget_s=0.5)
        if i >= args.warmup:
            vals.append(v)
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": len(vals), "warmup": args.warmup,
            "ms_per_step": round((time.perf_counter() - t_all) * 1e3 / (len(vals) + args.warmup), 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "configs[1] Qwen3-8B-like Q4_K projections, decode M=1 (CPU: gate_up slice)"},
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", **desc},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------------------------
def make_weights(torch, layers, seed=0):
    """Q4_K weights for one layer, copied to `layers` distinct buffers (rotated so they exceed L2). q, k and v are
    row slices of one contiguous "qkv" tensor, the fused attn_qkv layout the reference also loads (gen_llm.py:99-100):
    the decode reads them as three weights of one launch, the prefill as one N = 6144 GEMM."""
    rng = np.random.default_rng(seed)
    base = {name: torch.from_numpy(synth_q4k(rng, n, k)).cuda() for name, k, n in SHAPES if name not in ("q", "k", "v")}
    base["qkv"] = torch.from_numpy(synth_q4k(rng, 6144, 4096)).cuda()
    out = []
    for li in range(layers):
        w = {name: (t if li == 0 else t.clone()) for name, t in base.items()}
        w["q"], w["k"], w["v"] = w["qkv"][:4096], w["qkv"][4096:5120], w["qkv"][5120:]
        out.append(w)
    return out


def bench_gemv_forms(args, torch, wstack, xs, pk, time_steps):
    """Each decode launch form alone: 32 back-to-back launches per graph replay, rotated over enough copies of its
    weights to exceed twice the L2, so every launch streams its weights from HBM. Per launch: device time, weight
    GB/s and the fraction of the measured HBM copy. The four Q4_K forms of the step on int8 codes (and, beside them,
    the form that quantises its activation row in its own prologue), and configs[0]'s Q4_0 4096 x 4096 GEMV (the
    reference's CPU-runnable case) both at its stated precision
    -- fp16 activations through lk_mv, the reference's default f32-dot numerics for Q4_0 (formats.py:24-27) -- and on
    int8 activations."""
    from loom_skills_b200 import ops
    gen = torch.Generator(device=wstack[0]["o"].device)
    gen.manual_seed(7)
    q40 = synth_blocks(torch, wstack[0]["o"].device, 4096, 4096, "q4_0", gen)
    # Q4_K_M keeps ffn_down (half the layers) and attn_v in Q6_K: the down projection's shape in Q6_K
    q6d = torch.from_numpy(synth_q6k(np.random.default_rng(8), 4096, 12288)).to(wstack[0]["o"].device)
    x16 = xs[4096].to(torch.float16)
    forms = [("q|k|v", wstack[0]["qkv"], "q4_k", 4096, [4096, 1024, 1024], "int8"),
             ("o", wstack[0]["o"], "q4_k", 4096, [4096], "int8"),
             ("gate_up", wstack[0]["gate_up"], "q4_k", 4096, [24576], "int8"),
             ("down", wstack[0]["down"], "q4_k", 12288, [4096], "int8"),
             ("q4_0 4096x4096 fp16 (configs[0])", q40, "q4_0", 4096, [4096], "fp16"),
             ("q4_0 4096x4096 int8 (configs[0])", q40, "q4_0", 4096, [4096], "int8"),
             ("down q6_k (Q4_K_M)", q6d, "q6_k", 12288, [4096], "int8")]
    chain = 32
    out = {}
    xq = {k: ops.quant_q8(xs[k]) for k in xs}
    for label, base, fmt, k, ns, acts in forms:
        nbytes = base.numel()
        copies = max(2, -(-256_000_000 // nbytes))
        ws = [base] + [base.clone() for _ in range(copies - 1)]
        ys = [torch.empty(1, n, device=base.device) for n in ns]
        r0 = np.cumsum([0] + ns)
        x = xs[k]

        def body(fused=False):
            for i in range(chain):
                w = ws[i % copies]
                parts = [w[r0[j]:r0[j + 1]] for j in range(len(ns))]
                if acts == "fp16":
                    ops.mv(fmt, w, x16, ns[0], k, y=ys[0])
                elif fused:
                    ops.mv_q8_fused_multi(fmt, parts, x, ns, k, ys=ys)
                else:
                    ops.mv_q8_multi(fmt, parts, xq[k], ns, k, 1, ys=ys)

        def timed(fused):
            g = Timed(torch, lambda: body(fused))
            for _ in range(max(3, args.warmup)):
                g.replay()
            return time_steps(g.replay, max(5, args.steps)) * 1e3 / chain
        us = timed(False)
        gbs = nbytes / (us * 1e-6) / 1e9
        out[label] = {"format": fmt, "activations": acts, "us_per_launch": round(us, 2),
                      "weight_mb": round(nbytes / 1e6, 1), "weight_gbs": round(gbs, 1),
                      "hbm_frac": round(gbs / pk["hbm_gbs"], 4), "weight_copies": copies,
                      "kernel": "k_mv (lk_mv.cu)" if acts == "fp16" else
                                "k_mv_q8_rows on lk_quant_q8 codes" if fmt in ("q4_0", "q4_k") else
                                "k_mvq8g on lk_quant_q8 codes (lk_mvq8g.cu)"}
        if acts == "int8" and fmt in ("q4_0", "q4_k"):
            out[label]["fused_us_per_launch"] = round(timed(True), 2)   # the row quantised in the prologue
        del ws
    return out


def bench_pairs(args, torch, dev, time_steps):
    """Gate and up in two formats (Q4_K_M's Q4_K gate + Q6_K up; LK_FMT_PAIR) on a Qwen3-8B-like FFN, K=4096
    N=12288 each: the one-token decode (bf16 x) as one pair launch and as the reference's dense fallback -- two
    projections + g_silu_mul (gen_llm.py:6280-6283) -- over weights rotated past L2; and the prefill swiglu GEMM at
    M=2048 as one pair launch, beside two store GEMMs + silu_mul and the one-format Q4_K swiglu GEMM."""
    from loom_skills_b200 import ops
    rng = np.random.default_rng(11)
    k, n, m = 4096, 12288, 2048
    wg = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
    wu = torch.from_numpy(synth_q6k(rng, n, k)).to(dev)
    nbytes = wg.numel() + wu.numel()
    copies = max(2, -(-256_000_000 // nbytes))
    ws = [(wg, wu)] + [(wg.clone(), wu.clone()) for _ in range(copies - 1)]
    x = torch.randn(1, k, device=dev).to(torch.bfloat16)
    y, yu = torch.empty(1, n, device=dev), torch.empty(1, n, device=dev)
    chain = 16

    def mv_pair():
        for i in range(chain):
            g, u = ws[i % copies]
            ops.mv("q4_k+q6_k", g, x, n, k, w2=u, y=y)

    def mv_two():
        for i in range(chain):
            g, u = ws[i % copies]
            ops.mv("q4_k", g, x, n, k, y=y)
            ops.mv("q6_k", u, x, n, k, y=yu)
            ops.silu_mul(y, yu)

    xq = ops.quant_q8(x)

    def mv_q8_two():   # the reference's default decode of a mixed layer: two int8 projections + g_silu_mul
        for i in range(chain):
            g, u = ws[i % copies]
            ops.mv_q8("q4_k", g, xq, n, k, 1, y=y)
            ops.mv_q8("q6_k", u, xq, n, k, 1, y=yu)
            ops.silu_mul(y, yu)

    def timed(body, steps, per):
        g = Timed(torch, body)
        for _ in range(max(3, args.warmup)):
            g.replay()
        return time_steps(g.replay, steps) / per

    out = {"shape": {"k": k, "n": n, "gate": "q4_k", "up": "q6_k", "weight_mb": round(nbytes / 1e6, 1)}}
    steps = max(5, min(args.steps, 200))
    us_pair = timed(mv_pair, steps, chain) * 1e3
    us_two = timed(mv_two, steps, chain) * 1e3
    us_q8 = timed(mv_q8_two, steps, chain) * 1e3
    out["decode"] = {"pair_us": round(us_pair, 2), "pair_weight_gbs": round(nbytes / (us_pair * 1e-6) / 1e9, 1),
                     "two_projections_silu_mul_us": round(us_two, 2),
                     "int8_two_projections_silu_mul_us": round(us_q8, 2),
                     "int8_weight_gbs": round(nbytes / (us_q8 * 1e-6) / 1e9, 1), "weight_copies": copies,
                     "kernel": "k_mvs<kFmtPair> (lk_mv with LK_FMT_PAIR, bf16 x); int8: k_mv_q8_rows<Q4_K> + "
                               "k_mvq8g<Q6_K> on one lk_quant_q8 row, then lk_silu_mul"}
    del ws
    x16, sc = ops.row_scale_f16(torch.randn(m, k, device=dev).to(torch.bfloat16))
    yp, yq = torch.empty(m, n, device=dev), torch.empty(m, n, device=dev)
    wg2 = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
    flops = 2.0 * 2 * m * n * k
    gsteps = max(3, min(args.steps, 50))
    ms_pair = timed(lambda: ops.gemm("q4_k+q6_k", "swiglu", x16, sc, wg, n, w2=wu, y=yp), gsteps, 1)

    def gemm_two():
        ops.gemm("q4_k", "store", x16, sc, wg, n, y=yp)
        ops.gemm("q6_k", "store", x16, sc, wu, n, y=yq)
        ops.silu_mul(yp, yq)
    ms_two = timed(gemm_two, gsteps, 1)
    ms_one = timed(lambda: ops.gemm("q4_k", "swiglu", x16, sc, wg, n, w2=wg2, y=yp), gsteps, 1)
    out["prefill"] = {"rows": m, "pair_tflops": round(flops / (ms_pair * 1e-3) / 1e12, 1),
                      "pair_ms": round(ms_pair, 4), "two_gemms_silu_mul_ms": round(ms_two, 4),
                      "q4_k_swiglu_ms": round(ms_one, 4),
                      "kernel": "two passes of k_gemm_p (tcgen05 kind::f16): Q4_K store, Q6_K store with the act "
                                "epilogue against the stored gate"}
    return out


class Timed:
    """A step's launches captured as one CUDA graph (the kernels then run back to back, without host gaps)."""

    def __init__(self, torch, body):
        body()   # eager first call: per-device kernel set-up happens outside the capture
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                body()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = g

    def replay(self):
        self.graph.replay()


F16_SCALE = {"q4_0": 5.6e-3, "iq4_nl": 3.5e-4}   # block scales of quantised N(0, 0.02): amax / 8, amax / 127


def synth_blocks(torch, dev, rows, k, fmt, gen):
    """Packed 18-byte blocks synthesised on the device for timing: uniform 4-bit codes, the f16 scale a block of
    N(0, 0.02) weights gets (the values do not change the work; parity is tested on quantised weights)."""
    w = torch.randint(0, 256, (rows, k // 32, 18), dtype=torch.uint8, device=dev, generator=gen)
    d = np.frombuffer(np.float16(F16_SCALE[fmt]).tobytes(), np.uint8)
    w[:, :, 0] = int(d[0])
    w[:, :, 1] = int(d[1])
    return w.view(rows, -1)


def synth_kquant(torch, dev, rows, k, fmt, gen):
    """Q4_K / Q6_K super-blocks synthesised on the device: uniform bytes, the f16 scale(s) of the host forms."""
    bb, offs = {"q4_k": (144, [(0, Q4K_D)]), "q6_k": (210, [(208, np.frombuffer(np.float16(2e-4).tobytes(), np.uint8))])}[fmt]
    w = torch.randint(0, 256, (rows, k // 256, bb), dtype=torch.uint8, device=dev, generator=gen)
    for o, b in offs:
        for i, v in enumerate(b):
            w[:, :, o + i] = int(v)
    return w.view(rows, -1)


def synth_mxfp4(torch, dev, rows, k, gen):
    """MXFP4 split planes synthesised on the device: uniform nibbles, E8M0 exponents 119..121 (N(0, 0.02) blocks)."""
    nib = torch.randint(0, 256, (rows, k // 2), dtype=torch.uint8, device=dev, generator=gen)
    sc = torch.randint(119, 122, (rows, k // 32), dtype=torch.uint8, device=dev, generator=gen)
    return nib, sc


def bench_sharded(args, torch, dist, dev, world, rank, time_steps):
    """IQ4_NL K=5120 N=27648 and K=27648 N=5120 at M=4096, output columns sharded over the ranks and
    all-gathered; one step = both GEMMs. Strong scaling (the job is fixed). Exchanges: 'p2p' (tiles stored into
    every rank's y by the GEMM epilogue) and 'collective' (local GEMM + NCCL all-gather + column interleave)."""
    from loom_skills_b200 import ops
    from loom_skills_b200.parallel import ShardedGemm, shard_range
    M = 4096
    shapes = [("gate_up", 5120, 27648), ("down", 27648, 5120)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    xgen = torch.Generator(device=dev)
    xgen.manual_seed(99)   # the same activations on every rank
    parts = []
    for name, k, n in shapes:
        c0, c1 = shard_range(n, world, rank)
        w = synth_blocks(torch, dev, c1 - c0, k, "iq4_nl", gen)
        x = torch.randn(M, k, device=dev, generator=xgen).to(torch.bfloat16)
        x16, sc = ops.row_scale_f16(x)
        parts.append((name, k, n, w, x16, sc))
    flops = sum(2.0 * M * k * n for _, k, n, *_ in parts)
    out = {"workload": "configs[4] Qwen2.5-32B-like IQ4_NL, M=4096: K=5120 N=27648 and K=27648 N=5120",
           "data": "IQ4_NL blocks synthesised on the device (uniform indices, f16 scale 3.5e-4); bf16 N(0,1) x",
           "n_gpus": world, "scaling": "strong", "sharding": "output columns (weight rows) per rank, y all-gathered"}
    steps = max(5, min(20, args.steps // 50))
    # the parts on their own: this rank's shard GEMMs without any exchange, and the NCCL all-gather of f32 shards of
    # the step's output sizes without any GEMM (max over ranks, like every line)
    ys = [torch.empty(M, w.shape[0], device=dev) for _, _, _, w, _, _ in parts]

    def gemm_step():
        for (_, _, _, w, x16, sc), y in zip(parts, ys):
            ops.gemm("iq4_nl", "store", x16, sc, w, w.shape[0], y=y)
    for _ in range(3):
        gemm_step()
    g_ms = time_steps(gemm_step, steps)
    out["gemm_only"] = {"ms_per_step": round(g_ms, 4), "tflops_per_rank": round(flops / world / (g_ms * 1e-3) / 1e12, 1)}
    if world > 1:
        gbufs = [torch.empty(world * M, y.shape[1], device=dev) for y in ys]

        def gather_step():
            for y, gb in zip(ys, gbufs):
                dist.all_gather_into_tensor(gb, y)
        for _ in range(3):
            gather_step()
        a_ms = time_steps(gather_step, steps)
        moved = sum((world - 1) * M * y.shape[1] * 4 for y in ys)
        out["gather_only"] = {"ms_per_step": round(a_ms, 4), "recv_gbs_per_rank": round(moved / (a_ms * 1e-3) / 1e9, 1)}
        del gbufs
    del ys
    for exchange in ("p2p", "collective"):
        sgs = [ShardedGemm("iq4_nl", "store", w, n, k, exchange=exchange) for _, k, n, w, _, _ in parts]

        def step():
            for sg, (_, _, _, _, x16, sc) in zip(sgs, parts):
                sg(x16, sc)
        for _ in range(max(3, args.warmup // 3)):
            step()
        ms = time_steps(step, steps)
        out[exchange] = {"ms_per_step": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                         "steps": steps}
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for sg in sgs:
            sg.close()
    # fused compute + collective roofline: the slower of the GEMM at the measured tensor peak and the bytes each rank
    # must push over NVLink (its f32 shard to world - 1 peers) at the measured 770 GB/s per direction
    pk, _ = peaks()
    t_math = flops / world / (pk["bf16_tflops_sustained"] * 1e12)
    t_link = sum((world - 1) * M * (n / world) * 4 for _, _, n, *_ in parts) / 770e9
    target = max(t_math, t_link)
    out["roofline"] = {"target_ms": round(target * 1e3, 4), "t_math_ms": round(t_math * 1e3, 4),
                       "t_link_ms": round(t_link * 1e3, 4), "frac": round(target * 1e3 / out["p2p"]["ms_per_step"], 4),
                       "peaks": "measured bf16 sustained; NVLink 770 GB/s per direction (measured peer copy)"}
    return out


def bench_ep_moe(args, torch, dist, dev, world, rank, time_steps):
    """configs[2] with its experts sharded over the ranks (expert parallelism): every rank routes its own 4096 tokens,
    the assignments are sorted by destination rank and gathered on the GPU, NCCL all-to-all moves the rows there and
    back, the owning rank runs its experts (grouped GEMMs), and the weighted combine reads the returned rows in place.
    Weak scaling: 4096 tokens per rank. With one GPU the same tokens run the local MoE layer (no exchange)."""
    from loom_skills_b200 import ops
    from loom_skills_b200.parallel import ExpertParallelMoE
    E, ku, h, f, m = 128, 8, 2048, 768, 4096
    gen = torch.Generator(device=dev)
    gen.manual_seed(777)   # the same experts on every rank; each rank keeps its slice
    w_gu = synth_blocks(torch, dev, E * 2 * f, h, "q4_0", gen)
    w_dn = synth_blocks(torch, dev, E * h, f, "q4_0", gen)
    tgen = torch.Generator(device=dev)
    tgen.manual_seed(1000 + rank)
    x = torch.randn(m, h, device=dev, generator=tgen).to(torch.bfloat16)
    lg = torch.randn(m, E, device=dev, generator=tgen)
    flops = 2.0 * m * ku * 3 * h * f
    out = {"workload": "configs[2] Qwen3-30B-A3B-like Q4_0 MoE layer, E=128 top-8, H=2048, F=768, 4096 tokens per rank",
           "n_gpus": world, "scaling": "weak",
           "data": "Q4_0 blocks synthesised on the device; bf16 N(0,1) x, N(0,1) logits per rank"}
    steps = max(3, min(10, args.steps // 100))
    if world == 1:
        fn = lambda: ops.moe_ffn("q4_0", x, lg, w_gu, w_dn, h, f, E, ku)   # noqa: E731
        for _ in range(3):
            fn()
        ms = time_steps(fn, steps)
        out["local"] = {"ms_per_step": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1)}
        return out
    nl = E // world
    moe = ExpertParallelMoE("q4_0", w_gu[rank * nl * 2 * f:(rank + 1) * nl * 2 * f].contiguous(),
                            w_dn[rank * nl * h:(rank + 1) * nl * h].contiguous(), h, f, E, ku)
    del w_gu, w_dn
    for _ in range(3):
        moe(x, lg)
    ms = time_steps(lambda: moe(x, lg), steps)
    moe(x, lg, timed=True)   # one more call with per-stage events (the stage times are max over ranks)
    st = {}
    for k, v in moe.times.items():
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        st[k] = round(float(t.item()), 4)
    out["expert_parallel"] = {"ms_per_step": round(ms, 4), "tflops": round(world * flops / (ms * 1e-3) / 1e12, 1),
                              "stages_ms": st}
    return out


def moe_path(ops, torch, lg, E, ku, m, expert_bytes, ms, matvec_below=64):
    """Which pipeline a MoE layer of m tokens runs (Q4 on these shapes: expert matvecs up to 1024 assignments, grouped
    by expert from 128; MXFP4: matvecs for at most 16 assignments), and for the matvecs the weight GB/s over the
    experts the routing touches."""
    if m >= matvec_below:
        return {"path": "grouped GEMMs"}
    ids, _ = ops.moe_route(lg, E, ku)
    eu = int(torch.unique(ids).numel())
    return {"path": "expert matvecs", "touched_experts": eu,
            "weight_gbs": round(eu * expert_bytes / (ms * 1e-3) / 1e9, 1)}


def moe_inputs(torch, dev, gen, m, h, E):
    """The (x, logits) pairs one timed MoE step walks: at decode sizes (m <= 32) 8 different routings, so the experts a
    step touches (8 x the routing's) exceed the L2 and every expert streams from HBM; one pair for larger m, where
    all experts are touched."""
    r = 8 if m <= 32 else 1
    return [(torch.randn(m, h, device=dev, generator=gen).to(torch.bfloat16), torch.randn(m, E, device=dev, generator=gen))
            for _ in range(r)]


def timed_layers(torch, time_steps, pairs, layer):
    """ms per MoE layer over the pairs (one CUDA graph runs `layer` once per pair)."""
    g = Timed(torch, lambda: [layer(x, lg) for x, lg in pairs])
    for _ in range(3):
        g.replay()
    return time_steps(g.replay, 20) / len(pairs)


def bench_moe(args, torch, dev, time_steps, pk):
    """configs[2] (Q4_0 MoE, Qwen3-30B-A3B-like) and configs[3] (MXFP4 x e4m3 MoE, gpt-oss-20b-like): one MoE layer
    (route, schedule, expert GEMMs / matvecs, combine) per step as a CUDA graph; plus the dense MXFP4 x FP8 GEMM."""
    from loom_skills_b200 import ops
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321)
    out = {}
    E, ku, h, f = 128, 8, 2048, 768
    w_gu = synth_blocks(torch, dev, E * 2 * f, h, "q4_0", gen)
    w_dn = synth_blocks(torch, dev, E * h, f, "q4_0", gen)
    q = {}
    for m in (1, 16, 64, 256, 4096):
        pairs = moe_inputs(torch, dev, gen, m, h, E)
        ms = timed_layers(torch, time_steps, pairs, lambda x, lg: ops.moe_ffn("q4_0", x, lg, w_gu, w_dn, h, f, E, ku))
        q[str(m)] = {"ms": round(ms, 4), "tflops": round(2.0 * m * ku * 3 * h * f / (ms * 1e-3) / 1e12, 2),
                     "routings_per_step": len(pairs),
                     **moe_path(ops, torch, pairs[0][1], E, ku, m, 3 * h * f * 18 // 32, ms, 1024 // ku + 1)}
    out["q4_0_qwen3_30b"] = {"experts": E, "top_k": ku, "hidden": h, "intermediate": f, "by_tokens": q,
                             "data": "Q4_0 blocks synthesised on the device; bf16 N(0,1) x, N(0,1) logits"}
    del w_gu, w_dn
    # the same layer in a Q4_K_M-like mix (Q4_K gate/up, Q6_K down) at decode sizes: the reference's default MOE_Q8
    # numerics (int8 expert matvecs, lk_moe_expert_mv_q8) beside the f32-activation expert matvecs
    w_gu = synth_kquant(torch, dev, E * 2 * f, h, "q4_k", gen)
    w_dn = synth_kquant(torch, dev, E * h, f, "q6_k", gen)
    kq = {}
    ebytes = 2 * f * h // 256 * 144 + h * f // 256 * 210
    for m in (1, 4):
        pairs = moe_inputs(torch, dev, gen, m, h, E)
        row = {"routings_per_step": len(pairs)}
        for name, q8 in (("int8", True), ("f32", False)):
            ms = timed_layers(torch, time_steps, pairs,
                              lambda x, lg: ops.moe_ffn("q4_k", x, lg, w_gu, w_dn, h, f, E, ku, prefill=False,
                                                        fmt_down="q6_k", act_q8=q8))
            row[name] = {"ms": round(ms, 4), **moe_path(ops, torch, pairs[0][1], E, ku, m, ebytes, ms, 1 << 30)}
        kq[str(m)] = row
    out["q4_k_m_mix_qwen3_30b"] = {"experts": E, "top_k": ku, "hidden": h, "intermediate": f, "gate_up": "q4_k",
                                   "down": "q6_k", "by_tokens": kq,
                                   "data": "Q4_K / Q6_K blocks synthesised on the device; bf16 N(0,1) x, N(0,1) logits"}
    del w_gu, w_dn
    E, ku, h, f = 32, 4, 2880, 2880
    gu, gus = synth_mxfp4(torch, dev, E * 2 * f, h, gen)
    dn, dns = synth_mxfp4(torch, dev, E * h, f, gen)
    # gpt-oss numerics: softmax of the picked biased logits (gating 3), swiglu_oai, per-expert biases
    rbias = torch.randn(E, device=dev, generator=gen) * 0.1
    bg, bu = (torch.randn(E, f, device=dev, generator=gen) * 0.05 for _ in range(2))
    bd = torch.randn(E, h, device=dev, generator=gen) * 0.05
    oai = dict(gating=3, router_bias=rbias, norm=False, act="swiglu_oai", b_gate=bg, b_up=bu, b_down=bd)
    mx = {}
    for m in (1, 32, 1024, 8192):
        pairs = moe_inputs(torch, dev, gen, m, h, E)
        ms = timed_layers(torch, time_steps, pairs,
                          lambda x, lg: ops.moe_ffn_mxfp4s(x, lg, gu, gus, dn, dns, h, f, E, ku, **oai))
        mx[str(m)] = {"ms": round(ms, 4), "tflops": round(2.0 * m * ku * 3 * h * f / (ms * 1e-3) / 1e12, 2),
                      "routings_per_step": len(pairs),
                      **moe_path(ops, torch, pairs[0][1], E, ku, m, 3 * h * f // 2 + 3 * h * f // 32, ms, 16 // ku + 1)}
    # the dense kernel alone: fused gate/up shape, M=8192
    M = 8192
    x8, s8 = ops.row_scale_f8(torch.randn(M, h, device=dev, generator=gen))
    yg = torch.empty(M, f, device=dev)
    g = Timed(torch, lambda: ops.gemm_mxfp4s_f8("swiglu", x8, s8, gu[:f], gus[:f], f, w2=gu[f:2 * f],
                                                 w2s=gus[f:2 * f], y=yg))
    for _ in range(3):
        g.replay()
    ms = time_steps(g.replay, 50)
    tf = 2.0 * M * h * 2 * f / (ms * 1e-3) / 1e12
    f8_peak = 2 * pk["bf16_tflops_sustained"]
    out["mxfp4_gpt_oss_20b"] = {
        "experts": E, "top_k": ku, "hidden": h, "intermediate": f, "by_tokens": mx,
        "numerics": "gating 3 with router bias, swiglu_oai (alpha 1.702, limit 7), per-expert gate/up/down biases",
        "data": "MXFP4 planes synthesised on the device (uniform nibbles, E8M0 119..121); bf16 N(0,1) x",
        "dense_gemm": {"shape": [M, h, 2 * f], "mode": "swiglu", "ms": round(ms, 4), "tflops": round(tf, 1),
                       "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": round(f8_peak, 1),
                                    "unit": "TFLOP/s", "frac": round(tf / f8_peak, 4),
                                    "frac_of_fp4_dense_peak": round(tf / (4 * pk["bf16_tflops_sustained"]), 4),
                                    "peak_source": "2 x measured bf16 sustained: kind::mxf8f6f4 runs at the fp8 rate "
                                                   "(e4m3 activations keep it off the fp4 rate)",
                                    "kernel": "k_gemm_mx (tcgen05 kind::mxf8f6f4.block_scale, lk_mxfp4)"}}}
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    from loom_skills_b200 import ops

    rank, local, world = rank_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    pk, pk_src = peaks()
    wstack = make_weights(torch, args.layers, seed=rank)
    torch.manual_seed(rank)
    # the step's two activation vectors are views of one buffer, so the e2e step brings them in with one copy
    xbuf = torch.randn(1, 4096 + 12288, device=dev).to(torch.bfloat16)
    xs = {4096: xbuf[:, :4096], 12288: xbuf[:, 4096:]}
    # every projection output of the step is a view of one buffer, so the e2e step reads them back with one copy
    ncols = sum(n for _, _, n in SHAPES)
    yall = torch.empty(args.layers, ncols, device=dev)
    offs = np.cumsum([0] + [n for _, _, n in SHAPES])
    ys = [{name: yall[li, offs[j]:offs[j + 1]].view(1, n) for j, (name, _, n) in enumerate(SHAPES)}
          for li in range(args.layers)]
    wbytes_layer = sum(wstack[0][name].numel() for name, _, _ in SHAPES)
    act_bytes = sum(k * 2 + n * 4 for _, k, n in SHAPES)   # bf16 x read + f32 y written, per layer
    mv_per_step = args.layers * 4          # matvec launches: q|k|v, o, gate_up, down
    launches_per_step = mv_per_step + args.layers * 2   # + one quantisation per distinct activation row
    step_bytes = args.layers * wbytes_layer

    # int8 activations per layer: the reference's default decode numerics (ACT_Q8=1, gen_llm.py:514-518)
    xq = [{k: torch.empty(k + (k // 32) * 8, dtype=torch.uint8, device=dev) for k in xs} for _ in range(args.layers)]

    def quant_layer(li):
        for k in xs:
            ops.quant_q8(xs[k], out=xq[li][k])

    def mv_layer(li):
        # q | k | v share the activation: one launch over the three weights (lk_mv_q8_multi)
        w, y = wstack[li], ys[li]
        ops.mv_q8_multi("q4_k", [w["q"], w["k"], w["v"]], xq[li][4096], [4096, 1024, 1024], 4096, 1,
                        ys=[y["q"], y["k"], y["v"]])
        for name, k, n in SHAPES[3:]:
            ops.mv_q8("q4_k", w[name], xq[li][k], n, k, 1, y=y[name])

    def fused_layer(li):
        # the activation quantised inside each matvec (lk_mv_q8_fused): four launches per layer, q | k | v in one
        w, y = wstack[li], ys[li]
        ops.mv_q8_fused_multi("q4_k", [w["q"], w["k"], w["v"]], xs[4096], [4096, 1024, 1024], 4096,
                              ys=[y["q"], y["k"], y["v"]])
        for name, k, n in SHAPES[3:]:
            ops.mv_q8_fused("q4_k", w[name], xs[k], n, k, y=y[name])

    def decode_body():   # one decode step: the six projections of every layer, int8 numerics (16 + 32 launches)
        for li in range(args.layers):
            quant_layer(li)
            mv_layer(li)

    def mv_body():       # the step's 32 matvec launches alone (the codes of every layer already in place)
        for li in range(args.layers):
            mv_layer(li)

    def fused_body():    # every matvec quantising its own activation row in its prologue (32 launches)
        for li in range(args.layers):
            fused_layer(li)

    def decode_bf16_body():   # the f32/bf16-activation path (ACT_Q8=0)
        for li in range(args.layers):
            for name, k, n in SHAPES:
                ops.mv("q4_k", wstack[li][name], xs[k], n, k, y=ys[li][name])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_steps(fn, steps, clk=None):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        barrier()
        if clk:
            clk.mark(True)
        t0.record()
        for _ in range(steps):
            fn()
        t1.record()
        barrier()
        if clk:
            clk.mark(False)
        return max_over_ranks(t0.elapsed_time(t1)) / steps

    # ---- decode: device-resident inputs, one graph replay per step (16 quantisations + 32 matvec launches)
    dec = Timed(torch, decode_body)
    for _ in range(args.warmup):
        dec.replay()
    clk = Clocks("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    clk.start()
    ms = time_steps(dec.replay, args.steps, clk)
    clocks = clk.stop()
    value = world * step_bytes / (ms * 1e-3) / 1e9
    # the matvec kernel: a graph of the step's 32 matvec launches alone, between CUDA events, so its average launch is
    # that graph's time over the launches
    mg = Timed(torch, mv_body)
    for _ in range(args.warmup):
        mg.replay()
    mv_ms = time_steps(mg.replay, args.steps)
    code_bytes = {k: k + k // 32 * 8 for k in xs}             # int8 codes + (d, sum) per group, read by every CTA once
    act_bytes_l = sum(code_bytes[k] + n * 4 for _, k, n in SHAPES[2:])   # q|k|v read one row: counted once
    alg_per_launch = (step_bytes + args.layers * act_bytes_l) / mv_per_step
    kavg = mv_ms / mv_per_step
    achieved = alg_per_launch / (kavg * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": int(TRAFFIC_RATIO_DECODE * alg_per_launch), "peak_source": pk_src,
            "kernel": "k_mv_q8_rows (Q4_K x int8 codes, dp4a; lk_mvq8)",
            "avg_launch_us": round(kavg * 1e3, 2), "alg_bytes_per_launch": int(alg_per_launch),
            "mv_ms_per_step": round(mv_ms, 4)}
    # the same step with the quantisation folded into each matvec's prologue (lk_mv_q8_fused), for comparison: every
    # launch quantises its own row, so the step quantises 32 rows where the graph above quantises 16
    fg = Timed(torch, fused_body)
    for _ in range(args.warmup):
        fg.replay()
    fu_ms = time_steps(fg.replay, max(3, args.steps // 4))
    decode_fused = {"value": round(world * step_bytes / (fu_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_step": round(fu_ms, 4), "launches_per_step": mv_per_step,
                    "kernel": "k_mv_q8_rows<.., LK_BF16> (activation row quantised in the prologue)"}
    bf = Timed(torch, decode_bf16_body)
    for _ in range(args.warmup):
        bf.replay()
    bf_ms = time_steps(bf.replay, max(3, args.steps // 4))
    decode_bf16 = {"value": round(world * step_bytes / (bf_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                   "ms_per_step": round(bf_ms, 4), "numerics": "bf16 activations (ACT_Q8=0), k_mv (lk_mv)"}

    # ---- e2e through the public API: pinned host x in, every projection output back, each step (one graph)
    hx = torch.empty_like(xbuf, device="cpu").pin_memory()
    hx.copy_(xbuf.cpu())
    hy = torch.empty(args.layers, ncols).pin_memory()
    h2d = hx.numel() * 2
    d2h = hy.numel() * 4

    side = torch.cuda.Stream()

    def e2e_body():
        # x in, then each layer's outputs copied back on a side stream while the next layers compute (every output of
        # every layer still crosses to the host each step; the step ends when the last copy has)
        xbuf.copy_(hx, non_blocking=True)
        main = torch.cuda.current_stream()
        for li in range(args.layers):
            quant_layer(li)
            mv_layer(li)
            done = torch.cuda.Event()
            done.record(main)
            side.wait_event(done)
            with torch.cuda.stream(side):
                hy[li].copy_(yall[li], non_blocking=True)
        main.wait_stream(side)

    e2e_g = Timed(torch, e2e_body)
    for _ in range(args.warmup):
        e2e_g.replay()
    e2e_ms = time_steps(e2e_g.replay, args.steps)
    e2e = {"value": round(world * step_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4)}

    # ---- prefill: M rows through the same shapes (row scale to f16 + tcgen05 GEMM), one layer
    M = args.prefill_rows
    xp = {k: torch.randn(M, k, device=dev).to(torch.bfloat16) for k in (4096, 12288)}
    yp = {name: torch.empty(M, n, device=dev) for name, _, n in SHAPES}
    flops = sum(2.0 * M * n * k for _, k, n in SHAPES)
    prefill_bytes = sum(M * k * 2 + n * k // 256 * 144 + M * n * 4 for _, k, n in SHAPES)   # x16 + weights + y

    x16p = {}

    def scale_body():
        for k in xp:
            x16p[k] = ops.row_scale_f16(xp[k])

    yqkv = torch.empty(M, 6144, device=dev)

    def gemm_body():   # q | k | v as one GEMM over the fused qkv rows, then o, gate_up, down
        ops.gemm("q4_k", "store", x16p[4096][0], x16p[4096][1], wstack[0]["qkv"], 6144, y=yqkv)
        for name, k, n in SHAPES[3:]:
            ops.gemm("q4_k", "store", x16p[k][0], x16p[k][1], wstack[0][name], n, y=yp[name])

    scale_g = Timed(torch, scale_body)
    gemm_g = Timed(torch, gemm_body)
    ge = []

    def prefill_step():
        # the GEMM graph between CUDA events: the dominant kernel's time, live inside the timed region
        scale_g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        gemm_g.replay()
        b.record()
        ge.append((a, b))

    for _ in range(args.warmup):
        prefill_step()
    ge.clear()
    psteps = max(3, args.steps // 8)
    pms = time_steps(prefill_step, psteps)
    gms = statistics.mean(a.elapsed_time(b) for a, b in ge)
    ptflops = flops / (pms * 1e-3) / 1e12
    gemm_tf = flops / (gms * 1e-3) / 1e12
    peak_tf = pk["bf16_tflops_sustained"]
    prefill = {"rows": M, "tflops": round(world * ptflops, 1), "ms_per_step": round(pms, 4), "steps": psteps,
               "roofline": {"bound": "tensor", "achieved": round(gemm_tf, 1), "peak": peak_tf, "unit": "TFLOP/s",
                            "frac": round(gemm_tf / peak_tf, 4), "traffic": int(TRAFFIC_RATIO_PREFILL * prefill_bytes / len(SHAPES)),
                            "peak_source": pk_src + " sustained", "kernel": "k_gemm<Q4_K> (tcgen05 kind::f16, lk_gemm)"}}

    # ---- sweep over the config's token counts (one layer, per-step ms; row scale included for M >= 64)
    sweep = {}
    if not args.no_sweep:
        for m in (1, 8, 64, 512, 2048):
            xm = {k: torch.randn(m, k, device=dev).to(torch.bfloat16) for k in (4096, 12288)}
            ym = {name: torch.empty(m, n, device=dev) for name, _, n in SHAPES}

            def body_m():
                if m < 64:   # gen_llm.py:6107: matvecs below 64 tokens (int8 activations), GEMMs from 64
                    xqm = {k: ops.quant_q8(xm[k]) for k in xm}
                    for name, k, n in SHAPES:
                        ops.mv_q8("q4_k", wstack[0][name], xqm[k], n, k, m, y=ym[name])
                else:
                    x16 = {k: ops.row_scale_f16(xm[k]) for k in xm}
                    for name, k, n in SHAPES:
                        ops.gemm("q4_k", "store", x16[k][0], x16[k][1], wstack[0][name], n, y=ym[name])
            tm = Timed(torch, body_m)
            for _ in range(3):
                tm.replay()
            mms = time_steps(tm.replay, 20)
            sweep[str(m)] = {"ms": round(mms, 4), "weight_gbs": round(wbytes_layer / (mms * 1e-3) / 1e9, 1),
                             "tflops": round(sum(2.0 * m * n * k for _, k, n in SHAPES) / (mms * 1e-3) / 1e12, 2)}

    # ---- each decode launch form alone (its weights rotated past L2): the GEMV's own fraction of HBM per shape
    gemv = bench_gemv_forms(args, torch, wstack, xs, pk, time_steps) if not args.no_extra else None
    # ---- the IQ4_NL GEMMs N-sharded over the ranks, all-gather fused into the epilogue (strong scaling)
    sharded = bench_sharded(args, torch, dist, dev, world, rank, time_steps) if not args.no_extra else None
    # ---- configs[2] with its experts sharded over the ranks (expert parallelism, NCCL all-to-all)
    ep = bench_ep_moe(args, torch, dist, dev, world, rank, time_steps) if not args.no_extra else None
    # ---- the MoE layers, and the dense MXFP4 x FP8 GEMM (each rank a replica)
    moe = bench_moe(args, torch, dev, time_steps, pk) if not args.no_extra else None
    # ---- gate and up in two formats (Q4_K_M's Q4_K + Q6_K), decode and prefill (each rank a replica)
    pairs = bench_pairs(args, torch, dev, time_steps) if not args.no_extra else None

    gpu_launches = args.steps * launches_per_step   # 16 quantisations + 32 matvec launches per step
    if rank == 0:
        cpu_v, cpu_desc = cpu_decode_gbs(budget_s=args.cpu_seconds)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k x int8 (Q8_1 activations, integer dot, f32 group scaling)",
            "data": "synthetic: seeded Q4_K blocks (f16 d/dmin of N(0,0.02) weights, uniform 6-bit fields and nibbles), N(0,1) bf16 activations",
            "config": {"workload": "configs[1] Qwen3-8B-like Q4_K projections, decode M=1",
                       "shapes_k_n": [[k, n] for _, k, n in SHAPES], "layers": args.layers,
                       "weight_bytes_per_step": step_bytes,
                       "l2": f"inputs larger than L2: {step_bytes / 1e6:.0f} MB of weights rotated over "
                             f"{args.layers} layer copies",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "launch": "one CUDA graph replay per step"},
            "roofline": roof, "cpu_baseline": {"value": round(cpu_v, 4), "unit": "GB/s", **cpu_desc}, "e2e": e2e,
            "gpu_launches": gpu_launches, "clocks": clocks, "prefill": prefill, "sweep": sweep,
            "hbm_frac": round(value / world / pk["hbm_gbs"], 4), "decode_gemv": gemv, "decode_bf16": decode_bf16,
            "decode_fused": decode_fused,
            "sharded_iq4_nl": sharded, "ep_moe": ep, "moe": moe, "gate_up_pair": pairs}
        print(json.dumps(line), flush=True)
    if world > 1:
        del dec, mg, fg, bf, e2e_g, scale_g, gemm_g
        dist.barrier()
        dist.destroy_process_group()


def run_profile_case(args):
    """A few launches of one hot kernel at one bench shape, for ncu captures (profiles/): warm-up launches, then
    `--steps` profiled ones. Cases: mv_gate_up (Q4_K q8 matvec, K=4096 N=24576), mv_down (K=12288 N=4096),
    mv8_gate_up (the gate_up matvec on 8 tokens), gemm_gate_up (Q4_K GEMM, M=2048 K=4096 N=24576), gemm64_down
    (Q4_K GEMM, M=64 K=12288 N=4096), mx_gate_up (MXFP4 x e4m3 swiglu, M=8192 K=2880 N=2880), mxmv_gate_up (the
    MXFP4S expert matvecs of one gpt-oss token: 4 assignments of 32 experts, h = f = 2880, bf16 x), mvf_gate_up (the
    gate_up matvec quantising its bf16 row in the prologue), mvg_q6k (the generic-format matvec, Q6_K K=4096
    N=4096, f32 x), gemm_q6k (the window-producer GEMM, Q6_K M=2048 K=4096 N=4096), moeq8 (the int8 decode MoE layer
    of configs[2] at one token: E=128 top-8, H=2048, F=768, Q4_0), mvp_gate_up / gemmp_gate_up (a Q4_K gate and Q6_K
    up pair, K=4096 N=12288: the one-token matvec on bf16 x, and the swiglu GEMM at M=2048), mvq8_q6k_down (the int8
    matvec over Q6_K, K=12288 N=4096), mv_bf16_gate_up (the persistent one-token matvec on bf16 x, Q4_K K=4096
    N=24576)."""
    import torch

    from loom_skills_b200 import ops
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    case = args.profile_case
    if case == "mvf_gate_up":
        k, n = 4096, 24576
        w = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
        x = torch.randn(1, k, device=dev).to(torch.bfloat16)
        y = torch.empty(1, n, device=dev)
        fn = lambda: ops.mv_q8_fused("q4_k", w, x, n, k, y=y)   # noqa: E731
    elif case in ("mvp_gate_up", "gemmp_gate_up"):
        k, n = 4096, 12288
        wg = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
        wu = torch.from_numpy(synth_q6k(rng, n, k)).to(dev)
        if case == "mvp_gate_up":
            x = torch.randn(1, k, device=dev).to(torch.bfloat16)
            y = torch.empty(1, n, device=dev)
            fn = lambda: ops.mv("q4_k+q6_k", wg, x, n, k, w2=wu, y=y)   # noqa: E731
        else:
            m = 2048
            x16, sc = ops.row_scale_f16(torch.randn(m, k, device=dev).to(torch.bfloat16))
            y = torch.empty(m, n, device=dev)
            fn = lambda: ops.gemm("q4_k+q6_k", "swiglu", x16, sc, wg, n, w2=wu, y=y)   # noqa: E731
    elif case in ("mvg_q6k", "gemm_q6k"):
        k, n = 4096, 4096
        w = torch.from_numpy(synth_q6k(rng, n, k)).to(dev)
        if case == "mvg_q6k":
            x = torch.randn(1, k, device=dev)
            y = torch.empty(1, n, device=dev)
            fn = lambda: ops.mv("q6_k", w, x, n, k, y=y)   # noqa: E731
        else:
            m = 2048
            x16, sc = ops.row_scale_f16(torch.randn(m, k, device=dev).to(torch.bfloat16))
            y = torch.empty(m, n, device=dev)
            fn = lambda: ops.gemm("q6_k", "store", x16, sc, w, n, y=y)   # noqa: E731
    elif case == "moeq8":
        E, ku, h, f = 128, 8, 2048, 768
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)
        wgu = synth_blocks(torch, dev, E * 2 * f, h, "q4_0", gen)
        wdn = synth_blocks(torch, dev, E * h, f, "q4_0", gen)
        x = torch.randn(1, h, device=dev, generator=gen).to(torch.bfloat16)
        lg = torch.randn(1, E, device=dev, generator=gen)
        y = torch.empty(1, h, device=dev)
        act = torch.empty(ku, f, device=dev)
        fn = lambda: ops.moe_ffn_decode_q8("q4_0", x, lg, wgu, wdn, h, f, E, ku, y=y, act_buf=act)   # noqa: E731
    elif case == "mv_bf16_gate_up":
        k, n = 4096, 24576
        w = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
        x = torch.randn(1, k, device=dev).to(torch.bfloat16)
        y = torch.empty(1, n, device=dev)
        fn = lambda: ops.mv("q4_k", w, x, n, k, y=y)   # noqa: E731
    elif case == "mvq8_q6k_down":
        k, n = 12288, 4096
        w = torch.from_numpy(synth_q6k(rng, n, k)).to(dev)
        xq = ops.quant_q8(torch.randn(1, k, device=dev))
        y = torch.empty(1, n, device=dev)
        fn = lambda: ops.mv_q8("q6_k", w, xq, n, k, 1, y=y)   # noqa: E731
    elif case.startswith("mv"):
        k, n = (12288, 4096) if case == "mv_down" else (4096, 24576)
        t = 8 if case == "mv8_gate_up" else 1
        w = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
        xq = ops.quant_q8(torch.randn(t, k, device=dev))
        y = torch.empty(t, n, device=dev)
        fn = lambda: ops.mv_q8("q4_k", w, xq, n, k, t, y=y)   # noqa: E731
    elif case.startswith("gemm"):
        m, k, n = (64, 12288, 4096) if case == "gemm64_down" else (2048, 4096, 24576)
        w = torch.from_numpy(synth_q4k(rng, n, k)).to(dev)
        x16, sc = ops.row_scale_f16(torch.randn(m, k, device=dev).to(torch.bfloat16))
        y = torch.empty(m, n, device=dev)
        fn = lambda: ops.gemm("q4_k", "store", x16, sc, w, n, y=y)   # noqa: E731
    elif case == "mx_gate_up":
        m, k, n = 8192, 2880, 2880
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)
        g, gs = synth_mxfp4(torch, dev, n, k, gen)
        u, us = synth_mxfp4(torch, dev, n, k, gen)
        x8, s8 = ops.row_scale_f8(torch.randn(m, k, device=dev))
        y = torch.empty(m, n, device=dev)
        fn = lambda: ops.gemm_mxfp4s_f8("swiglu", x8, s8, g, gs, n, w2=u, w2s=us, y=y)   # noqa: E731
    elif case == "mxmv_gate_up":
        E, ku, h, f = 32, 4, 2880, 2880
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)
        gu, gus = synth_mxfp4(torch, dev, E * 2 * f, h, gen)
        x = torch.randn(1, h, device=dev).to(torch.bfloat16)
        ids = torch.tensor([3, 11, 17, 29], dtype=torch.int32, device=dev)
        y = torch.empty(ku, f, device=dev)
        fn = lambda: ops.moe_expert_mv_mxfp4s("gu", ids, x, gu, gus, f, h, ku, E, y=y)   # noqa: E731
    else:
        raise SystemExit(f"unknown --profile-case {case}")
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": case, "launches": args.warmup + args.steps}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--prefill-rows", type=int, default=2048)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the sharded-GEMM and MoE sections")
    ap.add_argument("--profile-case", default=None, help="run one kernel a few times for an ncu capture")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_case:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

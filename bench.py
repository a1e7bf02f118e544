"""bench.py -- W8A8 ConvRot linear throughput on B200, one JSON line on rank 0.

A step is one pass of the DiT block's four int8 ConvRot linears over one 32760-token batch (BASELINE.json
configs[1]): qkv 5120->15360, fc1 5120->13824, out-proj 5120->5120, fc2 13824->5120.  Each linear is the
reference's fused path (attn8::gemm_s8 with rotate): the fused Hadamard-256 rotation + per-token int8
quantization kernel, then the tcgen05 int8 GEMM with its fused scale/bias epilogue, bf16 out.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun the step's 32760 tokens are split over the ranks (BASELINE config 4's M sharding, 4095 tokens per
GPU at 8 GPUs; strong scaling, weights replicated, no collective on the data path); times are CUDA events, max
over ranks.  The same line carries, at N > 1, the weak-scaling run (32760 tokens per GPU), the N-split linears and
the query-sharded attention, each checked against the single-GPU result; at N = 1, the other configs (c2, c3, c4's
attention), the DiT call sites and the cuBLASLt comparator.  --impl reference times the reference's CPU path for
the same linears (rotate -> dequantise -> float matmul, portable/kernels.rs:220-242) on the host cores over the
whole 32760-token workload.
"""
from __future__ import annotations

import argparse
import datetime
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "h3-rs_b200"))

METRIC = "W8A8 ConvRot linear TOPS (% of int8 peak) at DiT shapes, 1/2/4/8 B200"
M_TOKENS = 32760
LINEARS = [("qkv", 5120, 15360), ("fc1", 5120, 13824), ("out", 5120, 5120), ("fc2", 13824, 5120)]
WORKLOAD = ("BASELINE c1: DiT-scale int8 ConvRot linears, M=32760 tokens; qkv 5120->15360, fc1 5120->13824, "
            "out 5120->5120, fc2 13824->5120; bf16 in/out, per-token int8 activations, int8 weights")
NOMINAL_INT8_TOPS = 4500.0
E2E_CHUNK = int(os.environ.get("H3Q_E2E_CHUNK", "2048"))  # rows per chunk of the host-memory path (e2e)
E2E_IN_SLOTS = int(os.environ.get("H3Q_E2E_IN_SLOTS", "32"))  # input chunk buffers of the host-memory path


def ops_per_step(m: int) -> float:
    return float(sum(2.0 * m * k * n for _, k, n in LINEARS))


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms around the timed region; the summary keeps the samples
    whose timestamps fall inside the `with` block (the timed region: the block ends after a device synchronize),
    or every sample when the region is shorter than the sampling interval."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        self.t0 = datetime.datetime.now()
        return self

    def __exit__(self, *exc):
        self.t1 = datetime.datetime.now()
        time.sleep(0.06)  # one more sample interval, so a sample taken just before the exit is flushed
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def when(r):
            try:
                return datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                return None
        inside = [r for r in rows if when(r) is not None and self.t0 <= when(r) <= self.t1]
        use = inside or rows
        sm = [float(r[2]) for r in use if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in use for i in range(4) if r[6 + i].lower() == "active"})
        loaded = [v for v in sm if mx and v > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "samples_in_region": len(inside)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# --------------------------------------------------------------------------------------------- CPU baseline

def cpu_baseline(rows: int = 4096) -> dict:
    """The reference's CPU path (oracle port of portable/kernels.rs:220-242) for every linear of the workload:
    each call dequantises the whole weight (timed in full, once per linear, as the reference does per call), then
    rotates and multiplies the activations (timed on a `rows`-token sample and scaled to 32760 tokens).  The
    default sample is about 10 s of host work on a 16-thread host.
    TOPS = algorithmic ops of the full workload / that extrapolated time.  numpy BLAS uses every host core."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    cores = _blas_threads()
    t_full, t_deq, t_rows_s = 0.0, 0.0, 0.0
    for _, k, n in LINEARS:
        w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        ws = (rng.random(n, dtype=np.float32) * 9e-3 + 1e-3).astype(np.float32)
        b = O.bf16_round((rng.standard_normal(n) * 0.02).astype(np.float32))
        x = O.f32_to_bf16_bits(rng.standard_normal((rows, k)).astype(np.float32))
        t0 = time.perf_counter()
        wd = O.cpu_dequant_weight(w, ws)
        t1 = time.perf_counter()
        O.cpu_linear_rows(x, wd, b, rotate=True)
        t2 = time.perf_counter()
        t_deq += t1 - t0
        t_rows_s += t2 - t1
        t_full += (t1 - t0) + (t2 - t1) * (M_TOKENS / rows)
    value = ops_per_step(M_TOKENS) / t_full / 1e12
    return {"value": value, "unit": "TOPS", "cores": cores, "kind": "port",
            "sample": f"all 4 linears: full weight dequantisation timed ({t_deq:.1f} s, single-threaded like "
                      f"portable/kernels.rs:14-27), rotate+matmul timed on {rows} of {M_TOKENS} tokens "
                      f"({t_rows_s:.1f} s, numpy BLAS on {cores} threads) and scaled linearly to {M_TOKENS} tokens "
                      f"(extrapolated full-step time {t_full:.1f} s)",
            "seconds": t_deq + t_rows_s}


def _blas_threads() -> int:
    """Every host core for numpy's BLAS, whatever OMP_NUM_THREADS the launcher set (torchrun sets 1)."""
    cores = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(cores)
    except ImportError:
        pass
    return cores


def run_reference(args) -> None:
    """--impl reference: the reference's CPU implementation of the path (oracle port of portable/kernels.rs:220-242,
    the Rust crate cannot be built here) on this host's cores, same metric, unit and workload; rank 0 only.

    The timed region is one whole reference call per linear over all 32760 tokens, nothing extrapolated: each
    linear's weight is dequantised once (as one call over the batch does), then the rows are rotated and
    multiplied.  The K timed steps split the rows into K consecutive slices of every linear (the dequantisation
    falls in the first step), so ms_per_step x K is the measured time of the full pass.  The W warm-up steps run
    64-row slices and are not timed."""
    import numpy as np
    from oracle import oracle as O
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    cores = _blas_threads()
    rng = np.random.default_rng(0)
    layers = []
    for _, k, n in LINEARS:
        w = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        wsc = (rng.random(n, dtype=np.float32) * 9e-3 + 1e-3).astype(np.float32)
        b = O.bf16_round((rng.standard_normal(n) * 0.02).astype(np.float32))
        x = rng.standard_normal((M_TOKENS, k), dtype=np.float32)
        x[:, rng.choice(k, 8, replace=False)] *= 20.0
        layers.append((w, wsc, b, O.f32_to_bf16_bits(x)))
        del x
    for _ in range(args.warmup):
        for w, wsc, b, x in layers:
            O.cpu_linear_rows(x[:64], O.cpu_dequant_weight(w[:256], wsc[:256]), b[:256], rotate=True)
    steps = max(1, args.steps)
    bounds = [M_TOKENS * s // steps for s in range(steps + 1)]
    deq = [None] * len(layers)
    t_deq = 0.0
    t0 = time.perf_counter()
    for s in range(steps):
        for i, (w, wsc, b, x) in enumerate(layers):
            if deq[i] is None:
                t1 = time.perf_counter()
                deq[i] = O.cpu_dequant_weight(w, wsc)
                t_deq += time.perf_counter() - t1
            O.cpu_linear_rows(x[bounds[s]:bounds[s + 1]], deq[i], b, rotate=True)
    total = time.perf_counter() - t0
    value = ops_per_step(M_TOKENS) / total / 1e12
    cb = {"value": value, "unit": "TOPS", "cores": cores, "kind": "port",
          "sample": f"the whole workload, unextrapolated: one reference call per linear over all {M_TOKENS} tokens "
                    f"(weight dequantisation {t_deq:.1f} s, single-threaded like portable/kernels.rs:14-27; rotate + "
                    f"matmul with numpy BLAS on {cores} threads), split into {steps} row slices, {total:.1f} s "
                    f"in total"}
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": ws, "steps": steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(ws), "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_block(n_gpus: int) -> dict:
    m_r = [hi - lo for lo, hi in (row_range(M_TOKENS, n_gpus, r) for r in range(n_gpus))]
    par = ("x1: all 32760 tokens on one GPU" if n_gpus == 1 else
           f"token-sharded x{n_gpus} (strong: the 32760 tokens split over the GPUs, {min(m_r)}-{max(m_r)} per GPU, "
           "weights replicated, no collective)")
    return {"workload": WORKLOAD, "M_total": M_TOKENS, "M_per_gpu": max(m_r),
            "linears": [f"{nm}:{k}x{n}" for nm, k, n in LINEARS],
            "rotate": "ConvRot Hadamard-256, fused into the quantizer", "epilogue": "xs*ws*acc + bias -> bf16",
            "l2": "no flush: at 32760 tokens every activation (335-905 MB) and output is larger than the 126 MB L2; "
                  "at 4095 tokens per GPU a step's inputs (247 MB of weights plus 240 MB of activations) and "
                  "outputs (323 MB) are over six times L2, so nothing a linear reads survives to its next run",
            "parallelism": par}


def row_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows of rank r: [floor(r total / g), floor((r + 1) total / g)) (h3q.parallel.row_range)."""
    return total * rank // world, total * (rank + 1) // world


# --------------------------------------------------------------------------------------------- our arm

def nvfp4_c3(dev, peaks: dict, reps: int = 10) -> dict:
    """the text encoder's NVFP4+AWQ linears at 512 prompt tokens (5120 -> 25600 and
    25600 -> 5120), fused fp4-decode + bf16 tcgen05 GEMM; CUDA-event time per layer and TFLOP/s against the measured
    bf16 peak (the tensor cores run bf16 here, because the reference keeps the activations bf16)."""
    import torch
    import h3q
    g = torch.Generator(device=dev).manual_seed(99)
    pool = torch.tensor([(e << 3) | m for e in (6, 7, 8) for m in range(8)] + [9 << 3], dtype=torch.uint8, device=dev)
    res = []
    for K, N in ((5120, 25600), (25600, 5120)):
        M = 512
        x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
        q = torch.randint(0, 256, (N, K // 2), generator=g, device=dev, dtype=torch.uint8)
        nbytes = ((N + 127) // 128) * ((K // 16 + 3) // 4) * 512
        bs = pool[torch.randint(0, pool.numel(), (nbytes,), generator=g, device=dev)]
        gs = torch.tensor([1.0 / 448.0], device=dev)
        pqs = (torch.rand(K, generator=g, device=dev) * 1.5 + 0.5).to(torch.bfloat16)
        ms = time_steps(lambda: h3q.nvfp4_linear(x, q, bs, gs, pqs), reps, dev)
        # the reference's GPU path on the same box: dequant_nvfp4 of the whole weight to bf16 (this library's
        # bit-exact kernel for kernels.rs:65-81), the AWQ multiply (weights.rs:617-620) and a bf16 cuBLAS matmul
        # (weights.rs:632), as QLinear::apply runs them for every call
        wbf = torch.empty((N, K), dtype=torch.bfloat16, device=dev)

        def ref_path():
            wd = h3q.dequant_nvfp4(q, bs, gs, torch.bfloat16)
            x2 = (x.float() * pqs.float()).to(torch.bfloat16)
            return torch.matmul(x2, wd.t())
        ref_ms = time_steps(ref_path, reps, dev)
        mm_ms = time_steps(lambda: torch.matmul(x, wbf.t()), reps, dev)
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        wbytes = N * K // 2 + nbytes
        res.append({"linear": f"{K}->{N}", "M": M, "ms": round(ms, 4), "tflops": round(tf, 1),
                    "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 3),
                    "weight_gbs": round(wbytes / (ms * 1e-3) / 1e9, 1),
                    "reference_gpu_path_ms": round(ref_ms, 4), "speedup_vs_reference_gpu_path": round(ref_ms / ms, 2),
                    "cublas_bf16_matmul_alone_ms": round(mm_ms, 4)})
    return {"workload": "BASELINE c3: NVFP4+AWQ text-encoder linears, M=512", "layers": res,
            "note": "time per call includes the AWQ pre-pass and, for 25600->5120, the stream-K fix-up; "
                    "cublas_bf16_matmul_alone_ms: the bf16 GEMM of the same shape with a resident bf16 weight"}


def attention_c4(dev, peaks: dict, reps: int = 5, S: int = 32760, H: int = 40) -> dict:
    """BASELINE config 4's attention: SageAttention-style int8 Q.K^T + f16 P.V at batch 1, 40 heads, head_dim 128,
    32760 tokens.  CUDA-event time of the whole attn8::attention pipeline (K mean, Q/K quantisation, V relayout,
    the tcgen05 attention kernel) and of the attention kernel alone; TOPS counted as the reference's attention bench
    counts them (4 S^2 D H, examples/attn_bench.rs), plus each half against its own peak."""
    import torch
    import h3q
    g = torch.Generator(device=dev).manual_seed(41)
    q = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
    k = (torch.randn((S, H, 128), generator=g, device=dev) +
         3.0 * torch.randn((1, H, 128), generator=g, device=dev)).to(torch.bfloat16)
    v = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
    res = {}
    for name, flags in (("per_token_f16", 0), ("block128_bf16", h3q.ATTN_SCALE_BLOCK128 | h3q.ATTN_PV_BF16)):
        for _ in range(2):
            h3q.attention(q, k, v, flags)
        km = h3q.attn_kmean(k)
        q8, qs = h3q.attn_quant_heads(q, None, flags)
        k8, ks = h3q.attn_quant_heads(k, km, flags)
        vt = h3q.attn_v_layout(v.reshape(S, H * 128), H * 128, 0, S, H, flags)
        h3q.attention_core(q8, qs, k8, ks, vt, flags)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        for _ in range(reps):
            h3q.attention(q, k, v, flags)
        ev[1].record()
        for _ in range(reps):
            h3q.attention_core(q8, qs, k8, ks, vt, flags)
        ev[2].record()
        torch.cuda.synchronize()
        ms_all = ev[0].elapsed_time(ev[1]) / reps
        ms_core = ev[1].elapsed_time(ev[2]) / reps
        half = 2.0 * S * S * 128 * H
        res[name] = {"ms_pipeline": round(ms_all, 3), "ms_kernel": round(ms_core, 3),
                     "tops_pipeline": round(2 * half / (ms_all * 1e-3) / 1e12, 1),
                     "tops_kernel": round(2 * half / (ms_core * 1e-3) / 1e12, 1),
                     "kernel_time_at_peaks_ms": round((half / (2 * peaks["bf16_tflops"] * 1e12) +
                                                       half / (peaks["bf16_tflops"] * 1e12)) * 1e3, 3)}
        res[name]["frac_of_tensor_roofline"] = round(res[name]["kernel_time_at_peaks_ms"] / ms_core, 3)
    res["device_status"] = h3q.device_status(dev.index or 0)
    return {"workload": f"BASELINE c4 attention: B1 H{H} D128 S{S}, non-causal", "modes": res,
            "note": "tops = 4 S^2 D H / time (the reference's count); roofline = QK at 2x bf16 burst + PV at bf16 "
                    "burst, serial"}


def attend_step_c4(dev, reps: int = 5, S: int = 32760, H: int = 40, rot: int = 96) -> dict:
    """The DiT's whole attention step (dit.rs:741-757) at config 4's shape: q / k RMSNorm + RoPE out of the fused
    qkv [S, 3 H 128], then the int8 attention with V read from the qkv rows (block-128 scales, bf16 P.V).  "fused"
    is h3q_attend_qkv (the normalised, rotated q / k never reach memory); "unfused" is h3q_qk_norm_rope twice then
    h3q_attention_qkv, as the reference runs it.  The rope table is [2, S, 48] (three axes of 16 frequencies)."""
    import torch
    import h3q
    g = torch.Generator(device=dev).manual_seed(43)
    inner = H * 128
    qkv = (2.0 * torch.randn((S, 3 * inner), generator=g, device=dev)).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    kw = (1 + 0.2 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    ang = 100.0 * torch.rand((S, rot // 2), generator=g, device=dev)
    cs = torch.stack([ang.cos(), ang.sin()]).to(torch.bfloat16).float().contiguous()
    flags = h3q.ATTN_SCALE_BLOCK128 | h3q.ATTN_PV_BF16

    def unfused():
        q = h3q.qk_norm_rope(qkv, 0, H, 128, (qw, 1e-6), cs, rot)
        k = h3q.qk_norm_rope(qkv, inner, H, 128, (kw, 1e-6), cs, rot)
        return h3q.attention_qkv(q, k, qkv, 2 * inner, flags)

    res = {}
    for name, fn in (("fused", lambda: h3q.attend_qkv(qkv, H, (qw, kw), 1e-6, cs, rot, flags)), ("unfused", unfused)):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name + "_ms"] = round(e0.elapsed_time(e1) / reps, 3)
    res["workload"] = f"DiT attention step: qk RMSNorm + RoPE (rot {rot}) + int8 attention, B1 H{H} D128 S{S}"
    res["device_status"] = h3q.device_status(dev.index or 0)
    return res


def streaming_c1(layers, M: int, dev, reps: int = 3) -> dict:
    """The config-1 step with its weights kept in pinned host memory and streamed to the GPU through a 2-slot ring
    (h3q_streamer; the reference's copy-stream uploads for weights that do not stay on the GPU, weights.rs:185-273):
    the copy of linear i+1 runs on the copy stream while linear i computes.  Compared with the same step on resident
    weights and with the copies alone; the weight bytes cross PCIe every step, so the bound is the slower of the
    two."""
    import torch
    import h3q
    from h3q.streaming import WeightStreamer
    host = [(ly["w"].cpu().pin_memory(), ly["ws"].cpu().pin_memory(), ly["b"].cpu().pin_memory()) for ly in layers]
    slot = max(w.numel() + 4 * (s.numel() + b.numel()) for w, s, b in host) + 1024
    ws = WeightStreamer(slot, 2, dev)
    L = h3q.lib()
    sp = torch.cuda.current_stream(dev).cuda_stream

    def linear(ly, w, s, b):
        h3q.check(L.h3q_quant_rows_i8(ly["x"].data_ptr(), 2, ly["q"].data_ptr(), ly["xs"].data_ptr(), M, ly["k"], 1, sp))
        h3q.check(L.h3q_gemm_s8_quantized(ly["q"].data_ptr(), ly["xs"].data_ptr(), w.data_ptr(), s.data_ptr(), ly["n"],
                                          b.data_ptr(), ly["out"].data_ptr(), 2, M, ly["n"], ly["k"], h3q.EPI_LINEAR,
                                          None, None, None, sp))

    pending = []

    def streamed():
        # enqueue linear i, then fetch linear i+1: the fetch's wait lands on the compute stream after linear i, so
        # the copy overlaps it (the first fetch of a step overlaps the previous step's last linear)
        if not pending:
            pending.append(ws.fetch(list(host[0])))
        for i, ly in enumerate(layers):
            (w, s, b), k = pending.pop(0)
            linear(ly, w, s, b)
            ws.release(k)
            pending.append(ws.fetch(list(host[(i + 1) % len(layers)])))

    def resident():
        for ly in layers:
            linear(ly, ly["w"], ly["ws"], ly["b"])

    def copies_only():
        while pending:
            ws.release(pending.pop(0)[1])
        for i in range(len(layers)):
            _, k = ws.fetch(list(host[i]))
            ws.release(k)

    res = {}
    for name, fn in (("resident", resident), ("streamed", streamed), ("copies_only", copies_only)):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name + "_ms"] = round(e0.elapsed_time(e1) / reps, 3)
    wbytes = sum(w.numel() + 4 * (s.numel() + b.numel()) for w, s, b in host)
    res["weight_bytes_per_step"] = wbytes
    res["h2d_gbs"] = round(wbytes / (res["copies_only_ms"] * 1e-3) / 1e9, 1)
    # the step can be no faster than the slower of its compute and its weight copies
    res["overlap_efficiency"] = round(max(res["resident_ms"], res["copies_only_ms"]) / res["streamed_ms"], 3)
    torch.cuda.synchronize()
    for (_, k) in pending:
        ws.release(k)
    ws.close()
    return res


def modulate_fused(dev, peaks: dict, reps: int = 10, M: int = 32760, C: int = 5120) -> dict:
    """The step in front of the qkv and fc1 linears: RMSNorm + adaLN modulate, then the rotated int8 quantizer.
    "two_pass" runs h3q_rms_modulate (bf16 row to memory) then h3q_quant_rows_i8, as the reference's
    rms_modulate + gemm_s8 do; "fused" is h3q_rms_modulate_quant.  HBM bytes counted as the fused pass's:
    2C read + C + 4 written per row (the adaLN tables stay in L2)."""
    import torch
    import h3q
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn((M, C), generator=g, device=dev).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    sc = 0.5 * torch.randn((6, C), generator=g, device=dev)
    sh = 0.5 * torch.randn((6, C), generator=g, device=dev)
    # table row of each token: its latent frame (21 frames of 1560 tokens at c1), as the DiT indexes its adaLN rows
    idx = ((torch.arange(M, device=dev) // 1560) % 6).to(torch.int32)
    res = {}
    for name, fn in (("two_pass", lambda: h3q.quant_rows(h3q.rms_modulate(x, w, 1e-6, sc, sh, idx), True)),
                     ("fused", lambda: h3q.rms_modulate_quant(x, w, 1e-6, sc, sh, idx))):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[name] = {"ms": round(ms, 4), "gbs_of_fused_bytes": round((3.0 * M * C + 4.0 * M) / (ms * 1e-3) / 1e9, 1)}
    res["workload"] = f"rms_modulate + rotated int8 quantization of the qkv input, M={M} C={C}"
    res["frac_of_hbm"] = round(res["fused"]["gbs_of_fused_bytes"] / peaks["hbm_gbs"], 3)
    return res


def lora_merge(dev, reps: int = 3, n: int = 15360, k: int = 5120, rank: int = 64) -> dict:
    """Load-time LoRA merge (QLinear::merge_loras, weights.rs:716-757) of the c1 qkv layer: dequantize, undo ConvRot,
    add one rank-64 bf16 delta, rotate, requantize per row (h3q_lora_merge_i8).  Work counted: the delta's
    2 n k r flops and the int8 weight read and written."""
    import torch
    import h3q
    g = torch.Generator(device=dev).manual_seed(13)
    w = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
    s = torch.rand(n, generator=g, device=dev) * 1e-2 + 1e-3
    a = (0.05 * torch.randn((rank, k), generator=g, device=dev)).to(torch.bfloat16)
    b = (0.05 * torch.randn((n, rank), generator=g, device=dev)).to(torch.bfloat16)
    loras = [(a, b, 0.5)]
    out = torch.empty_like(w)
    out_s = torch.empty(n, dtype=torch.float32, device=dev)
    for _ in range(2):
        h3q.lora_merge_i8(w, s, loras, out=out, out_scale=out_s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        h3q.lora_merge_i8(w, s, loras, out=out, out_scale=out_s)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    return {"workload": f"int8 ConvRot layer [{n}, {k}] + one rank-{rank} bf16 delta", "ms": round(ms, 3),
            "delta_tflops": round(2.0 * n * k * rank / (ms * 1e-3) / 1e12, 1),
            "note": "includes the workspace allocation of each call; f32 FMA chains on the CUDA cores"}


def dit_block_c4(dev, reps: int = 3, S: int = 32760, H: int = 40, F: int = 13824, rot: int = 96) -> dict:
    """One whole DiT block (Dit::run_block, dit.rs:969-1021) at config 4's shape: modulate, qkv, the attention step,
    out + gated residual, modulate, fc1 + SwiGLU, fc2 + gated residual.  "ops" issues the reference's calls one by
    one (h3q.dit.run_block_ops); "fused" is h3q.dit.run_block (the modulation feeds the quantizer, SwiGLU and the
    gated residuals run in the GEMM epilogues).  gemm_tops counts the four linears' 2 S N K only."""
    import torch
    import h3q
    from h3q import dit as D
    g = torch.Generator(device=dev).manual_seed(47)
    C = H * 128

    def lin(n, k):
        return D.Linear(torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8),
                        torch.rand(n, generator=g, device=dev) * 2e-3 + 5e-4,
                        0.02 * torch.randn(n, generator=g, device=dev))
    nw = lambda: (1 + 0.1 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    hw = lambda: (1 + 0.2 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    blk = D.Block(lin(3 * C, C), lin(C, C), lin(2 * F, C), lin(C, F), nw(), nw(), hw(), hw(), H)
    tab = lambda: 0.5 * torch.randn((6, C), generator=g, device=dev)
    gate = lambda: torch.rand((6, C), generator=g, device=dev)
    idx = ((torch.arange(S, device=dev) // 1560) % 6).to(torch.int32)
    ang = 100.0 * torch.rand((S, rot // 2), generator=g, device=dev)
    cs = torch.stack([ang.cos(), ang.sin()]).to(torch.bfloat16).float().contiguous()
    cx = D.StepCtx(tab(), tab(), gate(), tab(), tab(), gate(), idx, cs, rot,
                   h3q.ATTN_SCALE_BLOCK128 | h3q.ATTN_PV_BF16)
    x = torch.randn((S, C), generator=g, device=dev).to(torch.bfloat16)
    res = {}
    for name, fn in (("fused", D.run_block), ("ops", D.run_block_ops)):
        for _ in range(2):
            fn(x, blk, cx)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn(x, blk, cx)
        e1.record()
        torch.cuda.synchronize()
        res[name + "_ms"] = round(e0.elapsed_time(e1) / reps, 3)
    ops = 2.0 * S * C * (3 * C + C + 2 * F + F)
    res["gemm_tops_per_block"] = round(ops / 1e12, 2)
    res["same_bits"] = bool(torch.equal(D.run_block(x, blk, cx).view(torch.int16),
                                        D.run_block_ops(x, blk, cx).view(torch.int16)))
    res["workload"] = f"DiT block S{S} C{C} H{H} F{F} (fc1 {2 * F} interleaved rows), rope rot {rot}"
    res["device_status"] = h3q.device_status(dev.index or 0)
    return res


def make_layers(M: int, dev, rank: int = 0) -> list:
    """The four c1 linears with M activation rows: weights from one seed shared by every rank (replicated),
    activations ~N(0, 1) with 8 outlier channels x20 from a per-rank seed."""
    import torch
    gw = torch.Generator(device=dev).manual_seed(1234)
    gx = torch.Generator(device=dev).manual_seed(4321 + rank)
    layers = []
    for name, k, n in LINEARS:
        x = torch.randn((M, k), generator=gx, device=dev)
        oc = torch.randperm(k, generator=gx, device=dev)[:8]
        x[:, oc] *= 20.0
        x = x.to(torch.bfloat16)
        w = torch.randint(-127, 128, (n, k), generator=gw, device=dev, dtype=torch.int8)
        wsc = torch.rand(n, generator=gw, device=dev) * 9e-3 + 1e-3
        b = (torch.randn(n, generator=gw, device=dev) * 0.02).to(torch.bfloat16).float()
        layers.append(dict(name=name, k=k, n=n, m=M, x=x, w=w, ws=wsc, b=b,
                           q=torch.empty((M, k), dtype=torch.int8, device=dev),
                           xs=torch.empty(M, dtype=torch.float32, device=dev),
                           out=torch.empty((M, n), dtype=torch.bfloat16, device=dev)))
    return layers


def run_linear(L, ly, sp) -> None:
    """One c1 linear through the C ABI: the rotated quantizer, then the GEMM with the linear epilogue."""
    import h3q
    h3q.check(L.h3q_quant_rows_i8(ly["x"].data_ptr(), 2, ly["q"].data_ptr(), ly["xs"].data_ptr(), ly["m"], ly["k"],
                                  1, sp))
    h3q.check(L.h3q_gemm_s8_quantized(ly["q"].data_ptr(), ly["xs"].data_ptr(), ly["w"].data_ptr(),
                                      ly["ws"].data_ptr(), ly["n"], ly["b"].data_ptr(), ly["out"].data_ptr(),
                                      2, ly["m"], ly["n"], ly["k"], h3q.EPI_LINEAR, None, None, None, sp))


def tile_waves(M: int, N: int, units: int = 74) -> dict:
    """How a linear's 256 x 256 GEMM tiles fill the persistent grid (one CTA pair per tile, `units` pairs)."""
    tiles = -(-M // 256) * -(-N // 256)
    waves = -(-tiles // units)
    return {"tiles": tiles, "waves": round(tiles / units, 2), "wave_efficiency": round(tiles / (waves * units), 3)}


def time_steps(fn, reps: int, dev) -> float:
    """CUDA-event ms per call of fn (after two untimed calls)."""
    import torch
    for _ in range(2):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / reps


def c2_block(dev, peaks: dict, reps: int = 5) -> dict:
    """the fused-epilogue DiT linears at M = 65520 (a CFG pair of 32760-token halves sharing the
    weights).  up-proj 5120 -> 13824 with the GELU-tanh epilogue, whose output is the down-proj's input,
    13824 -> 5120 with the residual + gate epilogue (gate bf16 per channel ~U(0,1), residual bf16 ~N(0,1)).  Each
    linear is the rotated quantizer then the GEMM; CUDA-event time per linear."""
    import torch
    import h3q
    M, C, F = 65520, 5120, 13824
    g = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn((M, C), generator=g, device=dev)
    x[:, torch.randperm(C, generator=g, device=dev)[:8]] *= 20.0
    x = x.to(torch.bfloat16)
    w1 = torch.randint(-127, 128, (F, C), generator=g, device=dev, dtype=torch.int8)
    w2 = torch.randint(-127, 128, (C, F), generator=g, device=dev, dtype=torch.int8)
    ws1, ws2 = (torch.rand(n, generator=g, device=dev) * 9e-3 + 1e-3 for n in (F, C))
    b1, b2 = ((torch.randn(n, generator=g, device=dev) * 0.02).to(torch.bfloat16).float() for n in (F, C))
    gate = torch.rand((1, C), generator=g, device=dev).to(torch.bfloat16).float()
    resid = torch.randn((M, C), generator=g, device=dev).to(torch.bfloat16)
    up = torch.empty((M, F), dtype=torch.bfloat16, device=dev)
    down = torch.empty((M, C), dtype=torch.bfloat16, device=dev)

    def up_proj():
        q, xs = h3q.quant_rows(x, True)
        h3q.gemm_s8_quantized(q, xs, w1, ws1, b1, h3q.EPI_GELU_TANH, out=up)

    def down_proj():
        q, xs = h3q.quant_rows(up, True)
        h3q.gemm_s8_quantized(q, xs, w2, ws2, b2, h3q.EPI_GATE_RESID, gate=gate, resid=resid, out=down)

    res = {}
    for name, fn, k, n in (("up_gelu", up_proj, C, F), ("down_gate_resid", down_proj, F, C)):
        ms = time_steps(fn, reps, dev)
        tops = 2.0 * M * k * n / (ms * 1e-3) / 1e12
        res[name] = {"linear": f"{k}->{n}", "ms": round(ms, 3), "tops": round(tops, 1),
                     "frac_of_2x_bf16_burst": round(tops / (2 * peaks["bf16_tflops"]), 3)}
    res["workload"] = "BASELINE c2: M=65520 (CFG pair), fc1 GELU-tanh epilogue, fc2 residual + gate epilogue"
    res["note"] = "time per linear includes its rotated quantizer; workspace allocations by torch's caching allocator"
    res["device_status"] = h3q.device_status(dev.index or 0)
    return res


def gpu_comparators(layers, dev, per_linear, reps: int = 5) -> dict:
    """The reference's cuBLASLt path on the same GPU, GEMM part: int8 x int8 -> int32 (the H3_GEMM=cublaslt GEMM of
    kernels.rs:1008-1044; here through torch._int_mm, which issues the same cuBLASLt IMMA: row-major [M, K] codes
    times the [N, K] weight transposed) at each c1 shape, against this library's GEMM writing the same int32
    accumulators (H3Q_EPI_ACC_I32) and its fused bf16 epilogue.  The reference adds a separate epilogue kernel
    reading the int32 result back (kernels.rs:333-373), not timed here; the fused GEMM needs none."""
    import torch
    import h3q
    res = []
    for ly, pl in zip(layers, per_linear):
        acc = torch.empty((ly["m"], ly["n"]), dtype=torch.int32, device=dev)
        wt = ly["w"].t()
        lt_ms = time_steps(lambda: torch._int_mm(ly["q"], wt), reps, dev)
        ours_ms = time_steps(lambda: h3q.gemm_s8_quantized(ly["q"], ly["xs"], ly["w"], ly["ws"], None,
                                                           h3q.EPI_ACC_I32, out=acc), reps, dev)
        same = bool(torch.equal(torch._int_mm(ly["q"], wt), acc))
        ops = 2.0 * ly["m"] * ly["k"] * ly["n"]
        res.append({"linear": f"{ly['name']}:{ly['k']}x{ly['n']}", "cublaslt_int32_ms": round(lt_ms, 4),
                    "cublaslt_tops": round(ops / (lt_ms * 1e-3) / 1e12, 1),
                    "ours_int32_ms": round(ours_ms, 4), "ours_int32_tops": round(ops / (ours_ms * 1e-3) / 1e12, 1),
                    "ours_fused_bf16_ms": pl["gemm_ms"],
                    "speedup_int32": round(lt_ms / ours_ms, 3), "speedup_vs_fused": round(lt_ms / pl["gemm_ms"], 3),
                    "same_int32": same})
        del acc
    return {"layers": res, "M": layers[0]["m"],
            "note": "cuBLASLt via torch._int_mm; time of the GEMM only; same_int32 = identical accumulators"}


def _max_over_ranks(ms: float, dist, dev) -> float:
    import torch
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def multi_gpu_extras(dist, dev, reps: int = 3) -> dict:
    """At N > 1 GPUs, besides the strong-scaling headline (all ranks take part; times are CUDA events, max over
    ranks; every result is checked against the single-GPU result on the same rank and `parity` is the AND over
    ranks and checks):
      weak:      every rank runs the four c1 linears on its own 32760 tokens (no collective);
      nsplit:    the four c1 linears with the weight rows split over the ranks and the activations replicated
                 (M = 32760 in total, strong scaling), through h3q_gemm_s8_nsplit: "fused" is one GEMM per rank
                 storing its column block into every rank's output over NVLink, "push" the GEMM in row chunks with
                 the copy engines forwarding each finished chunk, "nccl" a local GEMM + ncclAllGather + relayout,
                 "peer" the GEMM then a kernel on every SM storing the column block into the peers' outputs,
                 "push_shard_quant" push with each rank quantizing only its row block and all-gathering the codes;
                 exchange_ms = the form's time minus the local work alone (compute_only_ms); each output must
                 equal, bit for bit, the whole linear computed on one GPU (the weak run's output of the same
                 activations); allgather_alone times the all-gather of the nccl form's column blocks by itself,
                 the link's ceiling for the exchange;
      attention: query-sharded c4 attention (S = 32760, H = 40 in total): K/V rows all-gathered, each rank attends
                 its 32760 / N queries (h3q_attention_rows); its rows must equal those of the whole-sequence
                 attention computed on one GPU."""
    import torch
    import h3q
    from h3q import parallel as P
    world = dist.get_world_size()
    rank = dist.get_rank()
    M = M_TOKENS
    L = h3q.lib()
    sp = torch.cuda.current_stream(dev).cuda_stream
    layers = make_layers(M, dev, rank=0)  # the same activations on every rank (the N split replicates them)
    checks = {}

    def step_weak():
        for ly in layers:
            run_linear(L, ly, sp)
    step_weak()
    torch.cuda.synchronize()
    dist.barrier()
    ms = _max_over_ranks(time_steps(step_weak, reps, dev), dist, dev)
    weak = {"ms_per_step": round(ms, 3), "tops": round(world * ops_per_step(M) / (ms * 1e-3) / 1e12, 1),
            "note": "32760 tokens per GPU, value = all ranks' ops / max time"}
    rows = torch.tensor([0, 1, 4095, 16380, 24571, M - 1], device=dev)
    comm = P.Comm(dev)
    res = {}
    # the local work alone (quantize all rows, GEMM of this rank's columns), to itemise the exchange
    lins = [P.NSplitLinear(ly["w"], ly["ws"], ly["b"], comm, mode="nccl") for ly in layers]

    def compute_only():
        for lin, ly in zip(lins, layers):
            q, xs = h3q.quant_rows(ly["x"], True)
            h3q.gemm_s8_quantized(q, xs, lin.w, lin.ws, lin.bias, h3q.EPI_LINEAR)
    dist.barrier()
    compute_ms = _max_over_ranks(time_steps(compute_only, reps, dev), dist, dev)
    del lins
    for name, mode, shard in (("fused", "fused", False), ("push", "push", False), ("nccl", "nccl", False),
                              ("peer", "peer", False), ("push_shard_quant", "push", True)):
        lins = [P.NSplitLinear(ly["w"], ly["ws"], ly["b"], comm, mode=mode, shard_quant=shard) for ly in layers]
        outs = [None] * len(lins)

        def step():
            for i, (lin, ly) in enumerate(zip(lins, layers)):
                outs[i] = lin.forward(ly["x"])
        step()
        torch.cuda.synchronize()
        ok = all(torch.equal(o.index_select(0, rows).view(torch.int16), ly["out"].index_select(0, rows).view(torch.int16))
                 for o, ly in zip(outs, layers))
        checks["nsplit_" + name] = ok
        dist.barrier()
        ms = _max_over_ranks(time_steps(step, reps, dev), dist, dev)
        res[name] = {"ms_per_step": round(ms, 3), "tops": round(ops_per_step(M) / (ms * 1e-3) / 1e12, 1),
                     "exchange_ms": round(ms - compute_ms, 3)}
        outs = None
        for lin in lins:
            lin.close()
        torch.cuda.synchronize()
        dist.barrier()
    res["compute_only_ms"] = round(compute_ms, 3)
    res["output_bytes_received_per_rank"] = int(sum(M * ly["n"] * 2 for ly in layers) * (world - 1) / world)
    # the exchange alone: the library's all-gather (NCCL) of each layer's [M, n_max] column blocks, the bytes the
    # nccl form moves, with no GEMM and no relayout -- what the link delivers to the N split
    widths = [max(hi - lo for lo, hi in (P.nsplit_range(ly["n"], world, r) for r in range(world))) for ly in layers]
    send = torch.zeros(M * max(widths), dtype=torch.bfloat16, device=dev)
    recv = torch.empty(world * M * max(widths), dtype=torch.bfloat16, device=dev)

    def gather_only():
        for wd in widths:
            comm.allgather(send[:M * wd], recv[:world * M * wd])
    gather_only()
    dist.barrier()
    ms = _max_over_ranks(time_steps(gather_only, reps, dev), dist, dev)
    moved = sum((world - 1) * M * wd * 2 for wd in widths)
    res["allgather_alone"] = {"ms": round(ms, 3), "bytes_received_per_rank": moved,
                              "gbs_received_per_rank": round(moved / (ms * 1e-3) / 1e9, 1)}
    del send, recv
    del layers
    S, H = 32760, 40
    lo, hi = P.row_range(S, world, rank)
    g = torch.Generator(device=dev).manual_seed(77)  # the same sequence on every rank; each keeps its rows
    q = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
    k = (torch.randn((S, H, 128), generator=g, device=dev) +
         3.0 * torch.randn((1, H, 128), generator=g, device=dev)).to(torch.bfloat16)
    v = torch.randn((S, H, 128), generator=g, device=dev).to(torch.bfloat16)
    ql, kl, vl = (t[lo:hi].contiguous() for t in (q, k, v))
    got = P.sharded_attention(ql, kl, vl, S, comm=comm)
    whole = h3q.attention(q, k, v)
    torch.cuda.synchronize()
    checks["attention_query_sharded"] = bool(torch.equal(got.view(torch.int16), whole[lo:hi].view(torch.int16)))
    del whole, q, k, v
    dist.barrier()
    ms = _max_over_ranks(time_steps(lambda: P.sharded_attention(ql, kl, vl, S, comm=comm), reps, dev), dist, dev)
    att = {"ms": round(ms, 3), "tops": round(4.0 * S * S * 128 * H / (ms * 1e-3) / 1e12, 1),
           "note": "K/V all-gather + kmean/quant of the full K + attention of this rank's query rows"}
    flag = torch.tensor([1 if all(checks.values()) else 0], device=dev, dtype=torch.int32)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    comm.close()
    return {"weak_c1_linears": weak,
            "nsplit_c1_linears": dict(res, workload="c1 linears, N split, M=32760 in total (strong scaling)"),
            "attention_c4_query_sharded": att, "parity": bool(flag.item()), "parity_checks_rank0": checks,
            "device_status": h3q.device_status(dev.index or 0)}


def run_profile_case(args) -> None:
    """One fc1-shaped linear at 4096 tokens (A 21 MB, W 71 MB, out 113 MB: more than L2 in total, a few hundred
    MB on the device): warmup + steps launches of the quantizer and the GEMM, for ncu --set full captures."""
    import torch
    import h3q
    dev = torch.device("cuda", 0)
    M, K, N = 4096, 5120, 13824
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn((M, K), generator=g, device=dev).to(torch.bfloat16)
    w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
    wsc = torch.rand(N, generator=g, device=dev) * 9e-3 + 1e-3
    b = torch.zeros(N, device=dev)
    for _ in range(args.warmup + args.steps):
        q, xs = h3q.quant_rows(x, True)
        h3q.gemm_s8_quantized(q, xs, w, wsc, b, h3q.EPI_LINEAR)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": f"M={M} K={K} N={N}", "launches": 2 * (args.warmup + args.steps),
                      "device_status": h3q.device_status(0)}))


def run_profile_linears(args) -> None:
    """The four c1 linears (quantizer + GEMM each) at args.profile_linears tokens: warmup + steps passes, for
    ncu DRAM-traffic captures on a smaller case than the bench's 32760 tokens (8192 tokens hold ~1.5 GB)."""
    import torch
    import h3q
    dev = torch.device("cuda", 0)
    layers = make_layers(args.profile_linears, dev)
    L = h3q.lib()
    sp = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(args.warmup + args.steps):
        for ly in layers:
            run_linear(L, ly, sp)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": f"c1 linears at M={args.profile_linears}",
                      "launches": 8 * (args.warmup + args.steps), "device_status": h3q.device_status(0)}))


def run_profile_rope(args) -> None:
    """qk_norm_rope of the q part of a fused qkv, S=16384, H=40, rot 96: warmup + steps launches of
    qk_norm_rope128_kernel (q heads 168 MB in, 168 MB out)."""
    import torch
    import h3q
    dev = torch.device("cuda", 0)
    S, H = 16384, 40
    g = torch.Generator(device=dev).manual_seed(3)
    qkv = (2.0 * torch.randn((S, 3 * H * 128), generator=g, device=dev)).to(torch.bfloat16)
    qw = (1 + 0.2 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    ang = 100.0 * torch.rand((S, 48), generator=g, device=dev)
    cs = torch.stack([ang.cos(), ang.sin()]).to(torch.bfloat16).float().contiguous()
    for _ in range(args.warmup + args.steps):
        h3q.qk_norm_rope(qkv, 0, H, 128, (qw, 1e-6), cs, 96)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": f"qk_norm_rope S={S} H={H} rot=96", "launches": args.warmup + args.steps,
                      "device_status": h3q.device_status(0)}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-nvfp4", action="store_true",
                    help="small case for ncu captures: the two NVFP4 text-encoder linears only")
    ap.add_argument("--profile-attn", action="store_true",
                    help="small case for ncu captures: the attention pipeline at S=8192, H=4")
    ap.add_argument("--profile-rope", action="store_true",
                    help="small case for ncu captures: qk_norm_rope of the q heads at S=16384, H=40, rot 96")
    ap.add_argument("--profile-modulate", action="store_true",
                    help="small case for ncu captures: rms_modulate + rotated int8 quantization at M=8192, C=5120")
    ap.add_argument("--profile-lora", action="store_true",
                    help="small case for ncu captures: the LoRA merge of a 4096 x 5120 int8 layer, rank 64")
    ap.add_argument("--profile", action="store_true",
                    help="small case for ncu captures: one 4096-token fc1 linear (quant + GEMM), nothing else")
    ap.add_argument("--profile-linears", type=int, default=0, metavar="M",
                    help="small case for ncu captures: the four c1 linears at M tokens, nothing else")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.profile:
        run_profile_case(args)
        return
    if args.profile_linears:
        run_profile_linears(args)
        return
    if args.profile_rope:
        run_profile_rope(args)
        return
    if args.profile_modulate:
        import torch
        print(json.dumps(modulate_fused(torch.device("cuda", 0), load_peaks(), reps=args.steps, M=8192)))
        return
    if args.profile_lora:
        import torch
        print(json.dumps(lora_merge(torch.device("cuda", 0), reps=args.steps, n=4096)))
        return
    if args.profile_nvfp4:
        import torch
        print(json.dumps(nvfp4_c3(torch.device("cuda", 0), load_peaks(), reps=args.steps)))
        return
    if args.profile_attn:
        import torch
        print(json.dumps(attention_c4(torch.device("cuda", 0), load_peaks(), reps=args.steps, S=8192, H=4)))
        return

    import torch
    import h3q

    ws_n, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if ws_n > 1:
        import datetime
        import torch.distributed as dist
        # NCCL announces its version on stdout while the communicator is created; keep stdout for the JSON line
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    if not h3q.available_arch(local):
        raise SystemExit("bench.py: this library needs an sm_100 (B200) GPU")

    # strong scaling: the 32760 tokens of the step split over the ranks (row_range), weights replicated
    lo_r, hi_r = row_range(M_TOKENS, ws_n, rank)
    M = hi_r - lo_r
    layers = make_layers(M, dev, rank)
    L = h3q.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def one_step(events=None):
        for i, ly in enumerate(layers):
            if events is not None:
                events[i][0].record(stream)
            h3q.check(L.h3q_quant_rows_i8(ly["x"].data_ptr(), 2, ly["q"].data_ptr(), ly["xs"].data_ptr(), M, ly["k"],
                                          1, sp))
            if events is not None:
                events[i][1].record(stream)
            h3q.check(L.h3q_gemm_s8_quantized(ly["q"].data_ptr(), ly["xs"].data_ptr(), ly["w"].data_ptr(),
                                              ly["ws"].data_ptr(), ly["n"], ly["b"].data_ptr(), ly["out"].data_ptr(),
                                              2, M, ly["n"], ly["k"], h3q.EPI_LINEAR, None, None, None, sp))
            if events is not None:
                events[i][2].record(stream)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in LINEARS] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record(stream)
        for s in range(args.steps):
            one_step(ev[s])
        stop.record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(stop)
    if dist is not None:
        t = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_step = elapsed_ms / args.steps
    # strong scaling: every step of the job processes the 32760 tokens once, split over the ranks
    value = ops_per_step(M_TOKENS) / (ms_step * 1e-3) / 1e12
    status = h3q.device_status(local)
    if status:
        raise SystemExit(f"bench.py: a kernel reported device error {status}")

    # per-kernel averages inside the timed region
    gemm_ms = sum(ev[s][i][1].elapsed_time(ev[s][i][2]) for s in range(args.steps) for i in range(len(LINEARS)))
    quant_ms = sum(ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps) for i in range(len(LINEARS)))
    launches = args.steps * len(LINEARS)
    gemm_ops_launch = ops_per_step(M) / len(LINEARS)
    gemm_avg_ms = gemm_ms / launches
    quant_bytes_launch = sum(3.0 * M * k + 4.0 * M for _, k, _ in LINEARS) / len(LINEARS)
    quant_avg_ms = quant_ms / launches
    per_linear = []
    for i, (nm, k, n) in enumerate(LINEARS):
        g_ms = sum(ev[s][i][1].elapsed_time(ev[s][i][2]) for s in range(args.steps)) / args.steps
        q_ms = sum(ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps)) / args.steps
        per_linear.append({"linear": f"{nm}:{k}x{n}", "m": M, "gemm_ms": round(g_ms, 4),
                           "gemm_tops": round(2.0 * M * k * n / (g_ms * 1e-3) / 1e12, 1), "quant_ms": round(q_ms, 4),
                           "quant_gbs": round((3.0 * M * k + 4.0 * M) / (q_ms * 1e-3) / 1e9, 1),
                           **tile_waves(M, n)})
    peaks = load_peaks()
    # the GEMM runs inside the timed step: when the power cap engaged during it (sw_power_cap among the reasons the
    # clock samples inside the region show), the denominator is the sustained (power-capped) bf16 figure, else the
    # burst figure; both fractions are reported
    clocks = clk.summary()
    capped = "sw_power_cap" in clocks.get("reasons", [])
    int8_burst = 2.0 * peaks["bf16_tflops"]
    int8_sustained = 2.0 * peaks["bf16_tflops_sustained"]
    int8_peak = int8_sustained if capped else int8_burst
    achieved = gemm_ops_launch / (gemm_avg_ms * 1e-3) / 1e12
    q_achieved = quant_bytes_launch / (quant_avg_ms * 1e-3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemm_i8_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")

    # end to end through the C ABI with host buffers: every linear's input comes from pinned host memory and its
    # output goes back to it.  The step's four linears go to h3q_host_pipeline_run as one batch: chunked copies in
    # and out overlap the GEMMs, and each linear's copies in overlap the previous linear's last GEMMs and copies out.
    e2e = None
    if rank == 0 or True:
        host_x = [ly["x"].cpu().pin_memory() for ly in layers]
        host_o = [torch.empty((M, ly["n"]), dtype=torch.bfloat16).pin_memory() for ly in layers]
        pipe = ctypes.c_void_p()
        # 32 input chunk buffers (1.8 GB): fc2's wide inputs cross PCIe while qkv and fc1 are bound by their copies out
        h3q.check(L.h3q_host_pipeline_create_ex(E2E_CHUNK, max(ly["k"] for ly in layers),
                                                max(ly["n"] for ly in layers), E2E_IN_SLOTS, 2, ctypes.byref(pipe)))

        items = (h3q.HostLinear * len(layers))()
        for i, ly in enumerate(layers):
            items[i] = h3q.HostLinear(host_x[i].data_ptr(), ly["w"].data_ptr(), ly["ws"].data_ptr(), ly["n"],
                                      ly["b"].data_ptr(), host_o[i].data_ptr(), M, ly["n"], ly["k"], 0, 1)

        def e2e_step():
            h3q.check(L.h3q_host_pipeline_run(pipe, items, len(layers), sp))

        e2e_step()
        torch.cuda.synchronize()
        e_steps = max(2, min(args.steps, 5))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / e_steps
        if dist is not None:
            t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        # the link bound of the same step: its copies alone, in the same chunks, both directions at once
        cin, cout = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        dx = torch.empty(E2E_CHUNK * max(ly["k"] for ly in layers), dtype=torch.bfloat16, device=dev)
        do = torch.empty(E2E_CHUNK * max(ly["n"] for ly in layers), dtype=torch.bfloat16, device=dev)

        def copies_only():
            cin.wait_stream(stream)
            cout.wait_stream(stream)
            for h, ly in zip(host_x, layers):
                flat = h.view(-1)
                with torch.cuda.stream(cin):
                    for r0 in range(0, M, E2E_CHUNK):
                        n_el = (min(M, r0 + E2E_CHUNK) - r0) * ly["k"]
                        dx[:n_el].copy_(flat[r0 * ly["k"]:r0 * ly["k"] + n_el], non_blocking=True)
            for h, ly in zip(host_o, layers):
                flat = h.view(-1)
                with torch.cuda.stream(cout):
                    for r0 in range(0, M, E2E_CHUNK):
                        n_el = (min(M, r0 + E2E_CHUNK) - r0) * ly["n"]
                        flat[r0 * ly["n"]:r0 * ly["n"] + n_el].copy_(do[:n_el], non_blocking=True)
            stream.wait_stream(cin)
            stream.wait_stream(cout)

        copies_only()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(e_steps):
            copies_only()
        e1.record(stream)
        torch.cuda.synchronize()
        link_ms = e0.elapsed_time(e1) / e_steps
        e2e = {"value": ops_per_step(M_TOKENS) / (e_ms * 1e-3) / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": int(sum(h.numel() * 2 for h in host_x)),
               "d2h_bytes_per_step": int(sum(h.numel() * 2 for h in host_o)), "ms_per_step": e_ms,
               "link_bound": {"copies_only_ms": link_ms, "frac": link_ms / e_ms,
                              "note": "the step's copies alone, same chunks, both PCIe directions at once"},
               "path": f"h3q_host_pipeline_run (C ABI), the four linears as one batch: pinned host input and output, "
                       f"{E2E_CHUNK}-row chunks, {E2E_IN_SLOTS} input chunk buffers, "
                       "whose copies in and out overlap the GEMMs, copies inside the timed region"}
        L.h3q_host_pipeline_destroy(pipe)

    extras = None
    if dist is not None:
        try:
            extras = multi_gpu_extras(dist, dev)
        except Exception as e:  # the headline line must still print; the failure is reported in it
            extras = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.synchronize()
        dist.barrier()
    # single-GPU measurements of the other configs and call sites: at N = 1 only
    solo = rank == 0 and ws_n == 1
    q_alone = None
    if solo:
        # the same four quantizer launches back to back, no GEMM between them: inside the step the quantizer runs
        # at the SM clock the power-capped GEMMs leave behind, and it is issue-bound
        def quants():
            for ly in layers:
                h3q.check(L.h3q_quant_rows_i8(ly["x"].data_ptr(), 2, ly["q"].data_ptr(), ly["xs"].data_ptr(), M,
                                              ly["k"], 1, sp))
        qa_ms = time_steps(quants, 10, dev) / len(LINEARS)
        q_alone = {"avg_launch_ms": qa_ms, "achieved": quant_bytes_launch / (qa_ms * 1e-3) / 1e9,
                   "frac": quant_bytes_launch / (qa_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                   "note": "the four quantizer launches alone, back to back (CUDA events)"}
    comp = gpu_comparators(layers, dev, per_linear) if solo else None
    c2 = c2_block(dev, load_peaks()) if solo else None
    nv = nvfp4_c3(dev, load_peaks()) if solo else None
    att = attention_c4(dev, load_peaks()) if solo else None
    modq = modulate_fused(dev, load_peaks()) if solo else None
    lmerge = lora_merge(dev) if solo else None
    attend = attend_step_c4(dev) if solo else None
    stream_c1 = streaming_c1(layers, M, dev) if solo else None
    block = dit_block_c4(dev) if solo else None

    cb = None
    if rank == 0 and ws_n == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline()
        cb.pop("seconds", None)

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": ws_n, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": config_block(ws_n),
        "frac_of_int8_peak": value / ws_n / int8_peak,
        "roofline": {"kernel": "gemm_i8_kernel (tcgen05 kind::i8, fused epilogue)", "bound": "tensor",
                     "achieved": achieved, "peak": int8_peak, "unit": "TOPS", "frac": achieved / int8_peak,
                     "peak_note": (f"2 x {peaks['source']} bf16 {'sustained' if capped else 'burst'} "
                                   f"{int8_peak / 2:.0f} TF/s (dense int8 issues at twice the bf16 rate; "
                                   f"{'sw_power_cap active in the timed region' if capped else 'no power cap seen'})"
                                   f"; frac of nominal 4500: {achieved / NOMINAL_INT8_TOPS:.3f}"),
                     "frac_of_burst": achieved / int8_burst, "frac_of_sustained": achieved / int8_sustained,
                     "traffic": traffic, "avg_launch_ms": gemm_avg_ms, "ops_per_launch": gemm_ops_launch},
        "roofline_quant": {"kernel": "quant_rows_kernel<2> (rotate + per-token int8)", "bound": "hbm",
                           "achieved": q_achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                           "frac": q_achieved / peaks["hbm_gbs"], "avg_launch_ms": quant_avg_ms,
                           "bytes_per_launch": quant_bytes_launch, "alone": q_alone},
        "per_linear": per_linear,
        "gpu_comparators": comp,
        "c2": c2,
        "nvfp4_c3": nv,
        "attention_c4": att,
        "modulate_quant": modq,
        "lora_merge": lmerge,
        "attend_step_c4": attend,
        "weight_streaming_c1": stream_c1,
        "dit_block_c4": block,
        "multi_gpu": extras,
        "cpu_baseline": cb, "e2e": e2e, "clocks": clocks,
        "gpu_launches": 2 * launches,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

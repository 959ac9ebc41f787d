#!/usr/bin/env python3
"""Benchmark of the B200 quantized linear layer (one JSON line on rank 0).

Workload (the decode sweep the metric is quoted on):
  one *step* = the W4A16 GEMMs of one 27B decoder layer -- QKV (K=5120,N=7168),
  O (5120,5120), gate_up (5120,34816), down (17408,5120) -- at every
  M in {1,2,4,8,16}: 20 GEMMs, int4 group-128 weights, fp16 activations ~N(0,1),
  fp16 scales ~U(0.005,0.02), fp16 out, fp32 accumulate.  Synthetic seeded data.
  value = weight bytes streamed per step (int4 codes + fp16 scales) / step time.
With --gpus N > 1 (torchrun, one rank per GPU) the same sweep runs tensor-parallel
(Megatron): QKV and gate_up split by columns, O and down split by rows on
group boundaries with an NCCL all-reduce of the fp16 output after each; value is
the whole layer's weight bytes per step / max-over-ranks step time.

Sub-object "tp_stack" (every N): BASELINE configs[4], the 64-layer 27B linear stack
tensor-parallel over the N ranks, 2304 rows (256 decode + a 2048-token prefill
chunk) per step, NCCL all-reduce after O and down; TFLOP/s of the whole job.

--impl reference times the reference's algorithm on the host cores: the CPU
restatement in oracle/ (the reference has no CPU GEMM of its own), same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [("qkv", 5120, 7168), ("o", 5120, 5120), ("gate_up", 5120, 34816), ("down", 17408, 5120)]
MS = [1, 2, 4, 8, 16]
GROUP = 128
L2_BYTES = 126 * 1024 * 1024  # B200 L2
METRIC = "W4A16 GEMM weight TB/s (M≤16) & TFLOPS (M≥1024) at 1–8 B200 vs roofline"


def weight_bytes(K, N, wbits=4, group=GROUP):
    return K * N * wbits // 8 + (K // group) * N * 2


def kernels_per_gemm(M, K, N):
    """Kernels one int4 decode hq_gemm launches (hq_decode.cu launch_decode): two for a wide layer
    (>= 128 strip groups of 128 columns) at M <= 4 with 16-bit activations, which runs the
    activation prep kernel before the integer-MMA kernel; one otherwise."""
    return 2 if (M <= 4 and N // 128 >= 128) else 1


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- CPU (oracle)

class CpuSweep:
    """The decode sweep on the host cores through the oracle's dequant-then-matmul."""

    def __init__(self, nthreads: int):
        import numpy as np
        from oracle import oracle as o
        self.o, self.nthreads = o, nthreads
        rng = np.random.default_rng(0)
        self.data = []
        for name, K, N in SHAPES:
            lin = rng.integers(0, 2**32, size=(K // 8, N), dtype=np.uint32)
            S = o.round_to(rng.uniform(0.005, 0.02, size=(K // GROUP, N)).astype(np.float32), "f16")
            As = {M: o.round_to(rng.standard_normal((M, K), dtype=np.float32), "f16") for M in MS}
            self.data.append((K, N, lin, S, As))
        self.bytes_per_pass = sum(weight_bytes(K, N) for _, K, N in SHAPES) * len(MS)

    def one_pass(self):
        for K, N, lin, S, As in self.data:
            for M in MS:
                self.o.w4_gemm(As[M], lin, S, group=GROUP, nthreads=self.nthreads)

    def run(self, seconds: float):
        """Passes until >= seconds elapsed (at least one); returns (TB/s, seconds, passes)."""
        t0 = time.perf_counter()
        passes = 0
        while True:
            self.one_pass()
            passes += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                return self.bytes_per_pass * passes / el / 1e12, el, passes


class CpuTq1:
    """The TQ1_0 GEMV (M = 1, fp32 x) on the host cores through the oracle's restatement of
    kernel_gemv_tq1_0 (native_decoder.cu:155-206): the output projection (vocab 248320 x hidden
    5120) and the four 27B layer shapes, the set the GPU's tq1_0 sub-object times.  Blocks are
    seeded random trit bytes (< 243) with fp16 d in [0.01, 0.05)."""

    SHAPES = [("output_proj", 5120, 248320)] + SHAPES

    def __init__(self, nthreads: int):
        import numpy as np
        from oracle import oracle as o
        self.o, self.nthreads = o, nthreads
        rng = np.random.default_rng(5)
        self.data = []
        for name, K, N in self.SHAPES:
            blob = rng.integers(0, 243, size=(N, K // 256, 56), dtype=np.uint8)
            d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16)
            blob[..., 0:2] = d.view(np.uint8).reshape(N, K // 256, 2)
            blob[..., 54:56] = 0
            x = rng.standard_normal(K).astype(np.float32)
            self.data.append((K, N, blob.reshape(-1), x))
        self.bytes_per_pass = sum(N * (K // 256) * 56 for _, K, N in self.SHAPES)

    def one_pass(self):
        for K, N, blob, x in self.data:
            self.o.gemv_tq1_0(x, blob, K, N, nthreads=self.nthreads)

    run = CpuSweep.run


def reference_kernel_sweep(args):
    """The reference's own CUDA kernels timed on this GPU beside hq_gemm on identical inputs.

    kernel_marlin_gemm_int4_templated (marlin_gemm.cu:130-237, through
    MarlinGemmEngine::forward_marlin_int4, :570-613, which also clears Y) and
    kernel_baseline_int4_gemm (:76-117, through forward_baseline_int4, :552-568) from the
    reference's unmodified marlin_gemm.cu compiled for sm_100a into
    oracle/_ref/libref_marlin.so, at the four 27B layer shapes and M in {1, 2, 4, 8}, on the
    reference's own conventions: fp32 X [M][K], fp32 scales and biases [K/128][N], fp32 Y; int4
    codes as Marlin quads (marlin) or linear words (baseline).  hq_gemm gets the same codes in
    tile order with the same fp32 X, scales and biases.  Each launch runs on the legacy default
    stream, where the reference launches; CUDA events on that stream bracket `reps` launches
    that rotate over enough weight copies that every copy was last read more than two L2 sizes
    earlier.  GB/s counts the int4 codes plus fp32 scales and biases."""
    import ctypes

    import torch
    from oracle import oracle as o
    r = o.ref_lib()
    if r is None:
        return {"unavailable": "oracle/_ref/libref_marlin.so is not built (the reference sources were absent "
                               "when the package was built)"}
    from nebula_b200 import _lib, hq
    vp = ctypes.c_void_p
    r.ref_forward_marlin.argtypes = [vp] * 6 + [ctypes.c_uint32]
    r.ref_forward_baseline.argtypes = [vp] * 6 + [ctypes.c_uint32]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ds = torch.cuda.default_stream(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    rows = []
    L = _lib.lib()
    for name, K, N in SHAPES:
        nbytes = K * N // 2 + 2 * (K // GROUP) * N * 4
        n_copies = min(32, -(-int(2.5 * L2_BYTES) // nbytes) + 1)
        lin = [torch.randint(-2**31, 2**31 - 1, (K // 8, N), dtype=torch.int32, device=dev, generator=g)
               for _ in range(n_copies)]
        # Marlin quad (marlin_gemm.cu:446-455): words 4q..4q+3 of column n side by side
        quad = [w.view(K // 32, 4, N).permute(0, 2, 1).contiguous() for w in lin]
        tile = [hq.repack(w.view(torch.uint8).reshape(-1), _lib.HQ_WFMT_LINEAR_U4, _lib.HQ_WFMT_TILE_U4, K, N)
                for w in lin]
        S = [(torch.rand((K // GROUP, N), device=dev, generator=g) * 0.01 + 0.005) for _ in range(n_copies)]
        B = [-8.0 * s for s in S]
        eng = r.ref_engine_create(8, K, N, GROUP)
        if not eng:
            return {"unavailable": "ref_engine_create failed: " + r.ref_last_error().decode()}
        try:
            for M in (1, 2, 4, 8):
                X = torch.randn((M, K), device=dev, generator=g)
                Y = torch.empty((M, N), device=dev)
                ws = hq.make_workspace(M, N, K, GROUP, _lib.HQ_WFMT_TILE_U4, dev)

                def marlin(c):
                    if r.ref_forward_marlin(vp(eng), vp(X.data_ptr()), vp(quad[c].data_ptr()), vp(S[c].data_ptr()),
                                            vp(B[c].data_ptr()), vp(Y.data_ptr()), M) != 0:
                        raise RuntimeError(r.ref_last_error().decode())

                def baseline(c):
                    if r.ref_forward_baseline(vp(eng), vp(X.data_ptr()), vp(lin[c].data_ptr()), vp(S[c].data_ptr()),
                                              vp(B[c].data_ptr()), vp(Y.data_ptr()), M) != 0:
                        raise RuntimeError(r.ref_last_error().decode())

                def ours(c):
                    st = L.hq_gemm(vp(X.data_ptr()), _lib.HQ_F32, vp(tile[c].data_ptr()), _lib.HQ_WFMT_TILE_U4,
                                   vp(S[c].data_ptr()), _lib.HQ_F32, vp(B[c].data_ptr()), vp(Y.data_ptr()),
                                   _lib.HQ_F32, M, N, K, GROUP, vp(ws.data_ptr()), ws.numel(), None)
                    if st != 0:
                        raise RuntimeError(L.hq_last_error_string().decode())
                row = {"shape": name, "M": M, "K": K, "N": N, "copies": n_copies}
                reps = max(10, n_copies)
                for key, fn in (("ref_marlin", marlin), ("ref_baseline", baseline), ("hq", ours)):
                    ms = _time_launches(torch, ds, fn, n_copies, reps=reps)
                    row[key + "_us"] = round(ms * 1e3, 2)
                    row[key + "_GBps"] = round(nbytes / (ms / 1e3) / 1e9, 1)
                row["hq_over_ref_marlin"] = round(row["ref_marlin_us"] / row["hq_us"], 2)
                row["hq_over_ref_baseline"] = round(row["ref_baseline_us"] / row["hq_us"], 2)
                rows.append(row)
                del X, Y, ws
        finally:
            torch.cuda.synchronize()
            r.ref_engine_destroy(vp(eng))
        del lin, quad, tile, S, B
        torch.cuda.empty_cache()
    hq.check_device_error()
    tot = {k: sum(rw[k + "_us"] for rw in rows) for k in ("ref_marlin", "ref_baseline", "hq")}
    return {"rows": rows, "sum_us": {k: round(v, 1) for k, v in tot.items()},
            "hq_over_ref_marlin": round(tot["ref_marlin"] / tot["hq"], 2),
            "hq_over_ref_baseline": round(tot["ref_baseline"] / tot["hq"], 2),
            "timing": "per row: CUDA events on the legacy default stream around max(10, copies) launches queued "
                      "behind a spin kernel (device time, back to back) after 3 warm-up launches; the reference's "
                      "Y memset included",
            "note": "the reference's CUDA kernels on this GPU: a comparison beside this arm's CPU value, not "
                    "part of it"}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    sweep = CpuSweep(nthreads)
    for _ in range(args.warmup):
        sweep.one_pass()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sweep.one_pass()
    step_s = (time.perf_counter() - t0) / args.steps
    value = sweep.bytes_per_pass / step_s / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u4", "data": "synthetic",
            "config": {"workload": "decode_sweep (BASELINE configs[1]): 27B layer QKV/O/gate_up/down x M in "
                                   "{1,2,4,8,16}, int4 g128, fp16 A/scales", "parallelism": "host cores"},
            "cpu_baseline": {"value": value, "unit": "TB/s", "cores": nthreads, "kind": "port",
                             "sample": "one full pass of the decode sweep (20 GEMMs) per step: the oracle's "
                                       "dequant-then-matmul (fp32, OpenMP) on all host threads"},
            "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_ref_kernels:
        try:
            import torch
            gpu = torch.cuda.is_available()
        except ImportError:
            gpu = False
        line["reference_kernels"] = reference_kernel_sweep(args) if gpu else {"unavailable": "no GPU visible"}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------- prefill / ternary sub-sweeps

def _time_launches(torch, stream, fn, n_copies, reps=10, warmup=3):
    """Average device time (ms) of fn(copy) over `reps` launches, CUDA events on `stream`.

    A ~5 ms spin kernel is queued ahead of the timed launches, so that the host has queued all of
    them before the first one starts: the events then bracket the launches running back to back
    on the device, not the host's per-call overhead."""
    with torch.cuda.stream(stream):
        for w in range(warmup):
            fn(w % n_copies)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(10_000_000)
        e0.record(stream)
        for r in range(reps):
            fn(r % n_copies)
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def _gemm_call(L, _lib, A, a_dt, W, wfmt, S, s_dt, C, c_dt, M, N, K, ws, stream):
    import ctypes
    vp = ctypes.c_void_p
    st = L.hq_gemm(vp(A.data_ptr()), a_dt, vp(W.data_ptr()), wfmt, vp(S.data_ptr()), s_dt, None, vp(C.data_ptr()),
                   c_dt, M, N, K, GROUP, vp(ws.data_ptr()) if ws is not None else None,
                   ws.numel() if ws is not None else 0, vp(stream.cuda_stream))
    if st != 0:
        raise RuntimeError(L.hq_last_error_string().decode())


def prefill_sweep(torch, L, _lib, hq, dev, stream, weights, peaks, args):
    """the four 27B shapes at M in --prefill-ms, bf16 activations and scales,
    int4 g128, bf16 out, through hq_gemm (the tcgen05 kernel for M > 16).  TFLOP/s = 2*M*N*K / time."""
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    Ms = [int(x) for x in args.prefill_ms.split(",") if x]
    rows, tot_flop, tot_ms = [], 0.0, 0.0
    for name, K, N in SHAPES:
        Kl, Nl, copies = weights[name]
        Sb = [S.bfloat16() for (_, S) in copies]
        for M in Ms:
            A = torch.randn((M, Kl), device=dev, generator=g).bfloat16()
            C = torch.empty((M, Nl), device=dev, dtype=torch.bfloat16)
            nb = int(L.hq_gemm_workspace_size(M, Nl, Kl, GROUP, _lib.HQ_WFMT_TILE_U4))
            ws = torch.zeros(max(nb, 16), dtype=torch.uint8, device=dev)

            def fn(c):
                _gemm_call(L, _lib, A, _lib.HQ_BF16, copies[c][0], _lib.HQ_WFMT_TILE_U4, Sb[c], _lib.HQ_BF16, C,
                           _lib.HQ_BF16, M, Nl, Kl, ws, stream)
            reps = 10 if M <= 2048 else 4
            ms = _time_launches(torch, stream, fn, len(copies), reps=reps)
            flop = 2.0 * M * Nl * Kl
            tot_flop += flop
            tot_ms += ms
            rows.append({"shape": name, "M": M, "K": Kl, "N": Nl, "us": round(ms * 1e3, 1),
                         "TFLOPS": round(flop / (ms / 1e3) / 1e12, 1)})
            del A, C, ws
    tf = tot_flop / (tot_ms / 1e3) / 1e12
    return {"metric": "prefill W4A16 GEMM TFLOP/s (BASELINE configs[2])", "value": tf, "unit": "TFLOP/s",
            "dtype": "bf16", "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"],
                                          "unit": "TFLOP/s", "frac": tf / peaks["bf16_tflops"],
                                          "peak_source": peaks["source"] + " (burst cuBLAS bf16)"},
            "timing": "per GEMM: CUDA events around 10 launches (4 at M=8192) after 3 warm-up, 2 rotating weight "
                      "copies; value = total FLOP / total time",
            "per_gemm": rows}


def tq1_sweep(torch, L, _lib, dev, stream, peaks, args):
    """The reference decoder's own ternary path: hq_tq1_0_gemv (drop-in for kernel_gemv_tq1_0,
    native_decoder.cu:155-206; fp32 x, M = 1) on TQ1_0 blocks (56 B per 256 weights) at the output
    projection (vocab 248320 x hidden 5120, native_decoder.hpp:180) and the four 27B layer shapes.
    GB/s of TQ1_0 bytes.  Each shape rotates enough weight copies that every timed launch reads a copy
    last touched more than 2 L2 sizes earlier."""
    import ctypes
    vp = ctypes.c_void_p
    g = torch.Generator(device=dev)
    g.manual_seed(321)
    rows, tot_b, tot_ms = [], 0.0, 0.0
    for name, K, N in [("output_proj", 5120, 248320)] + SHAPES:
        nbytes = N * (K // 256) * 56
        n_copies = min(64, max(2, -(-int(2.5 * L2_BYTES) // nbytes) + 1))
        W = torch.randint(0, 243, (n_copies, N, K // 256, 56), dtype=torch.uint8, device=dev, generator=g)
        d = (torch.rand((n_copies, N, K // 256), device=dev, generator=g) * 0.04 + 0.01).half()
        W[..., 0:2] = d.view(torch.uint8).view(n_copies, N, K // 256, 2)
        W[..., 54:56] = 0
        W = W.view(n_copies, -1)
        x = torch.randn(K, device=dev, generator=g)
        out = torch.empty(N, device=dev)

        def fn(c):
            st = L.hq_tq1_0_gemv(vp(x.data_ptr()), vp(W[c].data_ptr()), vp(out.data_ptr()), K, N,
                                 vp(stream.cuda_stream))
            if st != 0:
                raise RuntimeError(L.hq_last_error_string().decode())
        reps = max(10, n_copies)
        with torch.cuda.stream(stream):
            for c in range(3):
                fn(n_copies - 1 - c)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            torch.cuda._sleep(10_000_000)  # the host queues every timed launch before the first runs
            e0.record(stream)
            for r in range(reps):
                fn(r % n_copies)
            e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        rows.append({"shape": name, "K": K, "N": N, "copies": n_copies, "us": round(ms * 1e3, 2),
                     "GBps": round(nbytes / (ms / 1e3) / 1e9, 1)})
        tot_b += nbytes
        tot_ms += ms
        del W, d
    gbps = tot_b / (tot_ms / 1e3) / 1e9
    return {"metric": "TQ1_0 GEMV GB/s (M=1, fp32 x)", "value": gbps, "unit": "GB/s",
            "frac_hbm": gbps / peaks["hbm_gbs"], "per_gemv": rows,
            "timing": "per shape: CUDA events around max(10, copies) launches queued behind a spin kernel "
                      "(device time, back to back) after 3 warm-up launches on other copies"}


def proj_sweep(torch, L, _lib, dev, stream, peaks, args):
    """The output projection over GGML BF16 / Q8_0 / F32 rows (kernel_output_projection,
    forward_baseline.cu:178-257; TQ1_0 rows are the tq1_0 sub-object) at vocab 248320 x hidden 5120,
    fp32 x: GB/s of weight bytes, two rotating weight copies (each larger than L2)."""
    import ctypes
    vp = ctypes.c_void_p
    K, N = 5120, 248320
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    rows = []
    for name, w_type in (("bf16", _lib.HQ_GGML_BF16), ("q8_0", _lib.HQ_GGML_Q8_0), ("f32", _lib.HQ_GGML_F32)):
        if w_type == _lib.HQ_GGML_Q8_0:
            W = torch.randint(-128, 128, (2, N, K // 32, 34), dtype=torch.int8, device=dev, generator=g).view(torch.uint8)
            d = (torch.rand((2, N, K // 32), device=dev, generator=g) * 0.015 + 0.005).half()
            W[..., 0:2] = d.view(torch.uint8).view(2, N, K // 32, 2)
            del d
        elif w_type == _lib.HQ_GGML_BF16:
            W = torch.randn((2, N, K), device=dev, generator=g).bfloat16().view(torch.uint8)
        else:
            W = torch.randn((2, N, K), device=dev, generator=g).view(torch.uint8)
        W = W.reshape(2, -1)
        x = torch.randn(K, device=dev, generator=g)
        out = torch.empty(N, device=dev)

        def fn(c):
            st = L.hq_output_projection(vp(x.data_ptr()), vp(W[c].data_ptr()), w_type, vp(out.data_ptr()), K, N,
                                        vp(stream.cuda_stream))
            if st != 0:
                raise RuntimeError(L.hq_last_error_string().decode())
        ms = _time_launches(torch, stream, fn, 2, reps=10)
        nbytes = W.shape[1]
        rows.append({"type": name, "K": K, "N": N, "weight_bytes": nbytes, "us": round(ms * 1e3, 1),
                     "GBps": round(nbytes / (ms / 1e3) / 1e9, 1),
                     "frac_hbm": round(nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 3)})
        del W
    return {"metric": "output projection GEMV GB/s (vocab 248320 x 5120, M=1, fp32 x)", "per_type": rows,
            "timing": "CUDA events around 10 launches after 3 warm-up, 2 rotating weight copies"}


def w8_sweep(torch, L, _lib, dev, stream, peaks, args):
    """The reference engine's W8A8 path (forward_cutlass_int8, marlin_gemm.cu:327-377) through hq_w8_gemm:
    int8 W [K][N], fp32 X and per-column scales; GB/s of weight bytes, two rotating weight copies."""
    import ctypes
    vp = ctypes.c_void_p
    g = torch.Generator(device=dev)
    g.manual_seed(23)
    rows = []
    for M, K, N in ((1, 4096, 4096), (8, 4096, 4096), (1, 5120, 34816), (8, 5120, 34816)):
        W = torch.randint(-128, 128, (2, K, N), dtype=torch.int8, device=dev, generator=g)
        X = torch.randn((M, K), device=dev, generator=g) * 0.5
        S = torch.rand(N, device=dev, generator=g) * 0.015 + 0.005
        Y = torch.empty((M, N), device=dev)

        def fn(c):
            st = L.hq_w8_gemm(vp(X.data_ptr()), vp(W[c].data_ptr()), vp(S.data_ptr()), vp(Y.data_ptr()), M, K, N,
                              vp(stream.cuda_stream))
            if st != 0:
                raise RuntimeError(L.hq_last_error_string().decode())
        ms = _time_launches(torch, stream, fn, 2, reps=10)
        rows.append({"M": M, "K": K, "N": N, "us": round(ms * 1e3, 1),
                     "GBps": round(K * N / (ms / 1e3) / 1e9, 1)})
        del W
    return {"metric": "W8A8 GEMM weight GB/s (forward_cutlass_int8)", "per_gemm": rows,
            "timing": "CUDA events around 10 calls (one cluster kernel each) after 3 warm-up, 2 weight copies"}


def _ternary_tile(torch, nbytes, dev, g):
    f = torch.randint(0, 3, (nbytes, 4), dtype=torch.uint8, device=dev, generator=g)
    return (f[:, 0] | (f[:, 1] << 2) | (f[:, 2] << 4) | (f[:, 3] << 6)).contiguous()


def ternary_sweep(torch, L, _lib, hq, dev, stream, peaks, args):
    """ternary codes {-1,0,1} (2 bits), fp16 scales g128, fp16 activations, the 27B
    shapes at M in {1, 16} (weight TB/s) and M = 2048 (TFLOP/s)."""
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    rows = []
    dec_bytes, dec_ms, pf_flop, pf_ms = 0.0, 0.0, 0.0, 0.0
    for name, K, N in SHAPES:
        copies = []
        for c in range(args.copies):
            W = _ternary_tile(torch, hq.weight_bytes(_lib.HQ_WFMT_TILE_T2, K, N), dev, g)
            S = (torch.rand((K // GROUP, N), device=dev, generator=g) * 0.04 + 0.01).half()
            copies.append((W, S))
        for M in (1, 16, 2048):
            A = torch.randn((M, K), device=dev, generator=g).half()
            C = torch.empty((M, N), device=dev, dtype=torch.float16)
            nb = int(L.hq_gemm_workspace_size(M, N, K, GROUP, _lib.HQ_WFMT_TILE_T2))
            ws = torch.zeros(max(nb, 16), dtype=torch.uint8, device=dev)

            def fn(c):
                _gemm_call(L, _lib, A, _lib.HQ_F16, copies[c][0], _lib.HQ_WFMT_TILE_T2, copies[c][1], _lib.HQ_F16,
                           C, _lib.HQ_F16, M, N, K, ws, stream)
            ms = _time_launches(torch, stream, fn, len(copies), reps=20 if M <= 16 else 10)
            wb = weight_bytes(K, N, wbits=2)
            row = {"shape": name, "M": M, "K": K, "N": N, "us": round(ms * 1e3, 2)}
            if M <= 16:
                dec_bytes += wb
                dec_ms += ms
                row["GBps"] = round(wb / (ms / 1e3) / 1e9, 1)
            else:
                pf_flop += 2.0 * M * N * K
                pf_ms += ms
                row["TFLOPS"] = round(2.0 * M * N * K / (ms / 1e3) / 1e12, 1)
            rows.append(row)
            del A, C, ws
    dec = dec_bytes / (dec_ms / 1e3) / 1e9
    pf = pf_flop / (pf_ms / 1e3) / 1e12
    return {"metric": "ternary W2A16 GEMM (BASELINE configs[3])",
            "decode_GBps": dec, "decode_frac_hbm": dec / peaks["hbm_gbs"],
            "prefill_TFLOPS": pf, "prefill_frac_tensor": pf / peaks["bf16_tflops"], "dtype": "f16",
            "timing": "per GEMM: CUDA events around 20 (M<=16) / 10 launches queued behind a spin kernel, after 3 "
                      "warm-up, 2 rotating weight copies (not graph-captured)",
            "per_gemm": rows}


def q4_k_sweep(torch, L, _lib, hq, dev, stream, peaks, args):
    """GGUF Q4_K at model load: hq_q4_k_to_tile (GB/s of Q4_K blocks in) and the group-32 GEMM it
    feeds (fp16 activations, f32 scale and bias rows per 32 weights) at the 27B shapes, M in {1, 16}
    (decode kernel) and M = 2048 (tcgen05 kernel, TFLOP/s).
    Decode GB/s counts the bytes the kernel must read: codes (K N / 2) plus 8 bytes of scale and bias
    per 32 weights, activations and outputs."""
    import ctypes
    vp = ctypes.c_void_p
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    half_bits = torch.tensor([0.002], dtype=torch.float16).view(torch.uint8).to(dev)  # d = dmin = 0.002
    rows, conv = [], []
    dec_bytes, dec_ms, pf_flop, pf_ms = 0.0, 0.0, 0.0, 0.0
    for name, K, N in SHAPES:
        nblk = N * (K // 256)
        copies = []
        for c in range(args.copies):
            blob = torch.randint(0, 256, (nblk, 144), dtype=torch.uint8, device=dev, generator=g)
            blob[:, 0:2] = half_bits
            blob[:, 2:4] = half_bits
            tile = torch.empty(hq.weight_bytes(_lib.HQ_WFMT_TILE_U4_K32, K, N), dtype=torch.uint8, device=dev)
            S = torch.empty((K // 32, N), device=dev)
            B = torch.empty((K // 32, N), device=dev)
            copies.append((blob, tile, S, B))

        def cv(c):
            blob, tile, S, B = copies[c]
            st = L.hq_q4_k_to_tile(vp(blob.data_ptr()), vp(tile.data_ptr()), vp(S.data_ptr()), vp(B.data_ptr()),
                                      K, N, vp(stream.cuda_stream))
            if st != 0:
                raise RuntimeError(L.hq_last_error_string().decode())
        ms = _time_launches(torch, stream, cv, len(copies), reps=10)
        conv.append({"shape": name, "K": K, "N": N, "us": round(ms * 1e3, 1),
                     "GBps_in": round(nblk * 144 / (ms / 1e3) / 1e9, 1)})
        copies = [(t, s, b) for (_, t, s, b) in copies]
        for M in (1, 16, 2048):
            A = torch.randn((M, K), device=dev, generator=g).half()
            C = torch.empty((M, N), device=dev, dtype=torch.float16)
            nb = int(L.hq_gemm_workspace_size(M, N, K, 32, _lib.HQ_WFMT_TILE_U4_K32))
            ws = torch.zeros(max(nb, 16), dtype=torch.uint8, device=dev)

            def fn(c):
                t, s, b = copies[c]
                st = L.hq_gemm(vp(A.data_ptr()), _lib.HQ_F16, vp(t.data_ptr()), _lib.HQ_WFMT_TILE_U4_K32, vp(s.data_ptr()),
                               _lib.HQ_F32, vp(b.data_ptr()), vp(C.data_ptr()), _lib.HQ_F16, M, N, K, 32,
                               vp(ws.data_ptr()), ws.numel(), vp(stream.cuda_stream))
                if st != 0:
                    raise RuntimeError(L.hq_last_error_string().decode())
            ms = _time_launches(torch, stream, fn, len(copies), reps=20 if M <= 16 else 10)
            row = {"shape": name, "M": M, "K": K, "N": N, "us": round(ms * 1e3, 2)}
            if M <= 16:
                nbytes = K * N // 2 + 2 * (K // 32) * N * 4 + M * K * 2 + M * N * 2
                dec_bytes += nbytes
                dec_ms += ms
                row["GBps"] = round(nbytes / (ms / 1e3) / 1e9, 1)
            else:
                pf_flop += 2.0 * M * N * K
                pf_ms += ms
                row["TFLOPS"] = round(2.0 * M * N * K / (ms / 1e3) / 1e12, 1)
            rows.append(row)
            del A, C, ws
        del copies
    dec = dec_bytes / (dec_ms / 1e3) / 1e9
    pf = pf_flop / (pf_ms / 1e3) / 1e12
    return {"metric": "GGUF Q4_K: load-time conversion and group-32 GEMM",
            "decode_GBps": dec, "decode_frac_hbm": dec / peaks["hbm_gbs"],
            "prefill_TFLOPS": pf, "prefill_frac_tensor": pf / peaks["bf16_tflops"], "dtype": "f16",
            "timing": "per call: CUDA events around 20 (M<=16) / 10 GEMMs, 10 conversions, queued behind a spin kernel, after "
                      "3 warm-up, rotating weight copies (not graph-captured)",
            "conversion": conv, "per_gemm": rows}


# ------------------------------------------------- TP layer stack

def tp_stack(torch, dist, L, _lib, dev, world, rank, stream, peaks, args):
    """the 64-layer 27B linear stack (QKV, O, gate_up, down per layer, int4 g128,
    bf16 activations and scales, random weights from a per-(layer, projection, rank) seed), tensor-parallel
    over the `world` ranks (nebula_b200.tp: column-parallel QKV / gate_up, row-parallel O / down with an
    NCCL all-reduce of the bf16 output after each).  One step = one split-fuse batch of 256 decode rows +
    a 2048-token prefill chunk = 2304 rows through every GEMM of every layer.  Inputs of O and down are
    fixed synthetic tensors (attention and the MLP activation are outside this path)."""
    from nebula_b200 import tp
    rows, layers = 2304, args.stack_layers
    g = torch.Generator(device=dev)
    specs = {name: tp.shard_spec(name, K, N, world, rank) for name, K, N in tp.LAYER_SHAPES}
    W = []
    for layer in range(layers):
        per = {}
        for j, (name, K, N) in enumerate(tp.LAYER_SHAPES):
            sp = specs[name]
            g.manual_seed(1000003 * layer + 7919 * j + 104729 * rank + 17)
            Wt = torch.randint(0, 256, (int(L.hq_weight_bytes(_lib.HQ_WFMT_TILE_U4, sp.K, sp.N)),), dtype=torch.uint8,
                               device=dev, generator=g)
            St = (torch.rand((sp.K // GROUP, sp.N), device=dev, generator=g) * 0.015 + 0.005).bfloat16()
            per[name] = (Wt, St)
        W.append(per)
    g.manual_seed(4242 + rank)
    X = {name: torch.randn((rows, specs[name].K), device=dev, generator=g).bfloat16() for name, _, _ in tp.LAYER_SHAPES}
    Y = {name: torch.empty((rows, specs[name].N), device=dev, dtype=torch.bfloat16) for name, _, _ in tp.LAYER_SHAPES}
    # Micro-batches (rows split on 256-row tile boundaries): their GEMMs run in order on the
    # compute stream, their all-reduces in the same order on one communication stream, so one
    # micro-batch's all-reduce overlaps the next GEMM (of the other micro-batch), and each
    # micro-batch's next GEMM waits for its own all-reduce, as the next layer's input would.
    # One collective at a time per GPU: a spinning collective never waits for a peer whose
    # matching kernel is kept off its SMs by another spinning one.
    n_mb = max(1, min(args.stack_mb, rows // 256)) if world > 1 else 1
    tiles = rows // 256
    bounds = [0] + [256 * ((tiles * (i + 1) + n_mb - 1) // n_mb) for i in range(n_mb)]
    bounds[-1] = rows
    mbs = [(bounds[i], bounds[i + 1]) for i in range(n_mb)]
    comm = torch.cuda.Stream(device=dev) if world > 1 else stream
    ws_bytes = max(int(L.hq_gemm_workspace_size(rows, specs[n].N, specs[n].K, GROUP, _lib.HQ_WFMT_TILE_U4))
                   for n, _, _ in tp.LAYER_SHAPES)
    ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=dev)

    # The all-reduce after O and down: hq_allreduce_sum over NVLink peer memory
    # (the row-parallel outputs live in PyTorch symmetric memory), or NCCL.
    use_hq = world > 1 and args.stack_comm == "hq"
    epoch = [0]
    if use_hq:
        import ctypes
        import torch.distributed._symmetric_memory as symm
        flags = symm.empty(32, dtype=torch.int32, device=dev)
        flags.zero_()
        hf = symm.rendezvous(flags, dist.group.WORLD)
        fptrs = (ctypes.c_void_p * world)(*hf.buffer_ptrs)
        peers = {}
        for name in tp.ROW_PARALLEL:
            buf = symm.empty((rows, specs[name].N), dtype=torch.bfloat16, device=dev)
            hb = symm.rendezvous(buf, dist.group.WORLD)
            Y[name] = buf
            mc = int(hb.multicast_ptr or 0) if args.nvls else 0
            peers[name] = (list(hb.buffer_ptrs), hb, mc)
        torch.cuda.synchronize()
        dist.barrier()

    def all_reduce(name, mb):  # on the communication stream
        r0, r1 = mbs[mb]
        n_el = (r1 - r0) * specs[name].N
        if use_hq:
            epoch[0] += 1
            off = r0 * specs[name].N * 2
            ptrs, _, mc = peers[name]
            bp = (ctypes.c_void_p * world)(*[q + off for q in ptrs])
            st = L.hq_allreduce_sum(bp, fptrs, ctypes.c_void_p(mc + off if mc else 0), world, rank,
                                    _lib.HQ_BF16, n_el, epoch[0], args.ar_ctas, ctypes.c_void_p(comm.cuda_stream))
            if st != 0:
                raise RuntimeError(L.hq_last_error_string().decode())
        else:
            with torch.cuda.stream(comm):
                dist.all_reduce(Y[name][r0:r1])

    def step():
        pending = [None] * n_mb  # each micro-batch's last all-reduce, not yet waited for
        for layer in range(layers):
            for name, _, _ in tp.LAYER_SHAPES:
                sp = specs[name]
                Wt, St = W[layer][name]
                for mb, (r0, r1) in enumerate(mbs):
                    if pending[mb] is not None:
                        stream.wait_event(pending[mb])
                        pending[mb] = None
                    _gemm_call(L, _lib, X[name][r0:r1], _lib.HQ_BF16, Wt, _lib.HQ_WFMT_TILE_U4, St, _lib.HQ_BF16,
                               Y[name][r0:r1], _lib.HQ_BF16, r1 - r0, sp.N, sp.K, ws, stream)
                    if sp.row_parallel and world > 1:
                        done = torch.cuda.Event()
                        done.record(stream)
                        comm.wait_event(done)
                        all_reduce(name, mb)
                        pending[mb] = torch.cuda.Event()
                        pending[mb].record(comm)
        for ev in pending:  # the step ends when its last all-reduces have
            if ev is not None:
                stream.wait_event(ev)

    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps = args.stack_steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            step()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    flop = 2.0 * rows * sum(K * N for _, K, N in tp.LAYER_SHAPES) * layers
    tf = flop / (ms / 1e3) / 1e12
    collective = None
    if world > 1:
        collective = "NCCL all_reduce"
        if use_hq:
            collective = ("hq_allreduce_sum, NVLS multicast (multimem)" if any(v[2] for v in peers.values())
                          else "hq_allreduce_sum, NVLink peer loads")
            torch.cuda.synchronize()
            dist.barrier()
            peers.clear()
    del W, X, Y, ws
    torch.cuda.empty_cache()
    return {"metric": "TP layer-stack TFLOP/s (BASELINE configs[4])", "value": tf, "unit": "TFLOP/s",
            "tokens_per_s": rows / (ms / 1e3), "ms_per_step": ms, "n_gpus": world, "layers": layers,
            "rows_per_step": rows, "scaling": "strong", "dtype": "bf16",
            "frac_of_n_x_peak": tf / (world * peaks["bf16_tflops"]),
            "collective": collective, "micro_batches": [r1 - r0 for r0, r1 in mbs],
            "timing": f"{steps} steps after 2 warm-up, CUDA events on the compute stream, max over ranks; "
                      "64 x 4 hq_gemm launches + 128 all-reduces per step and micro-batch at TP; the "
                      "all-reduces run on a communication stream, overlapping the other micro-batch's GEMM"}


def run_case(args):
    """One hq_gemm problem launched --steps times (for ncu captures of a single kernel)."""
    import torch
    from nebula_b200 import _lib, hq
    f = args.case.split(",")
    dev = torch.device("cuda", 0)
    if f[0] == "proj":  # proj,TYPE,K,N: hq_output_projection over GGML TYPE (0 F32, 8 Q8_0, 30 BF16) rows
        w_type, K, N = int(f[1]), int(f[2]), int(f[3])
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        if w_type == _lib.HQ_GGML_Q8_0:
            W = torch.randint(-128, 128, (N, K // 32, 34), dtype=torch.int8, device=dev, generator=g).view(torch.uint8)
            W[..., 0:2] = (torch.rand((N, K // 32), device=dev, generator=g) * 0.015 + 0.005).half().view(
                torch.uint8).view(N, K // 32, 2)
        elif w_type == _lib.HQ_GGML_BF16:
            W = torch.randn((N, K), device=dev, generator=g).bfloat16().view(torch.uint8)
        else:
            W = torch.randn((N, K), device=dev, generator=g).view(torch.uint8)
        x = torch.randn(K, device=dev, generator=g)
        for _ in range(args.steps):
            y = hq.output_projection(x, W.reshape(-1), w_type, N)
        torch.cuda.synchronize()
        hq.check_device_error()
        print(json.dumps({"case": args.case, "checksum": float(y.abs().sum())}))
        return 0
    if f[0] == "tq1":  # tq1,K,N: hq_tq1_0_gemv on well-formed TQ1_0 blocks (packed 0..242, d ~ U(0.01, 0.05))
        K, N = int(f[1]), int(f[2])
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        W = torch.randint(0, 243, (N, K // 256, 56), dtype=torch.uint8, device=dev, generator=g)
        d = (torch.rand((N, K // 256), device=dev, generator=g) * 0.04 + 0.01).half()
        W[..., 0:2] = d.view(torch.uint8).view(N, K // 256, 2)
        W[..., 54:56] = 0
        x = torch.randn(K, device=dev, generator=g)
        for _ in range(args.steps):
            y = hq.tq1_0_gemv(x, W.view(-1), N)
        torch.cuda.synchronize()
        hq.check_device_error()
        print(json.dumps({"case": args.case, "checksum": float(y.abs().sum())}))
        return 0
    if f[0] == "q4k":  # q4k,K,N,M: GGUF Q4_K blocks (d = dmin = 0.002) converted once, then the group-32 GEMM
        K, N, M = int(f[1]), int(f[2]), int(f[3])
        g = torch.Generator(device=dev)
        g.manual_seed(5)
        blob = torch.randint(0, 256, (N * (K // 256), 144), dtype=torch.uint8, device=dev, generator=g)
        blob[:, 0:2] = torch.tensor([0.002], dtype=torch.float16).view(torch.uint8).to(dev)
        blob[:, 2:4] = blob[:, 0:2]
        tile, S, B = hq.q4_k_to_tile(blob.reshape(-1), K, N)
        A = torch.randn((M, K), device=dev, generator=g).half()
        for _ in range(args.steps):
            y = hq.gemm(A, tile, S, N=N, group=32, bias=B)
        torch.cuda.synchronize()
        hq.check_device_error()
        print(json.dumps({"case": args.case, "checksum": float(y.float().abs().sum())}))
        return 0
    K, N, M = int(f[0]), int(f[1]), int(f[2])
    dt = f[3] if len(f) > 3 else "f16"
    wfmt = _lib.HQ_WFMT_TILE_T2 if len(f) > 4 and f[4] == "t2" else _lib.HQ_WFMT_TILE_U4
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    W = torch.randint(0, 256, (hq.weight_bytes(wfmt, K, N),), dtype=torch.uint8, device=dev, generator=g)
    S = (torch.rand((K // GROUP, N), device=dev, generator=g) * 0.015 + 0.005).to(tdt)
    A = torch.randn((M, K), device=dev, generator=g).to(tdt)
    for _ in range(args.steps):
        y = hq.gemm(A, W, S, N=N, group=GROUP, wfmt=wfmt)
    torch.cuda.synchronize()
    hq.check_device_error()
    print(json.dumps({"case": args.case, "checksum": float(y.float().abs().sum())}))
    return 0


# ---------------------------------------------------------------- GPU arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hq", choices=["hq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--copies", type=int, default=len(MS),
                    help="weight copies per shape; the GEMM of a step at the i-th M reads copy i mod copies, so with "
                         "the default (one per M) every GEMM of a step reads its own weights")
    ap.add_argument("--no-extra", action="store_true", help="skip the prefill and ternary sweeps")
    ap.add_argument("--no-stack", action="store_true", help="skip the TP layer stack (configs[4])")
    ap.add_argument("--no-ref-kernels", action="store_true",
                    help="reference arm: skip timing the reference's CUDA kernels on the GPU")
    ap.add_argument("--case", default=None,
                    help="profiling aid: 'K,N,M[,f16|bf16[,u4|t2]]' runs that one hq_gemm `--steps` times and exits; "
                         "'tq1,K,N' runs hq_tq1_0_gemv, 'proj,TYPE,K,N' hq_output_projection, 'q4k,K,N,M' the "
                         "group-32 GEMM on converted Q4_K blocks instead")
    ap.add_argument("--stack-layers", type=int, default=64)
    ap.add_argument("--stack-steps", type=int, default=3)
    ap.add_argument("--stack-comm", default="hq", choices=["hq", "nccl"], help="collective of the TP stack")
    ap.add_argument("--stack-mb", type=int, default=1,
                    help="micro-batches of the TP stack at N > 1 (each step's rows split on 256-row tiles; two "
                         "measured slower at 2 GPUs: 1500 against 1760 TFLOP/s)")
    ap.add_argument("--ar-ctas", type=int, default=128, help="CTAs of hq_allreduce_sum in the TP stack")
    ap.add_argument("--sweep-parallel", default="replicas", choices=["replicas", "tp"],
                    help="decode sweep at N > 1.  'replicas': every GPU runs BASELINE configs[1] (a one-GPU "
                         "workload) on its own weights, no collective (weak scaling; the units are all ranks' "
                         "GEMMs).  'tp': its shapes sharded Megatron-style with an all-reduce after O and down "
                         "(strong scaling; each shard is latency-bound).  The sharded multi-GPU workload of the "
                         "north star is the layer stack, reported in tp_stack at every N.")
    ap.add_argument("--sweep-comm", default="nccl", choices=["hq", "nccl"],
                    help="all-reduce of the row-parallel outputs in the tensor-parallel decode sweep (10-160 KB "
                         "messages: NCCL measured faster than hq_allreduce_sum's two-barrier kernel there)")
    ap.add_argument("--sweep-ar-ctas", type=int, default=16, help="CTAs of hq_allreduce_sum in the decode sweep")
    ap.add_argument("--no-nvls", dest="nvls", action="store_false", help="hq_allreduce_sum without NVLink multicast")
    ap.add_argument("--prefill-ms", default="512,2048,8192", help="token counts of the prefill sweep")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.case:
        return run_case(args)

    import torch
    import torch.distributed as dist
    from nebula_b200 import _lib, hq

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    peaks = load_peaks()
    L = _lib.lib()

    # ------------------------------------------------------------ workload
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    tpw = world if args.sweep_parallel == "tp" else 1  # tensor-parallel width of the decode sweep
    replicas = world if args.sweep_parallel == "replicas" else 1
    gemms = []  # (name, M, K_local, N_local, allreduce)
    for M in MS:
        for name, K, N in SHAPES:
            if name in ("qkv", "gate_up"):
                gemms.append((name, M, K, N // tpw, False))
            else:
                gemms.append((name, M, K // tpw, N, tpw > 1))
    weights = {}
    for name, K, N in SHAPES:
        Kl, Nl = (K, N // tpw) if name in ("qkv", "gate_up") else (K // tpw, N)
        copies = []
        for c in range(args.copies):
            W = torch.randint(0, 256, (hq.weight_bytes(_lib.HQ_WFMT_TILE_U4, Kl, Nl),), dtype=torch.uint8,
                              device=dev, generator=g)
            S = (torch.rand((Kl // GROUP, Nl), device=dev, generator=g) * 0.015 + 0.005).half()
            copies.append((W, S))
        weights[name] = (Kl, Nl, copies)
    max_ws = max(int(L.hq_gemm_workspace_size(16, Nl, Kl, GROUP, _lib.HQ_WFMT_TILE_U4))
                 for Kl, Nl, _ in weights.values())
    ws = torch.zeros(max_ws, dtype=torch.uint8, device=dev)
    acts = {M: {name: torch.randn((M, weights[name][0]), device=dev, generator=g).half() for name, _, _ in SHAPES}
            for M in MS}
    outs = {M: {name: torch.empty((M, weights[name][1]), device=dev, dtype=torch.float16) for name, _, _ in SHAPES}
            for M in MS}

    import ctypes
    vp = ctypes.c_void_p

    # Tensor-parallel runs: the row-parallel (O, down) outputs are summed over the ranks
    # after each GEMM, by hq_allreduce_sum on PyTorch symmetric memory (epoch 0: the call
    # count lives in the flag area, so the calls replay inside the step's CUDA graph),
    # or by NCCL.
    sweep_hq = tpw > 1 and args.sweep_comm == "hq"
    ar_bufs = {}
    if sweep_hq:
        import torch.distributed._symmetric_memory as symm
        ar_flags = symm.empty(32, dtype=torch.int32, device=dev)
        ar_flags.zero_()
        hf = symm.rendezvous(ar_flags, dist.group.WORLD)
        ar_fptrs = (ctypes.c_void_p * world)(*hf.buffer_ptrs)
        for M in MS:
            for name, _, _ in SHAPES:
                if name in ("o", "down"):
                    buf = symm.empty((M, weights[name][1]), dtype=torch.float16, device=dev)
                    hb = symm.rendezvous(buf, dist.group.WORLD)
                    outs[M][name] = buf
                    mc = int(hb.multicast_ptr or 0) if args.nvls else 0
                    ar_bufs[(M, name)] = ((ctypes.c_void_p * world)(*hb.buffer_ptrs), hb, ctypes.c_void_p(mc))
        torch.cuda.synchronize()
        dist.barrier()

    def sweep_all_reduce(M, name, C):
        if sweep_hq:
            bp, _, mc = ar_bufs[(M, name)]
            st = L.hq_allreduce_sum(bp, ar_fptrs, mc, world, rank, _lib.HQ_F16, C.numel(), 0, args.sweep_ar_ctas,
                                    vp(sh))
            if st != 0:
                raise RuntimeError(L.hq_last_error_string().decode())
        else:
            dist.all_reduce(C)

    def launch(name, M, copy, stream_handle, A=None, C=None):
        Kl, Nl, copies = weights[name]
        W, S = copies[copy]
        A = acts[M][name] if A is None else A
        C = outs[M][name] if C is None else C
        st = L.hq_gemm(vp(A.data_ptr()), _lib.HQ_F16, vp(W.data_ptr()), _lib.HQ_WFMT_TILE_U4, vp(S.data_ptr()),
                       _lib.HQ_F16, None, vp(C.data_ptr()), _lib.HQ_F16, M, Nl, Kl, GROUP, vp(ws.data_ptr()),
                       ws.numel(), vp(stream_handle))
        if st != 0:
            raise RuntimeError(L.hq_last_error_string().decode())
        return C

    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream

    def copy_of(M):
        return MS.index(M) % args.copies

    def step(timing_events=None):
        for i, (name, M, Kl, Nl, ar) in enumerate(gemms):
            if timing_events is not None:
                timing_events[i][0].record(stream)
            C = launch(name, M, copy_of(M), sh)
            if timing_events is not None:
                timing_events[i][1].record(stream)
            if ar:
                sweep_all_reduce(M, name, C)

    # warm-up (also sets kernel attributes before graph capture)
    with torch.cuda.stream(stream):
        for w in range(args.warmup):
            step()
    torch.cuda.synchronize()

    # One graph holds a whole step.
    graphs = []
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        step()
    graphs.append(gr)
    graphs[0].replay()
    torch.cuda.synchronize()

    # ---------------------------------------------------------- timed region
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        time.sleep(0.3)
        ev0.record(stream)
        for s in range(args.steps):
            with torch.cuda.stream(stream):
                graphs[0].replay()
        ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    layer_bytes = sum(weight_bytes(K, N) for _, K, N in SHAPES)
    step_bytes = layer_bytes * len(MS) * replicas  # every rank's weight bytes (replicas: a full sweep each)
    value = step_bytes / (ms / 1e3) / 1e12

    # ----------------------------------------------- per-launch kernel timing
    # Every GEMM of a step bracketed by events on its stream (no graph, no
    # collectives), all queued behind a spin kernel so that they run back to
    # back on the device: the decode kernels' average launch duration per shape.
    per = []
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in gemms]
    reps = max(3, min(args.steps, 10))
    acc_ms = [0.0] * len(gemms)
    with torch.cuda.stream(stream):
        for r in range(reps):
            torch.cuda._sleep(10_000_000)
            for i, (name, M, Kl, Nl, ar) in enumerate(gemms):
                evs[i][0].record(stream)
                launch(name, M, copy_of(M), sh)
                evs[i][1].record(stream)
            torch.cuda.synchronize()
            for i in range(len(gemms)):
                acc_ms[i] += evs[i][0].elapsed_time(evs[i][1])
    for i, (name, M, Kl, Nl, ar) in enumerate(gemms):
        d = acc_ms[i] / reps
        b = weight_bytes(Kl, Nl)
        per.append({"shape": name, "M": M, "K": Kl, "N": Nl, "us": round(d * 1e3, 2),
                    "GBps": round(b / (d / 1e3) / 1e9, 1)})
    kern_bytes = sum(weight_bytes(Kl, Nl) for (_, _, Kl, Nl, _) in gemms)
    kern_s = sum(acc_ms) / reps / 1e3
    achieved = kern_bytes / kern_s / 1e9

    # DRAM bytes per launch: the ratio measured by ncu on the dominant launch
    # (dram__bytes_read + dram__bytes_write over the algorithmic bytes, recorded
    # in profiles/decode_traffic.json) times the average algorithmic bytes per launch.
    traffic = None
    tp = os.path.join(ROOT, "profiles", "decode_traffic.json")
    if os.path.exists(tp):
        try:
            ratio = json.load(open(tp)).get("traffic_ratio")
            traffic = ratio * kern_bytes / len(gemms) if ratio else None
        except (ValueError, OSError):
            traffic = None

    # ------------------------------------------------------------- e2e leg
    # Public API with host buffers: pinned host A -> device, hq_gemm, C -> pinned host.
    hostA = {M: {n: acts[M][n].cpu().pin_memory() for n, _, _ in SHAPES} for M in MS}
    hostC = {M: {n: torch.empty_like(outs[M][n], device="cpu").pin_memory() for n, _, _ in SHAPES} for M in MS}
    h2d = sum(hostA[M][n].numel() * 2 for (n, M, _, _, _) in gemms)
    d2h = sum(hostC[M][n].numel() * 2 for (n, M, _, _, _) in gemms)

    def e2e_step():
        for (name, M, Kl, Nl, ar) in gemms:
            acts[M][name].copy_(hostA[M][name], non_blocking=True)
            C = launch(name, M, copy_of(M), sh)
            if ar:
                sweep_all_reduce(M, name, C)
            hostC[M][name].copy_(C, non_blocking=True)

    with torch.cuda.stream(stream):
        for w in range(3):
            e2e_step()
    e2e_graphs = []
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        e2e_step()
    e2e_graphs.append(gr)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        with torch.cuda.stream(stream):
            e2e_graphs[0].replay()
    e1.record(stream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_val = step_bytes / (e2e_ms / 1e3) / 1e12

    hq.check_device_error()

    stack = None
    if not args.no_stack:
        stack = tp_stack(torch, dist, L, _lib, dev, world, rank, stream, peaks, args)
        hq.check_device_error()

    prefill = ternary = tq1 = proj = w8 = q4k = None
    if world == 1 and not args.no_extra:
        prefill = prefill_sweep(torch, L, _lib, hq, dev, stream, weights, peaks, args)
        ternary = ternary_sweep(torch, L, _lib, hq, dev, stream, peaks, args)
        tq1 = tq1_sweep(torch, L, _lib, dev, stream, peaks, args)
        proj = proj_sweep(torch, L, _lib, dev, stream, peaks, args)
        w8 = w8_sweep(torch, L, _lib, dev, stream, peaks, args)
        q4k = q4_k_sweep(torch, L, _lib, hq, dev, stream, peaks, args)
        hq.check_device_error()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        nth = os.cpu_count() or 1
        v, el, passes = CpuSweep(nth).run(args.cpu_seconds)
        v1, el1, passes1 = CpuSweep(1).run(args.cpu_seconds / 4)
        tq, elt, passest = CpuTq1(nth).run(args.cpu_seconds / 4)
        cpu = {"value": v, "unit": "TB/s", "cores": nth, "kind": "port",
               "sample": f"{passes} full pass(es) of the decode sweep (20 GEMMs) in {el:.1f} s: oracle "
                         "dequant-then-matmul, fp32 OpenMP, all host threads",
               "one_thread": {"value": v1, "unit": "TB/s", "cores": 1,
                              "sample": f"{passes1} full pass(es) of the same sweep in {el1:.1f} s on one thread"},
               "tq1_0": {"value": tq * 1e3, "unit": "GB/s", "cores": nth, "kind": "port",
                         "sample": f"{passest} pass(es) of the TQ1_0 GEMV set of the tq1_0 sub-object (output "
                                   f"projection + four layer shapes, M = 1, fp32 x) in {elt:.1f} s: the oracle's "
                                   "restatement of kernel_gemv_tq1_0, all host threads"}}

    for gr in graphs + e2e_graphs:
        del gr
    graphs.clear()
    e2e_graphs.clear()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if args.sweep_parallel == "tp" else "weak",
            "vs_baseline": None, "dtype": "u4", "data": "synthetic (seeded random int4 codes, fp16 A ~N(0,1), "
                                                         "fp16 scales ~U(0.005,0.02))",
            "config": {"workload": "decode_sweep (BASELINE configs[1]): 27B layer QKV 5120x7168, O 5120x5120, "
                                   "gate_up 5120x34816, down 17408x5120 at M in {1,2,4,8,16}; int4 g128, fp16 A",
                       "global_batch": "M in {1,2,4,8,16}" + (f" on each of {world} replicas" if replicas > 1 else ""),
                       "parallelism": (f"tp{world}" if tpw > 1 else f"replicas x{world}: every GPU runs the "
                                       "one-GPU sweep on its own weights, no collective") if world > 1 else "single",
                       "collective": None if tpw == 1 else (
                           "NCCL all_reduce" if not sweep_hq else
                           "hq_allreduce_sum, NVLS multicast" if any(v[2].value for v in ar_bufs.values())
                           else "hq_allreduce_sum, NVLink peer loads"),
                       "l2": f"inputs larger than L2: {args.copies} weight copies per shape "
                             f"({args.copies * layer_bytes / 1e6:.0f} MB); the GEMM at the i-th M reads copy i, so "
                             "every GEMM of a step reads weights no other GEMM of the step touched",
                       "graph": "each step is one CUDA graph replay"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "peak_source": peaks["source"], "frac_of_nominal_8000": achieved / 8000.0,
                         "kernel": "hq decode kernels: integer-MMA stream kernel (wide layers at M <= 4), "
                                   "cluster split-K mma.sync kernel (narrow layers, M <= 8), tcgen05 kernel "
                                   "(M > 8 on wide layers)",
                         "traffic_unit": "bytes per launch (avg)",
                         "algorithmic_bytes_per_step": kern_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "TB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": sum(kernels_per_gemm(M, Kl, Nl) for (_, M, Kl, Nl, _) in gemms) * args.steps,
            "clocks": clocks.summary(),
            "per_gemm": per,
        }
        if stack is not None:
            line["tp_stack"] = stack
        if prefill is not None:
            line["prefill"] = prefill
        if ternary is not None:
            line["ternary"] = ternary
        if tq1 is not None:
            line["tq1_0"] = tq1
        if proj is not None:
            line["output_projection"] = proj
        if w8 is not None:
            line["w8a8"] = w8
        if q4k is not None:
            line["q4_k"] = q4k
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

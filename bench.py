#!/usr/bin/env python3
"""Benchmark of the Acfun hot path on B200 — one JSON line on rank 0.

Workload (the int8 GEMM the metric is quoted on at one GPU):
    C[s8] = requant(A[s8, 4096x4096] . B[s8, 4096x4096] + bias[s32]) * scale[f32], ReLU
    A, B ~ U{-127..127}, bias ~ U{-1000..1000}, scale ~ U[1e-3, 1e-2], seeded.
A "step" is one acfun_gemm_s8_requant call on that input.

  value   device-resident inputs (acfun_gemm_s8_requant on CUDA pointers), CUDA-event time per
          step, L2 flushed (256 MiB write, then read back) before every timed step; TOPS = 2*M*N*K / t,
          summed over ranks (weak scaling: every rank runs its own 4096^3 problem).
  e2e     the same call through the C ABI with PINNED HOST buffers: H2D of A, B, bias,
          scale and D2H of C inside every timed step.
  roofline  the tcgen05 GEMM kernel (the only kernel a device-resident call launches):
          achieved = 2*M*N*K / mean kernel time; peak = 2 x the measured dense bf16 burst
          rate in MEASURED_PEAKS.json (B200 runs dense int8 at twice the bf16 rate);
          traffic from the committed ncu summary when present.
  cpu_baseline  the reference's own int8 GEMM (acfun_gemm_int8, AVX-512 VNNI + OpenMP, built
          from its sources into oracle/_ref) on the host cores, on a bounded row sample.

  --impl reference  times that reference CPU path alone, as the driver's reference arm.
Multi-GPU: launch with torch.distributed.run; one rank per GPU, NCCL only for the barrier
and the max-over-ranks of the measured time (the GEMMs are independent).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N = K = 4096
OPS = 2.0 * M * N * K
METRIC = "int8_gemm_tops"
UNIT = "TOPS"
WORKLOAD = "cfg2 int8 GEMM 4096^3 s8xs8->s32, fused +bias, *scale, ReLU, requant to s8"
VGG_CPU_IMAGES = 16   # reference CPU leg of cfg5: images timed one by one, median


def make_inputs(seed=1234):
    g = np.random.default_rng(seed)
    A = g.integers(-127, 128, (M, K), dtype=np.int8)
    B = g.integers(-127, 128, (K, N), dtype=np.int8)
    bias = g.integers(-1000, 1001, N, dtype=np.int32)
    scale = g.uniform(1e-3, 1e-2, N).astype(np.float32)
    return A, B, bias, scale


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 100 ms (line-buffered into a file)
    for the whole timed region, plus synchronous samples taken while queued work runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.extra = []
        import tempfile
        self.path = tempfile.mktemp(prefix="acfun_clocks_", suffix=".csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["stdbuf", "-oL", "nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def sample_now(self):
        try:
            out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                  "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10)
            self.extra += [ln for ln in out.stdout.splitlines() if ln.strip()]
        except (OSError, subprocess.TimeoutExpired):
            pass

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        lines = list(self.extra)
        try:
            lines += open(self.path).read().splitlines()
            os.unlink(self.path)
        except OSError:
            pass
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def flush_l2(buf):
    """L2 flush between timed steps: write a 256 MiB buffer (twice the 126 MB L2), then read it
    back, so the L2 holds none of the step's data and no dirty lines whose write-back the next
    timed kernel would otherwise pay for."""
    buf.fill_(1)
    buf.view(torch_mod().int32).amax()


def torch_mod():
    import torch
    return torch


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops"), d.get("hbm_gbs"), "measured"
    return 1590.0, 6650.0, "fallback"


def ncu_traffic():
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary (or None)."""
    p = os.path.join(ROOT, "profiles", "gemm_s8req_2sm_4096.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            return None
    return None


_HOST = None


def host_info():
    """What the CPU numbers were measured on: lscpu's model name, nproc, and the reference
    library's own view (acfun_effective_cores, acfun_backend_name) when it is built."""
    global _HOST
    if _HOST is None:
        model = None
        try:
            out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
            for ln in out.splitlines():
                if ln.startswith("Model name:"):
                    model = ln.split(":", 1)[1].strip()
        except (OSError, subprocess.TimeoutExpired):
            pass
        info = {"cpu_model": model, "nproc": os.cpu_count()}
        try:
            from oracle import pyoracle
            if pyoracle.ref_available():
                R = pyoracle.ref()
                info["acfun_effective_cores"] = int(R.acfun_effective_cores())
                info["acfun_backend_name"] = R.acfun_backend_name().decode()
        except OSError:
            pass
        _HOST = info
    return dict(_HOST)


def cpu_reference_sample(steps=5, rows=512):
    """The reference's int8 GEMM with its fused epilogue (acfun_gemm_int8_epi on u8 A = s8 A +
    128: the reference's own route for this config, dequantising alpha * acc + beta with ReLU in
    the same pass) on `rows` rows of the 4096^3 problem, all host threads, 3 warm-ups and the
    median of `steps` (>= 5) timed calls (the reference's own method, src/benchmark.cpp:98-111);
    returns TOPS and details."""
    from oracle import pyoracle
    kind = "reference" if pyoracle.ref_available() else "port"
    A, B, bias, scale = make_inputs()
    cores = os.cpu_count() or 1
    steps = max(steps, 5)
    Au = (A[:rows].astype(np.int16) + 128).astype(np.uint8)
    C = np.empty((rows, N), np.float32)
    alpha = scale.copy()
    beta = (bias.astype(np.float32) * scale).astype(np.float32)
    times = []
    if kind == "reference":
        R = pyoracle.ref()
        pyoracle.ref_set_threads(cores)
        for _ in range(3):
            R.acfun_gemm_int8_epi(rows, N, K, Au, B, C, alpha, beta, 1)
        for _ in range(steps):
            t0 = time.perf_counter()
            R.acfun_gemm_int8_epi(rows, N, K, Au, B, C, alpha, beta, 1)
            times.append(time.perf_counter() - t0)
    else:
        O = pyoracle.oracle()
        cores = 1
        r = min(rows, 16)
        Au = Au[:r].copy()
        C = C[:r]
        t0 = time.perf_counter()
        O.orc_gemm_int8_epi(r, N, K, Au, B, C, alpha, beta, 1)
        times.append(time.perf_counter() - t0)
        rows = r
    t = statistics.median(times)
    return {"value": round(2.0 * rows * N * K / t / 1e12, 4), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{rows} of {M} rows of the 4096^3 u8xs8 GEMM with its dequant + ReLU epilogue "
                      f"(acfun_gemm_int8_epi on A+128), 3 warm-ups, median of {len(times)}, {cores} threads",
            "host": host_info()}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    cb = cpu_reference_sample(steps=max(args.steps, 5), rows=args.cpu_rows)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _he(g, shape, fan_in):
    lim = np.sqrt(6.0 / fan_in)
    return g.uniform(-lim, lim, size=shape).astype(np.float32)


def _bn_fold(g, w, cout):
    """cfg3: BN gamma U[.5,1.5], beta U[-.1,.1], mean U[-.1,.1], var U[.5,1.5] folded into the
    conv (model.cpp:69-95 expression order), bias 0 before the fold."""
    gamma = g.uniform(0.5, 1.5, cout).astype(np.float32)
    beta = g.uniform(-0.1, 0.1, cout).astype(np.float32)
    mean = g.uniform(-0.1, 0.1, cout).astype(np.float32)
    var = g.uniform(0.5, 1.5, cout).astype(np.float32)
    s = (gamma / np.sqrt(var + np.float32(1e-5))).astype(np.float32)
    return (w * s).astype(np.float32), (beta - mean * s).astype(np.float32)


def measure_configs(acf, torch, stream, flush, steps, with_cpu=True, cfg_filter=None, vgg_images=256):
    """Every BASELINE config on one GPU (device-resident tensors, CUDA events, L2 flushed
    before each timed step), with its roofline and the reference timed on the host cores on a
    bounded sample of the same workload."""
    from oracle import pyoracle as P
    L = acf.lib()
    bf16, hbm, src = measured_peaks()
    peak = {"int8": (2 * bf16, "TOPS", f"2 x bf16 ({src})"), "bf16": (bf16, "TFLOP/s", src),
            "f32x3": (bf16 / 6, "TFLOP/s", f"3xTF32 ceiling = bf16/2/3 ({src})"),
            "f32bf3": (bf16 / 3, "TFLOP/s", f"3xBF16 ceiling = bf16/3 ({src})"),
            "hbm": (hbm, "GB/s", src)}
    cores = os.cpu_count() or 1
    R = P.ref() if (with_cpu and P.ref_available()) else None
    if R is not None:
        P.ref_set_threads(cores)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = {}

    def timeit(fn, n):
        # >= 3 warm-up calls and ~0.2 s of work: first calls grow the scratch workspace and
        # load modules, and an idle GPU needs a moment to reach its working clocks
        t0 = time.perf_counter()
        for i in range(200):
            fn()
            if i >= 2:
                torch.cuda.synchronize()
                if time.perf_counter() - t0 > 0.2:
                    break
        torch.cuda.synchronize()
        acf.check()
        evs = []
        for _ in range(n):
            flush_l2(flush)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            evs.append((s, e))
        torch.cuda.synchronize()
        acf.check()
        return sum(s.elapsed_time(e) for s, e in evs) / n / 1e3

    def cpu(fn, units, unit_scale, warm=3, reps=5):
        """The reference on `units` (images / rows) per call: `warm` warm-up calls, then the
        median of `reps` timed calls (src/benchmark.cpp:98-111) -> value per unit."""
        if R is None:
            return None
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return units * unit_scale / statistics.median(ts)

    def record(name, t, work, unit_div, bound, cpu_val=None, cpu_sample="", extra=None, nbytes=None):
        pk, punit, psrc = peak[bound]
        achieved = work / t / unit_div
        r = {"ms": round(t * 1e3, 4), "value": round(achieved, 3), "unit": punit,
             "roofline": {"bound": "hbm" if bound == "hbm" else "tensor", "achieved": round(achieved, 2),
                          "peak": round(pk, 1), "unit": punit, "frac": round(achieved / pk, 4),
                          "peak_source": psrc}}
        if nbytes is not None and bound != "hbm":
            # a tensor-core config whose compulsory HBM traffic takes longer than its math at
            # peak is HBM-bound: report that roofline, keep the tensor fraction beside it
            hpk = peak["hbm"][0]
            t_tensor, t_hbm = work / unit_div / pk, nbytes / 1e9 / hpk
            r["roofline"]["tensor_frac"] = round(achieved / pk, 4)
            r["roofline"]["hbm_frac"] = round(nbytes / 1e9 / t / hpk, 4)
            r["roofline"]["ideal_us"] = {"tensor": round(t_tensor * 1e6, 2), "hbm": round(t_hbm * 1e6, 2)}
            if t_hbm > t_tensor:
                r["roofline"].update({"bound": "hbm", "achieved": round(nbytes / 1e9 / t, 2), "peak": round(hpk, 1),
                                      "unit": "GB/s", "frac": round(nbytes / 1e9 / t / hpk, 4),
                                      "peak_source": peak["hbm"][2]})
        if cpu_val is not None:
            r["cpu_baseline"] = {"value": round(cpu_val, 4), "unit": punit, "cores": cores,
                                 "kind": "reference", "sample": cpu_sample + ", 3 warm-ups, median of 5",
                                 "host": host_info()}
        if extra:
            r.update(extra)
        out[name] = r

    want = (lambda n: cfg_filter is None or n in cfg_filter)
    g = np.random.default_rng(2024)

    if want("cfg1_sgemm_1024"):
        A = g.uniform(-1, 1, (1024, 1024)).astype(np.float32)
        B = g.uniform(-1, 1, (1024, 1024)).astype(np.float32)
        dA, dB, dC = dev(A), dev(B), torch.empty((1024, 1024), device="cuda")
        t = timeit(lambda: L.acfun_gemm(1024, 1024, 1024, dA.data_ptr(), dB.data_ptr(), dC.data_ptr()), steps)
        Cc = np.empty((1024, 1024), np.float32)
        cv = cpu(lambda: R.acfun_gemm(1024, 1024, 1024, A, B, Cc), 2 * 1024 ** 3, 1e-12)
        record("cfg1_sgemm_1024", t, 2 * 1024 ** 3, 1e12, "f32bf3", cv, "full 1024^3 acfun_gemm")

    if want("cfg2_bf16_4096"):
        A = g.uniform(-1, 1, (4096, 4096)).astype(np.float32)
        B = g.uniform(-1, 1, (4096, 4096)).astype(np.float32)
        dA, dB, dC = dev(A), dev(B), torch.empty((4096, 4096), device="cuda")
        t = timeit(lambda: L.acfun_gemm_bf16(4096, 4096, 4096, dA.data_ptr(), dB.data_ptr(), dC.data_ptr()), steps)
        rows = 256
        Cc = np.empty((rows, 4096), np.float32)
        As = np.ascontiguousarray(A[:rows])
        cv = cpu(lambda: R.acfun_gemm_bf16(rows, 4096, 4096, As, B, Cc), 2 * rows * 4096 * 4096, 1e-12)
        record("cfg2_bf16_4096", t, 2 * 4096 ** 3, 1e12, "bf16", cv, f"{rows} rows of 4096^3 acfun_gemm_bf16",
               {"note": "fp32 in/out API: includes the fp32->bf16 operand conversion"})

    def conv_cfg(name, N, H, W, Cin, Cout, KH, st, pd, int8=False, groups=1, dw=False, bound=None):
        if not want(name):
            return
        OH, OW = (H + 2 * pd - KH) // st + 1, (W + 2 * pd - KH) // st + 1
        x = g.uniform(0, 1, (N, H, W, Cin)).astype(np.float32)
        if dw:
            w = _he(g, (Cin, KH, KH), KH * KH)
            b = g.uniform(-0.1, 0.1, Cin).astype(np.float32)
        elif groups > 1:
            w = _he(g, (groups, KH * KH * (Cin // groups), Cout // groups), KH * KH * (Cin // groups))
            b = g.uniform(-0.1, 0.1, Cout).astype(np.float32)
        else:
            w, b = _bn_fold(g, _he(g, (KH * KH * Cin, Cout), KH * KH * Cin), Cout)
        flops = 2.0 * N * OH * OW * Cout * KH * KH * (Cin // groups if not dw else 1)
        nbytes = 4.0 * (N * H * W * Cin + N * OH * OW * Cout)
        dx, dout = dev(x), torch.empty((N, OH, OW, Cout), device="cuda")
        db = dev(b)
        ns = 2 if N >= 2 else 1
        xs = np.ascontiguousarray(x[:ns])
        os_ = np.empty((ns, OH, OW, Cout), np.float32)
        if int8:
            ws = np.empty(Cout, np.float32)
            wq = np.empty((KH * KH * Cin, Cout), np.int8)
            L.acfun_quantize_weights(acf.ptr(w), KH * KH * Cin, Cout, acf.ptr(ws), acf.ptr(wq))
            dwq, dws = dev(wq), dev(ws)
            fn = lambda: L.acfun_conv2d_int8(dx.data_ptr(), N, H, W, Cin, dwq.data_ptr(), dws.data_ptr(),
                                             db.data_ptr(), KH, KH, Cout, st, pd, 0.0, dout.data_ptr(), 1)
            cfn = lambda: R.acfun_conv2d_int8(xs, ns, H, W, Cin, wq, ws, b.ctypes.data, KH, KH, Cout, st, pd,
                                              0.0, os_, 1)
        elif dw:
            dw_ = dev(w)
            fn = lambda: L.acfun_conv2d_dw(dx.data_ptr(), N, H, W, Cin, dw_.data_ptr(), db.data_ptr(), KH, KH,
                                           st, pd, dout.data_ptr(), 1)
            cfn = lambda: R.acfun_conv2d_dw(xs, ns, H, W, Cin, w, b.ctypes.data, KH, KH, st, pd, os_, 1)
        else:
            dw_ = dev(w)
            fn = lambda: L.acfun_conv2d_g(dx.data_ptr(), N, H, W, Cin, dw_.data_ptr(), db.data_ptr(), KH, KH,
                                          Cout, st, pd, groups, dout.data_ptr(), 1)
            cfn = lambda: R.acfun_conv2d_g(xs, ns, H, W, Cin, np.ascontiguousarray(w), b.ctypes.data, KH, KH,
                                           Cout, st, pd, groups, os_, 1)
        t = timeit(fn, steps)
        bound = bound or ("int8" if int8 else "f32bf3")
        if bound == "hbm":
            cv = cpu(cfn, ns * nbytes / N, 1e-9)
            record(name, t, nbytes, 1e9, "hbm", cv, f"{ns} of {N} images, reference route",
                   {"us": round(t * 1e6, 2), "gflop": round(flops / 1e9, 4), "mbytes": round(nbytes / 1e6, 2),
                    "img_per_s": round(N / t, 1)})
        else:
            cv = cpu(cfn, ns * flops / N, 1e-12)
            record(name, t, flops, 1e12, bound, cv, f"{ns} of {N} images, reference route",
                   {"gflop_direct_count": round(flops / 1e9, 4), "mbytes": round(nbytes / 1e6, 2),
                    "img_per_s": round(N / t, 1)}, nbytes=nbytes)

    conv_cfg("cfg3a_conv3x3_f23_f32", 32, 56, 56, 64, 64, 3, 1, 1)
    conv_cfg("cfg3b_conv3x3_f43_f32", 8, 112, 112, 64, 64, 3, 1, 1)
    conv_cfg("cfg3a_conv3x3_int8", 32, 56, 56, 64, 64, 3, 1, 1, int8=True)
    conv_cfg("cfg4_depthwise_3x3", 32, 56, 56, 144, 144, 3, 1, 1, dw=True, bound="hbm")
    conv_cfg("cfg4_grouped_s1", 32, 14, 14, 24, 48, 3, 1, 1, groups=6, bound="hbm")
    conv_cfg("cfg4_grouped_s2", 32, 14, 14, 24, 48, 3, 2, 1, groups=6, bound="hbm")
    conv_cfg("cfg4_pointwise_s1", 32, 56, 56, 144, 24, 1, 1, 0, bound="hbm")
    conv_cfg("cfg4_pointwise_s2", 32, 56, 56, 32, 64, 1, 2, 0, bound="hbm")

    if want("cfg5_vgg11_b256"):
        import tempfile

        from acfun_b200 import acfun0
        path = os.path.join(tempfile.gettempdir(), "acfun_vgg11_seed5.acfun")
        if not os.path.exists(path):
            acfun0.vgg11(seed=5).save(path)
        m = acf.Model(path)
        n = vgg_images   # 256 = the config; smaller only for profiling captures
        x = g.uniform(0, 1, (n, 224, 224, 3)).astype(np.float32)
        dx, dy = dev(x), torch.empty((n, 1000), device="cuda")
        t = timeit(lambda: L.acfun_model_infer_batch(m.h, n, dx.data_ptr(), dy.data_ptr()), max(2, steps // 4))
        cv = None
        if R is not None:
            h = R.acfun_model_load(path.encode())
            o = np.empty(1000, np.float32)
            imgs = iter([np.ascontiguousarray(x[k]) for k in range(VGG_CPU_IMAGES + 1)])
            cv = cpu(lambda: R.acfun_model_infer(h, next(imgs), o), 1, 1.0, warm=1, reps=VGG_CPU_IMAGES)
            R.acfun_model_destroy(h)
        gf = 15.218e9
        record("cfg5_vgg11_b256", t, n * gf, 1e12, "f32bf3", None, "",
               {"img_per_s": round(n / t, 1), "gflop_per_img": 15.218, "images": n})
        if cv is not None:
            out["cfg5_vgg11_b256"]["cpu_baseline"] = {
                "value": round(cv, 3), "unit": "img/s", "cores": cores, "kind": "reference",
                "sample": f"acfun_model_infer (batch-1 API) on {VGG_CPU_IMAGES} different images of the batch "
                          f"after 1 warm-up: 1 / the median per-image time", "host": host_info()}
        m.close()

    if want("cfg5_vgg11_int8_b256"):
        # the survey's cfg5 int8 variant: every dense conv via quantize_weights + conv2d_int8 per
        # image (one activation scale per image), FC / pool / softmax fp32
        import tempfile

        from acfun_b200 import acfun0
        from oracle.model_oracle import OracleModel
        path = os.path.join(tempfile.gettempdir(), "acfun_vgg11_seed5.acfun")
        if not os.path.exists(path):
            acfun0.vgg11(seed=5).save(path)
        m = acf.Model(path)
        m.set_int8(True)
        n = vgg_images
        x = g.uniform(0, 1, (n, 224, 224, 3)).astype(np.float32)
        dx, dy = dev(x), torch.empty((n, 1000), device="cuda")
        t = timeit(lambda: L.acfun_model_infer_batch(m.h, n, dx.data_ptr(), dy.data_ptr()), max(2, steps // 4))
        cv = None
        if R is not None:
            om = OracleModel(open(path, "rb").read())
            imgs = iter([np.ascontiguousarray(x[k]) for k in range(VGG_CPU_IMAGES + 1)])
            cv = cpu(lambda: om.ref_infer(R, next(imgs), int8=True), 1, 1.0, warm=1, reps=VGG_CPU_IMAGES)
        gf = 15.218e9
        record("cfg5_vgg11_int8_b256", t, n * gf, 1e12, "int8", None, "",
               {"img_per_s": round(n / t, 1), "gop_per_img": 15.218, "images": n,
                "note": "conv ops on the int8 tensor pipe, FC (0.25 GFLOP/img) in 3xBF16"})
        if cv is not None:
            out["cfg5_vgg11_int8_b256"]["cpu_baseline"] = {
                "value": round(cv, 3), "unit": "img/s", "cores": cores, "kind": "reference",
                "sample": f"{VGG_CPU_IMAGES} different images (after 1 warm-up) through the reference's int8 "
                          "layer API (quantize_weights + conv2d_int8 per conv, fc / maxpool / softmax), the "
                          "composition its int8 path needs: 1 / the median per-image time",
                "host": host_info()}
        m.close()
    return out


def vgg_model_path(rank, world, dist):
    """The cfg5 VGG-11 ACFUN0 file (generated once per box by rank 0, seeded)."""
    import tempfile

    from acfun_b200 import acfun0
    path = os.path.join(tempfile.gettempdir(), "acfun_vgg11_seed5.acfun")
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".part"
        acfun0.vgg11(seed=5).save(tmp)
        os.replace(tmp, path)
    if world > 1:
        dist.barrier()
    return path


def measure_vgg_sharded(acf, torch, dist, stream, flush, rank, world, steps, n=256):
    """cfg5 end to end across `world` GPUs (world = 1 included): every step, rank r copies its
    contiguous share of the 256-image batch from pinned host memory to its GPU, runs
    acfun_model_infer_batch on it, the [256, 1000] outputs are all-gathered over NCCL (world >
    1) and the gathered result is copied back to pinned host memory.  Per step and rank the
    phases are timed with CUDA events on the launching stream; the step time is the max over
    ranks; img/s = 256 / that.  After timing, rank 0 infers the whole batch on its own GPU and
    compares it with the gathered result."""
    from acfun_b200.shard import gather_outputs, shard_bounds
    L = acf.lib()
    path = vgg_model_path(rank, world, dist)
    m = acf.Model(path)
    b, e = shard_bounds(n, world, rank)
    g = np.random.default_rng(77)
    x_all = g.uniform(0, 1, (n, 224, 224, 3)).astype(np.float32)
    hx = torch.from_numpy(np.ascontiguousarray(x_all[b:e])).pin_memory()
    dx = torch.empty(hx.shape, device="cuda")
    dy = torch.empty((e - b, 1000), device="cuda")
    hy = torch.empty((n, 1000)).pin_memory()

    def step(ev=None):
        if ev:
            ev[0].record(stream)
        dx.copy_(hx, non_blocking=True)
        if ev:
            ev[1].record(stream)
        if L.acfun_model_infer_batch(m.h, e - b, dx.data_ptr(), dy.data_ptr()) <= 0:
            acf.check()
        if ev:
            ev[2].record(stream)
        out = gather_outputs(dist, dy, n, world) if world > 1 else dy
        if ev:
            ev[3].record(stream)
        hy.copy_(out, non_blocking=True)
        if ev:
            ev[4].record(stream)
        return out

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    acf.check()
    evs = []
    for _ in range(steps):
        flush_l2(flush)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        step(ev)
        torch.cuda.synchronize()
        evs.append(ev)
    acf.check()
    ph = np.array([[ev[k].elapsed_time(ev[k + 1]) for k in range(4)] for ev in evs]).mean(0) / 1e3
    tt = float(np.mean([ev[0].elapsed_time(ev[4]) for ev in evs])) / 1e3
    vals = [tt] + list(ph)
    if world > 1:
        tv = torch.tensor(vals, device="cuda", dtype=torch.float64)
        dist.all_reduce(tv, op=dist.ReduceOp.MAX)
        vals = [float(v) for v in tv]
    tt, t_h2d, t_inf, t_gat, t_d2h = vals
    gathered = hy.numpy().copy()
    ok = bool(np.isfinite(gathered).all()) and abs(float(gathered.sum()) - n) < 1e-2 * n  # softmax rows
    parity = None
    if world > 1:
        dist.barrier()
        if rank == 0:
            # the whole batch on this one GPU (untimed) against the gathered shards
            dxa = torch.from_numpy(x_all).cuda()
            dya = torch.empty((n, 1000), device="cuda")
            if L.acfun_model_infer_batch(m.h, n, dxa.data_ptr(), dya.data_ptr()) <= 0:
                acf.check()
            one = dya.cpu().numpy()
            parity = {"bit_identical_to_1gpu": bool(np.array_equal(one.view(np.int32), gathered.view(np.int32))),
                      "max_abs_diff": float(np.abs(one - gathered).max())}
            del dxa, dya
        dist.barrier()
    m.close()
    bf16, _, src = measured_peaks()
    pk = bf16 / 3
    achieved = n * 15.218e9 / tt / 1e12
    return {"ms": round(tt * 1e3, 3), "value": round(n / tt, 1), "unit": "img/s", "n_gpus": world,
            "images_per_gpu": e - b, "outputs_valid": ok, "parity_vs_1gpu": parity,
            "phases_ms_max_over_ranks": {"h2d": round(t_h2d * 1e3, 3), "infer": round(t_inf * 1e3, 3),
                                         "gather": round(t_gat * 1e3, 3), "d2h": round(t_d2h * 1e3, 3)},
            "gather_share": round(t_gat / tt, 4),
            "h2d_bytes_per_step_per_rank": int(hx.numel() * 4), "d2h_bytes_per_step_per_rank": n * 1000 * 4,
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(pk * world, 1),
                         "unit": "TFLOP/s", "frac": round(achieved / (pk * world), 4),
                         "peak_source": f"3xBF16 ceiling = bf16/3 ({src}) x n_gpus"},
            "collective": "NCCL all-gather of the [256,1000] outputs (1 MB) only" if world > 1 else None,
            "timing": "events on the launching stream around H2D, infer, gather, D2H; mean over steps, "
                      "max over ranks; L2 flushed before every step"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="acfun_b200", choices=["acfun_b200", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=512)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-config measurements (every BASELINE config, N=1 only)")
    ap.add_argument("--configs", default=None, help="comma-separated subset of config names")
    ap.add_argument("--vgg-images", type=int, default=256,
                    help="cfg5 batch (256 = the config; smaller only for --only-configs profiling runs)")
    ap.add_argument("--only-configs", action="store_true",
                    help="print only the per-config measurements (profiling runs; not the bench line)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl != "reference" else args.warmup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    import acfun_b200 as acf

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    L = acf.lib()
    if L.acfun_set_device(local):
        acf.check()
    stream = torch.cuda.current_stream()
    L.acfun_set_stream(stream.cuda_stream)

    if args.only_configs:
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        filt = set(args.configs.split(",")) if args.configs else None
        res = measure_configs(acf, torch, stream, flush, steps=max(1, args.steps), vgg_images=args.vgg_images,
                              with_cpu=not args.no_cpu_baseline, cfg_filter=filt)
        print(json.dumps({"configs": res}), flush=True)
        return

    A, B, bias, scale = make_inputs(1234 + rank)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dbias, dscale = torch.from_numpy(bias).cuda(), torch.from_numpy(scale).cuda()
    dC = torch.empty((M, N), dtype=torch.int8, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def dev_step():
        L.acfun_gemm_s8_requant(M, N, K, dA.data_ptr(), dB.data_ptr(), dbias.data_ptr(), dscale.data_ptr(),
                                dC.data_ptr(), 1)

    # pinned host buffers for the end-to-end leg
    hA, hB = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    hbias, hscale = torch.from_numpy(bias).pin_memory(), torch.from_numpy(scale).pin_memory()
    hC = torch.empty((M, N), dtype=torch.int8).pin_memory()

    def e2e_step():
        L.acfun_gemm_s8_requant(M, N, K, hA.data_ptr(), hB.data_ptr(), hbias.data_ptr(), hscale.data_ptr(),
                                hC.data_ptr(), 1)

    # correctness spot check before timing: the first and last 8 rows of C against the CPU
    # oracle's restatement of the requantising GEMM, bit for bit (test infrastructure used as
    # the checker only)
    dev_step()
    torch.cuda.synchronize()
    acf.check()
    from oracle import pyoracle
    Cd = dC.cpu().numpy()
    for r0 in (0, M - 8):
        ref = np.empty((8, N), np.int8)
        pyoracle.oracle().orc_gemm_s8_requant(8, N, K, np.ascontiguousarray(A[r0:r0 + 8]), B,
                                              bias.ctypes.data, scale, ref, 1)
        if not np.array_equal(Cd[r0:r0 + 8], ref):
            raise SystemExit(f"bench: rows {r0}..{r0 + 7} of the int8 requant GEMM differ from the oracle")

    for _ in range(args.warmup):
        dev_step()
        e2e_step()
    torch.cuda.synchronize()
    acf.check()

    def timed(fn, steps, clk=None):
        total = 0.0
        evs = []
        for i in range(steps):
            if clk is not None and i == steps // 2:
                clk.sample_now()                 # the GPU is busy with the queued steps
            flush_l2(flush)                      # evict A, B, C from the 126 MB L2
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            evs.append((s, e))
        torch.cuda.synchronize()
        for s, e in evs:
            total += s.elapsed_time(e)
        return total / steps / 1e3             # seconds per step

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_dev = timed(dev_step, args.steps, clk)
        t_e2e = timed(e2e_step, args.steps)
    acf.check()
    t_dev_max, t_e2e_max = t_dev, t_e2e
    if world > 1:
        tt = torch.tensor([t_dev, t_e2e], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_dev_max, t_e2e_max = float(tt[0]), float(tt[1])
        dist.barrier()

    vgg = None
    if not args.no_configs:
        vgg = measure_vgg_sharded(acf, torch, dist, stream, flush, rank, world, steps=max(3, min(args.steps, 10)))

    if rank == 0:
        bf16_peak, hbm_peak, peak_src = measured_peaks()
        peak_tops = 2.0 * bf16_peak
        achieved = OPS / t_dev / 1e12
        traffic = ncu_traffic()
        sat = None
        Cn = dC.cpu().numpy()
        sat = float(((Cn == 127) | (Cn == 0)).mean())
        line = {
            "metric": METRIC, "value": round(world * OPS / t_dev_max / 1e12, 2), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_dev_max * 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "per_gpu_problems": 1,
                       "l2": "flushed before every timed step: 256 MiB write, then the same buffer read back (no step data and no dirty lines left in L2)",
                       "output_saturated_or_zero_frac": round(sat, 3)},
            "e2e": {"value": round(world * OPS / t_e2e_max / 1e12, 2), "unit": UNIT,
                    "h2d_bytes_per_step": A.nbytes + B.nbytes + bias.nbytes + scale.nbytes,
                    "d2h_bytes_per_step": M * N, "ms_per_step": round(t_e2e_max * 1e3, 4),
                    "api": "acfun_gemm_s8_requant on pinned host buffers"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak_tops, 1),
                         "unit": "TOPS", "frac": round(achieved / peak_tops, 4),
                         "peak_source": f"2 x bf16_tflops ({peak_src}, MEASURED_PEAKS.json): dense int8 = 2x bf16",
                         "kernel": "gemm_2sm_kernel<I8, S8_REQ> (256x256 tiles on SM pairs, tcgen05.mma.cta_group::2, "
                                   "6 stages)" if os.environ.get("ACFUN_GEMM_2SM", "1") != "0"
                                   else "gemm_tc_kernel<I8, BN=256, 4 stages, S8_REQ>",
                         "traffic": traffic},
            # our kernels in the two timed loops: one GEMM per device-resident call; the host-
            # buffer call splits A into min(8, A bytes / 2 MiB) row chunks, one GEMM each
            "gpu_launches": args.steps * (1 + max(1, min(8, (M * K) >> 21))),
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_sample(steps=3, rows=args.cpu_rows)
        if world == 1 and not args.no_configs:
            filt = set(args.configs.split(",")) if args.configs else None
            line["configs"] = measure_configs(acf, torch, stream, flush, steps=max(5, min(args.steps, 20)),
                                              with_cpu=not args.no_cpu_baseline, cfg_filter=filt)
        if vgg is not None:
            line.setdefault("configs", {})["cfg5_vgg11_b256_sharded"] = vgg
            line["vgg11_b256_e2e_img_per_s"] = vgg["value"]
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

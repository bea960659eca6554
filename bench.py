#!/usr/bin/env python
"""Benchmark of the B200 NVFP4 path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload ep|quant|gemm|moe] [--impl ours|reference]

Workloads (synthetic seeded inputs and random-init weights with the configs' shapes):
  ep (default)  cfg4: expert-parallel MoE stack on the N GPUs -- 30 MoE layers shaped as cfg3, 512 rows (32 sequences
                x 16 draft tokens) per step in total, split 512/N per GPU (strong scaling; --ep-scaling weak keeps
                512 rows per GPU), the 128 experts sharded 128/N per GPU, records and returned rows stored into the
                other GPUs' memory over NVLink by the kernels (one GPU runs the single-GPU layer); the step is
                replayed from one CUDA graph.  Metric tokens/s over all GPUs.  At N = 1 the line also carries the
                driver-visible sub-results `quant` (cfg1 T=8192) and `gemm` (cfg2 M=8192, K=4096, N=14336), timed in
                the same process under the same rules.
  quant         cfg1 at its largest size: bf16 [8192, 2816] ~ N(0,1) with 0.1% x50 outliers.  One step = device
                global amax + NVFP4 quantise (codes, tile-layout e4m3 scales, fp32 amax).  Metric GB/s of
                algorithmic bytes T*K*(2 + 1/2 + 1/16) + 4.
  moe           cfg3: one MoE layer, 4096 tokens, 128 experts, top-8: router + dispatch + grouped gate/up + grouped
                down with the weighted combine.  Metric tokens/s.
  gemm          cfg2 at its largest size: M=8192, K=4096, N=14336, NVFP4 A and W resident, bf16 out with the fused
                global-scale multiply.  One step = one GEMM.  Metric TFLOP/s of 2*M*N*K.
For N > 1 (torchrun, one process per GPU) quant, gemm and moe run one replica per rank (they do not shard):
value = sum over ranks of the work / the max over ranks of the device time.

Timing: W untimed warm-up steps; K timed steps, each bracketed by CUDA events on the launching stream; the L2 is
flushed between steps outside the events (a 256 MiB write, then a 256 MiB read so no dirty lines remain); barrier +
synchronize around the timed region; the max over ranks is taken.  `e2e` repeats the step through the public API
from pinned host memory with the host->device copy of the inputs and the device->host copy of the outputs inside
the timed region.

--impl reference times the reference's CPU implementation on the same config (rank 0 only): the quantiser (the
oracle's C port of scripts/nvfp4_ref.py:71-82, all host threads) for quant, the float64 dequant-matmul
(scripts/nvfp4_ref.py:102) on a row sample for gemm, the MoE experts() semantics of scripts/ref_forward.py:160-192
(numpy, all host threads, experts dequantised before timing) for moe and ep.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import pathlib
import re
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "NVFP4 GEMM TFLOPS & quant GB/s vs roofline; MoE tokens/s at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum (bytes) of the dominant kernel per launch, from the ncu captures
# summarised under profiles/ (quantize_bf16_rows_kernel, nvf4_gemm_pair_kernel, the MoE gate/up GEMM).
NCU_TRAFFIC = {"quant": 46.262272e6, "gemm": 335.105280e6, "moe": 366.175232e6,
               "ep": 320.639744e6}   # ep: the layer's dominant kernel, the grouped gate/up GEMM (one launch)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", choices=["quant", "gemm", "moe", "ep", "w4a16", "linear"], default="ep")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ep-rows", type=int, default=512, help="ep: rows per step (512 = 32 sequences x 16 drafts)")
    ap.add_argument("--ep-layers", type=int, default=30,
                    help="ep: MoE layers in the stack (30 = cfg4; 1 keeps the device footprint small for ncu captures)")
    ap.add_argument("--ep-scaling", choices=["strong", "weak"], default="strong",
                    help="ep: strong = --ep-rows in total, split over the GPUs (the cfg4 contract); weak = --ep-rows "
                         "per GPU")
    ap.add_argument("--no-sub", action="store_true", help="ep at N=1: skip the quant and gemm sub-results")
    ap.add_argument("--ep-exchange", choices=["auto", "p2p", "nccl", "local"], default="auto",
                    help="ep: records/rows stored over NVLink peer memory by the kernels (p2p), NCCL all-to-all "
                         "(nccl), the single-GPU MoE layer (local, 1 GPU only), or auto = p2p on 2+ GPUs, local on 1")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample length (rank 0, N=1)")
    ap.add_argument("--clock-seconds", type=float, default=1.5, help="sustained-load window for clock sampling")
    ap.add_argument("--profile-kernels", action="store_true",
                    help="after the timed steps, two eager steps under torch.profiler (CUPTI activity records): "
                         "per-kernel device time per step on every rank, to stderr (not a bench value)")
    ap.add_argument("--cuda-profiler-range", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


# ----------------------------------------------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ["clocks.sm", "clocks.max.sm", "power.draw", "utilization.gpu", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, device_index: int, uuid: str | None):
        self.proc = None
        sel = ["--id=" + uuid] if uuid else ["--id=" + str(device_index)]
        self.cmd = ["nvidia-smi", *sel, "--query-gpu=" + ",".join(self.FIELDS), "--format=csv,noheader,nounits",
                    "-lms", "100"]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for rec in csv.reader(io.StringIO(getattr(self, "out", "") or "")):
            if len(rec) != len(self.FIELDS):
                continue
            try:
                rows.append({"sm": float(rec[0]), "max": float(rec[1]), "util": float(rec[3]),
                             "reasons": {k: rec[i].strip() for i, k in enumerate(
                                 ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                  "sw_power_cap"], start=4)}})
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        busy = [r for r in rows if r["util"] > 0] or rows
        reasons = sorted({k for r in busy for k, v in r["reasons"].items() if k != "active" and v == "Active"})
        return {"sm_mhz": statistics.median(r["sm"] for r in busy), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": reasons, "samples": len(busy)}


# ----------------------------------------------------------------------------------------------------------------
# workloads
# ----------------------------------------------------------------------------------------------------------------

class QuantWorkload:
    name = "quant"
    unit = "GB/s"
    dtype = "f32"     # block arithmetic (f64 for the per-block scale), bf16 in, e2m1/e4m3 out

    def __init__(self, pkg, torch, orc, T=8192, K=2816):
        self.pkg, self.torch = pkg, torch
        self.T, self.K = T, K
        bits = orc.synth_bf16((T, K), 1.0, seed=2024, outlier_frac=0.001)
        self.host_bits = bits
        import numpy as np
        self.x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
        self.amax = torch.empty(1, dtype=torch.float32, device="cuda")
        self.packed = torch.empty((T, K // 2), dtype=torch.uint8, device="cuda")
        self.scales = torch.empty(pkg.nvfp4_scale_buffer_bytes(T, K), dtype=torch.uint8, device="cuda")
        self.units_per_step = T * K * 2.5625 + 4          # algorithmic bytes: bf16 in, codes, scales, amax
        self.kernel_bytes = T * K * 2.5625                 # the quantise kernel alone (input read + outputs)
        self.launches_per_step = 2
        self.kernel_name = "quantize_bf16_rows_kernel"
        self.config = {"workload": "cfg1 activation quantiser, dynamic global scale", "T": T, "K": K,
                       "input": "bf16 N(0,1), 0.1% entries x50", "l2": "flushed between steps (256 MiB write + 256 MiB read)",
                       "graph": "one CUDA graph per step (amax reset, amax, quantise)"}

    def step(self, mark=None):
        p = self.pkg
        p.amax(self.x, out=self.amax)
        if mark is not None:
            mark("kernel")
        p.quantize(self.x, amax_dev=self.amax, packed=self.packed, scales=self.scales)
        if mark is not None:
            mark("kernel_end")

    def value(self, seconds_per_step):
        return self.units_per_step / seconds_per_step / 1e9

    # end to end through the public API from pinned host buffers
    def e2e_setup(self):
        t = self.torch
        self.h_x = t.empty((self.T, self.K), dtype=t.bfloat16, pin_memory=True)
        self.h_x.copy_(self.x.cpu())
        self.h_packed = t.empty_like(self.packed, device="cpu").pin_memory()
        self.h_scales = t.empty_like(self.scales, device="cpu").pin_memory()
        self.h_amax = t.empty(1, dtype=t.float32, pin_memory=True)
        self.d_x = t.empty_like(self.x)
        return self.T * self.K * 2, self.packed.numel() + self.scales.numel() + 4

    def e2e_step(self):
        self.d_x.copy_(self.h_x, non_blocking=True)
        self.pkg.amax(self.d_x, out=self.amax)
        self.pkg.quantize(self.d_x, amax_dev=self.amax, packed=self.packed, scales=self.scales)
        self.h_packed.copy_(self.packed, non_blocking=True)
        self.h_scales.copy_(self.scales, non_blocking=True)
        self.h_amax.copy_(self.amax, non_blocking=True)

    def cpu_run(self, native, orc, seconds):
        """Oracle C port (all host threads) on the same input: amax + quantise, repeated for ~`seconds`."""
        n, t0 = 0, time.perf_counter()
        while True:
            a = native.amax_bf16(self.host_bits)
            native.quantize_bf16(self.host_bits, orc.global_scale_from_amax(a))
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        return self.units_per_step * n / el / 1e9, f"{n} passes over cfg1 T={self.T} x K={self.K} ({el:.1f} s)"


class GemmWorkload:
    name = "gemm"
    unit = "TFLOP/s"
    dtype = "nvfp4"   # e2m1 x e2m1 with e4m3 block scales, fp32 accumulate, bf16 out

    def __init__(self, pkg, torch, orc, M=8192, N=14336, K=4096):
        import numpy as np
        self.pkg, self.torch = pkg, torch
        self.M, self.N, self.K = M, N, K
        xb = orc.synth_bf16((M, K), 1.0, seed=11)
        wb = orc.synth_bf16((N, K), 0.02, seed=12)
        self.host_xb = xb
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        w = torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16).cuda()
        self.amax = pkg.amax(x)
        self.a, self.a_sf = pkg.quantize(x, amax_dev=self.amax)
        self.gw = float(orc.global_scale_from_amax(np.abs(orc.bf16_bits_to_f32(wb)).max()))
        self.b, self.b_sf = pkg.quantize(w, gscale=self.gw)
        self.x = x
        del w
        self.out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        self.units_per_step = 2.0 * M * N * K
        self.kernel_bytes = None
        self.launches_per_step = 1
        self.kernel_name = "nvf4_gemm_pair_kernel (256x256 tiles on a CTA pair, tcgen05 cta_group::2)"
        self.config = {"workload": "cfg2 dense prefill GEMM, largest config", "M": M, "N": N, "K": K,
                       "out": "bf16 row-major, alpha fused", "l2": "flushed between steps (256 MiB write + 256 MiB read)"}

    def step(self, mark=None):
        if mark is not None:
            mark("kernel")
        self.pkg.gemm(self.a, self.a_sf, 0.0, self.b, self.b_sf, 1.0 / self.gw, out=self.out, a_amax=self.amax)
        if mark is not None:
            mark("kernel_end")

    def value(self, seconds_per_step):
        return self.units_per_step / seconds_per_step / 1e12

    def e2e_setup(self):
        t = self.torch
        self.h_x = t.empty((self.M, self.K), dtype=t.bfloat16, pin_memory=True)
        self.h_x.copy_(self.x.cpu())
        self.h_out = t.empty((self.M, self.N), dtype=t.bfloat16, pin_memory=True)
        self.d_x = t.empty_like(self.x)
        return self.M * self.K * 2, self.M * self.N * 2

    def e2e_step(self):
        p = self.pkg
        self.d_x.copy_(self.h_x, non_blocking=True)
        p.amax(self.d_x, out=self.amax)
        p.quantize(self.d_x, amax_dev=self.amax, packed=self.a, scales=self.a_sf)
        p.gemm(self.a, self.a_sf, 0.0, self.b, self.b_sf, 1.0 / self.gw, out=self.out, a_amax=self.amax)
        self.h_out.copy_(self.out, non_blocking=True)

    def cpu_run(self, native, orc, seconds):
        """Oracle port: dequantise the NVFP4 operands and multiply in float64 (multithreaded BLAS) on a row sample."""
        import numpy as np
        rows = 64
        px = self.a[:rows].cpu().numpy()
        sx = orc.unswizzle_scales(self.a_sf.cpu().numpy(), self.M, self.K)[:rows]
        pw = self.b.cpu().numpy()
        sw = orc.unswizzle_scales(self.b_sf.cpu().numpy(), self.N, self.K)
        gx = float(orc.global_scale_from_amax(self.amax.item()))
        wd = orc.dequantize(pw, sw, self.gw)
        n, t0 = 0, time.perf_counter()
        while True:
            orc.dequantize(px, sx, gx) @ wd.T
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        return 2.0 * rows * self.N * self.K * n / el / 1e12, f"{n} x ({rows} rows of cfg2 M x N={self.N} x K={self.K}) float64"


class W4a16Workload:
    """The reference's W4A16 decode path at its largest call (src/forward.cu:596, fp4_gemv on the lm_head): NVFP4
    weights [N=262144, K=2816] (raw codes + e4m3 scales, 415 MB) times one fp16 activation row -> fp32 logits.  A
    weight stream: the roofline is HBM."""
    name = "w4a16"
    unit = "GB/s"
    dtype = "nvfp4 weights x fp16"

    def __init__(self, pkg, torch, orc, M=1, N=262144, K=2816):
        self.pkg, self.torch = pkg, torch
        self.M, self.N, self.K = M, N, K
        gen = torch.Generator(device="cuda").manual_seed(77)
        self.wp = torch.randint(0, 256, (N, K // 2), generator=gen, dtype=torch.uint8, device="cuda")
        self.ws = torch.randint(0x30, 0x40, (N, K // 16), generator=gen, dtype=torch.uint8, device="cuda")
        self.wg = 2688.0 / 0.1
        self.x = torch.randn((M, K), generator=gen, device="cuda").half()
        self.out = torch.empty((M, N), dtype=torch.float32, device="cuda")
        self.kernel_bytes = N * K // 2 + N * K // 16 + M * K * 2 + M * N * 4
        self.units_per_step = self.kernel_bytes
        self.launches_per_step = 1
        self.kernel_name = "w4a16_gemv_kernel" if M == 1 else "w4a16_fast_kernel"
        self.config = {"workload": "W4A16 decode GEMV (fp4_gemv), lm_head shape", "M": M, "N": N, "K": K,
                       "weights": "random NVFP4 codes and e4m3 scales (raw, unswizzled)",
                       "l2": "flushed between steps (256 MiB write + 256 MiB read); weights 415 MB > L2"}

    def step(self, mark=None):
        if mark is not None:
            mark("kernel")
        self.pkg.w4a16_gemm(self.out, self.wp, self.ws, self.wg, self.x, self.M, self.N, self.K)
        if mark is not None:
            mark("kernel_end")

    def value(self, seconds_per_step):
        return self.units_per_step / seconds_per_step / 1e9

    def e2e_setup(self):
        t = self.torch
        self.h_x = t.empty((self.M, self.K), dtype=t.float16, pin_memory=True)
        self.h_x.copy_(self.x.cpu())
        self.h_out = t.empty((self.M, self.N), dtype=t.float32, pin_memory=True)
        self.d_x = t.empty_like(self.x)
        return self.M * self.K * 2, self.M * self.N * 4

    def e2e_step(self):
        self.d_x.copy_(self.h_x, non_blocking=True)
        self.pkg.w4a16_gemm(self.out, self.wp, self.ws, self.wg, self.d_x, self.M, self.N, self.K)
        self.h_out.copy_(self.out, non_blocking=True)

    def cpu_run(self, native, orc, seconds):
        """Oracle port: dequantise a row sample of the weights (code * e4m3 / g) and multiply in float32 numpy."""
        import numpy as np
        rows = 8192
        wp = self.wp[:rows].cpu().numpy()
        ws = self.ws[:rows].cpu().numpy()
        x = self.x.float().cpu().numpy()
        n, t0 = 0, time.perf_counter()
        while True:
            wd = orc.dequantize(wp, ws, self.wg).astype(np.float32)
            x @ wd.T
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        b = rows * (self.K // 2 + self.K // 16)
        return b * n / el / 1e9, f"{n} x {rows} weight rows of the lm_head shape (dequantise + matmul, numpy)"


class LinearWorkload:
    """The dense Linear wired to the W4A4 path (src/forward.cu:424-445 at prefill): fp32 [M=4096, K=2816] in ->
    NVFP4 quantise (static activation scale) -> tcgen05 GEMM against NVFP4 W [N=2112, K] -> fp32 row-major out, one
    nvfp4b_linear call (the MLP gate/up projection shape of the model)."""
    name = "linear"
    unit = "TFLOP/s"
    dtype = "nvfp4"

    def __init__(self, pkg, torch, orc, M=4096, N=2112, K=2816):
        import numpy as np
        self.pkg, self.torch = pkg, torch
        self.M, self.N, self.K = M, N, K
        gen = torch.Generator(device="cuda").manual_seed(78)
        self.x = torch.randn((M, K), generator=gen, device="cuda")
        w = (torch.randn((N, K), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
        self.wg = float(orc.global_scale_from_amax(pkg.amax(w).item()))
        self.wp, self.ws_tiled = pkg.quantize(w, gscale=self.wg)
        self.ws_raw = torch.zeros((N, K // 16), dtype=torch.uint8, device="cuda")   # unused on the W4A4 path
        self.ag = float(orc.global_scale_from_amax(self.x.abs().max().item()))
        self.out = torch.empty((M, N), dtype=torch.float32, device="cuda")
        self.ws = pkg.linear_workspace(M, K)
        self.units_per_step = 2.0 * M * N * K
        self.launches_per_step = 2      # quantise + GEMM
        self.kernel_name = "nvfp4b_linear (quantize_kernel<float> + nvf4_gemm_pair_kernel, fp32 row-major out)"
        self.config = {"workload": "dense Linear, W4A4 prefill path (nvfp4b_linear)", "M": M, "N": N, "K": K,
                       "activation_scale": "static", "out": "fp32 row-major",
                       "l2": "flushed between steps (256 MiB write + 256 MiB read)"}

    def step(self, mark=None):
        if mark is not None:
            mark("kernel")
        self.pkg.linear(self.out, self.x, self.wp, self.ws_raw, self.ws_tiled, self.wg, a_gscale=self.ag,
                        mode=self.pkg.LINEAR_W4A4, workspace=self.ws)
        if mark is not None:
            mark("kernel_end")

    def value(self, seconds_per_step):
        return self.units_per_step / seconds_per_step / 1e12

    def e2e_setup(self):
        t = self.torch
        self.h_x = t.empty((self.M, self.K), dtype=t.float32, pin_memory=True)
        self.h_x.copy_(self.x.cpu())
        self.h_out = t.empty((self.M, self.N), dtype=t.float32, pin_memory=True)
        self.d_x = t.empty_like(self.x)
        return self.M * self.K * 4, self.M * self.N * 4

    def e2e_step(self):
        self.d_x.copy_(self.h_x, non_blocking=True)
        self.pkg.linear(self.out, self.d_x, self.wp, self.ws_raw, self.ws_tiled, self.wg, a_gscale=self.ag,
                        mode=self.pkg.LINEAR_W4A4, workspace=self.ws)
        self.h_out.copy_(self.out, non_blocking=True)

    def cpu_run(self, native, orc, seconds):
        """Oracle port: quantise a row sample of x (C port), dequantise, float64 matmul against the dequantised W."""
        import numpy as np
        rows = 64
        x = self.x[:rows].cpu().numpy()
        wd = orc.dequantize(self.wp.cpu().numpy(), orc.unswizzle_scales(self.ws_tiled.cpu().numpy(), self.N, self.K),
                            self.wg)
        n, t0 = 0, time.perf_counter()
        while True:
            px, sx = native.quantize_f32(x, self.ag)
            orc.dequantize(px, sx, self.ag) @ wd.T
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        return 2.0 * rows * self.N * self.K * n / el / 1e12, f"{n} x ({rows} rows of M x N={self.N} x K={self.K})"


class MoeWorkload:
    """cfg3: one MoE FFN layer, 4096 tokens, H=2816, 128 experts (I=704), top-8, GeLU-tanh gating."""
    name = "moe"
    unit = "tokens/s"
    dtype = "nvfp4"   # NVFP4 x NVFP4 grouped GEMMs, fp32 accumulate; bf16 router GEMM

    def __init__(self, pkg, torch, orc, T=4096, H=2816, I=704, E=128, topk=8):
        import numpy as np
        self.pkg, self.torch = pkg, torch
        self.T, self.H, self.I, self.E, self.topk = T, H, I, E, topk
        xb = orc.synth_bf16((T, H), 1.0, seed=31)
        rb = orc.synth_bf16((E, H), 0.02, seed=32)
        self.x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).cuda()
        self.proj = torch.from_numpy(rb.view(np.int16)).view(torch.bfloat16).cuda()
        gen = torch.Generator(device="cuda").manual_seed(33)
        arena = pkg.MoeExperts(E, H, I)
        for e in range(E):     # N(0, 0.02) bf16 weights, NVFP4-quantised straight into the arena layout
            w13 = (torch.randn((2 * I, H), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
            a = pkg.amax(w13)
            g = float(orc.global_scale_from_amax(a.item()))
            pkg.quantize(w13, gscale=g, packed=arena.w13[e], scales=arena.w13_scales[e])
            arena.w1_gscale[e] = g
            arena.w3_gscale[e] = g
            w2 = (torch.randn((H, I), generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
            g2 = float(orc.global_scale_from_amax(pkg.amax(w2).item()))
            pkg.quantize(w2, gscale=g2, packed=arena.w2[e], scales=arena.w2_scales[e])
            arena.w2_gscale[e] = g2
        self.arena = arena
        self.ws = pkg.moe_workspace(T, H, I, E, topk)
        self.in_amax = pkg.amax(self.x)
        self.ids, self.wts = pkg.moe_route(self.x, self.proj, topk, self.ws)
        h_amax = pkg.moe_calibrate(self.x, self.ids, self.wts, arena, self.ws, in_amax=self.in_amax)
        torch.cuda.synchronize()
        arena.a2_gscale.copy_(torch.from_numpy(np.array([orc.global_scale_from_amax(v) for v in h_amax.cpu().numpy()],
                                                        np.float32)))
        self.out = torch.empty((T, H), dtype=torch.float32, device="cuda")
        self.units_per_step = T
        self.kernel_flops = 2.0 * T * topk * (2 * I) * H          # grouped gate/up GEMM, routed rows only
        self.step_flops = 2.0 * T * topk * 3 * I * H + 2.0 * T * E * H
        self.launches_per_step = 9    # amax, router GEMM + top-k, hist-rank/plan/quantise-scatter, gate/up, down, combine
        self.kernel_name = "nvf4_gemm_kernel<GroupedSched, GateUpEpi> (grouped gate/up, GELU + NVFP4 requant)"
        self.config = {"workload": "cfg3 MoE FFN layer", "tokens": T, "hidden": H, "experts": E, "inter": I,
                       "topk": topk, "router": "bf16 [128, 2816], softmax-top8-renorm",
                       "scales": "x: dynamic global (device amax); h: static per-expert (calibrated once)",
                       "l2": "flushed between steps (256 MiB write + 256 MiB read)", "step_flops": self.step_flops}

    def step(self, mark=None):
        p, T, k = self.pkg, self.T, self.topk
        p.amax(self.x, out=self.in_amax)
        p.moe_route(self.x, self.proj, k, self.ws, ids=self.ids, weights=self.wts)
        p.moe_dispatch(self.x, self.ids, self.wts, self.arena, self.ws, in_amax=self.in_amax)
        if mark is not None:
            mark("kernel")
        p.moe_gate_up(T, k, self.arena, self.ws, in_amax=self.in_amax)
        if mark is not None:
            mark("kernel_end")
        p.moe_down(T, k, self.wts, self.arena, self.out, self.ws)    # fp32 row buffer + slot-ordered combine

    def value(self, seconds_per_step):
        return self.units_per_step / seconds_per_step

    def e2e_setup(self):
        t = self.torch
        self.h_x = t.empty((self.T, self.H), dtype=t.bfloat16, pin_memory=True)
        self.h_x.copy_(self.x.cpu())
        self.h_out = t.empty((self.T, self.H), dtype=t.float32, pin_memory=True)
        self.d_x = t.empty_like(self.x)
        return self.T * self.H * 2, self.T * self.H * 4

    def e2e_step(self):
        p = self.pkg
        self.d_x.copy_(self.h_x, non_blocking=True)
        p.amax(self.d_x, out=self.in_amax)
        p.moe_route(self.d_x, self.proj, self.topk, self.ws, ids=self.ids, weights=self.wts)
        p.moe_forward(self.d_x, self.ids, self.wts, self.arena, self.ws, in_amax=self.in_amax, out=self.out)
        self.h_out.copy_(self.out, non_blocking=True)

    def cpu_run(self, native, orc, seconds):
        """The reference's experts() semantics (scripts/ref_forward.py:175-192: per-token loop over the selected
        experts, gelu_tanh(gate) * up, down, weighted sum) in W4A4 on a token sample, numpy float32 on all host
        threads.  The sample's experts are dequantised BEFORE the timer (as the reference's experts() works on
        weights loaded once); the timed part is the per-token work: quantise x, the expert matmuls, requantise h."""
        import numpy as np
        S = 16
        ids = self.ids[:S].cpu().numpy()
        w = self.wts[:S].cpu().numpy()
        x = self.x[:S].float().cpu().numpy()
        gin = orc.global_scale_from_amax(self.in_amax.item())
        a2 = self.arena.a2_gscale.cpu().numpy()
        mats = {}
        for e in sorted(set(int(v) for v in ids.reshape(-1))):
            g = float(self.arena.w1_gscale[e].item())
            sf = orc.unswizzle_scales(self.arena.w13_scales[e].cpu().numpy(), 2 * self.I, self.H)
            sd = orc.unswizzle_scales(self.arena.w2_scales[e].cpu().numpy(), self.H, self.I)
            mats[e] = (native.dequantize(self.arena.w13[e].cpu().numpy(), sf, g).astype(np.float32),
                       native.dequantize(self.arena.w2[e].cpu().numpy(), sd,
                                         float(self.arena.w2_gscale[e].item())).astype(np.float32))
        n, t0 = 0, time.perf_counter()
        while True:
            _, _, xd = orc.quantize_rows(x.astype(np.float64), gin)
            xd = xd.astype(np.float32)
            out = np.zeros((S, self.H), np.float32)
            for t in range(S):
                for j in range(self.topk):
                    e = int(ids[t, j])
                    wgu, wd = mats[e]
                    y = wgu @ xd[t]
                    h = orc.gelu_tanh(y.reshape(-1, 2, 16)[:, 0].reshape(-1)) * y.reshape(-1, 2, 16)[:, 1].reshape(-1)
                    _, _, hd = orc.quantize_rows(h[None].astype(np.float64), a2[e])
                    out[t] += w[t, j] * (wd @ hd[0].astype(np.float32))
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        return S * n / el, (f"{n} x {S} tokens of cfg3 through the W4A4 experts() path (experts dequantised before "
                            f"timing, float32)")


class EpWorkload:
    """cfg4: expert-parallel decode/verify stack on G GPUs -- 30 stacked MoE FFN layers shaped as cfg3 (H=2816,
    128 experts of I=704, top-8), experts sharded 128/G per GPU, T rows per rank per step: 512/G of the 32 sequences
    x 16 draft tokens = 512 rows in total (scaling "strong", the cfg4 contract), or 512 per rank ("weak").  Exchange per layer: routed records and returned rows stored into the other ranks' memory over
    NVLink by the kernels (p2p, default on 2+ GPUs), or NCCL all-to-all (nccl); one GPU runs the single-GPU layer
    (local).  Layers are chained through an fp32 residual stream: each layer adds its MoE output, and its combine
    also leaves the next layer's bf16 input and amax."""
    name = "ep"
    unit = "tokens/s"
    dtype = "nvfp4"

    def __init__(self, pkg, torch, orc, rank=0, world=1, group=None, T=512, H=2816, I=704, E=128, topk=8, L=30,
                 exchange="p2p", scaling="strong"):
        import numpy as np
        import gemma_cuda_server_b200.expert_parallel as epm
        self.pkg, self.torch = pkg, torch
        self.exchange = exchange
        self.scaling = scaling
        self.ex = None
        if exchange == "p2p":       # one set of exchange buffers serves every layer (per-layer epochs)
            C = epm.P2PKernelOps.default_capacity(T, topk, world)
            self.ex = (epm.PeerExchange.create(pkg, world, C, H, group) if world > 1
                       else epm.PeerExchange.local_group(pkg, 1, C, H)[0])
        self.T, self.H, self.I, self.E, self.topk, self.L, self.G = T, H, I, E, topk, L, world
        El = E // world
        if scaling == "strong":      # this rank's slice of the one 512-row batch (the same rows at every G)
            gen = torch.Generator(device="cuda").manual_seed(4000)
            self.x0 = torch.randn((T * world, H), generator=gen, device="cuda")[rank * T:(rank + 1) * T]
            self.x0 = self.x0.to(torch.bfloat16).contiguous()
        else:
            gen = torch.Generator(device="cuda").manual_seed(4000 + rank)
            self.x0 = torch.randn((T, H), generator=gen, device="cuda").to(torch.bfloat16)
        self.x = torch.empty_like(self.x0)
        self.res = torch.empty((T, H), dtype=torch.float32, device="cuda")
        self.amax = torch.zeros(1, dtype=torch.float32, device="cuda")
        cal_ws = pkg.moe_workspace(T, H, I, El, topk)
        self.layers = []
        x = self.x0.clone()
        res = x.float()
        for l in range(L):
            lg = torch.Generator(device="cuda").manual_seed(5000 + l)              # router: same on every rank
            proj = (torch.randn((E, H), generator=lg, device="cuda") * 0.02).to(torch.bfloat16)
            wg = torch.Generator(device="cuda").manual_seed(6000 + 131 * l + rank)  # this rank's expert shard
            arena = pkg.MoeExperts(El, H, I)
            w13 = (torch.randn((El * 2 * I, H), generator=wg, device="cuda") * 0.02).to(torch.bfloat16)
            g = float(orc.global_scale_from_amax(pkg.amax(w13).item()))
            pkg.quantize(w13, gscale=g, packed=arena.w13.view(El * 2 * I, H // 2), scales=arena.w13_scales.view(-1))
            del w13
            arena.w1_gscale.fill_(g)
            arena.w3_gscale.fill_(g)
            w2 = (torch.randn((El * H, I), generator=wg, device="cuda") * 0.02).to(torch.bfloat16)
            g2 = float(orc.global_scale_from_amax(pkg.amax(w2).item()))
            pkg.quantize(w2, gscale=g2, packed=arena.w2.view(El * H, I // 2), scales=arena.w2_scales.view(-1))
            del w2
            arena.w2_gscale.fill_(g2)
            ops = (epm.P2PKernelOps(pkg, arena, E, topk, T, self.ex) if exchange == "p2p"
                   else epm.LocalOps(pkg, arena, E, topk, T) if exchange == "local"
                   else epm.KernelOps(pkg, arena, E, topk, T_cap=T, G=world))
            Ld = dict(proj=proj, arena=arena, ops=ops, layer=epm.ExpertParallelMoE(ops, group),
                      amax=torch.zeros(1, device="cuda"), ids=torch.empty((T, topk), dtype=torch.int32, device="cuda"),
                      w=torch.empty((T, topk), dtype=torch.float32, device="cuda"))
            # static down-projection input scales: calibrate this rank's experts on this layer's real input, with
            # every token sent to topk random local experts (each expert sees ~T*topk/El rows)
            pkg.amax(x, out=Ld["amax"])
            cal_ids = torch.argsort(torch.rand((T, El), generator=wg, device="cuda"), dim=1)[:, :topk].int().contiguous()
            cal_w = torch.full((T, topk), 1.0 / topk, device="cuda")
            h_amax = pkg.moe_calibrate(x, cal_ids, cal_w, arena, cal_ws, in_amax=Ld["amax"])
            arena.a2_gscale.copy_(torch.from_numpy(np.array(
                [orc.global_scale_from_amax(v) for v in h_amax.cpu().numpy()], np.float32)))
            pkg.moe_route(x, proj, topk, ops.src_ws, ids=Ld["ids"], weights=Ld["w"])
            Ld["layer"].forward(x, Ld["ids"], Ld["w"], res, in_amax=Ld["amax"], accumulate=True)
            x.copy_(res)
            self.layers.append(Ld)
        torch.cuda.synchronize()
        del cal_ws
        self.units_per_step = T                                   # rows of this rank; value() scales by G
        self.kernel_name = ("one MoE layer with its router (nvfp4b_moe_layer: router GEMM, top-k + dispatch ranking, "
                            "plan, quantise-scatter, grouped gate/up and down GEMMs, combine)"
                            if exchange == "local" else
                            "one expert-parallel layer on this rank with its router (nvfp4b_ep_p2p_layer: route, "
                            "records stored to the peers, local experts, rows stored back, combine), including its "
                            "waits for the other ranks" if exchange == "p2p" else
                            "expert side of one layer (record scatter, grouped gate/up and down GEMMs)")
        self.traffic_key = "ep" if exchange == "local" else None
        # one amax, then per layer -- local (nvfp4b_moe_layer): router GEMM, top-k + chunk ranking, plan,
        # quantise-scatter, gate/up, down, combine; p2p (nvfp4b_ep_p2p_layer): router GEMM, top-k + chunk ranking,
        # plan, pack, then meta + chunk ranking, plan, scatter, gate/up, down, and the combine with the next input
        # fused; nccl: router x2, hist-rank, plan, pack, meta + ranking, plan, scatter, gate/up, down, combine, amax
        self.launches_per_step = {"local": 7, "p2p": 10, "nccl": 12}[exchange] * L + 1
        self.kernel_flops = 2.0 * T * topk * 3 * I * H            # expert GEMMs of one layer at even routing
        self.step_flops = L * (2.0 * T * topk * 3 * I * H + 2.0 * T * E * H)
        self.config = {"workload": "cfg4 expert-parallel MoE stack", "layers": L, "rows_total": T * world,
                       "rows_per_gpu": T, "scaling": scaling, "hidden": H,
                       "experts": E, "experts_per_gpu": El, "inter": I, "topk": topk,
                       "capacity": self.ex.capacity if self.ex is not None else None,
                       "exchange": ("NVFP4 records and fp16 rows stored to peer memory over NVLink by the pack kernel "
                                    "and the down-GEMM epilogue, per-layer flags (no collective)") if exchange == "p2p"
                       else ("none: one GPU holds every expert (single-GPU MoE layer)" if exchange == "local"
                             else "NCCL all-to-all of NVFP4 records and fp16 rows per layer"),
                       "l2": "flushed between steps (256 MiB write + 256 MiB read)", "step_flops": self.step_flops}

    def step(self, mark=None):
        p, k = self.pkg, self.topk
        self.x.copy_(self.x0)
        self.res.copy_(self.x0)
        p.amax(self.x, out=self.amax)
        for li, Ld in enumerate(self.layers):
            # router + layer on the residual stream: res += MoE(x); the combine also leaves x = bf16(res) and its
            # amax for the next layer (one GPU: the router fused into the layer, nvfp4b_moe_layer)
            Ld["layer"].forward_routed(self.x, Ld["proj"], Ld["ids"], Ld["w"], self.res, in_amax=self.amax,
                                       accumulate=True, mark=mark if li == 0 else None, x_next=self.x,
                                       amax_next=self.amax)

    def value(self, seconds_per_step):
        return self.units_per_step / seconds_per_step

    def e2e_setup(self):
        t = self.torch
        self.h_x = t.empty((self.T, self.H), dtype=t.bfloat16, pin_memory=True)
        self.h_x.copy_(self.x0.cpu())
        self.h_out = t.empty((self.T, self.H), dtype=t.float32, pin_memory=True)
        return self.T * self.H * 2, self.T * self.H * 4

    def e2e_step(self):
        self.x0.copy_(self.h_x, non_blocking=True)
        if getattr(self, "graph", None) is not None:
            self.graph.replay()
        else:
            self.step()
        self.h_out.copy_(self.res, non_blocking=True)

    def _expert_bytes(self):
        I, H, p = self.I, self.H, self.pkg
        return (2 * I * H // 2 + p.nvfp4_scale_buffer_bytes(2 * I, H)) + (H * I // 2 + p.nvfp4_scale_buffer_bytes(H, I))

    def _rows_per_expert(self):
        """Rows each local expert ran in the last layer of the last step (host read of the dispatch plan)."""
        Ld = self.layers[-1]
        ops = Ld["ops"]
        El = self.E // self.G
        if self.exchange == "local":
            v = self.pkg.moe_view(ops.src_ws, self.T, self.H, self.I, El, self.topk)
        else:
            v = self.pkg.moe_view(ops.exp_ws, self.G * ops.capacity, self.H, self.I, El, 1)
        return v["seg_count"].cpu().tolist()

    def layer_bytes(self):
        """Algorithmic DRAM bytes of the timed part of one layer: the NVFP4 weights (codes + tile scales) of every
        local expert that received a row, read once, plus the layer's activations -- local layer (router included):
        x in (bf16), the residual read and written (fp32), the next input out (bf16) and the bf16 router weights;
        expert side of a rank: the records in (one per assignment) and one fp16 row per record out; the fused
        peer-memory layer runs both sides on every rank, so it counts both."""
        counts = self._rows_per_expert()
        hit = sum(1 for c in counts if c > 0)
        n = sum(counts)
        w = hit * self._expert_bytes()
        if self.exchange == "local":
            act = self.T * self.H * (2 + 4 + 4 + 2) + self.E * self.H * 2     # + the bf16 router weights
        elif self.exchange == "p2p":   # the whole layer on this rank: its tokens' side and its experts' side
            act = (self.T * self.H * (2 + 4 + 4 + 2) + self.E * self.H * 2 +
                   n * (self.pkg.ep_record_bytes(self.H) + 2 * self.H))
        else:
            act = n * (self.pkg.ep_record_bytes(self.H) + 2 * self.H)
        return {"weights": w, "activations": act, "total": w + act, "experts_hit": hit, "rows": n}

    def layer_flops(self):
        return 2.0 * sum(self._rows_per_expert()) * 3 * self.I * self.H

    def received(self, li=0):
        """Records this rank's experts ran in layer li's last run."""
        if self.exchange == "p2p":
            return sum(self.ex.recv_counts())        # one exchange for all layers: the last layer's counts
        if self.exchange == "local":
            return self.T * self.topk
        return int(self.layers[li]["ops"].counts[self.G:].sum().item())

    def close(self):
        if self.ex is not None:
            self.ex.close()
            self.ex = None

    def cpu_run(self, native, orc, seconds):
        """Layer 0 of the stack through the reference's experts() semantics (W4A4, dequantised experts, float32)
        on a token sample; tokens/s for the 30-layer stack = layer rate / 30."""
        Ld = self.layers[0]
        m = MoeWorkload.__new__(MoeWorkload)
        m.ids, m.wts, m.x, m.in_amax, m.arena = Ld["ids"], Ld["w"], self.x0, Ld["amax"], Ld["arena"]
        m.H, m.I, m.topk = self.H, self.I, self.topk
        rate, sample = MoeWorkload.cpu_run(m, native, orc, seconds)
        return rate / self.L, sample.replace("cfg3", "layer 0 of cfg4") + f"; stack rate = layer rate / {self.L}"


# ----------------------------------------------------------------------------------------------------------------

def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference_moe(args, world, orc):
    """The reference's CPU MoE semantics (scripts/ref_forward.py:160-192: softmax top-8 router, per-token loop over
    the selected experts, gelu_tanh(gate) * up, down, weighted sum) in W4A4 (x and h quantised with the NVFP4
    quantiser port), numpy float32 matmuls on all host threads.  Experts are dequantised once when first used; each
    step pushes a few tokens through one layer.  cfg4 (ep): tokens/s of the 30-layer stack = layer rate / 30."""
    import numpy as np
    import native
    H, I, E, topk = 2816, 704, 128, 8
    L = 30 if args.workload == "ep" else 1
    S = 4                                                     # tokens per step (bounded sample)
    rng = np.random.default_rng(7)
    proj = rng.standard_normal((E, H)).astype(np.float32) * 0.02
    experts = {}
    for e in range(E):        # N(0, 0.02) weights, NVFP4-quantised (C port), dequantised once -- before timing
        r = np.random.default_rng(1000 + e)
        mats = []
        for shape in ((2 * I, H), (H, I)):
            bits = orc.f32_to_bf16_bits(r.standard_normal(shape).astype(np.float32) * 0.02)
            g = orc.global_scale_from_amax(native.amax_bf16(bits))
            pk, sf = native.quantize_bf16(bits, g)
            mats.append(orc.dequantize(pk, sf, g).astype(np.float32))
        experts[e] = (mats[0], mats[1], 2688.0 / 0.05)         # static h scale (calibrated order of magnitude)

    def expert(e):
        return experts[e]

    def layer(x):
        logits = x @ proj.T
        p = np.exp(logits - logits.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        ids = np.argsort(-p, axis=1, kind="stable")[:, :topk]
        w = np.take_along_axis(p, ids, 1)
        w /= w.sum(1, keepdims=True)
        gin = orc.global_scale_from_amax(np.abs(x).max())
        _, _, xd = orc.quantize_rows(x.astype(np.float64), gin)
        xd = xd.astype(np.float32)
        out = np.zeros_like(x)
        for t in range(x.shape[0]):
            for j in range(topk):
                w13, w2, gh = expert(int(ids[t, j]))
                y = w13 @ xd[t]
                h = orc.gelu_tanh(y[:I]) * y[I:]
                _, _, hd = orc.quantize_rows(h[None].astype(np.float64), gh)
                out[t] += w[t, j] * (w2 @ hd[0].astype(np.float32))
        return out

    xs = rng.standard_normal((S * (args.warmup + args.steps), H)).astype(np.float32)
    for i in range(args.warmup):
        layer(xs[i * S:(i + 1) * S])
    t0 = time.perf_counter()
    for i in range(args.warmup, args.warmup + args.steps):
        layer(xs[i * S:(i + 1) * S])
    el = time.perf_counter() - t0
    val = S * args.steps / el / L
    workload = ("cfg4 expert-parallel MoE stack" if L > 1 else "cfg3 MoE FFN layer")
    sample = f"{S} tokens per step through one layer (E=128, top-8, H=2816, I=704); stack rate = layer rate / {L}"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "layers": L, "hidden": H, "experts": E, "inter": I, "topk": topk},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def run_reference_gemm(args, world, orc):
    """The reference's CPU GEMM (scripts/nvfp4_ref.py:102, gen_fp4_gemm_testcase.py:60): float64 X_deq @ W_deq^T of
    the NVFP4 operands, on cfg2's largest point (M=8192, K=4096, N=14336).  W is quantised and dequantised before
    timing; each step multiplies a sample of 64 activation rows (quantise + dequantise + matmul, BLAS threads)."""
    import numpy as np
    import native
    M, N, K, rows = 8192, 14336, 4096, 64
    wb = orc.synth_bf16((N, K), 0.02, seed=12)
    gw = orc.global_scale_from_amax(native.amax_bf16(wb))
    wd = native.dequantize(*native.quantize_bf16(wb, gw), gw)
    del wb
    xb = orc.synth_bf16((rows * (args.warmup + args.steps), K), 1.0, seed=11)
    gx = orc.global_scale_from_amax(native.amax_bf16(xb))

    def step(i):
        px, sx = native.quantize_bf16(xb[i * rows:(i + 1) * rows], gx)
        return native.dequantize(px, sx, gx) @ wd.T
    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.warmup, args.warmup + args.steps):
        step(i)
    el = time.perf_counter() - t0
    val = 2.0 * rows * N * K * args.steps / el / 1e12
    sample = f"{rows} of {M} rows per step, float64 dequant-matmul (N={N}, K={K})"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "cfg2 dense prefill GEMM, largest config", "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU implementation of the workload's path on the host cores; rank 0 only."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import native
    import nvfp4_oracle as orc
    if args.workload in ("moe", "ep"):
        run_reference_moe(args, world, orc)
        return
    if args.workload == "gemm":
        run_reference_gemm(args, world, orc)
        return
    if args.workload != "quant":
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU arm is timed for the quant and MoE workloads"}))
        return
    T, K = 8192, 2816
    rows = 1024                               # bounded sample per step
    bits = orc.synth_bf16((T, K), 1.0, seed=2024, outlier_frac=0.001)
    sample = bits[:rows]
    for _ in range(args.warmup):
        native.quantize_bf16(sample, orc.global_scale_from_amax(native.amax_bf16(sample)))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        native.quantize_bf16(sample, orc.global_scale_from_amax(native.amax_bf16(sample)))
    el = time.perf_counter() - t0
    val = rows * K * 2.5625 * args.steps / el / 1e9
    cores = native.num_threads()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "cfg1 activation quantiser, dynamic global scale", "T": T, "K": K},
        "cpu_baseline": {"value": val, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{rows} of {T} rows per step (C port of scripts/nvfp4_ref.py:71-82)"},
        "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def profile_kernels(torch, W, rank, world, barrier, steps=2):
    """Per-kernel device time per step of W on this rank (torch.profiler CUDA activity over `steps` eager steps,
    after the timed ones), printed to stderr rank by rank.  With several ranks a kernel that waits for another rank
    (record meta, combine) includes its wait."""
    import collections
    from torch.profiler import ProfilerActivity, profile
    barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            W.step()
        torch.cuda.synchronize()
    barrier()
    agg = collections.defaultdict(list)
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            name = e.name.replace("(anonymous namespace)::", "")
            epi = re.search(r"(\w+Epi)\b", name)          # the GEMM core's instances differ by epilogue policy
            agg[name.split("(")[0][:100] + (f" [{epi.group(1)}]" if epi else "")].append(e.device_time_total)
    rows = sorted(agg.items(), key=lambda kv: -sum(kv[1]))
    total = sum(sum(v) for _, v in rows) / steps
    text = "\n".join(f"kernels rank {rank}: {len(v) / steps:6.0f}/step {statistics.mean(v):9.2f} us  {k}"
                      for k, v in rows[:20])
    for r in range(world):
        if r == rank:
            print(text + f"\nkernels rank {rank}: device time per step {total:.1f} us", file=sys.stderr, flush=True)
        barrier()


def read_stream_ceiling(pkg, torch, W, flush, stream, barrier, reps=6):
    """The rate a pure TMA read of layer 0's expert weight codes reaches (nvfp4b_hbm_read_stream: the GEMMs' load
    path with no compute), one launch per arena as the layer's two grouped GEMMs stream them, L2 flushed before
    each launch, 3 untimed launches first.  A stream of a few hundred MB runs well below the 1 GiB copy peak (fixed
    ramp and tail), so this is the ceiling the layer's weight stream is compared with at its own size."""
    ar = W.layers[0]["arena"]
    out = {"kernel": "nvfp4b_hbm_read_stream (TMA boxes of 256 rows x 128 B, 4 stages, 1 CTA per SM, no compute)"}
    total_b, total_s = 0, 0.0
    for name, t in (("w13_codes", ar.w13), ("w2_codes", ar.w2)):
        nbytes = t.numel()
        rows = nbytes // 1408                     # [rows, 1408 B]: H/2 bytes per w13 row, 4 w2 rows (I/2 = 352 B)
        ms = []
        for i in range(3 + reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            pkg.hbm_read_stream(t, rows, 1408)
            b.record(stream)
            barrier()
            if i >= 3:
                ms.append(a.elapsed_time(b))
        sec = statistics.median(ms) / 1e3
        out[name] = {"bytes": rows * 1408, "us": sec * 1e6, "gbs": rows * 1408 / sec / 1e9}
        total_b += rows * 1408
        total_s += sec
    out["gbs"] = total_b / total_s / 1e9
    out["us"] = total_s * 1e6
    return out


def roofline_of(W, kern_s, peaks, peak_src, steps_s=None):
    """Roofline object of workload W's dominant kernel (or, for ep, one layer), from its event-timed duration."""
    hbm = peaks["hbm_gbs"]
    fp4_peak = peaks["bf16_tflops"] * 4.0
    fp4_src = f"{peak_src} bf16_tflops (burst) x 4 = dense FP4 rate of kind::mxf4nvf4"
    if W.name in ("quant", "w4a16"):
        achieved = W.kernel_bytes / kern_s / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": NCU_TRAFFIC.get(W.name), "kernel": W.kernel_name,
                "peak_source": f"{peak_src} hbm_gbs (copy, burst)"}
    if W.name == "ep":
        b = W.layer_bytes()
        achieved = b["total"] / kern_s / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": NCU_TRAFFIC.get(W.traffic_key), "kernel": W.kernel_name,
                "traffic_of": "the grouped gate/up GEMM, one launch (ncu dram__bytes_read + write; its algorithmic "
                              "bytes: 286 MB of w13 codes + scales and 5.8 MB of dispatched rows)",
                "algorithmic_bytes": b, "layer_us": kern_s * 1e6,
                "tensor": {"achieved": W.layer_flops() / kern_s / 1e12, "peak": fp4_peak, "unit": "TFLOP/s",
                           "frac": W.layer_flops() / kern_s / 1e12 / fp4_peak},
                "peak_source": f"{peak_src} hbm_gbs (copy, burst)"}
    flops = W.kernel_flops if W.name == "moe" else W.units_per_step
    achieved = flops / kern_s / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s", "frac": achieved / fp4_peak,
            "traffic": NCU_TRAFFIC.get(W.name), "kernel": W.kernel_name, "peak_source": fp4_src}
    if W.name == "moe" and steps_s:
        roof["step_tflops"] = W.step_flops / steps_s / 1e12
    return roof


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from __graft_entry__ import load_package
    sys.path.insert(0, str(ROOT / "oracle"))
    import nvfp4_oracle as orc   # seeded input generation; checker helpers

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    pkg = load_package()
    pkg.lib()
    if args.workload == "ep":
        exchange = args.ep_exchange if args.ep_exchange != "auto" else ("p2p" if world > 1 else "local")
        if exchange == "local" and world > 1:
            raise SystemExit("--ep-exchange local needs one GPU")
        if args.ep_scaling == "strong" and args.ep_rows % world:
            raise SystemExit(f"--ep-rows {args.ep_rows} does not split over {world} GPUs")
        rows = args.ep_rows // world if args.ep_scaling == "strong" else args.ep_rows
        W = EpWorkload(pkg, torch, orc, rank=rank, world=world, exchange=exchange, T=rows, scaling=args.ep_scaling,
                       L=args.ep_layers)
    else:
        W = {"quant": QuantWorkload, "gemm": GemmWorkload, "moe": MoeWorkload, "w4a16": W4a16Workload,
             "linear": LinearWorkload}[args.workload](pkg, torch, orc)
    # L2 flush between steps: write a 256 MiB buffer (evicts the step's data), then read another 256 MiB buffer so
    # the L2 is left holding clean lines (otherwise the next step would pay the flush's own write-backs).
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device="cuda")

    def flush():
        flush_w.zero_()
        flush_r.sum()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def eager_marks(Wk, n):
        """Kernel marks ("kernel" / "kernel_end" events on the launching stream) from n eager steps."""
        marks = [{} for _ in range(n)]
        for i in range(n):
            flush()

            def mark(name, i=i):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(stream)
                marks[i][name] = ev
            Wk.step(mark)
        barrier()
        return [m["kernel"].elapsed_time(m["kernel_end"]) for m in marks]

    def time_steps(Wk, steps, warmup, graph_capture, profiler_range=False):
        """W untimed warm-up steps, then `steps` timed steps (CUDA events on the launching stream around each, L2
        flushed before each outside the events).  Returns (step ms list, kernel ms list, graph or None)."""
        for _ in range(warmup):
            flush()
            Wk.step()
        barrier()
        graph = None
        if graph_capture:     # a launch-bound stack: one CUDA graph per step (fixed buffers, no host reads inside)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                Wk.step()
            barrier()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        marks = [{} for _ in range(steps)]
        if profiler_range:
            torch.cuda.profiler.start()
        for i in range(steps):
            flush()
            starts[i].record(stream)

            def mark(name, i=i):
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(stream)
                marks[i][name] = ev
            if graph is not None:
                graph.replay()
            else:
                Wk.step(mark)
            stops[i].record(stream)
        barrier()
        if profiler_range:
            torch.cuda.profiler.stop()
        step_ms = [a.elapsed_time(b) for a, b in zip(starts, stops)]
        if graph is not None:          # events cannot be taken inside a graph replay: marks from eager steps
            kern_ms = eager_marks(Wk, 3)
        else:
            kern_ms = [m["kernel"].elapsed_time(m["kernel_end"]) for m in marks]
        return step_ms, kern_ms, graph

    props = torch.cuda.get_device_properties(local)
    uuid = getattr(props, "uuid", None)
    uuid = ("GPU-" + str(uuid)) if uuid is not None and not str(uuid).startswith("GPU-") else uuid
    sampler = ClockSampler(local, uuid)

    with sampler:
        # the launch-bound steps (the 30-layer stack; the quantiser's memset + amax + quantise) replay one CUDA graph
        step_ms, kern_ms, graph = time_steps(W, args.steps, args.warmup, W.name in ("ep", "quant"),
                                             args.cuda_profiler_range)
        W.graph = graph
        # sustained window for the clock record (same steps, untimed); a step count all ranks agree on
        per_step = torch.tensor([sum(step_ms) / len(step_ms)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(per_step, op=dist.ReduceOp.MAX)
        n_clock = max(1, min(2000, int(args.clock_seconds * 1e3 / max(float(per_step.item()), 1e-3))))
        for i in range(n_clock):
            flush()
            if graph is not None:
                graph.replay()
            else:
                W.step()
            if i % 20 == 19:
                torch.cuda.synchronize()
        barrier()
    clocks = sampler.summary()

    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = W.value(ms_per_step / 1e3) * world

    # end to end through the public API with host buffers
    h2d, d2h = W.e2e_setup()
    for _ in range(3):
        W.e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(3, min(args.steps, 20))
    e0.record(stream)
    for _ in range(n_e2e):
        W.e2e_step()
    e1.record(stream)
    barrier()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = W.value(float(te.item()) / n_e2e / 1e3) * world

    if args.profile_kernels:
        profile_kernels(torch, W, rank, world, barrier)

    peaks, peak_src = load_peaks()
    kern_s = statistics.mean(kern_ms) / 1e3
    roof = roofline_of(W, kern_s, peaks, peak_src, steps_s=sum(step_ms) / 1e3 / args.steps)
    if W.name == "ep":
        roof["read_stream"] = read_stream_ceiling(pkg, torch, W, flush, stream, barrier)

    # driver-visible sub-results at N = 1: the quantiser (cfg1) and the dense GEMM (cfg2), same timing rules
    sub = None
    if W.name == "ep" and world == 1 and not args.no_sub:
        sub = {}
        sub_steps = max(10, min(args.steps, 50))
        for Wk in (QuantWorkload(pkg, torch, orc), GemmWorkload(pkg, torch, orc)):
            s_ms, k_ms, _ = time_steps(Wk, sub_steps, max(3, args.warmup), Wk.name == "quant")
            ks = statistics.mean(k_ms) / 1e3
            r = roofline_of(Wk, ks, peaks, peak_src)
            sub[Wk.name] = {"value": Wk.value(sum(s_ms) / len(s_ms) / 1e3), "unit": Wk.unit,
                            "ms_per_step": sum(s_ms) / len(s_ms), "steps": sub_steps, "config": Wk.config,
                            "roofline": r}
            del Wk
        torch.cuda.synchronize()

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        import native
        cv, sample = W.cpu_run(native, orc, args.cpu_seconds)
        cpu = {"value": cv, "unit": W.unit, "cores": native.num_threads() if W.name == "quant" else cpu_cores(),
               "kind": "port", "sample": sample}

    W.config["device_error"] = int(pkg.read_device_error())   # a bounded device wait that expired (0: none)
    if W.name == "ep":
        W.config["capacity_overflow"] = bool(sum(int(Ld["ops"].overflow.item()) for Ld in W.layers))
        W.config["graph"] = "one CUDA graph per step" if getattr(W, "graph", None) is not None else "eager"
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": W.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": getattr(W, "scaling", "weak"),
            "vs_baseline": None, "dtype": W.dtype, "data": "synthetic (seeded, shapes of BASELINE.json configs)",
            "config": {**W.config, "parallelism": f"expert parallel x{world}" if W.name == "ep" else f"replicas x{world}"},
            "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": W.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": W.launches_per_step * args.steps, "clocks": clocks}
        if sub is not None:
            line["sub_results"] = sub
        print(json.dumps(line))
    if getattr(W, "graph", None) is not None:      # a graph holding NCCL calls must go before the process group
        W.graph = None
        graph = None
        torch.cuda.synchronize()
    if W.name == "ep":                             # every rank done with every peer's buffers before they go
        barrier()
        W.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark of the fused decode-attention path on B200 (one JSON line on rank 0).

Default workload (batched): GQA fp16 single-query decode,
B=64 sequences per GPU, Hq=32, Hkv=8, N=16384 keys, D=128 -- the metric's
"decode-attn us/call & HBM GB/s at N=16K".  A step is one decode call over the
rank's batch.  Metric value = algorithmic HBM bytes (K, V, q, o, each byte once)
of all ranks / max-over-ranks device time, in GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Other workloads (--workload): fp16 (config 1), int8 / int8_b2048 (config 2),
int4 / int4_b2048 (config 3), sk (config 4 batch 1, gqa_sk_fast, L2-rotated).
Under torchrun (N>1) each rank runs the same per-rank workload on its own GPU
(sequences sharded, no collective on the data path: "scaling": "weak").
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import time

import torch

ROOT = pathlib.Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
PKG = "fused-quantized-kv-decode-attention_b200"
METRIC = "decode-attn µs/call & HBM GB/s (% of 8 TB/s) at N=16K; Llama-1B-arch tok/s"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    "gqa": dict(kind="gqa", B=64, Hq=32, Hkv=8, N=16384, D=128,
                desc="cfg4 batched: GQA fp16 decode B=64/GPU, Hq=32, Hkv=8, N=16384, D=128 (decode_attn_gqa)"),
    "gqa_int8": dict(kind="gqa_int8", B=64, Hq=32, Hkv=8, N=16384, D=128,
                     desc="cfg4 batched over an int8 KV cache: GQA int8 decode B=64/GPU, Hq=32, Hkv=8, N=16384, "
                          "D=128 (decode_attn_gqa_int8)"),
    "fp16": dict(kind="fp16", R=256, N=4096, D=128,
                 desc="cfg1: fp16 decode B=8 x 32 heads (R=256), N=4096, D=128 (decode_attn_fp16_mw)"),
    "int8": dict(kind="int8", R=8192, N=4096, D=128,
                 desc="cfg2: int8-KV decode B=256 x 32 heads (R=8192), N=4096, D=128 (decode_attn_int8_mw)"),
    "int8_b2048": dict(kind="int8", R=65536, N=4096, D=128,
                       desc="cfg2 sweep: int8-KV decode B=2048 x 32 heads, N=4096, D=128"),
    "int4": dict(kind="int4", R=8192, N=4096, D=128,
                 desc="cfg3: int4-KV decode B=256 x 32 heads (R=8192), N=4096, D=128 (decode_attn_int4)"),
    "int4_b2048": dict(kind="int4", R=65536, N=4096, D=128,
                       desc="cfg3 sweep: int4-KV decode B=2048 x 32 heads, N=4096, D=128"),
    "llama": dict(kind="llama", B=1, N=640, D=64, prompt=512, gen=128,
                  desc="cfg5: Llama-3.2-1B-architecture greedy decode, random N(0,0.02) bf16 weights, "
                       "prompt 512 + 128 generated tokens (KV cache type in config.kv_cache)"),
    "sk": dict(kind="sk", Hq=32, Hkv=8, N=16384, D=128, S=64,
               desc="cfg4: GQA split-K batch 1, Hq=32, Hkv=8, N=16384, D=128, S=64 (gqa_sk_fast), 8 rotated KV sets"),
    "qpt": dict(kind="quant8", R=8192, N=4096, D=128,
                desc="int8 per-token quantizer (qpt) over config 2's K: 8192 x 4096 tokens, D=128"),
    "quant_int4": dict(kind="quant4", R=8192, N=4096, D=128,
                       desc="int4 per-token quantizer + packer over config 3's K: 8192 x 4096 tokens, D=128"),
}

# Extra workloads timed in the default 1-GPU run (the "configs" key): the reference's published
# rows -- benchmarks/standalone_quant.json:6-33 (fp16 / int8 / int4), benchmarks/flashinfer_looptimed.json
# (split-K at D=64 and 128), the quantizers of nb:236-238 / nb:292-299 -- at BASELINE's configs.
CONFIG_SWEEP = [
    ("cfg1_fp16", "fp16", {}),
    ("cfg2_int8_b256", "int8", {}),
    ("cfg3_int4_b256_d128", "int4", {}),
    ("cfg3_int4_b256_d64", "int4", {"D": 64}),
    ("gqa_int8_b64_n16k", "gqa_int8", {}),
    ("sk_d128_n16k", "sk", {}),
    ("sk_d128_n64k", "sk", {"N": 65536, "S": 128}),
    ("sk_d64_n16k", "sk", {"D": 64}),
    ("sk_d64_n64k", "sk", {"D": 64, "N": 65536, "S": 128}),
] + [(f"sk_d{D}_n{N}", "sk", {"D": D, "N": N}) for D in (128, 64) for N in (512, 1024, 2048, 4096, 8192)] + [
    ("qpt_int8", "qpt", {}),
    ("quant_int4", "quant_int4", {}),
    ("cfg3_int4_b2048", "int4_b2048", {}),
    ("cfg2_int8_b2048", "int8_b2048", {}),
]


# The reference's published loop-timed gqa_sk_fast times (A100, us per call, Hq=32, Hkv=8, S=64;
# benchmarks/flashinfer_looptimed.json:6-149), printed beside the same shapes here.
REFERENCE_A100_SK_US = {
    64: {512: 10.48, 1024: 12.57, 2048: 16.93, 4096: 25.05, 8192: 39.23, 16384: 94.30},
    128: {512: 11.86, 1024: 14.71, 2048: 20.11, 4096: 30.63, 8192: 74.25, 16384: 129.34},
}


# ---------------------------------------------------------------------------- helpers
def algorithmic_bytes(w: dict) -> int:
    k = w["kind"]
    if k == "gqa":
        return 2 * w["B"] * w["Hkv"] * w["N"] * w["D"] * 2 + 2 * w["B"] * w["Hq"] * w["D"] * 2
    if k == "gqa_int8":
        return 2 * w["B"] * w["Hkv"] * w["N"] * (w["D"] + 2) + 2 * w["B"] * w["Hq"] * w["D"] * 2
    if k == "sk":
        return 2 * w["Hkv"] * w["N"] * w["D"] * 2 + 2 * w["Hq"] * w["D"] * 2
    R, N, D = w["R"], w["N"], w["D"]
    if k in ("quant8", "quant4"):   # per token: 2D read, D + 2 (int8) or D/2 + 2 (int4) written
        return R * N * (2 * D + (D if k == "quant8" else D // 2) + 2)
    qo = 2 * R * D * 2
    if k == "fp16":
        return 2 * R * N * D * 2 + qo
    code = R * N * D if k == "int8" else R * N * D // 2
    return 2 * code + 2 * R * N * 2 + qo


def path_dtype(kind: str) -> str:
    """Arithmetic types of the path: KV storage type and the accumulation type."""
    return {"int8": "i8 KV, f32 accumulate", "gqa_int8": "i8 KV, f32 accumulate",
            "int4": "i4 KV, f32 accumulate", "quant8": "f16 -> i8 codes + f16 scales",
            "quant4": "f16 -> packed i4 codes + f16 scales"}.get(kind, "f16 KV, f32 accumulate")


def plan_record(plan):
    """The library's launch plan (fqkv_decode_plan) as a JSON object."""
    if plan is None:
        return None
    kernels = ["fp16 (decode_f16_kernel)", "int8 CUDA-core (decode_quant_kernel)", "int4 CUDA-core (decode_quant_kernel)",
               "int8 tensor-core GQA (decode_qtc_kernel)", "int4 tensor-core (decode_qtc_kernel)"]
    merge = ("none" if plan[0] == 1 else "thread-block cluster / DSMEM, same launch" if plan[1]
             else "fp32 partials + PDL-chained combine kernel")
    return {"splits": plan[0], "cluster": plan[1], "ctas": plan[2], "keys_per_split": plan[3],
            "kernel": kernels[plan[4]], "split_merge": merge}


def dominant_kernel(w: dict, plan) -> str:
    """The library kernel(s) that take (nearly) all of a call's device time for workload `w` under `plan`."""
    k, D = w["kind"], w["D"]
    if k in ("quant8", "quant4"):
        return "quantize_tma_kernel<int4>" if k == "quant4" else "quantize_tma_kernel<int8>"
    names = {0: f"decode_f16_kernel<{D},{'1' if plan[1] else '0'}>", 1: f"decode_quant_kernel<false,{D}>",
             2: f"decode_quant_kernel<true,{D}>", 3: f"decode_qtc_kernel<{D},false,false>",
             4: f"decode_qtc_kernel<{D},true,true>"}
    name = names[plan[4]]
    return name + (" + combine_kernel (PDL-chained)" if plan[0] > 1 and not plan[1] else "")


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "measured (MEASURED_PEAKS.json hbm_gbs, copy read+write)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"


def committed_traffic(workload: str):
    """(DRAM bytes per launch of the dominant kernel, how they were measured) from the committed
    ncu summary ``profiles/dram_traffic.json``, or (None, reason)."""
    p = ROOT / "profiles" / "dram_traffic.json"
    try:
        d = json.loads(p.read_text())
    except Exception:
        return None, "no committed ncu traffic summary"
    e = d.get(workload)
    if e is None:
        return None, "no committed ncu capture for this workload"
    if isinstance(e, dict):
        return e.get("bytes"), e.get("source", d.get("_note", ""))
    return e, d.get("_note", "")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.gpu),
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        self.t0 = time.time()

    def stop(self) -> dict:
        self.t1 = time.time()
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------- workload setup
POOL_BYTES = 1 << 30
L2_ROTATE_BYTES = 537_000_000   # > 4 x the 126 MB L2: rotated input sets per call stream from HBM


def quantized_rows(quant, R: int, N: int, D: int, int4: bool, gen, dev):
    """codes [R, N, D or D/2] and fp16 scales [R, N]: the library's quantizer applied to N(0, 1) fp16 rows
    for the first 1 GiB of codes (the pool); rows past the pool repeat it (the B=2048 sweeps would
    otherwise spend minutes drawing 70-140 GB of fp16; every call still streams all R rows from HBM)."""
    H = D // 2 if int4 else D
    codes = torch.empty(R, N, H, device=dev, dtype=torch.uint8 if int4 else torch.int8)
    scales = torch.empty(R, N, device=dev, dtype=torch.float16)
    pool = max(1, min(R, POOL_BYTES // (N * H)))
    step = max(1, (1 << 29) // (N * D))  # quantize 1 GiB of fp16 at a time
    for r0 in range(0, pool, step):
        r1 = min(pool, r0 + step)
        x = torch.randn(r1 - r0, N, D, device=dev, generator=gen, dtype=torch.float16)
        c, sc = quant(x)
        codes[r0:r1].copy_(c)
        scales[r0:r1].copy_(sc)
        del x, c, sc
    for r0 in range(pool, R, pool):
        r1 = min(R, r0 + pool)
        codes[r0:r1].copy_(codes[:r1 - r0])
        scales[r0:r1].copy_(scales[:r1 - r0])
    return codes, scales


class Case:
    """Device-resident inputs and a zero-allocation launcher for one workload."""

    def __init__(self, pkg, w: dict, dev: torch.device, seed: int):
        self.pkg, self.w, self.dev = pkg, w, dev
        self.lib = pkg.native.lib()
        gen = torch.Generator(device=dev).manual_seed(seed)
        k = w["kind"]
        self.stream = torch.cuda.current_stream(dev)
        if k == "gqa":
            B, Hq, Hkv, N, D = w["B"], w["Hq"], w["Hkv"], w["N"], w["D"]
            # KV sets smaller than 4x L2 are rotated so every call streams from HBM
            self.n_sets = min(8, max(1, -(-L2_ROTATE_BYTES // (2 * B * Hkv * N * D * 2))))
            self.sets = [(torch.randn(B, Hq, D, device=dev, generator=gen, dtype=torch.float16),
                          torch.randn(B, Hkv, N, D, device=dev, generator=gen, dtype=torch.float16),
                          torch.randn(B, Hkv, N, D, device=dev, generator=gen, dtype=torch.float16))
                         for _ in range(self.n_sets)]
            self.q, self.K, self.V = self.sets[0]
            self.o = torch.empty(B, Hq, D, device=dev, dtype=torch.float16)
            nb = pkg.workspace_bytes("fp16", B, Hq, Hkv, N, D)
            self.ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
            self.nb = nb
            self.kernels_per_call = 1 + (1 if nb > 0 else 0)
        elif k == "gqa_int8":
            B, Hq, Hkv, N, D = w["B"], w["Hq"], w["Hkv"], w["N"], w["D"]
            self.q = torch.randn(B, Hq, D, device=dev, generator=gen, dtype=torch.float16)
            self.K = torch.empty(B, Hkv, N, D, device=dev, dtype=torch.int8)
            self.V = torch.empty_like(self.K)
            self.Ks = torch.empty(B, Hkv, N, device=dev, dtype=torch.float16)
            self.Vs = torch.empty_like(self.Ks)
            for b in range(B):  # quantize one sequence of fp16 at a time
                for dst, sdst in ((self.K, self.Ks), (self.V, self.Vs)):
                    x = torch.randn(Hkv, N, D, device=dev, generator=gen, dtype=torch.float16)
                    c, sc = pkg.qpt(x)
                    dst[b].copy_(c)
                    sdst[b].copy_(sc)
                    del x, c, sc
            self.o = torch.empty(B, Hq, D, device=dev, dtype=torch.float16)
            nb = pkg.workspace_bytes("int8", B, Hq, Hkv, N, D)
            self.ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
            self.nb = nb
            self.kernels_per_call = 1 + (1 if nb > 0 else 0)
        elif k == "sk":
            Hq, Hkv, N, D, S = w["Hq"], w["Hkv"], w["N"], w["D"], w["S"]
            self.sets = []
            for _ in range(8):  # 8 x 67 MB > 4 x L2: every call streams from HBM
                self.sets.append((torch.randn(Hq, D, device=dev, generator=gen, dtype=torch.float16),
                                  torch.randn(Hkv, N, D, device=dev, generator=gen, dtype=torch.float16),
                                  torch.randn(Hkv, N, D, device=dev, generator=gen, dtype=torch.float16)))
            self.mp = torch.empty(Hq, S, device=dev)
            self.lp = torch.empty(Hq, S, device=dev)
            self.op = torch.empty(Hq, S, D, device=dev)
            self.o = torch.empty(Hq, D, device=dev, dtype=torch.float16)
            self.i = 0
            self.kernels_per_call = 2
        elif k in ("quant8", "quant4"):
            R, N, D = w["R"], w["N"], w["D"]
            self.X = torch.empty(R * N, D, device=dev, dtype=torch.float16)
            step = (1 << 29) // D
            for t0 in range(0, R * N, step):
                self.X[t0:t0 + step].normal_(generator=gen)
            self.codes = torch.empty(R * N, D if k == "quant8" else D // 2, device=dev,
                                     dtype=torch.int8 if k == "quant8" else torch.uint8)
            self.scales = torch.empty(R * N, device=dev, dtype=torch.float16)
            self.kernels_per_call = 1
        else:
            R, N, D = w["R"], w["N"], w["D"]
            self.q = torch.randn(R, D, device=dev, generator=gen, dtype=torch.float16)
            self.o = torch.empty(R, D, device=dev, dtype=torch.float16)
            if k == "fp16":
                self.K = torch.randn(R, N, D, device=dev, generator=gen, dtype=torch.float16)
                self.V = torch.randn(R, N, D, device=dev, generator=gen, dtype=torch.float16)
            else:
                quant = pkg.qpt if k == "int8" else pkg.quant_int4_per_token
                self.K, self.Ks = quantized_rows(quant, R, N, D, k == "int4", gen, dev)
                self.V, self.Vs = quantized_rows(quant, R, N, D, k == "int4", gen, dev)
            fmt = {"fp16": "fp16", "int8": "int8", "int4": "int4"}[k]
            nb = pkg.workspace_bytes(fmt, R, 1, 1, N, D)
            self.ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
            self.nb = nb
            self.kernels_per_call = 1 + (1 if nb > 0 else 0)
        torch.cuda.synchronize(dev)
        self.plan = self._plan()
        if self.plan is not None:   # one kernel, plus the combine when splits merge through global partials
            self.kernels_per_call = 1 + (1 if self.plan[0] > 1 and self.plan[1] == 0 else 0)
        self._bind()

    def _plan(self):
        """The library's launch plan for this workload ([splits, cluster, CTAs, keys per split, kernel])."""
        import ctypes
        w, k = self.w, self.w["kind"]
        if k in ("quant8", "quant4"):
            return None
        out = (ctypes.c_int32 * 5)()
        if k in ("gqa", "gqa_int8", "sk"):
            fmt = 1 if k == "gqa_int8" else 0
            args = (1 if k == "sk" else w["B"], w["Hq"], w["Hkv"], w["N"], w["D"])
        else:
            fmt = {"fp16": 0, "int8": 1, "int4": 2}[k]
            args = (w["R"], 1, 1, w["N"], w["D"])
        rc = self.lib.fqkv_decode_plan(fmt, *args, getattr(self, "nb", 0) if k != "sk" else 1 << 40, out)
        if rc != 0:
            raise RuntimeError(f"plan failed: {self.pkg.native.last_error()}")
        return list(out)

    def _bind(self) -> None:
        """The C-ABI function and its argument list (all but the stream) for each call of the rotation,
        converted to ctypes values once, so a launch costs one foreign call."""
        import ctypes
        w, lib, k = self.w, self.lib, self.w["kind"]
        P, I = ctypes.c_void_p, ctypes.c_int64
        ws = (P(self.ws.data_ptr()) if self.nb else P(None), ctypes.c_size_t(self.nb)) if hasattr(self, "nb") else ()
        if k == "gqa":
            calls = [(lib.fqkv_decode_attn_gqa, (P(q.data_ptr()), P(K.data_ptr()), P(V.data_ptr()),
                                                 P(self.o.data_ptr()), I(w["B"]), I(w["Hq"]), I(w["Hkv"]), I(w["N"]),
                                                 I(w["D"]), I(8)) + ws) for q, K, V in self.sets]
        elif k == "gqa_int8":
            calls = [(lib.fqkv_decode_attn_gqa_int8, (P(self.q.data_ptr()), P(self.K.data_ptr()), P(self.V.data_ptr()),
                                                      P(self.Ks.data_ptr()), P(self.Vs.data_ptr()), P(self.o.data_ptr()),
                                                      I(w["B"]), I(w["Hq"]), I(w["Hkv"]), I(w["N"]), I(w["D"])) + ws)]
        elif k == "sk":
            calls = [(lib.fqkv_gqa_sk_fast, (P(q.data_ptr()), P(K.data_ptr()), P(V.data_ptr()), P(self.mp.data_ptr()),
                                             P(self.lp.data_ptr()), P(self.op.data_ptr()), P(self.o.data_ptr()),
                                             I(w["Hq"]), I(w["Hkv"]), I(w["N"]), I(w["D"]), I(w["S"]), I(8), I(8)))
                     for q, K, V in self.sets]
        elif k in ("quant8", "quant4"):
            fn = lib.fqkv_quantize_int8_per_token if k == "quant8" else lib.fqkv_quantize_int4_per_token
            calls = [(fn, (P(self.X.data_ptr()), P(self.codes.data_ptr()), P(self.scales.data_ptr()),
                           I(self.X.shape[0]), I(w["D"])))]
        elif k == "fp16":
            calls = [(lib.fqkv_decode_attn_fp16_mw, (P(self.q.data_ptr()), P(self.K.data_ptr()), P(self.V.data_ptr()),
                                                     P(self.o.data_ptr()), I(w["R"]), I(w["N"]), I(w["D"]), I(8)) + ws)]
        else:
            fn = lib.fqkv_decode_attn_int8_mw if k == "int8" else lib.fqkv_decode_attn_int4
            calls = [(fn, (P(self.q.data_ptr()), P(self.K.data_ptr()), P(self.V.data_ptr()), P(self.Ks.data_ptr()),
                           P(self.Vs.data_ptr()), P(self.o.data_ptr()), I(w["R"]), I(w["N"]), I(w["D"]), I(8)) + ws)]
        self._calls = calls
        self.i = 0

    def launch(self, stream: int | None = None) -> None:
        """One decode call through the C ABI, no allocation, on `stream` (a cudaStream_t handle; default:
        torch's current stream).  The arguments are bound once (see _bind)."""
        if stream is None:
            stream = torch.cuda.current_stream(self.dev).cuda_stream
        fn, args = self._calls[self.i % len(self._calls)]
        self.i += 1
        rc = fn(*args, stream)
        if rc != 0:
            raise RuntimeError(f"launch failed: {self.pkg.native.last_error()}")


def timing_methods(pkg, case: Case, w: dict, dev: torch.device, ms_call: float) -> dict:
    """The reference's other timing methods on the same workload and device-resident inputs: an
    eager loop of back-to-back C-ABI calls (flashinfer_looptimed.py:34-44), the median of single
    calls each bracketed by CUDA events and a synchronize (notebook lines 525-534), and the launch
    floor -- the same two on the op's smallest shape (flashinfer_looptimed.py:47-56).  Each part
    is capped at a few seconds of device time."""
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def loop_us(c: Case, n: int) -> float:
        s = torch.cuda.current_stream(dev).cuda_stream   # the caller's stream, resolved once
        for _ in range(3):
            c.launch(s)
        torch.cuda.synchronize(dev)
        a, b = ev(), ev()
        a.record()
        for _ in range(n):
            c.launch(s)
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) * 1e3 / n

    def single_median_us(c: Case, n: int) -> float:
        ts = []
        for _ in range(n):
            a, b = ev(), ev()
            a.record()
            c.launch()
            b.record()
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b) * 1e3)
        return statistics.median(ts)

    n_loop = max(20, min(200, int(3000.0 / max(ms_call, 1e-3))))
    n_single = max(10, min(100, int(2000.0 / max(ms_call, 1e-3))))
    small = dict(w)
    if w["kind"] in ("gqa", "gqa_int8"):
        small.update(B=1, N=64)
    elif w["kind"] == "sk":
        small.update(N=64)
    else:
        small.update(R=1, N=64)
    tiny = Case(pkg, small, dev, seed=7)
    return {"eager_loop_us_per_call": round(loop_us(case, n_loop), 3), "eager_loop_calls": n_loop,
            "single_call_median_us": round(single_median_us(case, n_single), 3), "single_calls": n_single,
            "launch_floor_us": round(loop_us(tiny, 200), 3),
            "launch_floor_single_call_median_us": round(single_median_us(tiny, 100), 3),
            "launch_floor_shape": {k: small[k] for k in ("B", "R", "Hq", "Hkv", "N", "D") if k in small}}


def e2e_run(pkg, case: Case, steps: int, dev: torch.device) -> dict:
    """Same metric through the public torch API with host (pinned) inputs copied in
    and the output read back every step, timed with CUDA events."""
    w = case.w
    k = w["kind"]
    if k == "gqa":
        host = [t.cpu().pin_memory() for t in (case.q, case.K, case.V)]
        dev_in = [torch.empty_like(t) for t in (case.q, case.K, case.V)]
        call = lambda: pkg.decode_attn_gqa(dev_in[0], dev_in[1], dev_in[2], 8)
    elif k == "gqa_int8":
        ts = (case.q, case.K, case.V, case.Ks, case.Vs)
        host = [t.cpu().pin_memory() for t in ts]
        dev_in = [torch.empty_like(t) for t in ts]
        call = lambda: pkg.decode_attn_gqa_int8(*dev_in)
    elif k == "sk":
        q, K, V = case.sets[0]
        host = [t.cpu().pin_memory() for t in (q, K, V)]
        dev_in = [torch.empty_like(t) for t in (q, K, V)]
        call = lambda: pkg.gqa_sk_fast(dev_in[0], dev_in[1], dev_in[2], case.mp, case.lp, case.op, case.o,
                                       w["S"], 8, 8) or case.o
    elif k in ("quant8", "quant4"):
        host = [case.X.cpu().pin_memory()]
        dev_in = [torch.empty_like(case.X)]
        quant = pkg.qpt if k == "quant8" else pkg.quant_int4_per_token
        call = lambda: quant(dev_in[0])
    elif k == "fp16":
        host = [t.cpu().pin_memory() for t in (case.q, case.K, case.V)]
        dev_in = [torch.empty_like(t) for t in (case.q, case.K, case.V)]
        call = lambda: pkg.decode_attn_fp16_mw(dev_in[0], dev_in[1], dev_in[2], 8)
    else:
        ts = (case.q, case.K, case.V, case.Ks, case.Vs)
        host = [t.cpu().pin_memory() for t in ts]
        dev_in = [torch.empty_like(t) for t in ts]
        op = pkg.decode_attn_int8_mw if k == "int8" else pkg.decode_attn_int4
        call = lambda: op(*dev_in, 8)
    h2d = sum(t.numel() * t.element_size() for t in host)
    if k in ("quant8", "quant4"):
        outs_host = [torch.empty(case.codes.shape, dtype=case.codes.dtype).pin_memory(),
                     torch.empty(case.scales.shape, dtype=torch.float16).pin_memory()]
    else:
        outs_host = [torch.empty(case.o.shape, dtype=torch.float16).pin_memory()]
    d2h = sum(t.numel() * t.element_size() for t in outs_host)

    def step():
        for d, h in zip(dev_in, host):
            d.copy_(h, non_blocking=True)
        o = call()
        for dst, src in zip(outs_host, o if isinstance(o, tuple) else (o,)):
            dst.copy_(src, non_blocking=True)

    step()
    torch.cuda.synchronize(dev)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(steps):
        step()
    s1.record()
    torch.cuda.synchronize(dev)
    ms = s0.elapsed_time(s1) / steps
    return {"ms": ms, "h2d": h2d, "d2h": d2h, "steps": steps}


# ---------------------------------------------------------------------------- CPU reference path
def cpu_reference_setup(w: dict):
    """The reference's CPU attention path (torch SDPA on fp16 CPU tensors, GQA by
    repeat_interleave, quantized KV dequantised first -- tests/test_kernels.py:14-16,
    :35-38, :49-50) on one sequence of the workload.  Returns (call, bytes, desc)."""
    from oracle import attention as oatt
    from oracle import quant as oq

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    k = w["kind"]
    if k == "gqa_int8":
        Hq, Hkv, N, D = w["Hq"], w["Hkv"], w["N"], w["D"]
        q = torch.randn(Hq, D, generator=g).half()
        Kc, Ks = oq.quantize_int8_per_token(torch.randn(Hkv, N, D, generator=g).half().numpy())
        Vc, Vs = oq.quantize_int8_per_token(torch.randn(Hkv, N, D, generator=g).half().numpy())
        G = Hq // Hkv

        def call():
            Kd = torch.from_numpy(oq.dequantize_int8(Kc, Ks)).half().repeat_interleave(G, 0)
            Vd = torch.from_numpy(oq.dequantize_int8(Vc, Vs)).half().repeat_interleave(G, 0)
            return oatt.sdpa_cpu_reference_path(q, Kd, Vd)
        nbytes = 2 * Hkv * N * (D + 2) + 2 * Hq * D * 2
        return call, nbytes, f"1 sequence (Hq={Hq}, Hkv={Hkv}, N={N}, D={D}, int8 KV dequantised) per call"
    if k in ("gqa", "sk"):
        Hq, Hkv, N, D = w["Hq"], w["Hkv"], w["N"], w["D"]
        q = torch.randn(Hq, D, generator=g).half()
        K = torch.randn(Hkv, N, D, generator=g).half()
        V = torch.randn(Hkv, N, D, generator=g).half()
        G = Hq // Hkv

        def call():
            return oatt.sdpa_cpu_reference_path(q, K.repeat_interleave(G, 0), V.repeat_interleave(G, 0))
        nbytes = 2 * Hkv * N * D * 2 + 2 * Hq * D * 2
        desc = f"1 sequence (Hq={Hq}, Hkv={Hkv}, N={N}, D={D}) per call"
        return call, nbytes, desc
    if k in ("quant8", "quant4"):
        N, D = w["N"], w["D"]
        X = torch.randn(32 * N, D, generator=g).half().numpy()   # one sequence's 32 heads of K
        quant = oq.quantize_int8_per_token if k == "quant8" else oq.quantize_int4_per_token
        nbytes = 32 * N * (2 * D + (D if k == "quant8" else D // 2) + 2)
        return (lambda: quant(X)), nbytes, f"1 sequence x 32 heads of K ({32 * N} tokens, D={D}) per call"
    rows, N, D = 32, w["N"], w["D"]  # one sequence's 32 heads
    q = torch.randn(rows, D, generator=g).half()
    Kf = torch.randn(rows, N, D, generator=g).half()
    Vf = torch.randn(rows, N, D, generator=g).half()
    desc = f"1 sequence x 32 heads (R=32, N={N}, D={D}) per call"
    if k == "fp16":
        return (lambda: oatt.sdpa_cpu_reference_path(q, Kf, Vf)), 2 * rows * N * D * 2 + 2 * rows * D * 2, desc
    if k == "int8":
        Kc, Ks = oq.quantize_int8_per_token(Kf.numpy())
        Vc, Vs = oq.quantize_int8_per_token(Vf.numpy())
        deq, code_bytes = oq.dequantize_int8, rows * N * D
    else:
        Kc, Ks = oq.quantize_int4_per_token(Kf.numpy())
        Vc, Vs = oq.quantize_int4_per_token(Vf.numpy())
        deq, code_bytes = oq.dequantize_int4, rows * N * D // 2

    def call():
        Kd = torch.from_numpy(deq(Kc, Ks)).half()
        Vd = torch.from_numpy(deq(Vc, Vs)).half()
        return oatt.sdpa_cpu_reference_path(q, Kd, Vd)
    return call, 2 * code_bytes + 2 * rows * N * 2 + 2 * rows * D * 2, desc


def cpu_reference_sample(w: dict, seconds: float) -> dict:
    call, nbytes, desc = cpu_reference_setup(w)
    call()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        call()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    per_call = el / n
    return {"value": nbytes / per_call / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{desc}; {n} calls in {el:.1f} s; {nbytes / 1e6:.1f} MB/call",
            "ms_per_call": per_call * 1e3}


# ---------------------------------------------------------------------------- config 5 (end to end)
def llama_1b_config():
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=128256, hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=64, max_position_embeddings=131072,
                       rms_norm_eps=1e-5, rope_theta=500000.0, tie_word_embeddings=True, initializer_range=0.02,
                       hidden_act="silu")


def run_llama(args, w) -> int:
    """Greedy decode tok/s: fqkv GraphDecoder vs transformers SDPA generate (the reference's stock path)
    and transformers + the fqkv hook (the reference's live-model path), same random weights."""
    from transformers import LlamaForCausalLM

    pkg = importlib.import_module(PKG)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, P, T = w["B"], w["prompt"], w["gen"]
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(llama_1b_config()).to(torch.bfloat16).eval()
    ids = torch.randint(0, model.config.vocab_size, (B, P), device=dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    # ---- ours: eager prefill + CUDA-graph decode steps
    dec = pkg.hf_integration.GraphDecoder(model, batch=B, max_len=P + T, kv_dtype=args.kv)
    dec.prefill(ids)
    dec.capture()
    best_pre, best_dec = 1e30, 1e30
    for _ in range(max(1, args.warmup // 3) + 2):
        e0, e1, e2 = ev(), ev(), ev()
        e0.record()
        dec.prefill(ids)
        e1.record()
        dec.generate(T - 1)
        e2.record()
        torch.cuda.synchronize(dev)
        best_pre, best_dec = min(best_pre, e0.elapsed_time(e1)), min(best_dec, e1.elapsed_time(e2))
    ours_tokens = torch.cat([dec.out_tokens[:, P:P + T]], dim=1).clone()
    decode_tps = B * (T - 1) / (best_dec / 1e3)
    e2e_tps = B * T / ((best_pre + best_dec) / 1e3)
    if args.profile_steps:
        # profiling run: a CUDA-profiler range (ncu --profile-from-start off) around K decode steps,
        # i.e. K replays of the step's graph after a fresh prefill; nothing else runs
        dec.prefill(ids)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.start()
        dec.generate(args.profile_steps)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        print(json.dumps({"workload": "llama", "batch": B, "kv": args.kv, "profile_steps": args.profile_steps,
                          "decode_tok_s": round(decode_tps, 2)}), flush=True)
        return 0

    # ---- stock transformers generate (SDPA) and the reference-style hook
    def hf_generate_tps(impl):
        model.config._attn_implementation = impl
        with torch.no_grad():
            model.generate(ids, max_new_tokens=8, do_sample=False, pad_token_id=0)
            torch.cuda.synchronize(dev)
            best = 1e30
            for _ in range(2):
                t0 = time.perf_counter()
                out = model.generate(ids, max_new_tokens=T, do_sample=False, pad_token_id=0)
                torch.cuda.synchronize(dev)
                best = min(best, time.perf_counter() - t0)
        model.config._attn_implementation = "sdpa"
        return B * T / best, out[:, P:]
    stock_tps, stock_tokens = hf_generate_tps("sdpa")
    hook_tps, hook_tokens = hf_generate_tps(pkg.hf_integration.register())

    # ---- agreement: teacher-forced SDPA logits on our sequence (first <= 4 sequences)
    nb = min(B, 4)
    seq = torch.cat([ids[:nb], ours_tokens[:nb]], dim=1)
    with torch.no_grad():
        ref_logits = model(seq).logits[:, P - 1:P - 1 + T].float()
    agree = (ref_logits.argmax(-1) == ours_tokens[:nb]).float().mean().item()
    # our own logits for the same steps (teacher forced by construction: same tokens)
    dec_chk = pkg.hf_integration.GraphDecoder(model, batch=B, max_len=P + T, keep_logits=True, kv_dtype=args.kv)
    dec_chk.prefill(ids)
    ours_logits = [dec_chk.logits[:nb].clone()]
    for _ in range(T - 1):
        dec_chk.step()
        ours_logits.append(dec_chk.logits[:nb].clone())
    ours_logits = torch.stack(ours_logits, dim=1)
    max_diff = (ours_logits - ref_logits).abs().max().item()
    line = {"metric": METRIC, "workload": "llama", "value": round(decode_tps, 2), "unit": "tok/s",
            "n_gpus": 1, "higher_is_better": True, "dtype": f"bf16 weights, {args.kv} KV", "data": "synthetic",
            "config": {"workload": w["desc"], "global_batch": B, "prompt": P, "gen": T, "head_dim": 64,
                       "kv_cache": f"{args.kv}, static, graph-captured decode step"
                       + (" (quantize-on-append)" if args.kv == "int8" else "")},
            "decode_tok_s": round(decode_tps, 2), "e2e_generate_tok_s": round(e2e_tps, 2),
            "prefill_ms": round(best_pre, 3), "decode_ms_per_step": round(best_dec / (T - 1), 4),
            "stock_sdpa_generate_tok_s": round(stock_tps, 2), "hf_hook_generate_tok_s": round(hook_tps, 2),
            "speedup_vs_stock_generate": round(e2e_tps / stock_tps, 3),
            "greedy_agreement_vs_sdpa_teacher_forced": round(agree, 4),
            "max_logit_diff_vs_sdpa": round(max_diff, 5),
            "token_match_stock_vs_ours": round((stock_tokens[:nb] == ours_tokens[:nb]).float().mean().item(), 4),
            "impl": "ours"}
    if args.split_mode != "auto":
        line["config"]["split_mode"] = args.split_mode
    print(json.dumps(line), flush=True)
    return 0


def run_llama_reference(args, w, rank: int) -> int:
    """Reference arm of config 5: the stock transformers SDPA decode (the reference notebook's baseline
    path) on the host cores, rank 0 only, on a bounded sample (1 sequence, prompt 512, 8 new tokens)."""
    if rank != 0:
        return 0
    from transformers import LlamaForCausalLM

    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(0)
    model = LlamaForCausalLM(llama_1b_config()).float().eval()
    model.config._attn_implementation = "sdpa"
    P, new = w["prompt"], 8
    ids = torch.randint(0, model.config.vocab_size, (1, P))
    with torch.no_grad():
        model.generate(ids, max_new_tokens=2, do_sample=False, pad_token_id=0)
        t0 = time.perf_counter()
        model.generate(ids, max_new_tokens=new, do_sample=False, pad_token_id=0)
        el = time.perf_counter() - t0
    value = new / el
    sample = f"1 sequence, prompt {P}, {new} generated tokens (prefill included), fp32 weights on CPU"
    line = {"impl": "reference", "metric": METRIC, "workload": "llama", "value": round(value, 3), "unit": "tok/s",
            "n_gpus": 1, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w["desc"], "global_batch": 1, "prompt": P, "gen": new},
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": torch.get_num_threads(),
                             "kind": "reference", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def tp_decode_measure(pkg, dist, model, ids, B: int, P: int, T: int, kv: str, world: int, rank: int,
                      local_rank: int, reps: int, fused: bool = False) -> dict | None:
    """One tensor-parallel decode configuration on every rank (collective): decode tok/s (CUDA events,
    max over ranks), tokens identical on all ranks, and -- on rank 0 -- agreement with the 1-GPU decoder
    on the same replicated weights and with teacher-forced SDPA logits (greedy agreement, max logit
    difference of the TP decoder's own logits).  Returns the record on rank 0, None elsewhere."""
    dev = torch.device("cuda", local_rank)
    GD = pkg.hf_integration.GraphDecoder
    ev = lambda: torch.cuda.Event(enable_timing=True)
    ids = ids[:B].contiguous()
    dec = GD(model, batch=B, max_len=P + T, kv_dtype=kv, tp_group=dist.group.WORLD, tp_fused=fused)
    dec.prefill(ids)
    dec.capture()
    best_pre, best_dec = 1e30, 1e30
    for _ in range(reps):
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)
        e0, e1, e2 = ev(), ev(), ev()
        e0.record()
        dec.prefill(ids)
        e1.record()
        dec.generate(T - 1)
        e2.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1), e1.elapsed_time(e2)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        best_pre, best_dec = min(best_pre, float(t[0])), min(best_dec, float(t[1]))
    ours = dec.out_tokens[:, P:P + T].clone()
    ref_tok = ours.clone()
    dist.broadcast(ref_tok, src=0)
    same = torch.tensor([float(torch.equal(ref_tok, ours))], device=dev)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    dec.release()
    # the TP decoder's own logits for the first sequences (eager steps, collective on every rank)
    nb = min(B, 4)
    chk = GD(model, batch=B, max_len=P + T, kv_dtype=kv, tp_group=dist.group.WORLD, keep_logits=True)
    chk.prefill(ids)
    tp_logits = [chk.logits[:nb].clone()]
    for _ in range(T - 1):
        chk.step()
        tp_logits.append(chk.logits[:nb].clone())
    tp_logits = torch.stack(tp_logits, dim=1)
    chk.release()
    rec = None
    if rank == 0:
        one = GD(model, batch=B, max_len=P + T, kv_dtype=kv)
        one.prefill(ids)
        one.capture()
        one.generate(T - 1)
        one_tok = one.out_tokens[:, P:P + T].clone()
        one.release()
        seq = torch.cat([ids[:nb], ours[:nb]], dim=1)
        with torch.no_grad():
            ref_logits = model(seq).logits[:, P - 1:P - 1 + T].float()
        rec = {"batch": B, "kv_cache": kv, "gather": "fused NVLink stores + bounded wait" if fused
               else "NCCL all_gather_into_tensor",
               "decode_tok_s": round(B * (T - 1) / (best_dec / 1e3), 2),
               "e2e_generate_tok_s": round(B * T / ((best_pre + best_dec) / 1e3), 2),
               "decode_ms_per_step": round(best_dec / (T - 1), 4), "prefill_ms": round(best_pre, 3),
               "tokens_identical_on_all_ranks": bool(same.item() == 1.0),
               "token_match_vs_1gpu_decoder": round((one_tok == ours).float().mean().item(), 4),
               "greedy_agreement_vs_sdpa_teacher_forced": round(
                   (ref_logits.argmax(-1) == ours[:nb]).float().mean().item(), 4),
               "max_logit_diff_vs_sdpa": round((tp_logits - ref_logits).abs().max().item(), 5)}
    dist.barrier(device_ids=[local_rank])
    return rec


def run_cfg5_1gpu(pkg, dev: torch.device) -> dict:
    """Config 5 on one GPU for the default run's record: the Llama-1B-architecture greedy decode
    (random N(0, 0.02) bf16 weights, seed 0, prompt 512, 128 generated tokens) at batch 1 and 64 with
    fp16 and int8 KV caches -- decode tok/s of the CUDA-graph step (CUDA events, best of 3), generate
    tok/s including the prefill, greedy agreement with and the largest logit difference from
    teacher-forced transformers SDPA logits (first 4 sequences), and stock transformers SDPA
    generate tok/s (the reference's baseline path) at each batch."""
    from transformers import LlamaForCausalLM

    GD = pkg.hf_integration.GraphDecoder
    P, T = WORKLOADS["llama"]["prompt"], WORKLOADS["llama"]["gen"]
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(llama_1b_config()).to(torch.bfloat16).eval()
    ids_all = torch.randint(0, model.config.vocab_size, (64, P), device=dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)
    recs = []
    for B in (1, 64):
        ids = ids_all[:B].contiguous()
        nb = min(B, 4)
        stock = None
        for kv in ("fp16", "int8"):
            dec = GD(model, batch=B, max_len=P + T, kv_dtype=kv)
            dec.prefill(ids)
            dec.capture()
            best_pre, best_dec = 1e30, 1e30
            for _ in range(3):
                e0, e1, e2 = ev(), ev(), ev()
                e0.record()
                dec.prefill(ids)
                e1.record()
                dec.generate(T - 1)
                e2.record()
                torch.cuda.synchronize(dev)
                best_pre, best_dec = min(best_pre, e0.elapsed_time(e1)), min(best_dec, e1.elapsed_time(e2))
            ours = dec.out_tokens[:, P:P + T].clone()
            dec.release()
            chk = GD(model, batch=B, max_len=P + T, kv_dtype=kv, keep_logits=True)
            chk.prefill(ids)
            lg = [chk.logits[:nb].clone()]
            for _ in range(T - 1):
                chk.step()
                lg.append(chk.logits[:nb].clone())
            lg = torch.stack(lg, dim=1)
            chk.release()
            seq = torch.cat([ids[:nb], ours[:nb]], dim=1)
            with torch.no_grad():
                ref_logits = model(seq).logits[:, P - 1:P - 1 + T].float()
            if stock is None:
                # the same generate call once untimed (first-call set-up of this shape), then timed
                model.config._attn_implementation = "sdpa"
                with torch.no_grad():
                    for rep in range(2):
                        torch.cuda.synchronize(dev)
                        t0 = time.perf_counter()
                        model.generate(ids, max_new_tokens=T, do_sample=False, pad_token_id=0)
                        torch.cuda.synchronize(dev)
                    stock = B * T / (time.perf_counter() - t0)
            recs.append({"batch": B, "kv_cache": kv,
                         "decode_tok_s": round(B * (T - 1) / (best_dec / 1e3), 2),
                         "e2e_generate_tok_s": round(B * T / ((best_pre + best_dec) / 1e3), 2),
                         "decode_ms_per_step": round(best_dec / (T - 1), 4), "prefill_ms": round(best_pre, 3),
                         "stock_sdpa_generate_tok_s": round(stock, 2),
                         "greedy_agreement_vs_sdpa_teacher_forced": round(
                             (ref_logits.argmax(-1) == ours[:nb]).float().mean().item(), 4),
                         "max_logit_diff_vs_sdpa": round((lg - ref_logits).abs().max().item(), 5)})
    del model
    torch.cuda.empty_cache()
    return {"workload": WORKLOADS["llama"]["desc"], "configs": recs,
            "timing": "decode: CUDA events around 127 graph-replayed steps, best of 3; stock: wall clock of "
                      "the second of two identical transformers generate calls"}


def tp_model(dist, dev, P: int):
    """The config-5 model (random N(0, 0.02) bf16 weights, seed 0) and prompt ids, identical on every rank."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(llama_1b_config()).to(torch.bfloat16).eval()
    for prm in model.parameters():          # identical replicated weights on every rank
        dist.broadcast(prm.data, src=0)
    ids = torch.randint(0, model.config.vocab_size, (64, P), device=dev)
    dist.broadcast(ids, src=0)
    return model, ids


def run_llama_tp(args, w, world: int, rank: int, local_rank: int) -> int:
    """Config 5 tensor-parallel over `world` GPUs by KV head (NCCL all-gather of the attention
    outputs every layer, inside the captured decode step); same model and workload as run_llama.
    Total work is fixed as the GPU count grows ("scaling": "strong")."""
    import torch.distributed as dist

    pkg = importlib.import_module(PKG)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    B, P, T = w["B"], w["prompt"], w["gen"]
    model, ids = tp_model(dist, dev, P)
    rec = tp_decode_measure(pkg, dist, model, ids, B, P, T, args.kv, world, rank, local_rank,
                            max(1, args.warmup // 3) + 2, fused=args.tp_gather == "fused")
    dist.destroy_process_group()
    if rank == 0:
        line = {"metric": METRIC, "workload": "llama", "value": rec["decode_tok_s"], "unit": "tok/s",
                "n_gpus": world, "higher_is_better": True, "scaling": "strong",
                "dtype": f"bf16 weights, {args.kv} KV", "data": "synthetic",
                "config": {"workload": w["desc"], "global_batch": B, "prompt": P, "gen": T, "head_dim": 64,
                           "parallelism": f"tp{world} by KV head (q/k/v rows, KV cache, attention sharded; "
                                          + rec["gather"] + " per layer; o_proj, MLP, LM head replicated)",
                           "kv_cache": f"{args.kv}, static, graph-captured decode step (collectives in the graph)"},
                "timing": "CUDA events, max over ranks", "gpu_launches_note": "per step: one CUDA graph replay",
                "impl": "ours", **{k: v for k, v in rec.items() if k not in ("batch", "kv_cache", "gather")}}
        print(json.dumps(line), flush=True)
    return 0


def run_multi_gpu_extras(pkg, dist, world: int, rank: int, local_rank: int, dev: torch.device,
                         gpu_index: int) -> dict | None:
    """Extra records of a multi-GPU run (every rank calls this; rank 0 gets the result):

    * ``cfg4_strong_kv_heads``: ONE batch-64 config-4 problem (Hq=32, Hkv=8, N=16384, D=128) with its KV
      heads sharded over the GPUs -- 8/world KV heads and their 32/world query heads per GPU, no
      collective on the data path; aggregate GB/s = the whole problem's bytes / the slowest GPU's time.
      Each rank checks one sequence of its shard against the float64 oracle.
    * ``cfg5_tensor_parallel``: the config-5 Llama-1B-architecture greedy decode tensor-parallel over
      all GPUs by KV head, batch 1 and 64, fp16 and int8 KV caches (tp_decode_measure)."""
    from oracle import attention as oatt

    out = {}
    full = dict(WORKLOADS["gqa"])
    if full["Hkv"] % world == 0:
        w = dict(full, Hq=full["Hq"] // world, Hkv=full["Hkv"] // world)
        case = Case(pkg, w, dev, seed=77 + rank)
        dist.barrier(device_ids=[local_rank])
        r = time_case(case, dev, gpu_index, min_seconds=0.3)
        ref = oatt.decode_attention_gqa(case.q[:1].cpu().numpy(), case.K[:1].cpu().numpy(), case.V[:1].cpu().numpy())
        case.launch()
        torch.cuda.synchronize(dev)
        err = float(abs(case.o[:1].float().cpu().numpy() - ref).max())
        t = torch.tensor([r["us"], err], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del case
        torch.cuda.empty_cache()
        us, err = float(t[0]), float(t[1])
        total = algorithmic_bytes(full)
        out["cfg4_strong_kv_heads"] = {
            "workload": full["desc"] + f", KV heads sharded {world} ways ({full['Hkv'] // world} KV / "
                                       f"{full['Hq'] // world} query heads per GPU)",
            "bytes_per_call": total, "us_per_call_max_over_ranks": round(us, 3),
            "aggregate_GB_s": round(total / (us * 1e-6) / 1e9, 1),
            "per_gpu_GB_s": round(total / world / (us * 1e-6) / 1e9, 1),
            "max_abs_err_vs_float64_oracle": err, "scaling": "strong",
            "timing": "CUDA-graph replays per rank, CUDA events, max over ranks"}
    if 8 % world == 0:
        P, T = 512, 128
        model, ids = tp_model(dist, dev, P)
        recs = []
        for B, kv in ((1, "fp16"), (64, "fp16"), (1, "int8"), (64, "int8")):
            rec = tp_decode_measure(pkg, dist, model, ids, B, P, T, kv, world, rank, local_rank, reps=3)
            if rank == 0:
                recs.append(rec)
        del model
        torch.cuda.empty_cache()
        out["cfg5_tensor_parallel"] = {
            "workload": WORKLOADS["llama"]["desc"] + f", tensor-parallel over {world} GPUs by KV head "
                                                     "(o_proj, MLP, LM head replicated)",
            "configs": recs, "scaling": "strong", "timing": "CUDA events, max over ranks"}
    return out if rank == 0 else None


# ---------------------------------------------------------------------------- every config in one run
def time_case(case: Case, dev: torch.device, gpu_index: int, min_seconds: float = 0.6) -> dict:
    """CUDA-event time per call of one workload: a CUDA graph of n back-to-back C-ABI calls replayed
    until the timed region lasts >= min_seconds, clocks sampled during it."""
    for _ in range(3):
        case.launch()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        case.launch()
    e1.record()
    torch.cuda.synchronize(dev)
    est_ms = max(e0.elapsed_time(e1) / 5, 1e-3)
    n = int(min(400, max(8, 50.0 / est_ms)))
    n -= n % 8                                     # whole rotations of the split-K KV sets
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(dev)):
        for _ in range(n):
            case.launch()
    graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(1, math.ceil(min_seconds * 1e3 / (n * est_ms)))
    sampler = ClockSampler(gpu_index)
    sampler.start()
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    del graph
    return {"us": e0.elapsed_time(e1) * 1e3 / (reps * n), "calls": reps * n, "clocks": clocks, "plan": case.plan}


def sk_l2_note(w: dict) -> str:
    """Where the rotated batch-1 split-K inputs live: 8 KV sets, streamed from HBM when they exceed L2."""
    tot = 8 * 2 * w["Hkv"] * w["N"] * w["D"] * 2
    if tot > 126e6:
        return f"8 rotated KV sets, {tot / 1e6:.0f} MB > L2"
    return (f"8 rotated KV sets, {tot / 1e6:.0f} MB: L2-resident (a latency-bound row, as the reference notes "
            "for its own short-N rows)")


def run_config_sweep(pkg, dev: torch.device, gpu_index: int, peak: float) -> dict:
    """Every BASELINE config (and the quantizers) timed on this GPU: one entry per workload."""
    out, t_start = [], time.time()
    for name, key, over in CONFIG_SWEEP:
        w = dict(WORKLOADS[key])
        w.update(over)
        t0 = time.time()
        case = None
        try:
            case = Case(pkg, w, dev, seed=4321)
            r = time_case(case, dev, gpu_index)
        except torch.cuda.OutOfMemoryError as exc:
            out.append({"name": name, "skipped": f"out of device memory: {str(exc).splitlines()[0]}"})
            continue
        finally:
            del case
            torch.cuda.empty_cache()
        nbytes = algorithmic_bytes(w)
        gbs = nbytes / (r["us"] * 1e-6) / 1e9
        plan = r["plan"]
        c = r["clocks"]
        out.append({"name": name, "workload": w["desc"] + "".join(f" [{k}={v}]" for k, v in over.items()),
                    "kernel": dominant_kernel(w, plan), "bytes_per_call": nbytes, "us_per_call": round(r["us"], 3),
                    "GB_s": round(gbs, 1), "pct_of_8TBps": round(100 * gbs / NOMINAL_HBM_GBS, 2),
                    "frac_of_measured_peak": round(gbs / peak, 4), "calls_timed": r["calls"],
                    "l2": sk_l2_note(w) if w["kind"] == "sk" else "inputs > L2",
                    "clocks": {"sm_mhz": c.get("sm_mhz"), "sm_max_mhz": c.get("sm_max_mhz"),
                               "reasons": c.get("reasons"), "samples": c.get("samples")},
                    "plan": plan_record(plan), "setup_plus_timing_s": round(time.time() - t0, 1)})
        ref_us = REFERENCE_A100_SK_US.get(w["D"], {}).get(w["N"]) if w["kind"] == "sk" else None
        if ref_us is not None:
            out[-1]["reference_a100_us"] = ref_us
    return {"entries": out, "wall_s": round(time.time() - t_start, 1),
            "timing": "CUDA-graph replays of back-to-back C-ABI calls with device-resident inputs, CUDA events",
            "data": "synthetic N(0,1) fp16; quantized KV: the library's quantizer on the first 1 GiB of codes, "
                    "repeated over the remaining rows"}


# ---------------------------------------------------------------------------- main
def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="gqa", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (sequences; 32 heads each for the row workloads)")
    ap.add_argument("--seq-len", type=int, default=None, help="override the context length N")
    ap.add_argument("--kv", default="fp16", choices=["fp16", "int8"], help="KV cache type of the llama workload")
    ap.add_argument("--tp-gather", default="nccl", choices=["nccl", "fused"],
                    help="llama workload under torchrun: NCCL all-gather or the attention kernel's fused NVLink gather")
    ap.add_argument("--head-dim", type=int, default=None, choices=[64, 128], help="override head_dim D")
    ap.add_argument("--no-clock-hold", action="store_true",
                    help="do not keep the GPU loaded for clock sampling after the timed region (profiling runs)")
    ap.add_argument("--eager", action="store_true",
                    help="time K eager C-ABI calls instead of one CUDA-graph replay of K calls")
    ap.add_argument("--no-extra-timing", action="store_true",
                    help="skip the eager-loop, single-call and launch-floor timings (1-GPU runs only)")
    ap.add_argument("--split-mode", default="auto", choices=["auto", "combine", "cluster"],
                    help="how split plans merge (fqkv_set_split_mode): the library's choice, partials + combine "
                         "kernel, or thread-block cluster")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="llama workload: after timing, run this many decode steps inside a CUDA-profiler range "
                         "(for ncu --profile-from-start off) and exit without the transformers comparison")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-config sweep of the default run (1 GPU: the 'configs' key; several "
                         "GPUs: the 'multi_gpu' key -- KV-head-sharded config 4 and tensor-parallel config 5)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    w = dict(WORKLOADS[args.workload])
    if args.batch is not None and w["kind"] != "sk":
        if w["kind"] in ("gqa", "gqa_int8"):
            w["B"] = args.batch
        else:
            w["R"] = 32 * args.batch
        w["desc"] += f" [batch overridden to {args.batch}]"
    if args.seq_len is not None:
        w["N"] = args.seq_len
        w["desc"] += f" [N overridden to {args.seq_len}]"
    if args.head_dim is not None:
        w["D"] = args.head_dim
        w["desc"] += f" [D overridden to {args.head_dim}]"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if w["kind"] == "llama":
        if args.batch is not None:
            w["B"] = args.batch
        if args.impl == "reference":
            return run_llama_reference(args, w, rank)
        if args.split_mode != "auto":  # how the attention's split plans merge (A/B of the merge modes)
            lib = importlib.import_module(PKG).native.lib()
            if lib.fqkv_set_split_mode({"combine": 1, "cluster": 2}[args.split_mode]) != 0:
                raise RuntimeError(importlib.import_module(PKG).native.last_error())
        return run_llama_tp(args, w, world, rank, local_rank) if world > 1 else run_llama(args, w)
    config = {"workload": w["desc"], "global_batch": None, "seq_len": w["N"], "head_dim": w["D"],
              "parallelism": f"{world} GPU(s), sequences sharded, no data-path collective",
              "l2": sk_l2_note(w) if w["kind"] == "sk" else "inputs larger than L2 per step (no flush needed)",
              "timing": "CUDA events around K eager C-ABI calls" if args.eager
              else "CUDA events around one CUDA-graph replay of K C-ABI calls"}
    if w["kind"] in ("gqa", "gqa_int8"):
        config["global_batch"] = w["B"] * world
    elif w["kind"] == "sk":
        config["global_batch"] = world
    else:
        config["global_batch"] = (w["R"] // 32) * world
    per_rank_bytes = algorithmic_bytes(w)

    # ---------------- reference arm: the reference's CPU path on host cores, rank 0 only
    if args.impl == "reference":
        if rank != 0:
            return 0
        call, nbytes, desc = cpu_reference_setup(w)
        for _ in range(args.warmup):
            call()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            call()
        ms = (time.perf_counter() - t0) * 1e3 / args.steps
        value = nbytes / (ms / 1e3) / 1e9
        res = {"cores": torch.get_num_threads(), "sample": desc}
        line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": path_dtype(w["kind"]), "data": "synthetic",
                "config": config,
                "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": res["cores"], "kind": "port",
                                 "sample": res["sample"] + f"; {args.steps} timed steps of one call"},
                "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    # ---------------- our arm
    pkg = importlib.import_module(PKG)
    mode = {"auto": 0, "combine": 1, "cluster": 2}[args.split_mode]
    if pkg.native.lib().fqkv_set_split_mode(mode) != 0:
        raise RuntimeError(pkg.native.last_error())
    if args.split_mode != "auto":
        config["split_mode"] = args.split_mode
    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    case = Case(pkg, w, dev, seed=1234 + rank)
    if getattr(case, "n_sets", 1) > 1:
        config["l2"] = f"{case.n_sets} rotated input sets > 4x L2"
    kernels_per_call = case.kernels_per_call
    main_plan = case.plan

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[local_rank]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local_rank
    sampler = ClockSampler(gpu_index)
    sampler.start()
    for _ in range(args.warmup):
        case.launch()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.eager:
        ev0.record()
        for _ in range(args.steps):
            case.launch()
        ev1.record()
    else:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch.cuda.Stream(dev)):
            for _ in range(args.steps):
                case.launch()
        graph.replay()  # untimed: first replay uploads the graph
        torch.cuda.synchronize(dev)
        barrier()
        ev0.record()
        graph.replay()
        ev1.record()
    torch.cuda.synchronize(dev)
    barrier()
    ms_total = ev0.elapsed_time(ev1)
    # keep the GPU loaded until the clock sampler has seen at least ~1 s of this kernel
    t_loaded = time.time() - sampler.t0
    while t_loaded < 1.2 and not args.no_clock_hold:
        for _ in range(50):
            case.launch()
        torch.cuda.synchronize(dev)
        t_loaded = time.time() - sampler.t0
    clocks = sampler.stop()

    t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
    methods = None
    if world == 1 and not args.no_extra_timing and w["kind"] not in ("quant8", "quant4"):
        methods = timing_methods(pkg, case, w, dev, ms_total / args.steps)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    value = per_rank_bytes * world / (ms_step / 1e3) / 1e9

    # e2e through the public torch API with host buffers
    e2e = None
    if not args.no_e2e:
        e_steps = max(3, min(args.steps, 10))
        r = e2e_run(pkg, case, e_steps, dev)
        te = torch.tensor([r["ms"]], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e_ms = float(te.item())
        e2e = {"value": round(per_rank_bytes * world / (e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
               "ms_per_step": round(e_ms, 3), "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]}

    sweep = multi = cfg5 = None
    if not args.no_configs and args.workload == "gqa" and not (args.batch or args.seq_len or args.head_dim):
        del case
        torch.cuda.empty_cache()
        if world == 1:
            sweep = run_config_sweep(pkg, dev, gpu_index, measured_peak()[0])
            cfg5 = run_cfg5_1gpu(pkg, dev)
        else:
            multi = run_multi_gpu_extras(pkg, dist, world, rank, local_rank, dev, gpu_index)

    if dist is not None:
        barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_src = measured_peak()
    achieved = per_rank_bytes / (ms_step / 1e3) / 1e9
    traffic, traffic_src = committed_traffic(args.workload) if not (args.batch or args.seq_len or args.head_dim) \
        else (None, "workload overridden: no committed capture")
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_src,
            "traffic": traffic, "traffic_source": traffic_src,
            "algorithmic_bytes_per_launch": per_rank_bytes,
            "note": "achieved = algorithmic bytes per call / CUDA-event time per call on the launch stream"
                    + (" (partial kernel + PDL-chained combine)" if kernels_per_call > 1 else "")}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        c = cpu_reference_sample(w, args.cpu_seconds)
        cpu = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in c.items() if k != "ms_per_call"}
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": path_dtype(w["kind"]), "data": "synthetic", "config": config,
            "us_per_call": round(ms_step * 1e3, 3), "pct_of_8TBps": round(100 * achieved / NOMINAL_HBM_GBS, 2),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": args.steps * kernels_per_call, "clocks": clocks, "impl": "ours",
            "plan": plan_record(main_plan)}
    if methods is not None:
        line["timing_methods"] = methods
    if sweep is not None:
        line["configs"] = sweep
    if cfg5 is not None:
        line["cfg5_llama_1gpu"] = cfg5
    if multi is not None:
        line["multi_gpu"] = multi
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

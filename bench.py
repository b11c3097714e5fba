"""Benchmark of the B200-native int8 LM path of OVNative.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (every N): BASELINE config 4.  64 CFG-paired utterances, lengths
uniform in [150, 800] tokens (seed 0), each a CFG pair of 2 x len rows (the
B = 2 batch the reference's CUDA path builds, cpp/src/model/tts.cpp:172-204),
are sharded over the N GPUs by longest-processing-time first (whole pairs per
GPU, no collective on the data path).  A step is one TTS diffusion step of
every utterance: the 28-layer Qwen3-0.6B-shaped LM forward of its CFG pair
(random-init int8 weights, 151,676-token vocabulary, int8 audio heads) and
the guided sampler on its logits.  Each GPU packs its pairs into forwards of
at most 16,384 rows.  value = tokens (rows) of all utterances x K / the
slowest rank's device time, in tokens/s; `scaling` is strong (the 64
utterances are the whole job at every N).

With N = 1 the line also carries config 1 (one layer's linear set at
M = 400, `layer_step`), configs 2 and 3 (`lm_forward`), the sampler, the
attention and the weight loader, each with its own device timing, bound and
the reference's CPU implementation timed beside it.

Numerics (--numerics): `fp16` (default) runs the fp16 tensor-core mainloops
(outputs within rel-L2 <= 1e-3 / max-abs <= 1e-2*rms of the reference);
`exact` the int8 mainloop that reproduces the reference bit for bit.

`--impl reference` times the reference's own CPU implementation of the
headline workload on the host cores (its LM forward, oracle/_ref, built from
the reference's sources).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_TOKENS = 400
N_LAYERS = 28
LAYER_METRIC = "int8 LM GEMM TOPS (one decoder layer's linear set, M=2x200)"
WORKLOAD = "config1: Qwen3-0.6B-shaped decoder layer linear set, int8, M=400"

# BASELINE config 4, the headline at every N: 64 CFG-paired utterances,
# lengths uniform in [150, 800] (seed 0), each a CFG pair of 2 x len rows,
# sharded over the GPUs by LPT; a step is one TTS diffusion step of every
# utterance (its LM forward + the guided sampler).
UTT_N, UTT_LO, UTT_HI, UTT_SEED = 64, 150, 800, 0
LM_LAYERS, LM_VOCAB = 28, 151676
MAX_ROWS = 16384
METRIC = ("LM forward tokens/s (config 4: 64 CFG-paired utterances, len U[150,800], "
          "utterance-parallel)")
UTT_WORKLOAD = ("config4: 64 CFG-paired utterances (2 x len rows each, len ~ U[150,800], seed "
                "0), one TTS step = 28-layer Qwen3-0.6B-shaped LM forward + guided sampler per "
                "utterance")


def env_int(k, d):
    v = os.environ.get(k)
    return int(v) if v not in (None, "") else d


def config(world: int) -> dict:
    return {
        "workload": WORKLOAD,
        "tokens_per_step": M_TOKENS,
        "hidden": 1024, "qkv": "2048|1024|1024", "o": "2048->1024", "gate_up": "3072|3072",
        "down": "3072->1024",
        "layers_rotated": N_LAYERS,
        "weights": "random int8 uniform[-127,127], scale |N(0,0.02)|/127, RMSNorm gains 1",
        "l2": "inputs larger than L2: each step reads a different layer's 15.7 MB of weights, "
              "28 layers = 440 MB",
        "parallelism": ("dp1" if world == 1 else
                        f"replicas x{world}: every GPU runs the same layer step (weak scaling of "
                        "the layer microbenchmark, no collectives)"),
        "attention": "out of scope; o_proj consumes the q projection (identity stand-in)",
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every `period` s."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, cuda_index: int, period: float = 0.01):
        self.samples = []
        self.reasons = 0
        self.pci_bus_id = None
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            # NVML numbers GPUs in PCI order and ignores CUDA_VISIBLE_DEVICES:
            # find the handle by the CUDA device's PCI bus id.
            self.pci_bus_id = _pci_bus_id(cuda_index)
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(self.pci_bus_id.encode())
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report why, keep running
            self.error = str(e)
        self.period = period
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception as e:
                self.error = str(e)
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t.is_alive():
            self._t.join()

    def summary(self) -> dict:
        names = sorted(k for k, bit in self.REASONS.items() if self.reasons & bit)
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}
        if self.pci_bus_id:
            out["pci_bus_id"] = self.pci_bus_id
        if self.error:
            out["error"] = self.error
        return out


def _pci_bus_id(cuda_index: int) -> str:
    """PCI bus id of CUDA device `cuda_index` in NVML's form
    (domain:bus:device.function)."""
    import torch
    p = torch.cuda.get_device_properties(cuda_index)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


# --------------------------------------------------------------- roofline
def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_traffic_config4(gemm: str, f16: bool) -> float | None:
    """DRAM bytes per launch of one of the config-4 forward's fp16 GEMMs (ncu,
    committed summary), or None."""
    p = os.path.join(ROOT, "profiles", "gemm_traffic_config4.json")
    if not f16 or not os.path.exists(p):
        return None
    with open(p) as f:
        k = json.load(f)["kernels"].get(gemm)
    return float(k["read"] + k["write"]) if k else None


def load_traffic(gemm: str, f16: bool) -> float | None:
    """DRAM bytes per launch of one of the step's GEMMs (ncu dram__bytes_read
    + dram__bytes_write) from the committed summary, or None."""
    p = os.path.join(ROOT, "profiles", "gemm_traffic_m400.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        v = d.get("fp16" if f16 else "exact", {}).get(gemm)
        return float(v) if v is not None else None
    return None


DTYPE = {
    "fp16": "fp16 x fp16 -> fp32 (int8 weights exact in fp16, activations fp16(q*asc))",
    "exact": "int8 (s8 x s8 -> s32 per 32-k block, fp32 epilogue)",
}
NUMERICS = {
    "fp16": "within rel-L2 <= 1e-3 / max-abs <= 1e-2*rms of the reference",
    "exact": "bit-identical to the reference",
}


def gemm_roofline(name: str, kernel: str, M: int, N: int, K: int, residual: bool,
                  out_bytes: int, gemm_us: float, f16: bool) -> dict:
    """Roofline of one GEMM of the step from its live launch time.
    Algorithmic bytes: s8 A + fp32 block scales (1.125*M*K), int8 W (N*K),
    fp32 wscale (4N), the output (`out_bytes`) and the residual read
    (4*M*N when accumulating).  The bound is the slower of HBM and the
    tensor pipe the kernel uses (dense bf16 for kind::f16; int8 = 2x bf16)."""
    peaks = load_peaks()
    alg_bytes = int(1.125 * M * K) + N * K + 4 * N + out_bytes + (4 * M * N if residual else 0)
    ops = 2 * M * N * K
    tensor_peak = peaks["bf16_tflops"] * (1 if f16 else 2)
    t_hbm = alg_bytes / (peaks["hbm_gbs"] * 1e9)
    t_tensor = ops / (tensor_peak * 1e12)
    if t_tensor >= t_hbm:
        achieved, peak, unit = ops / (gemm_us * 1e-6) / 1e12, tensor_peak, "TFLOP/s"
    else:
        achieved, peak, unit = alg_bytes / (gemm_us * 1e-6) / 1e9, peaks["hbm_gbs"], "GB/s"
    return {
        "kernel": f"{kernel} ({name}, M={M}, N={N}, K={K})",
        "bound": "tensor" if t_tensor >= t_hbm else "hbm",
        "achieved": round(achieved, 1),
        "peak": peak,
        "unit": unit,
        "frac": round(achieved / peak, 4),
        "peak_source": peaks["source"] + (" bf16 burst" if f16 else " 2x bf16 burst / hbm copy"),
        "algorithmic_bytes": alg_bytes,
        "algorithmic_ops": ops,
        "us_per_launch": round(gemm_us, 3),
        "roofline_us": round(max(t_hbm, t_tensor) * 1e6, 3),
        "traffic": load_traffic(name, f16),
    }


# ---------------------------------------------------------------- our arm
class LayerPath:
    """28 layers' weights, buffers and CUDA graphs of one numerics path."""

    def __init__(self, f16: bool, dev, stream, seed: int = 1000):
        import torch

        import ovnative_b200 as ovb
        from ovnative_b200 import layer as LY
        rng = np.random.default_rng(seed)
        self.f16 = f16
        self.layers = [LY.LayerWeights.from_host(LY.random_layer_host(rng), dev, f16=f16)
                       for _ in range(N_LAYERS)]
        self.buf = LY.LayerBuffers(M_TOKENS, dev, f16=f16)
        self.x0 = torch.from_numpy(
            rng.standard_normal((M_TOKENS, LY.HIDDEN)).astype(np.float32)).to(dev)
        self.x = self.x0.clone()
        # Eager warm-up sets the kernels' shared-memory attributes before capture.
        for lw in self.layers[:2]:
            LY.run(self.x, lw, self.buf)
        torch.cuda.synchronize()
        if ovb.device_status() != 0:
            raise RuntimeError("device wait timed out during warm-up")
        self.graphs = []
        with torch.cuda.stream(stream):
            for lw in self.layers:  # one graph per layer step
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    LY.run(self.x, lw, self.buf)
                self.graphs.append(g)
            self.chain = torch.cuda.CUDAGraph()  # all 28 steps; x reset first (1.6 MB)
            with torch.cuda.graph(self.chain, stream=stream):
                self.x.copy_(self.x0)
                for lw in self.layers:
                    LY.run(self.x, lw, self.buf)

    def run_steps(self, n: int):
        full, rest = divmod(n, N_LAYERS)
        for _ in range(full):
            self.chain.replay()
        for i in range(rest):
            self.graphs[i].replay()

    def release(self):
        for g in self.graphs + [self.chain]:
            g.reset()
        for lw in self.layers:
            lw.close()


def time_layer_step(args, dev, stream, world: int, barrier, max_over_ranks) -> dict:
    """one decoder layer's linear set at M = 400 (a CFG
    pair of 2 x 200 tokens), stepping through 28 layers' weights (L2-cold),
    replayed from CUDA graphs.  Returns the entry with its live per-GEMM
    roofline, the end-to-end pipelined step (host buffers in and out) and
    the other numerics path over the same steps."""
    import torch

    import ovnative_b200 as ovb
    from ovnative_b200 import layer as LY

    f16 = args.numerics == "fp16"
    path = LayerPath(f16, dev, stream)
    layers, buf, x0, x = path.layers, path.buf, path.x0, path.x
    graphs = path.graphs
    ops_step = M_TOKENS * LY.ops_per_token()

    with torch.cuda.stream(stream):
        path.run_steps(args.warmup)
    torch.cuda.synchronize()

    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        path.run_steps(args.steps)
        ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_max = max_over_ranks(ev0.elapsed_time(ev1))
    value = world * args.steps * ops_step / (ms_max * 1e-3) / 1e12

    # ---- the step's four GEMMs, each timed live: launches captured in a CUDA
    # graph so host launch cost is not timed, weights rotating over the 28
    # layers (L2-cold).  `roofline` is the one with the largest share.
    H, QKV, INTER = LY.HIDDEN, LY.QD + 2 * LY.KVD, LY.INTER
    kern = "gemm_h (fp16 mainloop)" if f16 else "gemm_s8_tc (int8 mainloop)"
    aq = buf.qh[0]
    xr = x0.clone()
    gemms = {
        # name: (launch(i), N, K, residual, output bytes)
        "qkv": ((lambda i: ovb.linear_h_sliced(aq, layers[i].qkv, [buf.q, buf.k, buf.v])) if f16
                else (lambda i: ovb.linear_s8_nk_packed_q_sliced(*buf.qh, layers[i].qkv,
                                                                 [buf.q, buf.k, buf.v])),
                QKV, H, False, 4 * M_TOKENS * QKV),
        "o": ((lambda i: ovb.linear_h(buf.qo[0], layers[i].o, xr, accumulate=True)) if f16
              else (lambda i: ovb.linear_s8_nk_packed_q_add(*buf.qo, layers[i].o, xr)),
              H, LY.QD, True, 4 * M_TOKENS * H),
        "gate_up+silu": ((lambda i: ovb.linear_h_silu(aq, layers[i].gate_up, out=buf.qi,
                                                      f16=True)) if f16
                         else (lambda i: ovb.linear_q_silu(*buf.qh, layers[i].gate_up,
                                                           out=buf.qi)),
                         2 * INTER, H, False,
                         M_TOKENS * INTER * (2 if f16 else 1) + 4 * M_TOKENS * INTER // 32),
        "down": ((lambda i: ovb.linear_h(buf.qi[0], layers[i].down, xr, accumulate=True)) if f16
                 else (lambda i: ovb.linear_s8_nk_packed_q_add(*buf.qi, layers[i].down, xr)),
                 H, INTER, True, 4 * M_TOKENS * H),
    }
    n_launch = 2 * N_LAYERS
    per_gemm = []
    with torch.cuda.stream(stream):
        ovb.rmsnorm_quantize_f32(x0, layers[0].post_ln, LY.RMS_EPS, out=buf.qh, f16=f16)
        ovb.s8_nk_quantize(buf.q, out=buf.qo, f16=f16)
        for name, (fn, N_g, K_g, res, ob) in gemms.items():
            gemm_us = _graph_time_us(stream, lambda i, fn=fn: fn(i % N_LAYERS), n_launch)
            per_gemm.append(gemm_roofline(name, kern, M_TOKENS, N_g, K_g, res, ob, gemm_us, f16))
    torch.cuda.synchronize()
    roofline = dict(max(per_gemm, key=lambda r: r["us_per_launch"]))
    roofline["all_gemms"] = [{k: r[k] for k in ("kernel", "us_per_launch", "bound", "achieved",
                                                "unit", "frac", "traffic")} for r in per_gemm]

    # ---- end to end through the public API with host buffers
    # Every step copies its own input from pinned host memory and reads its
    # result back.  Serial: copy in, step, copy out on one stream.  Pipelined
    # (the reported value), how a serving loop drives the layer: three device
    # buffers in rotation and one CUDA graph per (layer, rotation) holding
    # step i's compute (in place on buffer i%3), the host-to-device copy of
    # step i+1's input into buffer (i+1)%3 and the device-to-host copy of step
    # i-1's result from buffer (i-1)%3 on two copy streams, so the copies
    # overlap the compute and each step is one graph launch.
    rng = np.random.default_rng(77)
    h_in0 = torch.from_numpy(rng.standard_normal((M_TOKENS, LY.HIDDEN)).astype(np.float32))
    h_in0 = h_in0.pin_memory()
    h_out0 = torch.empty_like(h_in0).pin_memory()
    pipe = LY.StepPipeline(path.layers, path.buf, M_TOKENS, dev, stream)
    for r in range(3):
        pipe.host_in[r].copy_(h_in0)
    pipe.start()
    for r in range(3):  # warm
        pipe.step(r, 0)
    torch.cuda.synchronize()

    def timed_e2e(pipelined: bool) -> float:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        with torch.cuda.stream(stream):
            if not pipelined:
                for i in range(args.steps):
                    x.copy_(h_in0, non_blocking=True)
                    graphs[i % N_LAYERS].replay()
                    h_out0.copy_(x, non_blocking=True)
            else:
                pipe.start()
                for i in range(args.steps):
                    pipe.step(i, i % N_LAYERS)
                pipe.finish(args.steps - 1)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1))

    e2e_serial_ms = timed_e2e(False)
    e2e_ms = timed_e2e(True)
    io_bytes = M_TOKENS * LY.HIDDEN * 4
    e2e = {"value": world * args.steps * ops_step / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
           "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes,
           "ms_per_step": e2e_ms / args.steps,
           "mode": "pipelined: one CUDA graph per step holds its compute, the next step's "
                   "host-to-device copy and the previous step's device-to-host copy (two copy "
                   "streams, three buffers in rotation)",
           "serial_ms_per_step": e2e_serial_ms / args.steps}
    status = ovb.device_status()
    pipe.release()
    path.release()

    # ---- the other numerics path over the same K steps
    other_line = None
    if not args.skip_other:
        other = LayerPath(not f16, dev, stream)
        with torch.cuda.stream(stream):
            other.run_steps(args.warmup)
        barrier()
        torch.cuda.synchronize()
        o0 = torch.cuda.Event(enable_timing=True)
        o1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            o0.record(stream)
            other.run_steps(args.steps)
            o1.record(stream)
        torch.cuda.synchronize()
        barrier()
        o_ms = max_over_ranks(o0.elapsed_time(o1))
        status |= ovb.device_status()
        other.release()
        other_line = {"value": world * args.steps * ops_step / (o_ms * 1e-3) / 1e12,
                      "unit": "TOPS", "ms_per_step": o_ms / args.steps,
                      "numerics": NUMERICS["exact" if f16 else "fp16"]}
    if status != 0:
        raise RuntimeError(f"bounded device wait timed out (status {status})")
    return {
        "metric": LAYER_METRIC,
        "value": value,
        "unit": "TOPS",
        "steps": args.steps,
        "ms_per_step": ms_max / args.steps,
        "dtype": DTYPE[args.numerics],
        "numerics": NUMERICS[args.numerics],
        "config": config(world),
        ("exact" if f16 else "fp16"): other_line,
        "e2e": e2e,
        "gpu_launches": args.steps * LY.KERNELS_PER_LAYER,
        "roofline": roofline,
    }


def _graph_time_us(stream, fn, launches: int, warm: int = 3) -> float:
    """Device microseconds per call of fn(i): `warm` eager calls, then
    `launches` calls captured in one CUDA graph, replayed once untimed and
    once between CUDA events on `stream`."""
    import torch
    with torch.cuda.stream(stream):
        for i in range(warm):
            fn(i)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(launches):
                fn(i)
        g.replay()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
    e1.synchronize()
    g.reset()
    return e0.elapsed_time(e1) * 1e3 / launches


# ------------------------------------------------------ guided sampler
# The guided argmax pass of one TTS step at config 3's target (8 codebooks x
# 585 frames of the 1025-token audio vocabulary, cond plane of 700 tokens):
# HBM-bound, one read of both logits planes.
SAMPLER = {"codebooks": 8, "vocab": 1025, "target_len": 585, "cond_seq": 700,
           "uncond_seq": 585, "guidance": 3.0, "layer_penalty": 5.0, "mask_id": 1024}


def time_sampler(dev, stream, launches: int = 64, sets: int = 4) -> dict:
    """Device time per ovb_guided_sample launch, CUDA events around a graph
    of `launches` launches rotating over `sets` plane sets (168 MB > L2)."""
    import torch
    import ovnative_b200 as ovb
    sp = SAMPLER
    C, V, T = sp["codebooks"], sp["vocab"], sp["target_len"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    conds = [torch.randn((sp["cond_seq"], C * V), device=dev, generator=gen) * 3
             for _ in range(sets)]
    uncs = [torch.randn((sp["uncond_seq"], C * V), device=dev, generator=gen) * 3
            for _ in range(sets)]
    pred = torch.empty((C, T), dtype=torch.int32, device=dev)
    scores = torch.empty((C, T), dtype=torch.float32, device=dev)

    def one(i):
        ovb.guided_sample(conds[i % sets], uncs[i % sets], T, C, sp["guidance"],
                          sp["layer_penalty"], sp["mask_id"], pred, scores)

    with torch.cuda.stream(stream):
        for i in range(3):
            one(i)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(launches):
                one(i)
        g.replay()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / launches
    del g
    alg_bytes = 2 * C * T * V * 4 + C * T * 8
    peaks = load_peaks()
    achieved = alg_bytes / (us * 1e-6) / 1e9
    return {"kernel": "guided_sample_fixed_kernel<32, 1> (V = 1025; one warp per codebook x frame row)",
            "config": dict(sp), "us_per_launch": us, "rows": C * T, "bound": "hbm",
            "algorithmic_bytes": alg_bytes, "achieved": achieved, "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
            "peak_source": peaks["source"], "l2": "4 plane sets rotated, 168 MB > L2"}


def sampler_cpu_baseline(budget_s: float = 1.0) -> dict:
    """The C restatement of the reference's CPU loop (oracle port) on one
    whole step of SAMPLER, its frames split into one slice per host core and
    the slices run on concurrent threads (the ctypes calls release the GIL),
    as the reference's loop runs its rows in parallel: one warm-up step, then
    steps until `budget_s` (at least one)."""
    from concurrent.futures import ThreadPoolExecutor

    import oracle as O
    sp = SAMPLER
    C, V, T = sp["codebooks"], sp["vocab"], sp["target_len"]
    rng = np.random.default_rng(3)
    cond = (rng.standard_normal((sp["cond_seq"], C * V)) * 3).astype(np.float32)
    unc = (rng.standard_normal((sp["uncond_seq"], C * V)) * 3).astype(np.float32)
    cores = os.cpu_count() or 1
    bounds = np.linspace(0, T, min(cores, T) + 1).astype(int)
    off = sp["cond_seq"] - T  # the cond plane's target rows start here

    def part(i):
        t0, t1 = int(bounds[i]), int(bounds[i + 1])
        return O.guided_sample(cond[off + t0:off + t1], unc[t0:t1], t1 - t0, C, sp["guidance"],
                               sp["layer_penalty"], sp["mask_id"])

    with ThreadPoolExecutor(max_workers=len(bounds) - 1) as ex:
        list(ex.map(part, range(len(bounds) - 1)))
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget_s:
            list(ex.map(part, range(len(bounds) - 1)))
            n += 1
        sec = time.perf_counter() - t0
    return {"us_per_step": sec / n * 1e6, "cores": len(bounds) - 1, "kind": "port",
            "sample": f"{n} whole steps ({C} x {T} rows) in {sec:.2f} s, frames split over "
                      f"{len(bounds) - 1} threads"}


# ------------------------------------------------------------ GEMM M-sweep
# Config 4's isolated GEMM sweep: every LM projection shape at M = 16 ... 8192,
# both mainloops, weights rotating over enough copies to exceed L2.
SWEEP_SHAPES = {"q": (2048, 1024, False), "k/v": (1024, 1024, False), "o": (1024, 2048, True),
                "gate/up": (3072, 1024, False), "down": (1024, 3072, True),
                "qkv": (4096, 1024, False), "gate_up": (6144, 1024, False),
                "heads": (8200, 1024, False)}
SWEEP_M = (16, 64, 256, 1024, 4096, 8192)


def time_gemm_sweep(dev, stream, f16: bool, shapes=None, ms=SWEEP_M) -> list:
    """Device time per launch of one GEMM (CUDA events around a graph of
    launches) for every shape and M; weights rotate over copies totalling
    more than 150 MB so that every launch reads its weight from HBM."""
    import torch
    import ovnative_b200 as ovb
    out = []
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    kern = "gemm_h (fp16 mainloop)" if f16 else "gemm_s8_tc (int8 mainloop)"
    for name, (N, K, res) in (shapes or SWEEP_SHAPES).items():
        n_w = max(2, -(-150_000_000 // (N * K * (3 if f16 else 1))))
        ws = []
        for _ in range(n_w):
            W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=gen)
            sc = torch.rand((N,), device=dev, generator=gen) * (0.02 / 127)
            ws.append(ovb.Weight.from_nk(W, sc, f16=f16))
            del W
        for M in ms:
            A = torch.randn((M, K), device=dev, generator=gen)
            aq = ovb.s8_nk_quantize(A, f16=f16)
            C = torch.zeros((M, N), device=dev)
            if f16:
                fn = lambda w: ovb.linear_h(aq[0], w, C, accumulate=res)  # noqa: E731
            elif res:
                fn = lambda w: ovb.linear_s8_nk_packed_q_add(aq[0], aq[1], w, C)  # noqa: E731
            else:
                fn = lambda w: ovb.linear_s8_nk_packed_q(aq[0], aq[1], w, C)  # noqa: E731
            launches = max(2 * n_w, 8)
            with torch.cuda.stream(stream):
                for i in range(3):
                    fn(ws[i % n_w])
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for i in range(launches):
                        fn(ws[i % n_w])
                g.replay()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / launches
            g.reset()
            r = gemm_roofline(name, kern, M, N, K, res, 4 * M * N, us, f16)
            out.append({"shape": name, "M": M, "N": N, "K": K, "us": r["us_per_launch"],
                        "tops": round(2 * M * N * K / (us * 1e-6) / 1e12, 1),
                        "bound": r["bound"], "frac": r["frac"], "roofline_us": r["roofline_us"]})
            del A, aq, C
        for w in ws:
            w.close()
    if ovb.device_status() != 0:
        raise RuntimeError("bounded device wait timed out in the GEMM sweep")
    return out


def sweep_cpu_baseline(points, budget_s: float = 0.15) -> dict:
    """The reference's own int8 GEMM (linear_s8_nk_packed_q, AVX-VNNI,
    OpenMP on all host cores, through oracle/_ref) at every (shape, M) of the
    sweep: one warm-up call, then calls until `budget_s` (at least one);
    microseconds per call by (shape, M)."""
    import oracle as O
    if not O.ref_vnni():
        return {"unavailable": "the host has no AVX-VNNI (or oracle/_ref is not built)"}
    rng = np.random.default_rng(7)
    out, packed = {}, {}
    for name, M in points:
        N, K, res = SWEEP_SHAPES[name]
        if name not in packed:
            W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
            packed[name] = O.RefPacked(W, (np.abs(rng.standard_normal(N)) * 0.02 / 127)
                                       .astype(np.float32))
        pk = packed[name]
        aq, asc = O.ref_quantize(rng.standard_normal((M, K)).astype(np.float32))
        C0 = np.zeros((M, N), np.float32) if res else None
        pk.linear_q(aq, asc, C0)
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget_s:
            pk.linear_q(aq, asc, C0)
            n += 1
        out[f"{name}@{M}"] = round((time.perf_counter() - t0) / n * 1e6, 1)
    return {"us": out, "cores": os.cpu_count(), "kind": "reference",
            "what": "linear_s8_nk_packed_q[_add] (AVX-VNNI, OpenMP), activations pre-quantised"}


# ------------------------------------------------------------ weight load
def time_weight_load(dev, layers: int = 28) -> dict:
    """Load time of a synthetic checkpoint's int8 linear weights: a
    `layers`-layer OVW1 file of int8 [N, K] tensors (the reference's
    --int8-layout nk files; 440 MB at 28 layers), page cache warm.  Ours:
    ovb_ovw1_open + ovb_ovw1_weight per tensor (copy as stored, pack and
    widen to fp16 on the device), synchronised.  Reference: the host repack
    make_linear does per tensor (ov::s8_nk_pack into VNNI tiles + wsum,
    cpp/src/model/mat.cpp:95-101), one host thread as in the reference
    loader, on the same mapped payloads."""
    import shutil
    import tempfile

    import torch

    import oracle as O
    from ovnative_b200 import ovw1
    from ovnative_b200 import layer as LY
    rng = np.random.default_rng(11)
    shapes = [("q", LY.QD, LY.HIDDEN), ("k", LY.KVD, LY.HIDDEN), ("v", LY.KVD, LY.HIDDEN),
              ("o", LY.HIDDEN, LY.QD), ("gate", LY.INTER, LY.HIDDEN),
              ("up", LY.INTER, LY.HIDDEN), ("down", LY.HIDDEN, LY.INTER)]
    base = {n: rng.integers(-127, 128, size=(N, K), dtype=np.int8) for n, N, K in shapes}
    ts = []
    for li in range(layers):
        for n, N, K in shapes:
            ts.append((f"llm.layers.{li}.{n}_proj.weight", base[n], 0,
                       (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)))
    nbytes = sum(t[1].nbytes for t in ts)
    d = tempfile.mkdtemp(prefix="ovb_load_")
    try:
        path = os.path.join(d, "synthetic-int8-nk.ovw")
        ovw1.write(path, ts)
        with ovw1.OVW1File(path) as f:  # warm the page cache and the CUDA context
            for name, *_ in ts:
                f.array(name).sum()
        torch.cuda.synchronize()
        names = [t[0] for t in ts]

        def load_batch():
            with ovw1.OVW1File(path) as f:
                ws = f.weights(names, f16=True)
                torch.cuda.synchronize()
            return ws

        def load_one_by_one():
            with ovw1.OVW1File(path) as f:
                ws = [f.weight(name, f16=True) for name in names]
                torch.cuda.synchronize()
            return ws

        def timed(fn, reps=3):
            ts_ = []
            for _ in range(reps):
                t0 = time.perf_counter()
                ws = fn()
                ts_.append(time.perf_counter() - t0)
                for w in ws:
                    w.close()
            return float(np.median(ts_))

        ours = timed(load_batch)
        one_by_one = timed(load_one_by_one, reps=1)
        ref = None
        if O.ref_available():
            reps = []
            for _ in range(3):
                with ovw1.OVW1File(path) as f:
                    t0 = time.perf_counter()
                    for name in names:
                        O.RefPacked(f.array(name), f.scales(name))
                    reps.append(time.perf_counter() - t0)
            ref = float(np.median(reps))
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return {"what": f"{len(ts)} int8 [N, K] linear tensors of a {layers}-layer OVW1 file "
                    "(page cache warm)",
            "bytes": nbytes, "ms": round(ours * 1e3, 1), "GB/s": round(nbytes / ours / 1e9, 2),
            "one_by_one_ms": round(one_by_one * 1e3, 1), "fp16_copy": True,
            "cpu_baseline": None if ref is None else {
                "ms": round(ref * 1e3, 1), "cores": 1, "kind": "reference",
                "what": "ov::s8_nk_pack per tensor (make_linear's host repack)"}}


# ------------------------------------------------------------ LM forward
# BASELINE configs 2 and 3: the full 28-layer LM forward of a CFG pair
# (cond + uncond rows of S tokens each) with random-init int8 weights.
LM_CONFIGS = {"config2": 300, "config3": 700}


def _lm_inputs(rng, S, vocab, n_text=40):
    C, V = 8, 1025
    rows = 2 * S
    ids = rng.integers(0, V, size=(C, rows)).astype(np.int64)
    amask = np.ones(rows, np.uint8)
    amask[:n_text] = 0  # the conditional prompt's text ids
    ids[0, :n_text] = rng.integers(0, vocab, size=n_text)
    cond = np.ones((S, S), np.uint8)
    unc = np.ones((S, S), np.uint8)
    pos = np.concatenate([np.arange(S), np.arange(S)]).astype(np.int64)
    return ids, amask, cond, unc, pos


def time_lm_forward(dev, stream, f16: bool, layers: int = 28, vocab: int = 151676,
                    reps: int = 8, path: str | None = None, cpu: bool = True) -> dict:
    """LM forward tokens/s (cond + uncond rows per forward / time) at configs
    2 and 3 through ovb_lm: device-resident inputs, the forward captured in
    one CUDA graph, CUDA events around `reps` replays; e2e through
    ovb_lm_forward_cfg (host inputs in, host logits out, synchronous).  The
    reference's own LM::forward_cfg (oracle/_ref, OpenMP on all host cores)
    runs the same checkpoint and inputs on a bounded sample (one forward per
    config after one warm-up)."""
    import shutil
    import tempfile

    import torch

    import oracle as O
    import ovnative_b200 as ovb
    from ovnative_b200 import lm as LM
    from ovnative_b200 import ovw1
    d = None if path else tempfile.mkdtemp(prefix="ovb_lm_")
    out = {"layers": layers, "numerics": "fp16" if f16 else "exact", "vocab": vocab,
           "data": "synthetic (random-init int8 weights and embeddings, random ids)"}
    try:
        if path is None:
            path = os.path.join(d, "lm.ovw")
            ovw1.random_lm(path, n_layers=layers, vocab=vocab, seed=21)
        m = LM.LM(path, f16=f16)
        rng = np.random.default_rng(22)
        ref = O.RefLM(path, layers) if (cpu and O.ref_available()) else None
        for name, S in LM_CONFIGS.items():
            ids, amask, cond, unc, pos = _lm_inputs(rng, S, vocab)
            rows = 2 * S
            m.reserve(rows, 2 * S * S)
            t = [torch.from_numpy(np.ascontiguousarray(a)).to(dev)
                 for a in (ids, amask, cond, unc, pos)]
            with torch.cuda.stream(stream):
                for _ in range(3):
                    m.forward_cfg_device(*t)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    m.forward_cfg_device(*t)
                g.replay()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    g.replay()
                e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / reps
            g.reset()
            # end to end, host inputs: the TTS step as the reference's CUDA path
            # runs it (logits stay on the device, the guided sampler's
            # predictions and scores come back), and the forward alone with
            # the whole logits copied back (pinned staging)
            T = S - 40
            m.forward_cfg_sample(ids, amask, cond, unc, pos, T)
            t0 = time.perf_counter()
            for _ in range(3):
                m.forward_cfg_sample(ids, amask, cond, unc, pos, T)
            e2e_ms = (time.perf_counter() - t0) / 3 * 1e3
            m.forward_cfg(ids, amask, cond, unc, pos)
            t0 = time.perf_counter()
            for _ in range(3):
                m.forward_cfg(ids, amask, cond, unc, pos)
            e2e_logits_ms = (time.perf_counter() - t0) / 3 * 1e3
            entry = {"rows": rows, "ms": round(ms, 3), "tokens_per_s": round(rows / ms * 1e3, 1),
                     "e2e_ms": round(e2e_ms, 3),
                     "e2e_tokens_per_s": round(rows / e2e_ms * 1e3, 1),
                     "e2e_mode": "host ids in, forward with device logits, guided sampler, host "
                                 "pred/scores out (the reference CUDA path's device sampling)",
                     "e2e_host_logits_ms": round(e2e_logits_ms, 3)}
            if ref is not None:
                ref.forward_cfg(ids, amask, cond, unc, pos)
                t0 = time.perf_counter()
                ref.forward_cfg(ids, amask, cond, unc, pos)
                rs = time.perf_counter() - t0
                entry["cpu_baseline"] = {"ms": round(rs * 1e3, 1),
                                         "tokens_per_s": round(rows / rs, 1),
                                         "cores": os.cpu_count(), "kind": "reference",
                                         "what": "LM::forward_cfg (AVX-VNNI int8, OpenMP)"}
            out[name] = entry
        if ovb.device_status() != 0:
            raise RuntimeError("bounded device wait timed out in the LM forward")
        m.close()
        if ref is not None:
            ref.close()
    finally:
        if d:
            shutil.rmtree(d, ignore_errors=True)
    return out


# ------------------------------------------------------------ attention
# The attention of one layer at config 3's length: a CFG pair of 700-token
# segments (cond, uncond) with the reference's 0 / -1e30 padding bias, 16
# query heads over 8 kv heads of 128 dims.
ATTENTION = {"segments": [700, 700], "n_heads": 16, "n_kv": 8, "head_dim": 128,
             "pad_keys": 8}


def _attention_inputs(dev, gen, sets):
    import torch
    at = ATTENTION
    T = sum(at["segments"])
    H, KV, Dh = at["n_heads"], at["n_kv"], at["head_dim"]
    segs, r0 = [], 0
    for rows in at["segments"]:
        bias = torch.zeros((rows, rows), device=dev)
        bias[:, :at["pad_keys"]] = -1e30
        segs.append((bias, rows, r0 * H * Dh, r0 * KV * Dh))
        r0 += rows
    qs = [torch.randn((T, H * Dh), device=dev, generator=gen) for _ in range(sets)]
    ks = [torch.randn((T, KV * Dh), device=dev, generator=gen) for _ in range(sets)]
    vs = [torch.randn((T, KV * Dh), device=dev, generator=gen) for _ in range(sets)]
    return qs, ks, vs, segs


def attention_flops() -> int:
    """Algorithmic FLOPs of one layer's attention: 2 S^2 D for q k^T and
    2 S^2 D for p v, per segment and query head."""
    at = ATTENTION
    return sum(4 * s * s * at["head_dim"] * at["n_heads"] for s in at["segments"])


def time_attention(dev, stream, launches: int = 32, sets: int = 4) -> dict:
    """Device time per launch of the fp16-operand attention the LM runs
    (ovb_attention_h, the padding masks as a tile table) and of the
    fp32-operand ovb_attention, CUDA events around a graph of `launches`
    launches rotating over `sets` q/k/v sets (4 x 34 MB > L2)."""
    import torch
    import ovnative_b200 as ovb
    at = ATTENTION
    gen = torch.Generator(device=dev)
    gen.manual_seed(17)
    qs, ks, vs, segs = _attention_inputs(dev, gen, sets)
    outs = [torch.empty_like(q) for q in qs]
    q16s, k16s, v16s = ([t.half() for t in ts] for ts in (qs, ks, vs))
    masks = torch.cat([(b > -1e29).to(torch.uint8).reshape(-1) for b, _, _, _ in segs])
    tiles = ovb.attention_tiles([r for _, r, _, _ in segs], masks)
    segs_t = [(None, r, qo, ko) for _, r, qo, ko in segs]
    scale = 1.0 / float(np.sqrt(at["head_dim"]))

    def one_h(i):
        j = i % sets
        ovb.attention_h(q16s[j], k16s[j], v16s[j], segs_t, at["n_heads"], at["n_kv"], scale,
                        out=outs[j], tiles=tiles)

    def one_f32(i):
        j = i % sets
        ovb.attention(qs[j], ks[j], vs[j], segs, at["n_heads"], at["n_kv"], scale, out=outs[j])

    us = _graph_time_us(stream, one_h, launches)
    us32 = _graph_time_us(stream, one_f32, launches)
    flops = attention_flops()
    peaks = load_peaks()
    achieved = flops / (us * 1e-6) / 1e12
    return {"kernel": "attention_h_kernel (one CTA per segment x 128 query rows x kv head x "
                      "pair of query heads; fp16 q/k/v, tcgen05 kind::f16, S/P/O in TMEM)",
            "config": dict(at), "us_per_launch": us, "bound": "tensor",
            "algorithmic_flops": flops, "achieved": achieved, "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
            "peak_source": peaks["source"], "l2": "4 q/k/v sets rotated, 137 MB > L2",
            "fp32_operands": {"kernel": "attention_kernel (ovb_attention)", "us_per_launch": us32,
                              "frac": flops / (us32 * 1e-6) / 1e12 / peaks["bf16_tflops"]}}


def attention_cpu_baseline(budget_s: float = 1.0) -> dict:
    """The reference's own attention of one layer as LM::run_layer runs it
    (ov::attention_head_f32 per (segment, kv head, query head) in one OpenMP
    loop over all host cores, oracle/_ref) on the whole ATTENTION workload:
    one warm-up call, then calls until `budget_s` (at least one).  Without the
    reference library, the float64 restatement of the same loop on one core,
    on one (segment, head) unit scaled to the layer."""
    import oracle as O
    at = ATTENTION
    H, KV, Dh = at["n_heads"], at["n_kv"], at["head_dim"]
    rng = np.random.default_rng(5)
    scale = 1.0 / float(np.sqrt(Dh))
    if O.ref_available() and hasattr(O.ref_lib(), "ref_attention_layer"):
        T = sum(at["segments"])
        q = rng.standard_normal((T, H * Dh)).astype(np.float32)
        k = rng.standard_normal((T, KV * Dh)).astype(np.float32)
        v = rng.standard_normal((T, KV * Dh)).astype(np.float32)
        segs, r0 = [], 0
        for rows in at["segments"]:
            bias = np.zeros((rows, rows), np.float32)
            bias[:, :at["pad_keys"]] = -1e30
            segs.append((bias, rows, r0 * H * Dh, r0 * KV * Dh))
            r0 += rows
        O.attention_layer(q, k, v, segs, H, KV, Dh, scale)
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget_s:
            O.attention_layer(q, k, v, segs, H, KV, Dh, scale)
            n += 1
        sec = time.perf_counter() - t0
        return {"us_per_step": sec / n * 1e6, "cores": os.cpu_count(), "kind": "reference",
                "sample": f"{n} layer attentions (2 x {at['segments'][0]} rows, {H} heads) in "
                          f"{sec:.2f} s: ov::attention_head_f32 in the OpenMP loop of "
                          "LM::run_layer"}
    S = at["segments"][0]
    q = rng.standard_normal((S, Dh)).astype(np.float32)
    k = rng.standard_normal((S, Dh)).astype(np.float32)
    v = rng.standard_normal((S, Dh)).astype(np.float32)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s or n == 0:
        O.attention(q, k, v, [(None, S, 0, 0)], 1, 1, Dh, scale, use_ref=False)
        n += 1
    sec = time.perf_counter() - t0
    units = len(at["segments"]) * H
    return {"us_per_step": sec / n * units * 1e6, "cores": 1, "kind": "port",
            "sample": f"{n} (segment, head) units of {S} rows in {sec:.2f} s, scaled to {units}"}


# ------------------------------------------------- config 4: utterances
def utterance_lengths() -> dict:
    """uid -> length of the 64 config-4 utterances (seed 0)."""
    from ovnative_b200 import shard
    return dict(enumerate(int(x) for x in shard.synthetic_utterances(UTT_N, UTT_LO, UTT_HI,
                                                                      UTT_SEED)))


def config_utt(world: int, lengths: dict) -> dict:
    rows = sum(2 * v for v in lengths.values())
    return {
        "workload": UTT_WORKLOAD,
        "utterances": len(lengths),
        "rows_per_step": rows,
        "lengths": f"U[{UTT_LO},{UTT_HI}] seed {UTT_SEED}, sum {sum(lengths.values())}",
        "tts_step": "per utterance: LM forward of its B=2 CFG pair (cond = 40 text ids + "
                    "len-40 masked frames, uncond = the target slice; cpp/src/model/tts.cpp:"
                    "172-204) + guided sampler (guidance 2.0, layer_penalty 5.0)",
        "layers": LM_LAYERS, "vocab": LM_VOCAB, "audio_heads": "int8",
        "batching": f"each GPU packs its CFG pairs into forwards of <= {MAX_ROWS} rows "
                    "(attention segments stay per pair); with two or more batches, up to "
                    "four LM instances (--lanes) take the batches round-robin, each on its "
                    "own stream",
        "parallelism": f"dp{world}: utterance-parallel, LPT shards of whole CFG pairs, no "
                       "collective on the data path",
        "l2": "inputs larger than L2: every forward streams 449 MB of int8 weights (plus their "
              "fp16 copy on the fp16 path) and the batch's activations",
        "weights": "random-init int8, scale |N(0,0.02)|/127, RMSNorm gains 1 + N(0,0.05)",
    }


def shared_checkpoint(rank: int, world: int, dist=None) -> tuple[str, str]:
    """A 28-layer random-init checkpoint of the reference LM's shape (OVW1,
    151,676-token vocabulary, int8 heads), written once by rank 0 into a
    temporary directory whose path the other ranks receive.  Returns
    (path, directory)."""
    import tempfile

    from ovnative_b200 import ovw1
    obj = [None, None]
    if rank == 0:
        d = tempfile.mkdtemp(prefix="ovb_lm_")
        path = os.path.join(d, "lm28.ovw")
        ovw1.random_lm(path, n_layers=LM_LAYERS, vocab=LM_VOCAB, seed=21)
        obj = [path, d]
    if world > 1:
        dist.broadcast_object_list(obj, src=0)
    return obj[0], obj[1]


def cfg_attention_segments(seg_rows: list, dev):
    """The attention segments of packed CFG pairs (cond: every key attended;
    uncond: the target slice, then the tail rows seeing themselves,
    tts.cpp:186-198) over rows of the LM's q / k / v layout, and their tile
    table."""
    import torch

    import ovnative_b200 as ovb
    from ovnative_b200 import layer as LY
    segs, r0, masks = [], 0, []
    for si, rows in enumerate(seg_rows):
        mk = np.ones((rows, rows), np.uint8)
        if si % 2 == 1:
            T = max(1, rows - 40)
            mk[:] = 0
            mk[:T, :T] = 1
            mk[np.arange(T, rows), np.arange(T, rows)] = 1
        masks.append(mk.reshape(-1))
        segs.append((None, rows, r0 * LY.QD, r0 * LY.KVD))
        r0 += rows
    return segs, ovb.attention_tiles(seg_rows, torch.from_numpy(np.concatenate(masks)).to(dev))


def config4_biggest_batch_segments() -> list:
    """Segment rows of the largest config-4 batch one GPU runs (its CFG
    pairs' cond and uncond halves)."""
    from ovnative_b200 import shard
    from ovnative_b200 import tts_batch as TB
    lengths = utterance_lengths()
    uids = shard.lpt_assign([lengths[i] for i in range(len(lengths))], 1)[0]
    groups = TB.pack_batches(lengths, uids, MAX_ROWS)
    g = max(groups, key=lambda g: sum(2 * lengths[u] for u in g))
    return [lengths[u] for u in g for _ in range(2)]


def profile_attention() -> None:
    """Three launches of the forward's attention (fp16 operands, the CFG
    masks' tile table, the o projection's quantised input written by the
    epilogue) over the largest config-4 batch."""
    import torch

    import ovnative_b200 as ovb
    from ovnative_b200 import layer as LY
    dev = torch.device("cuda", 0)
    seg_rows = config4_biggest_batch_segments()
    M = sum(seg_rows)
    segs, tiles = cfg_attention_segments(seg_rows, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    q = torch.randn((M, LY.QD), device=dev, generator=gen).half()
    k = torch.randn((M, LY.KVD), device=dev, generator=gen).half()
    v = torch.randn((M, LY.KVD), device=dev, generator=gen).half()
    scale = 1.0 / float(np.sqrt(128))
    for _ in range(3):
        ovb.attention_h_q(q, k, v, segs, 16, 8, scale, tiles=tiles, f16=True)
    torch.cuda.synchronize()
    print(json.dumps({"attention": "config4", "rows": M, "segments": len(seg_rows),
                      "status": ovb.device_status()}), flush=True)


def time_forward_kernels(dev, stream, f16: bool, M: int, seg_rows: list,
                         n_layers: int = 8) -> dict:
    """Device time per launch of each GEMM and of the attention of a forward
    over M packed rows with the given attention segments: the GEMMs on
    random int8 weights of the LM's shapes rotating over `n_layers` layers
    (> L2), the attention on the segments with a 0 / -1e30 padding bias,
    each in a CUDA graph of launches between CUDA events.  Returns every
    kernel's roofline entry with its share of a 28-layer forward (time x
    launches per forward) and the dominant one."""
    import torch

    import ovnative_b200 as ovb
    from ovnative_b200 import layer as LY
    rng = np.random.default_rng(41)
    H, QD, KVD, INTER = LY.HIDDEN, LY.QD, LY.KVD, LY.INTER
    layers = [LY.LayerWeights.from_host(LY.random_layer_host(rng), dev, f16=f16)
              for _ in range(n_layers)]
    CV = 8 * 1025
    heads = [ovb.Weight.from_nk(rng.integers(-127, 128, size=(CV, H), dtype=np.int8),
                                (np.abs(rng.standard_normal(CV)) * 0.02 / 127).astype(np.float32),
                                f16=f16) for _ in range(3)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(42)
    x = torch.randn((M, H), device=dev, generator=gen)
    q = torch.randn((M, QD), device=dev, generator=gen)
    k = torch.randn((M, KVD), device=dev, generator=gen)
    v = torch.randn((M, KVD), device=dev, generator=gen)
    out = torch.empty_like(q)
    logits = torch.empty((M, CV), device=dev)
    qh = ovb.rmsnorm_quantize_f32(x, layers[0].input_ln, LY.RMS_EPS, f16=f16)
    qo = ovb.s8_nk_quantize(q, f16=f16)
    qi = ovb.linear_h_silu(qh[0], layers[0].gate_up) if f16 else \
        ovb.linear_q_silu(*qh, layers[0].gate_up)
    # at these batch sizes every fp16 GEMM runs on persistent CTA pairs
    kern = "gemm_h2_kernel (fp16 mainloop, CTA pairs)" if f16 else "gemm_s8_tc (int8 mainloop)"
    L_ = lambda i: layers[i % n_layers]  # noqa: E731
    # the fp16 forward's q|k|v GEMM carries the q/k norm + RoPE in its
    # epilogue and writes fp16 q / k / v (the LM's path, ovb_linear_h_qk_rope)
    tab = ovb.rope_table(torch.arange(M, device=dev, dtype=torch.int64))
    nrm = torch.ones(128, device=dev)
    qkv16 = (torch.empty((M, QD), dtype=torch.float16, device=dev),
             torch.empty((M, KVD), dtype=torch.float16, device=dev),
             torch.empty((M, KVD), dtype=torch.float16, device=dev))
    gemms = {
        "qkv": ((lambda i: ovb.linear_h_qk_rope(qh[0], L_(i).qkv, QD // 128, KVD // 128, nrm, nrm,
                                                LY.RMS_EPS, tab, out=qkv16)) if f16 else
                (lambda i: ovb.linear_s8_nk_packed_q_sliced(*qh, L_(i).qkv, [q, k, v])),
                QD + 2 * KVD, H, False, (2 if f16 else 4) * M * (QD + 2 * KVD), LM_LAYERS),
        "o": ((lambda i: ovb.linear_h(qo[0], L_(i).o, x, accumulate=True)) if f16 else
              (lambda i: ovb.linear_s8_nk_packed_q_add(*qo, L_(i).o, x)),
              H, QD, True, 4 * M * H, LM_LAYERS),
        "gate_up+silu": ((lambda i: ovb.linear_h_silu(qh[0], L_(i).gate_up, out=qi)) if f16 else
                         (lambda i: ovb.linear_q_silu(*qh, L_(i).gate_up, out=qi)),
                         2 * INTER, H, False, M * INTER * (2 if f16 else 1) + 4 * M * INTER // 32,
                         LM_LAYERS),
        "down": ((lambda i: ovb.linear_h(qi[0], L_(i).down, x, accumulate=True)) if f16 else
                 (lambda i: ovb.linear_s8_nk_packed_q_add(*qi, L_(i).down, x)),
                 H, INTER, True, 4 * M * H, LM_LAYERS),
        "heads": ((lambda i: ovb.linear_h(qh[0], heads[i % 3], logits)) if f16 else
                  (lambda i: ovb.linear_s8_nk_packed_q(*qh, heads[i % 3], logits)),
                  CV, H, False, 4 * M * CV, 1),
    }
    entries = []
    launches = 2 * n_layers
    for name, (fn, N_g, K_g, res, ob, per_fwd) in gemms.items():
        us = _graph_time_us(stream, fn, launches)
        r = gemm_roofline(name, kern, M, N_g, K_g, res, ob, us, f16)
        r["launches_per_forward"] = per_fwd
        r["us_per_forward"] = round(us * per_fwd, 1)
        r["traffic"] = load_traffic_config4(name, f16) if M == CONFIG4_BATCH_ROWS else None
        entries.append(r)
    # attention over the batch's segments with the LM's operands: fp16 q / k /
    # v and the tile table of the CFG masks
    segs, tiles = cfg_attention_segments(seg_rows, dev)
    q16, k16, v16 = q.half(), k.half(), v.half()
    scale = 1.0 / float(np.sqrt(128))
    us = _graph_time_us(stream, lambda i: ovb.attention_h(q16, k16, v16, segs, 16, 8, scale,
                                                          out=out, tiles=tiles), launches)
    flops = sum(4 * r * r * 128 * 16 for r in seg_rows)
    peaks = load_peaks()
    ach = flops / (us * 1e-6) / 1e12
    entries.append({"kernel": f"attention_h_kernel ({len(seg_rows)} segments, {M} rows)",
                    "bound": "tensor", "achieved": round(ach, 1), "peak": peaks["bf16_tflops"],
                    "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4),
                    "peak_source": peaks["source"] + " bf16 burst",
                    "algorithmic_flops": flops, "us_per_launch": round(us, 3),
                    "roofline_us": round(flops / (peaks["bf16_tflops"] * 1e12) * 1e6, 3),
                    "launches_per_forward": LM_LAYERS,
                    "us_per_forward": round(us * LM_LAYERS, 1), "traffic": None})
    for lw in layers:
        lw.close()
    for w in heads:
        w.close()
    if ovb.device_status() != 0:
        raise RuntimeError("bounded device wait timed out in the kernel timings")
    total = sum(e["us_per_forward"] for e in entries)
    for e in entries:
        e["share_of_timed_kernels"] = round(e["us_per_forward"] / total, 4)
    dom = dict(max(entries, key=lambda e: e["us_per_forward"]))
    dom["all_kernels"] = [{k: e[k] for k in ("kernel", "us_per_launch", "launches_per_forward",
                                             "share_of_timed_kernels", "bound", "achieved",
                                             "unit", "frac")} for e in entries]
    return dom


def time_utterances(args, rank: int, world: int, dev, stream, path: str, barrier,
                    max_over_ranks, sum_over_ranks, gather) -> dict:
    """The config-4 headline: this rank's LPT shard of the 64 utterances,
    packed into forwards, K TTS steps timed on the device (CUDA events on the
    launching stream, max over ranks), then the same K steps end to end (ids
    in from pinned host memory, predictions and scores back every step)."""
    import torch

    import ovnative_b200 as ovb
    from ovnative_b200 import lm as LM
    from ovnative_b200 import shard
    from ovnative_b200 import tts_batch as TB
    f16 = args.numerics == "fp16"
    lengths = utterance_lengths()
    plan = shard.lpt_assign([lengths[i] for i in range(len(lengths))], world)
    m = LM.LM(path, f16=f16)
    # with two or more batches, further LM instances (their own forward
    # buffers) let batches' forwards run on several streams at once
    n_batches = len(TB.pack_batches(lengths, plan[rank], MAX_ROWS)) if plan[rank] else 0
    extra = [LM.LM(path, f16=f16) for _ in range(min(args.lanes, n_batches) - 1)]
    sp = TB.Stepper(m, lengths, plan[rank], dev, stream, max_rows=MAX_ROWS, seed=rank,
                    extra_lms=extra)
    sp.warm_and_capture()
    for _ in range(args.warmup):
        sp.step()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            sp.step()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    my_ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(my_ms)
    rank_ms = gather(my_ms)
    rank_rows = gather(float(sp.rows_per_step))
    total_rows = sum(2 * v for v in lengths.values())
    value = args.steps * total_rows / (ms_max * 1e-3)

    # end to end: the same steps with host ids in and host predictions out
    for _ in range(2):
        sp.step_e2e()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        sp.step_e2e()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    h2d = int(sum_over_ranks(float(sp.h2d_bytes_per_step())))
    d2h = int(sum_over_ranks(float(sp.d2h_bytes_per_step())))
    # per forward: embedding gather, mask tile table, RoPE table; per layer
    # RMSNorm + quantise, q|k|v (+ q/k norm + RoPE in its epilogue on the fp16
    # path, a launch of its own on the int8 path), attention + o quantiser, o,
    # RMSNorm + quantise, gate|up + SiLU, down; final RMSNorm + quantise,
    # heads; then one sampler per CFG pair
    per_fwd = 3 + (7 if f16 else 8) * LM_LAYERS + 2
    # one batched sampler launch per batch (V = 1025)
    launches = int(sum_over_ranks(float(sum(per_fwd + 1 for b in sp.batches))))
    status = ovb.device_status()
    biggest = max(sp.batches, key=lambda b: b.rows) if sp.batches else None
    batches = [{"rows": b.rows, "pairs": len(b.pairs)} for b in sp.batches]
    sp.release()
    m.close()
    for e in extra:
        e.close()
    if status != 0:
        raise RuntimeError(f"bounded device wait timed out (status {status})")
    roofline = None
    if rank == 0 and biggest is not None and not args.no_roofline:
        roofline = time_forward_kernels(dev, stream, f16, biggest.rows, biggest.seg_rows)
    mean_ms = sum(rank_ms) / len(rank_ms)
    return {
        "value": value,
        "ms_per_step": ms_max / args.steps,
        "e2e": {"value": args.steps * total_rows / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms / args.steps,
                "mode": "every step, per batch: ids [C, rows] int64 copied in from pinned host "
                        "memory, the batch's CUDA graph (forward + samplers), predictions and "
                        "scores copied back to pinned host memory; a host synchronisation "
                        "ends the step"},
        "gpu_launches": launches * args.steps,
        "roofline": roofline,
        "ranks": {"device_ms": [round(x, 3) for x in rank_ms],
                  "rows_per_step": [int(x) for x in rank_rows],
                  "load_imbalance": round(max(rank_ms) / mean_ms, 4) if mean_ms > 0 else None,
                  "rank0_batches": batches},
        "clocks": clk.summary(),
        "config": config_utt(world, lengths),
    }


def utterance_cpu_baseline(path: str, budget_s: float, max_forwards: int = 1 << 30,
                           warmup: int = 1) -> dict:
    """The reference's own LM forward (LM::forward, B = 2 -- the CUDA path's
    CFG batch, cpp/src/model/tts.cpp:260-266 -- AVX-VNNI int8, OpenMP on all
    host cores, oracle/_ref) on a bounded sample of the config-4 utterances:
    one forward per utterance in id order after `warmup` untimed ones, until
    `budget_s` or `max_forwards`.  tokens/s = rows (2 x len) / time.  The
    sampler pass is not timed here (the reference's loop for it lives inside
    a Pipeline method; ~1 % of a CPU step)."""
    import oracle as O
    import oracle.cpu_baseline as CB
    from ovnative_b200 import tts_batch as TB
    if not O.ref_available():
        return {"unavailable": "oracle/_ref is not built"}
    lengths = utterance_lengths()
    rng = np.random.default_rng(3)
    ref = O.RefLM(path, LM_LAYERS)
    C = 8

    def b2(S):
        ids, amask, cond, unc, pos = TB.cfg_pair_inputs(rng, S, C)
        return (np.ascontiguousarray(ids.reshape(C, 2, S).transpose(1, 0, 2)),
                amask.reshape(2, S), np.stack([cond, unc]), pos.reshape(2, S))

    for u in range(warmup):
        ref.forward(*b2(lengths[u]))
    n, rows, t0 = 0, 0, time.perf_counter()
    u = warmup
    while n < max_forwards and (n == 0 or time.perf_counter() - t0 < budget_s):
        S = lengths[u % len(lengths)]
        ref.forward(*b2(S))
        rows += 2 * S
        n += 1
        u += 1
    sec = time.perf_counter() - t0
    ref.close()
    mode, kind = CB.pick_mode()
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return {"value": rows / sec, "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"{n} utterance forwards ({rows} rows, config-4 lengths in id order) in "
                      f"{sec:.1f} s: LM::forward B=2 (reference {mode} int8 path, OpenMP), "
                      "guided sampler not timed",
            "forwards": n, "seconds": sec, "host": CB.host_cpu()}


# --------------------------------------------------------------- our arm
def run_ours(args, rank: int, world: int, local_rank: int):
    import shutil

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def reduce(x: float, op) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max_over_ranks(ms: float) -> float:
        return reduce(ms, dist.ReduceOp.MAX if world > 1 else None)

    def sum_over_ranks(x: float) -> float:
        return reduce(x, dist.ReduceOp.SUM if world > 1 else None)

    def gather(x: float) -> list:
        if world == 1:
            return [x]
        t = torch.zeros(world, device=dev, dtype=torch.float64)
        t[rank] = x
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return [float(v) for v in t.tolist()]

    stream = torch.cuda.Stream(device=dev)
    f16 = args.numerics == "fp16"
    if args.workload == "layer":
        with ClockSampler(local_rank) as clk:
            out = time_layer_step(args, dev, stream, world, barrier, max_over_ranks)
        if world > 1:
            dist.destroy_process_group()
        if rank != 0:
            return None
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            import oracle.cpu_baseline as CB
            r = CB.run(M=M_TOKENS, layers=4, budget_s=args.cpu_seconds)
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "host")}
        out.update({"n_gpus": world, "warmup": args.warmup, "higher_is_better": True,
                    "scaling": "weak", "vs_baseline": None, "impl": "ours",
                    "data": "synthetic (seeded random-init int8 weights and N(0,1) activations)",
                    "cpu_baseline": cpu, "clocks": clk.summary()})
        return out

    path, tmpdir = shared_checkpoint(rank, world, dist if world > 1 else None)
    try:
        head = time_utterances(args, rank, world, dev, stream, path, barrier, max_over_ranks,
                               sum_over_ranks, gather)
        extras = {}
        if world == 1 and not args.headline_only:
            import ovnative_b200 as ovb
            # config 1's layer step is ~55 us: time 2800 of them (100 passes over
            # the 28 layers' weights) after 280 warm-up steps
            largs = argparse.Namespace(**{**vars(args), "steps": 2800, "warmup": 280})
            extras["layer_step"] = time_layer_step(largs, dev, stream, world, barrier,
                                                   max_over_ranks)
            extras["sampler"] = time_sampler(dev, stream)
            extras["attention"] = time_attention(dev, stream)
            if not args.no_cpu_baseline:
                extras["weight_load"] = time_weight_load(dev)
            extras["lm_forward"] = time_lm_forward(dev, stream, f16, path=path,
                                                   cpu=not args.no_cpu_baseline)
            if ovb.device_status() != 0:
                raise RuntimeError("bounded device wait timed out in the extra entries")
        barrier()
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            cpu = utterance_cpu_baseline(path, args.cpu_seconds)
            if "layer_step" in extras:
                import oracle.cpu_baseline as CB
                r = CB.run(M=M_TOKENS, layers=4, budget_s=min(args.cpu_seconds, 5.0))
                extras["layer_step"]["cpu_baseline"] = {
                    k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "host")}
            if "sampler" in extras:
                extras["sampler"]["cpu_baseline"] = sampler_cpu_baseline()
            if "attention" in extras:
                extras["attention"]["cpu_baseline"] = attention_cpu_baseline()
    finally:
        if rank == 0 and tmpdir:
            shutil.rmtree(tmpdir, ignore_errors=True)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    line = {
        "metric": METRIC,
        "value": head["value"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": DTYPE[args.numerics],
        "numerics": NUMERICS[args.numerics],
        "data": "synthetic (seeded random-init int8 weights and embeddings, random text ids, "
                "masked target frames)",
        "config": head["config"],
        "impl": "ours",
        "e2e": head["e2e"],
        "gpu_launches": head["gpu_launches"],
        "roofline": head["roofline"],
        "cpu_baseline": cpu,
        "ranks": head["ranks"],
        "clocks": head["clocks"],
    }
    line.update(extras)
    return line


# ---------------------------------------------------------- reference arm
def run_reference(args, rank: int, world: int):
    """The reference's own CPU implementation of the headline workload on
    the host cores (oracle/_ref: its LM forward), rank 0 only: after one
    untimed forward, one utterance forward per step, at most --steps of them
    and at most --ref-seconds, on the config-4 checkpoint and lengths."""
    if rank != 0:
        return None
    # torchrun sets OMP_NUM_THREADS=1 for every rank; rank 0 alone runs the
    # reference here, on all the host cores it may use.  OpenMP reads the
    # variable when its runtime loads, which has not happened yet (nothing
    # above imports torch or the reference library).
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    import shutil
    if args.workload == "layer":
        import oracle.cpu_baseline as CB
        r = CB.run(M=M_TOKENS, layers=4, max_steps=args.steps, budget_s=args.ref_seconds,
                   warmup=min(args.warmup, 3))
        return {
            "metric": LAYER_METRIC, "value": r["value"], "unit": "TOPS", "n_gpus": world,
            "steps": r["steps"], "warmup": min(args.warmup, 3),
            "ms_per_step": r["seconds"] * 1e3 / max(r["steps"], 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 (u8 x s8 VNNI per 32-k block, fp32 epilogue)",
            "data": "synthetic (seeded random-init int8 weights and N(0,1) activations)",
            "config": config(world), "impl": "reference",
            "cpu_baseline": {"value": r["value"], "unit": "TOPS", "cores": r["cores"],
                             "kind": r["kind"], "sample": r["sample"], "host": r["host"]},
            "e2e": {"value": r["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    path, tmpdir = shared_checkpoint(0, 1)
    try:
        r = utterance_cpu_baseline(path, args.ref_seconds, max_forwards=args.steps, warmup=1)
    finally:
        shutil.rmtree(tmpdir, ignore_errors=True)
    if "unavailable" in r:
        return {"impl": "reference", "unavailable": r["unavailable"]}
    return {
        "metric": METRIC,
        "value": r["value"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": r["forwards"],
        "warmup": 1,
        "ms_per_step": r["seconds"] * 1e3 / max(r["forwards"], 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8 (u8 x s8 VNNI per 32-k block, fp32 epilogue)",
        "data": "synthetic (seeded random-init int8 weights and embeddings, random text ids, "
                "masked target frames)",
        "config": config_utt(world, utterance_lengths()),
        "impl": "reference",
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "host")},
        "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# Rows of the largest batch one GPU runs at config 4 (bench.py
# --profile-forward prints it): the GEMM shapes the forward's launch list shows.
CONFIG4_BATCH_ROWS = 15408


def profile_gemm(name: str) -> None:
    """Three launches of one fp16 forward GEMM at the config-4 batch, as the LM
    calls it: q|k|v with the fused norm + RoPE, o and down accumulating into
    the residual stream, gate|up with the fused SiLU*up quantiser."""
    import torch

    import ovnative_b200 as ovb
    from ovnative_b200 import layer as LY
    dev = torch.device("cuda", 0)
    M = CONFIG4_BATCH_ROWS
    rng = np.random.default_rng(41)
    lw = LY.LayerWeights.from_host(LY.random_layer_host(rng), dev, f16=True)
    gen = torch.Generator(device=dev)
    gen.manual_seed(42)
    x = torch.randn((M, LY.HIDDEN), device=dev, generator=gen)
    qh = ovb.rmsnorm_quantize_f32(x, lw.input_ln, LY.RMS_EPS, f16=True)
    if name == "qkv":
        tab = ovb.rope_table(torch.arange(M, device=dev, dtype=torch.int64))
        nrm = torch.ones(128, device=dev)
        fn = lambda: ovb.linear_h_qk_rope(qh[0], lw.qkv, LY.QD // 128, LY.KVD // 128,  # noqa: E731
                                          nrm, nrm, LY.RMS_EPS, tab)
    elif name == "o":
        a = ovb.s8_nk_quantize(torch.randn((M, LY.QD), device=dev, generator=gen), f16=True)[0]
        fn = lambda: ovb.linear_h(a, lw.o, x, accumulate=True)  # noqa: E731
    elif name == "gate_up":
        fn = lambda: ovb.linear_h_silu(qh[0], lw.gate_up)  # noqa: E731
    else:
        qi = ovb.linear_h_silu(qh[0], lw.gate_up)
        fn = lambda: ovb.linear_h(qi[0], lw.down, x, accumulate=True)  # noqa: E731
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"gemm": name, "rows": M, "status": ovb.device_status()}), flush=True)
    lw.close()


def main():
    global MAX_ROWS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["utterances", "layer"], default="utterances",
                    help="utterances: BASELINE config 4 (the headline); layer: config 1's "
                         "layer step as the headline (profiling)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="skip the N=1 extra entries (layer step, sampler, attention, loader, "
                         "configs 2/3)")
    ap.add_argument("--no-roofline", action="store_true",
                    help="skip the per-kernel timings behind `roofline` (profiling runs)")
    ap.add_argument("--numerics", choices=["fp16", "exact"], default="fp16")
    ap.add_argument("--skip-other", action="store_true",
                    help="do not time the other numerics path of the layer step")
    ap.add_argument("--gemm-sweep", action="store_true",
                    help="only time the isolated GEMM M-sweep of config 4 (both mainloops)")
    ap.add_argument("--lm-only", action="store_true",
                    help="only time the 28-layer LM forward at configs 2 and 3")
    ap.add_argument("--load-only", action="store_true",
                    help="only time loading a synthetic OVW1 checkpoint's int8 weights")
    ap.add_argument("--attention-only", action="store_true",
                    help="only time the attention (one q/k/v set, 8 launches; for ncu)")
    ap.add_argument("--profile-forward", action="store_true",
                    help="build the 28-layer LM and the largest config-4 batch of one GPU and run "
                         "two eager forwards + samplers (for an ncu launch list)")
    ap.add_argument("--max-rows", type=int, default=MAX_ROWS,
                    help="rows per packed forward (at most 32 CFG pairs each)")
    ap.add_argument("--lanes", type=int, default=4,
                    help="LM instances per GPU whose batches' forwards run on their own streams")
    ap.add_argument("--profile-gemm", choices=["qkv", "o", "gate_up", "down"], default=None,
                    help="run one of the fp16 forward's GEMMs three times at the largest "
                         "config-4 batch of one GPU (15,408 rows; for ncu captures)")
    ap.add_argument("--profile-attention", action="store_true",
                    help="run the forward's attention three times over the largest config-4 "
                         "batch of one GPU (32 segments, 15,408 rows; for ncu captures)")
    ap.add_argument("--sampler-only", action="store_true",
                    help="only time the guided sampler (one plane set, 8 launches; for "
                         "profiling runs) and print its entry")
    args = ap.parse_args()
    MAX_ROWS = args.max_rows
    if args.profile_forward:
        import shutil

        import torch

        from ovnative_b200 import lm as LM
        from ovnative_b200 import shard
        from ovnative_b200 import tts_batch as TB
        dev = torch.device("cuda", 0)
        path, tmpdir = shared_checkpoint(0, 1)
        try:
            lengths = utterance_lengths()
            uids = shard.lpt_assign([lengths[i] for i in range(len(lengths))], 1)[0]
            m = LM.LM(path, f16=args.numerics == "fp16")
            st = torch.cuda.Stream(device=dev)
            sp = TB.Stepper(m, lengths, uids, dev, st, max_rows=MAX_ROWS)
            b = max(sp.batches, key=lambda x: x.rows)
            with torch.cuda.stream(st):
                for _ in range(2):
                    b.run()
            torch.cuda.synchronize()
            print(json.dumps({"rows": b.rows, "pairs": len(b.pairs), "segments": len(b.seg_rows)}),
                  flush=True)
            m.close()
        finally:
            shutil.rmtree(tmpdir, ignore_errors=True)
        return
    if args.profile_attention:
        profile_attention()
        return
    if args.profile_gemm:
        profile_gemm(args.profile_gemm)
        return
    if args.sampler_only:
        import torch
        dev = torch.device("cuda", 0)
        print(json.dumps(time_sampler(dev, torch.cuda.Stream(device=dev), launches=8, sets=1)),
              flush=True)
        return
    if args.gemm_sweep:
        import torch
        dev = torch.device("cuda", 0)
        st = torch.cuda.Stream(device=dev)
        res = {"gemm_sweep": {"fp16": time_gemm_sweep(dev, st, True),
                              "exact": time_gemm_sweep(dev, st, False)},
               "peaks": load_peaks(), "l2": "weights rotate over > 150 MB of copies",
               "cpu_baseline": sweep_cpu_baseline([(n, m) for n in SWEEP_SHAPES
                                                   for m in SWEEP_M])}
        print(json.dumps(res), flush=True)
        return
    if args.lm_only:
        import torch
        dev = torch.device("cuda", 0)
        print(json.dumps(time_lm_forward(dev, torch.cuda.Stream(device=dev),
                                         args.numerics == "fp16",
                                         cpu=not args.no_cpu_baseline)), flush=True)
        return
    if args.load_only:
        import torch
        print(json.dumps(time_weight_load(torch.device("cuda", 0))), flush=True)
        return
    if args.attention_only:
        import torch
        dev = torch.device("cuda", 0)
        print(json.dumps(time_attention(dev, torch.cuda.Stream(device=dev), launches=8, sets=1)),
              flush=True)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    else:
        out = run_ours(args, rank, world, local_rank)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark of the BF16X fused decode+GEMV hot path (the four-shape decode sweep).

One step = one pass of the fused decode+GEMV over the four benchmark weight
shapes ([out x in] = 4096x4096, 14336x4096, 4096x14336, 128256x4096) at the
chosen batch (default 1), weights resident in HBM in the kernel layout,
activations bf16 N(0,1).  ~950 MB of compressed weights per step, far larger
than the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Multi-GPU (launched by torchrun, one rank per GPU): weights are sharded by
output rows with no collective on the data path.  Default weak scaling: each
rank holds a [out x in] row shard of a [N*out x in] weight, so per-GPU work
is fixed; --scaling strong splits the [out x in] weights N ways instead.

Rank 0 prints one JSON line.  `value` is the whole-job compressed-byte
throughput (resident layout + patch table + activations + outputs, summed
over ranks, divided by the max-over-ranks device time of K steps).
`--impl reference` times the reference's CPU decode+matmul path (the C
oracle port, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode+GEMV GB/s (frac of 8 TB/s) & tok/s; decode+GEMM prefill TFLOPS"
SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong",
                    help="N>1: strong = the four weights row-sharded over the GPUs (tensor parallel, y "
                         "all-gathered); weak = every GPU an independent replica of the whole workload")
    ap.add_argument("--collective", choices=["peer", "nccl"], default="peer",
                    help="tensor parallel all-gather: inside the GEMV (peer stores over NVLink) or NCCL")
    ap.add_argument("--no-nccl-compare", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill and decode sub-records")
    ap.add_argument("--shapes", default="", help="e.g. 4096x4096,128256x4096 (default: all four)")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--mode", choices=["gemv", "gemm", "e2e", "kernels"], default="gemv",
                    help="gemv: decode+GEMV sweep (the headline); gemm: decode+GEMM prefill TFLOPS; "
                         "e2e: Llama-style decoder, ms per generated token against bf16 weights; "
                         "kernels: the stand-alone packer / repack / decode / GGUF kernels, GB/s each")
    ap.add_argument("--model", choices=["1b", "8b", "tiny"], default="1b", help="decoder for --mode e2e")
    ap.add_argument("--prompt", type=int, default=512, help="prompt tokens for --mode e2e")
    ap.add_argument("--new", type=int, default=128, help="generated tokens for --mode e2e")
    ap.add_argument("--seqs", type=int, default=1, help="sequences decoded together for --mode e2e (batch)")
    ap.add_argument("--tokens", type=int, default=2048, help="prefill tokens M for --mode gemm")
    ap.add_argument("--format", choices=["flat", "gguf", "gguf-lossless", "gguf-blocks", "gguf-blocks-lossless"],
                    default="flat",
                    help="weight source: the bf16x_quantize dict (flat), the 11.5-bpw GGUF blocks "
                         "(zero marker, lossy) or GGUF blocks + side table (exact), re-encoded into the "
                         "resident layout; gguf-blocks*: the GEMV reads the GGUF blocks in place")
    return ap.parse_args()


def gemm_kernel_name(rows, in_f, M, sms):
    """Which GEMM kernel ResidentWeight.gemm launches for (rows, in_f, M):
    the slab kernel when the shape takes a workspace, else the CTA-pair
    kernel for 256-token tiles that fill the GPU, else the single-CTA one."""
    from bfloat16x_b200 import _lib
    if _lib.lib().bf16x_gemm_workspace_bytes(rows, in_f, M) > 0:
        return "gemm_slab_kernel"
    bn = 64 if M <= 64 else 128 if M <= 128 else 256
    if bn == 256 and (rows + 127) // 128 * ((M + 255) // 256) < sms:
        bn = 128
    return "gemm2sm_kernel" if bn == 256 else f"gemm_kernel<{bn}>"


def make_resident(w, fmt, dev):
    """The fused kernels' resident weight built from `w` through the chosen format."""
    from bfloat16x_b200.opqk_linear import bf16x_quantize
    from bfloat16x_b200.resident import ResidentWeight
    if fmt == "flat":
        return ResidentWeight.from_packed(bf16x_quantize(w, device=dev), device=dev)
    from bfloat16x_b200.bf16x_gguf_block import GgufWeight
    if fmt.startswith("gguf-blocks"):
        # the GEMV reads the 46-byte blocks in place (prefill: resident layout)
        return GgufWeight.from_float(w, lossless=(fmt == "gguf-blocks-lossless"), native=True)
    return GgufWeight.from_float(w, lossless=(fmt == "gguf-lossless")).resident()


def shapes_of(args):
    if not args.shapes:
        return SHAPES
    return [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",")]


def workload_name(args, shapes):
    return ("configs[1] fused decode+GEMV sweep: " + ", ".join(f"{o}x{i}" for o, i in shapes) +
            f" at batch {args.batch}")


def peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_from_profile(kernel_key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get(kernel_key)
    except Exception:
        return None


# --------------------------------------------------------------------------- #
# CPU side (reference arm and cpu_baseline): the C oracle port                 #
# --------------------------------------------------------------------------- #
def cpu_sample(batch: int, seconds: float):
    """Time the CPU decode+matmul (oracle port of BF16XLinear.forward) on a
    4096x4096 sample; returns (bytes per pass, seconds per pass, cores, passes)."""
    import numpy as np
    import torch

    from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
    from oracle import oracle

    out_f, in_f = 4096, 4096
    w = synthetic_weight(out_f, in_f, seed=0)
    bits = w.view(torch.int16).numpy().view(np.uint16)
    p = oracle.quantize(bits, out_f, in_f)
    x = synthetic_activation(batch, in_f, seed=1).float().numpy()
    nbytes = workload_bytes(stored_weight_bytes(p, out_f, in_f), out_f, in_f, batch)
    oracle.linear(p, x)   # warm
    t0 = time.perf_counter()
    passes = 0
    while True:
        oracle.linear(p, x)
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return nbytes, el / passes, oracle.num_threads(), passes


def workload_bytes(weight_bytes, rows, in_f, batch, y_bytes=2):
    """Bytes one fused decode+GEMV launch must move: the stored weight
    (resident layout + patch records + record offsets, ResidentWeight.nbytes)
    + activations + outputs."""
    return weight_bytes + 2 * batch * in_f + y_bytes * batch * rows


def stored_weight_bytes(p, rows, in_f):
    """ResidentWeight.nbytes of a flat dict, computed on the host from its
    exact decode: 384 B per 256-column chunk of each row; one record per
    (16-row tile, chunk) of 32 emax words, 2 header words and one word per
    weight whose exponent is more than 15 below the largest of its row-local
    32-column group, padded to 4 words; tiles x chunks + 1 record offsets.
    Decoded 4096 rows at a time, so large weights stay within host memory."""
    import numpy as np
    from oracle import oracle
    nch = (in_f + 255) // 256
    n_tiles = (rows + 15) // 16
    rec_words = 0
    step = 4096
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        nt = (r1 - r0 + 15) // 16
        e = np.zeros((nt * 16, nch * 256), dtype=np.int16)
        e[:r1 - r0, :in_f] = ((oracle.decode(p, r0, r1).reshape(r1 - r0, in_f) >> 7) & 0xFF).astype(np.int16)
        valid = np.zeros_like(e, dtype=bool)
        valid[:r1 - r0, :in_f] = True
        g = e.reshape(nt * 16, nch * 8, 32)
        patch = ((g.max(axis=2, keepdims=True) - g) > 15) & valid.reshape(g.shape)
        counts = patch.reshape(nt, 16, nch, 256).sum(axis=(1, 3))
        rec_words += int(((34 + counts + 3) // 4 * 4).sum())
    return rows * nch * 384 + 4 * rec_words + 4 * (n_tiles * nch + 1)


def run_reference(args):
    """The reference's CPU decode+matmul path (BF16XLinear.forward,
    opqk_linear.py:390-404, restated in the C oracle: per-1024-row-tile decode
    with the overflow searchsorted, fp32 matmul) on this arm's workload: the
    same four weights (drawn with the same seeds, packed by the reference's
    quantize restated), the same activations, all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps, warmup = args.steps, args.warmup
    import numpy as np
    import torch

    from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
    from oracle import oracle

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    oracle.set_num_threads(cores)          # a launcher's OMP_NUM_THREADS=1 must not apply here
    world = int(os.environ.get("WORLD_SIZE", "1"))
    gen_dev = "cuda" if torch.cuda.is_available() else "cpu"
    shapes = shapes_of(args)
    B = args.batch
    layers = []
    nbytes = 0
    for si, (out_f, in_f) in enumerate(shapes):
        # the same inputs as the device arm at one GPU (seeds 1000*si and si+1)
        w = synthetic_weight(out_f, in_f, seed=1000 * si, device=gen_dev).cpu()
        bits = w.view(torch.int16).numpy().view(np.uint16)
        del w
        p = oracle.quantize(bits, out_f, in_f)
        nbytes += workload_bytes(stored_weight_bytes(p, out_f, in_f), out_f, in_f, B)
        del bits
        x = synthetic_activation(B, in_f, seed=si + 1, device=gen_dev).float().cpu().numpy()
        layers.append((p, x))

    def step():
        for p, x in layers:
            oracle.linear(p, x)
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    el = time.perf_counter() - t0
    v = nbytes * steps / el / 1e9
    sample = (f"the whole workload every step ({', '.join(f'{o}x{i}' for o, i in shapes)}, batch {B}): "
              f"CPU restatement of BF16XLinear.forward (opqk_linear.py:390-404) in C, OpenMP over {cores} "
              f"threads; GB/s counts the same bytes as the device arm (stored weight + x + y)")
    line = {
        "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": round(el / steps * 1e3, 3),
        "higher_is_better": True, "scaling": args.scaling if world > 1 else "strong", "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights with 0.5% x 2^U{4..8} outliers, bf16 N(0,1) activations)",
        "config": bench_config(args, shapes, world),
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- #
# GPU side                                                                     #
# --------------------------------------------------------------------------- #
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.strip().split(", ") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except Exception:
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _l2_flusher(dev):
    """A kernel that reads 256 MB (twice the 126 MB L2) on the current stream.
    Reading, not writing: a written flush buffer leaves L2 full of dirty lines
    whose write-back to HBM would then be charged to the kernel timed next."""
    import torch
    buf = torch.ones(64 << 20, dtype=torch.int32, device=dev)
    acc = torch.empty((), dtype=torch.int64, device=dev)

    def flush():
        torch.sum(buf, dim=0, dtype=torch.int64, out=acc)
    return flush


def prefill_record(layers, dev, steps, warmup, with_cublas):
    """Fused decode+GEMM over the same resident weights at M = 512 and 2048
    tokens: TFLOP/s per step, the dominant launch's fraction of the measured
    bf16 burst peak, cuBLAS bf16 on the uncompressed weights beside it."""
    import torch
    import torch.nn.functional as F

    from bfloat16x_b200.synthetic import synthetic_activation
    peak_tf, peak_kind = peak_tf_burst()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = {}
    for M in (512, 2048):
        xs = [synthetic_activation(M, L["in_f"], seed=31 + i, device=dev) for i, L in enumerate(layers)]
        ys = [torch.empty((M, L["rows"]), dtype=torch.bfloat16, device=dev) for L in layers]

        def step():
            for L, x, y in zip(layers, xs, ys):
                L["rw"].gemm(x, out=y)
        for _ in range(max(warmup, 3)):
            step()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in layers]
        per = [0.0] * len(layers)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            for i, (L, x, y) in enumerate(zip(layers, xs, ys)):
                ev[i][0].record()
                L["rw"].gemm(x, out=y)
                ev[i][1].record()
        b.record()
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b) / steps
        for i in range(len(layers)):
            per[i] = ev[i][0].elapsed_time(ev[i][1])
        flops = sum(2.0 * M * L["rows"] * L["in_f"] for L in layers)
        dom = max(range(len(layers)), key=lambda i: per[i])
        Ld = layers[dom]
        ach = 2.0 * M * Ld["rows"] * Ld["in_f"] / (per[dom] / 1e3) / 1e12
        rec = {"tokens": M, "TFLOPS": round(flops / (ms / 1e3) / 1e12, 1), "ms_per_step": round(ms, 4),
               "per_shape_ms": {f"{L['rows']}x{L['in_f']}": round(per[i], 4) for i, L in enumerate(layers)},
               "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak_tf, "unit": "TFLOP/s",
                            "frac": round(ach / peak_tf, 4), "peak_source": peak_kind + " (burst)",
                            "kernel": f"{gemm_kernel_name(Ld['rows'], Ld['in_f'], M, sms)} {Ld['rows']}x{Ld['in_f']}"}}
        if with_cublas:
            for L, x in zip(layers, xs):
                F.linear(x, L["w"])
            torch.cuda.synchronize(dev)
            a.record()
            for _ in range(steps):
                for L, x in zip(layers, xs):
                    F.linear(x, L["w"])
            b.record()
            torch.cuda.synchronize(dev)
            c_ms = a.elapsed_time(b) / steps
            rec["cublas_bf16"] = {"ms_per_step": round(c_ms, 4), "TFLOPS": round(flops / (c_ms / 1e3) / 1e12, 1),
                                  "ratio_vs_cublas": round(c_ms / ms, 3)}
        out[f"M{M}"] = rec
        del xs, ys
    return out


def gguf_record(layers, dev, steps, batch):
    """The same four weights quantized to the 11.5-bpw GGUF blocks (lossy:
    zero marker, no side table) and multiplied in place by bf16x_gguf_gemv:
    the step as one CUDA graph, each launch replayed back to back, the
    dominant launch's fraction of the measured HBM copy bandwidth
    (algorithmic bytes: 46 B per 32 weights + x + y)."""
    import torch

    from bfloat16x_b200.bf16x_gguf_block import GgufWeight
    if any(L.get("w") is None for L in layers) or any(L["in_f"] % 256 for L in layers):
        return None
    peak, kind = peak_hbm()
    gws = [GgufWeight.from_float(L["w"], lossless=False, native=True) for L in layers]
    ys = [torch.empty((batch, L["rows"]), dtype=torch.bfloat16, device=dev) for L in layers]

    def run(i):
        gws[i].gemv(layers[i]["x"], out=ys[i])

    def step():
        for i in range(len(layers)):
            run(i)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            step()                                  # scratch and counters exist before the capture
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
        gl = []
        for i in range(len(layers)):
            h = torch.cuda.CUDAGraph()
            with torch.cuda.graph(h, stream=s):
                run(i)
            gl.append(h)
    torch.cuda.synchronize(dev)
    for _ in range(3):
        g.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / steps
    per = []
    for h in gl:
        h.replay()
        a.record()
        for _ in range(steps):
            h.replay()
        b.record()
        torch.cuda.synchronize(dev)
        per.append(a.elapsed_time(b) / steps)
    nbytes = [gw.stream_bytes() + 2 * batch * (L["in_f"] + L["rows"]) for gw, L in zip(gws, layers)]
    dom = max(range(len(layers)), key=lambda i: per[i])
    ach = nbytes[dom] / (per[dom] / 1e3) / 1e9
    key = f"gemv_gguf-blocks_b{batch}_{layers[dom]['rows']}x{layers[dom]['in_f']}"
    out = {"format": "GGUF BF16X blocks, lossy (11.5 bits per weight), GEMV on the blocks in place",
           "ms_per_step": round(ms, 4), "GB/s": round(sum(nbytes) / (ms / 1e3) / 1e9, 1),
           "bits_per_weight": round(8 * sum(gw.stream_bytes() for gw in gws) /
                                    sum(L["rows"] * L["in_f"] for L in layers), 3),
           "per_shape_ms": {f"{L['rows']}x{L['in_f']}": round(per[i], 4) for i, L in enumerate(layers)},
           "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(ach / peak, 4), "peak_source": kind,
                        "kernel": f"gemv_kernel (GGUF blocks in place) {layers[dom]['rows']}x{layers[dom]['in_f']}",
                        "traffic": traffic_from_profile(key)},
           "gpu_launches": steps * len(layers)}
    _lib_check(dev)
    del g, gl, gws, ys
    return out


def _lib_check(dev):
    from bfloat16x_b200 import _lib
    _lib.check_device_status(dev.index)


def decode_record(dev, reps=20):
    """Stand-alone flat decode + overflow fix (bf16x_decode_triton) on 2048x1536
    and 4096x4096: bytes = 1.4375 B/weight of streams + 5 B per overflow entry
    in + 2 B/weight out, each launch timed alone after an L2 flush."""
    import torch

    from bfloat16x_b200.bf16x_decode import bf16x_decode_triton
    from bfloat16x_b200.opqk_linear import bf16x_quantize
    from bfloat16x_b200.synthetic import synthetic_weight
    peak, kind = peak_hbm()
    flush = _l2_flusher(dev)
    out = {}
    for (o, i) in ((2048, 1536), (4096, 4096)):
        w = synthetic_weight(o, i, seed=0, device=dev)
        p = bf16x_quantize(w, device=dev)
        args = (p["sign_packed"], p["mant_packed"], p["delta_packed"], p["emax"], o, i,
                p["delta_ovf_idx"], p["delta_ovf_val"])
        y = bf16x_decode_triton(*args)
        assert torch.equal(y.view(torch.int16), w.view(torch.int16)), "decode not bit-exact"
        nbytes = (4 * (p["sign_packed"].numel() + p["mant_packed"].numel() + p["delta_packed"].numel())
                  + p["emax"].numel() + 5 * p["delta_ovf_idx"].numel() + 2 * o * i)
        times = []
        for _ in range(reps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            bf16x_decode_triton(*args, out=y)
            b.record()
            torch.cuda.synchronize(dev)
            times.append(a.elapsed_time(b))
        t = statistics.median(times)
        out[f"{o}x{i}"] = {"us": round(t * 1e3, 2), "GB/s": round(nbytes / (t / 1e3) / 1e9, 1),
                           "frac": round(nbytes / (t / 1e3) / 1e9 / peak, 4), "bytes": int(nbytes),
                           "overflow_entries": int(p["delta_ovf_idx"].numel())}
    out["note"] = ("median of %d launches, each after reading a 256 MB buffer (L2 flushed, no dirty lines); "
                   "fraction of the %s HBM copy bandwidth (%.1f GB/s)" % (reps, kind, peak))
    return out


def peak_tf_burst():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    from bfloat16x_b200 import _lib
    from bfloat16x_b200.opqk_linear import bf16x_quantize
    from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight
    from bfloat16x_b200.tp import shard_bounds

    B = args.batch
    shapes = shapes_of(args)
    tp = world > 1 and args.scaling == "strong"
    peers = None
    collective_note = None
    if tp and args.collective == "peer":
        from bfloat16x_b200.peer import PeerGroup
        heap = sum(B * o * 8 + 256 for o, _ in shapes) + (1 << 20)
        try:
            peers = PeerGroup(None, dev, heap_bytes=heap)
        except _lib.Bf16xError as e:        # raised on every rank alike
            collective_note = f"NCCL all-gather: peer mapping unavailable ({e})"
    layers = []
    for si, (out_f, in_f) in enumerate(shapes):
        if args.scaling == "weak" or world == 1:
            r0, r1 = 0, out_f
            w = synthetic_weight(out_f, in_f, seed=1000 * si + rank, device=dev)
        else:
            # every rank draws the whole weight and packs its row shard, so the
            # N-GPU job computes exactly the 1-GPU job's outputs
            r0, r1 = shard_bounds(out_f, world, rank, 16)
            w = synthetic_weight(out_f, in_f, seed=1000 * si, device=dev)[r0:r1].contiguous()
        rows = r1 - r0
        rw = make_resident(w, args.format, dev)
        wb = None if args.no_cublas else w
        del w
        x = synthetic_activation(B, in_f, seed=si + 1, device=dev)
        L = dict(rw=rw, x=x, w=wb, rows=rows, r0=r0, out_f=out_f, in_f=in_f,
                 nbytes=workload_bytes(getattr(rw, "stream_bytes", rw.nbytes)(), rows, in_f, B))
        if peers is not None:
            L["lloff"] = peers.alloc(B * out_f * 8)          # exchange words of this layer
            L["y"] = torch.empty((B, out_f), dtype=torch.bfloat16, device=dev)
        elif tp:
            rmax = max(h - l for l, h in (shard_bounds(out_f, world, q, 16) for q in range(world)))
            L["y"] = torch.empty((B, rmax), dtype=torch.bfloat16, device=dev)
            L["yall"] = torch.empty((world * B, rmax), dtype=torch.bfloat16, device=dev)
        else:
            L["y"] = torch.empty((B, rows), dtype=torch.bfloat16, device=dev)
        layers.append(L)
    torch.cuda.synchronize()

    def run_layer(L, x=None):
        x = L["x"] if x is None else x
        if peers is not None:
            L["rw"].gemv_peers(x, peers, L["lloff"], L["out_f"], L["y"], mode=0, row0=L["r0"])
        elif tp:
            L["rw"].gemv(x, out=L["y"][:, :L["rows"]])
            dist.all_gather_into_tensor(L["yall"], L["y"])
        else:
            L["rw"].gemv(x, out=L["y"])

    def step():
        for L in layers:
            run_layer(L)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # ---------------- device-resident timing (value) --------------------------
    # One step (the four launches, with their all-gathers under tensor
    # parallelism) is captured once in a CUDA graph and replayed: what is
    # timed is device work, not Python launch overhead.
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    gstream = torch.cuda.Stream(device=dev)
    gstream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(gstream):
        step()                                   # per-stream scratch for the capture stream
        torch.cuda.synchronize(dev)
        barrier()
        g_step = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step, stream=gstream):
            step()
        g_layer = []
        for L in layers:
            gl = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gl, stream=gstream):
                run_layer(L)
            g_layer.append(gl)
    torch.cuda.synchronize(dev)
    for _ in range(max(args.warmup, 3)):
        g_step.replay()
    barrier()
    clock = ClockSampler(local)
    clock.start()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t_start.record()
    for _ in range(args.steps):
        g_step.replay()
    t_end.record()
    barrier()
    clocks = clock.stop()
    el_ms = t_start.elapsed_time(t_end)
    # per-launch device time of each layer (the same launch replayed back to back)
    per_layer_ms = []
    for gl in g_layer:
        gl.replay()
        barrier()
        a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_ev.record()
        for _ in range(args.steps):
            gl.replay()
        b_ev.record()
        torch.cuda.synchronize(dev)
        per_layer_ms.append(max_over_ranks(a_ev.elapsed_time(b_ev) / args.steps))
    el_max = max_over_ranks(el_ms)
    step_bytes = sum(L["nbytes"] for L in layers)
    total_bytes = sum_over_ranks(step_bytes * args.steps)
    value = total_bytes / (el_max / 1e3) / 1e9
    _lib.check_device_status(local)

    # the in-kernel all-gather against GEMV + NCCL all-gather on the same shards
    nccl_cmp = None
    if peers is not None and not args.no_nccl_compare:
        ys, yall = [], []
        for L in layers:
            rmax = max(h - l for l, h in (shard_bounds(L["out_f"], world, q, 16) for q in range(world)))
            ys.append(torch.empty((B, rmax), dtype=torch.bfloat16, device=dev))
            yall.append(torch.empty((world * B, rmax), dtype=torch.bfloat16, device=dev))

        def nccl_step():
            for L, y, ya in zip(layers, ys, yall):
                L["rw"].gemv(L["x"], out=y[:, :L["rows"]])
                dist.all_gather_into_tensor(ya, y)
        with torch.cuda.stream(gstream):
            nccl_step()
            torch.cuda.synchronize(dev)
            barrier()
            g_n = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_n, stream=gstream):
                nccl_step()
        for _ in range(3):
            g_n.replay()
        barrier()
        a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_ev.record()
        for _ in range(args.steps):
            g_n.replay()
        b_ev.record()
        barrier()
        n_ms = max_over_ranks(a_ev.elapsed_time(b_ev)) / args.steps
        nccl_cmp = {"ms_per_step": round(n_ms, 4), "GB/s": round(total_bytes / args.steps / (n_ms / 1e3) / 1e9, 1),
                    "speedup_of_fused": round(n_ms / (el_max / args.steps), 3),
                    "note": "the same row-shard GEMVs writing local rows, each followed by NCCL "
                            "all_gather_into_tensor, CUDA graph"}
        del g_n

    # dominant kernel: the launch with the largest share of device time
    dom = max(range(len(layers)), key=lambda i: per_layer_ms[i])
    Ld = layers[dom]
    achieved = Ld["nbytes"] / (per_layer_ms[dom] / 1e3) / 1e9
    peak, peak_kind = peak_hbm()
    kernel_key = (f"gemv_b{B}_{Ld['rows']}x{Ld['in_f']}" if args.format == "flat"
                  else f"gemv_{args.format}_b{B}_{Ld['rows']}x{Ld['in_f']}")

    # ---------------- end-to-end through the public API, host buffers ---------
    e2e = None
    if not args.no_e2e:
        hx = [L["x"].cpu().pin_memory() for L in layers]
        yout = [L["yall"] if "yall" in L else L["y"] for L in layers]     # the full y of each layer
        hy = [torch.empty(tuple(y.shape), dtype=torch.bfloat16).pin_memory() for y in yout]
        dx = [torch.empty_like(L["x"]) for L in layers]
        packed = world == 1
        if packed:
            # one staging buffer each way, as a serving loop keeps them: the
            # step's four inputs in one pinned host buffer copied in once,
            # the four outputs written into one device buffer read back once
            nx = [t.numel() for t in hx]
            ny = [y.numel() for y in yout]
            hx_all = torch.cat([t.reshape(-1) for t in hx]).pin_memory()
            dx_all = torch.empty_like(hx_all, device=dev)
            dy_all = torch.empty(sum(ny), dtype=torch.bfloat16, device=dev)
            hy_all = torch.empty(sum(ny), dtype=torch.bfloat16).pin_memory()
            ox = [sum(nx[:i]) for i in range(len(nx))]
            oy = [sum(ny[:i]) for i in range(len(ny))]
            dx = [dx_all[o:o + n].view(t.shape) for o, n, t in zip(ox, nx, hx)]
            saved_y = [L["y"] for L in layers]
            for L, o, n, y in zip(layers, oy, ny, yout):
                L["y"] = dy_all[o:o + n].view(y.shape)

        def e2e_step():
            if packed:
                dx_all.copy_(hx_all, non_blocking=True)
                for i, L in enumerate(layers):
                    run_layer(L, dx[i])
                hy_all.copy_(dy_all, non_blocking=True)
                return
            for i, L in enumerate(layers):
                dx[i].copy_(hx[i], non_blocking=True)
                run_layer(L, dx[i])
                hy[i].copy_(yout[i], non_blocking=True)

        for _ in range(max(args.warmup, 3)):
            e2e_step()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            e2e_step()
        b.record()
        barrier()
        e_max = max_over_ranks(a.elapsed_time(b))
        if packed:
            for i, L in enumerate(layers):
                assert torch.equal(hy_all[oy[i]:oy[i] + ny[i]].view(hy[i].shape), saved_y[i].cpu()), \
                    "packed end-to-end outputs differ from the device-timed step's"
                L["y"] = saved_y[i]
        e2e = {"value": round(total_bytes / (e_max / 1e3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": sum(t.numel() * 2 for t in hx) * world,
               "d2h_bytes_per_step": sum(t.numel() * 2 for t in hy) * world,
               "path": ("ResidentWeight.gemv_peers (row shards, all-gather inside the kernel)" if peers is not None else
                        "ResidentWeight.gemv (module forward path)") +
                       (": the step's inputs in one pinned buffer -> one H2D, the four fused GEMVs, one D2H of "
                        "their outputs" if packed else ": pinned x -> H2D, fused kernel, D2H y, every rank"),
               "ms_per_step": round(e_max / args.steps, 4)}

    # ---------------- cuBLAS bf16 GEMV on the same shapes ----------------------
    cublas = None
    if not args.no_cublas:
        import torch.nn.functional as F
        with torch.cuda.stream(gstream):
            for L in layers:
                F.linear(L["x"], L["w"])
            torch.cuda.synchronize(dev)
            gc = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gc, stream=gstream):
                for L in layers:
                    F.linear(L["x"], L["w"])
        for _ in range(3):
            gc.replay()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            gc.replay()
        b.record()
        barrier()
        c_ms = max_over_ranks(a.elapsed_time(b)) / args.steps
        cublas = {"ms_per_step": round(c_ms, 4), "speedup_vs_cublas_bf16": round(c_ms / (el_max / args.steps), 3),
                  "bf16_bytes_per_step": sum(L["rows"] * L["in_f"] * 2 for L in layers),
                  "note": "torch F.linear (cuBLAS) on the uncompressed bf16 weights (this rank's rows, no "
                          "all-gather), same shapes, CUDA graph"}

    prefill = decode = gguf = None
    if world == 1 and not args.no_prefill:
        prefill = prefill_record(layers, dev, min(args.steps, 10), args.warmup, not args.no_cublas)
        decode = decode_record(dev)
        if args.format == "flat":
            gguf = gguf_record(layers, dev, args.steps, B)

    # ---------------- CPU baseline (rank 0, N=1) ---------------------------------
    cpu = None
    if world == 1 and not args.no_cpu:
        nb, sec, cores, passes = cpu_sample(B, args.cpu_seconds)
        cpu = {"value": round(nb / sec / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"4096x4096 batch-{B} decode+matmul with the C oracle port of BF16XLinear.forward "
                         f"(OpenMP, {cores} threads), {passes} passes in {sec * passes:.1f} s"}

    if rank == 0:
        ms_step = el_max / args.steps
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": args.scaling if world > 1 else "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights with 0.5% x 2^U{4..8} outliers, bf16 N(0,1) activations)",
            "config": bench_config(args, shapes, world),
            "collective_note": collective_note,
            "resident_bpw": round(8 * sum(getattr(L['rw'], "stream_bytes", L['rw'].nbytes)() for L in layers) /
                                  sum(L['rows'] * L['in_f'] for L in layers), 3),
            "frac_of_8TBs": round(value / world / 8000.0, 4),
            "tok_s": round(B / (ms_step / 1e3), 1),
            "per_shape_ms": {f"{L['rows']}x{L['in_f']}": round(per_layer_ms[i], 4) for i, L in enumerate(layers)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "kernel": f"gemv_kernel{' (GGUF blocks in place)' if args.format.startswith('gguf-blocks') else ''} "
                                   f"(fused decode+GEMV) {Ld['rows']}x{Ld['in_f']} batch {B}",
                         "traffic": traffic_from_profile(kernel_key) if world == 1 else None},
            "gpu_launches": args.steps * len(layers),
            "timing": "CUDA-graph replay of the step; per_shape_ms from the same launch replayed back to back",
            "clocks": clocks,
            "e2e": e2e,
            "cublas_bf16": cublas,
            "allgather_nccl": nccl_cmp,
            "prefill": prefill,
            "decode": decode,
            "gguf": gguf,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        del g_step, g_layer
        barrier()
        if peers is not None:
            peers.close()
        dist.barrier()
        dist.destroy_process_group()


def bench_config(args, shapes, world):
    """The workload description, identical in both arms."""
    tp = world > 1 and args.scaling == "strong"
    par = (f"row-sharded tensor parallel x{world}, all-gather of y "
           + ("inside the GEMV kernel (epoch-tagged 64-bit stores to every GPU over NVLink)"
              if args.collective == "peer" else "by NCCL")
           if tp else f"row-shard x{world} (weak: independent replicas)" if world > 1 else "1 GPU")
    return {"workload": workload_name(args, shapes), "batch": args.batch, "format": args.format,
            "parallelism": par, "l2": "inputs larger than L2 (~1 GB of compressed weights per step)"}


def run_gemm(args):
    """Prefill: one step = the fused decode+GEMM over the four weight shapes at
    M tokens; value = TFLOPS (2*M*out*in per launch)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    from bfloat16x_b200 import _lib
    from bfloat16x_b200.opqk_linear import bf16x_quantize
    from bfloat16x_b200.resident import ResidentWeight
    from bfloat16x_b200.synthetic import synthetic_activation, synthetic_weight

    M = args.tokens
    shapes = shapes_of(args)
    layers = []
    for si, (out_f, in_f) in enumerate(shapes):
        rows = out_f if args.scaling == "weak" else out_f // world + (out_f % world if rank == world - 1 else 0)
        w = synthetic_weight(rows, in_f, seed=1000 * si + rank, device=dev)
        rw = make_resident(w, args.format, dev)
        x = synthetic_activation(M, in_f, seed=si + 1, device=dev)
        y = torch.empty((M, rows), dtype=torch.bfloat16, device=dev)
        layers.append(dict(rw=rw, x=x, y=y, w=None if args.no_cublas else w, rows=rows, in_f=in_f))
        del w

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def step():
        for L in layers:
            L["rw"].gemm(L["x"], out=L["y"])

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    clock = ClockSampler(local)
    clock.start()
    per_layer = [0.0] * len(layers)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in layers]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    a.record()
    for _ in range(args.steps):
        for i, L in enumerate(layers):
            ev[i][0].record()
            L["rw"].gemm(L["x"], out=L["y"])
            ev[i][1].record()
    b.record()
    barrier()
    clocks = clock.stop()
    el = a.elapsed_time(b)
    for i in range(len(layers)):
        per_layer[i] = ev[i][0].elapsed_time(ev[i][1])   # last step's launch
    if world > 1:
        t = torch.tensor([el], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        el = float(t.item())
    flops = sum(2.0 * M * L["rows"] * L["in_f"] for L in layers) * args.steps * world
    value = flops / (el / 1e3) / 1e12
    _lib.check_device_status(local)
    dom = max(range(len(layers)), key=lambda i: per_layer[i])
    Ld = layers[dom]
    ach = 2.0 * M * Ld["rows"] * Ld["in_f"] / (per_layer[dom] / 1e3) / 1e12
    peak_tf, peak_kind = 1688.4, "measured"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak_tf = float(json.load(f)["bf16_tflops"])
    except Exception:
        peak_tf, peak_kind = 1590.0, "fallback"
    cublas = None
    if not args.no_cublas:
        import torch.nn.functional as F
        for L in layers:
            F.linear(L["x"], L["w"])
        barrier()
        a.record()
        for _ in range(args.steps):
            for L in layers:
                F.linear(L["x"], L["w"])
        b.record()
        barrier()
        c_ms = a.elapsed_time(b) / args.steps
        cublas = {"ms_per_step": round(c_ms, 4), "TFLOPS": round(flops / args.steps / world / (c_ms / 1e3) / 1e12, 1),
                  "note": "torch F.linear (cuBLAS) on the uncompressed bf16 weights"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps, 4), "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "configs[2] fused decode+GEMM prefill: " + ", ".join(f"{o}x{i}" for o, i in shapes)
                                   + f" at M={M} tokens", "tokens": M, "format": args.format,
                       "l2": "inputs larger than L2"},
            "per_shape_ms": {f"{L['rows']}x{L['in_f']}": round(per_layer[i], 4) for i, L in enumerate(layers)},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": round(ach / peak_tf, 4), "peak_source": peak_kind,
                         "kernel": f"{gemm_kernel_name(Ld['rows'], Ld['in_f'], M, torch.cuda.get_device_properties(dev).multi_processor_count)} "
                                   f"{Ld['rows']}x{Ld['in_f']} M={M}", "traffic": None},
            "gpu_launches": args.steps * len(layers), "clocks": clocks, "cublas_bf16": cublas,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args):
    """Llama-style decoders (1B, 8B): greedy decode after a prompt prefill, ms per
    generated token with BF16X weights (every projection and lm_head through
    the fused kernels) and with the same weights in plain bf16.  Under
    torchrun the model is tensor-parallel over the ranks (one GPU each)."""
    import torch
    import torch.distributed as dist

    from bfloat16x_b200 import _lib
    from bfloat16x_b200.llama_e2e import (CONFIGS, LlamaModel, fp32_linears, generate, logits_rel_l2, pack_model,
                                          teacher_forced_logits)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = CONFIGS[args.model]
    max_seq = args.prompt + args.new + 8
    g = torch.Generator(device="cpu").manual_seed(7)
    prompt = torch.randint(0, cfg.vocab, (args.seqs, args.prompt), generator=g).to(dev)
    model = LlamaModel(cfg, max_seq, dev, seed=0, tp=world, batch=args.seqs)
    n_w = sum(m.weight.numel() for m in model.modules() if isinstance(m, torch.nn.Linear))
    generate(model, prompt, 4)                                   # warm-up
    ref_tok, ref_pre, ref_ms = generate(model, prompt, args.new)
    # logits of the bf16 weights on the prompt and on 16 teacher-forced steps
    n_tf = min(16, args.new)
    ref_logits = teacher_forced_logits(model, prompt, ref_tok[:n_tf])
    with fp32_linears(model):
        alt_logits = teacher_forced_logits(model, prompt, ref_tok[:n_tf])
    fl_max, fl_mean = logits_rel_l2(alt_logits, ref_logits)
    del alt_logits
    nbytes, _ = pack_model(model)
    got_logits = teacher_forced_logits(model, prompt, ref_tok[:n_tf])
    tf_max, tf_mean = logits_rel_l2(got_logits, ref_logits)
    del ref_logits, got_logits
    peers = None
    if world > 1 and args.collective == "peer":
        from bfloat16x_b200.llama_e2e import peer_heap_bytes, use_peer_collectives
        from bfloat16x_b200.peer import PeerGroup
        peers = PeerGroup(None, dev, heap_bytes=peer_heap_bytes(model))
        use_peer_collectives(model, peers)
    generate(model, prompt, 4)
    clock = ClockSampler(dev.index)
    clock.start()
    tok, pre, ms = generate(model, prompt, args.new)
    clocks = clock.stop()
    _lib.check_device_status(dev.index)
    t = torch.tensor([ms, ref_ms, pre, ref_pre, float(nbytes), float(n_w)], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t[:4].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t[4:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        t = torch.cat([mx, sm])
    ms, ref_ms, pre, ref_pre, nbytes, n_w = (float(v) for v in t.tolist())
    same = int((tok == ref_tok).all(dim=1).int().cumprod(0).sum().item())
    if rank == 0:
        line = {
            "metric": f"e2e greedy decode ms/token ({args.model} Llama-style, batch {args.seqs})", "value": round(ms, 4),
            "unit": "ms/token", "higher_is_better": False, "n_gpus": world, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) weights, random prompt ids)",
            "config": {"workload": f"configs[{3 if args.model == '1b' else 4}] {args.model}: prompt {args.prompt}, "
                                   f"{args.new} new tokens, batch {args.seqs}, every projection and lm_head "
                                   f"BF16X-packed" + (f", tensor-parallel over {world} GPUs" if world > 1 else ""),
                       "hidden": cfg.hidden, "layers": cfg.layers, "vocab": cfg.vocab, "tp": world,
                       "parallelism": f"tp{world}"},
            "bf16_ms_per_token": round(ref_ms, 4), "speedup_vs_bf16": round(ref_ms / ms, 3),
            "prefill_ms": round(pre, 3), "bf16_prefill_ms": round(ref_pre, 3),
            "linear_weight_bytes": {"bf16x_resident": int(nbytes), "bf16": int(2 * n_w)},
            "tokens_equal_to_bf16_run": same,
            "logits_rel_l2_vs_bf16": {"max": round(tf_max, 6), "mean": round(tf_mean, 6),
                                      "noise_floor_max": round(fl_max, 6), "noise_floor_mean": round(fl_mean, 6),
                                      "steps": 1 + n_tf, "how": "prompt's last position + teacher-forced decode "
                                                                "steps on the bf16 run's tokens; the floor is the "
                                                                "same bf16 weights with fp32-GEMM linears against "
                                                                "cuBLAS bf16"},
            "timing": "decode step as one CUDA graph replayed per token; max over ranks",
            "collectives": ("decode: o/down_proj partial sums and lm_head logits exchanged inside the fused GEMVs "
                            "(NVLink peer stores); prefill: NCCL") if peers is not None else "NCCL",
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if peers is not None:
            peers.close()
        dist.destroy_process_group()


def run_kernels(args):
    """The non-matmul kernels on one weight (default 8192x8192, 64 M weights,
    inputs and outputs larger than L2): the GPU packer (bf16x_quantize), the
    resident-layout repack, the flat decode + overflow fix, and the GGUF
    block quantize / dequantize / side-table count, pack and apply.  Each
    launch is timed alone after a 256 MB L2 flush (median of --steps); GB/s
    counts the bytes each kernel must read and write."""
    import torch

    from bfloat16x_b200 import _lib
    from bfloat16x_b200 import bf16x_gguf_block as gg
    from bfloat16x_b200._lib import BF16X_DTYPE_BF16, call, ptr
    from bfloat16x_b200.bf16x_decode import bf16x_decode_triton
    from bfloat16x_b200.opqk_linear import bf16x_quantize
    from bfloat16x_b200.resident import ResidentWeight, flat_args, flat_on_device
    from bfloat16x_b200.synthetic import synthetic_weight

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    out_f, in_f = shapes_of(args)[0] if args.shapes else (8192, 8192)
    n = out_f * in_f
    w = synthetic_weight(out_f, in_f, seed=0, device=dev)
    flush = _l2_flusher(dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    peak, kind = peak_hbm()

    def timed(fn):
        ts = []
        fn()
        for _ in range(max(args.steps, 3)):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    rec = {}

    def put(name, ms, nbytes, kernels):
        rec[name] = {"us": round(ms * 1e3, 2), "GB/s": round(nbytes / (ms / 1e3) / 1e9, 1),
                     "frac": round(nbytes / (ms / 1e3) / 1e9 / peak, 4), "bytes": int(nbytes), "kernels": kernels}

    # GPU packer: count pass + encode pass (bf16 in, streams + table out)
    p = bf16x_quantize(w, device=dev)
    n_ovf = p["delta_ovf_idx"].numel()
    stream_b = 4 * (p["sign_packed"].numel() + p["mant_packed"].numel() + p["delta_packed"].numel()) + p["emax"].numel()
    put("quantize", timed(lambda: bf16x_quantize(w, device=dev)), 2 * n + stream_b + 5 * n_ovf,
        "quantize count + encode (bf16x_quantize_count, bf16x_quantize)")
    # flat decode + overflow fix
    y = torch.empty((out_f, in_f), dtype=torch.bfloat16, device=dev)
    dargs = (p["sign_packed"], p["mant_packed"], p["delta_packed"], p["emax"], out_f, in_f,
             p["delta_ovf_idx"], p["delta_ovf_val"])
    bf16x_decode_triton(*dargs, out=y)
    assert torch.equal(y.view(torch.int16), w.view(torch.int16)), "decode not bit-exact"
    put("decode", timed(lambda: bf16x_decode_triton(*dargs, out=y)), stream_b + 5 * n_ovf + 2 * n,
        "flat_decode_kernel (bf16x_decode)")
    # repack: flat dict -> resident layout (count + scan + write)
    rw = ResidentWeight.from_packed(p, device=dev)
    f = flat_on_device(p, dev)
    ptile = torch.empty_like(rw.ptile_off)

    def repack():
        call("bf16x_repack_count", *flat_args(f), out_f, in_f, 0, out_f, ptr(ptile), st)
        call("bf16x_repack", *flat_args(f), out_f, in_f, 0, out_f, ptr(rw.ptile_off), ptr(rw.layout),
             ptr(rw.precs), st)
    put("repack", timed(repack), 2 * (stream_b + 5 * n_ovf) + rw.nbytes(),
        "repack count + write (streams read twice, resident layout + records written)")
    # resident decode: layout -> bf16
    put("resident_decode", timed(lambda: rw.decode(out=y)), rw.nbytes() + 2 * n, "resident_decode_kernel")
    # GGUF blocks
    blocks = torch.empty(n // 32 * 46, dtype=torch.uint8, device=dev)
    put("gguf_quantize", timed(lambda: call("bf16x_gguf_quantize", ptr(w), BF16X_DTYPE_BF16, n, ptr(blocks), st)),
        2 * n + n // 32 * 46, "bf16x_gguf_quantize (bf16 in)")
    put("gguf_dequantize", timed(lambda: call("bf16x_gguf_dequantize", ptr(blocks), n // 32, ptr(y),
                                              BF16X_DTYPE_BF16, st)),
        n // 32 * 46 + 2 * n, "bf16x_gguf_dequantize (bf16 out)")
    row_off = torch.empty(out_f + 1, dtype=torch.int32, device=dev)
    put("gguf_ovf_count", timed(lambda: call("bf16x_gguf_ovf_count", ptr(w), BF16X_DTYPE_BF16, out_f, in_f,
                                             ptr(row_off), st)), 2 * n + 4 * (out_f + 1), "bf16x_gguf_ovf_count")
    ro, ec, eb = gg._pack_ovf_dev(w, BF16X_DTYPE_BF16, out_f, in_f)
    ne = ec.numel()
    put("gguf_ovf_pack", timed(lambda: call("bf16x_gguf_ovf_pack", ptr(w), BF16X_DTYPE_BF16, out_f, in_f, ptr(ro),
                                            ptr(ec), ptr(eb), st)), 2 * n + 4 * (out_f + 1) + 4 * ne,
        "bf16x_gguf_ovf_pack")
    put("gguf_apply_ovf", timed(lambda: call("bf16x_gguf_apply_ovf", ptr(y), BF16X_DTYPE_BF16, out_f, in_f, ptr(ro),
                                             ptr(ec), ptr(eb), ne, st)), 4 * (out_f + 1) + 4 * ne + 4 * ne,
        "bf16x_gguf_apply_ovf (scattered 2-byte writes)")
    _lib.check_device_status(0)
    line = {"metric": "stand-alone BF16X kernels, GB/s of the bytes each must move", "unit": "GB/s",
            "config": {"workload": f"one {out_f}x{in_f} weight (synthetic, {n_ovf} overflow entries, "
                                   f"{ne} GGUF side-table entries)", "l2": "256 MB read before every launch (L2 flushed, no dirty lines)"},
            "peak": {"hbm_gbs": peak, "source": kind}, "kernels": rec}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "e2e":
        run_e2e(args)
    elif args.mode == "gemm":
        run_gemm(args)
    elif args.mode == "kernels":
        run_kernels(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

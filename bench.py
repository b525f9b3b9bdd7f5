#!/usr/bin/env python
"""Benchmark of the B200 attention backend (one JSON line on rank 0).

Headline workload (the one quoted at 1/2/4/8 GPUs):
batched GQA decode sweep, 64 independent sequences per GPU, Q16/KV2/D128,
18 layers of fp16 KV cache, context lengths U[512, 8192] (seeded), each step
appends one token to every sequence of every layer.  A bench "step" is one
decode step: 18 launches of the decode kernel (one per layer), each over the
64 sequences.  Metric: decode-attention HBM GB/s (algorithmic bytes: K/V rows
read + q/out + appended row, per launch) and tokens/s/GPU.  The KV caches
(~10 GB per GPU) are far larger than the 126 MB L2, so no flush is needed.

Components (rank 0): vision varlen prefill (configs[1], TFLOP/s) and decoder
causal prefill (configs[2], TFLOP/s), each timed with CUDA events; and on every
rank, end-to-end greedy OCR (configs[4]: random-init fp16 PaddleOCR-VL, 256
noise pages of 1024x1024 sharded by request, 512 tokens each) through the
engine's public API, tokens/s and requests/s (max time over ranks).

--impl reference times the reference's algorithm on the host cores (the C++
restatement of pvlc-cpu-ref in oracle/, because the Rust reference cannot be
built here) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import struct
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "paddleocr-vl-webgpu_b200"))

QH, KVH, HD = 16, 2, 128
LAYERS = 18
SEQS_PER_GPU = 64
L_MIN, L_MAX = 512, 8192
METRIC = "decode-attn HBM GB/s (64 seqs x 18 layers, L~U[512,8192])"
UNIT = "GB/s"

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of single launches
# captured with ncu on this workload's shapes (profiles/decode_kernel_64seq.txt,
# profiles/vision_tc_kernel_config1.txt, profiles/prefill_attn_kernel_config2.txt).
# The decode capture is one 64-sequence launch: its traffic / algorithmic-bytes
# ratio scales the figure to the bench's average launch.
DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE = 283.20e6 / 278.20e6
VISION_TC_TRAFFIC_BYTES = 61.00e6
PREFILL_ATTN_TRAFFIC_BYTES = 11.37e6
# checkpoint conversion, one launch over the whole payload
# (profiles/bf16_to_f16_kernel_checkpoint.txt: 5.820 TB/s x 651.3 us)
CONVERT_TRAFFIC_BYTES = 3.7907e9


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed region.

    Reads NVML (the library behind nvidia-smi) from a thread every 2 ms, so
    that a timed region of a few tens of milliseconds still gets samples;
    read-only queries, no setting of the GPU is touched.  The NVML device is
    found by the UUID of the CUDA device."""

    # NVML clock-event reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, cuda_index: int, period_s: float = 0.002):
        self.cuda_index = cuda_index
        self.period = period_s
        self.sm, self.bits = [], 0
        self.max_mhz = None
        self.error = None
        self.thread = None
        self.stop_flag = threading.Event()
        self.nvml = None
        self.handle = None

    def start(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = str(torch.cuda.get_device_properties(self.cuda_index).uuid)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                    uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle,
                                                                  pynvml.NVML_CLOCK_SM))
        except Exception as e:   # noqa: BLE001 - reported in the JSON line
            self.error = f"nvml unavailable: {type(e).__name__}"
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)))
                self.bits |= int(get_reasons(self.handle))
            except Exception as e:   # noqa: BLE001
                self.error = f"nvml query failed: {type(e).__name__}"
                return
            time.sleep(self.period)

    def stop(self):
        self.stop_flag.set()
        if self.thread:
            self.thread.join(timeout=2)
        reasons = sorted(n for b, n in self.REASONS.items() if self.bits & b)
        res = {"sm_mhz": statistics.median(self.sm) if self.sm else None,
               "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.sm),
               "source": "nvml"}
        if self.error:
            res["error"] = self.error
        return res


def algorithmic_decode_bytes(lengths_after_append):
    # K and V rows (2 heads x 128 fp16 each) + q + out (16 x 128 fp16) + appended K/V row
    return sum(1024 * n + 8192 + 1024 for n in lengths_after_append)


# --------------------------------------------------------------------- GPU arm
def run_gpu(args, rank, world, local_rank, dist):
    import numpy as np
    import torch

    from pvlc_b200 import abi, ops, positions

    abi.check(abi.lib().pvlc_attn_device_check(), "device check")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    hbm_peak, tf_peak, peak_src = peaks()

    # ---- synthetic workload (seeded per rank: this rank's request shard)
    rng = np.random.default_rng(1 + rank)
    L0 = rng.integers(L_MIN, L_MAX + 1, size=SEQS_PER_GPU).astype(np.int64)
    steps, warm = args.steps, args.warmup
    kernel_steps = 4                             # isolated per-launch kernel timing
    cap = int(L0.max()) + warm + 2 * steps + kernel_steps + 8   # timed + e2e + kernel steps
    B = SEQS_PER_GPU
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    kc = torch.empty((LAYERS, B, cap, KVH, HD), dtype=torch.float16, device=dev)
    vc = torch.empty_like(kc)
    kc.normal_(generator=g)
    vc.normal_(generator=g)
    kp = [torch.tensor([kc[l, b].data_ptr() for b in range(B)], dtype=torch.int64, device=dev)
          for l in range(LAYERS)]
    vp = [torch.tensor([vc[l, b].data_ptr() for b in range(B)], dtype=torch.int64, device=dev)
          for l in range(LAYERS)]
    q = torch.randn((LAYERS, B, QH, HD), generator=g, device=dev).half()
    kn = torch.randn((LAYERS, B, KVH, HD), generator=g, device=dev).half()
    vn = torch.randn((LAYERS, B, KVH, HD), generator=g, device=dev).half()
    out = torch.empty((LAYERS, B, QH, HD), dtype=torch.float16, device=dev)
    cos_np, sin_np = positions.linear_rope_tables(cap)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    ct0 = torch.tensor(L0, dtype=torch.int32, device=dev)
    ws = [ops.DecodeWorkspace(B, dev) for _ in range(LAYERS)]

    def step(ct, max_ct, ev=None, bufs=None):
        qq, kk, vv, oo = bufs if bufs is not None else (q, kn, vn, out)
        for l in range(LAYERS):
            if ev is not None:
                ev[l][0].record(stream)
            ops.decode(qq[l], kk[l], vv[l], cos, sin, kp[l], vp[l], ct, cap, max_ct, ws[l],
                       out=oo[l])
            if ev is not None:
                ev[l][1].record(stream)
        ct += 1

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    ct = ct0.clone()
    max_ct = int(L0.max())
    for i in range(warm):
        step(ct, max_ct + i)
    barrier()
    # ---- timed region: device-only (inputs resident in HBM)
    lengths = []
    sampler = ClockSampler(local_rank)
    sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    # launches back to back: an event recorded between two launches would
    # stop the next launch from being scheduled before the previous one ends
    barrier()
    t_start.record(stream)
    for s in range(steps):
        step(ct, max_ct + warm + s)
        lengths.extend([int(x) + warm + s + 1 for x in L0] * LAYERS)
    t_end.record(stream)
    barrier()
    clocks = sampler.stop()
    dev_ms = t_start.elapsed_time(t_end)
    # isolated kernel time: events around every launch of a few more steps
    kevs = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
             for _ in range(LAYERS)] for _ in range(kernel_steps)]
    k_lengths = []
    for s in range(kernel_steps):
        step(ct, max_ct + warm + steps + s, kevs[s])
        k_lengths.extend([int(x) + warm + steps + s + 1 for x in L0] * LAYERS)
    barrier()
    kernel_ms = [a.elapsed_time(b) for st in kevs for a, b in st]
    flags = sum(w.errors() for w in ws)
    if flags:
        raise RuntimeError(f"decode kernels raised fault flags {flags:#x}")
    bytes_rank = algorithmic_decode_bytes(lengths)
    launches = steps * LAYERS

    # ---- e2e: same steps through the public API with host buffers.  Every step
    # uploads its q / k_new / v_new from pinned host memory and reads its outputs
    # back; the copies run on their own streams into double-buffered device sets, so
    # step s + 1's upload and step s - 1's readback overlap step s's kernels.  The
    # timed region ends after the last readback.
    qh = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    knh = torch.empty(kn.shape, dtype=kn.dtype, pin_memory=True)
    vnh = torch.empty(vn.shape, dtype=vn.dtype, pin_memory=True)
    qh.copy_(q)
    knh.copy_(kn)
    vnh.copy_(vn)
    outh = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    sets = [(q, kn, vn, out), (torch.empty_like(q), torch.empty_like(kn), torch.empty_like(vn),
                               torch.empty_like(out))]
    h2d_stream, d2h_stream = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    read_back = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        with torch.cuda.stream(h2d_stream):
            for dst, src in zip(sets[i][:3], (qh, knh, vnh)):
                dst.copy_(src, non_blocking=True)
            uploaded[i].record(h2d_stream)

    e2e_steps = steps
    e_lengths = []
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    base = warm + steps + kernel_steps
    e0.record(stream)
    h2d_stream.wait_event(e0)
    d2h_stream.wait_event(e0)
    upload(0)
    for s in range(e2e_steps):
        i = s % 2
        if s + 1 < e2e_steps:
            if s >= 1:   # set 1 - i: step s - 1's kernels are done with its inputs
                h2d_stream.wait_event(computed[1 - i])
            upload(1 - i)
        stream.wait_event(uploaded[i])
        if s >= 2:       # set i's outputs of step s - 2 have been read back
            stream.wait_event(read_back[i])
        step(ct, max_ct + base + s, bufs=sets[i])
        computed[i].record(stream)
        d2h_stream.wait_event(computed[i])
        with torch.cuda.stream(d2h_stream):
            outh[i].copy_(sets[i][3], non_blocking=True)
            read_back[i].record(d2h_stream)
        e_lengths.extend([int(x) + base + s + 1 for x in L0] * LAYERS)
    stream.wait_stream(d2h_stream)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    e_bytes_rank = algorithmic_decode_bytes(e_lengths)
    h2d = (q.numel() + kn.numel() + vn.numel()) * 2
    d2h = out.numel() * 2

    # ---- aggregate over ranks: max time, summed bytes
    t = torch.tensor([dev_ms, e2e_ms, bytes_rank, e_bytes_rank], dtype=torch.float64, device=dev)
    if dist is not None:
        tmax = t[:2].clone()
        tsum = t[2:].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        dev_ms, e2e_ms = tmax.tolist()
        bytes_all, e_bytes_all = tsum.tolist()
    else:
        bytes_all, e_bytes_all = bytes_rank, e_bytes_rank
    value = bytes_all / (dev_ms * 1e-3) / 1e9
    e2e_value = e_bytes_all / (e2e_ms * 1e-3) / 1e9
    tok_per_s_per_gpu = B * steps / (dev_ms * 1e-3)
    # roofline: algorithmic bytes per launch over the timed region's time per
    # launch (any gap between launches counts against the kernel)
    launch_ms = dev_ms / launches
    achieved = (bytes_rank / launches) / (launch_ms * 1e-3) / 1e9
    avg_kernel_ms = statistics.mean(kernel_ms)
    kernel_achieved = (algorithmic_decode_bytes(k_lengths) / len(kernel_ms)) / (avg_kernel_ms * 1e-3) / 1e9

    components = {}
    del kc, vc, kp, vp, q, kn, vn, out, ws, qh, knh, vnh, outh, sets
    torch.cuda.empty_cache()
    if not args.skip_e2e:
        # every rank runs its request shard (the collectives inside are taken by all)
        e2e_res = run_e2e(args, dev, rank, world, dist)
        if rank == 0:
            components["e2e_greedy"] = e2e_res
    if rank != 0:
        return None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(dev_ms / steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) fp16 caches/q/k/v; per-rank request shard)",
        "config": {"workload": "configs[3] batched GQA decode sweep",
                   "seqs_per_gpu": B, "layers": LAYERS, "heads": "Q16/KV2/D128",
                   "context": f"U[{L_MIN},{L_MAX}] seed 1+rank, +1 row per step",
                   "parallelism": f"dp{world} (requests sharded, no hot-path collective)",
                   "l2": "inputs larger than L2 (~10 GB KV per GPU)"},
        "tokens_per_s_per_gpu": round(tok_per_s_per_gpu, 1),
        "gpu_launches": launches,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": "pvlc_b200.ops.decode -> C ABI pvlc_attn_decode, pinned host q/k/v in, out "
                        "back; copies on their own streams, double-buffered, overlapping the "
                        "neighbouring steps' kernels"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "peak_source": peak_src, "kernel": "pvlc::decode::decode_kernel",
                     "avg_launch_ms": round(launch_ms, 5),
                     "isolated_kernel": {"avg_ms": round(avg_kernel_ms, 5),
                                         "achieved": round(kernel_achieved, 1),
                                         "note": "events around each launch, separate steps"},
                     "traffic": round(args.traffic_bytes if args.traffic_bytes is not None else
                                      DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE * bytes_rank / launches),
                     "traffic_source": "--traffic-bytes" if args.traffic_bytes is not None else
                                       "ncu capture of one 64-sequence launch, scaled by algorithmic bytes"},
        "clocks": clocks,
        "components": components,
    }
    if not args.skip_cpu:
        line["cpu_baseline"] = cpu_decode_baseline(args.cpu_seconds)
    return line


def run_components(args, dev, tf_peak, peak_src,
                   which=("decode_b1", "vision", "prefill", "prefill_batch", "checkpoint",
                          "pack_blake3", "decode_linear"),
                   iters=20, warm=3):
    import torch
    cpu = not args.skip_cpu

    res = {}
    stream = torch.cuda.current_stream()

    def timeit(fn):
        # launches queued back to back: the device time per call, without the
        # host's per-call launch preparation showing up as device idle time
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(iters):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters

    if "decode_b1" in which:
        res["decode_b1"] = bench_decode_b1(dev, timeit)
        if cpu:
            res["decode_b1"]["cpu_baseline"] = cpu_decode_b1_baseline()
    if "vision" in which:
        res["vision_prefill"] = bench_vision(dev, timeit, tf_peak, peak_src, cpu)
    if "prefill" in which:
        res["decoder_prefill"] = bench_prefill(dev, timeit, tf_peak, peak_src, cpu)
    if "prefill_batch" in which:
        res["decoder_prefill_batch"] = bench_prefill_batch(dev, timeit, tf_peak, peak_src)
    if "checkpoint" in which:
        res["checkpoint_import"] = bench_checkpoint(dev, timeit)
    if "pack_blake3" in which:
        res["pack_blake3"] = bench_pack_blake3(dev, timeit, cpu)
    if "decode_linear" in which:
        res["decode_linear"] = bench_decode_linear(dev)
        if cpu:
            res["decode_linear"]["cpu_baseline"] = cpu_linear_baseline()
    return res


def bench_decode_linear(dev, rows=32, sets=16, reps=48):
    """The decode step's four projections of one decoder layer at the per-GPU decode batch
    of an 8-GPU configs[4] run (32 rows), through pvlc_linear (the gate-up with its fused
    SiLU gate) and through cuBLAS (+ the SiLU-gate pass), each timed as a CUDA graph of
    `reps` launches over `sets` weight sets (450 MB, larger than L2), device time with
    CUDA events.  value: the layer's weight bytes / our per-layer time."""
    import torch

    from pvlc_b200 import ops
    hbm_peak, _, peak_src = peaks()
    shapes = {"qkv": (1024, 2560, False), "o": (2048, 1024, False),
              "gate_up": (1024, 6144, True), "down": (3072, 1024, False)}

    def graph_ms(fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for i in range(3):
                fn(i)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(reps):
                fn(i)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(3):
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b) / reps)
        del g
        return best

    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    per, ours_ms, lib_ms, wbytes, checked = {}, 0.0, 0.0, 0, True
    for name, (K, N, gate) in shapes.items():
        x = torch.randn(rows, K, device=dev, generator=gen).half()
        ws = [(torch.randn(N, K, device=dev, generator=gen) * K ** -0.5).half()
              for _ in range(sets)]
        width = N // 2 if gate else N
        oo = [torch.empty(rows, width, device=dev, dtype=torch.float16) for _ in range(sets)]
        oc = [torch.empty(rows, N, device=dev, dtype=torch.float16) for _ in range(sets)]

        def ours(i):
            ops.linear(x, ws[i % sets], out=oo[i % sets], gate=gate)

        def lib(i):
            torch.mm(x, ws[i % sets].t(), out=oc[i % sets])
            if gate:
                ops.silu_mul(oc[i % sets], out=oo[i % sets])
        t_ours, t_lib = graph_ms(ours), graph_ms(lib)
        ref = x.float() @ ws[0].float().t()
        got = ops.linear(x, ws[0], gate=gate).float()
        if gate:
            r16 = ref.half().float().view(rows, N // 128, 2, 64)
            g16, u16 = r16[:, :, 0].reshape(rows, -1), r16[:, :, 1].reshape(rows, -1)
            want = g16 / (1 + torch.exp(-g16)) * u16
            ok = bool(((got - want).abs() <= want.abs() * 3e-3 + 2e-4).all())
        else:
            ok = bool(((got - ref).abs() <= ref.abs() * 2 ** -10 + 1e-4).all())
        checked = checked and ok
        per[name] = {"pvlc_linear_us": round(t_ours * 1e3, 2),
                     "cublas_us": round(t_lib * 1e3, 2),
                     "weights_mb": round(N * K * 2 / 1e6, 2)}
        ours_ms += t_ours
        lib_ms += t_lib
        wbytes += N * K * 2
        del ws, oo, oc
    gbs = wbytes / (ours_ms * 1e-3) / 1e9
    return {"workload": f"one decoder layer's QKV, O, gate-up (+SiLU gate), down projections "
                        f"at {rows} rows, fp16 weights in HBM",
            "value": round(gbs, 1), "unit": "GB/s", "layer_us": round(ours_ms * 1e3, 2),
            "cublas_layer_us": round(lib_ms * 1e3, 2), "per_projection": per,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(gbs / hbm_peak, 3),
                         "peak_source": peak_src},
            "kernel": "pvlc::lin::linear_kernel", "checked": checked,
            "note": "each launch is latency-bound (~2.5 us after the kernel ahead ends); "
                    "the engine keeps cuBLAS for these projections"}


def bench_pack_blake3(dev, timeit, cpu):
    """Model-pack verification: BLAKE3 of a 1 GiB section resident in HBM by pvlc_blake3
    (the digest PackReader.open checks), timed on the device; checked against the
    `blake3` package.  CPU baseline: the same package (the reference implementation's
    SIMD code) on host threads over a 256 MiB sample."""
    import torch

    from pvlc_b200 import ops
    n = 1 << 30
    g = torch.Generator(device=dev)
    g.manual_seed(6)
    data = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g)
    ws = torch.empty(int(ops.abi.lib().pvlc_blake3_workspace_bytes(n)), dtype=torch.uint8,
                     device=dev)
    dig = torch.empty(32, dtype=torch.uint8, device=dev)
    ms = timeit(lambda: ops.blake3(data, digest=dig, workspace=ws))
    res = {"workload": "BLAKE3 of one 1 GiB pack section in HBM (uniform random bytes)",
           "ms": round(ms, 4), "value": round(n / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
           "kernel": "pvlc::b3::chunk_kernel + parent_kernel",
           "bound": "integer ALU pipe (the XORs and rotates of the G function; the "
                    "additions issue to the FMA pipe); HBM traffic is 1 byte per byte"}
    try:
        import blake3
        host = data.cpu().numpy().tobytes()
        res["checked"] = bytes(dig.cpu().numpy()) == blake3.blake3(
            host, max_threads=blake3.blake3.AUTO).digest()
        if cpu:
            sample = host[:1 << 28]
            cores = os.cpu_count() or 1
            t0 = time.perf_counter()
            reps = 0
            while time.perf_counter() - t0 < 3.0:
                blake3.blake3(sample, max_threads=blake3.blake3.AUTO).digest()
                reps += 1
            dt = (time.perf_counter() - t0) / reps
            res["cpu_baseline"] = {"value": round(len(sample) / dt / 1e9, 2), "unit": "GB/s",
                                   "cores": cores, "kind": "reference",
                                   "sample": "256 MiB of the same section, the blake3 "
                                             f"package with all {cores} host threads, "
                                             f"{reps} passes"}
    except ImportError as e:
        res["checked"] = f"not checked: {e}"
    del data
    return res


def bench_checkpoint(dev, timeit):
    """Checkpoint import: the BF16 -> F16 conversion kernel over the whole
    PaddleOCR-VL-1.6 payload (958,588,736 elements, 1.92 GB; 4 bytes of HBM traffic per
    element), and the same payload from a file into HBM through load_payload_f16
    (page-cache read into pinned chunks, copy, in-place conversion)."""
    import tempfile

    import torch

    from pvlc_b200 import abi, checkpoint as C
    hbm_peak, _, peak_src = peaks()
    entries = C.name_sorted_layout(C.schema_specs())
    body = entries[-1][3][1]
    n = body // 2
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    src = torch.empty(n, dtype=torch.int16, device=dev)
    step = 1 << 27
    for i in range(0, n, step):
        m = min(step, n - i)
        src[i:i + m] = (torch.randn(m, generator=g, device=dev) * 0.02).to(
            torch.bfloat16).view(torch.int16)
    dst = torch.empty_like(src)
    word = torch.full((1,), -1, dtype=torch.int64, device=dev)
    lib, stream = abi.lib(), torch.cuda.current_stream(dev).cuda_stream

    def conv():
        abi.check(lib.pvlc_bf16_to_f16(src.data_ptr(), dst.data_ptr(), n, 0, word.data_ptr(),
                                       stream), "pvlc_bf16_to_f16")

    ms = timeit(conv)
    # the whole converted payload against torch's BF16 -> F16 rounding, in slices
    ok = int(word.item()) == -1
    for i in range(0, n, step):
        m = min(step, n - i)
        ok = ok and torch.equal(
            dst[i:i + m], src[i:i + m].view(torch.bfloat16).to(torch.float16).view(torch.int16))
    gbs = 4.0 * n / (ms * 1e-3) / 1e9
    res = {"workload": "PaddleOCR-VL-1.6 checkpoint payload, 958,588,736 BF16 elements "
                       "(1.92 GB) -> F16, N(0, 0.02^2) values",
           "ms": round(ms, 4), "value": round(gbs, 1), "unit": "GB/s", "checked": ok,
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                        "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                        "peak_source": peak_src, "traffic": CONVERT_TRAFFIC_BYTES,
                        "traffic_source": "ncu capture of one launch of this workload "
                                          "(DRAM bytes per second x duration)"},
           "kernel": "pvlc::convert::bf16_to_f16_kernel"}
    res["cpu_baseline"] = cpu_convert_baseline(src[:1 << 26].cpu().numpy())
    del dst
    path = None
    try:
        header = C.safetensors_header(entries, {"format": "pt"})
        fd, path = tempfile.mkstemp(suffix=".safetensors")
        with os.fdopen(fd, "wb") as f:
            f.write(struct.pack("<Q", len(header)) + header)
            host = src.cpu().numpy()
            f.write(memoryview(host))
        del host
        cat = C.SafetensorsCatalog.open(path)
        cat.validate_paddleocr_vl_16()
        C.load_payload_f16(cat, dev)       # warm: pinned buffers, page cache
        torch.cuda.synchronize()
        times = []
        for _ in range(2):
            t0 = time.perf_counter()
            blob = C.load_payload_f16(cat, dev)
            times.append(time.perf_counter() - t0)
            del blob
        ms_load = 1e3 * min(times)
        res["e2e"] = {"value": round(body / (ms_load * 1e-3) / 1e9, 2), "unit": "GB/s",
                      "ms": round(ms_load, 1), "h2d_bytes_per_step": body,
                      "d2h_bytes_per_step": 8,
                      "path": "pvlc_b200.checkpoint.load_payload_f16: checked header, file "
                              "(page cache) -> pinned 64 MiB chunks -> HBM -> pvlc_bf16_to_f16 "
                              "in place; best of 2"}
    except Exception as e:   # the kernel figure above stands without the file leg
        res["e2e"] = {"error": f"{type(e).__name__}: {e}"[:200]}
    finally:
        if path is not None and os.path.exists(path):
            os.unlink(path)
    return res


def bench_decode_b1(dev, timeit):
    """one decode call at batch 1 -- q [16,128], 1023 cached K/V rows + the
    appended one (1024 rows after the append), 1,056,768 algorithmic bytes per call.
    Calls rotate over 256 independent caches (272 MB, more than L2), so every call reads
    its cache from HBM."""
    import torch

    from pvlc_b200 import ops, positions
    hbm_peak, _, peak_src = peaks()
    n_sets, L, cap = 256, 1023, 1040
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    kc = torch.randn((n_sets, cap, KVH, HD), generator=g, device=dev).half()
    vc = torch.randn((n_sets, cap, KVH, HD), generator=g, device=dev).half()
    q = torch.randn((n_sets, 1, QH, HD), generator=g, device=dev).half()
    kn = torch.randn((n_sets, 1, KVH, HD), generator=g, device=dev).half()
    vn = torch.randn((n_sets, 1, KVH, HD), generator=g, device=dev).half()
    kp = [torch.tensor([kc[i].data_ptr()], dtype=torch.int64, device=dev) for i in range(n_sets)]
    vp = [torch.tensor([vc[i].data_ptr()], dtype=torch.int64, device=dev) for i in range(n_sets)]
    cos_np, sin_np = positions.linear_rope_tables(cap)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    ct = torch.tensor([L], dtype=torch.int32, device=dev)
    ws = ops.DecodeWorkspace(1, dev)
    out = torch.empty((1, QH, HD), dtype=torch.float16, device=dev)
    it = [0]

    def call():
        i = it[0] % n_sets
        it[0] += 1
        # the same row is appended again each time the set comes round: same bytes
        ops.decode(q[i], kn[i], vn[i], cos, sin, kp[i], vp[i], ct, cap, L, ws, out=out)

    # one call is a few microseconds of device time, less than the host's per-call
    # launch work: the 256 calls are captured once in a CUDA graph and replayed, so
    # the events see device time, not the host
    for _ in range(n_sets):
        call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            for _ in range(n_sets):
                call()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    reps = 8
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (reps * n_sets)
    host_ms = timeit(call)
    if ws.errors():
        raise RuntimeError("decode fault flags in the batch-1 component")
    nbytes = 2 * (L + 1) * KVH * HD * 2 + 2 * QH * HD * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "configs[0] decode, batch 1, Q16/KV2/D128, 1024 K/V rows after the "
                        "append, 256 rotating caches (> L2)",
            "ms": round(ms, 5), "value": round(gbs, 1), "unit": "GB/s",
            "algorithmic_bytes": nbytes,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                         "peak_source": peak_src},
            "host_launched_ms": round(host_ms, 5),
            "note": "device time per call from a CUDA graph of 256 calls; 1 MB per call, so "
                    "launch and pipeline latency, not bandwidth, set the time",
            "kernel": "pvlc::decode::decode_kernel"}


def cpu_decode_b1_baseline(seconds: float = 1.0):
    """configs[0] on the host: the oracle's decode step (C++ restatement of pvlc-cpu-ref:
    M-RoPE of q and the new key, append, GQA attention over 1024 rows) repeated for about a
    second; GB/s of the same algorithmic bytes as the device component."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pvlc_oracle as O
    from pvlc_b200 import positions
    L, cap = 1023, 1040
    cos, sin = positions.linear_rope_tables(cap)
    rng = np.random.default_rng(0)
    kc = rng.standard_normal((cap, KVH, HD)).astype(np.float16).astype(np.float32)
    vc = rng.standard_normal((cap, KVH, HD)).astype(np.float16).astype(np.float32)
    q = rng.standard_normal((QH * HD,)).astype(np.float32)
    kn = rng.standard_normal((KVH * HD,)).astype(np.float32)
    vn = rng.standard_normal((KVH * HD,)).astype(np.float32)
    nbytes = 2 * (L + 1) * KVH * HD * 2 + 2 * QH * HD * 2
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        O.decode_step(q, kn, vn, cos, sin, L, kc, vc, L)
        calls += 1
    el = time.perf_counter() - t0
    return {"value": round(nbytes * calls / el / 1e9, 3), "unit": "GB/s", "cores": O.threads(),
            "kind": "port",
            "sample": f"{calls} batch-1 decode calls at 1024 rows, {el:.2f} s"}


def cpu_linear_baseline(rows: int = 32, reps: int = 3):
    """The decode layer's four projections at `rows` rows through the oracle's linear (the
    reference's linear_f32 order, f32) on the host cores; GB/s of the fp16 weight bytes
    the device component reads."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pvlc_oracle as O
    rng = np.random.default_rng(8)
    shapes = [(1024, 2560), (2048, 1024), (1024, 6144), (3072, 1024)]
    mats = [(rng.standard_normal((rows, k)).astype(np.float32),
             (rng.standard_normal((n, k)) * k ** -0.5).astype(np.float32)) for k, n in shapes]
    wbytes = sum(n * k * 2 for k, n in shapes)
    t0 = time.perf_counter()
    for _ in range(reps):
        for x, w in mats:
            O.linear(x, w)
    el = (time.perf_counter() - t0) / reps
    return {"value": round(wbytes / el / 1e9, 3), "unit": "GB/s", "cores": O.threads(),
            "kind": "port", "layer_us": round(el * 1e6, 1),
            "sample": f"one decoder layer's four projections at {rows} rows, {reps} passes"}


def cpu_attention_baseline(kind, args_np, flops):
    """The oracle (C++ restatement of pvlc-cpu-ref) on the full component workload, on the
    host cores; returns the cpu_baseline record in TFLOP/s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pvlc_oracle as O
    t0 = time.perf_counter()
    if kind == "vision":
        q, k, v, T, cu, c, s_ = args_np
        qr, kr = O.vision_rope_apply_tables(q, k, T, 16, 72, c, s_)
        O.segmented_attention(qr, kr, v, T, 16, 72, cu)
        what = "vision_rope_2d (tables) + materialized_segmented_attention_f32, all 8000 tokens"
    else:
        q, k, v, T, c, s_, cap = args_np
        import numpy as np
        kc = np.zeros((cap, 2, 128), np.float32)
        vc = np.zeros_like(kc)
        O.decoder_prefill(q, k, v, c, s_, T, kc, vc)
        what = "apply_multimodal_rope_f32 + KV write + causal_gqa_f32, all 1564 tokens"
    el = time.perf_counter() - t0
    return {"value": round(flops / el / 1e12, 5), "unit": "TFLOP/s", "cores": O.threads(),
            "kind": "port", "sample": f"the full workload once ({what}), {el:.2f} s"}


def library_sdpa(dev, q, k, v, causal, gqa, segments=None):
    """Context only: the same attention through torch's scaled_dot_product_attention
    (cuDNN's fused attention where torch picks it), on pre-rotated inputs; not this
    library's code.  Returns ms per call or an error string."""
    import torch
    import torch.nn.functional as F
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        segs = segments or [(0, q.shape[0])]
        qs = [q[a:b].transpose(0, 1).unsqueeze(0) for a, b in segs]
        ks = [k[a:b].transpose(0, 1).unsqueeze(0) for a, b in segs]
        vs = [v[a:b].transpose(0, 1).unsqueeze(0) for a, b in segs]

        def run():
            for x, y, z in zip(qs, ks, vs):
                F.scaled_dot_product_attention(x, y, z, is_causal=causal, enable_gqa=gqa)

        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
                          SDPBackend.EFFICIENT_ATTENTION]):
            for _ in range(3):
                run()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(20):
                run()
            b.record()
            torch.cuda.synchronize()
        return a.elapsed_time(b) / 20
    except Exception as e:   # noqa: BLE001 - context figure only
        return f"{type(e).__name__}: {e}"[:160]


def bench_vision(dev, timeit, tf_peak, peak_src, cpu=True):
    """Vision varlen prefill, configs[1]."""
    import torch

    from pvlc_b200 import ops, positions
    grids = [(1, 32, 32), (1, 48, 48), (1, 24, 24), (1, 64, 64)]
    cu = [0, 1024, 3328, 3904, 8000]
    T = 8000
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    nrot = 8   # rotate input sets so consecutive launches do not hit the same L2 lines
    qs = [torch.randn((T, 16, 72), generator=g, device=dev).half() for _ in range(nrot)]
    ks = [torch.randn((T, 16, 72), generator=g, device=dev).half() for _ in range(nrot)]
    vs = [torch.randn((T, 16, 72), generator=g, device=dev).half() for _ in range(nrot)]
    c_np, s_np = positions.vision_rope_tables(grids)
    vcos, vsin = torch.from_numpy(c_np).to(dev), torch.from_numpy(s_np).to(dev)
    vout = torch.empty_like(qs[0])
    vws = torch.empty(ops.vision_workspace_bytes(T, 16), dtype=torch.uint8, device=dev)
    it = [0]

    def vis():
        i = it[0] % nrot
        it[0] += 1
        ops.vision_varlen_attention(qs[i], ks[i], vs[i], cu, vcos, vsin, out=vout, workspace=vws)

    ms = timeit(vis)
    flops = 4.0 * 72 * 16 * sum((cu[i + 1] - cu[i]) ** 2 for i in range(4))
    tf = flops / (ms * 1e-3) / 1e12
    res = {"workload": "configs[1] 8000 tokens, segments 1024/2304/576/4096, H16 D72, 2-D RoPE",
           "ms": round(ms, 4), "value": round(tf, 2), "unit": "TFLOP/s",
           "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": tf_peak,
                        "unit": "TFLOP/s", "frac": round(tf / tf_peak, 4),
                        "peak_source": peak_src, "traffic": VISION_TC_TRAFFIC_BYTES,
                        "traffic_kernel": "pvlc::vtc::vision_tc_kernel (ncu, one launch)"},
           "kernel": "pvlc::vtc::vision_rope_kernel + pvlc::vtc::vision_tc_kernel"}
    lib_ms = library_sdpa(dev, qs[0], ks[0], vs[0], False, False,
                          [(cu[i], cu[i + 1]) for i in range(4)])
    res["library_reference"] = {
        "what": "torch scaled_dot_product_attention per image (4 calls), q/k not rotated",
        "ms": round(lib_ms, 4) if isinstance(lib_ms, float) else lib_ms,
        "tflops": round(flops / (lib_ms * 1e-3) / 1e12, 1) if isinstance(lib_ms, float) else None}
    if cpu:
        f = lambda t: t.float().cpu().numpy()   # noqa: E731
        res["cpu_baseline"] = cpu_attention_baseline(
            "vision", (f(qs[0]), f(ks[0]), f(vs[0]), T, cu, c_np, s_np), flops)
    return res


def bench_prefill(dev, timeit, tf_peak, peak_src, cpu=True):
    """Decoder causal prefill, configs[2]."""
    import torch

    from pvlc_b200 import ops, positions
    nrot = 8
    it = [0]
    g = torch.Generator(device=dev)
    ids = [7] * 19 + [101305] + [100295] * 1480 + [9] * 64
    pos, delta = positions.mrope_position_ids(ids, [(1, 80, 74)])
    Tp = len(ids)
    pc, ps = positions.mrope_tables(pos, delta, Tp + 256)
    pcos, psin = torch.from_numpy(pc).to(dev), torch.from_numpy(ps).to(dev)
    g.manual_seed(3)
    pq = [torch.randn((Tp, 16, 128), generator=g, device=dev).half() for _ in range(nrot)]
    pk = [torch.randn((Tp, 2, 128), generator=g, device=dev).half() for _ in range(nrot)]
    pv = [torch.randn((Tp, 2, 128), generator=g, device=dev).half() for _ in range(nrot)]
    kcache = torch.empty((Tp + 256, 2, 128), dtype=torch.float16, device=dev)
    vcache = torch.empty_like(kcache)
    pout = torch.empty_like(pq[0])

    def pre():
        i = it[0] % nrot
        it[0] += 1
        ops.decoder_prefill(pq[i], pk[i], pv[i], pcos, psin, kcache, vcache, out=pout)

    ms = timeit(pre)
    flops = 4.0 * 128 * 16 * Tp * (Tp + 1) / 2
    tf = flops / (ms * 1e-3) / 1e12
    res = {"workload": "configs[2] T=1564 (20 text + 40x37 image + 64 text), Q16/KV2/D128, M-RoPE",
           "ms": round(ms, 4), "value": round(tf, 2), "unit": "TFLOP/s",
           "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": tf_peak,
                        "unit": "TFLOP/s", "frac": round(tf / tf_peak, 4),
                        "peak_source": peak_src, "traffic": PREFILL_ATTN_TRAFFIC_BYTES,
                        "traffic_kernel": "pvlc::ptc::prefill_attn_kernel (ncu, one launch)"},
           "kernel": "pvlc::ptc::kv_rope_kernel + pvlc::ptc::prefill_attn_kernel"}
    lib_ms = library_sdpa(dev, pq[0], pk[0], pv[0], True, True)
    res["library_reference"] = {
        "what": "torch scaled_dot_product_attention, causal GQA, q/k not rotated, no cache write",
        "ms": round(lib_ms, 4) if isinstance(lib_ms, float) else lib_ms,
        "tflops": round(flops / (lib_ms * 1e-3) / 1e12, 1) if isinstance(lib_ms, float) else None}
    if cpu:
        f = lambda t: t.float().cpu().numpy()   # noqa: E731
        res["cpu_baseline"] = cpu_attention_baseline(
            "prefill", (f(pq[0]), f(pk[0]), f(pv[0]), Tp, pc, ps, Tp + 256), flops)
    return res


def bench_prefill_batch(dev, timeit, tf_peak, peak_src):
    """Decoder causal prefill of one layer over the configs[4] batch: 256 OCR prompts of
    1238 tokens (1225 image tokens of a 980x980 page) packed back to back, one
    pvlc_attn_decoder_prefill_batch launch pair -- the e2e engine's per-layer call."""
    import numpy as np
    import torch

    from pvlc_b200 import ops, positions
    from pvlc_b200 import model as M
    B = 256
    ids = M.ocr_prompt_ids(1225)
    T = len(ids)
    pos, delta = positions.mrope_position_ids(ids, [(1, 70, 70)])
    cap = T + 16
    pc, ps = positions.mrope_tables(pos, delta, cap)
    tab = (torch.from_numpy(pc).to(dev), torch.from_numpy(ps).to(dev))
    offs = np.arange(B + 1, dtype=np.int64) * T
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    # 0.8 GB of q per set: larger than L2, so no rotation of input sets is needed
    q = torch.randn((B * T, 16, 128), generator=g, device=dev).half()
    k = torch.randn((B * T, 2, 128), generator=g, device=dev).half()
    v = torch.randn((B * T, 2, 128), generator=g, device=dev).half()
    kc = torch.empty((B, cap, 2, 128), dtype=torch.float16, device=dev)
    vc = torch.empty_like(kc)
    out = torch.empty_like(q)
    tables = [tab] * B

    def pre():
        ops.decoder_prefill_packed(q, k, v, offs, tables, kc, vc, out)

    ms = timeit(pre)
    flops = B * 4.0 * 128 * 16 * T * (T + 1) / 2
    tf = flops / (ms * 1e-3) / 1e12
    res = {"workload": f"configs[4] decoder prefill, {B} prompts x {T} tokens packed, one "
                       "launch pair per layer, Q16/KV2/D128, M-RoPE",
           "ms": round(ms, 4), "value": round(tf, 2), "unit": "TFLOP/s",
           "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": tf_peak,
                        "unit": "TFLOP/s", "frac": round(tf / tf_peak, 4),
                        "peak_source": peak_src},
           "kernel": "pvlc::ptc::kv_rope_kernel<256> + pvlc::ptc::prefill_persist_kernel<256>"}
    # context: the same causal GQA as one batched torch SDPA call (all prompts have the
    # same length here, so a [B, heads, T, 128] batch needs no packing)
    try:
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel
        qb = q.view(B, T, 16, 128).transpose(1, 2)
        kb = k.view(B, T, 2, 128).transpose(1, 2)
        vb = v.view(B, T, 2, 128).transpose(1, 2)
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
                          SDPBackend.EFFICIENT_ATTENTION]):
            lib_ms = timeit(lambda: F.scaled_dot_product_attention(qb, kb, vb, is_causal=True,
                                                                   enable_gqa=True))
        res["library_reference"] = {
            "what": "torch scaled_dot_product_attention, [256, 16, 1238, 128] causal GQA, q/k "
                    "not rotated, no cache write",
            "ms": round(lib_ms, 4), "tflops": round(flops / (lib_ms * 1e-3) / 1e12, 1)}
    except Exception as e:   # noqa: BLE001 - context figure only
        res["library_reference"] = {"error": f"{type(e).__name__}: {e}"[:160]}
    return res


def run_e2e(args, dev, rank, world, dist):
    """end-to-end greedy OCR through the public engine API.

    Random-init fp16 PaddleOCR-VL weights; seeded uniform-noise 1024x1024 RGB pages
    (smart_resize -> 980x980 -> 4900 patches -> 1225 image tokens, 1238-token prompts);
    args.e2e_requests requests sharded by index over the ranks; args.e2e_tokens greedy
    tokens each (EOS stops a request early).  Timed per rank with CUDA events around
    OcrEngine.recognize(): host->device page copies from pinned memory, device
    preprocessing, vision encoder, projector, decoder prefill, CUDA-graph decode and the
    token readbacks; max over ranks."""
    import numpy as np
    import torch

    from pvlc_b200 import dist as pdist
    from pvlc_b200 import model as M

    cfg = M.ModelConfig()
    weights = M.init_weights(cfg, seed=0, device=dev)
    eng = M.OcrEngine(cfg, weights, dev)
    mine = pdist.shard(args.e2e_requests, rank, world)
    pages = [request_page(i, pin=True) for i in mine]

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # warm-up: one call of the timed batch shape -- kernels, cuBLAS heuristics, the
    # allocator's pool, and the engine's KV caches and decode-step graph, which the
    # engine keeps for the next call of the same shape (a serving engine's steady state)
    eng.recognize(pages, args.e2e_tokens)
    barrier()
    timings = {}
    # clocks at a 20 ms period: the engine's host thread shares the interpreter lock
    # with the sampler, so it samples less often than around the kernel-only regions
    sampler = ClockSampler(torch.cuda.current_device(), period_s=0.02)
    load0 = os.getloadavg()[0]
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    res = eng.recognize(pages, args.e2e_tokens, timings=timings)
    e1.record()
    barrier()
    clocks = sampler.stop()
    clocks["host_loadavg_1m"] = [round(load0, 2), round(os.getloadavg()[0], 2)]
    # every rank's own breakdown, for the record (stderr: stdout carries the JSON line)
    print(f"e2e rank {rank}/{world}: {e0.elapsed_time(e1):.1f} ms {timings}", file=sys.stderr,
          flush=True)
    ms = e0.elapsed_time(e1)
    tokens = sum(len(t) for t in res["tokens"])
    eos = sum(1 for r in res["stop"] if r == "eos_token")
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    n = torch.tensor([tokens, len(mine), eos], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
    ms_max = float(t.item())
    tokens_all, reqs_all, eos_all = (int(x) for x in n.tolist())
    # after the timed region: every request's token ids and every rank's phase times
    # to rank 0 (NCCL all-gather of a fixed-size id block per rank, then a small object
    # gather), the only cross-GPU traffic of the run
    gathered = pdist.gather_token_ids(res["tokens"], args.e2e_requests, args.e2e_tokens, dev)
    phases = dict(rank=rank, ms=round(ms, 2), requests=len(mine),
                  **{k: (round(v, 2) if isinstance(v, float) else v) for k, v in timings.items()})
    per_rank = pdist.gather_to_rank0(phases) if dist is not None else [phases]
    out = {"workload": "configs[4] e2e greedy OCR, random-init fp16 PaddleOCR-VL, 1024x1024 "
                       "noise pages -> 980x980 (1225 image tokens), OCR prompt",
           "requests": reqs_all, "max_new_tokens": args.e2e_tokens, "n_gpus": world,
           "generated_tokens": tokens_all, "eos_stops": eos_all, "ms": round(ms_max, 2),
           "tokens_per_s": round(tokens_all / (ms_max * 1e-3), 1),
           "tokens_per_s_per_gpu": round(tokens_all / (ms_max * 1e-3) / world, 1),
           "requests_per_s": round(reqs_all / (ms_max * 1e-3), 3),
           "rank0_breakdown_ms": {k: (round(v, 2) if isinstance(v, float) else v)
                                  for k, v in timings.items()},
           "h2d_bytes_per_request": 1024 * 1024 * 3,
           "decode_batch_per_gpu": len(mine),
           "per_rank": per_rank,
           "clocks": clocks,
           "path": "pvlc_b200.model.OcrEngine.recognize (host pages in, token ids out)"}
    if rank == 0:
        out["tokens_digest"] = pdist.tokens_digest(gathered)
        # the gathered ids of a sample of requests -- the first one of every rank's shard
        # (at one GPU the first eight) -- against the same requests run again on rank 0
        # as one batch of their own
        sample = list(range(min(args.e2e_requests, max(world, 8))))
        again = eng.recognize([request_page(i, pin=True) for i in sample], args.e2e_tokens)
        first_diff = {}
        for i, toks in zip(sample, again["tokens"]):
            a, g = [int(x) for x in toks], gathered[i]
            if a != g:
                first_diff[i] = next((s for s, (x, y) in enumerate(zip(a, g)) if x != y),
                                     min(len(a), len(g)))
        out["rerun_check"] = {"requests": sample, "rerun_batch": len(sample),
                              "identical": len(sample) - len(first_diff),
                              "first_divergent_step": first_diff}
    if dist is not None:
        dist.barrier()
    if rank == 0 and not args.skip_cpu:
        out["cpu_baseline"] = cpu_e2e_baseline(cfg, weights)
    del eng, weights
    torch.cuda.empty_cache()
    return out


def request_page(i, pin=False):
    """configs[4] request i: a seeded uniform-noise 1024x1024 RGB page (host memory)."""
    import numpy as np
    import torch
    rng = np.random.default_rng(10_000 + i)
    t = torch.from_numpy(rng.integers(0, 256, (1024, 1024, 3), dtype=np.uint8))
    return t.pin_memory() if pin else t


# --------------------------------------------------------------- CPU (oracle)
def cpu_e2e_baseline(cfg, weights):
    """The reference's f32 composition (the oracle) on one reduced request: a 112x112 page
    (8x8 patches, 16 image tokens) and 4 greedy tokens, on the host cores."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pvlc_oracle as O
    from pvlc_b200 import model as M
    from pvlc_b200 import preprocess as P

    host = [[t.cpu().numpy() for t in part]
            for part in (weights.vision, weights.projector, weights.decoder)]
    rgb = np.random.default_rng(10_000).integers(0, 256, (112, 112, 3), dtype=np.uint8)
    pre = P.canonical_rgb8_to_patches(rgb, P.VisionPreprocessConfig(min_pixels=112 * 112,
                                                                     max_pixels=112 * 112))
    g = pre.image_grid_thw
    ids = M.ocr_prompt_ids(g[0] * g[1] * g[2] // 4, cfg)
    t0 = time.perf_counter()
    r = O.generate(cfg.oracle_dims(), *host, pre.values, [g], ids, 4, fp16_storage=False)
    el = time.perf_counter() - t0
    return {"value": round(len(r["tokens"]) / el, 4), "unit": "tokens/s", "cores": O.threads(),
            "kind": "port",
            "sample": f"1 request, 112x112 page (16 image tokens, {len(ids)}-token prompt), "
                      f"{len(r['tokens'])} greedy tokens, {el:.1f} s end to end "
                      "(reduced: a 980x980 page is ~4e12 FLOP of vision encoder on the CPU)"}



def cpu_convert_baseline(sample_bits):
    """The reference's host conversion (fp16.rs:171-276, one element at a time), restated
    in the oracle, over a bounded sample of the payload; GB/s at 4 bytes per element."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pvlc_oracle as O
    O.bf16_to_f16_bits(sample_bits[:1024])
    t0 = time.perf_counter()
    _, status = O.bf16_to_f16_bits(sample_bits)
    dt = time.perf_counter() - t0
    return {"value": round(4.0 * sample_bits.size / dt / 1e9, 3), "unit": "GB/s", "cores": 1,
            "kind": "port", "checked": bool((status == 0).all()),
            "sample": f"{sample_bits.size:,} BF16 elements of the bench payload, "
                      f"{dt:.2f} s, one thread"}


def cpu_decode_baseline(seconds: float):
    """The C++ restatement of pvlc-cpu-ref's decode step on the host cores, over a
    bounded sample of the decode-sweep workload (same length distribution)."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pvlc_oracle as O
    from pvlc_b200 import positions

    rng = np.random.default_rng(1)
    L0 = rng.integers(L_MIN, L_MAX + 1, size=SEQS_PER_GPU)
    cap = L_MAX + 64
    cos, sin = positions.linear_rope_tables(cap)
    data_rng = np.random.default_rng(5)
    kc = data_rng.standard_normal((cap, KVH, HD)).astype(np.float16).astype(np.float32)
    vc = data_rng.standard_normal((cap, KVH, HD)).astype(np.float16).astype(np.float32)
    q = data_rng.standard_normal((QH * HD,)).astype(np.float32)
    kn = data_rng.standard_normal((KVH * HD,)).astype(np.float32)
    vn = data_rng.standard_normal((KVH * HD,)).astype(np.float32)
    done_bytes, calls = 0, 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        L = int(L0[calls % len(L0)])
        O.decode_step(q, kn, vn, cos, sin, L, kc, vc, L)
        done_bytes += 1024 * (L + 1) + 8192 + 1024
        calls += 1
    el = time.perf_counter() - t0
    return {"value": round(done_bytes / el / 1e9, 4), "unit": UNIT, "cores": O.threads(),
            "kind": "port",
            "sample": f"{calls} sequence-layer decode steps (L from the seed-1 U[512,8192] draw), "
                      f"{el:.1f} s, OpenMP over query heads",
            "tokens_per_s": round(calls / el / LAYERS, 3)}


def run_reference(args, rank):
    if rank != 0:
        return None
    base = cpu_decode_baseline(args.cpu_seconds)
    return {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "configs[3] batched GQA decode sweep (bounded CPU sample)"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference is Rust (no cargo/rustc here); its f32 algorithm is timed via the "
                    "C++ restatement in oracle/"}


_JSON_FD = None


def _stdout_for_json_only():
    """Keep the process's stdout for the JSON line alone: libraries that print to file
    descriptor 1 (NCCL's version banner at communicator creation, among others) are sent
    to stderr, and emit() writes the line to the saved descriptor."""
    global _JSON_FD
    if _JSON_FD is None:
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)


def emit(obj) -> None:
    data = (json.dumps(obj) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def main():
    global LAYERS, SEQS_PER_GPU, METRIC
    _stdout_for_json_only()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-components", action="store_true")
    ap.add_argument("--traffic-bytes", type=float, default=None,
                    help="ncu dram bytes per decode launch, when measured")
    ap.add_argument("--seqs", type=int, default=SEQS_PER_GPU,
                    help="sequences per GPU (profiling runs use a smaller case)")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--skip-e2e", action="store_true", help="skip configs[4] e2e greedy OCR")
    ap.add_argument("--e2e-requests", type=int, default=256)
    ap.add_argument("--e2e-tokens", type=int, default=512)
    ap.add_argument("--only", choices=["decode_b1", "vision", "prefill", "prefill_batch",
                                       "checkpoint", "pack_blake3", "decode_linear", "e2e"],
                    default=None,
                    help="time one prefill component alone (profiling runs); prints its line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.seqs != SEQS_PER_GPU or args.layers != LAYERS:
        METRIC = f"decode-attn HBM GB/s ({args.seqs} seqs x {args.layers} layers, reduced case)"
    LAYERS, SEQS_PER_GPU = args.layers, args.seqs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if args.only == "e2e" and args.impl == "ours":
        import torch
        torch.cuda.set_device(0)
        emit(run_e2e(args, torch.device("cuda", 0), 0, 1, None))
        return
    if args.only is not None and args.impl == "ours":
        import torch
        hbm_peak, tf_peak, peak_src = peaks()
        res = run_components(args, torch.device("cuda", 0), tf_peak, peak_src,
                             which=(args.only,), iters=args.steps, warm=args.warmup)
        emit(res)
        return
    if args.impl == "reference":
        line = run_reference(args, rank)
    else:
        if world > 1:
            import torch
            import torch.distributed as tdist

            from pvlc_b200 import dist as pdist
            torch.cuda.set_device(local_rank)
            pdist.init("nccl", timeout_s=120.0, device_id=torch.device("cuda", local_rank))
            dist = tdist
        line = run_gpu(args, rank, world, local_rank, dist)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        # the single-GPU components run on rank 0 after the last collective, so no
        # rank waits in one while they run
        if line is not None and not args.skip_components:
            import torch
            _, tf_peak, peak_src = peaks()
            comps = run_components(args, torch.device("cuda", local_rank), tf_peak, peak_src)
            comps.update(line["components"])
            line["components"] = comps
    if line is not None:
        emit(line)


if __name__ == "__main__":
    main()

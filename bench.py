#!/usr/bin/env python
"""Benchmark of the B200 attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline line (one JSON line on rank 0): decode-attention HBM GB/s on BASELINE
config 3 -- 64 independent sequences per GPU, 24 layers, 14 query / 2 KV heads,
head_dim 64, f16 head-major KV cache with lengths drawn U{256..4096}, one new
token per sequence with RoPE and the KV append fused. A step is one decode of
all 24 layers for every sequence (one C-ABI call). `value` is whole-job
throughput over all ranks with inputs resident in HBM; `e2e` is the same metric
through the host-pointer C-ABI path (pinned host inputs copied in and outputs
read back inside the timed region). Per GPU the work is fixed (weak scaling);
sequences are independent, so no collective touches the data path.

The `prefill` object reports BASELINE config 2 (causal prefill, bf16) in
TFLOPS with its own roofline. `cpu_baseline` times the CPU restatement of the
reference's attention (oracle/, f64 accumulation as the reference's JS does)
on a bounded sample of the same workload on this host's cores.

--impl reference times the reference's CPU path restated in C (the reference is
JavaScript and no JS runtime exists on this machine) on the same workload and
prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "llm-inference-webgpu_b200")
for _p in (ROOT, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

H, KVH, D, THETA = 14, 2, 64, 1e6
SEQS, LAYERS, LMIN, LMAX = 64, 24, 256, 4096
CAP = 4160                       # >= LMAX + 1, a multiple of 64
METRIC = "decode-attn HBM GB/s"


# ----------------------------------------------------------------- helpers --

def peaks() -> dict:
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
            if k in m:
                p[k] = float(m[k])
        p["source"] = "measured"
    return p


def ncu_traffic(kernel: str, workload: str):
    """dram read+write bytes per launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#") and parts[0] == kernel and parts[1] == workload:
                return float(parts[2])
    return None


def workload_name() -> str:
    if (SEQS, LAYERS) == (64, 24):
        return "config3-batched-decode"
    return f"config3-batched-decode-reduced(seqs={SEQS},layers={LAYERS})"


def config3_lengths(rank: int) -> np.ndarray:
    rng = np.random.default_rng(1234 + rank)
    return rng.integers(LMIN, LMAX + 1, size=SEQS).astype(np.int32)


def config3_bytes(lengths: np.ndarray, cache_es: int = 2, in_es: int = 2, out_es: int = 4) -> dict:
    """Algorithmic bytes of one config-3 step (all layers, all sequences)."""
    kv_read = int(LAYERS * KVH * D * cache_es * 2 * int((lengths.astype(np.int64) + 1).sum()))
    q = SEQS * LAYERS * H * D * in_es
    kv_new = 2 * SEQS * LAYERS * KVH * D * in_es
    append = 2 * SEQS * LAYERS * KVH * D * cache_es
    out = SEQS * LAYERS * H * D * out_es
    return {"kv_read": kv_read, "q": q, "kv_new": kv_new, "append": append, "out": out,
            "attention_kernel": kv_read + q + kv_new + append, "step": kv_read + q + kv_new + append + out}


def config3_block(world: int) -> dict:
    """The headline workload's `config`, the same on both arms."""
    nb = config3_bytes(config3_lengths(0))
    return {"workload": workload_name(), "sequences_per_gpu": SEQS, "layers": LAYERS,
            "heads": "14q/2kv", "head_dim": D, "kv_len": f"U{{{LMIN}..{LMAX}}} seeded per rank",
            "cache_dtype": "f16", "q_dtype": "f16", "out_dtype": "f32", "rope_theta": THETA,
            "bytes_per_step_per_gpu": nb["step"], "parallelism": f"dp{world} (sequences)",
            "l2": "inputs larger than L2 (KV read per step per GPU %.2f GB)" % (nb["kv_read"] / 1e9)}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float) -> dict:
        rows = [s for t, s in self.samples if t0 <= t <= t1] or [s for _, s in self.samples]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            f = [x.strip() for x in r.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for(torch, dev: int) -> str:
    try:
        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[dev]
        return str(dev)


class _CAI:
    """__cuda_array_interface__ over a device pointer, so torch can view the cache pools."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


# ------------------------------------------------------- parity samples ---
# A check of the measured runs' outputs, outside every timed region: sampled
# rows recomputed in float64 with PyTorch on the same device inputs (the
# reference's decode, src/cpu/model.js:103-123 over src/core/attention.js:32-66:
# RoPE of the query at its absolute position, scores scaled by 1/sqrt(64), a
# max-shifted softmax, the weighted sum of values). The CPU oracle is the
# tests' checker; this is the benchmark's own sanity check of the same runs.

def _rope_f64(torch, x, positions, dev):
    """Half-split rotation (src/core/ops.js:147-158) of x [..., rows, 64] at positions [rows], f64."""
    half = D // 2
    inv = torch.tensor([THETA ** (-2.0 * j / D) for j in range(half)], dtype=torch.float64, device=dev)
    ang = torch.as_tensor(np.asarray(positions, np.float64), device=dev)[:, None] * inv[None, :]
    c, s_ = torch.cos(ang), torch.sin(ang)
    lo, hi = x[..., :half], x[..., half:]
    return torch.cat([lo * c - hi * s_, hi * c + lo * s_], dim=-1)


def _attend_f64(torch, qr, k, v):
    """qr [heads, 64]; k, v [kv_heads, n, 64] (f64): softmax(q k^T / 8) v per head, heads grouped."""
    group = qr.shape[0] // k.shape[0]
    kk = k.repeat_interleave(group, dim=0)
    vv = v.repeat_interleave(group, dim=0)
    sc = torch.einsum("hd,hnd->hn", qr, kk) / math.sqrt(D)
    return torch.einsum("hn,hnd->hd", torch.softmax(sc, dim=-1), vv)


def _summary(errs, scales) -> dict:
    mx = max(errs) if errs else 0.0
    rel = max(e / s for e, s in zip(errs, scales) if s > 0) if errs else 0.0
    return {"max_abs": float(f"{mx:.3g}"), "rel": float(f"{rel:.3g}"), "ok": bool(mx <= 2e-3 and rel <= 1e-2)}


def parity_decode(torch, dev, kp, vp, shape, q, out, lengths, picks) -> dict:
    """Sampled (sequence, layer) rows of a decode whose cache pools are viewed as `shape`
    [seqs][layers][kv_heads][cap][64] f16; q [seqs][layers][heads][64]; out likewise (f32)."""
    kv = torch.as_tensor(_CAI(kp, shape, "<f2"), device=dev)
    vv = torch.as_tensor(_CAI(vp, shape, "<f2"), device=dev)
    errs, scales = [], []
    for b, layer in picks:
        n = int(lengths[b]) + 1
        qr = _rope_f64(torch, q[b, layer].double(), [n - 1] * q.shape[2], dev)
        ref = _attend_f64(torch, qr, kv[b, layer, :, :n].double(), vv[b, layer, :, :n].double())
        errs.append(float((out[b, layer].double() - ref).abs().max()))
        scales.append(float(ref.abs().max()))
    res = _summary(errs, scales)
    res["rows"] = len(picks)
    return res


def parity_prefill(torch, dev, q, k, v, o, rows) -> dict:
    """Query rows of a causal prefill from position 0: q, o [S][heads][64]; k, v [S][kv][64]
    (the inputs before RoPE; keys rotated in f64, as exact as an f32 cache allows)."""
    S = q.shape[0]
    kr = _rope_f64(torch, k.double().transpose(0, 1), list(range(S)), dev)   # [kv][S][64]
    vt = v.double().transpose(0, 1)
    errs, scales = [], []
    for t in rows:
        qr = _rope_f64(torch, q[t].double(), [t] * q.shape[1], dev)
        ref = _attend_f64(torch, qr, kr[:, :t + 1], vt[:, :t + 1])
        # bf16 output: its own rounding (half an ulp) is not an error of the kernel
        errs.append(float(((o[t].double() - ref).abs() - ref.abs() * 2.0 ** -8).clamp_min(0).max()))
        scales.append(float(ref.abs().max()))
    res = _summary(errs, scales)
    res["rows"] = len(rows)
    return res


# ---------------------------------------------------------- CPU baselines --

def cpu_decode_sample(lengths: np.ndarray, target_s: float, threads: int = 0):
    """The reference's attention (restated in C, f64 accumulation) over config-3
    sequences, one layer's worth of data reused for `n` layers. Returns
    (GB/s, threads, description)."""
    from oracle import oracle as o
    rng = np.random.default_rng(99)
    cap = int(lengths.max()) + 1
    seq_stride = KVH * cap * D
    kb = rng.standard_normal(SEQS * seq_stride, dtype=np.float32).astype(np.float16).view(np.uint16)
    vb = rng.standard_normal(SEQS * seq_stride, dtype=np.float32).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(SEQS * H * D, dtype=np.float32)
    b = config3_bytes(lengths)
    per_layer = b["step"] / LAYERS
    t0 = time.perf_counter()
    _, used = o.batched_decode_f16(q, H * D, kb, vb, seq_stride, lengths, SEQS, cap, H, KVH, D, H * D, threads)
    t1 = time.perf_counter() - t0
    n = max(1, int(target_s / max(t1, 1e-6)))   # layers timed (the step has LAYERS; more repeat them)
    t0 = time.perf_counter()
    for _ in range(n):
        o.batched_decode_f16(q, H * D, kb, vb, seq_stride, lengths, SEQS, cap, H, KVH, D, H * D, threads)
    dt = time.perf_counter() - t0
    return per_layer * n / dt / 1e9, used, (f"{SEQS} sequences x {n} layer(s) of config 3 "
                                           f"({n * per_layer / 1e9:.3f} GB), {dt:.2f} s")


# ------------------------------------------------------------------ ours ----

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import b2a

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # NCCL's banner ("NCCL version ...") goes to stdout, where rank 0's one JSON
        # line must stand alone: keep NCCL to warnings unless asked for more
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.Stream(device=dev)
    ctx = b2a.Context(local)
    ctx.set_stream(stream)
    if args.generation_only:   # config 4 alone (a short run to profile its launches)
        res = bench_generation(torch, b2a, ctx, stream, dev, peaks()["hbm_gbs"], args)
        if rank == 0:
            print(json.dumps(res))
        return
    lengths = config3_lengths(rank)
    nb = config3_bytes(lengths)
    with torch.cuda.stream(stream):
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(LAYERS, KVH, D, H), CAP, batch=SEQS, dtype="f16")
        rope = b2a.RopeTable(ctx, D, THETA, 32769)
        kp, vp, strides = cache.pools()
        shape = (SEQS, LAYERS, KVH, CAP, D)
        gen = torch.Generator(device=dev)
        gen.manual_seed(4321 + rank)
        torch.as_tensor(_CAI(kp, shape, "<f2"), device=dev).normal_(generator=gen)
        torch.as_tensor(_CAI(vp, shape, "<f2"), device=dev).normal_(generator=gen)
        cache.setLengths(lengths)
        q = torch.randn(SEQS, LAYERS, H, D, device=dev, generator=gen).half()
        kn = torch.randn(SEQS, LAYERS, KVH, D, device=dev, generator=gen).half()
        vn = torch.randn(SEQS, LAYERS, KVH, D, device=dev, generator=gen).half()
        out = torch.empty(SEQS, LAYERS, H, D, device=dev, dtype=torch.float32)
    torch.cuda.synchronize(dev)

    def step():
        b2a.attentionDecode(ctx, cache, rope, 0, q, kn, vn, out, H, numLayers=LAYERS)

    clocks = ClockSampler(gpu_id_for(torch, local)) if rank == 0 else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if clocks:
        clocks.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize(dev)
    t_wall0 = time.time()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    t_wall1 = time.time()
    ms = e0.elapsed_time(e1)
    if clocks:
        time.sleep(0.2)
        clocks.stop()
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    value = world * nb["step"] * args.steps / (ms_max / 1e3) / 1e9

    # per-kernel device time (events around each launch on the launching stream)
    ktimes_steps = max(3, min(args.steps, 50))
    ctx.enable_timing(True)
    for _ in range(ktimes_steps):
        step()
    kt = ctx.read_timing()
    ctx.enable_timing(False)
    attn_name = "attention_mma" if "attention_mma" in kt else "attention_simt"
    attn_ms = kt[attn_name][1] / kt[attn_name][0]
    launches_per_step = sum(v[0] for v in kt.values()) / ktimes_steps

    # end to end through the host-pointer C ABI: every step copies its pinned
    # inputs in and its output back to pinned host memory inside the timed
    # region. Headline: b2a_attention_decode_host_async, the steps enqueued back
    # to back (two host buffer sets in turn) and one synchronisation at the end,
    # so a step's copies run under its neighbours' kernels. Beside it: the
    # synchronous call (each call returns with its results, as the reference's
    # groupedAttention does).
    e2e_steps = max(3, min(args.steps, 200))
    host_sets = [(q.cpu().pin_memory(), kn.cpu().pin_memory(), vn.cpu().pin_memory(),
                  torch.empty(out.shape, dtype=torch.float32).pin_memory()) for _ in range(2)]
    qh, knh, vnh, outh = host_sets[0]

    def e2e_timed(fn, n):
        torch.cuda.synchronize(dev)
        barrier()
        t0 = time.perf_counter()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        fn(n)
        f1.record(stream)
        torch.cuda.synchronize(dev)
        ms = max(f0.elapsed_time(f1), (time.perf_counter() - t0) * 1e3)   # the host wait counts too
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def run_async(n):
        for i in range(n):
            hq, hk, hv, ho = host_sets[i & 1]
            b2a.attentionDecodeAsync(ctx, cache, rope, 0, hq, hk, hv, ho, H, numLayers=LAYERS)
        ctx.synchronize()

    def run_sync(n):
        for _ in range(n):
            b2a.attentionDecode(ctx, cache, rope, 0, qh, knh, vnh, outh, H, numLayers=LAYERS)

    run_async(max(2, min(args.warmup, 5)))
    e2e_ms = e2e_timed(run_async, e2e_steps)
    run_sync(max(1, min(args.warmup, 5)))
    e2e_sync_ms = e2e_timed(run_sync, e2e_steps)
    e2e_value = world * nb["step"] * e2e_steps / (e2e_ms / 1e3) / 1e9
    e2e_sync_value = world * nb["step"] * e2e_steps / (e2e_sync_ms / 1e3) / 1e9
    link = host_link_gbs(torch, stream, dev, nb["q"] + nb["kv_new"], nb["out"])

    # parity of the measured step (outside the timed regions): the device call's
    # output and the host-pointer call's, on 16 sampled rows
    step()
    torch.cuda.synchronize(dev)
    rng = np.random.default_rng(5)
    picks = [(int(np.argmax(lengths)), 0), (int(np.argmax(lengths)), LAYERS - 1), (int(np.argmin(lengths)), 0)]
    picks += [(int(rng.integers(SEQS)), int(rng.integers(LAYERS))) for _ in range(13)]
    parity = {"config3": parity_decode(torch, dev, kp, vp, shape, q, out, lengths, picks),
              "config3_e2e": parity_decode(torch, dev, kp, vp, shape, q, outh.to(dev), lengths, picks[:4]),
              "config3_e2e_async": parity_decode(torch, dev, kp, vp, shape, q, host_sets[1][3].to(dev), lengths,
                                                 picks[:4])}

    pk = peaks()
    # one launch of the attention kernel per step: its average launch time over
    # the timed region is the step time (CUDA events on the launching stream)
    launch_ms = ms / args.steps
    achieved = nb["attention_kernel"] / (launch_ms / 1e3) / 1e9
    traffic = ncu_traffic(attn_name, workload_name())
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config3_block(world),
        "roofline": {"bound": "hbm", "kernel": attn_name, "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "peak_source": pk["source"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": nb["attention_kernel"],
                     "launch_ms": round(launch_ms, 4),
                     "launch_ms_bracketed": round(attn_ms, 4),
                     "note": ("launch_ms: the timed region over its K launches (one per step); "
                              "launch_ms_bracketed: a separate pass with events around each launch, which "
                              "also stops the next launch's prologue from overlapping this one's tail")},
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": nb["q"] + nb["kv_new"],
                "d2h_bytes_per_step": nb["out"], "ms_per_step": round(e2e_ms / e2e_steps, 4),
                "frac_of_value": round(e2e_value / value, 4),
                "path": ("b2a_attention_decode_host_async: pinned host inputs copied in and f32 outputs copied back "
                         "every step, steps enqueued back to back, one synchronisation at the end of the timed region"),
                "sync_per_call": {"value": round(e2e_sync_value, 1), "unit": "GB/s",
                                  "ms_per_step": round(e2e_sync_ms / e2e_steps, 4),
                                  "path": "b2a_attention_decode with B2A_HOST pointers: each call returns with its results"},
                "host_link": link},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "kernels": {k: {"launches": v[0], "avg_ms": round(v[1] / v[0], 4)} for k, v in kt.items()},
    }
    if clocks:
        line["clocks"] = clocks.summary(t_wall0, t_wall1)

    if world == 1 and not args.no_paged:
        line["paged"] = bench_paged(torch, b2a, ctx, stream, dev, rope, lengths, nb, q, kn, vn, out, ms_max / args.steps,
                                    args)
    if not args.no_splitkv:
        line["split_kv"] = bench_splitkv(torch, dist, b2a, ctx, stream, dev, rank, world, args)
        # the same with 24 layers per step (one launch per rank), so that a GPU's
        # share of the stream outweighs the exchange's fixed latency
        line["split_kv_24"] = bench_splitkv(torch, dist, b2a, ctx, stream, dev, rank, world, args, layers=24)
    if world == 1 and not args.no_prefill:
        line["prefill"] = bench_prefill(torch, b2a, ctx, stream, dev, pk, args)
    if world == 1 and not args.no_layer:
        line["layer"] = bench_layer(torch, b2a, ctx, stream, dev, args)
    if world == 1 and not args.no_generation:
        line["generation"] = bench_generation(torch, b2a, ctx, stream, dev, pk["hbm_gbs"], args)
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, used, sample = cpu_decode_sample(lengths, target_s=args.cpu_seconds)
        # the reference itself is single-threaded JavaScript: the same restatement on one thread beside it
        gbs1, _, sample1 = cpu_decode_sample(lengths, target_s=args.cpu_seconds / 2, threads=1)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": "port",
                                "sample": sample,
                                "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                                  "sample": sample1}}
    line["parity"] = parity
    for key in ("split_kv", "split_kv_24", "prefill"):   # their own parity samples, gathered in one place
        if isinstance(line.get(key), dict) and "parity" in line[key]:
            parity[key] = line[key]["parity"]
    # the bulky objects first and the compact summaries last, so a reader of the
    # line's tail sees parity, split-KV and prefill
    for key in ("kernels", "layer", "generation", "paged", "parity", "split_kv", "split_kv_24", "prefill"):
        if key in line:
            line[key] = line.pop(key)
    barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    cache.close()
    rope.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def host_link_gbs(torch, stream, dev, h2d_bytes: int, d2h_bytes: int, reps: int = 20) -> dict:
    """The host link alone: pinned-host <-> device copies of one step's input and output
    sizes, each direction by itself and both at once (two streams), CUDA-event timed."""
    hin = torch.empty(h2d_bytes, dtype=torch.uint8).pin_memory()
    hout = torch.empty(d2h_bytes, dtype=torch.uint8).pin_memory()
    din = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    dout = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    other = torch.cuda.Stream(device=dev)

    def timed(fn):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    def both():
        other.wait_stream(stream)
        with torch.cuda.stream(other):
            hout.copy_(dout, non_blocking=True)
        with torch.cuda.stream(stream):
            din.copy_(hin, non_blocking=True)
        stream.wait_stream(other)

    with torch.cuda.stream(stream):
        t_in = timed(lambda: din.copy_(hin, non_blocking=True))
        t_out = timed(lambda: hout.copy_(dout, non_blocking=True))
        t_both = timed(both)
    return {"h2d_gbs": round(h2d_bytes / (t_in / 1e3) / 1e9, 1), "d2h_gbs": round(d2h_bytes / (t_out / 1e3) / 1e9, 1),
            "both_ms": round(t_both, 4), "h2d_ms": round(t_in, 4), "d2h_ms": round(t_out, 4)}


def bench_paged(torch, b2a, ctx, stream, dev, rope, lengths, nb, q, kn, vn, out, contiguous_ms, args,
                page_size: int = 256) -> dict:
    """The config-3 decode step over a paged cache (b2a_kvcache_create_paged): the same 64
    sequences, lengths and inputs, the pool sized for the positions they hold. Pages are
    mapped in rounds of one page per sequence, so each sequence's pages are spread over
    the pool as they would be after interleaved growth."""
    pages = int(sum(-(-(int(L) + 1) // page_size) for L in lengths))
    with torch.cuda.stream(stream):
        pc = b2a.GpuKVCache(ctx, b2a.CacheConfig(LAYERS, KVH, D, H), CAP, batch=SEQS, dtype="f16",
                            pageSize=page_size, numPages=pages)
        kp, vp, _ = pc.pools()
        shape = ((pages + 1) * LAYERS * KVH * page_size, D)
        gen = torch.Generator(device=dev)
        gen.manual_seed(99)
        torch.as_tensor(_CAI(kp, shape, "<f2"), device=dev).normal_(generator=gen)
        torch.as_tensor(_CAI(vp, shape, "<f2"), device=dev).normal_(generator=gen)
    torch.cuda.synchronize(dev)
    target = np.asarray(lengths, np.int64) + 1   # the new token's slot too
    r = 1
    while True:
        pc.setLengths(np.minimum(target, r * page_size).astype(np.int32))
        if r * page_size >= target.max():
            break
        r += 1
    pc.setLengths(np.asarray(lengths, np.int32))
    assert pc.freePages == 0

    def step():
        b2a.attentionDecode(ctx, pc, rope, 0, q, kn, vn, out, H, numLayers=LAYERS)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(3, min(args.steps, 500))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    ctx.enable_timing(True)
    for _ in range(10):
        step()
    kt = ctx.read_timing()
    ctx.enable_timing(False)
    pool_bytes = pc.byteLength
    contiguous_bytes = 2 * SEQS * LAYERS * KVH * CAP * D * 2
    res = {"page_size": page_size, "pages": pages, "value": round(nb["step"] / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
           "ms_per_step": round(ms, 4), "contiguous_ms_per_step": round(contiguous_ms, 4),
           "pool_bytes": pool_bytes, "contiguous_cache_bytes": contiguous_bytes,
           "kernels": {k: {"launches": v[0], "avg_ms": round(v[1] / v[0], 4)} for k, v in kt.items()}}
    pc.close()
    return res


def bench_splitkv(torch, dist, b2a, ctx, stream, dev, rank, world, args, layers: int = 1) -> dict:
    """8 sequences with a 32768-position f16 cache and one new
    token each, the KV positions split across the ranks (layers > 1: that many
    layers per step, all in one launch per rank). One GPU: the plain decode call.
    Several: the exchange inside the attention kernel (peer stores over NVLink),
    with the NCCL all-gather path (partials kernel, all-gather, combine) beside it."""
    from b2a import dist as bd
    nseq, total = 8, 32768
    lo, hi = bd.position_slice(total, world, rank)
    n_local = hi - lo
    with torch.cuda.stream(stream):
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(layers, KVH, D, H), n_local + 1, batch=nseq, dtype="f16")
        rope = b2a.RopeTable(ctx, D, THETA, total + 1)
        kp, vp, _ = cache.pools()
        gen = torch.Generator(device=dev)
        gen.manual_seed(777 + rank)
        shape = (nseq, layers, KVH, n_local + 1, D)
        torch.as_tensor(_CAI(kp, shape, "<f2"), device=dev).normal_(generator=gen)
        torch.as_tensor(_CAI(vp, shape, "<f2"), device=dev).normal_(generator=gen)
        cache.setLengths([n_local] * nseq)
        g2 = torch.Generator(device=dev)
        g2.manual_seed(4242)   # the same query and new token on every rank
        q = torch.randn(nseq, layers, H, D, device=dev, generator=g2).half()
        kn = torch.randn(nseq, layers, KVH, D, device=dev, generator=g2).half()
        vn = torch.randn(nseq, layers, KVH, D, device=dev, generator=g2).half()
        pos = torch.full((nseq,), total, dtype=torch.int32, device=dev)
        local = torch.empty(nseq, layers, H, D + 4, device=dev)
        out = torch.empty(nseq, layers, H, D, device=dev)
    def timed(step_fn, n):
        """Device time of n back-to-back steps (max over ranks)."""
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):   # graph replays launch on the current stream
            e0.record(stream)
            for _ in range(n):
                step_fn()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    steps = max(10, min(args.steps, 300))
    extra = {}
    peer, peer_error = None, None
    if world > 1:
        try:
            peer = bd.PeerSplitKV(ctx, cache, rope, 0, H, rank, world, num_layers=layers)
        except RuntimeError as e:   # raised on every rank alike
            peer_error = str(e)[:200]
    if peer is not None:
        # the in-kernel exchange (peer stores + flags over NVLink), one launch
        # per step, replayed from a CUDA graph so the host adds nothing per step
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                peer.step(q, kn, vn, pos, out)
            ctx.enable_timing(True)
            for _ in range(10):
                peer.step(q, kn, vn, pos, out)
            kt = ctx.read_timing()
            ctx.enable_timing(False)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            peer.step(q, kn, vn, pos, out)
        ms = timed(graph.replay, steps)
        # the NCCL all-gather baseline (partials kernel, all-gather, combine kernel)
        nccl = bd.cuda_split_kv(ctx, cache, rope, 0, H, rank, world, num_layers=layers)
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                nccl.step(q, kn, vn, pos, local, out)
        ms_nccl = timed(lambda: nccl.step(q, kn, vn, pos, local, out), steps)
        extra = {"nccl_baseline": {"ms_per_step": round(ms_nccl / steps, 4),
                                   "path": "partials kernel + NCCL all_gather + combine kernel, eager"}}
        del graph
        peer.close()
    elif world > 1:
        # no peer mapping: the NCCL path is the measured one
        nccl = bd.cuda_split_kv(ctx, cache, rope, 0, H, rank, world, num_layers=layers)
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                nccl.step(q, kn, vn, pos, local, out)
            ctx.enable_timing(True)
            for _ in range(10):
                nccl.step(q, kn, vn, pos, local, out)
            kt = ctx.read_timing()
            ctx.enable_timing(False)
        ms = timed(lambda: nccl.step(q, kn, vn, pos, local, out), steps)
        extra = {"peer_error": peer_error}
    else:
        # one GPU holds the whole context: the plain decode call, whose kernel
        # splits the positions over the CTAs and merges the chunks itself
        def one():
            b2a.attentionDecode(ctx, cache, rope, 0, q, kn, vn, out, H, numLayers=layers)
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                one()
            ctx.enable_timing(True)
            for _ in range(10):
                one()
            kt = ctx.read_timing()
            ctx.enable_timing(False)
            ms = timed(one, steps)
        picks = [(b, (5 * b) % layers) for b in range(nseq)]
        extra = {"parity": parity_decode(torch, dev, kp, vp, shape, q, out, [total] * nseq, picks)}
    kv_bytes = nseq * layers * KVH * (total + 1) * D * 2 * 2
    cache.close()
    rope.close()
    gbs = kv_bytes * steps / (ms / 1e3) / 1e9   # the whole context's bytes over the max-over-ranks time
    return {"metric": "split-KV decode GB/s", "value": round(gbs, 1),
            "unit": "GB/s", "ms_per_step": round(ms / steps, 4), "steps": steps,
            "hbm_frac_per_gpu": round(gbs / world / peaks()["hbm_gbs"], 4), **extra,
            "kernels": {k: {"launches": v[0], "avg_ms": round(v[1] / v[0], 4)} for k, v in kt.items()},
            "config": {"workload": "config5-split-kv-decode" + (f"-{layers}-layers" if layers > 1 else ""),
                       "sequences": nseq, "kv_len": total,
                       "cache_dtype": "f16", "layers": layers, "kv_bytes_per_step": kv_bytes,
                       "parallelism": f"context-parallel over {world} GPU(s)",
                       "collective": ("in-kernel exchange: peer stores of (o, m, l) partials + flags over NVLink, "
                                      "LSE combine in rank order (CUDA graph replay)" if peer is not None else
                                      "NCCL all_gather of (o, m, l) partials, then LSE combine in rank order")
                       if world > 1 else "none (b2a_attention_decode: chunks merged inside the kernel)"}}


def bench_layer(torch, b2a, ctx, stream, dev, args) -> dict:
    """The attention block's neighbours: one decode step of one Qwen2.5 layer's
    attention block through the library - fused int8 q/k/v projection (bias, f16 row scales),
    RoPE + append + attention over the cache, int8 o_proj with the residual add - replayed from a
    CUDA graph. Two shapes: BASELINE config 4 (one sequence, ~128 cached positions, the
    generation loop's per-layer step) and config 3 (64 sequences, lengths U{256..4096})."""
    hidden, rows = H * D, H * D + 2 * KVH * D
    g = torch.Generator(device=dev)
    g.manual_seed(31)

    def codes(r, c):
        return torch.randint(-127, 128, (r, c), generator=g, device=dev, dtype=torch.int8)

    with torch.cuda.stream(stream):
        wqkv, wo = codes(rows, hidden), codes(hidden, hidden)
        sqkv = (torch.rand(rows, generator=g, device=dev) * 1e-3).half()
        so = (torch.rand(hidden, generator=g, device=dev) * 1e-3).half()
        bias = torch.randn(rows, generator=g, device=dev) * 0.1
    res = {"metric": "attention-block decode step", "unit": "us/layer", "weights": "int8 per-row, f16 scales",
           "kernels_per_layer": 3, "shapes": {}}
    weight_bytes = rows * hidden + hidden * hidden
    for name, batch, lens in (("config4-generation", 1, [128]),
                              ("config3-batch64", SEQS, [int(x) for x in config3_lengths(0)])):
        with torch.cuda.stream(stream):
            cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), max(lens) + 1, batch=batch, dtype="f16")
            rope = b2a.RopeTable(ctx, D, THETA, max(lens) + 1)
            cache.setLengths(lens)
            x = torch.randn(batch, hidden, generator=g, device=dev)
            q = torch.empty(batch, H * D, device=dev, dtype=torch.float16)
            kn = torch.empty(batch, KVH * D, device=dev, dtype=torch.float16)
            vn = torch.empty(batch, KVH * D, device=dev, dtype=torch.float16)
            att = torch.empty(batch, H * D, device=dev)
            xo = torch.empty(batch, hidden, device=dev)

            def step():
                b2a.qkvInt8(ctx, wqkv, sqkv, bias, x, q, kn, vn, hidden, H * D, KVH * D, batch)
                b2a.attentionDecode(ctx, cache, rope, 0, q.view(batch, 1, H, D), kn.view(batch, 1, KVH, D),
                                    vn.view(batch, 1, KVH, D), att.view(batch, 1, H, D), H)
                b2a.linearInt8(ctx, wo, so, None, att, xo, hidden, hidden, batch, residual=x)
            for _ in range(5):
                step()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        n = 200
        with torch.cuda.stream(stream):
            for _ in range(5):
                graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / n * 1e3
        # per-kernel device times from eager steps with the library's event timing
        with torch.cuda.stream(stream):
            ctx.enable_timing(True)
            for _ in range(20):
                step()
            kt = ctx.read_timing()
            ctx.enable_timing(False)
        kv_bytes = sum(lens) * KVH * D * 2 * 2
        res["shapes"][name] = {"batch": batch, "kv_positions": int(sum(lens)), "us_per_layer": round(us, 2),
                               "bytes_per_layer": int(weight_bytes + kv_bytes),
                               "gb_s": round((weight_bytes + kv_bytes) / (us * 1e-6) / 1e9, 1),
                               "kernels_us": {k: round(v[1] / v[0] * 1e3, 2) for k, v in kt.items()}}
        del graph
        cache.close()
        rope.close()
    return res


def bench_generation(torch, b2a, ctx, stream, dev, peak_gbs, args) -> dict:
    """Qwen2.5-0.5B-architecture greedy generation with random-init
    N(0, 0.02) weights quantized to int8 per output row (f16 scales; norm gains 1, biases 0),
    a 64-token seeded prompt, then 128 greedy tokens, through the public generate call (host
    prompt in, host tokens out). The prompt runs the per-layer kernels (tensor-core attention);
    every decode token is one cooperative kernel over all 24 layers, the output projection and
    the pick. Roofline: the bytes a decode token must read (every weight byte once, plus the
    cached keys/values) over its device time, against the measured HBM copy bandwidth."""
    cfg = b2a.ModelConfig.qwen25_05b()
    Hd, I, V, L = cfg.hiddenSize, cfg.intermediateSize, cfg.vocabSize, cfg.numLayers
    Q = Hd + 2 * cfg.kvDim
    n_prompt, n_new = 64, args.gen_new_tokens
    g = torch.Generator(device=dev)
    g.manual_seed(44)

    def quant(rows, cols):
        # quantizeInt8PerChannel's rule (src/core/quantize.js:36-58) on the device
        w = torch.randn(rows, cols, generator=g, device=dev) * 0.02
        scale = (w.abs().amax(dim=1) / 127.0).half()
        s32 = scale.float().clamp_min(1e-30)[:, None]
        lv = w / s32
        codes = (lv.sign() * (lv.abs() + 0.5).floor()).clamp(-127, 127).to(torch.int8)
        return codes.contiguous(), scale.contiguous()

    model = b2a.Model(ctx, cfg, n_prompt + n_new, scale_dtype="f16")
    with torch.cuda.stream(stream):
        ones = torch.ones(Hd, device=dev)
        host = {"layers": []}
        for layer in range(L):
            qkv, sqkv = quant(Q, Hd)
            o, so = quant(Hd, Hd)
            gate, sg = quant(I, Hd)
            up, su = quant(I, Hd)
            down, sd = quant(Hd, I)
            w = dict(input_norm=ones, post_attn_norm=ones, qkv=qkv, qkv_scales=sqkv,
                     qkv_bias=torch.zeros(Q, device=dev), o=o, o_scales=so, gate=gate, gate_scales=sg,
                     up=up, up_scales=su, down=down, down_scales=sd)
            torch.cuda.synchronize(dev)
            model.load_layer(layer, w)
            if not args.no_cpu:
                host["layers"].append({k: (v.float().cpu().numpy() if k.endswith("scales") else v.cpu().numpy())
                                       for k, v in w.items()})
        emb, semb = quant(V, Hd)
        torch.cuda.synchronize(dev)
        model.load_embedding(emb, semb)
        model.load_final_norm(ones)
        if not args.no_cpu:
            host["embedding"] = (emb.cpu().numpy(), semb.float().cpu().numpy())
            host["final_norm"] = ones.cpu().numpy()
        del emb
    prompt = np.random.default_rng(4).integers(0, V, n_prompt).astype(np.int32).tolist()
    for _ in range(2):
        model.generate_all(prompt, n_new)
    reps = args.gen_reps
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    walls = []
    for _ in range(reps):
        t0 = time.perf_counter()
        if _ == reps - 1:
            e0.record(stream)
        toks, best = model.generate_all(prompt, n_new)
        if _ == reps - 1:
            e1.record(stream)
        walls.append(time.perf_counter() - t0)
    torch.cuda.synchronize(dev)
    dev_ms = e0.elapsed_time(e1)
    wall = float(np.median(walls))
    # per-kernel device time of one more run
    ctx.enable_timing(True)
    model.generate_all(prompt, n_new)
    kt = ctx.read_timing()
    ctx.enable_timing(False)
    step = kt.get("decode_step", (0, 0.0))
    step_us = step[1] / max(1, step[0]) * 1e3
    prefill_ms = sum(v[1] for k, v in kt.items() if k != "decode_step")
    weight_bytes = L * (Q * Hd + Hd * Hd + 2 * I * Hd + Hd * I) + V * Hd
    scale_bytes = 2 * (L * (Q + Hd + 2 * I + Hd) + V)
    mean_ctx = n_prompt + (n_new - 1) / 2.0
    kv_bytes = L * 2 * cfg.numKVHeads * mean_ctx * D * 2
    token_bytes = weight_bytes + scale_bytes + kv_bytes
    achieved = token_bytes / (step_us * 1e-6) / 1e9 if step_us > 0 else None
    res = {
        "metric": "config 4 greedy generation", "unit": "tokens/s",
        "value": round(n_new / wall, 1),
        "device_tokens_per_s": round(n_new / (dev_ms / 1e3), 1),
        "config": {"model": "Qwen2.5-0.5B architecture, random-init N(0,0.02)", "layers": L, "hidden": Hd,
                   "intermediate": I, "vocab": V, "weights": "int8 per output row, f16 scales",
                   "prompt": n_prompt, "new_tokens": n_new, "batch": 1, "data": "synthetic"},
        "e2e": {"value": round(n_new / wall, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * n_prompt,
                "d2h_bytes_per_step": 8 * n_new},
        "prefill_ms": round(prefill_ms, 3),
        "decode_us_per_token": round(step_us, 2),
        "decode_path": model.decode_path,
        "roofline": {"bound": "hbm", "kernel": "decode_step", "achieved": round(achieved, 1) if achieved else None,
                     "peak": peak_gbs, "unit": "GB/s", "frac": round(achieved / peak_gbs, 3) if achieved else None,
                     "traffic": ncu_traffic("decode_step", "config4-generation-ctx64"),
                     "traffic_note": "one launch at context 64 (ncu)", "bytes_per_token": int(token_bytes)},
        "kernels_ms": {k: round(v[1], 3) for k, v in kt.items()},
        "gpu_launches_per_generation": int(sum(v[0] for v in kt.values())),
        "tokens_head": [int(t) for t in toks[:8]],
    }
    model.decode_path = "layered"
    t0 = time.perf_counter()
    model.generate_all(prompt, n_new)
    res["layered_tokens_per_s"] = round(n_new / (time.perf_counter() - t0), 1)
    model.close()
    if not args.no_cpu:
        res["cpu_baseline"] = cpu_generation_sample(host, cfg, prompt, min(args.cpu_seconds, 20.0))
    return res


def cpu_generation_sample(host: dict, cfg, prompt, target_s: float) -> dict:
    """The oracle's ReferenceModel restatement (C, f64 reductions, int8 weights widened per
    element) on the host cores: a short prompt, then decode tokens until target_s passes;
    tokens/s of the decode tokens."""
    import os as _os
    from oracle import oracle as o
    threads = _os.cpu_count() or 1
    om = o.OracleModel(host, cfg.hiddenSize, cfg.intermediateSize, cfg.numLayers, cfg.numHeads, cfg.numKVHeads,
                       cfg.vocabSize, cfg.ropeTheta, cfg.rmsNormEps, 256, threads)
    _, nxt = om.forward(prompt[:4])
    n, t0 = 0, time.perf_counter()
    while n < 64 and (n < 2 or time.perf_counter() - t0 < target_s):
        _, nxt = om.forward([nxt])
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"4-token prompt, then {n} greedy decode tokens of the full config-4 model"}


def bench_prefill(torch, b2a, ctx, stream, dev, pk, args) -> dict:
    """causal prefill, bf16 Q/K/V, RoPE at 0..S-1, fused append, bf16 out."""
    res = {"metric": "prefill-attn TFLOPS", "unit": "TFLOPS", "dtype": "bf16", "sweep": {}}
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)   # > L2, rewritten between steps
    for S in args.prefill_seqs:
        with torch.cuda.stream(stream):
            cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), S, batch=1, dtype=args.prefill_cache)
            rope = b2a.RopeTable(ctx, D, THETA, S)
            q = torch.randn(S, H, D, device=dev).bfloat16()
            k = torch.randn(S, KVH, D, device=dev).bfloat16()
            v = torch.randn(S, KVH, D, device=dev).bfloat16()
            o = torch.empty(S, H, D, device=dev, dtype=torch.bfloat16)
        flops = 4 * D * H * S * (S + 1) / 2
        steps = max(3, min(50, int(2e9 / max(flops, 1))))
        for _ in range(3):
            b2a.attentionPrefill(ctx, cache, rope, 0, q, k, v, o, S, H)
        # call time: steps enqueued back to back (L2 flush, event, call, event) and
        # synchronised once, so the host's per-call overhead overlaps the previous
        # step's device work instead of idling the GPU inside the timed bracket
        evs = []
        for _ in range(steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            b2a.attentionPrefill(ctx, cache, rope, 0, q, k, v, o, S, H)
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize(dev)
        total = sum(a.elapsed_time(b) for a, b in evs)
        # per-kernel times: a second pass with the library's event timing on
        ctx.enable_timing(True)
        for _ in range(steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            b2a.attentionPrefill(ctx, cache, rope, 0, q, k, v, o, S, H)
        torch.cuda.synchronize(dev)
        kt = ctx.read_timing()
        ctx.enable_timing(False)
        attn = next((k for k in ("prefill_pair", "prefill_tc", "attention_simt") if k in kt), None)
        kms = kt[attn][1] / kt[attn][0] if attn else None
        res["sweep"][str(S)] = {"ms": round(total / steps, 4), "tflops": round(flops / (total / steps / 1e3) / 1e12, 3),
                                "kernel": attn, "kernel_ms": round(kms, 4) if kms else None,
                                "kernel_tflops": round(flops / (kms / 1e3) / 1e12, 3) if kms else None,
                                "launches_per_step": sum(x[0] for x in kt.values()) / steps}
        if S == 512 or S == max(args.prefill_seqs):
            # the measured call's output: query rows of the first, middle and last tiles
            rows = sorted({0, 1, min(S - 1, 127), S // 2, max(0, S - 128), S - 1})
            res.setdefault("parity", {})[str(S)] = parity_prefill(torch, dev, q, k, v, o, rows)
        cache.close()
        rope.close()
    # many short prompts at once (b2a_attention_prefill_batch): config 2's S=512 for 32
    # sequences in one call, the way a server fills the GPU with short prefills
    nseq, S = 32, 512
    with torch.cuda.stream(stream):
        cache = b2a.GpuKVCache(ctx, b2a.CacheConfig(1, KVH, D, H), S, batch=nseq, dtype=args.prefill_cache)
        rope = b2a.RopeTable(ctx, D, THETA, S)
        q = torch.randn(nseq, S, H, D, device=dev).bfloat16()
        k = torch.randn(nseq, S, KVH, D, device=dev).bfloat16()
        v = torch.randn(nseq, S, KVH, D, device=dev).bfloat16()
        o = torch.empty(nseq, S, H, D, device=dev, dtype=torch.bfloat16)
    flops = nseq * 4 * D * H * S * (S + 1) / 2
    for _ in range(3):
        b2a.attentionPrefillBatch(ctx, cache, rope, 0, q, k, v, o, S, H, 0, nseq)
    evs = []
    for _ in range(20):
        with torch.cuda.stream(stream):
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        b2a.attentionPrefillBatch(ctx, cache, rope, 0, q, k, v, o, S, H, 0, nseq)
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize(dev)
    ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
    res["batched"] = {"sequences": nseq, "seq": S, "ms": round(ms, 4),
                      "tflops": round(flops / (ms / 1e3) / 1e12, 3),
                      "frac": round(flops / (ms / 1e3) / 1e12 / pk["bf16_tflops"], 4),
                      "call": "b2a_attention_prefill_batch (one append launch, one attention launch)"}
    cache.close()
    rope.close()
    main = res["sweep"].get("512") or next(iter(res["sweep"].values()))
    res["value"] = main["tflops"]
    res["config"] = {"workload": "config2-causal-prefill", "seq": 512, "heads": "14q/2kv", "head_dim": D,
                     "qkv_dtype": "bf16", "out_dtype": "bf16", "cache_dtype": args.prefill_cache,
                     "flops": "4*D*H*S(S+1)/2", "l2": "flushed (256 MiB write) between timed steps"}
    best_s = max(res["sweep"], key=lambda s: res["sweep"][s]["kernel_tflops"] or 0)
    bk = res["sweep"][best_s]
    if bk["kernel_tflops"]:
        res["roofline"] = {"bound": "tensor", "kernel": bk["kernel"], "seq": int(best_s),
                           "achieved": bk["kernel_tflops"], "peak": pk["bf16_tflops"], "peak_source": pk["source"],
                           "unit": "TFLOP/s", "frac": round(bk["kernel_tflops"] / pk["bf16_tflops"], 4),
                           "traffic": ncu_traffic(bk["kernel"], f"prefill{best_s}")}
        # scalar copies of the headline figures (for readers that keep only scalars)
        res["roofline_seq"] = int(best_s)
        res["roofline_tflops"] = bk["kernel_tflops"]
        res["roofline_frac"] = res["roofline"]["frac"]
    for S_ in ("2048", "16384"):
        if S_ in res["sweep"] and res["sweep"][S_]["kernel_tflops"]:
            res[f"s{S_}_kernel_tflops"] = res["sweep"][S_]["kernel_tflops"]
            res[f"s{S_}_frac"] = round(res["sweep"][S_]["kernel_tflops"] / pk["bf16_tflops"], 4)
    res["batched_tflops"] = res["batched"]["tflops"]
    res["batched_frac"] = res["batched"]["frac"]
    # the bulky sweep before the summaries
    for key in ("sweep", "batched", "config", "parity", "roofline"):
        if key in res:
            res[key] = res.pop(key)
    return res


# -------------------------------------------------------------- reference ---

def run_reference(args) -> None:
    """The reference's CPU attention path (restated in C: no JS runtime exists here),
    all host threads, rank 0 only, same metric and workload."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import oracle as o
    o.build()
    lengths = config3_lengths(0)
    # each step: a bounded sample of config 3 sized so the whole run ends in ~2 minutes
    budget = 120.0 / max(1, args.steps + args.warmup)
    rng = np.random.default_rng(99)
    cap = int(lengths.max()) + 1
    seq_stride = KVH * cap * D
    kb = rng.standard_normal(SEQS * seq_stride, dtype=np.float32).astype(np.float16).view(np.uint16)
    vb = rng.standard_normal(SEQS * seq_stride, dtype=np.float32).astype(np.float16).view(np.uint16)
    q = rng.standard_normal(SEQS * H * D, dtype=np.float32)
    per_seq = config3_bytes(lengths)["step"] / LAYERS / SEQS
    t0 = time.perf_counter()
    _, used = o.batched_decode_f16(q, H * D, kb, vb, seq_stride, lengths, SEQS, cap, H, KVH, D, H * D, 0)
    t_layer = time.perf_counter() - t0
    nseq = max(1, min(SEQS, int(SEQS * budget / max(t_layer, 1e-6))))
    sel = np.arange(nseq)
    sample_bytes = per_seq * nseq
    for _ in range(args.warmup):
        o.batched_decode_f16(q, H * D, kb, vb, seq_stride, lengths[sel], nseq, cap, H, KVH, D, H * D, 0)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        o.batched_decode_f16(q, H * D, kb, vb, seq_stride, lengths[sel], nseq, cap, H, KVH, D, H * D, 0)
    dt = time.perf_counter() - t0
    value = sample_bytes * args.steps / dt / 1e9
    sample = f"{nseq} of {SEQS} sequences x 1 layer of config 3 per step ({sample_bytes / 1e6:.1f} MB)"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config3_block(world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": used, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference is JavaScript (src/core/attention.js); no JS runtime exists on this machine, "
                 "so its CPU path runs as the C restatement in oracle/ with f64 accumulation, all host threads"),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    global SEQS, LAYERS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-splitkv", action="store_true")
    ap.add_argument("--no-paged", action="store_true", help="skip the config-3 decode over a paged cache")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-layer", action="store_true", help="skip the attention-block (projections) measurement")
    ap.add_argument("--no-generation", action="store_true", help="skip the config-4 generation measurement")
    ap.add_argument("--generation-only", action="store_true", help="only the config-4 generation measurement")
    ap.add_argument("--gen-new-tokens", type=int, default=128, help="greedy tokens per generation (config 4: 128)")
    ap.add_argument("--gen-reps", type=int, default=5, help="timed generations")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--prefill-seqs", type=int, nargs="+", default=[8, 64, 512, 2048, 8192, 16384])
    ap.add_argument("--prefill-cache", choices=["f16", "bf16"], default="f16",
                    help="KV cache dtype for the prefill sweep: bf16 inputs are exact in f16, and the f16 "
                         "tensor-core path needs no split products")
    ap.add_argument("--seqs", type=int, default=SEQS,
                    help="sequences per GPU (profiling of a smaller case; the headline is 64)")
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers per step (the headline is 24)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    SEQS, LAYERS = args.seqs, args.layers
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

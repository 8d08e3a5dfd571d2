#!/usr/bin/env python3
"""Benchmark of the gemma3.c attention hot path on B200.

Headline workload: batched decode, B=64
independent sequences, each with 32,768 cached positions (new token at
position 32768), all 34 layers (29 local: 1024-row window; 5 global: full
causal), BF16 KV cache ~N(0,1), sequences sharded across the GPUs (strong
scaling: 64/N per GPU, no collective on the data path).

One step = one decode token for every sequence through all 34 layers' attention
core (QK-norm, RoPE, cache append, GQA), i.e. 34 calls of
gemma3_cuda_attn_decode_dev per rank.  Metric: algorithmic KV bytes read per
second (50.73 GB/step at BF16) -- "decode HBM GB/s".  The reference arm
(--impl reference) runs the reference's own CPU attention (oracle/_ref,
compiled from gemma3.c's sources) on the same workload and is credited the
same algorithmic bytes per step, so the driver's ratio of the two values is
the ratio of step rates.

Secondary figures in the same JSON line (rank 0): the 34-layer T=8192 prefill
stack (configs[2], tensor-core prefill) and the B=1 global-layer decode at
8192 keys.

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Under torchrun (N>1) one process per GPU; timing is max over ranks.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gemma3.c_b200")
sys.path.insert(0, PKG)

N_LAYERS = 34
GLOBAL_LAYERS = [l for l in range(N_LAYERS) if (l + 1) % 6 == 0]
B_TOTAL = 64
CTX = 32768                      # cached positions per sequence
POS = CTX                        # position of the new token
ROW_BYTES_BF16 = 4 * 256 * 2 * 2  # K+V of one cache row, 4 kv heads, bf16
ROWS_PER_SEQ = len(GLOBAL_LAYERS) * (POS + 1) + (N_LAYERS - len(GLOBAL_LAYERS)) * 1024
BYTES_PER_SEQ_STEP = ROWS_PER_SEQ * ROW_BYTES_BF16   # 792.7 MB


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true", help="skip the configs[1]/[2] figures")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", choices=["decode", "prefill", "prefill_stack", "proj", "model_decode"],
                    help="tiny workload for ncu captures: 3 launches of the kernel, ~1-2 GB on the device")
    ap.add_argument("--seqs", type=int, default=B_TOTAL,
                    help="override the 64 sequences (small cases for ncu captures only)")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class Clocks:
    """Clock / throttle-reason sampler for the GPU this rank uses, during the
    timed region: NVML read every 10 ms from a thread (a timed region of
    tens of ms then still yields several samples), else nvidia-smi every
    200 ms.  Reads only; no GPU setting is changed."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    REASON_BITS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
                   ("hw_thermal_slowdown", 0x40))

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.f = None
        self.p = None
        self.nv = None
        self.rows = []

    def _nvml_loop(self):
        nv, h = self.nv, self.h
        while not self.stop.is_set():
            try:
                self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                  nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM),
                                  nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                break
            self.stop.wait(0.01)

    def __enter__(self):
        try:
            import threading
            import pynvml
            pynvml.nvmlInit()
            # the GPU of this CUDA ordinal, matched by UUID (NVML numbers every
            # GPU of the box, whatever CUDA_VISIBLE_DEVICES exposes)
            import torch
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.idx).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.stop = threading.Event()
            self.t = threading.Thread(target=self._nvml_loop, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nv = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.nv:
            self.stop.set()
            self.t.join()
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        if self.nv:
            rows = self.rows
            if not rows:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML returned no sample"], "samples": 0}
            reasons = {name for _, _, r in rows for name, bit in self.REASON_BITS if r & bit}
            return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                    "reasons": sorted(reasons), "samples": len(rows), "source": "NVML, 10 ms"}
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows), "source": "nvidia-smi, 200 ms"}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend):
        import torch
        if self.world > 1:
            import torch.distributed as dist
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group("gloo")
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x):
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# The reference's CPU path (oracle/_ref = gemma3.c's own C, blas-threads
# flags).  One "unit" = one sequence's decode token through all 34 layers'
# attention core (gemma3_transformer.c:294-352 minus the projections):
# rmsnorm per head, RoPE, cache_kv, gemma3_gqa over 32769 rows (global) or
# the 1024-row ring (local).  gemma3_gqa is single-threaded in every
# reference build, so the host's cores are used by running independent
# sequences on parallel threads (ctypes releases the GIL).
# ---------------------------------------------------------------------------
class CpuReference:
    """Per thread, one sequence's full set of caches as gemma3_kv_cache_alloc
    lays them out (gemma3_transformer.c:180-214): 29 local 1024-row rings and
    the global caches of 32,769 rows (5, or 1 shared by the 5 global layers
    when host memory is short; a 268 MB global cache is far larger than L3
    either way).  A thread runs its sequences one after another on its own
    caches, so no sequence-step finds another layer's cache in L3."""

    def __init__(self, threads, separate_globals=True):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracles import RefOracle  # the reference's own code
        import synth
        self.ref = RefOracle()
        self.kind = "reference"
        self.threads = threads
        max_seq = POS + 1
        self.rope_l = self.ref.rope_table(max_seq, 10000.0)
        self.rope_g = self.ref.rope_table(max_seq, 1000000.0)
        self.qn, self.kn = synth.qk_norm_gains(11)
        base_g = synth.normal(5, (CTX, 4, 256))
        base_l = synth.normal(6, (1024, 4, 256))
        g_bytes = 2 * max_seq * 4 * 256 * 4
        avail = os.sysconf("SC_AVPHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
        self.n_global = (len(GLOBAL_LAYERS) if separate_globals and threads * len(GLOBAL_LAYERS) * g_bytes < 0.6 * avail
                         else 1)
        self.caches = []
        for _ in range(threads):
            per = {}
            for i, layer in enumerate(range(N_LAYERS)):
                glob = layer in GLOBAL_LAYERS
                if glob and GLOBAL_LAYERS.index(layer) >= self.n_global:
                    per[layer] = per[GLOBAL_LAYERS[0]]
                    continue
                c = self.ref.new_cache(glob, max_seq)
                base = base_g if glob else base_l
                k, v = self.ref.cache_arrays(c)
                k[:base.shape[0]] = base
                v[:base.shape[0]] = base
                per[layer] = c
            self.caches.append(per)
        self.q = synth.normal(7, (1, 2048))
        self.k = synth.normal(8, (1, 1024))
        self.v = synth.normal(9, (1, 1024))

    def caches_note(self):
        return (f"per thread 29 local caches + {self.n_global} global cache(s) of 32769 rows"
                + ("" if self.n_global == len(GLOBAL_LAYERS) else " shared by the 5 global layers"))

    def unit(self, tid):
        per = self.caches[tid]
        for layer in range(N_LAYERS):
            glob = layer in GLOBAL_LAYERS
            self.ref.attn_core_tokens(per[layer], self.q, self.k, self.v, self.qn, self.kn,
                                      self.rope_g if glob else self.rope_l, POS)

    def run(self, units):
        """Runs `units` sequence-steps, thread t taking sequences t, t+th, ...
        on its own caches; returns seconds."""
        from concurrent.futures import ThreadPoolExecutor

        def worker(t):
            for _ in range(t, units, self.threads):
                self.unit(t)

        t0 = time.perf_counter()
        with ThreadPoolExecutor(self.threads) as ex:
            list(ex.map(worker, range(min(self.threads, units))))
        return time.perf_counter() - t0

    def close(self):
        seen = set()
        for per in self.caches:
            for c in per.values():
                if id(c) not in seen:
                    seen.add(id(c))
                    self.ref.free_cache(c)


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline_sample(target_s=12.0):
    """Times the reference on a bounded sample of the headline workload."""
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    th = cpu_threads()
    cpu = CpuReference(th, separate_globals=False)  # bounded set-up time inside the GPU bench
    cpu.run(th)  # warm
    units, secs = 0, 0.0
    while secs < target_s:
        secs += cpu.run(th)
        units += th
    note = cpu.caches_note()
    cpu.close()
    gbs = units * BYTES_PER_SEQ_STEP / secs / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": th, "kind": "reference",
            "sample": f"{units} sequence-steps (each: 34 layers, 5 x 32769-row global + 29 x 1024-row local "
                      f"gemma3_gqa, fp32 cache; {note}) on {th} threads, {secs:.1f} s; credited "
                      f"{BYTES_PER_SEQ_STEP / 1e6:.1f} MB (BF16 algorithmic bytes) per sequence-step"}


def run_reference_arm(args, dist):
    """--impl reference: the reference's CPU path on the same workload.  Every
    step runs all 64 sequence-steps (34 layers each) on the host's threads."""
    if dist.rank != 0:
        return None
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    th = cpu_threads()
    cpu = CpuReference(th)
    for _ in range(args.warmup):
        cpu.run(B_TOTAL)
    secs = [cpu.run(B_TOTAL) for _ in range(args.steps)]
    note = cpu.caches_note()
    cpu.close()
    t = sum(secs)
    gbs = args.steps * B_TOTAL * BYTES_PER_SEQ_STEP / t / 1e9
    step_ms = t / args.steps * 1e3
    return {
        "metric": "decode attention KV throughput, 34-layer Gemma-3-4B, B=64 @ 32768 ctx",
        "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) cache and q/k/v)",
        "config": {"workload": "configs[3] batched decode B=64, ctx 32768, 34 layers (5 global + 29 local)",
                   "batch": B_TOTAL, "context": CTX, "layers": N_LAYERS, "kv_cache": "fp32 (reference dtype)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": th, "kind": "reference",
                         "sample": f"every step: all {B_TOTAL} sequence-steps on {th} threads ({note}); "
                                   f"timed region {t:.1f} s"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def ev_time(torch, stream, fn):
    """Runs fn() between two CUDA events on `stream`; returns ms."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    fn()
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b)


def headline(args, dist, torch, gc, synth, pk):
    dev = dist.local
    N = dist.world
    assert B_TOTAL % N == 0, "64 sequences must split evenly over the GPUs"
    Bl = B_TOTAL // N
    ctx = gc.Context(max_context=POS + 1, max_batch=Bl, kv_dtype=gc.KV_BF16, device=dev, max_prefill=64)
    ctx.upload_rope(gc.rope_table(POS + 1, 10000.0), gc.rope_table(POS + 1, 1000000.0))
    for l in range(N_LAYERS):
        qn, kn = synth.qk_norm_gains(100 + l)
        ctx.set_qk_norm(l, qn, kn)
        rows = CTX if l in GLOBAL_LAYERS else 1024
        for s in range(Bl):
            ctx.fill_cache_random(l, s, rows, 1000 * (dist.rank * Bl + s) + l)
    ctx.synchronize()
    g = torch.Generator(device=f"cuda:{dev}").manual_seed(1234 + dist.rank)
    q = torch.randn(N_LAYERS, Bl, 2048, device=f"cuda:{dev}", generator=g)
    k = torch.randn(N_LAYERS, Bl, 1024, device=f"cuda:{dev}", generator=g)
    v = torch.randn(N_LAYERS, Bl, 1024, device=f"cuda:{dev}", generator=g)
    out = torch.empty(N_LAYERS, Bl, 2048, device=f"cuda:{dev}")
    seqs = list(range(Bl))
    pos = [POS] * Bl
    stream = torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{dev}")
    # The step calls gemma3_cuda_attn_decode_dev once per layer, as a C host
    # would: arguments converted once, outside the loop, so the Python
    # wrapper's per-call conversions do not starve the GPU on short layers.
    seq_a = np.arange(Bl, dtype=np.int32)
    pos_a = np.full(Bl, POS, dtype=np.int32)
    sp = seq_a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    pp = pos_a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    ptrs = [(q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), out[l].data_ptr()) for l in range(N_LAYERS)]
    fn, h = ctx.lib.gemma3_cuda_attn_decode_dev, ctx.h

    def step():
        for l in range(N_LAYERS):
            if fn(h, l, Bl, sp, pp, *ptrs[l]) != 0:
                raise RuntimeError(ctx.last_error())

    for _ in range(args.warmup):
        step()
    ctx.synchronize()
    # timed region: inputs (50.7 GB of cache) are far larger than L2
    dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = ctx.launch_count()
    with Clocks(dev) as clk:
        ms = ev_time(torch, stream, lambda: [step() for _ in range(args.steps)])
    ctx.synchronize()
    launches = ctx.launch_count() - launches0
    torch.cuda.synchronize(dev)
    dist.barrier()
    # kernel statistics (CUDA events around every split-KV launch) from a
    # separate pass, so the event records stay out of the timed region
    ctx.profile(True)
    for _ in range(2):
        step()
    ctx.synchronize()
    n_dec, dec_ms, dec_bytes = ctx.profile_read(0)
    ctx.profile(False)
    clocks = clk.summary()
    ms_max = dist.max(ms)
    total_bytes = args.steps * B_TOTAL * BYTES_PER_SEQ_STEP
    value = total_bytes / (ms_max / 1e3) / 1e9

    # e2e through the host-pointer C-ABI call: pinned host q/k/v in, out back
    qh = q.cpu().pin_memory().numpy()
    kh = k.cpu().pin_memory().numpy()
    vh = v.cpu().pin_memory().numpy()
    oh = torch.empty(N_LAYERS, Bl, 2048).pin_memory().numpy()

    # the host-pointer entry point called per layer as a C host calls it:
    # host pointers converted once, outside the timed loop
    fn_h = ctx.lib.gemma3_cuda_attn_decode
    hptrs = [tuple(a[l].ctypes.data_as(ctypes.POINTER(ctypes.c_float)) for a in (qh, kh, vh, oh))
             for l in range(N_LAYERS)]

    def step_e2e():
        for l in range(N_LAYERS):
            if fn_h(h, l, Bl, sp, pp, *hptrs[l]) != 0:
                raise RuntimeError(ctx.last_error())

    step_e2e()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step_e2e()
    e2e_s = dist.max(time.perf_counter() - t0)
    e2e = total_bytes / e2e_s / 1e9
    h2d = N_LAYERS * B_TOTAL * (2048 + 1024 + 1024) * 4
    d2h = N_LAYERS * B_TOTAL * 2048 * 4
    # correctness guard: outputs finite
    assert np.isfinite(oh).all()

    achieved = dec_bytes / (dec_ms / 1e3) / 1e9 if dec_ms > 0 else None
    res = {
        "value": value, "ms_per_step": ms_max / args.steps, "e2e": e2e, "h2d": h2d, "d2h": d2h,
        "gpu_launches": launches, "clocks": clocks,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"] if achieved else None,
                     "kernel": "decode_tc (BF16 cache, tcgen05)", "launches": n_dec,
                     "avg_launch_us": dec_ms / max(n_dec, 1) * 1e3,
                     "bytes_per_launch": dec_bytes / max(n_dec, 1)},
        "decode_kernel_share": dec_ms / ms if ms > 0 else None,
    }
    ctx.close()
    del q, k, v, out
    torch.cuda.empty_cache()
    return res


def secondary_prefill(args, torch, gc, pk, dev):
    """34-layer attention stack in prefill, B=1, T=8192."""
    T = 8192
    ctx = gc.Context(max_context=T, max_batch=1, kv_dtype=gc.KV_BF16, device=dev, max_prefill=T)
    ctx.upload_rope(gc.rope_table(T, 10000.0), gc.rope_table(T, 1000000.0))
    import synth
    for l in range(N_LAYERS):
        qn, kn = synth.qk_norm_gains(200 + l)
        ctx.set_qk_norm(l, qn, kn)
    g = torch.Generator(device=f"cuda:{dev}").manual_seed(99)
    q = torch.randn(N_LAYERS, T, 2048, device=f"cuda:{dev}", generator=g)
    k = torch.randn(N_LAYERS, T, 1024, device=f"cuda:{dev}", generator=g)
    v = torch.randn(N_LAYERS, T, 1024, device=f"cuda:{dev}", generator=g)
    out = torch.empty(T, 2048, device=f"cuda:{dev}")
    stream = torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{dev}")

    def step():
        for l in range(N_LAYERS):
            ctx.attn_prefill_dev(l, 0, q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), T, 0, out.data_ptr())

    for _ in range(max(1, args.warmup)):
        step()
    ctx.synchronize()
    steps = max(2, args.steps // 2)
    ctx.profile(True)
    ms = ev_time(torch, stream, lambda: [step() for _ in range(steps)])
    ctx.synchronize()
    n, kms, flops = ctx.profile_read(1)
    ctx.profile(False)
    ctx.close()
    del q, k, v
    torch.cuda.empty_cache()
    step_flops = flops / steps
    tf_step = step_flops / (ms / steps / 1e3) / 1e12
    tf_kernel = flops / (kms / 1e3) / 1e12
    return {"workload": "configs[2] 34-layer prefill stack, T=8192 (29 local + 5 global layers)",
            "tok_per_s": round(T * steps / (ms / 1e3), 1), "ms_per_step": round(ms / steps, 3),
            "algorithmic_tflop_per_step": round(step_flops / 1e12, 4),
            "tflops_step": round(tf_step, 1),
            "roofline": {"bound": "tensor", "kernel": "prefill_fa_sm100 (fp16 tcgen05, fp32 acc)",
                         "achieved": round(tf_kernel, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(tf_kernel / pk["bf16_tflops"], 4), "launches": n,
                         "avg_launch_us": round(kms / max(n, 1) * 1e3, 2)}}


def secondary_config0(args, torch, gc, pk, dev, with_cpu):
    """one local layer's attention core in prefill, B=1, T=512,
    positions 0..511, seed 0.  Q/K/V come from the projections of seeded
    N(0,1) activations through N(0,0.02) BF16 weights, computed on the host
    by the reference's own matvec (layer_attention through oracle/_ref), as
    the config prescribes; the timed region is the attention core (QK-norm,
    RoPE, cache append, GQA) on the GPU and, beside it, the reference's own
    CPU loop (gemma3_transformer.c:641-692 body, single-threaded as the
    reference runs it)."""
    import synth
    T, layer = 512, 0
    flops = 8.0 * 4 * 256 * (T * (T + 1) // 2)          # 1.076 GFLOP
    qn, kn = synth.qk_norm_gains(0)
    rope_l = gc.rope_table(1024, 10000.0)
    res = {"workload": "configs[0] one local layer prefill, T=512, positions 0..511, seed 0",
           "algorithmic_gflop": round(flops / 1e9, 4)}
    Q = K = V = None
    ref = None
    if with_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        try:
            from oracles import RefOracle
            ref = RefOracle()
        except Exception as e:  # reported, the GPU figure stays
            res["cpu_baseline"] = {"value": None, "error": f"{type(e).__name__}: {e}"}
    if ref is not None:
        x = synth.normal(0, (T, gc.HIDDEN))
        w = [synth.bf16_trunc(synth.normal(s_, shape, 0.02)) for s_, shape in
             ((1, (gc.Q_SIZE, gc.HIDDEN)), (2, (gc.KV_SIZE, gc.HIDDEN)), (3, (gc.KV_SIZE, gc.HIDDEN)),
              (4, (gc.HIDDEN, gc.Q_SIZE)))]
        c = ref.new_cache(False, 1024)
        rope_ref = ref.rope_table(1024, 10000.0)
        # the raw (pre-norm) projections layer_attention computes
        _, Q, K, V, _ = ref.layer_attention_tokens(c, x, *w, qn, kn, rope_ref, layer, 0)
        ref.free_cache(c)
    if Q is None:
        Q, K, V = synth.normal(10, (T, gc.Q_SIZE)), synth.normal(11, (T, gc.KV_SIZE)), synth.normal(12, (T, gc.KV_SIZE))
        res["inputs"] = "seeded N(0,1) q/k/v (reference projections unavailable)"
    else:
        res["inputs"] = "q/k/v = reference matvec projections of x~N(0,1) through W~N(0,0.02) (host)"
    # GPU: attention core through the C-ABI, device buffers (value) and host buffers (e2e)
    ctx = gc.Context(max_context=1024, max_batch=1, kv_dtype=gc.KV_F32, device=dev, max_prefill=T, num_layers=1)
    if ref is not None:
        rope_l = rope_ref  # the host's own table, as the integration uploads it
    ctx.upload_rope(rope_l, rope_l)
    ctx.set_qk_norm(layer, qn, kn)
    d = f"cuda:{dev}"
    q, k, v = (torch.from_numpy(np.ascontiguousarray(a)).to(d) for a in (Q, K, V))
    o = torch.empty(T, gc.Q_SIZE, device=d)
    stream = torch.cuda.ExternalStream(ctx.stream, device=d)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=d)
    call = lambda: ctx.attn_prefill_dev(layer, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), T, 0, o.data_ptr())
    for _ in range(5):
        call()
    ctx.synchronize()
    iters, tot = 50, 0.0
    ctx.profile(True)
    for _ in range(iters):
        with torch.cuda.stream(stream):
            flush.zero_()
        tot += ev_time(torch, stream, call)
    n, kms, _ = ctx.profile_read(1)
    ctx.profile(False)
    us = tot / iters * 1e3
    # pinned host buffers, as for the headline's e2e
    Qh, Kh, Vh = (torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).pin_memory().numpy()
                  for a in (Q, K, V))
    oh = torch.empty(T, gc.Q_SIZE).pin_memory().numpy()
    for _ in range(3):
        ctx.attn_prefill(layer, 0, Qh, Kh, Vh, 0, out=oh)
    t0 = time.perf_counter()
    reps = 50
    for _ in range(reps):
        ctx.attn_prefill(layer, 0, Qh, Kh, Vh, 0, out=oh)
    e2e_s = (time.perf_counter() - t0) / reps
    ctx.close()
    del flush
    res["gpu"] = {"us_per_call": round(us, 2), "tok_per_s": round(T / (us / 1e6), 1),
                  "kernel_us": round(kms / max(n, 1) * 1e3, 2) if n else None,
                  "e2e_us_per_call": round(e2e_s * 1e6, 2), "e2e_tok_per_s": round(T / e2e_s, 1),
                  "roofline": {"bound": "tensor", "achieved": round(flops / (us / 1e6) / 1e12, 2),
                               "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                               "frac": round(flops / (us / 1e6) / 1e12 / pk["bf16_tflops"], 4),
                               "note": "1.08 GFLOP: too small to fill 148 SMs; latency-bound"},
                  "api": "gemma3_cuda_attn_prefill_dev (value) / gemma3_cuda_attn_prefill host buffers (e2e)"}
    if ref is not None:
        c = ref.new_cache(False, 1024)
        ref.attn_core_tokens(c, Q, K, V, qn, kn, rope_ref, 0)  # warm
        runs, secs = 0, 0.0
        while secs < 2.0:
            ref.free_cache(c)
            c = ref.new_cache(False, 1024)
            t0 = time.perf_counter()
            ref.attn_core_tokens(c, Q, K, V, qn, kn, rope_ref, 0)
            secs += time.perf_counter() - t0
            runs += 1
        ref.free_cache(c)
        res["cpu_baseline"] = {"value": round(T * runs / secs, 1), "unit": "tok/s", "cores": 1, "kind": "reference",
                               "ms_per_call": round(secs / runs * 1e3, 2),
                               "sample": f"the whole T=512 layer, {runs} runs; gemma3_gqa and the token loop are "
                                         "single-threaded in the reference"}
    return res


def cpu_prefill_stack_sample(target_s=8.0):
    """Reference CPU baseline for configs[2] (34-layer prefill, T=8192),
    sampled: the whole stack is ~10 minutes of CPU.  Query tokens at evenly
    spaced positions of a local and of a global layer run through the
    reference's own per-token attention core (norm, RoPE, cache_kv,
    gemma3_gqa) over caches already holding the earlier positions; each
    host thread takes its own positions on its own cache.  The measured
    FLOP rate of each layer type, applied to that type's algorithmic FLOPs
    (29 x 7,864,832 and 5 x 33,558,528 (query, key) pairs x 8192 FLOP),
    gives the projected stack time."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracles import RefOracle
    from concurrent.futures import ThreadPoolExecutor
    import synth
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    ref = RefOracle()
    T = 8192
    th = cpu_threads()
    rope = {True: ref.rope_table(T, 1e6), False: ref.rope_table(T, 1e4)}
    qn, kn = synth.qk_norm_gains(3)
    base = synth.normal(17, (T, 4, 256))
    q1, k1, v1 = synth.normal(18, (1, 2048)), synth.normal(19, (1, 1024)), synth.normal(20, (1, 1024))
    rates = {}
    for glob in (False, True):
        caches = []
        for _ in range(th):
            c = ref.new_cache(glob, T)
            k, v = ref.cache_arrays(c)
            k[:] = base[:k.shape[0]]
            v[:] = base[:v.shape[0]]
            caches.append(c)
        # positions spread evenly over [0, T): position j*stride + offset
        per_thread = 4
        npos = th * per_thread
        positions = [int((i + 0.5) * T / npos) for i in range(npos)]

        def worker(t):
            pairs = 0
            for p in positions[t::th]:
                ref.attn_core_tokens(caches[t], q1, k1, v1, qn, kn, rope[glob], p)
                pairs += p + 1 if glob else min(p + 1, 1024)
            return pairs

        with ThreadPoolExecutor(th) as ex:
            list(ex.map(worker, range(th)))  # warm
        pairs, secs = 0, 0.0
        while secs < target_s / 2:
            t0 = time.perf_counter()
            with ThreadPoolExecutor(th) as ex:
                pairs += sum(ex.map(worker, range(th)))
            secs += time.perf_counter() - t0
        rates[glob] = pairs * 8192.0 / secs
        for c in caches:
            ref.free_cache(c)
    fl_local, fl_global = 29 * 7864832 * 8192.0, 5 * 33558528 * 8192.0
    stack_s = fl_local / rates[False] + fl_global / rates[True]
    return {"value": round(T / stack_s, 2), "unit": "tok/s", "cores": th, "kind": "reference",
            "tflops": round((fl_local + fl_global) / stack_s / 1e12, 5),
            "projected_stack_s": round(stack_s, 1),
            "sample": f"{th * 4} query positions spread over 0..8191 per layer type (local / global), "
                      f"each through the reference's per-token attention core on a pre-filled cache, "
                      f"{th} threads, ~{target_s:.0f} s; stack time projected from the measured "
                      f"GFLOP/s per layer type ({rates[False] / 1e9:.2f} local, {rates[True] / 1e9:.2f} global)"}


def secondary_decode_f32(args, torch, gc, pk, dev):
    """configs[3] with the reference's own cache dtype (fp32): 101.5 GB of KV
    per step on one GPU."""
    import synth
    Bl = B_TOTAL
    ctx = gc.Context(max_context=POS + 1, max_batch=Bl, kv_dtype=gc.KV_F32, device=dev, max_prefill=64)
    ctx.upload_rope(gc.rope_table(POS + 1, 10000.0), gc.rope_table(POS + 1, 1000000.0))
    for l in range(N_LAYERS):
        qn, kn = synth.qk_norm_gains(100 + l)
        ctx.set_qk_norm(l, qn, kn)
        rows = CTX if l in GLOBAL_LAYERS else 1024
        for s_ in range(Bl):
            ctx.fill_cache_random(l, s_, rows, 1000 * s_ + l)
    ctx.synchronize()
    d = f"cuda:{dev}"
    g = torch.Generator(device=d).manual_seed(1234)
    q = torch.randn(N_LAYERS, Bl, 2048, device=d, generator=g)
    k = torch.randn(N_LAYERS, Bl, 1024, device=d, generator=g)
    v = torch.randn(N_LAYERS, Bl, 1024, device=d, generator=g)
    out = torch.empty(N_LAYERS, Bl, 2048, device=d)
    seq_a = np.arange(Bl, dtype=np.int32)
    pos_a = np.full(Bl, POS, dtype=np.int32)
    sp = seq_a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    pp = pos_a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    ptrs = [(q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), out[l].data_ptr()) for l in range(N_LAYERS)]
    fn, h = ctx.lib.gemma3_cuda_attn_decode_dev, ctx.h
    stream = torch.cuda.ExternalStream(ctx.stream, device=d)

    def step():
        for l in range(N_LAYERS):
            if fn(h, l, Bl, sp, pp, *ptrs[l]) != 0:
                raise RuntimeError(ctx.last_error())

    for _ in range(3):
        step()
    ctx.synchronize()
    steps = max(3, args.steps // 2)
    ms = ev_time(torch, stream, lambda: [step() for _ in range(steps)])
    ctx.profile(True)
    step()
    ctx.synchronize()
    n, kms, byts = ctx.profile_read(0)
    ctx.profile(False)
    ctx.close()
    del q, k, v, out
    torch.cuda.empty_cache()
    step_bytes = Bl * BYTES_PER_SEQ_STEP * 2
    gbs = step_bytes * steps / (ms / 1e3) / 1e9
    kg = byts / (kms / 1e3) / 1e9
    return {"workload": "configs[3] batched decode B=64, ctx 32768, 34 layers, fp32 KV cache (reference dtype)",
            "value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms / steps, 3),
            "algorithmic_bytes_per_step": step_bytes,
            "roofline": {"bound": "hbm", "kernel": "decode_splitkv<f32>", "achieved": round(kg, 1),
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(kg / pk["hbm_gbs"], 4),
                         "avg_launch_us": round(kms / max(n, 1) * 1e3, 2)}}


def secondary_decode1(args, torch, gc, pk, dev):
    """one token at position 8191 over an 8192-row global cache,
    B=1.  A model step reads each layer's cache once, with the other layers'
    data in between; here 8 global layers, each with its own 8192-row cache
    (8 x 33.5 MB BF16 = 268 MB, twice L2), are decoded in rotation, calls
    queued back to back as a decode step issues them, so every call streams
    its cache from HBM.  us_per_call = CUDA-event time of the whole rotation
    / calls; kernel_us = events around each launch in a separate pass."""
    res = {}
    NG, NL = 8, 48  # global layers 5, 11, ..., 47
    glob = [l for l in range(NL) if (l + 1) % 6 == 0]
    for name, dt in (("bf16", gc.KV_BF16), ("f32", gc.KV_F32)):
        ctx = gc.Context(max_context=8192, max_batch=1, kv_dtype=dt, device=dev, max_prefill=64, num_layers=NL)
        ctx.upload_rope(gc.rope_table(8192, 10000.0), gc.rope_table(8192, 1000000.0))
        for i, l in enumerate(glob):
            ctx.fill_cache_random(l, 0, 8191, 7 + i)
        q = torch.randn(NG, 2048, device=f"cuda:{dev}")
        k = torch.randn(NG, 1024, device=f"cuda:{dev}")
        v = torch.randn(NG, 1024, device=f"cuda:{dev}")
        o = torch.empty(NG, 2048, device=f"cuda:{dev}")
        stream = torch.cuda.ExternalStream(ctx.stream, device=f"cuda:{dev}")
        seq_a = np.zeros(1, dtype=np.int32)
        pos_a = np.full(1, 8191, dtype=np.int32)
        sp = seq_a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
        pp = pos_a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
        fn, h = ctx.lib.gemma3_cuda_attn_decode_dev, ctx.h
        ptrs = [(q[i].data_ptr(), k[i].data_ptr(), v[i].data_ptr(), o[i].data_ptr()) for i in range(NG)]

        def rotation():
            for i, l in enumerate(glob):
                if fn(h, l, 1, sp, pp, *ptrs[i]) != 0:
                    raise RuntimeError(ctx.last_error())

        for _ in range(3):
            rotation()
        ctx.synchronize()
        reps = 25
        ms = ev_time(torch, stream, lambda: [rotation() for _ in range(reps)])
        ctx.profile(True)
        for _ in range(5):
            rotation()
        ctx.synchronize()
        n, kms, byts = ctx.profile_read(0)
        ctx.profile(False)
        ctx.close()
        calls = reps * NG
        per = byts / n
        us = ms / calls * 1e3
        res[name] = {"us_per_call": round(us, 2), "gbs_per_call": round(per / (us / 1e6) / 1e9, 1),
                     "frac_hbm_per_call": round(per / (us / 1e6) / 1e9 / pk["hbm_gbs"], 4),
                     "kernel_us": round(kms / n * 1e3, 2), "kv_bytes": per,
                     "kernel_gbs": round(byts / (kms / 1e3) / 1e9, 1),
                     "frac_hbm": round(byts / (kms / 1e3) / 1e9 / pk["hbm_gbs"], 4)}
    torch.cuda.empty_cache()
    return {"workload": "configs[1] global-layer decode, B=1, 8192 keys; 8 layers' caches (268 MB > L2) in rotation",
            **res}


def secondary_projections(args, torch, gc, pk, dev):
    """Q/K/V + O projections (fp16 tcgen05 GEMM): configs[2]'s T=8192 prefill
    block (tensor-bound) and configs[3]'s B=64 decode batch (weight-streaming,
    HBM-bound).  Eight layers of weights (252 MB, more than L2) are used in
    turn so the decode figure streams weights from HBM."""
    NL = 8
    T = 8192
    ctx = gc.Context(max_context=1024, max_batch=64, kv_dtype=gc.KV_BF16, device=dev, max_prefill=T, num_layers=NL)
    gen = torch.Generator().manual_seed(5)

    def w(shape):
        return (torch.randn(*shape, generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16).numpy().view("uint16")

    for l in range(NL):
        ctx.set_proj_weights(l, w((gc.Q_SIZE, gc.HIDDEN)), w((gc.KV_SIZE, gc.HIDDEN)), w((gc.KV_SIZE, gc.HIDDEN)),
                             w((gc.HIDDEN, gc.Q_SIZE)))
    d = f"cuda:{dev}"
    x = torch.randn(T, gc.HIDDEN, device=d)
    a = torch.randn(T, gc.Q_SIZE, device=d)
    q = torch.empty(T, gc.Q_SIZE, device=d)
    k = torch.empty(T, gc.KV_SIZE, device=d)
    v = torch.empty(T, gc.KV_SIZE, device=d)
    o = torch.empty(T, gc.HIDDEN, device=d)
    stream = torch.cuda.ExternalStream(ctx.stream, device=d)
    res = {}
    for name, rows in (("prefill_T8192", T), ("decode_B64", 64)):
        def step():
            for l in range(NL):
                ctx.project_qkv_dev(l, rows, x.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr())
                ctx.project_o_dev(l, rows, a.data_ptr(), o.data_ptr())
        for _ in range(3):
            step()
        ctx.synchronize()
        reps = 3 if rows == T else 20
        ctx.profile(True)
        ms = ev_time(torch, stream, lambda: [step() for _ in range(reps)])
        ctx.synchronize()
        n, kms, flops = ctx.profile_read(2)
        ctx.profile(False)
        calls = reps * NL
        wbytes = (gc.Q_SIZE + 2 * gc.KV_SIZE) * gc.HIDDEN * 2 + gc.HIDDEN * gc.Q_SIZE * 2
        if rows == T:
            tf = flops / (kms / 1e3) / 1e12
            res[name] = {"gflop_per_layer": round(flops / calls / 1e9, 1), "us_per_layer": round(ms / calls * 1e3, 1),
                         "roofline": {"bound": "tensor", "kernel": "proj_gemm_sm100 (fp16 tcgen05, fp32 acc)",
                                      "achieved": round(tf, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                                      "frac": round(tf / pk["bf16_tflops"], 4)}}
        else:
            gbs = wbytes * calls / (kms / 1e3) / 1e9
            res[name] = {"weight_mb_per_layer": round(wbytes / 1e6, 1), "us_per_layer": round(ms / calls * 1e3, 2),
                         "roofline": {"bound": "hbm", "kernel": "proj_gemm_sm100 + split-K reduce",
                                      "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                                      "frac": round(gbs / pk["hbm_gbs"], 4)}}
    ctx.close()
    del x, a, q, k, v, o
    torch.cuda.empty_cache()
    return {"workload": "Q/K/V + O projections, 8 layers of fp16 weights in turn", **res}


def secondary_model(args, torch, gc, pk, dev):
    """All 34 transformer blocks on the device (gemma3_cuda_prefill_forward_dev /
    gemma3_cuda_forward_dev): a T=8192 prompt (configs[2]'s length) and a B=64
    decode step at 4,096 cached positions per sequence.  One layer's random
    BF16 weights (N(0, 0.02), norm gains N(0, 0.1)) are uploaded to all 34
    layers; the embeddings, final norm and logits are outside the timed calls."""
    T, B, CTXD = 8192, 64, 4096
    d = f"cuda:{dev}"
    gen = torch.Generator().manual_seed(11)

    def w(shape, std=0.02):
        return (torch.randn(*shape, generator=gen) * std).to(torch.bfloat16).view(torch.int16).numpy().view("uint16")

    H, I = gc.HIDDEN, 10240
    lw = dict(input_layernorm=w((H,), 0.1), q_proj=w((gc.Q_SIZE, H)), k_proj=w((gc.KV_SIZE, H)),
              v_proj=w((gc.KV_SIZE, H)), o_proj=w((H, gc.Q_SIZE)), q_norm=w((256,), 0.1), k_norm=w((256,), 0.1),
              post_attention_layernorm=w((H,), 0.1), gate_proj=w((I, H)), up_proj=w((I, H)), down_proj=w((H, I)),
              pre_feedforward_layernorm=w((H,), 0.1), post_feedforward_layernorm=w((H,), 0.1))
    ctx = gc.Context(max_context=T, max_batch=B, kv_dtype=gc.KV_BF16, device=dev, max_prefill=T)
    ctx.upload_rope(gc.rope_table(T, 10000.0), gc.rope_table(T, 1000000.0))
    for l in range(N_LAYERS):
        ctx.set_layer_weights(l, **lw)
    stream = torch.cuda.ExternalStream(ctx.stream, device=d)
    res = {}
    # prefill: 34 blocks over 8192 tokens
    x0 = torch.randn(T, H, device=d)
    x = torch.empty_like(x0)

    def pstep():
        x.copy_(x0)
        ctx.prefill_forward_dev(0, x.data_ptr(), T, 0)

    with torch.cuda.stream(stream):
        pstep()
    ctx.synchronize()
    reps = 2
    with torch.cuda.stream(stream):
        ms = ev_time(torch, stream, lambda: [pstep() for _ in range(reps)])
    ctx.synchronize()
    attn_flops = 3.243e12
    proj_flops = N_LAYERS * 2.0 * T * H * (gc.Q_SIZE + 2 * gc.KV_SIZE + gc.Q_SIZE)
    mlp_flops = N_LAYERS * 2.0 * T * H * 3 * I
    tot = attn_flops + proj_flops + mlp_flops
    res["prefill_T8192"] = {"ms": round(ms / reps, 2), "tok_per_s": round(T * reps / (ms / 1e3), 1),
                            "tflop_per_prompt": round(tot / 1e12, 2),
                            "tflops": round(tot * reps / (ms / 1e3) / 1e12, 1),
                            "frac_of_peak": round(tot * reps / (ms / 1e3) / 1e12 / pk["bf16_tflops"], 4)}
    del x0, x
    # decode: B=64 tokens at position CTXD over random caches
    ctx.reset()
    for l in range(N_LAYERS):
        for s_ in range(B):
            ctx.fill_cache_random(l, s_, CTXD if gc.is_global_layer(l) else 1024, 1000 + 97 * l + s_)
    xd0 = torch.randn(B, H, device=d)
    xd = torch.empty_like(xd0)
    seqs, poss = list(range(B)), [CTXD] * B

    def dstep():
        xd.copy_(xd0)
        ctx.forward_dev(seqs, poss, xd.data_ptr())

    with torch.cuda.stream(stream):
        for _ in range(3):
            dstep()
    ctx.synchronize()
    reps = 10
    with torch.cuda.stream(stream):
        ms = ev_time(torch, stream, lambda: [dstep() for _ in range(reps)])
    ctx.synchronize()
    wbytes = N_LAYERS * 2 * (H * (gc.Q_SIZE + 2 * gc.KV_SIZE) + H * gc.Q_SIZE + 3 * H * I)
    kvbytes = B * (5 * (CTXD + 1) + 29 * 1024) * 4096
    gbs = (wbytes + kvbytes) * reps / (ms / 1e3) / 1e9
    res["decode_B64_ctx4096"] = {"ms_per_step": round(ms / reps, 3), "tok_per_s": round(B * reps / (ms / 1e3), 1),
                                 "weight_gb": round(wbytes / 1e9, 2), "kv_gb": round(kvbytes / 1e9, 2),
                                 "gbs": round(gbs, 1), "frac_hbm": round(gbs / pk["hbm_gbs"], 4)}
    # greedy step: token ids in, ids out (embedding, 34 blocks, final norm,
    # 262,208-way tied-embedding logits, argmax), same caches and positions
    emb = w((262208, H))
    ctx.set_embeddings(emb, w((H,), 0.1))
    del emb
    toks = list(range(1000, 1000 + B))
    for _ in range(2):
        ctx.greedy_step(seqs, poss, toks)
    reps = 5
    import time as _t
    t0 = _t.perf_counter()
    for _ in range(reps):
        ctx.greedy_step(seqs, poss, toks)  # synchronous: ids back on the host each step
    wall = (_t.perf_counter() - t0) / reps
    res["greedy_step_B64_ctx4096"] = {"ms_per_step_wall": round(wall * 1e3, 3), "tok_per_s": round(B / wall, 1),
                                      "note": "host-synchronous call incl. 1.34 GB logits GEMM and argmax"}
    ctx.close()
    del xd0, xd
    torch.cuda.empty_cache()
    return {"workload": "34 Gemma-3-4B blocks on the device (attention, projections, norms, GELU MLP)", **res}


def model_decode_case(torch, gc, dev, steps):
    """`steps` whole-model decode steps (34 blocks, B=64 at 4,096 cached
    positions, one layer's random BF16 weights on every layer)."""
    B, CTXD, H, I = 64, 4096, gc.HIDDEN, 10240
    gen = torch.Generator().manual_seed(11)

    def w(shape, std=0.02):
        return (torch.randn(*shape, generator=gen) * std).to(torch.bfloat16).view(torch.int16).numpy().view("uint16")

    lw = dict(input_layernorm=w((H,), 0.1), q_proj=w((gc.Q_SIZE, H)), k_proj=w((gc.KV_SIZE, H)),
              v_proj=w((gc.KV_SIZE, H)), o_proj=w((H, gc.Q_SIZE)), q_norm=w((256,), 0.1), k_norm=w((256,), 0.1),
              post_attention_layernorm=w((H,), 0.1), gate_proj=w((I, H)), up_proj=w((I, H)), down_proj=w((H, I)),
              pre_feedforward_layernorm=w((H,), 0.1), post_feedforward_layernorm=w((H,), 0.1))
    ctx = gc.Context(max_context=CTXD + 1, max_batch=B, kv_dtype=gc.KV_BF16, device=dev, max_prefill=64)
    ctx.upload_rope(gc.rope_table(CTXD + 1, 10000.0), gc.rope_table(CTXD + 1, 1000000.0))
    for l in range(N_LAYERS):
        ctx.set_layer_weights(l, **lw)
        for s_ in range(B):
            ctx.fill_cache_random(l, s_, CTXD if gc.is_global_layer(l) else 1024, 1000 + 97 * l + s_)
    xd = torch.randn(B, H, device=f"cuda:{dev}")
    for _ in range(steps):
        ctx.forward_dev(list(range(B)), [CTXD] * B, xd.data_ptr())
    ctx.synchronize()
    ctx.close()


def secondary_context_parallel(args, dist, torch, gc, pk):
    """B=4 sequences at 131,072 keys, BF16 KV; the 5 global layers'
    KV range is split over the N ranks (partials merged with an NCCL
    all-gather inside the library), the 29 local layers run on every rank.
    Metric: the job's algorithmic KV bytes per step / max-over-ranks time."""
    B, ctxlen = 4, 131072
    pos = ctxlen - 1
    dev = dist.local
    c = gc.Context(max_context=ctxlen, max_batch=B, kv_dtype=gc.KV_BF16, device=dev, max_prefill=64,
                   kv_rank=dist.rank, kv_ranks=dist.world)
    c.upload_rope(gc.rope_table(ctxlen, 1e4), gc.rope_table(ctxlen, 1e6))
    S = -(-ctxlen // dist.world)
    lo = min(ctxlen, dist.rank * S)
    for l in range(N_LAYERS):
        for s_ in range(B):
            rows = max(0, min(lo + S, pos) - lo) if l in GLOBAL_LAYERS else 1024
            if rows:
                c.fill_cache_random(l, s_, rows, 77 * s_ + l + (1000003 * dist.rank if l in GLOBAL_LAYERS else 0))
    if dist.world > 1:
        uid = [gc.Context.comm_unique_id() if dist.rank == 0 else None]
        dist.pg.broadcast_object_list(uid, src=0)
        c.comm_init(uid[0])
    g = torch.Generator(device=f"cuda:{dev}").manual_seed(4321)
    q = torch.randn(N_LAYERS, B, 2048, device=f"cuda:{dev}", generator=g)
    k = torch.randn(N_LAYERS, B, 1024, device=f"cuda:{dev}", generator=g)
    v = torch.randn(N_LAYERS, B, 1024, device=f"cuda:{dev}", generator=g)
    out = torch.empty(N_LAYERS, B, 2048, device=f"cuda:{dev}")
    stream = torch.cuda.ExternalStream(c.stream, device=f"cuda:{dev}")
    seqs, poss = list(range(B)), [pos] * B

    def step():
        for l in range(N_LAYERS):
            c.attn_decode_dev(l, seqs, poss, q[l].data_ptr(), k[l].data_ptr(), v[l].data_ptr(), out[l].data_ptr())

    steps = max(args.steps, 10)

    def timed():
        for _ in range(args.warmup):
            step()
        c.synchronize()
        dist.barrier()
        t = dist.max(ev_time(torch, stream, lambda: [step() for _ in range(steps)]))
        c.synchronize()
        return t

    ms = ms_nccl = timed()
    peer_note = None
    if dist.world > 1:
        # fused exchange: merged partials stored into the peers' buffers over
        # NVLink by the merge kernel, flags instead of a library collective.
        # Every rank must have mapped its peers before any uses the path, so
        # the ranks agree on the set-up outcome first.
        try:
            c.peer_init()
            ok = 1.0
        except Exception as e:  # reported in the line, the NCCL figure stays
            peer_note = f"peer exchange unavailable: {type(e).__name__}: {e}"
            ok = 0.0
        if dist.sum(ok) == dist.world:
            try:
                ms = timed()
            except Exception as e:  # a device-side failure is seen by every rank alike
                peer_note = f"peer exchange failed: {type(e).__name__}: {e}"
                ms = ms_nccl
        else:
            peer_note = peer_note or "peer exchange unavailable on another rank"
            if ok:
                c.set_exchange(gc.XCHG_NCCL)
    dist.barrier()
    c.close()
    del q, k, v, out
    torch.cuda.empty_cache()
    byts = (len(GLOBAL_LAYERS) * ctxlen + (N_LAYERS - len(GLOBAL_LAYERS)) * 1024) * B * ROW_BYTES_BF16
    gbs = byts * steps / (ms / 1e3) / 1e9
    xchg = ("no exchange" if dist.world == 1 else "NCCL all-gather + LSE merge" if peer_note else
            "merge kernel stores partials into peers' buffers over NVLink + flag wait + LSE merge")
    res = {"workload": "configs[4] long-context decode, B=4 @ 131072 keys, global-layer KV split over "
                       f"{dist.world} GPU(s), {xchg}; local layers on every rank",
           "value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms / steps, 3),
           "algorithmic_bytes_per_step": byts, "frac_of_n_x_hbm": round(gbs / (pk["hbm_gbs"] * dist.world), 4)}
    if dist.world > 1 and not peer_note:
        res["nccl_allgather"] = {"value": round(byts * steps / (ms_nccl / 1e3) / 1e9, 1),
                                 "ms_per_step": round(ms_nccl / steps, 3)}
    if peer_note:
        res["note"] = peer_note
    return res


def ncu_traffic(kernel, bytes_per_launch):
    """DRAM bytes per launch of `kernel`: the per-launch algorithmic bytes
    scaled by the DRAM/algorithmic ratio of the committed ncu capture
    (profiles/ncu_traffic.txt, measured on a smaller case of the same
    kernel: traffic grows in proportion to the rows streamed), or None."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if not os.path.exists(p) or not bytes_per_launch:
        return None
    for line in open(p):
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel:
            return round(float(parts[1]) * bytes_per_launch, 0)
    return None


def profile_case(args):
    """Few-launch cases for `ncu --set full` (one GPU, about 1-2 GB resident,
    inputs still larger than L2): decode = global layer, 8 sequences x 32769
    rows (1.07 GB of BF16 KV); prefill = one global and one local layer at
    T=8192; proj = the Q/K/V projection of a T=8192 block, twice (a
    302 MB fp16 input / output set)."""
    import torch
    import gemma3_cuda as gc
    import synth
    if args.profile_case == "decode":
        B = 8
        ctx = gc.Context(max_context=POS + 1, max_batch=B, kv_dtype=gc.KV_BF16, max_prefill=64, num_layers=6)
        ctx.upload_rope(gc.rope_table(POS + 1, 1e4), gc.rope_table(POS + 1, 1e6))
        for s in range(B):
            ctx.fill_cache_random(5, s, CTX, s)
        q = torch.randn(B, 2048, device="cuda")
        k = torch.randn(B, 1024, device="cuda")
        v = torch.randn(B, 1024, device="cuda")
        o = torch.empty(B, 2048, device="cuda")
        for _ in range(3):
            ctx.attn_decode_dev(5, list(range(B)), [POS] * B, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr())
    elif args.profile_case == "proj":
        T = 8192
        ctx = gc.Context(max_context=1024, max_batch=1, kv_dtype=gc.KV_BF16, max_prefill=T, num_layers=1)
        gen = torch.Generator().manual_seed(5)

        def w(shape):
            return (torch.randn(*shape, generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16).numpy().view(
                "uint16")

        ctx.set_proj_weights(0, w((2048, 2560)), w((1024, 2560)), w((1024, 2560)), w((2560, 2048)))
        x = torch.randn(T, 2560, device="cuda")
        q = torch.empty(T, 2048, device="cuda")
        k = torch.empty(T, 1024, device="cuda")
        v = torch.empty(T, 1024, device="cuda")
        for _ in range(2):
            ctx.project_qkv_dev(0, T, x.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr())
    elif args.profile_case == "model_decode":
        # 3 whole-model decode steps (34 blocks, B=64 at 4096 cached positions),
        # the workload of secondary.model.decode_B64_ctx4096
        model_decode_case(torch, gc, 0, steps=3)
        print(json.dumps({"profile_case": args.profile_case, "ok": True}))
        return
    elif args.profile_case == "prefill_stack":
        # the configs[2] stack exactly as the bench times it, 2 steps (for a
        # one-pass launch list: every prologue and attention launch)
        import types
        secondary_prefill(types.SimpleNamespace(steps=2, warmup=1), torch, gc, peaks(), 0)
        print(json.dumps({"profile_case": args.profile_case, "ok": True}))
        return
    else:
        T = 8192
        ctx = gc.Context(max_context=T, max_batch=1, kv_dtype=gc.KV_BF16, max_prefill=T, num_layers=6)
        ctx.upload_rope(gc.rope_table(T, 1e4), gc.rope_table(T, 1e6))
        for l in (0, 5):
            qn, kn = synth.qk_norm_gains(l)
            ctx.set_qk_norm(l, qn, kn)
        q = torch.randn(T, 2048, device="cuda")
        k = torch.randn(T, 1024, device="cuda")
        v = torch.randn(T, 1024, device="cuda")
        o = torch.empty(T, 2048, device="cuda")
        for l in (5, 0, 5):
            ctx.attn_prefill_dev(l, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), T, 0, o.data_ptr())
    ctx.synchronize()
    ctx.close()
    print(json.dumps({"profile_case": args.profile_case, "ok": True}))


def main():
    global B_TOTAL
    args = parse_args()
    B_TOTAL = args.seqs
    # rank 0 prints exactly one JSON line on stdout: keep NCCL's version
    # banner (printed to stdout at NCCL_DEBUG=VERSION) out of it
    if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.profile_case:
        return profile_case(args)
    dist = Dist()
    if args.impl == "reference":
        dist.init("gloo")
        res = run_reference_arm(args, dist)
        if res is not None:
            print(json.dumps(res), flush=True)
        dist.close()
        return
    import torch
    if not torch.cuda.is_available():
        raise SystemExit("bench.py --impl ours needs a CUDA device (there is no CPU fallback)")
    dist.init("nccl")
    torch.cuda.set_device(dist.local)
    import gemma3_cuda as gc
    import synth
    pk = peaks()
    h = headline(args, dist, torch, gc, synth, pk)
    line = {
        "metric": "decode attention KV throughput, 34-layer Gemma-3-4B, B=64 @ 32768 ctx",
        "value": round(h["value"], 2), "unit": "GB/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(h["ms_per_step"], 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) BF16 KV cache, random q/k/v projections)",
        "config": {"workload": "configs[3] batched decode B=64, ctx 32768, 34 layers (5 global + 29 local)",
                   "batch": B_TOTAL, "per_gpu_batch": B_TOTAL // dist.world, "context": CTX,
                   "layers": N_LAYERS, "kv_cache": "bf16, head-major device-resident",
                   "parallelism": f"sequence-sharded x{dist.world}, no data-path collective",
                   "algorithmic_bytes_per_step": B_TOTAL * BYTES_PER_SEQ_STEP,
                   "l2": "inputs (50.7 GB of KV) larger than L2; no flush needed"},
        "e2e": {"value": round(h["e2e"], 2), "unit": "GB/s", "h2d_bytes_per_step": h["h2d"],
                "d2h_bytes_per_step": h["d2h"],
                "api": "gemma3_cuda_attn_decode (host pointers, pinned), 34 calls per step per rank"},
        "gpu_launches": int(dist.sum(h["gpu_launches"])),
        "clocks": h["clocks"],
    }
    rf = dict(h["roofline"])
    tr = ncu_traffic("decode_tc_bf16", rf.get("bytes_per_launch"))
    rf["traffic"] = tr
    rf["peak_src"] = f"{pk['src']} hbm_gbs (MEASURED_PEAKS.json)" if pk["src"] == "measured" else "fallback 6.65 TB/s"
    for kk in ("achieved", "frac", "avg_launch_us", "bytes_per_launch"):
        if rf.get(kk) is not None:
            rf[kk] = round(rf[kk], 4 if kk == "frac" else 2)
    line["roofline"] = rf
    if not args.no_secondary:
        cp = secondary_context_parallel(args, dist, torch, gc, pk)
    if dist.rank == 0 and dist.world == 1:
        if not args.no_secondary:
            line["secondary"] = {"config0": secondary_config0(args, torch, gc, pk, dist.local,
                                                              not args.no_cpu_baseline),
                                 "decode_f32": secondary_decode_f32(args, torch, gc, pk, dist.local),
                                 "prefill": secondary_prefill(args, torch, gc, pk, dist.local),
                                 "decode_b1": secondary_decode1(args, torch, gc, pk, dist.local),
                                 "projections": secondary_projections(args, torch, gc, pk, dist.local),
                                 "model": secondary_model(args, torch, gc, pk, dist.local)}
    if not args.no_secondary:
        line.setdefault("secondary", {})["context_parallel"] = cp
        if not args.no_cpu_baseline and dist.rank == 0 and dist.world == 1:
            try:
                line["cpu_baseline"] = cpu_baseline_sample()
            except Exception as e:  # reported, never silently replaced
                line["cpu_baseline"] = {"value": None, "error": f"{type(e).__name__}: {e}"}
            try:
                line["secondary"]["prefill"]["cpu_baseline"] = cpu_prefill_stack_sample()
            except Exception as e:
                line["secondary"]["prefill"]["cpu_baseline"] = {"value": None, "error": f"{type(e).__name__}: {e}"}
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()

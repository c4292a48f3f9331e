"""Benchmark: decode tok/s of the 8B-shaped Q4_K decoder at batch 64 with fp8 paged KV, and % of the HBM roofline.

Workload: Llama-3-8B shape (32 layers, d 4096, 32/8 heads of 128, FFN 14336, vocab 128256),
random N(0, 0.02) weights quantized to Q4_K (every matrix, embedding and head included), fp8 e4m3 KV with per-page
scales in 16-token pages; 64 sequences with contexts log-normal over 512-8192 (numpy default_rng(0), median 2147,
sum 168,356); sequences 0-31 share a 1024-token radix prefix (the same 64 pages in every table). Synthetic data: there
is no network for checkpoints or datasets.

One step = one gc_step of 64 one-token greedy decode items (device argmax) through the C ABI of libgck.so.
  value  tok/s from the device time of the steps' kernels (CUDA events on the library's stream, gck_ext.h)
  e2e    tok/s from the host clock around the synchronous gc_step calls: plan upload (tokens, block tables) H2D,
         the kernels, the argmax tokens D2H
Inputs (13 GB of weights and KV) are far larger than L2 (126 MB), so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Under torchrun (N > 1) every rank runs an independent replica on its GPU (the 8B configs do not shard).
"""
import argparse
import json
import math
import os
import subprocess
import tempfile
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SPEC8B = dict(vocab=128256, d=4096, layers=32, heads=32, kv_heads=8, ffn=14336, eps=1e-5, theta=5e5, wtype="q4_k",
              std=0.02, seed=0, ctx=8192 + 128, name="llama3-8b-shape-q4k")
B, PREFIX = 64, 1024
METRIC = "decode tok/s (8B Q4_K, batch 64, fp8 KV)"
# DRAM bytes (read + write) per launch from single-kernel ncu captures of this workload (the 8B shape with 2 of its 32
# layers: a layer's launches have the full-size weights and KV); each names the library build it was captured on, and
# is reported beside the live timing, never in place of it
ATTN_TRAFFIC = dict(bytes=287_385_088, build="13d6345", kernel="attn_kernel<128, fp8, 1 warp, 1 row tile>")
# one layer's three GEMM launches (q/k/v, o, gate/up chained with down): 128.1 MB of DRAM traffic against 122.7 MB of
# Q4_K weights (1.044); "bytes" is their mean per launch, "gateup_down" the chained launch alone (the head launch was
# not captured)
GEMM_TRAFFIC = dict(bytes=42_703_701, gateup_down=103_319_040, build="dbd0dbe", ratio_to_weight_bytes=1.044)


def contexts():
    rng = np.random.default_rng(0)
    ctx = np.clip(np.rint(np.exp(rng.normal(math.log(2048), math.log(4) / 2, B))), 512, 8192).astype(int)
    ctx[:32] = np.maximum(ctx[:32], PREFIX + 16)
    return ctx


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        return {}


class Clocks:
    """SM clock and throttle reasons sampled during the timed region: NVML every 10 ms (reads only), else nvidia-smi
    every 200 ms."""

    def __init__(self, gpu):
        self.gpu, self.rows, self.p, self.stop, self.t = gpu, [], None, None, None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.stop = threading.Event()
            bits = [("hw_slowdown", pynvml.nvmlClocksEventReasonHwSlowdown),
                    ("hw_thermal_slowdown", pynvml.nvmlClocksEventReasonHwThermalSlowdown),
                    ("sw_thermal_slowdown", pynvml.nvmlClocksEventReasonSwThermalSlowdown),
                    ("sw_power_cap", pynvml.nvmlClocksEventReasonSwPowerCap)]

            def poll():
                mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                while not self.stop.is_set():
                    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.rows.append([str(sm), str(mx), "", ""] + ["Active" if r & m else "Not Active" for _, m in bits])
                    time.sleep(0.01)
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.stop = None
        q = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
            "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
            "clocks_event_reasons.sw_power_cap"
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.p = None
        return self

    def _read(self):
        for line in self.p.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.stop is not None:
            self.stop.set()
            self.t.join(timeout=2)
        if self.p:
            self.p.terminate()
            self.p.wait()
            self.t.join(timeout=2)

    def summary(self):
        sm = [float(r[0]) for r in self.rows if r and r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if len(r) > 1 and r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm), "source": "nvml 10 ms" if self.stop is not None else "nvidia-smi"}


def model_dir():
    from goethe_engine_b200 import synth
    spec = synth.Spec(**SPEC8B)
    d = os.path.join(os.environ.get("GCK_BENCH_DIR", "/tmp/gck_bench"), f"{spec.name}-s{spec.seed}")
    return spec, d


def ensure_model(rank, world, barrier):
    from goethe_engine_b200 import synth
    spec, d = model_dir()
    if rank == 0:
        t0 = time.time()
        synth.make(d, spec, ncol=B, maxctx=spec.ctx, kv="fp8", tune=dict(max_cols=2048, kv_scale="page"))
        print(f"[bench] model ready in {d} ({time.time() - t0:.1f}s)", file=sys.stderr, flush=True)
    if world > 1:
        barrier()
    return spec, d, [os.path.join(d, "model.gguf")]


def setup_sequences(be, ctx, steps_total):
    """Block tables and the prefill of every sequence's context (the shared prefix once)."""
    from goethe_engine_b200 import gck
    bs = be.block_size
    nxt = [0]

    def alloc(n):
        out = list(range(nxt[0], nxt[0] + n))
        nxt[0] += n
        return out
    rng = np.random.default_rng(1)
    prefix_tok = [int(x) for x in rng.integers(1, 128000, PREFIX)]
    shared = alloc(PREFIX // bs)
    tables, toks, start = [], [], []
    for i, c in enumerate(ctx):
        own = -(-(int(c) + steps_total + 1) // bs)
        if i < 32:
            tables.append(shared + alloc(own - len(shared)))
            toks.append(prefix_tok + [int(x) for x in rng.integers(1, 128000, int(c) - PREFIX)])
            start.append(PREFIX if i else 0)
        else:
            tables.append(alloc(own))
            toks.append([int(x) for x in rng.integers(1, 128000, int(c))])
            start.append(0)
    assert nxt[0] <= be.num_blocks, (nxt[0], be.num_blocks)
    # prefill: chunks packed into steps of at most max_cols tokens; the last token of each context is left for decode
    queue = [[i, start[i], int(ctx[i]) - 1] for i in range(len(ctx))]
    queue[0][2] = int(ctx[0]) - 1
    # sequence 0 computes the shared prefix before anyone else reads it
    order = [queue[0]] + queue[1:]
    cap = be.layout.max_cols
    t0 = time.time()
    while any(q[1] < q[2] for q in order):
        budget, items = cap, []
        for q in order:
            if q[1] >= q[2] or budget == 0:
                continue
            if q[0] in range(1, 32) and order[0][1] < PREFIX:
                continue
            n = min(budget, q[2] - q[1])
            items.append(gck.Work(q[0], toks[q[0]][q[1]:q[1] + n], q[1], tables[q[0]], 0))
            q[1] += n
            budget -= n
        be.step(items)
    # block tables as uint32 arrays: the binding hands them to gc_step without a copy
    return [np.asarray(t, np.uint32) for t in tables], toks, time.time() - t0


def kv_unique_bytes(ctx_now, layout):
    """Algorithmic KV bytes one decode step reads over all layers: every distinct row once (the shared prefix once)."""
    rows = int(np.sum(ctx_now + 1)) - 31 * PREFIX
    per_row = 2 * layout.kv_heads * layout.head_dim * 1        # K and V, fp8
    return rows * per_row * layout.layers


def weight_bytes(spec):
    from goethe_engine_b200.synth import Spec
    s = Spec(**spec)
    n = sum(r * c for _, (r, c), t in s.tensors() if t != "f32" and _ != "token_embd.weight")
    return n * 144 // 256


class Stats:
    """gck_ext.h step statistics of a handle: enable(mask) starts them, read() stops and returns them."""

    def __init__(self, be):
        import ctypes as C

        class S(C.Structure):
            _fields_ = [("size", C.c_uint32), ("steps", C.c_uint32), ("launches", C.c_uint64),
                        ("forward_ms", C.c_double), ("class_ms", C.c_double * 16), ("class_launches", C.c_uint64 * 16),
                        ("h2d_bytes", C.c_uint64), ("graph_steps", C.c_uint32), ("graph_captures", C.c_uint32),
                        ("gemm_pairs", C.c_uint32)]
        self.S, self.be, self.C = S, be, C
        be.L.gck_stats_enable.argtypes = [C.c_void_p, C.c_uint32]
        be.L.gck_stats_read.argtypes = [C.c_void_p, C.c_void_p]

    def enable(self, mask=0):
        self.be.L.gck_stats_enable(self.be.h, mask)

    def read(self):
        st = self.S(size=self.C.sizeof(self.S))
        self.be.L.gck_stats_read(self.be.h, self.C.byref(st))
        return st


GEMMS = (2, 6, 7, 8, 9)           # gck_ext.h classes of the tcgen05 GEMM launches: q/k/v, o, gate/up, down, head
ATTN, GATEUP, DOWN = 4, 7, 8


def run_mine(args, rank, world, barrier, maxreduce):
    from goethe_engine_b200 import build, gck
    if rank == 0:
        build.build()
    if world > 1:
        barrier()
    spec, d, ws = ensure_model(rank, world, barrier)
    ctx = contexts()
    PASS = args.steps                   # steps of each per-kernel pass after the timed region
    steps_total = args.warmup + args.steps + 2 * PASS
    dev = int(os.environ.get("LOCAL_RANK", 0))
    t0 = time.time()
    be = gck.Backend(d, ws, pool_blocks=int(np.sum(ctx)) // 16 + 2 * B + 64, device=dev)
    t_open = time.time() - t0
    stats = Stats(be)
    stats.enable(0)
    tables, toks, t_prefill = setup_sequences(be, ctx, steps_total)
    st0 = stats.read()
    last = np.array([t[-1] for t in toks], np.int32)
    pos = np.array([int(c) - 1 for c in ctx], np.int64)
    sids = np.arange(B)

    def step():
        # one token per sequence through gc_step (Backend.decode: the work records built from columns)
        last[:] = be.decode(sids, last, pos, tables)
        pos[:] += 1
    stats.enable(0)
    for _ in range(args.warmup):
        step()
    stw = stats.read()
    kv_bytes = np.mean([kv_unique_bytes(np.array(pos) + k, be.layout) for k in range(args.steps)])
    import torch
    torch.cuda.synchronize()
    if world > 1:
        barrier()
    # the timed region: whole-step events only (events around single launches would cut the programmatic overlap)
    stats.enable(0xFFFF if args.profile else 0)
    # GCK_PROFILE_WINDOW=1: the CUDA profiler window covers the first timed step only (ncu --profile-from-start off)
    window = bool(os.environ.get("GCK_PROFILE_WINDOW"))
    with Clocks(dev) as clk:
        t0 = time.perf_counter()
        for k in range(args.steps):
            if window and k == 0:
                torch.cuda.profiler.start()
            step()
            if window and k == 0:
                torch.cuda.profiler.stop()
        wall = time.perf_counter() - t0
    st = stats.read()
    torch.cuda.synchronize()
    # per-kernel device time: the same decode steps again (PASS each, the positions one further every step), events
    # around every launch of the GEMM classes, then around every attention launch. Those events cut the programmatic
    # overlap at the bracketed launches, so the per-launch times are upper bounds.
    stats.enable(sum(1 << c for c in GEMMS))
    for _ in range(PASS):
        step()
    sg = stats.read()
    stats.enable(1 << ATTN)
    for _ in range(PASS):
        step()
    sa = stats.read()
    stats.enable(0)
    if world > 1:
        barrier()
    dev_s = maxreduce(st.forward_ms / 1e3)
    wall = maxreduce(wall)
    value, e2e = aggregate(B * args.steps, world, dev_s, wall)
    pk = peaks()
    hbm = pk.get("hbm_gbs", 6650.0)
    psrc = "MEASURED_PEAKS.json hbm_gbs (burst copy)" if "hbm_gbs" in pk else "fallback 6650 GB/s"
    attn_ms = sa.class_ms[ATTN] / max(1, sa.class_launches[ATTN])
    attn_bytes = kv_bytes / be.layout.layers
    wbytes = weight_bytes(SPEC8B)
    step_bytes = kv_bytes + wbytes
    ms_step = dev_s / args.steps * 1e3
    gemm = gemm_roofline(sg, PASS, hbm, psrc)
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_k x f16 -> f32; fp8 e4m3 KV", "data": "synthetic (seeded N(0,0.02) weights, uniform tokens)",
        "config": {"workload": "C3: Llama-3-8B shape, Q4_K weights, fp8 paged KV (per-page scale), 64-sequence greedy "
                               "decode, log-normal contexts 512-8192 (sum 168356), 32 sequences share a 1024-token prefix",
                   "batch": B, "context_sum": int(np.sum(ctx)), "block_size": be.block_size, "layers": SPEC8B["layers"],
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (13 GB per step), no flush"},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": int(st.h2d_bytes // max(1, st.steps)),
                "d2h_bytes_per_step": B * 4 + 4, "path": "gc_step through the C ABI (ctypes), host buffers",
                "h2d_source": "the library's own count of its plan and block-table patch uploads (gck_stats.h2d_bytes)",
                "captured_steps": f"{st.graph_steps} of {st.steps} timed steps replayed a captured CUDA graph"},
        "roofline": gemm,
        "roofline_attention": {
            "bound": "hbm", "kernel": "attn_kernel (paged fp8 KV attention), one launch per layer",
            "achieved": round(attn_bytes / (attn_ms / 1e3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(attn_bytes / (attn_ms / 1e3) / 1e9 / hbm, 4),
            "traffic": ATTN_TRAFFIC["bytes"], "traffic_build": ATTN_TRAFFIC["build"],
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch (single-kernel capture)",
            "algorithmic_bytes_per_launch": int(attn_bytes), "launch_ms": round(attn_ms, 4),
            "timing": f"CUDA events around each attention launch, {PASS} decode steps after the timed region",
            "peak_source": psrc},
        "step_roofline": {"algorithmic_bytes": int(step_bytes), "weights_bytes": int(wbytes), "kv_bytes": int(kv_bytes),
                          "achieved_gbs": round(step_bytes / (ms_step / 1e3) / 1e9, 1),
                          "frac_of_measured": round(step_bytes / (ms_step / 1e3) / 1e9 / hbm, 4),
                          "frac_of_8tbs": round(step_bytes / (ms_step / 1e3) / 1e9 / 8000, 4)},
        "gpu_launches": int(st.launches),
        "clocks": clk.summary(),
        "setup": {"open_s": round(t_open, 1), "prefill_s": round(t_prefill, 1), "prefill_tokens": int(np.sum(ctx) - 31 * PREFIX),
                  "launches_before_timed": int(st0.launches + stw.launches)},
    }
    if args.profile:
        print_classes(st, args.steps)
    be.close()
    if rank == 0:
        if world == 1 and not args.no_cpu:
            res["parity"] = c3_parity()
            res["cpu_baseline"] = cpu_baseline()
        return res
    return None


def gemm_roofline(sg, steps, hbm, peak_source):
    """HBM roofline of the dominant kernel of a C3 step, the tcgen05 GEMM (every projection and the head): the Q4_K
    weight bytes the step's GEMM launches read (each weight once) over their summed device time, i.e. the algorithmic
    bytes of the average launch over its average duration; and the gate/up launch alone (66.06 MB of weights, 0.5 MB
    of activations, 1.8 MB of f16 output)."""
    ms = sum(sg.class_ms[c] for c in GEMMS) / steps
    launches = sum(sg.class_launches[c] for c in GEMMS) // steps
    wb = weight_bytes(SPEC8B)
    gu_ms = sg.class_ms[GATEUP] / max(1, sg.class_launches[GATEUP])
    gu_bytes = 2 * 14336 * 4096 * 144 // 256 + 64 * 4096 * 2 + 64 * 14336 * 2
    # chained: one launch per layer runs gate/up and down_proj (the down class launches nothing)
    chained = sg.class_launches[DOWN] == 0 and sg.class_launches[GATEUP] > 0
    if chained:
        gu_bytes += 4096 * 14336 * 144 // 256 + 64 * 14336 * 2 + 64 * 4096 * 4
    out = {"bound": "hbm", "kernel": "gemm_tc_kernel<Q4_K, 64> (q/k/v, o, gate/up "
                                     + ("chained with down in one launch" if chained else "and down")
                                     + " in every layer, and the head)",
           "achieved": round(wb / (ms / 1e3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
           "frac": round(wb / (ms / 1e3) / 1e9 / hbm, 4), "ms_per_step": round(ms, 4), "launches_per_step": int(launches),
           "algorithmic_bytes_per_launch": int(wb / max(1, launches)), "launch_ms": round(ms / max(1, launches), 5),
           "algorithmic_bytes_per_step": int(wb),
           "traffic": GEMM_TRAFFIC["bytes"] if GEMM_TRAFFIC else None,
           "traffic_build": GEMM_TRAFFIC["build"] if GEMM_TRAFFIC else None,
           "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, mean per launch over one layer's three GEMM "
                             "launches (--layers 2 case, full-size weights); 1.044 x their weight bytes",
           ("gateup_down" if chained else "gateup"): {
               "launch_ms": round(gu_ms, 4), "algorithmic_bytes_per_launch": int(gu_bytes),
               "achieved": round(gu_bytes / (gu_ms / 1e3) / 1e9, 1),
               "frac": round(gu_bytes / (gu_ms / 1e3) / 1e9 / hbm, 4),
               "traffic": GEMM_TRAFFIC.get("gateup_down" if chained else "gateup") if GEMM_TRAFFIC else None},
           "timing": f"CUDA events around each GEMM launch, {steps} decode steps after the timed region (upper bound: "
                     "the events cut the programmatic overlap)", "peak_source": peak_source}
    return out


# ------------------------------------------------------------------------------------------- C3 parity sample
def c3_sample():
    """A C3-shaped decode step of 64 sequences that the oracle can check: eight with contexts from the benchmark's own
    draw (7969, 838 and 856 tokens of their own; 2234 and four of 1040 on the shared 1024-token prefix pages), and 56
    that share the prefix pages with 16-48 tokens of their own (the step's token tile is the benchmark's 64 rows).
    Returns contexts, block tables, tokens, the pool size, the prefill chunks (sequence, start, end; the shared prefix
    first) and the decode items."""
    ctx = contexts()
    pick = [47, 54, 40, 0, 9, 12, 30, 14]
    rng = np.random.default_rng(3)
    cs = [int(ctx[i]) for i in pick] + [PREFIX + int(x) for x in rng.integers(16, 49, 56)]
    share = [i < 32 for i in pick] + [True] * 56
    rng = np.random.default_rng(1)
    prefix = [int(x) for x in rng.integers(1, 128000, PREFIX)]
    nxt, tabs, toks = PREFIX // 16, [], []
    for c, sh in zip(cs, share):
        own = -(-(c + 1) // 16) - (PREFIX // 16 if sh else 0)
        tabs.append((list(range(PREFIX // 16)) if sh else []) + list(range(nxt, nxt + own)))
        toks.append((prefix if sh else []) + [int(x) for x in rng.integers(1, 128000, c - (PREFIX if sh else 0))])
        nxt += own
    first = share.index(True)
    pre = [(first, 0, PREFIX)] + [(i, PREFIX if sh else 0, c - 1) for i, (c, sh) in enumerate(zip(cs, share))
                                  if i != first] + [(first, PREFIX, cs[first] - 1)]
    dec = [dict(sid=i, tokens=[t[-1]], pos=c - 1, blocks=tabs[i], want=1) for i, (c, t) in enumerate(zip(cs, toks))]
    return dict(cs=cs, tabs=tabs, toks=toks, nblk=nxt + 8, pre=pre, dec=dec)


def c3_sample_run(be, smp):
    """The library's half: the prefill (the shared prefix alone, then steps of at most 2048 tokens), then the decode
    step twice: float32 host logits, and greedy tokens from the device argmax (the same KV rows rewritten with the
    same values)."""
    from goethe_engine_b200 import gck
    toks, tabs = smp["toks"], smp["tabs"]
    (i0, a0, b0), queue = smp["pre"][0], [list(x) for x in smp["pre"][1:]]
    be.step([gck.Work(i0, toks[i0][a0:b0], a0, tabs[i0], 0)])
    while queue:
        budget, items = 2048, []
        for q in queue:
            if budget and q[1] < q[2]:
                n = min(budget, q[2] - q[1])
                items.append(gck.Work(q[0], toks[q[0]][q[1]:q[1] + n], q[1], tabs[q[0]], 0))
                q[1] += n
                budget -= n
        queue = [q for q in queue if q[1] < q[2]]
        be.step(items)
    dec = smp["dec"]
    got = be.step([gck.Work(d["sid"], d["tokens"], d["pos"], d["blocks"], 1) for d in dec])
    greedy = be.step([gck.Work(d["sid"], d["tokens"], d["pos"], d["blocks"], 1, greedy=True) for d in dec])
    return got, np.array([g[0] for g in greedy])


def c3_sample_oracle(gguf_path, smp, kv="fp8"):
    """The oracle's half over the same GGUF: the shared prefix, then every other prefill chunk in one step, then the
    decode step (oracle/ is test infrastructure; the benchmark runs it only in its CPU leg, as the checker)."""
    from oracle.load import weights_from_gguf
    from oracle.model import PagedOracle
    toks, tabs, pre = smp["toks"], smp["tabs"], smp["pre"]
    o = PagedOracle(weights_from_gguf(gguf_path), num_blocks=smp["nblk"], kv=kv,
                    kv_scale="page" if kv == "fp8" else "unit")
    o.step([dict(sid=i, tokens=toks[i][a:b], pos=a, blocks=tabs[i], want=0) for i, a, b in pre[:1]])
    o.step([dict(sid=i, tokens=toks[i][a:b], pos=a, blocks=tabs[i], want=0) for i, a, b in pre[1:]])
    return o.step(smp["dec"])


def c3_parity(tol=5e-2):
    """Outside the timed region, on rank 0 at N = 1: the C3 shape with 2 of its 32 layers (its own GGUF, the same
    synthesis), the 64-sequence c3_sample decode step through the C ABI against the oracle. max_rel_err: the largest
    per-row max |a - b| / max |b|, checked at the fp8-KV tolerance of the parity tests (5e-2: e4m3's 3 mantissa bits
    make the oracle itself move by up to 0.028 at this shape when its inputs carry f16 roundings); tokens: the device
    argmax against the oracle's."""
    from goethe_engine_b200 import gck, synth
    t0 = time.time()
    spec = synth.Spec(**dict(SPEC8B, layers=2, name=SPEC8B["name"] + "-L2"))
    d = os.path.join(os.environ.get("GCK_BENCH_DIR", "/tmp/gck_bench"), f"{spec.name}-s{spec.seed}")
    pack, ws = synth.make(d, spec, ncol=B, maxctx=spec.ctx, kv="fp8", tune=dict(max_cols=2048, kv_scale="page"))
    smp = c3_sample()
    with gck.Backend(pack, ws, pool_blocks=smp["nblk"]) as be:
        got, greedy = c3_sample_run(be, smp)
    ref = c3_sample_oracle(ws[0], smp)
    a, r = got.astype(np.float64), ref.astype(np.float64)
    err = np.abs(a - r).max(-1) / np.abs(r).max(-1)
    top2 = np.sort(r, -1)[:, -2:]
    sure = (top2[:, 1] - top2[:, 0]) / np.abs(r).max(-1) > 2 * tol
    return {"workload": "C3 shape with 2 of 32 layers: one 64-sequence decode step (contexts 838-7969, 61 on the shared "
                        "prefix pages), Q4_K, fp8 page-scaled KV, vocabulary 128256",
            "rows": int(len(err)), "max_rel_err": round(float(err.max()), 6), "tolerance": tol,
            "within_tolerance": bool((err <= tol).all()),
            "tokens_equal": int((greedy == r.argmax(-1)).sum()),
            "tokens_equal_where_margin_exceeds_2tol": f"{int((greedy == r.argmax(-1))[sure].sum())}/{int(sure.sum())}",
            "device_argmax_equals_host_argmax": bool(np.array_equal(greedy, got.argmax(-1))),
            "seconds": round(time.time() - t0, 1)}


# ------------------------------------------------------------------------------------------- CPU baselines
def reference_module():
    """goethe_engine.ref and .backend from the reference installed offline in baseline/_ref, or None."""
    p = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(p, "goethe_engine")):
        return None
    if p not in sys.path:
        sys.path.insert(0, p)
    import goethe_engine.backend as Bk
    import goethe_engine.ref as R
    return R, Bk


class RefSample:
    """The reference's own CPU implementation of the path, ref.py's RefModel + TorchBackend (ref.py:18-126), on a
    bounded sample of the C3 decode step: the first `seqs` C3 sequences at their contexts, `layers` layers of the 8B
    shape (d 4096, 32/8 heads of 128, FFN 14336) and a head of VS rows; the step time is scaled to 32 layers and the
    full 128256-row head. RefModel draws its own seeded f32 weights (ref.py computes in f32 whatever the checkpoint's
    storage); the fp8 KV pool holds random finite e4m3 codes (a decode step's time does not depend on the values)."""

    VS, MAX_STEPS, TARGET_S = 8192, 200, 10.0

    def __init__(self, R, Bk, seqs=8, layers=2):
        import torch
        self.torch, self.Bk = torch, Bk
        self.m = R.RefModel(vocab=self.VS, d=4096, layers=layers, heads=32, kv_heads=8, ffn=14336, seed=0)
        self.ctx = contexts()[:seqs]
        tabs, k = [], 0
        for c in self.ctx:
            n = -(-(int(c) + 2 + self.MAX_STEPS) // 16)
            tabs.append(list(range(k, k + n)))
            k += n
        self.be = R.TorchBackend(self.m, num_blocks=k, block_size=16, kv="fp8", max_seqs=seqs)
        g = torch.Generator().manual_seed(2)
        for c in (self.be.kc, self.be.vc):
            c.view(torch.uint8).copy_(torch.randint(0, 0x78, c.shape, generator=g, dtype=torch.uint8))
        self.tabs, self.seqs, self.layers = tabs, seqs, layers

    def run(self):
        torch = self.torch
        cores = len(os.sched_getaffinity(0))
        prev = torch.get_num_threads()
        torch.set_num_threads(cores)          # torchrun sets one thread per rank; the sample uses every host core
        try:
            pos = [int(c) for c in self.ctx]
            n, t_sum = 0, 0.0
            with torch.no_grad():
                while n < self.MAX_STEPS and t_sum < self.TARGET_S:
                    work = [self.Bk.Work(i, [7], pos[i], self.tabs[i], 1) for i in range(self.seqs)]
                    t0 = time.perf_counter()
                    self.be.step(work)
                    t_sum += time.perf_counter() - t0
                    pos = [p + 1 for p in pos]
                    n += 1
                x = torch.ones(4096)
                t0 = time.perf_counter()
                for _ in range(3 * self.seqs):
                    self.m.head @ x
                t_head = (time.perf_counter() - t0) / 3
        finally:
            torch.set_num_threads(prev)
        t_all = t_sum / n
        per_step = max(t_all - t_head, 1e-9) * 32 / self.layers + t_head * 128256 / self.VS
        return {"value": round(self.seqs / per_step, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
                "sample": f"ref.py RefModel + TorchBackend (torch {torch.__version__}, {cores} threads): decode step of "
                          f"{self.seqs} C3 sequences (contexts {list(map(int, self.ctx))}), {self.layers}/32 layers and "
                          f"{self.VS}/128256 head rows, {n} steps timed ({t_sum:.1f}s, {t_all:.2f}s each), scaled to "
                          f"the full model: {per_step:.2f}s per step"}


class PortSample:
    """The oracle (numpy restatement of ref.py) on the same bounded sample: `seqs` C3 sequences, `layers` layers of
    the 8B shape with seeded N(0, 0.02) f32 weights, a head of VS rows, random finite e4m3 KV codes; scaled the same
    way."""

    VS, MAX_STEPS, TARGET_S = 8192, 40, 10.0

    def __init__(self, seqs=8, layers=2):
        from oracle.model import PagedOracle, Weights
        rng = np.random.default_rng(0)
        mk = lambda *s: (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02))
        lw = [dict(q=mk(4096, 4096), k=mk(1024, 4096), v=mk(1024, 4096), o=mk(4096, 4096), g=mk(14336, 4096),
                   u=mk(14336, 4096), dn=mk(4096, 14336)) for _ in range(layers)]
        self.head = mk(self.VS, 4096)
        w = Weights(self.head, self.head, lw, eps=1e-5, theta=5e5, heads=32, kv_heads=8)
        self.ctx = contexts()[:seqs]
        nb = int(sum(-(-(c + 2 + self.MAX_STEPS) // 16) for c in self.ctx))
        self.o = PagedOracle(w, num_blocks=nb, kv="fp8", kv_scale="page")
        self.o.kc[:] = rng.integers(0, 0x78, self.o.kc.shape, dtype=np.uint8)
        self.o.vc[:] = rng.integers(0, 0x78, self.o.vc.shape, dtype=np.uint8)
        tabs, k = [], 0
        for c in self.ctx:
            n = -(-(int(c) + 2 + self.MAX_STEPS) // 16)
            tabs.append(list(range(k, k + n)))
            k += n
        self.items = [dict(sid=i, tokens=[7], pos=int(c), blocks=tabs[i], want=1) for i, c in enumerate(self.ctx)]
        self.seqs, self.layers = seqs, layers

    def run(self):
        from threadpoolctl import threadpool_limits
        cores = len(os.sched_getaffinity(0))
        with threadpool_limits(limits=cores, user_api="blas"):
            for it, c in zip(self.items, self.ctx):
                it["pos"] = int(c)
            n, t_sum = 0, 0.0
            while n < self.MAX_STEPS and t_sum < self.TARGET_S:
                for it in self.items:
                    it["pos"] += 1
                t0 = time.perf_counter()
                self.o.step(self.items)
                t_sum += time.perf_counter() - t0
                n += 1
            h = np.ones((self.seqs, 4096), np.float32)
            t0 = time.perf_counter()
            for _ in range(3):
                h @ self.head.T
            t_head = (time.perf_counter() - t0) / 3
        t_all = t_sum / n
        per_step = max(t_all - t_head, 1e-9) * 32 / self.layers + t_head * 128256 / self.VS
        return {"value": round(self.seqs / per_step, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                "sample": f"numpy oracle decode step of {self.seqs} C3 sequences, {self.layers}/32 layers and "
                          f"{self.VS}/128256 head rows, {n} steps timed ({t_sum:.1f}s, {t_all:.2f}s each), scaled to the "
                          f"full model: {per_step:.2f}s per step"}


def cpu_baseline():
    """ref.py itself (kind "reference") when the reference is installed in baseline/_ref, with the numpy port as a
    second figure; the port alone otherwise."""
    port = PortSample().run()
    ref = reference_module()
    if ref is None:
        port["note"] = "baseline/_ref absent: the reference's ref.py could not be imported"
        return port
    out = RefSample(*ref).run()
    out["port"] = port
    return out


SPEC8B_Q8 = dict(SPEC8B, wtype="q8_0", ctx=4096, name="llama3-8b-shape-q80")


def open_q8(tune, ncol, bucket="b200.BI.main", **extra):
    """The 8B shape with Q8_0 weights (C2, C4) and f16 KV in one bucket; returns (pack dir, [weights])."""
    from goethe_engine_b200 import build, gck, synth
    build.build()
    spec = synth.Spec(**SPEC8B_Q8)
    d = os.path.join(os.environ.get("GCK_BENCH_DIR", "/tmp/gck_bench"), f"{spec.name}-s{spec.seed}")
    t0 = time.time()
    synth.make(d, spec, buckets=[dict(id=bucket, ncol=ncol, maxctx=spec.ctx, kv="f16", tune=tune, **extra)])
    print(f"[bench] model ready in {d} ({time.time() - t0:.1f}s)", file=sys.stderr, flush=True)
    return d, [os.path.join(d, "model.gguf")]


def stats_api(be):
    import ctypes as C

    class Stats(C.Structure):
        _fields_ = [("size", C.c_uint32), ("steps", C.c_uint32), ("launches", C.c_uint64), ("forward_ms", C.c_double),
                    ("class_ms", C.c_double * 16), ("class_launches", C.c_uint64 * 16), ("h2d_bytes", C.c_uint64),
                    ("graph_steps", C.c_uint32), ("graph_captures", C.c_uint32), ("gemm_pairs", C.c_uint32)]
    be.L.gck_stats_enable.argtypes = [C.c_void_p, C.c_uint32]
    be.L.gck_stats_read.argtypes = [C.c_void_p, C.c_void_p]

    def read():
        st = Stats(size=C.sizeof(Stats))
        be.L.gck_stats_read(be.h, C.byref(st))
        return st
    return lambda prof=False: be.L.gck_stats_enable(be.h, 0xFFFF if prof else 0), read


CLASS_NAMES = ["embed", "rmsnorm", "gemm_qkv", "rope_kv", "attention", "attn_combine", "gemm_o", "gemm_gateup",
               "gemm_down", "gemm_head", "argmax", "splitk_reduce", "tp_allreduce", "a8_quant"]


def print_classes(st, steps, label=""):
    """The per-class device-time table (events around each launch) on stderr."""
    tot = sum(st.class_ms[i] for i in range(len(CLASS_NAMES)))
    lines = [f"{n:14s} {st.class_ms[i] / steps:8.3f} ms/step  {st.class_launches[i] // max(1, steps):5d} "
             f"launches/step  {100 * st.class_ms[i] / max(tot, 1e-9):5.1f}%" for i, n in enumerate(CLASS_NAMES)]
    print(f"[bench] {label}per-class device time (events around each launch):\n" + "\n".join(lines) +
          f"\n  sum {tot / steps:.3f} ms/step, step {st.forward_ms / steps:.3f} ms", file=sys.stderr, flush=True)


def run_c2(args):
    """C2: the 8B shape, Q8_0 weights, f16 KV, one sequence decoding at context 2048 (HBM-bound: every weight byte and
    the KV once per token). A single-stream bucket (ncol 1, not batched) with "tolerance" determinism, the one the
    reference's single-stream selection takes for one sequence (pack.py:619-633): its decode runs the GEMV."""
    import torch
    from goethe_engine_b200 import gck
    d, ws = open_q8(dict(max_cols=2048), 1, bucket="b200.FAST.single", determinism="tolerance", batch=False)
    ctx, steps_total = 2048, args.warmup + args.steps
    per_seq = -(-(ctx + steps_total + 1) // 16)
    be = gck.Backend(d, ws, buckets=("b200.FAST.single",), pool_blocks=per_seq + 4)
    on, read = stats_api(be)
    rng = np.random.default_rng(0)
    toks = [int(x) for x in rng.integers(1, 128000, ctx)]
    tab = np.arange(per_seq, dtype=np.uint32)
    be.step([gck.Work(0, toks[:-1], 0, tab, 0)])
    last, pos = toks[-1], ctx - 1
    for _ in range(args.warmup):
        last = int(be.decode([0], [last], [pos], [tab])[0])
        pos += 1
    torch.cuda.synchronize()
    on(args.profile)
    window = bool(os.environ.get("GCK_PROFILE_WINDOW"))   # the CUDA profiler window covers the first timed step
    with Clocks(0) as clk:
        t0 = time.perf_counter()
        for k in range(args.steps):
            if window and k == 0:
                torch.cuda.profiler.start()
            last = int(be.decode([0], [last], [pos], [tab])[0])
            if window and k == 0:
                torch.cuda.profiler.stop()
            pos += 1
        wall = time.perf_counter() - t0
    st = read()
    if args.profile:
        print_classes(st, args.steps)
    be.close()
    ms = st.forward_ms / args.steps
    wbytes = weight_bytes(SPEC8B_Q8) * 272 // 144         # Q8_0: 34 B per 32 weights
    kv = (ctx + args.warmup + args.steps / 2) * 32 * 8 * 128 * 2 * 2
    hbm = peaks().get("hbm_gbs", 6650.0)
    gbs = (wbytes + kv) / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "decode tok/s (8B Q8_0, batch 1, f16 KV)", "value": round(1e3 / ms, 2), "unit": "tok/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 x f16 -> f32; f16 KV",
        "data": "synthetic (seeded N(0,0.02) weights, uniform tokens)",
        "config": {"workload": "C2: Llama-3-8B shape, Q8_0 weights, a16, f16 paged KV, one sequence at context 2048",
                   "bucket": "single-stream, determinism tolerance (GEMV decode)",
                   "batch": 1, "context": ctx, "l2": "inputs larger than L2, no flush"},
        "e2e": {"value": round(args.steps / wall, 2), "unit": "tok/s", "h2d_bytes_per_step": int(st.h2d_bytes // max(1, st.steps)),
                "d2h_bytes_per_step": 8, "path": "gc_step through the C ABI (ctypes), host buffers",
                "h2d_source": "the library's own count of its plan and block-table patch uploads (gck_stats.h2d_bytes)",
                "captured_steps": f"{st.graph_steps} of {st.steps} timed steps replayed a captured CUDA graph"},
        "step_roofline": {"algorithmic_bytes": int(wbytes + kv), "achieved_gbs": round(gbs, 1),
                          "frac_of_measured": round(gbs / hbm, 4), "frac_of_8tbs": round(gbs / 8000, 4)},
        "gpu_launches": int(st.launches), "clocks": clk.summary()}), flush=True)


def run_c4(args):
    """C4: the 8B shape, a8 activations (every GEMM input quantized per token to int8, bucket field act "a8") x Q8_0
    weights, f16 KV; prefill of 32 sequences x 2048 uniform tokens in 2048-token steps (tensor-bound), then one tree
    verify of a 16-node draft tree per sequence (anchor + 15 drafts, each parent uniform over earlier nodes of depth
    < 4, random.Random(1) per sequence). --act a16 runs the same workload with f16 activations."""
    import random
    import torch
    from goethe_engine_b200 import gck
    d, ws = open_q8(dict(max_cols=2048), 32, bucket="b200.BI.a8" if args.act == "a8" else "b200.BI.main", act=args.act)
    n_seq, ctx = 32, 2048
    per_seq = -(-(ctx + 64) // 16)
    be = gck.Backend(d, ws, pool_blocks=n_seq * per_seq + 4, buckets=("b200.BI.a8" if args.act == "a8" else "b200.BI.main",))
    on, read = stats_api(be)
    rng = np.random.default_rng(0)
    toks = [[int(x) for x in rng.integers(1, 128000, ctx)] for _ in range(n_seq)]
    tabs = [np.arange(i * per_seq, (i + 1) * per_seq, dtype=np.uint32) for i in range(n_seq)]
    # warm-up: one sequence's prefill
    be.step([gck.Work(99, toks[0], 0, tabs[0], 0)])
    be.release(99)
    torch.cuda.synchronize()
    on(args.profile)
    window = bool(os.environ.get("GCK_PROFILE_WINDOW"))   # the CUDA profiler window: the first prefill, the first verify
    with Clocks(0) as clk:
        t0 = time.perf_counter()
        for i in range(n_seq):
            if window and i == 0:
                torch.cuda.profiler.start()
            be.step([gck.Work(i, toks[i], 0, tabs[i], 1, greedy=True)])
            if window and i == 0:
                torch.cuda.profiler.stop()
        wall_p = time.perf_counter() - t0
    st_p = read()
    if args.profile:
        print_classes(st_p, n_seq, "prefill ")
    parents = []
    r = random.Random(1)
    depth = [0]
    par = [-1]
    for i in range(1, 16):
        cands = [j for j in range(i) if depth[j] < 4]
        pj = r.choice(cands)
        par.append(pj)
        depth.append(depth[pj] + 1)
    parents = par
    draft = [[int(x) for x in rng.integers(1, 128000, 16)] for _ in range(n_seq)]
    verify = [gck.Work(i, draft[i], ctx, tabs[i], 16, greedy=True, parents=parents) for i in range(n_seq)]
    be.step(verify)                      # warm
    on(args.profile)
    t0 = time.perf_counter()
    for k in range(args.steps):
        if window and k == 0:
            torch.cuda.profiler.start()
        be.step(verify)
        if window and k == 0:
            torch.cuda.profiler.stop()
    wall_v = time.perf_counter() - t0
    st_v = read()
    if args.profile:
        print_classes(st_v, args.steps, "verify ")
    be.close()
    pre_ms = st_p.forward_ms
    sp = SPEC8B_Q8
    lin = sp["layers"] * sp["d"] * (sp["d"] * 2 + 2 * sp["d"] // sp["heads"] * sp["kv_heads"] + 3 * sp["ffn"])
    # linear layers for every token, causal QK^T and PV (2 x 2 x pos x d per layer), the head for the wanted row
    flop = n_seq * (2 * lin * ctx + sp["layers"] * 4 * sp["d"] * ctx * (ctx + 1) / 2 + 2 * sp["d"] * sp["vocab"])
    tc = peaks().get("bf16_tflops_sustained", 1400.0)
    ver_ms = st_v.forward_ms / args.steps
    # verify step: every weight byte once, every sequence's KV (ctx rows, f16, all layers) once; FLOPs of 512 token rows
    # through the linear layers, the head for 16 wanted rows per sequence, attention over ctx + path rows
    v_bytes = weight_bytes(sp) * 272 // 144 + n_seq * ctx * sp["layers"] * sp["kv_heads"] * (sp["d"] // sp["heads"]) * 2 * 2
    v_flop = 2 * lin * n_seq * 16 + 2 * sp["d"] * sp["vocab"] * n_seq * 16 + sp["layers"] * 4 * sp["d"] * ctx * n_seq * 16
    print(json.dumps({
        "metric": f"prefill tok/s (8B {args.act} x Q8_0, 32 x 2048) and tree-verify step ms (32 x 16-node trees)",
        "value": round(n_seq * ctx / (pre_ms / 1e3), 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": 1, "ms_per_step": round(pre_ms / n_seq, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": ("per-token int8 activations (f16-held codes) x q8_0 -> f32, scale in the epilogue"
                                       if args.act == "a8" else "q8_0 x f16 -> f32") + "; f16 KV",
        "data": "synthetic (seeded N(0,0.02) weights, uniform tokens, seeded draft trees)",
        "config": {"workload": f"C4: Llama-3-8B shape, {args.act} activations x Q8_0 weights, prefill 32 x 2048 then "
                               "verify 32 x 16-node trees",
                   "batch": n_seq, "context": ctx, "tree_parents": parents, "l2": "inputs larger than L2, no flush",
                   "gemm_cta_pairs": int(st_p.gemm_pairs)},
        "roofline": {"bound": "tensor", "achieved": round(flop / (pre_ms / 1e3) / 1e12, 1), "peak": tc, "unit": "TFLOP/s",
                     "frac": round(flop / (pre_ms / 1e3) / 1e12 / tc, 4),
                     "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained"},
        "verify": {"ms_per_step": round(ver_ms, 4), "tokens_per_step": n_seq * 16,
                   "tok_per_s": round(n_seq * 16 / (ver_ms / 1e3), 1), "e2e_ms_per_step": round(wall_v / args.steps * 1e3, 4),
                   # mixed bound: the step's weights and KV bytes, and its linear + head + attention FLOPs
                   "bytes": int(v_bytes), "achieved_gbs": round(v_bytes / (ver_ms / 1e3) / 1e9, 1),
                   "frac_of_measured_hbm": round(v_bytes / (ver_ms / 1e3) / 1e9 / peaks().get("hbm_gbs", 6650.0), 4),
                   "flop": v_flop, "achieved_tflops": round(v_flop / (ver_ms / 1e3) / 1e12, 1),
                   "frac_of_sustained_bf16": round(v_flop / (ver_ms / 1e3) / 1e12 / tc, 4)},
        "e2e": {"value": round(n_seq * ctx / wall_p, 1), "unit": "tok/s", "h2d_bytes_per_step": int(ctx * 4 + per_seq * 4),
                "d2h_bytes_per_step": 4, "path": "gc_step through the C ABI (ctypes), host buffers"},
        "gpu_launches": int(st_p.launches + st_v.launches), "clocks": clk.summary()}), flush=True)


SPEC70B = dict(vocab=128256, d=8192, layers=80, heads=64, kv_heads=8, ffn=28672, eps=1e-5, theta=5e5, wtype="q4_k",
               std=0.02, seed=0, ctx=4096 + 64, name="llama3-70b-shape-q4k")
B70, CTX70 = 128, 4096


def c5_measure(tp, steps, warmup, prefill=True, profile_steps=3):
    """The C5 decode step on one tensor-parallel handle over devices 0 .. tp-1 (one process; the library runs a thread
    per rank and its own all-reduce over peer memory). Returns the measurement as a dict: device and e2e tok/s, the step
    time, the per-GPU HBM roofline, and the per-class device time of profile_steps more steps (events around every
    launch) with the all-reduce separated and the largest class named. prefill False leaves the 4096-token contexts'
    KV pages as the pool's zero bytes (a decode step reads every page and does every product whatever the values; the
    prefill is not part of the metric), which keeps the scaling run short."""
    import torch
    from goethe_engine_b200 import build, gck, synth
    build.build()
    spec = synth.Spec(**SPEC70B)
    d = os.path.join(os.environ.get("GCK_BENCH_DIR", "/tmp/gck_bench"), f"{spec.name}-s{spec.seed}")
    t0 = time.time()
    synth.make(d, spec, buckets=[dict(id="b200.BI.main", ncol=B70, maxctx=spec.ctx, kv="fp8", tp=tp,
                                      tune=dict(max_cols=2048, kv_scale="page"))])
    t_model = time.time() - t0
    steps_total = warmup + steps + profile_steps
    per_seq = -(-(CTX70 + steps_total + 1) // 16)
    t0 = time.time()
    be = gck.Backend(d, [os.path.join(d, "model.gguf")], pool_blocks=B70 * per_seq + 16, device=0)
    t_open = time.time() - t0
    stats = Stats(be)
    rng = np.random.default_rng(0)
    toks = [[int(x) for x in rng.integers(1, 128000, CTX70)] for _ in range(B70)]
    tables = [np.arange(i * per_seq, (i + 1) * per_seq, dtype=np.uint32) for i in range(B70)]
    t0 = time.time()
    if prefill:
        cap = be.layout.max_cols
        queue = [[i, 0] for i in range(B70)]
        while any(q[1] < CTX70 - 1 for q in queue):
            budget, items = cap, []
            for q in queue:
                if q[1] >= CTX70 - 1 or budget == 0:
                    continue
                n = min(budget, CTX70 - 1 - q[1])
                items.append(gck.Work(q[0], toks[q[0]][q[1]:q[1] + n], q[1], tables[q[0]], 0))
                q[1] += n
                budget -= n
            be.step(items)
    t_prefill = time.time() - t0
    last = np.array([t[-1] for t in toks], np.int32)
    pos = np.full(B70, CTX70 - 1, np.int64)
    sids = np.arange(B70)

    def step():
        last[:] = be.decode(sids, last, pos, tables)
        pos[:] += 1
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    stats.enable(0)
    with Clocks(0) as clk:
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        wall = time.perf_counter() - t0
    st = stats.read()
    stats.enable(0xFFFF)
    for _ in range(profile_steps):
        step()
    sp = stats.read()
    be.close()
    dev_s = st.forward_ms / 1e3
    ms_step = dev_s / steps * 1e3
    wbytes = weight_bytes(SPEC70B)
    kv = (CTX70 + warmup + steps / 2) * B70 * 2 * 8 * 128 * SPEC70B["layers"]
    per_gpu = (wbytes + kv) / tp
    hbm = peaks().get("hbm_gbs", 6650.0)
    cls = {n: round(sp.class_ms[i] / profile_steps, 4) for i, n in enumerate(CLASS_NAMES) if sp.class_launches[i]}
    top = max(cls, key=cls.get) if cls else None
    return {"tp": tp, "value": round(B70 * steps / dev_s, 1), "unit": "tok/s", "ms_per_step": round(ms_step, 4),
            "e2e": round(B70 * steps / wall, 1), "steps": steps, "warmup": warmup,
            "bytes_per_gpu": int(per_gpu), "achieved_gbs_per_gpu": round(per_gpu / (ms_step / 1e3) / 1e9, 1),
            "frac_of_measured_hbm_per_gpu": round(per_gpu / (ms_step / 1e3) / 1e9 / hbm, 4),
            "class_ms_per_step": cls, "allreduce_ms_per_step": cls.get("tp_allreduce", 0.0),
            "largest_class": top,
            "class_timing": f"events around every launch, {profile_steps} steps after the timed region (upper bounds)",
            "gpu_launches": int(st.launches), "clocks": clk.summary(),
            "kv": "prefilled contexts" if prefill else "4096-token contexts, pages left as the pool's zero bytes",
            "setup_s": {"model": round(t_model, 1), "open": round(t_open, 1), "prefill": round(t_prefill, 1)}}


def run_c5(args):
    """C5: the 70B shape (Q4_K, fp8 paged KV with per-page scales), 128 sequences at context 4096 each (uniform tokens,
    seed 0), greedy decode on one tensor-parallel handle over --gpus devices (one process, NCCL all-reduces inside)."""
    tp = args.gpus
    r = c5_measure(tp, args.steps, args.warmup, prefill=True, profile_steps=3 if args.profile else 1)
    res = {
        "metric": "decode tok/s (70B Q4_K, batch 128, fp8 KV, tensor parallel)", "value": r["value"],
        "unit": "tok/s", "n_gpus": tp, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "q4_k x f16 -> f32; fp8 e4m3 KV",
        "data": "synthetic (seeded N(0,0.02) weights, uniform tokens)",
        "config": {"workload": "C5: Llama-3-70B shape, Q4_K weights, fp8 paged KV (per-page scale), 128 sequences at "
                               "context 4096, greedy decode", "batch": B70, "context": CTX70, "layers": SPEC70B["layers"],
                   "parallelism": f"tp{tp} (one handle; after o_proj and down_proj a deterministic all-reduce over "
                                  "peer memory, NCCL where peer access is missing)",
                   "l2": "inputs larger than L2, no flush"},
        "e2e": {"value": r["e2e"], "unit": "tok/s", "h2d_bytes_per_step": int(B70 * (CTX70 // 16 + 8) * 4 + B70 * 64),
                "d2h_bytes_per_step": B70 * 4, "path": "gc_step through the C ABI (ctypes), host buffers"},
        "step_roofline": {"bytes_per_gpu": r["bytes_per_gpu"], "achieved_gbs_per_gpu": r["achieved_gbs_per_gpu"],
                          "frac_of_measured": r["frac_of_measured_hbm_per_gpu"]},
        "tp_detail": r, "gpu_launches": r["gpu_launches"], "clocks": r["clocks"]}
    print(json.dumps(res), flush=True)


def collectives(world, backend="nccl", timeout_s=600):
    """The benchmark's only cross-rank steps, for one process per GPU (torchrun's RANK / WORLD_SIZE / MASTER_*): a
    barrier, and the max over ranks of a time (the job takes as long as its slowest rank). Replicas exchange no data.
    The process group's timeout ends a rank that waits for one which never arrives with an error. nccl on the GPU
    box; gloo (host tensors) for the CPU tests of this logic. Returns (barrier, maxreduce)."""
    if world == 1:
        return (lambda: None), (lambda x: x)
    import datetime
    import torch
    import torch.distributed as dist
    if backend == "nccl":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    dev = "cuda" if backend == "nccl" else "cpu"

    def barrier():
        dist.barrier()

    def maxreduce(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return barrier, maxreduce


def aggregate(units_per_rank, world, dev_s_max, wall_s_max):
    """Whole-job throughput: the units all ranks processed over the slowest rank's time (device, and host clock around
    the C-ABI calls for e2e)."""
    units = units_per_rank * world
    return units / dev_s_max, units / wall_s_max


def run_reference(args, rank, world):
    """The reference arm: ref.py's RefModel + TorchBackend (the reference's CPU implementation of the path) on the
    bounded C3 sample, all host cores, rank 0 only; the numpy port where baseline/_ref is absent. Nothing of this
    repository's native code is loaded."""
    if rank != 0:
        return
    ref = reference_module()
    smp = RefSample(*ref) if ref is not None else PortSample()
    cb, vals = None, []
    for _ in range(max(1, min(args.steps, 3))):
        cb = smp.run()
        vals.append(cb["value"])
    v = float(np.median(vals))
    cb["value"] = v
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                      "dtype": "f32 weights and activations (ref.py), fp8 e4m3 KV" if ref else "f32 (numpy port), fp8 KV",
                      "data": "synthetic",
                      "config": {"workload": "C3 decode step, bounded CPU sample (cpu_baseline.sample)"},
                      "cpu_baseline": cb, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0,
                                                   "d2h_bytes_per_step": 0}}), flush=True)


def main():
    # rank 0 prints one JSON line on stdout: NCCL's banner and logs (NCCL_DEBUG) go to a file instead
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    os.environ.setdefault("NCCL_DEBUG_FILE", os.path.join(tempfile.gettempdir(), "gck_nccl.%h.%p.log"))
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU leg (parity check and CPU baselines)")
    ap.add_argument("--no-tp", action="store_true", help="N > 1: skip the 70B tensor-parallel sub-record")
    ap.add_argument("--act", default="a8", choices=["a8", "a16"], help="c4: activation type (BASELINE config 4: a8)")
    ap.add_argument("--profile", action="store_true", help="time every kernel class (stderr table)")
    ap.add_argument("--workload", default="c3", choices=["c2", "c3", "c4", "c5"],
                    help="c3: the headline (8B, replicas over --gpus); c2: 8B Q8_0 batch-1 decode; c4: 8B Q8_0 prefill "
                         "and tree verify; c5: 70B tensor parallel over --gpus in one process")
    ap.add_argument("--layers", type=int, default=32,
                    help="layers of the 8B shape (default 32; fewer only for small profiling cases, not a headline)")
    args = ap.parse_args()
    if args.layers != 32:
        for sp, full in ((SPEC8B, 32), (SPEC8B_Q8, 32), (SPEC70B, 80)):
            sp["layers"] = min(args.layers, full)
            sp["name"] += f"-L{sp['layers']}"
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    if args.workload in ("c2", "c4"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": f"{args.workload}: the CPU baseline is measured on C3 "
                              "(bench.py --impl reference)"}), flush=True)
            return
        return run_c2(args) if args.workload == "c2" else run_c4(args)
    if args.workload == "c5":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "C5 (70B) on the CPU needs about 278 GB of f32 weights: "
                              "not run"}), flush=True)
            return
        return run_c5(args)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    barrier, maxreduce = collectives(world)
    try:
        res = run_mine(args, rank, world, barrier, maxreduce)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if rank != 0:
        return          # the replica ranks are done: their GPUs are free for rank 0's tensor-parallel handle
    if world > 1 and not args.no_tp:
        res["tp"] = tp_record(args, world)
    print(json.dumps(res), flush=True)


def tp_record(args, n):
    """The 70B shape (C5) on one tensor-parallel handle over the job's n GPUs, run by rank 0 after the C3 replicas
    (the other ranks have exited): BASELINE's TP curve. An error here is reported in the record, not raised, so the
    headline line is still printed."""
    try:
        r = c5_measure(n, args.steps, args.warmup, prefill=False, profile_steps=2)
        r["workload"] = ("C5: Llama-3-70B shape, Q4_K, fp8 paged KV, 128 sequences at context 4096, greedy decode, "
                         f"tensor parallel over {n} GPUs (heads and FFN columns split, all-reduce after o_proj and "
                         "down_proj)")
        return r
    except Exception as e:                                   # noqa: BLE001
        return {"tp": n, "error": f"{type(e).__name__}: {e}"}


if __name__ == "__main__":
    main()

"""Per-phase timeline of the resident 28-layer decode, from the phase-trace build.

    python macbook-hardware-linux-lab_b200/phase_trace.py [--steps 4] [--warmup 20]

Builds libgqa_b200_trace.so (the library with -DGQA_PHASE_TRACE) when it is
missing or stale, runs the default benchmark's workload through it (one
sequence, 28 layers of 12 q / 2 KV heads, t_max 4096, a CUDA graph of the 28
layer calls with the device position advanced, positions from 3840) and prints,
for the layers of the middle steps, the median over launches of each phase's
median CTA time in microseconds after the launch's median dependency release,
and the layer period.  Needs a GPU.  The traced build's stamps cost a few
percent, so its period is a little longer than the benchmark's.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys
from collections import defaultdict

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
PHASES = ["dependency released", "q staged", "warp 0 loop done", "partial stored",
          "every merging warp's slice sums in shared memory", "merged slice stored"]
WORDS = 4 + len(PHASES)


def _load(trace_lib):
    os.environ["GQA_LIB"] = trace_lib
    sys.path.insert(0, REPO)
    import __graft_entry__
    return __graft_entry__.load_package()


def collect(g, steps, warmup, layers=28, t_max=4096, pos_lo=3840, pos_hi=4096):
    import numpy as np
    import torch
    lib = g.lib()
    with g.Context(t_max=t_max) as ctx:
        caches = torch.empty((layers, 2, 2, t_max, 128), device="cuda")
        ctx.fill_normal(caches, caches.numel(), 4242, g.seeded.K_CACHE)
        kvs = [g.kv_of(caches[l, 0], caches[l, 1]) for l in range(layers)]
        qkv = torch.empty((layers, 2048), device="cuda")
        ctx.fill_normal(qkv, qkv.numel(), 4242, g.seeded.QKV)
        out = torch.empty((layers, 1536), device="cuda")
        d_pos = torch.tensor([pos_lo], dtype=torch.int32, device="cuda")
        ctx.reserve(1, t_max)
        graph = ctx.graph_create_layers(kvs, qkv, 2048, out, 1536, d_pos, advance=True,
                                        wrap_lo=pos_lo, wrap_hi=pos_hi)
        stream = torch.cuda.current_stream()
        for _ in range(warmup):
            graph.launch(stream)
        torch.cuda.synchronize()
        n = ctypes.c_int(0)
        g.gqa._check(lib.gqa_phase_trace_read(None, 0, 1, ctypes.byref(n)))
        for _ in range(steps):
            graph.launch(stream)
        torch.cuda.synchronize()
        g.gqa._check(lib.gqa_phase_trace_read(None, 0, 0, ctypes.byref(n)))
        rec = np.zeros((n.value, WORDS), dtype=np.uint64)
        g.gqa._check(lib.gqa_phase_trace_read(rec.ctypes.data, n.value, 1, ctypes.byref(n)))
        graph.destroy()
        if ctx.device_status() != 0:
            raise RuntimeError("device status set during the traced run")
    return rec.astype(np.int64)


def max_sm_mhz():
    import pynvml
    pynvml.nvmlInit()
    try:
        h = pynvml.nvmlDeviceGetHandleByIndex(0)
        return float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
    finally:
        pynvml.nvmlShutdown()


def analyse(rec, steps, clock_ghz, layers=28):
    import numpy as np
    tag, g0, c0 = rec[:, 0], rec[:, 2], rec[:, 3]
    ev = rec[:, 4:].astype(np.float64)
    t = (ev - c0[:, None]) / clock_ghz + g0[:, None]  # ns, common axis
    t[rec[:, 4:] == 0] = np.nan
    by_tag = defaultdict(list)
    for i in range(len(rec)):
        by_tag[tag[i]].append(i)
    launches = []
    for idx in by_tag.values():
        per = len(idx) // steps
        for s in range(steps):
            launches.append(np.array(idx[s * per:(s + 1) * per]))
    launches.sort(key=lambda ix: g0[ix].min())
    release = [np.nanmedian(t[ix, 0]) for ix in launches]
    first, last = layers + 1, len(launches) - layers - 1  # skip the first and last steps
    rows = []
    for li in range(max(first, 1), max(last, 2)):
        ix = launches[li]
        rows.append([np.nanmedian(t[ix, j]) - release[li] for j in range(len(PHASES))])
    rows = np.array(rows) / 1000.0
    period = np.median(np.diff(release[max(first, 1):max(last, 2)])) / 1000.0
    # Each CTA's own phases after its own release, from clock64 differences
    # alone (exact; the globaltimer that places CTAs on a common axis ticks
    # in coarse steps, so the table above moves in those steps).
    steady = np.concatenate([launches[li] for li in range(max(first, 1), max(last, 2))])
    own = (ev[steady] - ev[steady, :1]) / clock_ghz / 1000.0
    own[rec[steady, 4:] == 0] = np.nan
    return np.nanmedian(rows, axis=0), period, len(rows), np.nanmedian(own, axis=0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--clock-mhz", type=float, default=0.0,
                    help="SM clock for clock64 stamps (default: the device's maximum)")
    ap.add_argument("--save", default="", help="also write the raw records (.npy) here")
    args = ap.parse_args()
    sys.path.insert(0, HERE)
    import build  # noqa: E402  (this directory's build.py)
    trace_lib = build.build(phase_trace=True)
    g = _load(trace_lib)
    import torch
    rec = collect(g, args.steps, args.warmup)
    if args.save:
        import numpy as np
        np.save(args.save, rec)
    mhz = args.clock_mhz or max_sm_mhz()
    med, period, n, own = analyse(rec, args.steps, mhz / 1000.0)
    print(f"resident28 phase trace: {len(rec)} CTA records, {n} steady-state launches, "
          f"SM clock {mhz:.0f} MHz for clock64 stamps, {torch.cuda.get_device_name(0)}")
    print("| phase | us after the launch's median release (median CTA) | us after the CTA's own release (median, exact) |")
    print("|---|---|---|")
    for name, v, o in zip(PHASES, med, own):
        print(f"| {name} | {v:.2f} | {o:.3f} |")
    print(f"| layer period (release to next release) | {period:.2f} |")


if __name__ == "__main__":
    main()

"""Benchmark of the fp32 GQA decode attention path on B200.

Default workload (one line of JSON on rank 0): the 28-layer resident decode --
per GPU one sequence, 28 layers of 12 q / 2 KV heads, d = 128, an fp32 KV cache
of t_max = 4096 rows per layer (235 MB), and decode steps at positions
3840..4095 (each step: RoPE + append + attention in all 28 layers; the window
wraps after 256 steps).  A step is one replay of a CUDA graph holding the 28
layer calls; inputs are resident in HBM.

  value    KV-read GB/s: algorithmic K+V bytes (2048 B per attended row per
           layer) of all ranks / max-over-ranks device time of the timed steps
  e2e      the same metric through the C ABI with HOST buffers: each step
           copies its 28 x 2048 fp32 q/k/v rows from pinned host memory,
           replays the graph and copies the 28 x 1536 outputs back
  roofline dominant kernel (decode_split_kernel) against the measured HBM peak
  cpu_baseline  the reference's own CPU attention (oracle/_ref, compiled from
           its sources) on this host's cores, on a bounded sample

Multi-GPU (torchrun, one process per GPU): every rank decodes its own
sequence (sharding by sequence, no collective on the data path); "scaling":
"weak".  --impl reference runs the reference's CPU implementation instead
(rank 0 only).  Other workloads (--workload batched|long|single) measure the
remaining decode configurations.
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "GQA decode attn: KV-read HBM GB/s (% of peak) and tok/s at 1/2/4/8 B200"
N_Q, N_KV, D = 12, 2, 128
ROW_BYTES = 2 * N_KV * D * 4  # K + V bytes of one attended position, all KV heads (2048)
QKV_W, OUT_W = (N_Q + 2 * N_KV) * D, N_Q * D
HBM_FALLBACK = 6650.0

WORKLOADS = {
    "resident28": dict(layers=28, t_max=4096, pos_lo=3840, pos_hi=4096, seqs=1),
    "batched": dict(layers=1, seqs=64, len_lo=256, len_hi=8192, window=256),
    "long": dict(layers=1, seqs=256, t_max=32768, window=64),
    "single": dict(layers=1, t_max=512, pos_lo=511, pos_hi=512, seqs=1),
    "long1": dict(layers=1, seqs=1, t_max=32768, window=64),
    "prefill": dict(layers=1, seqs=8, t_max=2048),
    "block28": dict(layers=28, t_max=4096, pos_lo=3840, pos_hi=4096, seqs=1),
    "layer28": dict(layers=28, t_max=4096, pos_lo=3840, pos_hi=4096, seqs=1),
    "head": dict(layers=0, t_max=1, seqs=1, vocab=151936),
    "token28": dict(layers=28, t_max=4096, pos_lo=3840, pos_hi=4096, seqs=1, vocab=151936),
    # Qwen2.5-0.5B attention shape (head_dim 64, 14 q / 2 KV heads), 24 layers
    "resident05b": dict(layers=24, t_max=4096, pos_lo=3840, pos_hi=4096, seqs=1, n_q=14, n_kv=2,
                        d=64),
    # the Qwen2.5-0.5B model's ends (Q8_0 head) and its whole greedy step
    "head05b": dict(layers=0, t_max=1, seqs=1, vocab=151936, n_q=14, n_kv=2, d=64, model="0.5b"),
    "token24_05b": dict(layers=24, t_max=4096, pos_lo=3840, pos_hi=4096, seqs=1, vocab=151936,
                        n_q=14, n_kv=2, d=64, model="0.5b"),
}

BLOCK_METRIC = ("GQA attention block (RMSNorm, Q4_0 QKV + bias, attention, Q4_0 Wo + residual): "
                "HBM GB/s of KV + weights and tok/s")
Q4_ROW = (1536 // 32) * 18  # bytes of one Q4_0 row of d_model = 1536 inputs
BLOCK_WEIGHT_BYTES = (QKV_W + OUT_W) * Q4_ROW + (QKV_W + OUT_W) * 4  # W_qkv, W_o, b_qkv, gamma
D_FFN = 8960
FFN_WEIGHT_BYTES = 2 * D_FFN * Q4_ROW + OUT_W * (D_FFN // 32) * 18 + OUT_W * 4  # gate, up, down, gamma
LAYER_METRIC = ("decoder layer step (attention block + RMSNorm/SwiGLU/down FFN, Q4_0): HBM GB/s "
                "of KV + weights and tok/s")

PREFILL_METRIC = "GQA causal prefill: bf16 tensor-core TFLOP/s (fp32 accumulation)"
VOCAB = 151936
HEAD_BYTES = VOCAB * 1260 + OUT_W * 4 * 2  # Q6_K output.weight, gamma_output, state
HEAD_METRIC = ("Q6_K LM head (output RMSNorm, 151936x1536 GEMV, greedy pick): HBM GB/s of "
               "weights and logits/s")
TOKEN_METRIC = ("whole-model greedy decode step (Q4_0 embedding, 28 decoder layers, Q6_K LM head, "
                "pick): tok/s and HBM GB/s of KV + weights")
# Qwen2.5-0.5B sizes (generate_stream_05b.c:19-35)
D05, QKV05, DFFN05 = 896, 1152, 4864
Q4_ROW05 = (D05 // 32) * 18
ROW05 = 2 * 2 * 64 * 4  # K + V bytes of one attended position, both KV heads (1024)
BLOCK05_BYTES = (QKV05 + D05) * Q4_ROW05 + (QKV05 + D05) * 4
FFN05_BYTES = 2 * DFFN05 * Q4_ROW05 + D05 * (DFFN05 // 32) * 18 + D05 * 4
HEAD05_BYTES = VOCAB * 952 + D05 * 4 * 2  # Q8_0 output.weight, gamma_output, state
HEAD05_METRIC = ("Q8_0 LM head of Qwen2.5-0.5B (output RMSNorm, 151936x896 GEMV, greedy pick): "
                 "HBM GB/s of weights and logits/s")
TOKEN05_METRIC = ("Qwen2.5-0.5B whole-model greedy decode step (Q4_0 embedding, 24 decoder layers, "
                  "Q8_0 LM head, pick): tok/s and HBM GB/s of KV + weights")


def measured_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK, "fallback"


def profile_traffic(workload, alg_bytes=None, scale=1.0):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary.
    Where the summary also gives the algorithmic bytes of the captured launch
    (`algorithmic_bytes_per_launch`, a sharded workload captured on one GPU),
    the traffic is scaled to this run's launch by `alg_bytes` / that figure;
    `scale` multiplies it otherwise (prefill: the share of the sequences)."""
    path = os.path.join(REPO, "profiles", f"traffic_{workload}.txt")
    try:
        vals = {}
        for line in open(path):
            if "=" in line and not line.startswith("#"):
                k, v = line.split("=", 1)
                vals[k.strip()] = v.strip()
        traffic = float(vals["bytes_per_launch"])
        if "algorithmic_bytes_per_launch" in vals and alg_bytes:
            return round(traffic * alg_bytes / float(vals["algorithmic_bytes_per_launch"]))
        return round(traffic * scale)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML polling thread)
# ---------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index, period=0.002):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self.period = period
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report what we can
            self._nv = None
            self.error = str(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self._nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        names = [n for b, n in _REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(n_gpus):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


MIN_TIMED_S = 0.2    # the K-step region is repeated until this much device time is timed
MAX_ROUNDS = 200


def timed_rounds(body, world, stream, before=None):
    """Times `body` (which enqueues exactly the K timed steps) in rounds.

    Each round is bracketed by a barrier and a device synchronisation on both
    sides and timed with CUDA events on `stream`; its time is the maximum over
    ranks.  The number of rounds is fixed after the first (every rank gets the
    same maximum, so every rank runs the same rounds): enough for MIN_TIMED_S of
    timed device time in all.  `before()` (optional) runs untimed before each
    round.  Returns the per-round times in seconds; callers report the median.
    """
    import torch
    times, n_rounds = [], None
    while n_rounds is None or len(times) < n_rounds:
        if before is not None:
            before()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        body()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        t = max_over_ranks(e0.elapsed_time(e1) / 1e3, world)
        times.append(t)
        if n_rounds is None:
            n_rounds = max(1, min(MAX_ROUNDS, int(-(-MIN_TIMED_S // max(t, 1e-9)))))
            if MIN_TIMED_S <= 0:
                n_rounds = 1
    return times


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU reference / baseline (oracle/_ref: the reference's own function)
# ---------------------------------------------------------------------------
def cpu_reference_run(steps, warmup, budget_s, pos_lo=3840, layers=28):
    """Times the reference's cpu_attention_gqa_pipeline on the resident
    workload: per step, its 28 layer calls (independent inputs) spread over all
    host threads.  Returns (GB/s, cores, sample description, kind)."""
    import __graft_entry__
    orc = __graft_entry__.load_oracle()
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    if orc.have_reference():
        kind, T = "reference", orc.REF_T_MAX
    else:
        kind, T = "port", 4096
    kcs = [rng.standard_normal((2, T, 128), dtype=np.float32) for _ in range(layers)]
    vcs = [rng.standard_normal((2, T, 128), dtype=np.float32) for _ in range(layers)]
    qkvs = [rng.standard_normal(QKV_W, dtype=np.float32) for _ in range(layers)]

    def one_step(pos):
        if kind == "reference":
            orc.ref_bench_attention_many([q.copy() for q in qkvs], kcs, vcs, [pos] * layers,
                                         [pos + 1] * layers, cores)
        else:
            orc.decode_batched([q.copy() for q in qkvs], kcs, vcs, [pos + 1] * layers,
                               n_threads=cores)
        return layers * ROW_BYTES * (pos + 1)

    for i in range(warmup):
        one_step(pos_lo + i % 256)
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    while done < steps:
        nbytes += one_step(pos_lo + done % 256)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    sample = (f"{done} decode step(s) x {layers} layers at positions {pos_lo}.."
              f"{pos_lo + min(done, 256) - 1} (L = pos+1, window of 256 wraps), layer calls "
              f"spread over {cores} threads")
    return nbytes / dt / 1e9, cores, sample, kind, done / dt


def cpu_port_05b_run(budget_s, pos_lo=3840, layers=24):
    """The reference has no CPU attention for the 0.5B shape: the restatement
    (oracle/gqa_oracle.c, its loops at head_dim 64, group 7); per step the 24
    layer calls (independent inputs) spread over all host threads, as the
    reference's own function is timed for the 1.5B shape."""
    import __graft_entry__
    orc = __graft_entry__.load_oracle()
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    T, nq, nkv, d = 4096, 14, 2, 64
    kcs = [rng.standard_normal((nkv, T, d), dtype=np.float32) for _ in range(layers)]
    vcs = [rng.standard_normal((nkv, T, d), dtype=np.float32) for _ in range(layers)]
    qkvs = [rng.standard_normal((nq + 2 * nkv) * d, dtype=np.float32) for _ in range(layers)]
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    while True:
        pos = pos_lo + done % 256
        orc.decode_batched([q.copy() for q in qkvs], kcs, vcs, [pos + 1] * layers, n_heads_q=nq,
                           n_heads_kv=nkv, n_threads=cores, head_dim=d)
        nbytes += layers * 2 * nkv * d * 4 * (pos + 1)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    sample = (f"{done} decode step(s) x {layers} layers at positions {pos_lo}.."
              f"{pos_lo + min(done, 256) - 1}, the C restatement, layer calls spread over "
              f"{cores} threads")
    return nbytes / dt / 1e9, cores, sample, "port", done / dt


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = WORKLOADS["resident28"]
    gbs, cores, sample, kind, steps_per_s = cpu_reference_run(
        args.steps, min(args.warmup, 2), budget_s=90.0, pos_lo=wl["pos_lo"])
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / steps_per_s, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "tok_per_s": round(steps_per_s, 3),
        "config": workload_config("resident28"),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(name, exchange="peer"):
    if name == "head":
        return {"workload": "head: output RMSNorm + Q6_K LM head 151936x1536 (191 MB) + greedy "
                            "pick, one token's state per step",
                "vocab": VOCAB, "bytes_per_step": HEAD_BYTES,
                "l2": "two copies of the head weights used alternately (383 MB > 126 MB L2); "
                      "no flush",
                "parallelism": "replicas"}
    if name == "token28":
        return {"workload": "token28: one greedy decode step of the whole model per step -- Q4_0 "
                            "embedding of the previous pick, 28 decoder layers as in layer28, "
                            "output RMSNorm, Q6_K LM head 151936x1536, pick -- token and position "
                            "kept on the device, one CUDA graph per step",
                "layers": 28, "t_max": 4096, "positions": [3840, 4095], "vocab": VOCAB,
                "bytes_per_step": "28*(2048*(pos+1) + %d) + %d"
                                  % (BLOCK_WEIGHT_BYTES + FFN_WEIGHT_BYTES, HEAD_BYTES + Q4_ROW),
                "l2": "KV 235 MB + weights 928 MB per GPU > 126 MB L2; no flush",
                "parallelism": "sequence-sharded replicas"}
    if name == "head05b":
        return {"workload": "head05b: output RMSNorm + Q8_0 LM head 151936x896 (145 MB) of "
                            "Qwen2.5-0.5B + greedy pick, one token's state per step",
                "vocab": VOCAB, "bytes_per_step": HEAD05_BYTES,
                "l2": "two copies of the head weights used alternately (289 MB > 126 MB L2); "
                      "no flush",
                "parallelism": "replicas"}
    if name == "token24_05b":
        return {"workload": "token24_05b: one greedy decode step of the whole Qwen2.5-0.5B model "
                            "per step -- Q4_0 embedding of the previous pick, 24 decoder layers "
                            "(d_model 896, 14 q / 2 KV heads of 64, d_ffn 4864, Q4_0), output "
                            "RMSNorm, Q8_0 LM head 151936x896, pick -- token and position kept "
                            "on the device, one CUDA graph per step",
                "layers": 24, "t_max": 4096, "positions": [3840, 4095], "vocab": VOCAB,
                "bytes_per_step": "24*(1024*(pos+1) + %d) + %d"
                                  % (BLOCK05_BYTES + FFN05_BYTES, HEAD05_BYTES + Q4_ROW05),
                "l2": "KV 50 MB + weights 346 MB per GPU > 126 MB L2; no flush",
                "parallelism": "sequence-sharded replicas"}
    if name == "layer28":
        return {"workload": "layer28: 28 whole decoder layers per token (attention block as in "
                            "block28, then RMSNorm, Q4_0 gate/up 8960x1536 with SiLU, Q4_0 down "
                            "1536x8960 + residual), 1 sequence per GPU, positions 3840..4095, "
                            "no LM head",
                "layers": 28, "t_max": 4096, "positions": [3840, 4095],
                "bytes_per_layer": "2048*(pos+1) KV + %d weights"
                                   % (BLOCK_WEIGHT_BYTES + FFN_WEIGHT_BYTES),
                "l2": "KV 235 MB + weights 737 MB per GPU > 126 MB L2; no flush",
                "parallelism": "sequence-sharded replicas"}
    if name == "block28":
        return {"workload": "block28: 28 attention blocks per token (RMSNorm, Q4_0 QKV 2048x1536 + "
                            "bias, RoPE/append + GQA attention over fp32 KV t_max=4096, Q4_0 Wo "
                            "1536x1536 + residual), 1 sequence per GPU, positions 3840..4095",
                "layers": 28, "t_max": 4096, "positions": [3840, 4095],
                "bytes_per_layer": "2048*(pos+1) KV + %d weights" % BLOCK_WEIGHT_BYTES,
                "l2": "KV 235 MB + weights 87 MB per GPU > 126 MB L2; no flush",
                "parallelism": "sequence-sharded replicas"}
    if name == "resident05b":
        return {"workload": "resident05b: 24-layer resident decode attention of the Qwen2.5-0.5B "
                            "shape (head_dim 64, 14 q / 2 KV heads, 7 per KV head), 1 sequence "
                            "per GPU, fp32 KV t_max=4096 per layer (50 MB), steps at positions "
                            "3840..4095 (window wraps), shape-generic kernels",
                "layers": 24, "t_max": 4096, "positions": [3840, 4095], "global_batch": None,
                "l2": "KV 50 MB per GPU < 126 MB L2: read from L2 after the first pass",
                "parallelism": "sequence-sharded replicas"}
    if name == "resident28":
        return {"workload": "resident28: 28-layer resident decode attention, 1 sequence per GPU, "
                            "12 q / 2 KV heads, d=128, fp32 KV t_max=4096 per layer (235 MB), "
                            "steps at positions 3840..4095 (window wraps)",
                "layers": 28, "t_max": 4096, "positions": [3840, 4095], "global_batch": None,
                "l2": "KV 235 MB per GPU > 126 MB L2, read cyclically; no flush",
                "parallelism": "sequence-sharded replicas"}
    if name == "batched":
        return {"workload": "batched: 64 sequences, lengths U[256,8192] (seeded), fp32 KV, "
                            "one new token per sequence per step", "seqs": 64,
                "l2": "KV > 126 MB L2; no flush", "parallelism": "sequence-sharded"}
    if name == "long":
        return {"workload": "long: 256 sequences x 32768 fp32 KV rows (17.2 GB per layer)",
                "seqs": 256, "t_max": 32768, "l2": "KV > L2; no flush",
                "parallelism": "sequence-sharded"}
    if name == "prefill":
        return {"workload": "prefill: 8 sequences x 2048 tokens, 12 q / 2 KV heads, d=128, RoPE "
                            "theta 1e6, fp32 inputs cast to bf16, causal, fp32 accumulation",
                "seqs": 8, "seq_len": 2048, "flops_per_step": "4*B*Hq*d*S*(S+1)/2",
                "l2": "inputs 134 MB > L2; no flush", "parallelism": "sequence-sharded"}
    if name == "long1":
        how = ("merged partials exchanged by one kernel over NVLink peer memory (IPC inboxes, "
               "epoch flags) and LSE-combined" if exchange == "peer" else
               "partials all-gathered (NCCL) and LSE-combined")
        return {"workload": "long1: one sequence, 32768 fp32 KV rows (67 MB per layer) split by "
                            "KV range across the GPUs, " + how + " every step", "seqs": 1,
                "t_max": 32768, "l2": "KV > L2 at 1-2 GPUs; no flush",
                "parallelism": "kv-range split", "exchange": exchange}
    return {"workload": "single: one step, 12/2 heads, d=128, pos 511, seq_len 512",
            "l2": "1 MB KV fits in L2 (latency-bound)"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_resident(args, g, ctx, rank, world, local):
    import torch
    wl = WORKLOADS[args.workload]
    L_layers, t_max, pos_lo, pos_hi = wl["layers"], wl["t_max"], wl["pos_lo"], wl["pos_hi"]
    n_q, n_kv, d = wl.get("n_q", N_Q), wl.get("n_kv", N_KV), wl.get("d", D)
    qkv_w, out_w, row_bytes = (n_q + 2 * n_kv) * d, n_q * d, 2 * n_kv * d * 4
    generic = d != D
    seed = 4242 + 1000 * rank
    caches = torch.empty((L_layers, 2, n_kv, t_max, d), device="cuda")  # [layer][k/v][h][t][d]
    ctx.fill_normal(caches, caches.numel(), seed, g.seeded.K_CACHE)
    kvs = [g.kv_of(caches[l, 0], caches[l, 1]) for l in range(L_layers)]
    n_slots = 8
    qkv_slots = torch.empty((n_slots, L_layers, qkv_w), device="cuda")
    ctx.fill_normal(qkv_slots, qkv_slots.numel(), seed, g.seeded.QKV)
    out = torch.empty((L_layers, out_w), device="cuda")
    d_pos = torch.tensor([pos_lo], dtype=torch.int32, device="cuda")
    ctx.reserve(1, t_max)
    graphs = [ctx.graph_create_layers(kvs, qkv_slots[s], qkv_w, out, out_w, d_pos, advance=True,
                                      wrap_lo=pos_lo, wrap_hi=pos_hi) for s in range(n_slots)]
    # e2e: host-buffer steps through the C ABI (gqa_graph_step_host)
    d_qkv_e2e = torch.empty((L_layers, qkv_w), device="cuda")
    g_e2e = ctx.graph_create_layers(kvs, d_qkv_e2e, qkv_w, out, out_w, d_pos, advance=True,
                                    wrap_lo=pos_lo, wrap_hi=pos_hi)
    h_qkv = qkv_slots.cpu().pin_memory()
    h_out = torch.empty((n_slots, L_layers, out_w)).pin_memory()
    n_window = pos_hi - pos_lo

    def step_bytes(i):
        pos = pos_lo + i % n_window
        return L_layers * row_bytes * (pos + 1)

    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        graphs[i % n_slots].launch(stream)
    for i in range(args.warmup):
        g_e2e.step_host(h_qkv[i % n_slots], h_out[i % n_slots], stream)
    torch.cuda.synchronize()
    if ctx.device_status() != 0:
        raise RuntimeError("device status set during warm-up")

    # ---- kernel-only timed region (rounds of K steps, median) ----
    def reset_pos():
        d_pos.fill_(pos_lo)

    def body():
        for i in range(args.steps):
            graphs[i % n_slots].launch(stream)

    with ClockSampler(local) as clk:
        rounds = timed_rounds(body, world, stream, before=reset_pos)
    t_local = statistics.median(rounds)
    total_bytes = sum(step_bytes(i) for i in range(args.steps))

    # ---- the layer kernels' own in-graph time: the same 28 layer calls in a
    # graph without the position advance, replayed at position pos_lo ----
    g_layers = ctx.graph_create_layers(kvs, qkv_slots[0], qkv_w, out, out_w, d_pos,
                                       advance=False)
    reset_pos()
    for _ in range(3):
        g_layers.launch(stream)
    t_layers = statistics.median(timed_rounds(
        lambda: [g_layers.launch(stream) for _ in range(args.steps)], world, stream))
    g_layers.destroy()
    kernel_s = t_layers / args.steps / L_layers
    kernel_bytes = row_bytes * (pos_lo + 1)

    # ---- e2e timed region (host buffers in, host buffers out) ----
    def body_e2e():
        for i in range(args.steps):
            g_e2e.step_host(h_qkv[i % n_slots], h_out[i % n_slots], stream)

    t_e2e_local = statistics.median(timed_rounds(body_e2e, world, stream, before=reset_pos))
    status = ctx.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status} after the timed regions")

    # mirrors the library's split plan for pos read from the device (planned for t_max)
    n_sm = torch.cuda.get_device_properties(local).multi_processor_count
    if generic:  # split (RoPE + append fused), merge per layer (csrc/gqa_generic.cu)
        kernels_per_step = L_layers * 2 + 1
    elif args.grid_merge and args.variant in (-1, 0, 3, 5):
        # one grid-merged split kernel per layer (csrc/gqa_decode.cu), + the advance
        kernels_per_step = L_layers + 1
    else:
        target = args.target_ctas or n_sm
        quant = g.gqa.VARIANT_QUANT[3 if args.variant < 0 else args.variant]
        n_splits = min(-(-target // n_kv), -(-t_max // quant))
        kernels_per_step = L_layers * (2 if n_splits > 1 else 1) + 1
    for gr in graphs + [g_e2e]:
        gr.destroy()
    res = dict(t=t_local, t_e2e=t_e2e_local, bytes=total_bytes, clocks=clk.summary(),
               launches=kernels_per_step * args.steps, launches_per_step=kernels_per_step,
               h2d=L_layers * qkv_w * 4, d2h=L_layers * out_w * 4, tokens=args.steps,
               dominant_launches=L_layers * args.steps, rounds=len(rounds),
               timed_s=sum(rounds), kernel_s=kernel_s, kernel_bytes=kernel_bytes,
               layers=L_layers, kernel_pos=pos_lo,
               kernel_per_layer="split kernel + merge kernel" if generic or
               kernels_per_step != L_layers + 1 else "one grid-merged split kernel")
    if generic:
        res.update(kernel="split_generic_kernel<64, 7> (+ merge)",
                   data="synthetic: seeded N(0,1) q/k/v and KV caches (gqa_fill_normal), "
                        "Qwen2.5-0.5B attention shape")
    return res


def run_block(args, g, ctx, rank, world, local):
    import torch
    full = args.workload == "layer28"
    wl = WORKLOADS[args.workload]
    L_layers, t_max, pos_lo, pos_hi = wl["layers"], wl["t_max"], wl["pos_lo"], wl["pos_hi"]
    seed = 5353 + 1000 * rank
    caches = torch.empty((L_layers, 2, 2, t_max, D), device="cuda")
    ctx.fill_normal(caches, caches.numel(), seed, g.seeded.K_CACHE)
    kvs = [g.kv_of(caches[l, 0], caches[l, 1]) for l in range(L_layers)]
    scale = 1.0 / (4.6 * np.sqrt(OUT_W))
    keep, ws, fws = [], [], []
    for l in range(L_layers):
        wq = torch.from_numpy(g.seeded.q4_0_matrix(seed + l, g.seeded.W_QKV, QKV_W, OUT_W, scale))
        wo = torch.from_numpy(g.seeded.q4_0_matrix(seed + l, g.seeded.W_O, OUT_W, OUT_W, scale))
        bq = torch.from_numpy(0.1 * g.seeded.normal(seed + l, g.seeded.B_QKV, QKV_W))
        gm = torch.from_numpy(1.0 + 0.1 * g.seeded.normal(seed + l, g.seeded.GAMMA, OUT_W))
        dev = [wq.cuda(), bq.float().cuda(), wo.cuda(), gm.float().cuda()]
        keep += dev
        ws.append(g.block_weights_of(*dev))
        if full:
            fdev = [torch.from_numpy(a).cuda() for a in g.seeded.ffn_block_inputs(seed + l)]
            keep += fdev
            fws.append(g.ffn_weights_of(*fdev))
    state0 = torch.empty(OUT_W, device="cuda")
    ctx.fill_normal(state0, OUT_W, seed, g.seeded.STATE)
    state = state0.clone()
    d_pos = torch.tensor([pos_lo], dtype=torch.int32, device="cuda")
    ctx.reserve(1, t_max)
    n_window = pos_hi - pos_lo

    w_bytes = BLOCK_WEIGHT_BYTES + (FFN_WEIGHT_BYTES if full else 0)

    def step_bytes(i):
        pos = pos_lo + i % n_window
        return L_layers * (ROW_BYTES * (pos + 1) + w_bytes)

    def token_step():
        if full:
            ctx.decoder_layers(ws, fws, kvs, state, d_pos, True, pos_lo, pos_hi)
        else:
            ctx.attention_block_layers(ws, kvs, state, d_pos, True, pos_lo, pos_hi)

    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        token_step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            token_step()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    if ctx.device_status() != 0:
        raise RuntimeError("device status set during warm-up")

    d_pos.fill_(pos_lo)
    state.copy_(state0)
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    t_local = ev0.elapsed_time(ev1) / 1e3
    total_bytes = sum(step_bytes(i) for i in range(args.steps))

    # e2e: the token's residual state from pinned host memory in, the state out
    h_state = state0.cpu().pin_memory()
    h_out = torch.empty(OUT_W).pin_memory()
    d_pos.fill_(pos_lo)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        state.copy_(h_state, non_blocking=True)
        graph.replay()
        h_out.copy_(state, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    if ctx.device_status() != 0:
        raise RuntimeError("device status set after the timed regions")
    del graph
    # per layer: QKV GEMV, split, combine, Wo GEMV (+ gate/up, down); plus the position advance
    per_step = (6 if full else 4) * L_layers + 1
    return dict(t=t_local, t_e2e=e0.elapsed_time(e1) / 1e3, bytes=total_bytes,
                clocks=clk.summary(), launches=per_step * args.steps,
                launches_per_step=per_step, h2d=OUT_W * 4, d2h=OUT_W * 4, tokens=args.steps,
                dominant_launches=L_layers * args.steps,
                metric=LAYER_METRIC if full else BLOCK_METRIC,
                kernel="decode_split_kernel + gemv_q4_kernel (one %s)"
                       % ("decoder layer" if full else "attention block"),
                data="synthetic: seeded N(0,1) state and KV caches, seeded Q4_0 weights "
                     "(scales for unit-RMS projections)")


def run_head(args, g, ctx, rank, world, local):
    """The LM head alone ("head", "head05b") or the whole greedy decode step
    ("token28", "token24_05b"): Qwen2.5-1.5B with its Q6_K head, or
    Qwen2.5-0.5B with its Q8_0 head."""
    import torch
    wl = WORKLOADS[args.workload]
    whole = args.workload in ("token28", "token24_05b")
    small = wl.get("model") == "0.5b"
    d_model, qkv_w, d_ffn = (D05, QKV05, DFFN05) if small else (OUT_W, QKV_W, D_FFN)
    hd, n_kv = wl.get("d", D), wl.get("n_kv", N_KV)
    head_bytes = HEAD05_BYTES if small else HEAD_BYTES
    seed = 6464 + 1000 * rank
    s = g.seeded
    if small:
        w_head, gamma_out, embd = s.head_q8_inputs(seed, VOCAB, d_model)
        packed_bytes, pack, head = (g.Context.lm_head_q8_0_packed_bytes, ctx.lm_head_q8_0_pack,
                                    ctx.lm_head_q8_0)
    else:
        w_head, gamma_out, embd = s.head_inputs(seed, VOCAB, d_model)
        packed_bytes, pack, head = g.Context.lm_head_packed_bytes, ctx.lm_head_pack, ctx.lm_head
    n_copies = 1 if whole else 2
    packed = []
    raw = torch.from_numpy(w_head).cuda()
    for _ in range(n_copies):
        p = torch.empty(packed_bytes(VOCAB), dtype=torch.uint8, device="cuda")
        pack(raw, VOCAB, p)
        packed.append(p)
    del raw
    d_gamma = torch.from_numpy(gamma_out).cuda()
    d_embd = torch.from_numpy(embd).cuda()
    d_tok = torch.tensor([17], dtype=torch.int32, device="cuda")
    logits = torch.empty(VOCAB, device="cuda")
    state0 = torch.empty(d_model, device="cuda")
    ctx.fill_normal(state0, d_model, seed, s.STATE)
    state = state0.clone()
    keep = []
    if whole:
        L_layers, t_max, pos_lo, pos_hi = wl["layers"], wl["t_max"], wl["pos_lo"], wl["pos_hi"]
        caches = torch.empty((L_layers, 2, n_kv, t_max, hd), device="cuda")
        ctx.fill_normal(caches, caches.numel(), seed, s.K_CACHE)
        kvs = [g.kv_of(caches[l, 0], caches[l, 1]) for l in range(L_layers)]
        scale = 1.0 / (4.6 * np.sqrt(d_model))
        ws, fws = [], []
        for l in range(L_layers):
            wq = s.q4_0_matrix(seed + l, s.W_QKV, qkv_w, d_model, scale)
            wo = s.q4_0_matrix(seed + l, s.W_O, d_model, d_model, scale)
            bq = (0.1 * s.normal(seed + l, s.B_QKV, qkv_w)).astype(np.float32)
            gm = (1.0 + 0.1 * s.normal(seed + l, s.GAMMA, d_model)).astype(np.float32)
            dev = [torch.from_numpy(a).cuda() for a in (wq, bq, wo, gm)]
            fdev = [torch.from_numpy(a).cuda()
                    for a in s.ffn_block_inputs(seed + l, d_model=d_model, d_ffn=d_ffn)]
            keep += dev + fdev
            ws.append(g.block_weights_of(*dev))
            fws.append(g.ffn_weights_of(*fdev))
        model = g.ModelHandle(ws, fws, kvs, d_embd, d_gamma, packed[0], VOCAB,
                              g.gqa.HEAD_Q8_0 if small else g.gqa.HEAD_Q6_K)
        d_pos = torch.tensor([pos_lo], dtype=torch.int32, device="cuda")
        ctx.reserve(1, t_max)
        n_window = pos_hi - pos_lo
        w_bytes = (BLOCK05_BYTES + FFN05_BYTES) if small else (BLOCK_WEIGHT_BYTES + FFN_WEIGHT_BYTES)
        row_bytes = 2 * n_kv * hd * 4
        embd_row = (d_model // 32) * 18

        def step_bytes(i):
            pos = pos_lo + i % n_window
            return L_layers * (row_bytes * (pos + 1) + w_bytes) + head_bytes + embd_row

        def graph_body(i):
            ctx.decode_token(model, state, d_tok, d_pos, logits, pos_lo, pos_hi)
    else:
        def step_bytes(i):
            return head_bytes

        def graph_body(i):
            head(packed[i % n_copies], VOCAB, d_gamma, state, logits, d_tok)

    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        graph_body(i)
    torch.cuda.synchronize()
    graphs = []
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    for i in range(n_copies):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(gr, stream=cap):
                graph_body(i)
        graphs.append(gr)
    torch.cuda.synchronize()
    for gr in graphs:
        gr.replay()
    torch.cuda.synchronize()
    if ctx.device_status() != 0:
        raise RuntimeError("device status set during warm-up")
    if whole:
        d_pos.fill_(pos_lo)
    d_tok.fill_(17)
    state.copy_(state0)
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            graphs[i % n_copies].replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    t_local = ev0.elapsed_time(ev1) / 1e3
    total_bytes = sum(step_bytes(i) for i in range(args.steps))

    # e2e: the previous token in from pinned host memory, the pick out
    h_tok = torch.tensor([17], dtype=torch.int32).pin_memory()
    h_out = torch.empty(1, dtype=torch.int32).pin_memory()
    if whole:
        d_pos.fill_(pos_lo)
    state.copy_(state0)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        d_tok.copy_(h_tok, non_blocking=True)
        graphs[i % n_copies].replay()
        h_out.copy_(d_tok, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    if ctx.device_status() != 0:
        raise RuntimeError("device status set after the timed regions")
    del graphs
    # embedding, per layer 6 kernels, head, position advance
    per_step = (1 + 6 * wl["layers"] + 2) if whole else 1
    if small:
        metric = TOKEN05_METRIC if whole else HEAD05_METRIC
        data = ("synthetic: seeded Q8_0 head (uniform int8 codes, fp16 d ~ 2^-8), seeded Q4_0 "
                "embedding/layer weights at the Qwen2.5-0.5B sizes, N(0,1) state and KV caches")
    else:
        metric = TOKEN_METRIC if whole else HEAD_METRIC
        data = ("synthetic: seeded Q6_K head (uniform codes/scales, fp16 d ~ 2^-12), seeded "
                "Q4_0 embedding/layer weights, N(0,1) state and KV caches")
    return dict(t=t_local, t_e2e=e0.elapsed_time(e1) / 1e3, bytes=total_bytes,
                clocks=clk.summary(), launches=per_step * args.steps,
                launches_per_step=per_step, h2d=4, d2h=4, tokens=args.steps,
                dominant_launches=args.steps, metric=metric,
                kernel="whole decode step" if whole else
                ("lm_head_q8_kernel" if small else "lm_head_kernel"),
                head_bytes=head_bytes, data=data)


def cpu_head_run(budget_s, whole=False, pos_lo=3840, layers=28):
    """The reference's CPU path on the host cores: its Q6_K GEMV
    (cpu_gemv_q6_k_ref, OpenMP over rows) after the output norm, with the
    pick; for the whole step also the embedding lookup and its decoder-layer
    step 28 times (OpenMP GEMVs, serial attention)."""
    import __graft_entry__
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    if not orc.have_reference():
        return None
    s = g.seeded
    w_head = s.q6_k_matrix(901, s.W_HEAD, VOCAB)
    gamma = (1.0 + 0.1 * s.normal(901, s.GAMMA_OUT, OUT_W)).astype(np.float32)
    state = s.normal(901, s.STATE, OUT_W)
    if whole:
        table = s.q4_0_matrix(901, s.TOKEN_EMBD, VOCAB, OUT_W, 1.0 / 4.6)
        blocks = [s.attention_block_inputs(900 + l) for l in range(layers)]
        ffns = [s.ffn_block_inputs(900 + l) for l in range(layers)]
    tok = 17
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    while True:
        if whole:
            pos = pos_lo + done % 256
            x = orc.ref_token_embedding(table, tok)
            for l, L in enumerate(blocks):
                x = orc.ref_decoder_layer(x, (L[1], L[2], L[3], L[4]), ffns[l], L[5], L[6], pos,
                                          pos + 1)
            nbytes += layers * (ROW_BYTES * (pos + 1) + BLOCK_WEIGHT_BYTES + FFN_WEIGHT_BYTES)
            _, tok = orc.ref_lm_head(x, gamma, w_head)
            nbytes += HEAD_BYTES + Q4_ROW
        else:
            _, tok = orc.ref_lm_head(state, gamma, w_head)
            nbytes += HEAD_BYTES
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    what = ("whole decode step(s): embedding, 28 decoder layers, output norm, Q6_K head, pick"
            if whole else "LM head call(s): output norm, Q6_K GEMV over 151936 rows, pick")
    sample = (f"{done} {what}; the reference's OpenMP GEMVs on {os.cpu_count()} threads")
    return nbytes / dt / 1e9, os.cpu_count() or 1, sample, "reference", done / dt


def cpu_head05b_run(budget_s, whole=False, pos_lo=3840, layers=24):
    """The 0.5B model's step on the host cores.  The reference runs it only
    in OpenCL (generate_stream_05b.c), so this is the oracle: the reference's
    compiled OpenMP GEMVs for every projection, the restated Q8_0 head
    (gemv_q8_0) and attention, one thread for the restated parts."""
    import __graft_entry__
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    if not orc.have_reference():
        return None
    s = g.seeded
    w_head = s.q8_0_matrix(901, s.W_HEAD, VOCAB, D05)
    gamma = (1.0 + 0.1 * s.normal(901, s.GAMMA_OUT, D05)).astype(np.float32)
    state = s.normal(901, s.STATE, D05)
    if whole:
        table = s.q4_0_matrix(901, s.TOKEN_EMBD, VOCAB, D05, 1.0 / 4.6)
        blocks = [s.attention_block_inputs(900 + l, d_model=D05, n_heads_kv=2, head_dim=64)
                  for l in range(layers)]
        ffns = [s.ffn_block_inputs(900 + l, d_model=D05, d_ffn=DFFN05) for l in range(layers)]
        lay = [((L[1], L[2], L[3], L[4]), f) for L, f in zip(blocks, ffns)]
        kv = [(L[5], L[6]) for L in blocks]
    tok = 17
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    while True:
        if whole:
            pos = pos_lo + done % 256
            _, tok = orc.ref_decode_token(table, lay, kv, gamma, w_head, tok, pos, model="0.5b")
            nbytes += (layers * (ROW05 * (pos + 1) + BLOCK05_BYTES + FFN05_BYTES) +
                       HEAD05_BYTES + Q4_ROW05)
        else:
            _, tok = orc.lm_head_q8_0(state, gamma, w_head, VOCAB)
            nbytes += HEAD05_BYTES
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    what = ("whole 0.5B decode step(s): embedding, 24 decoder layers, output norm, Q8_0 head, "
            "pick" if whole else "Q8_0 LM head call(s) over 151936 rows with the pick")
    sample = (f"{done} {what}; the reference's compiled OpenMP GEMVs on {os.cpu_count()} "
              "threads, the restated Q8_0 head and attention on one")
    return nbytes / dt / 1e9, os.cpu_count() or 1, sample, "port", done / dt


def cpu_block_run(budget_s, pos_lo=3840, layers=28, full=False):
    """The reference's decoder-layer step on the host cores -- with zero FFN
    weights (the attention block) or whole -- per step its 28 layer calls in a
    row, each with the reference's OpenMP GEMVs and serial attention."""
    import __graft_entry__
    g = __graft_entry__.load_package()
    orc = __graft_entry__.load_oracle()
    if not orc.have_reference():
        return None
    blocks = [g.seeded.attention_block_inputs(900 + l) for l in range(layers)]
    ffns = [g.seeded.ffn_block_inputs(900 + l) for l in range(layers)] if full else None
    state = blocks[0][0].copy()
    w_bytes = BLOCK_WEIGHT_BYTES + (FFN_WEIGHT_BYTES if full else 0)
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    while True:
        pos = pos_lo + done % 256
        for l, L in enumerate(blocks):
            if full:
                state = orc.ref_decoder_layer(state, (L[1], L[2], L[3], L[4]), ffns[l], L[5], L[6],
                                              pos, pos + 1)
            else:
                state = orc.ref_attention_block(state, L[1], L[2], L[3], L[4], L[5], L[6], pos,
                                                pos + 1)
        nbytes += layers * (ROW_BYTES * (pos + 1) + w_bytes)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    what = "decoder layers" if full else "attention blocks"
    sample = (f"{done} token step(s) x {layers} {what} at positions {pos_lo}.."
              f"{pos_lo + min(done, 256) - 1}, the reference's OpenMP GEMVs on "
              f"{os.cpu_count()} threads, attention serial")
    return nbytes / dt / 1e9, os.cpu_count() or 1, sample, "reference", done / dt


def run_batched(args, g, ctx, rank, world, local):
    import torch
    wl = WORKLOADS[args.workload]
    seed = 777 + 1000 * rank
    if args.workload == "batched":
        n_all, window = wl["seqs"], wl["window"]
        lens_all = [int(x) for x in g.seeded.uniform_int(777, g.seeded.LENGTHS, n_all,
                                                         wl["len_lo"], wl["len_hi"])]
        t_max = wl["len_hi"] + window
    else:
        n_all, window, t_max = wl["seqs"], wl["window"], wl["t_max"]
        lens_all = [t_max - window] * n_all
    # Sequences are dealt to ranks (longest first to the least-loaded rank).
    # --share-of W (one process): time the share rank 0 gets at W ranks.
    if args.share_of > 1 and world == 1:
        mine = g.shard.plan_sequence_shards(lens_all, args.share_of)[0]
    else:
        mine = g.shard.plan_sequence_shards(lens_all, world)[rank]
    lens0 = [lens_all[i] for i in mine]
    n = len(lens0)
    k = torch.empty((n, 2, t_max, D), device="cuda")
    v = torch.empty((n, 2, t_max, D), device="cuda")
    ctx.fill_normal(k, k.numel(), seed, g.seeded.K_CACHE)
    ctx.fill_normal(v, v.numel(), seed, g.seeded.V_CACHE)
    qkv = torch.empty((n, QKV_W), device="cuda")
    ctx.fill_normal(qkv, qkv.numel(), seed, g.seeded.QKV)
    out = torch.empty((n, OUT_W), device="cuda")
    stride = 2 * t_max * D * 4
    kp = torch.tensor([k.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                      device="cuda")
    vp = torch.tensor([v.data_ptr() + s * stride for s in range(n)], dtype=torch.int64,
                      device="cuda")
    lens_base = torch.tensor(lens0, dtype=torch.int32, device="cuda")
    dl = lens_base.clone()
    max_len = max(lens0) + window - 1
    ctx.reserve(n, max_len)
    # Consecutive steps overlap their launches (programmatic dependent launch:
    # the preceding kernel is the previous step's combine, which writes no
    # cache row), and each step's combine advances the device lengths by one.
    ctx.set_option(g.gqa.GQA_OPT_PDL, 1)
    ctx.set_option(g.gqa.GQA_OPT_BATCH_ADVANCE, 1)
    stream = torch.cuda.current_stream()

    def step(i, st=None):
        if i % window == 0:
            dl.copy_(lens_base)
        ctx.decode_batched(n, kp, vp, qkv, QKV_W, dl, max_len, out, OUT_W,
                           st if st is not None else stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # The K timed steps as CUDA graphs of at most one window of steps each
    # (lengths reset at a graph's start, advanced by one after every step):
    # replays are not bound by the host's launch rate when a GPU's share of
    # the batch is small.  K = full * window + rem.
    def capture(n_steps):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            cap = torch.cuda.current_stream()
            for i in range(n_steps):
                step(i, cap)
        gr.replay()
        torch.cuda.synchronize()
        return gr

    full, rem = divmod(args.steps, window)
    graphs = ([capture(window)] * full) + ([capture(rem)] if rem else [])

    def body():
        for gr in graphs:
            gr.replay()

    with ClockSampler(local) as clk:
        rounds = timed_rounds(body, world, stream)
    t_local = statistics.median(rounds)
    total_bytes = sum(ROW_BYTES * (L + i % window) for i in range(args.steps) for L in lens0)
    # e2e: q/k/v rows from pinned host memory, outputs back, every step
    h_qkv = qkv.cpu().pin_memory()
    h_out = torch.empty((n, OUT_W)).pin_memory()

    def body_e2e():
        for i in range(args.steps):
            if i % window == 0:
                dl.copy_(lens_base)
            # host qkv in, the step, host outputs back: one C-ABI call
            ctx.decode_batched_host(n, kp, vp, h_qkv, qkv, QKV_W, dl, max_len, out, OUT_W, h_out,
                                    stream)

    t_e2e = statistics.median(timed_rounds(body_e2e, world, stream))
    status = ctx.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}")
    del graphs
    return dict(t=t_local, t_e2e=t_e2e, bytes=total_bytes,
                clocks=clk.summary(), launches=2 * args.steps, launches_per_step=2,
                h2d=n * QKV_W * 4, d2h=n * OUT_W * 4, tokens=n * args.steps,
                dominant_launches=args.steps, rounds=len(rounds), timed_s=sum(rounds))


def run_long1(args, g, ctx, rank, world, local):
    import torch
    wl = WORKLOADS["long1"]
    T, window = wl["t_max"], wl["window"]
    b, n = g.shard.plan_kv_ranges(T, world)[rank]
    seed = 5151
    k = torch.empty((N_KV, max(n, 1), D), device="cuda")
    v = torch.empty((N_KV, max(n, 1), D), device="cuda")
    for h in range(N_KV):  # this rank's rows of the one seeded global cache
        ctx.fill_normal(k[h], n * D, seed, g.seeded.K_CACHE, offset=(h * T + b) * D)
        ctx.fill_normal(v[h], n * D, seed, g.seeded.V_CACHE, offset=(h * T + b) * D)
    qkv = torch.empty(QKV_W, device="cuda")
    ctx.fill_normal(qkv, QKV_W, seed, g.seeded.QKV)
    out = torch.empty(OUT_W, device="cuda")
    if args.exchange == "peer":
        dec = g.shard.KvShardExchangeDecoder(ctx, k, v, b, n)
        per_step = 2  # split kernel + exchange-merge kernel
    else:
        dec = g.shard.KvShardDecoder(ctx, k, v, b, n)
        per_step = 3  # split + local merge + merge of the gathered partials (NCCL not counted)
    pos0 = T - window
    stream = torch.cuda.current_stream()

    def my_bytes(i):
        pos = pos0 + i % window
        return ROW_BYTES * max(0, min(n, pos + 1 - b))

    ctx.reserve(1, max(n, 1))  # split scratch for every position, before any capture
    for i in range(args.warmup):
        dec.step(qkv, pos0 + i % window, out)
    torch.cuda.synchronize()
    graph = None
    if args.exchange == "peer":
        # One CUDA graph holds the window's steps (positions pos0 .. pos0+window-1); the
        # exchange's step epoch lives on the device, so every replay is a new set of steps.
        # The NCCL arm stays eager (its collective is issued from the host).
        if args.steps % window:
            raise SystemExit(f"long1 with the peer exchange times whole windows: --steps must be "
                             f"a multiple of {window}")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(window):
                dec.step(qkv, pos0 + i, out)
        graph.replay()
        torch.cuda.synchronize()
    def body():
        if graph is not None:
            for _ in range(args.steps // window):
                graph.replay()
        else:
            for i in range(args.steps):
                dec.step(qkv, pos0 + i % window, out)

    with ClockSampler(local) as clk:
        rounds = timed_rounds(body, world, stream)
    t_local = statistics.median(rounds)
    h_qkv = qkv.cpu().pin_memory()
    h_out = torch.empty(OUT_W).pin_memory()

    def body_e2e():
        for i in range(args.steps):
            qkv.copy_(h_qkv, non_blocking=True)
            dec.step(qkv, pos0 + i % window, out)
            h_out.copy_(out, non_blocking=True)

    t_e2e = statistics.median(timed_rounds(body_e2e, world, stream))
    if ctx.device_status() != 0:
        raise RuntimeError("device status set")
    if args.exchange == "peer":
        barrier(world)  # no rank unmaps its inbox while a peer may still store into it
        del graph
        dec.close()
    return dict(t=t_local, t_e2e=t_e2e,
                bytes=sum(my_bytes(i) for i in range(args.steps)), clocks=clk.summary(),
                launches=per_step * args.steps, launches_per_step=per_step, h2d=QKV_W * 4,
                d2h=OUT_W * 4, tokens=args.steps / world, dominant_launches=args.steps,
                rounds=len(rounds), timed_s=sum(rounds))


def run_prefill(args, g, ctx, rank, world, local):
    import torch
    wl = WORKLOADS["prefill"]
    mine = g.shard.plan_sequence_shards([wl["t_max"]] * wl["seqs"], world)[rank]
    n, S = len(mine), wl["t_max"]
    x = torch.empty((max(n, 1), S, QKV_W), device="cuda")
    ctx.fill_normal(x, x.numel(), 9090 + rank, g.seeded.PREFILL_Q)
    out = torch.empty((max(n, 1), S, OUT_W), device="cuda")
    stream = torch.cuda.current_stream()
    flops = 4.0 * N_Q * D * S * (S + 1) / 2 * n
    for _ in range(args.warmup):
        ctx.prefill_bf16(n, S, x, out)
    torch.cuda.synchronize()

    def body():
        for _ in range(args.steps):
            ctx.prefill_bf16(n, S, x, out)

    with ClockSampler(local) as clk:
        rounds = timed_rounds(body, world, stream)
    t_local = statistics.median(rounds)
    h_x = x.cpu().pin_memory()
    h_out = torch.empty(out.shape).pin_memory()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        x.copy_(h_x, non_blocking=True)
        ctx.prefill_bf16(n, S, x, out)
        h_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    if ctx.device_status() != 0:
        raise RuntimeError("device status set")
    return dict(t=t_local, t_e2e=e0.elapsed_time(e1) / 1e3, flops=flops * args.steps,
                clocks=clk.summary(), launches=2 * args.steps, launches_per_step=2,
                h2d=x.numel() * 4, d2h=out.numel() * 4, tokens=n * S * args.steps,
                dominant_launches=args.steps, rounds=len(rounds), timed_s=sum(rounds))


def run_ours(args):
    import torch
    rank, world, local = dist_setup(args.gpus)
    import __graft_entry__
    g = __graft_entry__.load_package()
    wl = WORKLOADS[args.workload]
    t_max = wl.get("t_max") or (wl["len_hi"] + wl["window"])
    if args.workload == "long1":
        t_max = max(n for _, n in g.shard.plan_kv_ranges(t_max, world))
    ctx = g.Context(n_heads_q=wl.get("n_q", N_Q), n_heads_kv=wl.get("n_kv", N_KV),
                    head_dim=wl.get("d", D), t_max=t_max, device=local)
    if args.variant >= 0:
        ctx.set_option(g.gqa.GQA_OPT_KERNEL_VARIANT, args.variant)
    if args.target_ctas:
        ctx.set_option(g.gqa.GQA_OPT_TARGET_CTAS, args.target_ctas)
    if args.batch_chunk:
        ctx.set_option(g.gqa.GQA_OPT_BATCH_CHUNK, args.batch_chunk)
    if not args.grid_merge:
        ctx.set_option(g.gqa.GQA_OPT_GRID_MERGE, 0)
    if args.workload == "prefill":
        return report_prefill(args, run_prefill(args, g, ctx, rank, world, local), ctx, rank,
                              world)
    if args.workload in ("block28", "layer28"):
        r = run_block(args, g, ctx, rank, world, local)
    elif args.workload in ("head", "token28", "head05b", "token24_05b"):
        r = run_head(args, g, ctx, rank, world, local)
    elif args.workload in ("resident28", "single", "resident05b"):
        r = run_resident(args, g, ctx, rank, world, local)
    elif args.workload == "long1":
        r = run_long1(args, g, ctx, rank, world, local)
    else:
        r = run_batched(args, g, ctx, rank, world, local)
    t = max_over_ranks(r["t"], world)
    t_e2e = max_over_ranks(r["t_e2e"], world)
    total_bytes = sum_over_ranks(r["bytes"], world)
    tokens = sum_over_ranks(r["tokens"], world)
    peak, peak_kind = measured_peak()
    gbs = total_bytes / t / 1e9
    gbs_e2e = total_bytes / t_e2e / 1e9
    per_gpu_bytes = r["bytes"] / r["dominant_launches"]
    if "kernel_s" in r:
        # the dominant kernel's own in-graph time (its graph replayed without the advance)
        achieved = r["kernel_bytes"] / r["kernel_s"] / 1e9
        per_gpu_bytes = r["kernel_bytes"]
        basis = (f"in-graph: the {r['layers']} layer calls ({r['kernel_per_layer']}) replayed "
                 f"as a graph without the position advance, at position {r['kernel_pos']}; "
                 "median of rounds; per layer")
    else:
        achieved = r["bytes"] / r["t"] / 1e9  # this rank's kernel bytes over its timed region
        basis = ("timed-region device time / launches of the dominant kernel (includes its "
                 "merge and gaps)")
    extra = None
    if args.workload == "resident28" and not args.no_extra:
        extra = {}
        for name in ("batched", "long1", "prefill", "token28", "head"):
            try:
                extra[name] = run_extra(args, g, name, rank, world, local)
            except Exception as exc:  # a sharded extra never takes the headline line down
                extra[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if args.workload in ("block28", "layer28"):
            res = cpu_block_run(budget_s=12.0, full=args.workload == "layer28")
        elif args.workload in ("head", "token28"):
            res = cpu_head_run(budget_s=12.0, whole=args.workload == "token28")
        elif args.workload == "resident05b":
            res = cpu_port_05b_run(budget_s=12.0)
        elif args.workload in ("head05b", "token24_05b"):
            res = cpu_head05b_run(budget_s=12.0, whole=args.workload == "token24_05b")
        else:
            res = cpu_reference_run(10 ** 6, 1, budget_s=12.0)
        if res is not None:
            cgbs, cores, sample, kind, _ = res
            cpu = {"value": round(cgbs, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                   "sample": sample}
    if rank == 0:
        line = {
            "metric": r.get("metric", METRIC), "value": round(gbs, 2), "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t / args.steps * 1e3, 5), "higher_is_better": True,
            "scaling": "weak" if args.workload in ("resident28", "single", "block28", "layer28",
                                                   "head", "token28", "resident05b",
                                                   "head05b", "token24_05b")
            else "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": r.get("data", "synthetic: seeded N(0,1) q/k/v and KV caches (gqa_fill_normal)"),
            "config": workload_config(args.workload, args.exchange),
            "tok_per_s": round(tokens / t, 1),
            "hbm_frac_of_measured": round(gbs / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "kernel": r.get("kernel", "decode_split_kernel"),
                         "algorithmic_bytes_per_launch": round(per_gpu_bytes),
                         "duration_us": round(per_gpu_bytes / achieved / 1e3, 3),
                         "duration_basis": basis,
                         "traffic": profile_traffic(args.workload, per_gpu_bytes)},
            "timing": {"rounds": r.get("rounds", 1), "timed_s": round(r.get("timed_s", t), 4),
                       "statistic": "median over rounds of the K timed steps (each round "
                                    "barrier + synchronize on both sides, max over ranks); "
                                    f"rounds until >= {MIN_TIMED_S} s timed"},
            "e2e": {"value": round(gbs_e2e, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                    "tok_per_s": round(tokens / t_e2e, 1)},
            "gpu_launches": r["launches"],
            "clocks": r["clocks"],
            "cpu_baseline": cpu,
        }
        if extra:
            line["extra"] = extra
        if k_nondefault(args):  # tuning knobs away from the library's defaults
            line["tuning"] = {"kernel_variant": args.variant, "target_ctas": args.target_ctas,
                              "batch_chunk": args.batch_chunk, "grid_merge": args.grid_merge,
                              "share_of": args.share_of}
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def k_nondefault(args):
    return (args.variant >= 0 or args.target_ctas or args.batch_chunk or not args.grid_merge
            or args.share_of > 1)


def run_extra(args, g, name, rank, world, local):
    """One of the other configurations timed in the default run: `batched`
    (64 sequences dealt to the ranks, strong scaling), `long1` (one 32768-row
    sequence split by KV range over the ranks, merged over peer memory),
    `prefill` (8 prompts of 2048 tokens dealt to the ranks, strong scaling),
    `token28` (the whole greedy decode step of the 28-layer model, one model
    per rank) or `head` (the output RMSNorm + Q6_K LM head + pick, one per
    rank)."""
    import copy
    sub = copy.copy(args)
    sub.workload = name
    if name in ("token28", "head"):
        wl = WORKLOADS[name]
        ctx = g.Context(t_max=wl["t_max"], device=local)
        try:
            r = run_head(sub, g, ctx, rank, world, local)
        finally:
            ctx.close()
        t = max_over_ranks(r["t"], world)
        total = sum_over_ranks(r["bytes"], world)
        tokens = sum_over_ranks(r["tokens"], world)
        return {"workload": workload_config(name)["workload"],
                "value": round(total / t / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(t / sub.steps * 1e3, 5), "steps": sub.steps,
                "tok_per_s": round(tokens / t, 1), "scaling": "weak",
                "rounds": r.get("rounds", 1), "clocks": r["clocks"]}
    if name == "long1":
        sub.steps = WORKLOADS["long1"]["window"]  # the peer-exchange graph holds one window
        t_max = max(n for _, n in g.shard.plan_kv_ranges(WORKLOADS["long1"]["t_max"], world))
    elif name == "prefill":
        t_max = WORKLOADS["prefill"]["t_max"]
    else:
        t_max = WORKLOADS[name]["len_hi"] + WORKLOADS[name]["window"]
    ctx = g.Context(t_max=t_max, device=local)
    try:
        runner = {"long1": run_long1, "prefill": run_prefill}.get(name, run_batched)
        r = runner(sub, g, ctx, rank, world, local)
    finally:
        ctx.close()
    t = max_over_ranks(r["t"], world)
    tokens = sum_over_ranks(r["tokens"], world)
    if name == "prefill":
        flops = sum_over_ranks(r["flops"], world)
        return {"workload": workload_config(name)["workload"],
                "value": round(flops / t / 1e12, 1), "unit": "TFLOP/s",
                "ms_per_step": round(t / sub.steps * 1e3, 5), "steps": sub.steps,
                "tok_per_s": round(tokens / t, 1), "scaling": "strong",
                "rounds": r["rounds"], "clocks": r["clocks"]}
    total = sum_over_ranks(r["bytes"], world)
    return {"workload": workload_config(name, args.exchange)["workload"],
            "value": round(total / t / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(t / sub.steps * 1e3, 5), "steps": sub.steps,
            "tok_per_s": round(tokens / t, 1), "scaling": "strong",
            "rounds": r["rounds"], "clocks": r["clocks"]}


def report_prefill(args, r, ctx, rank, world):
    t = max_over_ranks(r["t"], world)
    t_e2e = max_over_ranks(r["t_e2e"], world)
    flops = sum_over_ranks(r["flops"], world)
    tokens = sum_over_ranks(r["tokens"], world)
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            # the step is timed alone (short, not power-capped): the burst figure
            peak, src = float(json.load(f)["bf16_tflops"]), "measured bf16_tflops (burst)"
    except Exception:
        peak, src = 1590.0, "fallback burst"
    tf = flops / t / 1e12
    if rank == 0:
        line = {
            "metric": PREFILL_METRIC, "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) q/k/v (gqa_fill_normal)",
            "config": workload_config("prefill"), "tok_per_s": round(tokens / t, 1),
            "roofline": {"bound": "tensor", "achieved": round(tf / world, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tf / world / peak, 4),
                         "peak_source": src, "kernel": "prefill_attn_kernel (+ prep kernel)",
                         "algorithmic_flops_per_step": 4.0 * N_Q * D * 2048 * 2049 / 2 * 8,
                         "achieved_scope": "whole step (prep + attention kernels)",
                         "traffic": profile_traffic("prefill", scale=1.0 / world)},
            "e2e": {"value": round(flops / t_e2e / 1e12, 1), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
            "gpu_launches": r["launches"], "clocks": r["clocks"], "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def main():
    global MIN_TIMED_S
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="resident28")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--min-timed-s", type=float, default=MIN_TIMED_S,
                    help="repeat the K timed steps until this much device time is timed "
                         "(0: one round, e.g. under a profiler)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the sharded configurations the default run also times")
    # tuning knobs (defaults are the library's own choices)
    ap.add_argument("--variant", type=int, default=-1, help=argparse.SUPPRESS)
    ap.add_argument("--target-ctas", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--batch-chunk", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--share-of", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--grid-merge", type=int, default=1, help=argparse.SUPPRESS)
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer", help=argparse.SUPPRESS)
    args = ap.parse_args()
    MIN_TIMED_S = max(0.0, args.min_timed_s)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

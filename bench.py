"""Embedded tokens/s of the B200 executor on BASELINE's wave configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1] [--impl b200|reference]

One step = one packed wave through the whole 24-layer graph on each GPU
(config 1: 16 sequences x 128 tokens = 2048 tokens; config 2: 1 x 2048;
config 0: the 4-sequence parity wave).  Every rank holds its own weight
replica and embeds its own wave (weak scaling, no data-path collective); the
process group only provides the barrier and the max-over-ranks time.

value  -- device time of K graph replays with inputs resident in HBM, CUDA
          events on the executor's stream, an L2 flush (256 MiB write) between
          steps outside the timed events; whole-job tokens / max-rank time.
e2e    -- the same waves through ei_gemma2_kfd_batch with host buffers: ids /
          bounds / positions H2D and the embeddings D2H every step, wall time.
--impl reference runs the reference's own CPU graph (oracle/_ref, compiled
from its sources) on the same workload on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "embedded tokens/s per box (2048-token waves)"
CONFIGS = {0: ("config0: 4 sequences, bodies 8/17/33/64 + BOS/EOS (130 tokens)", (8, 17, 33, 64)),
           1: ("config1: 16 x 128-token sequences = one 2048-token wave", (126,) * 16),
           2: ("config2: 1 x 2048-token sequence", (2046,))}


def q8_gemm_ops(n_tokens: int) -> float:
    """Algorithmic int8 ops (2*M*N*K) of the Q8_0 GEMMs for one wave."""
    per_tok = 0
    for l in range(24):
        d = 512 if l % 6 == 5 else 256
        per_tok += 512 * (4 * d + 1024)  # q, k, v
        per_tok += 4 * d * 512           # attn_output
        per_tok += 512 * 4096            # ffn up + gate
        per_tok += 2048 * 512            # ffn_down
        per_tok += 2 * 512 * 512         # inp_gate, proj
    per_tok += 512 * 768                 # output
    return 2.0 * per_tok * n_tokens


# DRAM bytes (read + write) per q8gemm launch, averaged over the 145 GEMM
# launches of one config-1 wave in one ncu capture (cold cache); the command
# and the totals are in profiles/q8gemm_wave_dram.md.
GEMM_DRAM_BYTES_PER_LAUNCH = 3.07e6


# The executor uploads each wave's inputs as one block: ids, bounds (2 words),
# positions, offsets (2048 tokens each) and the sequence count.
H2D_BYTES_PER_WAVE = (5 * 2048 + 2) * 4


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc = device, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        rows = []
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) >= 9:
                try:
                    rows.append((float(f[1]), float(f[2]), f[5:9]))
                except ValueError:
                    pass
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline_run(model_path, lengths, steps, warmup, seed):
    """The reference's own CPU graph (oracle/_ref) on the same waves."""
    import oracle
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    ids, off = syn.wave(lengths, seed=seed)
    ref = oracle.RefGraph(model_path, 0)
    for _ in range(warmup):
        ref.embed(ids, off)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        ref.embed(ids, off)
        times.append(time.perf_counter() - t0)
    n = int(off[-1])
    med = statistics.median(times)
    res = {"value": n / med, "unit": "tokens/s", "cores": ref.threads, "kind": "reference",
           "tier": ref.tier,
           "sample": f"{len(lengths)} x {n // len(lengths)}-token wave ({n} tokens), median of {steps} after "
                     f"{warmup} warm-up, ei_gemma2_embed_batch_fast_ctx with {ref.threads} threads"}
    ref.close()
    return res


def dist_init(backend="nccl"):
    """One process per GPU (torchrun env); the group carries only the barrier and
    the max-over-ranks time, never embedding data."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        kw = {}
        if backend == "nccl":
            import torch
            kw["device_id"] = torch.device(f"cuda:{local}")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
    return rank, world, local


def rank_wave(lengths, rank):
    """Each rank embeds its own wave of the same shape (weak scaling): the units
    are whole waves, so ranks share nothing on the data path."""
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    return syn.wave(lengths, seed=100 + rank)


def whole_job_rate(tokens_per_rank, world, steps, ms_max):
    """Tokens all ranks embedded / the slowest rank's time."""
    return tokens_per_rank * world * steps / (ms_max * 1e-3)


def reference_arm(args, rank, world):
    if rank != 0:
        return
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    desc, lengths = CONFIGS[args.config]
    model = syn.model_path(1234, "baseline")
    cpu = cpu_baseline_run(model, lengths, args.steps, args.warmup, seed=100)
    n = sum(l + 2 for l in lengths)
    line = {"metric": METRIC, "value": cpu["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * n / cpu["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8+fp32", "data": "synthetic",
            "config": {"workload": desc, "model": "EmbeddingGemma 2 text graph, seeded synthetic GGUF (seed 1234, "
                       "BASELINE weight distributions)", "tokens_per_wave": n},
            "impl": "reference", "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_init()
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return finalize(world)

    import torch
    eg2 = importlib.import_module("embeddinggemma2-amdkfd_b200")
    syn = eg2.synthetic
    desc, lengths = CONFIGS[args.config]
    model_path = syn.model_path(1234, "baseline")
    torch.cuda.set_device(local)
    model = eg2.GGUFModel(model_path)
    ex = eg2.Gemma2Executor(model, local)
    ids, off = rank_wave(lengths, rank)
    n, batch = int(off[-1]), len(off) - 1
    stream = torch.cuda.ExternalStream(ex.stream, device=local)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=local)

    # ---- value: device-resident waves
    ex.stage(ids, off)
    for _ in range(args.warmup):
        ex.launch(1)
    ex.finish()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.zero_()  # L2 flush, outside the timed events
                starts[i].record(stream)
                ex.launch(1)
                ends[i].record(stream)
        torch.cuda.synchronize()
    barrier(world)
    out_dev = ex.finish()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    dev_ms = sum(step_ms)
    dev_ms_max = reduce_max(dev_ms, world, f"cuda:{local}")

    # ---- e2e: the public C ABI with host buffers every step
    for _ in range(args.warmup):
        ex.batch(ids, off)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = ex.batch(ids, off)
    e2e_ms = (time.perf_counter() - t0) * 1000.0
    barrier(world)
    e2e_ms_max = reduce_max(e2e_ms, world, f"cuda:{local}")
    assert np.isfinite(out).all() and np.allclose(out, out_dev, atol=1e-6)

    # ---- dominant kernel: per-group event timing of one eager wave
    ex.stage(ids, off)
    prof = ex.profile()
    gemm_ms = sum(v for k, v in prof.items() if k.startswith("gemm_"))
    pk, src = peaks()
    int8_peak = 2.0 * pk["bf16_tflops_sustained"]
    achieved = q8_gemm_ops(n) / (gemm_ms * 1e-3) / 1e12
    line = {
        "metric": METRIC,
        "value": whole_job_rate(n, world, args.steps, dev_ms_max),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8+fp32", "data": "synthetic",
        "config": {"workload": desc, "model": "EmbeddingGemma 2 text graph, seeded synthetic GGUF (seed 1234, "
                   "BASELINE weight distributions)", "tokens_per_wave_per_gpu": n, "sequences_per_wave": batch,
                   "parallelism": f"replicas x{world} (whole waves per GPU, no collective)",
                   "l2": "256 MiB write between timed steps; per-wave working set > L2 (151 MB weights, 100 MB PLE)"},
        "e2e": {"value": whole_job_rate(n, world, args.steps, e2e_ms_max), "unit": "tokens/s",
                "h2d_bytes_per_step": H2D_BYTES_PER_WAVE,
                "d2h_bytes_per_step": batch * 768 * 4},
        "gpu_launches": ex.kernels_per_wave * args.steps,
        "roofline": {"kernel": "q8gemm_kernel (all Q8_0 GEMM launches of a wave)", "bound": "tensor",
                     "achieved": achieved, "peak": int8_peak, "unit": "TOP/s", "frac": achieved / int8_peak,
                     "peak_source": f"2 x bf16_tflops_sustained of {src} MEASURED_PEAKS (dense int8 = 2x bf16)",
                     "traffic": GEMM_DRAM_BYTES_PER_LAUNCH,
                     "traffic_note": "dram read+write bytes per launch, ncu capture averaged over one wave's GEMMs"},
        "profile_ms": {k: round(v, 4) for k, v in prof.items()},
    }
    c = clocks.summary()
    line["clocks"] = c
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_run(model_path, lengths, 3, 1, seed=100)
    if rank == 0:
        print(json.dumps(line), flush=True)
    del ex
    finalize(world)


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_max(v, world, device):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def finalize(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

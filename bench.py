#!/usr/bin/env python3
"""Throughput benchmark of the B200 encoder layer (UserOptimizedTransformer.forward).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload batch|dense|short|long|refN]

Metric: layer-forward tokens/s = B*S / step time (padded tokens counted, the
reference's definition, torch_transformer_benchmark.py:565-567), whole job.

Default workload (`batch`): one global batch of B=32 sequences of S=4096,
d_model=1024, 16 heads, FFN 4096, one layer, non-causal, right-padded mask
with lengths ~ U[1024, 4096], LayerNorm gamma ~ 1+0.02N(0,1), beta ~
0.02N(0,1), seeded default-init weights.  The batch is split over the N
ranks (one process per GPU, torchrun, NCCL), B/N samples each balanced by
work; a step is the forward of every rank's share AND the output gather
(every rank ends with the [B, S, D] output: the valid rows are pushed over
NVLink by the copy engines, overlapped with the next micro-batch), timed
together, so the
curve over N is strong scaling with the gather inside.  The step time is the
max over ranks of the CUDA-event time of the K timed steps.

The same JSON line nests, measured in the same run at the same N:
  dense_b8_s2048     the single-GPU dense layer (B=8 S=2048, lengths U[S/2,S])
                     per rank (weak scaling), with its attention roofline;
  short_b64_s128     the short-sequence heavy-padding layer (B=64 S=128
                     d_model=768 H=12 FFN=3072, lengths U[1,S]) per rank;
  context_parallel   one sequence of S=131072 (lengths U[0.9S, S]) over the
                     N ranks (context parallel; the plain model at N=1), with
                     peak memory per GPU;
  sustained          >= 3 s of back-to-back headline steps with the SM clock
                     sampled, against the sustained tensor peak;
  official_shapes    (N=1) the reference's official shapes #1-#13, each gated
                     and timed, with the ratio to its published RTX 5090 numbers.
Every timed workload except the long sequence is first gated against the CPU
FP32 oracle on one sample of the timed input (the reference's strict gate); a
failure stops the run before any timing (torch_transformer_benchmark.py:725-728).

Rank 0 prints one JSON line.  `--impl reference` times the reference's CPU
FP32 path (the oracle restatement of BaselineTransformer) on the host cores,
rotating through the samples of the same batch.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: (B, S, D, H, F, layers, causal, padding_ratio, ln_perturb, description)
    "batch": (32, 4096, 1024, 16, 4096, 1, False, 0.75, True,
              "batch-sharded encoder layer B=32 S=4096 d_model=1024 H=16 FFN=4096, L~U[S/4,S]"),
    "dense": (8, 2048, 1024, 16, 4096, 1, False, 0.5, True,
              "dense encoder layer B=8 S=2048 d_model=1024 H=16 FFN=4096, L~U[S/2,S]"),
    "short": (64, 128, 768, 12, 3072, 1, False, 0.999, False,
              "short-sequence heavy-padding layer B=64 S=128 d_model=768 H=12 FFN=3072, L~U[1,S]"),
    "long": (1, 131072, 1024, 16, 4096, 1, False, 0.1, False,
             "long single sequence B=1 S=131072 d_model=1024 H=16 FFN=4096, L~U[0.9S,S]"),
}

# The reference's official test shapes (STATEMENT.md 3.7, tools/matrix_runner.py:49-64):
# (id, batch, d_model, heads, seq_len, layers, ffn_dim), all causal, no padding.
REFERENCE_SHAPES = (
    (1, 64, 128, 4, 128, 4, 128), (2, 1, 128, 4, 128, 4, 128), (3, 4, 128, 4, 128, 4, 128),
    (4, 16, 128, 4, 128, 4, 128), (5, 128, 128, 4, 128, 4, 128), (6, 10000, 128, 4, 128, 4, 128),
    (7, 64, 32, 4, 128, 4, 32), (8, 64, 1024, 4, 128, 4, 1024), (9, 64, 128, 1, 128, 4, 128),
    (10, 64, 128, 2, 128, 4, 128), (11, 64, 128, 16, 128, 4, 128), (12, 64, 128, 4, 32, 4, 128),
    (13, 64, 128, 4, 1024, 4, 128), (14, 32, 1024, 16, 100000, 2, 1024),
)
for _sid, _b, _d, _h, _s, _l, _f in REFERENCE_SHAPES:
    WORKLOADS[f"ref{_sid}"] = (_b, _s, _d, _h, _f, _l, True, 0.0, False,
                               f"reference official shape #{_sid}: B={_b} S={_s} d_model={_d} H={_h} "
                               f"FFN={_f} layers={_l} causal, no padding")

# The reference's published throughput (tokens/s, B*S basis) for its official
# shapes on one RTX 5090: results/final/main_shapes_1_13.csv (optimized_throughput)
# and results/final/main_shape14_summary.json (#14).
PUBLISHED_RTX5090 = {
    1: 60995948.61, 2: 1155401.48, 3: 4621605.94, 4: 18317114.73, 5: 77929982.39, 6: 50831314.74,
    7: 73268458.91, 8: 2932400.22, 9: 54151242.44, 10: 58340931.34, 11: 44046799.59, 12: 18653453.54,
    13: 60721063.02, 14: 457962.98,
}

# Workloads whose global batch is split over the ranks (strong scaling, output gather timed).
SPLIT_BATCH = ("batch",)
TIMING_SEED = 1234 + 100000  # timing inputs use seed + 100000 (torch_transformer_benchmark.py:533)

PEAK_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAK_FALLBACK, "fallback"


def workload_config(workload):
    """The `config` object of the JSON line (the same in both arms)."""
    B, S, D, H, F, L, causal, pad, ln, desc = WORKLOADS[workload]
    min_valid = S if pad <= 0 else max(1, int(round(S * (1.0 - pad))))
    return {"workload": desc, "global_batch": B, "seq_len": S, "d_model": D, "heads": H, "ffn_dim": F,
            "layers": L, "causal": causal, "valid_lengths": f"U[{min_valid}, {S}]", "seed": TIMING_SEED}


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, backend):
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))


def barrier(world, device=None):
    if world > 1:
        import torch.distributed as dist

        if device is not None:
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


def reduce_over_ranks(world, value, device, op="max"):
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
    return float(t.item())


def gather_to_all(world, values, device):
    """List of every rank's `values` (a flat list of floats), by rank."""
    if world == 1:
        return [list(values)]
    import torch.distributed as dist

    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [p.tolist() for p in parts]


# ---------------------------------------------------------------------------
# Clock sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sms, maxes, power, reasons = [], [], [], {}
        for r in rows:
            try:
                sm = float(r[1])
                mx = float(r[2])
            except (ValueError, IndexError):
                continue
            sms.append(sm)
            maxes.append(mx)
            try:
                power.append(float(r[3]))
            except (ValueError, IndexError):
                pass
            for n, v in zip(self.REASONS, r[5:9]):
                if v.strip().lower() == "active":
                    reasons[n] = reasons.get(n, 0) + 1
        if not sms:
            return None
        loaded = [s for s in sms if s > 0.5 * max(sms)]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "reason_samples": reasons, "samples": len(sms), "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------
# Workload construction
# ---------------------------------------------------------------------------
class Case:
    """One rank's view of a workload: the global batch, the work-balanced
    assignment (split workloads), this rank's share and the parameters."""

    def __init__(self, workload, rank, world):
        import oracle

        B, S, D, H, F, L, causal, pad, ln, _ = WORKLOADS[workload]
        self.workload = workload
        self.split = workload in SPLIT_BATCH
        self.cfg_global = oracle.TransformerConfig(B, S, D, H, F, L, causal)
        sd = oracle.make_state_dict(self.cfg_global, seed=1234)
        self.sd = oracle.perturb_layernorm(sd, 1234) if ln else sd
        seed = TIMING_SEED if self.split else TIMING_SEED + 7919 * rank  # weak scaling: a batch per rank
        self.x, self.mask = oracle.generate_random_case(self.cfg_global, seed=seed, padding_ratio=pad)
        self.lengths = self.mask.to(torch.int64).sum(1).tolist()
        self.right_padded = bool(all(bool(self.mask[b, :n].all()) for b, n in enumerate(self.lengths)))
        if self.split and world > 1:
            if B % world != 0:
                raise SystemExit(f"--workload {workload}: batch {B} does not split over {world} GPUs")
            from techjam_b200 import sharding

            self.assignment = sharding.balanced_assignment(self.lengths, world, D, F)
            self.mine = self.assignment[rank]
        else:
            self.assignment = [list(range(B))] if self.split else None
            self.mine = list(range(B))
        idx = torch.tensor(self.mine, dtype=torch.int64)
        self.x_local = self.x[idx].contiguous()
        self.mask_local = self.mask[idx].contiguous()
        self.cfg_local = oracle.TransformerConfig(len(self.mine), S, D, H, F, L, causal)

    def model(self, pkg, device):
        c = self.cfg_global
        m = pkg.UserOptimizedTransformer(pkg.TransformerConfig(*c.__dict__.values()))
        m.load_state_dict(self.sd, strict=True)
        return m.to(device).eval()


def algorithmic_work(cfg, lengths):
    """Valid-token FLOPs of one layer forward over samples of these lengths:
    (valid tokens, GEMM FLOPs, attention FLOPs)."""
    lens = torch.tensor(lengths, dtype=torch.float64)
    D, F = cfg.d_model, cfg.ffn_dim
    nv = float(lens.sum())
    attn = float((4.0 * lens * lens * D).sum())  # QK^T + PV
    if cfg.causal:
        attn = float((2.0 * lens * (lens + 1) * D).sum())  # the lower triangle
    gemm = nv * (8.0 * D * D + 4.0 * D * F)
    return nv, gemm * cfg.num_layers, attn * cfg.num_layers


def accuracy_gate(out, case, sample, what, world):
    """The reference refuses to benchmark an implementation that fails its
    accuracy check (torch_transformer_benchmark.py:725-728): output row
    `sample` of the timed input against the CPU FP32 oracle, strict gate."""
    import oracle

    threads = torch.get_num_threads()
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    try:
        c = case.cfg_global
        one = oracle.TransformerConfig(1, c.seq_len, c.d_model, c.num_heads, c.ffn_dim, c.num_layers, c.causal)
        xs, ms = case.x[sample : sample + 1], case.mask[sample : sample + 1]
        if c.seq_len > 8192:
            ref = oracle.encoder_forward_blocked(case.sd, one, xs, ms, query_chunk=512)
        else:
            ref = oracle.encoder_forward(case.sd, one, xs, ms)
        r = oracle.compare_outputs(ref, out.detach().float().cpu().view_as(ref))
    finally:
        torch.set_num_threads(threads)
    return {"what": what, "sample": sample, "passed": r.passed, "failed_elements": r.failed_elements,
            "max_abs_error": r.max_abs_error}


def fail_on_gate(world, device, gate):
    ok = reduce_over_ranks(world, 1.0 if gate["passed"] else 0.0, device, op="min")
    if ok < 1.0:
        raise SystemExit(f"accuracy gate failed, refusing to time: {gate}")


def timed(fn, steps, world, device, sample_clocks=True, local=0):
    """Device time (ms, max over ranks) of `steps` calls of fn, bracketed by
    barrier + synchronize on both sides; nvidia-smi clocks sampled meanwhile."""
    stream = torch.cuda.current_stream(device)
    sampler = ClockSampler(local).start() if sample_clocks else None
    if sampler is not None:
        time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world, device)
    torch.cuda.synchronize(device)
    start.record(stream)
    for i in range(steps):
        fn(i)
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier(world, device)
    clocks = sampler.stop() if sampler is not None else None
    ms_local = start.elapsed_time(end)
    return reduce_over_ranks(world, ms_local, device), ms_local, clocks


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def run_ours(args, world, rank, local):
    import __graft_entry__

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_dist(world, "nccl")
    pkg = __graft_entry__.load_package()
    try:
        if args.workload == "long":
            line = measure_long(pkg, args, world, rank, local, device, headline=True)
        else:
            line = measure_headline(pkg, args, world, rank, local, device)
            if args.workload == "batch" and not args.no_extras:
                dense = measure_headline(pkg, argparse.Namespace(**{**vars(args), "workload": "dense"}), world,
                                         rank, local, device, nested=True)
                short = measure_headline(pkg, argparse.Namespace(**{**vars(args), "workload": "short"}), world,
                                         rank, local, device, nested=True)
                cp = measure_long(pkg, args, world, rank, local, device, headline=False)
                shapes = measure_official_shapes(pkg, args, device) if world == 1 else None
                if rank == 0:
                    line["dense_b8_s2048"] = dense
                    line["short_b64_s128"] = short
                    line["context_parallel"] = cp
                    line["official_shapes"] = shapes
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[device.index])
            dist.destroy_process_group()
    return line


def measure_headline(pkg, args, world, rank, local, device, nested=False):
    from techjam_b200 import sharding

    case = Case(args.workload, rank, world)
    cfg = case.cfg_global
    B, S = cfg.batch_size, cfg.seq_len
    model = case.model(pkg, device)
    encoder = sharding.BatchShardedEncoder(model, micro_batches=args.micro_batches,
                                           transport=args.gather_transport, copy_streams=args.copy_streams)
    gather = case.split and world > 1
    lengths = case.lengths if case.right_padded else None
    mask_local = case.mask_local.to(device)
    # Inputs larger than L2 between timed steps: x rotates over buffers whose
    # total exceeds the 126 MB L2 (and every step writes ~1 GB of activations).
    x_bytes = max(1, case.x_local.numel() * 4)
    big = x_bytes > 2**31
    n_rot = 1 if (big or x_bytes >= 256e6) else max(2, math.ceil(256e6 / x_bytes))
    xs = [case.x_local.to(device) for _ in range(n_rot)]

    def step(i):
        if gather:
            return encoder.forward(xs[i % n_rot], mask_local, gather=True, assignment=case.assignment,
                                   valid_lengths=lengths)
        return model(xs[i % n_rot], mask_local)

    with torch.inference_mode():
        for i in range(args.warmup):
            out = step(i)
        torch.cuda.synchronize(device)
        pkg._lib.device_status(torch.cuda.current_stream(device).cuda_stream)
        # accuracy gate on the timed input: at N>1 a sample another rank computed
        if case.split:
            owner = (rank + 1) % world
            sample = (case.assignment[owner] or case.mine or [0])[0]
            row = out[sample] if gather else out[case.mine.index(sample)]
        else:
            sample, row = 0, out[0]
        gate = accuracy_gate(row, case, sample, args.workload, world)
        fail_on_gate(world, device, gate)
        del out, row

        ms_total, ms_local, clocks = timed(step, args.steps, world, device, local=local)
        pkg._lib.device_status(torch.cuda.current_stream(device).cuda_stream)
    ms_step = ms_total / args.steps
    tokens_per_step = B * S * (1 if case.split else world)
    value = tokens_per_step / (ms_step / 1e3)
    nv_local, _, _ = algorithmic_work(cfg, [case.lengths[j] for j in case.mine])
    per_rank = gather_to_all(world, [len(case.mine), nv_local, ms_local / args.steps], device)
    nv_all, gemm_f, attn_f = algorithmic_work(cfg, case.lengths)
    flops_step = (gemm_f + attn_f) * (1 if case.split else world)

    sustained = None
    if not nested and not args.no_extras:
        sustained = measure_sustained(step, ms_step, world, device, local, flops_step)
    e2e = None if big else measure_e2e(case, model, device, args, world, gather, lengths)
    kernels = kernel_breakdown(pkg, model, case, device, args) if (rank == 0 and not big) else None
    if gather:
        encoder.close()

    if rank != 0:
        return None
    peaks, peak_kind = load_peaks()
    roof = roofline(kernels, peaks, peak_kind, args.workload) if kernels else None
    line = {
        "metric": "layer-forward tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong" if case.split else "weak",
        "vs_baseline": None,
        "dtype": "fp16 operands, fp32 accumulate/LayerNorm/residual/output",
        "data": "synthetic (seeded N(0,1) inputs, default-init weights, right-padded masks)",
        "config": workload_config(args.workload),
        "parallelism": (f"batch split x{world}: {B // world} samples per GPU balanced by work; the step includes "
                        "the output gather (valid rows pushed over NVLink into every "
                        f"GPU's [B,S,D] output, {encoder.micro_batches} micro-batches overlapping it, "
                        f"transport: {encoder.transport}"
                        + (f", {encoder.copy_streams} stream{'s' if encoder.copy_streams > 1 else ''} per "
                           "destination)" if encoder.transport == "copy_engine" else ")")
                        if gather else
                        (f"batch split x{world}" if case.split else
                         f"x{world}: each GPU runs its own batch of {B} (weak scaling, no collective)")),
        "l2_policy": (f"inputs larger than L2: x rotates over {n_rot} buffer(s) of {x_bytes / 2**20:.0f} MiB; "
                      "each step writes ~1 GB or more of activations"),
        "valid_tokens": int(nv_all) * (1 if case.split else world),
        "ranks": [{"rank": r, "samples": int(p[0]), "valid_tokens": int(p[1]), "ms_per_step": p[2]}
                  for r, p in enumerate(per_rank)],
        "tflops_valid": flops_step / (ms_step / 1e3) / 1e12,
        "accuracy_gate": gate,
        "gpu_launches": launches_per_step(case, gather, encoder.micro_batches,
                                          encoder.transport == "kernel") * args.steps,
        "roofline": roof,
        "kernels": kernels,
        "clocks": clocks,
        "e2e": e2e,
        "sustained": sustained,
    }
    if not nested:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args.workload, budget_s=args.cpu_budget)
        line["cpu_baseline"] = cpu
    return line


def measure_official_shapes(pkg, args, device):
    """The reference's official shapes #1-#13 (causal, no padding, 4 layers;
    tools/matrix_runner.py:49-64) on this GPU: each gated on sample 0 against
    the FP32 oracle (the accuracy check the reference's runner makes before
    timing a shape), then K forwards timed back to back with CUDA events, and
    the ratio to the reference's published RTX 5090 throughput.  #14 (13 GB of
    input) runs with --workload ref14."""
    rows = []
    for sid in range(1, 14):
        case = Case(f"ref{sid}", 0, 1)
        cfg = case.cfg_global
        model = case.model(pkg, device)
        x = case.x.to(device)
        m = case.mask.to(device)
        with torch.inference_mode():
            for _ in range(args.warmup):
                out = model(x, m)
            torch.cuda.synchronize(device)
            gate = accuracy_gate(out[0], case, 0, f"ref{sid}", 1)
            if not gate["passed"]:
                raise SystemExit(f"accuracy gate failed at official shape #{sid}, refusing to time: {gate}")
            steps = max(args.steps, 20)
            ms_total, _, _ = timed(lambda i: model(x, m), steps, 1, device, sample_clocks=False)
        ms = ms_total / steps
        value = cfg.batch_size * cfg.seq_len / (ms / 1e3)
        rows.append({"shape": sid, "B": cfg.batch_size, "S": cfg.seq_len, "d_model": cfg.d_model,
                     "heads": cfg.num_heads, "ffn_dim": cfg.ffn_dim, "layers": cfg.num_layers, "ms": ms,
                     "tokens_per_s": value, "reference_rtx5090_tokens_per_s": PUBLISHED_RTX5090[sid],
                     "ratio": value / PUBLISHED_RTX5090[sid], "gate_max_abs": gate["max_abs_error"]})
        del model, x, m, out
    ratios = [r["ratio"] for r in rows]
    return {"shapes": rows, "geomean_ratio_1_13": math.exp(sum(math.log(r) for r in ratios) / len(ratios)),
            "note": "ratio = tokens/s here / the reference's published RTX 5090 tokens/s "
                    "(results/final/main_shapes_1_13.csv); every shape gated on sample 0 first"}


def launches_per_step(case, gather, micro_batches, push_kernel):
    """Our kernels per step: per forward the token plan, 7 per layer and the
    final LayerNorm; with the kernel transport, one push kernel per micro-batch."""
    from techjam_b200 import sharding

    L = case.cfg_global.num_layers
    forwards = len(sharding.micro_batch_ranges(len(case.mine), micro_batches)) if gather else (1 if case.mine else 0)
    return forwards * (2 + 7 * L + (1 if gather and push_kernel else 0))


def measure_sustained(step, ms_step, world, device, local, flops_step):
    """>= 3 s of back-to-back steps: the throughput a long run holds once the
    GPU sits at its power cap, with the SM clock sampled meanwhile."""
    n = max(10, int(math.ceil(3000.0 / max(ms_step, 1e-3))))
    with torch.inference_mode():
        ms_total, _, clocks = timed(step, n, world, device, local=local)
    peaks, kind = load_peaks()
    ms = ms_total / n
    tflops = flops_step / (ms / 1e3) / 1e12
    sus = peaks.get("bf16_tflops_sustained", PEAK_FALLBACK["bf16_tflops_sustained"])
    return {"steps": n, "seconds": ms_total / 1e3, "ms_per_step": ms, "tflops_valid": tflops,
            "tflops_valid_per_gpu": tflops / world, "frac_of_sustained_peak": tflops / world / sus,
            "sustained_peak_tflops_per_gpu": sus, "peak_source": kind, "clocks": clocks}


def measure_long(pkg, args, world, rank, local, device, headline):
    """One sequence of S=131072 (lengths U[0.9S, S]): context parallel over the
    ranks (valid-token balanced chunks, K/V all-gathered over NCCL every
    layer); at N=1 the plain model.  Peak memory per GPU reported."""
    from techjam_b200 import sharding

    case = Case("long", 0, 1)  # the same sequence on every rank
    cfg = case.cfg_global
    S = cfg.seq_len
    model = case.model(pkg, device)
    steps = args.steps if headline else max(3, min(args.steps, 10))
    warm = args.warmup if headline else 3
    torch.cuda.synchronize(device)
    torch.cuda.reset_peak_memory_stats(device)
    if world > 1:
        ranges = sharding.sequence_ranges(case.mask[0], world)
        a, b = ranges[rank]
        slab = max(e - s for s, e in ranges)
        cp = sharding.ContextParallelEncoder(model)
        x = case.x[:, a:b].contiguous().to(device)
        m = case.mask[:, a:b].contiguous().to(device)
        fn = lambda i: cp.forward(x, m, slab)  # noqa: E731
    else:
        ranges = [(0, S)]
        x = case.x.to(device)
        m = case.mask.to(device)
        fn = lambda i: model(x, m)  # noqa: E731
    with torch.inference_mode():
        for i in range(warm):
            fn(i)
        torch.cuda.synchronize(device)
        ms_total, _, clocks = timed(fn, steps, world, device, local=local)
    ms = ms_total / steps
    peak_gib = reduce_over_ranks(world, torch.cuda.max_memory_allocated(device) / 2**30, device)
    nv, gemm_f, attn_f = algorithmic_work(cfg, case.lengths)
    del model, x, m, fn
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    d = {
        "value": S / (ms / 1e3),
        "unit": "tokens/s",
        "ms_per_step": ms,
        "steps": steps,
        "n_gpus": world,
        "parallelism": (f"context parallel x{world}: valid-token balanced chunks, NCCL all-gather of K/V"
                        if world > 1 else "one GPU"),
        "chunk_ranges": ranges,
        "valid_tokens": int(nv),
        "tflops_valid": (gemm_f + attn_f) / (ms / 1e3) / 1e12,
        "peak_memory_gib_per_gpu": peak_gib,
        "clocks": clocks,
        "gated_by": "tests/test_gpu_layer.py (one GPU) and tests/multi_gpu_worker.py (context parallel): "
                    "three 256-row query blocks against the query-row oracle",
    }
    if headline:
        d.update({"metric": "layer-forward tokens/s", "warmup": args.warmup,
                  "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                  "dtype": "fp16 operands, fp32 accumulate/LayerNorm/residual/output",
                  "data": "synthetic (seeded N(0,1) input, default-init weights, right-padded mask)",
                  "config": workload_config("long"), "gpu_launches": (2 + 7 * cfg.num_layers) * steps})
    return d


def measure_e2e(case, model, device, args, world, gather, lengths):
    """Same metric through the public API with host buffers: every step copies
    its input share from pinned host memory to the device, runs the forward
    (and, split over N GPUs, the output gather) and copies this rank's share
    of the output back to pinned host memory, all inside the timed region.
    With right-padded masks only the valid rows cross the host link in
    either direction (techjam_b200.hostio): the layer never reads x at a
    padded row and writes exact zeros there, so the host writes those zero
    rows of its output itself, inside the timed region too.
    Steps are pipelined the way a serving loop runs them: the upload of step
    i+1 and the download of step i-1 (two copy streams) overlap the forward of
    step i (compute stream), with events ordering each step's three stages.
    The pinned-copy bandwidth of rank 0, measured alone, is reported beside
    it so the host-link limit can be located."""
    from techjam_b200 import hostio, sharding

    steps = max(3, min(args.steps, 60))
    nbuf = 3
    x_cpu, mask_cpu = case.x_local, case.mask_local
    # three exchange buffers: the download of step i-3 is the last reader of
    # the buffer the gather of step i writes, and it completes before step i-1
    encoder = sharding.BatchShardedEncoder(model, micro_batches=args.micro_batches, buffers=3,
                                           transport=args.gather_transport, copy_streams=args.copy_streams)
    mine = torch.tensor(case.mine, dtype=torch.int64, device=device)
    x_host = [x_cpu.clone().pin_memory() for _ in range(nbuf)]
    m_host = mask_cpu.pin_memory()
    out_host = [torch.empty_like(x_cpu).pin_memory() for _ in range(nbuf)]
    x_dev = [torch.zeros_like(x_cpu, device=device) for _ in range(nbuf)]
    # Right-padded masks: upload only each sample's valid rows, the rows the
    # layer reads (its output at padded rows is zero whatever x holds there).
    local_lengths = [int(lengths[b]) for b in case.mine] if lengths is not None else None
    m_dev = [torch.empty_like(mask_cpu, device=device) for _ in range(nbuf)]
    outs = [None] * nbuf
    compute = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    up_done = [torch.cuda.Event() for _ in range(nbuf)]
    fwd_done = [torch.cuda.Event() for _ in range(nbuf)]
    down_done = [torch.cuda.Event() for _ in range(nbuf)]

    def forward(b):
        if gather:
            full = encoder.forward(x_dev[b], m_dev[b], gather=True, assignment=case.assignment,
                                   valid_lengths=lengths)
            return full.index_select(0, mine)  # this rank's share of the gathered output
        return model(x_dev[b], m_dev[b])

    def run(n):
        for i in range(n + 2):
            if i < n:  # upload step i
                b = i % nbuf
                h2d.wait_event(fwd_done[b])  # buffer b's previous forward has read x_dev[b]
                with torch.cuda.stream(h2d):
                    if local_lengths is None:
                        x_dev[b].copy_(x_host[b], non_blocking=True)
                    else:
                        hostio.upload_valid_rows(x_host[b], x_dev[b], local_lengths)
                    m_dev[b].copy_(m_host, non_blocking=True)
                up_done[b].record(h2d)
            if 1 <= i <= n:  # forward step i-1
                b = (i - 1) % nbuf
                compute.wait_event(up_done[b])
                compute.wait_event(down_done[b])  # the download of step i-4 (same host buffer) is done
                outs[b] = forward(b)
                fwd_done[b].record(compute)
            if i >= 2:  # download step i-2
                b = (i - 2) % nbuf
                d2h.wait_event(fwd_done[b])
                with torch.cuda.stream(d2h):
                    if local_lengths is None:
                        out_host[b].copy_(outs[b], non_blocking=True)
                    else:
                        # the host zero fill below must not race the previous
                        # download into the same host buffer
                        down_done[b].synchronize()
                        hostio.download_valid_rows(outs[b], out_host[b], local_lengths)
                outs[b].record_stream(d2h)
                down_done[b].record(d2h)

    with torch.inference_mode():
        for e in down_done + fwd_done:
            e.record(compute)
        run(3)
        torch.cuda.synchronize(device)
        barrier(world, device)
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(compute)
        h2d.wait_stream(compute)
        d2h.wait_stream(compute)
        run(steps)
        compute.wait_stream(d2h)
        compute.wait_stream(h2d)
        end.record(compute)
        torch.cuda.synchronize(device)
        ms = reduce_over_ranks(world, start.elapsed_time(end), device) / steps
        # the host output of the last step equals the device output it came from
        last = (steps - 1) % nbuf
        host_ok = bool(torch.equal(out_host[last], outs[last].cpu()))
        # pinned copy bandwidth of each rank alone (all ranks at once)
        bw = {}
        for name, src, dst in (("h2d", x_host[0], x_dev[0]), ("d2h", x_dev[0], out_host[0])):
            torch.cuda.synchronize(device)
            barrier(world, device)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(compute)
            for _ in range(3):
                dst.copy_(src, non_blocking=True)
            e.record(compute)
            torch.cuda.synchronize(device)
            bw[name] = 3 * src.numel() * src.element_size() / max(s.elapsed_time(e), 1e-6) / 1e6
    if gather:
        encoder.close()
    B, S = case.cfg_global.batch_size, case.cfg_global.seq_len
    tokens = B * S * (1 if case.split else world)
    return {
        "value": tokens / (ms / 1e3),
        "unit": "tokens/s",
        "ms_per_step": ms,
        "steps": steps,
        "h2d_bytes_per_step": (x_cpu.numel() if local_lengths is None else sum(local_lengths) * x_cpu.shape[-1]) * 4
                              + mask_cpu.numel(),
        "d2h_bytes_per_step": (x_cpu.numel() if local_lengths is None else sum(local_lengths) * x_cpu.shape[-1]) * 4,
        "bytes_per": "rank (each rank uploads its share and downloads its share of the gathered output)",
        "upload": ("the valid rows of x (the rows the layer reads) and the mask" if local_lengths is not None
                   else "x and the mask"),
        "download": ("the valid rows of the output; the host writes the zero rows of the padded positions "
                     "itself (inside the timed region)" if local_lengths is not None else "the whole output"),
        "pinned_copy_gbs_rank0": {k: round(v, 1) for k, v in bw.items()},
        "host_output_equals_device": host_ok,
        "pipeline": "upload i+1 / forward i / download i-1 overlapped on 3 streams",
    }


def kernel_breakdown(pkg, model, case, device, args):
    """Times each kernel alone through its C-ABI entry point on this rank's
    buffers (CUDA events on the launching stream, averaged over repeats)."""
    k = pkg.kernels
    cfg = case.cfg_local
    B, S, D, H, F = cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim
    if B == 0:
        return None
    dh = D // H
    rows = B * S
    layer = model.layers[0]
    att = layer.attention
    mask = case.mask_local.to(device)
    x = case.x_local.to(device)
    plan = k.token_plan(mask, B, S, device)
    nv_t, cu, cnt, orig, inv = k.plan_views(plan, B, S)
    nv = int(nv_t.item())
    lens = cnt.double().cpu()
    a16 = torch.empty(rows, D, dtype=torch.float16, device=device)
    qkv = torch.empty(3, H, rows, k.head_pad(dh), dtype=torch.float16, device=device)
    ctx = torch.empty(rows, D, dtype=torch.float16, device=device)
    h16 = torch.empty(rows, F, dtype=torch.float16, device=device)
    y16 = torch.empty(rows, D, dtype=torch.float16, device=device)
    y16b = torch.empty(rows, D, dtype=torch.float16, device=device)
    out = torch.empty(rows, D, dtype=torch.float32, device=device)
    xf = x.view(rows, D)
    kv_off = cu[:-1].contiguous()
    ops = {
        "token_plan": (lambda: k.token_plan(mask, B, S, device), "hbm", rows * (1 + 8)),
        "ln1_cast_f16": (lambda: k.ln_cast_f16(xf, layer.norm1.weight, layer.norm1.bias, row_map=orig,
                                               row_count=nv_t, out=a16), "hbm", nv * D * (4 + 2)),
        "gemm_qkv": (lambda: k.gemm_qkv_headmajor(a16, att._qkv_weight_mixed, att._qkv_bias_mixed, H,
                                                  row_count=nv_t, out=qkv), "tensor", 2.0 * nv * 3 * D * D),
        "flash_attn": (lambda: k.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], cu, kv_off.view(-1, 1),
                                                cnt.view(-1, 1), S, dh**-0.5, causal=bool(cfg.causal),
                                                out=ctx, head_dim=dh), "tensor",
                       float(((2.0 * lens * (lens + 1)) if cfg.causal else (4.0 * lens * lens)).mul(D).sum())),
        "gemm_out_f16": (lambda: k.gemm_bias_f16(ctx, att._out_weight_mixed, att.out_proj.bias, row_count=nv_t,
                                                 out=y16), "tensor", 2.0 * nv * D * D),
        "add_ln2_f16": (lambda: k.add_ln_cast_f16(xf, y16, layer.norm2.weight, layer.norm2.bias, row_map=orig,
                                                  row_count=nv_t, out=a16), "hbm", nv * D * (4 + 2 + 2)),
        "gemm_ffn_in_gelu": (lambda: k.gemm_bias_gelu_f16(a16, layer._ffn_in_weight_mixed, layer.ffn_in.bias,
                                                          row_count=nv_t, out=h16), "tensor", 2.0 * nv * F * D),
        "gemm_ffn_out_f16": (lambda: k.gemm_bias_f16(h16, layer._ffn_out_weight_mixed, layer.ffn_out.bias,
                                                     row_count=nv_t, out=y16b), "tensor", 2.0 * nv * D * F),
        "add2_ln_final_mask": (lambda: k.add2_ln_final_mask(xf, y16, y16b, model.final_norm.weight,
                                                            model.final_norm.bias, inv_map=inv,
                                                            x_at_original=True, rows=rows, out=out), "hbm",
                               nv * D * (4 + 2 + 2 + 4) + (rows - nv) * D * 4),
    }
    reps = max(3, min(50, args.steps))
    res = {}
    with torch.inference_mode():
        for name, (fn, bound, work) in ops.items():
            fn()
            fn()
            torch.cuda.synchronize(device)
            # The reps launches replay from one CUDA graph, so host launch cost
            # (a ctypes call per launch) does not hide the device time of the
            # short kernels.
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(reps):
                    fn()
            graph.replay()
            torch.cuda.synchronize(device)
            stream = torch.cuda.current_stream(device)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            graph.replay()
            e.record(stream)
            torch.cuda.synchronize(device)
            del graph
            ms = s.elapsed_time(e) / reps
            res[name] = {"ms": ms, "bound": bound, "work": work,
                         "rate": work / (ms / 1e3) / (1e12 if bound == "tensor" else 1e9),
                         "unit": "TFLOP/s" if bound == "tensor" else "GB/s"}
    return res


def roofline(kernels, peaks, peak_kind, workload):
    name, k = max(kernels.items(), key=lambda kv: kv[1]["ms"])
    if k["bound"] == "tensor":
        peak = peaks["bf16_tflops"]
        unit = "TFLOP/s"
    else:
        peak = peaks["hbm_gbs"]
        unit = "GB/s"
    traffic, source = load_traffic(workload, name)
    return {
        "kernel": name,
        "bound": "tensor" if k["bound"] == "tensor" else "hbm",
        "achieved": k["rate"],
        "peak": peak,
        "unit": unit,
        "frac": k["rate"] / peak,
        "peak_source": f"{peak_kind} ({'bf16_tflops burst, kernel timed alone' if unit == 'TFLOP/s' else 'hbm_gbs'})",
        "traffic": traffic,
        "traffic_source": source,
        "algorithmic_per_launch": k["work"],
    }


def load_traffic(workload, kernel):
    """DRAM bytes per launch of `kernel` on this workload (one GPU's share)
    from the committed ncu summaries, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None, None
    try:
        e = json.loads(p.read_text()).get(workload, {}).get(kernel, {})
        return e.get("dram_bytes_per_launch"), e.get("source")
    except (ValueError, AttributeError):
        return None, None


# ---------------------------------------------------------------------------
# CPU baseline / reference arm (the oracle restatement of the reference's
# FP32 BaselineTransformer on the host cores)
# ---------------------------------------------------------------------------
def cpu_step_fn(case, sample):
    """The FP32 oracle forward of one sample of the workload's batch."""
    import oracle

    c = case.cfg_global
    one = oracle.TransformerConfig(1, c.seq_len, c.d_model, c.num_heads, c.ffn_dim, c.num_layers, c.causal)
    xs, ms = case.x[sample : sample + 1].contiguous(), case.mask[sample : sample + 1].contiguous()
    if c.seq_len > 8192:
        return lambda: oracle.encoder_forward_blocked(case.sd, one, xs, ms, query_chunk=1024)
    return lambda: oracle.encoder_forward(case.sd, one, xs, ms)


def cpu_rotation(workload, steps, budget_s, threads):
    """Times the oracle on samples 0, 1, 2, ... of the batch in turn (one
    sample per step, so the steps together cover the batch's length mix),
    stopping after `steps` steps or the time budget.  Returns (tokens/s on
    the B*S basis, steps run, seconds, batch size)."""
    torch.set_num_threads(threads)
    case = Case(workload, 0, 1)
    B, S = case.cfg_global.batch_size, case.cfg_global.seq_len
    cpu_step_fn(case, 0)()  # warm-up (allocator, thread pool)
    total, n = 0.0, 0
    t_stop = time.perf_counter() + budget_s
    while n < steps and (n == 0 or time.perf_counter() < t_stop):
        fn = cpu_step_fn(case, n % B)
        t0 = time.perf_counter()
        fn()
        total += time.perf_counter() - t0
        n += 1
    return n * S / total, n, total, B


def cpu_baseline(workload, budget_s=20.0):
    threads = torch.get_num_threads()
    value, n, total, B = cpu_rotation(workload, 10**6, budget_s, threads)
    return {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"samples 0..{n - 1} of the {B}-sequence batch, one per step (the FP32 oracle "
                      f"restatement of BaselineTransformer, {total:.1f} s)"}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    value, n, total, B = cpu_rotation(args.workload, args.steps, args.cpu_budget * 6, threads)
    return {
        "metric": "layer-forward tokens/s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": n,
        "steps_requested": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total / n * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if args.workload in SPLIT_BATCH else "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded N(0,1) inputs, default-init weights, right-padded masks)",
        "config": workload_config(args.workload),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"samples 0..{n - 1} of the {B}-sequence batch, one per step (the FP32 oracle "
                                   "restatement of BaselineTransformer on all host threads)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def attention_length_scan(args):
    """Attention alone (head dim 64, 16 heads, non-causal, every sample of
    length L, B*L fixed where possible) over L = 256 .. 65536: throughput per
    length and the time per CTA and per 128-key step, which separates the
    per-CTA fixed cost (set-up, pipeline fill, output) from the steady state.
    Synthetic N(0,1) Q/K/V resident in HBM; CUDA events on the launching
    stream; one JSON line per length."""
    import __graft_entry__

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    pkg = __graft_entry__.load_package()
    k = pkg.kernels
    peaks, _ = load_peaks()
    H, dh = 16, 64
    g = torch.Generator(device=device).manual_seed(1234)
    for B, L in ((64, 256), (32, 512), (16, 1024), (8, 2048), (4, 4096), (2, 8192), (1, 16384), (1, 65536)):
        rows = B * L
        cu = torch.arange(B + 1, dtype=torch.int32, device=device) * L
        cnt = torch.full((B, 1), L, dtype=torch.int32, device=device)
        qkv = torch.randn(3, H, rows, dh, device=device, generator=g).half()
        ctx = torch.empty(rows, H * dh, dtype=torch.float16, device=device)
        fn = lambda: k.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], cu, cu[:-1].contiguous().view(-1, 1), cnt, L,  # noqa: E731
                                      dh ** -0.5, out=ctx)
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(device)
        n = max(3, min(args.steps, 20 if L < 65536 else 3))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize(device)
        us = s.elapsed_time(e) * 1e3 / n
        flops = 4.0 * B * H * L * L * dh
        ctas = B * H * ((L + 255) // 256)  # two 128-query tiles per CTA
        steps = (L + 127) // 128            # 128-key steps per CTA
        print(json.dumps({"attention_scan": {"B": B, "L": L, "H": H, "head_dim": dh, "us": us,
                                              "tflops": flops / us / 1e6,
                                              "of_measured_peak": flops / us / 1e6 / peaks["bf16_tflops"],
                                              "ctas": ctas, "steps_per_cta": steps,
                                              "us_per_cta_step_per_sm": us * 148 / (ctas * steps)}}),
              flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="batch")
    ap.add_argument("--micro-batches", type=int, default=0,
                    help="micro-batches per rank in the split-batch gather (0 = 2 up to 2 GPUs, 4 above)")
    ap.add_argument("--gather-transport", choices=("copy_engine", "kernel", "nccl"), default="copy_engine",
                    help="how the output gather moves rows over NVLink: the copy engines (default), "
                         "the push kernel or NCCL point-to-point")
    ap.add_argument("--copy-streams", type=int, default=1,
                    help="copy-engine gather: streams per destination, each pushing an equal share")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline only (no nested dense / context-parallel / sustained measurements)")
    ap.add_argument("--attention-scan", action="store_true",
                    help="time the attention kernel alone over sequence lengths 256..65536 instead")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    world, rank, local = dist_env()
    if world != args.gpus and world > 1:
        ap.error(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.attention_scan:
        attention_length_scan(args)
        return
    if args.impl == "reference":
        line = run_reference(args, world, rank)
    else:
        line = run_ours(args, world, rank, local)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

"""Worker for tests/test_gpu_multi.py, launched with torchrun (one rank per GPU).

Checks, on N GPUs over NCCL:
  * batch sharding: each rank runs its balanced range of the batch; the
    gathered output (NCCL point-to-point, the copy engines over NVLink, or the
    push kernel; valid rows only for right-padded masks, whole samples
    otherwise; 1-3 micro-batches) is bit-identical to the whole batch on one
    GPU;
  * context parallelism: one sequence split into valid-token balanced chunks,
    K/V exchanged every layer (copy engines overlapped with attention over
    the own keys, then a merged launch over the others; and the plain
    NCCL all-gather form); the gathered output passes the reference's
    strict gate against the single-GPU model (non-causal one layer, and
    causal two layers);
  * context parallelism at the long-sequence config (B1 S131072 D1024 H16
    F4096): three 256-row query blocks against the query-row oracle with the
    strict gate, padded rows exactly zero.
Exits non-zero on any failure.
"""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402
import oracle  # noqa: E402


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    pkg = __graft_entry__.load_package()
    from techjam_b200 import sharding

    pkg._lib.set_sync_check(True)
    failures = []

    def model_for(cfg, sd):
        m = pkg.UserOptimizedTransformer(pkg.TransformerConfig(*cfg.__dict__.values()))
        m.load_state_dict(sd, strict=True)
        return m.to(dev).eval()

    with torch.inference_mode():
        # ---- batch sharding ------------------------------------------------
        cfg = oracle.TransformerConfig(6, 512, 1024, 16, 4096, 1, False)
        sd = oracle.make_state_dict(cfg, seed=5)
        x, mask = oracle.generate_random_case(cfg, seed=5, padding_ratio=0.5)
        model = model_for(cfg, sd)
        a, b = sharding.batch_ranges(cfg.batch_size, world)[rank]
        bs = sharding.BatchShardedEncoder(model)
        out = bs.forward(x[a:b].to(dev), mask[a:b].to(dev), gather=True)
        full = model(x.to(dev), mask.to(dev))
        if not torch.equal(out, full):
            failures.append(f"batch sharding differs from one GPU: {float((out - full).abs().max())}")
        # work-balanced sample sets, gathered back into batch order
        assign = bs.assignment(mask)
        mine = torch.tensor(assign[rank], dtype=torch.int64)
        out = bs.forward(x[mine].to(dev), mask[mine].to(dev), gather=True, assignment=assign)
        if not torch.equal(out, full):
            failures.append(f"balanced batch sharding differs from one GPU: {float((out - full).abs().max())}")
        # right-padded masks: only valid rows cross NVLink, padded rows zero-filled
        # by the receiver; one to three micro-batches per rank, and twice in a
        # row so both exchange buffers (with the other call's stale rows) are used
        lengths = mask.sum(1).tolist()
        for mb in (1, 3):
            bs.micro_batches = mb
            for rep in range(2):
                out = bs.forward(x[mine].to(dev), mask[mine].to(dev), gather=True, assignment=assign,
                                 valid_lengths=lengths)
                if not torch.equal(out, full):
                    failures.append(f"valid-row gather (micro-batches {mb}, call {rep}) differs from one GPU")
        # the other transports of the same gather (push kernel, NCCL point-to-point,
        # copy engines with three streams per destination)
        for transport, k in (("kernel", 1), ("nccl", 1), ("copy_engine", 3)):
            pk = sharding.BatchShardedEncoder(model, micro_batches=2, transport=transport, copy_streams=k)
            for rep in range(2):
                out = pk.forward(x[mine].to(dev), mask[mine].to(dev), gather=True, assignment=assign,
                                 valid_lengths=lengths)
                if not torch.equal(out, full):
                    failures.append(f"{transport} gather ({k} streams, call {rep}) differs from one GPU")
            pk.close()
        # a non-prefix mask: whole samples are copied
        mask2 = mask.clone()
        mask2[:, 1::3] = False
        full2 = model(x.to(dev), mask2.to(dev))
        out = bs.forward(x[mine].to(dev), mask2[mine].to(dev), gather=True, assignment=assign)
        if not torch.equal(out, full2):
            failures.append("whole-sample gather of a non-prefix mask differs from one GPU")
        bs.close()

        # ---- context parallelism -------------------------------------------
        for cfg_t, pad in (((1, 4096, 1024, 16, 4096, 1, False), 0.1), ((1, 3000, 512, 8, 1024, 2, True), 0.2)):
            cfg = oracle.TransformerConfig(*cfg_t)
            sd = oracle.make_state_dict(cfg, seed=7)
            x, mask = oracle.generate_random_case(cfg, seed=7, padding_ratio=pad)
            model = model_for(cfg, sd)
            ranges = sharding.sequence_ranges(mask[0], world)
            slab = max(e - s for s, e in ranges)
            s0, e0 = ranges[rank]
            ref = model(x.to(dev), mask.to(dev))
            # overlapped K/V exchange (split attention + merge) and the plain
            # all-gather form; the overlapped one twice, so both K/V buffers are used
            for overlap, reps in ((True, 2), (False, 1)):
                cp = sharding.ContextParallelEncoder(model, overlap=overlap)
                for _ in range(reps):
                    out_local = cp.forward(x[:, s0:e0].contiguous().to(dev), mask[:, s0:e0].contiguous().to(dev),
                                           slab)
                    padded = torch.zeros(1, slab, cfg.d_model, device=dev)
                    padded[:, : e0 - s0] = out_local
                    parts = [torch.empty_like(padded) for _ in range(world)]
                    dist.all_gather(parts, padded)
                    out = torch.cat([parts[r][:, : e - s] for r, (s, e) in enumerate(ranges)], dim=1)
                    r = oracle.compare_outputs(ref.cpu(), out.cpu())
                    if not r.passed:
                        failures.append(f"context parallel {cfg_t} overlap={overlap}: {r}")
                    if torch.count_nonzero(out.cpu()[~mask]) != 0:
                        failures.append(f"context parallel {cfg_t} overlap={overlap}: padded rows not zero")
                cp.close()

        # ---- context parallelism at the long-sequence config ----------------
        # B1 S131072 D1024 H16 F4096, valid length ~ U[0.9S, S]: every rank
        # checks its chunk (finite, padded rows exactly zero); the rows of three
        # 256-row query blocks are summed to rank 0 (each row is owned by one
        # rank, the others add zeros), which gates them against the query-row
        # oracle after the process group is gone.
        cfg = oracle.TransformerConfig(1, 131072, 1024, 16, 4096, 1, False)
        sd = oracle.make_state_dict(cfg, seed=1234)
        x, mask = oracle.generate_random_case(cfg, seed=1234, padding_ratio=0.1)
        model = model_for(cfg, sd)
        ranges = sharding.sequence_ranges(mask[0], world)
        slab = max(e - s for s, e in ranges)
        s0, e0 = ranges[rank]
        cp = sharding.ContextParallelEncoder(model)
        out_local = cp.forward(x[:, s0:e0].contiguous().to(dev), mask[:, s0:e0].contiguous().to(dev), slab)[0]
        if not bool(torch.isfinite(out_local).all()):
            failures.append("context parallel S=131072: non-finite output")
        if torch.count_nonzero(out_local[~mask[0, s0:e0].to(dev)]) != 0:
            failures.append("context parallel S=131072: padded rows not zero")
        L = int(mask.sum())
        check_rows = oracle.long_sequence_check_rows(L, cfg.seq_len)
        picked = torch.zeros(check_rows.numel(), cfg.d_model, device=dev)
        own = (check_rows >= s0) & (check_rows < e0)
        picked[own.to(dev)] = out_local[(check_rows[own] - s0).to(dev)]
        dist.all_reduce(picked)
        picked = picked.cpu()
        cp.close()
        del model, cp, out_local
        pkg._lib.device_status(torch.cuda.current_stream().cuda_stream)

    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    if rank == 0:
        ref = oracle.encoder_forward_query_rows(sd, cfg, x, mask, check_rows)
        r = oracle.compare_outputs(ref, picked)
        print(f"context parallel S=131072 over {world} GPUs: {check_rows.numel()} rows, "
              f"max_abs={r.max_abs_error:.3g}, failed={r.failed_elements}", flush=True)
        if not r.passed:
            failures.append(f"context parallel S=131072 against the query-row oracle: {r}")
    if failures:
        print(f"rank {rank} FAILED:\n" + "\n".join(failures), flush=True)
        return 1
    print(f"rank {rank} OK", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

"""Host-side multi-GPU logic on CPU: shard ranges, the output gather's copy
plan, the split-attention merge formula, and the context-parallel
decomposition run by two gloo ranks.

The gloo test mirrors what ContextParallelEncoder does on GPUs -- valid-token
balanced chunks, compact local K/V padded to a common slab,
all_gather_into_tensor into [G][2][H][slab][dh], key-segment tables from
`segment_metadata`, attention walking the segments in order -- with the
oracle's FP32 math in place of the kernels, and checks each rank's queries
against the oracle's full-sequence attention.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle


def test_batch_ranges(pkg):
    from techjam_b200 import sharding

    for batch in (0, 1, 7, 8, 32, 33):
        for world in (1, 2, 3, 8):
            r = sharding.batch_ranges(batch, world)
            assert len(r) == world and r[0][0] == 0 and r[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            sizes = [e - s for s, e in r]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_balanced_assignment(pkg, world):
    """Every sample exactly once, the per-rank counts of batch_ranges, and the
    most loaded rank no worse than with contiguous ranges."""
    from techjam_b200 import sharding

    g = torch.Generator().manual_seed(world)
    for B in (0, 1, 7, 32, 33):
        lengths = torch.randint(1, 4097, (B,), generator=g).tolist()
        a = sharding.balanced_assignment(lengths, world, 1024, 4096)
        assert sorted(i for r in a for i in r) == list(range(B))
        assert [len(r) for r in a] == [e - s for s, e in sharding.batch_ranges(B, world)]
        assert a == sharding.balanced_assignment(lengths, world, 1024, 4096)  # deterministic
        w = 2.0 * 4096 / (8 * 1024 * 1024 + 4 * 1024 * 4096)
        cost = [L + w * L * L for L in lengths]
        worst = max((sum(cost[i] for i in r) for r in a), default=0.0)
        worst_ranges = max((sum(cost[s:e]) for s, e in sharding.batch_ranges(B, world)), default=0.0)
        assert worst <= worst_ranges + 1e-6


@pytest.mark.parametrize("world,micro", [(2, 1), (3, 2), (4, 3), (8, 2)])
@pytest.mark.parametrize("prefix", [True, False])
def test_gather_plan_rebuilds_the_batch_output(pkg, world, micro, prefix):
    """The output gather's copy plan, replayed on CPU byte arrays: every
    rank's pushes of its micro-batches (gather_segments) plus the receiver's
    zero fill (zero_fill_segments, right-padded masks) rebuild the full
    [B, S, D] output exactly, over a buffer holding a previous call's rows."""
    from techjam_b200 import sharding

    g = torch.Generator().manual_seed(world * 10 + micro)
    B, S, D = 13, 9, 3
    row = D * 4
    lengths = torch.randint(0, S + 1, (B,), generator=g).tolist()
    full = torch.randn(B, S, D, generator=g)
    for b, n in enumerate(lengths):
        full[b, n:] = 0  # padded rows of the model's output are zero
    assign = sharding.balanced_assignment(lengths, world, 64, 256)
    dest = torch.randn(B, S, D, generator=g)  # stale rows of an earlier call
    d_bytes = dest.view(-1).view(torch.uint8)
    if prefix:
        for off, n in sharding.zero_fill_segments(lengths, S, row):
            d_bytes[off : off + n] = 0
    for r in range(world):
        mine = assign[r]
        local = full[torch.tensor(mine, dtype=torch.int64)] if mine else torch.zeros(0, S, D)
        for j0, j1 in sharding.micro_batch_ranges(len(mine), micro):
            src = local[j0:j1].contiguous().view(-1).view(torch.uint8)
            for do, so, n in sharding.gather_segments(assign, r, (j0, j1), S, row, lengths if prefix else None):
                d_bytes[do : do + n] = src[so : so + n]
    assert torch.equal(dest, full)
    with pytest.raises(ValueError):
        sharding.zero_fill_segments([S + 1], S, row)
    assert sharding.micro_batch_ranges(0, 2) == []
    assert sharding.micro_batch_ranges(5, 2) == [(0, 3), (3, 5)]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_sequence_ranges_balance_valid_tokens(pkg, world):
    from techjam_b200 import sharding

    g = torch.Generator().manual_seed(world)
    for S in (1, 100, 4096):
        for kind in ("prefix", "random", "none", "empty"):
            if kind == "prefix":
                valid = torch.arange(S) < int(torch.randint(1, S + 1, (1,), generator=g))
            elif kind == "random":
                valid = torch.rand(S, generator=g) < 0.6
            elif kind == "none":
                valid = torch.ones(S, dtype=torch.bool)
            else:
                valid = torch.zeros(S, dtype=torch.bool)
            r = sharding.sequence_ranges(valid, world)
            assert len(r) == world and r[0][0] == 0 and r[-1][1] == S
            assert all(a[1] == b[0] and a[0] <= a[1] for a, b in zip(r, r[1:]))
            counts = [int(valid[s:e].sum()) for s, e in r]
            assert max(counts) - min(counts) <= 1, (kind, S, counts)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _project(sd, p, x, name):
    return torch.nn.functional.linear(x, sd[p + name + ".weight"], sd[p + name + ".bias"])


def _cp_rank(rank, world, port, causal, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__

        __graft_entry__.load_package()
        from techjam_b200 import sharding

        cfg = oracle.TransformerConfig(1, 300, 64, 2, 128, 1, causal)
        sd = oracle.make_state_dict(cfg, seed=11)
        x, mask = oracle.generate_random_case(cfg, seed=11, padding_ratio=0.3)
        mask[0, 40:47] = False  # a hole inside the valid prefix
        H, D = cfg.num_heads, cfg.d_model
        dh = D // H
        ranges = sharding.sequence_ranges(mask[0], world)
        a, b = ranges[rank]
        slab = max(e - s for s, e in ranges)
        p = "layers.0."
        h = torch.nn.functional.layer_norm(x, (D,), sd[p + "norm1.weight"], sd[p + "norm1.bias"], 1e-5)[0]
        # Compact local valid tokens, as the token plan orders them.
        local_valid = torch.nonzero(mask[0, a:b]).flatten() + a
        n_local = local_valid.numel()
        hl = h[local_valid]
        q = _project(sd, p, hl, "attention.q_proj").view(n_local, H, dh).transpose(0, 1)
        k = _project(sd, p, hl, "attention.k_proj").view(n_local, H, dh).transpose(0, 1)
        v = _project(sd, p, hl, "attention.v_proj").view(n_local, H, dh).transpose(0, 1)
        slab_kv = torch.full((2, H, slab, dh), float("nan"))  # rows past the count stay garbage
        slab_kv[0, :, :n_local] = k
        slab_kv[1, :, :n_local] = v
        kv_all = torch.empty(world, 2, H, slab, dh)
        dist.all_gather_into_tensor(kv_all.view(-1), slab_kv.reshape(-1))
        counts = torch.empty(world, dtype=torch.int32)
        dist.all_gather_into_tensor(counts, torch.tensor([n_local], dtype=torch.int32))
        kv_off, kv_len, q_pos0 = sharding.segment_metadata(counts, rank, causal)
        # Walk the segments in order, as the attention kernel does.
        ks, vs = [], []
        for gidx in range(world):
            o, l = int(kv_off[0, gidx]), int(kv_len[0, gidx])
            ks.append(kv_all[gidx, 0, :, o : o + l])
            vs.append(kv_all[gidx, 1, :, o : o + l])
        kk, vv = torch.cat(ks, 1), torch.cat(vs, 1)
        s = torch.matmul(q, kk.transpose(-1, -2)) * dh**-0.5
        if causal:
            qp = int(q_pos0[0]) + torch.arange(n_local)[:, None]
            kp = torch.arange(kk.shape[1])[None, :]
            s = s.masked_fill(kp > qp, float("-inf"))
        ctx = torch.matmul(torch.softmax(s, -1), vv).transpose(0, 1).reshape(n_local, D)

        # Oracle: full-sequence attention context for the same query rows.
        full_valid = torch.nonzero(mask[0]).flatten()
        qf = _project(sd, p, h, "attention.q_proj").view(300, H, dh).transpose(0, 1)
        kf = _project(sd, p, h, "attention.k_proj").view(300, H, dh).transpose(0, 1)
        vf = _project(sd, p, h, "attention.v_proj").view(300, H, dh).transpose(0, 1)
        sf = torch.matmul(qf, kf.transpose(-1, -2)) * dh**-0.5
        if causal:
            sf = sf.masked_fill(torch.ones(300, 300, dtype=torch.bool).triu(1), float("-inf"))
        sf = sf.masked_fill(~mask[0][None, None, :], float("-inf"))
        ref = torch.matmul(torch.softmax(sf, -1), vf).transpose(0, 1).reshape(300, D)[local_valid]
        assert set(full_valid.tolist()) >= set(local_valid.tolist())
        err = float((ctx - ref).abs().max()) if n_local else 0.0
        result_q.put((rank, n_local, err, None))
    except Exception as e:  # report to the parent instead of hanging it
        result_q.put((rank, -1, float("inf"), repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("causal", [False, True])
def test_context_parallel_decomposition_two_gloo_ranks(pkg, causal):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cp_rank, args=(r, world, port, causal, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, n_local, err, exc in sorted(results):
        assert exc is None, f"rank {rank}: {exc}"
        assert n_local > 0
        assert err < 1e-5, f"rank {rank}: max abs error {err}"


def test_split_attention_merge_formula():
    """The merge the split attention performs (part_mode 2), restated on CPU:
    with the first key set's normalised context o1 and base-2 log-sum-exp
    lse1, and the second set's unnormalised context O2 and sum l2 relative to
    2^m2, (O2*a + o1*c) / (l2*a + c), a = 2^(m2-M), c = 2^(lse1-M),
    M = max(m2, lse1), equals one softmax over both sets; an empty set
    (lse = -inf or l2 = 0) drops out."""
    g = torch.Generator().manual_seed(0)
    log2e = 1.4426950408889634
    for n1, n2 in ((50, 70), (1, 200), (0, 30), (40, 0)):
        s = torch.randn(n1 + n2, generator=g, dtype=torch.float64) * 4 * log2e  # base-2 scores
        v = torch.randn(n1 + n2, 8, generator=g, dtype=torch.float64)
        full = (torch.softmax(s / log2e, 0)[:, None] * v).sum(0)
        s1, s2, v1, v2 = s[:n1], s[n1:], v[:n1], v[n1:]
        if n1:
            m1 = s1.max()
            l1 = torch.exp2(s1 - m1).sum()
            o1 = (torch.exp2(s1 - m1)[:, None] * v1).sum(0) / l1
            lse1 = m1 + torch.log2(l1)
        else:
            o1, lse1 = torch.zeros(8, dtype=torch.float64), torch.tensor(float("-inf"), dtype=torch.float64)
        if n2:
            m2 = s2.max() - 3.0  # a stale running max, as the kernel keeps it
            p2 = torch.exp2(s2 - m2)
            O2, l2 = (p2[:, None] * v2).sum(0), p2.sum()
            e2 = m2
        else:
            O2, l2, e2 = torch.zeros(8, dtype=torch.float64), torch.tensor(0.0, dtype=torch.float64), float("-inf")
        M = max(float(e2), float(lse1))
        a = 0.0 if e2 == float("-inf") else 2.0 ** (float(e2) - M)
        c = 0.0 if float(lse1) == float("-inf") else 2.0 ** (float(lse1) - M)
        merged = (O2 * a + o1 * c) / (l2 * a + c)
        torch.testing.assert_close(merged, full, rtol=1e-12, atol=1e-12)


def _p2p_gather_rank(rank, world, port, micro, prefix, result_q):
    """One gloo rank of the point-to-point gather: the plan of p2p_step_plan
    run with real sends and receives (dist.batch_isend_irecv, as the NCCL
    transport issues them) over CPU tensors standing in for each micro-batch's
    output."""
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import __graft_entry__

        __graft_entry__.load_package()
        from techjam_b200 import sharding

        g = torch.Generator().manual_seed(99 + world + micro)
        B, S, D = 11, 7, 5
        lengths = torch.randint(0, S + 1, (B,), generator=g).tolist()
        full = torch.randn(B, S, D, generator=g)
        for b, n in enumerate(lengths):
            full[b, n:] = 0
        assign = sharding.balanced_assignment(lengths, world, 64, 256)
        valid = lengths if prefix else None
        out_all = torch.full((B, S, D), float("nan"))
        if prefix:  # the receiver's zero fill of padded rows
            for b, n in enumerate(lengths):
                out_all[b, n:] = 0
        mine = assign[rank]
        steps = sharding.p2p_steps(assign, micro)
        for k in range(steps):
            rng, sends, recvs, keeps = sharding.p2p_step_plan(assign, rank, k, micro, S, valid)
            ops = []
            if rng is not None:
                j0, j1 = rng
                out = full[torch.tensor(mine[j0:j1], dtype=torch.int64)].contiguous()  # "the forward"
                for jl, b, n in keeps:
                    out_all[b, :n].copy_(out[jl, :n])
                for d, jl, n in sends:
                    ops.append(dist.P2POp(dist.isend, out[jl, :n].contiguous(), d))
            recv_bufs = []
            for src, b, n in recvs:
                t = torch.empty(n, D)
                recv_bufs.append((b, n, t))
                ops.append(dist.P2POp(dist.irecv, t, src))
            if ops:
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
            for b, n, t in recv_bufs:
                out_all[b, :n] = t
        ok = torch.equal(out_all, full)
        result_q.put((rank, ok, None))
    except Exception as e:  # report to the parent instead of hanging it
        result_q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,micro", [(2, 2), (3, 4)])
@pytest.mark.parametrize("prefix", [True, False])
def test_p2p_gather_plan_gloo_ranks(pkg, world, micro, prefix):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_p2p_gather_rank, args=(r, world, port, micro, prefix, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, exc in sorted(results):
        assert exc is None, f"rank {rank}: {exc}"
        assert ok, f"rank {rank}: gathered output differs"


def test_p2p_plan_matches_pairwise(pkg):
    """Sender and receiver enumerate the same transfers in the same order, for
    every ordered rank pair and step (NCCL matches point-to-point operations
    between two ranks in posting order)."""
    from techjam_b200 import sharding

    g = torch.Generator().manual_seed(5)
    for world in (2, 3, 8):
        for B in (1, 6, 13, 32):
            lengths = torch.randint(0, 50, (B,), generator=g).tolist()
            assign = sharding.balanced_assignment(lengths, world, 64, 256)
            for micro in (1, 2, 4):
                for k in range(sharding.p2p_steps(assign, micro)):
                    plans = [sharding.p2p_step_plan(assign, r, k, micro, 50, lengths) for r in range(world)]
                    for s in range(world):
                        for d in range(world):
                            if s == d:
                                continue
                            sent = [n for dd, _, n in plans[s][1] if dd == d]
                            got = [n for ss, _, n in plans[d][2] if ss == s]
                            assert sent == got, (world, B, micro, k, s, d)


def test_split_segments_covers_the_same_rows(pkg):
    """The copy-engine gather's per-stream shares: every byte once, in order,
    cut only at whole rows, about equal shares."""
    from techjam_b200 import sharding

    g = torch.Generator().manual_seed(3)
    for row in (4, 12, 4096):
        for _ in range(200):
            segs, off = [], 0
            for _ in range(int(torch.randint(0, 6, (1,), generator=g))):
                n = row * int(torch.randint(1, 60, (1,), generator=g))
                segs.append((3 * off + 7, off, n))
                off += n
            for parts in (1, 2, 3, 4, 7):
                shares = sharding.split_segments(segs, parts, row)
                assert len(shares) == parts
                flat = [c for s in shares for c in s]
                assert all(n > 0 and n % row == 0 for _, _, n in flat)
                want = [(do + i, so + i) for do, so, n in segs for i in range(0, n, row)]
                got = [(do + i, so + i) for do, so, n in flat for i in range(0, n, row)]
                assert got == want
                total = sum(n for _, _, n in segs)
                if total:
                    cap = -(-total // parts)
                    assert max(sum(n for _, _, n in s) for s in shares) <= cap + row

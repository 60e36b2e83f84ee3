"""Multi-GPU execution of the encoder: batch sharding and context parallelism.

One process per GPU (torchrun), torch.distributed for the plumbing.

* Batch sharding: samples are independent in the reference model (every op
  is per sample), so each rank runs a contiguous, balanced range of the batch
  (the balanced-range split of the reference's multi-stream variant,
  candidates/v19/parallel_batch_common.py:31-51) or, balanced by estimated
  work rather than count, the sample set of `balanced_assignment`, with no
  data-path collective in the forward itself; `BatchShardedEncoder.forward(
  ..., gather=True)` ends with the output gather: the valid rows of every
  finished micro-batch go into every rank's [B, S, D] output over NVLink
  (copy engines into peer mappings), overlapped with the next micro-batch.
* Context parallelism for one long sequence: rank g holds a contiguous chunk
  of the sequence.  Attention is the only op that mixes tokens, so each rank
  computes LN1 and the QKV projection for its own tokens, all-gathers the
  K/V slabs with NCCL (all_gather_into_tensor into [G][2][H][slab][P], which
  the attention kernel reads as G key segments), runs attention for its own
  queries over every segment, and the rest of the layer is token-local.

Chunk boundaries are chosen so every rank gets the same number of VALID
tokens (`sequence_ranges`): with a right-padded mask the padded tail then
lands on the last rank and costs nothing, instead of idling it.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import kernels


def batch_ranges(batch: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous ranges covering [0, batch), sizes differing by at most one."""
    if batch < 0 or world <= 0:
        raise ValueError("batch must be >= 0 and world > 0")
    base, extra = divmod(batch, world)
    out, start = [], 0
    for r in range(world):
        size = base + (1 if r < extra else 0)
        out.append((start, start + size))
        start += size
    return out


def sequence_ranges(valid: torch.Tensor, world: int) -> List[Tuple[int, int]]:
    """Contiguous ranges covering [0, S) of one sequence with (as nearly as
    possible) equal numbers of valid tokens per range.  Padded positions after
    the last valid token go to the last range."""
    if valid.dim() != 1:
        raise ValueError("valid must be a [S] mask")
    S = valid.numel()
    if world <= 0:
        raise ValueError("world must be positive")
    counts = torch.cumsum(valid.to(torch.int64).cpu(), 0)
    total = int(counts[-1]) if S else 0
    bounds = [0]
    for r in range(1, world):
        target = (total * r + world - 1) // world  # valid tokens before range r
        # first position whose prefix count reaches target
        pos = int(torch.searchsorted(counts, torch.tensor(target), right=False).item()) + 1 if target > 0 else 0
        pos = max(bounds[-1], min(S, pos))
        bounds.append(pos)
    bounds.append(S)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def balanced_assignment(lengths: Sequence[int], world: int, d_model: int, ffn_dim: int) -> List[List[int]]:
    """Samples per rank, balanced by estimated work instead of sample count.

    Each rank gets as many samples as `batch_ranges` gives it (equal shapes
    everywhere), chosen greedily, largest first, for the rank with the least
    work so far (ties to the lower rank, so every rank computes the same
    assignment).  A sample of L valid tokens costs L (projections, per
    token) + w * L^2 (attention), w = attention FLOPs per token pair over
    projection FLOPs per token, doubled because attention runs at about half
    the projections' tensor-core rate.  Each rank's list is in decreasing
    order of cost (ties by index), so when a rank runs its samples in
    micro-batches the last one -- whose output gather nothing overlaps -- holds
    its cheapest samples."""
    B = len(lengths)
    caps = [e - s for s, e in batch_ranges(B, world)]
    w = 2.0 * (4.0 * d_model) / (8.0 * d_model * d_model + 4.0 * d_model * ffn_dim)
    cost = [float(L) + w * float(L) * float(L) for L in lengths]
    out: List[List[int]] = [[] for _ in range(world)]
    load = [0.0] * world
    for i in sorted(range(B), key=lambda i: (-cost[i], i)):
        r = min((r for r in range(world) if len(out[r]) < caps[r]), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += cost[i]
    return [sorted(o, key=lambda i: (-cost[i], i)) for o in out]


def micro_batch_ranges(n: int, parts: int) -> List[Tuple[int, int]]:
    """Splits n local samples into at most `parts` contiguous micro-batches
    (sizes differing by at most one, the larger ones first)."""
    if n <= 0:
        return []
    return [r for r in batch_ranges(n, max(1, min(parts, n))) if r[1] > r[0]]


def gather_segments(assignment: Sequence[Sequence[int]], rank: int, group: Tuple[int, int], seq_len: int,
                    row_bytes: int, valid_lengths: Optional[Sequence[int]]) -> List[Tuple[int, int, int]]:
    """Copies one destination needs for micro-batch `group` = local samples
    [j0, j1) of `rank`: (byte offset in the [B, S, D] output, byte offset in
    the micro-batch's [j1-j0, S, D] output, bytes).  With right-padded masks
    (valid_lengths given) only a sample's valid rows are copied; otherwise the
    whole sample, its zero rows included."""
    j0, j1 = group
    mine = assignment[rank]
    sample_bytes = seq_len * row_bytes
    out = []
    for j in range(j0, j1):
        b = mine[j]
        n = sample_bytes if valid_lengths is None else int(valid_lengths[b]) * row_bytes
        if n > 0:
            out.append((b * sample_bytes, (j - j0) * sample_bytes, n))
    return out


def p2p_step_plan(assignment: Sequence[Sequence[int]], rank: int, step: int, micro_batches: int,
                  seq_len: int, valid_lengths: Optional[Sequence[int]]):
    """Point-to-point transfers of micro-batch step `step` of the NCCL gather,
    the same on every rank: step k is the k-th range of
    micro_batch_ranges(len(assignment[r]), micro_batches) on each rank r (empty
    when r has fewer).  Returns (local_range, sends, recvs, keeps):
      local_range  this rank's [j0, j1) of the step (None when empty);
      sends        (peer, local row j - j0 of the micro-batch, rows) per peer,
                   peers in rank order and, per peer, samples in local order;
      recvs        (peer, sample b of the batch, rows), the matching order;
      keeps        (local row, sample b, rows): this rank's own samples.
    rows = the sample's valid rows (right-padded masks) or seq_len; samples
    with no rows are skipped on both sides."""
    world = len(assignment)

    def step_range(r):
        rs = micro_batch_ranges(len(assignment[r]), micro_batches)
        return rs[step] if step < len(rs) else None

    def rows(b):
        return seq_len if valid_lengths is None else int(valid_lengths[b])

    mine = step_range(rank)
    sends, recvs, keeps = [], [], []
    if mine is not None:
        j0, j1 = mine
        for j in range(j0, j1):
            b = assignment[rank][j]
            if rows(b) > 0:
                keeps.append((j - j0, b, rows(b)))
        for d in range(world):
            if d == rank:
                continue
            for j in range(j0, j1):
                b = assignment[rank][j]
                if rows(b) > 0:
                    sends.append((d, j - j0, rows(b)))
    for src in range(world):
        if src == rank:
            continue
        theirs = step_range(src)
        if theirs is None:
            continue
        for j in range(theirs[0], theirs[1]):
            b = assignment[src][j]
            if rows(b) > 0:
                recvs.append((src, b, rows(b)))
    return mine, sends, recvs, keeps


def split_segments(segs: Sequence[Tuple[int, int, int]], parts: int, row_bytes: int) -> List[List[Tuple[int, int, int]]]:
    """Deals copies (dst offset, src offset, bytes) to `parts` queues of
    about equal bytes, cutting a copy at whole rows where it straddles two
    queues; concatenated in queue order they cover the same bytes."""
    parts = max(1, int(parts))
    total = sum(n for _, _, n in segs)
    share = -(-total // parts)
    share = -(-share // row_bytes) * row_bytes if row_bytes > 0 else share
    out: List[List[Tuple[int, int, int]]] = [[] for _ in range(parts)]
    q, room = 0, share
    for do, so, n in segs:
        while n > 0:
            if room == 0 and q + 1 < parts:
                q, room = q + 1, share
            take = n if q + 1 == parts else min(n, room)
            out[q].append((do, so, take))
            do, so, n, room = do + take, so + take, n - take, room - take
    return out


def p2p_steps(assignment: Sequence[Sequence[int]], micro_batches: int) -> int:
    """Micro-batch steps of the NCCL gather: the most any rank has."""
    return max((len(micro_batch_ranges(len(a), micro_batches)) for a in assignment), default=0)


def zero_fill_segments(valid_lengths: Sequence[int], seq_len: int, row_bytes: int) -> List[Tuple[int, int]]:
    """(byte offset, bytes) of every sample's padded tail in the [B, S, D]
    output of a right-padded batch: the rows no rank sends."""
    out = []
    for b, L in enumerate(valid_lengths):
        L = int(L)
        if not 0 <= L <= seq_len:
            raise ValueError(f"valid length {L} of sample {b} outside [0, {seq_len}]")
        if L < seq_len:
            out.append(((b * seq_len + L) * row_bytes, (seq_len - L) * row_bytes))
    return out


class _Exchange:
    """A few [B, S, D] fp32 output buffers per rank (used in turn), each mapped
    into every other rank of the group (CUDA IPC), plus the transfer streams."""

    def __init__(self, key, bufs, ptrs, mapped, streams, flag):
        self.key = key
        self.bufs = bufs          # this rank's output buffers
        self.ptrs = ptrs          # ptrs[d][i]: address of rank d's buffer i in this process
        self.mapped = mapped      # peer allocation bases opened here (closed on release)
        self.streams = streams    # copy engines: streams[d] copies into rank d; kernel: [the push stream]
        self.flag = flag          # one-element tensor all-reduced as the completion barrier


class BatchShardedEncoder:
    """Runs `model` on this rank's share of the batch: a contiguous range
    (`local_range`), or the work-balanced sample set of `balanced_assignment`.

    forward(..., gather=True) also gathers the [B, S, D] output of the whole
    batch on every rank.  The samples run in micro-batches; as soon as one
    micro-batch is finished, the valid rows of its samples go into every
    rank's output buffer over NVLink (no padded rows on the link) while the
    next micro-batch computes.  Transports:
      "copy_engine" (default): copy-engine pushes into the peers' buffers
          (CUDA IPC peer mappings, one stream per destination);
      "kernel": one push kernel on a high-priority side stream
          (tj_push_segments);
      "nccl": NCCL point-to-point sends of each finished sample's valid rows
          to every peer, received straight into the peer's output rows
          (dist.batch_isend_irecv per micro-batch, on NCCL's stream, so the
          next micro-batch computes meanwhile); each rank waits for its own
          receives.  Measured on two B200s at B32 S4096: 26 M tokens/s with
          2 micro-batches and 48 M with 4, against 56 M for the copy engines.
    With the two push transports an all-reduce of one element on the current
    stream, after this rank's last push, is the barrier after which every
    rank's buffer is complete.  Each rank zero-fills the padded rows of its
    own buffer.

    The gathered output is one of `buffers` persistent buffers used in turn:
    the output of call i stays intact until this rank's current stream
    reaches the end of call i + buffers - 1 (peers start writing a buffer
    again only after every rank has passed the previous call's barrier);
    clone it to keep it longer.  Call `close()` (on every rank) before the
    process group goes away."""

    def __init__(self, model, group=None, micro_batches: Optional[int] = None, buffers: int = 2,
                 push_blocks: int = 64, transport: str = "copy_engine", copy_streams: int = 1) -> None:
        import torch.distributed as dist

        self.model = model
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.world > 8:
            raise ValueError("the output gather pushes to at most 8 GPUs (one node)")
        # measured on B200s (B32 S4096): 2 micro-batches best at 2 GPUs, 4 from 4 GPUs up
        self.micro_batches = max(1, int(micro_batches)) if micro_batches else (2 if self.world <= 2 else 4)
        self.push_blocks = int(push_blocks)
        if transport not in ("nccl", "kernel", "copy_engine"):
            raise ValueError("transport must be 'nccl', 'kernel' or 'copy_engine'")
        self.transport = transport
        # copy engines: streams per destination, each pushing an equal share of
        # every micro-batch's rows (so several engines can serve one peer)
        self.copy_streams = max(1, int(copy_streams))
        if buffers < 2:
            raise ValueError("the gather needs at least two output buffers")
        self.buffers = int(buffers)
        self._exchange: Optional[_Exchange] = None
        self._turn = 0

    def local_range(self, batch: int) -> Tuple[int, int]:
        return batch_ranges(batch, self.world)[self.rank]

    def assignment(self, valid_token_mask: torch.Tensor) -> List[List[int]]:
        """The work-balanced split of a [B, S] mask (the same on every rank)."""
        cfg = self.model.config
        lengths = valid_token_mask.to(torch.int64).sum(1).tolist()
        return balanced_assignment(lengths, self.world, cfg.d_model, cfg.ffn_dim)

    def forward(self, x_local: torch.Tensor, mask_local: Optional[torch.Tensor], gather: bool = False,
                assignment: Optional[Sequence[Sequence[int]]] = None,
                valid_lengths: Optional[Sequence[int]] = None):
        """x_local [B_r, S, D] holds this rank's samples in the order of
        `assignment[rank]` (contiguous batch ranges when assignment is None).
        valid_lengths: per-sample valid counts of the GLOBAL batch when the
        mask is right-padded (valid tokens first); then only valid rows cross
        NVLink.  Without it whole samples are copied (any mask)."""
        if not gather or self.world == 1:
            return self.model(x_local, mask_local)  # a rank may hold no samples (batch < world)
        return self._gather_forward(x_local, mask_local, assignment, valid_lengths)

    # ---- the gather ---------------------------------------------------------
    def _global_assignment(self, n_local: int, device) -> List[List[int]]:
        import torch.distributed as dist

        sizes = [torch.zeros(1, dtype=torch.int64, device=device) for _ in range(self.world)]
        dist.all_gather(sizes, torch.tensor([n_local], dtype=torch.int64, device=device), group=self.group)
        out, start = [], 0
        for s in sizes:
            n = int(s.item())
            out.append(list(range(start, start + n)))
            start += n
        return out

    def _exchange_for(self, B: int, S: int, D: int, device) -> _Exchange:
        import torch.distributed as dist

        from . import _lib

        key = (B, S, D, device)
        if self._exchange is not None and self._exchange.key == key:
            return self._exchange
        self.close()
        bufs = [torch.empty(B, S, D, dtype=torch.float32, device=device) for _ in range(self.buffers)]
        if self.transport == "nccl":  # no peer mappings: NCCL moves the rows
            self._exchange = _Exchange(key, bufs, None, [], [], None)
            self._turn = 0
            return self._exchange
        mine = [_lib.ipc_export(b.data_ptr()) for b in bufs]
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=self.group)
        ptrs: List[List[int]] = []
        mapped = {}
        for d in range(self.world):
            if d == self.rank:
                ptrs.append([b.data_ptr() for b in bufs])
                continue
            row = []
            for handle, offset in every[d]:
                if handle not in mapped:  # several buffers may share one allocation
                    mapped[handle] = _lib.ipc_open(handle)
                row.append(mapped[handle] + offset)
            ptrs.append(row)
        # kernel: one high-priority stream, its push kernel's CTAs scheduled
        # ahead of the next micro-batch's waiting CTAs; copy engines: one
        # stream per destination, so the copies run on several engines
        n_streams = 1 if self.transport == "kernel" else self.world * self.copy_streams
        streams = [torch.cuda.Stream(device, priority=-1) for _ in range(n_streams)]
        flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._exchange = _Exchange(key, bufs, ptrs, list(mapped.values()), streams, flag)
        self._turn = 0
        return self._exchange

    def close(self) -> None:
        """Unmaps the peers' buffers (collective: every rank calls it, so no
        rank frees a buffer another still maps)."""
        ex = self._exchange
        if ex is None:
            return
        import torch.distributed as dist

        from . import _lib

        for s in ex.streams:
            s.synchronize()
        dev = ex.bufs[0].device
        torch.cuda.current_stream(dev).synchronize()
        for base in ex.mapped:
            _lib.ipc_close(base)
        dist.barrier(group=self.group, device_ids=[dev.index])
        self._exchange = None

    def _gather_forward(self, x_local, mask_local, assignment, valid_lengths):
        import torch.distributed as dist

        from . import _lib

        dev = x_local.device
        n_local, S, D = x_local.shape
        if assignment is None:
            assignment = self._global_assignment(n_local, dev)
        if len(assignment) != self.world or len(assignment[self.rank]) != n_local:
            raise ValueError("assignment does not match the ranks' local batches")
        B = sum(len(a) for a in assignment)
        if valid_lengths is not None and len(valid_lengths) != B:
            raise ValueError(f"valid_lengths has {len(valid_lengths)} entries for a batch of {B}")
        ex = self._exchange_for(B, S, D, dev)
        buf = self._turn
        self._turn = (self._turn + 1) % self.buffers
        row_bytes = D * 4
        compute = torch.cuda.current_stream(dev)
        if valid_lengths is not None:
            base = ex.bufs[buf].data_ptr()
            _lib.copy_segments([(base + off, 0, n) for off, n in zero_fill_segments(valid_lengths, S, row_bytes)],
                               compute.cuda_stream)
        if self.transport == "nccl":
            return self._gather_nccl(x_local, mask_local, assignment, valid_lengths, ex.bufs[buf])
        push = ex.streams[0]
        dsts = [ex.ptrs[d][buf] for d in range(self.world)]
        for j0, j1 in micro_batch_ranges(n_local, self.micro_batches):
            out = self.model(x_local[j0:j1], None if mask_local is None else mask_local[j0:j1])
            done = torch.cuda.Event()
            done.record(compute)
            segs = gather_segments(assignment, self.rank, (j0, j1), S, row_bytes, valid_lengths)
            src = out.data_ptr()
            if self.transport == "kernel":
                push.wait_event(done)
                _lib.push_segments(dsts, [(do, src + so, n) for do, so, n in segs], push.cuda_stream,
                                   blocks=self.push_blocks)
                out.record_stream(push)
            else:
                k = self.copy_streams
                shares = split_segments(segs, k, row_bytes)
                for d in range(self.world):
                    for i in range(k):
                        stream = ex.streams[d * k + i]
                        stream.wait_event(done)
                        if shares[i]:
                            _lib.copy_segments([(dsts[d] + do, src + so, n) for do, so, n in shares[i]],
                                               stream.cuda_stream)
                        out.record_stream(stream)
        for stream in ex.streams:
            compute.wait_stream(stream)
        # Completes on a rank only after every rank has reached it, i.e. after
        # every rank's pushes (ordered before it on that rank's stream) landed.
        dist.all_reduce(ex.flag, group=self.group)
        return ex.bufs[buf]

    def _gather_nccl(self, x_local, mask_local, assignment, valid_lengths, out_all):
        """Micro-batch k on every rank, then one batch_isend_irecv per step:
        the step's valid rows to every peer, the peers' step-k rows straight
        into out_all; NCCL runs them on its own stream after the step's
        forward, while the next step computes.  The current stream waits for
        this rank's receives at the end."""
        import torch.distributed as dist

        S = out_all.shape[1]
        works, keep_alive = [], []
        group_ranks = None if self.group is None else dist.get_process_group_ranks(self.group)

        def peer(r):  # group rank -> global rank for P2POp
            return r if group_ranks is None else group_ranks[r]

        for k in range(p2p_steps(assignment, self.micro_batches)):
            mine, sends, recvs, keeps = p2p_step_plan(assignment, self.rank, k, self.micro_batches, S,
                                                      valid_lengths)
            ops = []
            if mine is not None:
                j0, j1 = mine
                out = self.model(x_local[j0:j1], None if mask_local is None else mask_local[j0:j1])
                keep_alive.append(out)
                for jl, b, n in keeps:
                    out_all[b, :n].copy_(out[jl, :n])
                for d, jl, n in sends:
                    ops.append(dist.P2POp(dist.isend, out[jl, :n], peer(d), group=self.group))
            for src, b, n in recvs:
                ops.append(dist.P2POp(dist.irecv, out_all[b, :n], peer(src), group=self.group))
            if ops:
                works.extend(dist.batch_isend_irecv(ops))
        for w in works:
            w.wait()
        return out_all


def segment_metadata(counts: torch.Tensor, rank: int, causal: bool):
    """Attention key-segment tables for context parallelism: one segment per
    rank (offset 0 in its slab, length = its valid tokens) and, for causal
    masking, the position of this rank's first valid token in the sequence."""
    G = counts.numel()
    kv_off = torch.zeros(1, G, dtype=torch.int32, device=counts.device)
    kv_len = counts.to(torch.int32).view(1, G).contiguous()
    q_pos0 = None
    if causal:
        q_pos0 = counts[:rank].to(torch.int32).sum().view(1).contiguous()
    return kv_off, kv_len, q_pos0


class _KvExchange:
    """Context parallelism's K/V exchange: two [G][2][H][slab][P] buffers per
    rank (used by alternate layers), each mapped into every other rank (CUDA
    IPC), one copy stream per peer, the partial-attention buffers and the
    one-element barrier tensor."""

    def __init__(self, key, bufs, ptrs, mapped, streams, part_o, part_lse, flag):
        self.key = key
        self.bufs = bufs
        self.ptrs = ptrs          # ptrs[d][i]: address of rank d's buffer i in this process
        self.mapped = mapped
        self.streams = streams    # streams[d]: copies into rank d
        self.part_o = part_o      # [slab, H*dh] fp32: attention over the rank's own keys
        self.part_lse = part_lse  # [slab, H] fp32: its log2-sum-exp
        self.flag = flag


class ContextParallelEncoder:
    """Context-parallel forward of one long sequence (batch 1) over a process
    group; each rank passes its chunk x_local [1, S_r, D] and mask_local
    [1, S_r] and gets its chunk of the output.  `slab` is the largest S_r over
    the ranks (all K/V slabs are padded to it).

    Per layer, after the QKV projection of its own tokens, each rank pushes its
    K/V slab ([2][H][slab][P], one contiguous block) into slot `rank` of every
    peer's K/V buffer with the copy engines over NVLink (CUDA IPC mappings) and,
    meanwhile, runs attention of its queries over its OWN keys, keeping the
    partial result (normalised fp32 context + log2-sum-exp).  An all-reduce of
    one element on the current stream is the barrier after which every peer's
    K/V has landed; attention over the other ranks' keys then merges with the
    partial (tj_flash_attn_fwd_partial).  With causal masking the keys of
    later ranks are all masked and those of earlier ranks all visible, so the
    second launch walks only the earlier ranks, unmasked.  The K/V buffers
    alternate between layers: a peer writes a buffer again only after every
    rank has passed the barrier of the layer in between, by which time this
    rank's attention over it has finished.

    overlap=False runs the plain form instead: a blocking NCCL all-gather of
    the K/V slabs, then one attention launch over every rank's keys."""

    def __init__(self, model, group=None, overlap: bool = True) -> None:
        import torch.distributed as dist

        self.model = model
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.overlap = bool(overlap)
        self._ex: Optional[_KvExchange] = None
        self._turn = 0

    def _exchange_for(self, slab: int, H: int, P: int, dh: int, device) -> _KvExchange:
        import torch.distributed as dist

        from . import _lib

        key = (slab, H, P, dh, device)
        if self._ex is not None and self._ex.key == key:
            return self._ex
        self.close()
        bufs = [torch.empty(self.world, 2, H, slab, P, dtype=torch.float16, device=device) for _ in range(2)]
        mine = [_lib.ipc_export(b.data_ptr()) for b in bufs]
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=self.group)
        ptrs, mapped = [], {}
        for d in range(self.world):
            if d == self.rank:
                ptrs.append([b.data_ptr() for b in bufs])
                continue
            row = []
            for handle, offset in every[d]:
                if handle not in mapped:
                    mapped[handle] = _lib.ipc_open(handle)
                row.append(mapped[handle] + offset)
            ptrs.append(row)
        streams = [torch.cuda.Stream(device) for _ in range(self.world)]  # streams[d]: pushes into rank d
        part_o = torch.empty(slab, H * dh, dtype=torch.float32, device=device)
        part_lse = torch.empty(slab, H, dtype=torch.float32, device=device)
        flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._ex = _KvExchange(key, bufs, ptrs, list(mapped.values()), streams, part_o, part_lse, flag)
        self._turn = 0
        return self._ex

    def close(self) -> None:
        """Unmaps the peers' K/V buffers (collective: every rank calls it)."""
        ex = self._ex
        if ex is None:
            return
        import torch.distributed as dist

        from . import _lib

        for s in ex.streams:
            s.synchronize()
        torch.cuda.current_stream(ex.flag.device).synchronize()
        for base in ex.mapped:
            _lib.ipc_close(base)
        dist.barrier(group=self.group, device_ids=[ex.flag.device.index])
        self._ex = None

    def forward(self, x_local: torch.Tensor, mask_local: Optional[torch.Tensor], slab: int) -> torch.Tensor:
        import torch.distributed as dist

        from . import _lib

        m = self.model
        cfg = m.config
        if m.training:
            raise RuntimeError("inference only; call .eval()")
        if x_local.dim() != 3 or x_local.shape[0] != 1:
            raise ValueError("context parallelism takes one sequence: x_local must be [1, S_r, D]")
        if x_local.dtype != torch.float32 or x_local.device.type != "cuda":
            raise TypeError("x_local must be a float32 CUDA tensor")
        dev = x_local.device
        _, Sl, D = x_local.shape
        if Sl > slab:
            raise ValueError(f"local chunk {Sl} longer than slab {slab}")
        H, F = cfg.num_heads, cfg.ffn_dim
        if D % 8 or F % 8:
            # The per-kernel entry points take dense fp16 rows, which TMA needs
            # to be whole 16-byte units; the single-GPU encoder pads its own
            # buffers instead (tj_encoder_forward).
            raise ValueError(f"context parallelism needs d_model and ffn_dim that are multiples of 8 "
                             f"(got {D} and {F}); run such a model on one GPU")
        dh = D // H
        causal = bool(cfg.causal)
        x = x_local.contiguous().view(Sl, D)
        if mask_local is not None:
            mask_u8 = mask_local.contiguous().view(torch.uint8) if mask_local.dtype == torch.bool else mask_local.contiguous()
        else:
            mask_u8 = None
        plan = kernels.token_plan(mask_u8, 1, Sl, dev)
        nv, cu, cnt, orig, inv = kernels.plan_views(plan, 1, Sl)
        counts = torch.empty(self.world, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(counts, cnt.contiguous(), group=self.group)
        kv_off, kv_len, q_pos0 = segment_metadata(counts, self.rank, causal)
        P = kernels.head_pad(dh)  # heads zero-padded to P halves
        if self.overlap:
            ex = self._exchange_for(slab, H, P, dh, dev)
            own_off = torch.zeros(1, 1, dtype=torch.int32, device=dev)
            own_len = cnt.view(1, 1).contiguous()
            # the second launch's keys: every other rank's (causal: the earlier ranks')
            remote_len = kv_len.clone()
            if causal:
                remote_len[:, self.rank:] = 0
            else:
                remote_len[:, self.rank] = 0
            has_remote = self.world > 1 and (not causal or self.rank > 0)
            seg_bytes = 2 * H * slab * P * 2
        else:
            kv_all = torch.empty(self.world, 2, H, slab, P, dtype=torch.float16, device=dev)

        a16 = torch.empty(slab, D, dtype=torch.float16, device=dev)
        qkv = torch.empty(3, H, slab, P, dtype=torch.float16, device=dev)
        ctx = torch.empty(slab, D, dtype=torch.float16, device=dev)
        h16 = torch.empty(slab, F, dtype=torch.float16, device=dev)
        y16 = torch.empty(Sl, D, dtype=torch.float16, device=dev)
        x1 = torch.empty(Sl, D, dtype=torch.float32, device=dev)
        x2 = torch.empty(Sl, D, dtype=torch.float32, device=dev)
        compute = torch.cuda.current_stream(dev)

        # Residual stream as in tj_encoder_forward: layer 0 reads x through the
        # plan's gather map; the out-projection and FFN-out write fp16 (y16) and
        # the next LayerNorm adds them to the fp32 stream (x1 after attention,
        # x2 = input of the next layer).  GEMM outputs only reach the first nv
        # (<= S_r) rows, so the fp32 buffers hold S_r rows.
        for i, layer in enumerate(m.layers):
            att = layer.attention
            if i == 0:
                xin, in_map = x, orig
                kernels.ln_cast_f16(x, layer.norm1.weight, layer.norm1.bias, layer.norm1.eps,
                                    row_map=orig, row_count=nv, out=a16)
            else:
                xin, in_map = x2, None
                kernels.add_ln_cast_f16(x1, y16, layer.norm1.weight, layer.norm1.bias, layer.norm1.eps,
                                        row_count=nv, sum_out=x2, out=a16)
            kernels.gemm_qkv_headmajor(a16, att._qkv_weight_mixed, att._qkv_bias_mixed, H,
                                       row_count=nv, out=qkv)
            if self.overlap:
                buf = self._turn
                self._turn ^= 1
                kv_ready = torch.cuda.Event()
                kv_ready.record(compute)
                for d in range(self.world):  # copy engines, one stream per peer
                    if d == self.rank:
                        continue
                    st = ex.streams[d]
                    st.wait_event(kv_ready)
                    _lib.copy_segments([(ex.ptrs[d][buf] + self.rank * seg_bytes, qkv[1].data_ptr(), seg_bytes)],
                                       st.cuda_stream)
                    qkv.record_stream(st)
                # attention over this rank's own keys while the K/V blocks travel
                kernels.flash_attn_fwd(qkv[0], qkv[1:2], qkv[2:3], cu, own_off, own_len, Sl, att.scale,
                                       causal=causal, out=None if has_remote else ctx, head_dim=dh,
                                       part_o=ex.part_o if has_remote else None,
                                       part_lse=ex.part_lse if has_remote else None,
                                       part_mode=1 if has_remote else 0)
                for d in range(self.world):
                    if d != self.rank:
                        compute.wait_stream(ex.streams[d])
                # completes once every rank's pushes (ordered before it on that
                # rank's stream) have landed
                dist.all_reduce(ex.flag, group=self.group)
                if has_remote:
                    kv = ex.bufs[buf]
                    kernels.flash_attn_fwd(qkv[0], kv[:, 0], kv[:, 1], cu, kv_off, remote_len, Sl, att.scale,
                                           causal=False, out=ctx, head_dim=dh, part_o=ex.part_o,
                                           part_lse=ex.part_lse, part_mode=2)
            else:
                dist.all_gather_into_tensor(kv_all.view(-1), qkv[1:3].reshape(-1), group=self.group)
                kernels.flash_attn_fwd(qkv[0], kv_all[:, 0], kv_all[:, 1], cu, kv_off, kv_len, Sl, att.scale,
                                       causal=causal, q_pos0=q_pos0, out=ctx, head_dim=dh)
            kernels.gemm_bias_f16(ctx[:Sl], att._out_weight_mixed, att.out_proj.bias, row_count=nv, out=y16)
            kernels.add_ln_cast_f16(xin, y16, layer.norm2.weight, layer.norm2.bias, layer.norm2.eps,
                                    row_map=in_map, row_count=nv, sum_out=x1, out=a16)
            kernels.gemm_bias_gelu_f16(a16, layer._ffn_in_weight_mixed, layer.ffn_in.bias, row_count=nv, out=h16)
            kernels.gemm_bias_f16(h16[:Sl], layer._ffn_out_weight_mixed, layer.ffn_out.bias, row_count=nv,
                                  out=y16)
        out = kernels.add_ln_final_mask(x1, y16, m.final_norm.weight, m.final_norm.bias, m.final_norm.eps,
                                        inv_map=inv, rows=Sl)
        return out.view(1, Sl, D)

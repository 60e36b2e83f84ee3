"""Multi-GPU execution of the encoder: batch sharding and context parallelism.

One process per GPU (torchrun), torch.distributed for the plumbing.

* Batch sharding: samples are independent in the reference model (every op
  is per sample), so each rank runs a contiguous, balanced range of the batch
  (the balanced-range split of the reference's multi-stream variant,
  candidates/v19/parallel_batch_common.py:31-51) or, balanced by estimated
  work rather than count, the sample set of `balanced_assignment`, with no
  data-path collective; `BatchShardedEncoder.forward(..., gather=True)`
  optionally all-gathers the outputs (back in batch order).
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
    the projections' tensor-core rate.  Returns sorted index lists."""
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
    return [sorted(o) for o in out]


class BatchShardedEncoder:
    """Runs `model` on this rank's share of the batch: a contiguous range
    (`local_range`), or the work-balanced sample set of `balanced_assignment`
    (`local_samples`), in which case `forward(..., gather=True, assignment=a)`
    puts the gathered outputs back in batch order."""

    def __init__(self, model, group=None) -> None:
        import torch.distributed as dist

        self.model = model
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def local_range(self, batch: int) -> Tuple[int, int]:
        return batch_ranges(batch, self.world)[self.rank]

    def assignment(self, valid_token_mask: torch.Tensor) -> List[List[int]]:
        """The work-balanced split of a [B, S] mask (the same on every rank)."""
        cfg = self.model.config
        lengths = valid_token_mask.to(torch.int64).sum(1).tolist()
        return balanced_assignment(lengths, self.world, cfg.d_model, cfg.ffn_dim)

    def forward(self, x_local: torch.Tensor, mask_local: Optional[torch.Tensor], gather: bool = False,
                assignment: Optional[Sequence[Sequence[int]]] = None):
        # A rank may hold no samples (batch < world); it still joins the gather.
        out = self.model(x_local, mask_local)
        if not gather or self.world == 1:
            return out
        import torch.distributed as dist

        sizes = [torch.zeros(1, dtype=torch.int64, device=out.device) for _ in range(self.world)]
        dist.all_gather(sizes, torch.tensor([out.shape[0]], dtype=torch.int64, device=out.device), group=self.group)
        sizes = [int(s.item()) for s in sizes]
        parts = [torch.empty((n,) + tuple(out.shape[1:]), dtype=out.dtype, device=out.device) for n in sizes]
        dist.all_gather(parts, out.contiguous(), group=self.group)
        full = torch.cat(parts, 0)
        if assignment is None:
            return full
        order = torch.tensor([i for r in assignment for i in r], dtype=torch.int64, device=full.device)
        if order.numel() != full.shape[0]:
            raise ValueError("assignment does not cover the gathered batch")
        result = torch.empty_like(full)
        result[order] = full
        return result


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


class ContextParallelEncoder:
    """Context-parallel forward of one long sequence (batch 1) over a process
    group; each rank passes its chunk x_local [1, S_r, D] and mask_local
    [1, S_r] and gets its chunk of the output.  `slab` is the largest S_r over
    the ranks (all K/V slabs are padded to it so they can be all-gathered)."""

    def __init__(self, model, group=None) -> None:
        import torch.distributed as dist

        self.model = model
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def forward(self, x_local: torch.Tensor, mask_local: Optional[torch.Tensor], slab: int) -> torch.Tensor:
        import torch.distributed as dist

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
        dh = D // H
        x = x_local.contiguous().view(Sl, D)
        if mask_local is not None:
            mask_u8 = mask_local.contiguous().view(torch.uint8) if mask_local.dtype == torch.bool else mask_local.contiguous()
        else:
            mask_u8 = None
        plan = kernels.token_plan(mask_u8, 1, Sl, dev)
        nv, cu, cnt, orig, inv = kernels.plan_views(plan, 1, Sl)
        counts = torch.empty(self.world, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(counts, cnt.contiguous(), group=self.group)
        kv_off, kv_len, q_pos0 = segment_metadata(counts, self.rank, bool(cfg.causal))

        a16 = torch.empty(slab, D, dtype=torch.float16, device=dev)
        P = kernels.head_pad(dh)  # heads zero-padded to P halves
        qkv = torch.empty(3, H, slab, P, dtype=torch.float16, device=dev)
        kv_all = torch.empty(self.world, 2, H, slab, P, dtype=torch.float16, device=dev)
        ctx = torch.empty(slab, D, dtype=torch.float16, device=dev)
        h16 = torch.empty(slab, F, dtype=torch.float16, device=dev)
        y16 = torch.empty(Sl, D, dtype=torch.float16, device=dev)
        x1 = torch.empty(Sl, D, dtype=torch.float32, device=dev)
        x2 = torch.empty(Sl, D, dtype=torch.float32, device=dev)

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
            dist.all_gather_into_tensor(kv_all.view(-1), qkv[1:3].reshape(-1), group=self.group)
            kernels.flash_attn_fwd(qkv[0], kv_all[:, 0], kv_all[:, 1], cu, kv_off, kv_len, Sl, att.scale,
                                   causal=bool(cfg.causal), q_pos0=q_pos0, out=ctx, head_dim=dh)
            kernels.gemm_bias_f16(ctx[:Sl], att._out_weight_mixed, att.out_proj.bias, row_count=nv, out=y16)
            kernels.add_ln_cast_f16(xin, y16, layer.norm2.weight, layer.norm2.bias, layer.norm2.eps,
                                    row_map=in_map, row_count=nv, sum_out=x1, out=a16)
            kernels.gemm_bias_gelu_f16(a16, layer._ffn_in_weight_mixed, layer.ffn_in.bias, row_count=nv, out=h16)
            kernels.gemm_bias_f16(h16[:Sl], layer._ffn_out_weight_mixed, layer.ffn_out.bias, row_count=nv,
                                  out=y16)
        out = kernels.add_ln_final_mask(x1, y16, m.final_norm.weight, m.final_norm.bias, m.final_norm.eps,
                                        inv_map=inv, rows=Sl)
        return out.view(1, Sl, D)

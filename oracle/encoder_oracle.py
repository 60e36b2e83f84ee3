"""CPU FP32 restatement of the reference Transformer encoder (the oracle).

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path: it
is imported by tests/, by __graft_entry__.smoke() and by bench.py's
CPU-baseline leg, never by the product package.

It restates, in functional PyTorch FP32 form over a state_dict, the
reference's own FP32 model `BaselineTransformer` and its helpers, which live
in the reference repository's `torch_transformer_benchmark.py`:

  TransformerConfig            torch_transformer_benchmark.py:29-56
  BaselineSelfAttention        torch_transformer_benchmark.py:59-122
  BaselineTransformerBlock     torch_transformer_benchmark.py:125-145
  BaselineTransformer          torch_transformer_benchmark.py:148-172
  generate_random_case         torch_transformer_benchmark.py:234-272
  compare_outputs              torch_transformer_benchmark.py:289-356
and the query-blocked (memory-bounded) variant and streaming comparator of
  tools/shape14/accuracy.py:68-156 (memory_bounded_attention/_baseline)
  tools/shape14/accuracy.py:160-201 (StreamingAccuracy, update_accuracy).

Pinning: tests/golden/ holds outputs of the real reference (imported from its
own source by tests/golden/make_golden.py) and tests/test_oracle_golden.py
checks this restatement against them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class TransformerConfig:
    """Same fields and validation as torch_transformer_benchmark.py:29-56."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")


# ---------------------------------------------------------------------------
# Parameters
# ---------------------------------------------------------------------------
def make_state_dict(config: TransformerConfig, seed: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """Default-initialised parameters with the reference's names and RNG order.

    BaselineTransformer (torch_transformer_benchmark.py:148-160) builds, per
    layer, norm1, attention.{q,k,v,out}_proj, norm2, ffn_in, ffn_out and then
    final_norm; nn.Linear draws Kaiming-uniform weights then uniform biases
    from the global generator, nn.LayerNorm draws nothing.  Building the same
    modules in the same order after torch.manual_seed(seed) reproduces the
    reference's weights bit for bit.
    """
    if seed is not None:
        torch.manual_seed(seed)
    D, H, Fd = config.d_model, config.num_heads, config.ffn_dim
    sd: Dict[str, torch.Tensor] = {}
    for i in range(config.num_layers):
        p = f"layers.{i}."
        norm1 = nn.LayerNorm(D)
        q, k, v, o = (nn.Linear(D, D, bias=True) for _ in range(4))
        norm2 = nn.LayerNorm(D)
        ffn_in = nn.Linear(D, Fd)
        ffn_out = nn.Linear(Fd, D)
        for name, mod in (
            ("norm1", norm1),
            ("attention.q_proj", q),
            ("attention.k_proj", k),
            ("attention.v_proj", v),
            ("attention.out_proj", o),
            ("norm2", norm2),
            ("ffn_in", ffn_in),
            ("ffn_out", ffn_out),
        ):
            sd[p + name + ".weight"] = mod.weight.detach().clone()
            sd[p + name + ".bias"] = mod.bias.detach().clone()
    fn = nn.LayerNorm(D)
    sd["final_norm.weight"] = fn.weight.detach().clone()
    sd["final_norm.bias"] = fn.bias.detach().clone()
    return sd


def perturb_layernorm(sd: Dict[str, torch.Tensor], seed: int, scale: float = 0.02) -> Dict[str, torch.Tensor]:
    """LayerNorm gamma ~ 1 + scale*N(0,1), beta ~ scale*N(0,1) (the GPU configs'
    LayerNorm distribution), drawn from a private generator in key order."""
    g = torch.Generator().manual_seed(seed)
    out = dict(sd)
    for name in sd:
        if ".norm" in name or name.startswith("final_norm"):
            t = sd[name]
            noise = torch.randn(t.shape, generator=g, dtype=torch.float32)
            out[name] = (1.0 + scale * noise) if name.endswith(".weight") else scale * noise
    return out


# ---------------------------------------------------------------------------
# Inputs
# ---------------------------------------------------------------------------
def generate_random_case(
    config: TransformerConfig,
    seed: int,
    padding_ratio: float,
    input_scale: float = 1.0,
    device: str | torch.device = "cpu",
    dtype: torch.dtype = torch.float32,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Restates torch_transformer_benchmark.py:234-272: x ~ N(0,1)*scale from a
    seeded generator, right-padded lengths ~ U{round(S(1-p)), .., S} drawn from
    the same generator, x zeroed at padded positions."""
    device = torch.device(device)
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    B, S, D = config.batch_size, config.seq_len, config.d_model
    x = torch.randn(B, S, D, generator=generator, device=device, dtype=dtype) * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(B, S, device=device, dtype=torch.bool)
    min_valid = max(1, int(round(S * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=S + 1, size=(B,), generator=generator, device=device)
    positions = torch.arange(S, device=device)[None, :]
    mask = positions < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


# ---------------------------------------------------------------------------
# Model
# ---------------------------------------------------------------------------
def _split_heads(t: torch.Tensor, H: int) -> torch.Tensor:
    B, S, D = t.shape
    return t.view(B, S, H, D // H).transpose(1, 2).contiguous()


def _attention(sd, p, x, mask, causal, H):
    """BaselineSelfAttention.forward, torch_transformer_benchmark.py:85-122."""
    B, S, D = x.shape
    scale = (D // H) ** -0.5
    q = _split_heads(F.linear(x, sd[p + "q_proj.weight"], sd[p + "q_proj.bias"]), H)
    k = _split_heads(F.linear(x, sd[p + "k_proj.weight"], sd[p + "k_proj.bias"]), H)
    v = _split_heads(F.linear(x, sd[p + "v_proj.weight"], sd[p + "v_proj.bias"]), H)
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        cm = torch.ones((S, S), device=x.device, dtype=torch.bool).triu(diagonal=1)
        scores = scores.masked_fill(cm, float("-inf"))
    if mask is not None:
        scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
    ctx = torch.matmul(probs, v).transpose(1, 2).contiguous().view(B, S, D)
    out = F.linear(ctx, sd[p + "out_proj.weight"], sd[p + "out_proj.bias"])
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


def _attention_blocked(sd, p, x, mask, causal, H, query_chunk):
    """memory_bounded_attention, tools/shape14/accuracy.py:68-122: the same
    formula evaluated query block by query block (no S x S score tensor)."""
    B, S, D = x.shape
    if B != 1:
        raise ValueError("the blocked oracle evaluates one sample at a time")
    scale = (D // H) ** -0.5
    q = _split_heads(F.linear(x, sd[p + "q_proj.weight"], sd[p + "q_proj.bias"]), H)
    k = _split_heads(F.linear(x, sd[p + "k_proj.weight"], sd[p + "k_proj.bias"]), H)
    v = _split_heads(F.linear(x, sd[p + "v_proj.weight"], sd[p + "v_proj.bias"]), H)
    ctx = torch.empty_like(q)
    key_pos = torch.arange(S, device=x.device)[None, :]
    invalid_keys = None if mask is None else ~mask[:, None, None, :]
    kt = k.transpose(-2, -1)
    for start in range(0, S, query_chunk):
        end = min(start + query_chunk, S)
        scores = torch.matmul(q[:, :, start:end], kt)
        scores.mul_(scale)
        if causal:
            qp = torch.arange(start, end, device=x.device)[:, None]
            scores.masked_fill_(key_pos > qp, float("-inf"))
        if invalid_keys is not None:
            scores.masked_fill_(invalid_keys, float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
        ctx[:, :, start:end].copy_(torch.matmul(probs, v))
    merged = ctx.transpose(1, 2).contiguous().view(B, S, D)
    out = F.linear(merged, sd[p + "out_proj.weight"], sd[p + "out_proj.bias"])
    if mask is not None:
        out.masked_fill_(~mask[..., None], 0)
    return out


def _encoder(sd, config, x, mask, attention_fn):
    """BaselineTransformer/Block.forward, torch_transformer_benchmark.py:134-145,162-172."""
    H = config.num_heads
    for i in range(config.num_layers):
        p = f"layers.{i}."
        D = x.shape[-1]
        h = F.layer_norm(x, (D,), sd[p + "norm1.weight"], sd[p + "norm1.bias"], 1e-5)
        x = x + attention_fn(sd, p + "attention.", h, mask, config.causal, H)
        h = F.layer_norm(x, (D,), sd[p + "norm2.weight"], sd[p + "norm2.bias"], 1e-5)
        h = F.gelu(F.linear(h, sd[p + "ffn_in.weight"], sd[p + "ffn_in.bias"]), approximate="none")
        x = x + F.linear(h, sd[p + "ffn_out.weight"], sd[p + "ffn_out.bias"])
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
    D = x.shape[-1]
    x = F.layer_norm(x, (D,), sd["final_norm.weight"], sd["final_norm.bias"], 1e-5)
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x


@torch.inference_mode()
def encoder_forward(sd, config: TransformerConfig, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    """FP32 forward of the reference encoder on x [B,S,D] with optional bool mask [B,S]."""
    return _encoder(sd, config, x, mask, _attention)


@torch.inference_mode()
def encoder_forward_blocked(
    sd, config: TransformerConfig, x: torch.Tensor, mask: Optional[torch.Tensor], query_chunk: int = 256
) -> torch.Tensor:
    """FP32 forward with query-blocked attention, one sample at a time (samples
    are independent in the reference: every op is per sample)."""
    outs = []
    for b in range(x.shape[0]):
        mb = None if mask is None else mask[b : b + 1]
        outs.append(
            _encoder(
                sd,
                config,
                x[b : b + 1],
                mb,
                lambda s, p, h, m, c, H: _attention_blocked(s, p, h, m, c, H, query_chunk),
            )
        )
    return torch.cat(outs, dim=0)


@torch.inference_mode()
def encoder_forward_query_rows(
    sd, config: TransformerConfig, x: torch.Tensor, mask: Optional[torch.Tensor], rows, query_chunk: int = 64
) -> torch.Tensor:
    """Output rows `rows` (sequence positions) of a ONE-layer encoder on ONE
    sample, without evaluating the other rows.

    The query-blocked oracle (memory_bounded_baseline, tools/shape14/accuracy.py:125-156,
    attention :68-122) restricted to a subset of query blocks.  Keys and values
    depend on every token, so LN1 and the K/V projections run over the whole
    sequence; Q, the attention rows, the out-projection, the residual adds,
    LN2, the FFN and the final LayerNorm are evaluated for `rows` only (every
    op except attention is per token, and with one layer the other rows'
    outputs never feed these).  The formula is the reference's unchanged:
    scores * scale, causal and key masks as -inf, FP32 softmax, probs @ v,
    invalid query rows zeroed after attention, after the block and after the
    final LayerNorm.  Returns [len(rows), D]."""
    if x.shape[0] != 1:
        raise ValueError("the query-row oracle evaluates one sample")
    if config.num_layers != 1:
        raise ValueError("the query-row oracle needs one layer (later layers read every row)")
    rows = torch.as_tensor(rows, dtype=torch.int64).reshape(-1)
    _, S, D = x.shape
    H = config.num_heads
    if rows.numel() and (int(rows.min()) < 0 or int(rows.max()) >= S):
        raise ValueError("query rows out of range")
    p = "layers.0."
    a = p + "attention."
    scale = (D // H) ** -0.5
    h = F.layer_norm(x, (D,), sd[p + "norm1.weight"], sd[p + "norm1.bias"], 1e-5)
    k = _split_heads(F.linear(h, sd[a + "k_proj.weight"], sd[a + "k_proj.bias"]), H)
    v = _split_heads(F.linear(h, sd[a + "v_proj.weight"], sd[a + "v_proj.bias"]), H)
    q = _split_heads(F.linear(h[:, rows], sd[a + "q_proj.weight"], sd[a + "q_proj.bias"]), H)
    del h
    ctx = torch.empty_like(q)
    key_pos = torch.arange(S, device=x.device)[None, :]
    invalid_keys = None if mask is None else ~mask[:, None, None, :]
    kt = k.transpose(-2, -1)
    for start in range(0, rows.numel(), query_chunk):
        end = min(start + query_chunk, rows.numel())
        scores = torch.matmul(q[:, :, start:end], kt)
        scores.mul_(scale)
        if config.causal:
            scores.masked_fill_(key_pos > rows[start:end, None], float("-inf"))
        if invalid_keys is not None:
            scores.masked_fill_(invalid_keys, float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
        ctx[:, :, start:end].copy_(torch.matmul(probs, v))
        del scores, probs
    merged = ctx.transpose(1, 2).contiguous().view(1, rows.numel(), D)
    attn = F.linear(merged, sd[a + "out_proj.weight"], sd[a + "out_proj.bias"])
    qmask = None if mask is None else mask[:, rows]
    if qmask is not None:
        attn = attn.masked_fill(~qmask[..., None], 0)
    xr = x[:, rows] + attn
    h2 = F.layer_norm(xr, (D,), sd[p + "norm2.weight"], sd[p + "norm2.bias"], 1e-5)
    h2 = F.gelu(F.linear(h2, sd[p + "ffn_in.weight"], sd[p + "ffn_in.bias"]), approximate="none")
    xr = xr + F.linear(h2, sd[p + "ffn_out.weight"], sd[p + "ffn_out.bias"])
    if qmask is not None:
        xr = xr.masked_fill(~qmask[..., None], 0)
    out = F.layer_norm(xr, (D,), sd["final_norm.weight"], sd["final_norm.bias"], 1e-5)
    if qmask is not None:
        out = out.masked_fill(~qmask[..., None], 0)
    return out[0]


def long_sequence_check_rows(valid_len: int, seq_len: int, block: int = 256) -> torch.Tensor:
    """Query rows a long-sequence parity check evaluates: the first, a middle
    and the last block of `block` valid positions (the shape-#14 accuracy
    tool's query blocks, tools/shape14/accuracy.py:92-119, at the start,
    middle and end of the valid prefix), plus the first padded position when
    there is one."""
    L = int(valid_len)
    if L <= 0:
        return torch.zeros(0, dtype=torch.int64)
    b = min(block, L)
    mid = max(0, min(L - b, L // 2 - b // 2))
    picks = [torch.arange(0, b), torch.arange(mid, mid + b), torch.arange(L - b, L)]
    if L < seq_len:
        picks.append(torch.tensor([L]))
    return torch.unique(torch.cat(picks))


# ---------------------------------------------------------------------------
# Comparator
# ---------------------------------------------------------------------------
@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    failed_feature_dims: List[int]
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float


def compare_outputs(reference: torch.Tensor, optimized: torch.Tensor, rtol: float = 0.02, atol: float = 0.002) -> AccuracyResult:
    """torch_transformer_benchmark.py:289-356: element passes iff finite on both
    sides and (|d| < atol or |d| < rtol*|ref|), strict inequalities."""
    if reference.shape != optimized.shape:
        raise AssertionError(f"shape mismatch: {tuple(reference.shape)} vs {tuple(optimized.shape)}")
    ref = reference.detach().float().cpu()
    opt = optimized.detach().float().cpu()
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    abs_err = (opt - ref).abs()
    passed_mask = finite & ((abs_err < atol) | (abs_err < rtol * ref.abs()))
    failed_mask = ~passed_mask
    failed = int(failed_mask.sum().item())
    flat = int(torch.nan_to_num(abs_err, nan=float("inf")).reshape(-1).argmax().item()) if ref.numel() else 0
    idx = []
    rem = flat
    for size in reversed(ref.shape):
        idx.append(rem % size)
        rem //= size
    worst = tuple(reversed(idx))
    rel = abs_err / ref.abs().clamp_min(1e-12)
    if ref.ndim >= 2:
        dims = torch.nonzero(failed_mask.any(dim=tuple(range(ref.ndim - 1))), as_tuple=False).flatten().tolist()
    else:
        dims = torch.nonzero(failed_mask, as_tuple=False).flatten().tolist()
    return AccuracyResult(
        passed=failed == 0,
        total_elements=ref.numel(),
        failed_elements=failed,
        max_abs_error=float(abs_err.max().item()) if ref.numel() else 0.0,
        max_relative_error=float(rel.max().item()) if ref.numel() else 0.0,
        mean_abs_error=float(abs_err.mean().item()) if ref.numel() else 0.0,
        failed_feature_dims=dims,
        worst_index=worst,
        reference_at_worst=float(ref[worst].item()) if ref.numel() else 0.0,
        optimized_at_worst=float(opt[worst].item()) if ref.numel() else 0.0,
    )


@dataclass
class StreamingAccuracy:
    """tools/shape14/accuracy.py:160-170."""

    total: int = 0
    failed: int = 0
    abs_sum: float = 0.0
    max_abs: float = 0.0
    max_rel: float = 0.0

    @property
    def passed(self) -> bool:
        return self.failed == 0


def update_accuracy(summary: StreamingAccuracy, reference: torch.Tensor, candidate: torch.Tensor,
                    token_chunk: int = 2048, rtol: float = 0.02, atol: float = 0.002) -> None:
    """tools/shape14/accuracy.py:172-201: the strict OR comparator over token slices."""
    if reference.shape != candidate.shape:
        raise AssertionError(f"shape mismatch: {tuple(reference.shape)} != {tuple(candidate.shape)}")
    for start in range(0, reference.shape[1], token_chunk):
        end = min(start + token_chunk, reference.shape[1])
        ref = reference[:, start:end].float()
        opt = candidate[:, start:end].float().to(ref.device)
        finite = torch.isfinite(ref) & torch.isfinite(opt)
        err = (opt - ref).abs()
        ok = finite & ((err < atol) | (err < rtol * ref.abs()))
        rel = err / ref.abs().clamp_min(1e-12)
        summary.total += ref.numel()
        summary.failed += int((~ok).sum().item())
        summary.abs_sum += float(err.double().sum().item())
        summary.max_abs = max(summary.max_abs, float(err.max().item()))
        summary.max_rel = max(summary.max_rel, float(rel.max().item()))

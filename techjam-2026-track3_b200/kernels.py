"""Torch-facing wrappers of the single-kernel C-ABI entry points.

Each wrapper validates device, dtype, contiguity and shape the way the
reference's custom op does (v16_1_clean.py:323-335: TypeError/ValueError on
bad inputs), then passes raw pointers and the current CUDA stream to the
library.  They exist for the per-kernel parity tests and for callers that
compose the layer themselves; UserOptimizedTransformer uses the single
tj_encoder_forward entry point.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def head_pad(head_dim: int) -> int:
    """Row length (halves) of the head-major q/k/v buffers: heads are
    zero-padded to 64, 128 or 256."""
    if not 1 <= head_dim <= 256:
        raise ValueError(f"head_dim must be in 1..256, got {head_dim}")
    return 64 if head_dim <= 64 else (128 if head_dim <= 128 else 256)


def _require(t: torch.Tensor, name: str, dtype: torch.dtype, device: torch.device) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.device != device:
        raise ValueError(f"{name} must be on {device}, got {t.device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _require_out(out: torch.Tensor, name: str, shape, dtype: torch.dtype, device: torch.device) -> None:
    """A caller-provided output must be exactly the buffer the kernel writes:
    the C ABI takes raw pointers and cannot check sizes itself."""
    _require(out, name, dtype, device)
    if tuple(out.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(out.shape)}")


def token_plan(mask: Optional[torch.Tensor], batch: int, seq_len: int, device) -> torch.Tensor:
    lib = _lib.load()
    n = lib.tj_token_plan_ints(batch, seq_len)
    plan = torch.empty(n, dtype=torch.int32, device=device)
    mptr = None
    if mask is not None:
        if mask.shape != (batch, seq_len):
            raise ValueError(f"mask must be [{batch}, {seq_len}], got {tuple(mask.shape)}")
        m = mask.contiguous()
        if m.dtype == torch.bool:
            m = m.view(torch.uint8)
        _require(m, "mask", torch.uint8, plan.device)
        mptr = m.data_ptr()
    _lib.check(lib.tj_token_plan(mptr, batch, seq_len, plan.data_ptr(), _stream(plan)), "token_plan")
    return plan


def plan_views(plan: torch.Tensor, batch: int, seq_len: int):
    """(nv[1], cu[B+1], counts[B], orig[BS], inv[BS]) views of a token plan (it
    ends with order[B], the samples by decreasing count: plan_order)."""
    B, BS = batch, batch * seq_len
    nv = plan[0:1]
    cu = plan[1 : B + 2]
    cnt = plan[B + 2 : 2 * B + 2]
    orig = plan[2 * B + 2 : 2 * B + 2 + BS]
    inv = plan[2 * B + 2 + BS : 2 * B + 2 + 2 * BS]
    return nv, cu, cnt, orig, inv


def plan_order(plan: torch.Tensor, batch: int, seq_len: int) -> torch.Tensor:
    """order[B] of a token plan: samples by decreasing valid count (stable;
    the identity for batches above 256)."""
    off = 2 * batch + 2 + 2 * batch * seq_len
    return plan[off : off + batch]


def ln_cast_f16(x, gamma, beta, eps=1e-5, row_map=None, row_count=None, out=None):
    dev = x.device
    _require(x, "x", torch.float32, dev)
    D = x.shape[-1]
    rows = x.numel() // D if row_map is None else row_map.numel()
    if out is None:
        out = torch.empty(rows, D, dtype=torch.float16, device=dev)
    if out.dim() != 2 or out.shape[1] != D or out.shape[0] < rows:
        raise ValueError(f"out must be [>= {rows}, {D}], got {tuple(out.shape)}")
    _require(out, "out", torch.float16, dev)
    lib = _lib.load()
    rc = lib.tj_ln_cast_f16(
        x.data_ptr(), _ptr(row_map), _ptr(row_count), rows, D, gamma.data_ptr(), beta.data_ptr(),
        float(eps), out.data_ptr(), _stream(x),
    )
    _lib.check(rc, "ln_cast_f16")
    return out


def ln_final_mask(x, gamma, beta, eps=1e-5, inv_map=None, rows=None, out=None):
    dev = x.device
    _require(x, "x", torch.float32, dev)
    D = x.shape[-1]
    if rows is None:
        rows = x.numel() // D if inv_map is None else inv_map.numel()
    if out is None:
        out = torch.empty(rows, D, dtype=torch.float32, device=dev)
    _require_out(out, "out", (rows, D), torch.float32, dev)
    lib = _lib.load()
    rc = lib.tj_ln_final_mask(
        x.data_ptr(), _ptr(inv_map), rows, D, gamma.data_ptr(), beta.data_ptr(), float(eps),
        out.data_ptr(), _stream(x),
    )
    _lib.check(rc, "ln_final_mask")
    return out


def add_ln_cast_f16(x, add16, gamma, beta, eps=1e-5, row_map=None, row_count=None, sum_out=None,
                    out=None):
    """s = x[row_map[r]] + add16[r] (fp32); sum_out[r] = s; out[r] = fp16(LayerNorm(s))."""
    dev = x.device
    _require(x, "x", torch.float32, dev)
    _require(add16, "add16", torch.float16, dev)
    D = x.shape[-1]
    rows = x.numel() // D if row_map is None else row_map.numel()
    if add16.dim() != 2 or add16.shape[1] != D or add16.shape[0] < rows:
        raise ValueError(f"add16 must be [>= {rows}, {D}], got {tuple(add16.shape)}")
    if out is None:
        out = torch.empty(rows, D, dtype=torch.float16, device=dev)
    if out.dim() != 2 or out.shape[1] != D or out.shape[0] < rows:
        raise ValueError(f"out must be [>= {rows}, {D}], got {tuple(out.shape)}")
    _require(out, "out", torch.float16, dev)
    if sum_out is not None:
        _require(sum_out, "sum_out", torch.float32, dev)
        if sum_out.dim() != 2 or sum_out.shape[1] != D or sum_out.shape[0] < rows:
            raise ValueError(f"sum_out must be [>= {rows}, {D}], got {tuple(sum_out.shape)}")
    lib = _lib.load()
    rc = lib.tj_add_ln_cast_f16(
        x.data_ptr(), _ptr(row_map), add16.data_ptr(), _ptr(row_count), rows, D, gamma.data_ptr(),
        beta.data_ptr(), float(eps), _ptr(sum_out), out.data_ptr(), _stream(x),
    )
    _lib.check(rc, "add_ln_cast_f16")
    return out


def add_ln_final_mask(x, add16, gamma, beta, eps=1e-5, inv_map=None, rows=None, out=None):
    """out[m] = LayerNorm(x[c] + add16[c]), c = inv_map[m] (zeros where c < 0)."""
    dev = x.device
    _require(x, "x", torch.float32, dev)
    _require(add16, "add16", torch.float16, dev)
    D = x.shape[-1]
    if add16.shape != x.shape:
        raise ValueError(f"add16 must match x {tuple(x.shape)}, got {tuple(add16.shape)}")
    if rows is None:
        rows = x.numel() // D if inv_map is None else inv_map.numel()
    if out is None:
        out = torch.empty(rows, D, dtype=torch.float32, device=dev)
    _require_out(out, "out", (rows, D), torch.float32, dev)
    lib = _lib.load()
    rc = lib.tj_add_ln_final_mask(
        x.data_ptr(), add16.data_ptr(), _ptr(inv_map), rows, D, gamma.data_ptr(), beta.data_ptr(),
        float(eps), out.data_ptr(), _stream(x),
    )
    _lib.check(rc, "add_ln_final_mask")
    return out


def add2_ln_final_mask(x, attn16, ffn16, gamma, beta, eps=1e-5, inv_map=None, x_at_original=False,
                       rows=None, out=None):
    """out[m] = LayerNorm((x[r] + attn16[c]) + ffn16[c]), c = inv_map[m], r = m if
    x_at_original else c (zeros where c < 0)."""
    dev = x.device
    _require(x, "x", torch.float32, dev)
    _require(attn16, "attn16", torch.float16, dev)
    _require(ffn16, "ffn16", torch.float16, dev)
    D = x.shape[-1]
    if attn16.shape != ffn16.shape or attn16.dim() != 2 or attn16.shape[1] != D:
        raise ValueError("attn16 and ffn16 must both be [compact_rows, D]")
    if rows is None:
        rows = x.numel() // D if inv_map is None else inv_map.numel()
    if x_at_original and (inv_map is None or x.numel() // D < rows):
        raise ValueError("x_at_original needs inv_map and x holding every output row")
    if out is None:
        out = torch.empty(rows, D, dtype=torch.float32, device=dev)
    _require_out(out, "out", (rows, D), torch.float32, dev)
    lib = _lib.load()
    rc = lib.tj_add2_ln_final_mask(
        x.data_ptr(), 1 if x_at_original else 0, attn16.data_ptr(), ffn16.data_ptr(), _ptr(inv_map), rows,
        D, gamma.data_ptr(), beta.data_ptr(), float(eps), out.data_ptr(), _stream(x),
    )
    _lib.check(rc, "add2_ln_final_mask")
    return out


def gemm_qkv_headmajor(a16, w_qkv16, b_qkv, num_heads, row_count=None, out=None):
    dev = a16.device
    _require(a16, "a16", torch.float16, dev)
    _require(w_qkv16, "w_qkv16", torch.float16, dev)
    _require(b_qkv, "b_qkv", torch.float32, dev)
    rows, D = a16.shape
    if w_qkv16.shape != (3 * D, D):
        raise ValueError(f"w_qkv16 must be [{3 * D}, {D}], got {tuple(w_qkv16.shape)}")
    if out is None:
        # head-major, each head zero-padded to head_pad(D // H) halves
        out = torch.empty(3, num_heads, rows, head_pad(D // num_heads), dtype=torch.float16, device=dev)
    _require_out(out, "out", (3, num_heads, rows, head_pad(D // num_heads)), torch.float16, dev)
    lib = _lib.load()
    rc = lib.tj_gemm_qkv_headmajor(
        a16.data_ptr(), w_qkv16.data_ptr(), b_qkv.data_ptr(), _ptr(row_count), rows, D, num_heads,
        out.data_ptr(), _stream(a16),
    )
    _lib.check(rc, "gemm_qkv_headmajor")
    return out


def gemm_bias_residual_f32(a16, w16, bias, resid, resid_map=None, row_count=None, out=None):
    dev = a16.device
    _require(a16, "a16", torch.float16, dev)
    _require(w16, "w16", torch.float16, dev)
    _require(bias, "bias", torch.float32, dev)
    _require(resid, "resid", torch.float32, dev)
    rows, K = a16.shape
    N = w16.shape[0]
    if w16.shape[1] != K:
        raise ValueError("w16 inner dimension does not match a16")
    if out is None:
        out = torch.empty(rows, N, dtype=torch.float32, device=dev)
    if out.dim() != 2 or out.shape[1] != N or out.shape[0] < (rows if row_count is None else 1):
        raise ValueError(f"out must be [rows, {N}], got {tuple(out.shape)}")
    _require(out, "out", torch.float32, dev)
    if resid.dim() != 2 or resid.shape[1] != N:
        raise ValueError(f"resid must be [rows, {N}], got {tuple(resid.shape)}")
    if resid_map is None and row_count is None and resid.shape[0] < rows:
        raise ValueError("resid has fewer rows than a16")
    lib = _lib.load()
    rc = lib.tj_gemm_bias_residual_f32(
        a16.data_ptr(), w16.data_ptr(), bias.data_ptr(), resid.data_ptr(), _ptr(resid_map),
        _ptr(row_count), rows, N, K, out.data_ptr(), _stream(a16),
    )
    _lib.check(rc, "gemm_bias_residual_f32")
    return out


def gemm_bias_f16(a16, w16, bias, row_count=None, out=None):
    """fp16 out = a16 @ w16^T + bias (the reference's fp16 F.linear)."""
    dev = a16.device
    _require(a16, "a16", torch.float16, dev)
    _require(w16, "w16", torch.float16, dev)
    _require(bias, "bias", torch.float32, dev)
    rows, K = a16.shape
    N = w16.shape[0]
    if w16.shape[1] != K:
        raise ValueError("w16 inner dimension does not match a16")
    if out is None:
        out = torch.empty(rows, N, dtype=torch.float16, device=dev)
    _require_out(out, "out", (rows, N), torch.float16, dev)
    lib = _lib.load()
    rc = lib.tj_gemm_bias_f16(
        a16.data_ptr(), w16.data_ptr(), bias.data_ptr(), _ptr(row_count), rows, N, K, out.data_ptr(),
        _stream(a16),
    )
    _lib.check(rc, "gemm_bias_f16")
    return out


def gemm_bias_gelu_f16(a16, w16, bias, row_count=None, out=None):
    dev = a16.device
    _require(a16, "a16", torch.float16, dev)
    _require(w16, "w16", torch.float16, dev)
    _require(bias, "bias", torch.float32, dev)
    rows, K = a16.shape
    N = w16.shape[0]
    if w16.shape[1] != K:
        raise ValueError("w16 inner dimension does not match a16")
    if out is None:
        out = torch.empty(rows, N, dtype=torch.float16, device=dev)
    _require_out(out, "out", (rows, N), torch.float16, dev)
    lib = _lib.load()
    rc = lib.tj_gemm_bias_gelu_f16(
        a16.data_ptr(), w16.data_ptr(), bias.data_ptr(), _ptr(row_count), rows, N, K,
        out.data_ptr(), _stream(a16),
    )
    _lib.check(rc, "gemm_bias_gelu_f16")
    return out


def flash_attn_fwd(q, k, v, q_cu, kv_off, kv_len, max_q_per_sample, scale, causal=False,
                   q_pos0=None, out=None, head_dim=64, part_o=None, part_lse=None, part_mode=0):
    """q: [H, q_rows, P]; k, v: [G, H, kv_rows, P] with P = head_pad(head_dim) (any strides
    with unit inner stride; rows hold head_dim values then zeros up to P); q_cu: [B+1];
    kv_off/kv_len: [B, G]
    int32.  Returns ctx [q_rows, H*head_dim] fp16.

    Split attention (tj_flash_attn_fwd_partial): part_mode 1 writes the partial
    result of these keys into part_o [q_rows, H*head_dim] fp32 and part_lse
    [q_rows, H] fp32 and returns None; part_mode 2 merges these keys with that
    partial into ctx."""
    dev = q.device
    _require(q, "q", torch.float16, dev)
    if k.dim() == 3:
        k = k.unsqueeze(0)
        v = v.unsqueeze(0)
    G, H, kv_rows, row = k.shape
    dh = head_dim
    P = head_pad(dh)
    if row != P or q.shape[0] != H or q.shape[2] != P:
        raise ValueError(f"q, k, v rows must be {P} halves (head dim {dh} zero-padded)")
    if k.stride() != v.stride() or k.stride(-1) != 1 or k.stride(-2) != P:
        raise ValueError(f"k and v must share strides with contiguous [rows, {P}] slabs")
    B = q_cu.numel() - 1
    if part_mode not in (0, 1, 2):
        raise ValueError(f"part_mode must be 0, 1 or 2, got {part_mode}")
    if part_mode:
        _require_out(part_o, "part_o", (q.shape[1], H * dh), torch.float32, dev)
        _require_out(part_lse, "part_lse", (q.shape[1], H), torch.float32, dev)
    if part_mode == 1:
        out = None
    elif out is None:
        out = torch.empty(q.shape[1], H * dh, dtype=torch.float16, device=dev)
    # out may be a column slice of a wider context (a head group's columns):
    # rows of H*head_dim contiguous halves at any row stride.
    if out is not None:
        if not isinstance(out, torch.Tensor) or out.dtype != torch.float16 or out.device != dev:
            raise TypeError(f"out must be a float16 tensor on {dev}")
        if tuple(out.shape) != (q.shape[1], H * dh) or out.stride(1) != 1 or out.stride(0) < H * dh:
            raise ValueError(f"out must be [{q.shape[1]}, {H * dh}] with contiguous rows, got "
                             f"{tuple(out.shape)} strides {out.stride()}")
    for name, t in (("q_cu", q_cu), ("kv_off", kv_off), ("kv_len", kv_len)):
        _require(t, name, torch.int32, dev)
    if kv_off.numel() != B * G or kv_len.numel() != B * G:
        raise ValueError(f"kv_off/kv_len must hold {B}x{G} entries")
    lib = _lib.load()
    rc = lib.tj_flash_attn_fwd_partial(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), H, dh, q.shape[1], kv_rows, k.stride(1),
        k.stride(0), G, B, max_q_per_sample, q_cu.data_ptr(), kv_off.data_ptr(),
        kv_len.data_ptr(), float(scale), 1 if causal else 0, _ptr(q_pos0), _ptr(out),
        0 if out is None else out.stride(0), _ptr(part_o), _ptr(part_lse), part_mode, _stream(q),
    )
    _lib.check(rc, "flash_attn_fwd")
    return out

"""Host <-> device transfers of a padded batch that move only the valid rows.

With a right-padded mask (the reference's padding: sample b holds L_b valid
tokens followed by padding, torch_transformer_benchmark.py:260-271), the
encoder never reads x at a padded position (the token plan drops those rows)
and writes exact zeros there (torch_transformer_benchmark.py:143-144,169-171).
So a serving loop that keeps its batches in host memory only has to move
each sample's first L_b rows over the host link in either direction:

* `upload_valid_rows` copies rows [0, L_b) of every sample of a pinned host x
  into the device x (the device rows past L_b keep whatever they held; the
  layer does not read them);
* `download_valid_rows` copies rows [0, L_b) of the device output into a
  pinned host output and writes the zero rows [L_b, S) on the host, so the
  host tensor equals the device output element for element.

Both issue one asynchronous copy per sample on the current CUDA stream.  The
zero fill runs on the calling CPU thread when `download_valid_rows` is
called, so no earlier copy into the same host rows may still be in flight
then (wait for the event of the previous transfer into that buffer first).
Masks that are not right-padded have no per-sample prefix; `valid_lengths`
returns None for them and the caller moves whole tensors instead.
"""
from __future__ import annotations

import torch


def valid_lengths(mask: torch.Tensor | None) -> list[int] | None:
    """Per-sample valid lengths of a right-padded bool mask [B, S] held on the
    host, or None when some row is not a prefix of ones (or mask is None)."""
    if mask is None:
        return None
    if mask.dim() != 2 or mask.dtype != torch.bool or mask.is_cuda:
        raise ValueError("valid_lengths: mask must be a bool [B, S] tensor in host memory")
    lengths = mask.sum(dim=1)
    pos = torch.arange(mask.shape[1]).unsqueeze(0)
    if not torch.equal(mask, pos < lengths.unsqueeze(1)):
        return None
    return [int(n) for n in lengths]


def _check(host: torch.Tensor, dev: torch.Tensor, lengths, what: str) -> None:
    if host.is_cuda or not dev.is_cuda:
        raise ValueError(f"{what}: expected a host tensor and a CUDA tensor")
    if host.shape != dev.shape or host.dtype != dev.dtype or host.dim() != 3:
        raise ValueError(f"{what}: host {tuple(host.shape)} {host.dtype} and device {tuple(dev.shape)} "
                         f"{dev.dtype} must be the same [B, S, D] shape and dtype")
    if not (host.is_contiguous() and dev.is_contiguous()):
        raise ValueError(f"{what}: tensors must be contiguous")
    if len(lengths) != host.shape[0] or any(n < 0 or n > host.shape[1] for n in lengths):
        raise ValueError(f"{what}: need {host.shape[0]} lengths in [0, {host.shape[1]}]")


def upload_valid_rows(x_host: torch.Tensor, x_dev: torch.Tensor, lengths) -> int:
    """Copies rows [0, lengths[b]) of each sample of x_host (pinned, [B, S, D])
    into x_dev on the current stream; returns the bytes copied."""
    _check(x_host, x_dev, lengths, "upload_valid_rows")
    row_bytes = x_host.shape[2] * x_host.element_size()
    total = 0
    for b, n in enumerate(lengths):
        if n:
            x_dev[b, :n].copy_(x_host[b, :n], non_blocking=True)
            total += n * row_bytes
    return total


def download_valid_rows(out_dev: torch.Tensor, out_host: torch.Tensor, lengths) -> int:
    """Copies rows [0, lengths[b]) of each sample of out_dev into out_host
    (pinned, [B, S, D]) on the current stream and zero-fills rows
    [lengths[b], S) of out_host on this thread; returns the bytes copied.
    The valid rows are in place once the stream reaches this point; the zero
    rows already are when the call returns."""
    _check(out_host, out_dev, lengths, "download_valid_rows")
    S = out_host.shape[1]
    row_bytes = out_host.shape[2] * out_host.element_size()
    total = 0
    for b, n in enumerate(lengths):
        if n:
            out_host[b, :n].copy_(out_dev[b, :n], non_blocking=True)
            total += n * row_bytes
        if n < S:
            out_host[b, n:].zero_()
    return total

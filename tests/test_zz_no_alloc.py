"""tj_encoder_forward_noalloc: the encoder forward without a caller workspace.

Some callers cannot allocate device memory where they run the encoder -- a
host binding the library through a thin FFI with no device allocator, or
serving code whose device memory is planned in advance (and cudaMalloc/cudaFree
may synchronise the device).  For them the library keeps a fixed static device
workspace.  This test calls that entry point through the C ABI twice in a row
and checks each result against the workspace entry point (tj_encoder_forward,
via the model) with the reference's strict gate, and that a shape too large
for the static workspace is refused with a clear error.

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _noalloc(lib, model, desc, x, mask, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tj_encoder_forward_noalloc(
        ctypes.byref(desc), model._layer_weights(x.device), model.final_norm.weight.data_ptr(),
        model.final_norm.bias.data_ptr(), x.data_ptr(),
        None if mask is None else mask.view(torch.uint8).data_ptr(), out.data_ptr(),
        ctypes.c_void_p(stream),
    )


def test_noalloc_matches_workspace_entry_point_twice(cuda_pkg):
    lib = cuda_pkg._lib.load()
    cfg = oracle.TransformerConfig(2, 256, 256, 4, 1024, 1, False)
    sd = oracle.make_state_dict(cfg, seed=1234)
    model = cuda_pkg.UserOptimizedTransformer(cuda_pkg.TransformerConfig(2, 256, 256, 4, 1024, 1, False))
    model.load_state_dict(sd, strict=True)
    model = model.to(DEV).eval()
    desc = cuda_pkg._lib.EncoderDesc(2, 256, 256, 4, 1024, 1, 0, 1e-5)
    assert lib.tj_encoder_workspace_bytes(ctypes.byref(desc)) <= (64 << 20)

    # Two calls in a row with different inputs and masks: the second must not
    # be affected by what the first left in the shared static workspace.
    for seed, pad in ((1234, 0.5), (4321, 0.9)):
        x, mask = oracle.generate_random_case(cfg, seed=seed, padding_ratio=pad)
        xd, md = x.to(DEV).contiguous(), mask.to(DEV).contiguous()
        with torch.inference_mode():
            expected = model(xd, md)
        out = torch.full_like(xd, float("nan"))
        rc = _noalloc(lib, model, desc, xd, md, out)
        assert rc == 0, cuda_pkg._lib.last_error()
        torch.cuda.synchronize()
        r = oracle.compare_outputs(expected.cpu(), out.cpu(), rtol=0.02, atol=0.002)
        assert r.passed, r
        assert torch.count_nonzero(out.cpu()[~mask]) == 0


def _near_bound_seq_len(cuda_pkg, lib, B, D, H, F, L):
    """Largest S (multiple of 64) whose workspace still fits the static array."""
    S = 64
    while True:
        desc = cuda_pkg._lib.EncoderDesc(B, S + 64, D, H, F, L, 0, 1e-5)
        if lib.tj_encoder_workspace_bytes(ctypes.byref(desc)) > (64 << 20):
            return S
        S += 64


@pytest.mark.parametrize("case", ["two_layers_causal", "near_the_bound"])
def test_noalloc_multi_layer_and_near_the_bound(cuda_pkg, case):
    """Every workspace buffer in use (two layers: x1, x2 and the last layer's
    FFN-out all live in the static array), and a shape whose workspace fills
    the array to within one 64-token step, where a layout error would first
    show: two calls in a row, each against tj_encoder_forward."""
    lib = cuda_pkg._lib.load()
    if case == "two_layers_causal":
        t = (2, 320, 256, 4, 1024, 2, True)
    else:
        t = (4, _near_bound_seq_len(cuda_pkg, lib, 4, 256, 4, 1024, 2), 256, 4, 1024, 2, False)
    cfg = oracle.TransformerConfig(*t)
    desc = cuda_pkg._lib.EncoderDesc(*t[:6], 1 if t[6] else 0, 1e-5)
    need = lib.tj_encoder_workspace_bytes(ctypes.byref(desc))
    assert 0 < need <= (64 << 20)
    if case == "near_the_bound":
        assert need > (64 << 20) - 4 * 64 * 8192  # within one 64-token step of the limit
    sd = oracle.make_state_dict(cfg, seed=77)
    model = cuda_pkg.UserOptimizedTransformer(cuda_pkg.TransformerConfig(*t))
    model.load_state_dict(sd, strict=True)
    model = model.to(DEV).eval()
    for seed, pad in ((77, 0.3), (78, 0.7)):
        x, mask = oracle.generate_random_case(cfg, seed=seed, padding_ratio=pad)
        xd, md = x.to(DEV).contiguous(), mask.to(DEV).contiguous()
        with torch.inference_mode():
            expected = model(xd, md)
        out = torch.full_like(xd, float("nan"))
        rc = _noalloc(lib, model, desc, xd, md, out)
        assert rc == 0, cuda_pkg._lib.last_error()
        torch.cuda.synchronize()
        r = oracle.compare_outputs(expected.cpu(), out.cpu(), rtol=0.02, atol=0.002)
        assert r.passed, (case, seed, r)
        assert torch.count_nonzero(out.cpu()[~mask]) == 0


def test_noalloc_rejects_shapes_beyond_the_static_workspace(cuda_pkg):
    lib = cuda_pkg._lib.load()
    desc = cuda_pkg._lib.EncoderDesc(8, 2048, 1024, 16, 4096, 1, 0, 1e-5)
    need = lib.tj_encoder_workspace_bytes(ctypes.byref(desc))
    assert need > (64 << 20)
    dummy = torch.zeros(1, device=DEV)
    arr = (cuda_pkg._lib.LayerWeights * 1)()
    rc = lib.tj_encoder_forward_noalloc(
        ctypes.byref(desc), arr, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None,
        dummy.data_ptr(), None,
    )
    assert rc == cuda_pkg._lib.TJ_ERR_WORKSPACE
    assert "static workspace" in cuda_pkg._lib.last_error()

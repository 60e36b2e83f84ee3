"""The fused small-model path of tj_encoder_forward (csrc/small_encoder.cu:
one CTA per sample through every layer, for S <= 128, d_model <= 128,
ffn_dim <= 128) on the B200: against the CPU FP32 oracle with the reference's
strict gate, and against the layer-by-layer path (tj_set_small_encoder(0)),
over head dims 4..128 (heads padded to 16 columns, several QKV head groups),
odd widths, padding (right-padded, non-prefix, a fully padded sample), no
mask, causal and several layers.  The reference's own small configurations
(tests/golden mask-path cases, the official 128-token shapes) also run this
path through the other GPU tests.
"""
from __future__ import annotations

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"

CASES = [
    # (B, S, D, H, F, layers, causal), padding ratio
    ((4, 128, 128, 4, 128, 4, True), 0.0),     # official shape #1 dims
    ((3, 100, 96, 3, 128, 2, False), 0.3),     # head dim 32, S < 128
    ((2, 128, 128, 1, 128, 1, True), 0.2),     # head dim 128 (one head)
    ((2, 128, 128, 2, 128, 2, False), 0.5),    # head dim 64
    ((2, 64, 32, 4, 32, 2, True), 0.0),        # head dim 8
    ((2, 128, 128, 16, 128, 1, False), 0.4),   # 16 heads of dim 8: two QKV head groups
    ((3, 37, 36, 4, 72, 2, False), 0.5),       # odd widths, head dim 9
    ((2, 1, 16, 4, 16, 1, False), 0.0),        # one token
    ((2, 32, 128, 4, 128, 4, True), 0.0),      # official shape #12 dims
]


def _model(pkg, cfg, sd):
    m = pkg.UserOptimizedTransformer(pkg.TransformerConfig(*cfg.__dict__.values()))
    m.load_state_dict(sd, strict=True)
    return m.to(DEV).eval()


def _forward(pkg, model, x, mask, fused):
    lib = pkg._lib.load()
    prev = lib.tj_set_small_encoder(1 if fused else 0)
    try:
        with torch.inference_mode():
            out = model(x.to(DEV), None if mask is None else mask.to(DEV))
        torch.cuda.synchronize()
    finally:
        lib.tj_set_small_encoder(prev)
    return out.cpu()


@pytest.fixture(autouse=True)
def _sync_check(cuda_pkg):
    prev = cuda_pkg._lib.set_sync_check(True)
    yield
    cuda_pkg._lib.set_sync_check(prev)


@pytest.mark.parametrize("cfg_t,pad", CASES, ids=[str(c[0]) for c in CASES])
def test_fused_small_encoder_against_oracle_and_layer_path(cuda_pkg, cfg_t, pad):
    cfg = oracle.TransformerConfig(*cfg_t)
    sd = oracle.make_state_dict(cfg, seed=41)
    x, mask = oracle.generate_random_case(cfg, seed=41, padding_ratio=pad)
    m = mask if pad > 0 else None
    model = _model(cuda_pkg, cfg, sd)
    fused = _forward(cuda_pkg, model, x, m, True)
    layered = _forward(cuda_pkg, model, x, m, False)
    ref = oracle.encoder_forward(sd, cfg, x, m)
    r = oracle.compare_outputs(ref, fused)
    assert r.passed, f"fused {cfg_t}: {r}"
    assert oracle.compare_outputs(ref, layered).passed
    assert float((fused - layered).abs().max()) < 2e-3
    if m is not None:
        assert torch.count_nonzero(fused[~m]) == 0


def test_fused_small_encoder_masks(cuda_pkg):
    """A fully padded sample (exact zeros, no NaN) and a non-prefix mask."""
    cfg = oracle.TransformerConfig(3, 96, 64, 2, 128, 2, False)
    sd = oracle.make_state_dict(cfg, seed=43)
    x, _ = oracle.generate_random_case(cfg, seed=43, padding_ratio=0.0)
    mask = torch.ones(3, 96, dtype=torch.bool)
    mask[1] = False
    mask[2, 1::3] = False
    model = _model(cuda_pkg, cfg, sd)
    out = _forward(cuda_pkg, model, x, mask, True)
    assert torch.isfinite(out).all()
    assert torch.count_nonzero(out[1]) == 0
    r = oracle.compare_outputs(oracle.encoder_forward(sd, cfg, x, mask), out)
    assert r.passed, r


def test_fused_small_encoder_is_deterministic_and_used(cuda_pkg):
    """Two runs give identical bits, and the fused path is the one that runs
    (its results differ from the layer path's in the last bits)."""
    cfg = oracle.TransformerConfig(8, 128, 128, 4, 128, 4, True)
    sd = oracle.make_state_dict(cfg, seed=47)
    x, _ = oracle.generate_random_case(cfg, seed=47, padding_ratio=0.0)
    model = _model(cuda_pkg, cfg, sd)
    a = _forward(cuda_pkg, model, x, None, True)
    b = _forward(cuda_pkg, model, x, None, True)
    c = _forward(cuda_pkg, model, x, None, False)
    assert torch.equal(a, b)
    assert not torch.equal(a, c)

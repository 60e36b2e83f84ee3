"""CPU checks of the C ABI and the host API (no kernel launches).

* the library loads and exports every entry point include/techjam_b200.h declares;
* argument validation fails with a status code and a message, not a crash;
* the Python model keeps the reference's parameter tree and strict state_dict
  (the contract of the reference's tests/test_state_dict.py:12-23).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

import oracle

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "techjam_b200.h"


def _declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TJ_API\s+[\w\s\*]+?\b(tj_\w+)\s*\(", text)))


def test_header_declares_and_binding_covers_all(pkg):
    names = _declared_symbols()
    assert len(names) >= 15
    assert sorted(pkg._lib.SIGNATURES) == names


def test_library_exports_every_symbol(pkg):
    lib = pkg._lib.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    assert lib.tj_abi_version() == 1


def test_argument_errors_are_reported_without_gpu(pkg):
    lib = pkg._lib.load()
    assert lib.tj_token_plan_ints(2, 8) == 2 + 3 * 2 + 2 * 16  # nv, cu, counts, orig, inv, order
    assert lib.tj_token_plan_ints(0, 8) == 0
    desc = pkg._lib.EncoderDesc(8, 2048, 1024, 16, 4096, 1, 0, 1e-5)
    need = lib.tj_encoder_workspace_bytes(ctypes.byref(desc))
    rows = 8 * 2048
    assert need >= rows * (1024 * 2 * 4 + 1024 * 4 * 2 + 4096 * 2)
    bad = pkg._lib.EncoderDesc(8, 2048, 1000, 16, 4096, 1, 0, 1e-5)  # D % H != 0
    assert lib.tj_encoder_workspace_bytes(ctypes.byref(bad)) == 0
    # Widths that are not multiples of 8: fp16 rows padded to 8 columns, so
    # the workspace is that of the padded widths (same plan and fp32 rows).
    odd = pkg._lib.EncoderDesc(2, 64, 100, 4, 200, 1, 0, 1e-5)
    pad = pkg._lib.EncoderDesc(2, 64, 104, 4, 200, 1, 0, 1e-5)
    n_odd = lib.tj_encoder_workspace_bytes(ctypes.byref(odd))
    n_pad = lib.tj_encoder_workspace_bytes(ctypes.byref(pad))
    assert 0 < n_odd <= n_pad
    rows = 2 * 64
    assert n_pad - n_odd <= 2 * rows * 4 * 4 + 4 * 256  # only the two fp32 row buffers differ (+ alignment)
    # Without a CUDA device every compute entry point refuses with a status code.
    rc = lib.tj_token_plan(None, 2, 8, None, None)
    assert rc != 0
    assert pkg._lib.last_error() != ""


def test_state_dict_matches_reference_layout(pkg):
    cfg = oracle.TransformerConfig(2, 8, 16, 4, 16, 2, True)
    sd = oracle.make_state_dict(cfg, seed=1234)
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(2, 8, 16, 4, 16, 2, True))
    model.load_state_dict({k: v.clone() for k, v in sd.items()}, strict=True)
    got = model.state_dict()
    assert tuple(got) == tuple(sd)
    for k in sd:
        assert torch.equal(got[k], sd[k]), k
    # fp16 caches are rebuilt on load and are not part of the state_dict
    att = model.layers[0].attention
    assert att._qkv_weight_mixed.dtype == torch.float16
    assert att._qkv_weight_mixed.shape == (48, 16)
    assert torch.equal(att._qkv_weight_mixed, torch.cat([sd["layers.0.attention.q_proj.weight"],
                                                         sd["layers.0.attention.k_proj.weight"],
                                                         sd["layers.0.attention.v_proj.weight"]]).half())


def test_same_seed_same_init_as_reference(pkg):
    """Constructing the model after torch.manual_seed(s) gives the reference's weights."""
    cfg = oracle.TransformerConfig(1, 4, 32, 2, 64, 2, False)
    sd = oracle.make_state_dict(cfg, seed=5)
    torch.manual_seed(5)
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(1, 4, 32, 2, 64, 2, False))
    for k, v in model.state_dict().items():
        assert torch.equal(v, sd[k]), k


def test_forward_refuses_cpu_and_training(pkg):
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(1, 4, 32, 2, 64, 1, False)).eval()
    with pytest.raises(ValueError, match="CUDA"):
        model(torch.zeros(1, 4, 32))
    with pytest.raises(TypeError):
        model(torch.zeros(1, 4, 32, dtype=torch.float64))
    model.train()
    with pytest.raises(RuntimeError, match="inference"):
        model(torch.zeros(1, 4, 32))


def test_config_validation_matches_reference(pkg):
    with pytest.raises(ValueError, match="divisible"):
        pkg.UserOptimizedTransformer(pkg.TransformerConfig(1, 4, 30, 4, 64, 1, False))
    with pytest.raises(ValueError):
        pkg.TransformerConfig(0, 4, 32, 2, 64, 1, False).validate()

"""Pins the oracle restatement (oracle/) to outputs of the real reference.

tests/golden/reference_outputs.pt was produced by tests/golden/make_golden.py,
which imports the reference's own torch_transformer_benchmark.py and
tools/shape14/accuracy.py.  CPU only.
"""
from __future__ import annotations

import hashlib

import pytest
import torch

import oracle


def _digest(tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().contiguous().cpu()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.numpy().tobytes())
    return h.hexdigest()


def _rebuild(entry):
    cfg = oracle.TransformerConfig(*entry["config"])
    sd = oracle.make_state_dict(cfg, seed=entry["seed"])
    if entry["ln_perturb_seed"] is not None:
        sd = oracle.perturb_layernorm(sd, entry["ln_perturb_seed"])
    x, mask = oracle.generate_random_case(cfg, seed=entry["seed"], padding_ratio=entry["padding_ratio"])
    return cfg, sd, x, mask


def test_full_cases_match_reference(golden):
    names = [n for n, e in golden.items() if e["kind"] == "full"]
    assert len(names) == 4
    for name in names:
        e = golden[name]
        cfg = oracle.TransformerConfig(*e["config"])
        out = oracle.encoder_forward(e["state_dict"], cfg, e["x"], e["mask"])
        torch.testing.assert_close(out, e["out"], rtol=0, atol=1e-6, msg=name)


@pytest.mark.parametrize(
    "name",
    [
        "cfg1_b2_s256_d256",
        "cfg1_trial1",
        "short_heavy_pad_b4_s128_d768",
        "dense_ln_b2_s512_d1024",
        "causal_two_layers_b2_s256",
        "no_padding_b2_s192_d128",
        "blocked_b1_s2048_d128",
    ],
)
def test_seeded_cases_match_reference(golden, name):
    e = golden[name]
    cfg, sd, x, mask = _rebuild(e)
    # The oracle's generators reproduce the reference's parameters and inputs bit for bit.
    assert _digest([sd[k] for k in sd]) == e["sd_sha256"], "parameter generator drifted"
    assert _digest([x]) == e["x_sha256"], "input generator drifted"
    assert torch.equal(mask, e["mask"])
    if e["blocked_query_chunk"]:
        out = oracle.encoder_forward_blocked(sd, cfg, x, mask, query_chunk=e["blocked_query_chunk"])
    else:
        out = oracle.encoder_forward(sd, cfg, x, mask)
    rows = out.reshape(-1, out.shape[-1]).double()
    torch.testing.assert_close(rows.sum(1), e["row_sum"], rtol=1e-6, atol=1e-4)
    torch.testing.assert_close((rows * rows).sum(1), e["row_sqsum"], rtol=1e-6, atol=1e-4)
    torch.testing.assert_close(out.reshape(-1, out.shape[-1])[:, :16], e["head"], rtol=0, atol=1e-5)
    if "out" in e:
        torch.testing.assert_close(out, e["out"], rtol=0, atol=1e-5)
    # Padded rows are exact zeros (torch_transformer_benchmark.py:169-171).
    flat_mask = mask.reshape(-1)
    assert torch.count_nonzero(out.reshape(-1, out.shape[-1])[~flat_mask]) == 0


def test_blocked_equals_dense_oracle():
    cfg = oracle.TransformerConfig(2, 320, 128, 2, 256, 1, False)
    sd = oracle.make_state_dict(cfg, seed=3)
    x, mask = oracle.generate_random_case(cfg, seed=3, padding_ratio=0.4)
    dense = oracle.encoder_forward(sd, cfg, x, mask)
    blocked = oracle.encoder_forward_blocked(sd, cfg, x, mask, query_chunk=64)
    torch.testing.assert_close(dense, blocked, rtol=0, atol=2e-5)


def test_query_row_oracle_matches_reference_blocked_outputs(golden):
    """The query-row oracle (the long-sequence checker) on the reference's own
    memory-bounded case: its rows match the reference's stored row sums,
    sums of squares and first 16 features at those rows."""
    e = golden["blocked_b1_s2048_d128"]
    cfg, sd, x, mask = _rebuild(e)
    rows = oracle.long_sequence_check_rows(int(mask.sum()), cfg.seq_len)
    assert rows.numel() == 3 * 256 + 1  # three blocks + the first padded row
    out = oracle.encoder_forward_query_rows(sd, cfg, x, mask, rows).double()
    torch.testing.assert_close(out.sum(1), e["row_sum"][rows], rtol=1e-6, atol=1e-4)
    torch.testing.assert_close((out * out).sum(1), e["row_sqsum"][rows], rtol=1e-6, atol=1e-4)
    torch.testing.assert_close(out[:, :16].float(), e["head"][rows], rtol=0, atol=1e-5)


@pytest.mark.parametrize("cfg_t,pad", [((1, 1500, 96, 3, 192, 1, True), 0.2),
                                       ((1, 1024, 64, 2, 128, 1, False), 0.0),
                                       ((1, 700, 40, 4, 80, 1, False), 0.6)])
def test_query_row_oracle_equals_blocked_oracle(cfg_t, pad):
    cfg = oracle.TransformerConfig(*cfg_t)
    sd = oracle.make_state_dict(cfg, seed=11)
    x, mask = oracle.generate_random_case(cfg, seed=11, padding_ratio=pad)
    m = mask if pad > 0 else None
    full = oracle.encoder_forward_blocked(sd, cfg, x, m, query_chunk=128)[0]
    rows = oracle.long_sequence_check_rows(int(mask.sum()), cfg.seq_len, block=100)
    sub = oracle.encoder_forward_query_rows(sd, cfg, x, m, rows)
    torch.testing.assert_close(sub, full[rows], rtol=0, atol=1e-5)
    with pytest.raises(ValueError):
        oracle.encoder_forward_query_rows(sd, oracle.TransformerConfig(1, 10, 40, 4, 80, 2, False), x, m, rows)


def test_comparator_is_strict_or():
    ref = torch.tensor([0.01, 0.0, 100.0, float("nan")])
    # abs 0.0025 and rel 25% fail; abs 0.0019 passes; rel 1.9% of 100 passes; NaN fails.
    opt = torch.tensor([0.0125, 0.0019, 101.9, float("nan")])
    r = oracle.compare_outputs(ref, opt)
    assert r.failed_elements == 2
    assert not r.passed
    s = oracle.StreamingAccuracy()
    oracle.update_accuracy(s, ref.view(1, 4, 1), opt.view(1, 4, 1), token_chunk=3)
    assert s.failed == 2 and s.total == 4

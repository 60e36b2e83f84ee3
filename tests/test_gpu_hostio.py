"""Valid-row host transfers (techjam_b200.hostio) on the B200: a batch whose
valid rows alone were uploaded (padded device rows hold NaN) gives the same
output as the whole batch, and the downloaded host output with its
host-written zero rows equals the device output bit for bit."""
from __future__ import annotations

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_valid_row_round_trip_matches_whole_tensors(cuda_pkg):
    pkg = cuda_pkg
    cfg = oracle.TransformerConfig(6, 384, 256, 4, 1024, 2, False)
    sd = oracle.make_state_dict(cfg, seed=77)
    x, mask = oracle.generate_random_case(cfg, seed=77, padding_ratio=0.8)
    mask[3] = False  # one sample without valid tokens
    x[3] = 0.0
    model = pkg.UserOptimizedTransformer(pkg.TransformerConfig(*cfg.__dict__.values()))
    model.load_state_dict(sd, strict=True)
    model = model.cuda().eval()
    lengths = pkg.hostio.valid_lengths(mask)
    assert lengths is not None and lengths[3] == 0
    x_host = x.pin_memory()
    out_host = torch.full_like(x, float("nan")).pin_memory()
    x_dev = torch.full_like(x, float("nan"), device="cuda")
    with torch.inference_mode():
        up = pkg.hostio.upload_valid_rows(x_host, x_dev, lengths)
        out_dev = model(x_dev, mask.cuda())
        down = pkg.hostio.download_valid_rows(out_dev, out_host, lengths)
        torch.cuda.synchronize()
        ref = model(x.cuda(), mask.cuda())
    torch.cuda.synchronize()
    assert up == down == sum(lengths) * cfg.d_model * 4
    assert torch.equal(out_host, out_dev.cpu())
    assert torch.equal(out_host, ref.cpu())
    assert torch.count_nonzero(out_host[~mask]) == 0

"""Host-side logic of techjam_b200.hostio (valid-row transfers): the mask
prefix lengths and the argument checks; the copies themselves run in
tests/test_gpu_hostio.py."""
from __future__ import annotations

import pytest
import torch


def test_valid_lengths_prefix_and_not(pkg):
    h = pkg.hostio
    mask = torch.zeros(3, 8, dtype=torch.bool)
    mask[0, :8] = True
    mask[1, :3] = True
    assert h.valid_lengths(mask) == [8, 3, 0]
    mask[2, 5] = True  # not a prefix
    assert h.valid_lengths(mask) is None
    assert h.valid_lengths(None) is None
    with pytest.raises(ValueError):
        h.valid_lengths(mask.int())


def test_transfer_argument_checks(pkg):
    h = pkg.hostio
    x = torch.zeros(2, 4, 8)
    with pytest.raises(ValueError):
        h.upload_valid_rows(x, x, [4, 4])  # no CUDA tensor
    with pytest.raises(ValueError):
        h.download_valid_rows(x, x, [1])

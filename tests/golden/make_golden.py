"""Generates tests/golden/reference_outputs.pt from the REAL reference.

Run in a container that has the reference repository checked out (read-only
is fine):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference's own FP32 model, input generator and memory-bounded
oracle (torch_transformer_benchmark.py, tools/shape14/accuracy.py), runs them
on CPU in FP32, and stores their outputs.  The oracle restatement in oracle/
is then pinned against these fixtures by tests/test_oracle_golden.py; the GPU
parity tests use them as the ground truth for the cases they cover.

Small cases store inputs, parameters and outputs in full.  Larger cases store
SHA-256 digests of the parameters and inputs (so the oracle's own generator
must reproduce them exactly), the padded mask, and for every output row its
float64 sum and sum of squares plus its first 16 features.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_outputs.pt"
HEAD = 16


def digest(tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().contiguous().cpu()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.numpy().tobytes())
    return h.hexdigest()


def row_stats(out: torch.Tensor):
    rows = out.reshape(-1, out.shape[-1]).double()
    return {
        "row_sum": rows.sum(dim=1),
        "row_sqsum": (rows * rows).sum(dim=1),
        "head": out.reshape(-1, out.shape[-1])[:, :HEAD].clone(),
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference repository checkout")
    args = ap.parse_args()
    ref_root = Path(args.reference)
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(HERE.parents[1]))
    import torch_transformer_benchmark as bench  # the reference's own module
    from tools.shape14.accuracy import memory_bounded_baseline  # reference

    from oracle.encoder_oracle import perturb_layernorm  # LN distribution of the GPU configs

    torch.set_num_threads(max(1, torch.get_num_threads()))
    cases = {}

    # 1) The reference's own parity-test setup (tests/test_mask_paths.py:12-42):
    #    config (2, 8, 16, 4, 16, 2, causal), seed 1234, fixed right-padded mask.
    fixed_mask = torch.tensor(
        [
            [True, True, True, True, True, False, False, False],
            [True, True, True, False, False, False, False, False],
        ]
    )
    for causal in (False, True):
        for use_mask in (False, True):
            torch.manual_seed(1234)
            config = bench.TransformerConfig(2, 8, 16, 4, 16, 2, causal)
            baseline = bench.BaselineTransformer(config).eval()
            x = torch.randn(2, 8, 16)
            mask = None
            if use_mask:
                mask = fixed_mask.clone()
                x = x.masked_fill(~mask[..., None], 0)
            with torch.inference_mode():
                out = baseline(x, mask)
            cases[f"mask_paths_causal{int(causal)}_mask{int(use_mask)}"] = {
                "kind": "full",
                "config": tuple(config.__dict__.values()),
                "state_dict": {k: v.clone() for k, v in baseline.state_dict().items()},
                "x": x.clone(),
                "mask": None if mask is None else mask.clone(),
                "out": out.clone(),
            }

    # 2) Seeded cases rebuilt by the oracle's generator (weights from
    #    torch.manual_seed(seed) + default init, inputs from generate_random_case).
    seeded = [
        # name, (B, S, D, H, F, L, causal), seed, padding_ratio, ln_perturb_seed, blocked
        ("cfg1_b2_s256_d256", (2, 256, 256, 4, 1024, 1, False), 1234, 0.5, None, None),
        ("cfg1_trial1", (2, 256, 256, 4, 1024, 1, False), 1235, 0.5, None, None),
        ("short_heavy_pad_b4_s128_d768", (4, 128, 768, 12, 3072, 1, False), 1234, 0.999, None, None),
        ("dense_ln_b2_s512_d1024", (2, 512, 1024, 16, 4096, 1, False), 1234, 0.5, 4321, None),
        ("causal_two_layers_b2_s256", (2, 256, 256, 4, 1024, 2, True), 77, 0.5, None, None),
        ("no_padding_b2_s192_d128", (2, 192, 128, 2, 512, 1, False), 5, 0.0, None, None),
        ("blocked_b1_s2048_d128", (1, 2048, 128, 2, 256, 1, False), 99, 0.1, None, 256),
    ]
    for name, cfg, seed, pad, ln_seed, blocked in seeded:
        config = bench.TransformerConfig(*cfg)
        torch.manual_seed(seed)
        baseline = bench.BaselineTransformer(config).eval()
        sd = {k: v.clone() for k, v in baseline.state_dict().items()}
        if ln_seed is not None:
            sd = perturb_layernorm(sd, ln_seed)
            baseline.load_state_dict(sd, strict=True)
        x, mask = bench.generate_random_case(
            config=config, device=torch.device("cpu"), dtype=torch.float32, seed=seed,
            padding_ratio=pad, input_scale=1.0,
        )
        with torch.inference_mode():
            if blocked:
                out = memory_bounded_baseline(baseline, x, mask, query_chunk=blocked)
                dense = baseline(x, mask)
            else:
                out = baseline(x, mask)
                dense = None
        entry = {
            "kind": "seeded",
            "config": cfg,
            "seed": seed,
            "padding_ratio": pad,
            "ln_perturb_seed": ln_seed,
            "blocked_query_chunk": blocked,
            "sd_sha256": digest([sd[k] for k in sd]),
            "x_sha256": digest([x]),
            "mask": mask.clone(),
            **row_stats(out),
        }
        if dense is not None:
            entry["dense_max_abs_diff"] = float((dense - out).abs().max())
        if cfg == (2, 256, 256, 4, 1024, 1, False) and seed == 1234:
            entry["out"] = out.clone()  # full output of the CPU plumbing config
        cases[name] = entry
        print(f"{name}: out sum {float(out.double().sum()):.6f}")

    torch.save({"torch_version": str(torch.__version__), "cases": cases}, OUT)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()

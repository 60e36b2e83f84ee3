"""Test infrastructure: CPU FP32 restatement of the reference encoder layer.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker.  The product path
(techjam-2026-track3_b200) never imports it.
"""
from .encoder_oracle import (  # noqa: F401
    AccuracyResult,
    StreamingAccuracy,
    TransformerConfig,
    compare_outputs,
    encoder_forward,
    encoder_forward_blocked,
    encoder_forward_query_rows,
    generate_random_case,
    long_sequence_check_rows,
    make_state_dict,
    perturb_layernorm,
    update_accuracy,
)

"""B200-native (sm_100a) Transformer encoder layer, a drop-in for
`v16_1_clean.UserOptimizedTransformer` of wheres-my-perry/techjam-2026-track3.

The directory name is not a Python identifier; load it with
`load_package()` from any of the repository entry points, which registers it
as the importable module `techjam_b200`.
"""
from .model import TransformerConfig, UserOptimizedTransformer  # noqa: F401
from . import hostio, kernels  # noqa: F401

__all__ = ["TransformerConfig", "UserOptimizedTransformer", "hostio", "kernels"]

"""B200-native CCQ cleaning operator (sm_100a CUDA behind a C ABI; see include/ccq_b200.h)."""
from .ops import (  # noqa: F401
    FusedCCQCleanGated,
    FusedCCQCleanRead,
    FusedCCQCleanReadL2Norm,
    ccq_gate_lambda,
    decode_step,
    decode_step_l2norm,
    fused_ccq_clean,
    fused_ccq_clean_gated,
    fused_ccq_clean_read,
    fused_ccq_clean_read_l2norm,
    l2norm,
    reduce_lambda_grad,
    reshape_lambda_3d,
)
from ._lib import CCQError, last_launch_count, last_path  # noqa: F401

__version__ = '0.1.0'

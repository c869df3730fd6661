"""quant_2bit_b200 -- B200-native BCJR forward-backward for QTIP trellis QAT.

Drop-in for the BCJR hot path of Venugopalan2610/quant-2bit (src/bcjr):
the autograd Function, its eager-compatible wrapper and the caller-side
quantizer helpers, running hand-written sm_100a kernels through the C ABI of
libbcjr_b200.so (include/bcjr_b200.h).
"""
from .bcjr import (  # noqa: F401
    K_BITS,
    L_BITS,
    V_DIM,
    BcjrForwardBackwardMonolithic,
    bcjr_forward_backward,
    bcjr_forward_backward_monolithic,
    bcjr_soft_backward,
    bcjr_soft_forward,
    build_pred_succ_tables,
)

__version__ = "0.1.0"

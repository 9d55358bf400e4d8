"""orthossm_b200 — B200-native (sm_100a) OrthoSSM Cheby-RKV hot path.

Public API mirrors the reference's ``sdpc_kernel`` op surface; see
``orthossm_b200.sdpc_kernel``.  Kernels live in ``csrc/`` behind the C ABI of
``include/orthossm_b200.h``; ``python -m orthossm_b200.build`` builds it.
"""
from .sdpc_kernel import (  # noqa: F401
    BASELINE_LAMBDA, LUT_TABLE_SIZE, MAX_DEGREE, MULTI_SCALE_LAMBDA, FusedChebyRKVv10,
    GatedComplexityPredictor, apply_cheby_rkv_core, apply_cheby_rkv_v10, cheby_ema_forward,
    cheby_ema_forward_host, cheby_ema_forward_seqpar, cheby_ema_forward_shards_local, exchange_shard_totals, fold_shard_carries, forward_path, gate_decay,
    get_chebyshev_lut,
    init_chebyshev_coefficients, ttt_wpred_adam, workspace_status,
)

from .state import ChebyStreamState, StreamingChebyRKV  # noqa: F401

__version__ = "0.1.0"

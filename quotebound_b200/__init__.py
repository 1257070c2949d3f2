"""quotebound_b200 — quotebound's Gated DeltaNet recurrence (forward and backward) on B200.

The compute lives in libqb_gdn.so (C ABI, include/qb_gdn.h); this package is the host-side mirror of
the reference's entry points plus the multi-GPU partitioner.
"""
from ._lib import QbError, version  # noqa: F401
from .deltanet import (gated_delta, gated_delta_bwd, gated_delta_fwd, gated_delta_trainable,  # noqa: F401
                       gated_delta_vjp)
from .exact import keep_rows, step, verify  # noqa: F401
from .gate import gate_bwd, gate_fwd  # noqa: F401

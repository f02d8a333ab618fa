"""The oracle: a CPU restatement of dyn-quant's split GEMV path.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() and
by bench.py's CPU-baseline and reference legs, always as the checker or the
timed CPU baseline.  The product (include/dq_abi.h and the dyn_quant package)
never imports it.
"""
from .oracle import *  # noqa: F401,F403

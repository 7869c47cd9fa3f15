"""CPU oracle for the W4A16 MoE expert path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (``qwen-ascend_b200/``) imports this package.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may use it,
and only as the checker or the timed CPU baseline, never as the measured GPU path.

The oracle restates the reference's algorithm (``fnx/engine.py`` ``_moe`` and the
quantised containers, the ``kernels/*`` rounding sequences and the
``fnx/w4gemv_op.py`` contract) in torch-CPU / numpy code.  It is pinned against
golden vectors produced by importing the reference's own Python code in the build
container (``tests/golden/make_golden.py``); see ``tests/test_oracle_golden.py``.
"""
from .moe_oracle import *  # noqa: F401,F403

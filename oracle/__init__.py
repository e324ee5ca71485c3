"""CPU oracle for the DeltaAttention prefill/decode hot path.

TEST INFRASTRUCTURE ONLY. This package is a plain numpy / torch-CPU restatement of
the reference's Triton kernels and their PyTorch glue. It is imported only by
``tests/``, by ``__graft_entry__.smoke()`` (as the checker) and by ``bench.py``'s
CPU-baseline leg and ``--impl reference`` arm. The product path
(``deltaattention_b200``) never imports it and has no CPU fallback.

Pinning: the restatement is checked against golden vectors produced by running the
reference's own kernels under ``TRITON_INTERPRET=1`` in the build container
(``tests/golden/gen_golden.py``). The interpreter is valid for fp32 and fp16 data; it
computes bf16 arithmetic on raw uint16 bit patterns, so bf16 is pinned by sharing the
fp16 code path with bf16 rounding (see ``delta_oracle.round_to``).
"""
from .delta_oracle import *  # noqa: F401,F403

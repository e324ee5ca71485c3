"""Drop-in for the reference's deltaFlashAttention.py (two-phase count-weighted attention).

``hybrid_compressed_flash_kernel`` (deltaFlashAttention.py:9-146),
``hybrid_compressed_flash_kernel_sanity`` (:149-259) and ``pure_phase1_flash_kernel``
(:262-357) keep their launch syntax and argument lists (the wrappers at
modeling_llama.py:306-451 call them unchanged); bf16/fp16 inputs with head_dim 64/128 run
on the tcgen05 kernel, other shapes on the CUDA-core kernel.
"""
from deltaattention_b200.launch import (  # noqa: F401
    hybrid_compressed_flash_kernel,
    hybrid_compressed_flash_kernel_sanity,
    pure_phase1_flash_kernel,
)

__all__ = ["hybrid_compressed_flash_kernel", "hybrid_compressed_flash_kernel_sanity", "pure_phase1_flash_kernel"]

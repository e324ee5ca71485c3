"""Drop-in for the reference's tritonModules.py (anchor selection and packing kernels).

``chunked_eval_kernel`` (tritonModules.py:7-69) and ``parallel_scatter_pack_kv_kernel``
(tritonModules.py:72-132) keep their Triton launch syntax and argument lists; they run
the sm_100a kernels of deltaattention_b200. ``triton`` stays importable for callers that
use ``triton.next_power_of_2`` / ``triton.cdiv`` (modeling_llama.py:635,664).
"""
import triton  # noqa: F401  (callers reach triton helpers through this module's namespace)

from deltaattention_b200.launch import chunked_eval_kernel, parallel_scatter_pack_kv_kernel  # noqa: F401

__all__ = ["chunked_eval_kernel", "parallel_scatter_pack_kv_kernel"]

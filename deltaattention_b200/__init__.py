"""B200-native (sm_100a) DeltaAttention hot path.

* ``deltaattention_b200.launch`` - the reference's kernels with their Triton launch syntax
  (``kernel[grid](...)``), backed by hand-written CUDA;
* ``deltaattention_b200.dropin`` - drop-in modules under the reference's module names
  (tritonModules, deltaFlashAttention, flashAttention, deltaDecoding, nmDeltaFlashAttention);
* ``deltaattention_b200.ops`` - the native fused path (RoPE, packing, GQA by index);
* ``include/deltaattn_b200.h`` - the C ABI all of them call.
"""
__version__ = "0.1.0"

from . import _lib  # noqa: F401


def library_path() -> str:
    return _lib.LIB_PATH

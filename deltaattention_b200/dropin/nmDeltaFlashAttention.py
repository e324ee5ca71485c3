"""N:M structured delta attention (module name of the reference's nmDeltaFlashAttention).

The reference ships this module only as compiled bytecode (``delta_type = "nm"``,
globVR.py:66), so its semantics are specified here: selection is N:M structured over
candidate positions t % stride == 0 with stride = ratio * n / m, keeping in every run of
m candidates the n whose key moved most since the previous candidate (fp32 squared
distance; position 0 always kept). The result packs into the reference's format (anchor
timestamps, run-length counts) and runs the reference's two-phase attention, so the
compression ratio is exactly ``ratio`` and every head has the same packed length.
"""
import torch

from deltaattention_b200 import _lib as L
from deltaattention_b200 import ops


def nm_stride(n: int, m: int, ratio: int) -> int:
    if (ratio * n) % m:
        raise ValueError("ratio * n / m must be an integer")
    c = ratio * n // m
    if c < 1:
        raise ValueError("ratio * n / m must be >= 1")
    return c


def nm_num_packed(seq_len: int, n: int = 2, m: int = 4, ratio: int = 4) -> int:
    return int(L.load().dab_nm_num_packed(seq_len, n, m, nm_stride(n, m, ratio)))


def nm_keep_mask(key_states: torch.Tensor, n: int = 2, m: int = 4, ratio: int = 4) -> torch.Tensor:
    """Keep mask [B, H, N] int32 of post-RoPE keys [B, H, N, d] (any strides)."""
    L.require_cuda(key_states)
    B, H, N, D = key_states.shape
    keep = torch.empty((B, H, N), dtype=torch.int32, device=key_states.device)
    st = L.stream_of(key_states)
    L.check(L.load().dab_nm_select(L.ptr(key_states), L.strides(key_states.stride()), L.ptr(keep),
                                   L.strides(keep.stride()), L.dtype_code(key_states), B, H, N, D, n, m,
                                   nm_stride(n, m, ratio), st), "nm_keep_mask")
    return keep


def nm_delta_flash_attention(q_rot, k_rot, v, n: int = 2, m: int = 4, ratio: int = 4, dense_window: int = 128,
                             sm_scale=None, out=None, return_packed=False):
    """N:M selection + packing + two-phase attention on post-RoPE q / k (GQA by index)."""
    keep = nm_keep_mask(k_rot, n, m, ratio)
    packed = ops.pack_from_keep(k_rot, v, keep, num_packed=nm_num_packed(k_rot.shape[2], n, m, ratio))
    o = ops.attention(q_rot, k_rot, v, packed, sm_scale=sm_scale, dense_window=dense_window, out=out)
    return (o, packed) if return_packed else o


__all__ = ["nm_keep_mask", "nm_num_packed", "nm_delta_flash_attention", "nm_stride"]

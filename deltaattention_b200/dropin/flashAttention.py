"""Drop-in for the reference's flashAttention.py (dense causal flash attention).

``_attn_fwd_flat`` (flashAttention.py:5-91) keeps its launch syntax;
``triton_flash_attention`` (flashAttention.py:94-130) keeps its call signature and
behaviour: contiguous inputs, ``sm_scale`` defaulting to head_dim**-0.5, 128x128 blocks.
"""
import torch

from deltaattention_b200.launch import _attn_fwd_flat  # noqa: F401


def triton_flash_attention(q, k, v, causal=True, sm_scale=None):
    batch_size, num_heads, q_len, head_dim = q.shape
    q = q.contiguous()
    k = k.contiguous()
    v = v.contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / (head_dim ** 0.5)
    out = torch.empty_like(q)
    grid = ((q_len + 127) // 128, batch_size * num_heads, 1)
    _attn_fwd_flat[grid](
        q, k, v, sm_scale, out,
        q.stride(0), q.stride(1), q.stride(2), q.stride(3),
        k.stride(0), k.stride(1), k.stride(2), k.stride(3),
        v.stride(0), v.stride(1), v.stride(2), v.stride(3),
        out.stride(0), out.stride(1), out.stride(2), out.stride(3),
        batch_size, num_heads, q_len,
        HEAD_DIM=head_dim, BLOCK_M=128, BLOCK_N=128, IS_CAUSAL=causal,
    )
    return out


__all__ = ["_attn_fwd_flat", "triton_flash_attention"]

"""Seeded synthetic inputs with the BASELINE configurations' distributions.

No dataset or checkpoint is available, so the benchmark and the tests draw layer inputs:
queries / values are normal (scaled), keys follow an AR(1) process along the sequence,
k_t = 0.95 k_{t-1} + 0.31 eps_t with k_0 ~ N(0, 1), optionally plus a constant per
(head, channel) offset ~ N(0, 1). Tensors come out in the projection layout
[B, N, H, d] viewed as [B, H, N, d] (the layout modeling_llama.py:550-552 produces).
"""
from __future__ import annotations

import torch


def ar1(shape_bhnd, gen, device, coef=0.95, noise=0.31, block=256):
    """AR(1) along dim 2 of a [B, H, N, d] tensor, fp32, computed blockwise on `device`."""
    B, H, N, D = shape_bhnd
    eps = torch.randn((N, B * H * D), generator=gen, device=device, dtype=torch.float32)
    innov = eps * noise
    innov[0] = eps[0]  # k_0 ~ N(0, 1)
    T = min(block, N)
    i = torch.arange(T, device=device, dtype=torch.float32)
    decay = torch.where(i[:, None] >= i[None, :], coef ** (i[:, None] - i[None, :]), torch.zeros((), device=device))
    pw = coef ** (i + 1)
    out = torch.empty_like(innov)
    carry = torch.zeros((B * H * D,), device=device, dtype=torch.float32)
    for t0 in range(0, N, T):
        t1 = min(t0 + T, N)
        n = t1 - t0
        y = decay[:n, :n] @ innov[t0:t1] + pw[:n, None] * carry[None, :]
        out[t0:t1] = y
        carry = y[-1]
    return out.view(N, B, H, D).permute(1, 2, 0, 3)


def rope_tables(N, D, theta, dtype, device="cpu"):
    """cos / sin [1, N, d] by the reference's formula (modeling_llama.py:160-170)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
    pos = torch.arange(N, dtype=torch.int64).float()
    freqs = (inv_freq[None, :, None] @ pos[None, None, :]).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype).to(device), emb.sin().to(dtype).to(device)


def layer_inputs(B, Hq, Hkv, N, D, dtype, seed=0, device="cuda", qv_scale=0.5, key_offset=True):
    """Pre-RoPE q, k and v in projection layout (viewed [B, H, N, d]) for one layer."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q = torch.randn((B, N, Hq, D), generator=g, device=device, dtype=torch.float32) * qv_scale
    v = torch.randn((B, N, Hkv, D), generator=g, device=device, dtype=torch.float32) * qv_scale
    k = ar1((B, Hkv, N, D), g, device)
    if key_offset:
        k = k + torch.randn((B, Hkv, 1, D), generator=g, device=device, dtype=torch.float32)
    kb = torch.empty((B, N, Hkv, D), dtype=dtype, device=device)
    kb.copy_(k.transpose(1, 2))
    return (q.to(dtype).transpose(1, 2), kb.transpose(1, 2), v.to(dtype).transpose(1, 2))


CONFIGS = {
    # fp32, MHA, N=2048, d=64, theta 1e4, N(0,1) q/v, plain AR(1) keys
    "cfg1": dict(B=1, Hq=8, Hkv=8, N=2048, D=64, dtype=torch.float32, theta=1e4, qv_scale=1.0, key_offset=False,
                 r=4),
    # Llama-3.1-8B layer, bf16, N=32k, r=4, theta 5e5
    "cfg2": dict(B=1, Hq=32, Hkv=8, N=32768, D=128, dtype=torch.bfloat16, theta=5e5, qv_scale=0.5, key_offset=True,
                 r=4),
}

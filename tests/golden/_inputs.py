"""Deterministic inputs for the golden fixtures (numpy PCG64, seeded).

Shared by ``gen_golden.py`` (which runs the reference) and the tests (which replay the
same inputs through the oracle and the CUDA kernels). Distributions follow the
keys are an AR(1) process along the sequence
(k_t = 0.95 k_{t-1} + 0.31 eps_t) with RoPE applied, queries/values are normal.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle import delta_oracle as O  # noqa: E402


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def normal(shape, seed, scale=1.0):
    return (rng(seed).standard_normal(shape) * scale).astype(np.float32)


def ar1_keys(B, H, N, D, seed, offset=False):
    g = rng(seed)
    eps = g.standard_normal((B, H, N, D))
    k = np.empty((B, H, N, D), dtype=np.float64)
    k[:, :, 0] = eps[:, :, 0]
    for t in range(1, N):
        k[:, :, t] = 0.95 * k[:, :, t - 1] + 0.31 * eps[:, :, t]
    if offset:
        k += g.standard_normal((B, H, 1, D))
    return k.astype(np.float32)


def cos_sin(N, D, theta, dtype):
    return O.rope_cos_sin(N, D, theta, dtype)


def post_rope_keys(B, H, N, D, theta, dtype, seed, offset=False):
    k = torch.from_numpy(ar1_keys(B, H, N, D, seed, offset)).to(dtype)
    cos, sin = cos_sin(N, D, theta, dtype)
    return O.apply_rope(k, cos, sin).contiguous()


def median_threshold(k, use_cos):
    """Kernel threshold argument that keeps roughly half the tokens."""
    kk = k.float().numpy()
    a, b = kk[:, :, 1:], kk[:, :, :-1]
    if use_cos:
        c = (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1) + 1e-8)
        return float(np.median(c))
    return float(np.median(((a - b) ** 2).sum(-1)))


def attn_inputs(B, H, N, D, dtype, seed):
    scale = 1.0 if dtype == torch.float32 else 0.5
    q = torch.from_numpy(normal((B, H, N, D), seed, scale)).to(dtype)
    k = post_rope_keys(B, H, N, D, 1e4, dtype, seed + 1000)
    v = torch.from_numpy(normal((B, H, N, D), seed + 2000, scale)).to(dtype)
    return q, k, v


def hetero_keep(B, H, N, seed):
    """Head h keeps each position with probability 1/2**(1+2h); position 0 always."""
    g = rng(seed + 5000)
    keep = np.zeros((B, H, N), dtype=np.int32)
    for h in range(H):
        p = 1.0 / (2 ** (1 + 2 * h))
        keep[:, h] = (g.random((B, N)) < p).astype(np.int32)
    keep[:, :, 0] = 1
    return torch.from_numpy(keep)


def decode_setup(dtype, seed):
    """A prefilled hybrid cache plus ``steps`` new tokens (deltaDecoding.py layout).

    Lengths differ per (b, kv-head) so the merge, append and first-append paths of
    ``fused_hybrid_decode_update_kernel`` all run.
    """
    B, Hkv, Hq, D, W, cap, N0, steps = 2, 2, 4, 64, 16, 256, 100, 40
    keys = ar1_keys(B, Hkv, N0 + steps, D, seed)
    vals = normal((B, Hkv, N0 + steps, D), seed + 1)
    kp = torch.zeros((B, Hkv, cap, D), dtype=dtype)
    vp = torch.zeros_like(kp)
    counts = torch.zeros((B, Hkv, cap), dtype=torch.int32)
    ts = torch.zeros((B, Hkv, cap), dtype=torch.int32)
    lengths = torch.zeros((B * Hkv,), dtype=torch.int32)
    plen = [[25, 0], [3, 25]]
    for b in range(B):
        for h in range(Hkv):
            L = plen[b][h]
            idx = np.arange(L) * 4
            kp[b, h, :L] = torch.from_numpy(keys[b, h, idx]).to(dtype)
            vp[b, h, :L] = torch.from_numpy(vals[b, h, idx]).to(dtype)
            counts[b, h, :L] = 4
            ts[b, h, :L] = torch.from_numpy(idx.astype(np.int32))
            lengths[b * Hkv + h] = L
    ke = torch.from_numpy(keys[:, :, N0 - W:N0]).to(dtype).contiguous()
    ve = torch.from_numpy(vals[:, :, N0 - W:N0]).to(dtype).contiguous()
    new_k = [torch.from_numpy(keys[:, :, N0 + s:N0 + s + 1]).to(dtype).contiguous() for s in range(steps)]
    new_v = [torch.from_numpy(vals[:, :, N0 + s:N0 + s + 1]).to(dtype).contiguous() for s in range(steps)]
    q = [torch.from_numpy(normal((B, Hq, D), seed + 100 + s)).to(dtype) for s in range(steps)]
    kk = keys.astype(np.float64)
    d2 = ((kk[:, :, 1:] - kk[:, :, :-1]) ** 2).sum(-1)
    cs = (kk[:, :, 1:] * kk[:, :, :-1]).sum(-1) / (
        np.linalg.norm(kk[:, :, 1:], axis=-1) * np.linalg.norm(kk[:, :, :-1], axis=-1))
    return dict(B=B, Hkv=Hkv, Hq=Hq, D=D, W=W, cap=cap, steps=steps, kp=kp, vp=vp,
                counts=counts, ts=ts, lengths=lengths, ke=ke, ve=ve, new_k=new_k,
                new_v=new_v, q=q, exact_len=W, total=N0,
                thr_euclid_sq=float(np.quantile(d2, 0.6)), thr_cos=float(np.quantile(cs, 0.4)))


def quirk_keep(B, H, N):
    """Head 0 keeps 7 of every 8 positions; head 1 keeps only positions < 150.

    Head 1 then owns two real packed blocks followed by all-padding blocks (count 0,
    timestamp 0) inside M, which resets the reference's last_safe timestamp to 0.
    """
    pos = np.arange(N)
    keep = np.zeros((B, H, N), dtype=np.int32)
    keep[:, 0] = (pos % 8 != 7)
    for h in range(1, H):
        keep[:, h] = pos < 150
    return torch.from_numpy(keep)

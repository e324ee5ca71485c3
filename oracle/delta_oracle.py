"""CPU restatement of the DeltaAttention hot path (test infrastructure only).

Every function cites the reference file:line it restates. Paths are relative to the
reference project root (Emruur/DeltaAttention).

Numeric conventions (what "the reference" computes, as pinned by the Triton
interpreter goldens in ``tests/golden``):

* ``tl.sum`` of a 1-D fp32 vector is numpy's ``np.sum``: for n <= 128 that is eight
  strided fp32 accumulators combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)); fp16
  vectors are accumulated the same way in fp32 and rounded to fp16 once.
* fp16 elementwise arithmetic is computed in fp32 and rounded to fp16 (numpy half
  semantics). bf16 follows the same structure with bf16 rounding (nearest even). The
  stock interpreter operates on raw uint16 bit patterns for bf16, so the bf16 fixtures
  come from the reference kernels run on the interpreter with IEEE bf16 arithmetic
  (``tests/golden/bf16_interp.py``): selection, packing and decode state match them bit
  for bit, attention outputs to within one bf16 ulp.
* Attention dot products accumulate in fp32; the count-weighted probabilities are
  rounded to the value dtype before the PV product (deltaFlashAttention.py:98,137).
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

__all__ = [
    "round_to", "np_sum_f32", "rope_inv_freq", "rope_cos_sin", "apply_rope",
    "delta_keep_mask", "periodic_keep_mask", "random_keep_mask", "nm_keep_mask",
    "pack_from_keep", "hybrid_schedule", "tile_count", "hybrid_attention",
    "flash_attention", "decode_update", "decode_attention", "sq_dist_f32",
    "eager_attention", "proj_rope", "dpxa_keep", "dpxa_tile_stats", "dpxa_weights", "dpxa_select",
    "block_sparse_attention",
]

# ---------------------------------------------------------------------------
# numeric helpers
# ---------------------------------------------------------------------------

def _f32_to_bf16_bits_rne(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = np.isnan(x)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = ((u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).astype(np.uint32)
    r = np.where(nan, np.uint32(0x7FC00000), r)
    return r.view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` ('fp32' | 'fp16' | 'bf16') and return them as fp32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return _f32_to_bf16_bits_rne(x)
    raise ValueError(dtype)


def np_sum_f32(x: np.ndarray) -> np.ndarray:
    """Row sums over the last axis in numpy's order (the interpreter's ``tl.sum``)."""
    return np.sum(np.ascontiguousarray(x, dtype=np.float32), axis=-1, dtype=np.float32)


def _dtype_name(t: torch.Tensor) -> str:
    return {torch.float32: "fp32", torch.float16: "fp16", torch.bfloat16: "bf16"}[t.dtype]


def sq_dist_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """fp32 squared distance with fp32-upcast operands (deltaDecoding.py:74-75)."""
    d = (a.astype(np.float32) - b.astype(np.float32)).astype(np.float32)
    return np_sum_f32(d * d)


# ---------------------------------------------------------------------------
# RoPE  (modeling_llama.py:159-204; HF "default" rope init)
# ---------------------------------------------------------------------------

def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """``1 / theta ** (arange(0, d, 2) / d)`` in fp32, as HF's default rope init."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))


def rope_cos_sin(seq_len: int, head_dim: int, theta: float, dtype: torch.dtype,
                 batch: int = 1):
    """cos/sin tables [B, N, d] (modeling_llama.py:160-170): fp32 math, cast to dtype."""
    inv_freq = rope_inv_freq(head_dim, theta)
    pos = torch.arange(seq_len, dtype=torch.int64)[None, :].expand(batch, -1)
    inv_e = inv_freq[None, :, None].float().expand(batch, -1, 1)
    freqs = (inv_e.float() @ pos[:, None, :].float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_half(x):  # modeling_llama.py:173-177
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x*cos + rotate_half(x)*sin`` in x's dtype (modeling_llama.py:200-204); x is [B,H,N,d]."""
    cos = cos.unsqueeze(1)
    sin = sin.unsqueeze(1)
    return (x * cos) + (_rotate_half(x) * sin)


# ---------------------------------------------------------------------------
# anchor selection
# ---------------------------------------------------------------------------

def proj_rope(x: torch.Tensor, w: torch.Tensor, cos: Optional[torch.Tensor], sin: Optional[torch.Tensor],
              rope_lo: int, rope_hi: int, head_dim: int = 128) -> torch.Tensor:
    """``k_proj(hidden_states).view(B, N, H, d)`` then ``apply_rotary_pos_emb``
    (modeling_llama.py:550-555, :180-204), kept in the projection layout [rows, out].

    The Linear's product is accumulated in fp64 here and rounded to the input dtype once (a
    GEMM's fp32 accumulation order is implementation-defined, so parity with it is to
    within rounding); RoPE then follows eager rounding on columns [rope_lo, rope_hi).
    """
    y = (x.double() @ w.double().t()).to(x.dtype)
    if rope_hi <= rope_lo:
        return y
    rows = y.shape[0]
    part = y[:, rope_lo:rope_hi].reshape(rows, -1, head_dim).transpose(0, 1)   # [H, rows, d]
    rot = apply_rope(part.unsqueeze(0), cos.reshape(1, rows, head_dim), sin.reshape(1, rows, head_dim))[0]
    y = y.clone()
    y[:, rope_lo:rope_hi] = rot.transpose(0, 1).reshape(rows, -1)
    return y


def delta_keep_mask(k: torch.Tensor, threshold: float, use_cosine: bool,
                    chunk_size: int, num_chunks: int):
    """``chunked_eval_kernel`` (tritonModules.py:7-69) over grid (B*H, num_chunks).

    ``threshold`` is the kernel argument as passed (cosine threshold, or the squared
    Euclidean threshold). Returns (keep_mask int32 [B,H,N], chunk_counts int32
    [B,H,num_chunks]); positions no program visits stay 0 (the caller zero-inits).
    All chunks of all heads advance in lockstep, one token per step.
    """
    B, H, N, D = k.shape
    dt = _dtype_name(k)
    kk = k.detach().float().cpu().numpy().astype(np.float32)
    keep = np.zeros((B, H, N), dtype=np.int32)
    ccount = np.zeros((B, H, num_chunks), dtype=np.int32)
    starts = np.arange(num_chunks) * chunk_size
    live = starts < N
    if not live.any():
        return torch.from_numpy(keep), torch.from_numpy(ccount)
    cidx = np.nonzero(live)[0]
    st = starts[cidx]
    en = np.minimum(st + chunk_size, N)
    thr = np.float32(threshold)
    # lanes: (b, h, chunk)
    L_b, L_h, L_c = np.meshgrid(np.arange(B), np.arange(H), np.arange(len(cidx)), indexing="ij")
    L_b, L_h, L_c = L_b.ravel(), L_h.ravel(), L_c.ravel()
    lst = st[L_c]
    len_ = (en - st)[L_c]
    ref = kk[L_b, L_h, lst]                      # anchor rows (fp32 holding dtype values)
    keep[L_b, L_h, lst] = 1
    local = np.ones(len(L_b), dtype=np.int32)
    eps = np.float32(1e-8)
    for i in range(1, int(len_.max())):
        act = i < len_
        if not act.any():
            break
        ai = np.nonzero(act)[0]
        pos = lst[ai] + i
        cur = kk[L_b[ai], L_h[ai], pos]
        r = ref[ai]
        if use_cosine:
            dot = np_sum_f32(cur * r)
            nc = np.sqrt(np_sum_f32(cur * cur) + eps).astype(np.float32)
            nr = np.sqrt(np_sum_f32(r * r) + eps).astype(np.float32)
            cos = (dot / (nc * nr).astype(np.float32)).astype(np.float32)
            kp = cos < thr
        else:
            diff = round_to(cur - r, dt)
            sq = round_to(diff * diff, dt)
            s = np_sum_f32(sq)
            s = round_to(s, dt)
            kp = s > thr
        keep[L_b[ai], L_h[ai], pos] = kp.astype(np.int32)
        upd = ai[kp]
        ref[upd] = cur[kp]
        local[upd] += 1
    ccount[L_b, L_h, cidx[L_c]] = local
    return torch.from_numpy(keep), torch.from_numpy(ccount)


def periodic_keep_mask(B: int, H: int, N: int, keep_rate: float) -> torch.Tensor:
    """``packing_mode == 'periodic'`` (modeling_llama.py:626-632)."""
    period = max(1, round(1.0 / keep_rate))
    row = (torch.arange(N) % period == 0).to(torch.int32)
    return row[None, None, :].expand(B, H, N).contiguous()


def random_keep_mask(B: int, H: int, N: int, keep_rate: float, generator=None) -> torch.Tensor:
    """``packing_mode == 'random'`` (modeling_llama.py:620-624), on a CPU generator."""
    km = (torch.rand(B, H, N, generator=generator) < keep_rate).to(torch.int32)
    km[:, :, 0] = 1
    return km


def nm_keep_mask(k: torch.Tensor, n: int, m: int, ratio: int) -> torch.Tensor:
    """Builder-specified N:M structured selection (the reference ships no source for it).

    Candidates are positions ``t % c == 0`` with ``c = ratio * n / m``. Candidate ``t``
    scores ``+inf`` at t == 0, else the fp32 squared distance between K[t] and K[t-c]
    (numpy summation order). Consecutive runs of ``m`` candidates form groups; each
    group keeps its ``min(n, size)`` highest-scoring candidates, ties to the earlier
    position. Every head therefore keeps the same number of anchors.
    """
    if (ratio * n) % m:
        raise ValueError("ratio*n/m must be an integer candidate stride")
    c = ratio * n // m
    if c < 1:
        raise ValueError("candidate stride must be >= 1")
    B, H, N, D = k.shape
    kk = k.detach().float().cpu().numpy().astype(np.float32)
    cand = np.arange(0, N, c)
    G = len(cand)
    score = np.full((B, H, G), np.inf, dtype=np.float32)
    if G > 1:
        a = kk[:, :, cand[1:]]
        b = kk[:, :, cand[1:] - c]
        d = (a - b).astype(np.float32)
        score[:, :, 1:] = np_sum_f32(d * d)
    keep = np.zeros((B, H, N), dtype=np.int32)
    for g0 in range(0, G, m):
        g1 = min(g0 + m, G)
        s = score[:, :, g0:g1]
        # stable sort by descending score: ties keep the earlier candidate
        order = np.argsort(-s, axis=-1, kind="stable")[..., :min(n, g1 - g0)]
        sel = cand[g0:g1][order]
        bi, hi = np.meshgrid(np.arange(B), np.arange(H), indexing="ij")
        for j in range(sel.shape[-1]):
            keep[bi, hi, sel[..., j]] = 1
    return torch.from_numpy(keep)


# ---------------------------------------------------------------------------
# packing  (modeling_llama.py:655-685; tritonModules.py:72-132)
# ---------------------------------------------------------------------------

def pack_from_keep(k: torch.Tensor, v: torch.Tensor, keep_mask: torch.Tensor,
                   num_packed: Optional[int] = None):
    """index_map = cumsum(keep)-1; scatter kept K/V/positions; counts by scatter_add.

    Returns (index_map int32, k_packed, v_packed, timestamps int32, counts int32), packed
    buffers zero-initialised to ``num_packed`` rows (default: max kept over heads).
    """
    B, H, N, D = k.shape
    km = keep_mask.to(torch.int32)
    index_map = (torch.cumsum(km, dim=-1) - 1).to(torch.int32)
    M = int(km.sum(-1).max()) if num_packed is None else int(num_packed)
    kp = torch.zeros((B, H, M, D), dtype=k.dtype)
    vp = torch.zeros_like(kp)
    ts = torch.zeros((B, H, M), dtype=torch.int32)
    pos = torch.arange(N, dtype=torch.int32)
    for b in range(B):
        for h in range(H):
            sel = km[b, h] == 1
            idx = index_map[b, h, sel].long()
            kp[b, h, idx] = k[b, h, sel].cpu()
            vp[b, h, idx] = v[b, h, sel].cpu()
            ts[b, h, idx] = pos[sel]
    counts = torch.zeros((B, H, M), dtype=torch.int32)
    counts.scatter_add_(2, index_map.long(), torch.ones_like(index_map, dtype=torch.int32))
    return index_map, kp, vp, ts, counts


# ---------------------------------------------------------------------------
# two-phase schedule  (deltaFlashAttention.py:63-113)
# ---------------------------------------------------------------------------

def hybrid_schedule(ts_row: np.ndarray, num_packed: int, seq_len_k: int, start_m: int,
                    dense_window: int, block_m: int = 128, block_n: int = 128):
    """(n_packed_blocks, dense_start, dense_hi) for one query block of one head."""
    ts_row = np.asarray(ts_row)
    n1 = 0
    last_safe = -1
    start_n = 0
    while start_n < num_packed:
        idx = start_n + np.arange(block_n)
        t = np.where(idx < num_packed, ts_row[np.minimum(idx, num_packed - 1)], seq_len_k + 1)
        tmax = int(t.max())
        if tmax >= start_m - dense_window:
            break
        last_safe = tmax
        n1 += 1
        start_n += block_n
    dense_start = max(0, ((last_safe + 1) // block_n) * block_n)
    dense_hi = min(seq_len_k, start_m + block_m)
    return n1, dense_start, dense_hi


def tile_count(N: int, r: int, W: int = 128, block: int = 128) -> int:
    """128x128 tiles one head runs under the reference schedule with periodic-r packing."""
    if r == 1:
        nb = -(-N // block)
        return nb * (nb + 1) // 2
    M = -(-N // r)
    ts = np.arange(M) * r
    tot = 0
    for mb in range(-(-N // block)):
        n1, ds, hi = hybrid_schedule(ts, M, N, mb * block, W, block, block)
        tot += n1 + max(0, -(-(hi - ds) // block))
    return tot


# ---------------------------------------------------------------------------
# attention  (deltaFlashAttention.py:9-357; flashAttention.py:5-91)
# ---------------------------------------------------------------------------

def _blk(x, a, b):
    return x[a:b]


def hybrid_attention(q, k_dense, v_dense, k_packed, v_packed, timestamps, counts,
                     sm_scale: float, dense_window: int, variant: str = "hybrid",
                     n_rep: int = 1, block_m: int = 128, block_n: int = 128,
                     heads: Optional[list] = None, query_blocks: Optional[list] = None):
    """Two-phase count-weighted attention, one query block at a time.

    variant: 'hybrid' (deltaFlashAttention.py:9-146), 'sanity' (:149-259) or
    'pure_phase1' (:262-357). q is [B,Hq,Nq,d]; the K/V/ts/counts tensors have
    Hq/n_rep heads (q-head h reads kv-head h // n_rep; n_rep=1 is the reference's
    repeat_kv-expanded call). ``heads`` / ``query_blocks`` optionally restrict the q-heads
    and query blocks computed (others are returned as zeros). Returns the output in q's dtype.
    """
    B, Hq, Nq, D = q.shape
    Nk = k_dense.shape[2]
    M = k_packed.shape[2]
    dt = _dtype_name(v_dense)
    out = torch.zeros((B, Hq, Nq, D), dtype=torch.float32)
    qf = q.float()
    kdf, vdf = k_dense.float(), v_dense.float()
    kpf, vpf = k_packed.float(), v_packed.float()
    tsn = timestamps.to(torch.int64).numpy()
    cf = counts.float()
    rdt = {"fp32": None, "fp16": torch.float16, "bf16": torch.bfloat16}[dt]
    ninf = float("-inf")
    heads = list(range(Hq)) if heads is None else list(heads)

    def rnd(x):
        return x if rdt is None else x.to(rdt).float()

    for b in range(B):
        for hk in range(Hq // n_rep):
            hs = [h for h in range(hk * n_rep, (hk + 1) * n_rep) if h in heads]
            if not hs:
                continue
            pids = range(-(-Nq // block_m)) if query_blocks is None else query_blocks
            for pid in pids:
                m0 = pid * block_m
                m1 = min(Nq, m0 + block_m)
                rows = torch.arange(m0, m1)
                R = m1 - m0
                qb = torch.cat([qf[b, h, m0:m1] for h in hs], 0)   # [len(hs)*R, D]
                rowpos = rows.repeat(len(hs))
                m_i = torch.full((qb.shape[0],), ninf)
                l_i = torch.zeros(qb.shape[0])
                acc = torch.zeros(qb.shape[0], D)
                last_safe = -1
                start_n = 0
                if variant in ("hybrid", "sanity"):
                    while start_n < M:
                        idx = start_n + np.arange(block_n)
                        pm = idx < M
                        tsb = np.where(pm, tsn[b, hk, np.minimum(idx, M - 1)], Nk + 1)
                        tmax = int(tsb.max())
                        if tmax >= m0 - dense_window:
                            break
                        sl = slice(start_n, min(start_n + block_n, M))
                        nv = sl.stop - sl.start
                        if variant == "hybrid":
                            qk = torch.full((qb.shape[0], block_n), ninf)
                            qk[:, :nv] = (qb @ kpf[b, hk, sl].T) * sm_scale
                            m_ij = torch.maximum(m_i, qk.max(1).values)
                            p = torch.exp(qk - m_ij[:, None])
                            c = torch.zeros(block_n)
                            c[:nv] = cf[b, hk, sl]
                            pw = p * c[None, :]
                            l_ij = pw.sum(1)
                            alpha = torch.exp(m_i - m_ij)
                            l_i = l_i * alpha + l_ij
                            acc = acc * alpha[:, None]
                            acc = acc + rnd(pw[:, :nv]) @ vpf[b, hk, sl]
                            m_i = m_ij
                        last_safe = tmax
                        start_n += block_n
                    ds = max(0, ((last_safe + 1) // block_n) * block_n)
                    hi = min(Nk, m0 + block_m)
                    for sn in range(ds, hi, block_n):
                        se = min(sn + block_n, Nk)
                        cols = torch.arange(sn, sn + block_n)
                        qk = torch.full((qb.shape[0], block_n), ninf)
                        qk[:, : se - sn] = (qb @ kdf[b, hk, sn:se].T) * sm_scale
                        mask = (rowpos[:, None] >= cols[None, :]) & (cols[None, :] < Nk)
                        qk = torch.where(mask, qk, torch.tensor(ninf))
                        m_ij = torch.maximum(m_i, qk.max(1).values)
                        p = torch.exp(qk - m_ij[:, None])
                        l_ij = p.sum(1)
                        alpha = torch.exp(m_i - m_ij)
                        l_i = l_i * alpha + l_ij
                        acc = acc * alpha[:, None]
                        acc = acc + rnd(p[:, : se - sn]) @ vdf[b, hk, sn:se]
                        m_i = m_ij
                    o = acc / l_i[:, None]
                elif variant == "pure_phase1":
                    while start_n < M:
                        sl = slice(start_n, min(start_n + block_n, M))
                        nv = sl.stop - sl.start
                        tsb = torch.from_numpy(tsn[b, hk, sl])
                        c = torch.zeros(block_n)
                        c[:nv] = cf[b, hk, sl]
                        kv = torch.zeros(block_n, dtype=torch.bool)
                        kv[:nv] = c[:nv] > 0
                        tfull = torch.full((block_n,), Nk + 1, dtype=torch.int64)
                        tfull[:nv] = tsb
                        valid = (tfull[None, :] <= rowpos[:, None]) & kv[None, :]
                        qk = torch.full((qb.shape[0], block_n), ninf)
                        qk[:, :nv] = (qb @ kpf[b, hk, sl].T) * sm_scale
                        qk = torch.where(valid, qk, torch.tensor(ninf))
                        m_ij = torch.maximum(m_i, qk.max(1).values)
                        p = torch.exp(qk - m_ij[:, None])
                        pw = p * c[None, :]
                        l_ij = pw.sum(1)
                        alpha = torch.exp(m_i - m_ij)
                        l_i = l_i * alpha + l_ij
                        acc = acc * alpha[:, None]
                        acc = acc + rnd(pw[:, :nv]) @ vpf[b, hk, sl]
                        m_i = m_ij
                        start_n += block_n
                    safe = torch.where(l_i > 0, l_i, torch.ones_like(l_i))
                    o = acc / safe[:, None]
                else:
                    raise ValueError(variant)
                for j, h in enumerate(hs):
                    out[b, h, m0:m1] = o[j * R:(j + 1) * R]
    return out.to(q.dtype)


def flash_attention(q, k, v, causal: bool = True, sm_scale: Optional[float] = None,
                    block_m: int = 128, block_n: int = 128, n_rep: int = 1):
    """``_attn_fwd_flat`` (flashAttention.py:5-91): dense FA2 forward, natural exp."""
    B, H, N, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / (D ** 0.5)
    dt = _dtype_name(v)
    rdt = {"fp32": None, "fp16": torch.float16, "bf16": torch.bfloat16}[dt]
    qf, kf, vf = q.float(), k.float(), v.float()
    out = torch.zeros((B, H, N, D), dtype=torch.float32)
    ninf = float("-inf")
    for b in range(B):
        for h in range(H):
            hk = h // n_rep
            for pid in range(-(-N // block_m)):
                m0, m1 = pid * block_m, min(N, pid * block_m + block_m)
                rows = torch.arange(m0, m1)
                qb = qf[b, h, m0:m1]
                m_i = torch.full((m1 - m0,), ninf)
                l_i = torch.zeros(m1 - m0)
                acc = torch.zeros(m1 - m0, D)
                hi = min(N, (pid + 1) * block_m) if causal else N
                for sn in range(0, hi, block_n):
                    se = min(sn + block_n, N)
                    cols = torch.arange(sn, sn + block_n)
                    qk = torch.zeros(m1 - m0, block_n)
                    qk[:, : se - sn] = qb @ kf[b, hk, sn:se].T
                    qk = qk * sm_scale
                    if causal:
                        qk = torch.where(rows[:, None] >= cols[None, :], qk, torch.tensor(ninf))
                    m_ij = torch.maximum(m_i, qk.max(1).values)
                    p = torch.exp(qk - m_ij[:, None])
                    p = torch.where(cols[None, :] < N, p, torch.zeros(()))
                    l_ij = p.sum(1)
                    alpha = torch.exp(m_i - m_ij)
                    l_i = l_i * alpha + l_ij
                    acc = acc * alpha[:, None]
                    pr = p if rdt is None else p.to(rdt).float()
                    acc = acc + pr[:, : se - sn] @ vf[b, hk, sn:se]
                    m_i = m_ij
                out[b, h, m0:m1] = acc / l_i[:, None]
    return out.to(q.dtype)


def eager_attention(q, k, v, sm_scale: float, n_rep: int = 1, query_rows: Optional[slice] = None):
    """``eager_attention_forward`` (modeling_llama.py:235-276) with a causal mask, fp32 softmax.

    ``query_rows`` (a slice of positions) computes only those query rows against all N keys,
    with the causal mask at their absolute positions; the output then holds those rows."""
    k = k.repeat_interleave(n_rep, dim=1)
    v = v.repeat_interleave(n_rep, dim=1)
    N = k.shape[2]
    rows = torch.arange(N)
    if query_rows is not None:
        q = q[:, :, query_rows]
        rows = rows[query_rows]
    w = torch.matmul(q, k.transpose(2, 3)) * sm_scale
    mask = torch.where(torch.arange(N)[None, :] > rows[:, None], float("-inf"), 0.0).to(w.dtype)
    w = w + mask
    w = torch.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(w, v)


# ---------------------------------------------------------------------------
# DPXA: delta-based tile scoring for block-sparse prefill (Paper/src/methodology.tex:89-135)
#
# The paper describes the method without code; this is the builder's specification, which
# the CUDA path implements and these functions restate:
#   1. Compaction: Stage-1 delta selection (the chunked_eval_kernel rule, Euclidean, squared
#      threshold) over every 128-token block of post-RoPE Q (threshold tau_q) and of
#      post-RoPE K (tau_k); each block's first row is an anchor; anchors keep their order.
#   2. Sampled scores per tile (query block i of q-head h, key block j <= i of its kv-head):
#      S = scale * Q^d_i K^d_j^T over the anchors only, causal inside the diagonal tile
#      (anchor key position <= anchor query position).
#   3. Tile importance: the sum of exp(S) over the tile's valid cells, kept as (max, sum of
#      exp(S - max)) per tile so no exponential overflows.
#   4. Top-p selection: per q-head the tile weights of a query block are its tiles'
#      importance over their total (the sampled attention mass); the q-heads of a GQA group
#      share one selection (their weights averaged), so the group's K / V blocks are read
#      once. Tiles are taken in decreasing weight (ties to the lower block) until the
#      cumulative weight exceeds p; the diagonal tile is always taken.
#   5. Attention: causal softmax attention of the full Q against the full K / V of the
#      selected key blocks only.
# ---------------------------------------------------------------------------

def dpxa_keep(x: torch.Tensor, threshold: float, block: int = 128) -> torch.Tensor:
    """Step 1: anchor mask of every ``block``-token block (chunked_eval_kernel with chunk =
    block, Euclidean; ``threshold`` is the squared distance threshold)."""
    N = x.shape[2]
    keep, _ = delta_keep_mask(x, threshold, False, block, -(-N // block))
    return keep


def dpxa_tile_stats(q, k, keep_q, keep_k, sm_scale: float, n_rep: int, block: int = 128):
    """Steps 2-3: per (b, q-head, query block i, key block j <= i) the tile's maximum scaled
    sampled score and the sum of exp(S - max) over its valid cells (fp64 here). Tiles with
    j > i, or without a valid cell, hold (-inf, 0). Returns (tmax, tsum) [B, Hq, nb, nb]."""
    B, Hq, N, D = q.shape
    nb = -(-N // block)
    tmax = torch.full((B, Hq, nb, nb), float("-inf"), dtype=torch.float64)
    tsum = torch.zeros((B, Hq, nb, nb), dtype=torch.float64)
    qf, kf = q.double(), k.double()
    for b in range(B):
        for h in range(Hq):
            hk = h // n_rep
            kblocks = []
            for j in range(nb):
                idx = torch.nonzero(keep_k[b, hk, j * block:(j + 1) * block]).flatten() + j * block
                kblocks.append((idx, kf[b, hk, idx]))
            for i in range(nb):
                qi = torch.nonzero(keep_q[b, h, i * block:(i + 1) * block]).flatten() + i * block
                qa = qf[b, h, qi]
                for j in range(i + 1):
                    kj, ka = kblocks[j]
                    sc = (qa @ ka.T) * sm_scale
                    if j == i:
                        sc = torch.where(kj[None, :] <= qi[:, None], sc, torch.tensor(float("-inf"), dtype=sc.dtype))
                    m = sc.max() if sc.numel() else torch.tensor(float("-inf"))
                    if torch.isfinite(m):
                        tmax[b, h, i, j] = m
                        tsum[b, h, i, j] = torch.exp(sc - m).sum()
    return tmax, tsum


def dpxa_weights(tmax, tsum, n_rep: int):
    """Step 4 (weights): per q-head, tile importance over the query block's total; then the
    mean over each GQA group's q-heads. Returns [B, Hkv, nb, nb] (zero for j > i)."""
    B, Hq, nb, _ = tmax.shape
    M = tmax.max(dim=-1, keepdim=True).values
    M = torch.where(torch.isfinite(M), M, torch.zeros_like(M))
    imp = torch.where(torch.isfinite(tmax), torch.exp(tmax - M) * tsum, torch.zeros_like(tsum))
    tot = imp.sum(-1, keepdim=True)
    w = torch.where(tot > 0, imp / torch.where(tot > 0, tot, torch.ones_like(tot)), torch.zeros_like(imp))
    return w.view(B, Hq // n_rep, n_rep, nb, nb).mean(2)


def dpxa_select(w, p: float) -> torch.Tensor:
    """Step 4 (top-p): bool [B, Hkv, nb, nb], causal, the diagonal always selected."""
    B, Hk, nb, _ = w.shape
    sel = torch.zeros((B, Hk, nb, nb), dtype=torch.bool)
    for b in range(B):
        for h in range(Hk):
            for i in range(nb):
                wi = w[b, h, i, : i + 1]
                order = sorted(range(i + 1), key=lambda j: (-float(wi[j]), j))
                cum = 0.0
                for j in order:
                    sel[b, h, i, j] = True
                    cum += float(wi[j])
                    if cum > p:
                        break
                sel[b, h, i, i] = True
    return sel


def block_sparse_attention(q, k, v, sel, sm_scale: float, n_rep: int, block: int = 128,
                           heads: Optional[list] = None, query_blocks: Optional[list] = None):
    """Step 5: causal attention of each query block against the selected key blocks of its
    kv-head (``sel`` [B, Hkv, nb, nb]); P is rounded to v's dtype before PV as in the
    two-phase kernel. Returns q's dtype; heads / query blocks not listed are zero."""
    B, Hq, N, D = q.shape
    nb = -(-N // block)
    dt = _dtype_name(v)
    rdt = {"fp32": None, "fp16": torch.float16, "bf16": torch.bfloat16}[dt]
    out = torch.zeros((B, Hq, N, D), dtype=torch.float32)
    qf, kf, vf = q.float(), k.float(), v.float()
    heads = list(range(Hq)) if heads is None else list(heads)
    qbs = list(range(nb)) if query_blocks is None else list(query_blocks)
    for b in range(B):
        for h in heads:
            hk = h // n_rep
            for i in qbs:
                m0, m1 = i * block, min(N, (i + 1) * block)
                blocks = [j for j in range(i + 1) if bool(sel[b, hk, i, j])]
                cols = torch.cat([torch.arange(j * block, min(N, (j + 1) * block)) for j in blocks])
                sc = (qf[b, h, m0:m1] @ kf[b, hk, cols].T) * sm_scale
                rows = torch.arange(m0, m1)
                sc = torch.where(cols[None, :] <= rows[:, None], sc, torch.tensor(float("-inf")))
                mx = sc.max(1, keepdim=True).values
                pr = torch.exp(sc - mx)
                l = pr.sum(1, keepdim=True)
                pr = pr if rdt is None else pr.to(rdt).float()
                out[b, h, m0:m1] = (pr @ vf[b, hk, cols]) / l
    return out.to(q.dtype)


# ---------------------------------------------------------------------------
# decoding  (deltaDecoding.py:9-104, 236-362)
# ---------------------------------------------------------------------------

def decode_update(new_k, new_v, k_exact, v_exact, k_packed, v_packed, counts, timestamps,
                  lengths, exact_seq_len: int, total_seq_len: int, threshold: float,
                  window: int, use_cosine: bool):
    """``fused_hybrid_decode_update_kernel`` (deltaDecoding.py:9-104), in place on CPU tensors.

    new_k/new_v [B,H,1,d]; k_exact [B,H,W,d]; k_packed [B,H,cap,d]; counts/timestamps
    [B,H,cap] int32; lengths [B*H] int32.
    """
    B, H = new_k.shape[:2]
    w = exact_seq_len % window
    thr = np.float32(threshold)
    eps = np.float32(1e-8)
    for b in range(B):
        for h in range(H):
            pid = b * H + h
            plen = int(lengths[pid])
            if exact_seq_len >= window:
                ek = k_exact[b, h, w].clone()
                ev = v_exact[b, h, w].clone()
                if plen > 0:
                    last = k_packed[b, h, plen - 1]
                    e32 = ek.float().numpy()
                    l32 = last.float().numpy()
                    if use_cosine:
                        dot = np_sum_f32(e32 * l32)
                        ne = np.sqrt(np_sum_f32(e32 * e32) + eps).astype(np.float32)
                        nl = np.sqrt(np_sum_f32(l32 * l32) + eps).astype(np.float32)
                        cs = np.float32(dot / np.float32(ne * nl))
                        merge = cs >= thr
                    else:
                        merge = sq_dist_f32(e32, l32) <= thr
                    if merge:
                        counts[b, h, plen - 1] += 1
                    else:
                        k_packed[b, h, plen] = ek
                        v_packed[b, h, plen] = ev
                        counts[b, h, plen] = 1
                        timestamps[b, h, plen] = total_seq_len - window
                        lengths[pid] = plen + 1
                else:
                    k_packed[b, h, 0] = ek
                    v_packed[b, h, 0] = ev
                    counts[b, h, 0] = 1
                    timestamps[b, h, 0] = total_seq_len - window
                    lengths[pid] = 1
            k_exact[b, h, w] = new_k[b, h, 0]
            v_exact[b, h, w] = new_v[b, h, 0]


def decode_attention(q, k_packed, v_packed, counts, lengths, k_exact, v_exact,
                     sm_scale: float, exact_len: int, n_rep: int):
    """``fused_hybrid_decode_kernel`` (deltaDecoding.py:236-362) for one token.

    q [B,Hq,d]; packed/exact tensors [B,Hkv,...]; lengths [B,Hkv]. Phase 1 adds
    log(count) to the scaled logits; phase 2 attends the first ``exact_len`` ring
    slots. Returns [B,Hq,d] in q's dtype.
    """
    B, Hq, D = q.shape
    dt = _dtype_name(v_packed)
    rdt = {"fp32": None, "fp16": torch.float16, "bf16": torch.bfloat16}[dt]
    out = torch.zeros((B, Hq, D), dtype=torch.float32)
    for b in range(B):
        for h in range(Hq):
            kv = h // n_rep
            qv = q[b, h].float()
            L = int(lengths[b, kv])
            s1 = (k_packed[b, kv, :L].float() @ qv) * sm_scale
            s1 = s1 + torch.log(counts[b, kv, :L].float())
            s2 = (k_exact[b, kv, :exact_len].float() @ qv) * sm_scale
            s = torch.cat([s1, s2])
            vv = torch.cat([v_packed[b, kv, :L].float(), v_exact[b, kv, :exact_len].float()])
            m = s.max()
            p = torch.exp(s - m)
            pr = p if rdt is None else p.to(rdt).float()
            out[b, h] = (pr @ vv) / p.sum()
    return out.to(q.dtype)

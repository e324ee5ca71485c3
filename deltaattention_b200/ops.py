"""Native B200 entry points for the delta-attention prefill path.

``delta_prefill`` runs the whole hot path the reference spreads over
modeling_llama.py:555 and :600-749 (RoPE, anchor selection, index map, packing, counts,
GQA expansion, two-phase attention) with these B200-specific changes:

* GQA is index arithmetic (q-head h reads kv-head h // n_rep): the six ``repeat_kv`` copies
  of modeling_llama.py:700-708 are gone;
* periodic packing is a strided view of the rotated keys / values (row stride x period), so
  nothing is copied; timestamps and counts come from one tiny kernel;
* delta selection, with RoPE(k) and packing, is one launch whose packed length stays on the
  device (no host sync); explicit keep masks pack on the device with the reference's one read
  of the packed length (modeling_llama.py:656);
* the output can be written straight into the ``[B, N, H, d]`` layout ``o_proj`` consumes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib as L

VARIANTS = {"hybrid": 0, "sanity": 1, "pure_phase1": 2}


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, out: Optional[torch.Tensor] = None):
    """``apply_rotary_pos_emb`` for one [B, H, N, d] tensor (modeling_llama.py:180-204).

    cos / sin are [B or 1, N, d] in x's dtype; rounding follows eager torch exactly.
    """
    L.require_cuda(x, cos, sin)
    B, H, N, D = x.shape
    if out is None:
        out = torch.empty((B, H, N, D), dtype=x.dtype, device=x.device)
    cb = cos.stride(0) if cos.shape[0] > 1 else 0
    if cos.stride() != sin.stride():
        sin = sin.contiguous()
        cos = cos.contiguous()
        cb = cos.stride(0) if cos.shape[0] > 1 else 0
    st = L.stream_of(x)
    L.check(L.load().dab_rope(L.ptr(x), L.strides(x.stride()), L.ptr(out), L.strides(out.stride()), L.ptr(cos),
                              L.ptr(sin), L.strides([cb, cos.stride(1), cos.stride(2)]), L.dtype_code(x), B, H, N,
                              D, st), "rope")
    return out


def dpxa_select(q_rot: torch.Tensor, k_rot: torch.Tensor, tau_q: float, tau_k: float, top_p: float,
                sm_scale: Optional[float] = None, return_stats: bool = False):
    """DPXA tile selection (Paper/src/methodology.tex:89-135, as the library specifies it).

    q_rot [B, Hq, N, d], k_rot [B, Hkv, N, d] post-RoPE, bf16 / fp16, d 64 or 128. Steps: the
    delta selection (Euclidean, thresholds tau_q / tau_k, squared inside as the reference) on
    every 128-token block of Q and K; each block's anchors compacted; sampled tile scores
    Q^d K^d^T (causal on the diagonal) reduced to a tile importance; per query block the
    tiles taken by decreasing weight (the weights of a GQA group's q-heads averaged) until the
    cumulative weight exceeds ``top_p``, the diagonal always. Returns the selection bitmask
    [B, Hkv, nb, ceil(nb/32)] int32 (bit j of query block i: key block j attended), and with
    ``return_stats`` also (keep_q, keep_k, tile_max, tile_sum) [B, Hq, nb, nb].
    """
    L.require_cuda(q_rot, k_rot)
    B, Hq, N, D = q_rot.shape
    Hkv = k_rot.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must be a multiple of kv heads")
    if sm_scale is None:
        sm_scale = D ** -0.5
    nb = -(-N // 128)
    dev = q_rot.device
    lib = L.load()
    st = L.stream_of(q_rot)
    keep_q, _ = delta_keep_mask(q_rot, tau_q, "euclidean", 128)
    keep_k, _ = delta_keep_mask(k_rot, tau_k, "euclidean", 128)
    out = {}
    for name, x, keep, H in (("q", q_rot, keep_q, Hq), ("k", k_rot, keep_k, Hkv)):
        cx = torch.empty((B, H, nb, 128, D), dtype=x.dtype, device=dev)
        pos = torch.empty((B, H, nb, 128), dtype=torch.int32, device=dev)
        cnt = torch.empty((B, H, nb), dtype=torch.int32, device=dev)
        L.check(lib.dab_dpxa_compact(L.ptr(x), L.strides(x.stride()), L.ptr(keep), L.strides(keep.stride()), L.ptr(cx),
                                     L.ptr(pos), L.ptr(cnt), L.dtype_code(x), B, H, N, D, st), "dpxa_compact")
        out[name] = (cx, pos, cnt)
    tmax = torch.full((B, Hq, nb, nb), float("-inf"), dtype=torch.float32, device=dev)
    tsum = torch.zeros((B, Hq, nb, nb), dtype=torch.float32, device=dev)
    (cq, qp, qc), (ck, kp_, kc) = out["q"], out["k"]
    L.check(lib.dab_dpxa_score(L.ptr(cq), L.ptr(qp), L.ptr(qc), L.ptr(ck), L.ptr(kp_), L.ptr(kc), L.ptr(tmax),
                               L.ptr(tsum), float(sm_scale), L.dtype_code(q_rot), B, Hq, Hq // Hkv, N, D, st),
            "dpxa_score")
    sel = torch.empty((B, Hkv, nb, -(-nb // 32)), dtype=torch.int32, device=dev)
    L.check(lib.dab_dpxa_select(L.ptr(tmax), L.ptr(tsum), L.ptr(sel), float(top_p), B, Hkv, Hq // Hkv, N, st),
            "dpxa_select")
    if return_stats:
        return sel, (keep_q, keep_k, tmax, tsum)
    return sel


def selection_to_mask(sel: torch.Tensor, nb: int) -> torch.Tensor:
    """The bitmask of ``dpxa_select`` as bool [B, Hkv, nb, nb]."""
    j = torch.arange(nb, device=sel.device)
    words = sel.to(torch.int64) & 0xFFFFFFFF
    return ((words[..., j // 32] >> (j % 32)) & 1).bool()


def block_sparse_attention(q_rot, k_rot, v, sel, *, sm_scale=None, out=None):
    """Causal attention over the selected 128-key blocks only (DPXA step 5) on the tcgen05
    kernel: q_rot [B, Hq, N, d], k_rot / v [B, Hkv, N, d], ``sel`` from ``dpxa_select``."""
    L.require_cuda(q_rot, k_rot, v, sel, out)
    B, Hq, N, D = q_rot.shape
    Hkv = k_rot.shape[1]
    if sm_scale is None:
        sm_scale = D ** -0.5
    if out is None:
        out = torch.empty((B, Hq, N, D), dtype=q_rot.dtype, device=q_rot.device)
    nb = -(-N // 128)
    if tuple(sel.shape) != (B, Hkv, nb, -(-nb // 32)) or not sel.is_contiguous():
        raise ValueError("block_sparse_attention: selection must be a contiguous [B, Hkv, nb, words] bitmask")
    lib = L.load()
    st = L.stream_of(q_rot)
    ws = L.workspace(q_rot.device, st.value, 256)
    strides = [*q_rot.stride(), *k_rot.stride(), *v.stride(), *out.stride()]
    L.check(lib.dab_block_sparse_attention(L.ptr(q_rot), L.ptr(k_rot), L.ptr(v), L.ptr(sel), L.ptr(out),
                                           L.dtype_code(q_rot), L.strides(strides), float(sm_scale), B, Hq, Hq // Hkv,
                                           N, D, L.ptr(ws), ws.numel(), st), "block_sparse_attention")
    return out


def dpxa_prefill(q, k, v, cos, sin, *, tau_q: float, tau_k: float, top_p: float, sm_scale=None):
    """One DPXA attention layer-op: RoPE(q, k), tile selection, block-sparse attention."""
    q_rot, k_rot = rope(q, cos, sin), rope(k, cos, sin)
    sel = dpxa_select(q_rot, k_rot, tau_q, tau_k, top_p, sm_scale)
    return block_sparse_attention(q_rot, k_rot, v, sel, sm_scale=sm_scale)


def proj_rope(x: torch.Tensor, w: torch.Tensor, cos: Optional[torch.Tensor] = None,
              sin: Optional[torch.Tensor] = None, rope_cols: Optional[tuple] = None,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q / k / v projection with RoPE as the GEMM epilogue (modeling_llama.py:550-555).

    ``x`` [rows, in] (the hidden states, rows = B*N), ``w`` [out, in] (nn.Linear weight, no
    bias), bf16. Returns [rows, out] = x @ w.T rounded to bf16, with RoPE (eager bf16
    rounding, table row r of ``cos`` / ``sin`` [rows, 128]) applied to the output columns in
    ``rope_cols`` = (lo, hi), by default all of them when tables are given. Viewed as
    [B, N, H, 128] and transposed, this is the reference's rotated ``key_states`` (or
    ``query_states``) in the projection layout the attention kernels read through strides.
    """
    L.require_cuda(x, w)
    rows, kin = x.shape
    nout = w.shape[0]
    if w.shape[1] != kin:
        raise ValueError(f"proj_rope: x has {kin} features, w expects {w.shape[1]}")
    if rope_cols is None:
        rope_cols = (0, nout) if cos is not None else (0, 0)
    lo, hi = rope_cols
    if hi > lo:
        if cos is None or sin is None:
            raise ValueError("proj_rope: RoPE columns given without cos / sin tables")
        L.require_cuda(cos, sin)
        cos = cos.reshape(-1, cos.shape[-1])
        sin = sin.reshape(-1, sin.shape[-1])
        if cos.shape[0] != rows or cos.stride() != sin.stride() or cos.stride(1) != 1:
            raise ValueError("proj_rope: cos / sin must be [rows, 128] with unit column stride and equal strides")
    if out is None:
        out = torch.empty((rows, nout), dtype=x.dtype, device=x.device)
    st = L.stream_of(x)
    ws = L.workspace(x.device, st.value, 256, tag="proj")
    L.check(L.load().dab_proj_rope(L.ptr(x), x.stride(0), L.ptr(w), w.stride(0),
                                   L.ptr(cos) if hi > lo else None, L.ptr(sin) if hi > lo else None,
                                   cos.stride(0) if hi > lo else 0, L.ptr(out), out.stride(0), L.dtype_code(x),
                                   rows, kin, nout, 128, lo, hi, L.ptr(ws), ws.numel(), st), "proj_rope")
    return out


@dataclass
class Packed:
    """Packed history of one layer: K/V rows, anchor timestamps and run-length counts.

    With ``anchors`` set (device packing without a host sync) the tensors have a capacity of
    rows per head and ``anchors`` [B * Hkv] int32 holds each head's kept count on the device;
    the reference's packed length is their maximum (``packed_length()`` reads it back)."""
    k: torch.Tensor          # [B, Hkv, M, d] (possibly a strided view), or [B, Hkv, capacity, d]
    v: torch.Tensor
    timestamps: torch.Tensor  # [B, Hkv, M] int32
    counts: torch.Tensor      # [B, Hkv, M] int32 (the reference's format)
    keep_mask: Optional[torch.Tensor] = None
    counts_f32: Optional[torch.Tensor] = None  # the same counts as fp32 (what attention weights with)
    anchors: Optional[torch.Tensor] = None     # [B * Hkv] int32 kept count per head (device length)

    def weights(self) -> torch.Tensor:
        if self.counts_f32 is None:
            self.counts_f32 = self.counts.float()
        return self.counts_f32

    def packed_length(self) -> int:
        """The reference's packed length M (a host read when the length lives on the device)."""
        if self.anchors is None:
            return self.k.shape[2]
        return int(self.anchors.max().item())

    def materialize(self) -> "Packed":
        """The reference's packed tensors (modeling_llama.py:655-685): every head cut to the
        packed length M, slots past its own anchors zero (K, V, timestamp, count). The packing
        itself when the length is already on the host; otherwise one host read of M."""
        if self.anchors is None:
            return self
        M = self.packed_length()
        B, H = self.k.shape[:2]
        valid = torch.arange(M, device=self.k.device)[None, None, :] < self.anchors.view(B, H, 1)
        zero = torch.zeros((), dtype=self.k.dtype, device=self.k.device)
        k = torch.where(valid[..., None], self.k[:, :, :M], zero)
        v = torch.where(valid[..., None], self.v[:, :, :M], zero)
        ts = torch.where(valid, self.timestamps[:, :, :M], 0).to(torch.int32)
        cnt = torch.where(valid, self.counts[:, :, :M], 0).to(torch.int32)
        return Packed(k, v, ts, cnt, self.keep_mask)


def pack_periodic(k_rot: torch.Tensor, v: torch.Tensor, period: int) -> Packed:
    """Periodic packing (modeling_llama.py:626-632 + :655-685) without copies."""
    L.require_cuda(k_rot, v)
    B, H, N, D = k_rot.shape
    M = -(-N // period)
    ts = torch.empty((B, H, M), dtype=torch.int32, device=k_rot.device)
    cnt = torch.empty_like(ts)
    cnt_f = torch.empty((B, H, M), dtype=torch.float32, device=k_rot.device)
    st = L.stream_of(k_rot)
    L.check(L.load().dab_periodic_meta(L.ptr(ts), L.ptr(cnt), L.ptr(cnt_f), B * H, M, N, period, st),
            "periodic_meta")
    return Packed(k_rot[:, :, ::period], v[:, :, ::period], ts, cnt, counts_f32=cnt_f)


def delta_keep_mask(k_rot: torch.Tensor, threshold: float, similarity: str = "euclidean", chunk_size: int = 512):
    """Delta selection (modeling_llama.py:634-653): keep mask and per-chunk anchor counts.

    ``threshold`` is the raw threshold; like the reference, only ``similarity == 'cosine'``
    selects cosine, every other value selects squared Euclidean with threshold**2.
    """
    from .launch import chunked_eval_kernel
    L.require_cuda(k_rot)
    B, H, N, D = k_rot.shape
    cs = min(chunk_size, N) if chunk_size > 0 else N
    nch = max(1, -(-N // cs))
    use_cos = similarity == "cosine"
    thr = threshold if use_cos else threshold ** 2
    # the scan writes every position and every chunk count
    keep = torch.empty((B, H, N), dtype=torch.int32, device=k_rot.device)
    cc = torch.empty((B, H, nch), dtype=torch.int32, device=k_rot.device)
    bd = 1 << max(4, (D - 1).bit_length())
    chunked_eval_kernel[(B * H, nch)](
        k_rot, keep, cc, thr, *k_rot.stride(), *keep.stride(), *cc.stride(), N, D, cs, num_heads=H,
        BLOCK_D=bd, USE_COSINE=use_cos)
    return keep, cc


def pack_from_keep(k_rot: torch.Tensor, v: torch.Tensor, keep: torch.Tensor, num_packed: Optional[int] = None,
                   want_index_map: bool = False) -> Packed:
    """Device-side index map + scatter + counts (modeling_llama.py:655-685)."""
    L.require_cuda(k_rot, v, keep)
    B, H, N, D = k_rot.shape
    if num_packed is None:
        num_packed = int(keep.sum(-1).max().item())  # the reference's packed length (modeling_llama.py:656)
    M = int(num_packed)
    dev = k_rot.device
    # every slot is written by the library (padding past a head's anchors with zeros)
    kp = torch.empty((B, H, M, D), dtype=k_rot.dtype, device=dev)
    vp = torch.empty_like(kp)
    ts = torch.empty((B, H, M), dtype=torch.int32, device=dev)
    cnt = torch.empty_like(ts)
    anchors = torch.empty((B * H,), dtype=torch.int32, device=dev)
    mx = torch.empty((1,), dtype=torch.int32, device=dev)
    im = torch.empty((B, H, N), dtype=torch.int32, device=dev) if want_index_map else None
    lib = L.load()
    st = L.stream_of(k_rot)
    ws = L.workspace(dev, st.value, int(lib.dab_pack_from_keep_workspace_size(B, H, N)), tag="pack")
    L.check(lib.dab_pack_from_keep(
        L.ptr(keep), L.strides(keep.stride()), L.ptr(k_rot), L.strides(k_rot.stride()), L.ptr(v),
        L.strides(v.stride()), L.ptr(kp), L.ptr(vp), L.strides(kp.stride()), L.ptr(ts), L.ptr(cnt),
        L.strides(ts.stride()), L.ptr(im), L.dtype_code(k_rot), B, H, N, D, M, L.ptr(anchors), L.ptr(mx),
        L.ptr(ws), ws.numel(), st), "pack_from_keep")
    p = Packed(kp, vp, ts, cnt, keep)
    p.index_map = im
    return p


def delta_compress(k, v, cos, sin, threshold: float, similarity: str = "euclidean", chunk_size: int = 512,
                   capacity: Optional[int] = None, want_keep_mask: bool = True):
    """RoPE, delta selection and packing of one layer's keys in one launch, with no host sync
    (modeling_llama.py:555 + :600-685; the reference reads the packed length back at :656).

    k / v [B, Hkv, N, d] pre-RoPE keys and values (any 16-byte-aligned row layout, e.g. the
    projection layout); cos / sin [1 or B, N, d]. ``threshold`` is the raw threshold as in
    ``delta_keep_mask`` (squared for Euclidean). Returns (rotated keys [B, Hkv, N, d], Packed
    with ``anchors`` on the device and ``capacity`` rows per head, default N rounded up to 128).
    """
    L.require_cuda(k, v, cos, sin)
    B, H, N, D = k.shape
    cap = int(capacity) if capacity is not None else max(128, -(-N // 128) * 128)
    dev = k.device
    use_cos = similarity == "cosine"
    thr = threshold if use_cos else threshold ** 2
    cs = min(chunk_size, N) if chunk_size > 0 else N
    k_rot = torch.empty((B, H, N, D), dtype=k.dtype, device=dev)
    kp = torch.empty((B, H, cap, D), dtype=k.dtype, device=dev)
    vp = torch.empty_like(kp)
    ts = torch.empty((B, H, cap), dtype=torch.int32, device=dev)
    cnt = torch.empty_like(ts)
    cnt_f = torch.empty((B, H, cap), dtype=torch.float32, device=dev)
    anchors = torch.empty((B * H,), dtype=torch.int32, device=dev)
    keep = torch.empty((B, H, N), dtype=torch.int32, device=dev) if want_keep_mask else None
    if cos.stride() != sin.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    cb = cos.stride(0) if cos.shape[0] > 1 else 0
    lib = L.load()
    st = L.stream_of(k)
    ws = L.workspace(dev, st.value, lib.dab_delta_compress_workspace_size(B, H, N, cs), tag="compress")
    L.check(lib.dab_delta_compress(
        L.ptr(k), L.strides(k.stride()), L.ptr(v), L.strides(v.stride()), L.ptr(cos), L.ptr(sin),
        L.strides([cb, cos.stride(1), cos.stride(2)]), L.ptr(k_rot), L.strides(k_rot.stride()), L.ptr(keep),
        L.strides(keep.stride() if keep is not None else (0, 0, 0)), L.ptr(kp), L.ptr(vp), L.strides(kp.stride()),
        L.ptr(ts), L.ptr(cnt), L.ptr(cnt_f), L.strides(ts.stride()), L.ptr(anchors), L.dtype_code(k), B, H, N, D,
        float(thr), 1 if use_cos else 0, cs, cap, L.ptr(ws), ws.numel(), st), "delta_compress")
    return k_rot, Packed(kp, vp, ts, cnt, keep, counts_f32=cnt_f, anchors=anchors)


def fused_delta_ok(k, v, cos) -> bool:
    """Whether ``delta_compress`` and the device-length attention take these tensors (bf16 /
    fp16, head_dim 64 / 128, contiguous 16-byte-aligned rows)."""
    if k.dtype not in (torch.bfloat16, torch.float16) or k.shape[-1] not in (64, 128):
        return False
    for t in (k, v, cos):
        if t.stride(-1) != 1 or t.data_ptr() % 16 or any((st * 2) % 16 for st in t.stride()[:-1]):
            return False
    return True


def attention(q_rot, k_rot, v, packed: Optional[Packed], *, sm_scale=None, dense_window=128,
              variant="hybrid", out=None, force_simt=False):
    """Two-phase count-weighted attention (deltaFlashAttention.py:9-357) with GQA by index.

    q_rot [B, Hq, N, d]; k_rot / v / packed tensors [B, Hkv, ...]; out any [B, Hq, N, d] view.
    """
    L.require_cuda(q_rot, k_rot, v, out)
    B, Hq, N, D = q_rot.shape
    Hkv = k_rot.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must be a multiple of kv heads")
    if sm_scale is None:
        sm_scale = D ** -0.5
    if out is None:
        out = torch.empty((B, Hq, N, D), dtype=q_rot.dtype, device=q_rot.device)
    M = packed.k.shape[2] if packed is not None else 0
    kp = packed.k if packed is not None else k_rot
    vp = packed.v if packed is not None else v
    ts = packed.timestamps if packed is not None else torch.zeros((B, Hkv, 1), dtype=torch.int32,
                                                                   device=q_rot.device)
    cnt = packed.weights() if packed is not None else ts
    lib = L.load()
    st = L.stream_of(q_rot)
    wsb = lib.dab_hybrid_flash_workspace_size(B, Hkv, N, M)
    ws = L.workspace(q_rot.device, st.value, wsb)
    bd = 1 << max(4, (D - 1).bit_length())
    strides = [*q_rot.stride(), *k_rot.stride(), *v.stride(), *kp.stride(), *vp.stride(), *ts.stride(),
               *cnt.stride(), *out.stride()]
    if packed is not None and packed.anchors is not None:
        # packed length on the device (capacity rows per head; M = max of the anchors)
        if force_simt:
            raise ValueError("attention: a device packed length runs on the tcgen05 kernel only")
        L.check(lib.dab_hybrid_flash_devlen(
            VARIANTS[variant], L.ptr(q_rot), L.ptr(k_rot), L.ptr(v), L.ptr(kp), L.ptr(vp), L.ptr(ts), L.ptr(cnt),
            1 if cnt.dtype == torch.int32 else 0, L.ptr(packed.anchors), L.ptr(out), L.dtype_code(q_rot),
            L.strides(strides), float(sm_scale), N, k_rot.shape[2], M, D, Hq, int(dense_window), -(-N // 128),
            B * Hq, 128, 128, bd, Hq // Hkv, L.ptr(ws), ws.numel(), st), "attention")
        return out
    L.check(lib.dab_hybrid_flash(
        VARIANTS[variant], L.ptr(q_rot), L.ptr(k_rot), L.ptr(v), L.ptr(kp), L.ptr(vp), L.ptr(ts), L.ptr(cnt),
        1 if cnt.dtype == torch.int32 else 0, L.ptr(out), L.dtype_code(q_rot), L.strides(strides), float(sm_scale),
        N, k_rot.shape[2], M, D, Hq, int(dense_window), -(-N // 128), B * Hq, 128, 128, bd, Hq // Hkv, L.ptr(ws),
        ws.numel(), 1 if force_simt else 0, st), "attention")
    return out


def flash(q_rot, k_rot, v, *, causal=True, sm_scale=None, out=None, force_simt=False):
    """Dense flash attention (flashAttention.py:5-91) with GQA by index: the r = 1 comparator."""
    L.require_cuda(q_rot, k_rot, v, out)
    B, Hq, N, D = q_rot.shape
    Hkv = k_rot.shape[1]
    if sm_scale is None:
        sm_scale = D ** -0.5
    if out is None:
        out = torch.empty((B, Hq, N, D), dtype=q_rot.dtype, device=q_rot.device)
    lib = L.load()
    st = L.stream_of(q_rot)
    wsb = lib.dab_hybrid_flash_workspace_size(B, Hkv, N, 0)
    ws = L.workspace(q_rot.device, st.value, wsb)
    strides = [*q_rot.stride(), *k_rot.stride(), *v.stride(), *out.stride()]
    L.check(lib.dab_attn_fwd_flat(
        L.ptr(q_rot), L.ptr(k_rot), L.ptr(v), float(sm_scale), L.ptr(out), L.dtype_code(q_rot), L.strides(strides),
        B, Hq, N, D, 128, 128, 1 if causal else 0, -(-N // 128), B * Hq, Hq // Hkv, L.ptr(ws), ws.numel(),
        1 if force_simt else 0, st), "flash")
    return out


def delta_prefill(q, k, v, cos, sin, *, mode="periodic", keep_rate=0.25, threshold=None,
                  similarity="euclidean", chunk_size=512, dense_window=128, variant="hybrid", sm_scale=None,
                  out=None, keep_mask=None, return_packed=False, fused=True):
    """The whole delta-attention prefill layer-op on pre-RoPE q / k and v.

    q [B, Hq, N, d], k / v [B, Hkv, N, d] (any strides, e.g. the [B, N, H, d] projection
    layout viewed with transpose(1, 2)). mode: 'periodic' (keep t % round(1/keep_rate) == 0),
    'delta' (threshold selection in chunks of ``chunk_size``) or 'mask' (``keep_mask``).
    In delta mode with bf16 / fp16 keys of head_dim 64 / 128 (and ``fused``), RoPE(k),
    selection and packing are one launch (``delta_compress``) and the packed length stays on
    the device, so the layer-op makes no host sync; otherwise they run as separate kernels and
    the packed length is read back as the reference does (modeling_llama.py:656).
    Returns the attention output [B, Hq, N, d] (and the packed history when requested).
    """
    L.require_cuda(q, k, v, cos, sin)
    q_rot = rope(q, cos, sin)
    fused_delta = mode == "delta" and fused and fused_delta_ok(k, v, cos)
    k_rot = None if fused_delta else rope(k, cos, sin)
    if mode == "periodic":
        period = max(1, round(1.0 / keep_rate))
        packed = pack_periodic(k_rot, v, period)
    elif mode == "delta":
        if threshold is None:
            raise ValueError("delta mode needs a threshold")
        if fused_delta:
            # one launch for RoPE(k), selection and packing; the packed length stays on the device
            k_rot, packed = delta_compress(k, v, cos, sin, threshold, similarity, chunk_size)
        else:
            keep, _ = delta_keep_mask(k_rot, threshold, similarity, chunk_size)
            packed = pack_from_keep(k_rot, v, keep)
    elif mode == "mask":
        packed = pack_from_keep(k_rot, v, keep_mask.to(torch.int32))
    else:
        raise ValueError(f"unknown mode {mode}")
    o = attention(q_rot, k_rot, v, packed, sm_scale=sm_scale, dense_window=dense_window, variant=variant, out=out)
    if return_packed:
        return o, packed, k_rot
    return o


_varlen_streams = {}


def delta_prefill_varlen(q, k, v, cos, sin, cu_seqlens, *, selection="nm", n=2, m=4, ratio=4, keep_rate=0.25,
                         dense_window=128, sm_scale=None, out=None, streams=3, return_packed=False):
    """The delta-attention prefill layer-op over sequences packed back to back (cu_seqlens).

    q [1, Hq, T, d] and k / v [1, Hkv, T, d] (any strides, e.g. the [T, H, d] projection
    output viewed as [1, H, T, d]) hold the sequences at offsets ``cu_seqlens`` (a host list
    of B + 1 increasing ints, cu_seqlens[-1] = T); cos / sin are tables of at least the
    longest sequence (positions restart at 0 in every sequence). Every sequence runs RoPE,
    its own selection (``selection="nm"``: n:m structured at ``ratio``, the
    nmDeltaFlashAttention variant; ``"periodic"``: keep t % round(1 / keep_rate) == 0), packing
    and the two-phase attention, exactly as ``delta_prefill`` on that sequence alone.
    Sequences go round-robin to ``streams`` CUDA streams, so one sequence's RoPE / selection /
    packing overlaps another's attention; the caller's current stream is waited on first and
    waits for every stream before this returns.

    Returns out [1, Hq, T, d] (allocated when not given), and with ``return_packed`` also the
    list of per-sequence (Packed, post-RoPE keys) for the decode-cache hand-off.
    """
    from .dropin.nmDeltaFlashAttention import nm_keep_mask, nm_num_packed
    # argument checks first (host logic only), then the device requirement
    if q.shape[0] != 1 or k.shape[0] != 1:
        raise ValueError("delta_prefill_varlen: sequences are packed along dim 2 of [1, H, T, d] tensors")
    cu = [int(x) for x in cu_seqlens]
    T = q.shape[2]
    if len(cu) < 2 or cu[0] != 0 or cu[-1] != T or any(b <= a for a, b in zip(cu, cu[1:])):
        raise ValueError("delta_prefill_varlen: cu_seqlens must rise strictly from 0 to the packed length")
    if max(b - a for a, b in zip(cu, cu[1:])) > cos.shape[-2]:
        raise ValueError("delta_prefill_varlen: cos / sin are shorter than the longest sequence")
    if selection not in ("nm", "periodic"):
        raise ValueError(f"delta_prefill_varlen: unknown selection {selection}")
    L.require_cuda(q, k, v, cos, sin, out)
    dev = q.device
    if out is None:
        out = torch.empty((1, q.shape[1], T, q.shape[3]), dtype=q.dtype, device=dev)
    cur = torch.cuda.current_stream(dev)
    ns = max(1, int(streams))
    pool = _varlen_streams.setdefault(dev.index, [])
    while len(pool) < ns:
        pool.append(torch.cuda.Stream(dev))
    for s in pool[:ns]:
        s.wait_stream(cur)
    packed = []
    for i, (s0, s1) in enumerate(zip(cu, cu[1:])):
        st = pool[i % ns]
        with torch.cuda.stream(st):
            q_rot = rope(q[:, :, s0:s1], cos, sin)
            k_rot = rope(k[:, :, s0:s1], cos, sin)
            vi = v[:, :, s0:s1]
            if selection == "nm":
                keep = nm_keep_mask(k_rot, n, m, ratio)
                pk = pack_from_keep(k_rot, vi, keep, num_packed=nm_num_packed(s1 - s0, n, m, ratio))
            else:
                pk = pack_periodic(k_rot, vi, max(1, round(1.0 / keep_rate)))
            attention(q_rot, k_rot, vi, pk, sm_scale=sm_scale, dense_window=dense_window, out=out[:, :, s0:s1])
            if return_packed:
                # handed to the caller's stream: keep the allocator from reusing them early
                for t in (pk.k, pk.v, pk.timestamps, pk.counts, pk.counts_f32, k_rot):
                    if t is not None:
                        t.record_stream(cur)
                packed.append((pk, k_rot))
    for s in pool[:ns]:
        cur.wait_stream(s)
    return (out, packed) if return_packed else out


_side_streams = {}


def _streams_for(dev: torch.device):
    """One host->device and one device->host copy stream per device, created on first use."""
    key = dev.index
    if key not in _side_streams:
        _side_streams[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _side_streams[key]


def delta_prefill_host(q, k, v, cos, sin, *, out, kv_heads_per_group=1, q_heads_per_group=None, **kw):
    """delta_prefill on host-resident inputs, writing a host-resident output.

    q [B, Hq, N, d], k / v [B, Hkv, N, d] and out [B, Hq, N, d] are CPU tensors in head-major
    layout, pinned (``pin_memory()``) so that the copies run asynchronously; cos / sin are
    the device RoPE tables. Keyword arguments go to ``delta_prefill``.

    Every kv-head (with its group of query heads) is independent in this layer-op with periodic
    selection: packing and attention of kv-head h read only k / v head h and q heads
    h*G .. h*G+G-1. The
    heads are therefore processed in groups of ``kv_heads_per_group`` kv-heads (or, with
    ``q_heads_per_group`` below a kv-head's query-head count, groups of that many query heads
    of one kv-head, whose K / V are copied with its first group), and group g's
    host->device copies, group g-1's compute and group g-2's device->host copy run at the same
    time on three streams. Results equal one ``delta_prefill`` call on the whole tensors.

    Ordering: the current stream waits for the last device->host copy before this returns, so
    work enqueued on the current stream afterwards (an event, a synchronize) covers the whole
    layer-op. The device buffers are kept between calls with the same shapes (one set per
    device and shape; ``release_host_prefill_buffers`` frees them), and each group's next
    host->device copy waits only for this call's compute of the groups that read those
    buffers, so consecutive calls overlap: the next call's copies start while this call's
    last groups are still computing and draining.

    Only ``mode="periodic"``: the delta and mask modes size the packed history by the largest
    kept count over all heads (modeling_llama.py:656), and a head's padding changes its
    schedule, so their heads are not independent.
    """
    if kw.get("mode", "periodic") != "periodic":
        raise ValueError("delta_prefill_host: only mode='periodic' splits by kv-head (the delta and mask "
                         "modes pad every head to the largest kept count); use delta_prefill")
    for t in (q, k, v, out):
        if t.is_cuda or not t.is_pinned():
            raise RuntimeError("delta_prefill_host: q, k, v and out must be pinned host tensors")
    L.require_cuda(cos, sin)
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if Hq % Hkv or tuple(out.shape) != (B, Hq, N, D) or k.shape != v.shape or k.shape[0] != B:
        raise ValueError("delta_prefill_host: shapes must be q/out [B, Hq, N, d], k/v [B, Hkv, N, d]")
    G = Hq // Hkv
    dev = cos.device
    cur = torch.cuda.current_stream(dev)
    h2d, d2h = _streams_for(dev)
    # groups: (kv-heads [a, b), query heads [qa, qb), copy K / V of [a, b) with this group)
    qg = G if q_heads_per_group is None else int(q_heads_per_group)
    if 1 <= qg < G:
        if G % qg:
            raise ValueError("delta_prefill_host: q_heads_per_group must divide the query heads per kv-head")
        groups = [(a, a + 1, a * G + s, a * G + s + qg, s == 0) for a in range(Hkv) for s in range(0, G, qg)]
    else:
        step = max(1, int(kv_heads_per_group))
        groups = [(a, min(Hkv, a + step), a * G, min(Hkv, a + step) * G, True) for a in range(0, Hkv, step)]
    key = (dev.index, tuple(q.shape), tuple(k.shape), q.dtype, tuple(groups))
    ws = _host_ws.get(key)
    if ws is None:
        ws = {"dq": torch.empty(q.shape, dtype=q.dtype, device=dev),
              "dk": torch.empty(k.shape, dtype=k.dtype, device=dev),
              "dv": torch.empty(v.shape, dtype=v.dtype, device=dev),
              "do": torch.empty(out.shape, dtype=out.dtype, device=dev),
              "computed": [None] * len(groups), "drained": [None] * len(groups)}
        _host_ws[key] = ws
        # the buffers come from the current stream's pool: the copy streams start after it
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
    dq, dk, dv, do = ws["dq"], ws["dk"], ws["dv"], ws["do"]
    computed, drained = ws["computed"], ws["drained"]
    ev_in = []
    with torch.cuda.stream(h2d):
        for gi, (a, b, qa, qb, with_kv) in enumerate(groups):
            # overwrite this group's buffers once the previous call's compute has read them (K / V
            # of [a, b) are read by every group of those kv-heads)
            for gj, (a2, b2, _, _, _) in enumerate(groups):
                if computed[gj] is not None and (gj == gi or (with_kv and a2 < b and a < b2)):
                    h2d.wait_event(computed[gj])
            for bi in range(B):
                if with_kv:
                    dk[bi, a:b].copy_(k[bi, a:b], non_blocking=True)
                    dv[bi, a:b].copy_(v[bi, a:b], non_blocking=True)
                dq[bi, qa:qb].copy_(q[bi, qa:qb], non_blocking=True)
            e = torch.cuda.Event()
            e.record(h2d)
            ev_in.append(e)
    for gi, ((a, b, qa, qb, _), e) in enumerate(zip(groups, ev_in)):
        cur.wait_event(e)
        if drained[gi] is not None:
            cur.wait_event(drained[gi])  # the previous call's output of this group has left
        delta_prefill(dq[:, qa:qb], dk[:, a:b], dv[:, a:b], cos, sin, out=do[:, qa:qb], **kw)
        done = torch.cuda.Event()
        done.record(cur)
        computed[gi] = done
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            for bi in range(B):
                out[bi, qa:qb].copy_(do[bi, qa:qb], non_blocking=True)
            dr = torch.cuda.Event()
            dr.record(d2h)
            drained[gi] = dr
    cur.wait_stream(d2h)
    return out


_host_ws = {}


def release_host_prefill_buffers():
    """Free the device buffers ``delta_prefill_host`` keeps between calls (after the work that
    uses them has finished)."""
    _host_ws.clear()


def tile_count_periodic(N: int, r: int, W: int = 128) -> int:
    """128x128 tiles one head runs under the reference schedule with periodic-r packing."""
    nb = -(-N // 128)
    if r == 1:
        return nb * (nb + 1) // 2
    M = -(-N // r)
    nblk = -(-M // 128)
    T = [min(128 * j + 127, M - 1) * r if 128 * j + 127 < M else N + 1 for j in range(nblk)]
    tot = 0
    for mb in range(nb):
        thr = 128 * mb - W
        n1 = 0
        while n1 < nblk and T[n1] < thr:
            n1 += 1
        last = T[n1 - 1] if n1 else -1
        ds = max(0, (last + 1) // 128)
        de = -(-min(N, 128 * mb + 128) // 128)
        tot += n1 + max(0, de - ds)
    return tot


_ = math

"""Kernel objects with the reference's Triton launch syntax: ``kernel[grid](*args, **meta)``.

Each object binds the exact parameter list of the reference kernel it replaces (names,
order, constexpr keywords; ``num_warps`` / ``num_stages`` are accepted and ignored) and
forwards to the CUDA library through the C ABI. The grid is honoured: it selects which
(head, block) programs run, as in the reference.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L

_META_IGNORED = {"num_warps", "num_stages", "num_ctas", "maxnreg", "enable_fp_fusion"}


def _bind(params, args, kwargs, name):
    kw = {k: v for k, v in kwargs.items() if k not in _META_IGNORED}
    if len(args) > len(params):
        raise TypeError(f"{name}: too many positional arguments")
    bound = dict(zip(params, args))
    for k, v in kw.items():
        if k in bound:
            raise TypeError(f"{name}: duplicate argument {k}")
        if k not in params:
            raise TypeError(f"{name}: unexpected argument {k}")
        bound[k] = v
    missing = [p for p in params if p not in bound]
    if missing:
        raise TypeError(f"{name}: missing arguments {missing}")
    return bound


def _grid(grid, bound):
    g = grid(bound) if callable(grid) else grid
    g = tuple(int(x) for x in g)
    return g + (1,) * (3 - len(g))


class KernelShim:
    """``shim[grid](...)`` calls ``impl(grid_tuple, bound_args)``."""

    def __init__(self, name, params, impl):
        self.__name__ = name
        self.params = list(params)
        self._impl = impl

    def __getitem__(self, grid):
        def launch(*args, **kwargs):
            b = _bind(self.params, args, kwargs, self.__name__)
            return self._impl(_grid(grid, b), b)
        return launch

    def __repr__(self):
        return f"<deltaattention_b200 kernel {self.__name__}>"


def _f(b, k):
    return float(b[k])


def _i(b, k):
    return int(b[k])


# ---------------------------------------------------------------- tritonModules.py:7-69
CHUNKED_EVAL_PARAMS = [
    "in_ptr", "keep_mask_ptr", "chunk_counts_ptr", "threshold_sq",
    "stride_in_b", "stride_in_h", "stride_in_s", "stride_in_d",
    "stride_km_b", "stride_km_h", "stride_km_s",
    "stride_cc_b", "stride_cc_h", "stride_cc_c",
    "seq_len", "head_dim", "chunk_size", "num_heads", "BLOCK_D", "USE_COSINE",
]


def _chunked_eval(grid, b):
    x, km, cc = b["in_ptr"], b["keep_mask_ptr"], b["chunk_counts_ptr"]
    L.require_cuda(x, km, cc)
    lib = L.load()
    st = L.stream_of(x)
    L.check(lib.dab_chunked_eval(
        L.ptr(x), L.dtype_code(x),
        L.strides([b["stride_in_b"], b["stride_in_h"], b["stride_in_s"], b["stride_in_d"]]),
        L.ptr(km), L.strides([b["stride_km_b"], b["stride_km_h"], b["stride_km_s"]]),
        L.ptr(cc), L.strides([b["stride_cc_b"], b["stride_cc_h"], b["stride_cc_c"]]),
        _f(b, "threshold_sq"), _i(b, "seq_len"), _i(b, "head_dim"), _i(b, "chunk_size"), _i(b, "num_heads"),
        grid[0], grid[1], _i(b, "BLOCK_D"), 1 if b["USE_COSINE"] else 0, st), "chunked_eval_kernel")


chunked_eval_kernel = KernelShim("chunked_eval_kernel", CHUNKED_EVAL_PARAMS, _chunked_eval)

# ---------------------------------------------------------------- tritonModules.py:72-132
SCATTER_PARAMS = [
    "k_in_ptr", "v_in_ptr", "k_packed_ptr", "v_packed_ptr", "pt_ptr", "keep_mask_ptr", "index_map_ptr",
    "stride_kb", "stride_kh", "stride_ks", "stride_kd",
    "stride_vb", "stride_vh", "stride_vs", "stride_vd",
    "stride_kpb", "stride_kph", "stride_kpa", "stride_kpd",
    "stride_vpb", "stride_vph", "stride_vpa", "stride_vpd",
    "stride_ptb", "stride_pth", "stride_pta",
    "stride_km_b", "stride_km_h", "stride_km_s",
    "stride_im_b", "stride_im_h", "stride_im_s",
    "seq_len", "head_dim", "num_heads", "BLOCK_S", "BLOCK_D",
]


def _scatter(grid, b):
    k, v, kp, vp, pt = b["k_in_ptr"], b["v_in_ptr"], b["k_packed_ptr"], b["v_packed_ptr"], b["pt_ptr"]
    km, im = b["keep_mask_ptr"], b["index_map_ptr"]
    L.require_cuda(k, v, kp, vp, pt, km, im)
    if not (k.dtype == v.dtype == kp.dtype == vp.dtype):
        raise TypeError("parallel_scatter_pack_kv_kernel: K/V/packed dtypes differ")
    num_packed = int(kp.shape[-2]) if kp.dim() >= 2 else 0
    lib = L.load()
    st = L.stream_of(k)
    s = lambda *names: L.strides([b[n] for n in names])  # noqa: E731
    L.check(lib.dab_parallel_scatter_pack_kv(
        L.ptr(k), L.ptr(v), L.ptr(kp), L.ptr(vp), L.ptr(pt), L.ptr(km), L.ptr(im), L.dtype_code(k),
        s("stride_kb", "stride_kh", "stride_ks", "stride_kd"), s("stride_vb", "stride_vh", "stride_vs", "stride_vd"),
        s("stride_kpb", "stride_kph", "stride_kpa", "stride_kpd"),
        s("stride_vpb", "stride_vph", "stride_vpa", "stride_vpd"),
        s("stride_ptb", "stride_pth", "stride_pta"), s("stride_km_b", "stride_km_h", "stride_km_s"),
        s("stride_im_b", "stride_im_h", "stride_im_s"),
        _i(b, "seq_len"), _i(b, "head_dim"), _i(b, "num_heads"), num_packed, grid[0], grid[1], _i(b, "BLOCK_S"),
        st), "parallel_scatter_pack_kv_kernel")


parallel_scatter_pack_kv_kernel = KernelShim("parallel_scatter_pack_kv_kernel", SCATTER_PARAMS, _scatter)

# ---------------------------------------------------------------- deltaFlashAttention.py:10-26
HYBRID_PARAMS = [
    "Q", "K_dense", "V_dense", "K_packed", "V_packed", "Packed_Timestamps", "Packed_Counts", "Out",
    "stride_qb", "stride_qh", "stride_qm", "stride_qd",
    "stride_kdb", "stride_kdh", "stride_kdn", "stride_kdd",
    "stride_vdb", "stride_vdh", "stride_vdn", "stride_vdd",
    "stride_kpb", "stride_kph", "stride_kpn", "stride_kpd",
    "stride_vpb", "stride_vph", "stride_vpn", "stride_vpd",
    "stride_ptb", "stride_pth", "stride_ptn",
    "stride_pcb", "stride_pch", "stride_pcn",
    "stride_ob", "stride_oh", "stride_om", "stride_od",
    "sm_scale", "seq_len_q", "seq_len_k", "num_packed_keys", "head_dim", "num_heads", "denseWindowSize",
    "BLOCK_M", "BLOCK_N", "BLOCK_D",
]
_STRIDE_NAMES = HYBRID_PARAMS[8:38]


def hybrid_call(variant, grid, b, kv_group=1, force_simt=False):
    q, kd, vd = b["Q"], b["K_dense"], b["V_dense"]
    kp, vp, ts, pc, out = b["K_packed"], b["V_packed"], b["Packed_Timestamps"], b["Packed_Counts"], b["Out"]
    L.require_cuda(q, kd, vd, kp, vp, ts, pc, out)
    if not (q.dtype == kd.dtype == vd.dtype == out.dtype):
        raise TypeError("hybrid flash: Q/K/V/Out dtypes differ")
    if ts.dtype != torch.int32:
        raise TypeError("hybrid flash: Packed_Timestamps must be int32")
    if pc.dtype not in (torch.float32, torch.int32):
        raise TypeError("hybrid flash: Packed_Counts must be float32 or int32")
    num_heads = _i(b, "num_heads")
    B = grid[1] // num_heads if num_heads else 0
    M = _i(b, "num_packed_keys")
    lib = L.load()
    st = L.stream_of(q)
    ws_bytes = lib.dab_hybrid_flash_workspace_size(B, num_heads // kv_group, _i(b, "seq_len_q"), M)
    ws = L.workspace(q.device, st.value, ws_bytes)
    L.check(lib.dab_hybrid_flash(
        variant, L.ptr(q), L.ptr(kd), L.ptr(vd), L.ptr(kp), L.ptr(vp), L.ptr(ts), L.ptr(pc),
        1 if pc.dtype == torch.int32 else 0, L.ptr(out), L.dtype_code(q),
        L.strides([b[n] for n in _STRIDE_NAMES]), _f(b, "sm_scale"), _i(b, "seq_len_q"), _i(b, "seq_len_k"),
        M, _i(b, "head_dim"), num_heads, _i(b, "denseWindowSize"), grid[0], grid[1], _i(b, "BLOCK_M"),
        _i(b, "BLOCK_N"), _i(b, "BLOCK_D"), kv_group, L.ptr(ws), ws.numel(), 1 if force_simt else 0, st),
        "hybrid_compressed_flash_kernel")
    return ws


hybrid_compressed_flash_kernel = KernelShim(
    "hybrid_compressed_flash_kernel", HYBRID_PARAMS, lambda g, b: hybrid_call(0, g, b))
hybrid_compressed_flash_kernel_sanity = KernelShim(
    "hybrid_compressed_flash_kernel_sanity", HYBRID_PARAMS, lambda g, b: hybrid_call(1, g, b))
pure_phase1_flash_kernel = KernelShim(
    "pure_phase1_flash_kernel", HYBRID_PARAMS, lambda g, b: hybrid_call(2, g, b))

# ---------------------------------------------------------------- flashAttention.py:6-17
FLAT_PARAMS = [
    "Q", "K", "V", "sm_scale", "Out",
    "stride_qz", "stride_qh", "stride_qm", "stride_qk",
    "stride_kz", "stride_kh", "stride_kn", "stride_kk",
    "stride_vz", "stride_vh", "stride_vk", "stride_vn",
    "stride_oz", "stride_oh", "stride_om", "stride_on",
    "Z", "H", "N_CTX", "HEAD_DIM", "BLOCK_M", "BLOCK_N", "IS_CAUSAL",
]


def flat_call(grid, b, kv_group=1, force_simt=False):
    q, k, v, out = b["Q"], b["K"], b["V"], b["Out"]
    L.require_cuda(q, k, v, out)
    if not (q.dtype == k.dtype == v.dtype == out.dtype):
        raise TypeError("_attn_fwd_flat: dtypes differ")
    H = _i(b, "H")
    lib = L.load()
    st = L.stream_of(q)
    ws_bytes = lib.dab_hybrid_flash_workspace_size(max(grid[1] // H, 1), H // kv_group, _i(b, "N_CTX"), 0)
    ws = L.workspace(q.device, st.value, ws_bytes)
    L.check(lib.dab_attn_fwd_flat(
        L.ptr(q), L.ptr(k), L.ptr(v), _f(b, "sm_scale"), L.ptr(out), L.dtype_code(q),
        L.strides([b[n] for n in FLAT_PARAMS[5:21]]), _i(b, "Z"), H, _i(b, "N_CTX"), _i(b, "HEAD_DIM"),
        _i(b, "BLOCK_M"), _i(b, "BLOCK_N"), 1 if b["IS_CAUSAL"] else 0, grid[0], grid[1], kv_group, L.ptr(ws),
        ws.numel(), 1 if force_simt else 0, st), "_attn_fwd_flat")


_attn_fwd_flat = KernelShim("_attn_fwd_flat", FLAT_PARAMS, flat_call)

# ---------------------------------------------------------------- deltaDecoding.py:10-22
UPDATE_PARAMS = [
    "new_k_ptr", "new_v_ptr", "k_exact_ptr", "v_exact_ptr", "k_packed_ptr", "v_packed_ptr",
    "packed_counts_ptr", "packed_timestamps_ptr", "packed_lengths_ptr",
    "exact_seq_len", "total_seq_len", "threshold_sq", "exact_window_size",
    "stride_new_b", "stride_new_h", "stride_new_s", "stride_new_d",
    "stride_exact_b", "stride_exact_h", "stride_exact_s", "stride_exact_d",
    "stride_pack_b", "stride_pack_h", "stride_pack_s", "stride_pack_d",
    "stride_pc_b", "stride_pc_h", "stride_pc_s",
    "num_heads", "head_dim", "BLOCK_D", "USE_COSINE",
]


def _update(grid, b):
    nk, nv, ke, ve = b["new_k_ptr"], b["new_v_ptr"], b["k_exact_ptr"], b["v_exact_ptr"]
    kp, vp = b["k_packed_ptr"], b["v_packed_ptr"]
    pc, pt, pl = b["packed_counts_ptr"], b["packed_timestamps_ptr"], b["packed_lengths_ptr"]
    L.require_cuda(nk, nv, ke, ve, kp, vp, pc, pt, pl)
    lib = L.load()
    st = L.stream_of(nk)
    s = lambda *names: L.strides([b[n] for n in names])  # noqa: E731
    capacity = int(kp.shape[-2])
    L.check(lib.dab_decode_update(
        L.ptr(nk), L.ptr(nv), L.ptr(ke), L.ptr(ve), L.ptr(kp), L.ptr(vp), L.ptr(pc), L.ptr(pt), L.ptr(pl),
        _i(b, "exact_seq_len"), _i(b, "total_seq_len"), _f(b, "threshold_sq"), _i(b, "exact_window_size"),
        L.dtype_code(nk), s("stride_new_b", "stride_new_h", "stride_new_s", "stride_new_d"),
        s("stride_exact_b", "stride_exact_h", "stride_exact_s", "stride_exact_d"),
        s("stride_pack_b", "stride_pack_h", "stride_pack_s", "stride_pack_d"),
        s("stride_pc_b", "stride_pc_h", "stride_pc_s"), _i(b, "num_heads"), _i(b, "head_dim"), _i(b, "BLOCK_D"),
        1 if b["USE_COSINE"] else 0, grid[0], capacity, None, st), "fused_hybrid_decode_update_kernel")


fused_hybrid_decode_update_kernel = KernelShim("fused_hybrid_decode_update_kernel", UPDATE_PARAMS, _update)

# ---------------------------------------------------------------- deltaDecoding.py:237-259
DECODE_PARAMS = [
    "Q", "K_packed", "V_packed", "Packed_Counts", "Packed_Lengths", "K_exact", "V_exact", "Out",
    "stride_qb", "stride_qh", "stride_qd",
    "stride_kpb", "stride_kph", "stride_kpn", "stride_kpd",
    "stride_vpb", "stride_vph", "stride_vpn", "stride_vpd",
    "stride_cb", "stride_ch", "stride_cn",
    "stride_lb", "stride_lh",
    "stride_keb", "stride_keh", "stride_ken", "stride_ked",
    "stride_veb", "stride_veh", "stride_ven", "stride_ved",
    "stride_ob", "stride_oh", "stride_od",
    "sm_scale", "exact_len", "num_kv_groups", "head_dim", "BLOCK_M", "BLOCK_N", "BLOCK_D",
]


def _decode(grid, b):
    q, kp, vp, pc, pl = b["Q"], b["K_packed"], b["V_packed"], b["Packed_Counts"], b["Packed_Lengths"]
    ke, ve, out = b["K_exact"], b["V_exact"], b["Out"]
    L.require_cuda(q, kp, vp, pc, pl, ke, ve, out)
    batch, hq = grid[0], grid[1]
    capacity = int(kp.shape[-2])
    lib = L.load()
    st = L.stream_of(q)
    ws_bytes = lib.dab_decode_attention_workspace_size(batch, hq, capacity, _i(b, "exact_len"), _i(b, "head_dim"))
    ws = L.workspace(q.device, st.value, ws_bytes, tag="decode")
    L.check(lib.dab_decode_attention(
        L.ptr(q), L.ptr(kp), L.ptr(vp), L.ptr(pc), L.ptr(pl), L.ptr(ke), L.ptr(ve), L.ptr(out), L.dtype_code(q),
        L.strides([b[n] for n in DECODE_PARAMS[8:35]]), _f(b, "sm_scale"), _i(b, "exact_len"),
        _i(b, "num_kv_groups"), batch, hq, _i(b, "head_dim"), capacity, L.ptr(ws), ws.numel(), st),
        "fused_hybrid_decode_kernel")


fused_hybrid_decode_kernel = KernelShim("fused_hybrid_decode_kernel", DECODE_PARAMS, _decode)

ALL_KERNELS = [chunked_eval_kernel, parallel_scatter_pack_kv_kernel, hybrid_compressed_flash_kernel,
               hybrid_compressed_flash_kernel_sanity, pure_phase1_flash_kernel, _attn_fwd_flat,
               fused_hybrid_decode_update_kernel, fused_hybrid_decode_kernel]

__all__ = [k.__name__ for k in ALL_KERNELS] + ["KernelShim", "hybrid_call", "flat_call"]
_ = ctypes

"""Generate golden vectors by running the REFERENCE's own Triton kernels on CPU.

Run in the build container only (it needs the read-only reference checkout):

    python tests/golden/gen_golden.py --reference /path/to/DeltaAttention [--bf16]

The reference kernels execute under ``TRITON_INTERPRET=1``. Four harness shims are
needed to import ``modeling_llama`` with the installed transformers (stub seaborn /
matplotlib modules, a ``LossKwargs`` TypedDict); the kernel modules themselves import
unchanged. The stock interpreter stores bf16 as raw uint16 and applies numpy arithmetic
to those bits (``bf16_interp_probe`` below records the evidence), so the default run's
bf16 cases only exercise fp32-upcast math (cosine selection) or torch-eager glue (RoPE).
With ``--bf16`` the run then installs ``bf16_interp`` (IEEE bf16 arithmetic in the
interpreter: fp32 compute, one round-to-nearest-even per bf16 result, fp32 accumulation
in ``tl.dot`` and ``tl.sum``) and writes the bf16 fixtures from the same unmodified
reference kernels: Euclidean selection, packing, the three attention variants, flash
attention and the decode replay.

Inputs are regenerated from ``_inputs.py`` (numpy PCG64, seeded); each fixture stores
an input checksum so a drifting generator is detected instead of silently compared.
"""


import argparse
import importlib.machinery
import os
import sys
import types
import typing

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import _inputs as I  # noqa: E402


def _shim_and_import(ref_root: str):
    sys.path.insert(0, ref_root)
    for name in ["seaborn", "matplotlib", "matplotlib.pyplot"]:
        m = types.ModuleType(name)
        m.__spec__ = importlib.machinery.ModuleSpec(name, None)
        sys.modules[name] = m
    sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
    for n in ["histplot", "boxplot", "heatmap"]:
        setattr(sys.modules["seaborn"], n, lambda *a, **k: None)
    import transformers.utils as tu

    class LossKwargs(typing.TypedDict, total=False):
        pass

    tu.LossKwargs = LossKwargs
    import modeling_llama  # noqa: F401
    import tritonModules
    import deltaFlashAttention  # noqa: F401
    import flashAttention
    import deltaDecoding
    return modeling_llama, tritonModules, flashAttention, deltaDecoding


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DELTA_REFERENCE"),
                    help="checkout of the reference project (or set DELTA_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--bf16", action="store_true",
                    help="also write the bf16 fixtures (interpreter with IEEE bf16 arithmetic, "
                         "installed after every other fixture is written)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("pass --reference <reference checkout> (or set DELTA_REFERENCE)")
    import torch
    import triton
    import triton.language as tl  # noqa: F401  (annotation namespace of _sub_kernel)
    ml, tm, fa, dd = _shim_and_import(args.reference)
    out = {}

    def save(name, **arrs):
        path = os.path.join(args.out, name + ".npz")
        np.savez_compressed(path, **{k: (v.numpy() if hasattr(v, "numpy") else np.asarray(v))
                                      for k, v in arrs.items()})
        out[name] = path
        print("wrote", path, os.path.getsize(path), "bytes")

    # ---------------- evidence: interpreter bf16 arithmetic is bit-level -------------

    a = torch.tensor([1.5, 2.0, -3.0, 0.25], dtype=torch.bfloat16)
    b = torch.tensor([0.5, 1.0, 1.0, 0.125], dtype=torch.bfloat16)
    o = torch.zeros(4, dtype=torch.bfloat16)
    _make_sub_kernel()[(1,)](a, b, o, D=4)
    save("bf16_interp_probe", a=a.view(torch.int16), b=b.view(torch.int16),
         interp=o.view(torch.int16), true=(a.float() - b.float()).bfloat16().view(torch.int16))

    # ---------------- RoPE (torch eager glue, modeling_llama.py:180-204) -------------
    for dt_name, dt in [("bf16", torch.bfloat16), ("fp32", torch.float32)]:
        x = I.ar1_keys(1, 2, 300, 128, seed=11, offset=True)
        x = torch.from_numpy(x).to(dt)
        cos, sin = I.cos_sin(300, 128, 500000.0, dt)
        q_e, k_e = ml.apply_rotary_pos_emb(x, x, cos, sin)
        save(f"rope_{dt_name}", cos=cos.float(), sin=sin.float(), out=k_e.float(),
             in_sum=np.float64(x.double().sum()))

    # ---------------- selection: chunked_eval_kernel (tritonModules.py:7-69) ---------
    run_eval = _runner_eval(tm)

    sel_cases = [
        # name, dtype, B,H,N,D, chunk, cosine, theta, seed
        ("keep_euclid_fp32", torch.float32, 1, 2, 1000, 64, 256, False, 1e4, 1),
        ("keep_euclid_fp16", torch.float16, 1, 2, 1000, 128, 300, False, 5e5, 2),
        ("keep_cosine_fp32", torch.float32, 1, 2, 1000, 64, 256, True, 1e4, 3),
        ("keep_cosine_bf16", torch.bfloat16, 1, 2, 1000, 128, 300, True, 5e5, 4),
        ("keep_cosine_fp16", torch.float16, 1, 2, 700, 96, 512, True, 5e5, 5),
    ]
    for name, dt, B, H, N, D, chunk, use_cos, theta, seed in sel_cases:
        k = I.post_rope_keys(B, H, N, D, theta, dt, seed=seed)
        thr = I.median_threshold(k, use_cos)
        # modeling_llama.py:641-642: the kernel receives tau**2 for Euclid, tau for cosine
        keep, cc = run_eval(k, thr, use_cos, chunk)
        save(name, keep=keep, chunk_counts=cc, threshold=np.float64(thr), chunk=chunk,
             in_sum=np.float64(k.double().sum()), seed=seed, theta=theta)

    # BSHD-strided input (the layout modeling_llama.py:551 hands to the kernel)
    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1)
    kb = k.transpose(1, 2).contiguous().transpose(1, 2)
    thr = I.median_threshold(k, False)
    keep, cc = run_eval(kb, thr, False, 256)
    save("keep_euclid_fp32_bshd", keep=keep, chunk_counts=cc, threshold=np.float64(thr))

    # ---------------- pack: parallel_scatter_pack_kv_kernel + torch glue -------------
    run_pack = _runner_pack(tm)

    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1)
    v = torch.from_numpy(I.normal((1, 2, 1000, 64), seed=101)).float()
    keep, _ = run_eval(k, I.median_threshold(k, False), False, 256)
    im, kp, vp, ts, counts = run_pack(k, v, keep)
    save("pack_fp32", keep=keep, index_map=im, k_packed=kp, v_packed=vp, timestamps=ts,
         counts=counts, k_sum=np.float64(k.double().sum()), v_sum=np.float64(v.double().sum()))

    # ---------------- attention: wrappers of modeling_llama.py:306-451 ---------------
    run_variants = _runner_variants(ml)

    attn_cases = [
        # name, dtype, H, N, D, packing, W, seed
        ("attn_fp32_periodic", torch.float32, 2, 600, 64, "periodic", 128, 21),
        ("attn_fp32_delta", torch.float32, 2, 600, 64, "delta", 128, 22),
        ("attn_fp32_w0", torch.float32, 2, 600, 64, "periodic", 0, 23),
        ("attn_fp16_periodic", torch.float16, 2, 600, 128, "periodic", 128, 24),
        ("attn_fp16_delta", torch.float16, 2, 520, 128, "delta", 128, 25),
        ("attn_fp32_quirk", torch.float32, 2, 600, 64, "quirk", 128, 26),
    ]
    for name, dt, H, N, D, packing, W, seed in attn_cases:
        q, k, v = I.attn_inputs(1, H, N, D, dt, seed)
        if packing == "periodic":
            keep = ((torch.arange(N) % 4) == 0).to(torch.int32)[None, None].expand(1, H, N).contiguous()
        elif packing == "quirk":
            keep = I.quirk_keep(1, H, N)
        else:
            # heterogeneous heads: head 0 keeps ~1/2, head 1 keeps ~1/8 -> padding blocks
            keep = I.hetero_keep(1, H, N, seed)
        _, kp, vp, ts, counts = run_pack(k, v, keep)
        res = run_variants(q, k, v, kp, vp, ts, counts, W)
        flash_c = fa.triton_flash_attention(q, k, v, causal=True)
        flash_n = fa.triton_flash_attention(q, k, v, causal=False)
        save(name, keep=keep, W=W, seed=seed, hybrid=res["hybrid"].float(),
             sanity=res["sanity"].float(), pure_phase1=res["pure_phase1"].float(),
             flash_causal=flash_c.float(), flash_noncausal=flash_n.float(),
             q_sum=np.float64(q.double().sum()))

    # ---------------- decoding (deltaDecoding.py) --------------------------------------
    for name, dt, use_cos in [("decode_fp32_euclid", torch.float32, False),
                              ("decode_fp16_cosine", torch.float16, True)]:
        save(name, **_replay_decode(dd, dt, use_cos))

    if args.bf16:
        _bf16_fixtures(save, tm, ml, fa, dd, run_eval, run_pack, run_variants)
    print("done", len(out), "fixtures")


class _Self:
    """Stand-in ``self`` for the reference's attention wrappers (they read only these)."""


def _runner_eval(tm):
    """``chunked_eval_kernel`` launch as ``modeling_llama.py:635-653`` performs it."""
    import torch
    import triton

    def run_eval(k, threshold, use_cos, chunk):
        B, H, N, D = k.shape
        nch = -(-N // chunk)
        keep = torch.zeros((B, H, N), dtype=torch.int32)
        cc = torch.zeros((B, H, nch), dtype=torch.int32)
        tm.chunked_eval_kernel[(B * H, nch)](
            k, keep, cc, threshold,
            k.stride(0), k.stride(1), k.stride(2), k.stride(3),
            keep.stride(0), keep.stride(1), keep.stride(2),
            cc.stride(0), cc.stride(1), cc.stride(2),
            N, D, chunk, num_heads=H,
            BLOCK_D=triton.next_power_of_2(D), USE_COSINE=use_cos)
        return keep, cc
    return run_eval


def _runner_pack(tm):
    """Index map, ``parallel_scatter_pack_kv_kernel`` and counts (modeling_llama.py:655-685)."""
    import torch
    import triton

    def run_pack(k, v, keep):
        B, H, N, D = k.shape
        index_map = (torch.cumsum(keep, dim=-1) - 1).to(torch.int32)
        M = int(keep.sum(-1).max())
        kp = torch.zeros((B, H, M, D), dtype=k.dtype)
        vp = torch.zeros_like(kp)
        ts = torch.zeros((B, H, M), dtype=torch.int32)
        tm.parallel_scatter_pack_kv_kernel[(B * H, triton.cdiv(N, 64))](
            k, v, kp, vp, ts, keep, index_map,
            k.stride(0), k.stride(1), k.stride(2), k.stride(3),
            v.stride(0), v.stride(1), v.stride(2), v.stride(3),
            kp.stride(0), kp.stride(1), kp.stride(2), kp.stride(3),
            vp.stride(0), vp.stride(1), vp.stride(2), vp.stride(3),
            ts.stride(0), ts.stride(1), ts.stride(2),
            keep.stride(0), keep.stride(1), keep.stride(2),
            index_map.stride(0), index_map.stride(1), index_map.stride(2),
            N, D, H, BLOCK_S=64, BLOCK_D=triton.next_power_of_2(D))
        counts = torch.zeros((B, H, M), dtype=torch.int32)
        counts.scatter_add_(2, index_map.long(), torch.ones_like(index_map, dtype=torch.int32))
        return index_map, kp, vp, ts, counts
    return run_pack


def _runner_variants(ml):
    """The three attention wrappers of ``modeling_llama.py:306-451``."""
    def run_variants(q, kd, vd, kp, vp, ts, counts, W):
        s = _Self()
        s.scaling = q.shape[-1] ** -0.5
        A = ml.LlamaAttention
        return {
            "hybrid": A._forward_hybrid_flash(s, q, kd, vd, kp, vp, ts, counts, W),
            "sanity": A._forward_hybrid_flash_sanity(s, q, kd, vd, kp, vp, ts, counts, W),
            "pure_phase1": A._forward_pure_phase1(s, q, kd, vd, kp, vp, ts, counts, W),
        }
    return run_variants


def _replay_decode(dd, dt, use_cos):
    """``decode_setup``'s steps through ``fused_hybrid_decode_update_kernel`` and the
    decode attention launch; returns the arrays a decode fixture stores."""
    import torch
    import triton
    st = I.decode_setup(dt, seed=31)
    B, Hkv, Hq, D, W = st["B"], st["Hkv"], st["Hq"], st["D"], st["W"]
    thr = st["thr_cos"] if use_cos else st["thr_euclid_sq"]
    kp, vp, cnt, tss, lens = st["kp"], st["vp"], st["counts"], st["ts"], st["lengths"]
    ke, ve = st["ke"], st["ve"]
    exact_len, total = st["exact_len"], st["total"]
    outs, lens_hist = [], []
    s = _Self()
    s.scaling = D ** -0.5
    s.layer_idx = 0
    s.num_key_value_groups = Hq // Hkv
    s.config = types.SimpleNamespace(num_key_value_heads=Hkv)
    for step in range(st["steps"]):
        nk = st["new_k"][step]
        nv = st["new_v"][step]
        dd.fused_hybrid_decode_update_kernel[(B * Hkv,)](
            nk, nv, ke, ve, kp, vp, cnt, tss, lens, exact_len, total, thr, W,
            nk.stride(0), nk.stride(1), nk.stride(2), nk.stride(3),
            ke.stride(0), ke.stride(1), ke.stride(2), ke.stride(3),
            kp.stride(0), kp.stride(1), kp.stride(2), kp.stride(3),
            cnt.stride(0), cnt.stride(1), cnt.stride(2),
            Hkv, D, BLOCK_D=triton.next_power_of_2(D), USE_COSINE=use_cos)
        exact_len += 1
        total += 1
        pkv = types.SimpleNamespace(
            k_packed=kp[None], v_packed=vp[None], packed_counts=cnt[None],
            packed_lengths=lens[None], k_exact=ke[None], v_exact=ve[None],
            exact_seq_lens=[exact_len], exact_window_size=W)
        # the wrapper records CUDA events; run the kernel launch it performs directly
        q = st["q"][step][:, :, None, :]
        o = _decode_attn(dd, s, q, pkv, Hkv)
        outs.append(o.float())
        lens_hist.append(lens.clone())
    return dict(outputs=torch.stack(outs), lengths=torch.stack(lens_hist),
                k_packed=kp.float(), v_packed=vp.float(), counts=cnt, timestamps=tss,
                k_exact=ke.float(), v_exact=ve.float(), threshold=np.float64(thr))


def _bf16_fixtures(save, tm, ml, fa, dd, run_eval, run_pack, run_variants):
    """bf16 fixtures: the reference's kernels, unmodified, on the interpreter with IEEE
    bf16 arithmetic (``bf16_interp.install``)."""
    import torch
    import bf16_interp
    bf16_interp.install()

    # the probe kernel now gives the correctly rounded difference
    a = torch.tensor([1.5, 2.0, -3.0, 0.25, 1.0, 3.0e38, 1.0, -0.0], dtype=torch.bfloat16)
    b = torch.tensor([0.5, 1.0, 1.0, 0.125, 2.0 ** -9, -3.0e38, 2.0 ** -8, 0.0],
                     dtype=torch.bfloat16)
    o = torch.zeros(8, dtype=torch.bfloat16)
    _make_sub_kernel()[(1,)](a, b, o, D=8)
    save("bf16_interp_ieee_probe", a=a.view(torch.int16), b=b.view(torch.int16),
         interp=o.view(torch.int16), true=(a.float() - b.float()).bfloat16().view(torch.int16))

    # Euclidean selection: x - a, d * d and the sum all run in bf16 (tritonModules.py:54-56)
    for name, B, H, N, D, chunk, theta, seed in [
            ("keep_euclid_bf16", 1, 2, 1000, 128, 300, 5e5, 6),
            ("keep_euclid_bf16_d64", 2, 2, 777, 64, 256, 1e4, 7)]:
        k = I.post_rope_keys(B, H, N, D, theta, torch.bfloat16, seed=seed)
        thr = I.median_threshold(k, False)
        keep, cc = run_eval(k, thr, False, chunk)
        save(name, keep=keep, chunk_counts=cc, threshold=np.float64(thr), chunk=chunk,
             in_sum=np.float64(k.double().sum()), seed=seed, theta=theta)

    # packing of bf16 rows under a bf16 Euclidean keep mask
    k = I.post_rope_keys(1, 2, 1000, 128, 5e5, torch.bfloat16, seed=6)
    v = torch.from_numpy(I.normal((1, 2, 1000, 128), seed=106)).to(torch.bfloat16)
    keep, _ = run_eval(k, I.median_threshold(k, False), False, 300)
    im, kp, vp, ts, counts = run_pack(k, v, keep)
    save("pack_bf16", keep=keep, index_map=im, k_packed=kp.float(), v_packed=vp.float(),
         timestamps=ts, counts=counts, k_sum=np.float64(k.double().sum()),
         v_sum=np.float64(v.double().sum()))

    # attention: bf16 QK^T / PV on the tensor-core path, P rounded to bf16 before PV
    for name, H, N, D, packing, W, seed in [
            ("attn_bf16_periodic", 2, 600, 128, "periodic", 128, 27),
            ("attn_bf16_delta", 2, 520, 128, "delta", 128, 28),
            ("attn_bf16_d64_w0", 2, 400, 64, "periodic", 0, 29)]:
        q, k, v = I.attn_inputs(1, H, N, D, torch.bfloat16, seed)
        if packing == "periodic":
            keep = ((torch.arange(N) % 4) == 0).to(torch.int32)[None, None].expand(1, H, N).contiguous()
        else:
            keep = I.hetero_keep(1, H, N, seed)
        _, kp, vp, ts, counts = run_pack(k, v, keep)
        res = run_variants(q, k, v, kp, vp, ts, counts, W)
        flash_c = fa.triton_flash_attention(q, k, v, causal=True)
        flash_n = fa.triton_flash_attention(q, k, v, causal=False)
        save(name, keep=keep, W=W, seed=seed, hybrid=res["hybrid"].float(),
             sanity=res["sanity"].float(), pure_phase1=res["pure_phase1"].float(),
             flash_causal=flash_c.float(), flash_noncausal=flash_n.float(),
             q_sum=np.float64(q.double().sum()))

    save("decode_bf16_euclid", **_replay_decode(dd, torch.bfloat16, False))


def _make_sub_kernel():
    import triton
    import triton.language as tl

    @triton.jit
    def _sub_kernel(a_ptr, b_ptr, o_ptr, D: tl.constexpr):
        offs = tl.arange(0, D)
        a = tl.load(a_ptr + offs)
        b = tl.load(b_ptr + offs)
        tl.store(o_ptr + offs, a - b)
    return _sub_kernel


def _decode_attn(dd, s, q, pkv, Hkv):
    """The launch ``_forward_fused_hybrid_decode`` performs (modeling_llama.py:453-518),
    minus its CUDA-event timing, which cannot run on a CPU-only box."""
    import torch
    import triton
    bsz, num_heads, _, head_dim = q.shape
    q = q.squeeze(2).contiguous()
    k_packed = pkv.k_packed[0]
    v_packed = pkv.v_packed[0]
    counts = pkv.packed_counts[0]
    lengths = pkv.packed_lengths[0].view(bsz, Hkv)
    k_exact = pkv.k_exact[0]
    v_exact = pkv.v_exact[0]
    exact_len = min(pkv.exact_seq_lens[0], pkv.exact_window_size)
    out = torch.empty_like(q)
    dd.fused_hybrid_decode_kernel[(bsz, num_heads)](
        q, k_packed, v_packed, counts, lengths, k_exact, v_exact, out,
        q.stride(0), q.stride(1), q.stride(2),
        k_packed.stride(0), k_packed.stride(1), k_packed.stride(2), k_packed.stride(3),
        v_packed.stride(0), v_packed.stride(1), v_packed.stride(2), v_packed.stride(3),
        counts.stride(0), counts.stride(1), counts.stride(2),
        lengths.stride(0), lengths.stride(1),
        k_exact.stride(0), k_exact.stride(1), k_exact.stride(2), k_exact.stride(3),
        v_exact.stride(0), v_exact.stride(1), v_exact.stride(2), v_exact.stride(3),
        out.stride(0), out.stride(1), out.stride(2),
        s.scaling, exact_len, s.num_key_value_groups,
        head_dim=head_dim, BLOCK_M=16, BLOCK_N=128, BLOCK_D=triton.next_power_of_2(head_dim))
    return out


if __name__ == "__main__":
    main()

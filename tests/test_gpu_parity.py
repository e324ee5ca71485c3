"""GPU parity: the CUDA kernels (through the reference-facing launch API and the C ABI)
against the reference goldens and the CPU oracle.

Selection, packing, N:M selection, RoPE and decode-cache state must match bit for bit.
Attention outputs: fp32 within 1e-4 (max abs); bf16/fp16 within max-abs 2e-2 and
mean-abs 2e-3 (the tolerances BASELINE.json's north star states).
"""
import numpy as np
import pytest
import torch

import _inputs as I
from oracle import delta_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 1e-5), torch.float16: (2e-2, 2e-3), torch.bfloat16: (2e-2, 2e-3)}


@pytest.fixture(scope="module", autouse=True)
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import deltaattention_b200 as d
    d._lib.load()
    from deltaattention_b200.dropin import install
    install()
    return d


@pytest.fixture(autouse=True)
def _fresh_error_words():
    """Each test starts with cleared device error words (a failure cannot leak forward)."""
    from deltaattention_b200 import _lib as L
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        L.workspace_errors()
    yield


def _check_ws_clean():
    from deltaattention_b200 import _lib as L
    torch.cuda.synchronize()
    codes = L.workspace_errors()
    assert all(c == 0 for c in codes), f"a bounded device wait timed out: {[hex(c) for c in codes]}"


def _cmp(out, ref, dtype, what=""):
    out = out.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(out).all() == torch.isfinite(ref).all(), what
    err = (out - ref).abs()
    mx, mean = TOL[dtype]
    assert err.max().item() <= mx and err.mean().item() <= mean, (what, err.max().item(), err.mean().item())


# ------------------------------------------------------------------ selection / packing
SEL = [
    ("keep_euclid_fp32", torch.float32, 1, 2, 1000, 64, 256, False, 1e4, 1),
    ("keep_euclid_fp16", torch.float16, 1, 2, 1000, 128, 300, False, 5e5, 2),
    ("keep_cosine_fp32", torch.float32, 1, 2, 1000, 64, 256, True, 1e4, 3),
    ("keep_cosine_bf16", torch.bfloat16, 1, 2, 1000, 128, 300, True, 5e5, 4),
    ("keep_cosine_fp16", torch.float16, 1, 2, 700, 96, 512, True, 5e5, 5),
    ("keep_euclid_bf16", torch.bfloat16, 1, 2, 1000, 128, 300, False, 5e5, 6),
    ("keep_euclid_bf16_d64", torch.bfloat16, 2, 2, 777, 64, 256, False, 1e4, 7),
]


@pytest.mark.parametrize("case", SEL, ids=[c[0] for c in SEL])
def test_chunked_eval_matches_reference_bit_exact(golden, case):
    import tritonModules as tm
    name, dt, B, H, N, D, chunk, use_cos, theta, seed = case
    g = golden(name)
    k = I.post_rope_keys(B, H, N, D, theta, dt, seed=seed).cuda()
    nch = -(-N // chunk)
    keep = torch.zeros((B, H, N), dtype=torch.int32, device="cuda")
    cc = torch.zeros((B, H, nch), dtype=torch.int32, device="cuda")
    bd = 1 << (D - 1).bit_length()
    tm.chunked_eval_kernel[(B * H, nch)](
        k, keep, cc, float(g["threshold"]), k.stride(0), k.stride(1), k.stride(2), k.stride(3),
        keep.stride(0), keep.stride(1), keep.stride(2), cc.stride(0), cc.stride(1), cc.stride(2),
        N, D, chunk, num_heads=H, BLOCK_D=bd, USE_COSINE=use_cos, num_warps=4)
    np.testing.assert_array_equal(keep.cpu().numpy(), g["keep"])
    np.testing.assert_array_equal(cc.cpu().numpy(), g["chunk_counts"])


def test_chunked_eval_strided_bshd(golden):
    import tritonModules as tm
    g = golden("keep_euclid_fp32_bshd")
    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1)
    kb = k.transpose(1, 2).contiguous().transpose(1, 2).cuda()
    keep = torch.zeros((1, 2, 1000), dtype=torch.int32, device="cuda")
    cc = torch.zeros((1, 2, 4), dtype=torch.int32, device="cuda")
    tm.chunked_eval_kernel[(2, 4)](kb, keep, cc, float(g["threshold"]), *kb.stride(), *keep.stride(), *cc.stride(),
                                   1000, 64, 256, num_heads=2, BLOCK_D=64, USE_COSINE=False)
    np.testing.assert_array_equal(keep.cpu().numpy(), g["keep"])


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_chunked_eval_euclid_matches_oracle(dt):
    """bf16 Euclid has no interpreter golden (bf16 arithmetic there is bitwise); the oracle
    restates the reference's rounding and reduction order and the kernel must agree."""
    import tritonModules as tm
    B, H, N, D, chunk = 1, 4, 2048, 128, 512
    k = I.post_rope_keys(B, H, N, D, 5e5, dt, seed=77, offset=True)
    thr = I.median_threshold(k, False)
    ref_keep, ref_cc = O.delta_keep_mask(k, thr, False, chunk, N // chunk)
    kc = k.cuda()
    keep = torch.zeros((B, H, N), dtype=torch.int32, device="cuda")
    cc = torch.zeros((B, H, N // chunk), dtype=torch.int32, device="cuda")
    tm.chunked_eval_kernel[(B * H, N // chunk)](kc, keep, cc, thr, *kc.stride(), *keep.stride(), *cc.stride(), N, D,
                                                chunk, num_heads=H, BLOCK_D=128, USE_COSINE=False)
    np.testing.assert_array_equal(keep.cpu().numpy(), ref_keep.numpy())
    np.testing.assert_array_equal(cc.cpu().numpy(), ref_cc.numpy())


SCAN = [  # dtype, head_dim, chunk, cosine: row widths 128 B to 1 KiB, ragged and tiny chunks
    (torch.bfloat16, 256, 300, False), (torch.bfloat16, 64, 512, False), (torch.float16, 128, 13, False),
    (torch.float32, 32, 77, True), (torch.bfloat16, 128, 512, True), (torch.float32, 256, 100, False),
]


@pytest.mark.parametrize("level", range(4))
@pytest.mark.parametrize("dt,D,chunk,use_cos", SCAN)
def test_delta_scan_keep_rates_match_oracle(dt, D, chunk, use_cos, level):
    """The delta scan from almost every key kept (level 0) to almost none (level 3), on ragged
    chunks and row widths from 128 to 1024 bytes: keep mask and chunk counts equal the oracle's."""
    import tritonModules as tm
    B, H, N = 1, 3, 1000
    k = I.post_rope_keys(B, H, N, D, 5e5, dt, seed=91, offset=True)
    kk = k.float().numpy()
    a, b = kk[:, :, 1:], kk[:, :, :-1]
    if use_cos:
        c = (a * b).sum(-1) / (np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1) + 1e-8)
        lo = float(np.quantile(c, 0.03))
        thr = [float(np.quantile(c, 0.97)), lo, lo - 0.3, lo - 0.8][level]
    else:
        d = ((a - b) ** 2).sum(-1)
        hi = float(np.quantile(d, 0.97))
        thr = [float(np.quantile(d, 0.03)), hi, 4 * hi, 16 * hi][level]
    nch = -(-N // chunk)
    ref_keep, ref_cc = O.delta_keep_mask(k, thr, use_cos, chunk, nch)
    kc = k.cuda()
    keep = torch.zeros((B, H, N), dtype=torch.int32, device="cuda")
    cc = torch.zeros((B, H, nch), dtype=torch.int32, device="cuda")
    tm.chunked_eval_kernel[(B * H, nch)](kc, keep, cc, thr, *kc.stride(), *keep.stride(), *cc.stride(), N, D, chunk,
                                         num_heads=H, BLOCK_D=D, USE_COSINE=use_cos)
    np.testing.assert_array_equal(keep.cpu().numpy(), ref_keep.numpy())
    np.testing.assert_array_equal(cc.cpu().numpy(), ref_cc.numpy())


@pytest.mark.parametrize("similarity,threshold", [("euclidean", 11.0), ("cosine", 0.9)])
def test_delta_scan_full_size_matches_oracle(similarity, threshold):
    """cfg2 keys at full size (8 kv-heads x 32k tokens in the projection layout, chunk 512,
    bf16; the bench's keys and Euclidean threshold, which keep about 1 key in 4): keep mask
    and chunk counts equal the oracle's on the same post-RoPE keys, token for token."""
    from deltaattention_b200 import ops, synth
    dev = torch.device("cuda")
    _, k, _ = synth.layer_inputs(1, 8, 8, 32768, 128, torch.bfloat16, seed=2000, device=dev)
    cos, sin = synth.rope_tables(32768, 128, 5e5, torch.bfloat16, device=dev)
    k_rot = ops.rope(k, cos, sin)
    keep, cc = ops.delta_keep_mask(k_rot, threshold, similarity, 512)
    use_cos = similarity == "cosine"
    ref_keep, ref_cc = O.delta_keep_mask(k_rot.cpu(), threshold if use_cos else threshold ** 2, use_cos, 512, 64)
    bad = (keep.cpu() != ref_keep).nonzero().tolist()
    assert not bad, f"{len(bad)} decisions differ, first at (b, h, t) = {bad[:4]}"
    np.testing.assert_array_equal(cc.cpu().numpy(), ref_cc.numpy())


def test_scatter_pack_matches_reference(golden):
    import tritonModules as tm
    g = golden("pack_fp32")
    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1).cuda()
    v = torch.from_numpy(I.normal((1, 2, 1000, 64), seed=101)).cuda()
    keep = torch.from_numpy(g["keep"]).cuda()
    im = (torch.cumsum(keep, -1) - 1).to(torch.int32)
    M = int(keep.sum(-1).max())
    kp = torch.zeros((1, 2, M, 64), device="cuda")
    vp = torch.zeros_like(kp)
    ts = torch.zeros((1, 2, M), dtype=torch.int32, device="cuda")
    tm.parallel_scatter_pack_kv_kernel[(2, -(-1000 // 64))](
        k, v, kp, vp, ts, keep, im, *k.stride(), *v.stride(), *kp.stride(), *vp.stride(), *ts.stride(),
        *keep.stride(), *im.stride(), 1000, 64, 2, BLOCK_S=64, BLOCK_D=64)
    np.testing.assert_array_equal(kp.cpu().numpy(), g["k_packed"])
    np.testing.assert_array_equal(vp.cpu().numpy(), g["v_packed"])
    np.testing.assert_array_equal(ts.cpu().numpy(), g["timestamps"])


@pytest.mark.parametrize("dt,D,layout", [(torch.bfloat16, 128, "bhsd"), (torch.float16, 96, "bshd"),
                                          (torch.bfloat16, 100, "bhsd"), (torch.float16, 64, "dstride")])
def test_scatter_pack_layouts_match_oracle(dt, D, layout):
    """The reference-facing scatter pack on 16-byte row copies (unit head-dim strides,
    aligned rows) and element copies (200-byte rows, strided head dim): packed K / V and
    timestamps equal the oracle's packing of the same keep mask."""
    import tritonModules as tm
    B, H, N = 1, 3, 1500
    k = torch.from_numpy(I.normal((B, H, N, D), seed=7)).to(dt)
    v = torch.from_numpy(I.normal((B, H, N, D), seed=8)).to(dt)
    keep = O.periodic_keep_mask(B, H, N, 0.3).clone()
    keep[:, :, 7::11] = 1
    _, kp_ref, vp_ref, ts_ref, _ = O.pack_from_keep(k, v, keep)
    if layout == "bshd":
        kc, vc = (t.transpose(1, 2).contiguous().cuda().transpose(1, 2) for t in (k, v))
    elif layout == "dstride":
        kc, vc = (t.transpose(2, 3).contiguous().cuda().transpose(2, 3) for t in (k, v))
    else:
        kc, vc = k.cuda(), v.cuda()
    km = keep.cuda()
    im = (torch.cumsum(km, -1) - 1).to(torch.int32)
    M = int(keep.sum(-1).max())
    kp = torch.zeros((B, H, M, D), dtype=dt, device="cuda")
    vp = torch.zeros_like(kp)
    ts = torch.zeros((B, H, M), dtype=torch.int32, device="cuda")
    tm.parallel_scatter_pack_kv_kernel[(B * H, -(-N // 64))](
        kc, vc, kp, vp, ts, km, im, *kc.stride(), *vc.stride(), *kp.stride(), *vp.stride(), *ts.stride(),
        *km.stride(), *im.stride(), N, D, H, BLOCK_S=64, BLOCK_D=1 << (D - 1).bit_length())
    assert torch.equal(kp.cpu().view(torch.int16), kp_ref.view(torch.int16))
    assert torch.equal(vp.cpu().view(torch.int16), vp_ref.view(torch.int16))
    assert torch.equal(ts.cpu(), ts_ref)


def test_scatter_pack_bf16_matches_reference(golden):
    """bf16 Euclidean selection, the reference's cumsum index map and the scatter pack on
    the GPU against the reference kernels' bf16 fixture, bit for bit."""
    import tritonModules as tm
    g = golden("pack_bf16")
    k = I.post_rope_keys(1, 2, 1000, 128, 5e5, torch.bfloat16, seed=6).cuda()
    v = torch.from_numpy(I.normal((1, 2, 1000, 128), seed=106)).to(torch.bfloat16).cuda()
    keep = torch.zeros((1, 2, 1000), dtype=torch.int32, device="cuda")
    cc = torch.zeros((1, 2, 4), dtype=torch.int32, device="cuda")
    thr = I.median_threshold(k.cpu(), False)
    tm.chunked_eval_kernel[(2, 4)](k, keep, cc, thr, *k.stride(), *keep.stride(), *cc.stride(),
                                   1000, 128, 300, num_heads=2, BLOCK_D=128, USE_COSINE=False)
    np.testing.assert_array_equal(keep.cpu().numpy(), g["keep"])
    im = (torch.cumsum(keep, -1) - 1).to(torch.int32)
    M = int(keep.sum(-1).max())
    kp = torch.zeros((1, 2, M, 128), dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    ts = torch.zeros((1, 2, M), dtype=torch.int32, device="cuda")
    tm.parallel_scatter_pack_kv_kernel[(2, -(-1000 // 64))](
        k, v, kp, vp, ts, keep, im, *k.stride(), *v.stride(), *kp.stride(), *vp.stride(), *ts.stride(),
        *keep.stride(), *im.stride(), 1000, 128, 2, BLOCK_S=64, BLOCK_D=128)
    np.testing.assert_array_equal(im.cpu().numpy(), g["index_map"])
    np.testing.assert_array_equal(kp.float().cpu().numpy(), g["k_packed"])
    np.testing.assert_array_equal(vp.float().cpu().numpy(), g["v_packed"])
    np.testing.assert_array_equal(ts.cpu().numpy(), g["timestamps"])
    from deltaattention_b200 import ops
    p = ops.pack_from_keep(k, v, keep, want_index_map=True)
    np.testing.assert_array_equal(p.k.float().cpu().numpy(), g["k_packed"])
    np.testing.assert_array_equal(p.counts.cpu().numpy(), g["counts"])


def test_device_pack_from_keep_matches_reference(golden):
    from deltaattention_b200 import ops
    g = golden("pack_fp32")
    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1).cuda()
    v = torch.from_numpy(I.normal((1, 2, 1000, 64), seed=101)).cuda()
    keep = torch.from_numpy(g["keep"]).cuda()
    p = ops.pack_from_keep(k, v, keep, want_index_map=True)
    np.testing.assert_array_equal(p.index_map.cpu().numpy(), g["index_map"])
    np.testing.assert_array_equal(p.k.cpu().numpy(), g["k_packed"])
    np.testing.assert_array_equal(p.v.cpu().numpy(), g["v_packed"])
    np.testing.assert_array_equal(p.timestamps.cpu().numpy(), g["timestamps"])
    np.testing.assert_array_equal(p.counts.cpu().numpy(), g["counts"])


@pytest.mark.parametrize("dt_name,dt", [("bf16", torch.bfloat16), ("fp32", torch.float32)])
def test_rope_matches_reference(golden, dt_name, dt):
    from deltaattention_b200 import ops
    g = golden(f"rope_{dt_name}")
    x = torch.from_numpy(I.ar1_keys(1, 2, 300, 128, seed=11, offset=True)).to(dt)
    cos, sin = O.rope_cos_sin(300, 128, 500000.0, dt)
    y = ops.rope(x.cuda(), cos.cuda(), sin.cuda())
    np.testing.assert_array_equal(y.float().cpu().numpy(), g["out"])


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("layout", ["contiguous", "projection", "d_strided", "d96"])
def test_rope_layouts_match_oracle(dt, layout):
    """Both RoPE kernels (16-byte rows and the generic strided one) against the oracle, bit-exact."""
    from deltaattention_b200 import ops
    D = 96 if layout == "d96" else 128
    B, H, N = 2, 3, 257
    base = torch.from_numpy(I.ar1_keys(B, H, N, D, seed=12, offset=True)).to(dt)
    cos, sin = O.rope_cos_sin(N, D, 500000.0, dt)
    ref = O.apply_rope(base, cos, sin)
    if layout == "projection":      # [B, N, H, D] storage viewed as [B, H, N, D]
        x = base.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    elif layout == "d_strided":     # d is not the unit-stride axis: generic kernel
        x = base.transpose(2, 3).contiguous().cuda().transpose(2, 3)
    else:
        x = base.cuda()
    y = ops.rope(x, cos.cuda(), sin.cuda())
    np.testing.assert_array_equal(y.float().cpu().numpy(), ref.float().numpy())


def test_nm_select_matches_oracle():
    from deltaattention_b200.dropin import nmDeltaFlashAttention as nm
    for (n, m, r, N) in [(2, 4, 4, 2000), (2, 4, 2, 777), (1, 4, 4, 1024), (3, 8, 8, 1500)]:
        k = I.post_rope_keys(2, 2, N, 128, 5e5, torch.bfloat16, seed=N)
        ref = O.nm_keep_mask(k, n, m, r)
        got = nm.nm_keep_mask(k.cuda(), n, m, r)
        np.testing.assert_array_equal(got.cpu().numpy(), ref.numpy())
        assert int(got[0, 0].sum()) == nm.nm_num_packed(N, n, m, r)


NM_CASES = [  # dtype, head_dim, n, m, ratio, N, layout
    (torch.float32, 64, 2, 4, 4, 1999, "bhsd"), (torch.float16, 256, 2, 4, 4, 1500, "bhsd"),
    (torch.bfloat16, 128, 2, 4, 4, 3001, "bshd"), (torch.bfloat16, 96, 2, 4, 4, 1000, "bhsd"),
    (torch.bfloat16, 128, 1, 3, 3, 2000, "bhsd"), (torch.float16, 64, 8, 16, 4, 4099, "bshd"),
    (torch.bfloat16, 16, 2, 4, 8, 777, "bhsd"),
]


@pytest.mark.parametrize("dt,D,n,m,r,N,layout", NM_CASES)
def test_nm_select_layouts_match_oracle(dt, D, n, m, r, N, layout):
    """N:M selection over dtypes, head dims 16-256 (96 takes the unstaged kernel), group sizes
    that do not divide a CTA's candidate count, ragged tails and the projection layout."""
    from deltaattention_b200.dropin import nmDeltaFlashAttention as nm
    k = I.post_rope_keys(2, 3, N, D, 5e5, dt, seed=N + D)
    ref = O.nm_keep_mask(k, n, m, r)
    kc = k.cuda() if layout == "bhsd" else k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    got = nm.nm_keep_mask(kc, n, m, r)
    np.testing.assert_array_equal(got.cpu().numpy(), ref.numpy())
    assert (got.sum(-1) == nm.nm_num_packed(N, n, m, r)).all()


# ------------------------------------------------------------------ attention
ATTN = [
    ("attn_fp32_periodic", torch.float32, 2, 600, 64, "periodic", 21),
    ("attn_fp32_delta", torch.float32, 2, 600, 64, "delta", 22),
    ("attn_fp32_w0", torch.float32, 2, 600, 64, "periodic", 23),
    ("attn_fp16_periodic", torch.float16, 2, 600, 128, "periodic", 24),
    ("attn_fp16_delta", torch.float16, 2, 520, 128, "delta", 25),
    ("attn_fp32_quirk", torch.float32, 2, 600, 64, "quirk", 26),
    ("attn_bf16_periodic", torch.bfloat16, 2, 600, 128, "periodic", 27),
    ("attn_bf16_delta", torch.bfloat16, 2, 520, 128, "delta", 28),
    ("attn_bf16_d64_w0", torch.bfloat16, 2, 400, 64, "periodic", 29),
]
VARIANT_KERNEL = {"hybrid": "hybrid_compressed_flash_kernel", "sanity": "hybrid_compressed_flash_kernel_sanity",
                  "pure_phase1": "pure_phase1_flash_kernel"}


def _launch_variant(variant, q, kd, vd, kp, vp, ts, counts, W, force_simt=False):
    """The launch modeling_llama.py:306-451 performs, through the drop-in kernel objects."""
    import deltaFlashAttention as dfa
    from deltaattention_b200 import launch
    B, H, N, D = q.shape
    out = torch.empty_like(q)
    args = (q, kd, vd, kp, vp, ts, counts, out,
            *q.stride(), *kd.stride(), *vd.stride(), *kp.stride(), *vp.stride(), *ts.stride(), *counts.stride(),
            *out.stride(), D ** -0.5, N, kd.shape[2], kp.shape[2], D, H, W)
    grid = (-(-N // 128), B * H, 1)
    bd = 1 << (D - 1).bit_length()
    if force_simt:
        b = launch._bind(launch.HYBRID_PARAMS, args, dict(BLOCK_M=128, BLOCK_N=128, BLOCK_D=bd), "x")
        launch.hybrid_call({"hybrid": 0, "sanity": 1, "pure_phase1": 2}[variant], launch._grid(grid, b), b,
                           force_simt=True)
    else:
        getattr(dfa, VARIANT_KERNEL[variant])[grid](*args, BLOCK_M=128, BLOCK_N=128, BLOCK_D=bd, num_warps=8,
                                                    num_stages=1)
    return out


@pytest.mark.parametrize("case", ATTN, ids=[c[0] for c in ATTN])
@pytest.mark.parametrize("variant", ["hybrid", "sanity", "pure_phase1"])
def test_hybrid_variants_match_reference(golden, case, variant):
    name, dt, H, N, D, packing, seed = case
    g = golden(name)
    q, k, v = I.attn_inputs(1, H, N, D, dt, seed)
    keep = torch.from_numpy(g["keep"])
    _, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    c = lambda t: t.cuda().contiguous()  # noqa: E731
    out = _launch_variant(variant, c(q), c(k), c(v), c(kp), c(vp), c(ts), c(counts.float()), int(g["W"]))
    _cmp(out, torch.from_numpy(g[variant]), dt, f"{name}/{variant}")
    _check_ws_clean()


@pytest.mark.parametrize("case", [ATTN[0], ATTN[3], ATTN[6], ATTN[8]],
                         ids=[ATTN[0][0], ATTN[3][0], ATTN[6][0], ATTN[8][0]])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_matches_reference(golden, case, causal):
    import flashAttention as fa
    name, dt, H, N, D, packing, seed = case
    g = golden(name)
    q, k, v = I.attn_inputs(1, H, N, D, dt, seed)
    out = fa.triton_flash_attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    _cmp(out, torch.from_numpy(g["flash_causal" if causal else "flash_noncausal"]), dt, name)
    _check_ws_clean()


@pytest.mark.parametrize("variant", ["hybrid", "sanity", "pure_phase1"])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [128, 64])
def test_tcgen05_vs_simt_and_oracle(variant, dt, D):
    """Expanded-head call (repeat_kv layout): tcgen05 path vs the oracle, ragged N."""
    H, N = 3, 1000
    q, k, v = I.attn_inputs(1, H, N, D, dt, 90 + D)
    keep = O.periodic_keep_mask(1, H, N, 0.25)
    _, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    ref = O.hybrid_attention(q, k, v, kp, vp, ts, counts.float(), D ** -0.5, 128, variant)
    c = lambda t: t.cuda().contiguous()  # noqa: E731
    out = _launch_variant(variant, c(q), c(k), c(v), c(kp), c(vp), c(ts), c(counts.float()), 128)
    _cmp(out, ref, dt, f"tc/{variant}")
    simt = _launch_variant(variant, c(q), c(k), c(v), c(kp), c(vp), c(ts), c(counts.float()), 128, force_simt=True)
    _cmp(simt, ref, dt, f"simt/{variant}")
    _check_ws_clean()


@pytest.mark.parametrize("disorder", ["sorted", "permuted", "zero_count"])
def test_pure_phase1_prefix_and_general_masks(disorder):
    """Pure phase 1 (bf16): a packed block whose timestamps ascend and whose counts are positive
    takes a per-row prefix mask on the streaming path; a block with keys out of timestamp order
    (the packed rows permuted inside their 128-key block, K / V / timestamps / counts together)
    or a zero count below the packed length takes the general per-key mask. Each against the
    oracle on the same packed tensors, which does not depend on the key order."""
    dt, H, N, D = torch.bfloat16, 2, 1500, 128
    q, k, v = I.attn_inputs(1, H, N, D, dt, 61)
    keep = O.periodic_keep_mask(1, H, N, 0.25)
    _, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    counts = counts.float()
    if disorder == "permuted":
        g = torch.Generator().manual_seed(5)
        M = kp.shape[2]
        perm = torch.cat([b0 + torch.randperm(min(128, M - b0), generator=g) for b0 in range(0, M, 128)])
        kp, vp, ts, counts = kp[:, :, perm], vp[:, :, perm], ts[:, :, perm], counts[:, :, perm]
    elif disorder == "zero_count":
        counts[:, :, 5] = 0.0
        counts[:, :, 200] = 0.0
    ref = O.hybrid_attention(q, k, v, kp, vp, ts, counts, D ** -0.5, 128, "pure_phase1")
    c = lambda t: t.cuda().contiguous()  # noqa: E731
    out = _launch_variant("pure_phase1", c(q), c(k), c(v), c(kp), c(vp), c(ts), c(counts), 128)
    _cmp(out, ref, dt, f"pure/{disorder}")
    _check_ws_clean()


@pytest.mark.parametrize("variant", ["hybrid", "sanity", "pure_phase1"])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_tcgen05_score_jumps(variant, dt):
    """Keys planted with ever larger scores in the middle of blocks (later 32-column chunks of
    packed and dense tiles): every row's running maximum jumps far past its reference mid-tile,
    which exercises the rescale of partly written probabilities."""
    H, N, D = 2, 1500, 128
    q, k, v = I.attn_inputs(1, H, N, D, dt, 77)
    q = (q.float() + 1.0).to(dt)
    k = k.float()
    for i, t in enumerate([300, 400, 680, 700, 1100, 1400]):  # dense chunks 1-3; packed t % 4 == 0
        k[:, :, t, :] += 2.0 + 0.75 * i
    k = k.to(dt)
    keep = O.periodic_keep_mask(1, H, N, 0.25)
    _, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    ref = O.hybrid_attention(q, k, v, kp, vp, ts, counts.float(), D ** -0.5, 128, variant)
    c = lambda t: t.cuda().contiguous()  # noqa: E731
    out = _launch_variant(variant, c(q), c(k), c(v), c(kp), c(vp), c(ts), c(counts.float()), 128)
    _cmp(out, ref, dt, f"tc-jumps/{variant}")
    _check_ws_clean()


@pytest.mark.parametrize("mode", ["periodic", "delta"])
def test_native_gqa_prefill_matches_oracle(mode):
    """ops.delta_prefill: RoPE + selection + device packing + GQA-by-index attention."""
    from deltaattention_b200 import ops, synth
    B, Hq, Hkv, N, D = 1, 8, 2, 2304, 128
    q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.bfloat16, seed=5, device="cpu")
    cos, sin = synth.rope_tables(N, D, 5e5, torch.bfloat16)
    kw = dict(mode=mode, keep_rate=0.25) if mode == "periodic" else dict(mode="delta", threshold=1.6,
                                                                          chunk_size=512)
    out, packed, k_rot = ops.delta_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), return_packed=True,
                                           **kw)
    packed = packed.materialize()
    q_ref = O.apply_rope(q.contiguous(), cos, sin)
    k_ref = O.apply_rope(k.contiguous(), cos, sin)
    np.testing.assert_array_equal(k_rot.float().cpu().numpy(), k_ref.float().numpy())
    if mode == "periodic":
        keep = O.periodic_keep_mask(B, Hkv, N, 0.25)
    else:
        keep, _ = O.delta_keep_mask(k_ref, 1.6 ** 2, False, 512, N // 512 + 1)
        np.testing.assert_array_equal(packed.keep_mask.cpu().numpy(), keep.numpy())
    _, kp, vp, ts, counts = O.pack_from_keep(k_ref, v.contiguous(), keep)
    np.testing.assert_array_equal(packed.timestamps.cpu().numpy(), ts.numpy())
    np.testing.assert_array_equal(packed.counts.cpu().numpy(), counts.numpy())
    ref = O.hybrid_attention(q_ref, k_ref, v.contiguous(), kp, vp, ts, counts.float(), D ** -0.5, 128, "hybrid",
                             n_rep=Hq // Hkv)
    _cmp(out, ref, torch.bfloat16, f"native/{mode}")
    _check_ws_clean()


@pytest.mark.parametrize("threshold", [8.0, 11.0, 14.0])
def test_delta_mode_fused_matches_separate_kernels_and_oracle(threshold):
    """The fused key compression (RoPE + scan + packing in one launch, packed length on the
    device) against the separate RoPE / scan / pack kernels with the host length: rotated keys,
    keep mask, anchors and every packed row bit-identical, rows past each head's anchors zero up
    to its block end; the device-length attention (per-key count weights on the streaming path)
    agrees with the host-length call on the same packing, and both match the oracle within the
    bf16 tolerance (N = 4096, GQA 4:1)."""
    from deltaattention_b200 import ops, synth
    B, Hq, Hkv, N, D = 1, 8, 2, 4096, 128
    q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.bfloat16, seed=33, device="cuda")
    cos, sin = synth.rope_tables(N, D, 5e5, torch.bfloat16, device="cuda")
    out, pk, k_rot = ops.delta_prefill(q, k, v, cos, sin, mode="delta", threshold=threshold, return_packed=True)
    out2, pk2, k_rot2 = ops.delta_prefill(q, k, v, cos, sin, mode="delta", threshold=threshold, return_packed=True,
                                          fused=False)
    assert pk.anchors is not None and pk2.anchors is None
    assert torch.equal(k_rot.view(torch.int16), k_rot2.view(torch.int16))
    assert torch.equal(pk.keep_mask, pk2.keep_mask)
    A = pk.anchors.view(B, Hkv).cpu()
    assert torch.equal(A, pk2.keep_mask.sum(-1).cpu().int())
    for h in range(Hkv):
        a = int(A[0, h])
        z = min(pk.k.shape[2], -(-a // 128) * 128)
        assert torch.equal(pk.k[0, h, :a].view(torch.int16), pk2.k[0, h, :a].view(torch.int16))
        assert torch.equal(pk.v[0, h, :a].view(torch.int16), pk2.v[0, h, :a].view(torch.int16))
        assert torch.equal(pk.timestamps[0, h, :a], pk2.timestamps[0, h, :a])
        assert torch.equal(pk.counts[0, h, :a], pk2.counts[0, h, :a])
        assert (pk.k[0, h, a:z] == 0).all() and (pk.v[0, h, a:z] == 0).all()
        assert (pk.timestamps[0, h, a:z] == 0).all() and (pk.counts[0, h, a:z] == 0).all()
    m = pk.materialize()
    assert torch.equal(m.timestamps, pk2.timestamps) and torch.equal(m.counts, pk2.counts)
    c = m.counts
    assert (c[:, :, :128].amax(-1) != c[:, :, :128].amin(-1)).any(), "counts should differ within a block"
    # the device-length attention weights each key by its count on the streaming path; the
    # host-length call takes the exact two-pass path for those blocks: equal within rounding
    _cmp(out, out2, torch.bfloat16, f"delta fused vs separate kernels, threshold {threshold}")
    q_ref = O.apply_rope(q.cpu().contiguous(), cos.cpu(), sin.cpu())
    k_ref = k_rot.cpu()
    ref = O.hybrid_attention(q_ref, k_ref, v.cpu().contiguous(), m.k.cpu(), m.v.cpu(), m.timestamps.cpu(),
                             m.counts.cpu().float(), D ** -0.5, 128, n_rep=Hq // Hkv, heads=[0, 7])
    for h in (0, 7):
        _cmp(out[:, h], ref[:, h], torch.bfloat16, f"delta fused vs oracle, threshold {threshold}, head {h}")
    _check_ws_clean()


@pytest.mark.parametrize("B,group,qgroup", [(2, 1, None), (1, 2, None), (1, 3, None), (2, 1, 1), (1, 1, 2)])
def test_host_pipelined_prefill_equals_device_call(B, group, qgroup):
    """ops.delta_prefill_host (kv-head groups, copies overlapped with compute on three streams)
    writes exactly what one ops.delta_prefill call on the device tensors returns."""
    from deltaattention_b200 import ops, synth
    Hq, Hkv, N, D = 8, 4, 1536, 128
    q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.bfloat16, seed=11, device="cuda")
    cos, sin = synth.rope_tables(N, D, 5e5, torch.bfloat16, device="cuda")
    kw = dict(mode="periodic", keep_rate=0.25)
    want = ops.delta_prefill(q, k, v, cos, sin, **kw).cpu()
    hq, hk, hv = (t.contiguous().cpu().pin_memory() for t in (q, k, v))
    ho = torch.full((B, Hq, N, D), float("nan"), dtype=torch.bfloat16).pin_memory()
    for _ in range(2):  # a second call reuses the cached copy streams
        ops.delta_prefill_host(hq, hk, hv, cos, sin, out=ho, kv_heads_per_group=group, q_heads_per_group=qgroup,
                               **kw)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(ho.view(torch.int16), want.view(torch.int16))
    _check_ws_clean()


@pytest.mark.parametrize("group,qgroup", [(1, None), (2, None), (1, 2)])
def test_host_prefill_back_to_back_calls(group, qgroup):
    """Consecutive delta_prefill_host calls with no synchronisation between them (the next
    call's copies overwrite the kept device buffers while the previous call still computes and
    drains): every call's output equals its own device call, bit for bit."""
    from deltaattention_b200 import ops, synth
    B, Hq, Hkv, N, D = 1, 8, 4, 4096, 128
    cos, sin = synth.rope_tables(N, D, 5e5, torch.bfloat16, device="cuda")
    kw = dict(mode="periodic", keep_rate=0.25)
    ins, wants, outs = [], [], []
    for seed in range(4):
        q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.bfloat16, seed=100 + seed, device="cuda")
        wants.append(ops.delta_prefill(q, k, v, cos, sin, **kw).cpu())
        ins.append(tuple(t.contiguous().cpu().pin_memory() for t in (q, k, v)))
        outs.append(torch.full((B, Hq, N, D), float("nan"), dtype=torch.bfloat16).pin_memory())
    torch.cuda.synchronize()
    for (hq, hk, hv), ho in zip(ins, outs):
        ops.delta_prefill_host(hq, hk, hv, cos, sin, out=ho, kv_heads_per_group=group, q_heads_per_group=qgroup,
                               **kw)
    torch.cuda.current_stream().synchronize()
    for ho, want in zip(outs, wants):
        assert torch.equal(ho.view(torch.int16), want.view(torch.int16))
    ops.release_host_prefill_buffers()
    _check_ws_clean()


@pytest.mark.parametrize("selection", ["nm", "periodic"])
def test_varlen_prefill_equals_per_sequence_calls(selection):
    """ops.delta_prefill_varlen over ragged sequences packed back to back (several streams):
    every sequence's output and packed history equal a call on that sequence alone."""
    from deltaattention_b200 import ops, synth
    from deltaattention_b200.dropin import nmDeltaFlashAttention as nm
    lens = [700, 1536, 1000, 2048, 513, 129]
    cu = [0]
    for n_ in lens:
        cu.append(cu[-1] + n_)
    Hq, Hkv, D = 8, 2, 128
    q, k, v = synth.layer_inputs(1, Hq, Hkv, cu[-1], D, torch.bfloat16, seed=41, device="cuda", qv_scale=1.0,
                                 key_offset=False)
    cos, sin = synth.rope_tables(max(lens), D, 5e5, torch.bfloat16, device="cuda")
    out, packed = ops.delta_prefill_varlen(q, k, v, cos, sin, cu, selection=selection, streams=3,
                                           return_packed=True)
    torch.cuda.synchronize()
    for i, (s0, s1) in enumerate(zip(cu, cu[1:])):
        q_rot = ops.rope(q[:, :, s0:s1], cos, sin)
        k_rot = ops.rope(k[:, :, s0:s1], cos, sin)
        if selection == "nm":
            want, pk = nm.nm_delta_flash_attention(q_rot, k_rot, v[:, :, s0:s1], 2, 4, 4, return_packed=True)
        else:
            pk = ops.pack_periodic(k_rot, v[:, :, s0:s1], 4)
            want = ops.attention(q_rot, k_rot, v[:, :, s0:s1], pk)
        got_pk, got_k = packed[i]
        assert torch.equal(out[:, :, s0:s1].view(torch.int16), want.view(torch.int16)), (selection, i)
        assert torch.equal(got_k.view(torch.int16), k_rot.view(torch.int16))
        assert torch.equal(got_pk.k.view(torch.int16), pk.k.view(torch.int16))
        assert torch.equal(got_pk.timestamps, pk.timestamps) and torch.equal(got_pk.counts, pk.counts)
    _check_ws_clean()


def test_cfg1_fp32_full_size():
    """BASELINE config 1 (fp32, B=1, H=8, N=2048, d=64, r=4) at 1e-4."""
    from deltaattention_b200 import ops, synth
    c = synth.CONFIGS["cfg1"]
    q, k, v = synth.layer_inputs(1, 8, 8, 2048, 64, torch.float32, seed=0, device="cpu", qv_scale=1.0,
                                 key_offset=False)
    cos, sin = synth.rope_tables(2048, 64, c["theta"], torch.float32)
    out = ops.delta_prefill(q.cuda(), k.cuda(), v.cuda(), cos.cuda(), sin.cuda(), keep_rate=0.25)
    q_ref, k_ref = O.apply_rope(q.contiguous(), cos, sin), O.apply_rope(k.contiguous(), cos, sin)
    keep = O.periodic_keep_mask(1, 8, 2048, 0.25)
    _, kp, vp, ts, counts = O.pack_from_keep(k_ref, v.contiguous(), keep)
    ref = O.hybrid_attention(q_ref, k_ref, v.contiguous(), kp, vp, ts, counts.float(), 64 ** -0.5, 128)
    _cmp(out, ref, torch.float32, "cfg1")


def test_cfg2_full_size_sampled_heads():
    """BASELINE config 2 shape (bf16, Hq=32, Hkv=8, N=32768, d=128, r=4): all rows of two
    q-heads against the oracle, plus size-independent properties on every head."""
    from deltaattention_b200 import ops, synth
    N = 32768
    q, k, v = synth.layer_inputs(1, 32, 8, N, 128, torch.bfloat16, seed=1, device="cuda")
    cos, sin = synth.rope_tables(N, 128, 5e5, torch.bfloat16, device="cuda")
    out = ops.delta_prefill(q, k, v, cos, sin, keep_rate=0.25)
    assert torch.isfinite(out.float()).all()
    heads = [0, 13]
    qc, kc, vc = q.cpu().contiguous(), k.cpu().contiguous(), v.cpu().contiguous()
    cc, sc = cos.cpu(), sin.cpu()
    q_ref, k_ref = O.apply_rope(qc, cc, sc), O.apply_rope(kc, cc, sc)
    keep = O.periodic_keep_mask(1, 8, N, 0.25)
    _, kp, vp, ts, counts = O.pack_from_keep(k_ref, vc, keep)
    ref = O.hybrid_attention(q_ref, k_ref, vc, kp, vp, ts, counts.float(), 128 ** -0.5, 128, n_rep=4, heads=heads)
    for h in heads:
        _cmp(out[:, h], ref[:, h], torch.bfloat16, f"cfg2/head{h}")
    # attention rows are convex combinations of V rows: bounded by V's range
    vmax = v.abs().amax().float()
    assert out.float().abs().amax() <= vmax * 1.01
    _check_ws_clean()


def test_dense_r1_matches_flash_kernel():
    """r = 1 through the hybrid kernel equals plain causal flash (same kernel family)."""
    from deltaattention_b200 import ops, synth
    q, k, v = synth.layer_inputs(1, 8, 2, 2048, 128, torch.bfloat16, seed=3, device="cuda")
    cos, sin = synth.rope_tables(2048, 128, 5e5, torch.bfloat16, device="cuda")
    qr, kr = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
    dense = ops.flash(qr, kr, v)
    ref = O.flash_attention(qr.cpu(), kr.cpu(), v.cpu().contiguous(), n_rep=4)
    _cmp(dense, ref, torch.bfloat16, "flash-gqa")


# ------------------------------------------------------------------ decoding
@pytest.mark.parametrize("name,dt,use_cos", [("decode_fp32_euclid", torch.float32, False),
                                             ("decode_fp16_cosine", torch.float16, True),
                                             ("decode_bf16_euclid", torch.bfloat16, False)])
def test_decode_replay_matches_reference(golden, name, dt, use_cos):
    import deltaDecoding as dd
    g = golden(name)
    st = I.decode_setup(dt, seed=31)
    B, Hkv, Hq, D, W = st["B"], st["Hkv"], st["Hq"], st["D"], st["W"]
    thr = float(g["threshold"])
    c = lambda t: t.cuda()  # noqa: E731
    kp, vp, cnt, tss, lens = c(st["kp"]), c(st["vp"]), c(st["counts"]), c(st["ts"]), c(st["lengths"])
    ke, ve = c(st["ke"]), c(st["ve"])
    exact_len, total = st["exact_len"], st["total"]
    outs = []
    for step in range(st["steps"]):
        nk, nv = c(st["new_k"][step]), c(st["new_v"][step])
        dd.fused_hybrid_decode_update_kernel[(B * Hkv,)](
            nk, nv, ke, ve, kp, vp, cnt, tss, lens, exact_len, total, thr, W,
            *nk.stride(), *ke.stride(), *kp.stride(), *cnt.stride(), Hkv, D, BLOCK_D=D, USE_COSINE=use_cos)
        exact_len += 1
        total += 1
        np.testing.assert_array_equal(lens.cpu().numpy(), g["lengths"][step])
        q = c(st["q"][step])
        out = torch.empty_like(q)
        lv = lens.view(B, Hkv)
        dd.fused_hybrid_decode_kernel[(B, Hq)](
            q, kp, vp, cnt, lv, ke, ve, out, *q.stride(), *kp.stride(), *vp.stride(), *cnt.stride(), *lv.stride(),
            *ke.stride(), *ve.stride(), *out.stride(), D ** -0.5, min(exact_len, W), Hq // Hkv, head_dim=D,
            BLOCK_M=16, BLOCK_N=128, BLOCK_D=D)
        outs.append(out.float().cpu())
    np.testing.assert_array_equal(cnt.cpu().numpy(), g["counts"])
    np.testing.assert_array_equal(tss.cpu().numpy(), g["timestamps"])
    np.testing.assert_array_equal(kp.float().cpu().numpy(), g["k_packed"])
    np.testing.assert_array_equal(ke.float().cpu().numpy(), g["k_exact"])
    _cmp(torch.stack(outs), torch.from_numpy(g["outputs"]), dt, name)


@pytest.mark.parametrize("dt,D,G,B,Hkv", [(torch.bfloat16, 128, 4, 3, 2), (torch.float16, 64, 8, 2, 1),
                                          (torch.bfloat16, 128, 1, 2, 2), (torch.bfloat16, 64, 2, 1, 3)])
def test_decode_attention_16bit_matches_oracle(dt, D, G, B, Hkv):
    """The 16-bit decode path (tensor-core split-K chunks of 128 keys, then the combine) on
    ragged packed lengths (0, short, not multiples of 128, several chunks) plus an exact
    window, against the oracle's fused_hybrid_decode_kernel restatement."""
    import deltaDecoding as dd
    g = torch.Generator().manual_seed(40 + D + G)
    cap, W = 700, 24
    Hq = Hkv * G
    kp = (torch.randn((B, Hkv, cap, D), generator=g) * 0.5).to(dt)
    vp = torch.randn((B, Hkv, cap, D), generator=g).to(dt)
    cnt = torch.randint(1, 9, (B, Hkv, cap), generator=g, dtype=torch.int32)
    lens_all = [0, 5, 127, 128, 129, 300, 650, 700]
    lens = torch.tensor([lens_all[(i * 3 + 1) % len(lens_all)] for i in range(B * Hkv)], dtype=torch.int32)
    lens = lens.view(B, Hkv)
    ke = (torch.randn((B, Hkv, W, D), generator=g) * 0.5).to(dt)
    ve = torch.randn((B, Hkv, W, D), generator=g).to(dt)
    q = (torch.randn((B, Hq, D), generator=g) * 0.5).to(dt)
    for exact_len in (W, 7):
        ref = O.decode_attention(q, kp, vp, cnt, lens, ke, ve, D ** -0.5, exact_len, G)
        c = lambda t: t.cuda()  # noqa: E731
        qc, kpc, vpc, cc, lc, kec, vec = c(q), c(kp), c(vp), c(cnt), c(lens), c(ke), c(ve)
        out = torch.empty_like(qc)
        dd.fused_hybrid_decode_kernel[(B, Hq)](
            qc, kpc, vpc, cc, lc, kec, vec, out, *qc.stride(), *kpc.stride(), *vpc.stride(), *cc.stride(),
            *lc.stride(), *kec.stride(), *vec.stride(), *out.stride(), D ** -0.5, exact_len, G, head_dim=D,
            BLOCK_M=16, BLOCK_N=128, BLOCK_D=D)
        _cmp(out, ref, dt, f"decode16/{D}/{G}/{exact_len}")
    _check_ws_clean()


def _device_cache_setup(layers, seed, dt=torch.bfloat16, D=128):
    """A prefilled DeviceDecodeCache plus the same state as plain tensors for the host-length
    launches of the reference API."""
    from deltaattention_b200.cache import DeviceDecodeCache
    g = torch.Generator().manual_seed(seed)
    B, Hkv, G, W, N0, cap = 2, 2, 4, 16, 240, 160
    thr = 8.0 * (D / 128) ** 0.5  # window keys merge into the last anchor, fresh tokens append
    c = DeviceDecodeCache(layers, B, Hkv, D, cap, W, dt, threshold=thr)
    for layer in range(layers):
        keys = torch.from_numpy(I.ar1_keys(B, Hkv, N0, D, seed=seed + layer)).to(dt)
        vals = (torch.randn((B, Hkv, N0, D), generator=g) * 0.5).to(dt)
        keep = O.periodic_keep_mask(B, Hkv, N0 - W, 0.25)
        _, kp, vp, ts, counts = O.pack_from_keep(keys[:, :, :N0 - W], vals[:, :, :N0 - W], keep)
        c.load_prefill(layer, kp.cuda(), vp.cuda(), counts.cuda(), ts.cuda(), keys[:, :, N0 - W:].cuda(),
                       vals[:, :, N0 - W:].cuda(), N0)
    host = dict(k_packed=c.k_packed.clone(), v_packed=c.v_packed.clone(), counts=c.packed_counts.clone(),
                ts=c.packed_timestamps.clone(), lens=c.packed_lengths.clone(), k_exact=c.k_exact.clone(),
                v_exact=c.v_exact.clone(), exact=[W] * layers, total=[N0] * layers)
    steps = []
    for _ in range(24):
        steps.append(((torch.randn((layers, B, Hkv * G, D), generator=g) * 0.5).to(dt).cuda(),
                      (torch.randn((layers, B, Hkv, 1, D), generator=g) * 0.5).to(dt).cuda(),
                      (torch.randn((layers, B, Hkv, 1, D), generator=g) * 0.5).to(dt).cuda()))
    return c, host, steps, dict(B=B, Hkv=Hkv, G=G, D=D, W=W, thr=thr)


def _host_length_step(host, layer, q, k_new, v_new, p):
    """One decode step through the reference-API kernels with host lengths (deltaDecoding.py)."""
    import deltaDecoding as dd
    B, Hkv, G, D, W = p["B"], p["Hkv"], p["G"], p["D"], p["W"]
    ke, ve, kp, vp = host["k_exact"][layer], host["v_exact"][layer], host["k_packed"][layer], host["v_packed"][layer]
    cnt, tss, lens = host["counts"][layer], host["ts"][layer], host["lens"][layer]
    dd.fused_hybrid_decode_update_kernel[(B * Hkv,)](
        k_new, v_new, ke, ve, kp, vp, cnt, tss, lens, host["exact"][layer], host["total"][layer], p["thr"] ** 2, W,
        *k_new.stride(), *ke.stride(), *kp.stride(), *cnt.stride(), Hkv, D, BLOCK_D=D, USE_COSINE=False)
    host["exact"][layer] += 1
    host["total"][layer] += 1
    out = torch.empty_like(q)
    lv = lens.view(B, Hkv)
    dd.fused_hybrid_decode_kernel[(B, Hkv * G)](
        q, kp, vp, cnt, lv, ke, ve, out, *q.stride(), *kp.stride(), *vp.stride(), *cnt.stride(), *lv.stride(),
        *ke.stride(), *ve.stride(), *out.stride(), D ** -0.5, min(host["exact"][layer], W), G, head_dim=D,
        BLOCK_M=16, BLOCK_N=128, BLOCK_D=D)
    return out


@pytest.mark.parametrize("dt,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_device_decode_cache_matches_host_lengths(dt, D):
    """DeviceDecodeCache (lengths on the device, advanced on the device) gives bit-identical
    outputs and cache contents to the reference-API launches with host lengths, over steps
    that both merge into and append to the packed history."""
    layers = 2
    c, host, steps, p = _device_cache_setup(layers, seed=61, dt=dt, D=D)
    for q, kn, vn in steps:
        for layer in range(layers):
            got = c.step(layer, q[layer], kn[layer], vn[layer])
            want = _host_length_step(host, layer, q[layer], kn[layer], vn[layer], p)
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    torch.cuda.synchronize()
    assert c.lengths() == [(host["exact"][i], host["total"][i]) for i in range(layers)]
    assert torch.equal(c.packed_lengths, host["lens"])
    assert torch.equal(c.packed_counts, host["counts"]) and torch.equal(c.packed_timestamps, host["ts"])
    assert torch.equal(c.k_packed.view(torch.int16), host["k_packed"].view(torch.int16))
    assert torch.equal(c.k_exact.view(torch.int16), host["k_exact"].view(torch.int16))
    grew = c.packed_lengths.max().item() > 40 and c.packed_counts.max().item() > 4
    assert grew, "the steps should both append anchors and merge into them"
    assert int(c.err.item()) == 0
    _check_ws_clean()


def test_device_decode_cache_folded_advance_equals_separate():
    """step() folds the length advance into the attention call (two launches); update with its
    own advance kernel followed by attend gives bit-identical outputs, lengths and cache."""
    layers = 2
    a, _, steps, _ = _device_cache_setup(layers, seed=63)
    b, _, _, _ = _device_cache_setup(layers, seed=63)
    for q, kn, vn in steps:
        for layer in range(layers):
            got = a.step(layer, q[layer], kn[layer], vn[layer])
            b.update(layer, kn[layer], vn[layer], advance=True)
            want = b.attend(layer, q[layer], advance=False)
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    torch.cuda.synchronize()
    assert a.lengths() == b.lengths()
    assert torch.equal(a.packed_counts, b.packed_counts) and torch.equal(a.packed_lengths, b.packed_lengths)
    assert torch.equal(a.k_exact.view(torch.int16), b.k_exact.view(torch.int16))
    _check_ws_clean()


@pytest.mark.parametrize("dt,D", [(torch.bfloat16, 128), (torch.float16, 64)])
def test_device_decode_cache_graph_replay(dt, D):
    """A decode step over every layer captured once in a CUDA graph and replayed per token
    equals the eager steps token by token."""
    layers = 2
    eager, _, steps, _ = _device_cache_setup(layers, seed=62, dt=dt, D=D)
    graphed, _, _, _ = _device_cache_setup(layers, seed=62, dt=dt, D=D)
    q0, k0, v0 = steps[0]
    for layer in range(layers):  # one eager step on both (kernel attributes are set outside capture)
        eager.step(layer, q0[layer], k0[layer], v0[layer])
        graphed.step(layer, q0[layer], k0[layer], v0[layer])
    sq, sk, sv = torch.empty_like(q0), torch.empty_like(k0), torch.empty_like(v0)
    sout = torch.empty_like(q0)
    graph = graphed.capture_step(sq, sk, sv, sout)
    for q, kn, vn in steps[1:]:
        want = torch.stack([eager.step(layer, q[layer], kn[layer], vn[layer]) for layer in range(layers)])
        sq.copy_(q)
        sk.copy_(kn)
        sv.copy_(vn)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(sout.view(torch.int16), want.view(torch.int16))
    assert eager.lengths() == graphed.lengths()
    del graph
    _check_ws_clean()


def test_hybrid_cache_end_to_end():
    """HybridCompressedCache: prefill hand-off then decode steps, against the oracle."""
    import types
    import deltaDecoding as dd
    cfg = types.SimpleNamespace(hidden_size=8 * 128, num_attention_heads=8, num_key_value_heads=2,
                                num_hidden_layers=1, head_dim=128)
    cache = dd.HybridCompressedCache(cfg, batch_size=1, dtype=torch.bfloat16, exact_window_size=32,
                                     initial_capacity=64)
    N0, D = 300, 128
    keys = torch.from_numpy(I.ar1_keys(1, 2, N0 + 20, D, seed=8)).bfloat16()
    vals = torch.from_numpy(I.normal((1, 2, N0 + 20, D), seed=9)).bfloat16()
    keep = O.periodic_keep_mask(1, 2, N0, 0.25)
    _, kp, vp, ts, counts = O.pack_from_keep(keys[:, :, :N0], vals[:, :, :N0], keep)
    cache.initialize_from_prefill(0, kp.cuda(), vp.cuda(), counts.cuda(), ts.cuda(), keys[:, :, N0 - 32:N0].cuda(),
                                  vals[:, :, N0 - 32:N0].cuda(), N0)
    assert cache.capacity >= kp.shape[2]
    ref_state = [kp.clone(), vp.clone(), counts.clone(), ts.clone(),
                 torch.tensor([kp.shape[2]] * 2, dtype=torch.int32), keys[:, :, N0 - 32:N0].clone(),
                 vals[:, :, N0 - 32:N0].clone()]
    cap = cache.capacity
    pad = lambda t, n: torch.cat([t, torch.zeros((*t.shape[:2], n - t.shape[2], *t.shape[3:]), dtype=t.dtype)], 2)  # noqa
    rk, rv, rc, rt = pad(ref_state[0], cap), pad(ref_state[1], cap), pad(ref_state[2], cap), pad(ref_state[3], cap)
    rl, rke, rve = ref_state[4], ref_state[5], ref_state[6]
    exact, total = 32, N0
    for s in range(20):
        nk, nv = keys[:, :, N0 + s:N0 + s + 1], vals[:, :, N0 + s:N0 + s + 1]
        cache.update(nk.cuda(), nv.cuda(), 0)
        O.decode_update(nk, nv, rke, rve, rk, rv, rc, rt, rl, exact, total, 0.0, 32, False)
        exact += 1
        total += 1
    np.testing.assert_array_equal(cache.packed_lengths[0].cpu().numpy(), rl.numpy())
    L = int(rl.max())
    np.testing.assert_array_equal(cache.packed_counts[0][:, :, :L].cpu().numpy(), rc[:, :, :L].numpy())
    np.testing.assert_array_equal(cache.packed_timestamps[0][:, :, :L].cpu().numpy(), rt[:, :, :L].numpy())

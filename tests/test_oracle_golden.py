"""Pin the CPU oracle against golden vectors produced by the reference's own kernels.

The fixtures in tests/golden were produced by ``gen_golden.py`` running the reference
Triton kernels under TRITON_INTERPRET=1 (the bf16 ones on the interpreter with IEEE bf16
arithmetic, ``bf16_interp``). Selection / packing / decode-cache state must match bit for
bit; attention outputs within the tolerances below.
"""
import numpy as np
import pytest
import torch

import _inputs as I
from oracle import delta_oracle as O


def test_interpreter_bf16_arithmetic_is_bitwise(golden):
    g = golden("bf16_interp_probe")
    # the interpreter subtracts raw bit patterns: not the bf16 difference
    assert not np.array_equal(g["interp"], g["true"])


def test_patched_interpreter_bf16_arithmetic_is_ieee(golden):
    g = golden("bf16_interp_ieee_probe")
    # with bf16_interp installed the same kernel gives the correctly rounded difference,
    # including a tie (1 - 2^-8 rounds to even), overflow to +inf and a signed zero
    np.testing.assert_array_equal(g["interp"], g["true"])


def test_bf16_rounding_helpers_agree_with_torch():
    import bf16_interp as BI
    x = np.random.default_rng(0).standard_normal(4096).astype(np.float32) * 10.0 ** np.arange(-20, 20, 10 / 1024)[:4096].astype(np.float32)
    x = np.concatenate([x, np.float32([0.0, -0.0, np.inf, -np.inf, 3.4e38, 1.0 + 2.0 ** -8,
                                      1.0 + 3 * 2.0 ** -8])])
    ours = BI.f32_to_bf16_bits(x)
    ref = torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, ref)
    np.testing.assert_array_equal(BI.bf16_bits_to_f32(ours), torch.from_numpy(ref.view(np.int16)).view(torch.bfloat16).float().numpy())


@pytest.mark.parametrize("dt_name,dt", [("bf16", torch.bfloat16), ("fp32", torch.float32)])
def test_rope_matches_reference_eager(golden, dt_name, dt):
    g = golden(f"rope_{dt_name}")
    x = torch.from_numpy(I.ar1_keys(1, 2, 300, 128, seed=11, offset=True)).to(dt)
    assert float(x.double().sum()) == pytest.approx(float(g["in_sum"]), rel=0, abs=1e-6)
    cos, sin = O.rope_cos_sin(300, 128, 500000.0, dt)
    np.testing.assert_array_equal(cos.float().numpy(), g["cos"])
    out = O.apply_rope(x, cos, sin)
    np.testing.assert_array_equal(out.float().numpy(), g["out"])


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
def test_delta_keep_mask_bit_exact(golden, case):
    name, dt, B, H, N, D, chunk, use_cos, theta, seed = case
    g = golden(name)
    k = I.post_rope_keys(B, H, N, D, theta, dt, seed=seed)
    assert float(k.double().sum()) == pytest.approx(float(g["in_sum"]), rel=1e-12)
    keep, cc = O.delta_keep_mask(k, float(g["threshold"]), use_cos, chunk, -(-N // chunk))
    np.testing.assert_array_equal(keep.numpy(), g["keep"])
    np.testing.assert_array_equal(cc.numpy(), g["chunk_counts"])
    frac = g["keep"].mean()
    assert 0.2 < frac < 0.9, frac   # the threshold exercises both branches


def test_delta_keep_mask_strided_input(golden):
    g = golden("keep_euclid_fp32_bshd")
    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1)
    kb = k.transpose(1, 2).contiguous().transpose(1, 2)
    keep, cc = O.delta_keep_mask(kb, float(g["threshold"]), False, 256, 4)
    np.testing.assert_array_equal(keep.numpy(), g["keep"])


def test_pack_bit_exact(golden):
    g = golden("pack_fp32")
    k = I.post_rope_keys(1, 2, 1000, 64, 1e4, torch.float32, seed=1)
    v = torch.from_numpy(I.normal((1, 2, 1000, 64), seed=101)).float()
    assert float(v.double().sum()) == pytest.approx(float(g["v_sum"]), rel=1e-12)
    keep = torch.from_numpy(g["keep"])
    im, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    np.testing.assert_array_equal(im.numpy(), g["index_map"])
    np.testing.assert_array_equal(kp.numpy(), g["k_packed"])
    np.testing.assert_array_equal(vp.numpy(), g["v_packed"])
    np.testing.assert_array_equal(ts.numpy(), g["timestamps"])
    np.testing.assert_array_equal(counts.numpy(), g["counts"])


def test_pack_bf16_bit_exact(golden):
    g = golden("pack_bf16")
    k = I.post_rope_keys(1, 2, 1000, 128, 5e5, torch.bfloat16, seed=6)
    v = torch.from_numpy(I.normal((1, 2, 1000, 128), seed=106)).to(torch.bfloat16)
    assert float(v.double().sum()) == pytest.approx(float(g["v_sum"]), rel=1e-12)
    keep, _ = O.delta_keep_mask(k, I.median_threshold(k, False), False, 300, 4)
    np.testing.assert_array_equal(keep.numpy(), g["keep"])
    im, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    np.testing.assert_array_equal(im.numpy(), g["index_map"])
    np.testing.assert_array_equal(kp.float().numpy(), g["k_packed"])
    np.testing.assert_array_equal(vp.float().numpy(), g["v_packed"])
    np.testing.assert_array_equal(ts.numpy(), g["timestamps"])
    np.testing.assert_array_equal(counts.numpy(), g["counts"])


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
TOL = {torch.float32: (2e-5, 2e-6), torch.float16: (4e-3, 2e-4), torch.bfloat16: (4e-3, 4e-5)}  # one bf16 ulp at |o| < 1


def attn_case(golden, case):
    name, dt, H, N, D, packing, seed = case
    g = golden(name)
    q, k, v = I.attn_inputs(1, H, N, D, dt, seed)
    assert float(q.double().sum()) == pytest.approx(float(g["q_sum"]), rel=1e-12)
    keep = torch.from_numpy(g["keep"])
    _, kp, vp, ts, counts = O.pack_from_keep(k, v, keep)
    return g, q, k, v, kp, vp, ts, counts, int(g["W"])


@pytest.mark.parametrize("case", ATTN, ids=[c[0] for c in ATTN])
@pytest.mark.parametrize("variant", ["hybrid", "sanity", "pure_phase1"])
def test_hybrid_attention_matches_reference(golden, case, variant):
    g, q, k, v, kp, vp, ts, counts, W = attn_case(golden, case)
    out = O.hybrid_attention(q, k, v, kp, vp, ts, counts.float(), q.shape[-1] ** -0.5, W, variant)
    ref = torch.from_numpy(g[variant])
    err = (out.float() - ref).abs()
    mx, mean = TOL[q.dtype]
    assert torch.isfinite(ref).all()
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())


@pytest.mark.parametrize("case", ATTN[:1] + ATTN[3:4] + ATTN[6:7], ids=[ATTN[0][0], ATTN[3][0], ATTN[6][0]])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_matches_reference(golden, case, causal):
    g, q, k, v, *_ = attn_case(golden, case)
    out = O.flash_attention(q, k, v, causal=causal)
    ref = torch.from_numpy(g["flash_causal" if causal else "flash_noncausal"])
    mx, mean = TOL[q.dtype]
    err = (out.float() - ref).abs()
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())


def test_delta_padding_block_restarts_dense_window(golden):
    """Reference quirk: a head with fewer anchors than M sees count-0 padding blocks
    whose max timestamp is 0, so last_safe drops to 0 and phase 2 restarts at key 0."""
    g, q, k, v, kp, vp, ts, counts, W = attn_case(golden, ATTN[5])
    M = kp.shape[2]
    n_h1 = int(counts[0, 1].gt(0).sum())
    assert n_h1 + 128 <= M          # head 1 has at least one all-padding block
    n1, ds, hi = O.hybrid_schedule(ts[0, 1].numpy(), M, 600, 512, W)
    assert ds == 0 and n1 == 4
    # head 0 (no padding) resumes dense attention near the diagonal
    n1, ds, hi = O.hybrid_schedule(ts[0, 0].numpy(), M, 600, 512, W)
    assert ds > 0


@pytest.mark.parametrize("name,dt,use_cos", [("decode_fp32_euclid", torch.float32, False),
                                             ("decode_fp16_cosine", torch.float16, True),
                                             ("decode_bf16_euclid", torch.bfloat16, False)])
def test_decode_replay_matches_reference(golden, name, dt, use_cos):
    g = golden(name)
    st = I.decode_setup(dt, seed=31)
    B, Hkv, Hq, D, W = st["B"], st["Hkv"], st["Hq"], st["D"], st["W"]
    thr = float(g["threshold"])
    kp, vp, cnt, tss, lens = st["kp"], st["vp"], st["counts"], st["ts"], st["lengths"]
    ke, ve = st["ke"], st["ve"]
    exact_len, total = st["exact_len"], st["total"]
    lens0 = lens.numpy().copy()
    outs = []
    for step in range(st["steps"]):
        O.decode_update(st["new_k"][step], st["new_v"][step], ke, ve, kp, vp, cnt, tss, lens,
                        exact_len, total, thr, W, use_cos)
        exact_len += 1
        total += 1
        np.testing.assert_array_equal(lens.numpy(), g["lengths"][step])
        o = O.decode_attention(st["q"][step], kp, vp, cnt, lens.view(B, Hkv), ke, ve,
                               D ** -0.5, min(exact_len, W), Hq // Hkv)
        outs.append(o.float())
    np.testing.assert_array_equal(cnt.numpy(), g["counts"])
    np.testing.assert_array_equal(tss.numpy(), g["timestamps"])
    np.testing.assert_array_equal(kp.float().numpy(), g["k_packed"])
    np.testing.assert_array_equal(ke.float().numpy(), g["k_exact"])
    out = torch.stack(outs)
    ref = torch.from_numpy(g["outputs"])
    mx, mean = TOL[dt]
    err = (out - ref).abs()
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())
    # the replay exercised both merges and appends
    grew = g["lengths"][-1] - lens0
    assert (grew > 0).any() and (grew < st["steps"]).any()


def test_tile_counts_match_reference_schedule():
    # tiles per head under the reference schedule (deltaFlashAttention.py:63-111 semantics),
    # periodic packing, W=128
    assert O.tile_count(2048, 4) == 84
    assert O.tile_count(8192, 1) == 2080
    assert O.tile_count(8192, 4) == 744
    assert O.tile_count(32768, 4) == 9144
    assert O.tile_count(32768, 1) == 32896

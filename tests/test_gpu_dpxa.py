"""GPU parity of DPXA (delta-based tile scoring, Paper/src/methodology.tex:89-135) against the
oracle's restatement of the library's specification (oracle.dpxa_*).

- anchors per 128-token block: bit-exact (the delta selection with chunk 128);
- tile statistics (from the compacted anchors): the kernel's fp32 (max, sum exp(S - max)) against the oracle's fp64 give
  tile weights within 1e-4;
- selection: equal to the oracle's top-p on the same weights, except where a tile's preceding
  cumulative weight lies within 1e-4 of p (a rounding-order tie), which is reported;
- block-sparse attention: within 2e-2 / 2e-3 (bf16) of the oracle on the kernel's own
  selection, and equal to dense causal attention when every tile is selected.
"""
import numpy as np
import pytest
import torch

import _inputs as I
from oracle import delta_oracle as O

pytestmark = pytest.mark.gpu

TOL_W = 1e-4
P_MARGIN = 1e-4


@pytest.fixture(scope="module", autouse=True)
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import deltaattention_b200 as d
    d._lib.load()
    return d


def _layer(B, Hq, Hkv, N, D, seed):
    # AR(1) keys; queries correlated with the keys at their own position, so attention is local
    # enough that top-p drops tiles
    k = torch.from_numpy(I.ar1_keys(B, Hkv, N, D, seed + 1))
    noise = torch.from_numpy(I.ar1_keys(B, Hq, N, D, seed))
    q = (0.5 * k.repeat_interleave(Hq // Hkv, 1) + 0.2 * noise).to(torch.bfloat16)
    k = k.to(torch.bfloat16)
    v = torch.from_numpy(I.normal((B, Hkv, N, D), seed + 2, 0.5)).to(torch.bfloat16)
    cos, sin = O.rope_cos_sin(N, D, 5e5, torch.bfloat16)
    return O.apply_rope(q, cos, sin).contiguous(), O.apply_rope(k, cos, sin).contiguous(), v


def _taus(q, k):
    # raw thresholds keeping about half of each block's rows (squared inside, as the reference)
    tq = float(np.quantile(((q[:, :, 1:].float() - q[:, :, :-1].float()) ** 2).sum(-1).numpy(), 0.9)) ** 0.5
    tk = float(np.quantile(((k[:, :, 1:].float() - k[:, :, :-1].float()) ** 2).sum(-1).numpy(), 0.9)) ** 0.5
    return tq, tk


def _ws_clean():
    from deltaattention_b200 import _lib as L
    torch.cuda.synchronize()
    assert all(c == 0 for c in L.workspace_errors())


CASES = [(1, 8, 2, 1000, 128, 11), (2, 4, 4, 640, 64, 12), (1, 6, 2, 777, 128, 13)]


@pytest.mark.parametrize("B,Hq,Hkv,N,D,seed", CASES)
def test_dpxa_selection_matches_oracle(B, Hq, Hkv, N, D, seed):
    from deltaattention_b200 import ops
    q, k, v = _layer(B, Hq, Hkv, N, D, seed)
    tq, tk = _taus(q, k)
    p = 0.8
    sel, (keep_q, keep_k, tmax, tsum) = ops.dpxa_select(q.cuda(), k.cuda(), tq, tk, p, return_stats=True)
    G = Hq // Hkv
    # anchors, bit-exact
    oq, ok_ = O.dpxa_keep(q, tq ** 2), O.dpxa_keep(k, tk ** 2)
    np.testing.assert_array_equal(keep_q.cpu().numpy(), oq.numpy())
    np.testing.assert_array_equal(keep_k.cpu().numpy(), ok_.numpy())
    assert 0.1 < oq.float().mean() < 0.9 and 0.1 < ok_.float().mean() < 0.9
    # tile weights
    rm, rs = O.dpxa_tile_stats(q, k, oq, ok_, D ** -0.5, G)
    w_ref = O.dpxa_weights(rm, rs, G)
    w_gpu = O.dpxa_weights(tmax.double().cpu(), tsum.double().cpu(), G)
    assert (w_gpu - w_ref).abs().max() <= TOL_W
    # selection: the oracle's top-p on the kernel's weights, flips only at cumulative-weight ties
    nb = -(-N // 128)
    got = ops.selection_to_mask(sel, nb).cpu()
    want = O.dpxa_select(w_ref, p)
    bad = 0
    for b in range(B):
        for h in range(Hkv):
            for i in range(nb):
                if torch.equal(got[b, h, i], want[b, h, i]):
                    continue
                wi = w_ref[b, h, i, : i + 1]
                order = sorted(range(i + 1), key=lambda j: (-float(wi[j]), j))
                cum = np.concatenate([[0.0], np.cumsum([float(wi[j]) for j in order])])
                flipped = [order.index(j) for j in range(i + 1) if got[b, h, i, j] != want[b, h, i, j]]
                if not all(abs(cum[r] - p) < P_MARGIN for r in flipped):
                    bad += 1
    assert bad == 0
    assert torch.equal(got, torch.tril(got))                       # causal
    assert bool(got.diagonal(dim1=2, dim2=3).all())                # the diagonal always
    frac = got.float().sum() / torch.tril(torch.ones(nb, nb)).sum() / (B * Hkv)
    assert 0.05 < frac < 1.0, frac
    _ws_clean()


@pytest.mark.parametrize("B,Hq,Hkv,N,D,seed", CASES)
def test_block_sparse_attention_matches_oracle(B, Hq, Hkv, N, D, seed):
    from deltaattention_b200 import ops
    q, k, v = _layer(B, Hq, Hkv, N, D, seed)
    tq, tk = _taus(q, k)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    sel = ops.dpxa_select(qc, kc, tq, tk, 0.8)
    out = ops.block_sparse_attention(qc, kc, vc, sel)
    nb = -(-N // 128)
    mask = ops.selection_to_mask(sel, nb).cpu()
    ref = O.block_sparse_attention(q, k, v, mask, D ** -0.5, Hq // Hkv)
    err = (out.float().cpu() - ref.float()).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
    _ws_clean()


def test_block_sparse_attention_all_tiles_equals_dense():
    """Every tile selected: the block-sparse kernel is dense causal attention."""
    from deltaattention_b200 import ops
    B, Hq, Hkv, N, D = 1, 8, 2, 1280, 128
    q, k, v = _layer(B, Hq, Hkv, N, D, 21)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    tq, tk = _taus(q, k)
    sel = ops.dpxa_select(qc, kc, tq, tk, 2.0)   # p above the total weight: every tile
    nb = N // 128
    assert bool(ops.selection_to_mask(sel, nb).cpu().equal(torch.tril(torch.ones(B, Hkv, nb, nb, dtype=torch.bool))))
    out = ops.block_sparse_attention(qc, kc, vc, sel)
    dense = ops.flash(qc, kc, vc)
    err = (out.float() - dense.float()).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3
    _ws_clean()


def test_dpxa_prefill_runs_whole_layer():
    """RoPE -> selection -> block-sparse attention through ops.dpxa_prefill, against the
    oracle's five steps on the same inputs (its own selection)."""
    from deltaattention_b200 import ops
    B, Hq, Hkv, N, D = 1, 4, 2, 896, 128
    kf = torch.from_numpy(I.ar1_keys(B, Hkv, N, D, 32))
    qr = (0.5 * kf.repeat_interleave(Hq // Hkv, 1) + 0.2 * torch.from_numpy(I.ar1_keys(B, Hq, N, D, 31))).to(torch.bfloat16)
    kr = kf.to(torch.bfloat16)
    v = torch.from_numpy(I.normal((B, Hkv, N, D), 33, 0.5)).to(torch.bfloat16)
    cos, sin = O.rope_cos_sin(N, D, 5e5, torch.bfloat16)
    q_rot, k_rot = O.apply_rope(qr, cos, sin), O.apply_rope(kr, cos, sin)
    tq, tk = _taus(q_rot, k_rot)
    out = ops.dpxa_prefill(qr.cuda(), kr.cuda(), v.cuda(), cos.cuda(), sin.cuda(), tau_q=tq, tau_k=tk, top_p=0.9)
    kq, kk = O.dpxa_keep(q_rot, tq ** 2), O.dpxa_keep(k_rot, tk ** 2)
    w = O.dpxa_weights(*O.dpxa_tile_stats(q_rot, k_rot, kq, kk, D ** -0.5, Hq // Hkv), Hq // Hkv)
    ref = O.block_sparse_attention(q_rot, k_rot, v, O.dpxa_select(w, 0.9), D ** -0.5, Hq // Hkv)
    err = (out.float().cpu() - ref.float()).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
    _ws_clean()

"""CPU checks of the DPXA restatement (oracle.dpxa_*; Paper/src/methodology.tex:89-135).

The paper ships no code, so these pin the specification's own invariants: per-block anchors
equal the chunked delta selection with chunk 128, tile weights of a query block sum to one,
the top-p selection is causal and always holds the diagonal, p above the total weight selects
every tile, and block-sparse attention over every tile is dense causal attention.
"""
import torch

import _inputs as I
from oracle import delta_oracle as O


def _layer(B, Hq, Hkv, N, D, seed):
    k = torch.from_numpy(I.ar1_keys(B, Hkv, N, D, seed + 1))
    q = (0.5 * k.repeat_interleave(Hq // Hkv, 1) + 0.2 * torch.from_numpy(I.ar1_keys(B, Hq, N, D, seed))).bfloat16()
    v = torch.from_numpy(I.normal((B, Hkv, N, D), seed + 2, 0.5)).bfloat16()
    return q, k.bfloat16(), v


def test_dpxa_keep_is_chunked_delta_selection_with_chunk_128():
    q, k, _ = _layer(1, 2, 1, 300, 64, 1)
    keep = O.dpxa_keep(k, 6.0)
    ref, _ = O.delta_keep_mask(k, 6.0, False, 128, 3)
    assert torch.equal(keep, ref)
    assert bool(keep[0, 0, ::128].eq(1).all())   # every block starts with an anchor


def test_dpxa_weights_selection_and_dense_limit():
    B, Hq, Hkv, N, D = 1, 4, 2, 520, 64
    q, k, v = _layer(B, Hq, Hkv, N, D, 5)
    kq, kk = O.dpxa_keep(q, 20.0), O.dpxa_keep(k, 20.0)
    tm, ts = O.dpxa_tile_stats(q, k, kq, kk, D ** -0.5, Hq // Hkv)
    w = O.dpxa_weights(tm, ts, Hq // Hkv)
    nb = 5
    assert torch.allclose(w.sum(-1), torch.ones(B, Hkv, nb, dtype=w.dtype))
    assert torch.equal(w, torch.tril(w))
    sel = O.dpxa_select(w, 0.5)
    assert torch.equal(sel, torch.tril(sel)) and bool(sel.diagonal(dim1=2, dim2=3).all())
    full = O.dpxa_select(w, 2.0)
    assert torch.equal(full, torch.tril(torch.ones_like(full)))
    out = O.block_sparse_attention(q, k, v, full, D ** -0.5, Hq // Hkv)
    ref = O.flash_attention(q, k, v, True, D ** -0.5, n_rep=Hq // Hkv)
    err = (out.float() - ref.float()).abs()
    assert err.max() <= 2e-2 and err.mean() <= 2e-3

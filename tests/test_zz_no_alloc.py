"""dab_hybrid_flash_noalloc (static device scratch, no caller workspace) against
dab_hybrid_flash with a workspace. Collected last (file name) so it also runs after every
other test has used the library in the same process."""
import ctypes
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from deltaattention_b200 import _lib as L  # noqa: E402

VARIANTS = {"hybrid": 0, "sanity": 1, "pure_phase1": 2}


def _noalloc(variant, q, k, v, packed, out):
    """The argument list ops.attention passes to dab_hybrid_flash, minus the workspace."""
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    kp, vp, ts, cnt = packed.k, packed.v, packed.timestamps, packed.weights()
    strides = [*q.stride(), *k.stride(), *v.stride(), *kp.stride(), *vp.stride(), *ts.stride(), *cnt.stride(),
               *out.stride()]
    lib = L.load()
    L.check(lib.dab_hybrid_flash_noalloc(
        VARIANTS[variant], L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(kp), L.ptr(vp), L.ptr(ts), L.ptr(cnt), 0, L.ptr(out),
        L.dtype_code(q), L.strides(strides), float(D ** -0.5), N, k.shape[2], kp.shape[2], D, Hq, 128,
        -(-N // 128), B * Hq, 128, 128, D, Hq // Hkv, 0, L.stream_of(q)), "hybrid_flash_noalloc")
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["hybrid", "sanity", "pure_phase1"])
def test_noalloc_matches_workspace_entry_point(variant):
    from deltaattention_b200 import ops, synth
    dev = torch.device("cuda:0")
    B, Hq, Hkv, N, D = 1, 8, 2, 1000, 128
    q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.bfloat16, seed=31, device=dev)
    cos, sin = synth.rope_tables(N, D, 5e5, torch.bfloat16, device=dev)
    qr, kr = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
    packed = ops.pack_periodic(kr, v, 4)
    ref = ops.attention(qr, kr, v, packed, variant=variant)
    for _ in range(2):  # two calls in a row reuse the same static scratch
        out = torch.full_like(ref, float("nan"))
        _noalloc(variant, qr, kr, v, packed, out)
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3, (variant, err.max().item())
        # the static scratch's own error word: no bounded in-kernel wait of this call timed out
        code = ctypes.c_int(-1)
        L.check(L.load().dab_noalloc_error(ctypes.byref(code), L.stream_of(q)), "noalloc_error")
        assert code.value == 0, hex(code.value)
    assert all(c == 0 for c in L.workspace_errors())


def test_noalloc_rejects_oversized_calls():
    """Sizes beyond the static scratch fail before any CUDA call, with both sizes named."""
    lib = L.load()
    B, Hq, N, M, D = 64, 64, 131072, 32768, 128
    need = lib.dab_hybrid_flash_workspace_size(B, Hq, N, M)
    assert need > (1 << 20)
    strides = L.strides([0] * 30)
    rc = lib.dab_hybrid_flash_noalloc(0, 16, 16, 16, 16, 16, 16, 16, 0, 16, 2, strides, 0.088, N, N, M, D, Hq, 128,
                                      N // 128, B * Hq, 128, 128, D, 1, 0, None)
    assert rc == 1
    msg = lib.dab_last_error().decode()
    assert str(need) in msg and str(1 << 20) in msg

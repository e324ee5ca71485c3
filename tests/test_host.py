"""CPU tests of the host side: the C-ABI library, the drop-in shims' argument handling and
the multi-process plumbing of bench.py (gloo, world size 2). No GPU is touched."""
import ctypes
import os
import re
import socket
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from deltaattention_b200 import _lib as L  # noqa: E402

HEADER = os.path.join(ROOT, "include", "deltaattn_b200.h")


def _header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return sorted(set(re.findall(r"\b(dab_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib_path():
    if not os.path.exists(L.LIB_PATH):
        from deltaattention_b200 import build
        build.build()
    return L.LIB_PATH


def test_library_exports_every_header_symbol(lib_path):
    syms = _header_symbols()
    assert len(syms) >= 15, syms
    so = ctypes.CDLL(lib_path)
    missing = [s for s in syms if not hasattr(so, s)]
    assert not missing, missing
    # the ctypes table binds exactly the declared ABI
    assert sorted(L.SIGNATURES) == syms


def test_host_only_entry_points(lib_path):
    lib = L.load()
    assert lib.dab_abi_version() >= 1
    r256 = lambda n: (n + 255) // 256 * 256  # noqa: E731
    for (B, H, N, M) in [(1, 8, 32768, 8192), (2, 3, 1000, 250), (1, 1, 1, 0)]:
        nmb, nblk = -(-N // 128), max(1, -(-M // 128))
        want = 256 + r256(B * H * nmb * 8) + 2 * r256(B * H * nblk * 4)
        assert lib.dab_hybrid_flash_workspace_size(B, H, N, M) == want
    assert lib.dab_pack_from_keep_workspace_size(2, 3, 5000) == 64 + 8 * 2 * 3 * 5  # header + a word per tile


def test_device_length_entries_reject_null_state(lib_path):
    """The device-length decode entries check their state pointer before touching the GPU."""
    lib = L.load()
    z = (ctypes.c_int64 * 4)(0, 0, 0, 0)
    assert lib.dab_decode_advance(None, 1, None) != 0
    assert b"seq_state" in lib.dab_last_error()
    assert lib.dab_decode_advance(None, 0, None) == 0  # nothing to advance
    rc = lib.dab_decode_update_dev(*([None] * 9), None, 0.0, 16, 2, z, z, z, z, 2, 128, 128, 0, 2, 64, None, None)
    assert rc != 0 and b"seq_state" in lib.dab_last_error()
    rc = lib.dab_decode_attention_dev(*([None] * 8), 2, z, 1.0, None, 1, 16, 4, 1, 8, 128, 64, None, 0, None)
    assert rc != 0 and b"seq_state" in lib.dab_last_error()


@pytest.mark.parametrize("n,m,r,N", [(2, 4, 4, 2000), (2, 4, 2, 777), (1, 4, 4, 1024), (3, 8, 8, 1500)])
def test_nm_packed_length_matches_oracle(lib_path, n, m, r, N):
    """dab_nm_num_packed (host arithmetic) equals the oracle's kept count per head."""
    from oracle import delta_oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import _inputs as I
    from deltaattention_b200.dropin import nmDeltaFlashAttention as nm
    k = I.post_rope_keys(1, 2, N, 64, 5e5, torch.float32, seed=N)
    keep = O.nm_keep_mask(k, n, m, r)
    counts = keep.sum(-1).flatten().tolist()
    assert len(set(counts)) == 1
    assert nm.nm_num_packed(N, n, m, r) == counts[0]


def test_product_path_refuses_cpu_tensors(lib_path):
    """No CPU fallback: the ops raise instead of computing on host tensors."""
    from deltaattention_b200 import ops
    x = torch.zeros(1, 2, 256, 128, dtype=torch.bfloat16)
    cos = torch.ones(1, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rope(x, cos, cos)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.flash(x, x, x)


def test_host_prefill_refuses_unpinned_or_device_buffers(lib_path):
    """delta_prefill_host takes pinned host q / k / v / out only (no silent synchronous copies)."""
    from deltaattention_b200 import ops
    x = torch.zeros(1, 2, 128, 64, dtype=torch.bfloat16)
    cos = torch.ones(128, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="pinned"):
        ops.delta_prefill_host(x, x, x, cos, cos, out=x)


def test_kernel_shim_binds_reference_argument_lists():
    """The drop-in kernel objects accept the reference launch's positional / keyword split and
    reject a call with a missing argument the way a Triton launch does (TypeError)."""
    from deltaattention_b200 import launch
    names = launch.HYBRID_PARAMS
    args = tuple(range(len(names) - 3))  # everything but BLOCK_M, BLOCK_N, BLOCK_D
    b = launch._bind(names, args, dict(BLOCK_M=128, BLOCK_N=128, BLOCK_D=64), "hybrid")
    assert b["BLOCK_D"] == 64 and b[names[0]] == 0 and b[names[len(args) - 1]] == len(args) - 1
    with pytest.raises(TypeError):
        launch._bind(names, args[:-1], dict(BLOCK_M=128, BLOCK_N=128, BLOCK_D=64), "hybrid")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        bench.barrier(world)
        # the bench's timing rule: every rank reports its own time, the job takes the maximum
        got = bench.max_over_ranks(1.5 + rank, world)
        out[rank] = got
    finally:
        dist.destroy_process_group()


def test_bench_max_over_ranks_gloo_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(out) == {0: 2.5, 1: 2.5}


def _shard_rank_main(rank, world, port, out):
    """One gloo rank of the kv-head partition: it runs the oracle layer-op on its kv-heads only
    and gathers every rank's output heads."""
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from deltaattention_b200 import shard, synth
        from oracle import delta_oracle as O
        B, Hq, Hkv, N, D = 1, 8, 4, 384, 64
        q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.float32, seed=3, device="cpu")
        cos, sin = synth.rope_tables(N, D, 1e4, torch.float32)
        ql, kl, vl = shard.shard_layer(q, k, v, world, rank)
        qr, kr = O.apply_rope(ql.contiguous(), cos, sin), O.apply_rope(kl.contiguous(), cos, sin)
        keep = O.periodic_keep_mask(B, kl.shape[1], N, 0.25)
        _, kp, vp, ts, cnt = O.pack_from_keep(kr, vl.contiguous(), keep)
        o = O.hybrid_attention(qr, kr, vl.contiguous(), kp, vp, ts, cnt.float(), D ** -0.5, 128, n_rep=Hq // Hkv)
        full = shard.gather_heads(o, world)
        out[rank] = (shard.kv_head_range(Hkv, world, rank), full.numpy())
    finally:
        dist.destroy_process_group()


def test_kv_head_shard_gloo_world2_equals_single_rank():
    """The bench's multi-GPU partition on two gloo ranks: each rank takes half the kv-heads
    (with their query heads) of one sequence, and the gathered output equals the one-rank
    computation of the whole layer exactly (the heads are independent)."""
    import numpy as np
    import torch.multiprocessing as mp
    from deltaattention_b200 import shard, synth
    from oracle import delta_oracle as O
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_shard_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert out[0][0] == (0, 2) and out[1][0] == (2, 4)
    B, Hq, Hkv, N, D = 1, 8, 4, 384, 64
    q, k, v = synth.layer_inputs(B, Hq, Hkv, N, D, torch.float32, seed=3, device="cpu")
    cos, sin = synth.rope_tables(N, D, 1e4, torch.float32)
    qr, kr = O.apply_rope(q.contiguous(), cos, sin), O.apply_rope(k.contiguous(), cos, sin)
    keep = O.periodic_keep_mask(B, Hkv, N, 0.25)
    _, kp, vp, ts, cnt = O.pack_from_keep(kr, v.contiguous(), keep)
    want = O.hybrid_attention(qr, kr, v.contiguous(), kp, vp, ts, cnt.float(), D ** -0.5, 128, n_rep=Hq // Hkv)
    for r in range(2):
        np.testing.assert_array_equal(out[r][1], want.numpy())


def test_kv_head_range_rejects_uneven_split():
    from deltaattention_b200 import shard
    assert [shard.kv_head_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError, match="divide"):
        shard.kv_head_range(8, 3, 0)
    with pytest.raises(ValueError, match="outside"):
        shard.kv_head_range(8, 2, 2)


@pytest.mark.parametrize("cu,msg", [([0, 100, 100, 300], "rise strictly"), ([0, 150, 299], "rise strictly"),
                                    ([5, 300], "rise strictly"), ([0, 300], "shorter than the longest")])
def test_varlen_prefill_rejects_bad_offsets(cu, msg):
    """delta_prefill_varlen checks cu_seqlens (strictly rising from 0 to the packed length) and
    the RoPE table length on the host, before any device work."""
    from deltaattention_b200 import ops
    q = torch.zeros((1, 4, 300, 64), dtype=torch.bfloat16)
    k = torch.zeros((1, 2, 300, 64), dtype=torch.bfloat16)
    cos = torch.zeros((1, 256, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match=msg):
        ops.delta_prefill_varlen(q, k, k, cos, cos, cu)


def test_varlen_prefill_rejects_unknown_selection():
    from deltaattention_b200 import ops
    q = torch.zeros((1, 4, 300, 64), dtype=torch.bfloat16)
    cos = torch.zeros((1, 512, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="unknown selection"):
        ops.delta_prefill_varlen(q, q, q, cos, cos, [0, 300], selection="delta")

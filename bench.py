"""Benchmark: delta-attention prefill tokens/s for BASELINE config 2 (one GPU per rank).

A step is one pass of the hot path over one layer of synthetic input: RoPE on q and k,
periodic r=4 packing (timestamps / counts; packed K/V are strided views) and the two-phase
count-weighted tcgen05 attention for B=1, Hq=32, Hkv=8, N=32768, d=128, bf16.

On N GPUs (torchrun, one rank per GPU) the one sequence is partitioned by kv-head, as the
(batch, kv-head) units of the path are independent: each rank runs Hkv/N kv-heads with their
query heads over the whole sequence, with no collective on the data path (strong scaling:
the job's work is fixed). ``--shard seq`` instead gives every rank a sequence of its own
(weak scaling). Per-GPU inputs larger than the 126 MB L2 need no flush between steps;
smaller ones (4 and 8 GPUs) get an L2 flush between steps (256 MiB written, then 256 MiB read,
so no dirty flush lines are left for the step to write back), outside the timed events.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--shard heads|seq]

Prints ONE JSON line (rank 0). ``--impl reference`` times the CPU restatement of the
reference's path (the oracle port) on this host's cores on a bounded sample of the same
workload (the reference's own code is Triton and cannot run on a host without the
interpreter and its source tree).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "delta-attn prefill tokens/s @N=32k, r=4 (one Llama-3.1-8B attention layer-op)"
UNIT = "tokens/s"
CFG = dict(B=1, Hq=32, Hkv=8, N=32768, D=128, r=4, W=128, theta=5e5)


def workload_config(n_gpus, shard="heads", flushed=False):
    if shard == "heads":
        par = (f"kv-head shard: {CFG['Hkv'] // n_gpus} kv-heads ({CFG['Hq'] // n_gpus} q-heads) of one sequence "
               f"per GPU, no data-path collective")
        gb = CFG["B"]
    else:
        par = f"dp{n_gpus} (one sequence per GPU, no data-path collective)"
        gb = CFG["B"] * n_gpus
    return {"workload": "cfg2: RoPE(q,k) + periodic r=4 packing + two-phase delta attention, one layer",
            "B": CFG["B"], "Hq": CFG["Hq"], "Hkv": CFG["Hkv"], "N": CFG["N"], "d": CFG["D"],
            "r": CFG["r"], "dense_window": CFG["W"], "global_batch": gb, "parallelism": par,
            "l2": ("per-GPU inputs smaller than 1.5x L2: L2 flushed between timed steps, 256 MiB written then "
                   "256 MiB read (outside the per-step events)") if flushed else "per-GPU inputs larger than L2; no flush"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except Exception:
        return 1590.0, 1400.0, "fallback"


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class L2Flush:
    """Evicts L2 between timed launches: writes a 256 MiB buffer (twice the 126 MB L2), then
    reads another 256 MiB buffer, so L2 ends up holding clean lines of the read buffer. After a
    write alone L2 would be full of the flush's dirty lines, and the timed kernel would pay for
    writing them back to HBM as its own reads evict them (~126 MB of extra traffic)."""

    def __init__(self, dev):
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
        self.out = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.fill_(1)
        torch.sum(self.r, dim=0, out=self.out)


def hbm_kernels(dev, seed):
    """HBM-bound kernels of the path, each launch timed alone with L2 flushed before it.

    Returns {name: {"us": t, "bytes": algorithmic bytes, "gbs": bytes / t, "frac": gbs / peak}}:
    delta selection (chunked_eval, cfg2 keys), device packing from a keep mask (cfg2 K/V), the
    reference-facing scatter pack of the same mask, 2:4 N:M selection (cfg2 keys),
    decode attention (16 sequences, packed lengths U[1024, 8192], window 100, 32 q-heads) and
    the decode cache update (one token per sequence)."""
    from deltaattention_b200 import ops, synth
    from deltaattention_b200.launch import fused_hybrid_decode_kernel, fused_hybrid_decode_update_kernel
    peak, _ = hbm_peak()
    flush = L2Flush(dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, reps=10):
        ts = []
        for _ in range(reps + 2):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts[2:])

    out = {}
    Hkv, N, D = CFG["Hkv"], CFG["N"], CFG["D"]
    _, k, v = synth.layer_inputs(1, Hkv, Hkv, N, D, torch.bfloat16, seed=seed, device=dev)
    cos, sin = synth.rope_tables(N, D, CFG["theta"], torch.bfloat16, device=dev)
    k_rot = ops.rope(k, cos, sin)
    thr = 11.0  # raw Euclidean threshold (squared inside, as the reference): keeps about 1 key in 4 here
    us = timed(lambda: ops.delta_keep_mask(k_rot, thr, "euclidean", 512))
    nbytes = k_rot.numel() * 2 + Hkv * N * 4
    out["delta_select"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak}
    keep, _ = ops.delta_keep_mask(k_rot, thr, "euclidean", 512)
    M = int(keep.sum(-1).max().item())
    kept = int(keep.sum().item())
    us = timed(lambda: ops.pack_from_keep(k_rot, v, keep, num_packed=M))
    nbytes = Hkv * N * 4 + kept * D * 2 * 2 * 2 + Hkv * M * 8
    out["pack_from_keep"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak,
                             "kept_fraction": kept / (Hkv * N)}
    # the reference-facing scatter pack (tritonModules.parallel_scatter_pack_kv_kernel) with the
    # index map the reference builds (cumsum - 1): keep / index map read, kept K / V rows moved,
    # timestamps written
    from deltaattention_b200.launch import parallel_scatter_pack_kv_kernel
    im = (torch.cumsum(keep, -1) - 1).to(torch.int32)
    kp_s = torch.zeros((1, Hkv, M, D), dtype=torch.bfloat16, device=dev)
    vp_s = torch.zeros_like(kp_s)
    ts_s = torch.zeros((1, Hkv, M), dtype=torch.int32, device=dev)
    us = timed(lambda: parallel_scatter_pack_kv_kernel[(Hkv, -(-N // 64))](
        k_rot, v, kp_s, vp_s, ts_s, keep, im, *k_rot.stride(), *v.stride(), *kp_s.stride(), *vp_s.stride(),
        *ts_s.stride(), *keep.stride(), *im.stride(), N, D, Hkv, BLOCK_S=64, BLOCK_D=D))
    nbytes = Hkv * N * 8 + kept * D * 2 * 2 * 2 + kept * 4
    out["scatter_pack"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak}
    del im, kp_s, vp_s, ts_s
    # the fused key compression of delta mode (RoPE(k) + delta scan + packing, one launch, packed
    # length left on the device): raw K read, rotated K written, the kept V rows read, packed K / V
    # and timestamps / counts (int32 + fp32) written, keep mask written, cos / sin read once
    _, k_raw, _ = synth.layer_inputs(1, Hkv, Hkv, N, D, torch.bfloat16, seed=seed, device=dev)
    us = timed(lambda: ops.delta_compress(k_raw, v, cos, sin, thr, "euclidean", 512))
    _, pkc = ops.delta_compress(k_raw, v, cos, sin, thr, "euclidean", 512)
    A = int(pkc.anchors.sum().item())
    nbytes = 2 * k_raw.numel() * 2 + A * D * 2 * 3 + A * 12 + Hkv * N * 4 + 2 * N * D * 2
    out["delta_compress"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak,
                             "kept_fraction": A / (Hkv * N),
                             "replaces": "rope(k) + delta_select + pack_from_keep + the packed-length read-back"}
    del k_raw, pkc
    # 2:4 N:M selection at r = 4: candidates every 2nd key, so half of K is read; keep mask written
    from deltaattention_b200.dropin.nmDeltaFlashAttention import nm_keep_mask
    us = timed(lambda: nm_keep_mask(k_rot, 2, 4, 4))
    nbytes = Hkv * (N // 2) * D * 2 + Hkv * N * 4
    out["nm_select"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak}
    del k, v, k_rot, keep
    # decode: cfg5-like cache state
    g = torch.Generator(device=dev).manual_seed(seed)
    Bd, Hq, W, cap = 16, CFG["Hq"], 100, N // CFG["r"]
    rnd = lambda *shape: torch.randn(shape, generator=g, device=dev).to(torch.bfloat16)  # noqa: E731
    lens = torch.randint(1024, cap + 1, (Bd, Hkv), generator=g, device=dev, dtype=torch.int32)
    kp, vp = rnd(Bd, Hkv, cap, D), rnd(Bd, Hkv, cap, D)
    cnt = torch.full((Bd, Hkv, cap), CFG["r"], dtype=torch.int32, device=dev)
    ke, ve = rnd(Bd, Hkv, W, D), rnd(Bd, Hkv, W, D)
    q = rnd(Bd, Hq, D)
    o = torch.empty_like(q)

    def dec():
        fused_hybrid_decode_kernel[(Bd, Hq)](
            q, kp, vp, cnt, lens, ke, ve, o, *q.stride(), *kp.stride(), *vp.stride(), *cnt.stride(), *lens.stride(),
            *ke.stride(), *ve.stride(), *o.stride(), D ** -0.5, W, Hq // Hkv, head_dim=D, BLOCK_M=16, BLOCK_N=128,
            BLOCK_D=D)
    us = timed(dec)
    nbytes = int(lens.sum().item()) * (D * 2 * 2 + 4) + Bd * Hkv * W * D * 2 * 2 + 2 * q.numel() * 2
    out["decode_attention"] = {"us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak,
                               "shape": f"B={Bd} Hq={Hq} Hkv={Hkv} d={D} packed U[1024,{cap}] window {W}"}
    nk, nv = rnd(Bd, Hkv, 1, D), rnd(Bd, Hkv, 1, D)
    lens_flat = lens.view(-1).clone()
    # every update may append one anchor and the kernel (like the reference's) has no capacity
    # argument: leave room for all timed calls
    spare = 32
    kp2 = torch.zeros((Bd, Hkv, cap + spare, D), dtype=torch.bfloat16, device=dev)
    vp2 = torch.zeros_like(kp2)
    cnt2 = torch.zeros((Bd, Hkv, cap + spare), dtype=torch.int32, device=dev)
    tss2 = torch.zeros_like(cnt2)
    kp2[:, :, :cap] = kp
    vp2[:, :, :cap] = vp
    cnt2[:, :, :cap] = cnt

    def upd():
        fused_hybrid_decode_update_kernel[(Bd * Hkv,)](
            nk, nv, ke, ve, kp2, vp2, cnt2, tss2, lens_flat, W, 100000, 16.0, W,
            *nk.stride(), *ke.stride(), *kp2.stride(), *cnt2.stride(), Hkv, D, BLOCK_D=D, USE_COSINE=False)
    us = timed(upd, reps=10)  # 12 calls in all: at most 12 appends per (sequence, kv-head)
    out["decode_update"] = {"us": us, "note": "one token per (sequence, kv-head); latency-bound"}
    return out


def decode_step(dev, seed, layers=32, steps=20):
    """One decode token over every layer of a Llama-3.1-8B-shaped model with the device-length
    cache (cache.DeviceDecodeCache): 16 sequences, Hq=32 / Hkv=8, d=128, packed lengths
    uniform in [1024, 8192] per (sequence, kv-head), exact window 100. Timed as eager
    launches (update, then attention + combine with the length advance, per layer) and as
    one replayed CUDA graph. HBM bytes per step: packed K / V rows, counts and the window read
    once per layer (516 B per key), as in hbm_kernels."""
    from deltaattention_b200.cache import DeviceDecodeCache
    from deltaattention_b200 import _lib as L
    B, Hq, Hkv, D, W, cap = 16, 32, 8, 128, 100, 8192 + 64
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    c = DeviceDecodeCache(layers, B, Hkv, D, cap, W, torch.bfloat16, device=dev, threshold=8.0)
    c.k_packed.normal_(generator=g)
    c.v_packed.normal_(generator=g)
    c.packed_counts.fill_(4)
    c.k_exact.normal_(generator=g)
    c.v_exact.normal_(generator=g)
    lens = torch.randint(1024, 8193, (B * Hkv,), generator=g, device=dev, dtype=torch.int32)
    c.packed_lengths.copy_(lens.expand(layers, -1))
    c.seq_state[:, 0] = W
    c.seq_state[:, 1] = 65536
    q = torch.randn((layers, B, Hq, D), generator=g, device=dev).bfloat16()
    kn = torch.randn((layers, B, Hkv, 1, D), generator=g, device=dev).bfloat16()
    vn = torch.randn((layers, B, Hkv, 1, D), generator=g, device=dev).bfloat16()
    out = torch.empty_like(q)

    def eager():
        for layer in range(layers):
            c.step(layer, q[layer], kn[layer], vn[layer], out[layer])

    for _ in range(3):
        eager()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        eager()
    e1.record()
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1) / steps
    graph = c.capture_step(q, kn, vn, out)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    graph_ms = e0.elapsed_time(e1) / steps
    keys = int(c.packed_lengths.sum().item()) + layers * B * Hkv * W
    nbytes = keys * 516
    err = int(c.err.item())
    del graph
    codes = L.workspace_errors()
    peak, _ = hbm_peak()
    return {"layers": layers, "shape": f"B={B} Hq={Hq} Hkv={Hkv} d={D} packed U[1024,8192] window {W}",
            "eager_ms": eager_ms, "graph_ms": graph_ms, "tokens_per_s": B / (graph_ms / 1000.0),
            "hbm_gbs": nbytes / (graph_ms / 1000.0) / 1e9, "frac": nbytes / (graph_ms / 1000.0) / 1e9 / peak,
            "launches_per_step": layers * 3, "err": err, "ws_errors": codes}


def serving(dev, seed, steps=256):
    """cfg5: batched varlen serving with Llama-3.1-8B layer shapes (one attention layer).

    16 sequences with lengths U[4096, 32768] packed back to back (cu_seqlens) in one
    projection-layout buffer; q / v ~ N(0, 1), keys AR(1) (config-1 distributions), RoPE
    theta 5e5, bf16. Prefill (ops.delta_prefill_varlen, sequences over three streams), per
    sequence: RoPE(q, k), 2:4 N:M selection at r = 4, device packing, two-phase attention
    (dense window 128); then the hand-off of each packed history and its last 100 keys into
    a DeviceDecodeCache. Then `steps` decode steps for all 16 sequences
    (cache update with raw Euclidean threshold 15, length advance, decode attention), new
    keys continuing each sequence's AR(1) process; the steps are captured in one CUDA graph
    and replayed. HBM bytes per decode step: every packed K / V row with its count and the
    window read once (516 B per key)."""
    from deltaattention_b200 import ops, synth
    from deltaattention_b200.cache import DeviceDecodeCache
    from deltaattention_b200.dropin.nmDeltaFlashAttention import nm_num_packed
    B, Hq, Hkv, D, W, Wd, thr = 16, CFG["Hq"], CFG["Hkv"], CFG["D"], CFG["W"], 100, 15.0
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(4096, 32769, (B,), generator=gen).tolist()
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T = cu[-1]
    q, k, v = synth.layer_inputs(1, Hq, Hkv, T, D, torch.bfloat16, seed=seed, device=dev, qv_scale=1.0,
                                 key_offset=False)
    cos, sin = synth.rope_tables(max(lens), D, CFG["theta"], torch.bfloat16, device=dev)
    o = torch.empty((1, T, Hq, D), dtype=torch.bfloat16, device=dev).transpose(1, 2)
    cap = max(nm_num_packed(n) for n in lens) + steps + 64
    cache = DeviceDecodeCache(1, B, Hkv, D, cap, Wd, torch.bfloat16, device=dev, threshold=thr)
    stream = torch.cuda.current_stream(dev)

    def prefill():
        _, packed = ops.delta_prefill_varlen(q, k, v, cos, sin, cu, selection="nm", n=2, m=4, ratio=4,
                                             dense_window=W, out=o, return_packed=True)
        for i, (pk, kr) in enumerate(packed):
            s0, s1 = cu[i], cu[i + 1]
            cache.load_prefill(0, pk.k, pk.v, pk.counts, pk.timestamps, kr[:, :, -Wd:], v[:, :, s1 - Wd:s1], s1 - s0,
                               batch_index=i)

    prefill()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    prefill()
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    packed0 = int(cache.packed_lengths.sum().item())

    # decode inputs: q ~ N(0, 1); keys continue each sequence's AR(1) from its last key
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 1)
    qs = torch.randn((steps, B, Hq, D), generator=g, device=dev).to(torch.bfloat16)
    vs = torch.randn((steps, B, Hkv, 1, D), generator=g, device=dev).to(torch.bfloat16)
    last = torch.stack([k[0, :, cu[i + 1] - 1].float() for i in range(B)])  # [B, Hkv, D]
    ks = torch.empty((steps, B, Hkv, 1, D), dtype=torch.bfloat16, device=dev)
    for t in range(steps):
        last = 0.95 * last + 0.31 * torch.randn(last.shape, generator=g, device=dev)
        ks[t, :, :, 0] = last.to(torch.bfloat16)
    outs = torch.empty_like(qs)
    names = ("seq_state", "packed_lengths", "packed_counts", "k_exact", "v_exact")
    snap = {n: getattr(cache, n).clone() for n in names}

    def restore():
        for n in names:
            getattr(cache, n).copy_(snap[n])

    for t in range(3):  # eager warm-up (kernel attributes are set outside capture)
        cache.step(0, qs[t], ks[t], vs[t], outs[t])
    restore()
    cache._workspace(Hq)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for t in range(steps):
            cache.step(0, qs[t], ks[t], vs[t], outs[t])
    stream.wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    restore()
    torch.cuda.synchronize()
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    decode_ms = e0.elapsed_time(e1)
    err = int(cache.err.item())
    packed1 = int(cache.packed_lengths.sum().item())
    del graph
    keys = steps * (packed0 + packed1) // 2 + steps * B * Hkv * Wd  # mean packed length over the steps
    nbytes = keys * 516
    peak, _ = hbm_peak()
    return {"sequences": B, "lengths": "U[4096, 32768]", "prefill_tokens": T, "prefill_ms": prefill_ms,
            "prefill_tokens_per_s": T / (prefill_ms / 1000.0), "selection": "2:4 N:M, r=4 (nmDeltaFlashAttention)",
            "decode_steps": steps, "decode_ms_per_step": decode_ms / steps,
            "decode_tokens_per_s": B * steps / (decode_ms / 1000.0),
            "decode_hbm_gbs": nbytes / (decode_ms / 1000.0) / 1e9,
            "decode_frac": nbytes / (decode_ms / 1000.0) / 1e9 / peak,
            "anchors_appended": packed1 - packed0, "anchor_slots_updated": steps * B * Hkv, "err": err}


def sweep(dev, seed, reps=3):
    """cfg3: the same layer-op at N in {8k .. 128k} and r in {2, 4, 8}, each against the same
    kernel family run dense (r = 1). Attention only, CUDA events, median of `reps` launches
    (every input is larger than L2 from N = 16k on; one head group per point is enough for
    the per-head rate, so the sweep uses B=1, Hq=32, Hkv=8 as cfg2)."""
    from deltaattention_b200 import ops, synth
    burst, _, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    out = []
    for N in (8192, 16384, 32768, 65536, 131072):
        q, k, v = synth.layer_inputs(1, CFG["Hq"], CFG["Hkv"], N, CFG["D"], torch.bfloat16, seed=seed, device=dev)
        cos, sin = synth.rope_tables(N, CFG["D"], CFG["theta"], torch.bfloat16, device=dev)
        qr, kr = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
        del q, k

        def timed(fn):
            fn()
            ts = []
            for _ in range(reps):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                torch.cuda.synchronize()
                ts.append(e0.elapsed_time(e1))
            return statistics.median(ts)
        dense = timed(lambda: ops.flash(qr, kr, v))
        row = {"N": N, "dense_r1_ms": dense}
        for r in (2, 4, 8):
            pk = ops.pack_periodic(kr, v, r)
            ms = timed(lambda: ops.attention(qr, kr, v, pk, dense_window=CFG["W"]))
            flops = CFG["Hq"] * ops.tile_count_periodic(N, r, CFG["W"]) * 4 * 128 * 128 * CFG["D"]
            row[f"r{r}"] = {"ms": ms, "tflops": flops / ms / 1e9, "frac": flops / ms / 1e9 / burst,
                            "speedup_vs_dense": dense / ms, "tokens_per_s": N / (ms / 1e3)}
        out.append(row)
        del qr, kr, v
        torch.cuda.empty_cache()
    return out


def proj_rope_bench(dev, seed, reps=5):
    """The k_proj / fused QKV projection with RoPE as the GEMM epilogue (modeling_llama.py:
    550-555) at cfg2 sizes (32768 tokens, hidden 4096), against the unfused path it replaces:
    torch's bf16 GEMM (cuBLAS) followed by the library's RoPE kernel. Inputs are larger than
    L2; CUDA events, median of `reps` launches after a warm-up launch."""
    from deltaattention_b200 import ops, synth
    burst, _, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    rows, kin = CFG["N"], 4096
    x = torch.randn(rows, kin, device=dev, dtype=torch.bfloat16, generator=g)
    cos, sin = synth.rope_tables(rows, CFG["D"], CFG["theta"], torch.bfloat16, device=dev)
    cos, sin = cos.reshape(rows, CFG["D"]), sin.reshape(rows, CFG["D"])

    def timed(fn):
        fn()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)
    out = {}
    for name, nout, rope_hi in (("k_proj", 1024, 1024), ("qkv_proj", 6144, 5120)):
        w = torch.randn(nout, kin, device=dev, dtype=torch.bfloat16, generator=g) * kin ** -0.5
        fused = timed(lambda: ops.proj_rope(x, w, cos, sin, rope_cols=(0, rope_hi)))
        gemm = timed(lambda: x @ w.t())

        def unfused():
            y = x @ w.t()
            h = rope_hi // CFG["D"]
            yr = y[:, :rope_hi].view(1, rows, h, CFG["D"]).transpose(1, 2)
            ops.rope(yr, cos[None], sin[None], out=yr)
            return y
        unf = timed(unfused)
        flops = 2 * rows * kin * nout
        out[name] = {"out_features": nout, "rope_columns": rope_hi, "fused_ms": fused, "cublas_gemm_ms": gemm,
                     "cublas_gemm_plus_rope_ms": unf, "fused_tflops": flops / fused / 1e9,
                     "frac_of_burst": flops / fused / 1e9 / burst, "speedup_vs_unfused": unf / fused}
        del w
    return out


def dpxa_bench(dev, seed, reps=3):
    """DPXA (delta-based tile scoring, Paper/src/methodology.tex:89-135) at cfg2 sizes: the
    selection (anchor masks of Q and K per 128-token block, compaction, sampled tile scores,
    top-p with p = 0.9) and the block-sparse attention over the selected tiles, against the
    same kernel dense. Queries correlated with the keys at their own position (so attention
    is local, as in a real layer) over AR(1) keys; thresholds keep about half the rows."""
    from deltaattention_b200 import ops, synth
    burst, _, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    B, Hq, Hkv, N, D = 1, CFG["Hq"], CFG["Hkv"], CFG["N"], CFG["D"]
    g = torch.Generator(device=dev).manual_seed(seed)
    k = synth.ar1((B, Hkv, N, D), g, dev).to(torch.bfloat16)
    q = (0.5 * k.repeat_interleave(Hq // Hkv, 1).float()
         + 0.2 * synth.ar1((B, Hq, N, D), g, dev)).to(torch.bfloat16)
    v = (0.5 * torch.randn((B, Hkv, N, D), device=dev, generator=g)).to(torch.bfloat16)
    cos, sin = synth.rope_tables(N, D, CFG["theta"], torch.bfloat16, device=dev)
    qr, kr = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
    del q, k
    dq = (qr[:, :, 1:].float() - qr[:, :, :-1].float()).pow(2).sum(-1).flatten()
    dk = (kr[:, :, 1:].float() - kr[:, :, :-1].float()).pow(2).sum(-1).flatten()
    tq = float(torch.quantile(dq[:: max(1, dq.numel() // 1000000)], 0.9)) ** 0.5
    tk = float(torch.quantile(dk[:: max(1, dk.numel() // 1000000)], 0.9)) ** 0.5
    del dq, dk

    def timed(fn):
        fn()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)
    p = 0.9
    sel_ms = timed(lambda: ops.dpxa_select(qr, kr, tq, tk, p))
    sel, (kq, kk, _, _) = ops.dpxa_select(qr, kr, tq, tk, p, return_stats=True)
    nb = N // 128
    mask = ops.selection_to_mask(sel, nb)
    tiles = int(mask.sum()) * (Hq // Hkv)        # q-head tiles the sparse attention runs
    attn_ms = timed(lambda: ops.block_sparse_attention(qr, kr, v, sel))
    dense_ms = timed(lambda: ops.flash(qr, kr, v))
    flops = tiles * 4 * 128 * 128 * D
    return {"top_p": p, "anchor_fraction_q": float(kq.float().mean()), "anchor_fraction_k": float(kk.float().mean()),
            "selected_tile_fraction": tiles / (Hq * nb * (nb + 1) / 2), "selection_ms": sel_ms,
            "sparse_attention_ms": attn_ms, "dense_r1_ms": dense_ms,
            "sparse_attention_tflops": flops / attn_ms / 1e9, "frac_of_burst": flops / attn_ms / 1e9 / burst,
            "speedup_vs_dense": dense_ms / (attn_ms + sel_ms)}


def traffic_per_launch():
    """DRAM bytes per attention launch from the committed ncu summary, if present."""
    try:
        with open(os.path.join(ROOT, "profiles", "attn_tc_cfg2_traffic.json")) as f:
            return json.load(f).get("bytes_per_launch")
    except Exception:
        return None


_SAMPLER = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
hs = []
for key in sys.argv[2:]:
    try:
        hs.append(pynvml.nvmlDeviceGetHandleByUUID(key))
    except Exception:
        hs.append(pynvml.nvmlDeviceGetHandleByIndex(int(key.split(":")[-1])))
mx = [pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in hs]
pw = [0.0] * len(hs)
out = open(sys.argv[1], "w", buffering=1)
n = 0
while True:
    for i, h in enumerate(hs):
        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
        if n % 16 == 0:
            pw[i] = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
        out.write(f"{time.time():.6f},{i},{sm},{mx[i]},{pw[i]:.1f},{rs}\n")
    n += 1
    time.sleep(0.0002)
"""


class ClockSampler:
    """SM clock, power and clock-event reasons sampled DURING the timed region.

    A separate process polls NVML (every ~0.3 ms; two queries per sample, the power every 16th)
    and timestamps each sample, so the sampling neither waits on this process's interpreter
    lock nor perturbs the launches; ``mark_start`` / ``mark_end`` bracket the timed region and
    the summary keeps the samples inside it. ``nvidia-smi -lms 200`` is the fallback when
    NVML cannot be loaded. GPUs are matched to NVML by UUID (CUDA ordinals `gpus`), so
    CUDA_VISIBLE_DEVICES remapping does not confuse them."""

    REASONS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("hw_power_brake_slowdown", 0x80))
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = list(gpus)
        self.proc = None
        self.kind = None
        self.t0 = self.t1 = None
        self.path = os.path.join("/tmp", f"dab_clocks_{os.getpid()}.csv")

    def _keys(self):
        keys = []
        for i in self.gpus:
            try:
                uid = str(torch.cuda.get_device_properties(i).uuid)
                keys.append(uid if uid.startswith("GPU-") else "GPU-" + uid)
            except Exception:
                keys.append(f"index:{i}")
        return keys

    def __enter__(self):
        if os.path.exists(self.path):
            os.remove(self.path)
        try:
            import pynvml  # noqa: F401  (the sampler process needs it)
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, self.path, *self._keys()],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            self.kind = "nvml"
            t_end = time.time() + 20.0
            while time.time() < t_end and self.proc.poll() is None:  # wait for the first sample
                if os.path.exists(self.path) and os.path.getsize(self.path) > 0:
                    break
                time.sleep(0.01)
            if self.proc.poll() is not None:
                raise RuntimeError("NVML sampler exited")
            return self
        except Exception:
            self.proc = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
            self.kind = "nvidia-smi"
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self.kind == "nvidia-smi":
                self.fh.close()

    def summary(self):
        sm, mx, reasons = [], [], set()
        if self.kind == "nvml":
            src = "nvml sampler process (~0.3 ms)"
            try:
                for line in open(self.path):
                    f = line.strip().split(",")
                    if len(f) != 6:
                        continue
                    t = float(f[0])
                    if (self.t0 is not None and t < self.t0) or (self.t1 is not None and t > self.t1):
                        continue
                    sm.append(float(f[2]))
                    mx.append(float(f[3]))
                    for name, bit in self.REASONS:
                        if int(f[5]) & bit:
                            reasons.add(name)
            except Exception:
                pass
        elif self.kind == "nvidia-smi":
            src = "nvidia-smi (200 ms)"
            try:
                for line in open(self.path):
                    f = [x.strip() for x in line.split(",")]
                    if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.gpus:
                        continue
                    sm.append(float(f[1]))
                    mx.append(float(f[2]))
                    for name, val in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                          "sw_power_cap"], f[5:9]):
                        if val.lower().startswith("active"):
                            reasons.add(name)
            except Exception:
                pass
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "source": src}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "sm_mhz_min": min(sm),
                "reasons": sorted(reasons), "samples": len(sm), "source": src}


SUSTAINED_S = 4.0  # length of the back-to-back GEMM loop behind the sustained bf16 figure


def pick_peak(clocks, timed_s):
    """The roofline denominator for the attention launch: the burst bf16 figure unless the timed
    region was at least as long as the loop the sustained figure was measured over and ran below
    95% of the maximum SM clock; then the sustained power-capped figure. (The sustained figure's
    GEMM loop settles at a lower clock than a shorter region reaches, so against a short region
    it would overstate the fraction.)"""
    burst, sustained, src = peaks()
    sm, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    if sm and mx:
        below_max = sm < 0.95 * mx
        why = f"median SM clock {sm:.0f} of max {mx:.0f} MHz over the timed region ({timed_s * 1e3:.0f} ms)"
    else:
        below_max = False
        why = f"no clock samples; timed region {timed_s * 1e3:.0f} ms"
    if below_max and timed_s >= SUSTAINED_S:
        return sustained, f"{src} bf16 sustained ({why}); burst {burst}", burst
    return burst, f"{src} bf16 burst ({why}); sustained {sustained}", sustained


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------ CPU side
_CPU_INPUTS = {}


def _cpu_inputs(N):
    from deltaattention_b200 import synth
    if N not in _CPU_INPUTS:
        q, k, v = synth.layer_inputs(1, CFG["Hq"], CFG["Hkv"], N, CFG["D"], torch.bfloat16, seed=0, device="cpu")
        _CPU_INPUTS[N] = (q, k, v) + synth.rope_tables(N, CFG["D"], CFG["theta"], torch.bfloat16)
    return _CPU_INPUTS[N]


def cpu_sample(heads=(0, 1, 2, 3), stride=1, N=CFG["N"]):
    """Oracle (CPU restatement of the reference path) on q-heads `heads` of one cfg2 layer:
    RoPE of the sampled query rows and of the heads' kv-heads, periodic packing, and the
    two-phase attention on every `stride`-th 128-row query block.

    `heads` should be whole GQA groups (the default is kv-head 0's four q-heads), so the
    kv-head's RoPE and packing are charged to all of its query heads. Returns (seconds,
    tokens-equivalent): the sample's share of one layer's N tokens."""
    from oracle import delta_oracle as O
    q, k, v, cos, sin = _cpu_inputs(N)
    G = CFG["Hq"] // CFG["Hkv"]
    kv_heads = sorted({h // G for h in heads})
    nmb = -(-N // 128)
    blocks = list(range(0, nmb, stride))
    t0 = time.perf_counter()
    qs = q[:, list(heads)].contiguous()
    if stride == 1:
        q_ref = O.apply_rope(qs, cos, sin)
    else:  # only the sampled rows' RoPE is charged (the other rows are zeros, not attended)
        q_ref = torch.zeros_like(qs)
        for b_ in blocks:
            sl = slice(128 * b_, min(N, 128 * b_ + 128))
            q_ref[:, :, sl] = O.apply_rope(qs[:, :, sl], cos[:, sl], sin[:, sl])
    k_ref = O.apply_rope(k[:, kv_heads].contiguous(), cos, sin)
    vv = v[:, kv_heads].contiguous()
    keep = O.periodic_keep_mask(1, len(kv_heads), N, 1.0 / CFG["r"])
    _, kp, vp, ts, counts = O.pack_from_keep(k_ref, vv, keep)
    n_rep = len(heads) // len(kv_heads)  # heads are whole GQA groups, or part of one group
    O.hybrid_attention(q_ref, k_ref, vv, kp, vp, ts, counts.float(), CFG["D"] ** -0.5, CFG["W"], n_rep=n_rep,
                       query_blocks=blocks)
    dt = time.perf_counter() - t0
    return dt, 128 * len(blocks) * len(heads) / CFG["Hq"]


def cpu_eager_dense_sample(heads=(0, 1, 2, 3), blocks=8, N=CFG["N"]):
    """The reference's eager dense attention (eager_attention_forward, modeling_llama.py:235-276:
    QK^T over all N keys, causal mask, fp32 softmax, PV) on CPU: the r = 1 CPU point.

    Runs `blocks` 128-row query blocks spread evenly over the sequence for q-heads `heads`
    (eager attention costs the same N keys per row at every position). Returns (seconds,
    tokens-equivalent)."""
    from oracle import delta_oracle as O
    q, k, v, cos, sin = _cpu_inputs(N)
    G = CFG["Hq"] // CFG["Hkv"]
    kv_heads = sorted({h // G for h in heads})
    k_ref = O.apply_rope(k[:, kv_heads].contiguous(), cos, sin)
    vv = v[:, kv_heads].contiguous()
    nmb = -(-N // 128)
    picks = sorted({min(nmb - 1, (i * nmb) // blocks) for i in range(blocks)})
    qs = q[:, list(heads)].contiguous()
    t0 = time.perf_counter()
    for b_ in picks:
        sl = slice(128 * b_, min(N, 128 * b_ + 128))
        qr = O.apply_rope(qs[:, :, sl], cos[:, sl], sin[:, sl])
        qfull = torch.zeros_like(qs)
        qfull[:, :, sl] = qr
        O.eager_attention(qfull, k_ref, vv, CFG["D"] ** -0.5, n_rep=len(heads) // len(kv_heads), query_rows=sl)
    dt = time.perf_counter() - t0
    return dt, 128 * len(picks) * len(heads) / CFG["Hq"]


def run_reference(args, world, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    heads = (0, 1, 2, 3)  # kv-head 0 with its whole GQA group
    # one step is the whole group over every query block when that fits the budget (the whole
    # run stays within about three minutes); otherwise every `stride`-th query block
    t_probe, _ = cpu_sample(heads, stride=8)
    t_group = t_probe * 8
    budget = 150.0 / (args.steps + args.warmup)
    stride = max(1, min(64, int(-(-t_group // budget))))
    for _ in range(args.warmup):
        cpu_sample(heads, stride)
    secs, toks = 0.0, 0.0
    for _ in range(args.steps):
        dt, tk = cpu_sample(heads, stride)
        secs += dt
        toks += tk
    value = toks / secs
    nmb = -(-CFG["N"] // 128)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * secs / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, BASELINE cfg2)",
            "config": workload_config(world, "heads"), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"per step: kv-head 0 with its 4 q-heads (one whole GQA group, 4 of 32 "
                                       f"q-heads) of one N={CFG['N']} layer: RoPE, periodic packing, two-phase "
                                       f"attention on every {stride}th of {nmb} query blocks; tokens scaled by "
                                       f"the sampled rows"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU side
def _timed_steps(step, steps, stream, flush=None):
    """Run `steps` steps; returns total device ms. Without `flush` one event pair brackets the
    loop; with it, L2 is flushed between steps (outside the timed events) and the per-step
    event times are summed."""
    if flush is None:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            step(True)
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)
    evs = []
    for _ in range(steps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step(True)
        e1.record(stream)
        evs.append((e0, e1))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs)


L2_BYTES = 126 * 10 ** 6


def run_ours(args, world, rank, local):
    from deltaattention_b200 import _lib as L
    from deltaattention_b200 import ops, synth
    from deltaattention_b200 import shard as shard_mod
    dev = torch.device("cuda", local)
    B, Hq, Hkv, N, D, r, W = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["N"], CFG["D"], CFG["r"], CFG["W"]
    shard = args.shard
    if shard == "heads" and Hkv % world:
        raise SystemExit(f"--shard heads needs the {Hkv} kv-heads to divide over {world} GPUs")
    # inputs: the one sequence every rank generates from the same seed (it keeps its kv-heads and
    # their query heads), or with --shard seq a sequence of its own per rank
    seed = 1000 if shard == "heads" else 1000 + rank
    q_all, k_all, v_all = synth.layer_inputs(B, Hq, Hkv, N, D, torch.bfloat16, seed=seed, device=dev)
    cos, sin = synth.rope_tables(N, D, CFG["theta"], torch.bfloat16, device=dev)
    if shard == "heads":
        q, k, v = shard_mod.shard_layer(q_all, k_all, v_all, world, rank)
        tokens = B * N
    else:
        q, k, v = q_all, k_all, v_all
        tokens = B * N * world
    my_hq, my_hkv = q.shape[1], k.shape[1]
    in_bytes = (q.numel() + k.numel() + v.numel()) * 2
    flush = L2Flush(dev) if in_bytes < 1.5 * L2_BYTES else None
    period = r
    stream = torch.cuda.current_stream(dev)
    attn_events = []
    launches_per_step = 5  # rope(q), rope(k), periodic_meta, schedule, attention

    def step(record=False):
        q_rot = ops.rope(q, cos, sin)
        k_rot = ops.rope(k, cos, sin)
        packed = ops.pack_periodic(k_rot, v, period)
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        o = ops.attention(q_rot, k_rot, v, packed, dense_window=W)
        if record:
            e1.record(stream)
            attn_events.append((e0, e1))
        return o

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(range(world) if rank == 0 else [local]) as clk:
        torch.cuda.synchronize()
        barrier(world)
        clk.mark_start()
        total_ms = _timed_steps(step, args.steps, stream, flush)
        clk.mark_end()
        barrier(world)
    clocks = clk.summary()
    ms = max_over_ranks(total_ms / args.steps, world)
    attn_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in attn_events) / len(attn_events), world)
    codes = L.workspace_errors()
    if any(codes):
        raise RuntimeError(f"bounded device wait timed out during the bench: {codes}")
    value = tokens / (ms / 1000.0)

    if args.only_step:
        if rank == 0:
            print(json.dumps({"ms_per_step": ms, "attn_ms": attn_ms, "clocks": clocks}), flush=True)
        return
    # dense (r = 1) comparator through the same kernel family: causal flash with GQA by index
    q_rot, k_rot = ops.rope(q, cos, sin), ops.rope(k, cos, sin)
    for _ in range(2):
        ops.flash(q_rot, k_rot, v)
    torch.cuda.synchronize()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nd = max(3, args.steps // 4)
    d0.record(stream)
    for _ in range(nd):
        ops.flash(q_rot, k_rot, v)
    d1.record(stream)
    torch.cuda.synchronize()
    dense_ms = max_over_ranks(d0.elapsed_time(d1) / nd, world)
    extra = {}
    if world == 1:
        # the reference's other two kernels of the same family (deltaFlashAttention.py:149-357):
        # the sanity variant (phase-1 QK^T computed and discarded) and pure phase 1
        variants = {}
        pk = ops.pack_periodic(k_rot, v, period)
        for name in ("sanity", "pure_phase1"):
            ops.attention(q_rot, k_rot, v, pk, dense_window=W, variant=name)
            torch.cuda.synchronize()
            d0.record(stream)
            for _ in range(nd):
                ops.attention(q_rot, k_rot, v, pk, dense_window=W, variant=name)
            d1.record(stream)
            torch.cuda.synchronize()
            variants[name] = {"ms": d0.elapsed_time(d1) / nd}
        extra["variants"] = variants
        del pk
        # the reference's threshold ("row" delta) mode as a whole layer-op: RoPE, delta scan,
        # device packing and the two-phase attention; raw Euclidean threshold 11 keeps about 1
        # key in 4 here
        for _ in range(2):
            ops.delta_prefill(q, k, v, cos, sin, mode="delta", threshold=11.0, dense_window=W)
        torch.cuda.synchronize()
        d0.record(stream)
        for _ in range(nd):
            ops.delta_prefill(q, k, v, cos, sin, mode="delta", threshold=11.0, dense_window=W)
        d1.record(stream)
        torch.cuda.synchronize()
        delta_ms = d0.elapsed_time(d1) / nd
        extra["delta_mode"] = {"ms_per_layer_op": delta_ms, "tokens_per_s": B * N / (delta_ms / 1000.0),
                               "threshold": 11.0, "selection": "Euclidean delta scan, chunk 512"}
    else:
        # verification, outside the timed region: the gathered kv-head shards equal one GPU's
        # computation of the whole layer, bit for bit (the heads are independent)
        if shard == "heads":
            full = shard_mod.gather_heads(step(), world)
            if rank == 0:
                qr_, kr_ = ops.rope(q_all, cos, sin), ops.rope(k_all, cos, sin)
                want = ops.attention(qr_, kr_, v_all, ops.pack_periodic(kr_, v_all, period), dense_window=W)
                extra["verify"] = {"gathered_shards_equal_one_gpu": bool(torch.equal(
                    full.view(torch.int16), want.contiguous().view(torch.int16)))}
                del qr_, kr_, want
            del full
            barrier(world)
        # beside the kv-head-sharded sequence: every GPU running a whole cfg2 layer of its own
        # (one sequence per GPU, the data-parallel alternative), timed the same way
        def dp_step(record=False):
            qr_, kr_ = ops.rope(q_all, cos, sin), ops.rope(k_all, cos, sin)
            ops.attention(qr_, kr_, v_all, ops.pack_periodic(kr_, v_all, period), dense_window=W)
        for _ in range(3):
            dp_step()
        torch.cuda.synchronize()
        barrier(world)
        dp_ms = max_over_ranks(_timed_steps(dp_step, args.steps, stream) / args.steps, world)
        barrier(world)
        extra["dp_one_sequence_per_gpu"] = {"value": B * N * world / (dp_ms / 1000.0), "unit": UNIT,
                                            "ms_per_step": dp_ms, "scaling": "weak"}
    del q_rot, k_rot

    # end to end through the public API: pinned host inputs (head-major [B, H, N, d]) -> device
    # -> pinned host output; ops.delta_prefill_host overlaps each kv-head group's copies with
    # the previous group's compute, every byte still crosses PCIe inside the timed region
    hq = q.contiguous().cpu().pin_memory()
    hk = k.contiguous().cpu().pin_memory()
    hv = v.contiguous().cpu().pin_memory()
    ho = torch.empty((B, my_hq, N, D), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        ops.delta_prefill_host(hq, hk, hv, cos, sin, out=ho, keep_rate=1.0 / r, dense_window=W)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    ne = max(3, args.steps // 2)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(ne):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(s0.elapsed_time(s1) / ne, world)
    # every rank copies its own share: the job's bytes are world x this rank's
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2 * world
    d2h = ho.numel() * 2 * world
    # DRAM bytes of the committed ncu capture (a whole cfg2 launch, 8 kv-heads) scaled to this
    # rank's kv-heads (the traffic is per head)
    traffic = traffic_per_launch()
    traffic = traffic * my_hkv / Hkv if traffic else None

    timed_s = total_ms / 1000.0
    peak, peak_kind, other = pick_peak(clocks, timed_s)
    tiles = ops.tile_count_periodic(N, r, W)
    flops = B * my_hq * tiles * 4 * 128 * 128 * D
    achieved = flops / (attn_ms / 1000.0) / 1e12
    burst, sustained, _ = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if shard == "heads" else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded AR(1) keys + offsets, 0.5*N(0,1) q/v: BASELINE cfg2 distributions)",
        "config": workload_config(world, shard, flush is not None),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "attn_tc_kernel<128,bf16>", "attn_ms_per_launch": attn_ms,
                     "flops_per_launch": flops, "tiles_per_head": tiles, "peak_kind": peak_kind,
                     "frac_of_burst": achieved / burst, "frac_of_sustained": achieved / sustained},
        "e2e": {"value": tokens / (e2e_ms / 1000.0), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "ops.delta_prefill_host (pinned head-major host buffers; one kv-head per group, "
                       "H2D / compute / D2H on three streams)",
                "pcie_gbs_per_gpu": {"h2d": h2d / world / (e2e_ms / 1000.0) / 1e9,
                                     "d2h": d2h / world / (e2e_ms / 1000.0) / 1e9}},
        "dense_r1": {"ms_per_step": dense_ms, "speedup_of_delta_attention": dense_ms / attn_ms},
        **extra,
        "gpu_launches": launches_per_step * args.steps * world,
        "clocks": clocks,
    }
    if world == 1 and not args.no_sweep:
        line["sweep"] = sweep(dev, 3000 + rank)
    if world == 1:
        hk_ = hbm_kernels(dev, 2000 + rank)
        line["hbm_kernels"] = {"peak_gbs": hbm_peak()[0], "peak_kind": hbm_peak()[1], **hk_}
    if world == 1 and not args.no_sweep:
        line["proj_rope"] = proj_rope_bench(dev, 6000 + rank)
        line["dpxa"] = dpxa_bench(dev, 7000 + rank)
        line["decode_step"] = decode_step(dev, 4000 + rank)
        line["serving_cfg5"] = serving(dev, 5000 + rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        dt, tk = cpu_sample(tuple(range(8)))
        de, te = cpu_eager_dense_sample()
        line["cpu_baseline"] = {"value": tk / dt, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                                "sample": f"8 of 32 q-heads (2 whole GQA groups) of one N={N} layer (RoPE, "
                                          f"packing, two-phase attention), {dt:.1f} s; tokens scaled by 8/32",
                                "eager_dense_r1": {"value": te / de, "unit": UNIT, "seconds": de,
                                                   "sample": "the reference's eager dense attention "
                                                             "(modeling_llama.py:235-276) for 8 query blocks of "
                                                             "q-heads 0-3 spread over the sequence, all N keys; "
                                                             "tokens scaled by the rows computed"},
                                "os_cpu_count": os.cpu_count()}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--shard", default="heads", choices=["heads", "seq"],
                    help="multi-GPU partition: kv-heads of one sequence (default) or one sequence per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the cfg3 N / r sweep")
    ap.add_argument("--n", type=int, default=None, help="sequence length override (profiling small cases)")
    ap.add_argument("--only-step", action="store_true",
                    help="time the hot-path step only (no comparator, e2e or CPU legs); for profiling")
    ap.add_argument("--only-hbm", action="store_true",
                    help="run the HBM-bound kernel measurements alone and print them; for profiling")
    ap.add_argument("--only-dpxa", action="store_true",
                    help="run the DPXA selection + block-sparse attention measurement alone (honours --n)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.n:
        CFG["N"] = args.n
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup()
    if args.only_dpxa:
        print(json.dumps(dpxa_bench(torch.device("cuda", local), 7000 + rank)), flush=True)
        return
    if args.only_hbm:
        dev = torch.device("cuda", local)
        print(json.dumps({**hbm_kernels(dev, 2000 + rank), "decode_step": decode_step(dev, 4000 + rank),
                          "serving_cfg5": serving(dev, 5000 + rank)}), flush=True)
        return
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Decode cache with device-resident lengths (native API).

``HybridCompressedCache`` (deltaDecoding.py:111-233, mirrored in ``dropin/deltaDecoding.py``)
keeps the exact-window and total lengths of every layer as Python integers, reads the
largest packed length back from the GPU every 256 tokens (deltaDecoding.py:216-221) and
grows its packed buffers by copying them. ``DeviceDecodeCache`` keeps the same buffers
(shapes, dtypes, layouts) and runs the same kernels, with three differences:

* the ``(exact, total)`` lengths of each layer live in an int64 device tensor, read by the
  update and attention kernels and advanced on the device (by the attention call's last
  kernel in ``step``), so a decode step issues kernel launches only (no host
  synchronisation, no host-side length bookkeeping);
* the packed capacity is fixed at construction (prefill anchors plus the decode steps
  planned: each step appends at most one anchor per head); a full cache sets the update
  kernel's error word (0x201) instead of growing;
* because nothing in a step depends on host values that change per token, a whole
  multi-layer step can be captured once in a CUDA graph and replayed per token
  (``capture_step``).

Outputs and cache contents are bit-identical to the host-length launches of the same
kernels (tests/test_gpu_parity.py).
"""
from __future__ import annotations

import torch

from . import _lib as L


class DeviceDecodeCache:
    """Per-layer hybrid compressed KV cache; lengths on the device."""

    def __init__(self, num_layers, batch, kv_heads, head_dim, capacity, exact_window, dtype=torch.bfloat16,
                 device="cuda", threshold=0.0, use_cosine=False):
        self.num_layers, self.bsz, self.n_kv_heads, self.head_dim = num_layers, batch, kv_heads, head_dim
        self.capacity, self.exact_window_size, self.dtype = int(capacity), int(exact_window), dtype
        self.device = torch.device(device)
        # the reference compares cosine similarity with the raw threshold and Euclidean
        # distance with its square (deltaDecoding.py:75-96)
        self.use_cosine = bool(use_cosine)
        self.threshold = float(threshold) if use_cosine else float(threshold) ** 2
        shp = (num_layers, batch, kv_heads)
        dev = self.device
        self.k_packed = torch.zeros((*shp, self.capacity, head_dim), device=dev, dtype=dtype)
        self.v_packed = torch.zeros_like(self.k_packed)
        self.packed_counts = torch.zeros((*shp, self.capacity), device=dev, dtype=torch.int32)
        self.packed_timestamps = torch.zeros((*shp, self.capacity), device=dev, dtype=torch.int32)
        self.packed_lengths = torch.zeros((num_layers, batch * kv_heads), device=dev, dtype=torch.int32)
        self.k_exact = torch.zeros((*shp, self.exact_window_size, head_dim), device=dev, dtype=dtype)
        self.v_exact = torch.zeros_like(self.k_exact)
        self.seq_state = torch.zeros((num_layers, 2), device=dev, dtype=torch.int64)  # (exact, total) per layer
        self.err = torch.zeros((1,), device=dev, dtype=torch.int32)
        self._ws = None
        self._ws_heads = 0

    def load_prefill(self, layer, k_packed, v_packed, counts, timestamps, k_exact, v_exact, total_len,
                     batch_index=None):
        """The prefill hand-off of ``HybridCompressedCache.initialize_from_prefill``.

        With ``batch_index`` the tensors hold one sequence ([1, Hkv, ...]) and fill that row of
        the batch, so sequences of different lengths (a varlen prefill) are loaded one by one.
        The batch shares the layer's (exact, total) pair, as the reference's cache does; the
        total only stamps the timestamps of anchors appended during decode."""
        p_len = k_packed.shape[2]
        if p_len > self.capacity:
            raise ValueError(f"DeviceDecodeCache: {p_len} packed anchors exceed the capacity {self.capacity}")
        b = slice(None) if batch_index is None else slice(int(batch_index), int(batch_index) + 1)
        self.k_packed[layer, b, :, :p_len] = k_packed
        self.v_packed[layer, b, :, :p_len] = v_packed
        self.packed_counts[layer, b, :, :p_len] = counts
        self.packed_timestamps[layer, b, :, :p_len] = timestamps
        self.packed_lengths[layer].view(self.bsz, self.n_kv_heads)[b] = p_len
        e_len = k_exact.shape[2]
        self.k_exact[layer, b, :, :e_len] = k_exact
        self.v_exact[layer, b, :, :e_len] = v_exact
        self.seq_state[layer, 0] = e_len
        self.seq_state[layer, 1] = int(total_len)

    def _workspace(self, hq):
        if self._ws is None or self._ws_heads != hq:
            lib = L.load()
            nbytes = lib.dab_decode_attention_workspace_size(self.bsz, hq, self.capacity, self.exact_window_size,
                                                             self.head_dim)
            self._ws = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=self.device)
            self._ws_heads = hq
        return self._ws

    def update(self, layer, k_new, v_new, advance=True):
        """Append one token per (batch, kv-head): k_new / v_new [B, Hkv, 1, d]. Advances the
        layer's lengths on the device (with ``advance=False`` the advance is left to the next
        ``attend(..., advance=True)``)."""
        L.require_cuda(k_new, v_new)
        lib = L.load()
        st = L.stream_of(k_new)
        ke, kp, pc = self.k_exact[layer], self.k_packed[layer], self.packed_counts[layer]
        bd = 16
        while bd < self.head_dim:
            bd <<= 1
        L.check(lib.dab_decode_update_dev(
            L.ptr(k_new), L.ptr(v_new), L.ptr(ke), L.ptr(self.v_exact[layer]), L.ptr(kp),
            L.ptr(self.v_packed[layer]), L.ptr(pc), L.ptr(self.packed_timestamps[layer]),
            L.ptr(self.packed_lengths[layer]), L.ptr(self.seq_state[layer]), self.threshold, self.exact_window_size,
            L.dtype_code(k_new), L.strides(k_new.stride()), L.strides(ke.stride()), L.strides(kp.stride()),
            L.strides(pc.stride()), self.n_kv_heads, self.head_dim, bd, 1 if self.use_cosine else 0,
            self.bsz * self.n_kv_heads, self.capacity, L.ptr(self.err), st), "decode_update_dev")
        if advance:
            L.check(lib.dab_decode_advance(L.ptr(self.seq_state[layer]), 1, st), "decode_advance")

    def attend(self, layer, q, out=None, sm_scale=None, advance=False):
        """Decode attention of q [B, Hq, d] over the layer's packed history and exact window.

        With ``advance`` the call also performs the length advance an ``update(...,
        advance=False)`` left pending: it attends with the advanced window length and steps
        the lengths after its last read."""
        L.require_cuda(q, out)
        B, hq, D = q.shape
        if out is None:
            out = torch.empty_like(q)
        if sm_scale is None:
            sm_scale = D ** -0.5
        lib = L.load()
        st = L.stream_of(q)
        kp, vp, pc = self.k_packed[layer], self.v_packed[layer], self.packed_counts[layer]
        pl = self.packed_lengths[layer].view(self.bsz, self.n_kv_heads)
        ke, ve = self.k_exact[layer], self.v_exact[layer]
        strides = [*q.stride(), *kp.stride(), *vp.stride(), *pc.stride(), *pl.stride(), *ke.stride(), *ve.stride(),
                   *out.stride()]
        ws = self._workspace(hq)
        L.check(lib.dab_decode_attention_dev(
            L.ptr(q), L.ptr(kp), L.ptr(vp), L.ptr(pc), L.ptr(pl), L.ptr(ke), L.ptr(ve), L.ptr(out), L.dtype_code(q),
            L.strides(strides), float(sm_scale), L.ptr(self.seq_state[layer]), 1 if advance else 0,
            self.exact_window_size,
            hq // self.n_kv_heads, B, hq, D, self.capacity, L.ptr(ws), ws.numel(), st), "decode_attention_dev")
        return out

    def step(self, layer, q, k_new, v_new, out=None):
        """One layer's decode step: update, length advance, attention (the reference's order),
        as two launches: the advance rides with the attention call."""
        self.update(layer, k_new, v_new, advance=False)
        return self.attend(layer, q, out, advance=True)

    def lengths(self):
        """(exact, total) per layer, read back to the host (a synchronising call)."""
        return [tuple(int(x) for x in row) for row in self.seq_state.cpu()]

    def capture_step(self, q, k_new, v_new, out):
        """Capture one decode step over every layer in a CUDA graph.

        q / out [layers, B, Hq, d], k_new / v_new [layers, B, Hkv, 1, d] are static device
        buffers: write a token's inputs into them, then ``graph.replay()`` runs the step and
        leaves the result in ``out``. Returns the ``torch.cuda.CUDAGraph``."""
        self._workspace(q.shape[2])
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for layer in range(self.num_layers):
                self.step(layer, q[layer], k_new[layer], v_new[layer], out[layer])
        torch.cuda.current_stream(self.device).wait_stream(s)
        return g

"""Drop-in for the reference's deltaDecoding.py (hybrid compressed KV cache for decoding).

``fused_hybrid_decode_update_kernel`` (deltaDecoding.py:9-104) and
``fused_hybrid_decode_kernel`` (deltaDecoding.py:236-362) keep their launch syntax.
``HybridCompressedCache`` (deltaDecoding.py:111-233) keeps its constructor, buffers
(shapes, dtypes, layouts), prefill hand-off and per-token ``update`` behaviour: a ring of
``exact_window_size`` exact tokens per (batch, kv-head); each evicted token merges into the
last packed anchor (count + 1) or is appended (count 1, timestamp = total - window).
"""
import torch

try:
    from transformers import Cache as _CacheBase
except Exception:  # pragma: no cover - transformers is optional for the kernels
    _CacheBase = object

from deltaattention_b200.launch import fused_hybrid_decode_kernel, fused_hybrid_decode_update_kernel  # noqa: F401


def _flags():
    try:
        import globVR  # the reference's flag module, when present on sys.path
        return globVR
    except ImportError:
        return None


def _next_pow2(n):
    p = 1
    while p < n:
        p <<= 1
    return p


class HybridCompressedCache(_CacheBase):
    def __init__(self, config, batch_size, dtype=torch.float16, exact_window_size=50, initial_capacity=1024,
                 device=None):
        try:
            super().__init__()
        except (TypeError, ValueError):
            # recent transformers Cache requires layer descriptions this cache does not use
            pass
        self.exact_window_size = exact_window_size
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        self.n_kv_heads = config.num_key_value_heads
        self.bsz = batch_size
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.num_layers = config.num_hidden_layers
        self.capacity = initial_capacity
        shp = (self.num_layers, self.bsz, self.n_kv_heads)
        self.k_packed = torch.zeros((*shp, self.capacity, self.head_dim), device=self.device, dtype=self.dtype)
        self.v_packed = torch.zeros_like(self.k_packed)
        self.packed_counts = torch.zeros((*shp, self.capacity), device=self.device, dtype=torch.int32)
        self.packed_timestamps = torch.zeros((*shp, self.capacity), device=self.device, dtype=torch.int32)
        self.packed_lengths = torch.zeros((self.num_layers, self.bsz * self.n_kv_heads), device=self.device,
                                          dtype=torch.int32)
        self.k_exact = torch.zeros((*shp, self.exact_window_size, self.head_dim), device=self.device,
                                   dtype=self.dtype)
        self.v_exact = torch.zeros_like(self.k_exact)
        self.exact_seq_lens = [0] * self.num_layers
        self.max_packed_len = [0] * self.num_layers
        self.total_seq_lens = [0] * self.num_layers

    def _expand_capacity(self, target_capacity):
        new_cap = max(self.capacity * 2, target_capacity)
        shp = (self.num_layers, self.bsz, self.n_kv_heads)
        nk = torch.zeros((*shp, new_cap, self.head_dim), device=self.device, dtype=self.dtype)
        nv = torch.zeros_like(nk)
        nc = torch.zeros((*shp, new_cap), device=self.device, dtype=torch.int32)
        nt = torch.zeros((*shp, new_cap), device=self.device, dtype=torch.int32)
        old = self.k_packed.shape[3]
        if old > 0:
            nk[..., :old, :] = self.k_packed
            nv[..., :old, :] = self.v_packed
            nc[..., :old] = self.packed_counts
            nt[..., :old] = self.packed_timestamps
        self.k_packed, self.v_packed, self.packed_counts, self.packed_timestamps = nk, nv, nc, nt
        self.capacity = new_cap

    def initialize_from_prefill(self, layer_idx, k_packed, v_packed, counts, timestamps, k_exact, v_exact,
                                original_q_len):
        p_len = k_packed.shape[2]
        self.max_packed_len[layer_idx] = p_len
        if p_len > self.capacity:
            self._expand_capacity(p_len + 1024)
        self.k_packed[layer_idx, :, :, :p_len, :] = k_packed
        self.v_packed[layer_idx, :, :, :p_len, :] = v_packed
        self.packed_counts[layer_idx, :, :, :p_len] = counts
        self.packed_timestamps[layer_idx, :, :, :p_len] = timestamps
        self.packed_lengths[layer_idx, :] = p_len
        e_len = k_exact.shape[2]
        self.k_exact[layer_idx, :, :, :e_len, :] = k_exact
        self.v_exact[layer_idx, :, :, :e_len, :] = v_exact
        self.exact_seq_lens[layer_idx] = e_len
        self.total_seq_lens[layer_idx] = original_q_len

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        if key_states.shape[2] > 1:
            return key_states, value_states
        if self.max_packed_len[layer_idx] + 1 >= self.capacity:
            self._expand_capacity(self.capacity + 1024)
        g = _flags()
        metric = getattr(g, "row_similarity_metric", "euclidean") if g else "euclidean"
        use_cosine = metric == "cosine"
        raw = getattr(g, "row_delta_threshold", 0.0) if g else 0.0
        thr = raw if use_cosine else raw ** 2
        L = layer_idx
        fused_hybrid_decode_update_kernel[(self.bsz * self.n_kv_heads,)](
            key_states, value_states,
            self.k_exact[L], self.v_exact[L], self.k_packed[L], self.v_packed[L],
            self.packed_counts[L], self.packed_timestamps[L], self.packed_lengths[L],
            self.exact_seq_lens[L], self.total_seq_lens[L], thr, self.exact_window_size,
            key_states.stride(0), key_states.stride(1), key_states.stride(2), key_states.stride(3),
            self.k_exact.stride(1), self.k_exact.stride(2), self.k_exact.stride(3), self.k_exact.stride(4),
            self.k_packed.stride(1), self.k_packed.stride(2), self.k_packed.stride(3), self.k_packed.stride(4),
            self.packed_counts.stride(1), self.packed_counts.stride(2), self.packed_counts.stride(3),
            self.n_kv_heads, self.head_dim,
            BLOCK_D=_next_pow2(self.head_dim), USE_COSINE=use_cosine,
        )
        if self.exact_seq_lens[L] >= self.exact_window_size:
            self.max_packed_len[L] += 1
            if self.total_seq_lens[L] % 256 == 0:
                self.max_packed_len[L] = int(self.packed_lengths[L].max().item())
        self.exact_seq_lens[L] += 1
        self.total_seq_lens[L] += 1
        return key_states, value_states

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.total_seq_lens[layer_idx]

    def get_max_length(self):
        return None

    def get_max_cache_shape(self):
        return None


__all__ = ["HybridCompressedCache", "fused_hybrid_decode_kernel", "fused_hybrid_decode_update_kernel"]

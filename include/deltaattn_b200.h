/* deltaattn_b200.h - C ABI of the B200 (sm_100a) DeltaAttention hot-path library.
 *
 * Conventions shared by every entry point:
 *   - pointers are device pointers; strides are in ELEMENTS, one int64 per dimension, in
 *     the same order as the reference kernel's stride arguments;
 *   - `dtype` is DAB_F32, DAB_F16 or DAB_BF16 and applies to the float tensors;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 *     asynchronous on it and allocates no device memory;
 *   - the return value is 0 on success; otherwise dab_last_error() describes the failure
 *     (its text contains "CUDA" when a CUDA call failed, matching the reference's
 *     classifier at eval_speedup.py:119-123).
 * Reference citations are file:line in the DeltaAttention project.
 */
#ifndef DELTAATTN_B200_H
#define DELTAATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DAB_F32 0
#define DAB_F16 1
#define DAB_BF16 2

#define DAB_HYBRID 0      /* hybrid_compressed_flash_kernel         deltaFlashAttention.py:9-146   */
#define DAB_SANITY 1      /* hybrid_compressed_flash_kernel_sanity  deltaFlashAttention.py:149-259 */
#define DAB_PURE_PHASE1 2 /* pure_phase1_flash_kernel               deltaFlashAttention.py:262-357 */

/* Message of the last failing call on this thread. */
const char* dab_last_error(void);
/* ABI revision of this header (1). */
int dab_abi_version(void);

/* Makes `device` current for this library's CUDA runtime on the calling thread (callers
 * that switch devices with another runtime instance call this before launching). */
int dab_set_device(int device);

/* Reads and clears the device error word at the start of an attention workspace (a bounded
 * in-kernel wait that timed out records a nonzero code there). Synchronises `stream`. */
int dab_workspace_error(void* workspace, int* code, void* stream);

/* chunked_eval_kernel[grid](in_ptr, keep_mask_ptr, chunk_counts_ptr, threshold_sq,
 *   stride_in_*(4), stride_km_*(3), stride_cc_*(3), seq_len, head_dim, chunk_size,
 *   num_heads, BLOCK_D, USE_COSINE) - tritonModules.py:7-69, launched at
 * modeling_llama.py:643-652 with grid (grid_bh, grid_chunks). Keep decisions are bit-exact
 * with the reference (same reduction order). */
int dab_chunked_eval(const void* in, int dtype, const int64_t* in_strides, int32_t* keep_mask,
                     const int64_t* km_strides, int32_t* chunk_counts, const int64_t* cc_strides,
                     float threshold, int64_t seq_len, int64_t head_dim, int64_t chunk_size,
                     int64_t num_heads, int64_t grid_bh, int64_t grid_chunks, int64_t block_d,
                     int use_cosine, void* stream);

/* parallel_scatter_pack_kv_kernel[grid](k_in, v_in, k_packed, v_packed, pt, keep_mask,
 *   index_map, strides k(4) v(4) kp(4) vp(4) pt(3) km(3) im(3), seq_len, head_dim,
 *   num_heads, BLOCK_S, BLOCK_D) - tritonModules.py:72-132, launched at
 * modeling_llama.py:667-680 with grid (grid_bh, grid_s). `num_packed` is the packed row
 * count (destinations outside [0, num_packed) are skipped instead of written). */
int dab_parallel_scatter_pack_kv(const void* k_in, const void* v_in, void* k_packed, void* v_packed,
                                 int32_t* packed_ts, const int32_t* keep_mask, const int32_t* index_map,
                                 int dtype, const int64_t* k_strides, const int64_t* v_strides,
                                 const int64_t* kp_strides, const int64_t* vp_strides,
                                 const int64_t* ts_strides, const int64_t* km_strides,
                                 const int64_t* im_strides, int64_t seq_len, int64_t head_dim,
                                 int64_t num_heads, int64_t num_packed, int64_t grid_bh, int64_t grid_s,
                                 int64_t block_s, void* stream);

/* Scratch bytes dab_hybrid_flash / dab_attn_fwd_flat need (batch, heads of the timestamp
 * tensor, query length, packed length). */
size_t dab_hybrid_flash_workspace_size(int64_t batch, int64_t ts_heads, int64_t seq_len_q, int64_t num_packed);

/* hybrid_compressed_flash_kernel / _sanity / pure_phase1_flash_kernel[grid](Q, K_dense,
 *   V_dense, K_packed, V_packed, Packed_Timestamps, Packed_Counts, Out, 30 strides in the
 *   reference order (q, kd, vd, kp, vp: 4 each; ts, counts: 3 each; out: 4), sm_scale,
 *   seq_len_q, seq_len_k, num_packed_keys, head_dim, num_heads, denseWindowSize,
 *   BLOCK_M, BLOCK_N, BLOCK_D) - deltaFlashAttention.py:9-357, wrappers at
 * modeling_llama.py:306-451, grid (grid_m, grid_bh).
 * Extensions: `counts_is_int` (counts given as int32 rather than the wrapper's fp32);
 * `kv_group` (q-head h reads K/V/timestamps/counts of head h / kv_group, which replaces the
 * repeat_kv copies of modeling_llama.py:700-708; 1 = the reference's expanded call);
 * `force_simt` (use the CUDA-core kernel even when the tcgen05 kernel applies).
 * bf16/fp16 with head_dim 64/128 and 128x128 blocks run on tcgen05; everything else on the
 * CUDA-core kernel. */
int dab_hybrid_flash(int variant, const void* q, const void* k_dense, const void* v_dense,
                     const void* k_packed, const void* v_packed, const int32_t* packed_ts,
                     const void* packed_counts, int counts_is_int, void* out, int dtype,
                     const int64_t* strides, float sm_scale, int64_t seq_len_q, int64_t seq_len_k,
                     int64_t num_packed, int64_t head_dim, int64_t num_heads, int64_t dense_window,
                     int64_t grid_m, int64_t grid_bh, int64_t block_m, int64_t block_n, int64_t block_d,
                     int64_t kv_group, void* workspace, size_t workspace_bytes, int force_simt, void* stream);

/* dab_hybrid_flash with the packed length kept on the device (native: the reference reads it
 * back to size the packed tensors, modeling_llama.py:655-656). `anchors_per_head` [B * Hts]
 * int32 holds every (batch, kv-head)'s kept count; the packed length M is their maximum,
 * taken on the device, and results equal dab_hybrid_flash on the same tensors cut to M rows.
 * The packed tensors (K/V, timestamps, counts) have `capacity` rows, a multiple of 128 and at
 * least M. For each head, rows [anchors, ceil(anchors / 128) * 128) must hold zero K / V,
 * timestamp 0 and count 0 (dab_delta_compress writes them); later rows are not read: rows
 * [anchors, M) are the reference's zero padding, scheduled (their zero timestamps enter the
 * phase-1 stop rule) but not loaded. The workspace is sized with num_packed = capacity.
 * tcgen05 path only (bf16 / fp16, head_dim 64 / 128, 128 x 128 blocks); other calls return 1. */
int dab_hybrid_flash_devlen(int variant, const void* q, const void* k_dense, const void* v_dense,
                            const void* k_packed, const void* v_packed, const int32_t* packed_ts,
                            const void* packed_counts, int counts_is_int, const int32_t* anchors_per_head,
                            void* out, int dtype, const int64_t* strides, float sm_scale, int64_t seq_len_q,
                            int64_t seq_len_k, int64_t capacity, int64_t head_dim, int64_t num_heads,
                            int64_t dense_window, int64_t grid_m, int64_t grid_bh, int64_t block_m, int64_t block_n,
                            int64_t block_d, int64_t kv_group, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Bytes of the library's static device scratch behind dab_hybrid_flash_noalloc. */
#define DAB_NOALLOC_SCRATCH_BYTES (1u << 20)

/* No counterpart in the reference (the reference's kernels need no scratch). The same call as
 * dab_hybrid_flash without the caller workspace: the phase schedule, the per-block
 * timestamp minima and count weights live in a file-scope device array of
 * DAB_NOALLOC_SCRATCH_BYTES per device, and the call allocates nothing (no cudaMalloc, no
 * allocator of any framework). For callers that hold no device allocator: a binding written
 * against the reference's launch signature alone, which has no scratch argument.
 * - Limit: dab_hybrid_flash_workspace_size(grid_bh / num_heads, num_heads / kv_group,
 *   seq_len_q, num_packed) must not exceed DAB_NOALLOC_SCRATCH_BYTES; larger calls return 1
 *   with a message naming both sizes. The size is 256 + 8*B*H*ceil(Nq/128) +
 *   8*B*H*ceil(num_packed/128) bytes (each array rounded up to 256; H = timestamp heads), so
 *   e.g. 128 k queries x 64 timestamp heads fit while num_packed <= 64 k (r >= 2), not at r = 1.
 * - The scratch used is the current device's copy; q must live on the current device (else
 *   the call returns 1).
 * - The first call on a device resolves the scratch address for that device (with that
 *   device current); make it before any stream capture. The address is kept for the life of
 *   the process: do not cudaDeviceReset a device this entry point has used.
 * - The array keeps the last call's contents. Only its 256-byte header (the device error word
 *   a timed-out in-kernel wait sets) must start at zero, and every call clears it on its stream
 *   first; every other scratch byte a call reads is written earlier in the same call.
 *   dab_noalloc_error reads that word after a call.
 * - Calls that overlap on one device (other streams or threads) share the scratch and race;
 *   serialise them. */
int dab_hybrid_flash_noalloc(int variant, const void* q, const void* k_dense, const void* v_dense,
                             const void* k_packed, const void* v_packed, const int32_t* packed_ts,
                             const void* packed_counts, int counts_is_int, void* out, int dtype,
                             const int64_t* strides, float sm_scale, int64_t seq_len_q, int64_t seq_len_k,
                             int64_t num_packed, int64_t head_dim, int64_t num_heads, int64_t dense_window,
                             int64_t grid_m, int64_t grid_bh, int64_t block_m, int64_t block_n, int64_t block_d,
                             int64_t kv_group, int force_simt, void* stream);

/* No counterpart in the reference. Reads and clears the error word of the current device's
 * dab_hybrid_flash_noalloc scratch (nonzero: a bounded in-kernel wait of the last call timed
 * out and its output is not valid); 0 when no call has run on the device. Synchronises
 * `stream`, so call it on the stream of the call it checks. */
int dab_noalloc_error(int* code, void* stream);

/* _attn_fwd_flat[grid](Q, K, V, sm_scale, Out, 16 strides (q, k, v, out), Z, H, N_CTX,
 *   HEAD_DIM, BLOCK_M, BLOCK_N, IS_CAUSAL) - flashAttention.py:5-91, wrapper
 * triton_flash_attention flashAttention.py:94-130, grid (grid_m, grid_zh). */
int dab_attn_fwd_flat(const void* q, const void* k, const void* v, float sm_scale, void* out, int dtype,
                      const int64_t* strides, int64_t Z, int64_t H, int64_t n_ctx, int64_t head_dim,
                      int64_t block_m, int64_t block_n, int is_causal, int64_t grid_m, int64_t grid_zh,
                      int64_t kv_group, void* workspace, size_t workspace_bytes, int force_simt, void* stream);

/* fused_hybrid_decode_update_kernel[(programs,)](new_k, new_v, k_exact, v_exact, k_packed,
 *   v_packed, packed_counts, packed_timestamps, packed_lengths, exact_seq_len,
 *   total_seq_len, threshold_sq, exact_window_size, strides new(4) exact(4) pack(4) pc(3),
 *   num_heads, head_dim, BLOCK_D, USE_COSINE) - deltaDecoding.py:9-104, launched at
 * deltaDecoding.py:197-211. `capacity` bounds appends; an append past it writes 0x201 into
 * `err_word` (may be NULL) instead of memory. */
int dab_decode_update(const void* new_k, const void* new_v, void* k_exact, void* v_exact, void* k_packed,
                      void* v_packed, int32_t* packed_counts, int32_t* packed_ts, int32_t* packed_lengths,
                      int64_t exact_seq_len, int64_t total_seq_len, float threshold, int64_t exact_window,
                      int dtype, const int64_t* new_strides, const int64_t* exact_strides,
                      const int64_t* pack_strides, const int64_t* pc_strides, int64_t num_heads,
                      int64_t head_dim, int64_t block_d, int use_cosine, int64_t programs, int64_t capacity,
                      int* err_word, void* stream);

/* Scratch bytes dab_decode_attention needs. */
size_t dab_decode_attention_workspace_size(int64_t batch, int64_t num_q_heads, int64_t capacity,
                                           int64_t exact_len, int64_t head_dim);

/* fused_hybrid_decode_kernel[(B, Hq)](Q, K_packed, V_packed, Packed_Counts, Packed_Lengths,
 *   K_exact, V_exact, Out, 27 strides (q 3, kp 4, vp 4, counts 3, lengths 2, ke 4, ve 4,
 *   out 3), sm_scale, exact_len, num_kv_groups, head_dim, BLOCK_M, BLOCK_N, BLOCK_D) -
 * deltaDecoding.py:236-362, wrapper modeling_llama.py:453-518. `capacity` is the packed
 * buffers' row capacity (bounds the split-K grid). */
int dab_decode_attention(const void* q, const void* k_packed, const void* v_packed, const int32_t* packed_counts,
                         const int32_t* packed_lengths, const void* k_exact, const void* v_exact, void* out,
                         int dtype, const int64_t* strides, float sm_scale, int64_t exact_len,
                         int64_t num_kv_groups, int64_t batch, int64_t num_q_heads, int64_t head_dim,
                         int64_t capacity, void* workspace, size_t workspace_bytes, void* stream);

/* Decode with device-resident sequence lengths (native; the reference keeps them on the host,
 * deltaDecoding.py:216-221). seq_state points to int64 {exact_seq_len, total_seq_len} in
 * device memory, the values dab_decode_update / dab_decode_attention take as host arguments.
 * dab_decode_update_dev is dab_decode_update reading them there; dab_decode_attention_dev is
 * dab_decode_attention with exact_len = min(seq_state[0], exact_window) read on the device
 * (the workspace is sized with exact_len = exact_window); dab_decode_advance adds 1 to both
 * lengths of `count` consecutive states. One decode step is update, advance, attention, the
 * order of modeling_llama.py's update, length increment and attention. With advance != 0,
 * dab_decode_attention_dev folds the advance into the attention call: it reads
 * exact_len = min(seq_state[0] + 1, exact_window) and adds 1 to both lengths after its last
 * read, so a step is update then attention (one launch fewer). */
int dab_decode_update_dev(const void* new_k, const void* new_v, void* k_exact, void* v_exact, void* k_packed,
                          void* v_packed, int32_t* packed_counts, int32_t* packed_ts, int32_t* packed_lengths,
                          const int64_t* seq_state, float threshold, int64_t exact_window, int dtype,
                          const int64_t* new_strides, const int64_t* exact_strides, const int64_t* pack_strides,
                          const int64_t* pc_strides, int64_t num_heads, int64_t head_dim, int64_t block_d,
                          int use_cosine, int64_t programs, int64_t capacity, int* err_word, void* stream);
int dab_decode_attention_dev(const void* q, const void* k_packed, const void* v_packed,
                             const int32_t* packed_counts, const int32_t* packed_lengths, const void* k_exact,
                             const void* v_exact, void* out, int dtype, const int64_t* strides, float sm_scale,
                             int64_t* seq_state, int advance, int64_t exact_window, int64_t num_kv_groups,
                             int64_t batch, int64_t num_q_heads, int64_t head_dim, int64_t capacity, void* workspace,
                             size_t workspace_bytes, void* stream);
int dab_decode_advance(int64_t* seq_state, int64_t count, void* stream);

/* apply_rotary_pos_emb for one tensor (modeling_llama.py:180-204): y = x*cos +
 * rotate_half(x)*sin with eager rounding to the tensor dtype after each op. x/y strides
 * (b, h, s, d); cos/sin strides (b, s, d) (b-stride 0 broadcasts). */
int dab_rope(const void* x, const int64_t* x_strides, void* y, const int64_t* y_strides, const void* cos_t,
             const void* sin_t, const int64_t* cs_strides, int dtype, int64_t batch, int64_t heads,
             int64_t seq_len, int64_t head_dim, void* stream);

/* q/k/v projection with RoPE as the GEMM epilogue (modeling_llama.py:550-555:
 * `k_proj(hidden_states).view(B, N, H, d).transpose(1, 2)` then apply_rotary_pos_emb at
 * :180-204). out[r, c] = x[r, :] . w[c, :] (nn.Linear, no bias), rounded to bf16; columns in
 * [rope_lo, rope_hi) (head-aligned) then get RoPE with eager bf16 rounding, using table row r
 * of cos / sin ([rows, 128]). x [rows, in_features], w [out_features, in_features], out
 * [rows, out_features]: unit column stride, 16-byte aligned row strides (elements). bf16,
 * head_dim 128, out_features a multiple of 128. `workspace` holds the 256-byte error header
 * (dab_workspace_error). */
int dab_proj_rope(const void* x, int64_t x_row_stride, const void* w, int64_t w_row_stride, const void* cos_t,
                  const void* sin_t, int64_t cs_row_stride, void* out, int64_t out_row_stride, int dtype,
                  int64_t rows, int64_t in_features, int64_t out_features, int64_t head_dim, int64_t rope_lo,
                  int64_t rope_hi, void* workspace, size_t workspace_bytes, void* stream);

/* DPXA: delta-based tile scoring for block-sparse prefill (Paper/src/methodology.tex:89-135;
 * the paper ships no code, so these entries implement the library's specification of it).
 *
 * dab_dpxa_compact: the anchors of every 128-token block (keep_mask from the delta selection
 * with chunk 128, e.g. dab_chunked_eval) gathered to the front of the block: `compact`
 * [B][H][nb][128][head_dim], their positions [B][H][nb][128] and counts [B][H][nb] int32.
 * x [B, H, N, d] with unit d-stride and 16-byte aligned rows; bf16 / fp16, d 64 or 128. */
int dab_dpxa_compact(const void* x, const int64_t* x_strides, const int32_t* keep_mask, const int64_t* km_strides,
                     void* compact, int32_t* positions, int32_t* counts, int dtype, int64_t batch, int64_t heads,
                     int64_t seq_len, int64_t head_dim, void* stream);
/* dab_dpxa_score: for every (batch, q-head, query block i, key block j <= i) the sampled tile
 * scores S = sm_scale * Q^d_i K^d_j^T over the compacted anchors (K of kv-head h / kv_group),
 * causal by anchor position on the diagonal tile, reduced to tile_max = max S and
 * tile_sum = sum exp(S - tile_max), fp32 [B][Hq][nb][nb]; entries j > i are not written. */
int dab_dpxa_score(const void* q_compact, const int32_t* q_positions, const int32_t* q_counts,
                   const void* k_compact, const int32_t* k_positions, const int32_t* k_counts, float* tile_max,
                   float* tile_sum, float sm_scale, int dtype, int64_t batch, int64_t num_q_heads, int64_t kv_group,
                   int64_t seq_len, int64_t head_dim, void* stream);
/* dab_dpxa_select: per (batch, kv-head, query block) the tiles' sampled attention mass
 * averaged over the group's q-heads, taken by decreasing weight (ties to the lower block)
 * until the cumulative weight exceeds top_p, plus the diagonal: bitmask `selection`
 * [B][Hkv][nb][ceil(nb / 32)] (bit j of word j / 32). nb <= 2048. */
int dab_dpxa_select(const float* tile_max, const float* tile_sum, uint32_t* selection, float top_p, int64_t batch,
                    int64_t num_kv_heads, int64_t kv_group, int64_t seq_len, void* stream);
/* Causal attention over the selected 128-key blocks only (the tcgen05 kernel walking the
 * bitmask), full K / V: q [B, Hq, N, d], k / v [B, Hq / kv_group, N, d], out [B, Hq, N, d];
 * `strides` q, k, v, out (4 each, elements). bf16 / fp16, d 64 or 128, unit d-stride,
 * 16-byte aligned rows. `workspace` holds the 256-byte error header. */
int dab_block_sparse_attention(const void* q, const void* k, const void* v, const uint32_t* selection, void* out,
                               int dtype, const int64_t* strides, float sm_scale, int64_t batch, int64_t num_q_heads,
                               int64_t kv_group, int64_t seq_len, int64_t head_dim, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Packed timestamps / counts of periodic packing (modeling_llama.py:626-632 followed by
 * :655-685): anchor j at j*period covering min(period, seq_len - j*period) tokens.
 * Buffers are [batch_heads][num_packed] contiguous; num_packed must be ceil(seq_len/period).
 * `packed_counts_f32` (optional, may be NULL) receives the counts as fp32, the form the
 * attention kernel weights probabilities with.
 * The packed K/V rows of periodic packing are a strided view of K/V (row stride x period),
 * so no copy is made. */
int dab_periodic_meta(int32_t* packed_ts, int32_t* packed_counts, float* packed_counts_f32, int64_t batch_heads,
                      int64_t num_packed, int64_t seq_len, int64_t period, void* stream);

/* Scratch bytes dab_pack_from_keep needs: a 64-byte header (error word first, then the
 * launch's ticket / done counters and epoch) and one status word per 1024-token tile. The
 * workspace must be zero-filled before its first use and is then reused as is, one
 * workspace per stream (each launch leaves the counters reset). */
size_t dab_pack_from_keep_workspace_size(int64_t batch, int64_t heads, int64_t seq_len);

/* Device-side packing from a keep mask (modeling_llama.py:655-685 without the host sync at
 * :656): index_map = cumsum(keep) - 1 (optional, [B][H][N] contiguous), packed K/V rows,
 * timestamps and run-length counts into buffers of `capacity` rows, anchors per head and
 * their maximum (the reference's M). Rows beyond a head's anchors are written with zero
 * K / V, timestamp 0 and count 0: the reference's zero-initialised padding, so the caller
 * need not clear the buffers. One launch: tiles find their packed offsets by a look-back
 * over the head's earlier tiles (bounded waits; a timeout sets the workspace's error word). */
int dab_pack_from_keep(const int32_t* keep_mask, const int64_t* km_strides, const void* k, const int64_t* k_strides,
                       const void* v, const int64_t* v_strides, void* k_packed, void* v_packed,
                       const int64_t* pack_strides, int32_t* packed_ts, int32_t* packed_counts,
                       const int64_t* meta_strides, int32_t* index_map, int dtype, int64_t batch, int64_t heads,
                       int64_t seq_len, int64_t head_dim, int64_t capacity, int32_t* anchors_per_head,
                       int32_t* max_anchors, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes dab_delta_compress needs (a 256-byte header, then 8 bytes per chunk). The
 * scratch must be zeroed once before its first use; the kernel leaves it ready for the next
 * call, so one scratch serves successive calls on one stream (not concurrent calls). */
size_t dab_delta_compress_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t chunk_size);

/* Threshold ("row" delta) key compression in one launch: apply_rotary_pos_emb on the raw keys
 * (modeling_llama.py:180-204, eager rounding, bit-identical to dab_rope) written to k_rot;
 * chunked_eval_kernel's selection on the rotated keys (tritonModules.py:7-69: squared Euclidean
 * distance > threshold_sq, or cosine < threshold_sq with use_cosine; bit-exact keep decisions,
 * written to keep_mask when it is not NULL); and the packing of modeling_llama.py:655-685 (K rows
 * from the rotated keys, V rows, timestamps, run-length counts as int32 and, when not NULL,
 * fp32), with the packed length left on the device: anchors_per_head[B * H] receives every
 * head's kept count (the reference's M = their maximum, modeling_llama.py:656, is taken by
 * dab_hybrid_flash_devlen on the device). Packed buffers have `capacity` rows per head (keep
 * it >= seq_len); for each head, rows [anchors, min(capacity, ceil(anchors / 128) * 128))
 * are written as zero K / V, timestamp 0 and count 0; later rows are left untouched.
 * Strides: k, v, k_rot, packed K / V (b, h, s, d); cos / sin (b, s, d), b-stride 0 broadcasts;
 * keep mask and packed metadata (b, h, s). Rows must be contiguous and 16-byte aligned,
 * bf16 / fp16, head_dim 64 or 128, chunk_size <= 1024. A bounded wait that times out or a
 * capacity overflow sets the workspace's first word (dab_workspace_error reads it). */
int dab_delta_compress(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       const void* cos_t, const void* sin_t, const int64_t* cs_strides, void* k_rot,
                       const int64_t* rot_strides, int32_t* keep_mask, const int64_t* km_strides, void* k_packed,
                       void* v_packed, const int64_t* pack_strides, int32_t* packed_ts, int32_t* packed_counts,
                       float* packed_counts_f32, const int64_t* meta_strides, int32_t* anchors_per_head, int dtype,
                       int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, float threshold_sq,
                       int use_cosine, int64_t chunk_size, int64_t capacity, void* workspace,
                       size_t workspace_bytes, void* stream);

/* N:M structured anchor selection (nmDeltaFlashAttention; the reference ships only a
 * compiled module for it, so the semantics are this library's own): candidates are the
 * positions t % stride == 0; candidate t scores +inf at t == 0, else the fp32 squared
 * distance between K[t] and K[t - stride]; every run of m_group consecutive candidates
 * keeps its min(n_keep, size) highest scores (ties to the earlier position). Writes the
 * whole keep mask (int32, 0/1). The packed length is dab_nm_num_packed(...) for every
 * head, so the result packs without a host sync. */
int dab_nm_select(const void* k, const int64_t* k_strides, int32_t* keep_mask, const int64_t* km_strides, int dtype,
                  int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t n_keep, int64_t m_group,
                  int64_t stride, void* stream);
/* Anchors per head that dab_nm_select keeps. */
int64_t dab_nm_num_packed(int64_t seq_len, int64_t n_keep, int64_t m_group, int64_t stride);

#ifdef __cplusplus
}
#endif
#endif /* DELTAATTN_B200_H */

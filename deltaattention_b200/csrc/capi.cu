// C ABI of the B200 delta-attention library (declared in include/deltaattn_b200.h).
//
// Every entry point takes plain device pointers, element strides, scalars and a CUDA
// stream, launches asynchronously on that stream and returns 0 or a nonzero status whose
// message `dab_last_error()` returns. No entry point allocates device memory: scratch is
// passed in by the caller (sizes from the *_workspace_size functions).
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <string>

#include "params.cuh"
#include "../../include/deltaattn_b200.h"

namespace dab {
cudaError_t launch_chunked_eval(int, int, bool, const void*, const int64_t*, int32_t*, const int64_t*, int32_t*,
                                const int64_t*, float, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                cudaStream_t);
cudaError_t launch_scatter_pack(int, const void*, const void*, void*, void*, int32_t*, const int32_t*,
                                const int32_t*, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                                const int64_t*, const int64_t*, const int64_t*, int64_t, int64_t, int64_t, int64_t,
                                int64_t, int64_t, cudaStream_t);
cudaError_t launch_rope(int, const void*, const int64_t*, void*, const int64_t*, const void*, const void*,
                        const int64_t*, int64_t, int64_t, int64_t, int64_t, cudaStream_t);
cudaError_t launch_periodic_meta(int32_t*, int32_t*, float*, int64_t, int64_t, int64_t, int64_t, cudaStream_t);
cudaError_t launch_pack_from_keep(int, const int32_t*, const int64_t*, const void*, const int64_t*, const void*,
                                  const int64_t*, void*, void*, const int64_t*, int32_t*, int32_t*, const int64_t*,
                                  int32_t*, int64_t, int64_t, int64_t, int64_t, int64_t, uint8_t*, int32_t*,
                                  int32_t*, cudaStream_t);
size_t pack_from_keep_workspace(int64_t, int64_t);
cudaError_t launch_attn_simt(int, const SimtParams&, cudaStream_t);
cudaError_t launch_attn_tc(int, bool, const TcParams&, int, cudaStream_t);
cudaError_t launch_schedule(const int32_t*, const int64_t*, const void*, const int64_t*, int, int, int, int, int,
                            int, int, int, int2*, int32_t*, int, float*, const int32_t*, int*, cudaStream_t);
cudaError_t launch_decode_update(int, int, bool, const void*, const void*, void*, void*, void*, void*, int32_t*,
                                 int32_t*, int32_t*, int64_t, int64_t, const int64_t*, float, int64_t, const int64_t*,
                                 const int64_t*, const int64_t*, const int64_t*, int64_t, int64_t, int64_t, int64_t,
                                 int*, cudaStream_t);
cudaError_t launch_decode_attn(int, const void*, const int64_t*, const void*, const int64_t*, const void*,
                               const int64_t*, const int32_t*, const int64_t*, const int32_t*, const int64_t*,
                               const void*, const int64_t*, const void*, const int64_t*, void*, const int64_t*,
                               float, int64_t, int64_t*, int, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                               float*, cudaStream_t);
cudaError_t launch_decode_advance(int64_t*, int64_t, cudaStream_t);
size_t decode_attn_workspace(int64_t, int64_t, int64_t, int64_t, int64_t);
cudaError_t launch_nm_select(int, const void*, const int64_t*, int32_t*, const int64_t*, int64_t, int64_t, int64_t,
                             int64_t, int, int, int64_t, cudaStream_t);
cudaError_t launch_key_compress(int, int, bool, CompressParams, cudaStream_t);
size_t key_compress_workspace(int64_t, int64_t, int64_t, int64_t);
cudaError_t launch_proj_rope(const ProjParams&, int, cudaStream_t);
cudaError_t launch_dpxa_compact(int, const void*, const int64_t*, const int32_t*, const int64_t*, void*, int32_t*,
                                int32_t*, int, int, int, int, cudaStream_t);
cudaError_t launch_dpxa_score(int, const void*, const int32_t*, const int32_t*, const void*, const int32_t*,
                              const int32_t*, float*, float*, float, int, int, int, int, int, cudaStream_t);
cudaError_t launch_dpxa_select(const float*, const float*, uint32_t*, float, int, int, int, int, cudaStream_t);
}  // namespace dab

using namespace dab;

namespace {
thread_local std::string g_err;
int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 0;
  return fail(2, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}
int elem_size(int dtype) { return dtype == F32 ? 4 : 2; }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// 4-D map over (d, rows, heads, batch) with a 64 x box_rows box and 128-byte swizzle.
bool encode_rows(CUtensorMap* m, const void* base, int dtype, int64_t d, int64_t rows, int64_t heads,
                 int64_t batch, int64_t s_row, int64_t s_head, int64_t s_batch, uint32_t box_rows = 128) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  const int es = elem_size(dtype);
  if (rows < 1 || heads < 1 || batch < 1) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(batch)};
  // extents of 1 never move: give them a harmless legal stride
  int64_t sr = s_row, sh = s_head, sb = s_batch;
  if (rows == 1) sr = d;
  if (heads == 1) sh = sr * rows;
  if (batch == 1) sb = sh * heads;
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(sr * es), static_cast<cuuint64_t>(sh * es),
                           static_cast<cuuint64_t>(sb * es)};
  for (auto s : strides)
    if (s % 16 != 0 || s == 0 || s >= (1ull << 40)) return false;
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

constexpr size_t WS_HEADER = 256;  // device error word + padding
size_t round256(size_t x) { return (x + 255) & ~size_t(255); }
}  // namespace

extern "C" {

const char* dab_last_error(void) { return g_err.c_str(); }

int dab_abi_version(void) { return 1; }

int dab_set_device(int device) { return cuda_status(cudaSetDevice(device), "dab_set_device"); }

int dab_workspace_error(void* workspace, int* code, void* stream) {
  if (!workspace || !code) return fail(1, "dab_workspace_error: null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int), st);
  if (e != cudaSuccess) return cuda_status(e, "dab_workspace_error");
  *code = v;
  return 0;
}

// ------------------------------------------------------------------------- selection
int dab_chunked_eval(const void* in, int dtype, const int64_t* in_strides, int32_t* keep_mask,
                     const int64_t* km_strides, int32_t* chunk_counts, const int64_t* cc_strides, float threshold,
                     int64_t seq_len, int64_t head_dim, int64_t chunk_size, int64_t num_heads, int64_t grid_bh,
                     int64_t grid_chunks, int64_t block_d, int use_cosine, void* stream) {
  if (!in || !keep_mask || !chunk_counts) return fail(1, "dab_chunked_eval: null pointer");
  if (block_d < head_dim || block_d > 256 || (block_d & (block_d - 1)))
    return fail(1, "dab_chunked_eval: BLOCK_D must be a power of two in [head_dim, 256]");
  if (chunk_size <= 0 || num_heads <= 0) return fail(1, "dab_chunked_eval: bad chunk_size / num_heads");
  const int bd = block_d < 16 ? 16 : static_cast<int>(block_d);
  return cuda_status(launch_chunked_eval(dtype, bd, use_cosine != 0, in, in_strides, keep_mask, km_strides,
                                         chunk_counts, cc_strides, threshold, seq_len, head_dim, chunk_size,
                                         num_heads, grid_bh, grid_chunks, static_cast<cudaStream_t>(stream)),
                     "chunked_eval");
}

int dab_parallel_scatter_pack_kv(const void* k_in, const void* v_in, void* k_packed, void* v_packed,
                                 int32_t* packed_ts, const int32_t* keep_mask, const int32_t* index_map, int dtype,
                                 const int64_t* k_strides, const int64_t* v_strides, const int64_t* kp_strides,
                                 const int64_t* vp_strides, const int64_t* ts_strides, const int64_t* km_strides,
                                 const int64_t* im_strides, int64_t seq_len, int64_t head_dim, int64_t num_heads,
                                 int64_t num_packed, int64_t grid_bh, int64_t grid_s, int64_t block_s,
                                 void* stream) {
  if (!k_in || !v_in || !keep_mask || !index_map) return fail(1, "dab_parallel_scatter_pack_kv: null pointer");
  if (num_packed > 0 && (!k_packed || !v_packed || !packed_ts))
    return fail(1, "dab_parallel_scatter_pack_kv: null packed buffer");
  if (num_heads <= 0) return fail(1, "dab_parallel_scatter_pack_kv: num_heads must be positive");
  return cuda_status(launch_scatter_pack(dtype, k_in, v_in, k_packed, v_packed, packed_ts, keep_mask, index_map,
                                         k_strides, v_strides, kp_strides, vp_strides, ts_strides, km_strides,
                                         im_strides, seq_len, head_dim, num_heads, grid_bh, grid_s * block_s,
                                         num_packed, static_cast<cudaStream_t>(stream)),
                     "parallel_scatter_pack_kv");
}

// ------------------------------------------------------------------------- attention
size_t dab_hybrid_flash_workspace_size(int64_t batch, int64_t ts_heads, int64_t seq_len_q, int64_t num_packed) {
  const int64_t nmb = (seq_len_q + 127) / 128;
  const int64_t nblk = (num_packed + 127) / 128;
  return WS_HEADER + round256(static_cast<size_t>(batch * ts_heads * nmb) * 8) +
         2 * round256(static_cast<size_t>(batch * ts_heads * (nblk > 0 ? nblk : 1)) * 4);
}

static int run_attention(int variant, int causal, const void* q, const void* kd, const void* vd, const void* kp,
                         const void* vp, const int32_t* ts, const void* counts, int counts_is_int, void* out,
                         int dtype, const int64_t* qs, const int64_t* kds, const int64_t* vds, const int64_t* kps,
                         const int64_t* vps, const int64_t* tss, const int64_t* cs, const int64_t* os,
                         float sm_scale, int64_t seq_q, int64_t seq_k, int64_t num_packed, int64_t head_dim,
                         int64_t num_heads, int64_t window, int64_t grid_m, int64_t grid_bh, int64_t block_m,
                         int64_t block_n, int64_t block_d, int64_t kv_group, void* workspace,
                         size_t workspace_bytes, int force_simt, cudaStream_t st, const char* name,
                         const int32_t* anchors = nullptr) {
  if (!q || !kd || !vd || !out) return fail(1, std::string(name) + ": null pointer");
  if (num_heads <= 0 || kv_group <= 0 || num_heads % kv_group) return fail(1, std::string(name) + ": bad heads");
  if (grid_bh % num_heads) return fail(1, std::string(name) + ": grid must cover whole batches of heads");
  if (block_d < head_dim) return fail(1, std::string(name) + ": BLOCK_D < head_dim");
  const int64_t B = grid_bh / num_heads;
  const int64_t Hts = num_heads / kv_group;
  const bool needs_packed = (variant != 3);
  if (needs_packed && num_packed > 0 && (!kp || !vp || !ts || !counts))
    return fail(1, std::string(name) + ": null packed tensor");
  const int64_t nmb = (seq_q + 127) / 128;
  const int64_t nblk = (num_packed + 127) / 128;

  // ---- tcgen05 path eligibility
  bool tc = !force_simt && (dtype == BF16 || dtype == F16) && (head_dim == 64 || head_dim == 128) &&
            block_d == head_dim && block_m == 128 && block_n == 128 && grid_m == nmb && sm_scale > 0.f &&
            seq_q > 0 && seq_k > 0 && seq_q < (1ll << 31) && seq_k < (1ll << 31) && num_packed < (1ll << 31);
  tc = tc && qs[3] == 1 && kds[3] == 1 && vds[3] == 1 && os[3] == 1 && aligned16(q) && aligned16(kd) &&
       aligned16(vd);
  if (needs_packed && num_packed > 0) tc = tc && kps[3] == 1 && vps[3] == 1 && aligned16(kp) && aligned16(vp);
  const size_t need_ws = dab_hybrid_flash_workspace_size(B, Hts, seq_q, num_packed);
  if (tc && (!workspace || workspace_bytes < need_ws)) tc = false;
  if (anchors) {
    // device packed length: tcgen05 path only, and the capacity a whole number of blocks (every
    // block a head holds is read whole; its rows past the anchors are zeros)
    if (!tc || !needs_packed || num_packed <= 0 || num_packed % 128)
      return fail(1, std::string(name) +
                         ": the device packed length needs the tcgen05 path (bf16 / fp16, head_dim 64 / 128, "
                         "128 x 128 blocks, unit inner strides, 16-byte aligned rows, a large enough workspace) "
                         "and a capacity that is a positive multiple of 128");
  }
  if (tc) {
    TcParams p;
    std::memset(&p, 0, sizeof(p));
    bool ok = encode_rows(&p.tm_q, q, dtype, head_dim, seq_q, num_heads, B, qs[2], qs[1], qs[0]);
    ok = ok && encode_rows(&p.tm_kd, kd, dtype, head_dim, seq_k, Hts, B, kds[2], kds[1], kds[0]);
    ok = ok && encode_rows(&p.tm_vd, vd, dtype, head_dim, seq_k, Hts, B, vds[2], vds[1], vds[0]);
    if (needs_packed && num_packed > 0) {
      ok = ok && encode_rows(&p.tm_kp, kp, dtype, head_dim, num_packed, Hts, B, kps[2], kps[1], kps[0]);
      ok = ok && encode_rows(&p.tm_vp, vp, dtype, head_dim, num_packed, Hts, B, vps[2], vps[1], vps[0]);
    } else {
      p.tm_kp = p.tm_kd;
      p.tm_vp = p.tm_vd;
    }
    if (ok) {
      uint8_t* ws = static_cast<uint8_t*>(workspace);
      p.err = reinterpret_cast<int*>(ws);
      p.sched = reinterpret_cast<const int2*>(ws + WS_HEADER);
      p.blkmin = reinterpret_cast<const int32_t*>(ws + WS_HEADER + round256(static_cast<size_t>(B * Hts * nmb) * 8));
      p.blkw = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(p.blkmin) +
                                              round256(static_cast<size_t>(B * Hts * (nblk > 0 ? nblk : 1)) * 4));
      p.out = out;
      p.os_b = os[0]; p.os_h = os[1]; p.os_m = os[2];
      p.ts = ts; p.ts_b = tss ? tss[0] : 0; p.ts_h = tss ? tss[1] : 0; p.ts_n = tss ? tss[2] : 0;
      p.counts = counts; p.cs_b = cs ? cs[0] : 0; p.cs_h = cs ? cs[1] : 0; p.cs_n = cs ? cs[2] : 0;
      p.counts_is_int = counts_is_int;
      p.scale_log2 = sm_scale * 1.4426950408889634f;
      p.seq_q = static_cast<int>(seq_q); p.seq_k = static_cast<int>(seq_k);
      p.num_packed = static_cast<int>(needs_packed ? num_packed : 0);
      p.B = static_cast<int>(B); p.Hq = static_cast<int>(num_heads); p.kv_group = static_cast<int>(kv_group);
      p.Hts = static_cast<int>(Hts);
      p.nmb = static_cast<int>(nmb); p.nblk = static_cast<int>(needs_packed ? nblk : 0);
      p.variant = variant; p.causal = causal;
      p.pair_heads = (kv_group % 2 == 0) ? 1 : 0;
      p.num_units = static_cast<int>(p.pair_heads ? nmb * B * Hts * (kv_group / 2) : ((nmb + 1) / 2) * B * num_heads);
      p.out_vec_ok = aligned16(out) && (os[0] * 2) % 16 == 0 && (os[1] * 2) % 16 == 0 && (os[2] * 2) % 16 == 0;
      // counts (and timestamps) rows: contiguous along keys with 16-byte aligned block starts
      p.anchors = anchors;
      p.len_dev = reinterpret_cast<const int*>(ws + 4);  // header word 1: the device packed length
      // device-packed (threshold) histories carry run-length counts that differ inside blocks
      p.keyed = anchors != nullptr;
      p.meta_bulk = needs_packed && num_packed > 0 && counts && cs && cs[2] == 1 && num_packed % 4 == 0 &&
                    aligned16(counts) && (cs[0] * 4) % 16 == 0 && (cs[1] * 4) % 16 == 0 &&
                    (variant != 2 || (ts && tss && tss[2] == 1 && aligned16(ts) && (tss[0] * 4) % 16 == 0 &&
                                      (tss[1] * 4) % 16 == 0));
      if (variant != 3 && num_packed > 0) {
        cudaError_t e = launch_schedule(ts, tss, counts, cs, counts_is_int, static_cast<int>(B),
                                        static_cast<int>(Hts), static_cast<int>(num_packed), static_cast<int>(seq_k),
                                        static_cast<int>(window), static_cast<int>(nmb), static_cast<int>(nblk),
                                        reinterpret_cast<int2*>(ws + WS_HEADER),
                                        reinterpret_cast<int32_t*>(const_cast<int32_t*>(p.blkmin)), variant == 2,
                                        const_cast<float*>(p.blkw), anchors, reinterpret_cast<int*>(ws + 4), st);
        if (e != cudaSuccess) return cuda_status(e, "schedule");
      } else if (variant != 3) {
        // no packed keys: phase 1 is empty and phase 2 starts at key 0
        cudaError_t e = cudaMemsetAsync(ws + WS_HEADER, 0, static_cast<size_t>(B * Hts * nmb) * 8, st);
        if (e != cudaSuccess) return cuda_status(e, "schedule");
      }
      return cuda_status(launch_attn_tc(static_cast<int>(head_dim), dtype == BF16, p, num_sms(), st), name);
    }
    // tensor maps not encodable (strides / alignment): fall through to the CUDA-core path
  }
  SimtParams sp;
  std::memset(&sp, 0, sizeof(sp));
  sp.q = q; sp.kd = kd; sp.vd = vd; sp.kp = kp; sp.vp = vp; sp.ts = ts; sp.counts = counts; sp.out = out;
  for (int i = 0; i < 4; ++i) {
    sp.qs[i] = qs[i]; sp.kds[i] = kds[i]; sp.vds[i] = vds[i]; sp.os[i] = os[i];
    sp.kps[i] = kps ? kps[i] : 0; sp.vps[i] = vps ? vps[i] : 0;
  }
  for (int i = 0; i < 3; ++i) { sp.tss[i] = tss ? tss[i] : 0; sp.cs[i] = cs ? cs[i] : 0; }
  sp.sm_scale = sm_scale;
  sp.seq_q = seq_q; sp.seq_k = seq_k; sp.num_packed = needs_packed ? num_packed : 0; sp.head_dim = head_dim;
  sp.num_heads = num_heads; sp.dense_window = window; sp.grid_m = grid_m; sp.grid_bh = grid_bh;
  sp.block_m = block_m; sp.block_n = block_n; sp.kv_group = kv_group; sp.counts_is_int = counts_is_int;
  sp.causal = causal; sp.variant = variant;
  if (head_dim > 128) return fail(1, std::string(name) + ": head_dim > 128 is not supported");
  if (block_m % 32) return fail(1, std::string(name) + ": BLOCK_M must be a multiple of 32");
  return cuda_status(launch_attn_simt(dtype, sp, st), name);
}

int dab_hybrid_flash(int variant, const void* q, const void* k_dense, const void* v_dense, const void* k_packed,
                     const void* v_packed, const int32_t* packed_ts, const void* packed_counts, int counts_is_int,
                     void* out, int dtype, const int64_t* strides, float sm_scale, int64_t seq_len_q,
                     int64_t seq_len_k, int64_t num_packed, int64_t head_dim, int64_t num_heads,
                     int64_t dense_window, int64_t grid_m, int64_t grid_bh, int64_t block_m, int64_t block_n,
                     int64_t block_d, int64_t kv_group, void* workspace, size_t workspace_bytes, int force_simt,
                     void* stream) {
  if (variant < 0 || variant > 2) return fail(1, "dab_hybrid_flash: variant must be 0, 1 or 2");
  if (!strides) return fail(1, "dab_hybrid_flash: null strides");
  const int64_t* s = strides;
  return run_attention(variant, 1, q, k_dense, v_dense, k_packed, v_packed, packed_ts, packed_counts,
                       counts_is_int, out, dtype, s + 0, s + 4, s + 8, s + 12, s + 16, s + 20, s + 23, s + 26,
                       sm_scale, seq_len_q, seq_len_k, num_packed, head_dim, num_heads, dense_window, grid_m,
                       grid_bh, block_m, block_n, block_d, kv_group, workspace, workspace_bytes, force_simt,
                       static_cast<cudaStream_t>(stream), "hybrid_flash");
}

int dab_hybrid_flash_devlen(int variant, const void* q, const void* k_dense, const void* v_dense,
                            const void* k_packed, const void* v_packed, const int32_t* packed_ts,
                            const void* packed_counts, int counts_is_int, const int32_t* anchors_per_head,
                            void* out, int dtype, const int64_t* strides, float sm_scale, int64_t seq_len_q,
                            int64_t seq_len_k, int64_t capacity, int64_t head_dim, int64_t num_heads,
                            int64_t dense_window, int64_t grid_m, int64_t grid_bh, int64_t block_m, int64_t block_n,
                            int64_t block_d, int64_t kv_group, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (variant < 0 || variant > 2) return fail(1, "dab_hybrid_flash_devlen: variant must be 0, 1 or 2");
  if (!strides || !anchors_per_head) return fail(1, "dab_hybrid_flash_devlen: null strides / anchors");
  const int64_t* s = strides;
  return run_attention(variant, 1, q, k_dense, v_dense, k_packed, v_packed, packed_ts, packed_counts,
                       counts_is_int, out, dtype, s + 0, s + 4, s + 8, s + 12, s + 16, s + 20, s + 23, s + 26,
                       sm_scale, seq_len_q, seq_len_k, capacity, head_dim, num_heads, dense_window, grid_m,
                       grid_bh, block_m, block_n, block_d, kv_group, workspace, workspace_bytes, 0,
                       static_cast<cudaStream_t>(stream), "hybrid_flash_devlen", anchors_per_head);
}

// Static scratch of dab_hybrid_flash_noalloc (one copy per device, zeroed at module load).
static __device__ __align__(256) uint8_t g_noalloc_scratch[DAB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

int dab_hybrid_flash_noalloc(int variant, const void* q, const void* k_dense, const void* v_dense,
                             const void* k_packed, const void* v_packed, const int32_t* packed_ts,
                             const void* packed_counts, int counts_is_int, void* out, int dtype,
                             const int64_t* strides, float sm_scale, int64_t seq_len_q, int64_t seq_len_k,
                             int64_t num_packed, int64_t head_dim, int64_t num_heads, int64_t dense_window,
                             int64_t grid_m, int64_t grid_bh, int64_t block_m, int64_t block_n, int64_t block_d,
                             int64_t kv_group, int force_simt, void* stream) {
  if (variant < 0 || variant > 2) return fail(1, "dab_hybrid_flash_noalloc: variant must be 0, 1 or 2");
  if (!strides) return fail(1, "dab_hybrid_flash_noalloc: null strides");
  if (num_heads <= 0 || kv_group <= 0 || num_heads % kv_group || grid_bh <= 0 || grid_bh % num_heads)
    return fail(1, "dab_hybrid_flash_noalloc: bad heads / grid");
  const size_t need = dab_hybrid_flash_workspace_size(grid_bh / num_heads, num_heads / kv_group, seq_len_q,
                                                      num_packed);
  if (need > DAB_NOALLOC_SCRATCH_BYTES)
    return fail(1, "dab_hybrid_flash_noalloc: this call needs " + std::to_string(need) +
                       " bytes of scratch but the static scratch holds " +
                       std::to_string(static_cast<size_t>(DAB_NOALLOC_SCRATCH_BYTES)) +
                       " (batch x heads x query blocks too large); use dab_hybrid_flash with a workspace");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "dab_hybrid_flash_noalloc (cudaGetDevice)");
  if (dev < 0 || dev >= kMaxDevices) return fail(1, "dab_hybrid_flash_noalloc: device ordinal out of range");
  // the scratch used is the current device's copy: the tensors must live on that device
  if (q) {
    cudaPointerAttributes pa;
    e = cudaPointerGetAttributes(&pa, q);
    if (e != cudaSuccess) return cuda_status(e, "dab_hybrid_flash_noalloc (cudaPointerGetAttributes)");
    if ((pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged) && pa.device != dev)
      return fail(1, "dab_hybrid_flash_noalloc: q lives on device " + std::to_string(pa.device) +
                         " but device " + std::to_string(dev) +
                         " is current; make the tensors' device current (dab_set_device) first");
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      // resolved with `dev` current: the address is that device's copy of the array
      e = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_noalloc_scratch);
      if (e != cudaSuccess) {
        g_noalloc_ptr[dev] = nullptr;
        return cuda_status(e, "dab_hybrid_flash_noalloc (cudaGetSymbolAddress)");
      }
    }
    scratch = g_noalloc_ptr[dev];
  }
  // the array keeps the previous call's contents: the header (device error word) must start
  // at zero so a timed-out wait of this call is recorded; everything else is written before read
  e = cudaMemsetAsync(scratch, 0, 256, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "dab_hybrid_flash_noalloc (clearing the scratch header)");
  const int64_t* s = strides;
  return run_attention(variant, 1, q, k_dense, v_dense, k_packed, v_packed, packed_ts, packed_counts,
                       counts_is_int, out, dtype, s + 0, s + 4, s + 8, s + 12, s + 16, s + 20, s + 23, s + 26,
                       sm_scale, seq_len_q, seq_len_k, num_packed, head_dim, num_heads, dense_window, grid_m,
                       grid_bh, block_m, block_n, block_d, kv_group, scratch, DAB_NOALLOC_SCRATCH_BYTES,
                       force_simt, static_cast<cudaStream_t>(stream), "hybrid_flash_noalloc");
}

int dab_noalloc_error(int* code, void* stream) {
  if (!code) return fail(1, "dab_noalloc_error: null argument");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "dab_noalloc_error (cudaGetDevice)");
  if (dev < 0 || dev >= kMaxDevices) return fail(1, "dab_noalloc_error: device ordinal out of range");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    scratch = g_noalloc_ptr[dev];
  }
  if (!scratch) {  // no dab_hybrid_flash_noalloc call on this device yet
    *code = 0;
    return 0;
  }
  return dab_workspace_error(scratch, code, stream);
}

int dab_attn_fwd_flat(const void* q, const void* k, const void* v, float sm_scale, void* out, int dtype,
                      const int64_t* strides, int64_t Z, int64_t H, int64_t n_ctx, int64_t head_dim,
                      int64_t block_m, int64_t block_n, int is_causal, int64_t grid_m, int64_t grid_zh,
                      int64_t kv_group, void* workspace, size_t workspace_bytes, int force_simt, void* stream) {
  if (!strides) return fail(1, "dab_attn_fwd_flat: null strides");
  (void)Z;
  const int64_t* s = strides;
  int bd = 16;
  while (bd < head_dim) bd <<= 1;
  return run_attention(3, is_causal, q, k, v, nullptr, nullptr, nullptr, nullptr, 0, out, dtype, s + 0, s + 4,
                       s + 8, nullptr, nullptr, nullptr, nullptr, s + 12, sm_scale, n_ctx, n_ctx, 0, head_dim, H, 0,
                       grid_m, grid_zh, block_m, block_n, bd, kv_group, workspace, workspace_bytes, force_simt,
                       static_cast<cudaStream_t>(stream), "attn_fwd_flat");
}

// ------------------------------------------------------------------------- decoding
int dab_decode_update(const void* new_k, const void* new_v, void* k_exact, void* v_exact, void* k_packed,
                      void* v_packed, int32_t* packed_counts, int32_t* packed_ts, int32_t* packed_lengths,
                      int64_t exact_seq_len, int64_t total_seq_len, float threshold, int64_t exact_window,
                      int dtype, const int64_t* new_strides, const int64_t* exact_strides,
                      const int64_t* pack_strides, const int64_t* pc_strides, int64_t num_heads, int64_t head_dim,
                      int64_t block_d, int use_cosine, int64_t programs, int64_t capacity, int* err_word,
                      void* stream) {
  if (!new_k || !new_v || !k_exact || !v_exact || !k_packed || !v_packed || !packed_counts || !packed_ts ||
      !packed_lengths)
    return fail(1, "dab_decode_update: null pointer");
  if (block_d < head_dim || block_d > 256 || (block_d & (block_d - 1)))
    return fail(1, "dab_decode_update: BLOCK_D must be a power of two in [head_dim, 256]");
  const int bd = block_d < 16 ? 16 : static_cast<int>(block_d);
  return cuda_status(launch_decode_update(dtype, bd, use_cosine != 0, new_k, new_v, k_exact, v_exact, k_packed,
                                          v_packed, packed_counts, packed_ts, packed_lengths, exact_seq_len,
                                          total_seq_len, nullptr, threshold, exact_window, new_strides, exact_strides,
                                          pack_strides, pc_strides, num_heads, head_dim, programs, capacity,
                                          err_word, static_cast<cudaStream_t>(stream)),
                     "decode_update");
}

size_t dab_decode_attention_workspace_size(int64_t batch, int64_t num_q_heads, int64_t capacity,
                                           int64_t exact_len, int64_t head_dim) {
  return decode_attn_workspace(batch, num_q_heads, capacity, exact_len, head_dim);
}

int dab_decode_attention(const void* q, const void* k_packed, const void* v_packed, const int32_t* packed_counts,
                         const int32_t* packed_lengths, const void* k_exact, const void* v_exact, void* out,
                         int dtype, const int64_t* strides, float sm_scale, int64_t exact_len,
                         int64_t num_kv_groups, int64_t batch, int64_t num_q_heads, int64_t head_dim,
                         int64_t capacity, void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k_packed || !v_packed || !packed_counts || !packed_lengths || !k_exact || !v_exact || !out)
    return fail(1, "dab_decode_attention: null pointer");
  if (!strides) return fail(1, "dab_decode_attention: null strides");
  if (num_kv_groups <= 0 || num_q_heads % num_kv_groups) return fail(1, "dab_decode_attention: bad kv groups");
  if (num_kv_groups > 8) return fail(1, "dab_decode_attention: more than 8 q-heads per kv-head");
  if (head_dim > 256) return fail(1, "dab_decode_attention: head_dim > 256");
  const size_t need = decode_attn_workspace(batch, num_q_heads, capacity, exact_len, head_dim);
  if (!workspace || workspace_bytes < need) return fail(1, "dab_decode_attention: workspace too small");
  // strides: q(3) kp(4) vp(4) counts(3) lengths(2) ke(4) ve(4) out(3) = 27 (deltaDecoding.py:244-251)
  const int64_t* s = strides;
  return cuda_status(launch_decode_attn(dtype, q, s + 0, k_packed, s + 3, v_packed, s + 7, packed_counts, s + 11,
                                        packed_lengths, s + 14, k_exact, s + 16, v_exact, s + 20, out, s + 24,
                                        sm_scale, exact_len, nullptr, 0, exact_len, num_kv_groups, batch,
                                        num_q_heads / num_kv_groups, head_dim, capacity,
                                        static_cast<float*>(workspace), static_cast<cudaStream_t>(stream)),
                     "decode_attention");
}

// ---------------------------------------------------- decode with device-resident lengths
// Same kernels as dab_decode_update / dab_decode_attention; the (exact, total) sequence
// lengths are read from device memory instead of host arguments, and dab_decode_advance
// steps them on the device, so a decode step issues no host-side length bookkeeping.
int dab_decode_update_dev(const void* new_k, const void* new_v, void* k_exact, void* v_exact, void* k_packed,
                          void* v_packed, int32_t* packed_counts, int32_t* packed_ts, int32_t* packed_lengths,
                          const int64_t* seq_state, float threshold, int64_t exact_window, int dtype,
                          const int64_t* new_strides, const int64_t* exact_strides, const int64_t* pack_strides,
                          const int64_t* pc_strides, int64_t num_heads, int64_t head_dim, int64_t block_d,
                          int use_cosine, int64_t programs, int64_t capacity, int* err_word, void* stream) {
  if (!seq_state) return fail(1, "dab_decode_update_dev: null seq_state");
  if (!new_k || !new_v || !k_exact || !v_exact || !k_packed || !v_packed || !packed_counts || !packed_ts ||
      !packed_lengths)
    return fail(1, "dab_decode_update_dev: null pointer");
  if (block_d < head_dim || block_d > 256 || (block_d & (block_d - 1)))
    return fail(1, "dab_decode_update_dev: BLOCK_D must be a power of two in [head_dim, 256]");
  const int bd = block_d < 16 ? 16 : static_cast<int>(block_d);
  return cuda_status(launch_decode_update(dtype, bd, use_cosine != 0, new_k, new_v, k_exact, v_exact, k_packed,
                                          v_packed, packed_counts, packed_ts, packed_lengths, 0, 0, seq_state,
                                          threshold, exact_window, new_strides, exact_strides, pack_strides,
                                          pc_strides, num_heads, head_dim, programs, capacity, err_word,
                                          static_cast<cudaStream_t>(stream)),
                     "decode_update_dev");
}

int dab_decode_attention_dev(const void* q, const void* k_packed, const void* v_packed,
                             const int32_t* packed_counts, const int32_t* packed_lengths, const void* k_exact,
                             const void* v_exact, void* out, int dtype, const int64_t* strides, float sm_scale,
                             int64_t* seq_state, int advance, int64_t exact_window, int64_t num_kv_groups,
                             int64_t batch, int64_t num_q_heads, int64_t head_dim, int64_t capacity, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (!seq_state) return fail(1, "dab_decode_attention_dev: null seq_state");
  if (!q || !k_packed || !v_packed || !packed_counts || !packed_lengths || !k_exact || !v_exact || !out)
    return fail(1, "dab_decode_attention_dev: null pointer");
  if (!strides) return fail(1, "dab_decode_attention_dev: null strides");
  if (exact_window <= 0) return fail(1, "dab_decode_attention_dev: exact_window must be positive");
  if (num_kv_groups <= 0 || num_q_heads % num_kv_groups) return fail(1, "dab_decode_attention_dev: bad kv groups");
  if (num_kv_groups > 8) return fail(1, "dab_decode_attention_dev: more than 8 q-heads per kv-head");
  if (head_dim > 256) return fail(1, "dab_decode_attention_dev: head_dim > 256");
  const size_t need = decode_attn_workspace(batch, num_q_heads, capacity, exact_window, head_dim);
  if (!workspace || workspace_bytes < need) return fail(1, "dab_decode_attention_dev: workspace too small");
  const int64_t* s = strides;
  return cuda_status(launch_decode_attn(dtype, q, s + 0, k_packed, s + 3, v_packed, s + 7, packed_counts, s + 11,
                                        packed_lengths, s + 14, k_exact, s + 16, v_exact, s + 20, out, s + 24,
                                        sm_scale, exact_window, seq_state, advance, exact_window, num_kv_groups,
                                        batch, num_q_heads / num_kv_groups, head_dim, capacity,
                                        static_cast<float*>(workspace), static_cast<cudaStream_t>(stream)),
                     "decode_attention_dev");
}

int dab_decode_advance(int64_t* seq_state, int64_t count, void* stream) {
  if (!seq_state && count > 0) return fail(1, "dab_decode_advance: null seq_state");
  return cuda_status(launch_decode_advance(seq_state, count, static_cast<cudaStream_t>(stream)), "decode_advance");
}

// ------------------------------------------------------------------------- native pieces
int dab_rope(const void* x, const int64_t* x_strides, void* y, const int64_t* y_strides, const void* cos_t,
             const void* sin_t, const int64_t* cs_strides, int dtype, int64_t batch, int64_t heads, int64_t seq_len,
             int64_t head_dim, void* stream) {
  if (!x || !y || !cos_t || !sin_t) return fail(1, "dab_rope: null pointer");
  return cuda_status(launch_rope(dtype, x, x_strides, y, y_strides, cos_t, sin_t, cs_strides, batch, heads, seq_len,
                                 head_dim, static_cast<cudaStream_t>(stream)),
                     "rope");
}

int dab_proj_rope(const void* x, int64_t x_row_stride, const void* w, int64_t w_row_stride, const void* cos_t,
                  const void* sin_t, int64_t cs_row_stride, void* out, int64_t out_row_stride, int dtype,
                  int64_t rows, int64_t in_features, int64_t out_features, int64_t head_dim, int64_t rope_lo,
                  int64_t rope_hi, void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !w || !out || !workspace) return fail(1, "dab_proj_rope: null pointer");
  if (dtype != BF16) return fail(1, "dab_proj_rope: bf16 only");
  if (head_dim != 128) return fail(1, "dab_proj_rope: head_dim must be 128");
  if (rows < 1 || in_features < 1 || out_features < 1) return fail(1, "dab_proj_rope: empty problem");
  if (out_features % 128 != 0) return fail(1, "dab_proj_rope: out_features must be a multiple of 128");
  if (rope_lo < 0 || rope_hi < rope_lo || rope_hi > out_features || rope_lo % 128 || rope_hi % 128)
    return fail(1, "dab_proj_rope: RoPE column range must be head-aligned inside [0, out_features]");
  if (rope_hi > rope_lo && (!cos_t || !sin_t)) return fail(1, "dab_proj_rope: RoPE tables missing");
  if (workspace_bytes < WS_HEADER) return fail(1, "dab_proj_rope: workspace smaller than 256 bytes");
  if (rows > INT32_MAX / 2 || in_features > INT32_MAX / 2 || out_features > INT32_MAX / 2)
    return fail(1, "dab_proj_rope: size too large");
  // TMA: 16-byte aligned bases and row strides; the epilogue: 16-byte output and table rows
  if (!aligned16(x) || !aligned16(w) || !aligned16(out) || x_row_stride % 8 || w_row_stride % 8 ||
      out_row_stride % 8 || (rope_hi > rope_lo && (!aligned16(cos_t) || !aligned16(sin_t) || cs_row_stride % 8)))
    return fail(1, "dab_proj_rope: pointers and row strides must be 16-byte aligned");
  ProjParams p{};
  if (!encode_rows(&p.tm_x, x, BF16, in_features, rows, 1, 1, x_row_stride, 0, 0, 128) ||
      !encode_rows(&p.tm_w, w, BF16, in_features, out_features, 1, 1, w_row_stride, 0, 0, 256))
    return fail(1, "dab_proj_rope: tensor map encoding failed (layout not TMA-compatible)");
  p.cos = cos_t;
  p.sin = sin_t;
  p.cs_row = cs_row_stride;
  p.out = out;
  p.os_row = out_row_stride;
  p.err = static_cast<int*>(workspace);
  p.rows = static_cast<int>(rows);
  p.K = static_cast<int>(in_features);
  p.Ho = static_cast<int>(out_features);
  p.rope_lo = static_cast<int>(rope_lo);
  p.rope_hi = static_cast<int>(rope_hi);
  p.n_tiles_n = static_cast<int>((out_features + 255) / 256);
  const int64_t tiles = ((rows + 127) / 128) * p.n_tiles_n;
  if (tiles > INT32_MAX) return fail(1, "dab_proj_rope: too many tiles");
  p.num_tiles = static_cast<int>(tiles);
  return cuda_status(launch_proj_rope(p, num_sms(), static_cast<cudaStream_t>(stream)), "proj_rope");
}

// ------------------------------------------------------------------------- DPXA
int dab_dpxa_compact(const void* x, const int64_t* x_strides, const int32_t* keep_mask, const int64_t* km_strides,
                     void* compact, int32_t* positions, int32_t* counts, int dtype, int64_t batch, int64_t heads,
                     int64_t seq_len, int64_t head_dim, void* stream) {
  if (!x || !x_strides || !keep_mask || !km_strides || !compact || !positions || !counts)
    return fail(1, "dab_dpxa_compact: null pointer");
  if (dtype != BF16 && dtype != F16) return fail(1, "dab_dpxa_compact: bf16 or fp16 only");
  if (head_dim != 64 && head_dim != 128) return fail(1, "dab_dpxa_compact: head_dim must be 64 or 128");
  if (x_strides[3] != 1 || x_strides[2] % 8 || !aligned16(x) || !aligned16(compact))
    return fail(1, "dab_dpxa_compact: rows must be contiguous and 16-byte aligned");
  if (batch * heads > 65535 || seq_len >= (int64_t{1} << 30)) return fail(1, "dab_dpxa_compact: size too large");
  return cuda_status(launch_dpxa_compact(dtype, x, x_strides, keep_mask, km_strides, compact, positions, counts,
                                         static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(seq_len),
                                         static_cast<int>(head_dim), static_cast<cudaStream_t>(stream)),
                     "dpxa_compact");
}

int dab_dpxa_score(const void* q_compact, const int32_t* q_positions, const int32_t* q_counts,
                   const void* k_compact, const int32_t* k_positions, const int32_t* k_counts, float* tile_max,
                   float* tile_sum, float sm_scale, int dtype, int64_t batch, int64_t num_q_heads, int64_t kv_group,
                   int64_t seq_len, int64_t head_dim, void* stream) {
  if (!q_compact || !q_positions || !q_counts || !k_compact || !k_positions || !k_counts || !tile_max || !tile_sum)
    return fail(1, "dab_dpxa_score: null pointer");
  if (dtype != BF16 && dtype != F16) return fail(1, "dab_dpxa_score: bf16 or fp16 only");
  if (head_dim != 64 && head_dim != 128) return fail(1, "dab_dpxa_score: head_dim must be 64 or 128");
  if (kv_group < 1 || num_q_heads % kv_group) return fail(1, "dab_dpxa_score: bad kv_group");
  if (batch * num_q_heads > 65535 || seq_len >= (int64_t{1} << 30)) return fail(1, "dab_dpxa_score: size too large");
  return cuda_status(launch_dpxa_score(dtype, q_compact, q_positions, q_counts, k_compact, k_positions, k_counts,
                                       tile_max, tile_sum, sm_scale, static_cast<int>(batch),
                                       static_cast<int>(num_q_heads), static_cast<int>(kv_group),
                                       static_cast<int>(seq_len), static_cast<int>(head_dim),
                                       static_cast<cudaStream_t>(stream)),
                     "dpxa_score");
}

int dab_dpxa_select(const float* tile_max, const float* tile_sum, uint32_t* selection, float top_p, int64_t batch,
                    int64_t num_kv_heads, int64_t kv_group, int64_t seq_len, void* stream) {
  if (!tile_max || !tile_sum || !selection) return fail(1, "dab_dpxa_select: null pointer");
  if (kv_group < 1 || batch * num_kv_heads > 65535) return fail(1, "dab_dpxa_select: bad sizes");
  if ((seq_len + 127) / 128 > 2048) return fail(1, "dab_dpxa_select: at most 2048 key blocks (256 k tokens)");
  return cuda_status(launch_dpxa_select(tile_max, tile_sum, selection, top_p, static_cast<int>(batch),
                                        static_cast<int>(num_kv_heads), static_cast<int>(kv_group),
                                        static_cast<int>(seq_len), static_cast<cudaStream_t>(stream)),
                     "dpxa_select");
}

int dab_block_sparse_attention(const void* q, const void* k, const void* v, const uint32_t* selection, void* out,
                               int dtype, const int64_t* strides, float sm_scale, int64_t batch, int64_t num_q_heads,
                               int64_t kv_group, int64_t seq_len, int64_t head_dim, void* workspace,
                               size_t workspace_bytes, void* stream) {
  const char* nm = "dab_block_sparse_attention";
  if (!q || !k || !v || !selection || !out || !strides || !workspace) return fail(1, std::string(nm) + ": null pointer");
  if (dtype != BF16 && dtype != F16) return fail(1, std::string(nm) + ": bf16 or fp16 only");
  if (head_dim != 64 && head_dim != 128) return fail(1, std::string(nm) + ": head_dim must be 64 or 128");
  if (kv_group < 1 || num_q_heads % kv_group || batch < 1 || seq_len < 1 || seq_len >= (int64_t{1} << 31))
    return fail(1, std::string(nm) + ": bad sizes");
  if (workspace_bytes < WS_HEADER) return fail(1, std::string(nm) + ": workspace smaller than 256 bytes");
  const int64_t* qs = strides;
  const int64_t* ks = strides + 4;
  const int64_t* vs = strides + 8;
  const int64_t* os = strides + 12;
  if (qs[3] != 1 || ks[3] != 1 || vs[3] != 1 || os[3] != 1 || !aligned16(q) || !aligned16(k) || !aligned16(v))
    return fail(1, std::string(nm) + ": unit head-dim strides and 16-byte aligned rows required");
  const int64_t Hts = num_q_heads / kv_group;
  const int64_t nmb = (seq_len + 127) / 128;
  TcParams p;
  std::memset(&p, 0, sizeof(p));
  bool ok = encode_rows(&p.tm_q, q, dtype, head_dim, seq_len, num_q_heads, batch, qs[2], qs[1], qs[0]);
  ok = ok && encode_rows(&p.tm_kd, k, dtype, head_dim, seq_len, Hts, batch, ks[2], ks[1], ks[0]);
  ok = ok && encode_rows(&p.tm_vd, v, dtype, head_dim, seq_len, Hts, batch, vs[2], vs[1], vs[0]);
  if (!ok) return fail(1, std::string(nm) + ": tensor map encoding failed (layout not TMA-compatible)");
  p.tm_kp = p.tm_kd;
  p.tm_vp = p.tm_vd;
  p.err = static_cast<int*>(workspace);
  p.out = out;
  p.os_b = os[0]; p.os_h = os[1]; p.os_m = os[2];
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.seq_q = static_cast<int>(seq_len); p.seq_k = static_cast<int>(seq_len);
  p.B = static_cast<int>(batch); p.Hq = static_cast<int>(num_q_heads); p.kv_group = static_cast<int>(kv_group);
  p.Hts = static_cast<int>(Hts);
  p.nmb = static_cast<int>(nmb);
  p.variant = 4;  // TC_SPARSE
  p.causal = 1;
  p.pair_heads = (kv_group % 2 == 0) ? 1 : 0;
  p.num_units = static_cast<int>(p.pair_heads ? nmb * batch * Hts * (kv_group / 2) : ((nmb + 1) / 2) * batch * num_q_heads);
  p.out_vec_ok = aligned16(out) && (os[0] * 2) % 16 == 0 && (os[1] * 2) % 16 == 0 && (os[2] * 2) % 16 == 0;
  p.len_dev = reinterpret_cast<const int*>(static_cast<uint8_t*>(workspace) + 4);
  p.sel = selection;
  p.sel_words = static_cast<int>((nmb + 31) / 32);
  return cuda_status(launch_attn_tc(static_cast<int>(head_dim), dtype == BF16, p, num_sms(), static_cast<cudaStream_t>(stream)),
                     nm);
}

int dab_periodic_meta(int32_t* packed_ts, int32_t* packed_counts, float* packed_counts_f32, int64_t batch_heads,
                      int64_t num_packed, int64_t seq_len, int64_t period, void* stream) {
  if (!packed_ts || !packed_counts) return fail(1, "dab_periodic_meta: null pointer");
  if (period < 1) return fail(1, "dab_periodic_meta: period must be >= 1");
  if (num_packed != (seq_len + period - 1) / period) return fail(1, "dab_periodic_meta: num_packed != ceil(N/period)");
  return cuda_status(launch_periodic_meta(packed_ts, packed_counts, packed_counts_f32, batch_heads, num_packed,
                                          seq_len, period,
                                          static_cast<cudaStream_t>(stream)),
                     "periodic_meta");
}

size_t dab_pack_from_keep_workspace_size(int64_t batch, int64_t heads, int64_t seq_len) {
  return pack_from_keep_workspace(batch * heads, seq_len);
}

int dab_pack_from_keep(const int32_t* keep_mask, const int64_t* km_strides, const void* k, const int64_t* k_strides,
                       const void* v, const int64_t* v_strides, void* k_packed, void* v_packed,
                       const int64_t* pack_strides, int32_t* packed_ts, int32_t* packed_counts,
                       const int64_t* meta_strides, int32_t* index_map, int dtype, int64_t batch, int64_t heads,
                       int64_t seq_len, int64_t head_dim, int64_t capacity, int32_t* anchors_per_head,
                       int32_t* max_anchors, void* workspace, size_t workspace_bytes, void* stream) {
  if (!keep_mask || !k || !v || !k_packed || !v_packed || !packed_ts || !packed_counts || !anchors_per_head ||
      !max_anchors)
    return fail(1, "dab_pack_from_keep: null pointer");
  if (workspace_bytes < dab_pack_from_keep_workspace_size(batch, heads, seq_len) || !workspace)
    return fail(1, "dab_pack_from_keep: workspace too small");
  if (k_strides[3] != 1 || v_strides[3] != 1 || pack_strides[3] != 1 || meta_strides[2] != 1)
    return fail(1, "dab_pack_from_keep: innermost strides must be 1");
  if (seq_len >= (int64_t{1} << 30) || capacity >= (int64_t{1} << 31))
    return fail(1, "dab_pack_from_keep: seq_len must be below 2^30 and capacity below 2^31");
  return cuda_status(launch_pack_from_keep(dtype, keep_mask, km_strides, k, k_strides, v, v_strides, k_packed,
                                           v_packed, pack_strides, packed_ts, packed_counts, meta_strides, index_map,
                                           batch, heads, seq_len, head_dim, capacity,
                                           static_cast<uint8_t*>(workspace), anchors_per_head, max_anchors,
                                           static_cast<cudaStream_t>(stream)),
                     "pack_from_keep");
}

size_t dab_delta_compress_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t chunk_size) {
  return key_compress_workspace(batch, heads, seq_len, chunk_size);
}

int dab_delta_compress(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       const void* cos_t, const void* sin_t, const int64_t* cs_strides, void* k_rot,
                       const int64_t* rot_strides, int32_t* keep_mask, const int64_t* km_strides, void* k_packed,
                       void* v_packed, const int64_t* pack_strides, int32_t* packed_ts, int32_t* packed_counts,
                       float* packed_counts_f32, const int64_t* meta_strides, int32_t* anchors_per_head, int dtype,
                       int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, float threshold_sq,
                       int use_cosine, int64_t chunk_size, int64_t capacity, void* workspace,
                       size_t workspace_bytes, void* stream) {
  const char* nm = "dab_delta_compress";
  if (!k || !v || !cos_t || !sin_t || !k_rot || !k_packed || !v_packed || !packed_ts || !packed_counts ||
      !anchors_per_head || !workspace || !k_strides || !v_strides || !cs_strides || !rot_strides || !pack_strides ||
      !meta_strides || (keep_mask && !km_strides))
    return fail(1, std::string(nm) + ": null pointer");
  if (dtype != BF16 && dtype != F16) return fail(1, std::string(nm) + ": keys must be bf16 or fp16");
  if (head_dim != 64 && head_dim != 128) return fail(1, std::string(nm) + ": head_dim must be 64 or 128");
  if (chunk_size < 1 || chunk_size > 1024) return fail(1, std::string(nm) + ": chunk_size must be in [1, 1024]");
  if (batch < 0 || heads < 0 || seq_len < 0 || capacity < 0 || seq_len >= (int64_t{1} << 31) ||
      capacity >= (int64_t{1} << 31))
    return fail(1, std::string(nm) + ": bad sizes");
  if (workspace_bytes < key_compress_workspace(batch, heads, seq_len, chunk_size))
    return fail(1, std::string(nm) + ": workspace too small");
  // 16-byte rows everywhere: unit inner strides, 16-byte aligned bases and row / head / batch strides
  auto ok16 = [](const void* ptr, std::initializer_list<int64_t> strides) {
    if (reinterpret_cast<uintptr_t>(ptr) & 15) return false;
    for (int64_t st : strides)
      if ((st * 2) % 16) return false;
    return true;
  };
  if (k_strides[3] != 1 || v_strides[3] != 1 || cs_strides[2] != 1 || rot_strides[3] != 1 || pack_strides[3] != 1 ||
      meta_strides[2] != 1 || !ok16(k, {k_strides[0], k_strides[1], k_strides[2]}) ||
      !ok16(v, {v_strides[0], v_strides[1], v_strides[2]}) || !ok16(cos_t, {cs_strides[0], cs_strides[1]}) ||
      !ok16(sin_t, {cs_strides[0], cs_strides[1]}) || !ok16(k_rot, {rot_strides[0], rot_strides[1], rot_strides[2]}) ||
      !ok16(k_packed, {pack_strides[0], pack_strides[1], pack_strides[2]}) ||
      !ok16(v_packed, {pack_strides[0], pack_strides[1], pack_strides[2]}))
    return fail(1, std::string(nm) + ": every row must be contiguous and 16-byte aligned");
  const int64_t nch = (seq_len + chunk_size - 1) / chunk_size;
  CompressParams p;
  std::memset(&p, 0, sizeof(p));
  p.k = k; p.ks_b = k_strides[0]; p.ks_h = k_strides[1]; p.ks_s = k_strides[2];
  p.v = v; p.vs_b = v_strides[0]; p.vs_h = v_strides[1]; p.vs_s = v_strides[2];
  p.cos = cos_t; p.sin = sin_t; p.cs_b = cs_strides[0]; p.cs_s = cs_strides[1];
  p.k_rot = k_rot; p.rs_b = rot_strides[0]; p.rs_h = rot_strides[1]; p.rs_s = rot_strides[2];
  p.keep = keep_mask;
  if (keep_mask) { p.km_b = km_strides[0]; p.km_h = km_strides[1]; p.km_s = km_strides[2]; }
  p.kp = k_packed; p.vp = v_packed; p.ps_b = pack_strides[0]; p.ps_h = pack_strides[1]; p.ps_s = pack_strides[2];
  p.ts = packed_ts; p.cnt = packed_counts; p.cnt_f = packed_counts_f32; p.ms_b = meta_strides[0];
  p.ms_h = meta_strides[1];
  p.anchors = anchors_per_head;
  p.ws = static_cast<uint8_t*>(workspace);
  p.thr = threshold_sq;
  p.H = static_cast<int>(heads); p.N = static_cast<int>(seq_len); p.chunk = static_cast<int>(chunk_size);
  p.nch = static_cast<int>(nch); p.cap = static_cast<int>(capacity);
  p.total_chunks = static_cast<unsigned>(batch * heads * nch);
  return cuda_status(launch_key_compress(dtype, static_cast<int>(head_dim), use_cosine != 0, p,
                                         static_cast<cudaStream_t>(stream)),
                     "delta_compress");
}

int64_t dab_nm_num_packed(int64_t seq_len, int64_t n_keep, int64_t m_group, int64_t stride) {
  if (seq_len <= 0 || n_keep <= 0 || m_group <= 0 || stride <= 0) return 0;
  const int64_t G = (seq_len + stride - 1) / stride;
  const int64_t full = G / m_group, rem = G % m_group;
  return full * (n_keep < m_group ? n_keep : m_group) + (rem < n_keep ? rem : n_keep);
}

int dab_nm_select(const void* k, const int64_t* k_strides, int32_t* keep_mask, const int64_t* km_strides, int dtype,
                  int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t n_keep, int64_t m_group,
                  int64_t stride, void* stream) {
  if (!k || !keep_mask) return fail(1, "dab_nm_select: null pointer");
  if (m_group < 1 || m_group > 16 || n_keep < 1 || stride < 1)
    return fail(1, "dab_nm_select: need 1 <= n, 1 <= m <= 16, stride >= 1");
  if (head_dim > 256) return fail(1, "dab_nm_select: head_dim > 256");
  return cuda_status(launch_nm_select(dtype, k, k_strides, keep_mask, km_strides, batch, heads, seq_len, head_dim,
                                      static_cast<int>(n_keep), static_cast<int>(m_group), stride,
                                      static_cast<cudaStream_t>(stream)),
                     "nm_select");
}

}  // extern "C"

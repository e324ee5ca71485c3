// Anchor selection, packing and RoPE kernels (HBM / latency bound integer+byte work).
//
//  * chunked_eval: the delta scan of tritonModules.py:7-69. One 8-lane group owns one
//    chunk and walks it token by token; the squared distance / cosine is reduced in
//    the reference's order (eight strided fp32 accumulators, then a pairwise tree,
//    identical to numpy's summation that the Triton interpreter uses), so keep
//    decisions are bit-exact with the reference.
//  * scatter_pack: parallel_scatter_pack_kv_kernel (tritonModules.py:72-132).
//  * rope: apply_rotary_pos_emb (modeling_llama.py:200-204) with eager rounding.
//  * periodic_meta / keep-mask packing for the native path (modeling_llama.py:626-685
//    without the host sync and without repeat_kv).
#include <type_traits>

#include "common.cuh"
#include "scan.cuh"

namespace dab {

// ---------------------------------------------------------------------------------------
// delta scan
// ---------------------------------------------------------------------------------------
// One step of the delta scan for one 8-lane group: lane g holds elements g, g + 8, ... of the
// current row and of the anchor (two halves of 128 for BD = 256). Returns whether the row is
// kept (a new anchor), computed in the reference's summation order.
template <typename T, int BD, bool COS>
__device__ __forceinline__ bool delta_decide(const float (&cur)[BD > 128 ? 2 : 1][BD / 8 / (BD > 128 ? 2 : 1)],
                                             const float (&ref)[BD > 128 ? 2 : 1][BD / 8 / (BD > 128 ? 2 : 1)],
                                             unsigned gmask, float thr) {
  constexpr int NH = BD > 128 ? 2 : 1;
  constexpr int PER = BD / 8 / NH;
  auto tree = [&](float v) {
    v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 2));
    v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 4));
    return v;
  };
  bool kp;
  if constexpr (COS) {
    float dot = 0.f, cc = 0.f, rr = 0.f;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        const float p0 = __fmul_rn(cur[hh][m], ref[hh][m]);
        const float p1 = __fmul_rn(cur[hh][m], cur[hh][m]);
        const float p2 = __fmul_rn(ref[hh][m], ref[hh][m]);
        a0 = m ? __fadd_rn(a0, p0) : p0;
        a1 = m ? __fadd_rn(a1, p1) : p1;
        a2 = m ? __fadd_rn(a2, p2) : p2;
      }
      a0 = tree(a0);
      a1 = tree(a1);
      a2 = tree(a2);
      dot = hh ? __fadd_rn(dot, a0) : a0;
      cc = hh ? __fadd_rn(cc, a1) : a1;
      rr = hh ? __fadd_rn(rr, a2) : a2;
    }
    const float nc = __fsqrt_rn(__fadd_rn(cc, 1e-8f));
    const float nr = __fsqrt_rn(__fadd_rn(rr, 1e-8f));
    const float cs = __fdiv_rn(dot, __fmul_rn(nc, nr));
    kp = cs < thr;
  } else {
    float tot = 0.f;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        // elementwise ops round to the input dtype (fp32 math, then RNE)
        const float d = round_as<T>(__fsub_rn(cur[hh][m], ref[hh][m]));
        const float sq = round_as<T>(__fmul_rn(d, d));
        acc = m ? __fadd_rn(acc, sq) : sq;
      }
      acc = tree(acc);
      tot = hh ? __fadd_rn(tot, acc) : acc;
    }
    tot = round_as<T>(tot);
    kp = tot > thr;
  }
  return kp;
}

template <typename T, int BD, bool COS>
__global__ void __launch_bounds__(256) chunked_eval_kernel(
    const T* __restrict__ x, int64_t xs_b, int64_t xs_h, int64_t xs_s, int64_t xs_d,
    int32_t* __restrict__ keep, int64_t km_b, int64_t km_h, int64_t km_s,
    int32_t* __restrict__ ccount, int64_t cc_b, int64_t cc_h, int64_t cc_c,
    float thr, int64_t seq_len, int64_t head_dim, int64_t chunk_size, int64_t num_heads,
    int64_t grid_bh, int64_t grid_chunks) {
  constexpr int NH = BD > 128 ? 2 : 1;      // numpy splits n > 128 into two halves
  constexpr int PER = BD / 8 / NH;          // elements per lane per half
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;                   // lane within the 8-lane group
  const unsigned gmask = 0xFFu << (lane & 24);
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 3) + (threadIdx.x >> 3);
  const int64_t bh = blockIdx.y;
  if (chunk >= grid_chunks || bh >= grid_bh) return;
  const int64_t b = static_cast<int>(bh) / static_cast<int>(num_heads), h = bh - b * num_heads;  // bh: a grid index
  const int64_t start = chunk * chunk_size;
  if (start >= seq_len) return;
  const int64_t end = min(start + chunk_size, seq_len);
  const T* row0 = x + b * xs_b + h * xs_h;
  int32_t* krow = keep + b * km_b + h * km_h;

  float ref[NH][PER], cur[NH][PER], nxt[NH][PER];
  auto load = [&](int64_t pos, float (&dst)[NH][PER]) {
    const T* r = row0 + pos * xs_s;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh)
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        const int e = hh * 128 + g + 8 * m;
        dst[hh][m] = (e < head_dim) ? to_f32(r[e * xs_d]) : 0.f;
      }
  };
  load(start, ref);
  if (g == 0) krow[start * km_s] = 1;
  int local = 1;
  if (start + 1 < end) load(start + 1, cur);
  for (int64_t i = start + 1; i < end; ++i) {
    if (i + 1 < end) load(i + 1, nxt);
    const bool kp = delta_decide<T, BD, COS>(cur, ref, gmask, thr);
    if (g == 0) krow[i * km_s] = kp ? 1 : 0;
    if (kp) {
#pragma unroll
      for (int hh = 0; hh < NH; ++hh)
#pragma unroll
        for (int m = 0; m < PER; ++m) ref[hh][m] = cur[hh][m];
      ++local;
    }
#pragma unroll
    for (int hh = 0; hh < NH; ++hh)
#pragma unroll
      for (int m = 0; m < PER; ++m) cur[hh][m] = nxt[hh][m];
  }
  if (g == 0) ccount[b * cc_b + h * cc_h + chunk * cc_c] = local;
}

// The scan with speculative rounds. While no key is kept the anchor stays fixed, so the
// decisions for the next SPEC_W tokens against it are independent of one another: each
// round decides SPEC_W candidates at once and the first kept one (found by ballot) becomes
// the new anchor; the decisions past it are discarded. The serial chain then advances one
// anchor (or SPEC_W rejected tokens) per round instead of one token per step.
//
// One warp owns one chunk (spec_warps chunks per CTA). Lane 4c + q scores candidate c with accumulators 2q and 2q + 1
// of the reference order (elements g, g + 8, ... for accumulator g): their sum is the first
// level of the pairwise tree and two shuffles finish it, so every decision is the one
// delta_decide makes. Rows are staged in a per-warp ring of SPEC_RING rows by 16-byte
// cp.async copies, one commit group per batch of 8 rows, SPEC_LA batches beyond the last
// row a round reads; the anchor is held in registers, so rows behind the scan position are
// free to be overwritten.
template <typename T, int BD, bool COS>
__global__ void __launch_bounds__(spec_warps<T, BD>() * 32) delta_scan_spec_kernel(
    const T* __restrict__ x, int64_t xs_b, int64_t xs_h, int64_t xs_s,
    int32_t* __restrict__ keep, int64_t km_b, int64_t km_h, int64_t km_s,
    int32_t* __restrict__ ccount, int64_t cc_b, int64_t cc_h, int64_t cc_c,
    float thr, int64_t seq_len, int64_t chunk_size, int64_t num_heads, int64_t num_chunks) {
  constexpr int NH = BD > 128 ? 2 : 1;
  constexpr int PER = BD / 8 / NH;
  constexpr int ROWB = BD * static_cast<int>(sizeof(T));  // bytes per row
  constexpr int NCP = ROWB / 16;                           // 16-byte copies per row
  constexpr int PITCH = ROWB + 16;                         // padded pitch: rows 4 banks apart
  extern __shared__ __align__(16) uint8_t spec_smem[];
  const int lane = threadIdx.x & 31;
  uint8_t* ring = spec_smem + (threadIdx.x >> 5) * (SPEC_RING * PITCH);
  const int c = lane >> 2;  // candidate of this lane
  const int q = lane & 3;   // its accumulators: 2q and 2q + 1
  const int64_t chunk = static_cast<int64_t>(blockIdx.x) * spec_warps<T, BD>() + (threadIdx.x >> 5);
  const int64_t bh = blockIdx.y;
  const int64_t b = static_cast<int>(bh) / static_cast<int>(num_heads), h = bh - b * num_heads;  // bh: a grid index
  const int64_t start = chunk * chunk_size;
  if (chunk >= num_chunks || start >= seq_len) return;  // whole warps leave; no CTA-wide barrier follows
  const int n = static_cast<int>(min(chunk_size, seq_len - start));
  const int64_t rstride = xs_s * static_cast<int64_t>(sizeof(T));
  const uint8_t* src0 = reinterpret_cast<const uint8_t*>(x + b * xs_b + h * xs_h) + start * rstride;
  int32_t* krow = keep + b * km_b + h * km_h + start * km_s;
  const int nbatch = (n + 7) >> 3;

  int req = 0;  // next batch to request
  auto top_up = [&](int need) {  // request through batch need + SPEC_LA (empty groups past the end)
    for (; req <= need + SPEC_LA; ++req) {
      if (req < nbatch) {
        for (int k = lane; k < 8 * NCP; k += 32) {
          const int r = 8 * req + k / NCP;
          if (r < n) cp_async16(ring + (r % SPEC_RING) * PITCH + (k % NCP) * 16, src0 + r * rstride + (k % NCP) * 16);
        }
      }
      cp_async_commit();
    }
  };
  float2 an[NH][PER];
  uint32_t aw[NH][PER];
  float rr = 0.f;  // cosine: the anchor's squared norm in the reference order
  auto load_anchor = [&](int r) {
    const uint8_t* row = ring + (r % SPEC_RING) * PITCH;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        if constexpr (!COS && sizeof(T) == 2) {
          aw[hh][m] = *reinterpret_cast<const uint32_t*>(row + (hh * 128 + 2 * q + 8 * m) * 2);
          continue;
        }
        const float2 y = load_pair<T>(row, hh * 128 + 2 * q + 8 * m);
        if constexpr (COS) {
          an[hh][m] = y;
          const float2 pr = fmul2(y, y);
          acc = m ? fadd2(acc, pr) : pr;
        } else {
          an[hh][m] = make_float2(-y.x, -y.y);
        }
      }
      if constexpr (COS) {
        const float v = spec_tree(__fadd_rn(acc.x, acc.y));
        rr = hh ? __fadd_rn(rr, v) : v;
      }
    }
  };

  top_up(0);
  cp_async_wait<SPEC_LA>();
  __syncwarp();
  load_anchor(0);
  if (lane == 0) krow[0] = 1;
  int count = 1;
  int p = 1;  // first undecided row
  while (p < n) {
    const int hi = min(p + SPEC_W - 1, n - 1);
    top_up(hi >> 3);
    cp_async_wait<SPEC_LA>();  // every batch through hi's has landed
    __syncwarp();
    const bool valid = p + c < n;
    const int r = valid ? p + c : n - 1;
    const bool kp = spec_decide<T, BD, COS>(ring + (r % SPEC_RING) * PITCH, an, aw, rr, q, thr);
    const unsigned kb = __ballot_sync(0xFFFFFFFFu, kp && valid) & 0x11111111u;
    const int first = kb ? (__ffs(kb) - 1) >> 2 : SPEC_W;
    if (q == 0 && valid && c <= first) krow[static_cast<int64_t>(p + c) * km_s] = c == first ? 1 : 0;
    if (first < SPEC_W) {
      ++count;
      load_anchor(p + first);
      p += first + 1;
    } else {
      p += SPEC_W;
    }
    __syncwarp();  // every lane is done with the ring before the next top-up refills it
  }
  cp_async_wait<0>();
  if (lane == 0) ccount[b * cc_b + h * cc_h + chunk * cc_c] = count;
}

template <typename T, int BD, bool COS>
static cudaError_t launch_chunked_eval_t(const void* x, const int64_t* xs, int32_t* keep, const int64_t* km,
                                         int32_t* cc, const int64_t* ccs, float thr, int64_t seq_len,
                                         int64_t head_dim, int64_t chunk_size, int64_t num_heads,
                                         int64_t grid_bh, int64_t grid_chunks, cudaStream_t st) {
  const bool staged = head_dim == BD && xs[3] == 1 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                      (xs[0] * static_cast<int64_t>(sizeof(T))) % 16 == 0 &&
                      (xs[1] * static_cast<int64_t>(sizeof(T))) % 16 == 0 &&
                      (xs[2] * static_cast<int64_t>(sizeof(T))) % 16 == 0 && BD * sizeof(T) >= 128;
  if (staged) {
    constexpr int WPC = spec_warps<T, BD>();
    const int smem = WPC * SPEC_RING * (BD * static_cast<int>(sizeof(T)) + 16);
    auto kfn = delta_scan_spec_kernel<T, BD, COS>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
    }
    dim3 g2(static_cast<unsigned>((grid_chunks + WPC - 1) / WPC), static_cast<unsigned>(grid_bh));
    kfn<<<g2, WPC * 32, smem, st>>>(static_cast<const T*>(x), xs[0], xs[1], xs[2], keep, km[0], km[1], km[2],
                                           cc, ccs[0], ccs[1], ccs[2], thr, seq_len, chunk_size, num_heads,
                                           grid_chunks);
    return cudaGetLastError();
  }
  const int groups_per_block = 8;  // 64 threads
  dim3 grid(static_cast<unsigned>((grid_chunks + groups_per_block - 1) / groups_per_block),
            static_cast<unsigned>(grid_bh));
  chunked_eval_kernel<T, BD, COS><<<grid, groups_per_block * 8, 0, st>>>(
      static_cast<const T*>(x), xs[0], xs[1], xs[2], xs[3], keep, km[0], km[1], km[2], cc, ccs[0], ccs[1],
      ccs[2], thr, seq_len, head_dim, chunk_size, num_heads, grid_bh, grid_chunks);
  return cudaGetLastError();
}

template <typename T, bool COS>
static cudaError_t launch_chunked_eval_bd(int bd, const void* x, const int64_t* xs, int32_t* keep,
                                          const int64_t* km, int32_t* cc, const int64_t* ccs, float thr,
                                          int64_t seq_len, int64_t head_dim, int64_t chunk_size,
                                          int64_t num_heads, int64_t grid_bh, int64_t grid_chunks,
                                          cudaStream_t st) {
#define DAB_BD_CASE(N)                                                                                     \
  case N:                                                                                                  \
    return launch_chunked_eval_t<T, N, COS>(x, xs, keep, km, cc, ccs, thr, seq_len, head_dim, chunk_size, \
                                            num_heads, grid_bh, grid_chunks, st);
  switch (bd) {
    DAB_BD_CASE(16)
    DAB_BD_CASE(32)
    DAB_BD_CASE(64)
    DAB_BD_CASE(128)
    DAB_BD_CASE(256)
    default:
      return cudaErrorInvalidValue;
  }
#undef DAB_BD_CASE
}

cudaError_t launch_chunked_eval(int dtype, int bd, bool cosine, const void* x, const int64_t* xs, int32_t* keep,
                                const int64_t* km, int32_t* cc, const int64_t* ccs, float thr, int64_t seq_len,
                                int64_t head_dim, int64_t chunk_size, int64_t num_heads, int64_t grid_bh,
                                int64_t grid_chunks, cudaStream_t st) {
  if (grid_bh <= 0 || grid_chunks <= 0) return cudaSuccess;
  if (grid_bh > 65535) return cudaErrorInvalidValue;
#define DAB_DT(TY)                                                                                           \
  return cosine ? launch_chunked_eval_bd<TY, true>(bd, x, xs, keep, km, cc, ccs, thr, seq_len, head_dim,   \
                                                   chunk_size, num_heads, grid_bh, grid_chunks, st)          \
                : launch_chunked_eval_bd<TY, false>(bd, x, xs, keep, km, cc, ccs, thr, seq_len, head_dim,  \
                                                    chunk_size, num_heads, grid_bh, grid_chunks, st);
  switch (dtype) {
    case F32: DAB_DT(float)
    case F16: DAB_DT(__half)
    case BF16: DAB_DT(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_DT
}

// ---------------------------------------------------------------------------------------
// scatter pack (drop-in): for kept s, Kp[idx[s]] = K[s], Vp[idx[s]] = V[s], ts[idx[s]] = s
// ---------------------------------------------------------------------------------------
constexpr int SP_TPG = 4;  // tokens per 8-lane group in scatter_pack_kernel

template <typename T>
__global__ void __launch_bounds__(256) scatter_pack_kernel(
    const T* __restrict__ k, const int64_t* __restrict__ unused, const T* __restrict__ v, T* __restrict__ kp,
    T* __restrict__ vp, int32_t* __restrict__ ts, const int32_t* __restrict__ km,
    const int32_t* __restrict__ im, int64_t ks_b, int64_t ks_h, int64_t ks_s, int64_t ks_d, int64_t vs_b,
    int64_t vs_h, int64_t vs_s, int64_t vs_d, int64_t kps_b, int64_t kps_h, int64_t kps_a, int64_t kps_d,
    int64_t vps_b, int64_t vps_h, int64_t vps_a, int64_t vps_d, int64_t tss_b, int64_t tss_h, int64_t tss_a,
    int64_t kms_b, int64_t kms_h, int64_t kms_s, int64_t ims_b, int64_t ims_h, int64_t ims_s, int64_t seq_len,
    int64_t head_dim, int64_t num_heads, int64_t rows_covered, int64_t num_packed, bool vec) {
  // SP_TPG consecutive tokens per 8-lane group: their keep flags and index-map entries load
  // together, then every kept row's loads are issued before its stores; rows move as 16-byte
  // pieces (`vec`: unit head-dim strides, 16-byte aligned rows) or element by element
  const int lane8 = threadIdx.x & 7;
  const int64_t s0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 3) + (threadIdx.x >> 3)) * SP_TPG;
  const int64_t bh = blockIdx.y;
  const int64_t lim = seq_len < rows_covered ? seq_len : rows_covered;
  if (s0 >= lim) return;
  const int64_t b = static_cast<int>(bh) / static_cast<int>(num_heads), h = bh - b * num_heads;  // bh: a grid index
  int64_t dst[SP_TPG];
#pragma unroll
  for (int t = 0; t < SP_TPG; ++t) {
    const int64_t s = s0 + t;
    dst[t] = -1;
    if (s < lim) {
      const int32_t kept = km[b * kms_b + h * kms_h + s * kms_s];
      const int64_t d = im[b * ims_b + h * ims_h + s * ims_s];
      // out-of-range destinations are dropped, not written
      if (kept == 1 && d >= 0 && d < num_packed) dst[t] = d;
    }
  }
  if (vec) {
    constexpr int MAXP = 2;  // 16-byte pieces per lane and row (rows up to 256 bytes; wider rows copy by element)
    const int64_t pieces = head_dim * static_cast<int64_t>(sizeof(T)) / 16;
    if (pieces <= 8 * MAXP) {
      uint4 kx[SP_TPG][MAXP], vx[SP_TPG][MAXP];
#pragma unroll
      for (int t = 0; t < SP_TPG; ++t) {
        if (dst[t] < 0) continue;
        const uint4* kr = reinterpret_cast<const uint4*>(k + b * ks_b + h * ks_h + (s0 + t) * ks_s);
        const uint4* vr = reinterpret_cast<const uint4*>(v + b * vs_b + h * vs_h + (s0 + t) * vs_s);
#pragma unroll
        for (int j = 0; j < MAXP; ++j) {
          const int64_t c = lane8 + 8 * j;
          if (c < pieces) {
            kx[t][j] = kr[c];
            vx[t][j] = vr[c];
          }
        }
      }
#pragma unroll
      for (int t = 0; t < SP_TPG; ++t) {
        if (dst[t] < 0) continue;
        uint4* kd = reinterpret_cast<uint4*>(kp + b * kps_b + h * kps_h + dst[t] * kps_a);
        uint4* vd = reinterpret_cast<uint4*>(vp + b * vps_b + h * vps_h + dst[t] * vps_a);
#pragma unroll
        for (int j = 0; j < MAXP; ++j) {
          const int64_t c = lane8 + 8 * j;
          if (c < pieces) {
            kd[c] = kx[t][j];
            vd[c] = vx[t][j];
          }
        }
        if (lane8 == 0) ts[b * tss_b + h * tss_h + dst[t] * tss_a] = static_cast<int32_t>(s0 + t);
      }
      return;
    }
  }
#pragma unroll
  for (int t = 0; t < SP_TPG; ++t) {
    if (dst[t] < 0) continue;
    const int64_t s = s0 + t;
    const T* krow = k + b * ks_b + h * ks_h + s * ks_s;
    const T* vrow = v + b * vs_b + h * vs_h + s * vs_s;
    T* kdst = kp + b * kps_b + h * kps_h + dst[t] * kps_a;
    T* vdst = vp + b * vps_b + h * vps_h + dst[t] * vps_a;
    for (int64_t d = lane8; d < head_dim; d += 8) {
      kdst[d * kps_d] = krow[d * ks_d];
      vdst[d * vps_d] = vrow[d * vs_d];
    }
    if (lane8 == 0) ts[b * tss_b + h * tss_h + dst[t] * tss_a] = static_cast<int32_t>(s);
  }
}


cudaError_t launch_scatter_pack(int dtype, const void* k, const void* v, void* kp, void* vp, int32_t* ts,
                                const int32_t* km, const int32_t* im, const int64_t* ks, const int64_t* vs,
                                const int64_t* kps, const int64_t* vps, const int64_t* tss, const int64_t* kms,
                                const int64_t* ims, int64_t seq_len, int64_t head_dim, int64_t num_heads,
                                int64_t grid_bh, int64_t rows_covered, int64_t num_packed, cudaStream_t st) {
  if (grid_bh <= 0 || rows_covered <= 0 || seq_len <= 0) return cudaSuccess;
  const int64_t rows = rows_covered < seq_len ? rows_covered : seq_len;
  constexpr int64_t per_cta = 32 * SP_TPG;  // 32 eight-lane groups per CTA
  dim3 grid(static_cast<unsigned>((rows + per_cta - 1) / per_cta), static_cast<unsigned>(grid_bh));
  const int64_t esz = dtype == F32 ? 4 : 2;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto rows16 = [&](const int64_t* st3) { return (st3[0] * esz) % 16 == 0 && (st3[1] * esz) % 16 == 0 &&
                                                 (st3[2] * esz) % 16 == 0; };
  const bool vec = ks[3] == 1 && vs[3] == 1 && kps[3] == 1 && vps[3] == 1 && (head_dim * esz) % 16 == 0 &&
                   al16(k) && al16(v) && al16(kp) && al16(vp) && rows16(ks) && rows16(vs) && rows16(kps) &&
                   rows16(vps);
#define DAB_SP(TY)                                                                                           \
  scatter_pack_kernel<TY><<<grid, 256, 0, st>>>(                                                             \
      static_cast<const TY*>(k), nullptr, static_cast<const TY*>(v), static_cast<TY*>(kp),                   \
      static_cast<TY*>(vp), ts, km, im, ks[0], ks[1], ks[2], ks[3], vs[0], vs[1], vs[2], vs[3], kps[0],      \
      kps[1], kps[2], kps[3], vps[0], vps[1], vps[2], vps[3], tss[0], tss[1], tss[2], kms[0], kms[1], kms[2], \
      ims[0], ims[1], ims[2], seq_len, head_dim, num_heads, rows_covered, num_packed, vec);                  \
  return cudaGetLastError();
  switch (dtype) {
    case F32: DAB_SP(float)
    case F16: DAB_SP(__half)
    case BF16: DAB_SP(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_SP
}

// ---------------------------------------------------------------------------------------
// RoPE: out = round(round(x*cos) + round(rotate_half(x)*sin)), eager-torch rounding
// ---------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const T* __restrict__ x, int64_t xb, int64_t xh, int64_t xs,
                                                   int64_t xd, T* __restrict__ y, int64_t yb, int64_t yh,
                                                   int64_t ys, int64_t yd, const T* __restrict__ cs,
                                                   const T* __restrict__ sn, int64_t cb, int64_t cs_s,
                                                   int64_t cd, int64_t H, int64_t N, int64_t D,
                                                   int64_t total_rows) {
  // one thread = one (row, i) pair with i < D/2: produces outputs i and i + D/2
  const int64_t half = D / 2;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total_rows * half) return;
  const int64_t row = idx / half, i = idx % half;
  const int64_t b = row / (H * N), rem = row % (H * N), h = rem / N, s = rem % N;
  const T* xr = x + b * xb + h * xh + s * xs;
  T* yr = y + b * yb + h * yh + s * ys;
  const int64_t c0 = b * cb + s * cs_s;
  const float x1 = to_f32(xr[i * xd]), x2 = to_f32(xr[(i + half) * xd]);
  const float c1 = to_f32(cs[c0 + i * cd]), c2 = to_f32(cs[c0 + (i + half) * cd]);
  const float s1 = to_f32(sn[c0 + i * cd]), s2 = to_f32(sn[c0 + (i + half) * cd]);
  // rotate_half: [-x2, x1]
  const float o1 = round_as<T>(__fadd_rn(round_as<T>(__fmul_rn(x1, c1)), round_as<T>(__fmul_rn(-x2, s1))));
  const float o2 = round_as<T>(__fadd_rn(round_as<T>(__fmul_rn(x2, c2)), round_as<T>(__fmul_rn(x1, s2))));
  yr[i * yd] = from_f32<T>(o1);
  yr[(i + half) * yd] = from_f32<T>(o2);
}

// Contiguous-row RoPE (unit stride along d in x, y and the tables): one thread takes 16 bytes
// of the first half of a row and the matching 16 bytes of the second half, for the same
// position in ROPE_HB heads, with the same per-element rounding sequence as rope_kernel. Its
// cos / sin vectors are loaded once for all those heads, and every head's inputs are
// requested before any is used. Grid: (rows of one head / rows per block, head groups,
// batch), so no index division by runtime sizes.
constexpr int ROPE_HB = 8;  // heads per thread: one cos / sin load serves ROPE_HB rows
template <typename T, int D>
__global__ void __launch_bounds__(256) rope_rows_kernel(const T* __restrict__ x, int64_t xb, int64_t xh, int64_t xs,
                                                        T* __restrict__ y, int64_t yb, int64_t yh, int64_t ys,
                                                        const T* __restrict__ cs, const T* __restrict__ sn,
                                                        int64_t cb, int64_t cs_s, int N, int H) {
  constexpr int V = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte vector
  constexpr int HALF = D / 2;
  constexpr int TPR = HALF / V;                          // threads per row
  constexpr int RPB = 256 / TPR;                         // rows per block
  const int s = blockIdx.x * RPB + static_cast<int>(threadIdx.x) / TPR;
  if (s >= N) return;
  const int i = (static_cast<int>(threadIdx.x) % TPR) * V;
  const int64_t b = blockIdx.z;
  const int h0 = blockIdx.y * ROPE_HB;
  const int nh = (H - h0) < ROPE_HB ? (H - h0) : ROPE_HB;
  const int64_t c0 = b * cb + s * cs_s;
  union Vec { uint4 u; T e[V]; };
  Vec c1, c2, s1, s2;
  c1.u = __ldg(reinterpret_cast<const uint4*>(cs + c0 + i));
  c2.u = __ldg(reinterpret_cast<const uint4*>(cs + c0 + i + HALF));
  s1.u = __ldg(reinterpret_cast<const uint4*>(sn + c0 + i));
  s2.u = __ldg(reinterpret_cast<const uint4*>(sn + c0 + i + HALF));
  // every head's two input vectors are requested before any is used
  Vec x1[ROPE_HB], x2[ROPE_HB];
#pragma unroll
  for (int hh = 0; hh < ROPE_HB; ++hh) {
    if (hh < nh) {
      const T* xr = x + b * xb + (h0 + hh) * xh + s * xs;
      x1[hh].u = *reinterpret_cast<const uint4*>(xr + i);
      x2[hh].u = *reinterpret_cast<const uint4*>(xr + i + HALF);
    }
  }
#pragma unroll
  for (int hh = 0; hh < ROPE_HB; ++hh) {
    if (hh >= nh) continue;
    Vec o1, o2;
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const float a1 = to_f32(x1[hh].e[e]), a2 = to_f32(x2[hh].e[e]);
      o1.e[e] = from_f32<T>(__fadd_rn(round_as<T>(__fmul_rn(a1, to_f32(c1.e[e]))),
                                      round_as<T>(__fmul_rn(-a2, to_f32(s1.e[e])))));
      o2.e[e] = from_f32<T>(__fadd_rn(round_as<T>(__fmul_rn(a2, to_f32(c2.e[e]))),
                                      round_as<T>(__fmul_rn(a1, to_f32(s2.e[e])))));
    }
    T* yr = y + b * yb + (h0 + hh) * yh + s * ys;
    *reinterpret_cast<uint4*>(yr + i) = o1.u;
    *reinterpret_cast<uint4*>(yr + i + HALF) = o2.u;
  }
}

template <typename T, int D>
static bool try_rope_rows(const void* x, const int64_t* xs, void* y, const int64_t* ys, const void* cs, const void* sn,
                          const int64_t* css, int64_t B, int64_t H, int64_t N, cudaStream_t st, cudaError_t* err) {
  constexpr int V = 16 / static_cast<int>(sizeof(T));
  constexpr int RPB = 256 / (D / 2 / V);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (xs[3] != 1 || ys[3] != 1 || css[2] != 1) return false;
  if (!al(x) || !al(y) || !al(cs) || !al(sn)) return false;
  for (int64_t v : {xs[0], xs[1], xs[2], ys[0], ys[1], ys[2], css[0], css[1]})
    if (v % V != 0) return false;
  if (B > 65535 || H > 65535 || N > (int64_t{1} << 30)) return false;
  const dim3 grid(static_cast<unsigned>((N + RPB - 1) / RPB), static_cast<unsigned>((H + ROPE_HB - 1) / ROPE_HB),
                  static_cast<unsigned>(B));
  rope_rows_kernel<T, D><<<grid, 256, 0, st>>>(static_cast<const T*>(x), xs[0], xs[1], xs[2], static_cast<T*>(y), ys[0],
                                               ys[1], ys[2], static_cast<const T*>(cs), static_cast<const T*>(sn),
                                               css[0], css[1], static_cast<int>(N), static_cast<int>(H));
  *err = cudaGetLastError();
  return true;
}

template <typename T>
static bool try_rope_rows_d(const void* x, const int64_t* xs, void* y, const int64_t* ys, const void* cs,
                            const void* sn, const int64_t* css, int64_t B, int64_t H, int64_t N, int64_t D,
                            cudaStream_t st, cudaError_t* err) {
  switch (D) {
    case 64: return try_rope_rows<T, 64>(x, xs, y, ys, cs, sn, css, B, H, N, st, err);
    case 128: return try_rope_rows<T, 128>(x, xs, y, ys, cs, sn, css, B, H, N, st, err);
    case 256: return try_rope_rows<T, 256>(x, xs, y, ys, cs, sn, css, B, H, N, st, err);
    default: return false;
  }
}

cudaError_t launch_rope(int dtype, const void* x, const int64_t* xs, void* y, const int64_t* ys, const void* cs,
                        const void* sn, const int64_t* css, int64_t B, int64_t H, int64_t N, int64_t D,
                        cudaStream_t st) {
  const int64_t rows = B * H * N;
  if (rows == 0) return cudaSuccess;
  if (D % 2) return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  // in-place calls (y == x) are safe on both paths: every element is read and written by one thread
  if (dtype == BF16 && try_rope_rows_d<__nv_bfloat16>(x, xs, y, ys, cs, sn, css, B, H, N, D, st, &e)) return e;
  if (dtype == F16 && try_rope_rows_d<__half>(x, xs, y, ys, cs, sn, css, B, H, N, D, st, &e)) return e;
  if (dtype == F32 && try_rope_rows_d<float>(x, xs, y, ys, cs, sn, css, B, H, N, D, st, &e)) return e;
  const int64_t work = rows * (D / 2);
  const unsigned blocks = static_cast<unsigned>((work + 255) / 256);
#define DAB_RP(TY)                                                                                              \
  rope_kernel<TY><<<blocks, 256, 0, st>>>(static_cast<const TY*>(x), xs[0], xs[1], xs[2], xs[3],               \
                                          static_cast<TY*>(y), ys[0], ys[1], ys[2], ys[3],                     \
                                          static_cast<const TY*>(cs), static_cast<const TY*>(sn), css[0],       \
                                          css[1], css[2], H, N, D, rows);                                       \
  return cudaGetLastError();
  switch (dtype) {
    case F32: DAB_RP(float)
    case F16: DAB_RP(__half)
    case BF16: DAB_RP(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_RP
}

// ---------------------------------------------------------------------------------------
// periodic packing metadata: anchor j sits at j*period and covers min(period, N - j*period)
// tokens (modeling_llama.py:626-632 + :655-685 for keep = t % period == 0)
// ---------------------------------------------------------------------------------------
__global__ void periodic_meta_kernel(int32_t* ts, int32_t* counts, float* counts_f, int64_t BH, int64_t M,
                                     int64_t N, int64_t period) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= BH * M) return;
  const int64_t j = idx % M;
  const int64_t p = j * period;
  const int64_t c = min(period, N - p);
  ts[idx] = static_cast<int32_t>(p);
  counts[idx] = static_cast<int32_t>(c);
  if (counts_f) counts_f[idx] = static_cast<float>(c);
}

cudaError_t launch_periodic_meta(int32_t* ts, int32_t* counts, float* counts_f, int64_t BH, int64_t M, int64_t N,
                                 int64_t period, cudaStream_t st) {
  if (BH * M == 0) return cudaSuccess;
  periodic_meta_kernel<<<static_cast<unsigned>((BH * M + 255) / 256), 256, 0, st>>>(ts, counts, counts_f, BH, M, N,
                                                                                   period);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// device-side packing from a keep mask (native path: no host sync, no repeat_kv), one launch
// (modeling_llama.py:655-685: index_map = cumsum(keep) - 1, the scatter of kept K / V rows and
// timestamps, run-length counts, zero padding up to the packed length).
// One CTA per 1024-token tile of one (batch, head). A CTA takes a ticket (head-major order),
// counts its tile's kept tokens, publishes that count, and finds its packed offset by a
// decoupled look-back over the head's earlier tiles: every tile publishes its own count before
// it waits on anything, and it waits only on tiles with smaller tickets (already running), so
// every wait ends. The run length of a tile's last anchor reaches the first kept token after
// the tile, found by scanning the keep mask forward 32 tokens at a time. The head's last tile
// writes the head's anchor count and zeroes the padding rows up to the capacity; the launch's
// last CTA writes the maximum anchor count, resets the ticket / done counters and advances the
// epoch that tags the status words, so the workspace is cleared once and then reused.
// ---------------------------------------------------------------------------------------
constexpr int PACK_TILE = 1024;    // tokens per tile (one CTA)
constexpr int PACK_THREADS = 256;  // threads per CTA: four consecutive tokens each
constexpr int PACK_HDR = 64;  // workspace header bytes; then one uint64 status word per tile
constexpr int PACK_PADDERS = 128;  // CTAs after the tiles that zero the padding rows

struct PackHdr {
  int err;  // first word: the error word dab_workspace_error reads
  unsigned ticket, done, epoch;
};
enum : int { ERR_PACK_LOOKBACK = 0x401 };  // a predecessor tile never published its count

__device__ __forceinline__ uint64_t pk_ld(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void pk_st(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// status word: epoch (32 bits) | flag (2 bits: 1 = the tile's count, 2 = inclusive prefix) | value
__device__ __forceinline__ uint64_t pk_word(unsigned ep, unsigned flag, unsigned val) {
  return (static_cast<uint64_t>(ep) << 32) | (static_cast<uint64_t>(flag) << 30) | val;
}

template <typename T>
__global__ void __launch_bounds__(PACK_THREADS) keep_pack_kernel(
    const int32_t* __restrict__ keep, int64_t kb, int64_t kh, int64_t ks, const T* __restrict__ k, int64_t xb,
    int64_t xh, int64_t xs, const T* __restrict__ v, int64_t vb, int64_t vh, int64_t vs, T* __restrict__ kp,
    T* __restrict__ vp, int64_t pb, int64_t ph, int64_t ps, int32_t* __restrict__ ts, int32_t* __restrict__ counts,
    int64_t mb, int64_t mh, int32_t* __restrict__ index_map, uint8_t* __restrict__ ws, int32_t* __restrict__ anchors,
    int32_t* __restrict__ max_anchors, int64_t H, int64_t N, int64_t D, int64_t ntile, int64_t capacity, int vec16) {
  constexpr int NW = PACK_THREADS / 32;
  constexpr int TPT = PACK_TILE / PACK_THREADS;  // consecutive tokens per thread
  __shared__ int32_t warp_tot[NW];
  __shared__ int32_t pos_of[PACK_TILE];
  __shared__ int32_t total, s_base, s_next;
  __shared__ unsigned s_ticket, s_ep;
  __shared__ int s_last;
  PackHdr* hdr = reinterpret_cast<PackHdr*>(ws);
  uint64_t* status = reinterpret_cast<uint64_t*>(ws + PACK_HDR);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    s_ticket = atomicAdd(&hdr->ticket, 1u);
    s_ep = *reinterpret_cast<volatile unsigned*>(&hdr->epoch) + 1u;
  }
  __syncthreads();
  const unsigned L = s_ticket, ep = s_ep;
  const int64_t BHt = (static_cast<int64_t>(gridDim.x) - PACK_PADDERS) / ntile;  // batch * heads
  const int nv = vec16 ? static_cast<int>(D * static_cast<int64_t>(sizeof(T)) / 16) : 0;
  if (static_cast<int64_t>(L) >= BHt * ntile) {
    // a padder: once every head's anchor count is out (the inclusive prefix of its last tile,
    // a smaller ticket), zero slice (L - tiles) of each head's padding rows [anchors, capacity)
    const int e = static_cast<int>(static_cast<int64_t>(L) - BHt * ntile);
    for (int64_t bh = 0; bh < BHt; ++bh) {
      if (tid == 0) {
        const uint64_t* sw = status + bh * ntile + ntile - 1;
        uint64_t w = pk_ld(sw);
        if ((w >> 32) != ep || ((w >> 30) & 3u) != 2u) {
          const uint64_t t0 = globaltimer();
          while ((w >> 32) != ep || ((w >> 30) & 3u) != 2u) {
            if (globaltimer() - t0 > DAB_WAIT_TIMEOUT_NS) {
              atomicCAS(&hdr->err, 0, static_cast<int>(ERR_PACK_LOOKBACK));
              w = pk_word(ep, 2u, static_cast<unsigned>(capacity < 0x3FFFFFFF ? capacity : 0x3FFFFFFF));
              break;
            }
            w = pk_ld(sw);
          }
        }
        s_base = static_cast<int32_t>(w & 0x3FFFFFFFu);
      }
      __syncthreads();
      const int64_t A = s_base;
      __syncthreads();
      if (A >= capacity) continue;
      const int64_t b = static_cast<int>(bh) / static_cast<int>(H), h = bh - b * H;
      const int64_t per = (capacity - A + PACK_PADDERS - 1) / PACK_PADDERS;
      const int64_t r0 = A + e * per, r1 = min(capacity, r0 + per);
      for (int64_t jj = r0 + tid; jj < r1; jj += PACK_THREADS) {
        ts[b * mb + h * mh + jj] = 0;
        counts[b * mb + h * mh + jj] = 0;
      }
      if (vec16) {
        for (int64_t i = tid; i < (r1 - r0) * nv; i += PACK_THREADS) {
          const int64_t off = (b * pb + h * ph + (r0 + i / nv) * ps) * static_cast<int64_t>(sizeof(T)) + (i % nv) * 16;
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(kp) + off) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(vp) + off) = make_uint4(0, 0, 0, 0);
        }
      } else {
        for (int64_t i = tid; i < (r1 - r0) * D; i += PACK_THREADS) {
          const int64_t off = b * pb + h * ph + (r0 + i / D) * ps + i % D;
          kp[off] = from_f32<T>(0.f);
          vp[off] = from_f32<T>(0.f);
        }
      }
    }
  } else {
    const int64_t bh = static_cast<int64_t>(L) / ntile, t = static_cast<int64_t>(L) - bh * ntile;
    const int64_t b = static_cast<int>(bh) / static_cast<int>(H), h = bh - b * H;
    const int32_t* krow = keep + b * kb + h * kh;
    // this thread's TPT consecutive tokens, their kept count and the block-wide exclusive scan
    const int64_t s0 = t * PACK_TILE + static_cast<int64_t>(tid) * TPT;
    int kv[TPT];
    int cnt = 0;
#pragma unroll
    for (int e = 0; e < TPT; ++e) {
      kv[e] = (s0 + e < N) ? (krow[(s0 + e) * ks] == 1) : 0;
      cnt += kv[e];
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int v0 = lane < NW ? warp_tot[lane] : 0;
      int wi = v0;
#pragma unroll
      for (int o = 1; o < NW; o <<= 1) {
        const int n = __shfl_up_sync(0xFFFFFFFFu, wi, o);
        if (lane >= o) wi += n;
      }
      if (lane < NW) warp_tot[lane] = wi - v0;  // exclusive offset of warp `lane`
      if (lane == NW - 1) total = wi;
    }
    __syncthreads();
    const int tbase = warp_tot[warp] + incl - cnt;  // kept tokens of the tile before this thread's
    if (warp == 0) {
      // publish this tile's count, then look back over the head's earlier tiles for the offset:
      // the warp reads 32 predecessors' status words at once, waits until each holds at least a
      // count, and adds counts up to the nearest one that holds an inclusive prefix
      if (lane == 0) pk_st(status + L, pk_word(ep, t == 0 ? 2u : 1u, static_cast<unsigned>(total)));
      int32_t base = 0;
      bool found = t == 0;
      for (int64_t i0 = static_cast<int64_t>(L) - 1; !found; i0 -= 32) {
        const int64_t i = i0 - lane;                          // lane l: predecessor i0 - l
        const bool mine = i >= static_cast<int64_t>(L) - t;  // within this head
        uint64_t w = mine ? pk_ld(status + i) : pk_word(ep, 2u, 0u);
        if (mine && ((w >> 32) != ep || ((w >> 30) & 3u) == 0)) {
          const uint64_t t0 = globaltimer();
          while ((w >> 32) != ep || ((w >> 30) & 3u) == 0) {
            if (globaltimer() - t0 > DAB_WAIT_TIMEOUT_NS) {
              atomicCAS(&hdr->err, 0, static_cast<int>(ERR_PACK_LOOKBACK));
              w = pk_word(ep, 2u, 0u);
              break;
            }
            w = pk_ld(status + i);
          }
        }
        const unsigned fl = __ballot_sync(0xFFFFFFFFu, ((w >> 30) & 3u) == 2u);  // lanes past the head count too
        const int stop = __ffs(fl) - 1;  // nearest predecessor with an inclusive prefix (-1: none)
        int32_t vsum = (stop < 0 || lane <= stop) ? static_cast<int32_t>(w & 0x3FFFFFFFu) : 0;
#pragma unroll
        for (int o = 16; o; o >>= 1) vsum += __shfl_xor_sync(0xFFFFFFFFu, vsum, o);
        base += vsum;
        found = stop >= 0;
      }
      if (lane == 0) {
        if (t != 0) pk_st(status + L, pk_word(ep, 2u, static_cast<unsigned>(base + total)));
        s_base = base;
      }
    } else if (warp == 1) {
      // first kept token after the tile (the run length of the tile's last anchor ends there)
      int64_t nf = N;
      for (int64_t q0 = (t + 1) * PACK_TILE; q0 < N; q0 += 32) {
        const int64_t sl = q0 + lane;
        const unsigned bb = __ballot_sync(0xFFFFFFFFu, sl < N && krow[sl * ks] == 1);
        if (bb) {
          nf = q0 + __ffs(bb) - 1;
          break;
        }
      }
      if (lane == 0) s_next = static_cast<int32_t>(nf);
    }
    __syncthreads();
    const int32_t base = s_base;
    int loc = tbase;
#pragma unroll
    for (int e = 0; e < TPT; ++e) {
      const int64_t s = s0 + e;
      if (s < N && index_map) index_map[bh * N + s] = base + loc + kv[e] - 1;  // cumsum(keep) - 1
      if (kv[e]) pos_of[loc++] = static_cast<int32_t>(s);
    }
    __syncthreads();
    const int tot = total;
    int32_t* tsr = ts + b * mb + h * mh;
    int32_t* cnr = counts + b * mb + h * mh;
    for (int i = tid; i < tot; i += PACK_THREADS) {
      const int32_t j = base + i;
      if (j >= capacity) break;
      // run length: distance to the next anchor (or to N after the last one)
      const int32_t sp = pos_of[i];
      const int32_t nxt = (i + 1 < tot) ? pos_of[i + 1] : s_next;
      tsr[j] = sp;
      cnr[j] = nxt - sp;
    }
    if (t == ntile - 1 && tid == 0) anchors[bh] = base + tot;
    if (vec16) {
      // 16-byte rows: the tile's kept rows as (row, 16-byte piece) items, thread i takes items
      // i, i + PACK_THREADS, ...; four items' loads are issued before their stores
      const int items = tot * nv;
      const T* kh0 = k + b * xb + h * xh;
      const T* vh0 = v + b * vb + h * vh;
      uint8_t* kd0 = reinterpret_cast<uint8_t*>(kp + b * pb + h * ph);
      uint8_t* vd0 = reinterpret_cast<uint8_t*>(vp + b * pb + h * ph);
      for (int i0 = tid; i0 < items; i0 += 4 * PACK_THREADS) {
        uint4 kr4[4], vr4[4];
        int64_t dst[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int idx = i0 + u * PACK_THREADS;
          dst[u] = -1;
          if (idx < items) {
            const int r = idx / nv, c = idx % nv;
            const int32_t jj = base + r;
            if (jj < capacity) {
              const int64_t ss = pos_of[r];
              kr4[u] = *(reinterpret_cast<const uint4*>(kh0 + ss * xs) + c);
              vr4[u] = *(reinterpret_cast<const uint4*>(vh0 + ss * vs) + c);
              dst[u] = static_cast<int64_t>(jj) * ps * static_cast<int64_t>(sizeof(T)) + c * 16;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (dst[u] < 0) continue;
          *reinterpret_cast<uint4*>(kd0 + dst[u]) = kr4[u];
          *reinterpret_cast<uint4*>(vd0 + dst[u]) = vr4[u];
        }
      }
    } else {
      // element copies: warp w takes kept rows w, w + NW, ...
      for (int r = warp; r < tot; r += NW) {
        const int32_t jj = base + r;
        if (jj >= capacity) break;
        const int64_t ss = pos_of[r];
        const T* kr = k + b * xb + h * xh + ss * xs;
        const T* vr = v + b * vb + h * vh + ss * vs;
        T* kd = kp + b * pb + h * ph + static_cast<int64_t>(jj) * ps;
        T* vd = vp + b * pb + h * ph + static_cast<int64_t>(jj) * ps;
        for (int64_t d = lane; d < D; d += 32) {
          kd[d] = kr[d];
          vd[d] = vr[d];
        }
      }
    }
  }  // tile CTAs
  // the launch's last CTA: the maximum anchor count, then the counters for the next launch
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned d = atomicAdd(&hdr->done, 1u);
    s_last = d == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    int32_t mx = 0;
    for (int64_t i = tid; i < BHt; i += PACK_THREADS) mx = max(mx, *reinterpret_cast<volatile int32_t*>(anchors + i));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if (lane == 0) warp_tot[warp] = mx;
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < NW; ++w) mx = max(mx, warp_tot[w]);
      *max_anchors = mx;
      hdr->ticket = 0u;
      hdr->done = 0u;
      hdr->epoch = ep;
      __threadfence();
    }
  }
}

size_t pack_from_keep_workspace(int64_t BH, int64_t N) {
  const int64_t ntile = (N + PACK_TILE - 1) / PACK_TILE;
  return static_cast<size_t>(PACK_HDR + 8 * (BH > 0 ? BH : 1) * (ntile > 0 ? ntile : 1));
}

cudaError_t launch_pack_from_keep(int dtype, const int32_t* keep, const int64_t* kms, const void* k,
                                  const int64_t* xs, const void* v, const int64_t* vs, void* kp, void* vp,
                                  const int64_t* ps, int32_t* ts, int32_t* counts, const int64_t* ms,
                                  int32_t* index_map, int64_t B, int64_t H, int64_t N, int64_t D,
                                  int64_t capacity, uint8_t* ws, int32_t* anchors, int32_t* max_anchors,
                                  cudaStream_t st) {
  const int64_t ntile = (N + PACK_TILE - 1) / PACK_TILE;
  const int64_t BH = B * H;
  if (BH == 0 || N == 0) return cudaSuccess;
  if (BH * ntile + PACK_PADDERS > (int64_t{1} << 31) - 1) return cudaErrorInvalidValue;
  const size_t es = dtype == F32 ? 4 : 2;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const int vec16 = al16(k) && al16(v) && al16(kp) && al16(vp) && (D * es) % 16 == 0 &&
                    ((xs[0] | xs[1] | xs[2] | vs[0] | vs[1] | vs[2] | ps[0] | ps[1] | ps[2]) * es) % 16 == 0;
  const unsigned grid = static_cast<unsigned>(BH * ntile + PACK_PADDERS);
#define DAB_KP(TY)                                                                                               \
  keep_pack_kernel<TY><<<grid, PACK_THREADS, 0, st>>>(                                                              \
      keep, kms[0], kms[1], kms[2], static_cast<const TY*>(k), xs[0], xs[1], xs[2],                             \
      static_cast<const TY*>(v), vs[0], vs[1], vs[2], static_cast<TY*>(kp), static_cast<TY*>(vp), ps[0],         \
      ps[1], ps[2], ts, counts, ms[0], ms[1], index_map, ws, anchors, max_anchors, H, N, D, ntile, capacity,     \
      vec16);                                                                                                    \
  return cudaGetLastError();
  switch (dtype) {
    case F32: DAB_KP(float)
    case F16: DAB_KP(__half)
    case BF16: DAB_KP(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_KP
}

// ---------------------------------------------------------------------------------------
// N:M structured selection (builder-specified: the reference ships no source for it).
// Candidates are positions t = i*c; candidate i scores +inf (i == 0) or the fp32 squared
// distance between K[t] and K[t-c] (numpy summation order). Each run of m consecutive
// candidates keeps its min(n, size) best (ties to the earlier position). One thread owns
// one group and writes the keep mask of every position the group spans.
// ---------------------------------------------------------------------------------------
template <typename T, int BD>
__global__ void __launch_bounds__(128) nm_select_kernel(const T* __restrict__ x, int64_t xb, int64_t xh, int64_t xs,
                                                        int64_t xd, int32_t* __restrict__ keep, int64_t kb,
                                                        int64_t kh, int64_t ks, int64_t H, int64_t N, int64_t D,
                                                        int n_keep, int m_group, int64_t c, int64_t groups) {
  constexpr int NH = BD > 128 ? 2 : 1;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t bh = blockIdx.y;
  if (gid >= groups) return;
  const int64_t b = static_cast<int>(bh) / static_cast<int>(H), h = bh - b * H;  // bh: a grid index
  const T* base = x + b * xb + h * xh;
  int32_t* kr = keep + b * kb + h * kh;
  const int64_t G = (N + c - 1) / c;  // candidates
  const int64_t i0 = gid * m_group;
  const int64_t left = G - i0;
  const int size = static_cast<int>(left < m_group ? left : m_group);
  float sc[16];
  for (int a = 0; a < size; ++a) {
    const int64_t i = i0 + a;
    if (i == 0) { sc[a] = INFINITY; continue; }
    const T* r1 = base + i * c * xs;
    const T* r0 = base + (i * c - c) * xs;
    float tot = 0.f;
    for (int hh = 0; hh < NH; ++hh) {
      float r[8];
      for (int k = 0; k < 8; ++k) {
        float acc = 0.f;
        for (int mm = 0; mm < BD / 8 / NH; ++mm) {
          const int e = hh * 128 + k + 8 * mm;
          const float d = (e < D) ? __fsub_rn(to_f32(r1[e * xd]), to_f32(r0[e * xd])) : 0.f;
          const float sq = __fmul_rn(d, d);
          acc = mm ? __fadd_rn(acc, sq) : sq;
        }
        r[k] = acc;
      }
      const float t = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                                __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
      tot = hh ? __fadd_rn(tot, t) : t;
    }
    sc[a] = tot;
  }
  const int nk = min(n_keep, size);
  const int64_t p0 = i0 * c;
  const int64_t p1e = (i0 + size) * c;
  const int64_t p1 = p1e < N ? p1e : N;
  for (int64_t p = p0; p < p1; ++p) kr[p * ks] = 0;
  for (int a = 0; a < size; ++a) {
    int rank = 0;
    for (int o = 0; o < size; ++o) rank += (sc[o] > sc[a]) || (sc[o] == sc[a] && o < a);
    if (rank < nk) kr[(i0 + a) * c * ks] = 1;
  }
}

// The same selection with candidate rows staged in shared memory. A CTA scores the candidates
// of NM_CAND_MAX / m whole groups of one (batch, head): their rows and the row of the candidate
// before them arrive by coalesced 16-byte cp.async copies, four lanes score each candidate (lane q holds
// accumulators 2q and 2q + 1 of the eight strided fp32 accumulators; their sum is the first
// level of the pairwise tree, two shuffles finish it), then one thread per group ranks it and
// the keep mask of every position the groups cover is written by consecutive threads. Used
// when the head dimension is the power of two BD with unit stride and rows start on 16-byte
// boundaries; the scores are the ones nm_select_kernel computes.
constexpr int NM_CAND_MAX = 64;  // candidates per CTA (whole groups)

template <typename T, int BD>
__global__ void __launch_bounds__(128) nm_select_staged_kernel(const T* __restrict__ x, int64_t xb, int64_t xh,
                                                               int64_t xs, int32_t* __restrict__ keep, int64_t kb,
                                                               int64_t kh, int64_t ks, int64_t H, int64_t N,
                                                               int n_keep, int m_group, int64_t c, int64_t groups) {
  constexpr int NH = BD > 128 ? 2 : 1;
  constexpr int PER = BD / 8 / NH;
  constexpr int ROWB = BD * static_cast<int>(sizeof(T));
  constexpr int NCP = ROWB / 16;
  constexpr int PITCH = ROWB + 16;
  extern __shared__ __align__(16) uint8_t nm_smem[];
  float* sc = reinterpret_cast<float*>(nm_smem);                 // scores of this CTA's candidates
  uint8_t* rows = nm_smem + NM_CAND_MAX * sizeof(float);         // row r holds candidate i0 - 1 + r
  const int gpc = NM_CAND_MAX / m_group;                         // groups per CTA
  const int64_t g0 = static_cast<int64_t>(blockIdx.x) * gpc;
  const int64_t bh = blockIdx.y;
  if (g0 >= groups) return;
  const int64_t b = static_cast<int>(bh) / static_cast<int>(H), h = bh - b * H;  // bh: a grid index
  const int64_t G = (N + c - 1) / c;  // candidates of the head
  const int64_t i0 = g0 * m_group;
  const int cn = static_cast<int>(min(static_cast<int64_t>(gpc) * m_group, G - i0));  // candidates here
  const uint8_t* base = reinterpret_cast<const uint8_t*>(x + b * xb + h * xh);
  const int64_t cstride = c * xs * static_cast<int64_t>(sizeof(T));  // bytes between candidates
  // stage candidates i0 - 1 .. i0 + cn - 1 (row 0 stays unused when i0 == 0); every copy in
  // flight at once
  for (int j = threadIdx.x; j < (cn + 1) * NCP; j += blockDim.x) {
    const int r = j / NCP, k = j % NCP;
    const int64_t i = i0 - 1 + r;
    if (i >= 0) cp_async16(rows + r * PITCH + k * 16, base + i * cstride + k * 16);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int q = threadIdx.x & 3;
  for (int a = threadIdx.x >> 2; a < ((cn + 7) & ~7); a += blockDim.x >> 2) {  // whole warps iterate together
    const int ra = a < cn ? a : cn - 1;
    const uint8_t* r1 = rows + (ra + 1) * PITCH;
    const uint8_t* r0 = rows + ra * PITCH;
    float tot = 0.f;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        const int e = hh * 128 + 2 * q + 8 * m;
        const float2 d = fadd2(load_pair<T>(r1, e), fneg2(load_pair<T>(r0, e)));
        const float2 sq = fmul2(d, d);
        acc = m ? fadd2(acc, sq) : sq;
      }
      const float t = spec_tree(__fadd_rn(acc.x, acc.y));
      tot = hh ? __fadd_rn(tot, t) : t;
    }
    if (q == 0 && a < cn) sc[a] = (i0 + a == 0) ? INFINITY : tot;
  }
  __syncthreads();
  // rank each group (one thread per group); the keep bits go to the row area, no longer read
  int32_t* kept = reinterpret_cast<int32_t*>(rows);
  const int ng = (cn + m_group - 1) / m_group;
  for (int gi = threadIdx.x; gi < ng; gi += blockDim.x) {
    const int a0 = gi * m_group;
    const int size = min(m_group, cn - a0);
    const int nk = min(n_keep, size);
    for (int a = 0; a < size; ++a) {
      int rank = 0;
      for (int o = 0; o < size; ++o)
        rank += (sc[a0 + o] > sc[a0 + a]) || (sc[a0 + o] == sc[a0 + a] && o < a);
      kept[a0 + a] = rank < nk ? 1 : 0;
    }
  }
  __syncthreads();
  int32_t* kr = keep + b * kb + h * kh;
  const int64_t p0 = i0 * c;
  const int64_t p1 = min((i0 + cn) * c, N);
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const int64_t off = p - p0;
    kr[p * ks] = (off % c == 0) ? kept[off / c] : 0;
  }
}

cudaError_t launch_nm_select(int dtype, const void* x, const int64_t* xs, int32_t* keep, const int64_t* kms,
                             int64_t B, int64_t H, int64_t N, int64_t D, int n_keep, int m_group, int64_t c,
                             cudaStream_t st) {
  if (B * H == 0 || N == 0) return cudaSuccess;
  if (m_group < 1 || m_group > 16 || n_keep < 1 || c < 1) return cudaErrorInvalidValue;
  int bd = 16;
  while (bd < D) bd <<= 1;
  if (bd > 256) return cudaErrorInvalidValue;
  const int64_t G = (N + c - 1) / c;
  const int64_t groups = (G + m_group - 1) / m_group;
  if (B * H > 65535) return cudaErrorInvalidValue;
  const int esz = dtype == F32 ? 4 : 2;
  const bool staged = D == bd && xs[3] == 1 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                      (xs[0] * esz) % 16 == 0 && (xs[1] * esz) % 16 == 0 && (xs[2] * esz) % 16 == 0;
  dim3 grid(static_cast<unsigned>((groups + 127) / 128), static_cast<unsigned>(B * H));
  const int gpc = NM_CAND_MAX / m_group;
  dim3 sgrid(static_cast<unsigned>((groups + gpc - 1) / gpc), static_cast<unsigned>(B * H));
  const int smem = NM_CAND_MAX * 4 + (NM_CAND_MAX + 1) * (bd * esz + 16);
#define DAB_NM(TY, BDV)                                                                                      \
  if (staged) {                                                                                              \
    auto kfn = nm_select_staged_kernel<TY, BDV>;                                                             \
    if (smem > 48 * 1024) {                                                                                  \
      cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);          \
      if (e != cudaSuccess) return e;                                                                        \
    }                                                                                                        \
    kfn<<<sgrid, 128, smem, st>>>(static_cast<const TY*>(x), xs[0], xs[1], xs[2], keep, kms[0], kms[1],     \
                                  kms[2], H, N, n_keep, m_group, c, groups);                                 \
    return cudaGetLastError();                                                                               \
  }                                                                                                          \
  nm_select_kernel<TY, BDV><<<grid, 128, 0, st>>>(static_cast<const TY*>(x), xs[0], xs[1], xs[2], xs[3], keep, \
                                                  kms[0], kms[1], kms[2], H, N, D, n_keep, m_group, c, groups); \
  return cudaGetLastError();
#define DAB_NM_BD(TY)                                                                                 \
  switch (bd) {                                                                                       \
    case 16: DAB_NM(TY, 16)                                                                           \
    case 32: DAB_NM(TY, 32)                                                                           \
    case 64: DAB_NM(TY, 64)                                                                           \
    case 128: DAB_NM(TY, 128)                                                                         \
    default: DAB_NM(TY, 256)                                                                          \
  }
  switch (dtype) {
    case F32: DAB_NM_BD(float)
    case F16: DAB_NM_BD(__half)
    case BF16: DAB_NM_BD(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_NM
#undef DAB_NM_BD
}

}  // namespace dab

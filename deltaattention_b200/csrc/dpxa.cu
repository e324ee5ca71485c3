// DPXA: delta-based tile scoring for block-sparse prefill (Paper/src/methodology.tex:89-135).
//
// The paper gives the method without code; the library implements this specification:
//   1. compaction: the Stage-1 delta selection (chunked_eval_kernel's rule with chunk = 128,
//      Euclidean, squared threshold) on every 128-token block of post-RoPE Q and K picks each
//      block's anchors; `dpxa_compact_kernel` gathers them to the front of the block;
//   2-3. scoring: `dpxa_score_kernel` multiplies each query block's anchors by the anchors of
//      every key block j <= i of its kv-head (mma.sync m16n8k16, fp32 accumulation), masks the
//      diagonal tile causally by anchor position, and keeps per tile (max S, sum exp(S - max));
//   4. selection: `dpxa_select_kernel` turns each q-head's tile statistics into the sampled
//      attention mass of each tile, averages the q-heads of a GQA group, sorts the tiles by
//      weight (ties to the lower block), takes them until the cumulative weight exceeds p and
//      always takes the diagonal: a bitmask per (batch, kv-head, query block);
//   5. attention: the tcgen05 attention kernel walks only the selected key blocks.
#include <type_traits>

#include "params.cuh"

namespace dab {

constexpr int DPX_B = 128;  // block (tile) size in tokens

__device__ __forceinline__ void dpx_cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void dpx_ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
template <typename T>
__device__ __forceinline__ void dpx_mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// ------------------------------------------------------------------ 1. compaction
// One CTA of 128 threads per (block, batch * head): the block's kept rows (keep mask from the
// delta scan with chunk 128) go to rows 0..cnt-1 of the block's slot in `cx` [BH][nb][128][D]
// (16-byte pieces), their positions to `cpos` [BH][nb][128], the count to `ccnt` [BH][nb].
template <typename T>
__global__ void __launch_bounds__(DPX_B) dpxa_compact_kernel(const T* __restrict__ x, int64_t xb, int64_t xh,
                                                             int64_t xs, const int32_t* __restrict__ keep,
                                                             int64_t kb, int64_t kh, int64_t ks, T* __restrict__ cx,
                                                             int32_t* __restrict__ cpos, int32_t* __restrict__ ccnt,
                                                             int H, int N, int D, int nb) {
  __shared__ int32_t wofs[DPX_B / 32];
  __shared__ int32_t pos[DPX_B];
  __shared__ int32_t total;
  const int blk = blockIdx.x, bh = blockIdx.y;
  const int b = bh / H, h = bh - b * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int s = blk * DPX_B + tid;
  const int kv = s < N ? (keep[b * kb + h * kh + static_cast<int64_t>(s) * ks] == 1) : 0;
  const unsigned bal = __ballot_sync(0xFFFFFFFFu, kv);
  if (lane == 0) wofs[warp] = __popc(bal);
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int w = 0; w < DPX_B / 32; ++w) {
      const int c = wofs[w];
      wofs[w] = run;
      run += c;
    }
    total = run;
  }
  __syncthreads();
  const int loc = wofs[warp] + __popc(bal & ((1u << lane) - 1));
  if (kv) pos[loc] = s;
  __syncthreads();
  const int64_t slot = static_cast<int64_t>(bh) * nb + blk;
  const int cnt = total;
  if (tid == 0) ccnt[slot] = cnt;
  cpos[slot * DPX_B + tid] = tid < cnt ? pos[tid] : 0;
  const int nv = D * static_cast<int>(sizeof(T)) / 16;
  const T* xr = x + b * xb + h * xh;
  uint8_t* dst = reinterpret_cast<uint8_t*>(cx + slot * DPX_B * D);
  for (int i = tid; i < cnt * nv; i += DPX_B) {
    const int r = i / nv, c = i - (i / nv) * nv;
    const uint4 val = *(reinterpret_cast<const uint4*>(xr + static_cast<int64_t>(pos[r]) * xs) + c);
    *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * D * sizeof(T) + c * 16) = val;
  }
}

// ------------------------------------------------------------------ 2-3. scoring
// One CTA of 8 warps per (query block i, batch * q-head). The query block's anchors sit in
// shared memory; warp w scores key blocks w, w+8, ... <= i on its own: it streams the block's
// anchors through a two-slot ring of 16-row chunks (cp.async, the next chunk loading while
// this one is multiplied), computes S for every 16-row tile of query anchors against the
// chunk (mma.sync m16n8k16, fp32; the chunk's key fragments held in registers and two query
// tiles multiplied per pass, four accumulator chains in flight), folds the scores into a
// running (max, sum exp(S - max)) and writes tile (i, j) after a warp reduction: no CTA-wide
// barrier per tile.
constexpr int DPX_KC = 16;  // key anchors per chunk
constexpr int DPX_SW = 8;   // warps per scoring CTA
template <typename T, int D>
__global__ void __launch_bounds__(DPX_SW * 32) dpxa_score_kernel(const T* __restrict__ cq, const int32_t* __restrict__ qpos,
                                                         const int32_t* __restrict__ qcnt, const T* __restrict__ ck,
                                                         const int32_t* __restrict__ kpos,
                                                         const int32_t* __restrict__ kcnt, float* __restrict__ tmax,
                                                         float* __restrict__ tsum, float sm_scale, int Hq, int G,
                                                         int nb) {
  constexpr int ROWB = D * 2, SEGS = D / 8;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* Qs = dsm;                                             // [128][D] swizzled 16-byte segments
  int32_t* qp = reinterpret_cast<int32_t*>(Qs + DPX_B * ROWB);   // [128]
  uint8_t* Kw = reinterpret_cast<uint8_t*>(qp + DPX_B);          // [warps][2 slots][DPX_KC][D]
  const int i = blockIdx.x, bq = blockIdx.y;
  const int b = bq / Hq, h = bq - b * Hq, hk = h / G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t qslot = static_cast<int64_t>(bq) * nb + i;
  const int64_t kbase = (static_cast<int64_t>(b) * (Hq / G) + hk) * nb;
  const int nq = qcnt[qslot];
  const int mtiles = (nq + 15) / 16;
  for (int e = tid; e < mtiles * 16 * SEGS; e += DPX_SW * 32) {
    const int r = e / SEGS, sg = e - (e / SEGS) * SEGS;
    dpx_cp16(smem_u32(Qs + r * ROWB + ((sg ^ (r & 7)) << 4)),
             cq + (qslot * DPX_B + (r < nq ? r : 0)) * D + sg * 8, r < nq);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (tid < DPX_B) qp[tid] = qpos[qslot * DPX_B + tid];
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  uint8_t* kring = Kw + warp * 2 * DPX_KC * ROWB;
  const int g = lane >> 2, c2 = (lane & 3) * 2;
  const float sl2 = sm_scale * 1.4426950408889634f;  // scores in log2 units
  // the warp's chunk `c` of key block j into ring slot `slot` (rows >= n zero)
  auto load_chunk = [&](int j, int c, int n, int slot) {
    const T* src = ck + ((kbase + j) * DPX_B + c * DPX_KC) * D;
    uint8_t* dst = kring + slot * DPX_KC * ROWB;
#pragma unroll 4
    for (int e = lane; e < DPX_KC * SEGS; e += 32) {
      const int r = e / SEGS, sg = e - (e / SEGS) * SEGS;
      const bool ok = c * DPX_KC + r < n;
      dpx_cp16(smem_u32(dst + r * ROWB + ((sg ^ (r & 7)) << 4)), src + static_cast<int64_t>(ok ? r : 0) * D + sg * 8, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int j = warp; j <= i; j += DPX_SW) {
    const int nk = kcnt[kbase + j];
    const int nch = (nk + DPX_KC - 1) / DPX_KC;
    const int32_t* kpj = kpos + (kbase + j) * DPX_B;
    float m = -INFINITY, sacc = 0.f;
    if (nch > 0) load_chunk(j, 0, nk, 0);
    for (int c = 0; c < nch; ++c) {
      if (c + 1 < nch) {
        load_chunk(j, c + 1, nk, (c + 1) & 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      __syncwarp();
      const uint8_t* Kb = kring + (c & 1) * DPX_KC * ROWB;
      const int nt_n = min(DPX_KC, nk - c * DPX_KC);  // valid key rows of the chunk
      const bool diag = j == i;
      // the chunk's B fragments (16 keys x D) in registers once, reused by every query tile
      uint32_t bf[D / 32][DPX_KC / 8][4];
#pragma unroll
      for (int kp2 = 0; kp2 < D / 32; ++kp2)
#pragma unroll
        for (int nt = 0; nt < DPX_KC / 8; ++nt) {
          const int r = nt * 8 + (lane & 7);
          const int sg = 4 * kp2 + (lane >> 3);
          dpx_ldsm_x4(bf[kp2][nt], smem_u32(Kb + r * ROWB + ((sg ^ (r & 7)) << 4)));
        }
      for (int mt0 = 0; mt0 < mtiles; mt0 += 2) {
        // S of two 16-row query tiles against the chunk's two 8-key tiles: four independent
        // mma chains in flight (the second tile only when it exists; warp-uniform)
        const bool two = mt0 + 1 < mtiles;
        float acc[2][DPX_KC / 8][4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int nt = 0; nt < DPX_KC / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[t][nt][e] = 0.f;
#pragma unroll
        for (int kp2 = 0; kp2 < D / 32; ++kp2) {
          const int sg0 = (2 * kp2) * 2 + (lane >> 4), sg1 = (2 * kp2 + 1) * 2 + (lane >> 4);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (t == 1 && !two) continue;
            uint32_t a0[4], a1[4];
            const int r = (mt0 + t) * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            dpx_ldsm_x4(a0, smem_u32(Qs + r * ROWB + ((sg0 ^ (r & 7)) << 4)));
            dpx_ldsm_x4(a1, smem_u32(Qs + r * ROWB + ((sg1 ^ (r & 7)) << 4)));
#pragma unroll
            for (int nt = 0; nt < DPX_KC / 8; ++nt) {
              dpx_mma<T>(acc[t][nt], a0, bf[kp2][nt][0], bf[kp2][nt][1]);
              dpx_mma<T>(acc[t][nt], a1, bf[kp2][nt][2], bf[kp2][nt][3]);
            }
          }
        }
        // fold the tiles' scores into (m, sum 2^(S' - m)), S' = S * scale * log2(e): the maximum
        // is taken on the raw accumulators and scaled once, each probability is one FMA and one
        // ex2; masks only where a tile crosses the anchor counts or the diagonal
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (t == 1 && !two) continue;
          const int mt = mt0 + t;
          const bool full_rows = mt * 16 + 16 <= nq;
#pragma unroll
          for (int nt = 0; nt < DPX_KC / 8; ++nt) {
            float x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = acc[t][nt][e];
            const bool full = full_rows && nt * 8 + 8 <= nt_n && !diag;
            if (!full) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int row = mt * 16 + g + (e >> 1) * 8, col = nt * 8 + c2 + (e & 1);
                bool ok = row < nq && col < nt_n;
                if (ok && diag) ok = kpj[c * DPX_KC + col] <= qp[row];
                if (!ok) x[e] = -INFINITY;
              }
            }
            const float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])) * sl2;
            if (mx > m) {
              sacc *= ex2(m - mx);
              m = mx;
            }
            if (m != -INFINITY)
              sacc += (ex2(fmaf(x[0], sl2, -m)) + ex2(fmaf(x[1], sl2, -m))) +
                      (ex2(fmaf(x[2], sl2, -m)) + ex2(fmaf(x[3], sl2, -m)));
          }
        }
      }
      __syncwarp();  // every lane is done with this slot before it is refilled
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xFFFFFFFFu, m, o), s2 = __shfl_xor_sync(0xFFFFFFFFu, sacc, o);
      const float mm = fmaxf(m, m2);
      sacc = (mm == -INFINITY) ? 0.f : sacc * ex2(m - mm) + s2 * ex2(m2 - mm);
      m = mm;
    }
    if (lane == 0) {
      tmax[qslot * nb + j] = m * 0.6931471805599453f;  // back to natural-log units
      tsum[qslot * nb + j] = sacc;
    }
  }
}

// ------------------------------------------------------------------ 4. selection
// One CTA of 256 threads per (query block i, batch * kv-head): tile weights averaged over the
// group's q-heads, a bitonic sort by (weight desc, block asc), an inclusive scan of the sorted
// weights, and the blocks whose preceding cumulative weight is <= p (plus the diagonal) set in
// the bitmask `sel` [B*Hkv][nb][words].
constexpr int DPX_SEL_MAX = 2048;  // key blocks per query block the selection handles (N <= 256k)
__global__ void __launch_bounds__(256) dpxa_select_kernel(const float* __restrict__ tmax, const float* __restrict__ tsum,
                                                          uint32_t* __restrict__ sel, float p, int Hkv, int G, int nb,
                                                          int words) {
  extern __shared__ __align__(16) uint8_t ssm[];
  float* wv = reinterpret_cast<float*>(ssm);            // [npad] weights
  int32_t* wi = reinterpret_cast<int32_t*>(wv + DPX_SEL_MAX);  // [npad] block index
  uint32_t* bits = reinterpret_cast<uint32_t*>(wi + DPX_SEL_MAX);  // [words]
  __shared__ float wred[8];
  const int i = blockIdx.x, bk = blockIdx.y;
  const int b = bk / Hkv, hk = bk - b * Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = i + 1;
  int npad = 1;
  while (npad < n) npad <<= 1;
  for (int j = tid; j < npad; j += 256) {
    wv[j] = j < n ? 0.f : -1.f;
    wi[j] = j;
  }
  for (int w = tid; w < words; w += 256) bits[w] = 0u;
  __syncthreads();
  for (int gq = 0; gq < G; ++gq) {
    const int64_t row = ((static_cast<int64_t>(b) * Hkv + hk) * G + gq) * nb + i;  // q-head hk*G+gq
    const float* mr = tmax + row * nb;
    const float* sr = tsum + row * nb;
    float M = -INFINITY;
    for (int j = tid; j < n; j += 256) M = fmaxf(M, mr[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    if (lane == 0) wred[warp] = M;
    __syncthreads();
    M = wred[0];
    for (int w = 1; w < 8; ++w) M = fmaxf(M, wred[w]);
    __syncthreads();
    if (M == -INFINITY) M = 0.f;
    float Z = 0.f;
    for (int j = tid; j < n; j += 256) Z += (mr[j] == -INFINITY) ? 0.f : __expf(mr[j] - M) * sr[j];
#pragma unroll
    for (int o = 16; o; o >>= 1) Z += __shfl_xor_sync(0xFFFFFFFFu, Z, o);
    if (lane == 0) wred[warp] = Z;
    __syncthreads();
    Z = 0.f;
    for (int w = 0; w < 8; ++w) Z += wred[w];
    __syncthreads();
    if (Z > 0.f)
      for (int j = tid; j < n; j += 256)
        wv[j] += ((mr[j] == -INFINITY) ? 0.f : __expf(mr[j] - M) * sr[j] / Z) / static_cast<float>(G);
    __syncthreads();
  }
  // bitonic sort: weight descending, block ascending
  for (int kk = 2; kk <= npad; kk <<= 1) {
    for (int jj = kk >> 1; jj > 0; jj >>= 1) {
      for (int t = tid; t < npad; t += 256) {
        const int u = t ^ jj;
        if (u > t) {
          const bool desc_first = (t & kk) == 0;
          // "a before b" in the final order: larger weight first, then smaller block index
          const float wa = wv[t], wb = wv[u];
          const int ia = wi[t], ib = wi[u];
          const bool a_before_b = (wa > wb) || (wa == wb && ia < ib);
          if (desc_first != a_before_b) {
            wv[t] = wb; wv[u] = wa;
            wi[t] = ib; wi[u] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
  // exclusive prefix of the sorted weights: block wi[k] is selected iff it is <= p
  if (warp == 0) {
    float run = 0.f;
    for (int k0 = 0; k0 < n; k0 += 32) {
      const int k = k0 + lane;
      const float v = k < n ? wv[k] : 0.f;
      float incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += y;
      }
      const float excl = run + incl - v;
      if (k < n && excl <= p) atomicOr(&bits[wi[k] >> 5], 1u << (wi[k] & 31));
      run += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) atomicOr(&bits[i >> 5], 1u << (i & 31));  // the diagonal tile
  }
  __syncthreads();
  uint32_t* out = sel + (static_cast<int64_t>(bk) * nb + i) * words;
  for (int w = tid; w < words; w += 256) out[w] = bits[w];
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_dpxa_compact(int dtype, const void* x, const int64_t* xs, const int32_t* keep, const int64_t* kms,
                                void* cx, int32_t* cpos, int32_t* ccnt, int B, int H, int N, int D, cudaStream_t st) {
  const int nb = (N + DPX_B - 1) / DPX_B;
  if (B * H == 0 || nb == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(nb), static_cast<unsigned>(B * H));
  if (dtype == BF16)
    dpxa_compact_kernel<__nv_bfloat16><<<grid, DPX_B, 0, st>>>(static_cast<const __nv_bfloat16*>(x), xs[0], xs[1], xs[2],
                                                              keep, kms[0], kms[1], kms[2],
                                                              static_cast<__nv_bfloat16*>(cx), cpos, ccnt, H, N, D, nb);
  else if (dtype == F16)
    dpxa_compact_kernel<__half><<<grid, DPX_B, 0, st>>>(static_cast<const __half*>(x), xs[0], xs[1], xs[2], keep, kms[0],
                                                       kms[1], kms[2], static_cast<__half*>(cx), cpos, ccnt, H, N, D, nb);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_score_t(const void* cq, const int32_t* qpos, const int32_t* qcnt, const void* ck,
                                  const int32_t* kpos, const int32_t* kcnt, float* tmax, float* tsum, float sm_scale,
                                  int B, int Hq, int G, int nb, cudaStream_t st) {
  const int smem = DPX_B * D * 2 + DPX_B * 4 + DPX_SW * 2 * DPX_KC * D * 2;
  auto kfn = dpxa_score_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kfn<<<dim3(static_cast<unsigned>(nb), static_cast<unsigned>(B * Hq)), DPX_SW * 32, smem, st>>>(
      static_cast<const T*>(cq), qpos, qcnt, static_cast<const T*>(ck), kpos, kcnt, tmax, tsum, sm_scale, Hq, G, nb);
  return cudaGetLastError();
}

cudaError_t launch_dpxa_score(int dtype, const void* cq, const int32_t* qpos, const int32_t* qcnt, const void* ck,
                              const int32_t* kpos, const int32_t* kcnt, float* tmax, float* tsum, float sm_scale, int B,
                              int Hq, int G, int N, int D, cudaStream_t st) {
  const int nb = (N + DPX_B - 1) / DPX_B;
  if (B * Hq == 0 || nb == 0) return cudaSuccess;
  if (dtype == BF16) {
    if (D == 128) return launch_score_t<__nv_bfloat16, 128>(cq, qpos, qcnt, ck, kpos, kcnt, tmax, tsum, sm_scale, B, Hq, G, nb, st);
    if (D == 64) return launch_score_t<__nv_bfloat16, 64>(cq, qpos, qcnt, ck, kpos, kcnt, tmax, tsum, sm_scale, B, Hq, G, nb, st);
  } else if (dtype == F16) {
    if (D == 128) return launch_score_t<__half, 128>(cq, qpos, qcnt, ck, kpos, kcnt, tmax, tsum, sm_scale, B, Hq, G, nb, st);
    if (D == 64) return launch_score_t<__half, 64>(cq, qpos, qcnt, ck, kpos, kcnt, tmax, tsum, sm_scale, B, Hq, G, nb, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_dpxa_select(const float* tmax, const float* tsum, uint32_t* sel, float p, int B, int Hkv, int G,
                               int N, cudaStream_t st) {
  const int nb = (N + DPX_B - 1) / DPX_B;
  if (B * Hkv == 0 || nb == 0) return cudaSuccess;
  if (nb > DPX_SEL_MAX) return cudaErrorInvalidValue;
  const int words = (nb + 31) / 32;
  const int smem = DPX_SEL_MAX * 8 + words * 4;
  cudaError_t e = cudaFuncSetAttribute(dpxa_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dpxa_select_kernel<<<dim3(static_cast<unsigned>(nb), static_cast<unsigned>(B * Hkv)), 256, smem, st>>>(
      tmax, tsum, sel, p, Hkv, G, nb, words);
  return cudaGetLastError();
}

}  // namespace dab

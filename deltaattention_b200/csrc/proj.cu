// Projection GEMM with a fused RoPE epilogue on B200 (sm_100a: TMA, tcgen05 / TMEM).
//
// out[r, c] = RoPE(round(sum_k X[r, k] * W[c, k])) is the q / k projection of one attention
// layer followed by the rotary embedding (modeling_llama.py:550-555: `k_proj(hidden_states)
// .view(B, N, H, d).transpose(1, 2)`, then `apply_rotary_pos_emb`), written once in the
// projection layout [rows, Ho] that the attention and selection kernels read through strides.
// The unfused path writes the projection to HBM, reads it back for RoPE and writes it again.
// Columns outside [rope_lo, rope_hi) are stored as the rounded projection (v_proj, or the V
// part of a fused QKV weight). The rounding matches eager bf16: the Linear's fp32 sum is
// rounded to bf16, then k*cos, rotate_half(k)*sin and their sum are each rounded to bf16.
//
// Structure (persistent, one CTA per SM, 192 threads):
//   warp 0     TMA producer: per 64-wide k-block a 128 x 64 tile of X and a 256 x 64 tile of W
//              into a 4-stage ring (48 KB per stage)
//   warp 1     MMA issuer (one elected lane): tcgen05.mma kind::f16 M128 N256 K16 into one of
//              two TMEM accumulators (256 columns each), so a tile's epilogue overlaps the next
//              tile's main loop; also allocates TMEM
//   warps 2-5  epilogue: one output row per thread (TMEM lane quarter = warp % 4), 32-column
//              chunks of the first and second half of a head together (rotate_half pairs
//              column i with i + 64), 16-byte stores
// Tiles are ordered row block major, so the Ho / 256 tiles sharing a 128-row block of X run at
// the same time on neighbouring SMs and X is read from HBM about once.
#include "params.cuh"

namespace dab {

constexpr int PJ_BM = 128, PJ_BN = 256, PJ_BK = 64, PJ_STAGES = 4, PJ_HD = 128;
constexpr int PJ_THREADS = 192;
constexpr int PJ_ABYTES = PJ_BM * PJ_BK * 2;  // 16 KB
constexpr int PJ_BBYTES = PJ_BN * PJ_BK * 2;  // 32 KB
constexpr int PJ_STAGE = PJ_ABYTES + PJ_BBYTES;
constexpr int PJ_OFF_BAR = PJ_STAGES * PJ_STAGE;
constexpr int PJ_NBAR = 2 * PJ_STAGES + 2 + 2 + 1;
constexpr int PJ_OFF_MISC = PJ_OFF_BAR + PJ_NBAR * 8;
constexpr int PJ_SMEM = PJ_OFF_MISC + 64 + 1024;  // + alignment slack

// every lane waits; the outcome is made warp-uniform so the warp-collective tcgen05
// instructions that follow stay converged
__device__ __forceinline__ bool pj_wait(uint64_t* bar, uint32_t par, const Abort& ab, int code) {
  const bool ok = mbar_wait(bar, par, ab, code);
  return __all_sync(0xFFFFFFFFu, ok);
}

// bf16 RoPE of one output pair (dims i and i + 64 of a head), eager rounding order
__device__ __forceinline__ void rope_pair(float x1, float x2, float c1, float s1, float c2, float s2, float& o1,
                                          float& o2) {
  o1 = __fadd_rn(round_as<__nv_bfloat16>(__fmul_rn(x1, c1)), round_as<__nv_bfloat16>(__fmul_rn(-x2, s1)));
  o2 = __fadd_rn(round_as<__nv_bfloat16>(__fmul_rn(x2, c2)), round_as<__nv_bfloat16>(__fmul_rn(x1, s2)));
}

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

__global__ void __launch_bounds__(PJ_THREADS, 1) proj_rope_kernel(const __grid_constant__ ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PJ_OFF_BAR);
  uint64_t* full = bars;                    // [STAGES] X and W tiles landed
  uint64_t* empty = full + PJ_STAGES;       // [STAGES] the MMAs reading a stage completed
  uint64_t* acc_full = empty + PJ_STAGES;   // [2] an accumulator holds a finished tile
  uint64_t* acc_empty = acc_full + 2;       // [2] the epilogue has read an accumulator
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PJ_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + PJ_OFF_MISC + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PJ_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(acc_full + a, 1);
      mbar_init(acc_empty + a, 4);  // one arrival per epilogue warp
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_x);
    tma_prefetch_desc(&p.tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Abort ab{abort_flag, p.err};
  const int kblocks = (p.K + PJ_BK - 1) / PJ_BK;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    int issued = 0;  // k-blocks issued so far (ring position)
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int m = tile / p.n_tiles_n, n = tile % p.n_tiles_n;
      for (int kb = 0; kb < kblocks; ++kb, ++issued) {
        const int s = issued % PJ_STAGES;
        if (!pj_wait(empty + s, ((issued / PJ_STAGES) & 1) ^ 1, ab, ERR_TIMEOUT_PRODUCER)) goto prod_done;
        if (lane == 0) {
          uint8_t* a = smem + s * PJ_STAGE;
          mbar_arrive_expect_tx(full + s, PJ_STAGE);
          tma_load_4d(a, &p.tm_x, full + s, kb * PJ_BK, m * PJ_BM, 0, 0);
          tma_load_4d(a + PJ_ABYTES, &p.tm_w, full + s, kb * PJ_BK, n * PJ_BN, 0, 0);
        }
      }
    }
  prod_done:
    // every copy issued must land before the CTA exits (bounded; reported as ERR_TIMEOUT_DRAIN)
    if (lane == 0) {
      bool drained = true;
      for (int q = (issued > PJ_STAGES ? issued - PJ_STAGES : 0); q < issued && drained; ++q)
        drained = mbar_drain(full + q % PJ_STAGES, (q / PJ_STAGES) & 1, p.err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = umma_idesc_f16(PJ_BM, PJ_BN, true, false);
    int pos = 0, t_local = 0;
    bool aborted = false;
    for (int tile = blockIdx.x; tile < p.num_tiles && !aborted; tile += gridDim.x, ++t_local) {
      const int a = t_local & 1;
      if (!pj_wait(acc_empty + a, ((t_local >> 1) & 1) ^ 1, ab, ERR_TIMEOUT_MMA)) break;
      tc_fence_after();
      const uint32_t tD = tmem + a * PJ_BN;
      for (int kb = 0; kb < kblocks; ++kb, ++pos) {
        const int s = pos % PJ_STAGES;
        if (!pj_wait(full + s, (pos / PJ_STAGES) & 1, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * PJ_STAGE), 16, 1024);
        const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * PJ_STAGE + PJ_ABYTES), 16, 1024);
#pragma unroll
        for (int k = 0; k < PJ_BK / 16; ++k)
          umma_ss(tD, ad + static_cast<uint64_t>(k * 2), bd + static_cast<uint64_t>(k * 2), IDESC,
                  (kb | k) != 0 ? 1u : 0u);
        umma_commit(empty + s);  // the stage is free once these MMAs have read it
      }
      if (!aborted) umma_commit(acc_full + a);
    }
    umma_commit(mma_done);
    if (lane == 0) mbar_drain(mma_done, 0, p.err);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int qtr = warp & 3;  // TMEM lane quarter this warp may access
    const int r = qtr * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(qtr * 32) << 16;
    const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(p.cos);
    const __nv_bfloat16* sn = static_cast<const __nv_bfloat16*>(p.sin);
    int t_local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++t_local) {
      const int a = t_local & 1;
      const int m = tile / p.n_tiles_n, n = tile % p.n_tiles_n;
      const int row = m * PJ_BM + r;
      const bool row_ok = row < p.rows;
      if (!pj_wait(acc_full + a, (t_local >> 1) & 1, ab, ERR_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t tD = tmem + lane_base + a * PJ_BN;
      __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + static_cast<int64_t>(row) * p.os_row;
#pragma unroll 1
      for (int hh = 0; hh < PJ_BN / PJ_HD; ++hh) {
        const int col0 = n * PJ_BN + hh * PJ_HD;  // first output column of this head
        if (col0 >= p.Ho) break;
        const bool rope = col0 >= p.rope_lo && col0 < p.rope_hi;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t lo[32], hi[32];
          __syncwarp();
          tmem_ld32(tD + hh * PJ_HD + c * 32, lo);       // dims 32c .. 32c+31
          tmem_ld32(tD + hh * PJ_HD + 64 + c * 32, hi);  // dims 64+32c .. 64+32c+31
          if (!row_ok) continue;  // no collective instruction follows before the next __syncwarp
          uint4* o1p = reinterpret_cast<uint4*>(orow + col0 + c * 32);
          uint4* o2p = reinterpret_cast<uint4*>(orow + col0 + 64 + c * 32);
          if (rope) {
            const uint4* c1p = reinterpret_cast<const uint4*>(cs + static_cast<int64_t>(row) * p.cs_row + c * 32);
            const uint4* c2p = reinterpret_cast<const uint4*>(cs + static_cast<int64_t>(row) * p.cs_row + 64 + c * 32);
            const uint4* s1p = reinterpret_cast<const uint4*>(sn + static_cast<int64_t>(row) * p.cs_row + c * 32);
            const uint4* s2p = reinterpret_cast<const uint4*>(sn + static_cast<int64_t>(row) * p.cs_row + 64 + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {  // 8 dims per 16-byte vector
              const uint4 c1 = __ldg(c1p + v), c2 = __ldg(c2p + v), s1 = __ldg(s1p + v), s2 = __ldg(s2p + v);
              const uint32_t c1w[4] = {c1.x, c1.y, c1.z, c1.w}, c2w[4] = {c2.x, c2.y, c2.z, c2.w};
              const uint32_t s1w[4] = {s1.x, s1.y, s1.z, s1.w}, s2w[4] = {s2.x, s2.y, s2.z, s2.w};
              uint32_t w1[4], w2[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = v * 8 + 2 * e;
                const float x1a = round_as<__nv_bfloat16>(__uint_as_float(lo[j]));
                const float x1b = round_as<__nv_bfloat16>(__uint_as_float(lo[j + 1]));
                const float x2a = round_as<__nv_bfloat16>(__uint_as_float(hi[j]));
                const float x2b = round_as<__nv_bfloat16>(__uint_as_float(hi[j + 1]));
                float o1a, o2a, o1b, o2b;
                rope_pair(x1a, x2a, bf16_lo(c1w[e]), bf16_lo(s1w[e]), bf16_lo(c2w[e]), bf16_lo(s2w[e]), o1a, o2a);
                rope_pair(x1b, x2b, bf16_hi(c1w[e]), bf16_hi(s1w[e]), bf16_hi(c2w[e]), bf16_hi(s2w[e]), o1b, o2b);
                w1[e] = pack2(o1a, o1b, 1);
                w2[e] = pack2(o2a, o2b, 1);
              }
              o1p[v] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
              o2p[v] = make_uint4(w2[0], w2[1], w2[2], w2[3]);
            }
          } else {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w1[4], w2[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = v * 8 + 2 * e;
                w1[e] = pack2(__uint_as_float(lo[j]), __uint_as_float(lo[j + 1]), 1);
                w2[e] = pack2(__uint_as_float(hi[j]), __uint_as_float(hi[j + 1]), 1);
              }
              o1p[v] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
              o2p[v] = make_uint4(w2[0], w2[1], w2[2], w2[3]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + a);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

cudaError_t launch_proj_rope(const ProjParams& p, int num_sms, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(proj_rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PJ_SMEM);
  if (e != cudaSuccess) return e;
  const int grid = p.num_tiles < num_sms ? p.num_tiles : num_sms;
  if (grid <= 0) return cudaSuccess;
  proj_rope_kernel<<<grid, PJ_THREADS, PJ_SMEM, st>>>(p);
  return cudaGetLastError();
}

}  // namespace dab

// Generic CUDA-core attention for the reference's prefill kernels.
//
// Covers every variant with any strides, block sizes and head_dim <= 128:
//   HYBRID      hybrid_compressed_flash_kernel          deltaFlashAttention.py:9-146
//   SANITY      hybrid_compressed_flash_kernel_sanity   deltaFlashAttention.py:149-259
//   PURE        pure_phase1_flash_kernel                deltaFlashAttention.py:262-357
//   DENSE       _attn_fwd_flat (causal or not)          flashAttention.py:5-91
// It is the fp32 path (no tensor-core format keeps fp32 accuracy) and the path for
// shapes the tcgen05 kernel does not take. A CTA owns 32 query rows of one (batch, head);
// four threads share a row (interleaved head-dim slices); keys stream through shared
// memory 32 at a time. The reference's logical BLOCK_M x BLOCK_N schedule (phase-1 stop
// rule, dense restart block) is evaluated per CTA, so results follow the reference's
// block semantics exactly; only the floating-point summation order differs.
#include "params.cuh"

namespace dab {

constexpr int SIMT_ROWS = 32;
constexpr int SIMT_KT = 32;
constexpr int SIMT_TPR = 4;

template <typename T, int BD>
__global__ void __launch_bounds__(128) attn_simt_kernel(const SimtParams p) {
  constexpr int NE = BD / SIMT_TPR;  // head-dim elements per thread
  __shared__ float sK[SIMT_KT][BD + 1];
  __shared__ float sV[SIMT_KT][BD + 1];
  __shared__ float sC[SIMT_KT];
  __shared__ int32_t sT[SIMT_KT];
  __shared__ int64_t sched[2];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int slice = lane & 3;
  const int rloc = tid >> 2;  // 0..31
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / p.num_heads, h = bh % p.num_heads;
  const int64_t hk = h / p.kv_group;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * SIMT_ROWS;
  const int64_t row = r0 + rloc;
  const int64_t pid = r0 / p.block_m;  // logical query block
  const int64_t m0 = pid * p.block_m;
  const bool row_ok = row < p.seq_q && row < p.grid_m * p.block_m;

  const T* Q = static_cast<const T*>(p.q);
  const T* KD = static_cast<const T*>(p.kd);
  const T* VD = static_cast<const T*>(p.vd);
  const T* KP = static_cast<const T*>(p.kp);
  const T* VP = static_cast<const T*>(p.vp);

  float q[NE], o[NE];
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    const int d = slice + SIMT_TPR * i;
    q[i] = (row_ok && d < p.head_dim) ? to_f32(Q[b * p.qs[0] + h * p.qs[1] + row * p.qs[2] + d * p.qs[3]]) : 0.f;
    o[i] = 0.f;
  }
  float m_i = -INFINITY, l_i = 0.f;

  auto count_at = [&](int64_t j) -> float {
    const int64_t off = b * p.cs[0] + hk * p.cs[1] + j * p.cs[2];
    return p.counts_is_int ? static_cast<float>(static_cast<const int32_t*>(p.counts)[off])
                           : static_cast<const float*>(p.counts)[off];
  };
  auto ts_at = [&](int64_t j) -> int64_t { return p.ts[b * p.tss[0] + hk * p.tss[1] + j * p.tss[2]]; };

  // ---- phase-1 schedule (deltaFlashAttention.py:66-111): first block whose max timestamp
  //      (masked lanes read seq_len_k + 1) reaches start_m - window stops the loop
  int64_t n_packed_keys = 0, dense_lo = 0, dense_hi = 0;
  if (p.variant == HYBRID || p.variant == SANITY) {
    if (tid < 32) {
      int64_t start_n = 0, last_safe = -1;
      while (start_n < p.num_packed) {
        int64_t tmax = INT64_MIN;
        for (int64_t jj = lane; jj < p.block_n; jj += 32) {
          const int64_t j = start_n + jj;
          const int64_t t = (j < p.num_packed) ? ts_at(j) : p.seq_k + 1;
          tmax = max(tmax, t);
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) tmax = max(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, off));
        if (tmax >= m0 - p.dense_window) break;
        last_safe = tmax;
        start_n += p.block_n;
      }
      if (lane == 0) {
        sched[0] = start_n;  // keys [0, start_n) of the packed sequence are consumed
        // ((last_safe + 1) // BLOCK_N) * BLOCK_N with Python floor division, last_safe >= -1
        const int64_t ds = ((last_safe + 1) / p.block_n) * p.block_n;
        sched[1] = ds > 0 ? ds : 0;
      }
    }
    __syncthreads();
    n_packed_keys = (p.variant == HYBRID) ? sched[0] : 0;  // sanity discards phase 1
    dense_lo = sched[1];
    dense_hi = min(p.seq_k, m0 + p.block_m);
  } else if (p.variant == PURE) {
    n_packed_keys = ((p.num_packed + p.block_n - 1) / p.block_n) * p.block_n;
  } else {  // DENSE
    dense_lo = 0;
    dense_hi = p.causal ? min(p.seq_k, (pid + 1) * p.block_m) : p.seq_k;
  }

  auto process_tile = [&](int64_t k0, bool packed) {
    // cooperative load of 32 keys (fp32 in shared memory)
    const int64_t lim = packed ? p.num_packed : p.seq_k;
    for (int idx = tid; idx < SIMT_KT * BD; idx += 128) {
      const int j = idx / BD, d = idx % BD;
      const int64_t key = k0 + j;
      float kv = 0.f, vv = 0.f;
      if (key < lim && d < p.head_dim) {
        if (packed) {
          kv = to_f32(KP[b * p.kps[0] + hk * p.kps[1] + key * p.kps[2] + d * p.kps[3]]);
          vv = to_f32(VP[b * p.vps[0] + hk * p.vps[1] + key * p.vps[2] + d * p.vps[3]]);
        } else {
          kv = to_f32(KD[b * p.kds[0] + hk * p.kds[1] + key * p.kds[2] + d * p.kds[3]]);
          vv = to_f32(VD[b * p.vds[0] + hk * p.vds[1] + key * p.vds[2] + d * p.vds[3]]);
        }
      }
      sK[j][d] = kv;
      sV[j][d] = vv;
    }
    if (tid < SIMT_KT) {
      const int64_t key = k0 + tid;
      if (packed && key < p.num_packed) {
        sC[tid] = count_at(key);
        sT[tid] = static_cast<int32_t>(ts_at(key));
      } else {
        sC[tid] = 0.f;
        sT[tid] = 0;
      }
    }
    __syncthreads();
    float s[SIMT_KT];
#pragma unroll
    for (int j = 0; j < SIMT_KT; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NE; ++i) acc = fmaf(q[i], sK[j][slice + SIMT_TPR * i], acc);
      s[j] = acc;
    }
#pragma unroll
    for (int j = 0; j < SIMT_KT; ++j) {
      s[j] += __shfl_xor_sync(0xFFFFFFFFu, s[j], 1);
      s[j] += __shfl_xor_sync(0xFFFFFFFFu, s[j], 2);
    }
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < SIMT_KT; ++j) {
      const int64_t key = k0 + j;
      bool ok;
      if (packed) {
        ok = key < p.num_packed;
        if (p.variant == PURE) ok = ok && sC[j] > 0.f && static_cast<int64_t>(sT[j]) <= row;
      } else {
        ok = key < p.seq_k;
        if (p.variant != DENSE || p.causal) ok = ok && key <= row;
      }
      s[j] = ok ? s[j] * p.sm_scale : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    const float m_new = fmaxf(m_i, mt);
    const float m_ref = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = expf(m_i - m_ref);
    float lsum = 0.f;
#pragma unroll
    for (int j = 0; j < SIMT_KT; ++j) {
      float pj = expf(s[j] - m_ref);
      if (packed) pj *= sC[j];
      lsum += pj;
      s[j] = round_as<T>(pj);  // probabilities are cast to V's dtype before the PV product
    }
    l_i = l_i * alpha + lsum;
#pragma unroll
    for (int i = 0; i < NE; ++i) {
      float acc = o[i] * alpha;
#pragma unroll
      for (int j = 0; j < SIMT_KT; ++j) acc = fmaf(s[j], sV[j][slice + SIMT_TPR * i], acc);
      o[i] = acc;
    }
    m_i = m_new;
    __syncthreads();
  };

  for (int64_t k0 = 0; k0 < n_packed_keys; k0 += SIMT_KT) process_tile(k0, true);
  for (int64_t k0 = dense_lo; k0 < dense_hi; k0 += SIMT_KT) process_tile(k0, false);

  if (!row_ok) return;
  float l = l_i;
  if (p.variant == PURE && !(l > 0.f)) l = 1.f;
  T* O = static_cast<T*>(p.out);
  const float inv = 1.f / l;
#pragma unroll
  for (int i = 0; i < NE; ++i) {
    const int d = slice + SIMT_TPR * i;
    if (d < p.head_dim) O[b * p.os[0] + h * p.os[1] + row * p.os[2] + d * p.os[3]] = from_f32<T>(o[i] * inv);
  }
}

template <typename T, int BD>
static cudaError_t launch_simt_t(const SimtParams& p, cudaStream_t st) {
  const int64_t rows = min(p.seq_q, p.grid_m * p.block_m);
  if (rows <= 0 || p.grid_bh <= 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((rows + SIMT_ROWS - 1) / SIMT_ROWS), static_cast<unsigned>(p.grid_bh));
  attn_simt_kernel<T, BD><<<grid, 128, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_attn_simt(int dtype, const SimtParams& p, cudaStream_t st) {
  if (p.block_m % SIMT_ROWS != 0 || p.block_m <= 0 || p.block_n <= 0) return cudaErrorInvalidValue;
  if (p.grid_bh > 65535) return cudaErrorInvalidValue;
  int bd = 16;
  while (bd < p.head_dim) bd <<= 1;
  if (bd > 128) return cudaErrorInvalidValue;
#define DAB_SIMT(TY)                                          \
  switch (bd) {                                               \
    case 16: return launch_simt_t<TY, 16>(p, st);             \
    case 32: return launch_simt_t<TY, 32>(p, st);             \
    case 64: return launch_simt_t<TY, 64>(p, st);             \
    default: return launch_simt_t<TY, 128>(p, st);            \
  }
  switch (dtype) {
    case F32: DAB_SIMT(float)
    case F16: DAB_SIMT(__half)
    case BF16: DAB_SIMT(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_SIMT
}

}  // namespace dab

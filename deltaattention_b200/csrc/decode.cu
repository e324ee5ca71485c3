// Delta decoding on B200: cache update and single-token attention (HBM bound).
//
//  * decode_update: fused_hybrid_decode_update_kernel (deltaDecoding.py:9-104). One warp
//    per (batch, kv-head). When the exact ring is full, the token it evicts is compared
//    with the last packed key (fp32, reduced in the reference's order so merge / append
//    decisions are bit-exact) and either merged into that anchor's count or appended.
//  * decode_attn: fused_hybrid_decode_kernel (deltaDecoding.py:236-362) as split-K
//    flash-decoding. A CTA owns 128 keys of one (batch, kv-head) for ALL q-heads of the
//    group, so the packed cache is read from HBM once per kv-head (the reference reads it
//    once per q-head). Each lane scores one key for every head; chunk max / sum use warp
//    shuffles; partials (m, l, acc) are merged by decode_combine.
#include <atomic>
#include <type_traits>

#include "common.cuh"

namespace dab {

template <typename T, int BD, bool COS>
__global__ void __launch_bounds__(128) decode_update_kernel(
    const T* __restrict__ nk, const T* __restrict__ nv, T* __restrict__ ke, T* __restrict__ ve,
    T* __restrict__ kp, T* __restrict__ vp, int32_t* __restrict__ counts, int32_t* __restrict__ ts,
    int32_t* __restrict__ lengths, int64_t exact_seq_len, int64_t total_seq_len, const int64_t* __restrict__ st,
    float thr, int64_t W, int64_t ns_b, int64_t ns_h, int64_t ns_s, int64_t ns_d, int64_t es_b, int64_t es_h,
    int64_t es_s, int64_t es_d, int64_t ps_b, int64_t ps_h, int64_t ps_s, int64_t ps_d, int64_t cs_b, int64_t cs_h,
    int64_t cs_s, int64_t num_heads, int64_t head_dim, int64_t programs, int64_t capacity, int* err) {
  if (st) {  // device-resident (exact, total) sequence state
    exact_seq_len = st[0];
    total_seq_len = st[1];
  }
  constexpr int NH = BD > 128 ? 2 : 1;
  constexpr int PER = BD / 8 / NH;
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  const int64_t pid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pid >= programs) return;
  const int pb = static_cast<int>(pid) / static_cast<int>(num_heads);  // 32-bit: pid < programs << 2^31
  const int64_t b = pb, h = static_cast<int>(pid) - pb * static_cast<int>(num_heads);
  const int64_t w = exact_seq_len % W;
  T* ek = ke + b * es_b + h * es_h + w * es_s;
  T* ev = ve + b * es_b + h * es_h + w * es_s;
  T* pk = kp + b * ps_b + h * ps_h;
  T* pv = vp + b * ps_b + h * ps_h;
  int32_t* cb = counts + b * cs_b + h * cs_h;
  int32_t* tb = ts + b * cs_b + h * cs_h;
  const int32_t plen = lengths[pid];
  // every load that does not depend on the decision is issued now: the new token and the
  // evicted V row (its K row is loaded below with the last anchor's key and count)
  constexpr int NV = BD / 32 > 0 ? BD / 32 : 1;  // elements per lane of a row
  T nkr[NV], nvr[NV], evr[NV];
  {
    const T* sk = nk + b * ns_b + h * ns_h;
    const T* sv = nv + b * ns_b + h * ns_h;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int64_t d = lane + 32 * j;
      if (d < head_dim) {
        nkr[j] = sk[d * ns_d];
        nvr[j] = sv[d * ns_d];
        evr[j] = ev[d * es_d];
      }
    }
  }
  if (exact_seq_len >= W) {
    bool merge = false;
    int32_t last_count = 0;
    if (plen > 0) {
      const T* lk = pk + static_cast<int64_t>(plen - 1) * ps_s;
      if (lane == 0) last_count = cb[static_cast<int64_t>(plen - 1) * cs_s];
      float ea[NH][PER], la[NH][PER];
#pragma unroll
      for (int hh = 0; hh < NH; ++hh)
#pragma unroll
        for (int m = 0; m < PER; ++m) {
          const int e = hh * 128 + g + 8 * m;
          ea[hh][m] = e < head_dim ? to_f32(ek[e * es_d]) : 0.f;
          la[hh][m] = e < head_dim ? to_f32(lk[e * ps_d]) : 0.f;
        }
      auto tree = [&](float v) {
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
        return v;
      };
      if constexpr (COS) {
        float dot = 0.f, n1 = 0.f, n2 = 0.f;
#pragma unroll
        for (int hh = 0; hh < NH; ++hh) {
          float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
          for (int m = 0; m < PER; ++m) {
            const float p0 = __fmul_rn(ea[hh][m], la[hh][m]);
            const float p1 = __fmul_rn(ea[hh][m], ea[hh][m]);
            const float p2 = __fmul_rn(la[hh][m], la[hh][m]);
            a0 = m ? __fadd_rn(a0, p0) : p0;
            a1 = m ? __fadd_rn(a1, p1) : p1;
            a2 = m ? __fadd_rn(a2, p2) : p2;
          }
          a0 = tree(a0); a1 = tree(a1); a2 = tree(a2);
          dot = hh ? __fadd_rn(dot, a0) : a0;
          n1 = hh ? __fadd_rn(n1, a1) : a1;
          n2 = hh ? __fadd_rn(n2, a2) : a2;
        }
        const float ne = __fsqrt_rn(__fadd_rn(n1, 1e-8f));
        const float nl = __fsqrt_rn(__fadd_rn(n2, 1e-8f));
        merge = __fdiv_rn(dot, __fmul_rn(ne, nl)) >= thr;
      } else {
        float tot = 0.f;
#pragma unroll
        for (int hh = 0; hh < NH; ++hh) {
          float acc = 0.f;
#pragma unroll
          for (int m = 0; m < PER; ++m) {
            const float d = __fsub_rn(ea[hh][m], la[hh][m]);
            const float sq = __fmul_rn(d, d);
            acc = m ? __fadd_rn(acc, sq) : sq;
          }
          acc = tree(acc);
          tot = hh ? __fadd_rn(tot, acc) : acc;
        }
        merge = tot <= thr;
      }
    }
    if (merge) {
      if (lane == 0) cb[static_cast<int64_t>(plen - 1) * cs_s] = last_count + 1;
    } else if (plen < capacity) {
      T* dk = pk + static_cast<int64_t>(plen) * ps_s;
      T* dv = pv + static_cast<int64_t>(plen) * ps_s;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int64_t d = lane + 32 * j;
        if (d < head_dim) {
          dk[d * ps_d] = ek[d * es_d];
          dv[d * ps_d] = evr[j];
        }
      }
      if (lane == 0) {
        cb[static_cast<int64_t>(plen) * cs_s] = 1;
        tb[static_cast<int64_t>(plen) * cs_s] = static_cast<int32_t>(total_seq_len - W);
        lengths[pid] = plen + 1;
      }
    } else if (lane == 0 && err) {
      atomicCAS(err, 0, 0x201);  // packed cache full: the caller must grow it first
    }
  }
  __syncwarp();  // the evicted row has been read by every lane before it is overwritten
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int64_t d = lane + 32 * j;
    if (d < head_dim) {
      ek[d * es_d] = nkr[j];
      ev[d * es_d] = nvr[j];
    }
  }
}

cudaError_t launch_decode_update(int dtype, int bd, bool cosine, const void* nk, const void* nv, void* ke,
                                 void* ve, void* kp, void* vp, int32_t* counts, int32_t* ts, int32_t* lengths,
                                 int64_t exact_seq_len, int64_t total_seq_len, const int64_t* seq_state, float thr,
                                 int64_t W,
                                 const int64_t* ns, const int64_t* es, const int64_t* ps, const int64_t* cs,
                                 int64_t num_heads, int64_t head_dim, int64_t programs, int64_t capacity, int* err,
                                 cudaStream_t st) {
  if (programs <= 0) return cudaSuccess;
  if (W <= 0) return cudaErrorInvalidValue;
  const unsigned blocks = static_cast<unsigned>((programs + 3) / 4);
#define DAB_UPD(TY, N, C)                                                                                     \
  decode_update_kernel<TY, N, C><<<blocks, 128, 0, st>>>(                                                     \
      static_cast<const TY*>(nk), static_cast<const TY*>(nv), static_cast<TY*>(ke), static_cast<TY*>(ve),      \
      static_cast<TY*>(kp), static_cast<TY*>(vp), counts, ts, lengths, exact_seq_len, total_seq_len, seq_state, \
      thr, W,                                                                                                 \
      ns[0], ns[1], ns[2], ns[3], es[0], es[1], es[2], es[3], ps[0], ps[1], ps[2], ps[3], cs[0], cs[1], cs[2], \
      num_heads, head_dim, programs, capacity, err);                                                          \
  return cudaGetLastError();
#define DAB_UPD_BD(TY, C)            \
  switch (bd) {                      \
    case 16: DAB_UPD(TY, 16, C)      \
    case 32: DAB_UPD(TY, 32, C)      \
    case 64: DAB_UPD(TY, 64, C)      \
    case 128: DAB_UPD(TY, 128, C)    \
    case 256: DAB_UPD(TY, 256, C)    \
    default: return cudaErrorInvalidValue; \
  }
#define DAB_UPD_DT(TY) \
  if (cosine) { DAB_UPD_BD(TY, true) } else { DAB_UPD_BD(TY, false) }
  switch (dtype) {
    case F32: DAB_UPD_DT(float)
    case F16: DAB_UPD_DT(__half)
    case BF16: DAB_UPD_DT(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_UPD
#undef DAB_UPD_BD
#undef DAB_UPD_DT
}

// ----------------------------------------------------------------------------- attention
constexpr int DEC_KC = 128;   // keys per CTA
constexpr int DEC_GMAX = 8;   // q-heads per kv-head handled by one CTA

template <typename T, int BD>
__global__ void __launch_bounds__(128) decode_attn_kernel(
    const T* __restrict__ q, int64_t qs_b, int64_t qs_h, int64_t qs_d, const T* __restrict__ kp, int64_t kps_b,
    int64_t kps_h, int64_t kps_n, int64_t kps_d, const T* __restrict__ vp, int64_t vps_b, int64_t vps_h,
    int64_t vps_n, int64_t vps_d, const int32_t* __restrict__ counts, int64_t cs_b, int64_t cs_h, int64_t cs_n,
    const int32_t* __restrict__ lengths, int64_t ls_b, int64_t ls_h, const T* __restrict__ ke, int64_t kes_b,
    int64_t kes_h, int64_t kes_n, int64_t kes_d, const T* __restrict__ ve, int64_t ves_b, int64_t ves_h,
    int64_t ves_n, int64_t ves_d, float sm_scale, int64_t exact_len, const int64_t* __restrict__ st, int64_t W,
    int64_t lag, int64_t G, int64_t Hkv, int64_t head_dim, int64_t nchunk, float* __restrict__ part) {
  if (st) {  // device-resident sequence state, `lag` steps behind when the advance follows
    const int64_t e = st[0] + lag;
    exact_len = e < W ? e : W;
  }
  __shared__ float sq[DEC_GMAX][BD];
  __shared__ float sp[DEC_GMAX][DEC_KC];
  __shared__ float swm[4][DEC_GMAX];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = blockIdx.x;
  const int64_t bk = blockIdx.y;
  const int b32 = static_cast<int>(bk) / static_cast<int>(Hkv);  // 32-bit: grid y extent << 2^31
  const int64_t b = b32, hk = static_cast<int>(bk) - b32 * static_cast<int>(Hkv);
  const int64_t plen = lengths[b * ls_b + hk * ls_h];
  const int64_t total = plen + exact_len;
  const int64_t k0 = chunk * DEC_KC;
  float* pout = part + ((bk * nchunk + chunk) * G) * (BD + 2);
  if (k0 >= total) {
    // empty partial: m = -inf, l = 0
    for (int g = 0; g < G; ++g)
      if (tid == 0) { pout[g * (BD + 2)] = -INFINITY; pout[g * (BD + 2) + 1] = 0.f; }
    return;
  }
  for (int i = tid; i < G * BD; i += 128) {
    const int g = i / BD, d = i % BD;
    sq[g][d] = d < head_dim ? to_f32(q[b * qs_b + (hk * G + g) * qs_h + d * qs_d]) : 0.f;
  }
  __syncthreads();
  // score: lane owns key k0 + warp*32 + lane
  const int64_t key = k0 + warp * 32 + lane;
  const bool valid = key < total;
  const bool packed = key < plen;
  float s[DEC_GMAX];
#pragma unroll
  for (int g = 0; g < DEC_GMAX; ++g) s[g] = 0.f;
  if (valid) {
    const T* kr = packed ? kp + b * kps_b + hk * kps_h + key * kps_n
                         : ke + b * kes_b + hk * kes_h + (key - plen) * kes_n;
    const int64_t sd = packed ? kps_d : kes_d;
    for (int d = 0; d < head_dim; ++d) {
      const float kv = to_f32(kr[d * sd]);
#pragma unroll
      for (int g = 0; g < DEC_GMAX; ++g)
        if (g < G) s[g] = fmaf(sq[g][d], kv, s[g]);
    }
  }
  float bias = 0.f;
  if (valid && packed) bias = logf(static_cast<float>(counts[b * cs_b + hk * cs_h + key * cs_n]));
  float mloc[DEC_GMAX];
#pragma unroll
  for (int g = 0; g < DEC_GMAX; ++g) {
    s[g] = valid ? s[g] * sm_scale + bias : -INFINITY;
    float m = s[g];
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    mloc[g] = m;
  }
  if (lane == 0)
    for (int g = 0; g < G; ++g) swm[warp][g] = mloc[g];
  __syncthreads();
  float m_c[DEC_GMAX];
#pragma unroll
  for (int g = 0; g < DEC_GMAX; ++g)
    m_c[g] = (g < G) ? fmaxf(fmaxf(swm[0][g], swm[1][g]), fmaxf(swm[2][g], swm[3][g])) : 0.f;
  __syncthreads();
  float lsum[DEC_GMAX];
#pragma unroll
  for (int g = 0; g < DEC_GMAX; ++g) {
    if (g >= G) continue;
    const float ref = (m_c[g] == -INFINITY) ? 0.f : m_c[g];
    const float pv = valid ? expf(s[g] - ref) : 0.f;
    sp[g][warp * 32 + lane] = round_as<T>(pv);  // P is cast to V's dtype before the PV product
    float l = pv;
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    lsum[g] = l;
  }
  if (lane == 0)
    for (int g = 0; g < G; ++g) swm[warp][g] = lsum[g];
  __syncthreads();
  // PV: thread owns head-dim column d = tid (and tid + 128 when BD = 256)
  const int64_t kend = (total - k0 < DEC_KC) ? (total - k0) : DEC_KC;
  for (int d = tid; d < BD; d += 128) {
    float acc[DEC_GMAX];
#pragma unroll
    for (int g = 0; g < DEC_GMAX; ++g) acc[g] = 0.f;
    if (d < head_dim) {
      for (int64_t j = 0; j < kend; ++j) {
        const int64_t kk = k0 + j;
        const float v = (kk < plen) ? to_f32(vp[b * vps_b + hk * vps_h + kk * vps_n + d * vps_d])
                                    : to_f32(ve[b * ves_b + hk * ves_h + (kk - plen) * ves_n + d * ves_d]);
#pragma unroll
        for (int g = 0; g < DEC_GMAX; ++g)
          if (g < G) acc[g] = fmaf(sp[g][j], v, acc[g]);
      }
    }
    for (int g = 0; g < G; ++g) pout[g * (BD + 2) + 2 + d] = acc[g];
  }
  if (tid < G) {
    pout[tid * (BD + 2)] = m_c[tid];
    pout[tid * (BD + 2) + 1] = swm[0][tid] + swm[1][tid] + swm[2][tid] + swm[3][tid];
  }
}

template <typename T, int BD>
__global__ void __launch_bounds__(128) decode_combine_kernel(const float* __restrict__ part, T* __restrict__ out,
                                                             int64_t os_b, int64_t os_h, int64_t os_d, int64_t G,
                                                             int64_t Hkv, int64_t nchunk, int64_t head_dim,
                                                             int64_t* __restrict__ adv) {
  // pass 1: every chunk's (max, sum) in parallel, the block maximum, and each chunk's scale
  // factor in shared memory (0 for chunks past the sequence, whose O was never written);
  // pass 2: warp w sums the scaled partial O of chunks w, w + 4, ..., each lane two adjacent
  // columns per 8-byte load, four chunks' loads in flight; the four warps' sums meet in
  // shared memory
  extern __shared__ float cmb[];  // f[nchunk], then l[nchunk]
  float* sf = cmb;
  float* sl = cmb + nchunk;
  __shared__ float red[4];
  __shared__ float2 wsum[4][BD / 2];
  // 32-bit division (grid extent and head counts are far below 2^31)
  const int hq32 = static_cast<int>(Hkv * G), g32 = static_cast<int>(G);
  const int b32 = static_cast<int>(blockIdx.x) / hq32, h32 = static_cast<int>(blockIdx.x) - b32 * hq32;
  const int hk32 = h32 / g32;
  const int64_t b = b32, h = h32, hk = hk32, g = h32 - hk32 * g32;
  const int64_t bk = b * Hkv + hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = part + (bk * nchunk * G + g) * (BD + 2);
  const int64_t cstride = G * (BD + 2);
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < nchunk; c += blockDim.x) {
    const float mc = base[c * cstride];
    sf[c] = mc;
    sl[c] = base[c * cstride + 1];
    m = fmaxf(m, mc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float ref = (m == -INFINITY) ? 0.f : m;
  float l = 0.f;
  for (int64_t c = threadIdx.x; c < nchunk; c += blockDim.x) {
    const float mc = sf[c];
    const float f = (mc == -INFINITY) ? 0.f : expf(mc - ref);
    sf[c] = f;
    l = fmaf(sl[c], f, l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
  __syncthreads();  // every f is in place; red[] is free again
  if (lane == 0) red[warp] = l;
  constexpr int NE = BD / 2 > 32 ? BD / 2 / 32 : 1;  // column pairs per lane
  float2 acc[NE];
#pragma unroll
  for (int k = 0; k < NE; ++k) acc[k] = make_float2(0.f, 0.f);
  for (int64_t c0 = warp; c0 < nchunk; c0 += 16) {
    float2 v[4][NE];
    float f[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t c = c0 + 4 * u;
      f[u] = c < nchunk ? sf[c] : 0.f;
      const float2* row = reinterpret_cast<const float2*>(base + c * cstride + 2);  // 8-byte aligned
#pragma unroll
      for (int k = 0; k < NE; ++k) {
        const int e = lane + 32 * k;
        v[u][k] = (f[u] != 0.f && e < BD / 2 && 2 * e < head_dim) ? row[e] : make_float2(0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int k = 0; k < NE; ++k) {
        acc[k].x = fmaf(v[u][k].x, f[u], acc[k].x);
        acc[k].y = fmaf(v[u][k].y, f[u], acc[k].y);
      }
  }
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    const int e = lane + 32 * k;
    if (e < BD / 2) wsum[warp][e] = acc[k];
  }
  __syncthreads();
  const float lt = (red[0] + red[1]) + (red[2] + red[3]);
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    const float* w0 = reinterpret_cast<const float*>(wsum[0]);
    const float* w1 = reinterpret_cast<const float*>(wsum[1]);
    const float* w2 = reinterpret_cast<const float*>(wsum[2]);
    const float* w3 = reinterpret_cast<const float*>(wsum[3]);
    const float a = (w0[d] + w1[d]) + (w2[d] + w3[d]);
    out[b * os_b + h * os_h + d * os_d] = from_f32<T>(a / lt);
  }
  // the step's length advance, after the attention kernel (the state's last reader this step)
  if (adv && blockIdx.x == 0 && threadIdx.x == 0) {
    adv[0] += 1;
    adv[1] += 1;
  }
}

// Tensor-core split-K decode for 16-bit types with unit head-dim strides and 16-byte rows.
// A CTA (DEC_NW = 8 warps) takes 128 keys of one (batch, kv-head) for all G (<= 8) q-heads:
//   * every thread copies 16-byte row segments of the block's K rows into shared memory with
//     cp.async (rows past the end are zero-filled), with the segment index XOR-swizzled by the
//     row so that ldmatrix reads are conflict-free; the V rows follow into the same buffer as
//     soon as every warp has read K, and land while the softmax runs (one 32 KB buffer instead
//     of two, so five CTAs share an SM);
//   * warp w scores keys 16w..16w+15 with mma.sync m16n8k16 (A = the q-heads padded to 16 rows,
//     B = K rows via ldmatrix);
//   * the chunk's row maximum per head goes through shared memory, and P = exp(s - max), cast
//     to V's dtype as the reference does before its PV product, is written to shared memory;
//   * warp w multiplies P by V for head-dim columns D/8*w.. over all 128 keys (V by
//     ldmatrix.trans), so the warps' outputs need no merge; (max, sum, O) form the chunk's
//     partial for the combine kernel.
// Against scoring one key per lane on CUDA cores (68 M instructions per launch, issue-bound at
// ~0.3 of HBM bandwidth) this issues a fraction of the instructions.
constexpr int DEC_VKC = 128;

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
// C (f32, 16x8) += A (16x16) * B (16x8), A row-major / B column-major, 16-bit inputs
template <typename T>
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}
template <typename T>
__device__ __forceinline__ uint32_t pack_t2(float lo, float hi) {
  return pack2(lo, hi, std::is_same<T, __nv_bfloat16>::value ? 1 : 0);
}

constexpr int DEC_NW = 8;  // warps per CTA: 16 keys each
constexpr int DEC_PROW = DEC_VKC + 8;  // padded P row (elements): conflict-free A-fragment loads
// K and V share one row buffer (V is copied in once every warp has read K), so five CTAs fit
// on an SM
template <int D>
constexpr int decode_mma_smem() {
  return 128 * D * 2 + 8 * D * 2 + 128 * 4 + 2 * DEC_NW * 8 * 4 + 8 * DEC_PROW * 2;
}

template <typename T, int D>
__global__ void __launch_bounds__(DEC_NW * 32, 5) decode_attn_mma_kernel(
    const T* __restrict__ q, int64_t qs_b, int64_t qs_h, const T* __restrict__ kp, int64_t kps_b, int64_t kps_h,
    int64_t kps_n, const T* __restrict__ vp, int64_t vps_b, int64_t vps_h, int64_t vps_n,
    const int32_t* __restrict__ counts, int64_t cs_b, int64_t cs_h, int64_t cs_n, const int32_t* __restrict__ lengths,
    int64_t ls_b, int64_t ls_h, const T* __restrict__ ke, int64_t kes_b, int64_t kes_h, int64_t kes_n,
    const T* __restrict__ ve, int64_t ves_b, int64_t ves_h, int64_t ves_n, float sm_scale, int64_t exact_len,
    const int64_t* __restrict__ st, int64_t W, int64_t lag, int G, int64_t Hkv, int64_t nchunk,
    float* __restrict__ part, bool qvec) {
  if (st) {  // device-resident sequence state, `lag` steps behind when the advance follows
    const int64_t e = st[0] + lag;
    exact_len = e < W ? e : W;
  }
  constexpr int ROWB = D * 2;   // bytes per K / V row
  constexpr int SEGS = D / 8;   // 16-byte segments per row
  constexpr int NT = DEC_NW * 32;        // threads
  constexpr int KPW = DEC_VKC / DEC_NW;  // keys per warp
  constexpr int NTW = KPW / 8;           // QK n-tiles per warp
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* Ks = dsm;                                          // [128][D], swizzled segments
  uint8_t* Vs = dsm;                                          // V over K once K has been read
  T* qsm = reinterpret_cast<T*>(dsm + DEC_VKC * ROWB);        // [8][D], rows >= G zero
  float* bias = reinterpret_cast<float*>(qsm + 8 * D);        // [128] log(count) of packed keys
  float* swm = bias + DEC_VKC;                                // [NW][8] per-warp max
  float* swl = swm + DEC_NW * 8;                              // [NW][8] per-warp sum
  T* Ps = reinterpret_cast<T*>(swl + DEC_NW * 8);             // [8][PROW] P of the chunk
  constexpr int PROW = DEC_PROW;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = blockIdx.x;
  const int64_t bk = blockIdx.y;
  // 32-bit division (the grid's y extent and the head count are far below 2^31)
  const int b32 = static_cast<int>(blockIdx.y) / static_cast<int>(Hkv);
  const int64_t b = b32, hk = static_cast<int>(blockIdx.y) - b32 * static_cast<int>(Hkv);
  const int64_t plen = lengths[b * ls_b + hk * ls_h];
  const int64_t total = plen + exact_len;
  const int64_t k0 = chunk * DEC_VKC;
  float* pout = part + ((bk * nchunk + chunk) * G) * (D + 2);
  if (k0 >= total) {
    if (tid < G) { pout[tid * (D + 2)] = -INFINITY; pout[tid * (D + 2) + 1] = 0.f; }
    return;
  }
  // ---- the block's K rows into shared memory (V follows into the same buffer once every warp
  // has read K), q and the count biases.
  // Thread t always copies 16-byte segment t % SEGS of rows t / SEGS + RPP*i; RPP is a multiple
  // of 8, so the swizzled segment (s ^ (row & 7)) is the same for all of this thread's rows.
  constexpr int RPP = NT / SEGS;
  const int cs_seg = tid % SEGS, r0 = tid / SEGS;
  const uint32_t rows_dst = smem_u32(Ks) + static_cast<uint32_t>(r0 * ROWB + ((cs_seg ^ (r0 & 7)) << 4));
  // rows k0 + r0 + RPP*i of the packed history (stride pn) continued by the exact window (stride en)
  auto issue_rows = [&](const T* pb, int64_t pn, const T* eb, int64_t en) {
    if (k0 + DEC_VKC <= plen) {
      const T* src = pb + (k0 + r0) * pn;
#pragma unroll 8
      for (int i = 0; i < DEC_VKC / RPP; ++i) cp_async16_zfill(rows_dst + i * RPP * ROWB, src + i * RPP * pn, true);
    } else {
      for (int i = 0; i < DEC_VKC / RPP; ++i) {
        const int64_t key = k0 + r0 + i * RPP;
        const bool ok = key < total;
        const T* src = !ok ? pb : (key < plen ? pb + key * pn : eb + (key - plen) * en);
        cp_async16_zfill(rows_dst + i * RPP * ROWB, src, ok);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // q rows 0..G-1 (A-fragment rows 0..7; rows 8..15 are never read, their fragments are 0):
  // 16-byte copies in K's commit group when q's rows allow it
  if (qvec) {
    if (tid < 8 * SEGS) {
      const int g = tid / SEGS, sq = tid % SEGS;
      cp_async16_zfill(smem_u32(qsm) + g * ROWB + sq * 16, q + b * qs_b + (hk * G + (g < G ? g : 0)) * qs_h + sq * 8,
                       g < G);
    }
  } else {
    for (int i = tid; i < 8 * D; i += NT) {
      const int g = i / D, d = i % D;
      qsm[i] = g < G ? q[b * qs_b + (hk * G + g) * qs_h + d] : from_f32<T>(0.f);
    }
  }
  issue_rows(kp + b * kps_b + hk * kps_h + cs_seg * 8, kps_n, ke + b * kes_b + hk * kes_h + cs_seg * 8, kes_n);
  if (tid < DEC_VKC) {
    const int64_t key = k0 + tid;
    bias[tid] = (key < plen) ? logf(static_cast<float>(counts[b * cs_b + hk * cs_h + key * cs_n])) : 0.f;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // K
  __syncthreads();

  const int g = lane >> 2;        // head row of this thread's accumulator fragments (rows g+8 are padding)
  const int c2 = (lane & 3) * 2;  // first of the two key / head-dim columns this thread holds
  // ---- S^T = q . K^T for this warp's KPW keys: n-tiles of 8 keys
  float acc[NTW][4];
#pragma unroll
  for (int j = 0; j < NTW; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
#pragma unroll
  for (int kp2 = 0; kp2 < D / 32; ++kp2) {
    uint32_t qa[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const T* qr = qsm + g * D + (2 * kp2 + h) * 16 + c2;
      qa[h][0] = *reinterpret_cast<const uint32_t*>(qr);
      qa[h][1] = *reinterpret_cast<const uint32_t*>(qr + 8);
    }
#pragma unroll
    for (int j = 0; j < NTW; ++j) {
      const int r = KPW * warp + 8 * j + (lane & 7);
      const int s = 4 * kp2 + (lane >> 3);
      uint32_t bb[4];
      ldsm_x4(bb, smem_u32(Ks + r * ROWB + ((s ^ (r & 7)) << 4)));
      mma16816<T>(acc[j], qa[0][0], 0u, qa[0][1], 0u, bb[0], bb[1]);
      mma16816<T>(acc[j], qa[1][0], 0u, qa[1][1], 0u, bb[2], bb[3]);
    }
  }
  // ---- softmax over the chunk's 128 keys for head g: each warp's maximum through shared
  // memory, one chunk maximum, P = exp(s - max) cast to V's dtype into shared memory
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < NTW; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int kl = KPW * warp + 8 * j + c2 + e;
      const bool ok = k0 + kl < total;
      acc[j][e] = ok ? acc[j][e] * sm_scale + bias[kl] : -INFINITY;
      mx = fmaxf(mx, acc[j][e]);
    }
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
  if ((lane & 3) == 0) swm[warp * 8 + g] = mx;
  __syncthreads();  // every warp is done with K: V's rows go into the same buffer
  issue_rows(vp + b * vps_b + hk * vps_h + cs_seg * 8, vps_n, ve + b * ves_b + hk * ves_h + cs_seg * 8, ves_n);
  float M = swm[g];
#pragma unroll
  for (int w = 1; w < DEC_NW; ++w) M = fmaxf(M, swm[w * 8 + g]);
  const float ref = (M == -INFINITY) ? 0.f : M;
  float l = 0.f;
#pragma unroll
  for (int j = 0; j < NTW; ++j) {
    const float p0 = acc[j][0] == -INFINITY ? 0.f : expf(acc[j][0] - ref);
    const float p1 = acc[j][1] == -INFINITY ? 0.f : expf(acc[j][1] - ref);
    l += p0 + p1;
    *reinterpret_cast<uint32_t*>(Ps + g * PROW + KPW * warp + 8 * j + c2) = pack_t2<T>(p0, p1);
  }
  l += __shfl_xor_sync(0xFFFFFFFFu, l, 1);
  l += __shfl_xor_sync(0xFFFFFFFFu, l, 2);
  if ((lane & 3) == 0) swl[warp * 8 + g] = l;
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // V
  __syncthreads();
  // ---- O = P . V: warp w owns head-dim columns (D / NW) * w .. over all 128 keys, so the
  // warps' outputs need no merge
  constexpr int NTD = D / 8 / DEC_NW;  // n-tiles of 8 columns per warp (2 for d = 128, 1 for 64)
  float o[NTD][4];
#pragma unroll
  for (int n = 0; n < NTD; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  const int mi = lane >> 3;
#pragma unroll
  for (int kk = 0; kk < DEC_VKC / 16; ++kk) {
    const uint32_t a0 = *reinterpret_cast<const uint32_t*>(Ps + g * PROW + 16 * kk + c2);
    const uint32_t a2 = *reinterpret_cast<const uint32_t*>(Ps + g * PROW + 16 * kk + 8 + c2);
    const int r = 16 * kk + (mi & 1) * 8 + (lane & 7);
    if constexpr (NTD == 2) {
      const int s = 2 * warp + (mi >> 1);
      uint32_t bb[4];
      ldsm_x4_t(bb, smem_u32(Vs + r * ROWB + ((s ^ (r & 7)) << 4)));
      mma16816<T>(o[0], a0, 0u, a2, 0u, bb[0], bb[1]);
      mma16816<T>(o[1], a0, 0u, a2, 0u, bb[2], bb[3]);
    } else {
      uint32_t bb[2];
      ldsm_x2_t(bb, smem_u32(Vs + r * ROWB + ((warp ^ (r & 7)) << 4)));
      mma16816<T>(o[0], a0, 0u, a2, 0u, bb[0], bb[1]);
    }
  }
  if (g < G) {
#pragma unroll
    for (int n = 0; n < NTD; ++n) {
      float* dst = pout + g * (D + 2) + 2 + (D / DEC_NW) * warp + 8 * n + c2;
      dst[0] = o[n][0];
      dst[1] = o[n][1];
    }
    if (warp == 0 && (lane & 3) == 0) {
      float lt = 0.f;
#pragma unroll
      for (int w = 0; w < DEC_NW; ++w) lt += swl[w * 8 + g];
      pout[g * (D + 2)] = M;
      pout[g * (D + 2) + 1] = lt;
    }
  }
}

// One decode step of device-resident sequence states: (exact, total) += 1 for `count` pairs.
__global__ void decode_advance_kernel(int64_t* st, int64_t count) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < count) {
    st[2 * i] += 1;
    st[2 * i + 1] += 1;
  }
}

cudaError_t launch_decode_advance(int64_t* st, int64_t count, cudaStream_t s) {
  if (count <= 0) return cudaSuccess;
  decode_advance_kernel<<<static_cast<unsigned>((count + 127) / 128), 128, 0, s>>>(st, count);
  return cudaGetLastError();
}

size_t decode_attn_workspace(int64_t B, int64_t Hq, int64_t capacity, int64_t exact_len, int64_t head_dim) {
  int bd = 16;
  while (bd < head_dim) bd <<= 1;
  const int64_t nchunk = (capacity + exact_len + DEC_KC - 1) / DEC_KC;
  return static_cast<size_t>(B * Hq * (nchunk > 0 ? nchunk : 1) * (bd + 2)) * sizeof(float);
}

cudaError_t launch_decode_attn(int dtype, const void* q, const int64_t* qs, const void* kp, const int64_t* kps,
                               const void* vp, const int64_t* vps, const int32_t* counts, const int64_t* cs,
                               const int32_t* lengths, const int64_t* ls, const void* ke, const int64_t* kes,
                               const void* ve, const int64_t* ves, void* out, const int64_t* os, float sm_scale,
                               int64_t exact_len, int64_t* seq_state, int advance, int64_t W, int64_t G,
                               int64_t B, int64_t Hkv, int64_t head_dim, int64_t capacity, float* part,
                               cudaStream_t st) {
  // advance: the kernels read exact = min(state[0] + 1, W) and the combine step then adds 1 to
  // both lengths (one launch fewer than a separate advance between update and attention)
  const int64_t lag = (seq_state && advance) ? 1 : 0;
  int64_t* adv = lag ? seq_state : nullptr;
  // with a device-resident state the window length is read on the device; `exact_len` is then
  // its bound (the window size) and sizes the split-K grid
  if (B * Hkv == 0) return cudaSuccess;
  if (G < 1 || G > DEC_GMAX) return cudaErrorInvalidValue;
  {
    // tensor-core path: 16-bit types, head_dim 64 / 128, unit head-dim strides, 16-byte rows
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    const bool shape_ok = (dtype == BF16 || dtype == F16) && (head_dim == 64 || head_dim == 128);
    const bool layout_ok = qs[2] == 1 && kps[3] == 1 && vps[3] == 1 && kes[3] == 1 && ves[3] == 1 && a16(kp) &&
                           a16(vp) && a16(ke) && a16(ve) && (kps[0] % 8 | kps[1] % 8 | kps[2] % 8) == 0 &&
                           (vps[0] % 8 | vps[1] % 8 | vps[2] % 8) == 0 && (kes[0] % 8 | kes[1] % 8 | kes[2] % 8) == 0 &&
                           (ves[0] % 8 | ves[1] % 8 | ves[2] % 8) == 0;
    if (shape_ok && layout_ok) {
      int64_t nc = (capacity + exact_len + DEC_VKC - 1) / DEC_VKC;
      if (nc < 1) nc = 1;
      dim3 g2(static_cast<unsigned>(nc), static_cast<unsigned>(B * Hkv));
      auto run = [&](auto tag, auto dd) -> cudaError_t {
        using TY = decltype(tag);
        constexpr int DD = decltype(dd)::value;
        constexpr int SM = decode_mma_smem<DD>();
        // the dynamic shared-memory limit is raised once per instantiation and device
        static std::atomic<uint64_t> attr_set{0};
        int dev = 0;
        cudaError_t ea = cudaGetDevice(&dev);
        if (ea != cudaSuccess) return ea;
        const uint64_t bit = 1ull << (dev & 63);
        if (!(attr_set.load() & bit)) {
          ea = cudaFuncSetAttribute(decode_attn_mma_kernel<TY, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM);
          if (ea != cudaSuccess) return ea;
          attr_set.fetch_or(bit);
        }
        decode_attn_mma_kernel<TY, DD><<<g2, DEC_NW * 32, SM, st>>>(
            static_cast<const TY*>(q), qs[0], qs[1], static_cast<const TY*>(kp), kps[0], kps[1], kps[2],
            static_cast<const TY*>(vp), vps[0], vps[1], vps[2], counts, cs[0], cs[1], cs[2], lengths, ls[0], ls[1],
            static_cast<const TY*>(ke), kes[0], kes[1], kes[2], static_cast<const TY*>(ve), ves[0], ves[1], ves[2],
            sm_scale, exact_len, seq_state, W, lag, static_cast<int>(G), Hkv, nc, part,
            a16(q) && (qs[0] % 8 | qs[1] % 8) == 0);
        const size_t csm = static_cast<size_t>(2 * nc) * sizeof(float);
        if (csm > 48 * 1024) {
          ea = cudaFuncSetAttribute(decode_combine_kernel<TY, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(csm));
          if (ea != cudaSuccess) return ea;
        }
        decode_combine_kernel<TY, DD><<<static_cast<unsigned>(B * Hkv * G), 128, csm, st>>>(
            part, static_cast<TY*>(out), os[0], os[1], os[2], G, Hkv, nc, head_dim, adv);
        return cudaGetLastError();
      };
      using I64 = std::integral_constant<int, 64>;
      using I128 = std::integral_constant<int, 128>;
      if (dtype == BF16) return head_dim == 64 ? run(__nv_bfloat16{}, I64{}) : run(__nv_bfloat16{}, I128{});
      return head_dim == 64 ? run(__half{}, I64{}) : run(__half{}, I128{});
    }
  }
  int bd = 16;
  while (bd < head_dim) bd <<= 1;
  if (bd > 256) return cudaErrorInvalidValue;
  int64_t nchunk = (capacity + exact_len + DEC_KC - 1) / DEC_KC;
  if (nchunk < 1) nchunk = 1;
  dim3 grid(static_cast<unsigned>(nchunk), static_cast<unsigned>(B * Hkv));
  const size_t csm = static_cast<size_t>(2 * nchunk) * sizeof(float);
#define DAB_DEC(TY, N)                                                                                          \
  if (csm > 48 * 1024) {                                                                                        \
    cudaError_t ea = cudaFuncSetAttribute(decode_combine_kernel<TY, N>,                                         \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(csm));  \
    if (ea != cudaSuccess) return ea;                                                                           \
  }                                                                                                             \
  decode_attn_kernel<TY, N><<<grid, 128, 0, st>>>(                                                              \
      static_cast<const TY*>(q), qs[0], qs[1], qs[2], static_cast<const TY*>(kp), kps[0], kps[1], kps[2], kps[3], \
      static_cast<const TY*>(vp), vps[0], vps[1], vps[2], vps[3], counts, cs[0], cs[1], cs[2], lengths, ls[0],  \
      ls[1], static_cast<const TY*>(ke), kes[0], kes[1], kes[2], kes[3], static_cast<const TY*>(ve), ves[0],    \
      ves[1], ves[2], ves[3], sm_scale, exact_len, seq_state, W, lag, G, Hkv, head_dim, nchunk, part);          \
  decode_combine_kernel<TY, N><<<static_cast<unsigned>(B * Hkv * G), 128, csm, st>>>(                           \
      part, static_cast<TY*>(out), os[0], os[1], os[2], G, Hkv, nchunk, head_dim, adv);                         \
  return cudaGetLastError();
#define DAB_DEC_BD(TY)           \
  switch (bd) {                  \
    case 16: DAB_DEC(TY, 16)     \
    case 32: DAB_DEC(TY, 32)     \
    case 64: DAB_DEC(TY, 64)     \
    case 128: DAB_DEC(TY, 128)   \
    default: DAB_DEC(TY, 256)    \
  }
  switch (dtype) {
    case F32: DAB_DEC_BD(float)
    case F16: DAB_DEC_BD(__half)
    case BF16: DAB_DEC_BD(__nv_bfloat16)
    default: return cudaErrorInvalidValue;
  }
#undef DAB_DEC
#undef DAB_DEC_BD
}

}  // namespace dab

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
#include <type_traits>

#include "common.cuh"

namespace dab {

template <typename T, int BD, bool COS>
__global__ void __launch_bounds__(128) decode_update_kernel(
    const T* __restrict__ nk, const T* __restrict__ nv, T* __restrict__ ke, T* __restrict__ ve,
    T* __restrict__ kp, T* __restrict__ vp, int32_t* __restrict__ counts, int32_t* __restrict__ ts,
    int32_t* __restrict__ lengths, int64_t exact_seq_len, int64_t total_seq_len, float thr, int64_t W,
    int64_t ns_b, int64_t ns_h, int64_t ns_s, int64_t ns_d, int64_t es_b, int64_t es_h, int64_t es_s, int64_t es_d,
    int64_t ps_b, int64_t ps_h, int64_t ps_s, int64_t ps_d, int64_t cs_b, int64_t cs_h, int64_t cs_s,
    int64_t num_heads, int64_t head_dim, int64_t programs, int64_t capacity, int* err) {
  constexpr int NH = BD > 128 ? 2 : 1;
  constexpr int PER = BD / 8 / NH;
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  const int64_t pid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pid >= programs) return;
  const int64_t b = pid / num_heads, h = pid % num_heads;
  const int64_t w = exact_seq_len % W;
  T* ek = ke + b * es_b + h * es_h + w * es_s;
  T* ev = ve + b * es_b + h * es_h + w * es_s;
  T* pk = kp + b * ps_b + h * ps_h;
  T* pv = vp + b * ps_b + h * ps_h;
  int32_t* cb = counts + b * cs_b + h * cs_h;
  int32_t* tb = ts + b * cs_b + h * cs_h;
  const int32_t plen = lengths[pid];
  if (exact_seq_len >= W) {
    bool merge = false;
    if (plen > 0) {
      const T* lk = pk + static_cast<int64_t>(plen - 1) * ps_s;
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
      if (lane == 0) cb[static_cast<int64_t>(plen - 1) * cs_s] += 1;
    } else if (plen < capacity) {
      T* dk = pk + static_cast<int64_t>(plen) * ps_s;
      T* dv = pv + static_cast<int64_t>(plen) * ps_s;
      for (int64_t d = lane; d < head_dim; d += 32) {
        dk[d * ps_d] = ek[d * es_d];
        dv[d * ps_d] = ev[d * es_d];
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
  __syncwarp();
  const T* sk = nk + b * ns_b + h * ns_h;
  const T* sv = nv + b * ns_b + h * ns_h;
  for (int64_t d = lane; d < head_dim; d += 32) {
    ek[d * es_d] = sk[d * ns_d];
    ev[d * es_d] = sv[d * ns_d];
  }
}

cudaError_t launch_decode_update(int dtype, int bd, bool cosine, const void* nk, const void* nv, void* ke,
                                 void* ve, void* kp, void* vp, int32_t* counts, int32_t* ts, int32_t* lengths,
                                 int64_t exact_seq_len, int64_t total_seq_len, float thr, int64_t W,
                                 const int64_t* ns, const int64_t* es, const int64_t* ps, const int64_t* cs,
                                 int64_t num_heads, int64_t head_dim, int64_t programs, int64_t capacity, int* err,
                                 cudaStream_t st) {
  if (programs <= 0) return cudaSuccess;
  if (W <= 0) return cudaErrorInvalidValue;
  const unsigned blocks = static_cast<unsigned>((programs + 3) / 4);
#define DAB_UPD(TY, N, C)                                                                                     \
  decode_update_kernel<TY, N, C><<<blocks, 128, 0, st>>>(                                                     \
      static_cast<const TY*>(nk), static_cast<const TY*>(nv), static_cast<TY*>(ke), static_cast<TY*>(ve),      \
      static_cast<TY*>(kp), static_cast<TY*>(vp), counts, ts, lengths, exact_seq_len, total_seq_len, thr, W,   \
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
    int64_t ves_n, int64_t ves_d, float sm_scale, int64_t exact_len, int64_t G, int64_t Hkv, int64_t head_dim,
    int64_t nchunk, float* __restrict__ part) {
  __shared__ float sq[DEC_GMAX][BD];
  __shared__ float sp[DEC_GMAX][DEC_KC];
  __shared__ float swm[4][DEC_GMAX];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = blockIdx.x;
  const int64_t bk = blockIdx.y;
  const int64_t b = bk / Hkv, hk = bk % Hkv;
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
                                                             int64_t Hkv, int64_t nchunk, int64_t head_dim) {
  // four warps take every fourth chunk, so the partials stream in parallel; a shared-memory
  // step merges the four running sums
  __shared__ float sm[4], sl[4];
  __shared__ float sacc[4][BD];
  const int64_t bh = blockIdx.x;  // (b, q-head)
  const int64_t Hq = Hkv * G;
  const int64_t b = bh / Hq, h = bh % Hq;
  const int64_t hk = h / G, g = h % G;
  const int64_t bk = b * Hkv + hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = part + (bk * nchunk * G + g) * (BD + 2);
  const int64_t cstride = G * (BD + 2);
  float m = -INFINITY;
  for (int64_t c = warp; c < nchunk; c += 4) m = fmaxf(m, base[c * cstride]);
  if (lane == 0) sm[warp] = m;
  __syncthreads();
  m = fmaxf(fmaxf(sm[0], sm[1]), fmaxf(sm[2], sm[3]));
  const float ref = (m == -INFINITY) ? 0.f : m;
  float l = 0.f;
  float acc[BD / 32 > 0 ? BD / 32 : 1];
#pragma unroll
  for (int j = 0; j < (BD / 32 > 0 ? BD / 32 : 1); ++j) acc[j] = 0.f;
  for (int64_t c = warp; c < nchunk; c += 4) {
    const float* pc = base + c * cstride;
    const float mc = pc[0];
    if (mc == -INFINITY) continue;
    const float f = expf(mc - ref);
    l = fmaf(pc[1], f, l);
#pragma unroll
    for (int j = 0; j < (BD / 32 > 0 ? BD / 32 : 1); ++j) {
      const int d = j * 32 + lane;
      if (d < head_dim) acc[j] = fmaf(pc[2 + d], f, acc[j]);
    }
  }
  if (lane == 0) sl[warp] = l;
#pragma unroll
  for (int j = 0; j < (BD / 32 > 0 ? BD / 32 : 1); ++j) {
    const int d = j * 32 + lane;
    if (d < BD) sacc[warp][d] = acc[j];
  }
  __syncthreads();
  const float lt = (sl[0] + sl[1]) + (sl[2] + sl[3]);
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    const float a = (sacc[0][d] + sacc[1][d]) + (sacc[2][d] + sacc[3][d]);
    out[b * os_b + h * os_h + d * os_d] = from_f32<T>(a / lt);
  }
}

// Vectorised split-K decode for 16-bit types with unit head-dim strides: a CTA (4 warps)
// scores 128 keys of one (batch, kv-head) for all G q-heads. QK: each lane owns one key and
// reads its row with 16-byte loads; PV: each warp reads whole V rows (every lane 8 bytes of a
// row, coalesced) for its 32 keys. Per-warp partial O are summed in shared memory.
constexpr int DEC_VKC = 128;
template <typename T, int D, int G>
__global__ void __launch_bounds__(128) decode_attn_vec_kernel(
    const T* __restrict__ q, int64_t qs_b, int64_t qs_h, const T* __restrict__ kp, int64_t kps_b, int64_t kps_h,
    int64_t kps_n, const T* __restrict__ vp, int64_t vps_b, int64_t vps_h, int64_t vps_n,
    const int32_t* __restrict__ counts, int64_t cs_b, int64_t cs_h, int64_t cs_n, const int32_t* __restrict__ lengths,
    int64_t ls_b, int64_t ls_h, const T* __restrict__ ke, int64_t kes_b, int64_t kes_h, int64_t kes_n,
    const T* __restrict__ ve, int64_t ves_b, int64_t ves_h, int64_t ves_n, float sm_scale, int64_t exact_len,
    int64_t Hkv, int64_t nchunk, float* __restrict__ part) {
  constexpr int NW = DEC_VKC / 32;
  constexpr int VE = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte load
  constexpr int PL = D / 32;                            // head-dim elements per lane in PV
  __shared__ float sq[G][D];
  __shared__ float sp[G][DEC_VKC];
  __shared__ float swm[NW][G], swl[NW][G];
  __shared__ float so[NW][G][D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t chunk = blockIdx.x;
  const int64_t bk = blockIdx.y;
  const int64_t b = bk / Hkv, hk = bk % Hkv;
  const int64_t plen = lengths[b * ls_b + hk * ls_h];
  const int64_t total = plen + exact_len;
  const int64_t k0 = chunk * DEC_VKC;
  float* pout = part + ((bk * nchunk + chunk) * G) * (D + 2);
  if (k0 >= total) {
    if (tid < G) { pout[tid * (D + 2)] = -INFINITY; pout[tid * (D + 2) + 1] = 0.f; }
    return;
  }
  for (int i = tid; i < G * D; i += DEC_VKC) sq[i / D][i % D] = to_f32(q[b * qs_b + (hk * G + i / D) * qs_h + i % D]);
  __syncthreads();
  // ---- scores: this lane's key
  const int64_t key = k0 + warp * 32 + lane;
  const bool valid = key < total;
  const bool packed = key < plen;
  float s[G];
#pragma unroll
  for (int g = 0; g < G; ++g) s[g] = 0.f;
  if (valid) {
    const T* kr = packed ? kp + b * kps_b + hk * kps_h + key * kps_n : ke + b * kes_b + hk * kes_h + (key - plen) * kes_n;
    // the whole row is requested before any of it is used (one memory round trip per key)
    union { uint4 u; T e[VE]; } raw[D / VE];
#pragma unroll
    for (int v = 0; v < D / VE; ++v) raw[v].u = __ldg(reinterpret_cast<const uint4*>(kr) + v);
#pragma unroll
    for (int v = 0; v < D / VE; ++v) {
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        const float kv = to_f32(raw[v].e[e]);
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = fmaf(sq[g][v * VE + e], kv, s[g]);
      }
    }
  }
  const float bias = (valid && packed) ? logf(static_cast<float>(counts[b * cs_b + hk * cs_h + key * cs_n])) : 0.f;
  // each warp runs its own softmax over its 32 keys (no CTA-wide step between QK and PV, so
  // one warp's V loads overlap another warp's K loads); the CTA merges the warps at the end
  float mw[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    s[g] = valid ? s[g] * sm_scale + bias : -INFINITY;
    float m = s[g];
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    mw[g] = m;
    const float ref = (m == -INFINITY) ? 0.f : m;
    const float pv = valid ? expf(s[g] - ref) : 0.f;
    sp[g][warp * 32 + lane] = round_as<T>(pv);  // P is cast to V's dtype before the PV product
    float l = pv;
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane == 0) { swm[warp][g] = m; swl[warp][g] = l; }
  }
  __syncwarp();
  // ---- PV over this warp's 32 keys: lane owns head-dim elements [lane * PL, lane * PL + PL)
  float o[G][PL];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < PL; ++e) o[g][e] = 0.f;
  const int64_t kw = k0 + warp * 32;
  const int nk = static_cast<int>((total - kw) < 32 ? (total - kw) : 32);
  // all of this warp's V rows are requested first (rows past the end read row 0, weighted 0)
  using VU = typename std::conditional<PL == 4, uint2, uint32_t>::type;
  union { VU u; T e[PL]; } vraw[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int64_t kk = (j < nk) ? kw + j : 0;
    const T* vr = (kk < plen) ? vp + b * vps_b + hk * vps_h + kk * vps_n : ve + b * ves_b + hk * ves_h + (kk - plen) * ves_n;
    vraw[j].u = __ldg(reinterpret_cast<const VU*>(vr + lane * PL));
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float pj = (j < nk) ? sp[g][warp * 32 + j] : 0.f;
#pragma unroll
      for (int e = 0; e < PL; ++e) o[g][e] = fmaf(pj, to_f32(vraw[j].e[e]), o[g][e]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < PL; ++e) so[warp][g][lane * PL + e] = o[g][e];
  __syncthreads();
  // merge the warps: reference = the chunk maximum, each warp's partial scaled to it
  for (int i = tid; i < G * D; i += DEC_VKC) {
    const int g = i / D, d = i % D;
    float M = swm[0][g];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, swm[w][g]);
    float acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w)
        if (swm[w][g] != -INFINITY) acc = fmaf(so[w][g][d], expf(swm[w][g] - M), acc);
    }
    pout[g * (D + 2) + 2 + d] = acc;
  }
  if (tid < G) {
    float M = swm[0][tid];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, swm[w][tid]);
    float l = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w)
        if (swm[w][tid] != -INFINITY) l = fmaf(swl[w][tid], expf(swm[w][tid] - M), l);
    }
    pout[tid * (D + 2)] = M;
    pout[tid * (D + 2) + 1] = l;
  }
  (void)mw;
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
                               int64_t exact_len, int64_t G, int64_t B, int64_t Hkv, int64_t head_dim,
                               int64_t capacity, float* part, cudaStream_t st) {
  if (B * Hkv == 0) return cudaSuccess;
  if (G < 1 || G > DEC_GMAX) return cudaErrorInvalidValue;
  {
    // vectorised path: 16-bit types, head_dim 64 / 128, unit head-dim strides, 16-byte rows
    auto a16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    const bool shape_ok = (dtype == BF16 || dtype == F16) && (head_dim == 64 || head_dim == 128) &&
                          (G == 1 || G == 2 || G == 4 || G == 8);
    const bool layout_ok = qs[2] == 1 && kps[3] == 1 && vps[3] == 1 && kes[3] == 1 && ves[3] == 1 && a16(kp) &&
                           a16(vp) && a16(ke) && a16(ve) && (kps[0] % 8 | kps[1] % 8 | kps[2] % 8) == 0 &&
                           (vps[0] % 8 | vps[1] % 8 | vps[2] % 8) == 0 && (kes[0] % 8 | kes[1] % 8 | kes[2] % 8) == 0 &&
                           (ves[0] % 8 | ves[1] % 8 | ves[2] % 8) == 0 && (reinterpret_cast<uintptr_t>(vp) & 7) == 0;
    if (shape_ok && layout_ok) {
      int64_t nc = (capacity + exact_len + DEC_VKC - 1) / DEC_VKC;
      if (nc < 1) nc = 1;
      dim3 g2(static_cast<unsigned>(nc), static_cast<unsigned>(B * Hkv));
#define DAB_DECV(TY, DD, GG)                                                                                       decode_attn_vec_kernel<TY, DD, GG><<<g2, DEC_VKC, 0, st>>>(                                                             static_cast<const TY*>(q), qs[0], qs[1], static_cast<const TY*>(kp), kps[0], kps[1], kps[2],                    static_cast<const TY*>(vp), vps[0], vps[1], vps[2], counts, cs[0], cs[1], cs[2], lengths, ls[0], ls[1],         static_cast<const TY*>(ke), kes[0], kes[1], kes[2], static_cast<const TY*>(ve), ves[0], ves[1], ves[2],         sm_scale, exact_len, Hkv, nc, part);                                                                         decode_combine_kernel<TY, DD><<<static_cast<unsigned>(B * Hkv * GG), 128, 0, st>>>(                                part, static_cast<TY*>(out), os[0], os[1], os[2], GG, Hkv, nc, head_dim);                                    return cudaGetLastError();
#define DAB_DECV_G(TY, DD) \
  switch (G) {             \
    case 1: DAB_DECV(TY, DD, 1) \
    case 2: DAB_DECV(TY, DD, 2) \
    case 4: DAB_DECV(TY, DD, 4) \
    default: DAB_DECV(TY, DD, 8) \
  }
#define DAB_DECV_D(TY)                         \
  if (head_dim == 64) { DAB_DECV_G(TY, 64) } \
  else { DAB_DECV_G(TY, 128) }
      if (dtype == BF16) { DAB_DECV_D(__nv_bfloat16) } else { DAB_DECV_D(__half) }
#undef DAB_DECV_D
#undef DAB_DECV_G
#undef DAB_DECV
    }
  }
  int bd = 16;
  while (bd < head_dim) bd <<= 1;
  if (bd > 256) return cudaErrorInvalidValue;
  int64_t nchunk = (capacity + exact_len + DEC_KC - 1) / DEC_KC;
  if (nchunk < 1) nchunk = 1;
  dim3 grid(static_cast<unsigned>(nchunk), static_cast<unsigned>(B * Hkv));
#define DAB_DEC(TY, N)                                                                                          \
  decode_attn_kernel<TY, N><<<grid, 128, 0, st>>>(                                                              \
      static_cast<const TY*>(q), qs[0], qs[1], qs[2], static_cast<const TY*>(kp), kps[0], kps[1], kps[2], kps[3], \
      static_cast<const TY*>(vp), vps[0], vps[1], vps[2], vps[3], counts, cs[0], cs[1], cs[2], lengths, ls[0],  \
      ls[1], static_cast<const TY*>(ke), kes[0], kes[1], kes[2], kes[3], static_cast<const TY*>(ve), ves[0],    \
      ves[1], ves[2], ves[3], sm_scale, exact_len, G, Hkv, head_dim, nchunk, part);                             \
  decode_combine_kernel<TY, N><<<static_cast<unsigned>(B * Hkv * G), 128, 0, st>>>(                             \
      part, static_cast<TY*>(out), os[0], os[1], os[2], G, Hkv, nchunk, head_dim);                              \
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

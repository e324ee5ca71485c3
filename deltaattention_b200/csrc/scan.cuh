// Device helpers of the speculative delta scan, shared by the scan kernel (select.cu) and the
// fused key-compression kernel (compress.cu): cp.async staging, the reference-order distance
// of one staged row against the anchor (tritonModules.py:40-60), and the round constants.
#pragma once
#include <type_traits>

#include "common.cuh"

namespace dab {

constexpr int SPEC_W = 8;       // candidates per round (4 lanes each)
constexpr int SPEC_RING = 64;   // rows in the ring
constexpr int SPEC_LA = 5;      // batches requested beyond the one a round reads (<= ring batches - 2)
// chains per CTA, one per warp (one per SM sub-partition); two when rows are wider than 512 B so
// that the rings fit in shared memory
template <typename T, int BD>
constexpr int spec_warps() { return BD * static_cast<int>(sizeof(T)) <= 512 ? 4 : 2; }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// elements e and e + 1 of a staged row (e even), one shared-memory load
template <typename T>
__device__ __forceinline__ float2 load_pair(const uint8_t* row, int e) {
  if constexpr (sizeof(T) == 4) {
    return *reinterpret_cast<const float2*>(row + e * 4);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + e * 2);
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(row + e * 2));
  }
}

__device__ __forceinline__ float2 fneg2(float2 v) { return make_float2(-v.x, -v.y); }

// levels 2 and 3 of the pairwise tree across the four lanes of a candidate (level 1 is the
// lane's own pair sum)
__device__ __forceinline__ float spec_tree(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
  v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
  return v;
}

// One candidate row against the anchor. Euclid: `aw` holds the anchor's 16-bit pairs as raw
// words, or (fp32) `an` the NEGATED anchor pairs. Cosine: `an` holds the anchor and `rr` its
// finished squared norm, which depends on the anchor alone.
// 16-bit Euclid: round(x - a) and round(d * d) as one packed 16-bit sub / mul. Both equal
// the fp32 operation followed by rounding to T: d * d is exact in fp32, and x - a is either
// exact in fp32 or (exponents more than 15 / 12 apart for bf16 / fp16) so close to x that
// neither rounding moves it off x's nearest value.
template <typename T>
struct Packed16;
template <>
struct Packed16<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ float2 sq_diff(uint32_t x, uint32_t a) {
    const T2 d = __hsub2(*reinterpret_cast<const T2*>(&x), *reinterpret_cast<const T2*>(&a));
    return __bfloat1622float2(__hmul2(d, d));
  }
};
template <>
struct Packed16<__half> {
  using T2 = __half2;
  static __device__ __forceinline__ float2 sq_diff(uint32_t x, uint32_t a) {
    const T2 d = __hsub2(*reinterpret_cast<const T2*>(&x), *reinterpret_cast<const T2*>(&a));
    return __half22float2(__hmul2(d, d));
  }
};

template <typename T, int BD, bool COS>
__device__ __forceinline__ bool spec_decide(const uint8_t* row, const float2 (&an)[BD > 128 ? 2 : 1][BD / 8 / (BD > 128 ? 2 : 1)],
                                            const uint32_t (&aw)[BD > 128 ? 2 : 1][BD / 8 / (BD > 128 ? 2 : 1)],
                                            float rr, int q, float thr) {
  constexpr int NH = BD > 128 ? 2 : 1;
  constexpr int PER = BD / 8 / NH;
  if constexpr (COS) {
    float dot = 0.f, cc = 0.f;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float2 d = make_float2(0.f, 0.f), c = d;
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        const float2 x = load_pair<T>(row, hh * 128 + 2 * q + 8 * m);
        const float2 pd = fmul2(x, an[hh][m]), pc = fmul2(x, x);
        d = m ? fadd2(d, pd) : pd;
        c = m ? fadd2(c, pc) : pc;
      }
      const float vd = spec_tree(__fadd_rn(d.x, d.y));
      const float vc = spec_tree(__fadd_rn(c.x, c.y));
      dot = hh ? __fadd_rn(dot, vd) : vd;
      cc = hh ? __fadd_rn(cc, vc) : vc;
    }
    const float nc = __fsqrt_rn(__fadd_rn(cc, 1e-8f));
    const float nr = __fsqrt_rn(__fadd_rn(rr, 1e-8f));
    return __fdiv_rn(dot, __fmul_rn(nc, nr)) < thr;
  } else {
    float tot = 0.f;
#pragma unroll
    for (int hh = 0; hh < NH; ++hh) {
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        const int e = hh * 128 + 2 * q + 8 * m;
        float2 sq;
        if constexpr (sizeof(T) == 2) {
          sq = Packed16<T>::sq_diff(*reinterpret_cast<const uint32_t*>(row + e * 2), aw[hh][m]);
        } else {  // fp32: x + (-a) is x - a exactly
          const float2 d = fadd2(load_pair<T>(row, e), an[hh][m]);
          sq = fmul2(d, d);
        }
        acc = m ? fadd2(acc, sq) : sq;
      }
      const float v = spec_tree(__fadd_rn(acc.x, acc.y));
      tot = hh ? __fadd_rn(tot, v) : v;
    }
    return round_as<T>(tot) > thr;
  }
}


}  // namespace dab

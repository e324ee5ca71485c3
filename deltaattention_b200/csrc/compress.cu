// Fused key compression for the threshold ("row" delta) selection: RoPE, the delta scan and
// the packing of one layer's keys in ONE launch, with the packed length left on the device.
//
// The reference runs these as separate steps with a host sync in between:
//   apply_rotary_pos_emb (modeling_llama.py:555, eager, three rounded ops per element),
//   chunked_eval_kernel (tritonModules.py:7-69, launched at modeling_llama.py:635-653),
//   index_map = cumsum(keep) - 1 and M = max(counts).item() (modeling_llama.py:655-656),
//   parallel_scatter_pack_kv_kernel and the counts (tritonModules.py:72-132,
//   modeling_llama.py:658-685).
//
// Here one warp owns one chunk of one (batch, kv-head):
//   1. Raw K rows and their cos / sin rows are staged by 16-byte cp.async copies (one commit
//      group per batch of 8 rows, KC_LA batches ahead). Each batch is rotated in shared memory
//      with the eager rounding sequence of apply_rotary_pos_emb (bit-identical to the RoPE
//      kernel) into a small ring of rotated rows, and written once to the rotated-K output
//      (the attention's dense phase reads it).
//   2. The speculative delta scan (scan.cuh: SPEC_W candidates per round, the reference's
//      summation order) runs on the rotated ring; the rotation of a batch happens just before
//      the first round that reads it. Kept positions go to a per-chunk bitmask (and the
//      int32 keep mask when one is requested).
//   3. The chunk publishes its anchor count, adds up the counts of the head's earlier chunks
//      (a bounded spin on each; chunks take tickets in head-major order, so every chunk waited
//      on has started and its scan does not wait), and writes its anchors' packed rows:
//      rotated K (re-read from L2), V, timestamp and run-length count (every chunk starts
//      with an anchor, so runs end inside the chunk). The head's last chunk writes the head's
//      anchor count and zero rows up to the end of its last 128-row block.
// The workspace header holds the ticket / done counters and an epoch that tags the status
// words of one launch; the launch's last warp resets the counters and advances the epoch,
// so the workspace needs clearing only once (it is reused launch after launch on one stream).
#include "params.cuh"
#include "scan.cuh"

namespace dab {

constexpr int KC_WARPS = 4;       // chunks (warps) per CTA
constexpr int KC_LA = 3;          // batches staged beyond the one being rotated
constexpr int KC_RING = 8 * (KC_LA + 2);  // rows of each staging ring (raw K, cos, sin)
constexpr int KC_ROT = 32;        // rows of the rotated ring (the scan reads at most 2 batches back)
constexpr int KC_MAXCHUNK = 1024; // tokens per chunk the keep bitmask holds
constexpr int KC_HDR = 256;       // workspace header bytes (then one uint64 status word per chunk)

enum : int { ERR_COMPRESS_LOOKBACK = 0x301, ERR_COMPRESS_CAPACITY = 0x302 };


struct CompressHdr {
  int err;
  unsigned ticket, done, epoch;
};

template <int D>
struct KcCfg {
  static constexpr int ROWB = D * 2;
  static constexpr int NCP = ROWB / 16;       // 16-byte pieces per row
  static constexpr int PITCH = ROWB + 16;     // padded pitch (rows 4 banks apart)
  static constexpr int RING = KC_RING * PITCH;
  static constexpr int ROT = KC_ROT * PITCH;
  static constexpr int WARP_SMEM = 3 * RING + ROT + KC_MAXCHUNK / 8;
  static constexpr int SMEM = KC_WARPS * WARP_SMEM;
};

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <typename T, int D, bool COS>
__global__ void __launch_bounds__(KC_WARPS * 32) key_compress_kernel(const __grid_constant__ CompressParams p) {
  using C = KcCfg<D>;
  constexpr int NH = 1;
  constexpr int PER = D / 8;
  constexpr int HALF = D / 2;
  constexpr int QW = HALF / 4;  // elements of each half a lane rotates
  extern __shared__ __align__(16) uint8_t kc_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring_x = kc_smem + warp * C::WARP_SMEM;
  uint8_t* ring_c = ring_x + C::RING;
  uint8_t* ring_s = ring_c + C::RING;
  uint8_t* ring_r = ring_s + C::RING;
  uint32_t* bits = reinterpret_cast<uint32_t*>(ring_r + C::ROT);
  CompressHdr* hdr = reinterpret_cast<CompressHdr*>(p.ws);
  uint64_t* status = reinterpret_cast<uint64_t*>(p.ws + KC_HDR);

  unsigned t = 0, ep = 0;
  if (lane == 0) {
    t = atomicAdd(&hdr->ticket, 1u);
    ep = *reinterpret_cast<volatile unsigned*>(&hdr->epoch) + 1u;
  }
  t = __shfl_sync(0xFFFFFFFFu, t, 0);
  ep = __shfl_sync(0xFFFFFFFFu, ep, 0);

  if (t < p.total_chunks) {
    const int bh = static_cast<int>(t) / p.nch, c = static_cast<int>(t) % p.nch;
    const int b = bh / p.H, h = bh % p.H;
    const int start = c * p.chunk;
    const int n = min(p.chunk, p.N - start);
    const int nbatch = (n + 7) >> 3;
    const uint8_t* xsrc = reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.k) + b * p.ks_b + h * p.ks_h +
                                                           static_cast<int64_t>(start) * p.ks_s);
    const uint8_t* csrc = reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.cos) + b * p.cs_b +
                                                           static_cast<int64_t>(start) * p.cs_s);
    const uint8_t* ssrc = reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.sin) + b * p.cs_b +
                                                           static_cast<int64_t>(start) * p.cs_s);
    const int64_t xrs = p.ks_s * 2, crs = p.cs_s * 2;  // row strides in bytes
    T* rdst = static_cast<T*>(p.k_rot) + b * p.rs_b + h * p.rs_h + static_cast<int64_t>(start) * p.rs_s;
    int32_t* krow = p.keep ? p.keep + b * p.km_b + h * p.km_h + static_cast<int64_t>(start) * p.km_s : nullptr;
    bits[lane] = 0u;
    __syncwarp();

    // ---------------- stage + rotate
    int req = 0;  // next batch to request
    auto top_up = [&](int need) {
      for (; req <= need + KC_LA; ++req) {
        if (req < nbatch) {
          for (int k = lane; k < 8 * C::NCP; k += 32) {
            const int r = 8 * req + k / C::NCP;
            const int pc = (k % C::NCP) * 16;
            if (r < n) {
              const int so = (r % KC_RING) * C::PITCH + pc;
              cp_async16(ring_x + so, xsrc + r * xrs + pc);
              cp_async16(ring_c + so, csrc + r * crs + pc);
              cp_async16(ring_s + so, ssrc + r * crs + pc);
            }
          }
        }
        cp_async_commit();
      }
    };
    int rot = 0;  // next batch to rotate
    auto rotate_through = [&](int need) {
      while (rot <= need && rot < nbatch) {
        top_up(rot);
        cp_async_wait<KC_LA>();  // every group through batch `rot` has landed
        __syncwarp();
        const int r = 8 * rot + (lane >> 2);
        if (r < n) {
          const int q = lane & 3;
          const uint8_t* rx = ring_x + (r % KC_RING) * C::PITCH;
          const uint8_t* rc = ring_c + (r % KC_RING) * C::PITCH;
          const uint8_t* rs = ring_s + (r % KC_RING) * C::PITCH;
          uint8_t* rr = ring_r + (r % KC_ROT) * C::PITCH;
          uint8_t* gr = reinterpret_cast<uint8_t*>(rdst + static_cast<int64_t>(r) * p.rs_s);
          union Vec { uint4 u; T e[8]; };
#pragma unroll
          for (int v0 = 0; v0 < QW; v0 += 8) {
            const int i = q * QW + v0;
            Vec x1, x2, c1, c2, s1, s2, o1, o2;
            x1.u = *reinterpret_cast<const uint4*>(rx + i * 2);
            x2.u = *reinterpret_cast<const uint4*>(rx + (i + HALF) * 2);
            c1.u = *reinterpret_cast<const uint4*>(rc + i * 2);
            c2.u = *reinterpret_cast<const uint4*>(rc + (i + HALF) * 2);
            s1.u = *reinterpret_cast<const uint4*>(rs + i * 2);
            s2.u = *reinterpret_cast<const uint4*>(rs + (i + HALF) * 2);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              // apply_rotary_pos_emb: x*cos + rotate_half(x)*sin, each op rounded to T
              const float a1 = to_f32(x1.e[e]), a2 = to_f32(x2.e[e]);
              o1.e[e] = from_f32<T>(__fadd_rn(round_as<T>(__fmul_rn(a1, to_f32(c1.e[e]))),
                                              round_as<T>(__fmul_rn(-a2, to_f32(s1.e[e])))));
              o2.e[e] = from_f32<T>(__fadd_rn(round_as<T>(__fmul_rn(a2, to_f32(c2.e[e]))),
                                              round_as<T>(__fmul_rn(a1, to_f32(s2.e[e])))));
            }
            *reinterpret_cast<uint4*>(rr + i * 2) = o1.u;
            *reinterpret_cast<uint4*>(rr + (i + HALF) * 2) = o2.u;
            *reinterpret_cast<uint4*>(gr + i * 2) = o1.u;
            *reinterpret_cast<uint4*>(gr + (i + HALF) * 2) = o2.u;
          }
        }
        __syncwarp();
        ++rot;
      }
    };

    // ---------------- speculative delta scan on the rotated rows
    const int cand = lane >> 2;  // candidate of this lane
    const int q = lane & 3;      // its accumulators: 2q and 2q + 1
    float2 an[NH][PER];
    uint32_t aw[NH][PER];
    float rr = 0.f;
    auto load_anchor = [&](int r) {
      const uint8_t* row = ring_r + (r % KC_ROT) * C::PITCH;
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int m = 0; m < PER; ++m) {
        if constexpr (!COS) {
          aw[0][m] = *reinterpret_cast<const uint32_t*>(row + (2 * q + 8 * m) * 2);
        } else {
          const float2 y = load_pair<T>(row, 2 * q + 8 * m);
          an[0][m] = y;
          const float2 pr = fmul2(y, y);
          acc = m ? fadd2(acc, pr) : pr;
        }
      }
      if constexpr (COS) rr = spec_tree(__fadd_rn(acc.x, acc.y));
    };
    rotate_through(0);
    load_anchor(0);
    if (lane == 0) {
      bits[0] = 1u;
      if (krow) krow[0] = 1;
    }
    int count = 1;
    int pos = 1;  // first undecided row
    while (pos < n) {
      const int hi = min(pos + SPEC_W - 1, n - 1);
      rotate_through(hi >> 3);
      const bool valid = pos + cand < n;
      const int r = valid ? pos + cand : n - 1;
      const bool kp = spec_decide<T, D, COS>(ring_r + (r % KC_ROT) * C::PITCH, an, aw, rr, q, p.thr);
      const unsigned kb = __ballot_sync(0xFFFFFFFFu, kp && valid) & 0x11111111u;
      const int first = kb ? (__ffs(kb) - 1) >> 2 : SPEC_W;
      if (krow && q == 0 && valid && cand <= first) krow[static_cast<int64_t>(pos + cand) * p.km_s] = cand == first;
      if (first < SPEC_W) {
        const int kpos = pos + first;
        if (lane == 0) bits[kpos >> 5] |= 1u << (kpos & 31);
        ++count;
        load_anchor(kpos);
        pos = kpos + 1;
      } else {
        pos += SPEC_W;
      }
      __syncwarp();
    }
    cp_async_wait<0>();
    __syncwarp();

    // ---------------- packed offset: anchors of the head's earlier chunks
    if (lane == 0) st_relaxed_u64(status + t, (static_cast<uint64_t>(ep) << 32) | static_cast<uint32_t>(count));
    int base = 0;
    const uint64_t* hs = status + (t - c);  // chunk 0 of this head
    for (int i = lane; i < c; i += 32) {
      uint64_t w = ld_relaxed_u64(hs + i);
      if (static_cast<unsigned>(w >> 32) != ep) {
        const uint64_t t0 = globaltimer();
        while (static_cast<unsigned>(w >> 32) != ep) {
          if (globaltimer() - t0 > DAB_WAIT_TIMEOUT_NS) {
            atomicCAS(&hdr->err, 0, static_cast<int>(ERR_COMPRESS_LOOKBACK));
            w = 0;
            break;
          }
          __nanosleep(200);
          w = ld_relaxed_u64(hs + i);
        }
      }
      base += static_cast<int>(static_cast<uint32_t>(w));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) base += __shfl_xor_sync(0xFFFFFFFFu, base, o);
    const bool last_chunk = c == p.nch - 1;
    if (last_chunk && lane == 0) p.anchors[bh] = base + count;
    if (base + count > p.cap && lane == 0) atomicCAS(&hdr->err, 0, static_cast<int>(ERR_COMPRESS_CAPACITY));

    // ---------------- anchor positions (the staging ring is free now)
    int32_t* apos = reinterpret_cast<int32_t*>(ring_x);
    const int nwords = (n + 31) >> 5;
    const uint32_t wb = lane < nwords ? bits[lane] : 0u;
    const int pcnt = __popc(wb);
    int incl = pcnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    int off = incl - pcnt;
    for (uint32_t m = wb; m; m &= m - 1) apos[off++] = lane * 32 + __ffs(m) - 1;
    __syncwarp();

    // ---------------- packed rows: timestamps, run lengths, rotated K and V
    int32_t* tsr = p.ts + b * p.ms_b + h * p.ms_h;
    int32_t* cnr = p.cnt + b * p.ms_b + h * p.ms_h;
    float* cfr = p.cnt_f ? p.cnt_f + b * p.ms_b + h * p.ms_h : nullptr;
    for (int i = lane; i < count; i += 32) {
      const int j = base + i;
      if (j >= p.cap) continue;
      const int s = apos[i];
      const int nx = (i + 1 < count) ? apos[i + 1] : n;
      tsr[j] = start + s;
      cnr[j] = nx - s;
      if (cfr) cfr[j] = static_cast<float>(nx - s);
    }
    const uint8_t* vsrc = reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.v) + b * p.vs_b + h * p.vs_h +
                                                           static_cast<int64_t>(start) * p.vs_s);
    const uint8_t* ksrc = reinterpret_cast<const uint8_t*>(rdst);
    uint8_t* kpd = reinterpret_cast<uint8_t*>(static_cast<T*>(p.kp) + b * p.ps_b + h * p.ps_h);
    uint8_t* vpd = reinterpret_cast<uint8_t*>(static_cast<T*>(p.vp) + b * p.ps_b + h * p.ps_h);
    const int items = count * C::NCP;
    for (int i0 = lane; i0 < items; i0 += 4 * 32) {
      uint4 kr4[4], vr4[4];
      int64_t dst[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = i0 + u * 32;
        dst[u] = -1;
        if (idx < items) {
          const int a = idx / C::NCP, pc = (idx % C::NCP) * 16;
          const int j = base + a;
          if (j < p.cap) {
            const int64_t s = apos[a];
            kr4[u] = *reinterpret_cast<const uint4*>(ksrc + s * p.rs_s * 2 + pc);
            vr4[u] = *reinterpret_cast<const uint4*>(vsrc + s * p.vs_s * 2 + pc);
            dst[u] = static_cast<int64_t>(j) * p.ps_s * 2 + pc;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (dst[u] < 0) continue;
        *reinterpret_cast<uint4*>(kpd + dst[u]) = kr4[u];
        *reinterpret_cast<uint4*>(vpd + dst[u]) = vr4[u];
      }
    }
    // the head's last chunk: zero rows from the head's anchor count to the end of its last
    // 128-row block (the reference's zero-initialised padding, as far as attention reads it)
    if (last_chunk) {
      const int A = base + count;
      const int Z = min(p.cap, (A + 127) & ~127);
      for (int j = A + lane; j < Z; j += 32) {
        tsr[j] = 0;
        cnr[j] = 0;
        if (cfr) cfr[j] = 0.f;
      }
      for (int i = lane; i < (Z - A) * C::NCP; i += 32) {
        const int64_t o = static_cast<int64_t>(A + i / C::NCP) * p.ps_s * 2 + (i % C::NCP) * 16;
        *reinterpret_cast<uint4*>(kpd + o) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vpd + o) = make_uint4(0, 0, 0, 0);
      }
    }
  }

  // ---------------- the launch's last warp resets the counters for the next launch
  if (lane == 0) {
    __threadfence();
    const unsigned d = atomicAdd(&hdr->done, 1u);
    if (d == p.total_warps - 1) {
      hdr->ticket = 0u;
      hdr->done = 0u;
      hdr->epoch = ep;
      __threadfence();
    }
  }
}

template <typename T, int D, bool COS>
static cudaError_t launch_kc_t(const CompressParams& p, cudaStream_t st) {
  using C = KcCfg<D>;
  auto kfn = key_compress_kernel<T, D, COS>;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const unsigned grid = p.total_warps / KC_WARPS;
  kfn<<<grid, KC_WARPS * 32, C::SMEM, st>>>(p);
  return cudaGetLastError();
}

size_t key_compress_workspace(int64_t B, int64_t H, int64_t N, int64_t chunk) {
  const int64_t nch = chunk > 0 ? (N + chunk - 1) / chunk : 0;
  return KC_HDR + static_cast<size_t>(B * H * (nch > 0 ? nch : 1)) * 8;
}

// p.total_chunks / total_warps are filled here; dtype 16-bit, D 64 / 128 (checked by the caller)
cudaError_t launch_key_compress(int dtype, int D, bool cosine, CompressParams p, cudaStream_t st) {
  p.total_warps = ((p.total_chunks + KC_WARPS - 1) / KC_WARPS) * KC_WARPS;
  if (p.total_chunks == 0) return cudaSuccess;
#define DAB_KC(TY, DD)                                                                                 \
  return cosine ? launch_kc_t<TY, DD, true>(p, st) : launch_kc_t<TY, DD, false>(p, st);
  if (dtype == BF16) {
    if (D == 128) { DAB_KC(__nv_bfloat16, 128) }
    if (D == 64) { DAB_KC(__nv_bfloat16, 64) }
  } else if (dtype == F16) {
    if (D == 128) { DAB_KC(__half, 128) }
    if (D == 64) { DAB_KC(__half, 64) }
  }
#undef DAB_KC
  return cudaErrorInvalidValue;
}

}  // namespace dab

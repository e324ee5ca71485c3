// tcgen05 / TMEM attention for the reference's prefill kernels on B200 (sm_100a).
//
// One kernel serves the four reference kernels (deltaFlashAttention.py:9-357 and
// flashAttention.py:5-91) for bf16/fp16 inputs with head_dim 64 or 128 and the
// reference's 128x128 logical blocks. The logical schedule (phase-1 stop rule, dense
// restart block, causal limit) comes from a small pre-pass (`schedule_kernel`), so the
// per-(query block, head) tile list is exactly the reference's.
//
// Structure (persistent, one CTA per SM, 384 threads):
//   warp 0      TMA producer: Q tiles and K tiles into a ring of shared-memory slots
//   warp 3      TMA producer: V tiles (ring), with the packed tile's counts (and timestamps)
//   warps 1, 2  MMA issuers for query tile 0 / 1 (one elected lane each): S = Q K^T into
//               TMEM, O += P V with P read from TMEM; warp 2 also allocates TMEM
//   warps 4-7   softmax + epilogue for query tile 0 (TMEM lanes 0..127, one row per thread)
//   warps 8-11  softmax + epilogue for query tile 1
// A work unit is two 128-row query tiles that share every K/V tile: two q-heads of one
// GQA group at the same query block (kv_group even) or two consecutive query blocks of
// one head. Units run heaviest first (latest query blocks first) in a serpentine static
// order across CTAs. Softmax keeps a stale running max unless it grows by more than 2^8,
// so the O correction pass is rare; O and l share the same reference so O / l is exact.
#include <type_traits>

#include "params.cuh"

namespace dab {

enum TcVariant : int { TC_HYBRID = 0, TC_SANITY = 1, TC_PURE = 2, TC_DENSE = 3, TC_SPARSE = 4 };

constexpr int TC_THREADS = 384;
constexpr int TC_BM = 128;
constexpr int TC_BN = 128;

template <int D> struct TcCfg {
  static constexpr int QBYTES = TC_BM * D * 2;
  static constexpr int KVBYTES = TC_BN * D * 2;
  // separate K and V rings, each with its own producer warp: the K tile of the next block is
  // loaded as soon as QK^T of the block two back completes, independent of V slot releases
  static constexpr int NK = (D == 128) ? 2 : 4;
  static constexpr int NV = (D == 128) ? 2 : 4;
  static constexpr int OFF_Q0 = 0;
  static constexpr int OFF_Q1 = QBYTES;
  static constexpr int OFF_K = 2 * QBYTES;
  static constexpr int OFF_V = OFF_K + NK * KVBYTES;
  static constexpr int OFF_AUXC = OFF_V + NV * KVBYTES;
  static constexpr int OFF_AUXT = OFF_AUXC + NV * TC_BN * 4;
  static constexpr int OFF_ONES = OFF_AUXT + NV * TC_BN * 4;  // 128 unit weights (dense blocks, KEYED)
  static constexpr int OFF_EPI = OFF_ONES + TC_BN * 4;  // per softmax warp: 32 rows x 80 B of output staging
  static constexpr int EPI_PITCH = 80;                  // 64 B of a 32-column chunk + 16 B (no bank conflicts)
  static constexpr int OFF_BAR = OFF_EPI + 8 * 32 * EPI_PITCH;
  static constexpr int NBAR = 2 + 2 * NK + 2 * NV + 2 * 6 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 64 + 1024;  // + alignment slack
};

// ----------------------------------------------------------------------------- schedule
// Per (batch, ts-head): packed-block max timestamps T_j (masked lanes read seq_k + 1), then
// for every query block mb: n1 = first j with T_j >= 128*mb - window, last_safe = T_{n1-1}
// (or -1), dense start block = (last_safe + 1) // 128. Also the smallest valid timestamp of
// every packed block for the pure-phase-1 variant (count > 0 and index < num_packed).
//
// Device packed length (`anchors` non-null): head bh keeps anchors[bh] rows and the packed
// length is M = max over heads (written to len_out[0]); keys in [anchors[bh], M) are the
// reference's zero padding (timestamp 0, count 0) and are scheduled as such without being
// read, keys >= M are the masked lanes. `nblk` is then the capacity in blocks (the row stride
// of blkmin / blkw); only the first ceil(M / 128) blocks are scheduled.
__global__ void __launch_bounds__(256) schedule_kernel(const int32_t* __restrict__ ts, int64_t tsb, int64_t tsh,
                                                       int64_t tsn, const void* counts, int64_t cb, int64_t ch,
                                                       int64_t cn, int counts_is_int, int Hts, int num_packed,
                                                       int seq_k, int window, int nmb, int nblk, int2* sched,
                                                       int32_t* blkmin, int want_blkmin, float* blkw,
                                                       const int32_t* __restrict__ anchors, int nheads_total,
                                                       int* len_out) {
  extern __shared__ int32_t sT[];  // nblk block maxima
  const int bh = blockIdx.x;
  const int b = bh / Hts, h = bh % Hts;
  const int32_t* tsr = ts + b * tsb + h * tsh;
  const int tid = threadIdx.x;
  const int wstride = nblk;  // row stride of blkmin / blkw (the capacity in blocks)
  int nreal = num_packed;  // keys of this head read from memory
  if (anchors) {
    __shared__ int red[8];
    int m = 0;
    for (int i = tid; i < nheads_total; i += blockDim.x) m = max(m, anchors[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = max(m, red[w]);
    num_packed = min(m, num_packed);
    nreal = min(anchors[bh], num_packed);
    nblk = (num_packed + TC_BN - 1) / TC_BN;
    if (bh == 0 && tid == 0) *len_out = num_packed;
  }
  // four threads per packed block, 32 consecutive keys each: every thread requests all of its
  // timestamps and counts before using any (one memory round trip per 64 blocks)
  for (int j0 = 0; j0 < nblk; j0 += 64) {
    const int j = j0 + (tid >> 2);
    const int k0 = j * TC_BN + (tid & 3) * 32;
    int tmax = INT32_MIN, tmin = INT32_MAX;
    float cmin = INFINITY, cmax = -INFINITY;
    if (j < nblk) {
      int tv[32];
      float cv[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int key = k0 + e;
        tv[e] = key < num_packed ? 0 : seq_k + 1;  // zero padding, or a masked lane
        cv[e] = 0.f;
        if (key < nreal) {
          tv[e] = tsr[static_cast<int64_t>(key) * tsn];
          const int64_t off = b * cb + h * ch + static_cast<int64_t>(key) * cn;
          cv[e] = counts_is_int ? static_cast<float>(static_cast<const int32_t*>(counts)[off])
                                : static_cast<const float*>(counts)[off];
        }
      }
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        if (k0 + e < num_packed) {
          if (cv[e] > 0.f) tmin = min(tmin, tv[e]);
          cmin = fminf(cmin, cv[e]);
          cmax = fmaxf(cmax, cv[e]);
        }
        tmax = max(tmax, tv[e]);
      }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      tmax = max(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, o));
      tmin = min(tmin, __shfl_xor_sync(0xFFFFFFFFu, tmin, o));
      cmin = fminf(cmin, __shfl_xor_sync(0xFFFFFFFFu, cmin, o));
      cmax = fmaxf(cmax, __shfl_xor_sync(0xFFFFFFFFu, cmax, o));
    }
    if ((tid & 3) == 0 && j < nblk) {
      sT[j] = tmax;
      if (want_blkmin) blkmin[static_cast<int64_t>(bh) * wstride + j] = tmin;
      // a block whose valid keys share one count c is weighted by adding log2(c) to the
      // exponent (exact for powers of two); mixed counts are applied per key
      blkw[static_cast<int64_t>(bh) * wstride + j] = (cmin == cmax) ? log2f(cmin) : __int_as_float(0x7FC00000);
    }
  }
  __syncthreads();
  for (int mb = threadIdx.x; mb < nmb; mb += blockDim.x) {
    const int thr = mb * TC_BM - window;
    int n1 = 0;
    while (n1 < nblk && sT[n1] < thr) ++n1;
    const int last_safe = n1 ? sT[n1 - 1] : -1;
    const int ds = max(0, (last_safe + 1) / TC_BN);
    sched[static_cast<int64_t>(bh) * nmb + mb] = make_int2(n1, ds);
  }
}

// ----------------------------------------------------------------------------- units
struct Unit {
  int b, hq[2], hts[2], mb[2];
  bool valid[2];
};

__device__ __forceinline__ Unit decode_unit(const TcParams& p, int u) {
  Unit U;
  if (p.pair_heads) {
    const int Hkv = p.Hq / p.kv_group;
    const int npair = p.kv_group / 2;
    const int per_mb = p.B * Hkv * npair;
    const int mb = p.nmb - 1 - u / per_mb;
    const int r = u % per_mb;
    const int bk = r / npair, pr = r % npair;
    U.b = bk / Hkv;
    const int hk = bk % Hkv;
    U.hq[0] = hk * p.kv_group + 2 * pr;
    U.hq[1] = U.hq[0] + 1;
    U.mb[0] = U.mb[1] = mb;
    U.valid[0] = U.valid[1] = true;
  } else {
    const int nmp = (p.nmb + 1) / 2;
    const int per = p.B * p.Hq;
    const int mp = nmp - 1 - u / per;
    const int bh = u % per;
    U.b = bh / p.Hq;
    U.hq[0] = U.hq[1] = bh % p.Hq;
    U.mb[0] = 2 * mp;
    U.mb[1] = 2 * mp + 1;
    U.valid[0] = true;
    U.valid[1] = U.mb[1] < p.nmb;
  }
  U.hts[0] = U.hq[0] / p.kv_group;
  U.hts[1] = U.hq[1] / p.kv_group;
  return U;
}

// Serpentine static assignment: round r covers units [r*G, (r+1)*G); odd rounds reverse.
__device__ __forceinline__ int unit_of(int iter, int cta, int G) {
  const int base = iter * G;
  return (iter & 1) ? base + (G - 1 - cta) : base + cta;
}

// the packed length: the host value, or (device packed length) the maximum of the heads' anchors
// that the schedule pre-pass, the previous launch on this stream, wrote to the workspace
__device__ __forceinline__ int packed_len(const TcParams& p) { return p.anchors ? *p.len_dev : p.num_packed; }

// the two query tiles' (phase-1 blocks, dense start block) entries of the schedule, fetched one
// unit ahead by the MMA and softmax warps so a unit boundary does not wait on the load
struct UnitSched {
  int2 s[2];
};
__device__ __forceinline__ UnitSched fetch_sched(const TcParams& p, const Unit& U) {
  UnitSched us;
  #pragma unroll
  for (int x = 0; x < 2; ++x) {
    us.s[x] = make_int2(0, 0);
    if (U.valid[x] && (p.variant == TC_HYBRID || p.variant == TC_SANITY))
      us.s[x] = __ldg(&p.sched[(static_cast<int64_t>(U.b) * p.Hts + U.hts[x]) * p.nmb + U.mb[x]]);
  }
  return us;
}

struct TileInfo {
  int packed;   // 1: packed block, 0: dense block
  int idx;      // block index (in 128-key blocks)
  int use;      // bit x set: query tile x attends this block
  int needs_v;  // the block's V is loaded and a PV product issued
};

// Enumerates the union of both query tiles' block lists in reference order (all packed
// blocks first, then dense blocks ascending). Every role walks the same sequence.
// SPARSE (DPXA block-sparse attention): the dense key blocks set in each tile's bitmask, up to
// and including its diagonal block, ascending.
template <bool SPARSE>
struct TileSeqT {
  int n1[2], ds[2], de[2];
  int pmax, dlo, dhi;
  int state, cur;  // state 0: packed, 1: dense, 2: done
  int mb_lo[2];
  const uint32_t* mrow[2];  // SPARSE: the tiles' bitmask rows
  int widx;                 // SPARSE: index of the mask word held in wrd
  uint32_t wrd[2];
  __device__ __forceinline__ void init(const TcParams& p, const Unit& U) { init(p, U, fetch_sched(p, U)); }
  __device__ __forceinline__ void init(const TcParams& p, const Unit& U, const UnitSched& us) {
    if constexpr (SPARSE) {
      dlo = 0;
      dhi = 0;
      #pragma unroll
      for (int x = 0; x < 2; ++x) {
        mb_lo[x] = U.mb[x];
        mrow[x] = U.valid[x] ? p.sel + (static_cast<int64_t>(U.b * p.Hts + U.hts[x]) * p.nmb + U.mb[x]) * p.sel_words
                             : nullptr;
        if (U.valid[x]) dhi = max(dhi, U.mb[x] + 1);
      }
      widx = -1;
      wrd[0] = wrd[1] = 0u;
      state = 1;
      cur = 0;
      return;
    }
    const int num_packed = packed_len(p);
    #pragma unroll
    for (int x = 0; x < 2; ++x) {
      n1[x] = 0; ds[x] = 0; de[x] = 0;
      mb_lo[x] = U.mb[x] * TC_BM;
      if (!U.valid[x]) continue;
      const int m0 = U.mb[x] * TC_BM;
      const int hi = min(p.seq_k, m0 + TC_BM);
      if (p.variant == TC_HYBRID || p.variant == TC_SANITY) {
        const int2 s = us.s[x];
        n1[x] = s.x;
        ds[x] = s.y;
        de[x] = (hi + TC_BN - 1) / TC_BN;
      } else if (p.variant == TC_PURE) {
        n1[x] = (num_packed + TC_BN - 1) / TC_BN;
      } else {
        ds[x] = 0;
        de[x] = p.causal ? (hi + TC_BN - 1) / TC_BN : (p.seq_k + TC_BN - 1) / TC_BN;
      }
    }
    const bool v0 = U.valid[0], v1 = U.valid[1];
    pmax = max(v0 ? n1[0] : 0, v1 ? n1[1] : 0);
    // with a device packed length, blocks past the head's own anchors are the reference's zero
    // padding: K = V = 0 and count 0 add nothing to O or l, so they are not loaded or computed
    // (the schedule pre-pass still counts their zero timestamps in the phase-1 stop rule)
    if (p.anchors) pmax = min(pmax, (p.anchors[U.b * p.Hts + U.hts[0]] + TC_BN - 1) / TC_BN);
    dlo = INT32_MAX; dhi = 0;
    #pragma unroll
    for (int x = 0; x < 2; ++x)
      if (U.valid[x] && de[x] > ds[x]) { dlo = min(dlo, ds[x]); dhi = max(dhi, de[x]); }
    if (dlo == INT32_MAX) { dlo = 0; dhi = 0; }
    state = 0;
    cur = 0;
  }

  __device__ __forceinline__ bool next(const TcParams& p, const Unit& U, TileInfo& t) {
    if constexpr (SPARSE) {
      // blocks up to each tile's diagonal (mb_lo holds the query block here), in mask order
      while (cur < dhi) {
        const int w = cur >> 5;
        if (w != widx) {
          widx = w;
          #pragma unroll
          for (int x = 0; x < 2; ++x) wrd[x] = mrow[x] ? __ldg(mrow[x] + w) : 0u;
        }
        const uint32_t any = (wrd[0] | wrd[1]) >> (cur & 31);
        if (!any) { cur = (w + 1) << 5; continue; }
        const int j = cur + __ffs(any) - 1;
        cur = j + 1;
        int use = 0;
        #pragma unroll
        for (int x = 0; x < 2; ++x)
          if (mrow[x] && j <= mb_lo[x] && ((wrd[x] >> (j & 31)) & 1u)) use |= 1 << x;
        if (!use) continue;
        t.packed = 0; t.idx = j; t.use = use; t.needs_v = 1;
        return true;
      }
      state = 2;
      return false;
    } else {
      return next_hybrid(p, U, t);
    }
  }

  __device__ __forceinline__ bool next_hybrid(const TcParams& p, const Unit& U, TileInfo& t) {
    while (state == 0) {
      if (cur >= pmax) { state = 1; cur = dlo; break; }
      const int j = cur++;
      int use = 0;
      #pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (!U.valid[x] || j >= n1[x]) continue;
        if (p.variant == TC_PURE) {
          const int tmin = p.blkmin[(static_cast<int64_t>(U.b) * p.Hts + U.hts[x]) * p.nblk + j];
          if (tmin > mb_lo[x] + TC_BM - 1) continue;  // block masked for every row: no-op
        }
        use |= 1 << x;
      }
      if (!use) continue;
      t.packed = 1; t.idx = j; t.use = use; t.needs_v = (p.variant != TC_SANITY);
      return true;
    }
    if (state == 1) {
      while (cur < dhi) {
        const int tb = cur++;
        int use = 0;
        #pragma unroll
        for (int x = 0; x < 2; ++x)
          if (U.valid[x] && tb >= ds[x] && tb < de[x]) use |= 1 << x;
        if (!use) continue;
        t.packed = 0; t.idx = tb; t.use = use; t.needs_v = 1;
        return true;
      }
      state = 2;
    }
    return false;
  }
};

// every lane of the warp waits; the outcome is made warp-uniform so warp-collective
// tcgen05 instructions that follow stay converged
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t par, const Abort& ab, int code) {
  const bool ok = mbar_wait(bar, par, ab, code);
  return __all_sync(0xFFFFFFFFu, ok);
}


// KEYED: the launch's packed blocks carry per-key counts that differ inside a block (the
// threshold selection's run lengths), given as fp32. The streaming fast path then weights each
// probability by its key's count (a multiply by the count staged with the V tile) instead of
// one per-block exponent offset, so such blocks stay off the exact two-pass path; one copy of
// the unrolled exponential loop either way (dense blocks read unit weights).
template <int D, bool BF16, bool KEYED, bool SPARSE>
__global__ void __launch_bounds__(TC_THREADS, 1) attn_tc_kernel(const __grid_constant__ TcParams p) {
  using C = TcCfg<D>;
  using TileSeq = TileSeqT<SPARSE>;
  constexpr int NK = C::NK, NV = C::NV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;                // [NK]
  uint64_t* k_empty = k_full + NK;            // [NK]
  uint64_t* v_full = k_empty + NK;            // [NV]
  uint64_t* v_empty = v_full + NV;            // [NV]
  uint64_t* s_full = v_empty + NV;            // [2]
  uint64_t* p_full = s_full + 2;              // [2] every P column of the block stored
  uint64_t* p_lo = p_full + 2;                // [2] P of keys 0..63 stored
  uint64_t* o_full = p_lo + 2;                // [2]
  uint64_t* tile_free = o_full + 2;           // [2]
  uint64_t* mma_done = tile_free + 2;
  uint64_t* turn = mma_done + 1;              // [2] MMA warp x finished issuing a batch
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 8);
  float* auxc = reinterpret_cast<float*>(smem + C::OFF_AUXC);
  int32_t* auxt = reinterpret_cast<int32_t*>(smem + C::OFF_AUXT);
  float* ones = reinterpret_cast<float*>(smem + C::OFF_ONES);
  if (KEYED && threadIdx.x < TC_BN) ones[threadIdx.x] = 1.f;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 2);  // one commit per MMA warp
    for (int s = 0; s < NK; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 2);
    }
    for (int s = 0; s < NV; ++s) {
      mbar_init(v_full + s, 1);
      mbar_init(v_empty + s, 2);
    }
    #pragma unroll
    for (int x = 0; x < 2; ++x) {
      mbar_init(s_full + x, 1);
      mbar_init(p_full + x, 4);
      mbar_init(p_lo + x, 4);
      mbar_init(o_full + x, 1);
      mbar_init(tile_free + x, 4);
    }
    mbar_init(mma_done, 2);
    mbar_init(turn + 0, 1);
    mbar_init(turn + 1, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_kd);
    tma_prefetch_desc(&p.tm_vd);
    tma_prefetch_desc(&p.tm_kp);
    tma_prefetch_desc(&p.tm_vp);
  }
  if (warp == 2) {
    tmem_alloc(tmem_base_smem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_smem;
  const Abort ab{abort_flag, p.err};
  const int G = gridDim.x;
  const int n_iter = (p.num_units + G - 1) / G;

  if (warp == 0) {
    // ================================================================ Q + K producer
    uint32_t q_par = 1;
    int kpos = 0, q_issued = 0;  // K ring positions issued so far (the last NK may be in flight)
    for (int it = 0; it < n_iter; ++it) {
      const int u = unit_of(it, blockIdx.x, G);
      if (u >= p.num_units) continue;
      const Unit U = decode_unit(p, u);
      if (!warp_wait(q_empty, q_par, ab, ERR_TIMEOUT_PRODUCER)) goto kprod_done;
      q_par ^= 1;
      if (lane == 0) {
        const uint32_t qb = (U.valid[0] ? C::QBYTES : 0) + (U.valid[1] ? C::QBYTES : 0);
        mbar_arrive_expect_tx(q_full, qb);
        #pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!U.valid[x]) continue;
          uint8_t* dst = smem + (x ? C::OFF_Q1 : C::OFF_Q0);
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_4d(dst + bx * (TC_BM * 128), &p.tm_q, q_full, bx * 64, U.mb[x] * TC_BM, U.hq[x], U.b);
        }
      }
      ++q_issued;
      TileSeq seq;
      seq.init(p, U);
      TileInfo t;
      while (seq.next(p, U, t)) {
        const int slot = kpos % NK;
        if (!warp_wait(k_empty + slot, ((kpos / NK) & 1) ^ 1, ab, ERR_TIMEOUT_PRODUCER)) goto kprod_done;
        if (lane == 0) {
          const CUtensorMap* tk = t.packed ? &p.tm_kp : &p.tm_kd;
          mbar_arrive_expect_tx(k_full + slot, C::KVBYTES);
          uint8_t* dst = smem + C::OFF_K + slot * C::KVBYTES;
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_4d(dst + bx * (TC_BN * 128), tk, k_full + slot, bx * 64, t.idx * TC_BN, U.hts[0], U.b);
        }
        ++kpos;
      }
    }
  kprod_done:
    // drain: every copy this warp issued must land before the CTA exits (bounded; a copy that
    // never lands is reported as ERR_TIMEOUT_DRAIN)
    if (lane == 0) {
      bool drained = true;
      for (int q = (kpos > NK ? kpos - NK : 0); q < kpos && drained; ++q)
        drained = mbar_drain(k_full + q % NK, (q / NK) & 1, p.err);
      if (drained && q_issued > 0) mbar_drain(q_full, (q_issued - 1) & 1, p.err);
    }
  } else if (warp == 3) {
    // ================================================================ V (+ counts) producer
    int vpos = 0;  // V ring positions issued so far (the last NV may be in flight)
    for (int it = 0; it < n_iter; ++it) {
      const int u = unit_of(it, blockIdx.x, G);
      if (u >= p.num_units) continue;
      const Unit U = decode_unit(p, u);
      const int hk = U.hts[0];  // both tiles of a unit share the K/V head
      TileSeq seq;
      seq.init(p, U);
      TileInfo t;
      while (seq.next(p, U, t)) {
        if (!t.needs_v) continue;
        const int slot = vpos % NV;
        if (!warp_wait(v_empty + slot, ((vpos / NV) & 1) ^ 1, ab, ERR_TIMEOUT_PRODUCER)) goto vprod_done;
        uint32_t meta_bytes = 0;
        if (t.packed) {
          // counts (and timestamps) of this packed block ride with its V tile: bulk copies on
          // the same barrier when rows are contiguous and aligned, else lane loads
          float* c = auxc + slot * TC_BN;
          int32_t* tt = auxt + slot * TC_BN;
          // with a device packed length every row of a block the head holds is written (rows
          // past its anchors up to the block end are zeros), so the whole block is copied
          const int nkeys = p.anchors ? TC_BN : min(TC_BN, p.num_packed - t.idx * TC_BN);
          if (p.meta_bulk) {
            meta_bytes = static_cast<uint32_t>(nkeys) * 4u * (p.variant == TC_PURE ? 2u : 1u);
            if (lane == 0) {
              const int64_t off_c = U.b * p.cs_b + static_cast<int64_t>(hk) * p.cs_h + static_cast<int64_t>(t.idx) * TC_BN;
              bulk_load(c, static_cast<const uint32_t*>(p.counts) + off_c, nkeys * 4u, v_full + slot);
              if (p.variant == TC_PURE) {
                const int64_t off_t = U.b * p.ts_b + static_cast<int64_t>(hk) * p.ts_h + static_cast<int64_t>(t.idx) * TC_BN;
                bulk_load(tt, p.ts + off_t, nkeys * 4u, v_full + slot);
              }
            }
          } else {
            for (int e = lane; e < TC_BN; e += 32) {
              const int key = t.idx * TC_BN + e;
              uint32_t cv = 0;
              int32_t tv2 = 0;
              if (p.anchors || key < p.num_packed) {
                const int64_t off = U.b * p.cs_b + static_cast<int64_t>(hk) * p.cs_h + static_cast<int64_t>(key) * p.cs_n;
                cv = static_cast<const uint32_t*>(p.counts)[off];
                if (p.variant == TC_PURE)
                  tv2 = p.ts[U.b * p.ts_b + static_cast<int64_t>(hk) * p.ts_h + static_cast<int64_t>(key) * p.ts_n];
              }
              reinterpret_cast<uint32_t*>(c)[e] = cv;
              tt[e] = tv2;
            }
            __syncwarp();
          }
        }
        if (lane == 0) {
          const CUtensorMap* tv = t.packed ? &p.tm_vp : &p.tm_vd;
          mbar_arrive_expect_tx(v_full + slot, C::KVBYTES + meta_bytes);
          uint8_t* dst = smem + C::OFF_V + slot * C::KVBYTES;
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_4d(dst + bx * (TC_BN * 128), tv, v_full + slot, bx * 64, t.idx * TC_BN, hk, U.b);
        }
        ++vpos;
      }
    }
  vprod_done:
    if (lane == 0) {
      bool drained = true;
      for (int q = (vpos > NV ? vpos - NV : 0); q < vpos && drained; ++q)
        drained = mbar_drain(v_full + q % NV, (q / NV) & 1, p.err);
    }
  } else if (warp == 1 || warp == 2) {
    // ================================================================ MMA issuers
    // One warp per query tile: warp 1 issues tile 0's MMAs, warp 2 tile 1's. Issuing tcgen05.mma
    // slows the other warps on the issuing warp's scheduler (the softmax warps of lane quarter
    // 1 ran ~300 cycles per block behind the others with one issuer for both tiles), so the
    // load is split over two schedulers. The tiles use disjoint TMEM columns, so the two issue
    // streams need no ordering between them; the K / V / Q slot releases take one commit from
    // each warp (barrier counts of 2). Both warps wait on every K / V fill they release, even
    // for blocks their tile skips, so a warp can never arrive for a later fill of a slot.
    // The two warps issue their batches (a block's PV plus the next block's S) strictly in
    // turn, tile 0 first, through the `turn` barriers: the tensor pipe then finishes tile 0's
    // S about one batch before tile 1's, and the two tiles' softmax passes stay half a period
    // apart instead of locking in phase and sharing the exponential unit.
    // Each warp runs converged (waits are warp-uniform) and the tcgen05 helpers issue from one
    // elected lane, which keeps descriptors and TMEM addresses warp-uniform.
    {
      const int x = warp - 1;
      constexpr uint32_t IDESC_S = umma_idesc_f16(TC_BM, TC_BN, BF16, false);
      constexpr uint32_t IDESC_PV = umma_idesc_f16(TC_BM, D, BF16, true);
      const uint32_t tS = tmem + 128 * x;
      const uint32_t tO = tmem + 256 + D * x;
      // shared-memory descriptors as base + constant: the start-address field (bits 0-13, in
      // 16-byte units) of every operand is the base's plus a fixed offset
      const uint64_t qdesc = umma_desc_sw128(smem_u32(smem + (x ? C::OFF_Q1 : C::OFF_Q0)), 16, 1024);
      const uint64_t kdesc0 = umma_desc_sw128(smem_u32(smem + C::OFF_K), 16, 1024);
      const uint64_t vdesc0 = umma_desc_sw128(smem_u32(smem + C::OFF_V), TC_BN * 128, 1024);
      const bool sanity = p.variant == TC_SANITY;
      int kpos = 0, vpos = 0;  // K / V ring positions
      uint32_t q_par = 0, free_par = 1, p_par = 0;
      uint32_t nbatch = 0;  // batches this warp has issued
      bool aborted = false;
      // before batch k: tile 1 waits for tile 0's batch k, tile 0 for tile 1's batch k-1
      auto my_turn = [&]() -> bool {
        if (x == 1) return warp_wait(turn + 0, nbatch & 1, ab, ERR_TIMEOUT_MMA);
        return nbatch == 0 || warp_wait(turn + 1, (nbatch - 1) & 1, ab, ERR_TIMEOUT_MMA);
      };
      auto end_turn = [&]() {
        __syncwarp();
        if (lane == 0) mbar_arrive(turn + x);
        ++nbatch;
      };
      UnitSched us_next{};
      bool us_have = false;
      for (int it = 0; it < n_iter && !aborted; ++it) {
        const int u = unit_of(it, blockIdx.x, G);
        if (u >= p.num_units) continue;
        const Unit U = decode_unit(p, u);
        const UnitSched us = us_have ? us_next : fetch_sched(p, U);
        {
          const int un = unit_of(it + 1, blockIdx.x, G);
          us_have = it + 1 < n_iter && un < p.num_units;
          if (us_have) us_next = fetch_sched(p, decode_unit(p, un));
        }
        const bool mine = x ? U.valid[1] : U.valid[0];
        if (!warp_wait(q_full, q_par, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
        q_par ^= 1;
        tc_fence_after();
        bool freed = false, o_init = false;
        auto ensure_free = [&]() -> bool {
          if (freed) return true;
          if (!warp_wait(tile_free + x, free_par, ab, ERR_TIMEOUT_MMA)) return false;
          free_par ^= 1;
          tc_fence_after();
          freed = true;
          return true;
        };
        auto issue_S = [&](int kslot) {
          const uint64_t kb = kdesc0 + static_cast<uint64_t>(kslot * (C::KVBYTES >> 4));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t off = ((kk >> 2) * (TC_BM * 128) + (kk & 3) * 32) >> 4;
            umma_ss(tS, qdesc + off, kb + off, IDESC_S, kk > 0);
          }
        };
        // PV over keys 64*half .. 64*half+63 (P columns 32*half .. 32*half+31)
        auto issue_PV = [&](int vslot, int half) {
          const uint64_t vb = vdesc0 + static_cast<uint64_t>(vslot * (C::KVBYTES >> 4));
#pragma unroll
          for (int k4 = 0; k4 < TC_BN / 32; ++k4) {
            const int kk = half * (TC_BN / 32) + k4;
            umma_ts(tO, tS + kk * 8, vb + static_cast<uint64_t>((kk * 2048) >> 4), IDESC_PV,
                    (o_init || kk > 0) ? 1u : 0u);
          }
          o_init = true;
        };
        auto uses = [&](const TileInfo& t) { return mine && (t.use >> x & 1); };

        TileSeq seq;
        seq.init(p, U, us);
        TileInfo cur, nxt;
        bool have_cur = seq.next(p, U, cur);
        int cur_v = -1;
        if (have_cur) {
          const int ck = kpos % NK;
          if (!warp_wait(k_full + ck, (kpos / NK) & 1, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
          ++kpos;
          tc_fence_after();
          if (!my_turn()) { aborted = true; break; }
          if (uses(cur)) {
            issue_S(ck);
            if (!(sanity && cur.packed)) umma_commit(s_full + x);
          }
          end_turn();
          umma_commit(k_empty + ck);
        }
        bool q_released = false;
        while (have_cur) {
          if (cur.needs_v) {
            cur_v = vpos % NV;
            if (!warp_wait(v_full + cur_v, (vpos / NV) & 1, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
            ++vpos;
            tc_fence_after();
          }
          const bool have_nxt = seq.next(p, U, nxt);
          if (!have_nxt && !q_released) {
            // every S of this unit is issued: Q may be refilled once they complete
            umma_commit(q_empty);
            q_released = true;
          }
          if (!my_turn()) { aborted = true; break; }
          if (cur.needs_v && uses(cur)) {
            // the first half of PV starts once the softmax has stored P of keys 0..63 (and
            // has checked that keys 64..127 need no rescale), overlapping the second half's
            // exponentials
            if (!warp_wait(p_lo + x, p_par, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
            tc_fence_after();
            // the first PV of a unit overwrites O: the previous unit's epilogue must be done
            if (!ensure_free()) { aborted = true; break; }
            issue_PV(cur_v, 0);
            if (!warp_wait(p_full + x, p_par, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
            p_par ^= 1;
            tc_fence_after();
            issue_PV(cur_v, 1);
          }
          int nk = -1;
          if (have_nxt) {
            nk = kpos % NK;
            if (!warp_wait(k_full + nk, (kpos / NK) & 1, ab, ERR_TIMEOUT_MMA)) { aborted = true; break; }
            ++kpos;
            tc_fence_after();
            if (uses(nxt)) {
              issue_S(nk);
              if (!(sanity && nxt.packed)) umma_commit(s_full + x);
            }
          }
          end_turn();
          if (cur.needs_v) umma_commit(v_empty + cur_v);
          if (have_nxt) umma_commit(k_empty + nk);
          if (!have_nxt) break;
          cur = nxt;
        }
        if (aborted) break;
        if (!q_released) umma_commit(q_empty);
        // Handshake per valid query tile and unit: the MMA warp waits tile_free once (before
        // the unit's first PV into the tile's O, or here) and always commits o_full; the
        // epilogue always waits o_full before arriving on tile_free. An epilogue therefore
        // never arrives before the matching wait, which keeps the parity waits unambiguous.
        // Invalid tiles take no part.
        if (mine) {
          if (!ensure_free()) { aborted = true; break; }
          umma_commit(o_full + x);
        }
      }
      // wait for every MMA this warp issued before TMEM can be released (one commit per warp)
      umma_commit(mma_done);
      if (lane == 0) mbar_drain(mma_done, 0, p.err);
      __syncwarp();
    }
  } else if (warp >= 4) {
    // ================================================================ softmax + epilogue
    const int x = (warp - 4) >> 2;          // query tile
    const int wq = warp & 3;                // TMEM lane quarter
    const int r = wq * 32 + lane;           // row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + 128 * x;
    const uint32_t tO = tmem + lane_base + 256 + D * x;
    const float sl2 = p.scale_log2;
    int vpos = 0;  // V ring position (the packed block's counts travel with its V tile)
    uint32_t s_par = 0, o_par = 0;
    UnitSched us_next{};
    bool us_have = false;
    for (int it = 0; it < n_iter; ++it) {
      const int u = unit_of(it, blockIdx.x, G);
      if (u >= p.num_units) continue;
      const Unit U = decode_unit(p, u);
      const UnitSched us = us_have ? us_next : fetch_sched(p, U);
      {
        const int un = unit_of(it + 1, blockIdx.x, G);
        us_have = it + 1 < n_iter && un < p.num_units;
        if (us_have) us_next = fetch_sched(p, decode_unit(p, un));
      }
      const bool my_valid = x ? U.valid[1] : U.valid[0];
      const int my_hts = x ? U.hts[1] : U.hts[0];
      const int my_hq = x ? U.hq[1] : U.hq[0];
      const int row = (x ? U.mb[1] : U.mb[0]) * TC_BM + r;
      float m_used = -INFINITY, l = 0.f;
      bool o_has = false;
      TileSeq seq;
      seq.init(p, U, us);
      const float* wrow = p.blkw + (static_cast<int64_t>(U.b) * p.Hts + my_hts) * p.nblk;
      TileInfo t;
      bool ok = true;
      while (seq.next(p, U, t)) {
        // log2 weight of a packed block (NaN when its counts differ)
        const float lw = t.packed ? wrow[t.idx] : 0.f;
        if (!t.needs_v) continue;
        const int vs = vpos % NV;
        const uint32_t vfp = (vpos / NV) & 1;
        ++vpos;
        if (!my_valid || !(t.use >> x & 1)) continue;
        // everything up to the first read of S depends only on the block: it is done before
        // waiting for S, off the softmax -> PV -> QK^T -> softmax chain
        const uint32_t* cnt = reinterpret_cast<const uint32_t*>(auxc + vs * TC_BN);
        const bool cint = p.counts_is_int != 0;
        // a packed block with one common count is weighted through the exponent (no per-key work)
        const bool perkey = t.packed && !(lw == lw);  // NaN: counts differ inside the block
        const int32_t* tsv = auxt + vs * TC_BN;
        // per-key weights of the streaming path (KEYED): the block's counts, or unit weights
        const float* wts = KEYED ? (t.packed ? auxc + vs * TC_BN : ones) : nullptr;
        if (perkey || (t.packed && (KEYED || p.variant == TC_PURE))) {
          // per-key counts (and timestamps) arrive with the block's V tile
          if (!warp_wait(v_full + vs, vfp, ab, ERR_TIMEOUT_SOFTMAX)) { ok = false; break; }
        }
        const int n0 = t.idx * TC_BN;
        const uint32_t NEG_INF = 0xFF800000u;
        // pure-phase-1 validity (count > 0, index < num_packed, timestamp <= row): 32 bits per
        // 32-column chunk, built before S is read
        uint32_t vm[4] = {~0u, ~0u, ~0u, ~0u};
        int lim = TC_BN;
        bool pure_prefix = false;  // pure phase 1 with a per-row prefix mask (below)
        if (!KEYED && p.variant == TC_PURE) {
          const int nval = packed_len(p) - n0;  // keys of this block below the packed length
          // Packed keys keep sequence order, so their timestamps ascend. When they do in this
          // block and every count below the packed length is positive, a row's valid keys are
          // the prefix with timestamp <= row: a per-row limit, which the streaming path handles.
          // (Not compiled into the KEYED kernels: the extra code slowed their streaming path;
          // pure phase 1 on device-packed histories keeps the general mask.)
          {
            const int j0 = 4 * lane;
            const int4 tv = *reinterpret_cast<const int4*>(tsv + j0);
            const uint4 cv = *reinterpret_cast<const uint4*>(cnt + j0);
            const int tn = __shfl_down_sync(0xFFFFFFFFu, tv.x, 1);  // the next lane's first key
            const int tt[4] = {tv.x, tv.y, tv.z, tv.w};
            const uint32_t cc[4] = {cv.x, cv.y, cv.z, cv.w};
            bool okp = true;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = j0 + e;
              const float cj = cint ? static_cast<float>(static_cast<int32_t>(cc[e])) : __uint_as_float(cc[e]);
              const int tnext = e < 3 ? tt[e + 1] : tn;
              if (j < nval && !(cj > 0.f)) okp = false;
              if (j + 1 < nval && j + 1 < TC_BN && tnext < tt[e]) okp = false;
            }
            pure_prefix = __all_sync(0xFFFFFFFFu, okp);
          }
          if (pure_prefix) {
            // keys with timestamp <= row among the first nval (a search over the sorted prefix)
            const int nv = max(0, min(nval, TC_BN));
            int pos = 0;
#pragma unroll
            for (int step = TC_BN; step > 0; step >>= 1)
              if (pos + step <= nv && tsv[pos + step - 1] <= row) pos += step;
            lim = pos;
          }
        }
        if (p.variant == TC_PURE && !pure_prefix) {
          const int nval = packed_len(p) - n0;
#pragma unroll 1
          for (int w = 0; w < 4; ++w) {
            uint32_t bits = 0;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int j = w * 32 + e;
              const float cj = cint ? static_cast<float>(static_cast<int32_t>(cnt[j])) : __uint_as_float(cnt[j]);
              const bool v = (j < nval) && cj > 0.f && tsv[j] <= row;
              bits |= (v ? 1u : 0u) << e;
            }
            if (w == 0) vm[0] = bits; else if (w == 1) vm[1] = bits; else if (w == 2) vm[2] = bits; else vm[3] = bits;
          }
        }
        if (p.variant != TC_PURE) {
          if (t.packed) {
            lim = packed_len(p) - n0;
          } else {
            lim = p.seq_k - n0;
            if (p.variant != TC_DENSE || p.causal) lim = min(lim, row - n0 + 1);
          }
        }
        // S chunk c (columns 32c..32c+31) with masked columns set to -inf
        const bool any_mask = __any_sync(0xFFFFFFFFu, (p.variant == TC_PURE && !pure_prefix) || lim < TC_BN);
        auto load_chunk = [&](int c, uint32_t* sc) {
          tmem_ld32(tS + c * 32, sc);
          if (any_mask) {
            const uint32_t bits = (c == 0) ? vm[0] : (c == 1) ? vm[1] : (c == 2) ? vm[2] : vm[3];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const bool v = ((bits >> e) & 1u) && (c * 32 + e < lim);
              sc[e] = v ? sc[e] : NEG_INF;
            }
          }
        };
        auto chunk_max = [&](const uint32_t* sc) {
          float m0 = __uint_as_float(sc[0]), m1 = __uint_as_float(sc[1]);
#pragma unroll
          for (int e = 2; e < 32; e += 4) {
            m0 = fmax3(m0, __uint_as_float(sc[e]), __uint_as_float(sc[e + 1]));
            m1 = fmax3(m1, __uint_as_float(sc[e + 2]), __uint_as_float(sc[e + 3]));
          }
          return fmaxf(m0, m1);
        };
        // probabilities 2^(s*scale + nb) of one 32-column chunk, packed as bf16x2 / f16x2
        // pairs into out[0..15]; row sums into la / lb
        float2 la = make_float2(0.f, 0.f), lb = la;
        // exponent arguments and row sums on packed fp32x2 FMA / add (one instruction per pair):
        // the softmax warps are issue-bound
        auto exp_plain = [&](const uint32_t* sc, float nb, uint32_t* out) {
          const float2 s2 = make_float2(sl2, sl2), n2 = make_float2(nb, nb);
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float2 a01 = ffma2(make_float2(__uint_as_float(sc[e]), __uint_as_float(sc[e + 1])), s2, n2);
            const float2 a23 = ffma2(make_float2(__uint_as_float(sc[e + 2]), __uint_as_float(sc[e + 3])), s2, n2);
            float pe[4];
            pe[0] = ex2(a01.x); pe[1] = ex2(a01.y); pe[2] = ex2(a23.x); pe[3] = ex2(a23.y);
            la = fadd2(la, make_float2(pe[0], pe[1]));
            lb = fadd2(lb, make_float2(pe[2], pe[3]));
            out[e / 2] = pack2(pe[0], pe[1], BF16);
            out[e / 2 + 1] = pack2(pe[2], pe[3], BF16);
          }
        };
        // the same with a per-key count weight (packed blocks whose counts differ)
        auto exp_counted = [&](int c, const uint32_t* sc, float nb, uint32_t* out) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const uint4 cb = *reinterpret_cast<const uint4*>(cnt + c * 32 + e);
            const uint32_t cu[4] = {cb.x, cb.y, cb.z, cb.w};
            float pe[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float ck = cint ? static_cast<float>(static_cast<int32_t>(cu[k])) : __uint_as_float(cu[k]);
              pe[k] = ex2(fmaf(__uint_as_float(sc[e + k]), sl2, nb)) * ck;
            }
            la.x += pe[0]; la.y += pe[1]; lb.x += pe[2]; lb.y += pe[3];
            out[e / 2] = pack2(pe[0], pe[1], BF16);
            out[e / 2 + 1] = pack2(pe[2], pe[3], BF16);
          }
        };
        // probabilities weighted by per-key counts (KEYED streaming path): 2^(s*scale + nb) * w
        auto exp_keyed = [&](int c, const uint32_t* sc, float nb, uint32_t* out) {
          const float2 s2 = make_float2(sl2, sl2), n2 = make_float2(nb, nb);
          const float* w = wts + c * 32;
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 w4 = *reinterpret_cast<const float4*>(w + e);
            const float2 a01 = ffma2(make_float2(__uint_as_float(sc[e]), __uint_as_float(sc[e + 1])), s2, n2);
            const float2 a23 = ffma2(make_float2(__uint_as_float(sc[e + 2]), __uint_as_float(sc[e + 3])), s2, n2);
            const float2 p01 = fmul2(make_float2(ex2(a01.x), ex2(a01.y)), make_float2(w4.x, w4.y));
            const float2 p23 = fmul2(make_float2(ex2(a23.x), ex2(a23.y)), make_float2(w4.z, w4.w));
            la = fadd2(la, p01);
            lb = fadd2(lb, p23);
            out[e / 2] = pack2(p01.x, p01.y, BF16);
            out[e / 2 + 1] = pack2(p23.x, p23.y, BF16);
          }
        };
        // one chunk of the streaming path
        auto exp_stream = [&](int c, const uint32_t* sc, float nb, uint32_t* out) {
          if constexpr (KEYED) exp_keyed(c, sc, nb, out);
          else exp_plain(sc, nb, out);
        };
        // fast path (warp-uniform; bf16, unmasked tile, one weight per block): S streams through
        // two register buffers (the load of chunk c+1 is in flight while chunk c is
        // exponentiated against the running reference) and
        // each P chunk is stored as soon as it is computed. P chunk c covers columns
        // 16c..16c+15, below every S chunk not yet read. A chunk that raises some row's maximum
        // more than 2^8 above its reference stops the stream: the repair path below takes over
        // from that chunk. P of keys 0..63 (chunks 0 and 1) is released to the MMA warp (p_lo)
        // only after chunks 2 and 3 have passed the same check, so released P is final.
        // (KEYED: per-key weights are fine too)
        // a tile masked only by a per-row key limit (the causal diagonal, the end of the keys, the
        // packed tail) also takes the fast path: its masked S entries are overwritten with -inf in
        // TMEM first, so the unmodified streaming code gives them probability 0
        const bool lim_mask = any_mask && (p.variant != TC_PURE || pure_prefix);
        const bool fast = BF16 && (KEYED || !perkey) && (!any_mask || lim_mask);
        if (!warp_wait(s_full + x, s_par, ab, ERR_TIMEOUT_SOFTMAX)) { ok = false; break; }
        s_par ^= 1;
        tc_fence_after();
        if (fast && lim_mask) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            if (!__any_sync(0xFFFFFFFFu, lim < c * 32 + 32)) continue;  // no masked column in chunk c
            uint32_t sc[32];
            tmem_ld32(tS + c * 32, sc);
#pragma unroll
            for (int e = 0; e < 32; ++e) sc[e] = (c * 32 + e < lim) ? sc[e] : NEG_INF;
            tmem_st32(tS + c * 32, sc);
          }
          tmem_st_wait();
        }
        int stop = 0;  // first chunk the fast path did not finish
        bool lo_sent = false;  // p_lo arrived (P of keys 0..63 final)
        if (fast) {
          uint32_t sa[32], sb[32];
          tmem_ld32_async(tS, sa);
          tmem_ld32_wait(sa);
          tmem_ld32_async(tS + 32, sb);
          // a row without a reference yet (the unit's first block) takes chunk 0's maximum: any
          // finite reference is exact once O / l divides it out, and a later chunk more than 2^8
          // above it takes the repair path like any other jump
          if (m_used == -INFINITY) {
            const float m0 = chunk_max(sa) * sl2;
            m_used = (m0 == -INFINITY) ? 0.f : m0;
          }
          const float nb = KEYED ? -m_used : lw - m_used;
          const float lim_raise = m_used + 8.f;
          // chunk c (0 or 1); false when it stops the stream (no load is left in flight then). On
          // success chunk c+1 has landed in sn and chunk c+2 is loading into sc.
          auto step = [&](int c, uint32_t(&sc)[32], uint32_t(&sn)[32]) -> bool {
            if (__any_sync(0xFFFFFFFFu, chunk_max(sc) * sl2 > lim_raise)) {
              tmem_ld32_wait(sn);
              stop = c;
              return false;
            }
            uint32_t pc[16];
            exp_stream(c, sc, nb, pc);
            tmem_st16(tS + c * 16, pc);
            tmem_ld32_wait(sn);
            tmem_ld32_async(tS + (c + 2) * 32, sc);
            return true;
          };
          if (step(0, sa, sb) && step(1, sb, sa)) {
            // chunk 2 is in sa, chunk 3 lands in sb: both are checked before P of keys 0..63
            // is released to the first half of PV, so nothing released is ever rescaled
            tmem_ld32_wait(sb);
            if (__any_sync(0xFFFFFFFFu, fmaxf(chunk_max(sa), chunk_max(sb)) * sl2 > lim_raise)) {
              stop = 2;
            } else {
              tmem_st_wait();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(p_lo + x);
              lo_sent = true;
              uint32_t pc[16];
              exp_stream(2, sa, nb, pc);
              tmem_st16(tS + 32, pc);
              exp_stream(3, sb, nb, pc);
              tmem_st16(tS + 48, pc);
              stop = 4;
            }
          }
        }
        if (stop < 4) {
          // exact / repair path from chunk `stop`: the row maximum over the chunks not yet done
          // (their S columns are intact), then a rescale of everything accumulated so far, then
          // P of the remaining chunks. After a fast-path stop the reference moves up by a whole
          // number of octaves, so the P chunks already stored rescale exactly (power of two).
          tmem_st_wait();
          float mt = -INFINITY;
#pragma unroll 1
          for (int c = stop; c < 4; ++c) {
            uint32_t sc[32];
            load_chunk(c, sc);
            mt = fmaxf(mt, chunk_max(sc));
          }
          mt *= sl2;
          const bool need = mt > m_used + (BF16 ? 8.f : 0.f);
          if (__any_sync(0xFFFFFFFFu, need)) {
            float m_new = m_used, f = 1.f;
            if (need) {
              if (stop > 0) {
                const int k = static_cast<int>(ceilf(mt - m_used));
                m_new = m_used + static_cast<float>(k);
                f = k < 127 ? __int_as_float((127 - k) << 23) : 0.f;
              } else {
                m_new = mt;
                f = ex2(m_used - m_new);
              }
            }
            l *= f;
            la.x *= f; la.y *= f; lb.x *= f; lb.y *= f;
            if (o_has) {
#pragma unroll 1
              for (int c = 0; c < D / 16; ++c) {
                uint32_t o[16];
                tmem_ld16(tO + c * 16, o);
#pragma unroll
                for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f);
                tmem_st16(tO + c * 16, o);
              }
            }
            if (BF16) {
#pragma unroll 1
              for (int c = 0; c < stop; ++c) {
                uint32_t pc[16];
                tmem_ld16(tS + c * 16, pc);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float lo = __uint_as_float(pc[j] << 16) * f;
                  const float hi = __uint_as_float(pc[j] & 0xFFFF0000u) * f;
                  pc[j] = pack2(lo, hi, true);
                }
                tmem_st16(tS + c * 16, pc);
              }
            }
            m_used = m_new;
          }
          const float msub = (m_used == -INFINITY) ? 0.f : m_used;
#pragma unroll 1
          for (int c = stop; c < 4; ++c) {
            uint32_t sc[32], pc[16];
            load_chunk(c, sc);
            if (perkey) exp_counted(c, sc, -msub, pc);
            else exp_plain(sc, lw - msub, pc);
            tmem_st16(tS + c * 16, pc);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (!lo_sent) mbar_arrive(p_lo + x);
          mbar_arrive(p_full + x);
        }
        l += (la.x + la.y) + (lb.x + lb.y);
        o_has = true;
      }
      if (!ok) break;
      if (!my_valid) continue;  // invalid tiles take no part in the o_full / tile_free handshake
      // ---------------- epilogue: O / l -> out
      float lf = l;
      if (p.variant == TC_PURE && !(lf > 0.f)) lf = 1.f;
      const float inv = 1.f / lf;
      const bool row_ok = row < p.seq_q;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = static_cast<T*>(p.out) + U.b * p.os_b + static_cast<int64_t>(my_hq) * p.os_h +
                static_cast<int64_t>(row) * p.os_m;
      if (!warp_wait(o_full + x, o_par, ab, ERR_TIMEOUT_EPILOGUE)) break;
      o_par ^= 1;
      tc_fence_after();
      if (o_has && p.out_vec_ok) {
        // each 32-column chunk goes through the warp's staging rows, so a 16-byte store
        // instruction covers 8 rows x 64 B (8 lines) instead of 32 rows x 16 B (32 lines)
        uint8_t* stg = smem + C::OFF_EPI + (warp - 4) * 32 * C::EPI_PITCH;
        const int rr = lane >> 2, seg = lane & 3;  // the row / 16-byte piece this lane stores
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ob[32];
          tmem_ld32(tO + c * 32, ob);
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 w;
            w.x = pack2(__uint_as_float(ob[j]) * inv, __uint_as_float(ob[j + 1]) * inv, BF16);
            w.y = pack2(__uint_as_float(ob[j + 2]) * inv, __uint_as_float(ob[j + 3]) * inv, BF16);
            w.z = pack2(__uint_as_float(ob[j + 4]) * inv, __uint_as_float(ob[j + 5]) * inv, BF16);
            w.w = pack2(__uint_as_float(ob[j + 6]) * inv, __uint_as_float(ob[j + 7]) * inv, BF16);
            *reinterpret_cast<uint4*>(stg + lane * C::EPI_PITCH + j * 2) = w;
          }
          __syncwarp();
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int lr = q4 * 8 + rr;  // lane (row) of the warp whose piece this is
            const uint4 w = *reinterpret_cast<const uint4*>(stg + lr * C::EPI_PITCH + seg * 16);
            if (row - lane + lr < p.seq_q)
              *reinterpret_cast<uint4*>(orow + static_cast<int64_t>(lr - lane) * p.os_m + c * 32 + seg * 8) = w;
          }
          __syncwarp();
        }
      } else if (o_has) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ob[32];
          tmem_ld32(tO + c * 32, ob);
          float o[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __uint_as_float(ob[j]);
          if (row_ok) {
            if (p.out_vec_ok) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 w;
                w.x = pack2(o[j] * inv, o[j + 1] * inv, BF16);
                w.y = pack2(o[j + 2] * inv, o[j + 3] * inv, BF16);
                w.z = pack2(o[j + 4] * inv, o[j + 5] * inv, BF16);
                w.w = pack2(o[j + 6] * inv, o[j + 7] * inv, BF16);
                *reinterpret_cast<uint4*>(orow + c * 32 + j) = w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) orow[c * 32 + j] = from_f32<T>(o[j] * inv);
            }
          }
        }
      } else if (row_ok) {
        // no block attended: the reference divides a zero accumulator by l
        const float v = 0.f * inv;
        for (int j = 0; j < D; ++j) orow[j] = from_f32<T>(v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tile_free + x);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, 512);
}

template <int D, bool BF16, bool KEYED, bool SPARSE = false>
static cudaError_t launch_tc_t(const TcParams& p, int num_sms, cudaStream_t st) {
  using C = TcCfg<D>;
  auto kfn = attn_tc_kernel<D, BF16, KEYED, SPARSE>;
  cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int grid = p.num_units < num_sms ? p.num_units : num_sms;
  if (grid <= 0) return cudaSuccess;
  kfn<<<grid, TC_THREADS, C::SMEM, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_attn_tc(int head_dim, bool bf16, const TcParams& p, int num_sms, cudaStream_t st) {
  if (p.variant == TC_SPARSE) {
    if (head_dim == 128)
      return bf16 ? launch_tc_t<128, true, false, true>(p, num_sms, st) : launch_tc_t<128, false, false, true>(p, num_sms, st);
    if (head_dim == 64)
      return bf16 ? launch_tc_t<64, true, false, true>(p, num_sms, st) : launch_tc_t<64, false, false, true>(p, num_sms, st);
    return cudaErrorInvalidValue;
  }
  // per-key weights on the streaming path only where it runs (bf16) and the counts are fp32
  const bool keyed = p.keyed && bf16 && !p.counts_is_int;
  if (head_dim == 128)
    return keyed ? launch_tc_t<128, true, true>(p, num_sms, st)
                 : bf16 ? launch_tc_t<128, true, false>(p, num_sms, st) : launch_tc_t<128, false, false>(p, num_sms, st);
  if (head_dim == 64)
    return keyed ? launch_tc_t<64, true, true>(p, num_sms, st)
                 : bf16 ? launch_tc_t<64, true, false>(p, num_sms, st) : launch_tc_t<64, false, false>(p, num_sms, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_schedule(const int32_t* ts, const int64_t* tss, const void* counts, const int64_t* cs,
                            int counts_is_int, int B, int Hts, int num_packed, int seq_k, int window, int nmb,
                            int nblk, int2* sched, int32_t* blkmin, int want_blkmin, float* blkw,
                            const int32_t* anchors, int* len_out, cudaStream_t st) {
  if (B * Hts == 0) return cudaSuccess;
  const size_t sm = static_cast<size_t>(nblk > 0 ? nblk : 1) * sizeof(int32_t);
  if (sm > 200 * 1024) return cudaErrorInvalidValue;
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(schedule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sm));
    if (e != cudaSuccess) return e;
  }
  schedule_kernel<<<B * Hts, 256, sm, st>>>(ts, tss[0], tss[1], tss[2], counts, cs[0], cs[1], cs[2], counts_is_int,
                                            Hts, num_packed, seq_k, window, nmb, nblk, sched, blkmin, want_blkmin,
                                            blkw, anchors, B * Hts, len_out);
  return cudaGetLastError();
}

}  // namespace dab

// Launch-parameter structs shared by the kernels and the C ABI layer.
#pragma once
#include "common.cuh"

namespace dab {

enum Variant : int { HYBRID = 0, SANITY = 1, PURE = 2, DENSE = 3 };

// CUDA-core attention (any dtype / strides / block sizes, head_dim <= 128)
struct SimtParams {
  const void* q; const void* kd; const void* vd; const void* kp; const void* vp;
  const int32_t* ts; const void* counts; void* out;
  int64_t qs[4], kds[4], vds[4], kps[4], vps[4], tss[3], cs[3], os[4];
  float sm_scale;
  int64_t seq_q, seq_k, num_packed, head_dim, num_heads, dense_window;
  int64_t grid_m, grid_bh, block_m, block_n;
  int64_t kv_group;      // q-head h reads K/V/ts/counts of head h / kv_group
  int counts_is_int;     // counts given as int32 (else fp32)
  int causal;            // DENSE only
  int variant;
};

// tcgen05 attention (bf16 / fp16, head_dim 64 or 128, 128x128 logical blocks)
struct TcParams {
  CUtensorMap tm_q, tm_kd, tm_vd, tm_kp, tm_vp;
  void* out;
  int64_t os_b, os_h, os_m;
  const int32_t* ts;
  int64_t ts_b, ts_h, ts_n;
  const void* counts;
  int64_t cs_b, cs_h, cs_n;
  const int2* sched;       // [B*Hts][nmb] = (phase-1 blocks, dense start block)
  const int32_t* blkmin;   // [B*Hts][nblk] smallest valid timestamp of each packed block
  const float* blkw;       // [B*Hts][nblk] log2 of the block's common count, NaN if counts differ
  int* err;
  float scale_log2;        // sm_scale * log2(e)
  int seq_q, seq_k, num_packed;
  int B, Hq, kv_group, Hts;
  int nmb, nblk;
  int variant, causal, counts_is_int, pair_heads;
  int num_units;
  int out_vec_ok;          // output rows are 16-byte aligned with unit d-stride
  int meta_bulk;           // counts / timestamps rows can be bulk-copied (contiguous, 16-byte aligned)
  // device-resident packed length (null: num_packed above is the packed length). anchors[b*Hts+h]
  // is the kept count of each head, len_dev[0] their maximum M (the reference's packed length,
  // written by the schedule pre-pass); num_packed / nblk then give the buffers' capacity.
  const int32_t* anchors;
  const int* len_dev;
  int keyed;               // packed blocks' counts differ inside blocks: weight per key on the fast path
  // block-sparse variant (DPXA): bitmask of the key blocks each (batch, kv-head, query block)
  // attends, `sel_words` 32-bit words per query block
  const uint32_t* sel;
  int sel_words;
};

// fused key compression (compress.cu): strides in elements
struct CompressParams {
  const void* k; int64_t ks_b, ks_h, ks_s;        // raw keys [B, H, N, D]
  const void* v; int64_t vs_b, vs_h, vs_s;        // values [B, H, N, D]
  const void* cos; const void* sin; int64_t cs_b, cs_s;  // RoPE tables [B or 1, N, D]
  void* k_rot; int64_t rs_b, rs_h, rs_s;          // rotated keys out
  int32_t* keep; int64_t km_b, km_h, km_s;        // keep mask out (may be null)
  void* kp; void* vp; int64_t ps_b, ps_h, ps_s;   // packed K / V [B, H, cap, D]
  int32_t* ts; int32_t* cnt; float* cnt_f; int64_t ms_b, ms_h;  // packed metadata [B, H, cap]
  int32_t* anchors;                               // [B * H] kept count per head
  uint8_t* ws;                                    // workspace: header, then a status word per chunk
  float thr;                                      // squared-distance (or cosine) threshold
  int H, N, chunk, nch, cap;
  unsigned total_chunks, total_warps;
};

// projection GEMM with a RoPE epilogue (proj.cu): out = RoPE(round(X W^T)) on [rope_lo, rope_hi)
struct ProjParams {
  CUtensorMap tm_x;                     // X [rows, K] bf16, box 64 x 128, 128-byte swizzle
  CUtensorMap tm_w;                     // W [Ho, K] bf16 (nn.Linear weight), box 64 x 256
  const void* cos; const void* sin;     // RoPE tables [rows, head_dim] bf16
  int64_t cs_row;                       // table row stride (elements)
  void* out; int64_t os_row;            // out [rows, Ho] bf16, row stride (elements)
  int* err;                             // device error word (bounded waits)
  int rows, K, Ho;
  int rope_lo, rope_hi;                 // output columns that get RoPE (multiples of 128)
  int n_tiles_n, num_tiles;             // 256-column tiles per row block; total tiles
};

}  // namespace dab

// Batched decode (up to 64 concurrent sequences, one token each per step) on
// tcgen05 tensor cores.  Included at the end of megakernel.cu.
//
// This file starts with the pieces every batched kernel shares: the hi/lo
// split of fp32 activations into the 128-row bf16 A operand, and a test entry
// point that runs one tcgen05 GEMM with a plain epilogue.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include <cuda_fp16.h>

#include "../../include/megakernel.h"
#include "tc_gemm.cuh"

namespace mk {

// x fp32 [rows x K] (rows <= 64) -> A bf16 [128 x K]: row r = bf16(x_r),
// row 64 + r = bf16(x_r - bf16(x_r)); rows >= `rows` of both halves are 0.
__global__ void hilo_split_kernel(const float* __restrict__ x, int rows, int K, __nv_bfloat16* __restrict__ a) {
  const int n = 64 * K;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int r = i / K;
    const float v = r < rows ? x[i] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    a[i] = hi;
    a[(size_t)n + i] = __float2bfloat16_rn(v - __bfloat162float(hi));
  }
}

// Plain epilogue: out[seq][64 t + c] = v[c] for seq < rows.
struct EpiStore {
  static constexpr bool kCols = false;
  // Prefetched inputs are the same for every tile.
  static constexpr bool kPrePerTile = false;
  static constexpr int kPre = 0;
  struct Params {
    float* out;
    int ldo;
    int rows;
  };
  __device__ __forceinline__ static void prefetch(const Params&, int, float*, int) {}
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, const float (&v)[64], const float*) {
    if (seq >= ep.rows) return;
    float* o = ep.out + (size_t)seq * ep.ldo + 64 * t;
#pragma unroll
    for (int c = 0; c < 64; c += 4) *reinterpret_cast<float4*>(o + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
  }
};


// ============================================================================
// Batched decode step (Qwen3 d64 shape): per-kernel device code.
// ============================================================================

constexpr int kBMax = 64;          // sequences per batch
constexpr int kBH = 1024, kBQ = 1024, kBKV = 512, kBI = 2816, kBD = 64, kBNQ = 16, kBNKV = 8, kBL = 28;
constexpr int kBV = 151936;
constexpr int kBHT = kBH / 64;     // 64-column tiles of the residual stream (sum-of-squares partials)
// Positions per attention chunk (K/V tile of a warp's pipeline).
#ifndef MK_BATTN_CHUNK
#define MK_BATTN_CHUNK 64
#endif
constexpr int kBChunk = MK_BATTN_CHUNK;
static_assert(kBChunk == 32 || kBChunk == 64, "attention chunk");
constexpr int kBNT = kBChunk / 8;      // 8-position n-tiles of a chunk (scores)
constexpr int kBKS = kBChunk / 16;     // 16-position k-steps of a chunk (P.V)
constexpr int kBLMTiles = kBV / 64;
static_assert(kBV % 64 == 0, "vocab tiles");

struct BatchDev {
  // activations
  float* x;              // [64][1024] residual stream
  float* ssq;            // [16][64] per-tile partial sums of squares of x
  __nv_bfloat16* a_x;    // [128][1024] hi/lo of (gain . x)
  __nv_bfloat16* a_att;  // [128][1024] hi/lo of the attention output
  __nv_bfloat16* a_h;    // [128][2816] hi/lo of silu(gate) * up
  float* q;              // [64][16][64] normed + roped queries
  float* part;           // attention partials [64][8][maxch][2][66]
  unsigned long long* lm_part;  // [2374][64] packed (orderable value, index)
  __nv_bfloat16* kv;     // [64][L][2][8][max_seq][64] bf16 cache (nullptr with an fp8 cache)
  uint8_t* kv8;          // same layout, e4m3 (nullptr with a bf16 cache)
  const float* rope_cos; // [max_seq][32]
  const float* rope_sin;
  int* pos;              // [64] position of each sequence's next token
  int* err;
  int* acnt;             // [64][8] attention chunk tickets (0 between layers)
  int batch, max_seq, maxch;
  int seq_mode;          // 0: row b is sequence b; 1: every row belongs to sequence 0 (prefill)
};

__device__ __forceinline__ size_t bkv_index(const BatchDev& d, int b, int l, int kv, int h, int p) {
  const size_t sq = d.seq_mode ? 0 : (size_t)b;
  return ((((sq * kBL + l) * 2 + kv) * kBNKV + h) * (size_t)d.max_seq + p) * kBD;
}
// Two e4m3 values (low byte first) -> two f16 (exact), and two fp32 -> e4m3
// (round to nearest, saturating).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// 1 / rms of row `seq` of x from the 16 tile partials (fixed order).
__device__ __forceinline__ float inv_rms(const float* ssq, int seq) {
  float s = 0.f;
#pragma unroll
  for (int t = 0; t < kBHT; ++t) s += ssq[t * kBMax + seq];
  return rsqrtf(s / (float)kBH + 1e-6f);
}
// Epilogue prefetch (128 threads, e = 0..127): 1 / rms of every row into
// pre[0..63].
__device__ __forceinline__ void prefetch_inv_rms(const float* ssq, float* pre, int e) {
  if (e < kBMax) pre[e] = inv_rms(ssq, e);
}
__device__ __forceinline__ void put_hilo(__nv_bfloat16* a, int K, int seq, int col, float v) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  a[(size_t)seq * K + col] = hi;
  a[(size_t)(kBMax + seq) * K + col] = __float2bfloat16_rn(v - __bfloat162float(hi));
}
// Orderable 64-bit key: larger value first, then the lower index.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (uint32_t)(0x7fffffff - idx);
}

// x[b] = E[tok_b]; ssq[0][b] = |x_b|^2 (other tiles 0); a_x = hi/lo(g . x).
// tok_b = forced[b] when forced != null, else prev_out[b].
__global__ void bembed_kernel(BatchDev d, const __nv_bfloat16* __restrict__ emb, const __nv_bfloat16* __restrict__ g,
                              const int* __restrict__ forced, const int* __restrict__ prev_out) {
  const int b = blockIdx.x;
  __shared__ float red[32];
  pdl_launch();
  pdl_wait();
  if (b >= kBMax) return;
  float ss = 0.f;
  const bool live = b < d.batch;
  const int tok = live ? (forced ? forced[b] : prev_out[b]) : 0;
  for (int i = threadIdx.x; i < kBH; i += blockDim.x) {
    const float v = live ? __bfloat162float(emb[(size_t)tok * kBH + i]) : 0.f;
    d.x[b * kBH + i] = v;
    ss += v * v;
    put_hilo(d.a_x, kBH, b, i, __bfloat162float(g[i]) * v);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < kBHT) {
    float t = 0.f;
    if (threadIdx.x == 0)
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    d.ssq[threadIdx.x * kBMax + b] = t;
  }
}

// QKV epilogue: tile t < 16: query head t; 16..23: key head t-16; 24..31:
// value head t-24.  Scales by 1/rms, applies q_norm / k_norm and RoPE at the
// sequence's position, writes q (fp32) or appends K / V (bf16) to the cache.
struct EpiQKV {
  static constexpr bool kCols = true;
  // Prefetched inputs depend on the tile index (re-fetched per 64-column tile).
  static constexpr bool kPrePerTile = true;
  // pre: [0, 64) 1/rms per row, [64, 128) head-norm gains, [128, 192) the
  // row's position (int bits), then [192 + 64 r, +64) cos | sin of row r.
  static constexpr int kPre = 3 * 64 + 64 * 64;
  struct Params {
    BatchDev d;
    int l;
    const __nv_bfloat16* qn;
    const __nv_bfloat16* kn;
  };
  __device__ __forceinline__ static void prefetch(const Params& ep, int t, float* pre, int e) {
    const BatchDev& d = ep.d;
    prefetch_inv_rms(d.ssq, pre, e);
    if (e < 64) {
      pre[64 + e] = t < 24 ? __bfloat162float((t < 16 ? ep.qn : ep.kn)[e]) : 0.f;
      pre[128 + e] = __int_as_float(e < d.batch ? __ldcg(d.pos + e) : 0);
    }
    if (t < 24) {
      // cos | sin rows of each sequence's position: thread e covers 32
      // consecutive floats of row e / 2 (lanes = consecutive addresses).
      const int r = e >> 1, half = e & 1;
      const int pr = r < d.batch ? __ldcg(d.pos + r) : 0;
      const float* src = (half ? d.rope_sin : d.rope_cos) + (size_t)pr * 32;
      float* dst = pre + 192 + 64 * r + 32 * half;
#pragma unroll
      for (int c = 0; c < 32; c += 4) *reinterpret_cast<float4*>(dst + c) = __ldg(reinterpret_cast<const float4*>(src + c));
    }
  }
  __device__ __forceinline__ static void apply(const Params&, int, int, float (&)[64], const float*) {}
  // 128 threads, two per row (lanes 2r, 2r + 1 of a warp pair up): thread
  // half h takes columns [16h, 16h + 16) and their RoPE partners 32 on, so
  // the head norm's sum of squares is one shuffle and every RoPE pair stays
  // in one thread.
  __device__ __forceinline__ static void cols(const Params& ep, int t, float* tile, int tid, const float* pre,
                                              int ra, int rb) {
    const BatchDev& d = ep.d;
    const int row = ra + (tid >> 1), h = tid & 1, c0 = 16 * h;
    const bool live = row < rb && row < d.batch;
    const int rr_ = live ? row : ra;            // a valid row for the (unused) loads of idle threads
    const float r = pre[rr_];
    float a[16], b[16];
    const float4* tr = reinterpret_cast<const float4*>(tile + rr_ * kTcCombStride);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 x = tr[(c0 >> 2) + k], y = tr[8 + (c0 >> 2) + k];
      a[4 * k] = x.x * r; a[4 * k + 1] = x.y * r; a[4 * k + 2] = x.z * r; a[4 * k + 3] = x.w * r;
      b[4 * k] = y.x * r; b[4 * k + 1] = y.y * r; b[4 * k + 2] = y.z * r; b[4 * k + 3] = y.w * r;
    }
    if (t < 24) {
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) ss = fmaf(b[c], b[c], fmaf(a[c], a[c], ss));
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rr = rsqrtf(ss / 64.f + 1e-6f);
      const float* gn = pre + 64;
      const float* cs = pre + 192 + 64 * rr_;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float x0 = gn[c0 + c] * (a[c] * rr), x1 = gn[32 + c0 + c] * (b[c] * rr);
        const float cc = cs[c0 + c], sn = cs[32 + c0 + c];
        a[c] = x0 * cc - x1 * sn;
        b[c] = x1 * cc + x0 * sn;
      }
    }
    if (!live) return;
    const int p = __float_as_int(pre[128 + row]);
    if (t < 16) {
      float* o = d.q + ((size_t)row * kBNQ + t) * kBD;
#pragma unroll
      for (int c = 0; c < 16; c += 4) {
        *reinterpret_cast<float4*>(o + c0 + c) = make_float4(a[c], a[c + 1], a[c + 2], a[c + 3]);
        *reinterpret_cast<float4*>(o + 32 + c0 + c) = make_float4(b[c], b[c + 1], b[c + 2], b[c + 3]);
      }
      return;
    }
    const int kv = t < 24 ? 0 : 1, hd = t < 24 ? t - 16 : t - 24;
    if (d.kv8 != nullptr) {
      // fp8 cache: e4m3, round to nearest, saturating (|K|, |V| << 448).
      uint8_t* o8 = d.kv8 + bkv_index(d, row, ep.l, kv, hd, p);
      uint4 w;
      w.x = (uint32_t)f32x2_to_e4m3x2(a[0], a[1]) | ((uint32_t)f32x2_to_e4m3x2(a[2], a[3]) << 16);
      w.y = (uint32_t)f32x2_to_e4m3x2(a[4], a[5]) | ((uint32_t)f32x2_to_e4m3x2(a[6], a[7]) << 16);
      w.z = (uint32_t)f32x2_to_e4m3x2(a[8], a[9]) | ((uint32_t)f32x2_to_e4m3x2(a[10], a[11]) << 16);
      w.w = (uint32_t)f32x2_to_e4m3x2(a[12], a[13]) | ((uint32_t)f32x2_to_e4m3x2(a[14], a[15]) << 16);
      *reinterpret_cast<uint4*>(o8 + c0) = w;
      w.x = (uint32_t)f32x2_to_e4m3x2(b[0], b[1]) | ((uint32_t)f32x2_to_e4m3x2(b[2], b[3]) << 16);
      w.y = (uint32_t)f32x2_to_e4m3x2(b[4], b[5]) | ((uint32_t)f32x2_to_e4m3x2(b[6], b[7]) << 16);
      w.z = (uint32_t)f32x2_to_e4m3x2(b[8], b[9]) | ((uint32_t)f32x2_to_e4m3x2(b[10], b[11]) << 16);
      w.w = (uint32_t)f32x2_to_e4m3x2(b[12], b[13]) | ((uint32_t)f32x2_to_e4m3x2(b[14], b[15]) << 16);
      *reinterpret_cast<uint4*>(o8 + 32 + c0) = w;
      return;
    }
    __nv_bfloat16* o = d.kv + bkv_index(d, row, ep.l, kv, hd, p);
#pragma unroll
    for (int c = 0; c < 16; c += 8) {
      uint4 w;
      w.x = pack_bf16x2(a[c], a[c + 1]); w.y = pack_bf16x2(a[c + 2], a[c + 3]);
      w.z = pack_bf16x2(a[c + 4], a[c + 5]); w.w = pack_bf16x2(a[c + 6], a[c + 7]);
      *reinterpret_cast<uint4*>(o + c0 + c) = w;
      w.x = pack_bf16x2(b[c], b[c + 1]); w.y = pack_bf16x2(b[c + 2], b[c + 3]);
      w.z = pack_bf16x2(b[c + 4], b[c + 5]); w.w = pack_bf16x2(b[c + 6], b[c + 7]);
      *reinterpret_cast<uint4*>(o + 32 + c0 + c) = w;
    }
  }
};

// Residual epilogue (O and down projections).  Column phase (thread = column
// c of the tile): x += v (coalesced), the new x goes back to the tile; then
// thread = row: sum of squares of the row's 64 new values -> ssq[t][row];
// then thread = column again: hi/lo of (g . x) into a_next.
struct EpiResid {
  static constexpr bool kCols = true;
  // Prefetched inputs depend on the tile index (re-fetched per 64-column tile).
  static constexpr bool kPrePerTile = true;
  // pre: [0, 64) gains of the tile's columns, then x[r][64 t + c] at
  // 64 + 64 r + c (the residual stream's tile, fetched during the MMAs).
  static constexpr int kPre = 64 + 64 * 64;
  struct Params {
    BatchDev d;
    __nv_bfloat16* a_next;
    const __nv_bfloat16* g;
  };
  __device__ __forceinline__ static void prefetch(const Params& ep, int t, float* pre, int e) {
    const BatchDev& d = ep.d;
    if (e < 64) pre[e] = __bfloat162float(ep.g[64 * t + e]);
    // Row r = e / 2, 32 columns per thread, 16-byte loads through L2 (the
    // previous kernel wrote x).
    const int r = e >> 1, c0 = 32 * (e & 1);
    const float* src = d.x + (size_t)r * kBH + 64 * t + c0;
    float* dst = pre + 64 + 64 * r + c0;
#pragma unroll
    for (int c = 0; c < 32; c += 4) *reinterpret_cast<float4*>(dst + c) = __ldcg(reinterpret_cast<const float4*>(src + c));
  }
  __device__ __forceinline__ static void apply(const Params&, int, int, float (&)[64], const float*) {}
  // 128 threads: column c = tid & 63 for every other row of [ra, rb), then
  // the per-row sum of squares on one thread per row.
  __device__ __forceinline__ static void cols(const Params& ep, int t, float* tile, int tid, const float* pre,
                                              int ra, int rb) {
    const BatchDev& d = ep.d;
    const int c = tid & 63;
    const int col = 64 * t + c;
    const float g = pre[c];
#pragma unroll 8
    for (int r = ra + (tid >> 6); r < rb; r += 2) {
      const float xn = pre[64 + 64 * r + c] + tile[r * kTcCombStride + c];
      __stcg(d.x + (size_t)r * kBH + col, xn);
      tile[r * kTcCombStride + c] = xn;
      put_hilo(ep.a_next, kBH, r, col, g * xn);
    }
    asm volatile("bar.sync 2, 128;" ::: "memory");
    if (tid < rb - ra) {
      const int row = ra + tid;
      float ss = 0.f;
      const float4* tr = reinterpret_cast<const float4*>(tile + row * kTcCombStride);
#pragma unroll 4
      for (int k = 0; k < 16; ++k) {
        const float4 xv = tr[k];
        ss = fmaf(xv.x, xv.x, ss);
        ss = fmaf(xv.y, xv.y, ss);
        ss = fmaf(xv.z, xv.z, ss);
        ss = fmaf(xv.w, xv.w, ss);
      }
      d.ssq[t * kBMax + row] = ss;
    }
  }
};

// Gate/up epilogue: columns 0..31 are gate rows 32t.., 32..63 the matching
// up rows.  Column phase on all 128 epilogue threads (lane = gate column c,
// so the hi/lo writes to a_h are coalesced): h = silu(gate / rms) *
// (up / rms), then hi/lo of h into a_h.
struct EpiSwiGLU {
  static constexpr bool kCols = true;
  // Prefetched inputs depend on the tile index (re-fetched per 64-column tile).
  static constexpr bool kPrePerTile = true;
  static constexpr int kPre = 64;   // 1 / rms per row
  struct Params {
    BatchDev d;
  };
  __device__ __forceinline__ static void prefetch(const Params& ep, int, float* pre, int e) {
    prefetch_inv_rms(ep.d.ssq, pre, e);
  }
  __device__ __forceinline__ static void apply(const Params&, int, int, float (&)[64], const float*) {}
  __device__ __forceinline__ static void cols(const Params& ep, int t, float* tile, int tid, const float* pre,
                                              int ra, int rb) {
    const int c = tid & 31;
    const int batch = ep.d.batch;
#pragma unroll 4
    for (int r = ra + (tid >> 5); r < rb; r += 4) {
      const float rr = pre[r];
      const float gt = tile[r * kTcCombStride + c] * rr, up = tile[r * kTcCombStride + 32 + c] * rr;
      put_hilo(ep.d.a_h, kBI, r, 32 * t + c, r < batch ? gt / (1.f + expf(-gt)) * up : 0.f);
    }
  }
};

// LM-head epilogue: logits of 64 vocabulary rows; per sequence the best
// (value, lowest index) of the tile -> lm_part[t][seq]; optional logits.
struct EpiArgmax {
  static constexpr bool kCols = false;
  // Prefetched inputs are the same for every tile.
  static constexpr bool kPrePerTile = false;
  static constexpr int kPre = 64;   // 1 / rms per row
  struct Params {
    BatchDev d;
    float* logits;  // [batch][V] or null
  };
  __device__ __forceinline__ static void prefetch(const Params& ep, int, float* pre, int e) {
    prefetch_inv_rms(ep.d.ssq, pre, e);
  }
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, float (&v)[64], const float* pre) {
    const BatchDev& d = ep.d;
    if (seq >= d.batch) return;
    const float r = pre[seq];
    float best = -INFINITY;
    int bi = 0;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      v[c] *= r;
      if (v[c] > best) { best = v[c]; bi = c; }
    }
    d.lm_part[(size_t)t * kBMax + seq] = argmax_key(best, 64 * t + bi);
    if (ep.logits) {
      float* o = ep.logits + (size_t)seq * kBV + 64 * t;
#pragma unroll
      for (int c = 0; c < 64; c += 4) *reinterpret_cast<float4*>(o + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
    }
  }
};

// Split-KV attention on tensor cores, one warp per item (sequence b, KV head
// h, span s of `span` chunks of 64 positions <= pos_b) for the GQA pair of
// query heads (2h, 2h+1).  Replaces warp_attention (src/attention.cuh:100-167)
// for many sequences at once.
//   - the warp walks its span's chunks with an online softmax, K and V of the
//     next chunk arriving by cp.async into the other half of a double buffer
//     while the current chunk is computed (64 rows of 128 B each, 16-byte
//     chunks XOR-swizzled by row so ldmatrix is bank-conflict free); rows
//     past pos are copied too but masked;
//   - S = Q K^T and O = P V run as mma.sync m16n8k16 (bf16, fp32 accumulate).
//     Q and P enter as two bf16 rows each (hi = bf16(v), lo = bf16(v - hi);
//     rows 0/1 = hi of heads 0/1, rows 2/3 = lo) so the products keep ~16
//     mantissa bits; the score accumulators are reused as the A operand of
//     P V (same fragment layout);
//   - a span that covers the whole context writes hi/lo of the two heads'
//     outputs into a_att directly; otherwise the partial {acc[2][64], m[2],
//     l[2]} goes to part[b][h][s] and the warp that completes the last span
//     of (b, h) (ticket in acnt) merges all spans in span order -- no
//     separate merge pass.
constexpr int kBAttnWarps = 2;
#ifndef MK_BATTN_BUFS
#define MK_BATTN_BUFS 3
#endif
constexpr int kBAttnBufs = MK_BATTN_BUFS;   // chunks of K/V per warp: current + in flight
// bf16 cache: K/V chunks land swizzled in kBAttnBufs buffers.  fp8 cache
// (e4m3): the chunks land unswizzled in kBAttnBufs staging buffers (4 KB
// each) and are converted into one f16 working tile (swizzled) before use.
template <bool F8>
struct AttnWarpSmemT {
  static constexpr int kTiles = F8 ? 1 : kBAttnBufs;
  alignas(128) uint16_t k[kTiles][kBChunk * kBD];  // 8 KB each, swizzled (bf16 or f16)
  alignas(128) uint16_t v[kTiles][kBChunk * kBD];
  alignas(128) uint8_t k8[F8 ? kBAttnBufs : 1][F8 ? kBChunk * kBD : 16];   // fp8 staging
  alignas(128) uint8_t v8[F8 ? kBAttnBufs : 1][F8 ? kBChunk * kBD : 16];
  alignas(16) float q[2][kBD];
};
template <bool F8>
constexpr size_t attn_smem_bytes() { return sizeof(AttnWarpSmemT<F8>) * kBAttnWarps; }


__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_n() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// byte offset of (row, 16-byte chunk) in a swizzled 64 x 128 B tile
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
// bf16 hi / lo terms of v packed as bf16x2 pairs
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
  hi = pack_bf16x2(__bfloat162float(ha), __bfloat162float(hb));
  lo = pack_bf16x2(a - __bfloat162float(ha), b - __bfloat162float(hb));
}

// f16 counterparts for the fp8-cache attention (e4m3 converts to f16
// exactly; all operands of one mma share a type).
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <bool F16>
__device__ __forceinline__ void split2t(float a, float b, uint32_t& hi, uint32_t& lo) {
  if constexpr (F16) {
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    hi = pack_f16x2(__half2float(ha), __half2float(hb));
    lo = pack_f16x2(a - __half2float(ha), b - __half2float(hb));
  } else {
    split2(a, b, hi, lo);
  }
}
template <bool F16>
__device__ __forceinline__ void mmat(float& d0, float& d1, float& d2, float& d3, uint32_t a0, uint32_t a1,
                                     uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (F16)
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    mma_bf16_16816(d0, d1, d2, d3, a0, a1, a2, a3, b0, b1);
}

// Merge of the chunk partials of (b, h) for both query heads: lanes load the
// chunks' (m, l) in parallel (32 chunks per round), then every lane sums its
// two output dimensions over the chunks with the weights broadcast by
// shuffle, loads batched eight chunks at a time.  Fixed summation order.
__device__ __forceinline__ void attn_merge(const BatchDev& d, int b, int h, int lane, int nc) {
  const float* base = d.part + ((size_t)b * kBNKV + h) * d.maxch * 132;
  float M[2] = {-INFINITY, -INFINITY};
  for (int c0 = 0; c0 < nc; c0 += 32) {
    const int c = c0 + lane;
    if (c < nc) {
      M[0] = fmaxf(M[0], __ldcg(base + (size_t)c * 132 + 64));
      M[1] = fmaxf(M[1], __ldcg(base + (size_t)c * 132 + 66 + 64));
    }
  }
  M[0] = warp_max(M[0]);
  M[1] = warp_max(M[1]);
  float den[2] = {0.f, 0.f}, o[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  for (int c0 = 0; c0 < nc; c0 += 32) {
    const int c = c0 + lane;
    float w[2] = {0.f, 0.f};
    if (c < nc) {
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        w[g] = expf(__ldcg(base + (size_t)c * 132 + g * 66 + 64) - M[g]);
        den[g] = fmaf(__ldcg(base + (size_t)c * 132 + g * 66 + 65), w[g], den[g]);
      }
    }
    const int cnt = min(32, nc - c0);
    for (int k0 = 0; k0 < cnt; k0 += 8) {
      float2 a[8][2];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int cc = min(k0 + k, cnt - 1);
#pragma unroll
        for (int g = 0; g < 2; ++g)
          a[k][g] = __ldcg(reinterpret_cast<const float2*>(base + (size_t)(c0 + cc) * 132 + g * 66 + 2 * lane));
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const float wk = __shfl_sync(0xffffffffu, w[g], (k0 + k) & 31);
          if (k0 + k < cnt) {
            o[g][0] = fmaf(a[k][g].x, wk, o[g][0]);
            o[g][1] = fmaf(a[k][g].y, wk, o[g][1]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const float inv = 1.f / warp_sum(den[g]);
    const int col = (2 * h + g) * kBD + 2 * lane;
    put_hilo(d.a_att, kBQ, b, col, o[g][0] * inv);
    put_hilo(d.a_att, kBQ, b, col + 1, o[g][1] * inv);
  }
}

template <bool F8>
__global__ void __launch_bounds__(kBAttnWarps * 32) battn_kernel(BatchDev d, int l, int span) {
  extern __shared__ __align__(128) uint8_t attn_smem_raw[];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  AttnWarpSmemT<F8>& sw = reinterpret_cast<AttnWarpSmemT<F8>*>(attn_smem_raw)[wid];
  const int wglob = blockIdx.x * kBAttnWarps + wid;
  const int nw = gridDim.x * kBAttnWarps;
  const int maxspan = (d.maxch + span - 1) / span;
  const int nitems = kBMax * kBNKV * maxspan;
  pdl_launch();
  pdl_wait();
  for (int it = wglob; it < nitems; it += nw) {
    const int s = it % maxspan, h = (it / maxspan) % kBNKV, b = it / (maxspan * kBNKV);
    if (b >= d.batch) continue;
    const int p = d.pos[b];
    const int nc = p / kBChunk + 1;              // chunks holding positions 0..p
    const int cs = s * span;
    if (cs >= nc) continue;
    const int ce = min(nc, cs + span);
    const int nspan = (nc + span - 1) / span;
    const size_t k_off = bkv_index(d, b, l, 0, h, 0), v_off = bkv_index(d, b, l, 1, h, 0);
    __syncwarp();   // the previous item's readers of sw are done
    // K and V of chunk c into buffer `buf`: bf16, 64 rows x 8 pieces of 16 B
    // swizzled; fp8, 64 rows x 4 pieces of 16 B plain.  Rows past max_seq
    // clamp (masked later).
    auto load = [&](int c, int buf) {
      if constexpr (F8) {
        const uint32_t ks = smem_u32(sw.k8[buf]), vs = smem_u32(sw.v8[buf]);
#pragma unroll
        for (int k = 0; k < kBChunk / 8; ++k) {
          const int idx = lane + 32 * k, row = idx >> 2, ch = idx & 3;
          const size_t src_row = (size_t)min(c * kBChunk + row, d.max_seq - 1);
          cp_async16(ks + (uint32_t)(row * 64 + ch * 16), d.kv8 + k_off + src_row * kBD + ch * 16);
          cp_async16(vs + (uint32_t)(row * 64 + ch * 16), d.kv8 + v_off + src_row * kBD + ch * 16);
        }
      } else {
        const uint32_t ks = smem_u32(sw.k[buf]), vs = smem_u32(sw.v[buf]);
#pragma unroll
        for (int k = 0; k < kBChunk / 4; ++k) {
          const int idx = lane + 32 * k, row = idx >> 3, ch = idx & 7;
          const size_t src_row = (size_t)min(c * kBChunk + row, d.max_seq - 1);
          cp_async16(ks + swz(row, ch), d.kv + k_off + src_row * kBD + ch * 8);
          cp_async16(vs + swz(row, ch), d.kv + v_off + src_row * kBD + ch * 8);
        }
      }
    };
#pragma unroll
    for (int i = 0; i < kBAttnBufs - 1; ++i) {
      if (cs + i < ce) load(cs + i, i);
      cp_async_commit();
    }
    {
      const float* qg = d.q + ((size_t)b * kBNQ + 2 * h) * kBD;
      *reinterpret_cast<float4*>(&sw.q[0][0] + 4 * lane) = __ldg(reinterpret_cast<const float4*>(qg) + lane);
    }
    __syncwarp();
    // A fragments of Q (rows 0/1: hi of heads 0/1, rows 2/3: lo), 4 k-steps
    uint32_t qa[4][2];   // a0 (cols 2tq..+1), a2 (cols 8+2tq..+1) for row g; rows >= 4 zero
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t hi0 = 0, lo0 = 0, hi1 = 0, lo1 = 0;
      if (g < 4) {
        const float* qr = &sw.q[g & 1][kk * 16 + 2 * tq];
        split2t<F8>(qr[0], qr[1], hi0, lo0);
        split2t<F8>(qr[8], qr[9], hi1, lo1);
      }
      qa[kk][0] = g < 2 ? hi0 : lo0;
      qa[kk][1] = g < 2 ? hi1 : lo1;
      if (g >= 4) { qa[kk][0] = 0; qa[kk][1] = 0; }
    }
    // Running softmax state of head g (lanes g < 2): max, denominator, and
    // the unnormalised output dims 8j + 2tq, +1.
    float M = -INFINITY, Lsum = 0.f, ro[8][2];
#pragma unroll
    for (int j = 0; j < 8; ++j) ro[j][0] = ro[j][1] = 0.f;
#pragma unroll 1
    for (int c = cs; c < ce; ++c) {
      const int buf = (c - cs) % kBAttnBufs;
      // Prefetch chunk c + bufs - 1 into the buffer freed by chunk c - 1,
      // then wait for chunk c (one commit group per chunk, empty past the
      // span).
      if (c + kBAttnBufs - 1 < ce) load(c + kBAttnBufs - 1, (c - cs + kBAttnBufs - 1) % kBAttnBufs);
      cp_async_commit();
      cp_async_wait_n<kBAttnBufs - 1>();
      __syncwarp();
      if constexpr (F8) {
        // e4m3 -> f16 (exact) into the swizzled working tile.
#pragma unroll
        for (int k = 0; k < kBChunk / 4; ++k) {
          const int idx = lane + 32 * k, row = idx >> 3, ch = idx & 7;
          const uint2 ka = *reinterpret_cast<const uint2*>(&sw.k8[buf][row * 64 + ch * 8]);
          const uint2 va = *reinterpret_cast<const uint2*>(&sw.v8[buf][row * 64 + ch * 8]);
          uint4 ko, vo;
          ko.x = e4m3x2_to_f16x2((uint16_t)ka.x); ko.y = e4m3x2_to_f16x2((uint16_t)(ka.x >> 16));
          ko.z = e4m3x2_to_f16x2((uint16_t)ka.y); ko.w = e4m3x2_to_f16x2((uint16_t)(ka.y >> 16));
          vo.x = e4m3x2_to_f16x2((uint16_t)va.x); vo.y = e4m3x2_to_f16x2((uint16_t)(va.x >> 16));
          vo.z = e4m3x2_to_f16x2((uint16_t)va.y); vo.w = e4m3x2_to_f16x2((uint16_t)(va.y >> 16));
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sw.k[0]) + swz(row, ch)) = ko;
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sw.v[0]) + swz(row, ch)) = vo;
        }
        __syncwarp();
      }
      const int tb = F8 ? 0 : buf;
      const uint32_t ks = smem_u32(sw.k[tb]), vs = smem_u32(sw.v[tb]);
      const int n = min(kBChunk, p + 1 - c * kBChunk);
      // S[16 x 64]: 8 n-tiles of 8 positions
      float sacc[kBNT][4];
#pragma unroll
      for (int j = 0; j < kBNT; ++j) { sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f; }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jp = 0; jp < kBNT / 2; ++jp) {
          // matrices: (n-tile 2jp, k lo), (2jp, k hi), (2jp+1, k lo), (2jp+1, k hi)
          const int mi = lane >> 3, r = lane & 7;
          const int row = (2 * jp + (mi >> 1)) * 8 + r, ch = kk * 2 + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(ks + swz(row, ch), b0, b1, b2, b3);
          mmat<F8>(sacc[2 * jp][0], sacc[2 * jp][1], sacc[2 * jp][2], sacc[2 * jp][3], qa[kk][0], 0u,
                         qa[kk][1], 0u, b0, b1);
          mmat<F8>(sacc[2 * jp + 1][0], sacc[2 * jp + 1][1], sacc[2 * jp + 1][2], sacc[2 * jp + 1][3],
                         qa[kk][0], 0u, qa[kk][1], 0u, b2, b3);
        }
      }
      // rows 0/1 (+ rows 2/3 from lane + 8): full scores of heads 0/1 in
      // lanes g = 0 / 1, positions 8j + 2tq, +1
      float sc[kBNT][2];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kBNT; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = sacc[j][e] + __shfl_down_sync(0xffffffffu, sacc[j][e], 8);
          const int pos = 8 * j + 2 * tq + e;
          sc[j][e] = pos < n ? v * 0.125f : -INFINITY;
          mx = fmaxf(mx, sc[j][e]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < kBNT; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sc[j][e] = expf(sc[j][e] - mx);
          ls += sc[j][e];
        }
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      ls += __shfl_xor_sync(0xffffffffu, ls, 2);
      // P as A operand: lanes g = 0/1 give hi of their head, lanes g = 2/3 the
      // lo of lane - 8's probabilities, other rows zero.
      uint32_t pa[kBKS][2];
#pragma unroll
      for (int kk = 0; kk < kBKS; ++kk) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int j = 2 * kk + hh;
          const float p0 = __shfl_up_sync(0xffffffffu, sc[j][0], 8), p1 = __shfl_up_sync(0xffffffffu, sc[j][1], 8);
          uint32_t hi, lo, hi2, lo2;
          split2t<F8>(sc[j][0], sc[j][1], hi, lo);
          split2t<F8>(p0, p1, hi2, lo2);
          pa[kk][hh] = g < 2 ? hi : (g < 4 ? lo2 : 0u);
        }
      }
      // O[16 x 64]: 8 n-tiles of 8 dims, K = positions
      float oacc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) { oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f; }
#pragma unroll
      for (int kk = 0; kk < kBKS; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
          // .trans matrices: (pos lo 8, dims 2jp), (pos hi 8, dims 2jp), (pos lo, 2jp+1), (pos hi, 2jp+1)
          const int mi = lane >> 3, r = lane & 7;
          const int row = kk * 16 + (mi & 1) * 8 + r, ch = 2 * jp + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vs + swz(row, ch), b0, b1, b2, b3);
          mmat<F8>(oacc[2 * jp][0], oacc[2 * jp][1], oacc[2 * jp][2], oacc[2 * jp][3], pa[kk][0], 0u,
                         pa[kk][1], 0u, b0, b1);
          mmat<F8>(oacc[2 * jp + 1][0], oacc[2 * jp + 1][1], oacc[2 * jp + 1][2], oacc[2 * jp + 1][3],
                         pa[kk][0], 0u, pa[kk][1], 0u, b2, b3);
        }
      }
      // Fold this chunk into the running state (lanes g < 2 hold head g).
      const float Mn = fmaxf(M, mx);
      const float ca = expf(M - Mn), cb = expf(mx - Mn);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v0 = oacc[j][0] + __shfl_down_sync(0xffffffffu, oacc[j][0], 8);
        const float v1 = oacc[j][1] + __shfl_down_sync(0xffffffffu, oacc[j][1], 8);
        ro[j][0] = ro[j][0] * ca + v0 * cb;
        ro[j][1] = ro[j][1] * ca + v1 * cb;
      }
      Lsum = Lsum * ca + ls * cb;
      M = Mn;
      __syncwarp();   // this buffer's readers are done before it is refilled
    }
    if (nspan == 1) {
      // The whole context in one item: normalise and write the outputs.
      if (g < 2) {
        const float inv = 1.f / Lsum;
        const int col = (2 * h + g) * kBD;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          put_hilo(d.a_att, kBQ, b, col + 8 * j + 2 * tq, ro[j][0] * inv);
          put_hilo(d.a_att, kBQ, b, col + 8 * j + 2 * tq + 1, ro[j][1] * inv);
        }
      }
      continue;
    }
    // Partial {acc[2][64], m[2], l[2]} of span s; the warp that completes
    // the last span of (b, h) merges them.
    float* o = d.part + (((size_t)b * kBNKV + h) * d.maxch + s) * 132;
    if (g < 2) {
#pragma unroll
      for (int j = 0; j < 8; ++j) __stcg(reinterpret_cast<float2*>(o + g * 66 + 8 * j + 2 * tq), make_float2(ro[j][0], ro[j][1]));
    }
    if (lane == 0 || lane == 4) {
      const int hh = lane >> 2;
      __stcg(o + hh * 66 + 64, M);
      __stcg(o + hh * 66 + 65, Lsum);
    }
    // Ticket: the acq_rel atomic releases this warp's partial stores (ordered
    // before it by __syncwarp; release is cumulative) and, for the last
    // warp, acquires every other span's.
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      const int old = atom_add_acq_rel(d.acnt + b * kBNKV + h, 1);
      last = old == nspan - 1;
      if (last) d.acnt[b * kBNKV + h] = 0;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) attn_merge(d, b, h, lane, nspan);
  }
}

// Per-sequence argmax over the LM tiles -> out[b]; advances pos[b].
__global__ void bargmax_kernel(BatchDev d, int* __restrict__ out) {
  const int b = blockIdx.x;
  __shared__ unsigned long long red[32];
  pdl_launch();
  pdl_wait();
  unsigned long long best = 0;
  for (int t = threadIdx.x; t < kBLMTiles; t += blockDim.x) {
    const unsigned long long k = d.lm_part[(size_t)t * kBMax + b];
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    best = red[0] > best ? red[0] : best;
    out[b] = 0x7fffffff - (int)(uint32_t)(best & 0xffffffffu);
    d.pos[b] += 1;
  }
}

}  // namespace mk

// Test entry point (see include/megakernel.h).
extern "C" int megakernel_tc_gemm_test_split(const float* d_x, int rows, const void* d_w, int K, int N, int ksplit,
                                             float* d_out, void* stream) {
  if (!d_x || !d_w || !d_out || rows < 1 || rows > 64 || K < 64 || K % 64 != 0 || N < 64 || N % 64 != 0 ||
      ksplit < 1 || ksplit > mk::kTcMaxSplit || (ksplit - 1) * ((K / 64 + ksplit - 1) / ksplit) >= K / 64)
    return MK_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return MK_ERR_CUDA;
  __nv_bfloat16* a = nullptr;
  CUtensorMap* maps = nullptr;
  int* err = nullptr;
  int rc = MK_OK;
  if (cudaMalloc(&a, (size_t)128 * K * 2) != cudaSuccess || cudaMalloc(&maps, 2 * sizeof(CUtensorMap)) != cudaSuccess ||
      cudaMalloc(&err, sizeof(int)) != cudaSuccess) {
    rc = MK_ERR_OOM;
  } else {
    CUtensorMap h[2];
    if (!mk::tc_make_map(&h[0], a, 128, (uint64_t)K, 128) || !mk::tc_make_map(&h[1], d_w, (uint64_t)N, (uint64_t)K, 32)) {
      rc = MK_ERR_INVALID_ARG;
    } else {
      cudaMemcpyAsync(maps, h, sizeof(h), cudaMemcpyHostToDevice, st);
      cudaMemsetAsync(err, 0, sizeof(int), st);
      mk::hilo_split_kernel<<<64, 256, 0, st>>>(d_x, rows, K, a);
      mk::TcGemmParams p{maps, maps + 1, K, N / 64, 0, err, 1000000000LL, ksplit, nullptr};
      mk::EpiStore::Params ep{d_out, N, rows};
      if (mk::tc_gemm_launch<mk::EpiStore>(p, ep, sms, st) != cudaSuccess) rc = MK_ERR_LAUNCH;
      int herr = 0;
      if (cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
          cudaStreamSynchronize(st) != cudaSuccess)
        rc = MK_ERR_CUDA;
      else if (rc == MK_OK)
        rc = herr;
    }
  }
  cudaFree(a);
  cudaFree(maps);
  cudaFree(err);
  return rc;
}

extern "C" int megakernel_tc_gemm_test(const float* d_x, int rows, const void* d_w, int K, int N, float* d_out,
                                       void* stream) {
  return megakernel_tc_gemm_test_split(d_x, rows, d_w, K, N, 1, d_out, stream);
}

// The same GEMM on e4m3 weights: d_w8 [N][K] e4m3 bytes, d_scale [N] per-row
// scales (W = scale * e4m3); the converter-warp path of the batched GEMMs.
extern "C" int megakernel_tc_gemm_test_e4m3(const float* d_x, int rows, const void* d_w8, const float* d_scale,
                                             int K, int N, float* d_out, void* stream) {
  if (!d_x || !d_w8 || !d_scale || !d_out || rows < 1 || rows > 64 || K < 64 || K % 64 != 0 || N < 64 ||
      N % 64 != 0)
    return MK_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return MK_ERR_CUDA;
  __nv_bfloat16* a = nullptr;
  CUtensorMap* maps = nullptr;
  int* err = nullptr;
  int rc = MK_OK;
  if (cudaMalloc(&a, (size_t)128 * K * 2) != cudaSuccess || cudaMalloc(&maps, 2 * sizeof(CUtensorMap)) != cudaSuccess ||
      cudaMalloc(&err, sizeof(int)) != cudaSuccess) {
    rc = MK_ERR_OOM;
  } else {
    CUtensorMap h[2];
    if (!mk::tc_make_map(&h[0], a, 128, (uint64_t)K, 128) ||
        !mk::tc_make_map_e4m3(&h[1], d_w8, (uint64_t)N, (uint64_t)K, 32)) {
      rc = MK_ERR_INVALID_ARG;
    } else {
      cudaMemcpyAsync(maps, h, sizeof(h), cudaMemcpyHostToDevice, st);
      cudaMemsetAsync(err, 0, sizeof(int), st);
      mk::hilo_split_kernel<<<64, 256, 0, st>>>(d_x, rows, K, a);
      mk::TcGemmParams p{maps, maps + 1, K, N / 64, 0, err, 1000000000LL, 1, d_scale};
      mk::EpiStore::Params ep{d_out, N, rows};
      if (mk::tc_gemm_launch<mk::EpiStore, true>(p, ep, sms, st) != cudaSuccess) rc = MK_ERR_LAUNCH;
      int herr = 0;
      if (cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
          cudaStreamSynchronize(st) != cudaSuccess)
        rc = MK_ERR_CUDA;
      else if (rc == MK_OK)
        rc = herr;
    }
  }
  cudaFree(a);
  cudaFree(maps);
  cudaFree(err);
  return rc;
}

// ============================================================================
// Batched decode: host side.
// ============================================================================
namespace {

struct BatchState {
  int device = 0, sms = 0, batch = 0, max_seq = 0;
  const __nv_bfloat16* wp[2 + 11 * mk::kBL] = {};
  mk::BatchDev d{};
  CUtensorMap* maps = nullptr;   // device copy: [0] a_x, [1] a_att, [2] a_h, [3 + 4l + k] layer maps, [3 + 4L] LM
  int last_error = 0;
  long long kv_bytes = 0;
  bool owns_kv = true;
  int* d_tmp = nullptr;          // [64] scratch tokens (prefill)
  // e4m3 weights (optional): per layer the q|k|v, O, gate|up and down
  // matrices, then the LM head, each row scaled by its own factor.
  uint8_t* w8 = nullptr;
  float* wsc = nullptr;
  size_t w8_off[4 * mk::kBL + 1] = {};
  size_t sc_off[4 * mk::kBL + 1] = {};
};

// Rows x cols of the matrix behind GEMM map k of a layer (0 q|k|v, 1 O,
// 2 gate|up, 3 down; 4: the LM head).
inline void gemm_matrix(int k, int& rows, int& cols) {
  using namespace mk;
  switch (k) {
    case 0: rows = kBQ + 2 * kBKV; cols = kBH; break;
    case 1: rows = kBH; cols = kBQ; break;
    case 2: rows = 2 * kBI; cols = kBH; break;
    case 3: rows = kBH; cols = kBI; break;
    default: rows = kBV; cols = kBH; break;
  }
}

// e4m3 copy of a bf16 matrix with one scale per row (max |w| / 448): one
// warp per row.
__global__ void quant_rows_kernel(const __nv_bfloat16* __restrict__ w, int rows, int cols, uint8_t* __restrict__ q,
                                  float* __restrict__ scale) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* wr = w + (size_t)row * cols;
  float amax = 0.f;
  for (int c = lane; c < cols; c += 32) amax = fmaxf(amax, fabsf(__bfloat162float(wr[c])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = 1.f / sc;
  uint16_t* qr = reinterpret_cast<uint16_t*>(q + (size_t)row * cols);
  for (int c = 2 * lane; c < cols; c += 64)
    qr[c >> 1] = mk::f32x2_to_e4m3x2(__bfloat162float(wr[c]) * inv, __bfloat162float(wr[c + 1]) * inv);
  if (lane == 0) scale[row] = sc;
}

enum { kMapAx = 0, kMapAatt = 1, kMapAh = 2, kMapLayer0 = 3 };
// GEMM launch parameters with K split over `ksplit` CTAs (one cluster) per
// output tile; every split keeps at least one K block.
mk::TcGemmParams gemm_params(const mk::BatchDev& d, const CUtensorMap* a, const CUtensorMap* w, int K, int ntiles,
                             int half_off, int ksplit) {
  const int kb = K / mk::kTcBK;
  if (ksplit > mk::kTcMaxSplit) ksplit = mk::kTcMaxSplit;
  while (ksplit > 1 && (ksplit - 1) * ((kb + ksplit - 1) / ksplit) >= kb) --ksplit;
  return mk::TcGemmParams{a, w, K, ntiles, half_off, d.err, 1000000000LL, ksplit, nullptr};
}
inline int map_layer(int l, int k) { return kMapLayer0 + 4 * l + k; }   // k: 0 qkv, 1 o, 2 gate/up, 3 down
inline int map_lm() { return kMapLayer0 + 4 * mk::kBL; }

void batch_free(BatchState* s) {
  if (!s) return;
  cudaFree(s->d.x); cudaFree(s->d.ssq); cudaFree(s->d.a_x); cudaFree(s->d.a_att); cudaFree(s->d.a_h);
  cudaFree(s->d.q); cudaFree(s->d.part); cudaFree(s->d.lm_part);
  if (s->owns_kv) { cudaFree(s->d.kv); cudaFree(s->d.kv8); }
  cudaFree(s->w8);
  cudaFree(s->wsc);
  cudaFree(s->d_tmp);
  cudaFree(const_cast<float*>(s->d.rope_cos)); cudaFree(const_cast<float*>(s->d.rope_sin));
  cudaFree(s->d.pos); cudaFree(s->d.err); cudaFree(s->maps); cudaFree(s->d.acnt);
  delete s;
}

template <class T>
bool balloc(T** p, size_t bytes) {
  return cudaMalloc(reinterpret_cast<void**>(p), bytes) == cudaSuccess && cudaMemset(*p, 0, bytes) == cudaSuccess;
}

// ext_kv: bind to a caller-owned cache of one sequence ([L][2][KVH][max_seq][hd])
// instead of allocating [batch] caches (used by the parallel prefill).
// kv_fp8: keep the cache in e4m3 (half the bytes; own cache only).
// w_fp8: run the GEMMs on an e4m3 copy of the weights (per-row scales).
BatchState* batch_init(const void* d_weights, const long long* offsets, int num_offsets, int batch, int max_seq,
                       __nv_bfloat16* ext_kv = nullptr, bool kv_fp8 = false, bool w_fp8 = false) {
  using namespace mk;
  if (!d_weights || !offsets || batch < 1 || batch > kBMax || max_seq < 1 || (kv_fp8 && ext_kv)) return nullptr;
  if (infer_shape(offsets, num_offsets) != 0) return nullptr;   // d64 shape only
  for (int i = 0; i < num_offsets; ++i)
    if (offsets[i] < 0 || (offsets[i] & 15) != 0) return nullptr;
  // The fused maps need w_q|w_k|w_v and w_gate|w_up back to back.
  for (int l = 0; l < kBL; ++l) {
    const long long* o = offsets + 2 + 11 * l;
    if (o[2] != o[1] + (long long)kBQ * kBH * 2 || o[3] != o[2] + (long long)kBKV * kBH * 2 ||
        o[9] != o[8] + (long long)kBI * kBH * 2)
      return nullptr;
  }
  BatchState* s = new BatchState();
  if (cudaGetDevice(&s->device) != cudaSuccess ||
      cudaDeviceGetAttribute(&s->sms, cudaDevAttrMultiProcessorCount, s->device) != cudaSuccess) {
    delete s;
    return nullptr;
  }
  s->batch = batch;
  s->max_seq = max_seq;
  for (int i = 0; i < num_offsets; ++i)
    s->wp[i] = reinterpret_cast<const __nv_bfloat16*>(static_cast<const char*>(d_weights) + offsets[i]);
  BatchDev& d = s->d;
  d.batch = batch;
  d.max_seq = max_seq;
  d.maxch = (max_seq + kBChunk - 1) / kBChunk;
  s->kv_bytes = ext_kv ? 0 : (long long)batch * kBL * 2 * kBNKV * (long long)max_seq * kBD * (kv_fp8 ? 1 : 2);
  s->owns_kv = ext_kv == nullptr;
  float *rc = nullptr, *rs = nullptr;
  const bool ok =
      balloc(&d.x, sizeof(float) * kBMax * kBH) && balloc(&d.ssq, sizeof(float) * kBHT * kBMax) &&
      balloc(&d.a_x, 2 * 128 * kBH) && balloc(&d.a_att, 2 * 128 * kBQ) && balloc(&d.a_h, 2 * 128 * kBI) &&
      balloc(&d.q, sizeof(float) * kBMax * kBNQ * kBD) &&
      balloc(&d.part, sizeof(float) * (size_t)kBMax * kBNKV * d.maxch * 132) &&
      balloc(&d.lm_part, sizeof(unsigned long long) * (size_t)kBLMTiles * kBMax) &&
      (ext_kv ? (d.kv = ext_kv) != nullptr
              : (kv_fp8 ? balloc(&d.kv8, (size_t)s->kv_bytes) : balloc(&d.kv, (size_t)s->kv_bytes))) &&
      balloc(&s->d_tmp, sizeof(int) * kBMax) && balloc(&rc, sizeof(float) * (size_t)max_seq * 32) &&
      balloc(&rs, sizeof(float) * (size_t)max_seq * 32) && balloc(&d.pos, sizeof(int) * kBMax) &&
      balloc(&d.err, sizeof(int) * 4) && balloc(&s->maps, sizeof(CUtensorMap) * (map_lm() + 1)) &&
      balloc(&d.acnt, sizeof(int) * kBMax * kBNKV);
  d.rope_cos = rc;
  d.rope_sin = rs;
  if (!ok) { batch_free(s); return nullptr; }
  {
    std::vector<float> hc((size_t)max_seq * 32), hs((size_t)max_seq * 32);
    host_rope(kBD, 1.0e6, max_seq, hc.data(), hs.data());
    if (cudaMemcpy(rc, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(rs, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
      batch_free(s);
      return nullptr;
    }
  }
  std::vector<CUtensorMap> h(map_lm() + 1);
  bool mok = tc_make_map(&h[kMapAx], d.a_x, 128, kBH, 128) && tc_make_map(&h[kMapAatt], d.a_att, 128, kBQ, 128) &&
             tc_make_map(&h[kMapAh], d.a_h, 128, kBI, 128);
  for (int l = 0; l < kBL && mok; ++l) {
    const int b = 2 + 11 * l;
    mok = tc_make_map(&h[map_layer(l, 0)], s->wp[b + 1], kBQ + 2 * kBKV, kBH, 32) &&
          tc_make_map(&h[map_layer(l, 1)], s->wp[b + 6], kBH, kBQ, 32) &&
          tc_make_map(&h[map_layer(l, 2)], s->wp[b + 8], 2 * kBI, kBH, 32) &&
          tc_make_map(&h[map_layer(l, 3)], s->wp[b + 10], kBH, kBI, 32);
  }
  mok = mok && tc_make_map(&h[map_lm()], s->wp[0], kBV, kBH, 32);
  if (mok && w_fp8) {
    // e4m3 copies of the GEMM weights; their maps replace the bf16 ones.
    size_t wo = 0, so = 0;
    for (int m = 0; m <= 4 * kBL; ++m) {
      int rows, cols;
      gemm_matrix(m == 4 * kBL ? 4 : m % 4, rows, cols);
      s->w8_off[m] = wo;
      s->sc_off[m] = so;
      wo += (size_t)rows * cols;
      so += (size_t)rows;
    }
    mok = balloc(&s->w8, wo) && balloc(&s->wsc, so * sizeof(float));
    for (int m = 0; m <= 4 * kBL && mok; ++m) {
      const int k = m == 4 * kBL ? 4 : m % 4, l = m / 4;
      int rows, cols;
      gemm_matrix(k, rows, cols);
      const int wkey = k == 0 ? 1 : (k == 1 ? 6 : (k == 2 ? 8 : 10));
      const __nv_bfloat16* src = k == 4 ? s->wp[0] : s->wp[2 + 11 * l + wkey];
      quant_rows_kernel<<<(rows + 7) / 8, 256>>>(src, rows, cols, s->w8 + s->w8_off[m], s->wsc + s->sc_off[m]);
      mok = cudaGetLastError() == cudaSuccess &&
            tc_make_map_e4m3(&h[k == 4 ? map_lm() : map_layer(l, k)], s->w8 + s->w8_off[m], rows, cols, 32);
    }
    mok = mok && cudaDeviceSynchronize() == cudaSuccess;
  }
  if (!mok || cudaMemcpy(s->maps, h.data(), sizeof(CUtensorMap) * h.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    batch_free(s);
    return nullptr;
  }
  return s;
}

// One step for every sequence: input tokens from `forced` (device, [batch])
// or, when null, from `prev_out`; next tokens to `out`; optional logits.
// Launch with programmatic stream serialization: the kernel may start while
// the previous one drains; it calls griddepcontrol.wait before reading it.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <class T>
struct Tag { using type = T; };

int batch_step(BatchState* s, const int* forced, const int* prev_out, int* out, float* logits, cudaStream_t st) {
  using namespace mk;
  const BatchDev& d = s->d;
  const CUtensorMap* M = s->maps;
  if (launch_pdl(bembed_kernel, kBMax, 256, 0, st, d, s->wp[0], s->wp[2], forced, prev_out) != cudaSuccess)
    return ::MK_ERR_LAUNCH;
  static bool attn_attr = false;
  if (!attn_attr) {
    if (cudaFuncSetAttribute(battn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<false>()) != cudaSuccess ||
        cudaFuncSetAttribute(battn_kernel<false>, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess ||
        cudaFuncSetAttribute(battn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<true>()) != cudaSuccess ||
        cudaFuncSetAttribute(battn_kernel<true>, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    attn_attr = true;
  }
  // 2-warp blocks, as many as are resident per SM at once (shared memory
  // and registers; the occupancy calculator's answer, asked once).
  static int bps_cache[2] = {0, 0};
  int& bps = bps_cache[d.kv8 != nullptr ? 1 : 0];
  if (bps == 0) {
    const cudaError_t e = d.kv8 != nullptr
        ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, battn_kernel<true>, kBAttnWarps * 32, attn_smem_bytes<true>())
        : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, battn_kernel<false>, kBAttnWarps * 32, attn_smem_bytes<false>());
    if (e != cudaSuccess || bps < 1) { bps = 0; return ::MK_ERR_LAUNCH; }
  }
  const int attn_blocks = s->sms * bps;
  // Chunks per attention item: split each (sequence, head) into as many
  // spans as there are warp slots for all of them at once, at the
  // engine's capacity; never more items than slots (a second wave of items
  // would double the layer's attention time).
  const int per_pair = std::max(1, s->sms * bps * kBAttnWarps / (d.batch * kBNKV));
  const int attn_span = (d.maxch + per_pair - 1) / per_pair;
  const bool f8 = d.kv8 != nullptr;
  // Split-K factors of the q/k/v, O, gate/up and down GEMMs (cluster
  // split K, partials pushed into rank 0's shared memory).  Measured on B200
  // (64 sequences at position 1024, ms per step): {1, 2, 1, 3} 2.049,
  // {1, 2, 1, 4} 2.030, {1, 1, 1, 4} 2.095, {2, 2, 1, 4} 2.033,
  // {1, 2, 2, 4} 2.178, {2, 2, 2, 4} 2.164; with the 256-column LM head,
  // {1, 2, 1, 4} 1.963 and {2, 2, 1, 4} 1.957, but over the bench's 256
  // steps (positions 1024-1279) 2.007 and 2.015: {1, 2, 1, 4} kept.  (The earlier form -- partials
  // through global memory, a ticket, the last CTA summing, epilogue inputs
  // loaded after the MMAs -- took 2.463 at {1, 2, 1, 3}.)
  int ks[4] = {1, 2, 1, 4};
  if (const char* e = getenv("MK_BATCH_KSPLIT")) {
    int t[4];
    if (sscanf(e, "%d,%d,%d,%d", &t[0], &t[1], &t[2], &t[3]) == 4)
      for (int k = 0; k < 4; ++k) ks[k] = t[k] < 1 ? 1 : (t[k] > kTcMaxSplit ? kTcMaxSplit : t[k]);
  }
  const bool w8 = s->w8 != nullptr;
  // GEMM of map slot m (layer l, kind k; m = 4L: LM head) on the bf16 or
  // the e4m3 weights.
#if MK_TC_STAMPS
  int tl_next = 0;
  {
    void* tl = nullptr;
    if (cudaGetSymbolAddress(&tl, g_tc_tl) == cudaSuccess) cudaMemsetAsync(tl, 0xff, sizeof(g_tc_tl), st);
    if (cudaGetSymbolAddress(&tl, g_tc_stamps) == cudaSuccess) cudaMemsetAsync(tl, 0, sizeof(g_tc_stamps), st);
  }
#endif
  auto gemm = [&](auto epi_tag, TcGemmParams p, const auto& ep, int m) -> cudaError_t {
    using Epi = typename decltype(epi_tag)::type;
#if MK_TC_STAMPS
    p.tl = tl_next++;
    const char* ss = getenv("MK_TC_STAMP_SLOT");
    p.stamp = ss != nullptr && atoi(ss) == p.tl;
#endif
    if (!w8) return tc_gemm_launch<Epi, false>(p, ep, s->sms, st);
    p.wscale = s->wsc + s->sc_off[m];
    return tc_gemm_launch<Epi, true>(p, ep, s->sms, st);
  };
  for (int l = 0; l < kBL; ++l) {
    const int b = 2 + 11 * l;
    const __nv_bfloat16* g_next = l + 1 < kBL ? s->wp[b + 11] : s->wp[1];
    if (gemm(Tag<EpiQKV>{}, gemm_params(d, M + kMapAx, M + map_layer(l, 0), kBH, (kBQ + 2 * kBKV) / 64, 0, ks[0]),
             EpiQKV::Params{d, l, s->wp[b + 4], s->wp[b + 5]}, 4 * l) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    if ((f8 ? launch_pdl(battn_kernel<true>, attn_blocks, kBAttnWarps * 32, attn_smem_bytes<true>(), st, d, l, attn_span)
            : launch_pdl(battn_kernel<false>, attn_blocks, kBAttnWarps * 32, attn_smem_bytes<false>(), st, d, l,
                         attn_span)) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    if (gemm(Tag<EpiResid>{}, gemm_params(d, M + kMapAatt, M + map_layer(l, 1), kBQ, kBH / 64, 0, ks[1]),
             EpiResid::Params{d, d.a_x, s->wp[b + 7]}, 4 * l + 1) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    if (gemm(Tag<EpiSwiGLU>{}, gemm_params(d, M + kMapAx, M + map_layer(l, 2), kBH, kBI / 32, kBI, ks[2]),
             EpiSwiGLU::Params{d}, 4 * l + 2) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    if (gemm(Tag<EpiResid>{}, gemm_params(d, M + kMapAh, M + map_layer(l, 3), kBI, kBH / 64, 0, ks[3]),
             EpiResid::Params{d, d.a_x, g_next}, 4 * l + 3) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
  }
  // LM head: bf16 weights in CTA tiles of 4 x 64 columns (the activation
  // operand is re-read a quarter as often); e4m3 weights in 64-column tiles.
  {
    TcGemmParams p = gemm_params(d, M + kMapAx, M + map_lm(), kBH, kBLMTiles, 0, 1);
    const EpiArgmax::Params ep{d, logits};
#if MK_TC_STAMPS
    p.tl = tl_next++;
#endif
    const cudaError_t e = w8 ? (p.wscale = s->wsc + s->sc_off[4 * kBL], tc_gemm_launch<EpiArgmax, true>(p, ep, s->sms, st))
                             : tc_gemm_launch<EpiArgmax, false, 4>(p, ep, s->sms, st);
    if (e != cudaSuccess) return ::MK_ERR_LAUNCH;
  }
  if (launch_pdl(bargmax_kernel, s->batch, 256, 0, st, d, out) != cudaSuccess) return ::MK_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? ::MK_OK : ::MK_ERR_LAUNCH;
}

int batch_finish(BatchState* s, cudaStream_t st, int rc) {
  int herr = 0;
  if (cudaMemcpyAsync(&herr, s->d.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    rc = MK_ERR_CUDA;
  else if (rc == MK_OK && herr != 0)
    rc = herr;
  if (herr != 0) cudaMemsetAsync(s->d.err, 0, sizeof(int), st);
  s->last_error = rc;
  return rc;
}

__global__ void bset_pos_kernel(int* pos, int base, int rows) {
  const int b = threadIdx.x;
  if (b < mk::kBMax) pos[b] = b < rows ? base + b : 0;
}

// Parallel prefill of n prompt tokens at positions pos0 .. pos0+n-1 of the
// bound cache: 64 positions per batched step (rows = consecutive positions
// of sequence 0; row r attends to positions <= pos0 + 64k + r, all written
// by the step's QKV epilogue before its attention kernel runs).  The greedy
// token after the last prompt token goes to d_next.
int batch_prefill(BatchState* s, const int* d_tokens, int n, int pos0, int* d_next, cudaStream_t st) {
  using namespace mk;
  s->d.seq_mode = 1;
  int rc = ::MK_OK;
  int rows = 0;
  for (int k = 0; k * kBMax < n && rc == ::MK_OK; ++k) {
    rows = n - k * kBMax < kBMax ? n - k * kBMax : kBMax;
    s->batch = rows;
    s->d.batch = rows;
    bset_pos_kernel<<<1, kBMax, 0, st>>>(s->d.pos, pos0 + k * kBMax, rows);
    rc = batch_step(s, d_tokens + (size_t)k * kBMax, nullptr, s->d_tmp, nullptr, st);
  }
  if (rc == ::MK_OK &&
      cudaMemcpyAsync(d_next, s->d_tmp + rows - 1, sizeof(int), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    rc = ::MK_ERR_CUDA;
  return batch_finish(s, st, rc);
}

// Frees the parallel-prefill state of a batch-1 engine (declared in megakernel.cu).
void prefill_free(void* p) {
  if (p) batch_free(static_cast<BatchState*>(p));
}

}  // namespace

// Parallel prefill for the batch-1 engine (see include/megakernel.h).
extern "C" int megakernel_prefill(void* handle, const int* d_tokens, int n_tokens, int* d_next, void* stream) {
  State* st = static_cast<State*>(handle);
  if (!st || !d_tokens || !d_next || n_tokens < 1) return MK_ERR_INVALID_ARG;
  if (st->shape_id != 0) return set_err(st, MK_ERR_SHAPE);
  if (st->pos + n_tokens > st->max_seq) return set_err(st, MK_ERR_CAPACITY);
  if (cudaSetDevice(st->device) != cudaSuccess) return set_err(st, MK_ERR_CUDA);
  if (!st->prefill) {
    st->prefill = batch_init(st->d_weights, st->offsets.data(), (int)st->offsets.size(), mk::kBMax, st->max_seq,
                             st->d_kv);
    if (!st->prefill) return set_err(st, MK_ERR_OOM);
  }
  // NULL: the default stream, as the reference's calls use, so the launch is
  // ordered after the caller's earlier default-stream work on its buffers.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = batch_prefill(static_cast<BatchState*>(st->prefill), d_tokens, n_tokens, st->pos, d_next, s);
  if (rc == MK_OK) st->pos += n_tokens;
  return set_err(st, rc);
}

#if MK_TC_STAMPS
// Profiling build only: copies the GEMM stamps [256][64] (u64 ns) to host.
extern "C" int megakernel_tc_stamps(void* h_out) {
  return cudaMemcpyFromSymbol(h_out, mk::g_tc_stamps, sizeof(mk::g_tc_stamps)) == cudaSuccess ? 0 : -2;
}
// Profiling build only: the last step's GEMM timeline [160][3] (u64 ns:
// first entry, first release from griddepcontrol.wait, ~last exit).
extern "C" int megakernel_tc_timeline(void* h_out) {
  return cudaMemcpyFromSymbol(h_out, mk::g_tc_tl, sizeof(mk::g_tc_tl)) == cudaSuccess ? 0 : -2;
}
#endif

extern "C" {

void* megakernel_batch_init(const void* d_weights, const long long* offsets, int num_offsets, int batch,
                            int max_seq) {
  return batch_init(d_weights, offsets, num_offsets, batch, max_seq);
}

void* megakernel_batch_init_ex(const void* d_weights, const long long* offsets, int num_offsets, int batch,
                               int max_seq, int flags) {
  if (flags & ~(MK_KV_FP8_E4M3 | MK_W_FP8_E4M3)) return nullptr;
  return batch_init(d_weights, offsets, num_offsets, batch, max_seq, nullptr, (flags & MK_KV_FP8_E4M3) != 0,
                    (flags & MK_W_FP8_E4M3) != 0);
}

void megakernel_batch_free(void* handle) {
  if (!handle) return;
  cudaDeviceSynchronize();
  batch_free(static_cast<BatchState*>(handle));
}

int megakernel_batch_size(void* handle) { return handle ? static_cast<BatchState*>(handle)->batch : MK_ERR_INVALID_ARG; }

int megakernel_batch_step(void* handle, const int* d_tokens, int* d_out, float* d_logits, void* stream) {
  if (!handle || !d_tokens || !d_out) return MK_ERR_INVALID_ARG;
  BatchState* s = static_cast<BatchState*>(handle);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return batch_finish(s, st, batch_step(s, d_tokens, nullptr, d_out, d_logits, st));
}

int megakernel_batch_decode_n(void* handle, const int* d_forced, int n_forced, int n_steps, int* d_out,
                              void* stream) {
  if (!handle || !d_forced || !d_out || n_forced < 1 || n_steps < n_forced) return MK_ERR_INVALID_ARG;
  BatchState* s = static_cast<BatchState*>(handle);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = MK_OK;
  for (int t = 0; t < n_steps && rc == MK_OK; ++t) {
    const int* f = t < n_forced ? d_forced + (size_t)t * s->batch : nullptr;
    const int* prev = t > 0 ? d_out + (size_t)(t - 1) * s->batch : nullptr;
    rc = batch_step(s, f, prev, d_out + (size_t)t * s->batch, nullptr, st);
  }
  return batch_finish(s, st, rc);
}

int megakernel_batch_set_pos(void* handle, const int* h_pos) {
  if (!handle || !h_pos) return MK_ERR_INVALID_ARG;
  BatchState* s = static_cast<BatchState*>(handle);
  for (int b = 0; b < s->batch; ++b)
    if (h_pos[b] < 0 || h_pos[b] >= s->max_seq) return MK_ERR_CAPACITY;
  return cudaMemcpy(s->d.pos, h_pos, sizeof(int) * s->batch, cudaMemcpyHostToDevice) == cudaSuccess ? MK_OK
                                                                                                   : MK_ERR_CUDA;
}

int megakernel_batch_get_pos(void* handle, int* h_pos) {
  if (!handle || !h_pos) return MK_ERR_INVALID_ARG;
  BatchState* s = static_cast<BatchState*>(handle);
  return cudaMemcpy(h_pos, s->d.pos, sizeof(int) * s->batch, cudaMemcpyDeviceToHost) == cudaSuccess ? MK_OK
                                                                                                   : MK_ERR_CUDA;
}

void* megakernel_batch_kv_ptr(void* handle) {
  if (!handle) return nullptr;
  const BatchState* s = static_cast<BatchState*>(handle);
  return s->d.kv8 ? static_cast<void*>(s->d.kv8) : static_cast<void*>(s->d.kv);
}

long long megakernel_batch_kv_bytes(void* handle) {
  return handle ? static_cast<BatchState*>(handle)->kv_bytes : 0;
}

int megakernel_batch_last_error(void* handle) {
  return handle ? static_cast<BatchState*>(handle)->last_error : MK_ERR_INVALID_ARG;
}

}  // extern "C"

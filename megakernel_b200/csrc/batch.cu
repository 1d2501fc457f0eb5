// Batched decode (up to 64 concurrent sequences, one token each per step) on
// tcgen05 tensor cores.  Included at the end of megakernel.cu.
//
// This file starts with the pieces every batched kernel shares: the hi/lo
// split of fp32 activations into the 128-row bf16 A operand, and a test entry
// point that runs one tcgen05 GEMM with a plain epilogue.
#include <cstdio>
#include <vector>

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
  struct Params {
    float* out;
    int ldo;
    int rows;
  };
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, const float (&v)[64]) {
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
constexpr int kBChunk = 64;        // positions per attention work item (one warp)
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
  __nv_bfloat16* kv;     // [64][L][2][8][max_seq][64]
  const float* rope_cos; // [max_seq][32]
  const float* rope_sin;
  int* pos;              // [64] position of each sequence's next token
  int* err;
  int batch, max_seq, maxch;
};

__device__ __forceinline__ size_t bkv_index(const BatchDev& d, int b, int l, int kv, int h, int p) {
  return (((((size_t)b * kBL + l) * 2 + kv) * kBNKV + h) * (size_t)d.max_seq + p) * kBD;
}
// 1 / rms of row `seq` of x from the 16 tile partials (fixed order).
__device__ __forceinline__ float inv_rms(const float* ssq, int seq) {
  float s = 0.f;
#pragma unroll
  for (int t = 0; t < kBHT; ++t) s += ssq[t * kBMax + seq];
  return rsqrtf(s / (float)kBH + 1e-6f);
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
  struct Params {
    BatchDev d;
    int l;
    const __nv_bfloat16* qn;
    const __nv_bfloat16* kn;
  };
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, float (&v)[64]) {
    const BatchDev& d = ep.d;
    if (seq >= d.batch) return;
    const float r = inv_rms(d.ssq, seq);
#pragma unroll
    for (int c = 0; c < 64; ++c) v[c] *= r;
    const int p = d.pos[seq];
    if (t < 24) {
      const __nv_bfloat16* gn = t < 16 ? ep.qn : ep.kn;
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < 64; ++c) ss = fmaf(v[c], v[c], ss);
      const float rr = rsqrtf(ss / 64.f + 1e-6f);
#pragma unroll
      for (int c = 0; c < 64; ++c) v[c] = __bfloat162float(gn[c]) * (v[c] * rr);
      const float* cs = d.rope_cos + (size_t)p * 32;
      const float* sn = d.rope_sin + (size_t)p * 32;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float x0 = v[c], x1 = v[c + 32], cc = cs[c], ssn = sn[c];
        v[c] = x0 * cc - x1 * ssn;
        v[c + 32] = x1 * cc + x0 * ssn;
      }
    }
    if (t < 16) {
      float* o = d.q + ((size_t)seq * kBNQ + t) * kBD;
#pragma unroll
      for (int c = 0; c < 64; c += 4) *reinterpret_cast<float4*>(o + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
    } else {
      const int kv = t < 24 ? 0 : 1, h = t < 24 ? t - 16 : t - 24;
      __nv_bfloat16* o = d.kv + bkv_index(d, seq, ep.l, kv, h, p);
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        uint4 w;
        w.x = pack_bf16x2(v[c], v[c + 1]);
        w.y = pack_bf16x2(v[c + 2], v[c + 3]);
        w.z = pack_bf16x2(v[c + 4], v[c + 5]);
        w.w = pack_bf16x2(v[c + 6], v[c + 7]);
        *reinterpret_cast<uint4*>(o + c) = w;
      }
    }
  }
};

// Residual epilogue (O and down projections): x += v, per-tile sum of
// squares of the new x, and hi/lo of (g . x) for the next GEMM.
struct EpiResid {
  struct Params {
    BatchDev d;
    __nv_bfloat16* a_next;
    const __nv_bfloat16* g;
  };
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, float (&v)[64]) {
    const BatchDev& d = ep.d;
    float* xr = d.x + (size_t)seq * kBH + 64 * t;
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 64; c += 4) {
      float4 o = *reinterpret_cast<float4*>(xr + c);
      o.x += v[c]; o.y += v[c + 1]; o.z += v[c + 2]; o.w += v[c + 3];
      *reinterpret_cast<float4*>(xr + c) = o;
      ss = fmaf(o.x, o.x, ss); ss = fmaf(o.y, o.y, ss); ss = fmaf(o.z, o.z, ss); ss = fmaf(o.w, o.w, ss);
      put_hilo(ep.a_next, kBH, seq, 64 * t + c, __bfloat162float(ep.g[64 * t + c]) * o.x);
      put_hilo(ep.a_next, kBH, seq, 64 * t + c + 1, __bfloat162float(ep.g[64 * t + c + 1]) * o.y);
      put_hilo(ep.a_next, kBH, seq, 64 * t + c + 2, __bfloat162float(ep.g[64 * t + c + 2]) * o.z);
      put_hilo(ep.a_next, kBH, seq, 64 * t + c + 3, __bfloat162float(ep.g[64 * t + c + 3]) * o.w);
    }
    d.ssq[t * kBMax + seq] = ss;
  }
};

// Gate/up epilogue: columns 0..31 are gate rows 32t.., 32..63 the matching
// up rows; h = silu(gate / rms) * (up / rms) -> hi/lo into a_h.
struct EpiSwiGLU {
  struct Params {
    BatchDev d;
  };
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, float (&v)[64]) {
    const BatchDev& d = ep.d;
    const float r = inv_rms(d.ssq, seq);
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float gt = v[c] * r, up = v[32 + c] * r;
      const float h = seq < d.batch ? gt / (1.f + expf(-gt)) * up : 0.f;
      put_hilo(d.a_h, kBI, seq, 32 * t + c, h);
    }
  }
};

// LM-head epilogue: logits of 64 vocabulary rows; per sequence the best
// (value, lowest index) of the tile -> lm_part[t][seq]; optional logits.
struct EpiArgmax {
  struct Params {
    BatchDev d;
    float* logits;  // [batch][V] or null
  };
  __device__ __forceinline__ static void apply(const Params& ep, int t, int seq, float (&v)[64]) {
    const BatchDev& d = ep.d;
    if (seq >= d.batch) return;
    const float r = inv_rms(d.ssq, seq);
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

// Split-KV attention, one warp per item (sequence b, KV head h, chunk c of
// 64 positions <= pos_b).  Lane = two positions for the scores, two output
// dimensions for P.V.  Writes {acc[2][64], m[2], l[2]} for the GQA pair of
// query heads (2h, 2h+1) to part[b][h][c].  Replaces warp_attention
// (src/attention.cuh:100-167) for many sequences at once.
__global__ void __launch_bounds__(256) battn_kernel(BatchDev d, int l) {
  const int lane = threadIdx.x & 31;
  const int wglob = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int nitems = d.batch * kBNKV * d.maxch;
  for (int it = wglob; it < nitems; it += nw) {
    const int c = it % d.maxch, h = (it / d.maxch) % kBNKV, b = it / (d.maxch * kBNKV);
    const int p = d.pos[b];
    const int c0 = c * kBChunk;
    if (c0 > p) continue;
    const int n = min(kBChunk, p + 1 - c0);
    const __nv_bfloat16* Kc = d.kv + bkv_index(d, b, l, 0, h, c0);
    const __nv_bfloat16* Vc = d.kv + bkv_index(d, b, l, 1, h, c0);
    const float* q0 = d.q + ((size_t)b * kBNQ + 2 * h) * kBD;
    const float* q1 = q0 + kBD;
    // scores: lane handles positions lane and lane + 32
    float s[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int pp = lane + 32 * j;
      float a0 = 0.f, a1 = 0.f;
      if (pp < n) {
        const uint4* kr = reinterpret_cast<const uint4*>(Kc + (size_t)pp * kBD);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint4 w = __ldg(kr + k);
          const float4 qa = __ldg(reinterpret_cast<const float4*>(q0) + 2 * k);
          const float4 qb = __ldg(reinterpret_cast<const float4*>(q0) + 2 * k + 1);
          const float4 ra = __ldg(reinterpret_cast<const float4*>(q1) + 2 * k);
          const float4 rb = __ldg(reinterpret_cast<const float4*>(q1) + 2 * k + 1);
          const float k0 = bf_lo(w.x), k1 = bf_hi(w.x), k2 = bf_lo(w.y), k3 = bf_hi(w.y);
          const float k4 = bf_lo(w.z), k5 = bf_hi(w.z), k6 = bf_lo(w.w), k7 = bf_hi(w.w);
          a0 = fmaf(k0, qa.x, a0); a0 = fmaf(k1, qa.y, a0); a0 = fmaf(k2, qa.z, a0); a0 = fmaf(k3, qa.w, a0);
          a0 = fmaf(k4, qb.x, a0); a0 = fmaf(k5, qb.y, a0); a0 = fmaf(k6, qb.z, a0); a0 = fmaf(k7, qb.w, a0);
          a1 = fmaf(k0, ra.x, a1); a1 = fmaf(k1, ra.y, a1); a1 = fmaf(k2, ra.z, a1); a1 = fmaf(k3, ra.w, a1);
          a1 = fmaf(k4, rb.x, a1); a1 = fmaf(k5, rb.y, a1); a1 = fmaf(k6, rb.z, a1); a1 = fmaf(k7, rb.w, a1);
        }
        s[j][0] = a0 * 0.125f;
        s[j][1] = a1 * 0.125f;
      } else {
        s[j][0] = -INFINITY;
        s[j][1] = -INFINITY;
      }
    }
    float m[2], lsum[2], pr[2][2];
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      m[g] = warp_max(fmaxf(s[0][g], s[1][g]));
      pr[0][g] = expf(s[0][g] - m[g]);
      pr[1][g] = expf(s[1][g] - m[g]);
      lsum[g] = warp_sum(pr[0][g] + pr[1][g]);
    }
    // P.V: lane owns dims 2*lane, 2*lane+1
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    const uint32_t* vr = reinterpret_cast<const uint32_t*>(Vc) + lane;
#pragma unroll 4
    for (int pp = 0; pp < n; ++pp) {
      const uint32_t w = __ldg(vr + (size_t)pp * (kBD / 2));
      const int src = pp & 31;
      const float p0 = __shfl_sync(0xffffffffu, pp < 32 ? pr[0][0] : pr[1][0], src);
      const float p1 = __shfl_sync(0xffffffffu, pp < 32 ? pr[0][1] : pr[1][1], src);
      const float v0 = bf_lo(w), v1 = bf_hi(w);
      acc[0][0] = fmaf(p0, v0, acc[0][0]);
      acc[0][1] = fmaf(p0, v1, acc[0][1]);
      acc[1][0] = fmaf(p1, v0, acc[1][0]);
      acc[1][1] = fmaf(p1, v1, acc[1][1]);
    }
    float* o = d.part + (((size_t)b * kBNKV + h) * d.maxch + c) * (2 * 66);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      *reinterpret_cast<float2*>(o + g * 66 + 2 * lane) = make_float2(acc[g][0], acc[g][1]);
      if (lane == 0) { o[g * 66 + 64] = m[g]; o[g * 66 + 65] = lsum[g]; }
    }
  }
}

// Merge of the chunk partials of (sequence b, query head qh): one warp, lane
// = two dims.  Writes hi/lo of the attention output into a_att.
__global__ void __launch_bounds__(256) bmerge_kernel(BatchDev d) {
  const int lane = threadIdx.x & 31;
  const int wi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wi >= kBMax * kBNQ) return;
  const int b = wi / kBNQ, qh = wi % kBNQ, h = qh / 2, g = qh % 2;
  float o0 = 0.f, o1 = 0.f;
  if (b < d.batch) {
    const int nc = d.pos[b] / kBChunk + 1;
    const float* base = d.part + ((size_t)b * kBNKV + h) * d.maxch * (2 * 66) + g * 66;
    float M = -INFINITY;
    for (int c = 0; c < nc; ++c) M = fmaxf(M, base[(size_t)c * 132 + 64]);
    float den = 0.f;
    for (int c = 0; c < nc; ++c) {
      const float* pc = base + (size_t)c * 132;
      const float w = expf(pc[64] - M);
      den = fmaf(pc[65], w, den);
      const float2 a = *reinterpret_cast<const float2*>(pc + 2 * lane);
      o0 = fmaf(a.x, w, o0);
      o1 = fmaf(a.y, w, o1);
    }
    const float inv = 1.f / den;
    o0 *= inv;
    o1 *= inv;
  }
  put_hilo(d.a_att, kBQ, b, qh * kBD + 2 * lane, o0);
  put_hilo(d.a_att, kBQ, b, qh * kBD + 2 * lane + 1, o1);
}

// Per-sequence argmax over the LM tiles -> out[b]; advances pos[b].
__global__ void bargmax_kernel(BatchDev d, int* __restrict__ out) {
  const int b = blockIdx.x;
  __shared__ unsigned long long red[32];
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
extern "C" int megakernel_tc_gemm_test(const float* d_x, int rows, const void* d_w, int K, int N, float* d_out,
                                       void* stream) {
  if (!d_x || !d_w || !d_out || rows < 1 || rows > 64 || K < 64 || K % 64 != 0 || N < 64 || N % 64 != 0)
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
      mk::TcGemmParams p{maps, maps + 1, K, N / 64, 0, err, 1000000000LL};
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
};

enum { kMapAx = 0, kMapAatt = 1, kMapAh = 2, kMapLayer0 = 3 };
inline int map_layer(int l, int k) { return kMapLayer0 + 4 * l + k; }   // k: 0 qkv, 1 o, 2 gate/up, 3 down
inline int map_lm() { return kMapLayer0 + 4 * mk::kBL; }

void batch_free(BatchState* s) {
  if (!s) return;
  cudaFree(s->d.x); cudaFree(s->d.ssq); cudaFree(s->d.a_x); cudaFree(s->d.a_att); cudaFree(s->d.a_h);
  cudaFree(s->d.q); cudaFree(s->d.part); cudaFree(s->d.lm_part); cudaFree(s->d.kv);
  cudaFree(const_cast<float*>(s->d.rope_cos)); cudaFree(const_cast<float*>(s->d.rope_sin));
  cudaFree(s->d.pos); cudaFree(s->d.err); cudaFree(s->maps);
  delete s;
}

template <class T>
bool balloc(T** p, size_t bytes) {
  return cudaMalloc(reinterpret_cast<void**>(p), bytes) == cudaSuccess && cudaMemset(*p, 0, bytes) == cudaSuccess;
}

BatchState* batch_init(const void* d_weights, const long long* offsets, int num_offsets, int batch, int max_seq) {
  using namespace mk;
  if (!d_weights || !offsets || batch < 1 || batch > kBMax || max_seq < 1) return nullptr;
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
  s->kv_bytes = (long long)batch * kBL * 2 * kBNKV * (long long)max_seq * kBD * 2;
  float *rc = nullptr, *rs = nullptr;
  const bool ok =
      balloc(&d.x, sizeof(float) * kBMax * kBH) && balloc(&d.ssq, sizeof(float) * kBHT * kBMax) &&
      balloc(&d.a_x, 2 * 128 * kBH) && balloc(&d.a_att, 2 * 128 * kBQ) && balloc(&d.a_h, 2 * 128 * kBI) &&
      balloc(&d.q, sizeof(float) * kBMax * kBNQ * kBD) &&
      balloc(&d.part, sizeof(float) * (size_t)kBMax * kBNKV * d.maxch * 132) &&
      balloc(&d.lm_part, sizeof(unsigned long long) * (size_t)kBLMTiles * kBMax) &&
      balloc(&d.kv, (size_t)s->kv_bytes) && balloc(&rc, sizeof(float) * (size_t)max_seq * 32) &&
      balloc(&rs, sizeof(float) * (size_t)max_seq * 32) && balloc(&d.pos, sizeof(int) * kBMax) &&
      balloc(&d.err, sizeof(int) * 4) && balloc(&s->maps, sizeof(CUtensorMap) * (map_lm() + 1));
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
  if (!mok || cudaMemcpy(s->maps, h.data(), sizeof(CUtensorMap) * h.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    batch_free(s);
    return nullptr;
  }
  return s;
}

// One step for every sequence: input tokens from `forced` (device, [batch])
// or, when null, from `prev_out`; next tokens to `out`; optional logits.
int batch_step(BatchState* s, const int* forced, const int* prev_out, int* out, float* logits, cudaStream_t st) {
  using namespace mk;
  const BatchDev& d = s->d;
  const long long to = 1000000000LL;
  const CUtensorMap* M = s->maps;
  bembed_kernel<<<kBMax, 256, 0, st>>>(d, s->wp[0], s->wp[2], forced, prev_out);
  const int attn_blocks = s->sms * 4;
  for (int l = 0; l < kBL; ++l) {
    const int b = 2 + 11 * l;
    const __nv_bfloat16* g_next = l + 1 < kBL ? s->wp[b + 11] : s->wp[1];
    if (tc_gemm_launch<EpiQKV>(TcGemmParams{M + kMapAx, M + map_layer(l, 0), kBH, (kBQ + 2 * kBKV) / 64, 0, d.err, to},
                               EpiQKV::Params{d, l, s->wp[b + 4], s->wp[b + 5]}, s->sms, st) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    battn_kernel<<<attn_blocks, 256, 0, st>>>(d, l);
    bmerge_kernel<<<(kBMax * kBNQ * 32 + 255) / 256, 256, 0, st>>>(d);
    if (tc_gemm_launch<EpiResid>(TcGemmParams{M + kMapAatt, M + map_layer(l, 1), kBQ, kBH / 64, 0, d.err, to},
                                 EpiResid::Params{d, d.a_x, s->wp[b + 7]}, s->sms, st) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    if (tc_gemm_launch<EpiSwiGLU>(TcGemmParams{M + kMapAx, M + map_layer(l, 2), kBH, kBI / 32, kBI, d.err, to},
                                  EpiSwiGLU::Params{d}, s->sms, st) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
    if (tc_gemm_launch<EpiResid>(TcGemmParams{M + kMapAh, M + map_layer(l, 3), kBI, kBH / 64, 0, d.err, to},
                                 EpiResid::Params{d, d.a_x, g_next}, s->sms, st) != cudaSuccess)
      return ::MK_ERR_LAUNCH;
  }
  if (tc_gemm_launch<EpiArgmax>(TcGemmParams{M + kMapAx, M + map_lm(), kBH, kBLMTiles, 0, d.err, to},
                                EpiArgmax::Params{d, logits}, s->sms, st) != cudaSuccess)
    return ::MK_ERR_LAUNCH;
  bargmax_kernel<<<s->batch, 256, 0, st>>>(d, out);
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

}  // namespace

extern "C" {

void* megakernel_batch_init(const void* d_weights, const long long* offsets, int num_offsets, int batch,
                            int max_seq) {
  return batch_init(d_weights, offsets, num_offsets, batch, max_seq);
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

void* megakernel_batch_kv_ptr(void* handle) { return handle ? static_cast<BatchState*>(handle)->d.kv : nullptr; }

long long megakernel_batch_kv_bytes(void* handle) {
  return handle ? static_cast<BatchState*>(handle)->kv_bytes : 0;
}

int megakernel_batch_last_error(void* handle) {
  return handle ? static_cast<BatchState*>(handle)->last_error : MK_ERR_INVALID_ARG;
}

}  // extern "C"

// Skinny tcgen05 GEMM for batched decode: C[64 x N] = X[64 x K] * W[N x K]^T
// with X in fp32 and W in bf16 (the reference's gemv_* functions,
// src/gemv.cuh:36-279, batched over up to 64 concurrent sequences).
//
// Operand A is 128 x K bf16: rows 0..63 are bf16(x) ("hi") and rows 64..127
// are bf16(x - hi) ("lo") of the 64 sequences, so one M=128 MMA computes the
// product with ~16 mantissa bits of x; the epilogue adds the two halves.
//
// Per CTA (persistent over 64-column output tiles, 256 threads):
//   warp 0      TMA producer: A block (64 K x 128 rows, SW128) and two 32-row
//               W blocks per stage into an 8-stage ring (full/empty mbarriers);
//   warp 1      TMEM owner and MMA issuer: 4 x tcgen05.mma (K=16 each) per
//               stage into one of two 64-column fp32 accumulators, commits to
//               the stage's empty barrier and, per tile, to tmem_full;
//   warps 4..7  epilogue: tcgen05.ld of their 32-lane quarter (one thread
//               per row), release the accumulator, add hi + lo through shared
//               memory, (split K) publish / collect the parts, then
//               Epi::apply(ep, tile, seq, v[64]) on 64 threads (one per row)
//               and, when Epi::kCols, Epi::cols(ep, tile, smem_tile, tid) on
//               all 128 epilogue threads with the 64 x 64 tile in shared
//               memory (lanes = consecutive columns, so global writes are
//               coalesced).
// Split K (ksplit = S, 2..4): the S CTAs of one output tile form a
// thread-block cluster (cluster rank = split index) and reduce-scatter their
// hi + lo partial tiles: rank k owns rows [64k/S, 64(k+1)/S) of the tile;
// every rank pushes the rows it does not own to their owners' receive
// buffers with st.async (distributed shared memory, completing on the
// owner's "recv" mbarrier by byte count, so no release fence is needed),
// sums its own rows over the S partials in rank order (deterministic), frees
// its buffers with a remote arrive on every peer's "free" mbarrier and runs
// the epilogue for its rows.  No partial crosses L2 and no counter is
// needed.
// Every wait is bounded (timeout_ns); on expiry the kernel records
// MK_ERR_TIMEOUT in *err and every role leaves its loop.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "../../include/megakernel.h"
#include "tc_ptx.cuh"

namespace mk {

constexpr int kTcBM = 128, kTcBN = 64, kTcBK = 64, kTcStages = 5;
constexpr int kTcABytes = kTcBM * kTcBK * 2;          // 16 KB
constexpr int kTcWBytes = kTcBN * kTcBK * 2;          //  8 KB
constexpr int kTcStageBytes = kTcABytes + kTcWBytes;  // 24 KB
constexpr int kTcThreads = 256;
// Floats per row of the 64 x 64 tile buffer (hi/lo combine, split-K
// partial, epilogue tile): 68 keeps rows 16-byte aligned, and row-wise float4
// accesses of 8 consecutive rows (one quarter warp) hit 32 distinct banks.
constexpr int kTcCombStride = 68;
// Epilogue side inputs fetched while the MMAs run (kTcPreFloats floats):
// [0, 64) the tile's per-column W scales (e4m3 weights), then the Epi's own
// region of Epi::kPre floats (at most kTcPreFloats - 64).
constexpr int kTcPreFloats = 64 + 64 * 64 + 3 * 64;
// Split K: at most 4 CTAs per tile, so rank 0 receives up to 3 partial tiles.
constexpr int kTcMaxSplit = 4;
constexpr int kTcRecvFloats = (kTcMaxSplit - 1) * 64 * kTcCombStride;
// Per-instance ring: 5 stages of A + W (measured on B200: 4 to 8 stages give
// the same step time); with e4m3 weights (W8) each stage also holds the 4 KB
// e4m3 W block that two converter warps expand into the bf16 W tile.
// NSUB = 4 (bf16 weights, no split K; the LM head): a CTA tile is 4 x 64 =
// 256 output columns, so each stage carries 32 KB of W against the same
// 16 KB of A and the activation operand is re-read a quarter as often; 4
// stages, two 256-column TMEM accumulators, the epilogue runs once per
// 64-column sub-tile.
template <bool W8, int NSUB = 1>
struct TcCfg {
  static_assert(NSUB == 1 || (NSUB == 4 && !W8), "wide tiles: bf16 weights only");
  static constexpr int kStages = NSUB == 1 ? kTcStages : 4;
  static constexpr int kW8Bytes = W8 ? kTcBN * kTcBK : 0;
  static constexpr int kWBytes = NSUB * kTcWBytes;            // bf16 W tile
  static constexpr int kStageBytes = kTcABytes + kWBytes + kW8Bytes;
  static constexpr uint32_t kTxBytes = W8 ? kTcABytes + kW8Bytes : kTcABytes + kWBytes;
  static constexpr uint32_t kTmemCols = 2 * 64 * NSUB;        // two accumulators
  // Prefetch region: wide tiles only take epilogues with small side inputs.
  static constexpr int kPreFloats = NSUB == 1 ? kTcPreFloats : 256;
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + 64 * kTcCombStride * 4 +
                                  (size_t)kPreFloats * 4 + (NSUB == 1 ? (size_t)kTcRecvFloats * 4 : 0);
  static_assert(kSmem + 1024 <= 232448, "shared memory (dynamic + static) per CTA");
};

struct TcGemmParams {
  const CUtensorMap* amap;  // A [128 x K] bf16, box {64, 128}, SW128
  const CUtensorMap* wmap;  // W rows, box {64, 32}, SW128
  int K;                    // multiple of 64
  int ntiles;               // output tiles of 64 columns
  int w_half_off;           // gate/up: row offset of the second matrix; 0: plain rows
  int* err;
  long long timeout_ns;
  int ksplit;               // K blocks split over this many CTAs (one cluster) per tile, 1..4
  const float* wscale;      // e4m3 weights only: per-W-row scale (the GEMM uses W = scale * e4m3)
  int tl = -1;              // profiling builds: this launch's slot in the step timeline
  int stamp = 0;            // profiling builds: record this launch's per-CTA stamps
};

// W rows of tile t: [r0, r0+32) then [r1, r1+32).  Plain: 64t and 64t+32;
// gate/up (w_half_off > 0): gate rows 32t, up rows w_half_off + 32t, so the
// tile's columns are 32 gate outputs followed by the matching 32 up outputs.
__device__ __forceinline__ void tc_tile_rows(const TcGemmParams& p, int t, int& r0, int& r1) {
  if (p.w_half_off > 0) { r0 = 32 * t; r1 = p.w_half_off + 32 * t; }
  else { r0 = 64 * t; r1 = 64 * t + 32; }
}

// Bounded mbarrier wait; false on timeout or when another role gave up.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, const TcGemmParams& p,
                                        volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if ((long long)(globaltimer_ns() - t0) > p.timeout_ns) {
        atomicCAS(p.err, 0, MK_ERR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Same, acquire at cluster scope (the arrivals come from other CTAs).
__device__ __forceinline__ bool tc_wait_cl(uint64_t* bar, uint32_t parity, const TcGemmParams& p,
                                           volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if ((long long)(globaltimer_ns() - t0) > p.timeout_ns) {
        atomicCAS(p.err, 0, MK_ERR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Profiling build only (-DMK_TC_STAMPS=1): %globaltimer stamps per CTA of
// the launch whose params carry `stamp` (batch_step marks the launch slot
// named by MK_TC_STAMP_SLOT), read back with megakernel_tc_stamps.
#ifndef MK_TC_STAMPS
#define MK_TC_STAMPS 0
#endif
#if MK_TC_STAMPS
__device__ unsigned long long g_tc_stamps[256][64];
#define TC_STAMP(k)                                                                  \
  do {                                                                              \
    if (p.stamp && blockIdx.x < 256) g_tc_stamps[blockIdx.x][(k)] = globaltimer_ns(); \
  } while (0)
// Step timeline: per GEMM launch of a step (slot p.tl), the earliest CTA
// entry, the earliest release from griddepcontrol.wait and the latest CTA
// exit (stored complemented so that all three are atomicMin), read back
// with megakernel_tc_timeline.
constexpr int kTcTimeline = 160;
__device__ unsigned long long g_tc_tl[kTcTimeline][3];
#define TC_TL(k, v)                                                      \
  do {                                                                   \
    if (p.tl >= 0 && p.tl < kTcTimeline) atomicMin(&g_tc_tl[p.tl][(k)], (v)); \
  } while (0)
#else
#define TC_STAMP(k) do {} while (0)
#define TC_TL(k, v) do {} while (0)
#endif

// e4m3 pair (low byte first) -> bf16 pair, exactly (through f16).
__device__ __forceinline__ uint32_t tc_e4m3x2_to_bf16x2(uint16_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v));
  const __half2 hh = *reinterpret_cast<const __half2*>(&h);
  const float2 f = __half22float2(hh);
  const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<const uint32_t*>(&b);
}

template <class Epi, bool W8 = false, int NSUB = 1>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ TcGemmParams p, const __grid_constant__ typename Epi::Params ep) {
  using C = TcCfg<W8, NSUB>;
  static_assert(NSUB == 1 || !Epi::kPrePerTile, "wide tiles prefetch once per CTA tile");
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
  float* comb = reinterpret_cast<float*>(smem + (size_t)C::kStages * C::kStageBytes);
  float* pre = comb + 64 * kTcCombStride;
  float* recv = pre + C::kPreFloats;       // split K: partial rows from the peers [S-1][64][kTcCombStride]
  static_assert(Epi::kPre <= C::kPreFloats - 64, "epilogue prefetch region");
  __shared__ alignas(8) uint64_t full[kTcStages], empty[kTcStages], conv[kTcStages], tfull[2], tempty[2];
  __shared__ alignas(8) uint64_t recv_bar, free_bar;   // split K (cluster) only
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); mbar_init(&conv[s], 2); }
    for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], 4); }
    // recv: one local arrival with the expected bytes per tile, the peers'
    // st.async bytes complete it; free: every peer arrives once per tile
    // when it has read its receive buffers.
    mbar_init(&recv_bar, 1);
    mbar_init(&free_bar, p.ksplit > 1 ? p.ksplit - 1 : 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) { tmem_alloc(&tmem_base_sh, C::kTmemCols); tmem_relinquish(); }
  if (warp == 0 && lane == 0) { prefetch_tmap(p.amap); prefetch_tmap(p.wmap); }
  pdl_launch();
  tc_fence_before();
  __syncthreads();
  // Peers arrive on each other's barriers: all are initialised first.
  if (p.ksplit > 1) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int kblocks = p.K / kTcBK;
  const int kper = (kblocks + p.ksplit - 1) / p.ksplit;   // K blocks per split
  const int nct = (p.ntiles + NSUB - 1) / NSUB;           // CTA tiles (NSUB 64-column sub-tiles each)
  const int nunits = nct * p.ksplit;

  if (threadIdx.x == 0) { TC_STAMP(0); TC_TL(0, globaltimer_ns()); }
  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    // Weights do not depend on the previous kernel: the W blocks of the first
    // stages are requested before waiting for it; A (its output) after.
    const int u0 = blockIdx.x;
    int pre = 0;
    if (u0 < nunits) {
      const int t = u0 / p.ksplit, sp = u0 % p.ksplit;
      int r0, r1;
      tc_tile_rows(p, t, r0, r1);
      const int kb0 = sp * kper, kb1 = min(kblocks, (sp + 1) * kper);
      pre = min(C::kStages, kb1 - kb0);
      for (int j = 0; j < pre; ++j) {
        const int kb = kb0 + j;
        uint8_t* st = smem + (size_t)j * C::kStageBytes;
        mbar_arrive_expect_tx(&full[j], C::kTxBytes);
        // bf16 W: the two 32-row halves of the SW128 tile; e4m3 W: the two
        // halves of the staging block after the tile (64 bytes per row).
        if constexpr (NSUB > 1) {
          for (int k = 0; k < 2 * NSUB; ++k) tma_load_2d(st + kTcABytes + 4096 * k, p.wmap, kb * kTcBK, 64 * NSUB * t + 32 * k, &full[j]);
        } else {
          uint8_t* wdst = W8 ? st + kTcABytes + kTcWBytes : st + kTcABytes;
          const int half = W8 ? C::kW8Bytes / 2 : kTcWBytes / 2;
          tma_load_2d(wdst, p.wmap, kb * kTcBK, r0, &full[j]);
          tma_load_2d(wdst + half, p.wmap, kb * kTcBK, r1, &full[j]);
        }
      }
    }
    TC_STAMP(1);
    pdl_wait();
    TC_STAMP(2);
    uint32_t s = 0, ph = 0;
    int issued = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int t = u / p.ksplit, sp = u % p.ksplit;
      int r0, r1;
      tc_tile_rows(p, t, r0, r1);
      for (int kb = sp * kper; kb < min(kblocks, (sp + 1) * kper); ++kb, ++issued) {
        uint8_t* st = smem + (size_t)s * C::kStageBytes;
        if (issued < pre) {
          tma_load_2d(st, p.amap, kb * kTcBK, 0, &full[s]);
        } else {
          if (!tc_wait(&empty[s], ph ^ 1u, p, &abort_flag)) goto done_producer;
          mbar_arrive_expect_tx(&full[s], C::kTxBytes);
          tma_load_2d(st, p.amap, kb * kTcBK, 0, &full[s]);
          if constexpr (NSUB > 1) {
            for (int k = 0; k < 2 * NSUB; ++k) tma_load_2d(st + kTcABytes + 4096 * k, p.wmap, kb * kTcBK, 64 * NSUB * t + 32 * k, &full[s]);
          } else {
            uint8_t* wdst = W8 ? st + kTcABytes + kTcWBytes : st + kTcABytes;
            const int half = W8 ? C::kW8Bytes / 2 : kTcWBytes / 2;
            tma_load_2d(wdst, p.wmap, kb * kTcBK, r0, &full[s]);
            tma_load_2d(wdst + half, p.wmap, kb * kTcBK, r1, &full[s]);
          }
        }
        if (++s == C::kStages) { s = 0; ph ^= 1u; }
      }
    }
  done_producer:;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = tc_idesc_bf16(kTcBM, kTcBN * NSUB);
    uint32_t s = 0, ph = 0;
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int sp = u % p.ksplit;
      const int kb0 = sp * kper, kb1 = min(kblocks, (sp + 1) * kper);
      const int buf = i & 1;
      if (!tc_wait(&tempty[buf], (((uint32_t)i >> 1) & 1u) ^ 1u, p, &abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * kTcBN * NSUB);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc_wait(W8 ? &conv[s] : &full[s], ph, p, &abort_flag)) { ok = false; break; }
        if (kb - kb0 < 24) TC_STAMP(4 + kb - kb0);
        tc_fence_after();
        const uint32_t a = smem_u32(smem + (size_t)s * C::kStageBytes);
        const uint32_t w = a + kTcABytes;
#pragma unroll
        for (int kk = 0; kk < kTcBK / 16; ++kk)
          tc_mma_bf16(d, tc_desc_sw128(a + kk * 32), tc_desc_sw128(w + kk * 32), idesc, (kb > kb0) || kk != 0);
        tc_commit(&empty[s]);
        if (++s == C::kStages) { s = 0; ph ^= 1u; }
      }
      if (!ok) break;
      tc_commit(&tfull[buf]);
      TC_STAMP(30);
    }
  } else if (W8 && (warp == 2 || warp == 3)) {
    // ---- e4m3 -> bf16 converter (W8 only) ----
    // Each lane expands one W row of the stage's e4m3 block (64 bytes) into
    // the 128-byte-swizzled bf16 tile the MMA reads, then the warp makes its
    // writes visible to the tensor core (async proxy) and arrives on conv.
    const int row = 32 * (warp - 2) + lane;
    uint32_t s = 0, ph = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
      const int sp = u % p.ksplit;
      const int kb0 = sp * kper, kb1 = min(kblocks, (sp + 1) * kper);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc_wait(&full[s], ph, p, &abort_flag)) { ok = false; break; }
        uint8_t* st = smem + (size_t)s * C::kStageBytes;
        const uint8_t* src = st + kTcABytes + kTcWBytes + row * 64;
        uint8_t* dst = st + kTcABytes + row * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint2 w = *reinterpret_cast<const uint2*>(src + 8 * j);
          uint4 o;
          o.x = tc_e4m3x2_to_bf16x2((uint16_t)w.x);
          o.y = tc_e4m3x2_to_bf16x2((uint16_t)(w.x >> 16));
          o.z = tc_e4m3x2_to_bf16x2((uint16_t)w.y);
          o.w = tc_e4m3x2_to_bf16x2((uint16_t)(w.y >> 16));
          *reinterpret_cast<uint4*>(dst + ((j ^ (row & 7)) << 4)) = o;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
        if (++s == C::kStages) { s = 0; ph ^= 1u; }
      }
      if (!ok) break;
    }
  } else if (warp >= 4) {
    // ---- epilogue ----
    const int q = warp - 4;          // TMEM lane quarter = rows 32q .. 32q+31
    const int row = 32 * q + lane;
    float* tile = comb;              // [64][kTcCombStride]: lo half, then the final tile
    pdl_wait();                      // epilogues read the previous kernel's outputs
    if (threadIdx.x == 128) { TC_STAMP(3); TC_TL(1, globaltimer_ns()); }
    int i = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++i) {
      const int S = p.ksplit, t = u / S, sp = u % S;
      const int buf = i & 1;
      const int ra = 64 * sp / S, rb = 64 * (sp + 1) / S;   // rows this CTA finishes
      // Split K: every peer must have read this CTA's previous rows before
      // they are rewritten in its receive buffers.
      if (S > 1 && i > 0 && bar_any(2, 128, !tc_wait_cl(&free_bar, (uint32_t)(i - 1) & 1u, p, &abort_flag)))
        break;
      // Side inputs of this tile's epilogue, fetched while the MMAs run
      // (the previous tile's epilogue is done with the region: loop-end
      // barrier).  Visible to all epilogue threads after the barrier below.
      {
        const int e = threadIdx.x - 128;
        if (S > 1 && e == 0) mbar_arrive_expect_tx(&recv_bar, (uint32_t)((S - 1) * (rb - ra) * 64 * 4));
        if constexpr (W8) {
          if (e < 64) {
            int r0, r1;
            tc_tile_rows(p, t, r0, r1);
            pre[e] = __ldg(p.wscale + (e < 32 ? r0 + e : r1 + e - 32));
          }
        }
        Epi::prefetch(ep, t, pre + 64, e);
      }
      // All four epilogue warps leave together (they share named barriers).
      if (bar_any(2, 128, !tc_wait(&tfull[buf], ((uint32_t)i >> 1) & 1u, p, &abort_flag))) break;
      if (threadIdx.x == 128) TC_STAMP(31);
      tc_fence_after();
      bool quit = false;
      // NSUB 64-column sub-tiles of the accumulator (sub-tile tt = t NSUB + h).
      for (int h = 0; h < NSUB; ++h) {
        const int tt = t * NSUB + h;
        float v[64];
        {
          uint32_t r[32];
          const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * kTcBN * NSUB + 64 * h);
          tmem_ld_32x32b_x32(ta, r);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]);
          tmem_ld_32x32b_x32(ta + 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[32 + c] = __uint_as_float(r[c]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && h == NSUB - 1) mbar_arrive(&tempty[buf]);
        if (q >= 2) {
          float4* tr = reinterpret_cast<float4*>(tile + (row - 64) * kTcCombStride);
#pragma unroll
          for (int c = 0; c < 16; ++c) tr[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (threadIdx.x == 128) TC_STAMP(32);
        if (q < 2) {
          float4* tr = reinterpret_cast<float4*>(tile + row * kTcCombStride);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float4 lo = tr[c];
            v[4 * c] += lo.x; v[4 * c + 1] += lo.y; v[4 * c + 2] += lo.z; v[4 * c + 3] += lo.w;
          }
          if (S > 1 && (row < ra || row >= rb)) {
            // Split K: a row another rank owns goes to slot (this rank's index
            // among the owner's peers) of the owner's receive buffers.
            int dest = 0;
            while (dest + 1 < S && row >= 64 * (dest + 1) / S) ++dest;
            const int slot = sp < dest ? sp : sp - 1;
            const uint32_t dst = mapa_shared(smem_u32(recv + (slot * 64 + row) * kTcCombStride), (uint32_t)dest);
            const uint32_t bar = mapa_shared(smem_u32(&recv_bar), (uint32_t)dest);
#pragma unroll
            for (int c = 0; c < 16; ++c)
              st_async_f32x4(dst + 16 * c, make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]), bar);
          }
        }
        if (S > 1) {
          // Own rows: the S partials summed in rank order (this rank's own
          // partial at position sp), then every peer is told that its rows
          // have been read.
          if (bar_any(2, 128, !tc_wait(&recv_bar, (uint32_t)i & 1u, p, &abort_flag))) { quit = true; break; }
          if (threadIdx.x == 128) TC_STAMP(33);
          if (q < 2 && row >= ra && row < rb) {
            float4 acc[16];
            const float4* r0p = reinterpret_cast<const float4*>(recv + row * kTcCombStride);
#pragma unroll
            for (int c = 0; c < 16; ++c)
              acc[c] = sp == 0 ? make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]) : r0p[c];
            for (int j = 1; j < S; ++j) {
              const float4* rj = reinterpret_cast<const float4*>(recv + ((j < sp ? j : j - 1) * 64 + row) * kTcCombStride);
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const float4 x = j == sp ? make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]) : rj[c];
                acc[c].x += x.x; acc[c].y += x.y; acc[c].z += x.z; acc[c].w += x.w;
              }
            }
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              v[4 * c] = acc[c].x; v[4 * c + 1] = acc[c].y; v[4 * c + 2] = acc[c].z; v[4 * c + 3] = acc[c].w;
            }
          }
          asm volatile("bar.sync 2, 128;" ::: "memory");
          // Arrivals come from the lo-half warps, which issued no st.async: a
          // release by a thread with stores in flight to another CTA waits for
          // them (measured ~1-2 us).
          const int e = threadIdx.x - 192;
          if (e >= 0 && e < S - 1) mbar_arrive_remote(mapa_shared(smem_u32(&free_bar), (uint32_t)(e < sp ? e : e + 1)));
          if (threadIdx.x == 128) TC_STAMP(36);
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (threadIdx.x == 128) TC_STAMP(34);
        if (q < 2 && row >= ra && row < rb && tt < p.ntiles) {
          if constexpr (W8) {
            // W = scale * e4m3: column c of the tile is W row r0 + c (c < 32)
            // or r1 + c - 32 (scales prefetched to pre[c]).
#pragma unroll
            for (int c = 0; c < 64; ++c) v[c] *= pre[c];
          }
          Epi::apply(ep, tt, row, v, pre + 64);
          if (threadIdx.x == 128) TC_STAMP(37);
          // Column phase: the row values go through shared memory so that
          // global writes are coalesced (lanes = consecutive columns).
          if constexpr (Epi::kCols) {
            float4* tr = reinterpret_cast<float4*>(tile + row * kTcCombStride);
#pragma unroll
            for (int c = 0; c < 16; ++c) tr[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
          }
        }
        if constexpr (Epi::kCols) {
          asm volatile("bar.sync 2, 128;" ::: "memory");
          Epi::cols(ep, tt, tile, threadIdx.x - 128, pre + 64, ra, rb);
          if (threadIdx.x == 128) TC_STAMP(38);
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
      }
      if (quit) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  // No CTA leaves while a peer may still read its shared memory or arrive on
  // its barriers.
  if (p.ksplit > 1) cluster_sync_all();
  if (threadIdx.x == 0) { TC_STAMP(35); TC_TL(2, ~globaltimer_ns()); }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ---- host side ---------------------------------------------------------------

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline PFN_encodeTiled tc_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// Row-major bf16 matrix [rows x cols] -> tensor map with a {64, box_rows}
// box and the 128-byte swizzle.  Returns false on failure.
inline bool tc_make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  PFN_encodeTiled enc = tc_encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols * 2) % 16 != 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major e4m3 matrix [rows x cols] (bytes) -> tensor map with a {64, box_rows}
// box, no swizzle (the converter warps swizzle while expanding to bf16).
inline bool tc_make_map_e4m3(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  PFN_encodeTiled enc = tc_encode_fn();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 16 != 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <class Epi, bool W8 = false, int NSUB = 1>
inline cudaError_t tc_gemm_launch(const TcGemmParams& p, const typename Epi::Params& ep, int max_ctas,
                                  cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<Epi, W8, NSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)TcCfg<W8, NSUB>::kSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  if (p.ksplit < 1 || p.ksplit > kTcMaxSplit || (NSUB > 1 && p.ksplit != 1)) return cudaErrorInvalidValue;
  const int units = (p.ntiles + NSUB - 1) / NSUB * p.ksplit;
  const int cap = max_ctas / p.ksplit * p.ksplit;   // whole clusters
  const int grid = units < cap ? units : cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = TcCfg<W8, NSUB>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = (unsigned)p.ksplit;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = p.ksplit > 1 ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<Epi, W8, NSUB>, p, ep);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace mk

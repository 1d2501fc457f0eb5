// Compile-time model shapes and the per-CTA work schedule.
//
// The reference fixes one shape in namespace config (src/config.cuh:13-29).
// Here the kernel is a template over a shape struct so that the graded
// head_dim-64 shape, the head_dim-128 shape of src/config.cuh and a tiny test
// shape share one code path.  Shape ids must match megakernel_b200/shapes.py.
#pragma once
#include <cstdint>

namespace mk {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
// Two consumer warpgroups plus a producer warpgroup of which only the first
// warp works.  Nine warps would cap every thread at 168 registers (three
// warps share a sub-partition's register file); with setmaxnreg the producer
// warpgroup drops to kProducerRegs and the consumers rise to kConsumerRegs.
// The split must not exceed what the launch allocates: 384 threads x 168.
constexpr int kThreads = kConsumerThreads + 128;
constexpr int kConsumerRegs = 232;
constexpr int kProducerRegs = 40;
static_assert(2 * 128 * kConsumerRegs + 128 * kProducerRegs <= kThreads * 168, "register split");
constexpr int kRingBytes = 176 * 1024;
constexpr int kMaxCtas = 256;
constexpr int kRowsMax = 256;           // weight rows one CTA owns in one phase
constexpr int kRowPad = 16;             // bytes between weight rows in a ring stage
// 64-bit words between consecutive elements of the all-read activation hops.
// A microbenchmark of a bare 148-CTA all-gather ran faster with elements one
// per 32-byte sector (4), but in this kernel 4 measured 530 against 510
// us/token for 1 (B200, 512-token launch at positions 128-639).
#ifndef MK_HOP_SPREAD
#define MK_HOP_SPREAD 1
#endif
constexpr int kHopSpread = MK_HOP_SPREAD;
constexpr int kMaxTP = 8;               // tensor-parallel GPUs at most
constexpr int kPvParts = 4;             // position parts of the attention P.V (warps / GRP)
constexpr int kMaxChunksPerHead = 16;   // attention split-KV chunks per KV head
// Cached positions per split-KV chunk (at most): smaller chunks spread the
// walk over more CTAs but cost more in the merge of their partials.
#ifndef MK_CHUNK_MIN_POS
#define MK_CHUNK_MIN_POS 128
#endif
constexpr int kChunkMinPos = MK_CHUNK_MIN_POS;
// From this many chunks per head on, the partials are merged in two levels
// (one CTA per KV head, then every CTA reads the merged heads).  Measured on
// B200 (64-token launches): the extra exchange costs more than it saves up to
// 4 chunks; at 5 chunks it wins, at 16 (p >= 1920) it saves ~150 us/token.
#ifndef MK_MERGE2_MIN_CHUNKS
#define MK_MERGE2_MIN_CHUNKS 5
#endif
constexpr int kMerge2MinChunks = MK_MERGE2_MIN_CHUNKS;

template <int H_, int L_, int NQ_, int NKV_, int D_, int I_, int V_, int STB_>
struct ShapeT {
  static constexpr int H = H_, L = L_, NQ = NQ_, NKV = NKV_, D = D_, I = I_, V = V_;
  static constexpr int Q = NQ * D, KV = NKV * D, QKV = Q + 2 * KV, GRP = NQ / NKV;
  static constexpr int STB = STB_;                          // ring stage bytes
  static constexpr int NST = kRingBytes / STB;              // ring stages
  static constexpr int SUBP = STB / (D * 2);                // KV positions per stage
  static constexpr int XIN = (H > Q ? (H > I ? H : I) : (Q > I ? Q : I));
  static constexpr int NOFF = 2 + 11 * L;
  // Weight rows sit in a stage at a pitch of 2K + 16 bytes, so the 8 rows an
  // ldmatrix reads fall in different shared-memory banks.
  template <int K> __host__ __device__ static constexpr int pitch() { return 2 * K + kRowPad; }
  template <int K> __host__ __device__ static constexpr int rows_per_stage() { return STB / pitch<K>(); }
  static_assert(H % 256 == 0 && Q % 256 == 0 && I % 256 == 0, "K dims must be multiples of 256");
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(STB % 16 == 0 && NST >= 4, "ring");
  static_assert(kPvParts * GRP == kConsumerWarps && GRP * D <= kConsumerThreads, "PV warp mapping");
};

// Shape 0: BASELINE configs[0] (head_dim 64, intermediate 2816).
using ShapeD64 = ShapeT<1024, 28, 16, 8, 64, 2816, 151936, 16944>;
// Shape 1: the shape src/config.cuh:13-22 compiles (head_dim 128, intermediate 3072).
using ShapeD128 = ShapeT<1024, 28, 16, 8, 128, 3072, 151936, 18480>;
// Shape 2: tiny test shape (small stages so the ring wraps many times).
using ShapeTiny = ShapeT<256, 2, 4, 2, 64, 512, 2048, 4160>;

// All schedule arithmetic is 32-bit: products stay below 2^31 for every
// supported shape and CTA count (148 * 151936 < 2^25), and 64-bit division is
// a long software sequence on the GPU.

// Even split of R rows over N CTAs, rotated so the CTAs that receive one
// extra row differ from phase to phase (keeps per-token bytes balanced).
__host__ __device__ inline void split_rows(int R, int N, int cta, int rot, int& start, int& end) {
  const unsigned c = (unsigned)((cta + rot) % N);
  start = (int)(c * (unsigned)R / (unsigned)N);
  end = (int)((c + 1u) * (unsigned)R / (unsigned)N);
}
// Rotation per (layer, phase); phase 0 qkv, 1 o, 2 gate/up, 3 down, 4 lm head.
__host__ __device__ inline int phase_rot(int layer, int phase, int N) {
  return (int)((unsigned)((layer * 5 + phase) * 37) % (unsigned)N);
}

// Attention split-KV plan for a step at position p (p cached positions): one
// chunk per kChunkMinPos positions (rounded up), at most kMaxChunksPerHead,
// so up to NKV * 16 = 128 CTAs walk the cache at once.
template <class S>
__host__ __device__ inline int chunks_per_head(int p) {
  int nc = (p + kChunkMinPos - 1) / kChunkMinPos;
  if (nc < 1) nc = 1;
  if (nc > kMaxChunksPerHead) nc = kMaxChunksPerHead;
  return nc;
}
// Item i (0 <= i < nitems = NKV * nc) of layer l runs on CTA
// (floor(i * N / nitems) + 53 l) mod N: items are spread evenly and the set
// rotates from layer to layer so the extra K/V bytes land on different CTAs.
// items_of_cta returns the (contiguous) items [lo, hi) that CTA `cta` owns.
__host__ __device__ inline void items_of_cta(int cta, int layer, int nitems, int N, int& lo, int& hi) {
  const unsigned shift = (unsigned)(layer * 53) % (unsigned)N;
  const unsigned c = ((unsigned)cta + (unsigned)N - shift) % (unsigned)N;
  lo = (int)((c * (unsigned)nitems + (unsigned)N - 1u) / (unsigned)N);
  hi = (int)(((c + 1u) * (unsigned)nitems + (unsigned)N - 1u) / (unsigned)N);
}
// Positions [c0, c1) of the cached prefix handled by chunk j of nc.
__host__ __device__ inline void chunk_range(int p, int nc, int j, int& c0, int& c1) {
  c0 = (int)((unsigned)j * (unsigned)p / (unsigned)nc);
  c1 = (int)((unsigned)(j + 1) * (unsigned)p / (unsigned)nc);
}

}  // namespace mk

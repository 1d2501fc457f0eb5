// The persistent decode megakernel (B200 / sm_100a).
//
// Replaces persistent_megakernel (src/megakernel.cu:86-339) and the device op
// library it inlines (src/gemv.cuh, rmsnorm.cuh, attention.cuh, kv_cache.cuh,
// sampling.cuh, barriers.cuh).  One cooperative launch of one CTA per SM runs
// `n_steps` whole decode steps (embedding -> L layers -> final norm -> LM-head
// argmax -> next input token) without returning to the host.
//
// Structure of a CTA:
//   * warp 8 (producer): walks this CTA's byte stream for every step --
//     its rows of each weight matrix and its share of the cached K/V -- and
//     issues 1-D TMA bulk copies into a ring of shared-memory stages, each
//     completing on a "full" mbarrier.  Weights do not depend on activations,
//     so the producer runs ahead of the math by up to the ring size, through
//     every inter-CTA dependency, keeping HBM busy.
//   * warps 0-7 (consumers): per phase, wait for the activation vector the
//     phase needs, then do the math on ring stages and release them on an
//     "empty" mbarrier.
//
// Inter-CTA dependencies: every activation element crosses between CTAs as a
// 64-bit word {tag, fp32 bits} written with one st.relaxed.gpu.  The tag names
// the (step, layer, phase), so a reader spins on the words it needs until the
// tags match: no counters, no grid barriers, no fences on the critical path.
// The reference instead runs 144 atomic grid barriers per token
// (src/barriers.cuh:38-73).  Every wait is bounded through a per-CTA watchdog
// thread (no progress for timeout_ns, or another CTA's error, raises the
// CTA's abort flag); the CTA then records an error code and all roles exit.
#pragma once
#include "ptx.cuh"
#include "shapes.cuh"

// Everything is inlined into the kernel body: the consumer and producer
// warpgroups run with different register budgets (setmaxnreg), and ptxas
// drops setmaxnreg when the kernel makes out-of-line calls.
#define MK_PHASE __forceinline__

// Sub-phase stamps of layer 1 (megakernel_set_trace_detail): a profiling
// build only (-DMK_DETAIL_STAMPS=1), since they add 6 KB to the kernel body.
#ifndef MK_DETAIL_STAMPS
#define MK_DETAIL_STAMPS 0
#endif
// Coarse per-phase trace stamps (megakernel_set_trace): also a profiling
// build only (-DMK_TRACE_POINTS=1, 4 KB of kernel code).
#ifndef MK_TRACE_POINTS
#define MK_TRACE_POINTS 0
#endif

// Unroll factor of the GEMV's streamed-slice loop: more ldmatrix loads in
// flight per warp (measured on B200: 1 -> +8 % per token, 2 -> 4 -> 8 each
// about -1.5 %; the code grows by under 1 KB).
#ifndef MK_GEMV_UNROLL
#define MK_GEMV_UNROLL 8
#endif
// Unroll of the attention P.V position loop (code size vs load overlap).
#ifndef MK_PV_UNROLL
#define MK_PV_UNROLL 4
#endif
// Weight slices per tile loaded into registers before the GEMV input arrives.
#ifndef MK_GEMV_PIT
#define MK_GEMV_PIT 2
#endif
// Pause between polling rounds of a tagged-word wait (ns).
#ifndef MK_POLL_BACKOFF_NS
#define MK_POLL_BACKOFF_NS 50
#endif

namespace mk {

constexpr int kGemvUnroll = MK_GEMV_UNROLL;
constexpr int kPvUnroll = MK_PV_UNROLL;

enum : int {
  MK_OK = 0,
  MK_ERR_INVALID_ARG = -1,
  MK_ERR_CUDA = -2,
  MK_ERR_TIMEOUT = -3,
  MK_ERR_CAPACITY = -4,
  MK_ERR_SHAPE = -5,
  MK_ERR_LAUNCH = -6,
  MK_ERR_OOM = -7,
};

struct KParams {
  const __nv_bfloat16* const* w;  // 2 + 11 L weight pointers (offsets order)
  __nv_bfloat16* kv;              // [L, 2, NKV, max_seq, D]
  const float* rope_cos;          // [max_seq, D/2]
  const float* rope_sin;          // [max_seq, D/2]
  uint64_t* hop;                  // tagged activation words (see HopLayout)
  int* err;                       // first error code (0 = ok)
  const int* forced;              // tokens fed at steps 0..n_forced-1
  int n_forced;                   // >= 1
  int n_steps;
  int* out_tokens;                // [n_steps] argmax of each step
  float* logits;                  // optional [n_steps, V] fp32 logits
  int pos0;                       // position of step 0
  uint32_t seq0;                  // tag sequence number of step 0
  int max_seq;
  int ncta;
  int nst;                        // ring stages in use (<= S::NST)
  int issue_gap_ns;               // producer pacing: min ns between stage issues (0 = off)
  long long timeout_ns;
  int debug_skip_cta;             // >= 0: that CTA never publishes layer-0 x (fault test)
  uint64_t* trace;                // optional stamps [trace_steps][ncta][Trace::kPoints]
  int trace_steps;
  uint64_t* detail;               // optional [trace_steps][ncta][64] sub-phase stamps of layer 1
  // Tensor-parallel launches (template TP > 1) only: this GPU's rank and the
  // hop buffer of every rank (peer_hop[tp_rank] is this GPU's own), mapped
  // into this process by CUDA IPC.
  int tp_rank;
  uint64_t* peer_hop[kMaxTP];
};

// Offsets (in 64-bit words) of the tagged activation buffers.  With tensor
// parallelism over TP GPUs, X holds one slot per rank (each rank's partial
// down projection, written by that rank over NVLink) and LM one (max, index)
// pair per (rank, CTA); the other hops stay on the GPU.
template <class S, int TP = 1>
struct HopLayout {
  static constexpr int kAttWords = S::NKV * kMaxChunksPerHead * S::GRP * (S::D + 2);
  // The GPU-local hops come first, so their offsets do not depend on TP.
  static constexpr long long QKV = 0;                      // [2][QKV]
  static constexpr long long ATT = QKV + 2 * S::QKV;       // [2][items][GRP][D+2]
  // The GEMV-input hops that every CTA reads (XA, HM, X) keep one element
  // per kHopSpread words (shapes.cuh).
  static constexpr long long XA = ATT + 2LL * kAttWords;   // [2][H]  after attention (spread)
  static constexpr long long HM = XA + 2LL * S::H * kHopSpread;     // [2][I]  silu(g)*u (spread)
  static constexpr long long X = HM + 2LL * S::I * kHopSpread;      // [2][TP][H]  layer input (spread)
  static constexpr long long LM = X + 2LL * TP * S::H * kHopSpread; // [2][TP * kMaxCtas][2]
  static constexpr long long MH = LM + 2LL * TP * kMaxCtas * 2;  // [2][Q]  merged heads (two-level merge)
  static constexpr long long TOTAL = MH + 2LL * S::Q;
};

// Tag of phase `k` (0 qkv, 1 att, 2 xa, 3 hm, 4 x-out) of layer `l` at step seq.
__device__ __forceinline__ uint32_t tag_of(uint32_t seq, int l, int k) {
  return (seq << 8) | (uint32_t)(l * 5 + k);
}

// Trace points per (step, CTA): per layer 7 (producer reaches the layer, x
// ready, qkv published, attention merged, x' published, h published, x''
// published), then lm start, lm partial published, next token known, the
// step's total ns consumer thread 0 spent in activation-hop waits, and the
// SM clock cycles (clock64) elapsed over the step.
template <class S>
struct Trace {
  static constexpr int kPoints = 7 * S::L + 5;
};

template <class S>
struct Smem;
template <class S>
__device__ __forceinline__ void trace_point(const KParams& P, Smem<S>& sm, int t, int cta, int k) {
  sm.progress = sm.progress + 1u;   // watchdog: this CTA is advancing
  if (MK_TRACE_POINTS && P.trace != nullptr && t < P.trace_steps)
    P.trace[((size_t)t * P.ncta + cta) * Trace<S>::kPoints + k] = globaltimer_ns();
}

// Sub-phase stamp k of layer 1 (profiling aid; off unless P.detail is set).

#if MK_DETAIL_STAMPS
#define MK_DP(k)                                                                      \
  do {                                                                                \
    if (P.detail != nullptr && l == 1 && t < P.trace_steps &&                         \
        (threadIdx.x == 0 || threadIdx.x == kConsumerThreads))                        \
      P.detail[((size_t)t * P.ncta + blockIdx.x) * 64 + (k)] = globaltimer_ns();      \
  } while (0)
#else
#define MK_DP(k) do {} while (0)
#endif

template <class S>
struct Smem {
  float xres[S::H];                   // residual stream x (fp32)
  float xin[S::XIN];                  // GEMV input vector (normed x, attn, h)
  // GEMV input split exactly into three bf16 terms, x = hi + mid + lo (each
  // term keeps 8 mantissa bits, together the 24 of fp32); padded rows keep
  // the three arrays in different banks.
  alignas(16) __nv_bfloat16 xs[3][S::XIN + 8];
  float partw[kConsumerWarps][64];    // per-warp row partials of one GEMV pass (<= 4 tiles)
  float rowsum[2][kRowsMax];          // GEMV results of this CTA's rows
  alignas(16) float qs[S::GRP][S::D];     // normed + roped queries (read as float4)
  float sc[S::GRP][S::SUBP + 2];      // scores / probabilities of one block
  float pv[kPvParts * S::GRP * S::D];  // PV partials [part][GRP][D]
  float mrun[S::GRP], lrun[S::GRP], corr[S::GRP];
  float gq[S::D], gk[S::D];           // q_norm / k_norm gains of the layer
  float rc[S::D / 2], rs[S::D / 2];   // RoPE cos / sin row of position p
  // K/V rows not in the ring (prev + current); read with 16-byte loads.
  alignas(16) __nv_bfloat16 kx[2][S::D];
  alignas(16) __nv_bfloat16 vx[2][S::D];
  float red[kConsumerWarps * 2];
  float mlbuf[S::NQ * kMaxChunksPerHead * 2];  // attention partials' (m, l), one copy per CTA
  int redi[kConsumerWarps];
  int next_token;
  volatile int abort_flag;
  volatile int tokens_done;
  volatile uint32_t progress;         // bumped at every phase (watchdog)
  volatile int done;                  // consumers finished (watchdog exits)
  unsigned long long wait_hop_ns;     // trace accounting (thread 0)
  const __nv_bfloat16* wtab[S::NOFF]; // weight pointer table (offsets order)
  // The copy engine's schedule, computed once per launch (every division by
  // the CTA count happens here, none in the producer's loops): rows [r0, r1)
  // of GEMV phase ph (0 q/k/v, 1 O, 2 gate/up, 3 down) at layer l packed as
  // r0 | r1 << 16 in rows[4 l + ph], the rotated CTA index that places
  // attention items per layer, the LM-head rows, and division magics
  // (magic_of) for the CTA count and for 1..16 chunks per head.
  uint32_t rows[4 * S::L];
  uint16_t itc[S::L];
  int lm0, lm1;
  uint32_t magic_n;
  uint32_t magic_c[kMaxChunksPerHead + 1];
  KParams prm;                        // copy of the launch parameters
  alignas(8) unsigned char prod[64];  // the producer's state (see Producer)
  alignas(8) uint64_t full[S::NST];
  alignas(8) uint64_t empty[S::NST];
};

// ---- failure handling -------------------------------------------------------
template <class S>
__device__ __forceinline__ void fail(const KParams& P, Smem<S>& sm, int code) {
  atomicCAS(P.err, 0, code);
  sm.abort_flag = 1;
}

// Spin helper of every wait: returns false when the wait must be abandoned
// (this CTA aborted).  Waits are bounded by the CTA's watchdog warp
// (decode_kernel), which raises abort_flag when the CTA has made no progress
// for timeout_ns or another CTA has reported an error; each wait site only
// reads the flag, which keeps the (inlined, instruction-cache-bound) wait
// code small.
struct Spin {
  template <class S>
  __device__ __forceinline__ bool keep_going(const KParams& P, Smem<S>& sm) {
    (void)P;
    return !sm.abort_flag;
  }
};

// Slow paths of the waits live out of line: the fast path (already complete)
// stays a couple of instructions at every call site, which keeps the kernel's
// hot loop small enough for the instruction caches.
template <class S>
__device__ __forceinline__ bool wait_bar_slow(const KParams& P, Smem<S>& sm, uint64_t* bar, uint32_t parity) {
  Spin sp;
  while (!mbar_try_wait(bar, parity)) {
    if (!sp.keep_going(P, sm)) return false;
  }
  return true;
}
template <class S>
__device__ __forceinline__ bool wait_bar(const KParams& P, Smem<S>& sm, uint64_t* bar, uint32_t parity) {
  if (mbar_test(bar, parity)) return true;
  return wait_bar_slow(P, sm, bar, parity);
}
// Re-poll one tagged word until it carries `tag` (bounded); returns the word.
template <class S>
__device__ __forceinline__ uint64_t poll_tagged_slow(const KParams& P, Smem<S>& sm, const uint64_t* src,
                                                  uint32_t tag) {
  uint64_t v;
  Spin sp;
  do {
    v = ld_relaxed(src);
    if ((uint32_t)(v >> 32) == tag) break;
    __nanosleep(MK_POLL_BACKOFF_NS);
  } while (sp.keep_going(P, sm));
  return v;
}

// ---- per-step plan shared by producer and consumers -------------------------
// This CTA owns rows [s, e) of the concatenated [Wq; Wk; Wv] matrix; the part
// that falls in tensor m (0 q, 1 k, 2 v) is rows [a, b) of that tensor and
// starts at output row o.  (Written without arrays so nothing lands in local
// memory.)
template <class S>
__device__ __forceinline__ bool qkv_part(int s, int e, int m, int& a, int& b, int& o) {
  const int base = m == 0 ? 0 : (m == 1 ? S::Q : S::Q + S::KV);
  const int len = m == 0 ? S::Q : S::KV;
  o = max(s, base);
  const int hi = min(e, base + len);
  a = o - base;
  b = hi - base;
  return o < hi;
}

// Weight pointer for layer l, key k (0 attn_norm .. 10 w_down), offsets order
// of src/megakernel.cu:518-532.  Read from the shared-memory copy of the
// table: almost no L1 is left beside the ring, so a global read would cost an
// L2 round trip on the critical path.
#define wptr(l, k) (sm.wtab[2 + 11 * (l) + (k)])
enum { W_ATTN_NORM = 0, W_Q, W_K, W_V, W_QNORM, W_KNORM, W_O, W_FFN_NORM, W_GATE, W_UP, W_DOWN };

template <class S>
__device__ __forceinline__ size_t kv_index(int l, int kind, int h, int pos, int max_seq) {
  return ((((size_t)l * 2 + kind) * S::NKV + h) * (size_t)max_seq + pos) * S::D;
}

}  // namespace mk

namespace mk {

// ---- schedule helpers ---------------------------------------------------------
// floor(x / d) for the small numerators of the schedule, from
// m = ceil(2^31 / d): floor(2x m / 2^32), exact while x d < 2^31 (x < 2^31).
__host__ __device__ __forceinline__ uint32_t magic_of(uint32_t d) {
  return (uint32_t)((0x80000000ull + d - 1) / d);
}
__device__ __forceinline__ uint32_t divm(uint32_t x, uint32_t m) { return __umulhi(x << 1, m); }

// ---- producer ---------------------------------------------------------------
// The copy issuer, one thread.  It walks this CTA's byte stream in the order
// the consumers use it -- per layer the q, k, v rows, the cached K/V of its
// attention items, the O rows, the gate and up rows and the down rows; per
// step the LM-head rows -- as a sequence of "segments", each a run of ring
// stages described by a few numbers, and issues every stage from one place:
// the producer's code is small because it shares the SM's instruction cache
// with the consumer warps (an earlier form, one inlined copy loop per weight
// matrix, was 39 KB of the kernel).  Stage q of a segment copies
//   cnt = min(per, total - g per) units,  g = q >> kv,
//   from base + (q & kv) kind_stride + g per unit_stride,
// either as cnt pieces of piece_bytes at row_stride, placed at `pitch` in the
// stage (weight rows for the tensor-core GEMV), or as one copy of
// cnt * unit_bytes bytes (LM-head rows, cached K/V).  kv = 1 interleaves the
// K and V streams of an attention item.  Bulk copies only, never multicast.
// With TP > 1 this GPU reads its rank's slice of the MLP (rows of gate/up,
// columns of down) and of the LM head.
template <class S, int TP>
__device__ __forceinline__ void producer(const KParams& P, Smem<S>& sm, uint8_t* ring, int cta) {
  constexpr int IR = S::I / TP, VR = S::V / TP;
  constexpr int LPC = S::STB / (2 * S::H);
  constexpr int RPC_H = S::STB / (2 * S::H + kRowPad), RPC_Q = S::STB / (2 * S::Q + kRowPad),
                RPC_I = S::STB / (2 * IR + kRowPad);
  const int rank = TP > 1 ? P.tp_rank : 0;
  if ((threadIdx.x & 31) != 0) return;
  const uint64_t pol = policy_evict_first();
  const uint32_t nst = (uint32_t)P.nst;
  uint32_t slot = 0, par = 0, issued = 0;
  bool ok = true;
  Spin spin;
#pragma unroll 1
  for (int t = 0; t < P.n_steps && ok; ++t) {
    const int p = P.pos0 + t;
    const int nc = chunks_per_head<S>(p);
    const uint32_t mc = sm.magic_c[nc];
    // seg 0-2 q, k, v; 3 the attention items' K/V (item index in `it`);
    // 4 O; 5 gate; 6 up; 7 down; then (l == L) the LM head.
    int l = 0, seg = 0, it = 0, ihi = 0;
    trace_point<S>(P, sm, t, cta, 0);
#pragma unroll 1
    while (ok) {
      const char* base = nullptr;
      size_t kind_stride = 0, unit_stride = 0, row_stride = 0;
      int total = 0, per = 1, kv = 0, pitch = 0;
      uint32_t unit_bytes = 0, piece_bytes = 0;
      bool pieces = false;
      if (l == S::L) {                                   // LM-head rows
        base = reinterpret_cast<const char*>(sm.wtab[0] + (size_t)(rank * VR + sm.lm0) * S::H);
        total = sm.lm1 - sm.lm0;
        per = LPC;
        unit_bytes = 2 * S::H;
        unit_stride = 2 * S::H;
      } else if (seg == 3) {                             // cached K/V of item `it`
        if (it == 0 && ihi == 0) {
          const uint32_t c = sm.itc[l], nit = (uint32_t)(S::NKV * nc);
          it = (int)divm(c * nit + P.ncta - 1, sm.magic_n);
          ihi = (int)divm((c + 1) * nit + P.ncta - 1, sm.magic_n);
        }
        if (it < ihi) {
          const int h = (int)divm(it, mc), j = it - h * nc;
          const int c0 = (int)divm(j * p, mc);
          const int te = min((int)divm((j + 1) * p, mc), p - 1);
          total = te - c0;
          if (total > 0 && t >= 2) {
            // Positions < p-1 were written by steps <= t-2 (or earlier
            // launches): wait until the consumers have finished step t-2.
            // Position p-1 is read by the consumers directly.
            while (sm.tokens_done < t - 1)
              if (!spin.keep_going(P, sm)) { ok = false; break; }
            fence_proxy_async_global();
          }
          base = reinterpret_cast<const char*>(P.kv + kv_index<S>(l, 0, h, c0, P.max_seq));
          kind_stride = (size_t)S::NKV * P.max_seq * S::D * 2;
          per = S::SUBP;
          unit_bytes = S::D * 2;
          unit_stride = S::D * 2;
          kv = 1;
        }
      } else {                                           // weight rows
        const int ph = seg < 3 ? 0 : seg - 3 - (seg >= 6 ? 1 : 0);
        const uint32_t rr = sm.rows[4 * l + ph];
        int r0 = (int)(rr & 0xffffu), r1 = (int)(rr >> 16);
        int K = S::H, wkey = W_Q + seg;
        row_stride = S::H;
        if (seg < 3) {
          int a, b, o;
          if (qkv_part<S>(r0, r1, seg, a, b, o)) { r0 = a; r1 = b; } else { r1 = r0; }
        } else if (seg == 4) {
          K = S::Q; row_stride = S::Q; wkey = W_O;
        } else if (seg < 7) {
          wkey = seg == 5 ? W_GATE : W_UP;
          r0 += rank * IR; r1 += rank * IR;
        } else {
          K = IR; row_stride = S::I; wkey = W_DOWN;
        }
        const __nv_bfloat16* wb = wptr(l, wkey) + (seg == 7 ? (size_t)rank * IR : 0);
        base = reinterpret_cast<const char*>(wb + (size_t)r0 * row_stride);
        total = r1 - r0;
        per = seg == 4 ? RPC_Q : (seg == 7 ? RPC_I : RPC_H);
        piece_bytes = 2 * K;
        row_stride *= 2;
        unit_stride = row_stride;
        pitch = 2 * K + kRowPad;
        pieces = true;
      }
      // ---- the segment's stages, issued from this one place ----
#pragma unroll 1
      for (int q = 0; ok && total > 0; ++q) {
        const int g = q >> kv;
        const int cnt = min(per, total - g * per);
        if (cnt <= 0) break;
        if (!wait_bar(P, sm, &sm.empty[slot], par ^ 1u)) { ok = false; break; }
        const char* src = base + (size_t)(q & kv) * kind_stride + (size_t)g * per * unit_stride;
        uint8_t* dst = ring + (size_t)slot * S::STB;
        const int n = pieces ? cnt : 1;
        const uint32_t bytes = pieces ? piece_bytes : (uint32_t)cnt * unit_bytes;
        mbar_arrive_expect_tx(&sm.full[slot], (uint32_t)n * bytes);
        for (int i = 0; i < n; ++i)
          bulk_g2s(dst + (size_t)i * pitch, src + (size_t)i * row_stride, bytes, &sm.full[slot], pol);
        ++issued;
        if (++slot == nst) { slot = 0; par ^= 1u; }
      }
      // ---- next segment ----
      if (l == S::L) break;
      if (seg == 3 && it < ihi) { ++it; if (it < ihi) continue; }
      if (++seg == 8) {
        seg = 0; it = 0; ihi = 0;
        ++l;
        if (l < S::L) trace_point<S>(P, sm, t, cta, 7 * l);
      }
    }
  }
  if (!ok) {
    // Abandoned: wait (bounded) for the copies already in flight so that no
    // bulk copy lands in shared memory after this CTA has exited.
    const uint32_t first = issued > nst ? issued - nst : 0;
    for (uint32_t c = first; c < issued; ++c) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sm.full[c % nst], (c / nst) & 1u))
        if ((long long)(globaltimer_ns() - t0) > P.timeout_ns) break;
    }
  }
}

}  // namespace mk

#ifndef MK_MERGE_ML_FIRST
#define MK_MERGE_ML_FIRST 1
#endif

namespace mk {

// Resolve up to NB tagged words already loaded into w[]: while any of them
// lacks `tag`, re-load ALL of the missing ones together, so a round of
// polling costs one L2 round trip however many words a thread owns.
// Bounded like every wait; on expiry the caller proceeds with stale values
// (the abort flag is set and the step is abandoned at the next barrier).
template <class S, int NB, bool SYS = false>
__device__ __forceinline__ void resolve_tagged(const KParams& P, Smem<S>& sm, uint64_t (&w)[NB],
                                               const uint64_t* (&src)[NB], int nvalid, uint32_t tag) {
  bool miss = false;
#pragma unroll
  for (int k = 0; k < NB; ++k) miss |= (k < nvalid) && (uint32_t)(w[k] >> 32) != tag;
  if (!miss) return;
  Spin sp;
  while (miss && sp.keep_going(P, sm)) {
    // Back off between rounds: every CTA polls the same words, and re-issuing
    // all of them back to back floods the L2 slices that hold them (the
    // writers' stores queue behind the polls).
    __nanosleep(MK_POLL_BACKOFF_NS);
#pragma unroll
    for (int k = 0; k < NB; ++k)
      if (k < nvalid && (uint32_t)(w[k] >> 32) != tag) w[k] = SYS ? ld_relaxed_sys(src[k]) : ld_relaxed(src[k]);
    miss = false;
#pragma unroll
    for (int k = 0; k < NB; ++k) miss |= (k < nvalid) && (uint32_t)(w[k] >> 32) != tag;
  }
}

// ---- consumer helpers (all 512 consumer threads call these) -----------------

// Spin on n tagged words src[i] until each carries `tag`; store the fp32
// payloads to dst[i].  Each thread first issues all of its loads (up to
// kBatch in flight) and only then checks tags, so a hop costs about one L2
// round trip instead of one per word.  No barrier inside.
template <class S>
__device__ MK_PHASE void wait_tagged(const KParams& P, Smem<S>& sm, const uint64_t* src,
                                            int n, uint32_t tag, float* dst) {
  constexpr int kBatch = 12;
  const uint64_t tw0 = (MK_TRACE_POINTS && P.trace != nullptr && threadIdx.x == 0) ? globaltimer_ns() : 0;
  for (int base = threadIdx.x; base < n; base += kConsumerThreads * kBatch) {
    uint64_t v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = base + k * kConsumerThreads;
      v[k] = i < n ? ld_relaxed(src + (size_t)i * kHopSpread) : 0;
    }
    const uint64_t* sp[kBatch];
    int nv = 0;
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      sp[k] = src + (size_t)(base + k * kConsumerThreads) * kHopSpread;
      nv += (base + k * kConsumerThreads < n) ? 1 : 0;
    }
    resolve_tagged<S, kBatch>(P, sm, v, sp, nv, tag);
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = base + k * kConsumerThreads;
      if (i < n) dst[i] = __uint_as_float((uint32_t)v[k]);
    }
  }
  if (tw0 != 0) sm.wait_hop_ns += globaltimer_ns() - tw0;
}

// One tagged word, returned as float.
template <class S>
__device__ __forceinline__ float wait_word(const KParams& P, Smem<S>& sm, const uint64_t* src,
                                           uint32_t tag) {
  uint64_t v = ld_relaxed(src);
  if ((uint32_t)(v >> 32) != tag) v = poll_tagged_slow(P, sm, src, tag);
  return __uint_as_float((uint32_t)v);
}

// Block-wide fp32 sum over the consumer threads (fixed reduction order).
template <class S>
__device__ __forceinline__ float consumer_sum(Smem<S>& sm, float v) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) sm.red[warp] = v;
  consumer_sync(kConsumerThreads);
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) s += sm.red[w];
  consumer_sync(kConsumerThreads);
  return s;
}

// xs[0..2][i] = bf16 terms hi, mid, lo of x with hi + mid + lo == x to fp32
// precision.  The tensor-core GEMV multiplies all three terms.
template <class S>
__device__ __forceinline__ void split_one(Smem<S>& sm, int i, float x) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(hi);
  const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(mid);
  sm.xs[0][i] = hi;
  sm.xs[1][i] = mid;
  sm.xs[2][i] = __float2bfloat16_rn(r2);
}
template <class S>
__device__ MK_PHASE void split_xin(Smem<S>& sm, int n) {
  for (int i = threadIdx.x; i < n; i += kConsumerThreads) split_one(sm, i, sm.xin[i]);
  consumer_sync(kConsumerThreads);
}

// Norm gains are loaded into registers BEFORE the caller waits for the
// activation hop, so their global-memory latency overlaps the wait.
template <class S>
struct GainRegs {
  static constexpr int kPer = (S::H + kConsumerThreads - 1) / kConsumerThreads;
  float g[kPer];
  __device__ __forceinline__ void load(const __nv_bfloat16* gp) {
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      const int i = threadIdx.x + e * kConsumerThreads;
      g[e] = i < S::H ? __bfloat162float(gp[i]) : 0.f;
    }
  }
};

// xin = g * (xres * rsqrt(mean(xres^2) + eps))   (Qwen3RMSNorm order), also
// split into xs.  Replaces rmsnorm_float_in (src/rmsnorm.cuh:87-108); computed
// redundantly in every CTA and kept in shared memory, never written back.
template <class S>
__device__ MK_PHASE void rmsnorm_to_xin(Smem<S>& sm, const GainRegs<S>& gr) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < S::H; i += kConsumerThreads) ss += sm.xres[i] * sm.xres[i];
  ss = consumer_sum(sm, ss);
  const float r = rsqrtf(ss / (float)S::H + 1e-6f);
#pragma unroll
  for (int e = 0; e < GainRegs<S>::kPer; ++e) {
    const int i = threadIdx.x + e * kConsumerThreads;
    if (i < S::H) {
      const float v = gr.g[e] * (sm.xres[i] * r);
      sm.xin[i] = v;
      split_one(sm, i, v);
    }
  }
  consumer_sync(kConsumerThreads);
}

// One tensor-core GEMV pass over up to three row segments that follow each
// other in the ring (this CTA's rows of Wq, Wk, Wv; or of Wgate and Wup; or
// of one matrix), all with K columns and the same input x:
//     out_s[r] = scale * (W_s[r, :] . x).
// The producer placed each segment's rows in consecutive stages at pitch
// 2K + 16 (RPC rows per stage).  Replaces gemv_block / gemv_qkv /
// gemv_gate_up_silu (src/gemv.cuh:36-279) with warp-level tensor-core MMAs:
//   A = 16 weight rows x 16 columns (ldmatrix from the stage),
//   B = 16 columns x 8, whose columns 0..2 are the hi/mid/lo bf16 terms of x
//       (sm.xs), so a row's dot product is D[r][0] + D[r][1] + D[r][2] in fp32.
// Warp w takes the 16-column slices w, w + 8, ... of up to four 16-row tiles.
//
// The pass is split in two so that everything that does not depend on x runs
// before the caller waits for x: prepare() waits for the stages, computes the
// fragment addresses and loads the first PIT slices of weight fragments into
// registers; finish() (after x is in sm.xs) runs the MMAs, reduces the 8
// warps' partials in a fixed order and releases the stages.  Each segment has
// <= 32 rows and the pass's stages fit the ring (checked on the host).  All
// consumer threads call both; the plan lives in registers (inlined).
template <class S, int K, int MAXT>
struct GemvPlan {
  static constexpr int PITCH = S::template pitch<K>();
  static constexpr int RPC = S::template rows_per_stage<K>();
  static constexpr int KS = K / 16;
  static constexpr int ITER = (KS + kConsumerWarps - 1) / kConsumerWarps;
  static constexpr int PIT = ITER < MK_GEMV_PIT ? ITER : MK_GEMV_PIT;   // slices preloaded per tile
  // Ragged K (a tensor-parallel column slice): the last slices exist for only
  // some warps, which skip the rest (a warp-uniform test).
  static constexpr bool kRag = KS % kConsumerWarps != 0;
  static_assert(RPC >= 1 && K % 16 == 0, "GEMV shape");
  uint32_t slot0;
  int nch, ntile, t0n, t1n, n0, n1, n2;
  bool ok;
  static_assert(MAXT >= 1 && MAXT <= 4, "tiles");
  uint32_t abase[MAXT];
  uint32_t pa[PIT][MAXT][4];

  __device__ __forceinline__ void prepare(const KParams& P, Smem<S>& sm, const uint8_t* ring, uint32_t kc,
                                          int m0, int m1, int m2) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t nst = (uint32_t)P.nst;
    n0 = m0; n1 = m1; n2 = m2;
    const int ch0 = (n0 + RPC - 1) / RPC, ch1 = (n1 + RPC - 1) / RPC, ch2 = (n2 + RPC - 1) / RPC;
    nch = ch0 + ch1 + ch2;
    t0n = (n0 + 15) >> 4;
    t1n = (n1 + 15) >> 4;
    ntile = t0n + t1n + ((n2 + 15) >> 4);
    slot0 = kc % nst;
    const uint32_t ph0 = (kc / nst) & 1u;
    ok = true;
    for (int c = 0; c < nch; ++c) {
      uint32_t sl = slot0 + c, ph = ph0;
      if (sl >= nst) { sl -= nst; ph ^= 1u; }
      if (!mbar_test(&sm.full[sl], ph)) ok = wait_bar_slow(P, sm, &sm.full[sl], ph) && ok;
    }
    ok = __all_sync(0xffffffffu, ok);
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
      const bool in0 = t < t0n, in1 = !in0 && t < t0n + t1n;
      const int tn = in0 ? n0 : (in1 ? n1 : n2);
      const int tc = in0 ? 0 : (in1 ? ch0 : ch0 + ch1);
      const int tr = in0 ? t * 16 : (in1 ? (t - t0n) * 16 : (t - t0n - t1n) * 16);
      int lrow = tr + ((lane >> 3) & 1) * 8 + (lane & 7);
      if (lrow >= tn) lrow = tr;  // rows past the segment: a valid address, result unused
      const int c = tc + lrow / RPC, rin = lrow % RPC;
      uint32_t sl = slot0 + c;
      if (sl >= nst) sl -= nst;
      abase[t] = smem_u32(ring + (size_t)sl * S::STB + (size_t)rin * PITCH) + (uint32_t)((lane >> 4) * 16);
    }
    if (ok) {
#pragma unroll
      for (int it = 0; it < PIT; ++it)
#pragma unroll
        for (int t = 0; t < MAXT; ++t)
          if (t < ntile && (!kRag || warp + it * kConsumerWarps < KS))
            ldmatrix_x4(abase[t] + (warp + it * kConsumerWarps) * 32, pa[it][t][0], pa[it][t][1],
                        pa[it][t][2], pa[it][t][3]);
    }
  }

  // scale: per-row factor applied to the dot products (the RMSNorm 1/rms when
  // the caller passes x without it), or 1.
  __device__ __forceinline__ uint32_t finish(const KParams& P, Smem<S>& sm, float* out0, float* out1,
                                             float* out2, bool norm_scale) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;
    const uint32_t nst = (uint32_t)P.nst;
    if (nch == 0) return 0;
    // Tile 0 alternates two accumulator sets so a single-tile pass (O,
    // down) does not chain every MMA on the previous one.
    float d[MAXT][4] = {}, e[4] = {};
    if (ok) {
      const uint32_t* xs0 = reinterpret_cast<const uint32_t*>(&sm.xs[g < 3 ? g : 0][0]);
      // Preloaded slices first ...
#pragma unroll
      for (int it = 0; it < PIT; ++it) {
        const int ks = warp + it * kConsumerWarps;
        if (kRag && ks >= KS) break;
        const uint32_t b0 = g < 3 ? xs0[ks * 8 + tq] : 0u;
        const uint32_t b1 = g < 3 ? xs0[ks * 8 + tq + 4] : 0u;
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
          if (t < ntile) {
            if (t == 0 && (it & 1))
              mma_bf16_16816(e[0], e[1], e[2], e[3], pa[it][t][0], pa[it][t][1], pa[it][t][2], pa[it][t][3], b0, b1);
            else
              mma_bf16_16816(d[t][0], d[t][1], d[t][2], d[t][3], pa[it][t][0], pa[it][t][1], pa[it][t][2],
                             pa[it][t][3], b0, b1);
          }
        }
      }
      // ... then the rest, loaded from the stages as they are used.
#pragma unroll kGemvUnroll
      for (int it = PIT; it < ITER; ++it) {
        const int ks = warp + it * kConsumerWarps;
        if (kRag && ks >= KS) break;
        const uint32_t b0 = g < 3 ? xs0[ks * 8 + tq] : 0u;
        const uint32_t b1 = g < 3 ? xs0[ks * 8 + tq + 4] : 0u;
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
          if (t < ntile) {
            uint32_t a0, a1, a2, a3;
            ldmatrix_x4(abase[t] + ks * 32, a0, a1, a2, a3);
            if (t == 0 && (it & 1)) mma_bf16_16816(e[0], e[1], e[2], e[3], a0, a1, a2, a3, b0, b1);
            else mma_bf16_16816(d[t][0], d[t][1], d[t][2], d[t][3], a0, a1, a2, a3, b0, b1);
          }
        }
      }
    }
    // Lane (g, tq=0) holds columns 0,1 of rows g, g+8; lane (g, tq=1) column 2.
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
      if (t < ntile) {
        if (t == 0) {
          d[0][0] += e[0]; d[0][1] += e[1]; d[0][2] += e[2]; d[0][3] += e[3];
        }
        float s0 = d[t][0] + d[t][1];
        float s1 = d[t][2] + d[t][3];
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        if (tq == 0) {
          sm.partw[warp][t * 16 + g] = s0;
          sm.partw[warp][t * 16 + g + 8] = s1;
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      for (int c = 0; c < nch; ++c) {
        uint32_t sl = slot0 + c;
        if (sl >= nst) sl -= nst;
        mbar_arrive(&sm.empty[sl]);
      }
    }
    consumer_sync(kConsumerThreads);
    if (threadIdx.x < ntile * 16) {
      const int t = threadIdx.x >> 4, r = threadIdx.x & 15;
      const int row = (t < t0n ? t * 16 : (t < t0n + t1n ? (t - t0n) * 16 : (t - t0n - t1n) * 16)) + r;
      const int n = t < t0n ? n0 : (t < t0n + t1n ? n1 : n2);
      float* out = t < t0n ? out0 : (t < t0n + t1n ? out1 : out2);
      if (row < n) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w += 2) {
          a0 += sm.partw[w][threadIdx.x];
          a1 += sm.partw[w + 1][threadIdx.x];
        }
        float v = a0 + a1;
        if (norm_scale) {
          float ss = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) ss += sm.red[w];
          v *= rsqrtf(ss / (float)S::H + 1e-6f);
        }
        out[row] = v;
      }
    }
    consumer_sync(kConsumerThreads);
    return (uint32_t)nch;
  }
};

// Wait for n tagged fp32 words of an activation hop and stage them for the
// next GEMV: optionally keep v in xres (residual stream), scale by the
// RMSNorm gain (GAIN) and write the three bf16 split terms of the result to
// xs.  Returns this thread's sum of v^2; callers that normalise reduce it
// into sm.red (per warp) before the barrier that precedes GemvPlan::finish.
template <class S, bool GAIN, bool RES, int kBatch>
__device__ __forceinline__ float hop_to_xs(const KParams& P, Smem<S>& sm, const uint64_t* src, int n,
                                           uint32_t tag, const GainRegs<S>& gr) {
  float ss = 0.f;
#pragma unroll 1
  for (int base = threadIdx.x; base < n; base += kConsumerThreads * kBatch) {
    uint64_t w[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = base + k * kConsumerThreads;
      w[k] = i < n ? ld_relaxed(src + (size_t)i * kHopSpread) : 0;
    }
    const uint64_t* sp[kBatch];
    int nv = 0;
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      sp[k] = src + (size_t)(base + k * kConsumerThreads) * kHopSpread;
      nv += (base + k * kConsumerThreads < n) ? 1 : 0;
    }
    resolve_tagged<S, kBatch>(P, sm, w, sp, nv, tag);
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = base + k * kConsumerThreads;
      if (i < n) {
        const float v = __uint_as_float((uint32_t)w[k]);
        if (RES) sm.xres[i] = v;
        ss = fmaf(v, v, ss);
        float x = v;
        if (GAIN) x = gr.g[k < GainRegs<S>::kPer ? k : 0] * v;
        split_one(sm, i, x);
      }
    }
  }
  return ss;
}

// Tensor-parallel layer input: x = x' + sum over ranks (in rank order, so
// every GPU computes the same fp32 value) of each rank's partial down
// projection, read from the TP slots src[j * H + i] that the ranks write over
// NVLink.  x' (the residual after attention) is in xres and is replaced by x.
// With SPLIT the (gain-scaled) x is also staged for the next GEMV as in
// hop_to_xs.  Returns this thread's sum of x^2.
template <class S, int TP, bool SPLIT>
__device__ __forceinline__ float hop_sum_to_xs(const KParams& P, Smem<S>& sm, const uint64_t* src,
                                               uint32_t tag, const GainRegs<S>& gr) {
  constexpr int PER = GainRegs<S>::kPer;
  static_assert(S::H % kConsumerThreads == 0, "whole rows per thread");
  // At most 16 words in flight per thread (registers); TP = 8 takes two rounds.
  constexpr int EG = PER * TP <= 16 ? PER : 16 / TP;
  float ss = 0.f;
#pragma unroll
  for (int e0 = 0; e0 < PER; e0 += EG) {
    uint64_t w[EG * TP];
    const uint64_t* sp[EG * TP];
#pragma unroll
    for (int e = 0; e < EG; ++e)
#pragma unroll
      for (int j = 0; j < TP; ++j) {
        sp[e * TP + j] = src + ((size_t)j * S::H + threadIdx.x + (e0 + e) * kConsumerThreads) * kHopSpread;
        w[e * TP + j] = ld_relaxed_sys(sp[e * TP + j]);
      }
    resolve_tagged<S, EG * TP, true>(P, sm, w, sp, EG * TP, tag);
#pragma unroll
    for (int e = 0; e < EG; ++e) {
      const int i = threadIdx.x + (e0 + e) * kConsumerThreads;
      float v = sm.xres[i];
#pragma unroll
      for (int j = 0; j < TP; ++j) v += __uint_as_float((uint32_t)w[e * TP + j]);
      sm.xres[i] = v;
      ss = fmaf(v, v, ss);
      if (SPLIT) split_one(sm, i, gr.g[e0 + e] * v);
    }
  }
  return ss;
}

// Per-warp partial of the RMSNorm sum of squares into sm.red[warp].
template <class S>
__device__ __forceinline__ void norm_partial(Smem<S>& sm, float ss) {
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) sm.red[threadIdx.x >> 5] = ss;
}

// LM head over rows [r0, r1) of the tied embedding: per-warp running argmax
// (strictly greater => lowest index kept), optional fp32 logits.  Replaces
// lm_head_argmax_phase1 (src/sampling.cuh:32-89): a warp reads whole 2*H-byte
// rows from shared memory instead of one thread walking each row.
template <class S>
__device__ MK_PHASE uint32_t lm_rows(const KParams& P, Smem<S>& sm, const uint8_t* ring,
                                        uint32_t kc, int r0, int r1, float* logits_row0,
                                        float& best_v, int& best_i) {
  const uint32_t kc0 = kc;
  constexpr int PPR = S::H / 256;
  constexpr int RB = 2 * S::H;
  constexpr int RPC = S::STB / RB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t nst = (uint32_t)P.nst;
  float xr[PPR][8];
#pragma unroll
  for (int q = 0; q < PPR; ++q) {
#pragma unroll
    for (int e = 0; e < 8; ++e) xr[q][e] = sm.xin[q * 256 + lane * 8 + e];
  }
  for (int cr = r0; cr < r1; cr += RPC) {
    const int n = min(RPC, r1 - cr);
    const uint32_t slot = kc % nst, ph = (kc / nst) & 1u;
    if (__all_sync(0xffffffffu, wait_bar(P, sm, &sm.full[slot], ph))) {
      const uint8_t* st = ring + (size_t)slot * S::STB + lane * 16;
      const int rel = cr - r0;
      for (int r = ((warp - rel) % kConsumerWarps + kConsumerWarps) % kConsumerWarps; r < n;
           r += kConsumerWarps) {
        float a = 0.f;
#pragma unroll
        for (int q = 0; q < PPR; ++q)
          a += dot8(*reinterpret_cast<const uint4*>(st + (size_t)r * RB + q * 512), xr[q]);
        a = warp_sum(a);
        const int row = cr + r;
        if (a > best_v) { best_v = a; best_i = row; }
        if (logits_row0 != nullptr && lane == 0) logits_row0[row] = a;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
    ++kc;
  }
  return kc - kc0;
}

}  // namespace mk

namespace mk {

// Online-softmax update over n1 + n2 positions whose K and V rows (D bf16
// each) sit contiguously in shared memory: [0, n1) at K1/V1 (a ring stage),
// [n1, n1 + n2) at K2/V2 (the previous and current positions).
// Scores: one thread per (head, position), a full D-long dot product with no
// cross-lane reduction; the 16-byte pieces of a row are visited in an order
// rotated by the position so the rows a warp reads hit distinct banks.
// PV: thread (part, g, d) sums positions = part (mod parts).  The running
// (m, l) live in sm.mrun/lrun; the PV accumulator stays in `acc`.
template <class S>
__device__ MK_PHASE void attend_block(Smem<S>& sm, const __nv_bfloat16* K1, const __nv_bfloat16* V1,
                                          int n1, const __nv_bfloat16* K2, const __nv_bfloat16* V2,
                                          int n2, float (&acc)[S::D / 32]) {
  constexpr int D = S::D, GRP = S::GRP;
  constexpr int PIECES = D / 8;  // 16-byte pieces per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = n1 + n2;
  const float scale = (D == 64) ? 0.125f : 0.08838834764831845f;  // D^-0.5
#pragma unroll 1
  for (int i = threadIdx.x; i < GRP * n; i += kConsumerThreads) {
    const int g = i / n, pos = i - g * n;
    const __nv_bfloat16* kr = pos < n1 ? K1 + (size_t)pos * D : K2 + (size_t)(pos - n1) * D;
    const uint4* k4 = reinterpret_cast<const uint4*>(kr);
    const float4* q4 = reinterpret_cast<const float4*>(&sm.qs[g][0]);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int jj = 0; jj < PIECES; ++jj) {
      const int j = (jj + pos) & (PIECES - 1);
      const uint4 w = k4[j];
      const float4 qa = q4[2 * j], qb = q4[2 * j + 1];
      s0 = fmaf(bf_lo(w.x), qa.x, s0);
      s1 = fmaf(bf_hi(w.x), qa.y, s1);
      s0 = fmaf(bf_lo(w.y), qa.z, s0);
      s1 = fmaf(bf_hi(w.y), qa.w, s1);
      s0 = fmaf(bf_lo(w.z), qb.x, s0);
      s1 = fmaf(bf_hi(w.z), qb.y, s1);
      s0 = fmaf(bf_lo(w.w), qb.z, s0);
      s1 = fmaf(bf_hi(w.w), qb.w, s1);
    }
    sm.sc[g][pos] = (s0 + s1) * scale;
  }
  consumer_sync(kConsumerThreads);
  if (warp < GRP) {
    const int g = warp;
    float mx = -INFINITY;
#pragma unroll 1
    for (int pos = lane; pos < n; pos += 32) mx = fmaxf(mx, sm.sc[g][pos]);
    mx = warp_max(mx);
    const float mold = sm.mrun[g];
    const float mnew = fmaxf(mold, mx);
    const float c = expf(mold - mnew);
    float sum = 0.f;
#pragma unroll 1
    for (int pos = lane; pos < n; pos += 32) {
      const float e = expf(sm.sc[g][pos] - mnew);
      sm.sc[g][pos] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    if (lane == 0) {
      sm.lrun[g] = sm.lrun[g] * c + sum;
      sm.mrun[g] = mnew;
      sm.corr[g] = c;
    }
  }
  consumer_sync(kConsumerThreads);
  {
    // P.V: warp w takes query head w % GRP and every kPvParts-th position
    // starting at w / GRP; lane l the DPL dims [l DPL, (l+1) DPL), loaded as
    // bf16 pairs (one 4- or 8-byte load per position and lane).
    constexpr int DPL = D / 32;
    const int g = warp % GRP, part = warp / GRP, d0 = lane * DPL;
    float a[DPL], b[DPL];
#pragma unroll
    for (int k = 0; k < DPL; ++k) a[k] = b[k] = 0.f;
    auto fma_row = [&](float (&c)[DPL], float pw, const __nv_bfloat16* vr) {
#pragma unroll
      for (int k = 0; k < DPL; k += 2) {
        const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vr + d0 + k));
        c[k] = fmaf(pw, v.x, c[k]);
        c[k + 1] = fmaf(pw, v.y, c[k + 1]);
      }
    };
    int pos = part;
#pragma unroll kPvUnroll
    for (; pos + kPvParts < n1; pos += 2 * kPvParts) {
      fma_row(a, sm.sc[g][pos], V1 + (size_t)pos * D);
      fma_row(b, sm.sc[g][pos + kPvParts], V1 + (size_t)(pos + kPvParts) * D);
    }
    for (; pos < n; pos += kPvParts)
      fma_row(a, sm.sc[g][pos], pos < n1 ? V1 + (size_t)pos * D : V2 + (size_t)(pos - n1) * D);
    const float c = sm.corr[g];
#pragma unroll
    for (int k = 0; k < DPL; ++k) acc[k] = acc[k] * c + (a[k] + b[k]);
  }
  consumer_sync(kConsumerThreads);
}

// Attention item (KV head h, chunk j of nc) for layer l at position p: QK-norm,
// RoPE, append of the current K/V (last chunk only), online softmax over the
// chunk, and a tagged partial {acc[GRP][D], m, l}.  Replaces qk_rmsnorm_inplace
// (src/rmsnorm.cuh:57-84), apply_rope_inplace (src/attention.cuh:22-44),
// append_kv (src/kv_cache.cuh:58-78) and warp_attention (src/attention.cuh:100-167).
template <class S>
__device__ MK_PHASE uint32_t attention_item(const KParams& P, Smem<S>& sm, const uint8_t* ring, uint32_t kc,
                                           int t, int l, int p, uint32_t seq, int h, int j, int nc,
                                           int item) {
  const uint32_t kc0 = kc;
  constexpr int D = S::D, GRP = S::GRP, HALF = D / 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t* qkv = P.hop + HopLayout<S>::QKV + (size_t)(l & 1) * S::QKV;
  const uint32_t tq = tag_of(seq, l, 0);
  const uint32_t nst = (uint32_t)P.nst;
  int c0, c1;
  chunk_range(p, nc, j, c0, c1);
  const bool last = (j == nc - 1);
  const bool prev = (p >= 1) && (c0 <= p - 1) && (p - 1 < c1);
  const int te = min(c1, p - 1);

  // Side inputs that do not depend on this step's activations are loaded into
  // registers first, so their latency overlaps the wait for q, k, v: threads
  // [0, D) load the q/k gains and the K/V of position p-1, threads [0, D/2)
  // the RoPE row of position p.
  static_assert(D <= kConsumerThreads, "one thread per head dimension");
  float pre0 = 0.f, pre1 = 0.f, rc = 0.f, rs = 0.f;
  unsigned short prek = 0, prev_v = 0;
  if (tid < D) {
    pre0 = __bfloat162float(wptr(l, W_QNORM)[tid]);
    pre1 = __bfloat162float(wptr(l, W_KNORM)[tid]);
    if (tid < HALF) {
      rc = P.rope_cos[(size_t)p * HALF + tid];
      rs = P.rope_sin[(size_t)p * HALF + tid];
    }
    if (prev) {
      // Written by the previous step (possibly another CTA): read through L2.
      const unsigned short* kvu = reinterpret_cast<const unsigned short*>(P.kv);
      prek = __ldcg(kvu + kv_index<S>(l, 0, h, p - 1, P.max_seq) + tid);
      prev_v = __ldcg(kvu + kv_index<S>(l, 1, h, p - 1, P.max_seq) + tid);
    }
  }
  // Raw q (GRP heads), k, v of this KV head -> sm.xin as scratch [GRP+2][D]
  // (xin is free between the q/k/v GEMV and the merge).
  static_assert((S::GRP + 2) * S::D <= S::XIN, "attention scratch");
  float* raw = sm.xin;
  {
    // q (GRP heads), k and v of head h: up to three words per thread,
    // resolved together (one L2 round trip per polling round).
    static_assert(GRP * D <= kConsumerThreads, "one q word per thread");
    const uint64_t* sp[3] = {qkv + h * GRP * D + tid, qkv + S::Q + h * D + tid,
                             qkv + S::Q + S::KV + h * D + tid};
    const int nv = tid < D ? 3 : (tid < GRP * D ? 1 : 0);
    uint64_t w[3] = {0, 0, 0};
    if (nv > 0) w[0] = ld_relaxed(sp[0]);
    if (nv > 1) { w[1] = ld_relaxed(sp[1]); w[2] = ld_relaxed(sp[2]); }
    resolve_tagged<S, 3>(P, sm, w, sp, nv, tq);
    if (nv > 0) raw[tid] = __uint_as_float((uint32_t)w[0]);
    if (nv > 1) {
      raw[GRP * D + tid] = __uint_as_float((uint32_t)w[1]);
      raw[(GRP + 1) * D + tid] = __uint_as_float((uint32_t)w[2]);
    }
  }
  if (tid < D) {
    sm.gq[tid] = pre0;
    sm.gk[tid] = pre1;
    if (tid < HALF) {
      sm.rc[tid] = rc;
      sm.rs[tid] = rs;
    }
    if (prev) {
      sm.kx[0][tid] = __ushort_as_bfloat16(prek);
      sm.vx[0][tid] = __ushort_as_bfloat16(prev_v);
    }
  }
  if (tid < GRP) { sm.mrun[tid] = -INFINITY; sm.lrun[tid] = 0.f; }
  consumer_sync(kConsumerThreads);
  MK_DP(4);

  // Per-head RMSNorm (q_norm / k_norm gains) then rotate-half RoPE at p.
  if (warp <= GRP) {
    float* x = raw + warp * D;
    const float* gn = warp < GRP ? sm.gq : sm.gk;
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) ss += x[d] * x[d];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + 1e-6f);
    float y[D / 32];
#pragma unroll
    for (int e = 0; e < D / 32; ++e) y[e] = gn[lane + 32 * e] * (x[lane + 32 * e] * r);
    __syncwarp();
#pragma unroll
    for (int e = 0; e < D / 32; ++e) x[lane + 32 * e] = y[e];
    __syncwarp();
    for (int d = lane; d < HALF; d += 32) {
      const float x0 = x[d], x1 = x[d + HALF], c = sm.rc[d], s = sm.rs[d];
      const float o0 = x0 * c - x1 * s;
      const float o1 = x1 * c + x0 * s;
      if (warp < GRP) {
        sm.qs[warp][d] = o0;
        sm.qs[warp][d + HALF] = o1;
      } else {
        sm.kx[1][d] = __float2bfloat16_rn(o0);
        sm.kx[1][d + HALF] = __float2bfloat16_rn(o1);
      }
    }
  } else if (warp == GRP + 1) {
    const float* v = raw + (GRP + 1) * D;
    for (int d = lane; d < D; d += 32) sm.vx[1][d] = __float2bfloat16_rn(v[d]);
  }
  consumer_sync(kConsumerThreads);
  MK_DP(5);

  float acc[D / 32];
#pragma unroll
  for (int k = 0; k < D / 32; ++k) acc[k] = 0.f;
  // Positions held outside the ring -- p-1 (slot 0) and the current p (slot
  // 1) -- ride along with the first ring block (or form the only block).
  // Cached positions [c0, te) stream through the ring as (K, V) stage pairs.
  // One call site for attend_block: it is inlined, and a second site would
  // add ~10 KB to a kernel body that already overflows the instruction cache.
  const int s0 = prev ? 0 : 1;
  int ne = (prev ? 1 : 0) + (last ? 1 : 0);
  for (int a = c0, first = 1; first || a < te; a += S::SUBP, first = 0) {
    const bool ring_blk = a < te;
    const int n = ring_blk ? min(S::SUBP, te - a) : 0;
    const uint32_t sk = kc % nst, pk = (kc / nst) & 1u;
    const uint32_t sv = (kc + 1) % nst, pv = ((kc + 1) / nst) & 1u;
    bool ok = true;
    if (ring_blk) {
      ok = wait_bar(P, sm, &sm.full[sk], pk);
      ok = ok && wait_bar(P, sm, &sm.full[sv], pv);
    }
    const int blk = (a - c0) / S::SUBP;
    if (blk < 4) MK_DP(20 + 2 * blk);
    if (!consumer_any(kConsumerThreads, !ok) && n + ne > 0) {
      attend_block(sm, reinterpret_cast<const __nv_bfloat16*>(ring + (size_t)sk * S::STB),
                   reinterpret_cast<const __nv_bfloat16*>(ring + (size_t)sv * S::STB), n,
                   &sm.kx[s0][0], &sm.vx[s0][0], ne, acc);
    }
    if (blk < 4) MK_DP(21 + 2 * blk);
    ne = 0;
    if (ring_blk) {
      if (lane == 0) { mbar_arrive(&sm.empty[sk]); mbar_arrive(&sm.empty[sv]); }
      kc += 2;
    }
  }
  MK_DP(7);
  {
    // This warp's head / part / dims, as attend_block's P.V assigns them.
    constexpr int DPL = D / 32;
    float* dst = &sm.pv[((warp / GRP) * GRP + warp % GRP) * D + lane * DPL];
#pragma unroll
    for (int k = 0; k < DPL; ++k) dst[k] = acc[k];
  }
  consumer_sync(kConsumerThreads);
  uint64_t* out = P.hop + HopLayout<S>::ATT + (size_t)(l & 1) * HopLayout<S>::kAttWords +
                  (size_t)item * GRP * (D + 2);
  const uint32_t ta = tag_of(seq, l, 1);
  if (tid < GRP * D) {
    constexpr int GD = GRP * D;
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kPvParts; ++q) s += sm.pv[q * GD + tid];
    const int g = tid / D, d = tid % D;
    st_tagged(out + g * (D + 2) + d, ta, __float_as_uint(s));
  }
  if (tid < GRP) {
    st_tagged(out + tid * (D + 2) + D, ta, __float_as_uint(sm.mrun[tid]));
    st_tagged(out + tid * (D + 2) + D + 1, ta, __float_as_uint(sm.lrun[tid]));
  }
  MK_DP(6);
  if (last && tid < D) {
    // Append the current K/V (bf16) at position p, after the partial is
    // published.  Its first reader is the next step, so the fences that make
    // it visible (to other CTAs' loads and TMA copies) are issued once per
    // step, before this CTA publishes its LM-head pair (fence_kv_appends).
    const int d = tid;
    P.kv[kv_index<S>(l, 0, h, p, P.max_seq) + d] = sm.kx[1][d];
    P.kv[kv_index<S>(l, 1, h, p, P.max_seq) + d] = sm.vx[1][d];
  }
  consumer_sync(kConsumerThreads);
  return kc - kc0;
}

// Two-level merge (nc >= kMerge2MinChunks): the CTA that walked chunk 0 of KV
// head h merges the nc partials of that head's GRP query heads and publishes
// the GRP x D results to the MH hop, so the other CTAs read Q words instead of
// every partial (at 16 chunks the direct merge had each of 148 CTAs read
// 135 KB of partials, about 9 us per layer).  Called after all of this CTA's
// items of the layer, so it never waits on a partial this CTA has yet to make.
template <class S, int TP>
__device__ MK_PHASE void merge_head(const KParams& P, Smem<S>& sm, int l, uint32_t seq, int nc, int h) {
  constexpr int D = S::D, GRP = S::GRP;
  static_assert(GRP * kMaxChunksPerHead <= kConsumerThreads && GRP * D <= kConsumerThreads, "merge_head");
  const int tid = threadIdx.x;
  const uint64_t* att = P.hop + HopLayout<S>::ATT + (size_t)(l & 1) * HopLayout<S>::kAttWords +
                        (size_t)h * nc * GRP * (D + 2);
  const uint32_t ta = tag_of(seq, l, 1);
  if (tid < GRP * nc) {
    const int g = tid / nc, j = tid % nc;
    const uint64_t* bj = att + ((size_t)j * GRP + g) * (D + 2) + D;
    uint64_t w2[2] = {ld_relaxed(bj), ld_relaxed(bj + 1)};
    const uint64_t* sp2[2] = {bj, bj + 1};
    resolve_tagged<S, 2>(P, sm, w2, sp2, 2, ta);
    sm.mlbuf[2 * tid] = __uint_as_float((uint32_t)w2[0]);
    sm.mlbuf[2 * tid + 1] = __uint_as_float((uint32_t)w2[1]);
  }
  consumer_sync(kConsumerThreads);
  if (tid < GRP * D) {
    const int g = tid / D, dd = tid % D;
    uint64_t w[kMaxChunksPerHead];
    const uint64_t* sp[kMaxChunksPerHead];
#pragma unroll
    for (int j = 0; j < kMaxChunksPerHead; ++j) {
      sp[j] = att + ((size_t)j * GRP + g) * (D + 2) + dd;
      w[j] = j < nc ? ld_relaxed(sp[j]) : 0;
    }
    resolve_tagged<S, kMaxChunksPerHead>(P, sm, w, sp, nc, ta);
    float M = -INFINITY;
    for (int j = 0; j < nc; ++j) M = fmaxf(M, sm.mlbuf[2 * (g * nc + j)]);
    float den = 0.f, acc = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxChunksPerHead; ++j) {
      if (j < nc) {
        const float cj = expf(sm.mlbuf[2 * (g * nc + j)] - M);
        den = fmaf(sm.mlbuf[2 * (g * nc + j) + 1], cj, den);
        acc = fmaf(__uint_as_float((uint32_t)w[j]), cj, acc);
      }
    }
    st_tagged(P.hop + HopLayout<S, TP>::MH + (size_t)(l & 1) * S::Q + (size_t)(h * GRP + g) * D + dd, ta,
              __float_as_uint(acc / den));
  }
  consumer_sync(kConsumerThreads);
}

// Merge the split-KV partials of layer l into xin[Q] (every CTA, redundantly):
// out = sum_j exp(m_j - M) acc_j / sum_j exp(m_j - M) l_j.
// Each CTA polls every partial word exactly once per round: the per-head
// (m, l) pairs by a few threads into shared memory, then each thread its EPT
// accumulator words of every chunk (resolved together, one L2 round trip per
// polling round).  Also writes the bf16 split terms of each output.
template <class S, int TP, bool M2>
__device__ MK_PHASE void merge_attention(const KParams& P, Smem<S>& sm, int l, uint32_t seq, int nc) {
  constexpr int D = S::D, GRP = S::GRP;
  if (M2 && nc >= kMerge2MinChunks) {
    // Two-level: the per-head results are in the MH hop.
    constexpr int EQ = (S::Q + kConsumerThreads - 1) / kConsumerThreads;
    const uint64_t* mh = P.hop + HopLayout<S, TP>::MH + (size_t)(l & 1) * S::Q;
    uint64_t w[EQ];
    const uint64_t* sp[EQ];
#pragma unroll
    for (int k = 0; k < EQ; ++k) {
      sp[k] = mh + threadIdx.x + k * kConsumerThreads;
      w[k] = threadIdx.x + k * kConsumerThreads < S::Q ? ld_relaxed(sp[k]) : 0;
    }
    const int nv = (S::Q - (int)threadIdx.x + kConsumerThreads - 1) / kConsumerThreads;
    resolve_tagged<S, EQ>(P, sm, w, sp, nv < EQ ? nv : EQ, tag_of(seq, l, 1));
#pragma unroll
    for (int k = 0; k < EQ; ++k) {
      const int i = threadIdx.x + k * kConsumerThreads;
      if (i < S::Q) {
        const float v = __uint_as_float((uint32_t)w[k]);
        sm.xin[i] = v;
        split_one(sm, i, v);
      }
    }
    return;
  }
  constexpr int EPT = S::Q >= kConsumerThreads ? S::Q / kConsumerThreads : 1;
  static_assert(D % EPT == 0, "a thread's outputs stay inside one head");
  const uint64_t* att = P.hop + HopLayout<S>::ATT + (size_t)(l & 1) * HopLayout<S>::kAttWords;
  const uint32_t ta = tag_of(seq, l, 1);
  const size_t stride = (size_t)GRP * (D + 2);
  // (m, l) of every (query head, chunk): word pairs at item * stride + g * (D+2) + D.
  for (int i = threadIdx.x; i < S::NQ * nc; i += kConsumerThreads) {
    const int qh = i / nc, j = i % nc;
    const uint64_t* bj = att + ((size_t)(qh / GRP) * nc + j) * stride + (size_t)(qh % GRP) * (D + 2) + D;
    uint64_t w2[2] = {ld_relaxed(bj), ld_relaxed(bj + 1)};
    const uint64_t* sp2[2] = {bj, bj + 1};
    resolve_tagged<S, 2>(P, sm, w2, sp2, 2, ta);
    sm.mlbuf[2 * i] = __uint_as_float((uint32_t)w2[0]);
    sm.mlbuf[2 * i + 1] = __uint_as_float((uint32_t)w2[1]);
  }
  const int e0 = threadIdx.x * EPT;
  const bool active = e0 < S::Q;
  const int qh = active ? e0 / D : 0, d0 = e0 % D, g = qh % GRP;
  const uint64_t* b = att + ((size_t)(qh / GRP) * nc * GRP + g) * (D + 2) + d0;
  // Accumulator words, kGroup chunks at a time (registers and code size bound
  // the group; from kMerge2MinChunks chunks on the two-level merge runs
  // instead, so one group covers every direct merge of a launch that picks
  // its kernel by position).  Word q of a group
  // is chunk j0 + q / EPT, element q % EPT.
  constexpr int kGroup = kMerge2MinChunks, NW = kGroup * EPT;
  uint64_t w[NW];
#if MK_MERGE_ML_FIRST
  // Poll the accumulator words only once every (m, l) pair is present: their
  // writers publish them together, so one round then finds nearly all of
  // them, instead of every thread of every CTA re-polling its words while
  // the items are still running (which also slows the writers' stores).
  consumer_sync(kConsumerThreads);
#pragma unroll
  for (int q = 0; q < NW; ++q)
    w[q] = (active && q / EPT < nc) ? ld_relaxed(b + (size_t)(q / EPT) * stride + q % EPT) : 0;
#else
#pragma unroll
  for (int q = 0; q < NW; ++q)
    w[q] = (active && q / EPT < nc) ? ld_relaxed(b + (size_t)(q / EPT) * stride + q % EPT) : 0;
  consumer_sync(kConsumerThreads);
#endif
  float M = -INFINITY, den = 0.f, acc[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) acc[k] = 0.f;
  if (active) {
    for (int j = 0; j < nc; ++j) M = fmaxf(M, sm.mlbuf[2 * (qh * nc + j)]);
    for (int j0 = 0; j0 < nc; j0 += kGroup) {
      const int nvw = min(kGroup, nc - j0) * EPT;
      const uint64_t* bg = b + (size_t)j0 * stride;
      if (j0 > 0) {
#pragma unroll
        for (int q = 0; q < NW; ++q) w[q] = q < nvw ? ld_relaxed(bg + (size_t)(q / EPT) * stride + q % EPT) : 0;
      }
      bool miss = false;
#pragma unroll
      for (int q = 0; q < NW; ++q) miss |= q < nvw && (uint32_t)(w[q] >> 32) != ta;
      Spin spn;
      while (miss && spn.keep_going(P, sm)) {
        __nanosleep(MK_POLL_BACKOFF_NS);
        miss = false;
#pragma unroll
        for (int q = 0; q < NW; ++q)
          if (q < nvw && (uint32_t)(w[q] >> 32) != ta) w[q] = ld_relaxed(bg + (size_t)(q / EPT) * stride + q % EPT);
#pragma unroll
        for (int q = 0; q < NW; ++q) miss |= q < nvw && (uint32_t)(w[q] >> 32) != ta;
      }
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        if (j * EPT < nvw) {
          const float cj = expf(sm.mlbuf[2 * (qh * nc + j0 + j)] - M);
          den = fmaf(sm.mlbuf[2 * (qh * nc + j0 + j) + 1], cj, den);
#pragma unroll
          for (int k = 0; k < EPT; ++k) acc[k] = fmaf(__uint_as_float((uint32_t)w[j * EPT + k]), cj, acc[k]);
        }
      }
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      sm.xin[e0 + k] = acc[k] * inv;
      split_one(sm, e0 + k, acc[k] * inv);
    }
  }
}

template <class S, int TP, bool M2>
__device__ __forceinline__ void consumers(const KParams& P, Smem<S>& sm, const uint8_t* ring, int cta) {
  const int N = P.ncta, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Tensor parallelism (TP > 1): this GPU computes the MLP rows [rank IR,
  // (rank + 1) IR) and the LM-head rows [rank VR, (rank + 1) VR); attention
  // and the O projection are replicated on every GPU.
  constexpr int IR = S::I / TP, VR = S::V / TP;
  const int rank = TP > 1 ? P.tp_rank : 0;
  uint32_t kc = 0;
  // Token ids come from the caller (forced) or from the argmax.  A forced
  // id outside the vocabulary is never used as an embedding row index: the
  // launch records MK_ERR_INVALID_ARG (which every CTA's watchdog turns
  // into an abort) and reads row 0 meanwhile.  (An early-exit path here
  // measured ~30 us/token slower: this kernel is sensitive to code layout.)
  int tok = P.forced[0];
  if (tok < 0 || tok >= S::V) {
    if (tid == 0) atomicCAS(P.err, 0, MK_ERR_INVALID_ARG);
    tok = 0;
  }
  #pragma unroll 1
  for (int t = 0; t < P.n_steps; ++t) {
    const int p = P.pos0 + t;
    const uint32_t seq = P.seq0 + (uint32_t)t;
    const int nc = chunks_per_head<S>(p);
    const int nitems = S::NKV * nc;
    const long long clk0 = clock64();
    bool appended = false;
    {
      const __nv_bfloat16* er = sm.wtab[0] + (size_t)tok * S::H;
      for (int i = tid; i < S::H; i += kConsumerThreads) sm.xres[i] = __bfloat162float(er[i]);
    }
    consumer_sync(kConsumerThreads);
    #pragma unroll 1
    for (int l = 0; l < S::L; ++l) {
      // ---- P1: x -> RMSNorm -> q, k, v rows --------------------------------
      // RMSNorm is folded into the GEMV: W (g . x / rms) = (W (g . x)) / rms,
      // so the GEMV runs on g . x while the sum of squares is reduced.
      GainRegs<S> gains;
      gains.load(wptr(l, W_ATTN_NORM));
      int s0, s1;
      split_rows(S::QKV, N, cta, phase_rot(l, 0, N), s0, s1);
      int rq[3], oq[3];
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        int a, b, o;
        rq[m] = qkv_part<S>(s0, s1, m, a, b, o) ? b - a : 0;
        oq[m] = rq[m] ? o - s0 : 0;
      }
      {
        GemvPlan<S, S::H, 4> gp;
        gp.prepare(P, sm, ring, kc, rq[0], rq[1], rq[2]);
        float ss = 0.f;
        if (l > 0) {
          if constexpr (TP == 1)
            ss = hop_to_xs<S, true, true, GainRegs<S>::kPer>(P, sm, P.hop + HopLayout<S>::X + (size_t)(l & 1) * S::H * kHopSpread, S::H,
                                          tag_of(seq, l - 1, 4), gains);
          else
            ss = hop_sum_to_xs<S, TP, true>(P, sm, P.hop + HopLayout<S, TP>::X + (size_t)(l & 1) * TP * S::H * kHopSpread,
                                            tag_of(seq, l - 1, 4), gains);
        } else {
#pragma unroll
          for (int e = 0; e < GainRegs<S>::kPer; ++e) {
            const int i = tid + e * kConsumerThreads;
            if (i < S::H) {
              const float v = sm.xres[i];
              ss = fmaf(v, v, ss);
              split_one(sm, i, gains.g[e] * v);
            }
          }
        }
        norm_partial(sm, ss);
        if (consumer_any(kConsumerThreads, sm.abort_flag != 0)) return;
        if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * l + 1);
        MK_DP(1);
        kc += gp.finish(P, sm, sm.rowsum[0] + oq[0], sm.rowsum[0] + oq[1], sm.rowsum[0] + oq[2], true);
      }
      MK_DP(2);
      {
        uint64_t* dst = P.hop + HopLayout<S>::QKV + (size_t)(l & 1) * S::QKV;
        const uint32_t tg = tag_of(seq, l, 0);
        for (int r = tid; r < s1 - s0; r += kConsumerThreads)
          st_tagged(dst + s0 + r, tg, __float_as_uint(sm.rowsum[0][r]));
        // (no barrier needed: the next writer of rowsum[0] is behind several)
        if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * l + 2);
      }
      // ---- P2: attention items owned by this CTA ------------------------------
      {
        int ilo, ihi;
        items_of_cta(cta, l, nitems, N, ilo, ihi);
        for (int i = ilo; i < ihi; ++i) {
          kc += attention_item<S>(P, sm, ring, kc, t, l, p, seq, i / nc, i % nc, nc, i);
          appended |= (i % nc == nc - 1);
        }
        if (M2 && nc >= kMerge2MinChunks)
          for (int i = ilo; i < ihi; ++i)
            if (i % nc == 0) merge_head<S, TP>(P, sm, l, seq, nc, i / nc);
      }
      // ---- P3: merge -> O projection + residual --------------------------------
      {
        int r0, r1;
        split_rows(S::H, N, cta, phase_rot(l, 1, N), r0, r1);
        GemvPlan<S, S::Q, 2> gp;
        gp.prepare(P, sm, ring, kc, r1 - r0, 0, 0);
        MK_DP(8);
        merge_attention<S, TP, M2>(P, sm, l, seq, nc);
        if (consumer_any(kConsumerThreads, sm.abort_flag != 0)) return;
        MK_DP(9);
        if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * l + 3);
        kc += gp.finish(P, sm, sm.rowsum[0], nullptr, nullptr, false);
        MK_DP(10);
        uint64_t* dst = P.hop + HopLayout<S>::XA + (size_t)(l & 1) * S::H * kHopSpread;
        const uint32_t tg = tag_of(seq, l, 2);
        for (int r = tid; r < r1 - r0; r += kConsumerThreads)
          st_tagged(dst + (size_t)(r0 + r) * kHopSpread, tg, __float_as_uint(sm.xres[r0 + r] + sm.rowsum[0][r]));
        if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * l + 4);
      }
      // ---- P4: x' -> RMSNorm -> silu(gate) * up ---------------------------------
      {
        gains.load(wptr(l, W_FFN_NORM));
        int r0, r1;
        split_rows(IR, N, cta, phase_rot(l, 2, N), r0, r1);
        GemvPlan<S, S::H, 4> gp;
        gp.prepare(P, sm, ring, kc, r1 - r0, r1 - r0, 0);
        // xres is rewritten by the hop below: every thread must be done with
        // the O epilogue's reads of it.
        consumer_sync(kConsumerThreads);
        const float ss = hop_to_xs<S, true, true, GainRegs<S>::kPer>(P, sm, P.hop + HopLayout<S>::XA + (size_t)(l & 1) * S::H * kHopSpread,
                                                  S::H, tag_of(seq, l, 2), gains);
        norm_partial(sm, ss);
        if (consumer_any(kConsumerThreads, sm.abort_flag != 0)) return;
        MK_DP(13);
        kc += gp.finish(P, sm, sm.rowsum[0], sm.rowsum[1], nullptr, true);
        MK_DP(15);
        uint64_t* dst = P.hop + HopLayout<S>::HM + (size_t)(l & 1) * S::I * kHopSpread;
        const uint32_t tg = tag_of(seq, l, 3);
        for (int r = tid; r < r1 - r0; r += kConsumerThreads) {
          const float g = sm.rowsum[0][r];
          const float u = sm.rowsum[1][r];
          const float hval = (g / (1.0f + expf(-g))) * u;
          st_tagged(dst + (size_t)(r0 + r) * kHopSpread, tg, __float_as_uint(hval));
        }
        if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * l + 5);
      }
      // ---- P5: h -> down projection + residual --------------------------------
      {
        int r0, r1;
        split_rows(S::H, N, cta, phase_rot(l, 3, N), r0, r1);
        GemvPlan<S, IR, 2> gp;
        gp.prepare(P, sm, ring, kc, r1 - r0, 0, 0);
        hop_to_xs<S, false, false, (IR + kConsumerThreads - 1) / kConsumerThreads>(P, sm, P.hop + HopLayout<S>::HM + (size_t)(l & 1) * S::I * kHopSpread, IR,
                                   tag_of(seq, l, 3), gains);
        if (consumer_any(kConsumerThreads, sm.abort_flag != 0)) return;
        MK_DP(17);
        kc += gp.finish(P, sm, sm.rowsum[0], nullptr, nullptr, false);
        MK_DP(18);
        uint64_t* dst = P.hop + HopLayout<S>::X + (size_t)((l + 1) & 1) * S::H * kHopSpread;
        const uint32_t tg = tag_of(seq, l, 4);
        const bool skip = (l == 0 && cta == P.debug_skip_cta);
        if constexpr (TP == 1) {
          if (!skip)
            for (int r = tid; r < r1 - r0; r += kConsumerThreads)
              st_tagged(dst + (size_t)(r0 + r) * kHopSpread, tg, __float_as_uint(sm.xres[r0 + r] + sm.rowsum[0][r]));
        } else {
          // This rank's partial rows (no residual: every rank adds x' itself)
          // into slot `rank` of every GPU's X hop, over NVLink for the peers.
          (void)dst;
          const size_t off = HopLayout<S, TP>::X + ((size_t)((l + 1) & 1) * TP * S::H + (size_t)rank * S::H + r0) * kHopSpread;
          if (!skip)
            for (int r = tid; r < r1 - r0; r += kConsumerThreads)
#pragma unroll
              for (int j = 0; j < TP; ++j)
                st_tagged_sys(P.peer_hop[j] + off + (size_t)r * kHopSpread, tg, __float_as_uint(sm.rowsum[0][r]));
        }
        // xres is rewritten by the next layer's hop: finish the reads first.
        consumer_sync(kConsumerThreads);
        if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * l + 6);
      }
    }
    // ---- final RMSNorm -> LM head -> argmax ------------------------------------
    // K/V appended during this step become visible before this CTA's LM-head
    // pair is published: every reader of them (next step's attention, the
    // copy engines two steps on) first observes all CTAs' pairs of this step.
    if (appended && tid < S::D) {
      fence_proxy_async_global();
      __threadfence();
    }
    appended = false;
    GainRegs<S> fgains;
    fgains.load(sm.wtab[1]);
    if constexpr (TP == 1)
      wait_tagged(P, sm, P.hop + HopLayout<S>::X + (size_t)(S::L & 1) * S::H * kHopSpread, S::H,
                  tag_of(seq, S::L - 1, 4), sm.xres);
    else
      hop_sum_to_xs<S, TP, false>(P, sm, P.hop + HopLayout<S, TP>::X + (size_t)(S::L & 1) * TP * S::H * kHopSpread,
                                  tag_of(seq, S::L - 1, 4), fgains);
    if (consumer_any(kConsumerThreads, sm.abort_flag != 0)) return;
    rmsnorm_to_xin(sm, fgains);
    if (tid == 0) trace_point<S>(P, sm, t, cta, 7 * S::L);
    {
      int r0, r1;
      split_rows(VR, N, cta, phase_rot(S::L, 4, N), r0, r1);
      r0 += rank * VR;
      r1 += rank * VR;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      float* lrow = P.logits ? P.logits + (size_t)t * S::V : nullptr;
      kc += lm_rows<S>(P, sm, ring, kc, r0, r1, lrow, bv, bi);
      if (lane == 0) { sm.red[warp] = bv; sm.redi[warp] = bi; }
      consumer_sync(kConsumerThreads);
      // (max, index) pair of CTA c of rank j at slot j * N + c.
      const size_t lm_off = HopLayout<S, TP>::LM + (size_t)(t & 1) * TP * kMaxCtas * 2;
      uint64_t* lm = P.hop + lm_off;
      const uint32_t tg = tag_of(seq, S::L, 0);
      if (tid == 0) {
        float v = sm.red[0];
        int ix = sm.redi[0];
        for (int w = 1; w < kConsumerWarps; ++w)
          if (sm.red[w] > v || (sm.red[w] == v && sm.redi[w] < ix)) { v = sm.red[w]; ix = sm.redi[w]; }
        if constexpr (TP == 1) {
          st_tagged(lm + 2 * cta, tg, __float_as_uint(v));
          st_tagged(lm + 2 * cta + 1, tg, (uint32_t)ix);
        } else {
          const size_t slot = (size_t)rank * N + cta;
#pragma unroll
          for (int j = 0; j < TP; ++j) {
            st_tagged_sys(P.peer_hop[j] + lm_off + 2 * slot, tg, __float_as_uint(v));
            st_tagged_sys(P.peer_hop[j] + lm_off + 2 * slot + 1, tg, (uint32_t)ix);
          }
        }
        trace_point<S>(P, sm, t, cta, 7 * S::L + 1);
      }
      // Every CTA reduces all CTAs' (max, index) pairs: lowest index wins ties.
      if constexpr (TP == 1) {
        float* pairs = &sm.partw[0][0];
        for (int c = tid; c < N; c += kConsumerThreads) {
          uint64_t w2[2] = {ld_relaxed(lm + 2 * c), ld_relaxed(lm + 2 * c + 1)};
          const uint64_t* sp2[2] = {lm + 2 * c, lm + 2 * c + 1};
          resolve_tagged<S, 2>(P, sm, w2, sp2, 2, tg);
          pairs[c] = __uint_as_float((uint32_t)w2[0]);
          pairs[kMaxCtas + c] = __uint_as_float((uint32_t)w2[1]);
        }
        consumer_sync(kConsumerThreads);
        if (warp == 0) {
          float v = -INFINITY;
          int ix = 0x7fffffff;
          for (int c = lane; c < N; c += 32) {
            const float cv = pairs[c];
            const int ci = (int)__float_as_uint(pairs[kMaxCtas + c]);
            if (cv > v || (cv == v && ci < ix)) { v = cv; ix = ci; }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
            if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
          }
          if (lane == 0) sm.next_token = ix;
        }
      } else {
        // TP * N pairs (all ranks): a running best per thread, then per warp,
        // then across the warps.
        float v = -INFINITY;
        int ix = 0x7fffffff;
        for (int c = tid; c < TP * N; c += kConsumerThreads) {
          uint64_t w2[2] = {ld_relaxed_sys(lm + 2 * c), ld_relaxed_sys(lm + 2 * c + 1)};
          const uint64_t* sp2[2] = {lm + 2 * c, lm + 2 * c + 1};
          resolve_tagged<S, 2, true>(P, sm, w2, sp2, 2, tg);
          const float cv = __uint_as_float((uint32_t)w2[0]);
          const int ci = (int)(uint32_t)w2[1];
          if (cv > v || (cv == v && ci < ix)) { v = cv; ix = ci; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, v, o);
          const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
          if (ov > v || (ov == v && oi < ix)) { v = ov; ix = oi; }
        }
        // sm.red / redi were last read by thread 0 before its publish above.
        consumer_sync(kConsumerThreads);
        if (lane == 0) { sm.red[warp] = v; sm.redi[warp] = ix; }
        consumer_sync(kConsumerThreads);
        if (tid == 0) {
          for (int w = 1; w < kConsumerWarps; ++w)
            if (sm.red[w] > sm.red[0] || (sm.red[w] == sm.red[0] && sm.redi[w] < sm.redi[0])) {
              sm.red[0] = sm.red[w];
              sm.redi[0] = sm.redi[w];
            }
          sm.next_token = sm.redi[0];
        }
      }
      if (consumer_any(kConsumerThreads, sm.abort_flag != 0)) return;
      const int best = sm.next_token;
      if (cta == 0 && tid == 0) P.out_tokens[t] = best;
      tok = (t + 1 < P.n_forced) ? P.forced[t + 1] : best;
      if (tok < 0 || tok >= S::V) {
        if (tid == 0) atomicCAS(P.err, 0, MK_ERR_INVALID_ARG);
        tok = 0;
      }
      if (tid == 0) {
        trace_point<S>(P, sm, t, cta, 7 * S::L + 2);
        if (MK_TRACE_POINTS && P.trace != nullptr && t < P.trace_steps) {
          uint64_t* tr = P.trace + ((size_t)t * P.ncta + cta) * Trace<S>::kPoints;
          tr[7 * S::L + 3] = sm.wait_hop_ns;
          tr[7 * S::L + 4] = (uint64_t)(clock64() - clk0);
        }
        sm.wait_hop_ns = 0;
        __threadfence();
        sm.tokens_done = t + 1;
      }
    }
  }
}

// Watchdog (one thread of the producer warpgroup): every wait in this CTA is
// bounded through it.  It records an error and raises abort_flag when the
// CTA's progress counter has not moved for timeout_ns (MK_ERR_TIMEOUT) or
// when another CTA has reported an error; every wait then gives up, the
// roles leave at their next barrier, and the producer drains its copies.
template <class S>
__device__ __forceinline__ void watchdog(const KParams& P, Smem<S>& sm) {
  uint32_t last = sm.progress;
  uint64_t t_last = globaltimer_ns();
  while (!sm.done && !sm.abort_flag) {
    __nanosleep(500);
    const uint64_t now = globaltimer_ns();
    const uint32_t pr = sm.progress;
    if (pr != last) {
      last = pr;
      t_last = now;
    } else if ((long long)(now - t_last) > P.timeout_ns) {
      fail(P, sm, MK_ERR_TIMEOUT);
      break;
    }
    if (ld_volatile_i32(P.err) != 0) {
      sm.abort_flag = 1;
      break;
    }
  }
}

// M2: compile the two-level attention merge (used from kMerge2MinChunks chunks
// per head on).  It is a separate instance because its code alone (about
// 19 KB) slows the short-context steps that never use it: the kernel body
// already exceeds the SM's instruction cache.
template <class S, int TP = 1, bool M2 = false>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ KParams P) {
  static_assert(TP >= 1 && TP <= kMaxTP && S::I % TP == 0 && S::V % TP == 0 && (S::I / TP) % 16 == 0,
                "tensor-parallel split");
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* ring = dsm;
  Smem<S>& sm = *reinterpret_cast<Smem<S>*>(dsm + (size_t)S::NST * S::STB);
  for (int i = threadIdx.x; i < S::NOFF; i += blockDim.x) sm.wtab[i] = P.w[i];
  if (threadIdx.x == 0) sm.prm = P;
  {
    // The producer's schedule (see Smem::rows): the same split_rows /
    // phase_rot / items_of_cta plan the consumers follow.
    constexpr int IR = S::I / TP, VR = S::V / TP;
    const int N = P.ncta, i = threadIdx.x;
    if (i < 4 * S::L) {
      const int l = i >> 2, ph = i & 3;
      const int R = ph == 0 ? S::QKV : (ph == 2 ? IR : S::H);
      int r0, r1;
      split_rows(R, N, blockIdx.x, phase_rot(l, ph, N), r0, r1);
      sm.rows[i] = (uint32_t)r0 | ((uint32_t)r1 << 16);
    } else if (i < 5 * S::L) {
      const int l = i - 4 * S::L;
      sm.itc[l] = (uint16_t)(((unsigned)blockIdx.x + (unsigned)N - (unsigned)(l * 53) % (unsigned)N) % (unsigned)N);
    } else if (i == 5 * S::L) {
      split_rows(VR, N, blockIdx.x, phase_rot(S::L, 4, N), sm.lm0, sm.lm1);
      sm.magic_n = magic_of((uint32_t)N);
    } else if (i > 5 * S::L && i <= 5 * S::L + kMaxChunksPerHead) {
      const uint32_t d = (uint32_t)(i - 5 * S::L);
      sm.magic_c[d] = magic_of(d);
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NST; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort_flag = 0;
    sm.tokens_done = 0;
    sm.progress = 0;
    sm.done = 0;
    sm.wait_hop_ns = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int cta = blockIdx.x;
  // The device functions read the parameters from shared memory.  The
  // producer warpgroup (one working warp) hands registers to the two
  // consumer warpgroups.
  if (threadIdx.x >= kConsumerThreads) {
    setmaxnreg_dec<kProducerRegs>();
    if (threadIdx.x < kConsumerThreads + 32) producer<S, TP>(sm.prm, sm, ring, cta);
    else if (threadIdx.x == kConsumerThreads + 32) watchdog<S>(sm.prm, sm);
  } else {
    setmaxnreg_inc<kConsumerRegs>();
    consumers<S, TP, M2>(sm.prm, sm, ring, cta);
    if (threadIdx.x == 0) sm.done = 1;
  }
}

template <class S>
constexpr size_t smem_bytes() { return (size_t)S::NST * S::STB + sizeof(Smem<S>); }

}  // namespace mk

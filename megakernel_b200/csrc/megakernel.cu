// Host state, launch and C ABI of libmegakernel.
//
// Replaces the host half of src/megakernel.cu (MegakernelState :345-353,
// decode_step :377-413, extern "C" API :535-624) and the allocators of
// src/kv_cache.cuh:84-92, src/barriers.cuh:155-187 and src/sampling.cuh:123-141.
// Differences that matter to a caller: every CUDA call is checked, errors are
// reported (NULL / -1 / negative status), the device is an option instead of
// device 0, the kernel launch is cooperative (it fails instead of deadlocking
// when the CTAs cannot all be resident), and the KV capacity is a runtime size.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/megakernel.h"
#include "decode_kernel.cuh"

namespace {

constexpr int kDefaultMaxSeq = 8448;
constexpr uint32_t kSeqLimit = 1u << 24;

struct State {
  int shape_id = -1;
  int device = 0;
  int ncta = 0;
  int nst = 0;                  // ring stages in use
  int issue_gap_ns = 0;         // producer pacing (MK_ISSUE_GAP_NS tuning knob)
  int max_seq = 0;
  int pos = 0;
  uint32_t seq = 1;
  int last_error = MK_OK;
  long long timeout_ns = 1000000000LL;
  int debug_skip_cta = -1;
  bool capture_logits = false;
  int merge_mode = 0;           // 0 auto, 1 direct, 2 two-level instance
  size_t smem = 0;
  int vocab = 0;
  const void* kernel = nullptr;         // direct attention merge
  const void* kernel_m2 = nullptr;      // two-level attention merge (long context)

  const __nv_bfloat16** d_wptr = nullptr;
  __nv_bfloat16* d_kv = nullptr;
  size_t kv_bytes = 0;
  float* d_cos = nullptr;
  float* d_sin = nullptr;
  uint64_t* d_hop = nullptr;
  size_t hop_bytes = 0;
  int* d_err = nullptr;
  int* d_tok = nullptr;         // [2]: input token, output token of megakernel_decode
  float* d_logits = nullptr;
  int* h_pinned = nullptr;      // [2]: output token, error code
  cudaStream_t stream = nullptr;
  uint64_t* d_trace = nullptr;  // caller-owned trace buffer
  int trace_steps = 0;
  uint64_t* d_detail = nullptr; // caller-owned sub-phase buffer (profiling)
  const void* d_weights = nullptr;       // caller's weight buffer and offsets (parallel prefill)
  std::vector<long long> offsets;
  void* prefill = nullptr;               // lazily built batched state bound to d_kv (batch.cu)
  // Tensor parallelism (megakernel_tp_*): rank, size, and every rank's hop
  // buffer (own at [tp_rank], peers mapped by CUDA IPC).
  int tp_rank = 0;
  int tp_size = 1;
  bool tp_connected = false;
  uint64_t* peer_hop[mk::kMaxTP] = {};
  bool peer_opened[mk::kMaxTP] = {};
};

void prefill_free(void* p);   // batch.cu

}  // namespace

namespace mk_tp {
const void* kernel(int shape_id, int tp, bool m2, size_t* hop_words);   // tp.cu
}

namespace {

struct ShapeInfo {
  int H, L, NQ, NKV, D, I, V;
};

template <class S>
ShapeInfo info_of() { return {S::H, S::L, S::NQ, S::NKV, S::D, S::I, S::V}; }

ShapeInfo shape_info(int id) {
  switch (id) {
    case 0: return info_of<mk::ShapeD64>();
    case 1: return info_of<mk::ShapeD128>();
    default: return info_of<mk::ShapeTiny>();
  }
}
constexpr int kNumShapes = 3;

#define MK_CUDA(call)                                                        \
  do {                                                                       \
    cudaError_t e_ = (call);                                                 \
    if (e_ != cudaSuccess) {                                                 \
      std::fprintf(stderr, "megakernel: %s failed: %s\n", #call,             \
                   cudaGetErrorString(e_));                                  \
      return e_ == cudaErrorMemoryAllocation ? MK_ERR_OOM : MK_ERR_CUDA;     \
    }                                                                        \
  } while (0)

void host_rope(int D, double theta, int positions, float* c, float* s) {
  const int half = D / 2;
  for (int i = 0; i < half; ++i) {
    // inv_freq = 1 / theta^(2i/D) in fp32, angle = inv_freq * pos in fp32
    // (transformers modeling_rope_utils.py:178, modeling_qwen3.py:140-144).
    // torch evaluates theta ** x like a double pow rounded to fp32.
    const float expo = (float)(2 * i) / (float)D;
    const float inv = 1.0f / (float)pow(theta, (double)expo);
    for (int p = 0; p < positions; ++p) {
      const float ang = (float)p * inv;
      c[(size_t)p * half + i] = (float)cos((double)ang);
      s[(size_t)p * half + i] = (float)sin((double)ang);
    }
  }
}

// Every phase's rows per CTA must fit the kernel's per-CTA row buffers.
bool rows_fit(const ShapeInfo& s, int N) {
  auto rows = [&](int R) { return (R + N - 1) / N; };
  const int Q = s.NQ * s.D, KV = s.NKV * s.D;
  return rows(Q + 2 * KV) <= mk::kRowsMax && rows(s.H) <= mk::kRowsMax &&
         rows(s.I) <= mk::kRowsMax && N <= mk::kMaxCtas;
}

// The tensor-core GEMV takes a phase's segments in one pass: every segment
// <= 32 rows, <= 4 tiles of 16 rows per pass, and all stages of the pass in
// the ring at once.
template <class S>
bool plan_fits(int N, int nst) {
  auto rows = [&](int R) { return (R + N - 1) / N; };
  auto chunks = [](int r, int rpc) { return (r + rpc - 1) / rpc; };
  const int rq = rows(S::QKV), rh = rows(S::H), ri = rows(S::I);
  const int rpc_h = S::template rows_per_stage<S::H>();
  if (rq > 32 || rh > 32 || ri > 32) return false;
  if ((rq + 15) / 16 + 2 > 4) return false;                        // q/k/v tiles
  if (chunks(rq, rpc_h) + 2 > nst) return false;
  if (2 * chunks(ri, rpc_h) > nst) return false;                   // gate + up
  if (chunks(rh, S::template rows_per_stage<S::Q>()) > nst) return false;
  if (chunks(rh, S::template rows_per_stage<S::I>()) > nst) return false;
  return N <= mk::kMaxCtas;
}

template <class S>
void kernel_info(State* st) {
  st->kernel = reinterpret_cast<const void*>(&mk::decode_kernel<S>);
  st->smem = mk::smem_bytes<S>();
  st->hop_bytes = mk::HopLayout<S>::TOTAL * 8;
  // MK_RING_STAGES (tuning knob): use fewer ring stages than fit.
  st->nst = S::NST;
  if (const char* e = std::getenv("MK_RING_STAGES")) {
    const int v = std::atoi(e);
    if (v >= 4 && v < S::NST) st->nst = v;
  }
  if (const char* e = std::getenv("MK_ISSUE_GAP_NS")) st->issue_gap_ns = std::atoi(e);
}

void free_state(State* st) {
  if (!st) return;
  for (int j = 0; j < mk::kMaxTP; ++j)
    if (st->peer_opened[j]) cudaIpcCloseMemHandle(st->peer_hop[j]);
  cudaFree(st->d_wptr);
  cudaFree(st->d_kv);
  cudaFree(st->d_cos);
  cudaFree(st->d_sin);
  cudaFree(st->d_hop);
  cudaFree(st->d_err);
  cudaFree(st->d_tok);
  cudaFree(st->d_logits);
  if (st->h_pinned) cudaFreeHost(st->h_pinned);
  if (st->stream) cudaStreamDestroy(st->stream);
  prefill_free(st->prefill);
  delete st;
}

int infer_shape(const long long* off, int n) {
  if (!off || n < 13 || (n - 2) % 11 != 0) return MK_ERR_SHAPE;
  const int L = (n - 2) / 11;
  const long long H = (off[2] - off[1]) / 2;
  if (H <= 0) return MK_ERR_SHAPE;
  for (int id = 0; id < kNumShapes; ++id) {
    const ShapeInfo s = shape_info(id);
    if (s.L != L || s.H != H) continue;
    const long long Q = (long long)s.NQ * s.D, KV = (long long)s.NKV * s.D;
    if (off[1] - off[0] != 2LL * s.V * s.H) continue;
    if (off[4] - off[3] != 2 * Q * s.H) continue;       // w_q
    if (off[5] - off[4] != 2 * KV * s.H) continue;      // w_k
    if (off[7] - off[6] != 2LL * s.D) continue;         // q_norm
    if (off[11] - off[10] != 2LL * s.I * s.H) continue; // w_gate
    return id;
  }
  return MK_ERR_SHAPE;
}

}  // namespace

namespace {

int init_impl(void* d_weights, const long long* offsets, int num_offsets, const mk_options* o,
              State** out, int tp_rank = 0, int tp_size = 1) {
  *out = nullptr;
  if (!d_weights || !offsets) return MK_ERR_INVALID_ARG;
  if (tp_size < 1 || tp_size > mk::kMaxTP || tp_rank < 0 || tp_rank >= tp_size) return MK_ERR_INVALID_ARG;
  const int id = o->shape_id >= 0 ? o->shape_id : infer_shape(offsets, num_offsets);
  if (id < 0 || id >= kNumShapes) return MK_ERR_SHAPE;
  const ShapeInfo s = shape_info(id);
  if (num_offsets != 2 + 11 * s.L) return MK_ERR_SHAPE;
  for (int i = 0; i < num_offsets; ++i)
    if (offsets[i] < 0 || (offsets[i] & 15) != 0) return MK_ERR_INVALID_ARG;  // TMA alignment
  if ((reinterpret_cast<uintptr_t>(d_weights) & 15) != 0) return MK_ERR_INVALID_ARG;

  State* st = new (std::nothrow) State();
  if (!st) return MK_ERR_OOM;
  auto bail = [&](int code) { free_state(st); return code; };
  st->shape_id = id;
  st->d_weights = d_weights;
  st->offsets.assign(offsets, offsets + num_offsets);
  st->vocab = s.V;
  st->max_seq = o->max_seq > 0 ? o->max_seq : kDefaultMaxSeq;
  st->timeout_ns = o->timeout_ns > 0 ? o->timeout_ns : 1000000000LL;
  st->debug_skip_cta = o->debug_skip_cta;
  int dev = o->device;
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return bail(MK_ERR_CUDA);
  st->device = dev;
  if (cudaSetDevice(dev) != cudaSuccess) return bail(MK_ERR_CUDA);

  switch (id) {
    case 0: kernel_info<mk::ShapeD64>(st); break;
    case 1: kernel_info<mk::ShapeD128>(st); break;
    default: kernel_info<mk::ShapeTiny>(st); break;
  }
  st->tp_rank = tp_rank;
  st->tp_size = tp_size;
  {
    size_t words = 0;
    st->kernel_m2 = mk_tp::kernel(id, tp_size, true, &words);
    if (!st->kernel_m2) return bail(MK_ERR_INVALID_ARG);   // (shape, TP size) not compiled
    if (tp_size > 1) {
      st->kernel = st->kernel_m2;
      st->hop_bytes = words * 8;
    }
  }
  int sms = 0, coop = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess)
    return bail(MK_ERR_CUDA);
  if (!coop) return bail(MK_ERR_LAUNCH);
  if (cudaFuncSetAttribute(st->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)st->smem) != cudaSuccess ||
      cudaFuncSetAttribute(st->kernel_m2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)st->smem) != cudaSuccess)
    return bail(MK_ERR_LAUNCH);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, st->kernel, mk::kThreads, st->smem) !=
          cudaSuccess || occ < 1)
    return bail(MK_ERR_LAUNCH);
  st->ncta = o->num_ctas > 0 ? o->num_ctas : sms;
  bool fits = false;
  switch (id) {
    case 0: fits = plan_fits<mk::ShapeD64>(st->ncta, st->nst); break;
    case 1: fits = plan_fits<mk::ShapeD128>(st->ncta, st->nst); break;
    default: fits = plan_fits<mk::ShapeTiny>(st->ncta, st->nst); break;
  }
  if (st->ncta > sms * occ || !rows_fit(s, st->ncta) || !fits) return bail(MK_ERR_INVALID_ARG);

  if (cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(MK_ERR_CUDA);
  // Weight pointer table (offsets order of src/megakernel.cu:518-532).
  {
    const __nv_bfloat16** h = new (std::nothrow) const __nv_bfloat16*[num_offsets];
    if (!h) return bail(MK_ERR_OOM);
    for (int i = 0; i < num_offsets; ++i)
      h[i] = reinterpret_cast<const __nv_bfloat16*>(static_cast<const char*>(d_weights) + offsets[i]);
    cudaError_t e = cudaMalloc(&st->d_wptr, sizeof(void*) * num_offsets);
    if (e == cudaSuccess)
      e = cudaMemcpy(st->d_wptr, h, sizeof(void*) * num_offsets, cudaMemcpyHostToDevice);
    delete[] h;
    if (e != cudaSuccess) return bail(MK_ERR_OOM);
  }
  st->kv_bytes = (size_t)s.L * 2 * s.NKV * (size_t)st->max_seq * s.D * sizeof(__nv_bfloat16);
  if (cudaMalloc(&st->d_kv, st->kv_bytes) != cudaSuccess) return bail(MK_ERR_OOM);
  if (cudaMemset(st->d_kv, 0, st->kv_bytes) != cudaSuccess) return bail(MK_ERR_CUDA);
  {
    const size_t n = (size_t)st->max_seq * (s.D / 2);
    float* hc = new (std::nothrow) float[n];
    float* hs = new (std::nothrow) float[n];
    if (!hc || !hs) { delete[] hc; delete[] hs; return bail(MK_ERR_OOM); }
    host_rope(s.D, 1.0e6, st->max_seq, hc, hs);
    cudaError_t e = cudaMalloc(&st->d_cos, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&st->d_sin, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(st->d_cos, hc, n * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(st->d_sin, hs, n * sizeof(float), cudaMemcpyHostToDevice);
    delete[] hc;
    delete[] hs;
    if (e != cudaSuccess) return bail(MK_ERR_OOM);
  }
  if (cudaMalloc(&st->d_hop, st->hop_bytes) != cudaSuccess) return bail(MK_ERR_OOM);
  if (cudaMemset(st->d_hop, 0, st->hop_bytes) != cudaSuccess) return bail(MK_ERR_CUDA);
  if (cudaMalloc(&st->d_err, sizeof(int)) != cudaSuccess) return bail(MK_ERR_OOM);
  if (cudaMalloc(&st->d_tok, 2 * sizeof(int)) != cudaSuccess) return bail(MK_ERR_OOM);
  if (cudaMallocHost(&st->h_pinned, 2 * sizeof(int)) != cudaSuccess) return bail(MK_ERR_OOM);
  if (cudaDeviceSynchronize() != cudaSuccess) return bail(MK_ERR_CUDA);
  *out = st;
  return MK_OK;
}

// One cooperative launch of n_steps steps; asynchronous on `stream`.
int launch(State* st, const int* d_forced, int n_forced, int n_steps, int* d_out,
           float* d_logits, cudaStream_t stream) {
  if (st->tp_size > 1 && !st->tp_connected) return MK_ERR_INVALID_ARG;
  if (st->seq + (uint32_t)n_steps >= kSeqLimit) {
    // Peers write into this GPU's hop buffer whenever they run ahead, so a
    // tensor-parallel engine cannot clear it on its own.
    if (st->tp_size > 1) return MK_ERR_CAPACITY;
    // Tag sequence numbers are 24 bits: start over from clean buffers.
    MK_CUDA(cudaMemsetAsync(st->d_hop, 0, st->hop_bytes, stream));
    st->seq = 1;
  }
  mk::KParams P;
  P.w = st->d_wptr;
  P.kv = st->d_kv;
  P.rope_cos = st->d_cos;
  P.rope_sin = st->d_sin;
  P.hop = st->d_hop;
  P.err = st->d_err;
  P.forced = d_forced;
  P.n_forced = n_forced;
  P.n_steps = n_steps;
  P.out_tokens = d_out;
  P.logits = d_logits;
  P.pos0 = st->pos;
  P.seq0 = st->seq;
  P.max_seq = st->max_seq;
  P.ncta = st->ncta;
  P.nst = st->nst;
  P.issue_gap_ns = st->issue_gap_ns;
  P.timeout_ns = st->timeout_ns;
  P.debug_skip_cta = st->debug_skip_cta;
  P.trace = st->d_trace;
  P.trace_steps = st->d_trace ? st->trace_steps : 0;
  P.detail = st->d_detail;
  P.tp_rank = st->tp_rank;
  for (int j = 0; j < mk::kMaxTP; ++j) P.peer_hop[j] = st->peer_hop[j];
  MK_CUDA(cudaMemsetAsync(st->d_err, 0, sizeof(int), stream));
  void* args[] = {&P};
  // The two-level merge kernel once the launch reaches more chunks per head
  // than the threshold at which that merge starts to pay (see shapes.cuh).
  const int nc_last = mk::chunks_per_head<mk::ShapeD64>(st->pos + n_steps - 1);
  // Auto: the two-level instance only when the launch goes past
  // kMerge2MinChunks chunks per head.  Measured on B200 (512-token launch at
  // positions 128-639, whose last 127 steps have 5 chunks): the two-level
  // instance took ~30 us/token longer over the launch than the direct one.
  const bool m2 = st->merge_mode == 2 || (st->merge_mode == 0 && nc_last > mk::kMerge2MinChunks);
  const void* kern = m2 ? st->kernel_m2 : st->kernel;
  cudaError_t e = cudaLaunchCooperativeKernel(kern, dim3(st->ncta), dim3(mk::kThreads), args,
                                              st->smem, stream);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "megakernel: launch failed: %s\n", cudaGetErrorString(e));
    cudaGetLastError();
    return MK_ERR_LAUNCH;
  }
  st->seq += (uint32_t)n_steps;
  return MK_OK;
}

// Launch, wait, and fold the in-kernel error word into the status.
int run_sync(State* st, const int* d_forced, int n_forced, int n_steps, int* d_out,
             float* d_logits, cudaStream_t stream) {
  if (st->pos + n_steps > st->max_seq) return MK_ERR_CAPACITY;
  int rc = launch(st, d_forced, n_forced, n_steps, d_out, d_logits, stream);
  if (rc != MK_OK) return rc;
  MK_CUDA(cudaMemcpyAsync(st->h_pinned + 1, st->d_err, sizeof(int), cudaMemcpyDeviceToHost, stream));
  MK_CUDA(cudaStreamSynchronize(stream));
  if (st->h_pinned[1] != 0) return st->h_pinned[1];
  st->pos += n_steps;
  return MK_OK;
}

State* as_state(void* h) { return static_cast<State*>(h); }

int set_err(State* st, int rc) {
  if (st) st->last_error = rc;
  return rc;
}

template <class S>
void plan_bytes_t(int N, int p, long long* out) {
  const int nc = mk::chunks_per_head<S>(p);
  const int nitems = S::NKV * nc;
  for (int c = 0; c < N; ++c) {
    long long b = 0;
    for (int l = 0; l < S::L; ++l) {
      int r0, r1;
      mk::split_rows(S::QKV, N, c, mk::phase_rot(l, 0, N), r0, r1);
      b += 2LL * S::H * (r1 - r0);
      int ilo, ihi;
      mk::items_of_cta(c, l, nitems, N, ilo, ihi);
      for (int i = ilo; i < ihi; ++i) {
        int c0, c1;
        mk::chunk_range(p, nc, i % nc, c0, c1);
        const int te = c1 < p - 1 ? c1 : p - 1;
        if (te > c0) b += 2LL * 2 * S::D * (te - c0);
      }
      mk::split_rows(S::H, N, c, mk::phase_rot(l, 1, N), r0, r1);
      b += 2LL * S::Q * (r1 - r0);
      mk::split_rows(S::I, N, c, mk::phase_rot(l, 2, N), r0, r1);
      b += 2LL * 2 * S::H * (r1 - r0);
      mk::split_rows(S::H, N, c, mk::phase_rot(l, 3, N), r0, r1);
      b += 2LL * S::I * (r1 - r0);
    }
    int r0, r1;
    mk::split_rows(S::V, N, c, mk::phase_rot(S::L, 4, N), r0, r1);
    b += 2LL * S::H * (r1 - r0);
    out[c] = b;
  }
}

}  // namespace

namespace {
// Payload (low 32 bits) of n tagged words at src with a stride, as fp32.
__global__ void tp_slots_kernel(const uint64_t* src, int n, int stride, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __uint_as_float((uint32_t)src[(size_t)i * stride]);
}
template <int TP>
long long tp_slot_offset(int shape_id, int parity) {
  switch (shape_id) {
    case 0: return mk::HopLayout<mk::ShapeD64, TP>::X + (long long)parity * TP * mk::ShapeD64::H * mk::kHopSpread;
    case 2: return mk::HopLayout<mk::ShapeTiny, TP>::X + (long long)parity * TP * mk::ShapeTiny::H * mk::kHopSpread;
    default: return -1;
  }
}
}  // namespace

extern "C" {

void megakernel_default_options(mk_options* o) {
  if (!o) return;
  o->device = -1;
  o->shape_id = -1;
  o->max_seq = 0;
  o->num_ctas = 0;
  o->timeout_ns = 0;
  o->debug_skip_cta = -1;
}

int megakernel_init_ex(void* d_weights, const long long* offsets, int num_offsets,
                       const mk_options* opts, void** out_handle) {
  if (!out_handle) return MK_ERR_INVALID_ARG;
  *out_handle = nullptr;
  mk_options def;
  megakernel_default_options(&def);
  State* st = nullptr;
  const int rc = init_impl(d_weights, offsets, num_offsets, opts ? opts : &def, &st);
  if (rc == MK_OK) *out_handle = st;
  return rc;
}

void* megakernel_init(void* d_weights, long long* offsets, int num_offsets) {
  void* h = nullptr;
  const int rc = megakernel_init_ex(d_weights, offsets, num_offsets, nullptr, &h);
  if (rc != MK_OK) {
    std::fprintf(stderr, "megakernel_init: %s\n", megakernel_error_string(rc));
    return nullptr;
  }
  return h;
}

int megakernel_decode(void* handle, int input_token) {
  State* st = as_state(handle);
  if (!st) return -1;
  if (input_token < 0 || input_token >= st->vocab) { set_err(st, MK_ERR_INVALID_ARG); return -1; }
  if (cudaSetDevice(st->device) != cudaSuccess) { set_err(st, MK_ERR_CUDA); return -1; }
  st->h_pinned[0] = input_token;
  if (cudaMemcpyAsync(st->d_tok, st->h_pinned, sizeof(int), cudaMemcpyHostToDevice, st->stream) !=
      cudaSuccess) { set_err(st, MK_ERR_CUDA); return -1; }
  int rc = run_sync(st, st->d_tok, 1, 1, st->d_tok + 1, st->capture_logits ? st->d_logits : nullptr,
                    st->stream);
  if (rc == MK_OK &&
      (cudaMemcpyAsync(st->h_pinned, st->d_tok + 1, sizeof(int), cudaMemcpyDeviceToHost, st->stream) !=
           cudaSuccess ||
       cudaStreamSynchronize(st->stream) != cudaSuccess))
    rc = MK_ERR_CUDA;
  set_err(st, rc);
  return rc == MK_OK ? st->h_pinned[0] : -1;
}

void megakernel_reset(void* handle) {
  State* st = as_state(handle);
  if (!st) return;
  cudaSetDevice(st->device);
  cudaMemsetAsync(st->d_kv, 0, st->kv_bytes, st->stream);
  cudaStreamSynchronize(st->stream);
  st->pos = 0;
}

int megakernel_get_pos(void* handle) {
  State* st = as_state(handle);
  return st ? st->pos : -1;
}

void megakernel_free(void* handle) {
  State* st = as_state(handle);
  if (!st) return;
  cudaSetDevice(st->device);
  cudaStreamSynchronize(st->stream);
  free_state(st);
}

void megakernel_sync(void) { cudaDeviceSynchronize(); }

int megakernel_decode_n(void* handle, const int* d_tokens, int n_forced, int n_steps, int* d_out,
                        float* d_logits, void* stream) {
  State* st = as_state(handle);
  if (!st) return MK_ERR_INVALID_ARG;
  if (!d_tokens || !d_out || n_forced < 1 || n_steps < 1 || n_forced > n_steps)
    return set_err(st, MK_ERR_INVALID_ARG);
  if (cudaSetDevice(st->device) != cudaSuccess) return set_err(st, MK_ERR_CUDA);
  // NULL: the default stream, as the reference's calls use, so the launch is
  // ordered after the caller's earlier default-stream work on its buffers.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return set_err(st, run_sync(st, d_tokens, n_forced, n_steps, d_out, d_logits, s));
}

int megakernel_prefill(void* handle, const int* d_tokens, int n_tokens, int* d_next, void* stream);  // batch.cu

int megakernel_generate(void* handle, const int* prompt, int n_prompt, int n_gen, int* out) {
  State* st = as_state(handle);
  if (!st) return MK_ERR_INVALID_ARG;
  if (!prompt || !out || n_prompt < 1 || n_gen < 1) return set_err(st, MK_ERR_INVALID_ARG);
  for (int i = 0; i < n_prompt; ++i)
    if (prompt[i] < 0 || prompt[i] >= st->vocab) return set_err(st, MK_ERR_INVALID_ARG);
  if (cudaSetDevice(st->device) != cudaSuccess) return set_err(st, MK_ERR_CUDA);
  const int steps = n_prompt + n_gen - 1;
  if (st->pos + steps > st->max_seq) return set_err(st, MK_ERR_CAPACITY);
  // The graded shape prefills the prompt in parallel (64 positions per
  // batched tcgen05 step); other shapes feed it token by token.
  const bool parallel = st->shape_id == 0 && std::getenv("MK_SERIAL_PREFILL") == nullptr;
  int* d_in = nullptr;
  int* d_out = nullptr;
  int rc = MK_OK;
  if (cudaMallocAsync(&d_in, sizeof(int) * n_prompt, st->stream) != cudaSuccess ||
      cudaMallocAsync(&d_out, sizeof(int) * steps, st->stream) != cudaSuccess)
    rc = MK_ERR_OOM;
  if (rc == MK_OK && cudaMemcpyAsync(d_in, prompt, sizeof(int) * n_prompt, cudaMemcpyHostToDevice,
                                     st->stream) != cudaSuccess)
    rc = MK_ERR_CUDA;
  int* res = d_out + (n_prompt - 1);
  if (rc == MK_OK && parallel) {
    rc = megakernel_prefill(handle, d_in, n_prompt, res, st->stream);
    if (rc == MK_OK && n_gen > 1) rc = run_sync(st, res, 1, n_gen - 1, res + 1, nullptr, st->stream);
  } else if (rc == MK_OK) {
    rc = run_sync(st, d_in, n_prompt, steps, d_out, nullptr, st->stream);
  }
  if (rc == MK_OK &&
      (cudaMemcpyAsync(out, res, sizeof(int) * n_gen, cudaMemcpyDeviceToHost, st->stream) != cudaSuccess ||
       cudaStreamSynchronize(st->stream) != cudaSuccess))
    rc = MK_ERR_CUDA;
  if (d_in) cudaFreeAsync(d_in, st->stream);
  if (d_out) cudaFreeAsync(d_out, st->stream);
  cudaStreamSynchronize(st->stream);
  return set_err(st, rc);
}

int megakernel_set_logits_capture(void* handle, int enable) {
  State* st = as_state(handle);
  if (!st) return MK_ERR_INVALID_ARG;
  if (enable && !st->d_logits) {
    if (cudaSetDevice(st->device) != cudaSuccess) return set_err(st, MK_ERR_CUDA);
    if (cudaMalloc(&st->d_logits, sizeof(float) * st->vocab) != cudaSuccess)
      return set_err(st, MK_ERR_OOM);
    cudaMemset(st->d_logits, 0, sizeof(float) * st->vocab);
  }
  st->capture_logits = enable != 0;
  return MK_OK;
}

int megakernel_get_logits(void* handle, float* out) {
  State* st = as_state(handle);
  if (!st || !out || !st->d_logits) return MK_ERR_INVALID_ARG;
  if (cudaSetDevice(st->device) != cudaSuccess ||
      cudaMemcpy(out, st->d_logits, sizeof(float) * st->vocab, cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_err(st, MK_ERR_CUDA);
  return MK_OK;
}

int megakernel_set_pos(void* handle, int pos) {
  State* st = as_state(handle);
  if (!st) return MK_ERR_INVALID_ARG;
  if (pos < 0 || pos >= st->max_seq) return set_err(st, MK_ERR_CAPACITY);
  st->pos = pos;
  return MK_OK;
}

void* megakernel_kv_ptr(void* handle) {
  State* st = as_state(handle);
  return st ? st->d_kv : nullptr;
}
long long megakernel_kv_bytes(void* handle) {
  State* st = as_state(handle);
  return st ? (long long)st->kv_bytes : -1;
}
int megakernel_max_seq(void* handle) {
  State* st = as_state(handle);
  return st ? st->max_seq : -1;
}
int megakernel_shape_id(void* handle) {
  State* st = as_state(handle);
  return st ? st->shape_id : -1;
}
int megakernel_num_ctas(void* handle) {
  State* st = as_state(handle);
  return st ? st->ncta : -1;
}
int megakernel_set_merge_mode(void* handle, int mode) {
  State* st = as_state(handle);
  if (!st || mode < 0 || mode > 2) return MK_ERR_INVALID_ARG;
  // Tensor-parallel engines run only the instance with the two-level merge.
  if (st->tp_size > 1 && mode == 1) return set_err(st, MK_ERR_INVALID_ARG);
  st->merge_mode = mode;
  return MK_OK;
}

int megakernel_last_error(void* handle) {
  State* st = as_state(handle);
  return st ? st->last_error : MK_ERR_INVALID_ARG;
}

const char* megakernel_error_string(int code) {
  switch (code) {
    case MK_OK: return "ok";
    case MK_ERR_INVALID_ARG: return "invalid argument";
    case MK_ERR_CUDA: return "CUDA runtime error";
    case MK_ERR_TIMEOUT: return "in-kernel wait timed out";
    case MK_ERR_CAPACITY: return "KV capacity exceeded";
    case MK_ERR_SHAPE: return "offsets match no compiled model shape";
    case MK_ERR_LAUNCH: return "cooperative launch not possible";
    case MK_ERR_OOM: return "device allocation failed";
    default: return "unknown error";
  }
}

int megakernel_set_trace(void* handle, void* d_buf, int steps) {
  State* st = as_state(handle);
  if (!st || steps < 0 || (steps > 0 && !d_buf)) return MK_ERR_INVALID_ARG;
  // Compiled in only with -DMK_TRACE_POINTS=1 (profiling builds).
  if (!MK_TRACE_POINTS && steps > 0) return MK_ERR_INVALID_ARG;
  st->d_trace = steps > 0 ? static_cast<uint64_t*>(d_buf) : nullptr;
  st->trace_steps = steps;
  return MK_OK;
}

int megakernel_trace_points(void* handle) {
  State* st = as_state(handle);
  if (!st) return MK_ERR_INVALID_ARG;
  switch (st->shape_id) {
    case 0: return mk::Trace<mk::ShapeD64>::kPoints;
    case 1: return mk::Trace<mk::ShapeD128>::kPoints;
    default: return mk::Trace<mk::ShapeTiny>::kPoints;
  }
}

int megakernel_set_trace_detail(void* handle, void* d_buf) {
  State* st = as_state(handle);
  if (!st) return MK_ERR_INVALID_ARG;
  // The sub-phase stamps are compiled in only with -DMK_DETAIL_STAMPS=1 (they
  // cost 6 KB of instruction-cache-bound kernel code).
  if (!MK_DETAIL_STAMPS && d_buf != nullptr) return MK_ERR_INVALID_ARG;
  st->d_detail = static_cast<uint64_t*>(d_buf);
  return MK_OK;
}

int megakernel_tp_init(void* d_weights, const long long* offsets, int num_offsets,
                       const mk_options* opts, int tp_rank, int tp_size, void** out_handle) {
  if (!out_handle) return MK_ERR_INVALID_ARG;
  *out_handle = nullptr;
  if (tp_size < 2) return MK_ERR_INVALID_ARG;
  mk_options def;
  megakernel_default_options(&def);
  State* st = nullptr;
  const int rc = init_impl(d_weights, offsets, num_offsets, opts ? opts : &def, &st, tp_rank, tp_size);
  if (rc == MK_OK) *out_handle = st;
  return rc;
}

int megakernel_tp_ipc_handle(void* handle, void* out) {
  State* st = as_state(handle);
  if (!st || !out || st->tp_size < 2) return MK_ERR_INVALID_ARG;
  MK_CUDA(cudaSetDevice(st->device));
  cudaIpcMemHandle_t h;
  MK_CUDA(cudaIpcGetMemHandle(&h, st->d_hop));
  std::memcpy(out, &h, sizeof(h));
  return MK_OK;
}

int megakernel_tp_connect(void* handle, const void* handles) {
  State* st = as_state(handle);
  if (!st || !handles || st->tp_size < 2 || st->tp_connected) return MK_ERR_INVALID_ARG;
  MK_CUDA(cudaSetDevice(st->device));
  for (int j = 0; j < st->tp_size; ++j) {
    if (j == st->tp_rank) {
      st->peer_hop[j] = st->d_hop;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + (size_t)j * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      std::fprintf(stderr, "megakernel: cudaIpcOpenMemHandle(rank %d) failed: %s\n", j, cudaGetErrorString(e));
      cudaGetLastError();
      return MK_ERR_CUDA;
    }
    st->peer_hop[j] = static_cast<uint64_t*>(p);
    st->peer_opened[j] = true;
  }
  st->tp_connected = true;
  return MK_OK;
}


int megakernel_tp_exchange_slots(void* handle, float* d_out) {
  State* st = as_state(handle);
  if (!st || !d_out || st->tp_size < 2) return MK_ERR_INVALID_ARG;
  const ShapeInfo s = shape_info(st->shape_id);
  // The last layer (L - 1) of a step writes the slots of parity L & 1.
  const int parity = s.L & 1;
  long long off = -1;
  switch (st->tp_size) {
    case 2: off = tp_slot_offset<2>(st->shape_id, parity); break;
    case 4: off = tp_slot_offset<4>(st->shape_id, parity); break;
    case 8: off = tp_slot_offset<8>(st->shape_id, parity); break;
  }
  if (off < 0) return set_err(st, MK_ERR_INVALID_ARG);
  MK_CUDA(cudaSetDevice(st->device));
  const int n = st->tp_size * s.H;
  tp_slots_kernel<<<(n + 255) / 256, 256, 0, st->stream>>>(st->d_hop + off, n, mk::kHopSpread, d_out);
  MK_CUDA(cudaGetLastError());
  MK_CUDA(cudaStreamSynchronize(st->stream));
  return MK_OK;
}

int megakernel_tp_info(void* handle, int* rank, int* size) {
  State* st = as_state(handle);
  if (!st || !rank || !size) return MK_ERR_INVALID_ARG;
  *rank = st->tp_rank;
  *size = st->tp_size;
  return MK_OK;
}

int megakernel_infer_shape(const long long* offsets, int num_offsets) {
  return infer_shape(offsets, num_offsets);
}

int megakernel_rope_table(int head_dim, double theta, int positions, float* cos_out, float* sin_out) {
  if (head_dim <= 0 || (head_dim & 1) || positions <= 0 || !cos_out || !sin_out)
    return MK_ERR_INVALID_ARG;
  host_rope(head_dim, theta, positions, cos_out, sin_out);
  return MK_OK;
}

int megakernel_plan_bytes(int shape_id, int num_ctas, int pos, long long* bytes_per_cta) {
  if (num_ctas < 1 || num_ctas > mk::kMaxCtas || pos < 0 || !bytes_per_cta) return MK_ERR_INVALID_ARG;
  switch (shape_id) {
    case 0: plan_bytes_t<mk::ShapeD64>(num_ctas, pos, bytes_per_cta); return MK_OK;
    case 1: plan_bytes_t<mk::ShapeD128>(num_ctas, pos, bytes_per_cta); return MK_OK;
    case 2: plan_bytes_t<mk::ShapeTiny>(num_ctas, pos, bytes_per_cta); return MK_OK;
    default: return MK_ERR_SHAPE;
  }
}

}  // extern "C"

// The allocation-free entry point lives in its own file; it is compiled in
// this translation unit so both entry points launch the same kernel image.
#include "noalloc.cu"
#include "batch.cu"

// megakernel_decode_noalloc: the decode megakernel for callers that cannot
// allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at all: a runtime that
// owns every device allocation itself, an allocator-free embedded loader, or
// a plugin that must not change the process's device-memory footprint after
// start-up.  They can still hand us their own buffers (weights, KV cache,
// token arrays), but not the kernel's scratch: the tagged activation words
// the CTAs exchange, the error word, the weight-pointer table and the RoPE
// tables.  Here that scratch is one file-scope __device__ array of a fixed
// size, so the entry point allocates nothing.
//
// Limits and behaviour (documented in include/megakernel.h):
//   * graded shape only (head_dim 64, intermediate 2816);
//   * positions: pos + n_steps <= MK_NOALLOC_MAX_POS (2048) and <= kv_max_seq;
//   * the array lives on every GPU that loads this library until exit;
//   * the first call on a device sets that device up (symbol address, kernel
//     attributes, RoPE table upload with a blocking copy), so make the first
//     call before any stream capture;
//   * every call shares the array: calls that overlap on the GPU (two streams,
//     two host threads) race.  Each call clears the parts that must start at
//     zero (activation tags, error word) before it launches.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/megakernel.h"
#include "decode_kernel.cuh"

namespace {

using SNA = mk::ShapeD64;
constexpr int kMaxPos = MK_NOALLOC_MAX_POS;
constexpr int kMaxDevices = 64;
constexpr size_t kHopBytes = mk::HopLayout<SNA>::TOTAL * sizeof(uint64_t);
constexpr size_t kErrOff = kHopBytes;                                   // int
constexpr size_t kWtabOff = kErrOff + 256;                              // NOFF pointers
constexpr size_t kCosOff = kWtabOff + ((SNA::NOFF * 8 + 255) / 256) * 256;
constexpr size_t kRopeBytes = (size_t)kMaxPos * (SNA::D / 2) * sizeof(float);
constexpr size_t kSinOff = kCosOff + kRopeBytes;
constexpr size_t kScratchBytes = kSinOff + kRopeBytes;                  // ~0.87 MB
static_assert(kScratchBytes == MK_NOALLOC_SCRATCH_BYTES, "header and layout agree");

// The only scratch this entry point uses.  In host code `g_scratch` is a
// host-side stand-in, not a device address: the device address comes from
// cudaGetSymbolAddress at set-up.
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

struct DeviceSetup {
  bool done = false;
  unsigned char* base = nullptr;  // device address of g_scratch on this device
  int sms = 0;
  const void* kernel_m2 = nullptr;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_mutex;

// Once per device, with that device current.
int setup_device(int dev, DeviceSetup** out) {
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceSetup& s = g_setup[dev];
  if (!s.done) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return MK_ERR_CUDA;
    int coop = 0;
    if (cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess)
      return MK_ERR_CUDA;
    if (!coop || s.sms > mk::kMaxCtas) return MK_ERR_LAUNCH;
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(&mk::decode_kernel<SNA>),
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)mk::smem_bytes<SNA>()) != cudaSuccess)
      return MK_ERR_LAUNCH;
    // The two-level-merge instance (compiled in tp.cu), used once a call
    // goes past kMerge2MinChunks chunks per head, as the allocating path does.
    size_t words = 0;
    s.kernel_m2 = mk_tp::kernel(0, 1, true, &words);
    if (!s.kernel_m2 || words * sizeof(uint64_t) != kHopBytes ||
        cudaFuncSetAttribute(s.kernel_m2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)mk::smem_bytes<SNA>()) != cudaSuccess)
      return MK_ERR_LAUNCH;
    // RoPE tables from the allocating path's host_rope (one formula for both
    // entry points), staged through fixed host buffers and copied with
    // blocking copies.
    static float cos_table[kMaxPos * (SNA::D / 2)];
    static float sin_table[kMaxPos * (SNA::D / 2)];
    host_rope(SNA::D, 1.0e6, kMaxPos, cos_table, sin_table);
    if (cudaMemcpy(static_cast<unsigned char*>(p) + kCosOff, cos_table, kRopeBytes, cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(static_cast<unsigned char*>(p) + kSinOff, sin_table, kRopeBytes, cudaMemcpyHostToDevice) !=
            cudaSuccess)
      return MK_ERR_CUDA;
    s.base = static_cast<unsigned char*>(p);
    s.done = true;
  }
  *out = &s;
  return MK_OK;
}

}  // namespace

extern "C" int megakernel_decode_noalloc(const void* d_weights, const long long* offsets,
                                         int num_offsets, void* d_kv, int kv_max_seq, int pos,
                                         const int* d_tokens, int n_forced, int n_steps, int* d_out,
                                         float* d_logits, void* stream) {
  if (!d_weights || !offsets || !d_kv || !d_tokens || !d_out) return MK_ERR_INVALID_ARG;
  if (num_offsets != SNA::NOFF || megakernel_infer_shape(offsets, num_offsets) != 0) return MK_ERR_SHAPE;
  if (n_forced < 1 || n_steps < 1 || n_forced > n_steps || pos < 0) return MK_ERR_INVALID_ARG;
  if (pos + n_steps > kMaxPos || pos + n_steps > kv_max_seq) {
    std::fprintf(stderr, "megakernel_decode_noalloc: positions up to %d exceed the limit of %d "
                 "(static scratch) or the KV capacity %d\n", pos + n_steps, kMaxPos, kv_max_seq);
    return MK_ERR_CAPACITY;
  }
  // The kernel's bulk copies read weights and cached K/V at 16-byte
  // granularity: both buffers must start on a 16-byte boundary.
  if ((reinterpret_cast<uintptr_t>(d_weights) & 15) != 0 || (reinterpret_cast<uintptr_t>(d_kv) & 15) != 0)
    return MK_ERR_INVALID_ARG;
  for (int i = 0; i < num_offsets; ++i)
    if (offsets[i] < 0 || (offsets[i] & 15) != 0) return MK_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MK_ERR_CUDA;
  DeviceSetup* s = nullptr;
  int rc = setup_device(dev, &s);
  if (rc != MK_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // Weight pointers into the scratch table (pageable source: the copy is
  // staged before cudaMemcpyAsync returns, so `ptrs` may go out of scope).
  const __nv_bfloat16* ptrs[SNA::NOFF];
  for (int i = 0; i < num_offsets; ++i)
    ptrs[i] = reinterpret_cast<const __nv_bfloat16*>(static_cast<const char*>(d_weights) + offsets[i]);
  if (cudaMemcpyAsync(s->base + kWtabOff, ptrs, sizeof(ptrs), cudaMemcpyHostToDevice, st) != cudaSuccess)
    return MK_ERR_CUDA;
  // Start from clean activation tags and error word: the array still holds
  // the previous call's contents.
  if (cudaMemsetAsync(s->base, 0, kWtabOff, st) != cudaSuccess) return MK_ERR_CUDA;

  mk::KParams P{};
  P.w = reinterpret_cast<const __nv_bfloat16* const*>(s->base + kWtabOff);
  P.kv = static_cast<__nv_bfloat16*>(d_kv);
  P.rope_cos = reinterpret_cast<const float*>(s->base + kCosOff);
  P.rope_sin = reinterpret_cast<const float*>(s->base + kSinOff);
  P.hop = reinterpret_cast<uint64_t*>(s->base);
  P.err = reinterpret_cast<int*>(s->base + kErrOff);
  P.forced = d_tokens;
  P.n_forced = n_forced;
  P.n_steps = n_steps;
  P.out_tokens = d_out;
  P.logits = d_logits;
  P.pos0 = pos;
  P.seq0 = 1;
  P.max_seq = kv_max_seq;
  P.ncta = s->sms;
  P.nst = SNA::NST;
  P.issue_gap_ns = 0;
  P.timeout_ns = 1000000000LL;
  P.debug_skip_cta = -1;
  P.trace = nullptr;
  P.trace_steps = 0;
  P.detail = nullptr;
  void* args[] = {&P};
  const bool m2 = mk::chunks_per_head<SNA>(pos + n_steps - 1) > mk::kMerge2MinChunks;
  const void* kern = m2 ? s->kernel_m2 : reinterpret_cast<const void*>(&mk::decode_kernel<SNA>);
  if (cudaLaunchCooperativeKernel(kern, dim3(s->sms),
                                  dim3(mk::kThreads), args, mk::smem_bytes<SNA>(), st) != cudaSuccess) {
    cudaGetLastError();
    return MK_ERR_LAUNCH;
  }
  int err = 0;
  if (cudaMemcpyAsync(&err, P.err, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return MK_ERR_CUDA;
  return err;
}

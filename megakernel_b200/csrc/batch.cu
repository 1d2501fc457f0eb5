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

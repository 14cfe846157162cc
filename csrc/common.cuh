// Shared helpers for the memory-bound row kernels (norms, RoPE, residual, optimiser).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

// Row kernels: vector count per row -> (vectors per thread VEC, threads per block TH).
#define DMAD_ROW_DISPATCH(nvec, ...)                                        \
  [&] {                                                                     \
    if ((nvec) <= 128) { constexpr int VEC = 1, TH = 128; __VA_ARGS__(); }  \
    else if ((nvec) <= 256) { constexpr int VEC = 2, TH = 128; __VA_ARGS__(); } \
    else if ((nvec) <= 512) { constexpr int VEC = 2, TH = 256; __VA_ARGS__(); } \
    else if ((nvec) <= 768) { constexpr int VEC = 3, TH = 256; __VA_ARGS__(); } \
    else { constexpr int VEC = 4, TH = 256; __VA_ARGS__(); }                \
  }()

// Optional index guards (build with DMAD_BOUNDS_CHECK=1): a guarded access whose index is out of
// range records status code 6 (bounds) in the device status word and is skipped instead of faulting.
#ifdef DMAD_BOUNDS_CHECK
#define DMAD_GUARD(cond, status)                          \
  if (!(cond)) {                                         \
    if ((status) != nullptr) atomicCAS((status), 0, 6);  \
  } else
#else
#define DMAD_GUARD(cond, status)
#endif

namespace dmad {

struct alignas(16) bf16x8 {
  uint32_t w[4];
};

__device__ __forceinline__ void bf16x8_to_float(const bf16x8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(v.w[i] << 16);
    f[2 * i + 1] = __uint_as_float(v.w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint32_t f2_to_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ bf16x8 float_to_bf16x8(const float (&f)[8]) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.w[i] = f2_to_bf16x2(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum for blocks of up to 1024 threads; `red` must hold 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float u = k0 * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.f + tanhf(u));
}

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f;
  const float x2 = x * x;
  const float u = k0 * (x + 0.044715f * x2 * x);
  const float th = tanhf(u);
  const float du = k0 * (1.f + 3.f * 0.044715f * x2);
  return 0.5f * (1.f + th) + 0.5f * x * (1.f - th * th) * du;
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

}  // namespace dmad

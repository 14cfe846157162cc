// Timestep embedding kernels (sm_100a).
//
// The reference computes `sinusoidal_embedding_1d` in fp64 and then runs
// time_embedding = Linear(256, D) -> SiLU -> Linear(D, D) and
// time_projection = SiLU -> Linear(D, 6D) under fp32 autocast
// (train/wan/rcm/networks/wan2pt1.py:181-190, 590-591, 772-784).  M (the number
// of distinct timesteps) is tiny, so these are weight-bandwidth-bound:
//   sinusoid_kernel      : fp64 phases, cos half then sin half, fp32 output
//   small_linear_kernel  : y = act_in(x) W^T + b for M <= 16 rows; every warp
//                          streams one weight row once and dots it against all
//                          M input rows held in shared memory (fp32 math).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace dmad {
namespace {

__global__ void sinusoid_kernel(const float* __restrict__ t, float* __restrict__ out, int M, int dim, double max_period) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int half = dim / 2;
  if (i >= M * half) return;
  const int m = i / half, j = i % half;
  const double freq = pow(max_period, -(double)j / half);
  const double ph = (double)t[m] * freq;
  out[(int64_t)m * dim + j] = (float)cos(ph);
  out[(int64_t)m * dim + half + j] = (float)sin(ph);
}

constexpr int kMaxM = 16;
constexpr int kKChunk = 512;  // 16 x 512 fp32 = 32 KB of static shared memory

// grid.x: output columns / 8 (one warp per column); x: [M, K] fp32 contiguous.
__global__ void __launch_bounds__(256)
small_linear_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ w, const float* __restrict__ bias,
                    float* __restrict__ y, int M, int K, int N, int act_in) {
  __shared__ float xs[kMaxM * kKChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  float acc[kMaxM];
#pragma unroll
  for (int m = 0; m < kMaxM; ++m) acc[m] = 0.f;
  for (int k0 = 0; k0 < K; k0 += kKChunk) {
    const int kc = min(kKChunk, K - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < M * kc; i += blockDim.x) {
      const int m = i / kc, k = i % kc;
      float v = x[(int64_t)m * K + k0 + k];
      if (act_in == 1) v = silu(v);
      xs[m * kKChunk + k] = v;
    }
    __syncthreads();
    if (n < N) {
      const __nv_bfloat16* wr = w + (int64_t)n * K + k0;
      for (int k = lane * 8; k < kc; k += 256) {
        float wv[8];
        bf16x8_to_float(*reinterpret_cast<const bf16x8*>(wr + k), wv);
#pragma unroll
        for (int m = 0; m < kMaxM; ++m) {
          if (m < M) {
            const float* xr = xs + m * kKChunk + k;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[m] += wv[e] * xr[e];
          }
        }
      }
    }
  }
  if (n < N) {
#pragma unroll
    for (int m = 0; m < kMaxM; ++m) {
      if (m < M) {
        const float s = warp_sum(acc[m]);
        if (lane == 0) y[(int64_t)m * N + n] = s + (bias != nullptr ? bias[n] : 0.f);
      }
    }
  }
}

}  // namespace

void sinusoid_embed(const at::Tensor& t, at::Tensor& out, int64_t dim, double max_period) {
  TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() && out.is_contiguous(), "sinusoid: fp32 contiguous");
  const int M = t.numel();
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(t.device());
  const int n = M * (dim / 2);
  sinusoid_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(t.data_ptr<float>(),
                                                                                 out.data_ptr<float>(), M, (int)dim,
                                                                                 max_period);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// y[M, N] = act_in(x[M, K]) @ w[N, K]^T + bias; act_in: 0 identity, 1 SiLU.
void small_linear(const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> bias, at::Tensor& y,
                  int64_t act_in) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.dim() == 2, "x: fp32 [M, K]");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous() && w.dim() == 2, "w: bf16 [N, K]");
  const int M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && K % 8 == 0, "small_linear: K mismatch or K % 8 != 0");
  TORCH_CHECK(M <= kMaxM, "small_linear: at most 16 rows");
  TORCH_CHECK(y.scalar_type() == at::kFloat && y.is_contiguous() && y.size(0) == M && y.size(1) == N, "y: fp32 [M, N]");
  const float* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N, "bias: fp32 [N]");
    bp = bias->data_ptr<float>();
  }
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  small_linear_kernel<<<(N + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), bp, y.data_ptr<float>(), M, K, N,
      (int)act_in);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmad

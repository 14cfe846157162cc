// Frozen-gain spectral norm of a segmented bf16 weight, fused: the power iteration, the scaled weight
// and its gradient, reading the weight directly in bf16 (fp32 accumulation).
//
// Functional parity target: the reference's frozen-gain spectral norm on the critic / generator Linears
// (train/wan/rcm/models/t2v_model_distill_dmad.py:488-507 with torch's spectral_norm parametrization:
// one power iteration per training forward, sigma = u^T W v with u, v held constant, W * gain / sigma).
// A weight W [O, I] is split by rows into segments (the q / k / v parts of a fused projection), each with
// its own u (rows), v [I] and gain; segments whose norm is off (zero-initialised) pass through.
//
// Training forward, per segment s (rows R_s):
//   t_s = W_s^T u_s,  v_s = t_s / |t_s|,  r = W_s v_s,  sigma_s = |r|,  u_s = r / |r|,
//   W_eff = bf16(W * gain_s / sigma_s)
// (sigma_s = u_s^T W_s v_s exactly, since u_s = r / |r|).  Evaluation: r = W_s v_s with the stored v,
// sigma_s = u_s^T r.  Backward, with G = dL/dW_eff and c_s = sum over R_s of G o W:
//   dW = bf16(G * gain_s / sigma_s - (gain_s c_s / sigma_s^2) u_s v_s^T)
// Three reads of W and one write per training forward, two reads of G, one of W and one write per
// backward: six launches per Linear instead of about fifteen per segment.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace dmad {
namespace {

constexpr int kMaxSeg = 8;

struct SnSegs {
  int n;
  int off[kMaxSeg + 1];  // row offsets of the segments
  int on[kMaxSeg];       // 1 = spectrally normed
};

__device__ __forceinline__ int seg_of(const SnSegs& m, int row) {
  int s = 0;
  while (s + 1 < m.n && row >= m.off[s + 1]) ++s;
  return s;
}

// t[s, :] += W[r, :] u[r] over a chunk of rows (segment-aware), one 8-column vector per thread.
__global__ void sn_wtu_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int O, int I,
                              const float* __restrict__ u, float* __restrict__ t, SnSegs m, int rows) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 * 8 >= I) return;
  const int r0 = blockIdx.y * rows, r1 = min(O, r0 + rows);
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  int s = seg_of(m, r0);
  if (r1 <= m.off[s + 1]) {  // the whole chunk in one segment (the usual case): four rows of loads at a time
    if (!m.on[s]) return;
    int r = r0;
    for (; r + 4 <= r1; r += 4) {
      bf16x8 raw[4];
      float ur[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        raw[k] = reinterpret_cast<const bf16x8*>(w + (int64_t)(r + k) * ldw)[c8];
        ur[k] = u[r + k];
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float wv[8];
        bf16x8_to_float(raw[k], wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(wv[e], ur[k], acc[e]);
      }
    }
    for (; r < r1; ++r) {
      float wv[8];
      bf16x8_to_float(reinterpret_cast<const bf16x8*>(w + (int64_t)r * ldw)[c8], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wv[e], u[r], acc[e]);
    }
    float* dst = t + (int64_t)s * I + c8 * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) atomicAdd(dst + e, acc[e]);
    return;
  }
  auto flush = [&](int seg) {
    if (!m.on[seg]) return;
    float* dst = t + (int64_t)seg * I + c8 * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      atomicAdd(dst + e, acc[e]);
      acc[e] = 0.f;
    }
  };
  for (int r = r0; r < r1; ++r) {
    if (r >= m.off[s + 1]) {
      flush(s);
      ++s;
    }
    if (!m.on[s]) continue;
    float wv[8];
    bf16x8_to_float(reinterpret_cast<const bf16x8*>(w + (int64_t)r * ldw)[c8], wv);
    const float ur = u[r];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = fmaf(wv[e], ur, acc[e]);
  }
  flush(s);
}

__device__ float block_sum_all(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float x = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
  return warp_sum(x);
}

// v[s, :] = t[s, :] / max(|t[s, :]|, 1e-12), one block per segment.
__global__ void sn_normalize_kernel(const float* __restrict__ t, float* __restrict__ v, int I, SnSegs m) {
  __shared__ float red[32];
  const int s = blockIdx.x;
  if (!m.on[s]) return;
  const float* ts = t + (int64_t)s * I;
  float ss = 0.f;
  for (int c = threadIdx.x; c < I; c += blockDim.x) ss = fmaf(ts[c], ts[c], ss);
  const float inv = 1.f / fmaxf(sqrtf(block_sum_all(ss, red)), 1e-12f);
  for (int c = threadIdx.x; c < I; c += blockDim.x) v[(int64_t)s * I + c] = ts[c] * inv;
}

// r[row] = W[row, :] . v[seg(row), :], one warp per row.
__global__ void sn_wv_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int O, int I,
                             const float* __restrict__ v, float* __restrict__ r, SnSegs m) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < O; row += gridDim.x * warps) {
    const int s = seg_of(m, row);
    if (!m.on[s]) {
      if (lane == 0) r[row] = 0.f;
      continue;
    }
    const bf16x8* wr = reinterpret_cast<const bf16x8*>(w + (int64_t)row * ldw);
    const float4* vs = reinterpret_cast<const float4*>(v + (int64_t)s * I);
    float acc = 0.f;
    for (int c8 = lane; c8 * 8 < I; c8 += 32) {
      float wv[8];
      bf16x8_to_float(wr[c8], wv);
      const float4 a = vs[2 * c8], b = vs[2 * c8 + 1];
      acc = fmaf(wv[0], a.x, acc);
      acc = fmaf(wv[1], a.y, acc);
      acc = fmaf(wv[2], a.z, acc);
      acc = fmaf(wv[3], a.w, acc);
      acc = fmaf(wv[4], b.x, acc);
      acc = fmaf(wv[5], b.y, acc);
      acc = fmaf(wv[6], b.z, acc);
      acc = fmaf(wv[7], b.w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) r[row] = acc;
  }
}

// Per segment: sigma (training: |r|, u <- r / max(|r|, 1e-12); evaluation: u . r), and the per-row
// scale gain / sigma (1 for segments without the norm).  One block per segment.
__global__ void sn_finish_kernel(const float* __restrict__ r, float* __restrict__ u, const float* __restrict__ gain,
                                 float* __restrict__ scale, float* __restrict__ sigma, SnSegs m, int train) {
  __shared__ float red[32];
  const int s = blockIdx.x;
  const int r0 = m.off[s], r1 = m.off[s + 1];
  if (!m.on[s]) {
    for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) scale[i] = 1.f;
    if (threadIdx.x == 0) sigma[s] = 1.f;
    return;
  }
  float acc = 0.f;
  for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) acc = fmaf(r[i], train ? r[i] : u[i], acc);
  acc = block_sum_all(acc, red);
  float sg;
  if (train) {
    const float nrm = sqrtf(acc);
    const float inv = 1.f / fmaxf(nrm, 1e-12f);
    sg = nrm * nrm * inv;  // u . r with u = r / max(|r|, eps)
    for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) u[i] = r[i] * inv;
  } else {
    sg = acc;
  }
  const float sc = gain[s] / sg;
  for (int i = r0 + threadIdx.x; i < r1; i += blockDim.x) scale[i] = sc;
  if (threadIdx.x == 0) sigma[s] = sg;
}

// out[r, :] = bf16(W[r, :] * scale[r]).
__global__ void sn_scale_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, __nv_bfloat16* __restrict__ out,
                                int O, int I, const float* __restrict__ scale) {
  const int nv = I / 8;
  const int64_t n = (int64_t)O * nv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / nv), c8 = (int)(i % nv);
    float wv[8];
    bf16x8_to_float(reinterpret_cast<const bf16x8*>(w + (int64_t)row * ldw)[c8], wv);
    const float sc = scale[row];
#pragma unroll
    for (int e = 0; e < 8; ++e) wv[e] *= sc;
    reinterpret_cast<bf16x8*>(out + (int64_t)row * I)[c8] = float_to_bf16x8(wv);
  }
}

// c[s] += sum over the rows of segment s of G o W, one warp per row.
__global__ void sn_gw_kernel(const __nv_bfloat16* __restrict__ g, int64_t ldg, const __nv_bfloat16* __restrict__ w,
                             int64_t ldw, int O, int I, float* __restrict__ c, SnSegs m) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  int cur = -1;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < O; row += gridDim.x * warps) {
    const int s = seg_of(m, row);
    if (!m.on[s]) continue;
    if (s != cur) {
      if (cur >= 0) {
        acc = warp_sum(acc);
        if (lane == 0) atomicAdd(c + cur, acc);
      }
      acc = 0.f;
      cur = s;
    }
    const bf16x8* gr = reinterpret_cast<const bf16x8*>(g + (int64_t)row * ldg);
    const bf16x8* wr = reinterpret_cast<const bf16x8*>(w + (int64_t)row * ldw);
    for (int c8 = lane; c8 * 8 < I; c8 += 32) {
      float gv[8], wv[8];
      bf16x8_to_float(gr[c8], gv);
      bf16x8_to_float(wr[c8], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(gv[e], wv[e], acc);
    }
  }
  if (cur >= 0) {
    acc = warp_sum(acc);
    if (lane == 0) atomicAdd(c + cur, acc);
  }
}

// dW[r, :] = bf16(scale[r] G[r, :] - (gain_s c_s / sigma_s^2) u[r] v[s, :]).
__global__ void sn_dw_kernel(const __nv_bfloat16* __restrict__ g, int64_t ldg, __nv_bfloat16* __restrict__ dw, int O,
                             int I, const float* __restrict__ scale, const float* __restrict__ u,
                             const float* __restrict__ v, const float* __restrict__ gain,
                             const float* __restrict__ sigma, const float* __restrict__ c, SnSegs m) {
  const int nv = I / 8;
  const int64_t n = (int64_t)O * nv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / nv), c8 = (int)(i % nv);
    const int s = seg_of(m, row);
    float gv[8];
    bf16x8_to_float(reinterpret_cast<const bf16x8*>(g + (int64_t)row * ldg)[c8], gv);
    const float sc = scale[row];
    if (m.on[s]) {
      const float b = gain[s] * c[s] / (sigma[s] * sigma[s]) * u[row];
      const float4 va = reinterpret_cast<const float4*>(v + (int64_t)s * I)[2 * c8];
      const float4 vb = reinterpret_cast<const float4*>(v + (int64_t)s * I)[2 * c8 + 1];
      gv[0] = sc * gv[0] - b * va.x;
      gv[1] = sc * gv[1] - b * va.y;
      gv[2] = sc * gv[2] - b * va.z;
      gv[3] = sc * gv[3] - b * va.w;
      gv[4] = sc * gv[4] - b * vb.x;
      gv[5] = sc * gv[5] - b * vb.y;
      gv[6] = sc * gv[6] - b * vb.z;
      gv[7] = sc * gv[7] - b * vb.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) gv[e] *= sc;
    }
    reinterpret_cast<bf16x8*>(dw + (int64_t)row * I)[c8] = float_to_bf16x8(gv);
  }
}

SnSegs make_segs(const std::vector<int64_t>& offsets, const std::vector<int64_t>& on, int64_t O) {
  TORCH_CHECK(offsets.size() >= 2 && (int)offsets.size() <= kMaxSeg + 1, "spectral norm: 1 to 8 segments");
  TORCH_CHECK(on.size() + 1 == offsets.size(), "spectral norm: one flag per segment");
  TORCH_CHECK(offsets.front() == 0 && offsets.back() == O, "spectral norm: segments must cover the rows");
  SnSegs m{};
  m.n = (int)on.size();
  for (size_t i = 0; i < offsets.size(); ++i) m.off[i] = (int)offsets[i];
  for (size_t i = 0; i < on.size(); ++i) {
    TORCH_CHECK(offsets[i + 1] > offsets[i], "spectral norm: empty segment");
    m.on[i] = on[i] ? 1 : 0;
  }
  return m;
}

void check_weight(const at::Tensor& w, const char* name) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.dim() == 2, name, " must be a CUDA bf16 matrix");
  TORCH_CHECK(w.stride(1) == 1 && w.stride(0) % 8 == 0 && w.size(1) % 8 == 0, name,
              " must have contiguous rows, a row stride and a width that are multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(w.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}

void check_f32(const at::Tensor& t, int64_t n, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() == n, name,
              " must be a contiguous CUDA fp32 tensor of ", n, " elements");
}

}  // namespace

// Spectrally normed weight of `w` [O, I] bf16: returns bf16(W * gain_s / sigma_s) and writes the per-row
// scale [O] and sigma [nseg].  `u` [O] and `v` [nseg, I] (fp32) hold the power-iteration state and are
// updated in place when `train`; `gain` [nseg] fp32.  `offsets`: nseg + 1 row offsets, `on`: per segment.
at::Tensor sn_weight_fwd(const at::Tensor& w, at::Tensor& u, at::Tensor& v, const at::Tensor& gain,
                         at::Tensor& scale, at::Tensor& sigma, std::vector<int64_t> offsets, std::vector<int64_t> on,
                         bool train) {
  check_weight(w, "w");
  const int64_t O = w.size(0), I = w.size(1);
  SnSegs m = make_segs(offsets, on, O);
  check_f32(u, O, "u");
  check_f32(v, m.n * I, "v");
  check_f32(gain, m.n, "gain");
  check_f32(scale, O, "scale");
  check_f32(sigma, m.n, "sigma");
  c10::cuda::CUDAGuard guard(w.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto f32 = w.options().dtype(at::kFloat);
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  if (train) {
    at::Tensor t = at::zeros({m.n, I}, f32);
    const int threads = 64, rows = 32;  // 8-column vectors per block x rows per chunk
    dim3 grid((unsigned)((I / 8 + threads - 1) / threads), (unsigned)((O + rows - 1) / rows));
    sn_wtu_kernel<<<grid, threads, 0, stream>>>(wp, w.stride(0), (int)O, (int)I, u.data_ptr<float>(),
                                                t.data_ptr<float>(), m, rows);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    sn_normalize_kernel<<<m.n, 256, 0, stream>>>(t.data_ptr<float>(), v.data_ptr<float>(), (int)I, m);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  at::Tensor r = at::empty({O}, f32);
  const int blocks_r = (int)std::min<int64_t>((O + 7) / 8, 148 * 8);
  sn_wv_kernel<<<blocks_r, 256, 0, stream>>>(wp, w.stride(0), (int)O, (int)I, v.data_ptr<float>(), r.data_ptr<float>(),
                                             m);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  sn_finish_kernel<<<m.n, 256, 0, stream>>>(r.data_ptr<float>(), u.data_ptr<float>(), gain.data_ptr<float>(),
                                            scale.data_ptr<float>(), sigma.data_ptr<float>(), m, train ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  at::Tensor out = at::empty({O, I}, w.options());
  const int64_t n = O * (I / 8);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  sn_scale_kernel<<<blocks, 256, 0, stream>>>(wp, w.stride(0), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                              (int)O, (int)I, scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Gradient of sn_weight_fwd's output with respect to w, from g = dL/dW_eff [O, I] bf16 and the u, v,
// scale, sigma of that forward.
at::Tensor sn_weight_bwd(const at::Tensor& g, const at::Tensor& w, const at::Tensor& u, const at::Tensor& v,
                         const at::Tensor& gain, const at::Tensor& scale, const at::Tensor& sigma,
                         std::vector<int64_t> offsets, std::vector<int64_t> on) {
  check_weight(g, "g");
  check_weight(w, "w");
  TORCH_CHECK(g.sizes() == w.sizes(), "g and w shapes differ");
  const int64_t O = w.size(0), I = w.size(1);
  SnSegs m = make_segs(offsets, on, O);
  check_f32(u, O, "u");
  check_f32(v, m.n * I, "v");
  check_f32(gain, m.n, "gain");
  check_f32(scale, O, "scale");
  check_f32(sigma, m.n, "sigma");
  c10::cuda::CUDAGuard guard(w.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  at::Tensor c = at::zeros({m.n}, w.options().dtype(at::kFloat));
  const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(g.data_ptr());
  const int blocks_r = (int)std::min<int64_t>((O + 7) / 8, 148 * 4);
  sn_gw_kernel<<<blocks_r, 256, 0, stream>>>(gp, g.stride(0), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                             w.stride(0), (int)O, (int)I, c.data_ptr<float>(), m);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  at::Tensor dw = at::empty({O, I}, w.options());
  const int64_t n = O * (I / 8);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  sn_dw_kernel<<<blocks, 256, 0, stream>>>(gp, g.stride(0), reinterpret_cast<__nv_bfloat16*>(dw.data_ptr()), (int)O,
                                           (int)I, scale.data_ptr<float>(), u.data_ptr<float>(), v.data_ptr<float>(),
                                           gain.data_ptr<float>(), sigma.data_ptr<float>(), c.data_ptr<float>(), m);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dw;
}

}  // namespace dmad

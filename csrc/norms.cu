// Row-wise memory-bound kernels of the DiT blocks (sm_100a, bf16 activations,
// fp32 math):
//   * ln_mod_fwd / ln_mod_bwd : LayerNorm or RMSNorm followed by a per-group
//     affine y = n * A + C.  Covers the adaLN "norm(x) * (1 + scale) + shift" of
//     the Wan and H3 blocks (train/wan/rcm/networks/wan2pt1.py:419-436,
//     dmad_h3/lowmem.py:436-458), the affine cross-attention LayerNorm and the
//     non-affine RMSNorm of the H3 critic heads.  The group of a row is
//     row / rows_per_group, or an explicit int32 index per row (H3 packed rows).
//     The backward optionally fuses a residual-gradient addend and the backward
//     of the gated residual that produced its input.
//   * gate_res_fwd : out = x + y * gate[g]  (gated residual, wan2pt1.py:426-436)
//   * qk_norm_rope_fwd / _bwd : RMSNorm over the full hidden size of q and k
//     (wan2pt1.py:193-211) followed by interleaved rotary embedding per head
//     (rcm/utils/rope.py:36-70) from cos/sin tables.
//   * gelu_tanh_fwd / _bwd.
#include <torch/extension.h>
#include <type_traits>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace dmad {
namespace {


// Row kernels are instantiated for the number of 8-element vectors each thread
// holds (VEC) and the block size (TH); rows of up to 8192 columns are covered.

struct ModSpec {
  const float* a;   // [G, D] fp32 (row stride a_sg; 0 = shared row) or nullptr
  const float* c;   // [G, D] fp32 or nullptr
  int64_t a_sg, c_sg;
  float a_add;      // A = a_add + a[g]
  int rows_per_group;
  const int* gidx;  // optional explicit group per row
};

__device__ __forceinline__ int row_group(const ModSpec& m, int64_t r) {
  return m.gidx != nullptr ? m.gidx[r] : (int)(r / m.rows_per_group);
}

template <int kMaxVec, int kTh>
__global__ void __launch_bounds__(kTh)
ln_mod_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, __nv_bfloat16* __restrict__ y, int64_t sy,
                  float* __restrict__ mean_out, float* __restrict__ rstd_out, ModSpec m, int64_t R, int D, float eps,
                  bool rms) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  if (r >= R) return;
  const int nvec = D >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + r * sx);
  float v[kMaxVec][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kTh;
    if (c < nvec) {
      bf16x8_to_float(xr[c], v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[i][e];
    }
  }
  const float mu = rms ? 0.f : block_sum(s, red) / D;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kTh;
    if (c < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i][e] - mu;
        ss += d * d;
      }
    }
  }
  const float rstd = rsqrtf(block_sum(ss, red) / D + eps);
  const int g = row_group(m, r);
  const float* ar = m.a != nullptr ? m.a + (int64_t)g * m.a_sg : nullptr;
  const float* cr = m.c != nullptr ? m.c + (int64_t)g * m.c_sg : nullptr;
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + r * sy);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kTh;
    if (c < nvec) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int col = c * 8 + e;
        const float A = m.a_add + (ar != nullptr ? ar[col] : 0.f);
        const float C = cr != nullptr ? cr[col] : 0.f;
        o[e] = (v[i][e] - mu) * rstd * A + C;
      }
      yr[c] = float_to_bf16x8(o);
    }
  }
  if (threadIdx.x == 0) {
    if (mean_out != nullptr) mean_out[r] = mu;
    rstd_out[r] = rstd;
  }
}

// Forward for rows of up to 1536 columns: one warp per row, every lane holding kV 8-column vectors of
// the row (all loads issued up front), shuffle reductions only (no shared memory, no block barriers).
// Each warp walks kRows consecutive rows; the modulation rows A / C (fp32, shared by the rows of a
// group) are re-read per row from L1 rather than held in registers, which keeps two CTAs per SM.
template <int kV, int kRows>
__global__ void __launch_bounds__(256, 2)
ln_mod_fwd_warp_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, __nv_bfloat16* __restrict__ y, int64_t sy,
                       float* __restrict__ mean_out, float* __restrict__ rstd_out, ModSpec m, int64_t R, int D,
                       float eps, bool rms) {
  const int lane = threadIdx.x & 31;
  const int64_t r0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kRows;
  const int nvec = D >> 3;
#pragma unroll 1
  for (int rr = 0; rr < kRows; ++rr) {
    const int64_t r = r0 + rr;
    if (r >= R) return;
    const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + r * sx);
    float v[kV][8];
    {
      bf16x8 raw[kV];
#pragma unroll
      for (int i = 0; i < kV; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) raw[i] = xr[c];
      }
#pragma unroll
      for (int i = 0; i < kV; ++i) {
        const int c = lane + 32 * i;
        if (c < nvec) bf16x8_to_float(raw[i], v[i]);
      }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
#pragma unroll
        for (int e = 0; e < 8; ++e) s += v[i][e];
      }
    }
    const float mu = rms ? 0.f : warp_sum(s) / D;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = v[i][e] - mu;
          ss += d * d;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / D + eps);
    const int g = row_group(m, r);
    const float* ar = m.a != nullptr ? m.a + (int64_t)g * m.a_sg : nullptr;
    const float* cr = m.c != nullptr ? m.c + (int64_t)g * m.c_sg : nullptr;
    bf16x8* yr = reinterpret_cast<bf16x8*>(y + r * sy);
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int c = lane + 32 * i;
      if (c < nvec) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; e += 4) {
          const float4 av = ar != nullptr ? __ldg(reinterpret_cast<const float4*>(ar + c * 8 + e))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 cv = cr != nullptr ? __ldg(reinterpret_cast<const float4*>(cr + c * 8 + e))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
          o[e] = (v[i][e] - mu) * rstd * (m.a_add + av.x) + cv.x;
          o[e + 1] = (v[i][e + 1] - mu) * rstd * (m.a_add + av.y) + cv.y;
          o[e + 2] = (v[i][e + 2] - mu) * rstd * (m.a_add + av.z) + cv.z;
          o[e + 3] = (v[i][e + 3] - mu) * rstd * (m.a_add + av.w) + cv.w;
        }
        yr[c] = float_to_bf16x8(o);
      }
    }
    if (lane == 0) {
      if (mean_out != nullptr) mean_out[r] = mu;
      rstd_out[r] = rstd;
    }
  }
}

// Backward arguments (the kernels follow).  Optional fusions:
//   dres   : dx_total = LN_bwd(dy) + dres
//   gate/yg: the input of the norm was out = xg + yg * gate[g]; additionally
//            write dyg = dx_total * gate and accumulate dgate += dx_total * yg.
struct LnBwdArgs {
  const __nv_bfloat16* dy;
  int64_t sdy;
  const __nv_bfloat16* x;
  int64_t sx;
  const float* mean;
  const float* rstd;
  __nv_bfloat16* dx;
  int64_t sdx;
  const __nv_bfloat16* dres;
  int64_t sdres;
  float* da;  // [G, D] accum (row stride D) or nullptr
  float* dc;
  // gated-residual fusion
  const float* gate;
  int64_t gate_sg;
  const __nv_bfloat16* yg;
  int64_t syg;
  __nv_bfloat16* dyg;
  int64_t sdyg;
  float* dgate;  // [G, D] accum
  int64_t R;
  int D;
  bool rms;
  int rows_per_block;
};

// Two-pass backward.  Pass 1, one warp per row: the row statistics mean(dn) and mean(dn * n) of
// dn = dy * A (no block barriers, two CTAs of 8 rows per SM).  Pass 2, one thread per 8-column vector
// (column tiles of 256 vectors) over a tile of consecutive rows per block: dx (plus the optional
// residual-gradient and gated-residual fusions) from those statistics, with the column sums dA, dC
// (and dgate) accumulated in registers over the tile and flushed once per tile and group.  A one-pass
// kernel with two block reductions per row was latency-bound; this reads x and dy twice but keeps
// four rows of loads in flight per thread.
__global__ void __launch_bounds__(256, 2)
ln_bwd_stats_kernel(LnBwdArgs p, ModSpec m, float2* __restrict__ stats) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= p.R) return;
  const int nvec = p.D >> 3;
  const float mu = p.rms ? 0.f : p.mean[r];
  const float rstd = p.rstd[r];
  const int g = row_group(m, r);
  const float* ar = m.a != nullptr ? m.a + (int64_t)g * m.a_sg : nullptr;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(p.x + r * p.sx);
  const bf16x8* dyr = reinterpret_cast<const bf16x8*>(p.dy + r * p.sdy);
  float s1 = 0.f, s2 = 0.f;
#pragma unroll 4
  for (int c = lane; c < nvec; c += 32) {
    float xv[8], gv[8];
    bf16x8_to_float(xr[c], xv);
    bf16x8_to_float(dyr[c], gv);
#pragma unroll
    for (int e = 0; e < 8; e += 4) {
      const float4 av = ar != nullptr ? __ldg(reinterpret_cast<const float4*>(ar + c * 8 + e))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
      const float aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float n = (xv[e + k] - mu) * rstd;
        const float dn = gv[e + k] * (m.a_add + aa[k]);
        s1 += dn;
        s2 = fmaf(dn, n, s2);
      }
    }
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) stats[r] = make_float2(p.rms ? 0.f : s1 / p.D, s2 / p.D);
}

template <int kChunk>
__global__ void __launch_bounds__(256)
ln_bwd_apply_kernel(LnBwdArgs p, ModSpec m, const float2* __restrict__ stats) {
  const int nvec = p.D >> 3;
  const int c = blockIdx.y * 256 + threadIdx.x;  // column tiles of 256 vectors (2048 columns)
  if (c >= nvec) return;
  const int64_t r0 = (int64_t)blockIdx.x * p.rows_per_block;
  const int64_t r1 = min(p.R, r0 + p.rows_per_block);
  const bool has_gate = p.gate != nullptr;
  float acc_a[8], acc_c[8], acc_g[8], A[8], Gt[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc_a[e] = acc_c[e] = acc_g[e] = A[e] = Gt[e] = 0.f;
  int cur = -1;
  auto flush = [&]() {
    if (cur < 0) return;
    const int64_t base = (int64_t)cur * p.D + c * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (p.da != nullptr) atomicAdd(p.da + base + e, acc_a[e]);
      if (p.dc != nullptr) atomicAdd(p.dc + base + e, acc_c[e]);
      if (has_gate && p.dgate != nullptr) atomicAdd(p.dgate + base + e, acc_g[e]);
      acc_a[e] = acc_c[e] = acc_g[e] = 0.f;
    }
  };
  for (int64_t rb = r0; rb < r1; rb += kChunk) {
    // loads of the chunk's rows first, then the arithmetic row by row
    bf16x8 xraw[kChunk], dyraw[kChunk], rraw[kChunk], yraw[kChunk];
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      const int64_t r = rb + k;
      if (r < r1) {
        xraw[k] = reinterpret_cast<const bf16x8*>(p.x + r * p.sx)[c];
        dyraw[k] = reinterpret_cast<const bf16x8*>(p.dy + r * p.sdy)[c];
        if (p.dres != nullptr) rraw[k] = reinterpret_cast<const bf16x8*>(p.dres + r * p.sdres)[c];
        if (has_gate) yraw[k] = reinterpret_cast<const bf16x8*>(p.yg + r * p.syg)[c];
      }
    }
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      const int64_t r = rb + k;
      if (r >= r1) break;
      const int g = row_group(m, r);
      if (g != cur) {
        flush();
        cur = g;
        const float* ar = m.a != nullptr ? m.a + (int64_t)g * m.a_sg + c * 8 : nullptr;
        const float* gr = has_gate ? p.gate + (int64_t)g * p.gate_sg + c * 8 : nullptr;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          A[e] = m.a_add + (ar != nullptr ? ar[e] : 0.f);
          Gt[e] = gr != nullptr ? gr[e] : 0.f;
        }
      }
      const float mu = p.rms ? 0.f : p.mean[r];
      const float rstd = p.rstd[r];
      const float2 st = stats[r];
      float xv[8], gv[8], o[8];
      bf16x8_to_float(xraw[k], xv);
      bf16x8_to_float(dyraw[k], gv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float n = (xv[e] - mu) * rstd;
        const float dn = gv[e] * A[e];
        acc_a[e] = fmaf(gv[e], n, acc_a[e]);
        acc_c[e] += gv[e];
        o[e] = rstd * (dn - st.x - n * st.y);
      }
      if (p.dres != nullptr) {
        float rv[8];
        bf16x8_to_float(rraw[k], rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] += rv[e];
      }
      reinterpret_cast<bf16x8*>(p.dx + r * p.sdx)[c] = float_to_bf16x8(o);
      if (has_gate) {
        float yv[8], d[8];
        bf16x8_to_float(yraw[k], yv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          d[e] = o[e] * Gt[e];
          acc_g[e] = fmaf(o[e], yv[e], acc_g[e]);
        }
        reinterpret_cast<bf16x8*>(p.dyg + r * p.sdyg)[c] = float_to_bf16x8(d);
      }
    }
  }
  flush();
}

__global__ void gate_res_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, const __nv_bfloat16* __restrict__ y,
                                    int64_t sy, __nv_bfloat16* __restrict__ out, int64_t so, ModSpec m, int64_t R,
                                    int D) {
  const int nvec = D >> 3;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= R * nvec) return;
  const int64_t r = idx / nvec;
  const int c = idx % nvec;
  const int g = row_group(m, r);
  float xv[8], yv[8], o[8];
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(x + r * sx)[c], xv);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(y + r * sy)[c], yv);
  const float* ar = m.a != nullptr ? m.a + (int64_t)g * m.a_sg : nullptr;
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = xv[e] + yv[e] * (m.a_add + (ar != nullptr ? ar[c * 8 + e] : 0.f));
  reinterpret_cast<bf16x8*>(out + r * so)[c] = float_to_bf16x8(o);
}

// Gated-residual backward: dy = dout * gate[g], dgate[g] += sum_rows dout * y.  One thread per 8-column
// vector (column tiles of 256 vectors) over a tile of consecutive rows, the loads of four rows issued
// before their arithmetic; the column sums stay in registers and are flushed once per tile and group.
template <int kChunk>
__global__ void __launch_bounds__(256)
gate_res_bwd_kernel(const __nv_bfloat16* __restrict__ dout, int64_t sdo, const __nv_bfloat16* __restrict__ y, int64_t sy,
                    __nv_bfloat16* __restrict__ dy, int64_t sdy, float* __restrict__ dgate, ModSpec m, int64_t R, int D,
                    int rows_per_block) {
  const int nvec = D >> 3;
  const int c = blockIdx.y * 256 + threadIdx.x;
  if (c >= nvec) return;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block, r1 = min(R, r0 + rows_per_block);
  float acc[8], Gt[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = Gt[e] = 0.f;
  int cur = -1;
  auto flush = [&]() {
    if (cur < 0 || dgate == nullptr) return;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      atomicAdd(dgate + (int64_t)cur * D + c * 8 + e, acc[e]);
      acc[e] = 0.f;
    }
  };
  for (int64_t rb = r0; rb < r1; rb += kChunk) {
    bf16x8 graw[kChunk], yraw[kChunk];
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      if (rb + k < r1) {
        graw[k] = reinterpret_cast<const bf16x8*>(dout + (rb + k) * sdo)[c];
        yraw[k] = reinterpret_cast<const bf16x8*>(y + (rb + k) * sy)[c];
      }
    }
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      const int64_t r = rb + k;
      if (r >= r1) break;
      const int g = row_group(m, r);
      if (g != cur) {
        flush();
        cur = g;
        const float* ar = m.a + (int64_t)g * m.a_sg + c * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) Gt[e] = ar[e];
      }
      float gv[8], yv[8], o[8];
      bf16x8_to_float(graw[k], gv);
      bf16x8_to_float(yraw[k], yv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        o[e] = gv[e] * Gt[e];
        acc[e] = fmaf(gv[e], yv[e], acc[e]);
      }
      reinterpret_cast<bf16x8*>(dy + r * sdy)[c] = float_to_bf16x8(o);
    }
  }
  flush();
}

// ------------------------------------------------------------------ q/k RMSNorm + RoPE
// src: q at column 0, k at column D of each row (row stride ss); writes q/k
// into dst (row stride sd, q at 0, k at D).  cos/sin: [Lrope, hd/2] fp32,
// row r uses table row (r % Lrope).  hd = head dim (128), heads = D / hd.
template <int kMaxVec, int kTh>
__global__ void __launch_bounds__(kTh)
qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ src, int64_t ss, __nv_bfloat16* __restrict__ dst, int64_t sd,
                        const float* __restrict__ wq, const float* __restrict__ wk, const float* __restrict__ cosT,
                        const float* __restrict__ sinT, float* __restrict__ rstd_q, float* __restrict__ rstd_k,
                        int64_t R, int D, int hd, int Lrope, float eps) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const int which = blockIdx.y;  // 0 = q, 1 = k
  const int nvec = D >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(src + r * ss + which * D);
  const float* w = which == 0 ? wq : wk;
  float v[kMaxVec][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kTh;
    if (c < nvec) {
      bf16x8_to_float(xr[c], v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[i][e] * v[i][e];
    }
  }
  const float rstd = rsqrtf(block_sum(s, red) / D + eps);
  const int64_t tr = (r % Lrope) * (hd >> 1);
  bf16x8* yr = reinterpret_cast<bf16x8*>(dst + r * sd + which * D);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kTh;
    if (c < nvec) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const int col = c * 8 + e;
        const float a0 = v[i][e] * rstd * w[col];
        const float a1 = v[i][e + 1] * rstd * w[col + 1];
        const int pi = (col % hd) >> 1;
        const float cs = cosT[tr + pi], sn = sinT[tr + pi];
        o[e] = a0 * cs - a1 * sn;
        o[e + 1] = a1 * cs + a0 * sn;
      }
      yr[c] = float_to_bf16x8(o);
    }
  }
  if (threadIdx.x == 0) (which == 0 ? rstd_q : rstd_k)[r] = rstd;
}

// Forward for rows of up to 2048 columns: one warp per row and per q / k (blockIdx.y), every lane holding
// kV 8-column vectors (all loads issued up front), a shuffle reduction for the RMS, the rotation angles
// and norm weights read as vectors.  Needs contiguous 16-byte aligned tables [L, hd / 2] and weights.
template <int kV>
__global__ void __launch_bounds__(256, 2)
qk_norm_rope_fwd_warp_kernel(const __nv_bfloat16* __restrict__ src, int64_t ss, __nv_bfloat16* __restrict__ dst,
                             int64_t sd, const float* __restrict__ wq, const float* __restrict__ wk,
                             const float* __restrict__ cosT, const float* __restrict__ sinT, float* __restrict__ rstd_q,
                             float* __restrict__ rstd_k, int64_t R, int D, int hd, int Lrope, float eps, bool hd_pow2) {
  const int lane = threadIdx.x & 31;
  const int which = blockIdx.y;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= R) return;
  const int nvec = D >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(src + r * ss + which * D);
  const float* w = which == 0 ? wq : wk;
  float v[kV][8];
  {
    bf16x8 raw[kV];
#pragma unroll
    for (int i = 0; i < kV; ++i)
      if (lane + 32 * i < nvec) raw[i] = xr[lane + 32 * i];
#pragma unroll
    for (int i = 0; i < kV; ++i)
      if (lane + 32 * i < nvec) bf16x8_to_float(raw[i], v[i]);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kV; ++i)
    if (lane + 32 * i < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[i][e], v[i][e], s);
    }
  const float rstd = rsqrtf(warp_sum(s) / D + eps);
  const float* cr = cosT + (int64_t)((int)r % Lrope) * (hd >> 1);
  const float* sr = sinT + (cr - cosT);
  bf16x8* yr = reinterpret_cast<bf16x8*>(dst + r * sd + which * D);
#pragma unroll
  for (int i = 0; i < kV; ++i) {
    const int c = lane + 32 * i;
    if (c < nvec) {
      const int pi = (hd_pow2 ? ((c * 8) & (hd - 1)) : ((c * 8) % hd)) >> 1;
      const float4 cs4 = *reinterpret_cast<const float4*>(cr + pi), sn4 = *reinterpret_cast<const float4*>(sr + pi);
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + c * 8));
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + c * 8 + 4));
      const float cs[4] = {cs4.x, cs4.y, cs4.z, cs4.w}, sn[4] = {sn4.x, sn4.y, sn4.z, sn4.w};
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float a0 = v[i][e] * rstd * wv[e];
        const float a1 = v[i][e + 1] * rstd * wv[e + 1];
        o[e] = a0 * cs[e >> 1] - a1 * sn[e >> 1];
        o[e + 1] = a1 * cs[e >> 1] + a0 * sn[e >> 1];
      }
      yr[c] = float_to_bf16x8(o);
    }
  }
  if (lane == 0) (which == 0 ? rstd_q : rstd_k)[r] = rstd;
}

// Backward: g (grad of the rotated output, q at col 0 / k at col D, row stride sg)
// -> dx (grad of the pre-norm input, row stride sdx); dw accumulates (fp32 [D]).
struct QkBwd {
  const __nv_bfloat16* g[2];  // gq, gk
  int64_t sg[2];
  const __nv_bfloat16* src;
  int64_t ss;
  __nv_bfloat16* dx;
  int64_t sdx;
  const float* w[2];
  const float* cosT;
  const float* sinT;
  const float* rstd[2];
  float* dw[2];
  int64_t R;
  int D, hd, Lrope, rows_per_block;
  bool hd_pow2;
};

// Pass 1, one warp per row and per q / k (blockIdx.y): mean(dn * n) of dn = rot^-1(g) * w, n = x * rstd.
__global__ void __launch_bounds__(256, 2) qk_bwd_stats_kernel(QkBwd p, float* __restrict__ stats) {
  const int which = blockIdx.y, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= p.R) return;
  const int nvec = p.D >> 3;
  const float rstd = p.rstd[which][r];
  const float* cr = p.cosT + (int64_t)((int)r % p.Lrope) * (p.hd >> 1);
  const float* sr = p.sinT + (cr - p.cosT);
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(p.src + r * p.ss + which * p.D);
  const bf16x8* gr = reinterpret_cast<const bf16x8*>(p.g[which] + r * p.sg[which]);
  const float* w = p.w[which];
  float s2 = 0.f;
#pragma unroll 4
  for (int c = lane; c < nvec; c += 32) {
    float xv[8], gv[8];
    bf16x8_to_float(xr[c], xv);
    bf16x8_to_float(gr[c], gv);
    // the vector's four rotation angles: table entries [pi, pi + 4) of the row (hd a multiple of 8)
    const int pi = (p.hd_pow2 ? ((c * 8) & (p.hd - 1)) : ((c * 8) % p.hd)) >> 1;
    const float4 cs4 = *reinterpret_cast<const float4*>(cr + pi), sn4 = *reinterpret_cast<const float4*>(sr + pi);
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + c * 8)), w1 = __ldg(reinterpret_cast<const float4*>(w + c * 8 + 4));
    const float cs[4] = {cs4.x, cs4.y, cs4.z, cs4.w}, sn[4] = {sn4.x, sn4.y, sn4.z, sn4.w};
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float da0 = gv[e] * cs[e >> 1] + gv[e + 1] * sn[e >> 1];  // inverse rotation of the output gradient
      const float da1 = -gv[e] * sn[e >> 1] + gv[e + 1] * cs[e >> 1];
      s2 = fmaf(da0 * wv[e], xv[e] * rstd, s2);
      s2 = fmaf(da1 * wv[e + 1], xv[e + 1] * rstd, s2);
    }
  }
  s2 = warp_sum(s2);
  if (lane == 0) stats[which * p.R + r] = s2 / p.D;
}

// Pass 2: dx = rstd (dn - n mean(dn n)) and dw += sum_rows rot^-1(g) * n, one thread per 8-column vector
// (column tiles of 256 vectors, blockIdx.z = q / k) over a tile of rows, four rows of loads at a time.
template <int kChunk>
__global__ void __launch_bounds__(256) qk_bwd_apply_kernel(QkBwd p, const float* __restrict__ stats) {
  const int which = blockIdx.z;
  const int nvec = p.D >> 3;
  const int c = blockIdx.y * 256 + threadIdx.x;
  if (c >= nvec) return;
  const int64_t r0 = (int64_t)blockIdx.x * p.rows_per_block, r1 = min(p.R, r0 + p.rows_per_block);
  const float* w = p.w[which];
  float W[8], acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    W[e] = w[c * 8 + e];
    acc[e] = 0.f;
  }
  const int pi0 = ((c * 8) % p.hd) >> 1;  // a vector never straddles a head (hd is a multiple of 8)
  int rot = (int)(r0 % p.Lrope);           // rotation-table row of the current row, advanced row by row
  for (int64_t rb = r0; rb < r1; rb += kChunk) {
    bf16x8 xraw[kChunk], graw[kChunk];
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      if (rb + k < r1) {
        xraw[k] = reinterpret_cast<const bf16x8*>(p.src + (rb + k) * p.ss + which * p.D)[c];
        graw[k] = reinterpret_cast<const bf16x8*>(p.g[which] + (rb + k) * p.sg[which])[c];
      }
    }
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
      const int64_t r = rb + k;
      if (r >= r1) break;
      const float rstd = p.rstd[which][r];
      const float mdnn = stats[which * p.R + r];
      const int64_t tr = (int64_t)rot * (p.hd >> 1) + pi0;
      if (++rot == p.Lrope) rot = 0;
      const float4 cs4 = *reinterpret_cast<const float4*>(p.cosT + tr);
      const float4 sn4 = *reinterpret_cast<const float4*>(p.sinT + tr);
      const float csv[4] = {cs4.x, cs4.y, cs4.z, cs4.w}, snv[4] = {sn4.x, sn4.y, sn4.z, sn4.w};
      float xv[8], gv[8], o[8];
      bf16x8_to_float(xraw[k], xv);
      bf16x8_to_float(graw[k], gv);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float cs = csv[e >> 1], sn = snv[e >> 1];
        const float da0 = gv[e] * cs + gv[e + 1] * sn;
        const float da1 = -gv[e] * sn + gv[e + 1] * cs;
        const float n0 = xv[e] * rstd, n1 = xv[e + 1] * rstd;
        acc[e] = fmaf(da0, n0, acc[e]);
        acc[e + 1] = fmaf(da1, n1, acc[e + 1]);
        o[e] = rstd * (da0 * W[e] - n0 * mdnn);
        o[e + 1] = rstd * (da1 * W[e + 1] - n1 * mdnn);
      }
      reinterpret_cast<bf16x8*>(p.dx + r * p.sdx + which * p.D)[c] = float_to_bf16x8(o);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) atomicAdd(p.dw[which] + c * 8 + e, acc[e]);
}

// Standalone interleaved RoPE on [R, H, hd] rows (forward sign +1, backward -1).
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, int64_t sx, __nv_bfloat16* __restrict__ y, int64_t sy,
                            const float* __restrict__ cosT, const float* __restrict__ sinT, int64_t R, int D, int hd,
                            int Lrope, float sign) {
  const int nvec = D >> 3;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= R * nvec) return;
  const int64_t r = idx / nvec;
  const int c = idx % nvec;
  const int64_t tr = (r % Lrope) * (hd >> 1);
  float v[8], o[8];
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(x + r * sx)[c], v);
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const int pi = ((c * 8 + e) % hd) >> 1;
    const float cs = cosT[tr + pi], sn = sign * sinT[tr + pi];
    o[e] = v[e] * cs - v[e + 1] * sn;
    o[e + 1] = v[e + 1] * cs + v[e] * sn;
  }
  reinterpret_cast<bf16x8*>(y + r * sy)[c] = float_to_bf16x8(o);
}

__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t nvec) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nvec) return;
  float v[8];
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(x)[i], v);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = gelu_tanh(v[e]);
  reinterpret_cast<bf16x8*>(y)[i] = float_to_bf16x8(v);
}

__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ dx, int64_t nvec) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nvec) return;
  float gv[8], xv[8];
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(g)[i], gv);
  bf16x8_to_float(reinterpret_cast<const bf16x8*>(x)[i], xv);
#pragma unroll
  for (int e = 0; e < 8; ++e) gv[e] *= gelu_tanh_grad(xv[e]);
  reinterpret_cast<bf16x8*>(dx)[i] = float_to_bf16x8(gv);
}

void check_rows(const at::Tensor& t, const char* name, int64_t D) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be CUDA bf16");
  TORCH_CHECK(t.dim() == 2 && t.size(1) == D && t.stride(1) == 1, name, " must be [R, D] with contiguous rows");
  TORCH_CHECK(t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name,
              " rows must be 16-byte aligned");
}

ModSpec make_mod(const c10::optional<at::Tensor>& a, const c10::optional<at::Tensor>& c, double a_add,
                 int64_t rows_per_group, const c10::optional<at::Tensor>& gidx, int64_t D) {
  ModSpec m;
  m.a = nullptr;
  m.c = nullptr;
  m.a_sg = m.c_sg = 0;
  if (a.has_value() && a->defined()) {
    TORCH_CHECK(a->scalar_type() == at::kFloat && a->dim() == 2 && a->size(1) == D && a->stride(1) == 1,
                "modulation A must be fp32 [G, D]");
    m.a = a->data_ptr<float>();
    m.a_sg = a->size(0) == 1 ? 0 : a->stride(0);
  }
  if (c.has_value() && c->defined()) {
    TORCH_CHECK(c->scalar_type() == at::kFloat && c->dim() == 2 && c->size(1) == D && c->stride(1) == 1,
                "modulation C must be fp32 [G, D]");
    m.c = c->data_ptr<float>();
    m.c_sg = c->size(0) == 1 ? 0 : c->stride(0);
  }
  m.a_add = (float)a_add;
  m.rows_per_group = (int)std::max<int64_t>(1, rows_per_group);
  m.gidx = nullptr;
  if (gidx.has_value() && gidx->defined()) {
    TORCH_CHECK(gidx->scalar_type() == at::kInt && gidx->is_contiguous(), "group index must be int32");
    m.gidx = gidx->data_ptr<int>();
  }
  return m;
}

}  // namespace

void ln_mod_fwd(const at::Tensor& x, at::Tensor& y, c10::optional<at::Tensor> mean, at::Tensor& rstd,
                c10::optional<at::Tensor> a, c10::optional<at::Tensor> c, double a_add, int64_t rows_per_group,
                c10::optional<at::Tensor> gidx, double eps, bool rms) {
  const int64_t D = x.size(1), R = x.size(0);
  TORCH_CHECK(D % 8 == 0 && D <= 8192, "ln_mod: D must be a multiple of 8 and <= 8192");
  check_rows(x, "x", D);
  check_rows(y, "y", D);
  c10::cuda::CUDAGuard guard(x.device());
  ModSpec m = make_mod(a, c, a_add, rows_per_group, gidx, D);
  float* mp = (mean.has_value() && mean->defined()) ? mean->data_ptr<float>() : nullptr;
  TORCH_CHECK(rms || mp != nullptr, "LayerNorm needs a mean buffer");
  if (R == 0) return;
  const auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  auto stream = at::cuda::getCurrentCUDAStream();
  // the modulation rows are read as float4: the warp kernel needs them 16-byte aligned
  const bool mod_aligned = (m.a == nullptr || (reinterpret_cast<uintptr_t>(m.a) % 16 == 0 && m.a_sg % 4 == 0)) &&
                           (m.c == nullptr || (reinterpret_cast<uintptr_t>(m.c) % 16 == 0 && m.c_sg % 4 == 0));
  if (D <= 1536 && mod_aligned) {
    constexpr int kRows = 4;
    const int64_t warps = (R + kRows - 1) / kRows;
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    auto launch = [&](auto kv) {
      constexpr int V = decltype(kv)::value;
      ln_mod_fwd_warp_kernel<V, kRows><<<blocks, 256, 0, stream>>>(xp, x.stride(0), yp, y.stride(0), mp,
                                                                   rstd.data_ptr<float>(), m, R, (int)D, (float)eps, rms);
    };
    const int nv = (int)((D / 8 + 31) / 32);
    if (nv <= 2) launch(std::integral_constant<int, 2>{});
    else if (nv <= 4) launch(std::integral_constant<int, 4>{});
    else launch(std::integral_constant<int, 6>{});
  } else {
    DMAD_ROW_DISPATCH(D / 8, [&] {
      ln_mod_fwd_kernel<VEC, TH><<<(unsigned)R, TH, 0, stream>>>(xp, x.stride(0), yp, y.stride(0), mp,
                                                                  rstd.data_ptr<float>(), m, R, (int)D, (float)eps, rms);
    });
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Rows per block of the tiled backward kernels: about two blocks per SM (one wave) over row tiles x
// column tiles, a multiple of their four-row load chunk.
static int row_tile(int64_t R, int64_t ctiles, int device) {
  static int sms = 0;
  if (sms == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const int64_t want = std::max<int64_t>(1, 2 * sms / ctiles);
  return (int)std::max<int64_t>(4, ((R + want - 1) / want + 3) / 4 * 4);
}

void ln_mod_bwd(const at::Tensor& dy, const at::Tensor& x, c10::optional<at::Tensor> mean, const at::Tensor& rstd,
                c10::optional<at::Tensor> a, double a_add, int64_t rows_per_group, c10::optional<at::Tensor> gidx,
                bool rms, at::Tensor& dx, c10::optional<at::Tensor> dres, c10::optional<at::Tensor> da,
                c10::optional<at::Tensor> dc, c10::optional<at::Tensor> gate, c10::optional<at::Tensor> yg,
                c10::optional<at::Tensor> dyg, c10::optional<at::Tensor> dgate) {
  const int64_t D = x.size(1), R = x.size(0);
  check_rows(dy, "dy", D);
  check_rows(x, "x", D);
  check_rows(dx, "dx", D);
  c10::cuda::CUDAGuard guard(x.device());
  // the statistics pass reads the modulation rows as float4: an unaligned view is copied first
  if (a.has_value() && a->defined() && a->dim() == 2 && a->size(0) > 1 &&
      ((reinterpret_cast<uintptr_t>(a->data_ptr()) & 15) != 0 || a->stride(0) % 4 != 0))
    a = a->contiguous().clone(at::MemoryFormat::Contiguous);
  else if (a.has_value() && a->defined() && (reinterpret_cast<uintptr_t>(a->data_ptr()) & 15) != 0)
    a = a->clone(at::MemoryFormat::Contiguous);
  ModSpec m = make_mod(a, c10::nullopt, a_add, rows_per_group, gidx, D);
  LnBwdArgs p{};
  p.dy = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  p.sdy = dy.stride(0);
  p.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  p.sx = x.stride(0);
  p.mean = (mean.has_value() && mean->defined()) ? mean->data_ptr<float>() : nullptr;
  p.rstd = rstd.data_ptr<float>();
  p.dx = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  p.sdx = dx.stride(0);
  if (dres.has_value() && dres->defined()) {
    check_rows(*dres, "dres", D);
    p.dres = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
    p.sdres = dres->stride(0);
  }
  auto acc_ptr = [&](const c10::optional<at::Tensor>& t) -> float* {
    if (!(t.has_value() && t->defined())) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->size(-1) == D, "accumulator must be fp32 [G, D]");
    return t->data_ptr<float>();
  };
  p.da = acc_ptr(da);
  p.dc = acc_ptr(dc);
  if (gate.has_value() && gate->defined()) {
    TORCH_CHECK(gate->scalar_type() == at::kFloat && gate->stride(1) == 1, "gate must be fp32 [G, D]");
    p.gate = gate->data_ptr<float>();
    p.gate_sg = gate->size(0) == 1 ? 0 : gate->stride(0);
    TORCH_CHECK(yg.has_value() && dyg.has_value() && dgate.has_value(), "gate fusion needs yg, dyg, dgate");
    check_rows(*yg, "yg", D);
    check_rows(*dyg, "dyg", D);
    p.yg = reinterpret_cast<const __nv_bfloat16*>(yg->data_ptr());
    p.syg = yg->stride(0);
    p.dyg = reinterpret_cast<__nv_bfloat16*>(dyg->data_ptr());
    p.sdyg = dyg->stride(0);
    p.dgate = acc_ptr(dgate);
  }
  p.R = R;
  p.D = (int)D;
  p.rms = rms;
  if (R == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  // two passes: row statistics, then dx and the column sums by row tiles
  at::Tensor stats = at::empty({R, 2}, x.options().dtype(at::kFloat));
  float2* sp = reinterpret_cast<float2*>(stats.data_ptr<float>());
  ln_bwd_stats_kernel<<<(unsigned)((R + 7) / 8), 256, 0, stream>>>(p, m, sp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t nvec = D / 8, ctiles = (nvec + 255) / 256;
  p.rows_per_block = row_tile(R, ctiles, x.get_device());
  const dim3 grid((unsigned)((R + p.rows_per_block - 1) / p.rows_per_block), (unsigned)ctiles);
  const int th = (int)std::min<int64_t>(256, (nvec + 31) / 32 * 32);
  ln_bwd_apply_kernel<4><<<grid, th, 0, stream>>>(p, m, sp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gate_res_fwd(const at::Tensor& x, const at::Tensor& y, at::Tensor& out, c10::optional<at::Tensor> gate,
                  int64_t rows_per_group, c10::optional<at::Tensor> gidx) {
  const int64_t D = x.size(1), R = x.size(0);
  check_rows(x, "x", D);
  check_rows(y, "y", D);
  check_rows(out, "out", D);
  c10::cuda::CUDAGuard guard(x.device());
  const bool has_gate = gate.has_value() && gate->defined();
  ModSpec m = make_mod(gate, c10::nullopt, has_gate ? 0.0 : 1.0, rows_per_group, gidx, D);
  const int64_t n = R * (D / 8);
  if (n == 0) return;
  gate_res_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), m, R, (int)D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gate_res_bwd(const at::Tensor& dout, const at::Tensor& y, at::Tensor& dy, const at::Tensor& gate,
                  at::Tensor& dgate, int64_t rows_per_group, c10::optional<at::Tensor> gidx) {
  const int64_t D = y.size(1), R = y.size(0);
  check_rows(dout, "dout", D);
  check_rows(y, "y", D);
  check_rows(dy, "dy", D);
  TORCH_CHECK(dgate.scalar_type() == at::kFloat && dgate.is_contiguous() && dgate.size(-1) == D, "dgate fp32 [G, D]");
  c10::cuda::CUDAGuard guard(y.device());
  ModSpec m = make_mod(gate, c10::nullopt, 0.0, rows_per_group, gidx, D);
  if (R == 0) return;
  const int64_t nvec = D / 8, ctiles = (nvec + 255) / 256;
  const int rpb = row_tile(R, ctiles, y.get_device());
  const dim3 grid((unsigned)((R + rpb - 1) / rpb), (unsigned)ctiles);
  const int th = (int)std::min<int64_t>(256, (nvec + 31) / 32 * 32);
  gate_res_bwd_kernel<4><<<grid, th, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0),
      reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()), dy.stride(0), dgate.data_ptr<float>(), m, R, (int)D, rpb);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope_fwd(const at::Tensor& src, at::Tensor& dst, const at::Tensor& wq, const at::Tensor& wk,
                      const at::Tensor& cosT, const at::Tensor& sinT, at::Tensor& rstd_q, at::Tensor& rstd_k,
                      int64_t D, int64_t hd, double eps) {
  TORCH_CHECK(src.dim() == 2 && src.size(1) >= 2 * D && src.stride(1) == 1, "src must be [R, >=2D]");
  TORCH_CHECK(dst.dim() == 2 && dst.size(1) >= 2 * D && dst.stride(1) == 1, "dst must be [R, >=2D]");
  TORCH_CHECK(src.stride(0) % 8 == 0 && dst.stride(0) % 8 == 0 && D % 8 == 0 && D <= 8192 && D % hd == 0, "bad layout");
  TORCH_CHECK(wq.scalar_type() == at::kFloat && wk.scalar_type() == at::kFloat, "norm weights must be fp32");
  TORCH_CHECK(cosT.is_contiguous() && sinT.is_contiguous() && cosT.size(1) == hd / 2, "rope tables must be [L, hd/2]");
  const int64_t R = src.size(0);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  const bool vec_ok = D <= 2048 && hd % 8 == 0 && D % hd == 0 && cosT.is_contiguous() && sinT.is_contiguous() &&
                      cosT.size(1) == hd / 2 && (reinterpret_cast<uintptr_t>(cosT.data_ptr()) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(sinT.data_ptr()) & 15) == 0 && wq.is_contiguous() &&
                      wk.is_contiguous() && (reinterpret_cast<uintptr_t>(wq.data_ptr()) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(wk.data_ptr()) & 15) == 0;
  if (vec_ok) {
    const int nvec = (int)(D / 8);
    const dim3 wgrid((unsigned)((R + 7) / 8), 2);
    auto launch = [&](auto kv) {
      qk_norm_rope_fwd_warp_kernel<decltype(kv)::value><<<wgrid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0),
          reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), dst.stride(0), wq.data_ptr<float>(), wk.data_ptr<float>(),
          cosT.data_ptr<float>(), sinT.data_ptr<float>(), rstd_q.data_ptr<float>(), rstd_k.data_ptr<float>(), R,
          (int)D, (int)hd, (int)cosT.size(0), (float)eps, (hd & (hd - 1)) == 0);
    };
    if (nvec <= 64)
      launch(std::integral_constant<int, 2>{});
    else if (nvec <= 128)
      launch(std::integral_constant<int, 4>{});
    else if (nvec <= 192)
      launch(std::integral_constant<int, 6>{});
    else
      launch(std::integral_constant<int, 8>{});
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid((unsigned)R, 2);
  DMAD_ROW_DISPATCH(D / 8, [&] {
    qk_norm_rope_fwd_kernel<VEC, TH><<<grid, TH, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0),
        reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), dst.stride(0), wq.data_ptr<float>(), wk.data_ptr<float>(),
        cosT.data_ptr<float>(), sinT.data_ptr<float>(), rstd_q.data_ptr<float>(), rstd_k.data_ptr<float>(), R,
        (int)D, (int)hd, (int)cosT.size(0), (float)eps);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope_bwd(const at::Tensor& gq, const at::Tensor& gk, const at::Tensor& src, at::Tensor& dx,
                      const at::Tensor& wq, const at::Tensor& wk, const at::Tensor& cosT, const at::Tensor& sinT,
                      const at::Tensor& rstd_q, const at::Tensor& rstd_k, at::Tensor& dwq, at::Tensor& dwk, int64_t D,
                      int64_t hd) {
  TORCH_CHECK(gq.stride(-1) == 1 && gk.stride(-1) == 1 && dx.stride(1) == 1, "contiguous rows required");
  const int64_t R = src.size(0);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  TORCH_CHECK(hd % 8 == 0 && D % hd == 0, "head dim must be a multiple of 8 dividing D");
  QkBwd p{};
  p.g[0] = reinterpret_cast<const __nv_bfloat16*>(gq.data_ptr());
  p.g[1] = reinterpret_cast<const __nv_bfloat16*>(gk.data_ptr());
  p.sg[0] = gq.stride(0);
  p.sg[1] = gk.stride(0);
  p.src = reinterpret_cast<const __nv_bfloat16*>(src.data_ptr());
  p.ss = src.stride(0);
  p.dx = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  p.sdx = dx.stride(0);
  p.w[0] = wq.data_ptr<float>();
  p.w[1] = wk.data_ptr<float>();
  p.cosT = cosT.data_ptr<float>();
  p.sinT = sinT.data_ptr<float>();
  p.rstd[0] = rstd_q.data_ptr<float>();
  p.rstd[1] = rstd_k.data_ptr<float>();
  p.dw[0] = dwq.data_ptr<float>();
  p.dw[1] = dwk.data_ptr<float>();
  p.R = R;
  p.D = (int)D;
  p.hd = (int)hd;
  p.hd_pow2 = (hd & (hd - 1)) == 0;
  p.Lrope = (int)cosT.size(0);
  TORCH_CHECK(cosT.is_contiguous() && sinT.is_contiguous() && cosT.size(1) == hd / 2 &&
                  (reinterpret_cast<uintptr_t>(cosT.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sinT.data_ptr()) & 15) == 0,
              "rotation tables must be contiguous 16-byte aligned fp32 [L, hd / 2]");
  TORCH_CHECK(wq.is_contiguous() && wk.is_contiguous() && (reinterpret_cast<uintptr_t>(wq.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(wk.data_ptr()) & 15) == 0,
              "norm weights must be contiguous and 16-byte aligned");
  auto stream = at::cuda::getCurrentCUDAStream();
  at::Tensor stats = at::empty({2, R}, src.options().dtype(at::kFloat));
  qk_bwd_stats_kernel<<<dim3((unsigned)((R + 7) / 8), 2), 256, 0, stream>>>(p, stats.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t nvec = D / 8, ctiles = (nvec + 255) / 256;
  p.rows_per_block = row_tile(R, 2 * ctiles, src.get_device());
  const dim3 grid((unsigned)((R + p.rows_per_block - 1) / p.rows_per_block), (unsigned)ctiles, 2);
  const int th = (int)std::min<int64_t>(256, (nvec + 31) / 32 * 32);
  qk_bwd_apply_kernel<4><<<grid, th, 0, stream>>>(p, stats.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_apply(const at::Tensor& x, at::Tensor& y, const at::Tensor& cosT, const at::Tensor& sinT, int64_t hd,
                bool inverse) {
  const int64_t R = x.size(0), D = x.size(1);
  check_rows(x, "x", D);
  check_rows(y, "y", D);
  const int64_t n = R * (D / 8);
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
      y.stride(0), cosT.data_ptr<float>(), sinT.data_ptr<float>(), R, (int)D, (int)hd, (int)cosT.size(0),
      inverse ? -1.f : 1.f);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_fwd(const at::Tensor& x, at::Tensor& y) {
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.numel() % 8 == 0, "gelu: contiguous, numel % 8 == 0");
  const int64_t n = x.numel() / 8;
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  gelu_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gelu_bwd(const at::Tensor& g, const at::Tensor& x, at::Tensor& dx) {
  TORCH_CHECK(g.is_contiguous() && x.is_contiguous() && dx.is_contiguous() && x.numel() % 8 == 0, "gelu_bwd layout");
  const int64_t n = x.numel() / 8;
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  gelu_bwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmad

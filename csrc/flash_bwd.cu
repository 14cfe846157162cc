// Flash-attention backward for sm_100a (bf16, head dim 64 or 128), two tcgen05 kernels.
//
// Functional parity target: the backward the reference pairs with its attention
// forward (flash-attn 2 `_flash_attn_backward`, called from
// train/wan/rcm/utils/flash_attention_jvp_triton.py:534-579, and cuDNN SDPA
// backward through attention.py:120-167): dQ, dK, dV of O = softmax(Q K^T s) V.
//
// Kernel A (dK, dV): one CTA per 128-key tile, looping over 128-query tiles.
//   S^T = K Q^T and dP^T = V dO^T go to TMEM; the row owner (thread = key)
//   forms P^T (written back as bf16 over S^T) and dS^T = P^T (dP^T - D) s
//   (written back as bf16 over dP^T); dV += P^T dO and dK += dS^T Q are
//   TMEM-A MMAs.  TMEM: S^T 0..127, dP^T 128..255, dV 256.., dK 384.. (d columns each).
// Kernel B (dQ): one CTA per 128-query tile, looping over 128-key tiles with
//   a double-buffered S, dP, and dQ += dS K as a TMEM-A MMA.
// Splitting dQ from dK/dV costs two extra GEMMs per tile pair but needs no
// atomics and no fp32 scratch accumulator.
// In both kernels two 128-thread groups (warps 4..7 and 8..11) share the elementwise work of a
// tile by columns: group g handles columns [64g, 64g + 64) and writes its bf16 P / dS packed over
// the first half of its own columns; the TMEM-A MMAs take the halves from [0, 32) and [64, 96).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "sm100.cuh"
#include "tma_host.h"

namespace dmad {

void check_bhld(const at::Tensor& x, const char* name, int64_t d = 128);
int* device_status_ptr(int device);
int64_t flash_lse_pad(int64_t L);

namespace {

constexpr int kHalfBytes = 128 * 128;
constexpr int kTileBytes = 2 * kHalfBytes;

struct BwdParams {
  __nv_bfloat16* out;  // dK/dV base (kernel A uses out & out2) or dQ (kernel B)
  __nv_bfloat16* out2;
  int64_t sb, sl, sh;     // strides of out
  int64_t sb2, sl2, sh2;  // strides of out2
  const float* lse2;      // [B, H, Lpad] log2-domain
  const float* dd;        // [B, H, Lpad] rowsum(dO * O)
  int Lq, Lk, H, Lpad;
  float scale_log2, scale;
  int* status;
};

// Columns [c_begin, c_begin + 32 * n_chunks) of one TMEM row as bf16.
__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* row, uint32_t tmem_row, float mul, int c_begin = 0,
                                               int n_chunks = 4) {
  if (row != nullptr) row += c_begin;
  tmem_row += c_begin;
#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    uint32_t r[32];
    tmem_ld32(tmem_row + c * 32, r);
    tmem_wait_ld();
    if (row != nullptr) {
      uint4* dst = reinterpret_cast<uint4*>(row + c * 32);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * mul, __uint_as_float(r[8 * v + 1]) * mul);
        w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * mul, __uint_as_float(r[8 * v + 3]) * mul);
        w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * mul, __uint_as_float(r[8 * v + 5]) * mul);
        w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * mul, __uint_as_float(r[8 * v + 7]) * mul);
        dst[v] = w;
      }
    }
  }
}

// TMEM column of the bf16 A operand for K step kk (16 elements = 8 columns): the two column groups'
// packed halves live at [0, 32) and [64, 96) of the region.
__device__ __forceinline__ uint32_t split_a_col(int kk) { return kk < 4 ? kk * 8 : 64 + (kk - 4) * 8; }

// ------------------------------------------------------------------ D = rowsum(dO * O)
template <int kD>
__global__ void bwd_dot_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                               float* __restrict__ dd, int64_t osb, int64_t osl, int64_t osh, int64_t gsb,
                               int64_t gsl, int64_t gsh, int B, int H, int Lq, int Lpad) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * H * Lpad) return;
  const int q = row % Lpad;
  const int h = (row / Lpad) % H;
  const int b = row / ((int64_t)Lpad * H);
  float acc = 0.f;
  if (q < Lq) {
    if constexpr (kD == 128) {  // four elements a lane
      const uint2 ov = *reinterpret_cast<const uint2*>(o + b * osb + q * osl + h * osh + lane * 4);
      const uint2 gv = *reinterpret_cast<const uint2*>(dout + b * gsb + q * gsl + h * gsh + lane * 4);
      const float2 o0 = unpack_bf16x2(ov.x), o1 = unpack_bf16x2(ov.y);
      const float2 g0 = unpack_bf16x2(gv.x), g1 = unpack_bf16x2(gv.y);
      acc = o0.x * g0.x + o0.y * g0.y + o1.x * g1.x + o1.y * g1.y;
    } else {  // two
      const float2 o0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(o + b * osb + q * osl + h * osh + lane * 2));
      const float2 g0 =
          unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dout + b * gsb + q * gsl + h * gsh + lane * 2));
      acc = o0.x * g0.x + o0.y * g0.y;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  }
  if (lane == 0) dd[row] = acc;
}

// ------------------------------------------------------------------ kernel A: dK, dV
template <int kD>
struct DkvSmem {
  static constexpr int kT = kD / 64 * kHalfBytes;  // 128 rows x kD bf16 as 64-column panels
  uint8_t k[kT];
  uint8_t v[kT];
  uint8_t q[2][kT];
  uint8_t g[2][kT];  // dO
  float lse[2][128];
  float dd[2][128];
  uint64_t kv_full;
  uint64_t q_full[2], q_empty[2];
  uint64_t s_full, dp_full, done;
  uint64_t p_part[4], ds_part[4];  // part 2g + c: query columns [64g + 32c, +32) of P^T / dS^T
  uint32_t tmem_base;
  int abort_flag;
};

template <int kD>
__global__ void __launch_bounds__(384, 1)
flash_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_g,
                      BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  using Smem = DkvSmem<kD>;
  constexpr int kPanels = kD / 64, kT = Smem::kT;
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.y, batch = blockIdx.z;
  const int k0 = blockIdx.x * 128;
  const int nq = (p.Lq + 127) / 128;
  const int64_t bh_off = ((int64_t)batch * p.H + head) * p.Lpad;

  if (threadIdx.x == 0) {
    mbar_init(&sm.kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.dp_full, 1);
    for (int q = 0; q < 4; ++q) {
      mbar_init(&sm.p_part[q], 128);
      mbar_init(&sm.ds_part[q], 128);
    }
    mbar_init(&sm.done, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&sm.kv_full, 2 * kT);
      for (int h = 0; h < kPanels; ++h) {
        tma_load_4d(sm.k + h * kHalfBytes, &tm_k, &sm.kv_full, h * 64, head, k0, batch);
        tma_load_4d(sm.v + h * kHalfBytes, &tm_v, &sm.kv_full, h * 64, head, k0, batch);
      }
      int last_s = -1;
      uint32_t last_ph = 0;
      for (int i = 0; i < nq; ++i) {
        const int s = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&sm.q_empty[s], ph ^ 1, kStatusTimeoutEmpty, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&sm.q_full[s], 2 * kT + 2 * 512);
        for (int h = 0; h < kPanels; ++h) {
          tma_load_4d(sm.q[s] + h * kHalfBytes, &tm_q, &sm.q_full[s], h * 64, head, i * 128, batch);
          tma_load_4d(sm.g[s] + h * kHalfBytes, &tm_g, &sm.q_full[s], h * 64, head, i * 128, batch);
        }
        bulk_load(sm.lse[s], p.lse2 + bh_off + i * 128, 512, &sm.q_full[s]);
        bulk_load(sm.dd[s], p.dd + bh_off + i * 128, 512, &sm.q_full[s]);
        last_s = s;
        last_ph = ph;
      }
      mbar_wait(&sm.kv_full, 0, kStatusTimeoutTmaFull, nullptr, p.status);
      if (last_s >= 0) mbar_wait(&sm.q_full[last_s], last_ph, kStatusTimeoutTmaFull, nullptr, p.status);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_kk = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_mn = idesc_bf16_f32(128, kD, false, true);
      const uint32_t ka = smem_u32(sm.k), va = smem_u32(sm.v);
      const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 384;
      auto gemm_kk = [&](uint32_t d, uint32_t a, uint32_t b) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16_ss(d, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(b + off, 16, 1024), idesc_kk, kk > 0);
        }
      };
      // D (+)= A B with A in TMEM (P^T or dS^T), handed over in four parts of 32 columns (K steps 2q and
      // 2q + 1 for part q), issued as each part lands: parts 0 and 2 (the first halves of the two
      // column groups, written at the same time) before 1 and 3.
      auto ts_parts = [&](uint64_t* parts, uint32_t parity, uint32_t d, uint32_t a_tmem, uint32_t b, bool acc) {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int q = (n & 1) * 2 + (n >> 1);
          if (!mbar_wait(&parts[q], parity, kStatusTimeoutSoftmax, abort_flag, p.status)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 2 * q; kk < 2 * q + 2; ++kk)
            mma_bf16_ts(d, a_tmem + split_a_col(kk), smem_desc_sw128(b + kk * 2048, kHalfBytes, 1024), idesc_mn,
                        (acc || kk > 0) ? 1u : 0u);
        }
        return true;
      };
      bool ok = mbar_wait(&sm.kv_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) ok = mbar_wait(&sm.q_full[0], 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
        gemm_kk(t_s, ka, smem_u32(sm.q[0]));
        mma_commit(&sm.s_full);
        gemm_kk(t_dp, va, smem_u32(sm.g[0]));
        mma_commit(&sm.dp_full);
      }
      for (int i = 0; ok && i < nq; ++i) {
        const int s = i & 1;
        const bool has_next = i + 1 < nq;
        const int s1 = (i + 1) & 1;
        const uint32_t ph1 = ((i + 1) >> 1) & 1;
        if (!(ok = ts_parts(sm.p_part, i & 1, t_dv, t_s, smem_u32(sm.g[s]), i > 0))) break;
        if (has_next) {
          if (!(ok = mbar_wait(&sm.q_full[s1], ph1, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
          tc_fence_after();
          gemm_kk(t_s, ka, smem_u32(sm.q[s1]));
          mma_commit(&sm.s_full);
        }
        if (!(ok = ts_parts(sm.ds_part, i & 1, t_dk, t_dp, smem_u32(sm.q[s]), i > 0))) break;
        mma_commit(&sm.q_empty[s]);
        if (has_next) {
          gemm_kk(t_dp, va, smem_u32(sm.g[s1]));
          mma_commit(&sm.dp_full);
        }
      }
      mma_commit(&sm.done);
      mbar_wait(&sm.done, 0, kStatusTimeoutMma, nullptr, p.status);
    }
  } else if (warp >= 4) {
    const int g = (warp - 4) >> 2;  // column group: query columns [64g, 64g + 64)
    const int c0 = 64 * g;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lb = (uint32_t)(wq * 32) << 16;
    const uint32_t t_s = tmem + lb + c0, t_dp = tmem + lb + 128 + c0;
    const float scale_log2 = p.scale_log2, scale = p.scale;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const int s = i & 1;
      const uint32_t ph = (i >> 1) & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_full[s], ph, kStatusTimeoutTmaFull, abort_flag, p.status));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full, i & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      float pv[64];
      {
        uint32_t r[2][32];
        tmem_ld32(t_s, r[0]);
        tmem_ld32(t_s + 32, r[1]);
        tmem_wait_ld();
        const float* lse = sm.lse[s] + c0;
        // every second exponential on the FMA pipe, two at a time as one packed polynomial
        // (padded query columns have lse = +inf: the polynomial's clamp gives ~1e-38 there,
        // against dO = 0)
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) x[u] = fmaf(__uint_as_float(r[c][e + u]), scale_log2, -lse[c * 32 + e + u]);
            const float2 pp = ex2_poly2(x[1], x[3]);
            pv[c * 32 + e] = ex2_approx(x[0]);
            pv[c * 32 + e + 1] = pp.x;
            pv[c * 32 + e + 2] = ex2_approx(x[2]);
            pv[c * 32 + e + 3] = pp.y;
          }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // P^T to the MMA thread in two parts of 32 query columns
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(pv[c * 32 + 2 * e], pv[c * 32 + 2 * e + 1]);
        tmem_st16(t_s + 16 * c, w);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.p_part[2 * g + c]);
      }

      ok = __all_sync(0xffffffffu, mbar_wait(&sm.dp_full, i & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t r[2][32];
        tmem_ld32(t_dp, r[0]);
        tmem_ld32(t_dp + 32, r[1]);
        tmem_wait_ld();
        const float* dd = sm.dd[s] + c0;
        const uint64_t sc2 = f2(scale, scale);
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {  // dS = P (dP - D) scale, two columns per packed op
            const int q = c * 32 + 2 * e;
            const uint64_t dp2 = f2(__uint_as_float(r[c][2 * e]), __uint_as_float(r[c][2 * e + 1]));
            const uint64_t ds2 = f2_mul(f2_mul(f2_sub(dp2, f2(dd[q], dd[q + 1])), f2(pv[q], pv[q + 1])), sc2);
            const float2 d = f2_split(ds2);
            w[c * 16 + e] = pack_bf16x2(d.x, d.y);
          }
          // hand this part of dS^T to the MMA thread
          tmem_st16(t_dp + 16 * c, *reinterpret_cast<const uint32_t(*)[16]>(w + 16 * c));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&sm.ds_part[2 * g + c]);
        }
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.done, 0, kStatusTimeoutMma, abort_flag, p.status));
    if (ok) {
      tc_fence_after();
      const int kr = k0 + row;
      const bool valid = kr < p.Lk;
      __nv_bfloat16* dv_row = valid ? p.out2 + batch * p.sb2 + (int64_t)kr * p.sl2 + head * p.sh2 : nullptr;
      __nv_bfloat16* dk_row = valid ? p.out + batch * p.sb + (int64_t)kr * p.sl + head * p.sh : nullptr;
      // group g stores output columns [g d / 2, (g + 1) d / 2)
      store_row_bf16(dv_row, tmem + lb + 256, 1.f, g * (kD / 2), kD / 64);
      store_row_bf16(dk_row, tmem + lb + 384, 1.f, g * (kD / 2), kD / 64);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ kernel B: dQ
template <int kD>
struct DqSmem {
  static constexpr int kT = kD / 64 * kHalfBytes;
  uint8_t q[kT];
  uint8_t g[kT];
  uint8_t k[2][kT];
  uint8_t v[2][kT];
  uint64_t q_full;
  uint64_t kv_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t dp_full, done;
  uint64_t ds_part[4];  // part 2g + c: key columns [64g + 32c, +32) of dS
  uint32_t tmem_base;
  int abort_flag;
};

template <int kD>
__global__ void __launch_bounds__(384, 1)
flash_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_g,
                    BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  using Smem = DqSmem<kD>;
  constexpr int kPanels = kD / 64, kT = Smem::kT;
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.y, batch = blockIdx.z;
  const int q0 = blockIdx.x * 128;
  const int nkv = (p.Lk + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.s_free[s], 256);
    }
    mbar_init(&sm.dp_full, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&sm.ds_part[q], 128);
    mbar_init(&sm.done, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&sm.q_full, 2 * kT);
      for (int h = 0; h < kPanels; ++h) {
        tma_load_4d(sm.q + h * kHalfBytes, &tm_q, &sm.q_full, h * 64, head, q0, batch);
        tma_load_4d(sm.g + h * kHalfBytes, &tm_g, &sm.q_full, h * 64, head, q0, batch);
      }
      int last_s = -1;
      uint32_t last_ph = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&sm.kv_empty[s], ph ^ 1, kStatusTimeoutEmpty, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&sm.kv_full[s], 2 * kT);
        for (int h = 0; h < kPanels; ++h) {
          tma_load_4d(sm.k[s] + h * kHalfBytes, &tm_k, &sm.kv_full[s], h * 64, head, j * 128, batch);
          tma_load_4d(sm.v[s] + h * kHalfBytes, &tm_v, &sm.kv_full[s], h * 64, head, j * 128, batch);
        }
        last_s = s;
        last_ph = ph;
      }
      mbar_wait(&sm.q_full, 0, kStatusTimeoutTmaFull, nullptr, p.status);
      if (last_s >= 0) mbar_wait(&sm.kv_full[last_s], last_ph, kStatusTimeoutTmaFull, nullptr, p.status);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_kk = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_mn = idesc_bf16_f32(128, kD, false, true);
      const uint32_t qa = smem_u32(sm.q), ga = smem_u32(sm.g);
      const uint32_t t_dp = tmem + 256, t_dq = tmem + 384;
      auto gemm_kk = [&](uint32_t d, uint32_t a, uint32_t b) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16_ss(d, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(b + off, 16, 1024), idesc_kk, kk > 0);
        }
      };
      auto ts_parts = [&](uint64_t* parts, uint32_t parity, uint32_t d, uint32_t a_tmem, uint32_t b, bool acc) {
#pragma unroll
        for (int n = 0; n < 4; ++n) {  // parts 0 and 2 first, as in the dK / dV kernel
          const int q = (n & 1) * 2 + (n >> 1);
          if (!mbar_wait(&parts[q], parity, kStatusTimeoutSoftmax, abort_flag, p.status)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 2 * q; kk < 2 * q + 2; ++kk)
            mma_bf16_ts(d, a_tmem + split_a_col(kk), smem_desc_sw128(b + kk * 2048, kHalfBytes, 1024), idesc_mn,
                        (acc || kk > 0) ? 1u : 0u);
        }
        return true;
      };
      bool ok = mbar_wait(&sm.q_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) ok = mbar_wait(&sm.kv_full[0], 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
        gemm_kk(tmem, qa, smem_u32(sm.k[0]));
        mma_commit(&sm.s_full[0]);
        gemm_kk(t_dp, ga, smem_u32(sm.v[0]));
        mma_commit(&sm.dp_full);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j & 1;
        const bool has_next = j + 1 < nkv;
        const int s1 = (j + 1) & 1;
        const uint32_t ph1 = ((j + 1) >> 1) & 1;
        if (has_next) {
          if (!(ok = mbar_wait(&sm.kv_full[s1], ph1, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
          if (j >= 1 && !(ok = mbar_wait(&sm.s_free[s1], ((j - 1) >> 1) & 1, kStatusTimeoutSoftmax, abort_flag, p.status)))
            break;
          tc_fence_after();
          gemm_kk(tmem + s1 * 128, qa, smem_u32(sm.k[s1]));
          mma_commit(&sm.s_full[s1]);
        }
        const uint32_t kb = smem_u32(sm.k[s]);
        if (!(ok = ts_parts(sm.ds_part, j & 1, t_dq, t_dp, kb, j > 0))) break;
        mma_commit(&sm.kv_empty[s]);
        if (has_next) {
          gemm_kk(t_dp, ga, smem_u32(sm.v[s1]));
          mma_commit(&sm.dp_full);
        }
      }
      mma_commit(&sm.done);
      mbar_wait(&sm.done, 0, kStatusTimeoutMma, nullptr, p.status);
    }
  } else if (warp >= 4) {
    const int g = (warp - 4) >> 2;  // column group: key columns [64g, 64g + 64)
    const int c0 = 64 * g;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int q_row = q0 + row;
    const uint32_t lb = (uint32_t)(wq * 32) << 16;
    const uint32_t t_dp = tmem + lb + 256 + c0;
    const float scale_log2 = p.scale_log2, scale = p.scale;
    const int64_t bh_off = ((int64_t)batch * p.H + head) * p.Lpad;
    const float lse2 = p.lse2[bh_off + q_row];
    const float dval = p.dd[bh_off + q_row];
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[s], (j >> 1) & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      float pv[64];
      const int kv_valid = p.Lk - j * 128 - c0;
      {
        uint32_t r[2][32];
        tmem_ld32(tmem + lb + s * 128 + c0, r[0]);
        tmem_ld32(tmem + lb + s * 128 + c0 + 32, r[1]);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&sm.s_free[s]);
        if (kv_valid >= 64) {  // full columns: packed scale-and-shift, every second exponential as
                               // half of a packed polynomial on the FMA pipe
          const uint64_t sc2 = f2(scale_log2, scale_log2), nl2 = f2(-lse2, -lse2);
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              const float2 xa = f2_split(f2_fma(f2(__uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1])), sc2, nl2));
              const float2 xb =
                  f2_split(f2_fma(f2(__uint_as_float(r[c][e + 2]), __uint_as_float(r[c][e + 3])), sc2, nl2));
              const float2 pp = ex2_poly2(xa.y, xb.y);
              pv[c * 32 + e] = ex2_approx(xa.x);
              pv[c * 32 + e + 1] = pp.x;
              pv[c * 32 + e + 2] = ex2_approx(xb.x);
              pv[c * 32 + e + 3] = pp.y;
            }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              pv[c * 32 + e] =
                  (c * 32 + e < kv_valid) ? ex2_approx(fmaf(__uint_as_float(r[c][e]), scale_log2, -lse2)) : 0.f;
        }
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.dp_full, j & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t r[2][32];
        tmem_ld32(t_dp, r[0]);
        tmem_ld32(t_dp + 32, r[1]);
        tmem_wait_ld();
        const uint64_t nd2 = f2(-dval, -dval), sc2 = f2(scale, scale);
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {  // dS = P (dP - D) scale, two columns per packed op
            const int kv = c * 32 + 2 * e;
            const uint64_t dp2 = f2(__uint_as_float(r[c][2 * e]), __uint_as_float(r[c][2 * e + 1]));
            const float2 d = f2_split(f2_mul(f2_mul(f2_add(dp2, nd2), f2(pv[kv], pv[kv + 1])), sc2));
            w[c * 16 + e] = pack_bf16x2(d.x, d.y);
          }
          // hand this part of dS to the MMA thread
          tmem_st16(t_dp + 16 * c, *reinterpret_cast<const uint32_t(*)[16]>(w + 16 * c));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&sm.ds_part[2 * g + c]);
        }
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.done, 0, kStatusTimeoutMma, abort_flag, p.status));
    if (ok) {
      tc_fence_after();
      __nv_bfloat16* dq_row = q_row < p.Lq ? p.out + batch * p.sb + (int64_t)q_row * p.sl + head * p.sh : nullptr;
      store_row_bf16(dq_row, tmem + lb + 384, 1.f, g * (kD / 2), kD / 64);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ fused kernel: dK, dV and dQ
// One CTA per 128-key tile, as kernel A, that also forms dQ_i = dS_i K for every query tile i and adds
// it into an fp32 accumulator [B, H, Lpad, 128] with vector reductions (red.global.add.v4.f32): five
// GEMMs per tile pair instead of seven.  TMEM: S^T / P^T 0..127, dP^T and then dQ_i 128..255,
// dV 256..383, dK 384..511.  dS^T of tile i is written over dO_i once dV_i (its last reader) is done,
// in the 128-byte-swizzled layout TMA gives a [128][64] box; dK += dS^T Q_i reads it as a K-major A
// and dQ_i = dS K as an MN-major A.  Per tile the tensor pipe runs dP_i, dV_i, S_{i+1}, dK_i, dQ_i
// and waits only while the softmax warps drain dQ_i out of TMEM (dP_{i+1} reuses its columns).
struct FusedSmem {
  uint8_t k[kTileBytes];
  uint8_t v[kTileBytes];
  uint8_t q[2][kTileBytes];
  uint8_t g[2][kTileBytes];  // dO_i, then dS_i^T
  float lse[2][128];
  float dd[2][128];
  uint64_t kv_full;
  uint64_t q_full[2], q_empty[2];
  uint64_t s_full, dp_full, p_full, dv_done, ds_full, dq_full, dq_free, done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__global__ void __launch_bounds__(384, 1)
flash_bwd_fused_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_g,
                       BwdParams p, float* __restrict__ dq_acc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  FusedSmem& sm = *reinterpret_cast<FusedSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = warp_id(), lane = lane_id();
  const int head = blockIdx.y, batch = blockIdx.z;
  const int k0 = blockIdx.x * 128;
  const int nq = (p.Lq + 127) / 128;
  const int64_t bh_off = ((int64_t)batch * p.H + head) * p.Lpad;

  if (threadIdx.x == 0) {
    mbar_init(&sm.kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 1);
    }
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.dp_full, 1);
    mbar_init(&sm.p_full, 256);
    mbar_init(&sm.dv_done, 1);
    mbar_init(&sm.ds_full, 256);
    mbar_init(&sm.dq_full, 1);
    mbar_init(&sm.dq_free, 256);
    mbar_init(&sm.done, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&sm.kv_full, 2 * kTileBytes);
      for (int h = 0; h < 2; ++h) {
        tma_load_4d(sm.k + h * kHalfBytes, &tm_k, &sm.kv_full, h * 64, head, k0, batch);
        tma_load_4d(sm.v + h * kHalfBytes, &tm_v, &sm.kv_full, h * 64, head, k0, batch);
      }
      int last_s = -1;
      uint32_t last_ph = 0;
      for (int i = 0; i < nq; ++i) {
        const int s = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!mbar_wait(&sm.q_empty[s], ph ^ 1, kStatusTimeoutEmpty, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&sm.q_full[s], 2 * kTileBytes + 2 * 512);
        for (int h = 0; h < 2; ++h) {
          tma_load_4d(sm.q[s] + h * kHalfBytes, &tm_q, &sm.q_full[s], h * 64, head, i * 128, batch);
          tma_load_4d(sm.g[s] + h * kHalfBytes, &tm_g, &sm.q_full[s], h * 64, head, i * 128, batch);
        }
        bulk_load(sm.lse[s], p.lse2 + bh_off + i * 128, 512, &sm.q_full[s]);
        bulk_load(sm.dd[s], p.dd + bh_off + i * 128, 512, &sm.q_full[s]);
        last_s = s;
        last_ph = ph;
      }
      mbar_wait(&sm.kv_full, 0, kStatusTimeoutTmaFull, nullptr, p.status);
      if (last_s >= 0) mbar_wait(&sm.q_full[last_s], last_ph, kStatusTimeoutTmaFull, nullptr, p.status);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_kk = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_mn = idesc_bf16_f32(128, 128, false, true);
      constexpr uint32_t idesc_dq = idesc_bf16_f32(128, 128, true, true);
      const uint32_t ka = smem_u32(sm.k), va = smem_u32(sm.v);
      const uint32_t t_s = tmem, t_y = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 384;
      auto gemm_kk = [&](uint32_t d, uint32_t a, uint32_t b) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16_ss(d, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(b + off, 16, 1024), idesc_kk, kk > 0);
        }
      };
      bool ok = mbar_wait(&sm.kv_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) ok = mbar_wait(&sm.q_full[0], 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
        gemm_kk(t_s, ka, smem_u32(sm.q[0]));
        mma_commit(&sm.s_full);
        gemm_kk(t_y, va, smem_u32(sm.g[0]));
        mma_commit(&sm.dp_full);
      }
      for (int i = 0; ok && i < nq; ++i) {
        const int s = i & 1;
        const bool has_next = i + 1 < nq;
        const int s1 = (i + 1) & 1;
        const uint32_t ph1 = ((i + 1) >> 1) & 1;
        const uint32_t ga = smem_u32(sm.g[s]), qa = smem_u32(sm.q[s]);
        if (i > 0) {  // dP_i into the columns dQ_{i-1} has left
          if (!(ok = mbar_wait(&sm.dq_free, (i - 1) & 1, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
          tc_fence_after();
          gemm_kk(t_y, va, ga);
          mma_commit(&sm.dp_full);
        }
        if (!(ok = mbar_wait(&sm.p_full, i & 1, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO_i
          mma_bf16_ts(t_dv, t_s + split_a_col(kk), smem_desc_sw128(ga + kk * 2048, kHalfBytes, 1024), idesc_mn,
                      (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&sm.dv_done);
        if (has_next) {
          if (!(ok = mbar_wait(&sm.q_full[s1], ph1, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
          tc_fence_after();
          gemm_kk(t_s, ka, smem_u32(sm.q[s1]));
          mma_commit(&sm.s_full);
        }
        if (!(ok = mbar_wait(&sm.ds_full, i & 1, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // dK += dS^T Q_i (dS^T K-major over dO_i's buffer)
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16_ss(t_dk, smem_desc_sw128(ga + off, 16, 1024), smem_desc_sw128(qa + kk * 2048, kHalfBytes, 1024),
                      idesc_mn, (i > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dQ_i = dS K (dS MN-major, K MN-major)
          mma_bf16_ss(t_y, smem_desc_sw128(ga + kk * 2048, kHalfBytes, 1024),
                      smem_desc_sw128(ka + kk * 2048, kHalfBytes, 1024), idesc_dq, kk > 0 ? 1u : 0u);
        mma_commit(&sm.dq_full);
        mma_commit(&sm.q_empty[s]);
      }
      mma_commit(&sm.done);
      mbar_wait(&sm.done, 0, kStatusTimeoutMma, nullptr, p.status);
    }
  } else if (warp >= 4) {
    const int g = (warp - 4) >> 2;  // column group: query columns (then dQ columns) [64g, 64g + 64)
    const int c0 = 64 * g;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lb = (uint32_t)(wq * 32) << 16;
    const uint32_t t_s = tmem + lb + c0, t_y = tmem + lb + 128 + c0;
    const float scale_log2 = p.scale_log2, scale = p.scale;
    bool ok = true;
    // dQ_j out of TMEM (lane = query row of tile j) into the fp32 accumulator
    auto drain_dq = [&](int j) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.dq_full, j & 1, kStatusTimeoutMma, abort_flag, p.status)))
        return false;
      tc_fence_after();
      uint32_t r[2][32];
      tmem_ld32(t_y, r[0]);
      tmem_ld32(t_y + 32, r[1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sm.dq_free);
      float* dst = dq_acc + (bh_off + (int64_t)j * 128 + row) * 128 + c0;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int v = 0; v < 8; ++v)
          red_add_v4(dst + c * 32 + 4 * v, __uint_as_float(r[c][4 * v]), __uint_as_float(r[c][4 * v + 1]),
                     __uint_as_float(r[c][4 * v + 2]), __uint_as_float(r[c][4 * v + 3]));
      return true;
    };
    for (int i = 0; i < nq; ++i) {
      const int s = i & 1;
      const uint32_t ph = (i >> 1) & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_full[s], ph, kStatusTimeoutTmaFull, abort_flag, p.status));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full, i & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      float pv[64];
      {
        uint32_t r[2][32];
        tmem_ld32(t_s, r[0]);
        tmem_ld32(t_s + 32, r[1]);
        tmem_wait_ld();
        const float* lse = sm.lse[s] + c0;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float x = fmaf(__uint_as_float(r[c][e]), scale_log2, -lse[c * 32 + e]);
            pv[c * 32 + e] = (e & 1) ? ex2_poly(x) : ex2_approx(x);
          }
      }
      {
        uint32_t w[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) w[e] = pack_bf16x2(pv[2 * e], pv[2 * e + 1]);
        tmem_st32(t_s, w);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.p_full);
      if (i > 0 && !(ok = drain_dq(i - 1))) break;

      ok = __all_sync(0xffffffffu, mbar_wait(&sm.dp_full, i & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      uint32_t w[32];
      {
        uint32_t r[2][32];
        tmem_ld32(t_y, r[0]);
        tmem_ld32(t_y + 32, r[1]);
        tmem_wait_ld();
        const float* dd = sm.dd[s] + c0;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int q = c * 32 + 2 * e;
            const float d0 = pv[q] * (__uint_as_float(r[c][2 * e]) - dd[q]) * scale;
            const float d1 = pv[q + 1] * (__uint_as_float(r[c][2 * e + 1]) - dd[q + 1]) * scale;
            w[c * 16 + e] = pack_bf16x2(d0, d1);
          }
      }
      // dO_i's buffer takes dS^T once dV_i has read it
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.dv_done, i & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      {
        uint8_t* dst = sm.g[s] + g * kHalfBytes + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(dst + ((c ^ (row & 7)) << 4)) =
              make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.ds_full);
    }
    if (ok && nq > 0) ok = drain_dq(nq - 1);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.done, 0, kStatusTimeoutMma, abort_flag, p.status));
    if (ok) {
      tc_fence_after();
      const int kr = k0 + row;
      const bool valid = kr < p.Lk;
      __nv_bfloat16* dv_row = valid ? p.out2 + batch * p.sb2 + (int64_t)kr * p.sl2 + head * p.sh2 : nullptr;
      __nv_bfloat16* dk_row = valid ? p.out + batch * p.sb + (int64_t)kr * p.sl + head * p.sh : nullptr;
      store_row_bf16(dv_row, tmem + lb + 256, 1.f, c0, 2);
      store_row_bf16(dk_row, tmem + lb + 384, 1.f, c0, 2);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dq (bf16, strided [B, Lq, H, 128]) from the fp32 accumulator [B, H, Lpad, 128]; 8 elements a thread
__global__ void dq_from_acc_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t sb,
                                   int64_t sl, int64_t sh, int B, int H, int Lq, int Lpad) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * Lq * H * 16;
  if (t >= total) return;
  const int c8 = t & 15;
  const int64_t r = t >> 4;  // (b, l, h) in dq's order
  const int h = r % H;
  const int l = (r / H) % Lq;
  const int b = r / ((int64_t)H * Lq);
  const float4* src = reinterpret_cast<const float4*>(acc + ((((int64_t)b * H + h) * Lpad + l) * 128 + c8 * 8));
  const float4 x = src[0], y = src[1];
  uint4 w;
  w.x = pack_bf16x2(x.x, x.y);
  w.y = pack_bf16x2(x.z, x.w);
  w.z = pack_bf16x2(y.x, y.y);
  w.w = pack_bf16x2(y.z, y.w);
  *reinterpret_cast<uint4*>(dq + b * sb + (int64_t)l * sl + h * sh + c8 * 8) = w;
}

CUtensorMap make_map(const at::Tensor& x) {
  const uint64_t dims[4] = {(uint64_t)x.size(3), (uint64_t)x.size(2), (uint64_t)x.size(1), (uint64_t)x.size(0)};
  const uint64_t strides[3] = {(uint64_t)x.stride(2) * 2, (uint64_t)x.stride(1) * 2, (uint64_t)x.stride(0) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(x.data_ptr(), 4, dims, strides, box);
}

}  // namespace

// [B, L, H, d] tensors, d = 64 or 128; dq, dk, dv may be strided views (e.g. slices of one fused
// [B, L, 3, H, d] buffer).
// lse2: [B, H, Lpad] log2-domain LSE from flash_fwd; dd_scratch: [B, H, Lpad] fp32 work
// buffer that receives rowsum(dO * O).
void flash_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
               const at::Tensor& dout, const at::Tensor& lse2, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
               at::Tensor& dd_scratch, double scale) {
  TORCH_CHECK(q.dim() == 4 && (q.size(3) == 64 || q.size(3) == 128), "q must be [B, L, H, 64 or 128]");
  const int d = (int)q.size(3);
  check_bhld(q, "q", d);
  check_bhld(k, "k", d);
  check_bhld(v, "v", d);
  check_bhld(o, "o", d);
  check_bhld(dout, "dout", d);
  check_bhld(dq, "dq", d);
  check_bhld(dk, "dk", d);
  check_bhld(dv, "dv", d);
  const int B = q.size(0), Lq = q.size(1), H = q.size(2), Lk = k.size(1);
  const int64_t Lpad = flash_lse_pad(Lq);
  TORCH_CHECK(lse2.is_contiguous() && lse2.scalar_type() == at::kFloat && lse2.dim() == 3 && lse2.size(2) == Lpad,
              "lse must be [B, H, round_up(Lq, 256)] fp32");
  TORCH_CHECK(dd_scratch.is_contiguous() && dd_scratch.scalar_type() == at::kFloat &&
                  dd_scratch.numel() >= (int64_t)B * H * Lpad,
              "dd_scratch too small");
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  {
    const int64_t rows = (int64_t)B * H * Lpad;
    const int warps = 8;
    auto dot = d == 64 ? bwd_dot_kernel<64> : bwd_dot_kernel<128>;
    dot<<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        dd_scratch.data_ptr<float>(), o.stride(0), o.stride(1), o.stride(2), dout.stride(0), dout.stride(1),
        dout.stride(2), B, H, Lq, (int)Lpad);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  CUtensorMap tq = make_map(q), tk = make_map(k), tv = make_map(v), tg = make_map(dout);
  BwdParams p;
  p.lse2 = lse2.data_ptr<float>();
  p.dd = dd_scratch.data_ptr<float>();
  p.Lq = Lq;
  p.Lk = Lk;
  p.H = H;
  p.Lpad = (int)Lpad;
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.status = device_status_ptr(q.get_device());
  {
    p.out = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
    p.sb = dk.stride(0);
    p.sl = dk.stride(1);
    p.sh = dk.stride(2);
    p.out2 = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
    p.sb2 = dv.stride(0);
    p.sl2 = dv.stride(1);
    p.sh2 = dv.stride(2);
    const size_t smem = (d == 64 ? sizeof(DkvSmem<64>) : sizeof(DkvSmem<128>)) + 1024;
    auto kern = d == 64 ? flash_bwd_dkdv_kernel<64> : flash_bwd_dkdv_kernel<128>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((Lk + 127) / 128, H, B);
    kern<<<grid, 384, smem, stream>>>(tq, tk, tv, tg, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  {
    p.out = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
    p.sb = dq.stride(0);
    p.sl = dq.stride(1);
    p.sh = dq.stride(2);
    p.out2 = nullptr;
    const size_t smem = (d == 64 ? sizeof(DqSmem<64>) : sizeof(DqSmem<128>)) + 1024;
    auto kern = d == 64 ? flash_bwd_dq_kernel<64> : flash_bwd_dq_kernel<128>;
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((Lq + 127) / 128, H, B);
    kern<<<grid, 384, smem, stream>>>(tq, tk, tv, tg, p);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}


// Single-kernel backward (dK, dV and an fp32 dQ accumulator in one pass over the tile pairs, then a
// conversion of the accumulator into dq).  dq_acc: fp32, at least B * H * round_up(Lq, 256) * 128
// elements, overwritten.
void flash_bwd_fused(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                     const at::Tensor& dout, const at::Tensor& lse2, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
                     at::Tensor& dd_scratch, at::Tensor& dq_acc, double scale) {
  check_bhld(q, "q");
  check_bhld(k, "k");
  check_bhld(v, "v");
  check_bhld(o, "o");
  check_bhld(dout, "dout");
  check_bhld(dq, "dq");
  check_bhld(dk, "dk");
  check_bhld(dv, "dv");
  const int B = q.size(0), Lq = q.size(1), H = q.size(2), Lk = k.size(1);
  const int64_t Lpad = flash_lse_pad(Lq);
  TORCH_CHECK(lse2.is_contiguous() && lse2.scalar_type() == at::kFloat && lse2.dim() == 3 && lse2.size(2) == Lpad,
              "lse must be [B, H, round_up(Lq, 256)] fp32");
  TORCH_CHECK(dd_scratch.is_contiguous() && dd_scratch.scalar_type() == at::kFloat &&
                  dd_scratch.numel() >= (int64_t)B * H * Lpad,
              "dd_scratch too small");
  TORCH_CHECK(dq_acc.is_cuda() && dq_acc.is_contiguous() && dq_acc.scalar_type() == at::kFloat &&
                  dq_acc.numel() >= (int64_t)B * H * Lpad * 128,
              "dq_acc must be contiguous fp32 with at least B * H * round_up(Lq, 256) * 128 elements");
  c10::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t rows = (int64_t)B * H * Lpad;
  {
    const int warps = 8;
    bwd_dot_kernel<128><<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
        dd_scratch.data_ptr<float>(), o.stride(0), o.stride(1), o.stride(2), dout.stride(0), dout.stride(1),
        dout.stride(2), B, H, Lq, (int)Lpad);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  C10_CUDA_CHECK(cudaMemsetAsync(dq_acc.data_ptr(), 0, (size_t)rows * 128 * sizeof(float), stream));
  CUtensorMap tq = make_map(q), tk = make_map(k), tv = make_map(v), tg = make_map(dout);
  BwdParams p;
  p.lse2 = lse2.data_ptr<float>();
  p.dd = dd_scratch.data_ptr<float>();
  p.Lq = Lq;
  p.Lk = Lk;
  p.H = H;
  p.Lpad = (int)Lpad;
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.status = device_status_ptr(q.get_device());
  p.out = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.sb = dk.stride(0);
  p.sl = dk.stride(1);
  p.sh = dk.stride(2);
  p.out2 = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.sb2 = dv.stride(0);
  p.sl2 = dv.stride(1);
  p.sh2 = dv.stride(2);
  const size_t smem = sizeof(FusedSmem) + 1024;
  C10_CUDA_CHECK(cudaFuncSetAttribute(flash_bwd_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  flash_bwd_fused_kernel<<<dim3((Lk + 127) / 128, H, B), 384, smem, stream>>>(tq, tk, tv, tg, p,
                                                                               dq_acc.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t threads = (int64_t)B * Lq * H * 16;
  dq_from_acc_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), dq.stride(0), dq.stride(1),
      dq.stride(2), B, H, Lq, (int)Lpad);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
}  // namespace dmad

// ============================================================================
// Allocation-free entry point (declaration, rules of use and the reason it
// exists: flash_bwd_noalloc.h).  No counterpart in the reference.
// ============================================================================
#include "flash_bwd_noalloc.h"
#include <cstdio>
#include <mutex>

namespace dmad {
namespace {

// rowsum(dO * O) work rows and the bounded-wait status word of the entry point
static __device__ __align__(256) float g_noalloc_rows[DMAD_NOALLOC_MAX_ROWS];
static __device__ __align__(256) int g_noalloc_status;

struct NoallocSymbols {
  float* rows = nullptr;
  int* status = nullptr;
};

// Device addresses of the static arrays, looked up once per device with that device current.
bool noalloc_symbols(NoallocSymbols& out) {
  static std::mutex mu;
  static NoallocSymbols table[64];
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> lock(mu);
  NoallocSymbols& s = table[dev];
  if (s.rows == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_rows) != cudaSuccess || p == nullptr) return false;
    void* st = nullptr;
    if (cudaGetSymbolAddress(&st, g_noalloc_status) != cudaSuccess || st == nullptr) return false;
    s.rows = static_cast<float*>(p);
    s.status = static_cast<int*>(st);
  }
  out = s;
  return true;
}

CUtensorMap map_raw(const void* base, int B, int L, int H, const int64_t* st) {
  const uint64_t dims[4] = {128, (uint64_t)H, (uint64_t)L, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(base, 4, dims, strides, box);
}

}  // namespace
}  // namespace dmad

extern "C" int dmad_flash_attn_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                           const void* dout, const float* lse2, void* dq, void* dk, void* dv, int B,
                                           int Lq, int Lk, int H, const int64_t* strides, float scale,
                                           void* stream) {
  using namespace dmad;
  const void* ptrs[10] = {q, k, v, o, dout, lse2, dq, dk, dv, strides};
  for (const void* p : ptrs)
    if (p == nullptr) {
      fprintf(stderr, "dmad_flash_attn_bwd_noalloc: null pointer argument\n");
      return DMAD_NOALLOC_ERR_ARGS;
    }
  if (B <= 0 || Lq <= 0 || Lk <= 0 || H <= 0) {
    fprintf(stderr, "dmad_flash_attn_bwd_noalloc: sizes must be positive\n");
    return DMAD_NOALLOC_ERR_ARGS;
  }
  // every tensor is moved with 16-byte vector accesses or bulk copies: a misaligned base would fault on the
  // GPU, so it is rejected here instead
  for (int i = 0; i < 9; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16 != 0) {
      fprintf(stderr, "dmad_flash_attn_bwd_noalloc: pointer argument %d is not 16-byte aligned\n", i);
      return DMAD_NOALLOC_ERR_ARGS;
    }
  {
    // the static array's address is per device: the stream must belong to the current device
    int cur = -1, sdev = -1;
    if (cudaGetDevice(&cur) != cudaSuccess ||
        cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess) {
      fprintf(stderr, "dmad_flash_attn_bwd_noalloc: cannot query the current device or the stream's device\n");
      return DMAD_NOALLOC_ERR_CUDA;
    }
    if (cur != sdev) {
      fprintf(stderr, "dmad_flash_attn_bwd_noalloc: stream belongs to device %d but device %d is current\n", sdev,
              cur);
      return DMAD_NOALLOC_ERR_ARGS;
    }
  }
  for (int i = 0; i < 24; ++i)
    if (strides[i] <= 0 || strides[i] % 8 != 0) {
      fprintf(stderr, "dmad_flash_attn_bwd_noalloc: stride %d must be a positive multiple of 8 elements\n", i);
      return DMAD_NOALLOC_ERR_ARGS;
    }
  const int64_t Lpad = flash_lse_pad(Lq);
  const int64_t rows = (int64_t)B * H * Lpad;
  if (rows > DMAD_NOALLOC_MAX_ROWS) {
    fprintf(stderr,
            "dmad_flash_attn_bwd_noalloc: B*H*round_up(Lq,256) = %lld exceeds the static work array of %d rows; "
            "use the regular entry point for this size\n",
            (long long)rows, DMAD_NOALLOC_MAX_ROWS);
    return DMAD_NOALLOC_ERR_TOO_LARGE;
  }
  NoallocSymbols sym;
  if (!noalloc_symbols(sym)) {
    fprintf(stderr, "dmad_flash_attn_bwd_noalloc: cudaGetSymbolAddress failed\n");
    return DMAD_NOALLOC_ERR_CUDA;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t* sq = strides + 0;
  const int64_t* sk = strides + 3;
  const int64_t* sv = strides + 6;
  const int64_t* so = strides + 9;
  const int64_t* sg = strides + 12;
  const int64_t* sdq = strides + 15;
  const int64_t* sdk = strides + 18;
  const int64_t* sdv = strides + 21;
  CUtensorMap tq, tk, tv, tg;
  try {
    tq = map_raw(q, B, Lq, H, sq);
    tk = map_raw(k, B, Lk, H, sk);
    tv = map_raw(v, B, Lk, H, sv);
    tg = map_raw(dout, B, Lq, H, sg);
  } catch (const std::exception& e) {
    fprintf(stderr, "dmad_flash_attn_bwd_noalloc: %s\n", e.what());
    return DMAD_NOALLOC_ERR_ARGS;
  }
  if (cudaMemsetAsync(sym.status, 0, sizeof(int), s) != cudaSuccess) return DMAD_NOALLOC_ERR_CUDA;
  {
    const int warps = 8;
    bwd_dot_kernel<128><<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, s>>>(
        static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(dout), sym.rows, so[0], so[1], so[2],
        sg[0], sg[1], sg[2], B, H, Lq, (int)Lpad);
  }
  BwdParams p;
  p.lse2 = lse2;
  p.dd = sym.rows;
  p.Lq = Lq;
  p.Lk = Lk;
  p.H = H;
  p.Lpad = (int)Lpad;
  p.scale = scale;
  p.scale_log2 = (float)((double)scale * 1.4426950408889634);
  p.status = sym.status;
  p.out = static_cast<__nv_bfloat16*>(dk);
  p.sb = sdk[0];
  p.sl = sdk[1];
  p.sh = sdk[2];
  p.out2 = static_cast<__nv_bfloat16*>(dv);
  p.sb2 = sdv[0];
  p.sl2 = sdv[1];
  p.sh2 = sdv[2];
  const size_t smem_a = sizeof(DkvSmem<128>) + 1024;
  if (cudaFuncSetAttribute(flash_bwd_dkdv_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_a) !=
      cudaSuccess)
    return DMAD_NOALLOC_ERR_CUDA;
  flash_bwd_dkdv_kernel<128><<<dim3((Lk + 127) / 128, H, B), 384, smem_a, s>>>(tq, tk, tv, tg, p);
  p.out = static_cast<__nv_bfloat16*>(dq);
  p.sb = sdq[0];
  p.sl = sdq[1];
  p.sh = sdq[2];
  p.out2 = nullptr;
  const size_t smem_b = sizeof(DqSmem<128>) + 1024;
  if (cudaFuncSetAttribute(flash_bwd_dq_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b) !=
      cudaSuccess)
    return DMAD_NOALLOC_ERR_CUDA;
  flash_bwd_dq_kernel<128><<<dim3((Lq + 127) / 128, H, B), 384, smem_b, s>>>(tq, tk, tv, tg, p);
  if (cudaGetLastError() != cudaSuccess) return DMAD_NOALLOC_ERR_CUDA;
  return DMAD_NOALLOC_OK;
}

extern "C" int dmad_flash_attn_bwd_noalloc_status(void* stream, int* out) {
  using namespace dmad;
  if (out == nullptr) return DMAD_NOALLOC_ERR_ARGS;
  int cur = -1, sdev = -1;
  if (cudaGetDevice(&cur) != cudaSuccess ||
      cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess)
    return DMAD_NOALLOC_ERR_CUDA;
  if (cur != sdev) return DMAD_NOALLOC_ERR_ARGS;
  // host code names the status word only through the symbol API (the name is a host-side stand-in)
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_noalloc_status, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return DMAD_NOALLOC_ERR_CUDA;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return DMAD_NOALLOC_ERR_CUDA;
  *out = v;
  return DMAD_NOALLOC_OK;
}

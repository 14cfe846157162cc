// Persistent tcgen05 GEMM for sm_100a with a LoRA K-extension and fused epilogues.
//
//   D[M, N] = act( alpha * (A[M, K] B[N, K]^T + A2[M, K2] B2[N, K2]^T) + bias[N] )      (bf16 out)
//
// A2 / B2 are optional extra K panels.  The LoRA-fused linear uses them as
//   Y = X W^T + s (X A^T) (B o mask)^T = [X | s X A^T] [W | B o mask]^T,
// so the adapter costs one extra 128-wide K panel of the same GEMM instead of two more GEMMs and
// an add (the reference runs cuBLAS for W plus PEFT's two LoRA GEMMs: nn.Linear + peft LoraLayer,
// train/h3/lightx2v_train/model_zoo/base.py:16-114; the rank-128 LoRA student of the 14B config).
// X A^T itself is this kernel with N = r (epilogue scale s).
//
// Kernel structure (one CTA per SM, persistent over 128 x 256 output tiles):
//   warp 0      TMA producer: 4-stage ring of (A 128x64, B 256x64) bf16 tiles, 128B swizzle
//   warp 1      TMEM owner; one thread issues tcgen05.mma (M=128, N=256, K=16) into one of two
//               256-column fp32 accumulators, so the epilogue of tile i overlaps tile i+1
//   warps 2..5  epilogue: tcgen05.ld (thread = output row), alpha, bias, optional GELU-tanh,
//               bf16 stores
// Every mbarrier wait is bounded (2 s), records a status code and makes all roles leave.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace dmad {

int* device_status_ptr(int device);

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB

struct GemmSmem {
  uint8_t a[kStages][kABytes];
  uint8_t b[kStages][kBBytes];
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct GemmParams {
  __nv_bfloat16* d;
  float* d32;   // split-K: fp32 [M, N] accumulation target (reduced with red.global.add), else null
  int64_t ldd;
  const float* bias;  // fp32 [N] or null
  int M, N, k1_steps, k2_steps;
  int tiles_m, tiles_n, num_tiles;
  int split, ksteps_per_split;  // split-K: tiles x split work items, each a range of K steps
  int a_mn, b_mn;               // operand majorness: 0 = K-major ([rows, K]), 1 = MN-major ([K, rows])
  float alpha;
  int act;  // 0 none, 1 gelu-tanh
  int* status;
};

__device__ __forceinline__ void red_add_v4f(float* dst, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// K-step range [k_begin, k_end) of work item t (split-K splits the K loop of one output tile)
__device__ __forceinline__ void k_range(const GemmParams& p, int t, int& k_begin, int& k_end) {
  const int ks = p.k1_steps + p.k2_steps;
  const int s = t % p.split;
  k_begin = s * p.ksteps_per_split;
  k_end = min(ks, k_begin + p.ksteps_per_split);
}

// Loads one operand tile of `rows` rows x 64 K-elements for K step k: K-major = one box [rows][64];
// MN-major = rows / 64 boxes [64 K][64 rows], each a 128-byte-swizzled 8 KB panel.
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int kcoord, int r0,
                                             int rows, bool mn) {
  if (!mn) {
    tma_load_2d(dst, tm, bar, kcoord, r0);
  } else {
    for (int j = 0; j < rows / 64; ++j) tma_load_2d(dst + j * 8192, tm, bar, r0 + 64 * j, kcoord);
  }
}

// Shared-memory descriptor of sub-step kk (16 K-elements) of an operand tile.
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk, bool mn) {
  return mn ? smem_desc_sw128(base + kk * 2048, 8192, 1024) : smem_desc_sw128(base + kk * 32, 16, 1024);
}

__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& m0, int& n0) {
  t /= p.split;
  // column-major raster within groups of 8 M-tiles: neighbouring CTAs share B (weight) tiles in L2
  constexpr int kGroup = 8;
  const int group = t / (kGroup * p.tiles_n);
  const int first_m = group * kGroup;
  const int gm = min(kGroup, p.tiles_m - first_m);
  const int in = t % (kGroup * p.tiles_n);
  m0 = (first_m + in % gm) * kBM;
  n0 = (in / gm) * kBN;
}

__global__ void __launch_bounds__(192, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
            const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ CUtensorMap tm_b2, GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 128);
    }
    mbar_init(&sm.drain, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    if (p.k2_steps > 0) {
      prefetch_tmap(&tm_a2);
      prefetch_tmap(&tm_b2);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int it = 0;  // global k-step counter (ring position)
      int last_stage = -1;
      uint32_t last_ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int m0, n0, kb, ke;
        tile_coords(p, t, m0, n0);
        k_range(p, t, kb, ke);
        for (int k = kb; k < ke; ++k, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!(ok = mbar_wait(&sm.empty[s], ph ^ 1, kStatusTimeoutEmpty, abort_flag, p.status))) break;
          mbar_arrive_expect_tx(&sm.full[s], kABytes + kBBytes);
          if (k < p.k1_steps) {
            load_operand(sm.a[s], &tm_a, &sm.full[s], k * kBK, m0, kBM, p.a_mn);
            load_operand(sm.b[s], &tm_b, &sm.full[s], k * kBK, n0, kBN, p.b_mn);
          } else {
            const int kk = (k - p.k1_steps) * kBK;
            load_operand(sm.a[s], &tm_a2, &sm.full[s], kk, m0, kBM, p.a_mn);
            load_operand(sm.b[s], &tm_b2, &sm.full[s], kk, n0, kBN, p.b_mn);
          }
          last_stage = s;
          last_ph = ph;
        }
      }
      if (last_stage >= 0) mbar_wait(&sm.full[last_stage], last_ph, kStatusTimeoutTmaFull, nullptr, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      const uint32_t idesc = idesc_bf16_f32(kBM, kBN, p.a_mn != 0, p.b_mn != 0);
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++tl) {
        const int buf = tl & 1;
        const uint32_t acc_ph = (tl >> 1) & 1;
        if (!(ok = mbar_wait(&sm.acc_empty[buf], acc_ph ^ 1, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kBN;
        int kb, ke;
        k_range(p, t, kb, ke);
        for (int k = kb; k < ke; ++k, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!(ok = mbar_wait(&sm.full[s], ph, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
          tc_fence_after();
          const uint32_t aa = smem_u32(sm.a[s]), bb = smem_u32(sm.b[s]);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_ss(d, operand_desc(aa, kk, p.a_mn), operand_desc(bb, kk, p.b_mn), idesc,
                        (k > kb || kk > 0) ? 1u : 0u);
          mma_commit(&sm.empty[s]);
        }
        if (!ok) break;
        mma_commit(&sm.acc_full[buf]);
      }
      if (!ok) *abort_flag = 1;
      mma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, kStatusTimeoutMma, nullptr, p.status);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int wq = warp & 3;  // TMEM lane quarter this warp may access
    const int row = wq * 32 + lane;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    int tl = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      const uint32_t acc_ph = (tl >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.acc_full[buf], acc_ph, kStatusTimeoutMma, abort_flag, p.status)))
        break;
      tc_fence_after();
      int m0, n0;
      tile_coords(p, t, m0, n0);
      const int m = m0 + row;
      __nv_bfloat16* drow = p.d + (int64_t)m * p.ldd + n0;
      int kb, ke;
      k_range(p, t, kb, ke);
      const bool empty = ke <= kb;  // a split past the end of K: nothing was accumulated
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + buf * kBN + c * 32, r);
        tmem_wait_ld();
        const int nc = n0 + c * 32;
        if (p.d32 != nullptr) {  // split-K: alpha-scaled fp32 partial sums reduced into d32
          if (!empty && m < p.M && nc < p.N) {
            float* d32 = p.d32 + (int64_t)m * p.ldd + nc;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (nc + q * 4 < p.N)
                red_add_v4f(d32 + q * 4, __uint_as_float(r[4 * q]) * p.alpha, __uint_as_float(r[4 * q + 1]) * p.alpha,
                            __uint_as_float(r[4 * q + 2]) * p.alpha, __uint_as_float(r[4 * q + 3]) * p.alpha);
          }
          continue;
        }
        if (m < p.M && nc < p.N) {
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float x = __uint_as_float(r[i]) * p.alpha;
            if (p.bias != nullptr) x += (nc + i < p.N) ? p.bias[nc + i] : 0.f;
            if (p.act == 1) x = gelu_tanh(x);
            v[i] = x;
          }
          uint4* dst = reinterpret_cast<uint4*>(drow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (nc + q * 8 < p.N)
              dst[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                                  pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

CUtensorMap make_operand_map(const at::Tensor& x, uint32_t box_rows, bool mn) {
  // K-major x: [rows, K]; MN-major x: [K, rows]; the contiguous dimension is innermost either way
  const uint64_t dims[2] = {(uint64_t)x.size(1), (uint64_t)x.size(0)};
  const uint64_t strides[1] = {(uint64_t)x.stride(0) * 2};
  const uint32_t box[2] = {(uint32_t)kBK, mn ? 64u : box_rows};
  return make_tmap_bf16(x.data_ptr(), 2, dims, strides, box);
}

void check_operand(const at::Tensor& x, const char* name) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2, name, " must be a 2-D CUDA bf16 tensor");
  TORCH_CHECK(x.stride(1) == 1 && x.stride(0) % 8 == 0 && x.size(1) % 8 == 0, name,
              ": the inner dimension must be contiguous, its size and the row stride multiples of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

}  // namespace

size_t gemm_smem_bytes() { return sizeof(GemmSmem) + 1024; }

// d = act(alpha * (A B^T + A2 B2^T) + bias) with A [M, K] / B [N, K] given K-major (as stored) or, with
// a_mn / b_mn, MN-major (stored transposed: a [K, M], b [K, N]); A2 / B2 follow A / B.  split > 1: the K
// loop of every output tile is split over `split` CTAs whose alpha-scaled fp32 partial sums are added into
// d32 [M, N] (zeroed by the caller; no bias or activation); d is then unused.
void gemm_bf16_ex(const at::Tensor& a, const at::Tensor& b, c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2,
                  c10::optional<at::Tensor> bias, c10::optional<at::Tensor> d, c10::optional<at::Tensor> d32,
                  double alpha, int64_t act, bool a_mn, bool b_mn, int64_t split) {
  check_operand(a, "a");
  check_operand(b, "b");
  const int64_t M = a_mn ? a.size(1) : a.size(0), K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0), Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "a and b must share K");
  const bool ext = a2.has_value() && a2->defined();
  int64_t K2 = 0;
  if (ext) {
    TORCH_CHECK(b2.has_value() && b2->defined(), "a2 needs b2");
    check_operand(*a2, "a2");
    check_operand(*b2, "b2");
    const int64_t M2 = a_mn ? a2->size(1) : a2->size(0), N2 = b_mn ? b2->size(1) : b2->size(0);
    K2 = a_mn ? a2->size(0) : a2->size(1);
    const int64_t K2b = b_mn ? b2->size(0) : b2->size(1);
    TORCH_CHECK(M2 == M && N2 == N && K2 == K2b, "a2 / b2 shapes must match a / b");
  }
  TORCH_CHECK(split >= 1, "split >= 1");
  const bool splitk = d32.has_value() && d32->defined();
  TORCH_CHECK(splitk || split == 1, "split > 1 needs the fp32 output d32");
  float* d32p = nullptr;
  __nv_bfloat16* dp = nullptr;
  int64_t ldd = 0;
  if (splitk) {
    TORCH_CHECK(d32->is_cuda() && d32->scalar_type() == at::kFloat && d32->dim() == 2 && d32->size(0) == M &&
                    d32->size(1) == N && d32->stride(1) == 1 && d32->stride(0) % 4 == 0 && N % 4 == 0,
                "d32 must be fp32 [M, N] with contiguous rows (N and row stride multiples of 4)");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(d32->data_ptr()) % 16 == 0, "d32 must be 16-byte aligned");
    TORCH_CHECK(!(bias.has_value() && bias->defined()) && act == 0, "split-K has no bias / activation epilogue");
    d32p = d32->data_ptr<float>();
    ldd = d32->stride(0);
  } else {
    TORCH_CHECK(d.has_value() && d->defined(), "d is required");
    TORCH_CHECK(d->is_cuda() && d->scalar_type() == at::kBFloat16 && d->dim() == 2 && d->size(0) == M &&
                    d->size(1) == N && d->stride(1) == 1 && d->stride(0) % 8 == 0 && N % 8 == 0,
                "d must be bf16 [M, N] with contiguous rows (N and row stride multiples of 8)");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(d->data_ptr()) % 16 == 0, "d must be 16-byte aligned");
    dp = reinterpret_cast<__nv_bfloat16*>(d->data_ptr());
    ldd = d->stride(0);
  }
  const float* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N && bias->is_contiguous(), "bias fp32 [N]");
    bp = bias->data_ptr<float>();
  }
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  CUtensorMap ma = make_operand_map(a, kBM, a_mn), mb = make_operand_map(b, kBN, b_mn);
  CUtensorMap ma2 = ext ? make_operand_map(*a2, kBM, a_mn) : ma, mb2 = ext ? make_operand_map(*b2, kBN, b_mn) : mb;
  GemmParams p;
  p.d = dp;
  p.d32 = d32p;
  p.ldd = ldd;
  p.bias = bp;
  p.M = (int)M;
  p.N = (int)N;
  p.k1_steps = (int)((K + kBK - 1) / kBK);
  p.k2_steps = ext ? (int)((K2 + kBK - 1) / kBK) : 0;
  p.tiles_m = (int)((M + kBM - 1) / kBM);
  p.tiles_n = (int)((N + kBN - 1) / kBN);
  const int ks = p.k1_steps + p.k2_steps;
  TORCH_CHECK(ks > 0, "empty K");
  p.split = (int)std::min<int64_t>(split, ks);
  p.ksteps_per_split = (ks + p.split - 1) / p.split;
  p.num_tiles = p.tiles_m * p.tiles_n * p.split;
  p.a_mn = a_mn ? 1 : 0;
  p.b_mn = b_mn ? 1 : 0;
  p.alpha = (float)alpha;
  p.act = (int)act;
  p.status = device_status_ptr(a.get_device());
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, a.get_device());
  const size_t smem = gemm_smem_bytes();
  C10_CUDA_CHECK(cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int grid = std::min(p.num_tiles, sms);
  gemm_kernel<<<grid, 192, smem, at::cuda::getCurrentCUDAStream()>>>(ma, mb, ma2, mb2, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// d = act(alpha * (a @ b^T + a2 @ b2^T) + bias); a [M, K], b [N, K], a2 [M, K2], b2 [N, K2], d [M, N].
void gemm_bf16(const at::Tensor& a, const at::Tensor& b, c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2,
               c10::optional<at::Tensor> bias, at::Tensor& d, double alpha, int64_t act) {
  gemm_bf16_ex(a, b, a2, b2, bias, d, c10::nullopt, alpha, act, false, false, 1);
}

}  // namespace dmad

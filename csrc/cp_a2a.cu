// Ulysses context-parallel all-to-all over NVLink peer memory, fused with the work around it.
//
// Layouts (cp ranks, rank r holds the contiguous token slice [r*Ll, (r+1)*Ll) of every sample;
// H heads of hd = 128 channels, Hl = H / cp heads per rank after the exchange):
//   sequence-sharded rows  [B*Ll, ld] bf16, head h at columns [h*hd, (h+1)*hd)
//   head-sharded slots     [B, L, n, Hl, hd] bf16 (n = 3 for q|k|v, 1 otherwise), L = cp * Ll
// Every store below goes to a peer's symmetric slot (or this GPU's own) through plain
// st.global.v4; completion is published by the bounded barrier that follows each push
// (collectives.cu), never by a spin inside these kernels.
//
// * cp_qkv_push: RMSNorm over the full hidden size of q and k, interleaved RoPE at the row's
//   global position, and the scatter of q, k, v to the rank that owns each head -- the
//   reference's qk-norm + rope + `_SeqAllToAllQKV` (train/wan/rcm/networks/wan2pt1.py:227-289,
//   train/wan/rcm/utils/a2a_cp.py:121-143) in one pass over the projection output.
// * cp_seq_to_head: plain sequence->head exchange of an [B*Ll, D] tensor (gradient of the
//   attention output in backward).
// * cp_head_to_seq: head->sequence exchange of [B, L, n, Hl, hd] into the owners' [B*Ll, ld]
//   rows at this rank's head columns (attention output, or dq|dk|dv in backward; the reverse
//   all-to-all of a2a_cp.py:108-118 / :141-143).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace dmad {

int* device_status_ptr(int device);

namespace {

constexpr int kMaxCp = 16;

struct PeerTable {
  int64_t p[kMaxCp];
};

// grid (B*Ll, 3); one block per (row, q|k|v)
template <int kMaxVec, int kTh>
__global__ void __launch_bounds__(kTh)
cp_qkv_push_kernel(const __nv_bfloat16* __restrict__ src, int64_t ss, PeerTable dst, const float* __restrict__ wq,
                   const float* __restrict__ wk, const float* __restrict__ cosT, const float* __restrict__ sinT,
                   float* __restrict__ rstd_q, float* __restrict__ rstd_k, int Ll, int L, int D, int hd, int Hl,
                   int rank, float eps, int cp, int* status) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const int which = blockIdx.y;
  const int b = (int)(r / Ll), lr = (int)(r % Ll);
  const int64_t grow = (int64_t)b * L + (int64_t)rank * Ll + lr;  // global row of the slot
  const int nvec = D >> 3;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(src + r * ss + which * D);
  float v[kMaxVec][8];
  float rstd = 1.f;
  if (which < 2) {
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
    rstd = rsqrtf(block_sum(s, red) / D + eps);
  } else {
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = threadIdx.x + i * kTh;
      if (c < nvec) bf16x8_to_float(xr[c], v[i]);
    }
  }
  const float* w = which == 0 ? wq : wk;
  const int64_t tr = (int64_t)lr * (hd >> 1);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * kTh;
    if (c < nvec) {
      const int col = c * 8;
      const int h = col / hd, hl = h % Hl, peer = h / Hl;
      float o[8];
      if (which < 2) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float a0 = v[i][e] * rstd * w[col + e];
          const float a1 = v[i][e + 1] * rstd * w[col + e + 1];
          const int pi = ((col + e) % hd) >> 1;
          const float cs = cosT[tr + pi], sn = sinT[tr + pi];
          o[e] = a0 * cs - a1 * sn;
          o[e + 1] = a1 * cs + a0 * sn;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = v[i][e];
      }
      __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst.p[peer]) +
                         ((grow * 3 + which) * Hl + hl) * (int64_t)hd + (col % hd);
      DMAD_GUARD(peer < cp && grow < (int64_t)(r / Ll + 1) * L, status)
      *reinterpret_cast<bf16x8*>(d) = float_to_bf16x8(o);
    }
  }
  if (which < 2 && threadIdx.x == 0) (which == 0 ? rstd_q : rstd_k)[r] = rstd;
}

// one thread per 8 elements of the local [B*Ll, n*D] source
__global__ void cp_seq_to_head_kernel(const __nv_bfloat16* __restrict__ src, int64_t ss, PeerTable dst, int64_t R,
                                      int Ll, int L, int D, int n, int hd, int Hl, int rank, int cp, int* status) {
  const int per_row = n * D / 8;
  const int64_t total = R * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row;
    const int cc = (int)(i % per_row) * 8;
    const int which = cc / D, col = cc % D;
    const int b = (int)(r / Ll), lr = (int)(r % Ll);
    const int64_t grow = (int64_t)b * L + (int64_t)rank * Ll + lr;
    const int h = col / hd, hl = h % Hl, peer = h / Hl;
    const bf16x8 x = *reinterpret_cast<const bf16x8*>(src + r * ss + cc);
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst.p[peer]) +
                       ((grow * n + which) * Hl + hl) * (int64_t)hd + (col % hd);
    DMAD_GUARD(peer < cp, status)
    *reinterpret_cast<bf16x8*>(d) = x;
  }
}

// src: this rank's [B, L, n, Hl, hd] (strides given per n-slot: the n slots may be separate
// tensors); one thread per 8 elements; row (b, g) goes to rank g / Ll, local row b*Ll + g % Ll,
// columns which*D + (rank*Hl + hl)*hd of a row of stride ld.
struct HeadSrc {
  int64_t p[3];
  int64_t sb, sl, sh;  // element strides of each [B, L, Hl, hd] source
};

__global__ void cp_head_to_seq_kernel(HeadSrc src, PeerTable dst, int64_t ld, int B, int Ll, int L, int D, int n,
                                      int hd, int Hl, int rank, int cp, int* status) {
  const int per_row = n * Hl * hd / 8;
  const int64_t total = (int64_t)B * L * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gr = i / per_row;  // b*L + g
    const int cc = (int)(i % per_row) * 8;
    const int which = cc / (Hl * hd), rem = cc % (Hl * hd);
    const int hl = rem / hd, e = rem % hd;
    const int b = (int)(gr / L), g = (int)(gr % L);
    const int peer = g / Ll, lr = g % Ll;
    const __nv_bfloat16* s =
        reinterpret_cast<const __nv_bfloat16*>(src.p[which]) + b * src.sb + (int64_t)g * src.sl + hl * src.sh + e;
    const bf16x8 x = *reinterpret_cast<const bf16x8*>(s);
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst.p[peer]) + ((int64_t)b * Ll + lr) * ld + which * D +
                       (int64_t)(rank * Hl + hl) * hd + e;
    DMAD_GUARD(peer < cp && which < n, status)
    *reinterpret_cast<bf16x8*>(d) = x;
  }
}

PeerTable make_table(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(!ptrs.empty() && ptrs.size() <= (size_t)kMaxCp, "cp group size must be 1..", kMaxCp);
  PeerTable t{};
  for (size_t i = 0; i < ptrs.size(); ++i) {
    TORCH_CHECK(ptrs[i] % 16 == 0, "peer slot must be 16-byte aligned");
    t.p[i] = ptrs[i];
  }
  return t;
}

int grid_1d(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)); }

}  // namespace

// src: [B*Ll, >=3D] local projection (q|k|v); dst: peer addresses of the [B, L, 3, Hl, hd] slots.
void cp_qkv_push(const at::Tensor& src, std::vector<int64_t> dst, const at::Tensor& wq, const at::Tensor& wk,
                 const at::Tensor& cosT, const at::Tensor& sinT, at::Tensor& rstd_q, at::Tensor& rstd_k, int64_t B,
                 int64_t D, int64_t hd, int64_t rank, double eps) {
  const int cp = (int)dst.size();
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(1) == 1 &&
                  src.stride(0) % 8 == 0 && src.size(1) >= 3 * D,
              "src must be bf16 [B*Ll, >=3D] with contiguous rows");
  TORCH_CHECK(D % hd == 0 && hd % 8 == 0 && (D / hd) % cp == 0 && D <= 8192, "heads must divide over the cp group");
  TORCH_CHECK(src.size(0) % B == 0, "rows must be B * Ll");
  TORCH_CHECK(wq.scalar_type() == at::kFloat && wk.scalar_type() == at::kFloat, "norm weights must be fp32");
  const int64_t R = src.size(0);
  const int Ll = (int)(R / B);
  TORCH_CHECK(cosT.is_contiguous() && sinT.is_contiguous() && cosT.size(0) >= Ll && cosT.size(1) == hd / 2,
              "rope tables must be [Ll, hd/2] for the local rows");
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  PeerTable t = make_table(dst);
  dim3 grid((unsigned)R, 3);
  DMAD_ROW_DISPATCH(D / 8, [&] {
    cp_qkv_push_kernel<VEC, TH><<<grid, TH, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0), t, wq.data_ptr<float>(),
        wk.data_ptr<float>(), cosT.data_ptr<float>(), sinT.data_ptr<float>(), rstd_q.data_ptr<float>(),
        rstd_k.data_ptr<float>(), Ll, Ll * cp, (int)D, (int)hd, (int)(D / hd / cp), (int)rank, (float)eps, cp,
        device_status_ptr(src.get_device()));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// src: [B*Ll, >= n*D] local rows; dst: peer addresses of [B, L, n, Hl, hd] slots.
void cp_seq_to_head(const at::Tensor& src, std::vector<int64_t> dst, int64_t B, int64_t D, int64_t n, int64_t hd,
                    int64_t rank) {
  const int cp = (int)dst.size();
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(1) == 1 &&
                  src.stride(0) % 8 == 0 && src.size(1) >= n * D,
              "src must be bf16 [B*Ll, >=n*D]");
  TORCH_CHECK(D % hd == 0 && (D / hd) % cp == 0 && hd % 8 == 0 && src.size(0) % B == 0, "bad cp layout");
  const int64_t R = src.size(0);
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  const int Ll = (int)(R / B);
  cp_seq_to_head_kernel<<<grid_1d(R * n * D / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.stride(0), make_table(dst), R, Ll, Ll * cp,
      (int)D, (int)n, (int)hd, (int)(D / hd / cp), (int)rank, cp, device_status_ptr(src.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// srcs: n local [B, L, Hl, hd] bf16 views with identical strides; dst: peer addresses of
// [B*Ll, ld] row buffers; this rank's heads land at columns which*D + rank*Hl*hd.
void cp_head_to_seq(std::vector<at::Tensor> srcs, std::vector<int64_t> dst, int64_t ld, int64_t D, int64_t rank) {
  const int cp = (int)dst.size();
  const int n = (int)srcs.size();
  TORCH_CHECK(n >= 1 && n <= 3, "1..3 sources");
  const at::Tensor& s0 = srcs[0];
  TORCH_CHECK(s0.is_cuda() && s0.scalar_type() == at::kBFloat16 && s0.dim() == 4 && s0.stride(3) == 1, "bad source");
  const int B = s0.size(0), L = s0.size(1), Hl = s0.size(2), hd = s0.size(3);
  TORCH_CHECK(L % cp == 0 && Hl * cp * hd == D && hd % 8 == 0 && ld % 8 == 0 && ld >= n * D, "bad cp layout");
  HeadSrc hs{};
  for (int i = 0; i < n; ++i) {
    TORCH_CHECK(srcs[i].sizes() == s0.sizes() && srcs[i].strides() == s0.strides(), "sources must share layout");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(srcs[i].data_ptr()) % 16 == 0, "sources must be 16-byte aligned");
    hs.p[i] = reinterpret_cast<int64_t>(srcs[i].data_ptr());
  }
  TORCH_CHECK(s0.stride(0) % 8 == 0 && s0.stride(1) % 8 == 0 && s0.stride(2) % 8 == 0, "strides must be x8");
  hs.sb = s0.stride(0);
  hs.sl = s0.stride(1);
  hs.sh = s0.stride(2);
  c10::cuda::CUDAGuard guard(s0.device());
  const int64_t total = (int64_t)B * L * n * Hl * hd / 8;
  if (total == 0) return;
  cp_head_to_seq_kernel<<<grid_1d(total), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      hs, make_table(dst), ld, B, L / cp, L, (int)D, n, hd, Hl, (int)rank, cp, device_status_ptr(s0.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmad

// Parameter all-gather over NVLink peer memory for sharded (FSDP-style) block weights.
//
// Every rank holds the shard [r * len, (r + 1) * len) of a block's flat bf16 weight vector in a
// symmetric buffer; this kernel pulls all shards into a local gathered buffer with 16-byte peer
// loads (rank order staggered per CTA so the ranks do not all read one GPU at a time).  The
// shards are written once at setup (frozen weights), so no flag protocol is needed per gather.
// Parity target: FSDP2's per-block parameter all-gather (train/wan/rcm/models/
// t2v_model_distill_rcm.py:175-195, train/h3/lightx2v_train/runtime/fsdp.py:60-85).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace dmad {

int* device_status_ptr(int device);

namespace {

constexpr int kMaxRanks = 16;

struct Shards {
  int64_t p[kMaxRanks];
};
static_assert(sizeof(Shards) == 8 * 16, "peer table");

__global__ void fsdp_gather_kernel(Shards src, uint4* __restrict__ dst, int world, int64_t len_vec,
                                   int64_t n_vec, int* status) {
  const int64_t total = len_vec * world;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    // (chunk, j) -> (rank, j) must be a bijection over the whole grid-stride range: the rank rotates
    // with the 64 KB segment of j, so concurrent CTAs spread their loads over the peers while every
    // (rank, j) is copied exactly once
    const int64_t chunk = i / len_vec;
    const int64_t j = i % len_vec;
    const int r = (int)((chunk + (j >> 12)) % world);
    const int64_t g = (int64_t)r * len_vec + j;  // element-vector index in the gathered buffer
    DMAD_GUARD(r < world && j < len_vec, status)
    if (g < n_vec) dst[g] = reinterpret_cast<const uint4*>(src.p[r])[j];
  }
}

// acc[j] (+)= sum over ranks r (in rank order) of slot_r[off + j], j < len: every rank's bf16 gradient of
// one block sits in its symmetric grad slot; this rank pulls the slice it owns from every peer with
// 16-byte loads and sums in fp32.  The rank order is fixed, so the result does not depend on timing.
__global__ void fsdp_reduce_scatter_kernel(Shards slots, float* __restrict__ acc, int world, int64_t off,
                                           int64_t len_vec, bool accumulate, int* status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len_vec; i += (int64_t)gridDim.x * blockDim.x) {
    float s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] = 0.f;
    for (int r = 0; r < world; ++r) {
      const uint4 v = reinterpret_cast<const uint4*>(slots.p[r] + off * 2)[i];  // off in bf16 elements
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[2 * e] += __uint_as_float(w[e] << 16);
        s[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
      }
    }
    float4* out = reinterpret_cast<float4*>(acc) + 2 * i;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (accumulate) {
      a = out[0];
      b = out[1];
    }
    out[0] = make_float4(a.x + s[0], a.y + s[1], a.z + s[2], a.w + s[3]);
    out[1] = make_float4(b.x + s[4], b.y + s[5], b.z + s[6], b.w + s[7]);
  }
}

}  // namespace

// acc (fp32, len elements) (+)= sum over ranks of the bf16 elements [off, off + len) of every rank's slot.
void fsdp_reduce_scatter(std::vector<int64_t> slot_ptrs, at::Tensor& acc, int64_t off, int64_t len, bool accumulate) {
  const int world = (int)slot_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "1..16 ranks");
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.numel() >= len,
              "acc must be a contiguous fp32 CUDA tensor of at least len elements");
  TORCH_CHECK(len % 8 == 0 && off % 8 == 0, "off / len must be multiples of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(acc.data_ptr()) % 16 == 0, "acc must be 16-byte aligned");
  Shards s{};
  for (int i = 0; i < world; ++i) {
    TORCH_CHECK(slot_ptrs[i] % 16 == 0, "slots must be 16-byte aligned");
    s.p[i] = slot_ptrs[i];
  }
  if (len == 0) return;
  c10::cuda::CUDAGuard guard(acc.device());
  const int64_t len_vec = len / 8;
  const int blocks = (int)std::min<int64_t>((len_vec + 255) / 256, 148 * 8);
  fsdp_reduce_scatter_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      s, acc.data_ptr<float>(), world, off, len_vec, accumulate, device_status_ptr(acc.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dst: local bf16 buffer of >= numel elements; shard_ptrs: every rank's shard address (len elements each).
void fsdp_gather(std::vector<int64_t> shard_ptrs, at::Tensor& dst, int64_t len, int64_t numel) {
  const int world = (int)shard_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "1..16 ranks");
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == at::kBFloat16 && dst.is_contiguous() && dst.numel() >= numel,
              "dst must be a contiguous bf16 CUDA tensor of at least numel elements");
  TORCH_CHECK(len % 8 == 0 && numel % 8 == 0 && numel <= len * world, "len / numel must be multiples of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0, "dst must be 16-byte aligned");
  Shards s{};
  for (int i = 0; i < world; ++i) {
    TORCH_CHECK(shard_ptrs[i] % 16 == 0, "shards must be 16-byte aligned");
    s.p[i] = shard_ptrs[i];
  }
  if (numel == 0) return;
  c10::cuda::CUDAGuard guard(dst.device());
  const int64_t len_vec = len / 8, total = len_vec * world;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  fsdp_gather_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      s, reinterpret_cast<uint4*>(dst.data_ptr()), world, len_vec, numel / 8, device_status_ptr(dst.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Copy engine transfer of nbytes from an address of another GPU's (mapped) memory into dst on the
// current stream: the ring-attention key/value blocks move without occupying SMs.
void peer_copy(at::Tensor& dst, int64_t src_ptr, int64_t nbytes) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && (int64_t)(dst.numel() * dst.element_size()) >= nbytes,
              "dst must be a contiguous CUDA tensor of at least nbytes");
  if (nbytes == 0) return;
  c10::cuda::CUDAGuard guard(dst.device());
  C10_CUDA_CHECK(cudaMemcpyAsync(dst.data_ptr(), reinterpret_cast<const void*>(src_ptr), (size_t)nbytes,
                                 cudaMemcpyDeviceToDevice, at::cuda::getCurrentCUDAStream()));
}

// Copy engine transfer of src into an address of another GPU's (mapped) memory.
void peer_copy_to(int64_t dst_ptr, const at::Tensor& src, int64_t nbytes) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous() && (int64_t)(src.numel() * src.element_size()) >= nbytes,
              "src must be a contiguous CUDA tensor of at least nbytes");
  if (nbytes == 0) return;
  c10::cuda::CUDAGuard guard(src.device());
  C10_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<void*>(dst_ptr), src.data_ptr(), (size_t)nbytes,
                                 cudaMemcpyDeviceToDevice, at::cuda::getCurrentCUDAStream()));
}

}  // namespace dmad

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

}  // namespace

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

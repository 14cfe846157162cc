// Collectives fused with compute over NVLink / NVSwitch peer memory (sm_100a).
//
// Peer buffers come from one symmetric allocation per tensor (every rank maps every other rank's
// copy); the host passes their addresses in rank order.  Remote traffic is either plain
// ld/st.global through those peer mappings (P2P) or `multimem` loads / stores through the
// NVSwitch multicast address of the allocation (NVLS: the switch sums on the way in and
// replicates on the way out).  No TMA load and no multicast TMA touches another GPU's memory.
//
// * symm_barrier: every rank optionally stores a float payload into slot [rank] of every peer's
//   slot array, then writes `epoch` into flag [rank] of every peer (system-scope release) and
//   waits, bounded by a globaltimer deadline, until all of its own flags reach `epoch` (acquire).
//   A wait that runs out records kStatusTimeoutPeer and returns; the kernels below then skip their
//   update so that no rank writes inconsistent weights.
// * dp_sumsq: sum of squares of this rank's shard of the rank-averaged gradient (for clipping by
//   the global norm; the partial travels to the peers as a barrier payload).
// * dp_adamw: the data-parallel optimiser step as one kernel.  Rank r owns the shard
//   [off, off + len) of the flat parameter vector.  Each thread gathers the gradient of its 8
//   elements from every rank (the reduce-scatter), averages, applies AdamW to the fp32 master shard
//   (decoupled weight decay, bias correction, optional clipping scale, optional EMA of the
//   weights), and stores the new weights into every rank's parameter buffer (the all-gather).
//   Parity target: the reference's FSDP2 gradient reduce-scatter + FusedAdam(master_weights) step
//   + parameter all-gather (train/wan/rcm/utils/fused_adam_dtensor.py:29-416; FSDP2 wrapping in
//   train/wan/rcm/models/t2v_model_distill_rcm.py:175-195).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"
#include "sm100.cuh"

namespace dmad {

int* device_status_ptr(int device);

namespace {

constexpr int kMaxWorld = 16;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// ------------------------------------------------------------------------------------ barrier
// Layout of the symmetric sync buffer of every rank: int32 flags[world], then float slots[world].
__global__ void symm_barrier_kernel(const int64_t* __restrict__ buf_ptrs, int rank, int world, int epoch,
                                    const float* __restrict__ payload, unsigned long long timeout_ns, int* status) {
  const int p = threadIdx.x;
  if (p < world) {
    int* peer = reinterpret_cast<int*>(buf_ptrs[p]);
    if (payload != nullptr) reinterpret_cast<float*>(peer + world)[rank] = *payload;
    __threadfence_system();
    st_release_sys(peer + rank, epoch);
  }
  __syncthreads();
  if (p < world) {
    const int* mine = reinterpret_cast<const int*>(buf_ptrs[rank]) + p;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(mine) < epoch) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_status(status, kStatusTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------ 8-wide I/O
template <typename T>
struct Io8;

template <>
struct Io8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&f)[8]) {
    bf16x8_to_float(*reinterpret_cast<const bf16x8*>(p), f);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&f)[8]) {
    *reinterpret_cast<bf16x8*>(p) = float_to_bf16x8(f);
  }
  // Sum over every rank through the switch (fp32 accumulation, bf16 result).
  static __device__ __forceinline__ void mc_load_sum(uint64_t mc, float (&f)[8]) {
    bf16x8 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(mc)
                 : "memory");
    bf16x8_to_float(v, f);
  }
  static __device__ __forceinline__ void mc_store(uint64_t mc, const float (&f)[8]) {
    const bf16x8 v = float_to_bf16x8(f);
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.w[0]),
                 "r"(v.w[1]), "r"(v.w[2]), "r"(v.w[3])
                 : "memory");
  }
};

template <>
struct Io8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&f)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
  static __device__ __forceinline__ void mc_load_sum(uint64_t mc, float (&f)[8]) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                   : "=f"(f[4 * h]), "=f"(f[4 * h + 1]), "=f"(f[4 * h + 2]), "=f"(f[4 * h + 3])
                   : "l"(mc + 16 * h)
                   : "memory");
  }
  static __device__ __forceinline__ void mc_store(uint64_t mc, const float (&f)[8]) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
      asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + 16 * h),
                   "f"(f[4 * h]), "f"(f[4 * h + 1]), "f"(f[4 * h + 2]), "f"(f[4 * h + 3])
                   : "memory");
  }
};

struct DpArgs {
  int64_t grads[kMaxWorld];   // peer addresses of the flat gradient buffer (P2P mode)
  int64_t params[kMaxWorld];  // peer addresses of the flat parameter buffer (P2P mode)
  uint64_t mc_grads, mc_params;  // multicast addresses (NVLS mode; 0 = P2P)
  float* master;
  float* m;
  float* v;
  float* ema;
  const float* slots;  // clipping: per-rank sums of squares (local sync buffer), or null
  const int* status;
  int64_t off, len;  // shard in elements (multiples of 8)
  int world;
  int force_finite;  // replace non-finite averaged gradients by 0 (GradClip(force_finite))
  float inv_world, lr, b1, b2, eps, wd, step_size, inv_sqrt_bc2, ema_beta, max_norm;
};

template <typename T>
__device__ __forceinline__ void gather_avg(const DpArgs& a, int64_t e, float (&g)[8]) {
  if (a.mc_grads != 0) {
    Io8<T>::mc_load_sum(a.mc_grads + e * sizeof(T), g);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = 0.f;
    // start at a different peer on every rank so that the ranks do not all read one GPU at a time
    for (int j = 0; j < a.world; ++j) {
      int p = j + (int)(a.off / a.len);
      p = p >= a.world ? p - a.world : p;
      float t[8];
      Io8<T>::load(reinterpret_cast<const T*>(a.grads[p]) + e, t);
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i] += t[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    g[i] *= a.inv_world;
    if (a.force_finite && !isfinite(g[i])) g[i] = 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) dp_sumsq_kernel(DpArgs a, float* __restrict__ acc) {
  if (ld_volatile(a.status) != 0) return;
  __shared__ float red[32];
  float s = 0.f;
  const int64_t nvec = a.len >> 3;
  for (int64_t vi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; vi < nvec; vi += (int64_t)gridDim.x * blockDim.x) {
    float g[8];
    gather_avg<T>(a, a.off + vi * 8, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += g[i] * g[i];
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) atomicAdd(acc, s);
}

template <typename T>
__global__ void __launch_bounds__(256) dp_adamw_kernel(DpArgs a) {
  if (ld_volatile(a.status) != 0) return;  // a barrier ran out: leave every weight as it was
  float scale = 1.f;
  if (a.slots != nullptr) {
    float tot = 0.f;
    for (int p = 0; p < a.world; ++p) tot += a.slots[p];
    const float n = sqrtf(tot);
    scale = isfinite(n) ? fminf(1.f, a.max_norm / (n + 1e-6f)) : 0.f;
  }
  const int64_t nvec = a.len >> 3;
  for (int64_t vi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; vi < nvec; vi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = a.off + vi * 8;
    float g[8];
    gather_avg<T>(a, e, g);
    const int64_t s = vi * 8;  // index inside the shard
    float w8[8], m8[8], v8[8];
    Io8<float>::load(a.master + s, w8);
    Io8<float>::load(a.m + s, m8);
    Io8<float>::load(a.v + s, v8);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gi = g[i] * scale;
      float w = w8[i] * (1.f - a.lr * a.wd);
      m8[i] = a.b1 * m8[i] + (1.f - a.b1) * gi;
      v8[i] = a.b2 * v8[i] + (1.f - a.b2) * gi * gi;
      w -= a.step_size * m8[i] / (sqrtf(v8[i]) * a.inv_sqrt_bc2 + a.eps);
      w8[i] = w;
    }
    Io8<float>::store(a.master + s, w8);
    Io8<float>::store(a.m + s, m8);
    Io8<float>::store(a.v + s, v8);
    if (a.ema != nullptr) {
      float e8[8];
      Io8<float>::load(a.ema + s, e8);
#pragma unroll
      for (int i = 0; i < 8; ++i) e8[i] = a.ema_beta * e8[i] + (1.f - a.ema_beta) * w8[i];
      Io8<float>::store(a.ema + s, e8);
    }
    if (a.mc_params != 0) {
      Io8<T>::mc_store(a.mc_params + e * sizeof(T), w8);
    } else {
      for (int j = 0; j < a.world; ++j) {
        int p = j + (int)(a.off / a.len);
        p = p >= a.world ? p - a.world : p;
        Io8<T>::store(reinterpret_cast<T*>(a.params[p]) + e, w8);
      }
    }
  }
}

DpArgs make_args(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs, int64_t mc_grads,
                 int64_t mc_params, int64_t elem_size, int64_t off, int64_t len, int device, bool force_finite) {
  const int world = (int)grad_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxWorld && (int)param_ptrs.size() == world, "bad world size ", world);
  TORCH_CHECK(off % 8 == 0 && len % 8 == 0 && len > 0, "shard offset / length must be positive multiples of 8");
  TORCH_CHECK(off % len == 0 && off / len < world, "shard offset must be rank * len");
  DpArgs a{};
  for (int p = 0; p < world; ++p) {
    TORCH_CHECK(grad_ptrs[p] % 16 == 0 && param_ptrs[p] % 16 == 0, "peer buffers must be 16-byte aligned");
    a.grads[p] = grad_ptrs[p];
    a.params[p] = param_ptrs[p];
  }
  TORCH_CHECK(mc_grads % 16 == 0 && mc_params % 16 == 0, "multicast addresses must be 16-byte aligned");
  TORCH_CHECK((mc_grads == 0) == (mc_params == 0), "multicast needs both the gradient and the parameter buffer");
  a.mc_grads = (uint64_t)mc_grads;
  a.mc_params = (uint64_t)mc_params;
  a.off = off;
  a.len = len;
  a.world = world;
  a.inv_world = 1.f / world;
  a.status = device_status_ptr(device);
  a.force_finite = force_finite ? 1 : 0;
  (void)elem_size;
  return a;
}

int grid_for(int64_t len) { return (int)std::min<int64_t>((len / 8 + 255) / 256, 148 * 8); }

}  // namespace

// buf_ptrs: int64 CUDA tensor [world] with every rank's address of the symmetric sync buffer
// (int32 flags[world] followed by float slots[world]); payload: optional one-float CUDA tensor.
void symm_barrier(const at::Tensor& buf_ptrs, int64_t rank, int64_t epoch, c10::optional<at::Tensor> payload,
                  double timeout_s) {
  TORCH_CHECK(buf_ptrs.is_cuda() && buf_ptrs.scalar_type() == at::kLong && buf_ptrs.dim() == 1,
              "buf_ptrs must be an int64 vector on the device");
  const int64_t world = buf_ptrs.numel();
  TORCH_CHECK(world >= 1 && world <= 1024 && rank >= 0 && rank < world, "bad rank / world");
  TORCH_CHECK(epoch > 0 && epoch < (1ll << 31), "epoch out of range");
  const float* pl = nullptr;
  if (payload.has_value() && payload->defined()) {
    TORCH_CHECK(payload->is_cuda() && payload->scalar_type() == at::kFloat && payload->numel() >= 1, "bad payload");
    pl = payload->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(buf_ptrs.device());
  symm_barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, at::cuda::getCurrentCUDAStream()>>>(
      buf_ptrs.data_ptr<int64_t>(), (int)rank, (int)world, (int)epoch, pl,
      (unsigned long long)(timeout_s * 1e9), device_status_ptr(buf_ptrs.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// acc: one-float CUDA tensor (zeroed by the caller) that receives this rank's partial sum of squares.
void dp_sumsq(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs, int64_t mc_grads, int64_t mc_params,
              int64_t elem_size, int64_t off, int64_t len, at::Tensor& acc, bool force_finite) {
  TORCH_CHECK(acc.is_cuda() && acc.scalar_type() == at::kFloat, "acc must be a float CUDA tensor");
  c10::cuda::CUDAGuard guard(acc.device());
  DpArgs a = make_args(grad_ptrs, param_ptrs, mc_grads, mc_params, elem_size, off, len, acc.get_device(), force_finite);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (elem_size == 2)
    dp_sumsq_kernel<__nv_bfloat16><<<grid_for(len), 256, 0, stream>>>(a, acc.data_ptr<float>());
  else if (elem_size == 4)
    dp_sumsq_kernel<float><<<grid_for(len), 256, 0, stream>>>(a, acc.data_ptr<float>());
  else
    TORCH_CHECK(false, "unsupported element size ", elem_size);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// master / exp_avg / exp_avg_sq (/ ema): fp32 shard state of `len` elements starting at `off`.
// slots: optional float CUDA tensor [world] of the ranks' sums of squares (enables clipping to max_norm).
void dp_adamw(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs, int64_t mc_grads, int64_t mc_params,
              int64_t elem_size, at::Tensor& master, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
              c10::optional<at::Tensor> ema, int64_t off, int64_t len, double lr, double beta1, double beta2,
              double eps, double weight_decay, int64_t step, double ema_beta, c10::optional<at::Tensor> slots,
              double max_norm, bool force_finite) {
  for (const at::Tensor* t : {&master, &exp_avg, &exp_avg_sq}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() >= len,
                "shard state must be contiguous fp32 CUDA tensors of at least len elements");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "shard state must be 16-byte aligned");
  }
  c10::cuda::CUDAGuard guard(master.device());
  DpArgs a = make_args(grad_ptrs, param_ptrs, mc_grads, mc_params, elem_size, off, len, master.get_device(),
                       force_finite);
  a.master = master.data_ptr<float>();
  a.m = exp_avg.data_ptr<float>();
  a.v = exp_avg_sq.data_ptr<float>();
  a.ema = nullptr;
  if (ema.has_value() && ema->defined()) {
    TORCH_CHECK(ema->scalar_type() == at::kFloat && ema->numel() >= len && ema->is_contiguous(), "bad ema shard");
    a.ema = ema->data_ptr<float>();
  }
  a.slots = nullptr;
  if (slots.has_value() && slots->defined()) {
    TORCH_CHECK(slots->is_cuda() && slots->scalar_type() == at::kFloat && slots->numel() >= a.world, "bad slots");
    a.slots = slots->data_ptr<float>();
  }
  const double bc1 = 1.0 - std::pow(beta1, (double)step), bc2 = 1.0 - std::pow(beta2, (double)step);
  a.lr = (float)lr;
  a.b1 = (float)beta1;
  a.b2 = (float)beta2;
  a.eps = (float)eps;
  a.wd = (float)weight_decay;
  a.step_size = (float)(lr / (bc1 > 0 ? bc1 : 1.0));
  a.inv_sqrt_bc2 = (float)(1.0 / std::sqrt(bc2 > 0 ? bc2 : 1.0));
  a.ema_beta = (float)ema_beta;
  a.max_norm = (float)max_norm;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (elem_size == 2)
    dp_adamw_kernel<__nv_bfloat16><<<grid_for(len), 256, 0, stream>>>(a);
  else if (elem_size == 4)
    dp_adamw_kernel<float><<<grid_for(len), 256, 0, stream>>>(a);
  else
    TORCH_CHECK(false, "unsupported element size ", elem_size);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmad

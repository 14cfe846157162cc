// Multi-tensor optimiser kernels (sm_100a).
//
// fused_adamw: one launch updates every tensor of a parameter group:
//   fp32 master weight, first/second moments (decoupled weight decay, bias
//   correction = torch.optim.AdamW semantics), optional bf16 working copy of
//   the weight, and an optional fp32 EMA copy (ema = b*ema + (1-b)*w), which
//   folds the reference's separate EMA pass
//   (train/wan/rcm/utils/dtensor_helper.py:43-51, minimax_h3_dmad_trainer.py:458-480)
//   into the optimiser.  Gradients may be bf16 or fp32 and are multiplied by a
//   device-side scale (gradient clipping without a host round trip).
// Parity target: the reference's FusedAdam / MasterWeightAdamW
// (train/wan/rcm/utils/fused_adam_dtensor.py:29-416).
// multi_sumsq: sum of squares over a tensor list (gradient-norm clipping).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "common.cuh"

namespace dmad {
namespace {

constexpr int kChunk = 16384;

struct TensorEntry {
  float* master;
  float* m;
  float* v;
  const void* grad;
  __nv_bfloat16* lowp;
  float* ema;
  int64_t numel;
};

struct ChunkEntry {
  int tensor;
  int chunk;
};

__global__ void __launch_bounds__(256)
adamw_kernel(const TensorEntry* __restrict__ tensors, const ChunkEntry* __restrict__ chunks, bool grad_bf16, float lr,
             float b1, float b2, float eps, float wd, float bc1, float bc2, const float* __restrict__ grad_scale,
             float ema_beta) {
  const ChunkEntry ce = chunks[blockIdx.x];
  const TensorEntry te = tensors[ce.tensor];
  const int64_t start = (int64_t)ce.chunk * kChunk;
  const int64_t end = min(te.numel, start + kChunk);
  const float gs = grad_scale != nullptr ? *grad_scale : 1.f;
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
    float g = grad_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(te.grad)[i])
                        : reinterpret_cast<const float*>(te.grad)[i];
    g *= gs;
    float w = te.master[i];
    w -= lr * wd * w;
    const float m = b1 * te.m[i] + (1.f - b1) * g;
    const float v = b2 * te.v[i] + (1.f - b2) * g * g;
    te.m[i] = m;
    te.v[i] = v;
    w -= step_size * m / (sqrtf(v) * inv_sqrt_bc2 + eps);
    te.master[i] = w;
    if (te.lowp != nullptr) te.lowp[i] = __float2bfloat16(w);
    if (te.ema != nullptr) te.ema[i] = ema_beta * te.ema[i] + (1.f - ema_beta) * w;
  }
}

__global__ void __launch_bounds__(256)
sumsq_kernel(const TensorEntry* __restrict__ tensors, const ChunkEntry* __restrict__ chunks, bool grad_bf16,
             float* __restrict__ out) {
  __shared__ float red[32];
  const ChunkEntry ce = chunks[blockIdx.x];
  const TensorEntry te = tensors[ce.tensor];
  const int64_t start = (int64_t)ce.chunk * kChunk;
  const int64_t end = min(te.numel, start + kChunk);
  float acc = 0.f;
  for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = grad_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(te.grad)[i])
                              : reinterpret_cast<const float*>(te.grad)[i];
    acc += g * g;
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(out, acc);
}

// Clip factor on the device: scale = min(1, max_norm / (sqrt(sumsq) + 1e-6)); non-finite -> 0.
__global__ void clip_scale_kernel(const float* sumsq, float* scale, float max_norm) {
  const float n = sqrtf(*sumsq);
  float s = max_norm / (n + 1e-6f);
  s = s < 1.f ? s : 1.f;
  if (!isfinite(n)) s = 0.f;
  *scale = s;
}

struct Tables {
  at::Tensor tensors, chunks;
  int nchunks;
};

Tables build_tables(const std::vector<at::Tensor>& master, const std::vector<at::Tensor>& m,
                    const std::vector<at::Tensor>& v, const std::vector<at::Tensor>& grads,
                    const std::vector<at::Tensor>& lowp, const std::vector<at::Tensor>& ema, bool& grad_bf16,
                    const at::Device& dev) {
  const size_t n = grads.size();
  std::vector<TensorEntry> te(n);
  std::vector<ChunkEntry> ce;
  grad_bf16 = n > 0 && grads[0].scalar_type() == at::kBFloat16;
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(grads[i].is_contiguous() && grads[i].is_cuda(), "grads must be contiguous CUDA tensors");
    TORCH_CHECK((grads[i].scalar_type() == at::kBFloat16) == grad_bf16, "mixed grad dtypes in one group");
    te[i].grad = grads[i].data_ptr();
    te[i].numel = grads[i].numel();
    te[i].master = master.empty() ? nullptr : master[i].data_ptr<float>();
    te[i].m = m.empty() ? nullptr : m[i].data_ptr<float>();
    te[i].v = v.empty() ? nullptr : v[i].data_ptr<float>();
    te[i].lowp = lowp.empty() ? nullptr : reinterpret_cast<__nv_bfloat16*>(lowp[i].data_ptr());
    te[i].ema = ema.empty() ? nullptr : ema[i].data_ptr<float>();
    if (!master.empty()) {
      TORCH_CHECK(master[i].is_contiguous() && master[i].numel() == te[i].numel &&
                      master[i].scalar_type() == at::kFloat,
                  "master weights must be contiguous fp32 matching the grads");
      TORCH_CHECK(m[i].numel() == te[i].numel && v[i].numel() == te[i].numel, "moment size mismatch");
      if (!lowp.empty()) TORCH_CHECK(lowp[i].is_contiguous() && lowp[i].numel() == te[i].numel, "lowp mismatch");
      if (!ema.empty()) TORCH_CHECK(ema[i].is_contiguous() && ema[i].numel() == te[i].numel, "ema mismatch");
    }
    const int nc = (int)((te[i].numel + kChunk - 1) / kChunk);
    for (int c = 0; c < nc; ++c) ce.push_back({(int)i, c});
  }
  Tables t;
  t.nchunks = (int)ce.size();
  auto opts = at::TensorOptions().dtype(at::kByte);
  at::Tensor ht = at::empty({(int64_t)(n * sizeof(TensorEntry))}, opts.pinned_memory(true));
  at::Tensor hc = at::empty({(int64_t)(std::max<size_t>(ce.size(), 1) * sizeof(ChunkEntry))}, opts.pinned_memory(true));
  if (n) memcpy(ht.data_ptr(), te.data(), n * sizeof(TensorEntry));
  if (!ce.empty()) memcpy(hc.data_ptr(), ce.data(), ce.size() * sizeof(ChunkEntry));
  t.tensors = ht.to(dev, /*non_blocking=*/true);
  t.chunks = hc.to(dev, /*non_blocking=*/true);
  return t;
}

}  // namespace

void fused_adamw(std::vector<at::Tensor> master, std::vector<at::Tensor> grads, std::vector<at::Tensor> exp_avg,
                 std::vector<at::Tensor> exp_avg_sq, std::vector<at::Tensor> lowp, std::vector<at::Tensor> ema,
                 double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step,
                 c10::optional<at::Tensor> grad_scale, double ema_beta) {
  if (grads.empty()) return;
  TORCH_CHECK(master.size() == grads.size() && exp_avg.size() == grads.size() && exp_avg_sq.size() == grads.size(),
              "adamw: list sizes differ");
  TORCH_CHECK(lowp.empty() || lowp.size() == grads.size(), "adamw: lowp list size");
  TORCH_CHECK(ema.empty() || ema.size() == grads.size(), "adamw: ema list size");
  c10::cuda::CUDAGuard guard(grads[0].device());
  bool gbf16;
  Tables t = build_tables(master, exp_avg, exp_avg_sq, grads, lowp, ema, gbf16, grads[0].device());
  const float bc1 = 1.f - (float)std::pow(beta1, (double)step);
  const float bc2 = 1.f - (float)std::pow(beta2, (double)step);
  const float* gs = nullptr;
  if (grad_scale.has_value() && grad_scale->defined()) gs = grad_scale->data_ptr<float>();
  adamw_kernel<<<t.nchunks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const TensorEntry*>(t.tensors.data_ptr()), reinterpret_cast<const ChunkEntry*>(t.chunks.data_ptr()),
      gbf16, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)weight_decay, bc1 > 0 ? bc1 : 1.f,
      bc2 > 0 ? bc2 : 1.f, gs, (float)ema_beta);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Adds the sum of squares of `grads` into out[0] (fp32 scalar on the device).
void multi_sumsq(std::vector<at::Tensor> grads, at::Tensor& out) {
  if (grads.empty()) return;
  c10::cuda::CUDAGuard guard(grads[0].device());
  bool gbf16;
  Tables t = build_tables({}, {}, {}, grads, {}, {}, gbf16, grads[0].device());
  sumsq_kernel<<<t.nchunks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const TensorEntry*>(t.tensors.data_ptr()), reinterpret_cast<const ChunkEntry*>(t.chunks.data_ptr()),
      gbf16, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void clip_scale(const at::Tensor& sumsq, at::Tensor& scale, double max_norm) {
  c10::cuda::CUDAGuard guard(sumsq.device());
  clip_scale_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(sumsq.data_ptr<float>(), scale.data_ptr<float>(),
                                                                    (float)max_norm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace dmad

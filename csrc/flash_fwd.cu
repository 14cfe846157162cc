// Flash-attention forward for sm_100a (bf16 in/out, fp32 accumulate, head dim 64 or 128).
//
// Functional parity target: the reference's attention entry point
// (train/wan/rcm/utils/attention.py:120-167, cuDNN SDPA on cc 100) and the
// forward half of its Triton kernel (train/wan/rcm/utils/flash_attention_jvp_triton.py:107-232):
// O = softmax(Q K^T * scale) V, plus the natural-log row LSE used by backward.
//
// Design (one CTA per pair of 128-row query tiles of one (batch, head)):
//   warp 0      : TMA producer; Q once, then a 2-stage ring of K and V tiles
//   warp 1      : TMEM owner and the single MMA-issuing thread
//   warps 4..7  : softmax for query tile 0   (thread i owns TMEM lane / query row i)
//   warps 8..11 : softmax for query tile 1
// TMEM (512 columns): per tile, S at [t*256, +128) and O at [t*256+128, +d).
// P is written back as bf16 over the first 64 columns of S and consumed by a
// TMEM-A (".kind::f16 [d], [a], b") MMA, so it never touches shared memory.
// Each tile alternates S = Q K_j^T -> softmax -> O += P V_j; the MMA thread
// interleaves the two tiles so the tensor core works on one tile while the
// other tile's softmax runs.  P reaches the MMA thread in four parts of 32 keys (one mbarrier
// each), so the PV MMAs of the first keys run while the softmax computes the rest.  O is rescaled lazily: only when a row maximum
// grows by more than 2^8 (values stay exact because the final normalisation
// uses the same stale maximum as the numerator).
#include <cuda_runtime.h>
#include <type_traits>
#include <cuda_bf16.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "sm100.cuh"
#include "tma_host.h"

namespace dmad {

int* device_status_ptr(int device);

namespace {

constexpr int kTileM = 128;   // query rows per tile
constexpr int kTileN = 128;   // keys per KV tile
constexpr int kStages = 2;
constexpr int kHalfBytes = 128 * 128;            // one 128-row x 64-col bf16 swizzle panel
constexpr float kRescaleThreshold = 8.0f;        // log2 units

template <int kD>
struct FwdSmem {
  static constexpr int kTileBytes = kD / 64 * kHalfBytes;  // 128 rows x kD bf16 as 64-column panels
  // 1024-byte aligned panels (required by the 128B swizzle atoms)
  uint8_t q[2][kTileBytes];
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], p_full[2][4], pv_done[2];  // p_full[t][q]: P columns of part q of tile t
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct FwdParams {
  __nv_bfloat16* o;  // [B, Lq, H, d] with strides below
  float* lse;        // [B, H, Lpad] log2-domain LSE (+inf on padding rows)
  int64_t o_sb, o_sl, o_sh;
  int Lq, Lk, H, Lpad;
  float scale_log2;
  int* status;       // device status word (bounded-wait failures)
  // optional second copy of every output row, scattered to the rank that owns the row
  // (context-parallel head->sequence exchange): row g of sample b goes to
  // scat[g / scat_ll] + (b * scat_ll + g % scat_ll) * scat_ld + scat_col + head * d
  int64_t scat[16];
  int scat_n, scat_ll, scat_col;
  int64_t scat_ld;
  // optional running merge over successive key blocks (ring context parallelism):
  // acc_o fp32 [B, Lq, H, d] and acc_lse (log2) [B, H, Lpad] hold the softmax-weighted output
  // of the blocks seen so far; acc_read merges into them, acc_final also writes the bf16 o
  float* acc_o;
  float* acc_lse;
  int acc_read, acc_final;
};

template <int kD, int kPolyPer8, int kPSplit>
__global__ void __launch_bounds__(384, 1)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, FwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  using Smem = FwdSmem<kD>;
  constexpr int kPanels = kD / 64, kTileBytes = Smem::kTileBytes;
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;

  const int warp = warp_id();
  const int lane = lane_id();
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int q0 = blockIdx.x * (2 * kTileM);
  const int nkv = (p.Lk + kTileN - 1) / kTileN;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&sm.p_full[t][q], 128);
      mbar_init(&sm.pv_done[t], 1);
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
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      mbar_arrive_expect_tx(&sm.q_full, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        for (int h = 0; h < kPanels; ++h)
          tma_load_4d(sm.q[t] + h * kHalfBytes, &tm_q, &sm.q_full, h * 64, head, q0 + t * kTileM, batch);
      int last_s = -1, last_ph = 0;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!mbar_wait(&sm.k_empty[s], ph ^ 1, kStatusTimeoutEmpty, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&sm.k_full[s], kTileBytes);
        for (int h = 0; h < kPanels; ++h)
          tma_load_4d(sm.k[s] + h * kHalfBytes, &tm_k, &sm.k_full[s], h * 64, head, j * kTileN, batch);
        if (!mbar_wait(&sm.v_empty[s], ph ^ 1, kStatusTimeoutEmpty, abort_flag, p.status)) {
          // K load of this stage is in flight: wait for it before leaving
          mbar_wait(&sm.k_full[s], ph, kStatusTimeoutTmaFull, nullptr, p.status);
          break;
        }
        mbar_arrive_expect_tx(&sm.v_full[s], kTileBytes);
        for (int h = 0; h < kPanels; ++h)
          tma_load_4d(sm.v[s] + h * kHalfBytes, &tm_v, &sm.v_full[s], h * 64, head, j * kTileN, batch);
        last_s = s;
        last_ph = ph;
      }
      // never leave while our own copies may still be landing
      mbar_wait(&sm.q_full, 0, kStatusTimeoutTmaFull, nullptr, p.status);
      if (last_s >= 0) {
        mbar_wait(&sm.k_full[last_s], last_ph, kStatusTimeoutTmaFull, nullptr, p.status);
        mbar_wait(&sm.v_full[last_s], last_ph, kStatusTimeoutTmaFull, nullptr, p.status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, kD, false, true);
      const uint32_t q_addr0 = smem_u32(sm.q[0]);
      const uint32_t q_addr1 = smem_u32(sm.q[1]);
      bool ok = mbar_wait(&sm.q_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);

      auto issue_qk = [&](int t, int s) {
        const uint32_t qa = t == 0 ? q_addr0 : q_addr1;
        const uint32_t ka = smem_u32(sm.k[s]);
        const uint32_t d_tmem = tmem + t * 256;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16_ss(d_tmem, smem_desc_sw128(qa + off, 16, 1024), smem_desc_sw128(ka + off, 16, 1024), idesc_qk,
                      kk > 0);
        }
      };
      auto issue_pv = [&](int t, int s, bool acc, int kk0, int kk1) {
        const uint32_t va = smem_u32(sm.v[s]);
        const uint32_t p_tmem = tmem + t * 256;        // bf16 P over S columns [0,64)
        const uint32_t o_tmem = tmem + t * 256 + 128;
#pragma unroll
        for (int kk = kk0; kk < kk1; ++kk) {
          mma_bf16_ts(o_tmem, p_tmem + kk * 8, smem_desc_sw128(va + kk * 2048, kHalfBytes, 1024), idesc_pv,
                      (acc || kk > 0) ? 1u : 0u);
        }
      };

      if (ok) ok = mbar_wait(&sm.k_full[0], 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        mma_commit(&sm.s_full[0]);
        issue_qk(1, 0);
        mma_commit(&sm.s_full[1]);
        mma_commit(&sm.k_empty[0]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        const int s1 = (j + 1) % kStages;
        const uint32_t ph1 = ((j + 1) / kStages) & 1;
        const bool has_next = j + 1 < nkv;
        if (!(ok = mbar_wait(&sm.v_full[s], ph, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
        for (int t = 0; t < 2; ++t) {
          // P arrives in kPSplit parts (keys [128q / kPSplit, ...)); each part's MMAs start as soon as
          // the softmax has stored it, overlapping the rest of the softmax
#pragma unroll
          for (int q = 0; q < kPSplit; ++q) {
            if (!(ok = mbar_wait(&sm.p_full[t][q], j & 1, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
            tc_fence_after();
            issue_pv(t, s, j > 0, q * (8 / kPSplit), (q + 1) * (8 / kPSplit));
          }
          if (!ok) break;
          mma_commit(&sm.pv_done[t]);
          if (has_next) {
            if (t == 0 && !(ok = mbar_wait(&sm.k_full[s1], ph1, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
            tc_fence_after();
            issue_qk(t, s1);
            mma_commit(&sm.s_full[t]);
          }
        }
        if (!ok) break;
        mma_commit(&sm.v_empty[s]);
        if (has_next) mma_commit(&sm.k_empty[s1]);
      }
      // drain: every MMA issued by this thread has completed before TMEM is freed
      mma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, kStatusTimeoutMma, nullptr, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax / epilogue
    const int t = (warp - 4) >> 2;           // query tile
    const int wq = warp & 3;                 // TMEM lane quarter
    const int row = wq * 32 + lane;          // row within the tile
    const int q_row = q0 + t * kTileM + row;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t s_tmem = tmem + lane_base + t * 256;
    const uint32_t o_tmem = s_tmem + 128;
    const float scale_log2 = p.scale_log2;
    float m_used = -INFINITY;
    float l_sum = 0.f;
    bool ok = true;

    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      const int kv_valid = p.Lk - j * kTileN;
      const bool masked = kv_valid < kTileN;  // only the last key tile (warp-uniform)
      float alpha = 1.f;
      float rsum[4] = {0.f, 0.f, 0.f, 0.f};
      // The softmax body is instantiated twice: unmasked (every key tile but the last) and
      // masked (keys >= Lk read as -inf).
      auto body = [&](auto masked_t) {
        constexpr bool kMasked = decltype(masked_t)::value;
        // pass 1: the whole S row in one TMEM read (four loads, one wait); row maximum with
        // eight independent 3-input-max chains
        float m_blk;
        {
          uint32_t sr[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + c * 32, sr[c]);
          tmem_wait_ld();
          auto sv = [&](int c, int i) -> float {
            const float v = __uint_as_float(sr[c][i]);
            return (kMasked && c * 32 + i >= kv_valid) ? -INFINITY : v;
          };
          float mc[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float a = sv(c, 0), b = sv(c, 1);
#pragma unroll
            for (int i = 2; i < 30; i += 4) {
              a = fmax3(a, sv(c, i), sv(c, i + 1));
              b = fmax3(b, sv(c, i + 2), sv(c, i + 3));
            }
            mc[c] = fmax3(a, b, fmaxf(sv(c, 30), sv(c, 31)));
          }
          m_blk = fmaxf(fmaxf(mc[0], mc[1]), fmaxf(mc[2], mc[3])) * scale_log2;
        }
        bool rescale = false;
        if (j == 0) {
          m_used = m_blk;
        } else if (m_blk > m_used + kRescaleThreshold) {
          alpha = ex2_approx(m_used - m_blk);
          m_used = m_blk;
          rescale = true;
        }
        // O holds the sum over tiles < j (PV(j-1) finished before S(j) completed).
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(o_tmem + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(o_tmem + c * 32, r);
          }
        }
        // pass 2: P = exp2(S * scale - m) and the row sum, 32 columns at a time with the next
        // chunk's TMEM read in flight.  Chunk c writes bf16 P columns [16c, 16c+16), which
        // only overlap S columns already read.  On full tiles every second exponential runs on
        // the FMA pipe (ex2_poly); masked columns of the last tile give exactly 0 via MUFU.
        const float neg_m = -m_used;
        uint32_t buf[2][32];
        tmem_ld32(s_tmem, buf[0]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_wait_ld();
          if (c + 1 < 4) tmem_ld32(s_tmem + (c + 1) * 32, buf[(c + 1) & 1]);
          const uint32_t(&r)[32] = buf[c & 1];
          uint32_t pk[16];
          if constexpr (!kMasked) {
            // packed fp32x2 scale-and-shift and row sums; in every group of eight columns
            // kPolyPer8 of the odd columns take the exponential as a packed polynomial on the FMA
            // pipe (ex2_poly2), the others on MUFU
            const uint64_t sc2 = f2(scale_log2, scale_log2), nm2 = f2(neg_m, neg_m);
            float x[32], e[32];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 xx =
                  f2_split(f2_fma(f2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), sc2, nm2));
              x[2 * i] = xx.x;
              x[2 * i + 1] = xx.y;
            }
#pragma unroll
            for (int g = 0; g < 32; g += 8) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int a = g + 4 * h + 1, b = a + 2;
                if constexpr (kPolyPer8 >= 2) {
                  if (kPolyPer8 >= 4 || h == 0) {
                    const float2 pp = ex2_poly2(x[a], x[b]);
                    e[a] = pp.x;
                    e[b] = pp.y;
                  } else {
                    e[a] = ex2_approx(x[a]);
                    e[b] = ex2_approx(x[b]);
                  }
                } else {
                  e[a] = ex2_approx(x[a]);
                  e[b] = ex2_approx(x[b]);
                }
                e[a - 1] = ex2_approx(x[a - 1]);
                e[b - 1] = ex2_approx(x[b - 1]);
              }
            }
            uint64_t acc_a = f2(0.f, 0.f), acc_b = f2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              acc_a = f2_add(acc_a, f2(e[2 * i], e[2 * i + 1]));
              acc_b = f2_add(acc_b, f2(e[2 * i + 2], e[2 * i + 3]));
              pk[i] = pack_bf16x2(e[2 * i], e[2 * i + 1]);
              pk[i + 1] = pack_bf16x2(e[2 * i + 2], e[2 * i + 3]);
            }
            const float2 a2 = f2_split(f2_add(acc_a, acc_b));
            rsum[c] += a2.x + a2.y;
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int col = c * 32 + 2 * i;
              float x0 = fmaf(__uint_as_float(r[2 * i]), scale_log2, neg_m);
              float x1 = fmaf(__uint_as_float(r[2 * i + 1]), scale_log2, neg_m);
              x0 = col < kv_valid ? x0 : -INFINITY;
              x1 = col + 1 < kv_valid ? x1 : -INFINITY;
              const float p0 = ex2_approx(x0);
              const float p1 = ex2_approx(x1);
              rsum[c] += p0 + p1;
              pk[i] = pack_bf16x2(p0, p1);
            }
          }
          tmem_st16(s_tmem + c * 16, pk);
          if ((c + 1) % (4 / kPSplit) == 0) {  // hand this part of P to the MMA thread
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&sm.p_full[t][(c + 1) / (4 / kPSplit) - 1]);
          }
        }
      };
      if (masked)
        body(std::true_type{});
      else
        body(std::false_type{});
      const float rs = (rsum[0] + rsum[1]) + (rsum[2] + rsum[3]);
      l_sum = l_sum * alpha + rs;
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.pv_done[t], (nkv - 1) & 1, kStatusTimeoutMma, abort_flag, p.status));
    if (ok && p.acc_o != nullptr) {
      // merge this key block into the running result: weights 2^(lse_prev - lse_new) and
      // 2^(m - lse_new) on the previous output and on this block's unnormalised O
      tc_fence_after();
      const bool valid = q_row < p.Lq;
      const float lse_j = m_used + __log2f(l_sum);
      float* lrow = p.acc_lse + ((int64_t)batch * p.H + head) * p.Lpad + q_row;
      const float lp = (p.acc_read && valid) ? *lrow : -INFINITY;
      const float mx = fmaxf(lp, lse_j);
      const float nl = mx + __log2f(exp2f(lp - mx) + exp2f(lse_j - mx));
      const float wa = p.acc_read ? exp2f(lp - nl) : 0.f;
      const float wb = exp2f(m_used - nl);
      float* arow = p.acc_o + (((int64_t)batch * p.Lq + q_row) * p.H + head) * kD;
      __nv_bfloat16* orow = p.o + batch * p.o_sb + (int64_t)q_row * p.o_sl + head * p.o_sh;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(o_tmem + c * 32, r);
        tmem_wait_ld();
        if (valid) {
          float4* a4 = reinterpret_cast<float4*>(arow + c * 32);
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            float4 prev = p.acc_read ? a4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 nw;
            nw.x = prev.x * wa + __uint_as_float(r[4 * v + 0]) * wb;
            nw.y = prev.y * wa + __uint_as_float(r[4 * v + 1]) * wb;
            nw.z = prev.z * wa + __uint_as_float(r[4 * v + 2]) * wb;
            nw.w = prev.w * wa + __uint_as_float(r[4 * v + 3]) * wb;
            a4[v] = nw;
            if (p.acc_final) {
              uint2 w2;
              w2.x = pack_bf16x2(nw.x, nw.y);
              w2.y = pack_bf16x2(nw.z, nw.w);
              reinterpret_cast<uint2*>(orow + c * 32)[v] = w2;
            }
          }
        }
      }
      if (q_row < p.Lpad) {
        *lrow = valid ? nl : INFINITY;
        if (p.lse != nullptr) p.lse[((int64_t)batch * p.H + head) * p.Lpad + q_row] = valid ? nl : INFINITY;
      }
    } else if (ok) {
      tc_fence_after();
      const float inv_l = 1.f / l_sum;
      const bool valid = q_row < p.Lq;
      __nv_bfloat16* orow = p.o + batch * p.o_sb + (int64_t)q_row * p.o_sl + head * p.o_sh;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(o_tmem + c * 32, r);
        tmem_wait_ld();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv_l, __uint_as_float(r[8 * v + 1]) * inv_l);
            w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv_l, __uint_as_float(r[8 * v + 3]) * inv_l);
            w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv_l, __uint_as_float(r[8 * v + 5]) * inv_l);
            w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv_l, __uint_as_float(r[8 * v + 7]) * inv_l);
            dst[v] = w;
            if (p.scat_n > 0) {
              const int peer = q_row / p.scat_ll, lr = q_row - peer * p.scat_ll;
              __nv_bfloat16* srow = reinterpret_cast<__nv_bfloat16*>(p.scat[peer]) +
                                    ((int64_t)batch * p.scat_ll + lr) * p.scat_ld + p.scat_col + head * kD;
              reinterpret_cast<uint4*>(srow + c * 32)[v] = w;
            }
          }
        }
      }
      if (p.lse != nullptr && q_row < p.Lpad)
        p.lse[((int64_t)batch * p.H + head) * p.Lpad + q_row] = valid ? (m_used + __log2f(l_sum)) : INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// q/k/v: [B, L, H, d] bf16 views, d = 64 or 128 (last dim contiguous, any row / head / batch
// stride that is a multiple of 8 elements); boxes of 128 rows x 64 columns.
CUtensorMap make_qkv_map(const at::Tensor& x) {
  const uint64_t dims[4] = {(uint64_t)x.size(3), (uint64_t)x.size(2), (uint64_t)x.size(1), (uint64_t)x.size(0)};
  const uint64_t strides[3] = {(uint64_t)x.stride(2) * 2, (uint64_t)x.stride(1) * 2, (uint64_t)x.stride(0) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(x.data_ptr(), 4, dims, strides, box);
}

}  // namespace

// d: the head dim the kernel was written for (64 or 128)
void check_bhld(const at::Tensor& x, const char* name, int64_t d) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16, name, " must be a CUDA bf16 tensor");
  TORCH_CHECK(x.dim() == 4 && x.size(3) == d, name, " must be [B, L, H, ", d, "]");
  TORCH_CHECK(x.stride(3) == 1, name, " last dim must be contiguous");
  TORCH_CHECK(x.stride(2) % 8 == 0 && x.stride(1) % 8 == 0 && x.stride(0) % 8 == 0, name,
              " strides must be multiples of 8 elements");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}

size_t flash_fwd_smem_bytes(int d) { return (d == 64 ? sizeof(FwdSmem<64>) : sizeof(FwdSmem<128>)) + 1024; }

int64_t flash_lse_pad(int64_t L) { return (L + 255) / 256 * 256; }

// Launches the forward; `scat` (optional) adds the owner-rank copy of every output row.
static void flash_fwd_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                             at::Tensor& lse, double scale, const std::vector<int64_t>& scat, int64_t scat_ld,
                             int64_t scat_col, float* acc_o = nullptr, float* acc_lse = nullptr, int acc_read = 0,
                             int acc_final = 0) {
  TORCH_CHECK(q.dim() == 4 && (q.size(3) == 64 || q.size(3) == 128), "q must be [B, L, H, 64 or 128]");
  const int d = (int)q.size(3);
  check_bhld(q, "q", d);
  check_bhld(k, "k", d);
  check_bhld(v, "v", d);
  check_bhld(o, "o", d);
  TORCH_CHECK(k.sizes() == v.sizes(), "k and v shapes differ");
  TORCH_CHECK(q.size(0) == k.size(0) && q.size(2) == k.size(2), "q/k batch or head mismatch");
  TORCH_CHECK(o.sizes() == q.sizes(), "o shape mismatch");
  const int B = q.size(0), Lq = q.size(1), H = q.size(2), Lk = k.size(1);
  TORCH_CHECK(Lk > 0 && Lq > 0, "empty attention");
  bool has_lse = lse.defined() && lse.numel() > 0;
  if (has_lse) {
    TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous(), "lse must be fp32 contiguous");
    TORCH_CHECK(lse.dim() == 3 && lse.size(0) == B && lse.size(1) == H && lse.size(2) == flash_lse_pad(Lq),
                "lse must be [B, H, round_up(Lq, 256)]");
  }
  c10::cuda::CUDAGuard guard(q.device());
  CUtensorMap tq = make_qkv_map(q), tk = make_qkv_map(k), tv = make_qkv_map(v);
  FwdParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = has_lse ? lse.data_ptr<float>() : nullptr;
  p.o_sb = o.stride(0);
  p.o_sl = o.stride(1);
  p.o_sh = o.stride(2);
  p.Lq = Lq;
  p.Lk = Lk;
  p.H = H;
  p.Lpad = has_lse ? (int)lse.size(2) : 0;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.status = device_status_ptr(q.get_device());
  p.scat_n = (int)scat.size();
  TORCH_CHECK(p.scat_n <= 16, "at most 16 scatter targets");
  for (int i = 0; i < 16; ++i) p.scat[i] = i < p.scat_n ? scat[i] : 0;
  p.scat_ll = p.scat_n > 0 ? Lq / p.scat_n : 1;
  p.scat_ld = scat_ld;
  p.scat_col = (int)scat_col;
  p.acc_o = acc_o;
  p.acc_lse = acc_lse;
  p.acc_read = acc_read;
  p.acc_final = acc_final;
  if (p.scat_n > 0) {
    TORCH_CHECK(Lq % p.scat_n == 0, "Lq must divide over the scatter targets");
    TORCH_CHECK(scat_ld % 8 == 0 && scat_col % 8 == 0, "scatter row stride / column must be multiples of 8");
    for (int i = 0; i < p.scat_n; ++i) TORCH_CHECK(scat[i] % 16 == 0, "scatter targets must be 16-byte aligned");
  }
  const size_t smem = flash_fwd_smem_bytes(d);
  // four P parts per tile (measured at L = 32760, H = 12: 5.65-5.75 ms against 5.85-5.91 ms with
  // P handed over whole); half of the exponentials on the FMA pipe (2 of 8: same time, none: +6 %)
  auto kern = d == 64 ? flash_fwd_kernel<64, 4, 4> : flash_fwd_kernel<128, 4, 4>;
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((Lq + 2 * kTileM - 1) / (2 * kTileM), H, B);
  kern<<<grid, 384, smem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Writes O (same layout rules as q) and the log2-domain LSE [B, H, Lpad] (fp32),
// Lpad = Lq rounded up to a multiple of 256 (padding rows hold +inf).
void flash_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
               double scale) {
  flash_fwd_launch(q, k, v, o, lse, scale, {}, 0, 0);
}

// One key block of ring attention: merges softmax(q k^T) v over this block into the fp32 running
// output acc_o [B, Lq, H, d] (contiguous) and its log2 LSE acc_lse [B, H, round_up(Lq, 256)];
// read = merge with the previous blocks, final = also write the bf16 result to o (and lse if given).
void flash_fwd_accumulate(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                          at::Tensor& lse, at::Tensor& acc_o, at::Tensor& acc_lse, bool read, bool final_,
                          double scale) {
  TORCH_CHECK(acc_o.is_cuda() && acc_o.scalar_type() == at::kFloat && acc_o.is_contiguous() && acc_o.dim() == 4 &&
                  acc_o.size(0) == q.size(0) && acc_o.size(1) == q.size(1) && acc_o.size(2) == q.size(2) &&
                  acc_o.size(3) == q.size(3),
              "acc_o must be contiguous fp32 [B, Lq, H, d]");
  TORCH_CHECK(acc_lse.is_cuda() && acc_lse.scalar_type() == at::kFloat && acc_lse.is_contiguous() &&
                  acc_lse.dim() == 3 && acc_lse.size(2) == flash_lse_pad(q.size(1)),
              "acc_lse must be fp32 [B, H, round_up(Lq, 256)]");
  flash_fwd_launch(q, k, v, o, lse, scale, {}, 0, 0, acc_o.data_ptr<float>(), acc_lse.data_ptr<float>(), read ? 1 : 0,
                   final_ ? 1 : 0);
}

// flash_fwd that also stores every output row into the [B*Ll, ld] row buffer of the rank that
// owns the row (scatter[r] = that rank's buffer address, Ll = Lq / #ranks), at columns
// col + head * d -- the reverse all-to-all of context parallelism fused into the epilogue.
void flash_fwd_scatter(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                       double scale, std::vector<int64_t> scatter, int64_t ld, int64_t col) {
  TORCH_CHECK(!scatter.empty(), "scatter targets required");
  flash_fwd_launch(q, k, v, o, lse, scale, scatter, ld, col);
}

}  // namespace dmad

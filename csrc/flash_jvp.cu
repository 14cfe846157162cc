// Flash-attention forward with its forward-mode tangent (JVP) for sm_100a: bf16 in/out,
// fp32 accumulation, head dim 128, non-causal.
//
// Given primals q, k, v and tangents tq, tk, tv, one pass computes
//   O  = softmax(S) V,                 S  = q k^T * scale
//   tO = P tV + (P * tS) V - rowsum(P * tS) * O,   tS = (tq k^T + q tk^T) * scale
// and the log2-domain LSE of S (the same [B, H, round_up(L, 256)] buffer as the plain forward,
// so the plain flash backward differentiates O).  Parity target: the reference's Triton kernel
// `_attn_fwd` (train/wan/rcm/utils/flash_attention_jvp_triton.py:107-232) and its autograd wrapper
// (`_attention`, :450-579), whose backward differentiates O only (tangents are detached).
//
// Online form (per query row, running maximum m, e_j = exp(s_j - m)):
//   l = sum e_j, r = sum e_j ts_j, O~ = sum e_j v_j, T~ = sum e_j (tv_j + ts_j v_j)
//   O = O~ / l,  tO = (T~ - (r / l) O~) / l
// A~ = P tV and B~ = (P * tS) V accumulate into ONE TMEM accumulator T~ (only their sum is needed),
// so one 128-row query tile needs S, tS, O~ and T~: 4 x 128 = all 512 TMEM columns.
//
// CTA (384 threads) = one 128-row query tile of one (batch, head):
//   warp 0      TMA producer: q and tq once; k, tk, tv, v tiles single-buffered (6 x 32 KB smem)
//   warp 1      TMEM owner and the single MMA-issuing thread
//   warps 4..7  softmax group 0: key columns [0, 64) of every tile (thread = query row)
//   warps 8..11 softmax group 1: key columns [64, 128)
// The two groups exchange their partial row maxima through shared memory (an mbarrier with a
// bounded wait), so both use the same maximum and rescale decisions.  Each group writes its bf16 P (and P * tS) packed
// over the first half of its OWN S (tS) columns, which it has already read; the TMEM-A MMAs take
// the two packed halves from columns [c, c+32) and [c+64, c+96).
// MMA order per key tile j (the tensor core runs them in issue order):
//   [wait P_j]   O~ += P_j V_j ; T~ += P_j tV_j ; S_{j+1} = q k_{j+1}^T
//   [wait PtS_j] T~ += (P_j * tS_j) V_j ; tS_{j+1} = tq k_{j+1}^T + q tk_{j+1}^T
// so the tensor core works on P V, P tV and the next S while the softmax groups process tS_j.
// O~ and T~ are rescaled lazily (row maximum grew by > 2^8), after the tile's last MMA into them
// completed.  Every wait is bounded (status word + abort flag), as in the plain forward.
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
void check_bhld(const at::Tensor& x, const char* name, int64_t d = 128);
int64_t flash_lse_pad(int64_t L);

namespace {

constexpr int kTileM = 128;
constexpr int kTileN = 128;
constexpr int kHalfBytes = 128 * 128;       // 128 rows x 64 bf16 (one 128B-swizzle panel)
constexpr int kTileBytes = 2 * kHalfBytes;  // 128 x 128 bf16
constexpr float kRescaleThreshold = 8.0f;   // log2 units

struct JvpSmem {
  uint8_t q[kTileBytes];
  uint8_t tq[kTileBytes];
  uint8_t k[kTileBytes];
  uint8_t tk[kTileBytes];
  uint8_t v[kTileBytes];
  uint8_t tv[kTileBytes];
  uint64_t q_full;
  uint64_t k_full, k_empty, tk_full, tk_empty, v_full, v_empty, tv_full, tv_empty;
  uint64_t s_full, ts_full, p_full, pts_full, acc_done, drain, xchg, fin_full;
  float red[2][2][128];  // [tile parity][group][row] partial row maxima (scaled, log2)
  float fin[2][2][128];  // [l | r][group][row] at the end
  uint32_t tmem_base;
  int abort_flag;
};

struct JvpParams {
  __nv_bfloat16* o;
  __nv_bfloat16* to;
  float* lse;  // [B, H, Lpad] log2 domain, +inf on padding rows
  int64_t o_sb, o_sl, o_sh, to_sb, to_sl, to_sh;
  int Lq, Lk, H, Lpad;
  float scale_log2, scale;
  int has_tk, has_tv;
  int* status;
  // accumulate mode (key blocks visited one launch at a time): acc_o / acc_u fp32 [B, Lq, H, 128] hold
  // O and T~ / l of the blocks seen so far, acc_lse (log2) / acc_mu [B, H, Lpad] their LSE and r / l
  float* acc_o;
  float* acc_u;
  float* acc_lse;
  float* acc_mu;
  int acc_read, acc_final;
};

// TMEM column map (lane = query row)
constexpr uint32_t kColS = 0, kColTS = 128, kColO = 256, kColT = 384;

__global__ void __launch_bounds__(384, 1)
flash_jvp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tq,
                 const __grid_constant__ CUtensorMap tm_tk, const __grid_constant__ CUtensorMap tm_tv, JvpParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  JvpSmem& sm = *reinterpret_cast<JvpSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  volatile int* abort_flag = &sm.abort_flag;

  const int warp = warp_id();
  const int lane = lane_id();
  const int head = blockIdx.y;
  const int batch = blockIdx.z;
  const int q0 = blockIdx.x * kTileM;
  const int nkv = (p.Lk + kTileN - 1) / kTileN;
  const bool has_tk = p.has_tk != 0, has_tv = p.has_tv != 0;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.k_full, 1);
    mbar_init(&sm.k_empty, 1);
    mbar_init(&sm.tk_full, 1);
    mbar_init(&sm.tk_empty, 1);
    mbar_init(&sm.v_full, 1);
    mbar_init(&sm.v_empty, 1);
    mbar_init(&sm.tv_full, 1);
    mbar_init(&sm.tv_empty, 1);
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.ts_full, 1);
    mbar_init(&sm.p_full, 256);
    mbar_init(&sm.pts_full, 256);
    mbar_init(&sm.acc_done, 1);
    mbar_init(&sm.drain, 1);
    mbar_init(&sm.xchg, 256);
    mbar_init(&sm.fin_full, 256);
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
    prefetch_tmap(&tm_tq);
    if (has_tk) prefetch_tmap(&tm_tk);
    if (has_tv) prefetch_tmap(&tm_tv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      mbar_arrive_expect_tx(&sm.q_full, 2 * kTileBytes);
      for (int h = 0; h < 2; ++h) {
        tma_load_4d(sm.q + h * kHalfBytes, &tm_q, &sm.q_full, h * 64, head, q0, batch);
        tma_load_4d(sm.tq + h * kHalfBytes, &tm_tq, &sm.q_full, h * 64, head, q0, batch);
      }
      // last tile index issued per buffer (k, tk, tv, v): never leave while one is landing
      int last[4] = {-1, -1, -1, -1};
      uint64_t* fulls[4] = {&sm.k_full, &sm.tk_full, &sm.tv_full, &sm.v_full};
      auto load = [&](int kind, uint64_t* empty, uint8_t* dst, const CUtensorMap* tm, int j) -> bool {
        if (!mbar_wait(empty, (j & 1) ^ 1, kStatusTimeoutEmpty, abort_flag, p.status)) return false;
        mbar_arrive_expect_tx(fulls[kind], kTileBytes);
        for (int h = 0; h < 2; ++h)
          tma_load_4d(dst + h * kHalfBytes, tm, fulls[kind], h * 64, head, j * kTileN, batch);
        last[kind] = j;
        return true;
      };
      for (int j = 0; j < nkv; ++j) {
        bool ok = load(0, &sm.k_empty, sm.k, &tm_k, j);
        if (ok && has_tk) ok = load(1, &sm.tk_empty, sm.tk, &tm_tk, j);
        if (ok && has_tv) ok = load(2, &sm.tv_empty, sm.tv, &tm_tv, j);
        if (ok) ok = load(3, &sm.v_empty, sm.v, &tm_v, j);
        if (!ok) break;
      }
      mbar_wait(&sm.q_full, 0, kStatusTimeoutTmaFull, nullptr, p.status);
      for (int i = 0; i < 4; ++i)
        if (last[i] >= 0) mbar_wait(fulls[i], last[i] & 1, kStatusTimeoutTmaFull, nullptr, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 128, false, true);
      const uint32_t qa = smem_u32(sm.q), tqa = smem_u32(sm.tq), ka = smem_u32(sm.k), tka = smem_u32(sm.tk);
      const uint32_t va = smem_u32(sm.v), tva = smem_u32(sm.tv);

      auto gemm_nt = [&](uint32_t d, uint32_t a, uint32_t b, bool acc) {  // D (+)= A B^T, both K-major
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16_ss(d, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(b + off, 16, 1024), idesc_qk,
                      (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto gemm_pv = [&](uint32_t d, uint32_t a_tmem, uint32_t b, bool acc) {  // D (+)= P[TMEM] B (MN-major)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t a_col = (kk < 4) ? kk * 8 : 64 + (kk - 4) * 8;  // the two packed halves
          mma_bf16_ts(d, a_tmem + a_col, smem_desc_sw128(b + kk * 2048, kHalfBytes, 1024), idesc_pv,
                      (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto issue_s = [&]() { gemm_nt(tmem + kColS, qa, ka, false); };
      auto issue_ts = [&]() {
        gemm_nt(tmem + kColTS, tqa, ka, false);
        if (has_tk) gemm_nt(tmem + kColTS, qa, tka, true);
      };

      bool ok = mbar_wait(&sm.q_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) ok = mbar_wait(&sm.k_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      if (ok) {
        tc_fence_after();
        issue_s();
        mma_commit(&sm.s_full);
        if (has_tk) ok = mbar_wait(&sm.tk_full, 0, kStatusTimeoutTmaFull, abort_flag, p.status);
      }
      if (ok) {
        tc_fence_after();
        issue_ts();
        mma_commit(&sm.ts_full);
        mma_commit(&sm.k_empty);
        if (has_tk) mma_commit(&sm.tk_empty);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const uint32_t ph = j & 1, ph1 = (j + 1) & 1;
        const bool has_next = j + 1 < nkv;
        if (!(ok = mbar_wait(&sm.p_full, ph, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
        if (!(ok = mbar_wait(&sm.v_full, ph, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
        if (has_tv && !(ok = mbar_wait(&sm.tv_full, ph, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
        tc_fence_after();
        gemm_pv(tmem + kColO, tmem + kColS, va, j > 0);
        if (has_tv) {
          gemm_pv(tmem + kColT, tmem + kColS, tva, j > 0);
          mma_commit(&sm.tv_empty);
        }
        if (has_next) {
          if (!(ok = mbar_wait(&sm.k_full, ph1, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
          tc_fence_after();
          issue_s();
          mma_commit(&sm.s_full);
        }
        if (!(ok = mbar_wait(&sm.pts_full, ph, kStatusTimeoutSoftmax, abort_flag, p.status))) break;
        tc_fence_after();
        gemm_pv(tmem + kColT, tmem + kColTS, va, has_tv || j > 0);
        mma_commit(&sm.v_empty);
        mma_commit(&sm.acc_done);
        if (has_next) {
          if (has_tk && !(ok = mbar_wait(&sm.tk_full, ph1, kStatusTimeoutTmaFull, abort_flag, p.status))) break;
          tc_fence_after();
          issue_ts();
          mma_commit(&sm.ts_full);
          mma_commit(&sm.k_empty);
          if (has_tk) mma_commit(&sm.tk_empty);
        }
      }
      if (!ok) *abort_flag = 1;
      mma_commit(&sm.drain);
      mbar_wait(&sm.drain, 0, kStatusTimeoutMma, nullptr, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax groups / epilogue
    const int g = (warp - 4) >> 2;  // column group
    const int wq = warp & 3;        // TMEM lane quarter
    const int row = wq * 32 + lane;
    const int q_row = q0 + row;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t c0 = 64u * g;
    const uint32_t s_t = tmem + lane_base + kColS + c0;
    const uint32_t ts_t = tmem + lane_base + kColTS + c0;
    const uint32_t o_t = tmem + lane_base + kColO + c0;
    const uint32_t t_t = tmem + lane_base + kColT + c0;
    const float scale_log2 = p.scale_log2, scale = p.scale;
    float m_used = -INFINITY, l_sum = 0.f, r_sum = 0.f;
    bool ok = true;

    for (int j = 0; j < nkv; ++j) {
      const uint32_t ph = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.s_full, ph, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      const int kv_valid = p.Lk - j * kTileN - (int)c0;  // valid columns of this group's 64
      float pv[64];
      {
        uint32_t sr[2][32];
        tmem_ld32(s_t, sr[0]);
        tmem_ld32(s_t + 32, sr[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float x = __uint_as_float(sr[c][i]);
            pv[c * 32 + i] = (c * 32 + i < kv_valid) ? x : -INFINITY;
          }
      }
      float a0 = pv[0], a1 = pv[1];
#pragma unroll
      for (int i = 2; i < 62; i += 4) {
        a0 = fmax3(a0, pv[i], pv[i + 1]);
        a1 = fmax3(a1, pv[i + 2], pv[i + 3]);
      }
      const float pm = fmax3(a0, a1, fmaxf(pv[62], pv[63])) * scale_log2;
      sm.red[ph][g][row] = pm;
      mbar_arrive(&sm.xchg);  // exchange with the other column group (bounded wait, no bar.sync)
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.xchg, ph, kStatusTimeoutSoftmax, abort_flag, p.status));
      if (!ok) break;
      const float m_blk = fmaxf(sm.red[ph][0][row], sm.red[ph][1][row]);
      float alpha = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_used = m_blk;
      } else if (m_blk > m_used + kRescaleThreshold) {
        alpha = ex2_approx(m_used - m_blk);
        m_used = m_blk;
        rescale = true;
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // every MMA into O~ / T~ of tile j-1 has completed before we touch them
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&sm.acc_done, (j - 1) & 1, kStatusTimeoutMma, abort_flag, p.status));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int acc = 0; acc < 2; ++acc)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t a = (acc == 0 ? o_t : t_t) + c * 32;
            uint32_t r[32];
            tmem_ld32(a, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(a, r);
          }
      }
      // P = exp2(S * scale - m), packed bf16 over this group's first 32 S columns (all 64 of its
      // S columns are already in registers)
      const float neg_m = -m_used;
      float ls = 0.f;
      {
        // packed fp32x2 scale-and-shift and row sums (masked columns hold -inf: exp2 gives 0)
        const uint64_t sc2 = f2(scale_log2, scale_log2), nm2 = f2(neg_m, neg_m);
        uint64_t acc2 = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = c * 32 + 2 * i;
            const float2 x = f2_split(f2_fma(f2(pv[col], pv[col + 1]), sc2, nm2));
            pv[col] = ex2_approx(x.x);
            pv[col + 1] = ex2_approx(x.y);
            acc2 = f2_add(acc2, f2(pv[col], pv[col + 1]));
            pk[i] = pack_bf16x2(pv[col], pv[col + 1]);
          }
          tmem_st16(s_t + c * 16, pk);
        }
        const float2 a2 = f2_split(acc2);
        ls = a2.x + a2.y;
      }
      l_sum = l_sum * alpha + ls;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.p_full);

      // P * tS (tS scaled to the true tangent of the logits), packed over this group's first 32 tS columns
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.ts_full, ph, kStatusTimeoutMma, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      float rs = 0.f;
      {
        uint32_t tr[2][32];
        tmem_ld32(ts_t, tr[0]);
        tmem_ld32(ts_t + 32, tr[1]);
        tmem_wait_ld();
        const uint64_t sc2 = f2(scale, scale);
        uint64_t acc2 = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {  // P * tS * scale, two columns per packed op
            const int col = c * 32 + 2 * i;
            const uint64_t x2 = f2_mul(f2_mul(f2(pv[col], pv[col + 1]),
                                              f2(__uint_as_float(tr[c][2 * i]), __uint_as_float(tr[c][2 * i + 1]))),
                                       sc2);
            acc2 = f2_add(acc2, x2);
            const float2 x = f2_split(x2);
            pk[i] = pack_bf16x2(x.x, x.y);
          }
          tmem_st16(ts_t + c * 16, pk);
        }
        const float2 a2 = f2_split(acc2);
        rs = a2.x + a2.y;
      }
      r_sum = r_sum * alpha + rs;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.pts_full);
    }
    if (ok)
      ok = __all_sync(0xffffffffu,
                      mbar_wait(&sm.acc_done, (nkv - 1) & 1, kStatusTimeoutMma, abort_flag, p.status));
    const bool valid = q_row < p.Lq;
    const int64_t lidx = ((int64_t)batch * p.H + head) * p.Lpad + q_row;
    // the previous block's LSE / mu are read before fin_full: group 0 rewrites them only after both
    // groups have arrived there
    float lp = -INFINITY, mp = 0.f;
    if (p.acc_o != nullptr && p.acc_read && valid) {
      lp = p.acc_lse[lidx];
      mp = p.acc_mu[lidx];
    }
    sm.fin[0][g][row] = l_sum;
    sm.fin[1][g][row] = r_sum;
    mbar_arrive(&sm.fin_full);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.fin_full, 0, kStatusTimeoutSoftmax, abort_flag, p.status));
    if (ok && !*abort_flag && p.acc_o != nullptr) {
      // merge this key block: O = wa O_acc + wb O~, U = wa U_acc + wb T~, mu = wa mu_acc + wb r, with
      // wa = 2^(lse_acc - lse_new), wb = 2^(m - lse_new); tO = U - mu O at the last block
      tc_fence_after();
      const float l_tot = sm.fin[0][0][row] + sm.fin[0][1][row];
      const float r_tot = sm.fin[1][0][row] + sm.fin[1][1][row];
      const float lse_j = m_used + __log2f(l_tot);
      const float mx = fmaxf(lp, lse_j);
      const float nl = mx + __log2f(exp2f(lp - mx) + exp2f(lse_j - mx));
      const float wa = p.acc_read ? exp2f(lp - nl) : 0.f;
      const float wb = exp2f(m_used - nl);
      const float nmu = mp * wa + r_tot * wb;
      const int64_t arow_off = (((int64_t)batch * p.Lq + q_row) * p.H + head) * 128 + c0;
      float* arow = p.acc_o + arow_off;
      float* urow = p.acc_u + arow_off;
      __nv_bfloat16* orow = p.o + batch * p.o_sb + (int64_t)q_row * p.o_sl + head * p.o_sh + c0;
      __nv_bfloat16* torow = p.to + batch * p.to_sb + (int64_t)q_row * p.to_sl + head * p.to_sh + c0;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t ro[32], rt[32];
        tmem_ld32(o_t + c * 32, ro);
        tmem_ld32(t_t + c * 32, rt);
        tmem_wait_ld();
        if (valid) {
          float4* a4 = reinterpret_cast<float4*>(arow + c * 32);
          float4* u4 = reinterpret_cast<float4*>(urow + c * 32);
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const float4 pa = p.acc_read ? a4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 pu = p.acc_read ? u4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 na, nu;
            na.x = pa.x * wa + __uint_as_float(ro[4 * v + 0]) * wb;
            na.y = pa.y * wa + __uint_as_float(ro[4 * v + 1]) * wb;
            na.z = pa.z * wa + __uint_as_float(ro[4 * v + 2]) * wb;
            na.w = pa.w * wa + __uint_as_float(ro[4 * v + 3]) * wb;
            nu.x = pu.x * wa + __uint_as_float(rt[4 * v + 0]) * wb;
            nu.y = pu.y * wa + __uint_as_float(rt[4 * v + 1]) * wb;
            nu.z = pu.z * wa + __uint_as_float(rt[4 * v + 2]) * wb;
            nu.w = pu.w * wa + __uint_as_float(rt[4 * v + 3]) * wb;
            a4[v] = na;
            u4[v] = nu;
            if (p.acc_final) {
              uint2 wo, wt;
              wo.x = pack_bf16x2(na.x, na.y);
              wo.y = pack_bf16x2(na.z, na.w);
              wt.x = pack_bf16x2(nu.x - nmu * na.x, nu.y - nmu * na.y);
              wt.y = pack_bf16x2(nu.z - nmu * na.z, nu.w - nmu * na.w);
              reinterpret_cast<uint2*>(orow + c * 32)[v] = wo;
              reinterpret_cast<uint2*>(torow + c * 32)[v] = wt;
            }
          }
        }
      }
      if (g == 0 && q_row < p.Lpad) {
        p.acc_lse[lidx] = valid ? nl : INFINITY;
        p.acc_mu[lidx] = valid ? nmu : 0.f;
        if (p.lse != nullptr) p.lse[lidx] = valid ? nl : INFINITY;
        if (blockIdx.x == gridDim.x - 1 && q_row + kTileM < p.Lpad) {
          p.acc_lse[lidx + kTileM] = INFINITY;
          p.acc_mu[lidx + kTileM] = 0.f;
          if (p.lse != nullptr) p.lse[lidx + kTileM] = INFINITY;
        }
      }
    } else if (ok && !*abort_flag) {
      tc_fence_after();
      const float l_tot = sm.fin[0][0][row] + sm.fin[0][1][row];
      const float r_tot = sm.fin[1][0][row] + sm.fin[1][1][row];
      const float inv_l = 1.f / l_tot;
      const float rl = r_tot * inv_l;
      __nv_bfloat16* orow = p.o + batch * p.o_sb + (int64_t)q_row * p.o_sl + head * p.o_sh + c0;
      __nv_bfloat16* torow = p.to + batch * p.to_sb + (int64_t)q_row * p.to_sl + head * p.to_sh + c0;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t ro[32], rt[32];
        tmem_ld32(o_t + c * 32, ro);
        tmem_ld32(t_t + c * 32, rt);
        tmem_wait_ld();
        if (valid) {
          uint4* dst_o = reinterpret_cast<uint4*>(orow + c * 32);
          uint4* dst_t = reinterpret_cast<uint4*>(torow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            float o8[8], t8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float ov = __uint_as_float(ro[8 * v + i]);
              o8[i] = ov * inv_l;
              t8[i] = (__uint_as_float(rt[8 * v + i]) - rl * ov) * inv_l;
            }
            dst_o[v] = make_uint4(pack_bf16x2(o8[0], o8[1]), pack_bf16x2(o8[2], o8[3]), pack_bf16x2(o8[4], o8[5]),
                                  pack_bf16x2(o8[6], o8[7]));
            dst_t[v] = make_uint4(pack_bf16x2(t8[0], t8[1]), pack_bf16x2(t8[2], t8[3]), pack_bf16x2(t8[4], t8[5]),
                                  pack_bf16x2(t8[6], t8[7]));
          }
        }
      }
      if (g == 0 && p.lse != nullptr) {
        float* lrow = p.lse + ((int64_t)batch * p.H + head) * p.Lpad;
        if (q_row < p.Lpad) lrow[q_row] = valid ? (m_used + __log2f(l_tot)) : INFINITY;
        // Lpad (a multiple of 256) can exceed the last tile by 128 rows: the last CTA pads them
        if (blockIdx.x == gridDim.x - 1 && q_row + kTileM < p.Lpad) lrow[q_row + kTileM] = INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

CUtensorMap make_bhld_map(const at::Tensor& x) {
  const uint64_t dims[4] = {128, (uint64_t)x.size(2), (uint64_t)x.size(1), (uint64_t)x.size(0)};
  const uint64_t strides[3] = {(uint64_t)x.stride(2) * 2, (uint64_t)x.stride(1) * 2, (uint64_t)x.stride(0) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return make_tmap_bf16(x.data_ptr(), 4, dims, strides, box);
}

}  // namespace

size_t flash_jvp_smem_bytes() { return sizeof(JvpSmem) + 1024; }

namespace {

void jvp_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& tq,
                const c10::optional<at::Tensor>& tk, const c10::optional<at::Tensor>& tv, at::Tensor& o,
                at::Tensor& to, const at::Tensor& lse, double scale, float* acc_o, float* acc_u, float* acc_lse,
                float* acc_mu, int acc_lpad, bool acc_read, bool acc_final) {
  check_bhld(q, "q");
  check_bhld(k, "k");
  check_bhld(v, "v");
  check_bhld(tq, "tq");
  check_bhld(o, "o");
  check_bhld(to, "to");
  const bool has_tk = tk.has_value() && tk->defined();
  const bool has_tv = tv.has_value() && tv->defined();
  if (has_tk) {
    check_bhld(*tk, "tk");
    TORCH_CHECK(tk->sizes() == k.sizes(), "tk shape mismatch");
  }
  if (has_tv) {
    check_bhld(*tv, "tv");
    TORCH_CHECK(tv->sizes() == v.sizes(), "tv shape mismatch");
  }
  TORCH_CHECK(k.sizes() == v.sizes(), "k and v shapes differ");
  TORCH_CHECK(tq.sizes() == q.sizes() && o.sizes() == q.sizes() && to.sizes() == q.sizes(), "q-shaped tensors differ");
  TORCH_CHECK(q.size(0) == k.size(0) && q.size(2) == k.size(2), "q/k batch or head mismatch");
  const int B = q.size(0), Lq = q.size(1), H = q.size(2), Lk = k.size(1);
  TORCH_CHECK(Lq > 0 && Lk > 0, "empty attention");
  const bool has_lse = lse.defined() && lse.numel() > 0;
  if (has_lse) {
    TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == at::kFloat && lse.is_contiguous(), "lse must be fp32 contiguous");
    TORCH_CHECK(lse.dim() == 3 && lse.size(0) == B && lse.size(1) == H && lse.size(2) == flash_lse_pad(Lq),
                "lse must be [B, H, round_up(Lq, 256)]");
  }
  c10::cuda::CUDAGuard guard(q.device());
  CUtensorMap mq = make_bhld_map(q), mk = make_bhld_map(k), mv = make_bhld_map(v), mtq = make_bhld_map(tq);
  CUtensorMap mtk = has_tk ? make_bhld_map(*tk) : mk, mtv = has_tv ? make_bhld_map(*tv) : mv;
  JvpParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.to = reinterpret_cast<__nv_bfloat16*>(to.data_ptr());
  p.lse = has_lse ? lse.data_ptr<float>() : nullptr;
  p.o_sb = o.stride(0);
  p.o_sl = o.stride(1);
  p.o_sh = o.stride(2);
  p.to_sb = to.stride(0);
  p.to_sl = to.stride(1);
  p.to_sh = to.stride(2);
  p.Lq = Lq;
  p.Lk = Lk;
  p.H = H;
  p.Lpad = acc_o != nullptr ? acc_lpad : (has_lse ? (int)lse.size(2) : 0);
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.scale = (float)scale;
  p.has_tk = has_tk;
  p.has_tv = has_tv;
  p.status = device_status_ptr(q.get_device());
  p.acc_o = acc_o;
  p.acc_u = acc_u;
  p.acc_lse = acc_lse;
  p.acc_mu = acc_mu;
  p.acc_read = acc_read ? 1 : 0;
  p.acc_final = acc_final ? 1 : 0;
  const size_t smem = flash_jvp_smem_bytes();
  C10_CUDA_CHECK(cudaFuncSetAttribute(flash_jvp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((Lq + kTileM - 1) / kTileM, H, B);
  flash_jvp_kernel<<<grid, 384, smem, at::cuda::getCurrentCUDAStream()>>>(mq, mk, mv, mtq, mtk, mtv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// q, k, v, tq: [B, L, H, 128] bf16 (last dim contiguous, strides multiples of 8 elements);
// tk / tv optional (undefined = zero tangent).  Writes o, to (shape of q) and the log2 LSE.
void flash_jvp_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& tq,
                   c10::optional<at::Tensor> tk, c10::optional<at::Tensor> tv, at::Tensor& o, at::Tensor& to,
                   at::Tensor& lse, double scale) {
  jvp_launch(q, k, v, tq, tk, tv, o, to, lse, scale, nullptr, nullptr, nullptr, nullptr, 0, false, false);
}

// One key block of a blockwise (ring) attention JVP: merges this block into acc_o / acc_u (contiguous
// fp32 [B, Lq, H, 128]) and acc_lse / acc_mu (fp32 [B, H, round_up(Lq, 256)]); read = false starts a
// fresh accumulation, final_ = true also writes the bf16 o and to.  lse (optional) receives the LSE.
void flash_jvp_accumulate(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& tq,
                          c10::optional<at::Tensor> tk, c10::optional<at::Tensor> tv, at::Tensor& o, at::Tensor& to,
                          at::Tensor& lse, at::Tensor& acc_o, at::Tensor& acc_u, at::Tensor& acc_lse,
                          at::Tensor& acc_mu, bool read, bool final_, double scale) {
  for (const at::Tensor* a : {&acc_o, &acc_u})
    TORCH_CHECK(a->is_cuda() && a->scalar_type() == at::kFloat && a->is_contiguous() && a->dim() == 4 &&
                    a->size(0) == q.size(0) && a->size(1) == q.size(1) && a->size(2) == q.size(2) &&
                    a->size(3) == 128,
                "acc_o / acc_u must be contiguous fp32 [B, Lq, H, 128]");
  for (const at::Tensor* a : {&acc_lse, &acc_mu})
    TORCH_CHECK(a->is_cuda() && a->scalar_type() == at::kFloat && a->is_contiguous() && a->dim() == 3 &&
                    a->size(0) == q.size(0) && a->size(1) == q.size(2) && a->size(2) == flash_lse_pad(q.size(1)),
                "acc_lse / acc_mu must be fp32 [B, H, round_up(Lq, 256)]");
  jvp_launch(q, k, v, tq, tk, tv, o, to, lse, scale, acc_o.data_ptr<float>(), acc_u.data_ptr<float>(),
             acc_lse.data_ptr<float>(), acc_mu.data_ptr<float>(), (int)acc_lse.size(2), read, final_);
}

}  // namespace dmad

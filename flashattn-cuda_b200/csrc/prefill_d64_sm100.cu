// prefill_d64_sm100.cu -- attention prefill forward for head dimension 64 on
// B200 (sm_100a): the reference's headline shape (cuda/flash_attn_fa3_db_full.cu,
// HD = 64, :23), with the same math as prefill_sm100.cu (O, L = m ln2 + ln l).
//
// At D = 64 a 128 x 128 score tile carries half the UMMA work it does at
// D = 128, so the softmax is what bounds the kernel.  This variant therefore
// splits every score row between two warpgroups:
//
//   * one CTA per (256 query rows = Q tiles 0/1, query head), 640 threads;
//   * warps 0-15: four softmax warpgroups (tile t, half h), warpgroup 2t+h.
//     Half h owns keys [64h, 64h+64) of every 128-key tile and runs an
//     independent online softmax over them, with its own running max, sum and
//     TMEM accumulator O_{t,h} -- a split of the key range inside the CTA.  At
//     the end the two halves of a row are merged with the log-sum-exp identity
//     (the rescale of cuda/flash_attn_fa3_db_full.cu:261-284 applied across
//     halves) and each thread writes 32 of the row's 64 output columns;
//   * warp 16: TMA producer (Q once, K/V tiles into a 4-stage ring, 128-byte
//     swizzle); warp 17: UMMA issuer and TMEM owner; warps 18-19 idle;
//   * UMMA: S_t = Q_t K_j^T (SS, M=128 N=128 K=64) into TMEM S_t;
//     O_{t,h} += P_{t,h} V_j[64h:64h+64] (TS, M=128 N=64 K=64), P_{t,h} written
//     by its warpgroup as packed 16-bit pairs over its half of S_t.
//
// TMEM (512 columns): S_0 [0,128) S_1 [128,256) O_{t,h} at 256 + 64 (2t + h).
#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace prefill64 {

constexpr int D = 64;
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int HALF = BN / 2;
constexpr int kRowsPerCta = 2 * BM;
constexpr int kSoftmaxWGs = 4;
constexpr int kThreads = (kSoftmaxWGs + 1) * 128;  // + {producer, MMA, 2 idle}
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kStages = 4;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;
// Launched at kLaunchRegs per thread (the most 20 warps can have); the
// control warpgroup gives registers to the softmax warpgroups.
constexpr uint32_t kLaunchRegs = 96;
constexpr uint32_t kRegsCtrl = 64;
constexpr uint32_t kRegsSoftmax = 104;
static_assert(128 * kRegsCtrl + 512 * kRegsSoftmax <= kThreads * kLaunchRegs,
              "register split must fit in the launch allocation");

constexpr uint32_t kQBytes = BM * D * 2;    // one Q tile, 16 KB
constexpr uint32_t kKVBytes = BN * D * 2;   // one K or V tile, 16 KB
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + 2 * kQBytes;
constexpr uint32_t kOffV = kOffK + kStages * kKVBytes;
constexpr uint32_t kOffML = kOffV + kStages * kKVBytes;  // epilogue exchange: [2][2][128] x (m, l)
constexpr uint32_t kOffBar = kOffML + 2 * 2 * 128 * 8;
// q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2][2], pv_done[2], epi[2]
constexpr int kNumBars = 1 + 3 * kStages + 2 + 4 + 2 + 2;
constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
constexpr uint32_t kOffAbort = kOffTmemSlot + 8;
constexpr uint32_t kSmemBytes = kOffAbort + 8 + 1024;
constexpr int kPolyPairsPer8 = 3;  // of 8 exponential pairs, on the FMA pipe
// Split-KV form (small grids): each CTA's partial O (fp32, normalised by its
// own sum, rows padded to 68 floats so that a warp's row-strided 16-B stores
// hit distinct banks) and its per-row (m, l), written over the drained K/V ring.
constexpr int kPartStride = D + 4;
constexpr uint32_t kOffPartO = kOffK;
constexpr uint32_t kOffPartML = kOffPartO + kRowsPerCta * kPartStride * 4;
static_assert(kOffPartML + kRowsPerCta * 8 <= kOffML, "split partials must fit in the K/V ring");
constexpr int kMaxSplits = 8;

// SPLIT: a cluster of `splits` CTAs along x shares one 256-row block; CTA
// rank r takes KV tiles [r * kv_per_split, ...) of those the block sees (under
// a causal mask possibly none) and the
// partial results are merged through distributed shared memory at the end
// (the LSE-weighted combine of the split-KV decode, done in-kernel).
template <bool BF16, bool CAUSAL, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_d64_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, void* __restrict__ out,
                       float* __restrict__ lse, int N, int Nk, int H, int group, float scale_log2,
                       int splits, int kv_per_split) {
  using E = Elem<BF16>;
  constexpr int S = kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw);
  const uint32_t sQ = sb + kOffQ, sK = sb + kOffK, sV = sb + kOffV;
  const uint32_t bar0 = sb + kOffBar;
  const uint32_t BAR_Q = bar0;
  auto BAR_KF = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_VF = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto BAR_KVE = [&](int s) { return bar0 + 8u * (1 + 2 * S + s); };
  auto BAR_SF = [&](int t) { return bar0 + 8u * (1 + 3 * S + t); };
  auto BAR_PF = [&](int t, int h) { return bar0 + 8u * (3 + 3 * S + 2 * t + h); };
  auto BAR_PVD = [&](int t) { return bar0 + 8u * (7 + 3 * S + t); };
  auto BAR_EPI = [&](int t) { return bar0 + 8u * (9 + 3 * S + t); };
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sp + kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sp + kOffAbort);
  float2* s_ml = reinterpret_cast<float2*>(sp + kOffML);  // [t][h][row]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = SPLIT ? (int)blockIdx.x / splits : (int)blockIdx.x;
  const uint32_t crank = SPLIT ? cluster_ctarank() : 0u;
  const int bhk = (bh / H) * (H / group) + (bh % H) / group;
  const int q0 = ((int)gridDim.y - 1 - (int)blockIdx.y) * kRowsPerCta;
  // keys: Nk (>= N when causal); the causal mask is aligned to the bottom
  // right, query row r sees keys <= r + (Nk - N)
  const int koff = Nk - N;
  const int nkv_all = (Nk + BN - 1) / BN;
  // this CTA's KV tiles: kv_base + [0, nkv_t[t]) for Q tile t (every loop below
  // runs over the local index j; kv_base + j is the tile's place in the sequence)
  const int kv_base = SPLIT ? (int)crank * kv_per_split : 0;
  // (split: a causal rank whose slice lies past the block's last visible key
  // has no tile at all and contributes an empty partial)
  int nkv_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    nkv_t[t] = CAUSAL ? min(nkv_all, (q0 + (t + 1) * BM + koff + BN - 1) / BN) : nkv_all;
    if (SPLIT) nkv_t[t] = max(0, min(kv_per_split, nkv_t[t] - kv_base));
  }
  const int nkv = nkv_t[1];  // >= nkv_t[0]

  if (warp == kProducerWarp && lane == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      // p_full / epi: one arrival per softmax warp (4 per half, 8 per tile);
      // the rest one arrival (expect_tx or tcgen05.commit)
      uint32_t cnt = 1;
      for (int t = 0; t < 2; ++t) {
        if (bar == BAR_PF(t, 0) || bar == BAR_PF(t, 1)) cnt = 4;
        if (bar == BAR_EPI(t)) cnt = 8;
      }
      mbar_init(bar, cnt);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32((const void*)tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 16) {
    setmaxnreg_dec<kRegsCtrl>();
    if (warp == kProducerWarp && lane == 0 && nkv > 0) {
      // ---------------------------------------------------------- producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(BAR_Q, 2 * kQBytes);
      tma_load_3d(sQ, &tmQ, BAR_Q, 0, q0, bh);
      tma_load_3d(sQ + kQBytes, &tmQ, BAR_Q, 0, q0 + BM, bh);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % S;
        if (j >= S && !mbar_wait(BAR_KVE(st), ((j / S) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(BAR_KF(st), kKVBytes);
        tma_load_3d(sK + st * kKVBytes, &tmK, BAR_KF(st), 0, (kv_base + j) * BN, bhk);
        mbar_arrive_expect_tx(BAR_VF(st), kKVBytes);
        tma_load_3d(sV + st * kKVBytes, &tmV, BAR_VF(st), 0, (kv_base + j) * BN, bhk);
      }
    } else if (warp == kMmaWarp && lane == 0) {
      // ---------------------------------------------------------- UMMA issuer
      constexpr uint32_t idesc_qk = idesc_f16(BM, BN, BF16, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(BM, D, BF16, false, true);
      const uint64_t dq0 = sdesc_sw128(sQ, 16, 1024);
      const uint64_t dk0 = sdesc_sw128(sK, 16, 1024);
      const uint64_t dv0 = sdesc_sw128(sV, 16, 1024);  // N = 64: one column block
      // Every commit point costs the tensor pipe a bubble of ~100 clocks, so each
      // Q tile's two PV products and its next S are issued as one run with one
      // commit point (pv_done and s_full committed back to back).
      auto issue_s = [&](int t, int j) {
        const uint64_t qd = dq0 + ((t * kQBytes) >> 4);
        const uint64_t kd = dk0 + (((j % S) * kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16_ss(tmem + t * 128, qd + kk * 2, kd + kk * 2, idesc_qk, kk > 0 ? 1u : 0u);
      };
      auto issue_pv = [&](int t, int h, int j) {
        const uint64_t vd = dv0 + (((j % S) * kKVBytes + h * HALF * 128) >> 4);
        const uint32_t a_p = tmem + t * 128 + h * HALF;
        const uint32_t d_o = tmem + 256 + 64 * (2 * t + h);
#pragma unroll
        for (int kk = 0; kk < HALF / 16; ++kk)
          umma_f16_ts(d_o, a_p + kk * 8, vd + kk * 128, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
      };
      bool ok = nkv > 0 && mbar_wait(BAR_Q, 0, abort_flag) && mbar_wait(BAR_KF(0), 0, abort_flag);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (nkv_t[t] == 0) continue;  // split-KV: no tile of this slice is visible
          issue_s(t, 0);
          umma_commit(BAR_SF(t));
        }
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % S;
        if (!mbar_wait(BAR_VF(st), (j / S) & 1, abort_flag)) break;
        bool k_next = false;
#pragma unroll
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= nkv_t[t]) continue;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!mbar_wait(BAR_PF(t, h), j & 1, abort_flag)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, h, j);
          }
          if (!ok) break;
          const bool s_next = j + 1 < nkv_t[t];
          if (s_next) {  // S_t(j+1) overwrites P_{t,*}(j): after both PVs
            if (!k_next) {
              if (!mbar_wait(BAR_KF((j + 1) % S), ((j + 1) / S) & 1, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              k_next = true;
            }
            issue_s(t, j + 1);
          }
          umma_commit(BAR_PVD(t));
          if (s_next) umma_commit(BAR_SF(t));
        }
        umma_commit(BAR_KVE(st));
      }
    }
    if constexpr (SPLIT) {
      __syncwarp();
      cluster_sync_all();
      cluster_sync_all();
    }
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax (t, h)
    const int wg = warp >> 2;
    const int t = wg >> 1, h = wg & 1;
    const int row = threadIdx.x & 127;
    const int grow = q0 + t * BM + row;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_base + t * 128 + h * HALF;  // S half, then P half
    const uint32_t t_o = tmem + lane_base + 256 + 64 * (2 * t + h);
    const int my_nkv = nkv_t[t];
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;

    for (int j = 0; j < my_nkv && ok; ++j) {
      if (!mbar_wait(BAR_SF(t), j & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[HALF];
      tmem_ld32(t_s, s);
      tmem_ld32(t_s + 32, s + 32);
      tmem_ld_wait();

      const int kv0 = (kv_base + j) * BN + h * HALF;
      const bool need_mask = (kv0 + HALF > Nk) || (CAUSAL && kv0 + HALF > q0 + t * BM + koff);
      if (need_mask) {
        const int lim = (CAUSAL ? min(Nk, grow + 1 + koff) : Nk) - kv0;
#pragma unroll
        for (int c = 0; c < HALF; ++c)
          if (c >= lim) s[c] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(s[i], s[i + 8]);
#pragma unroll
      for (int c = 16; c < HALF; c += 16)
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = fmax3(mx8[i], s[c + i], s[c + 8 + i]);
      const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                             fmaxf(mx8[6], mx8[7]));
      const float m_new = fmaxf(m_run, mx * scale_log2);
      const bool rescale = m_new > m_run + kRescaleThreshold;  // always on this half's first data
      float alpha = 1.f;
      if (rescale) {
        alpha = ex2_mufu(m_run - m_new);
        m_run = m_new;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      const float2 sc2 = make_float2(scale_log2, scale_log2);
      const float2 nm2 = make_float2(-m_use, -m_use);
      float2 rs[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rs[i] = make_float2(0.f, 0.f);
      uint32_t pk[HALF / 2];
#pragma unroll
      for (int c = 0; c < HALF; c += 2) {
        const float2 x = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
        float2 p;
        if (((c >> 1) & 7) < kPolyPairsPer8) {
          p = exp2_poly2(x);
        } else {
          p.x = ex2_mufu(x.x);
          p.y = ex2_mufu(x.y);
        }
        rs[(c >> 1) & 3] = fadd2(rs[(c >> 1) & 3], p);
        pk[c >> 1] = pack2_u32<BF16>(p.x, p.y);
      }
      const float2 r01 = fadd2(fadd2(rs[0], rs[1]), fadd2(rs[2], rs[3]));
      l_run = l_run * alpha + (r01.x + r01.y);

      // P_{t,h}(j) over this half of S_t (32 packed columns)
      tmem_st32u(t_s, pk);
      // O_{t,h} is still accumulated by the PV products of step j-1: rescale once
      // they are done
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        if (!mbar_wait(BAR_PVD(t), (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(t_o + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(t_o + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_PF(t, h));
    }

    // ---------------------------------------------------------- epilogue
    // exchange (m, l) with the other half of the row, then merge:
    //   M = max(m0, m1), w_i = 2^(m_i - M), L = l0 w0 + l1 w1,
    //   O = (w0 O_{t,0} + w1 O_{t,1}) / L   (this thread: columns [32h, 32h+32))
    if (ok && my_nkv > 0) ok = mbar_wait(BAR_PVD(t), (my_nkv - 1) & 1, abort_flag);
    s_ml[(t * 2 + h) * 128 + row] = make_float2(ok ? m_run : -INFINITY, ok ? l_run : 0.f);
    __syncwarp();
    if (lane == 0) mbar_arrive(BAR_EPI(t));
    if (ok) ok = mbar_wait(BAR_EPI(t), 0, abort_flag);
    float a[32], b[32];
    float M = -INFINITY, Lsum = 0.f, f0 = 0.f, f1 = 0.f;
    if (ok) {
      tc_fence_after();
      const float2 ml0 = s_ml[(t * 2 + 0) * 128 + row];
      const float2 ml1 = s_ml[(t * 2 + 1) * 128 + row];
      M = fmaxf(ml0.x, ml1.x);
      const float w0 = (ml0.x == -INFINITY) ? 0.f : ex2_mufu(ml0.x - M);
      const float w1 = (ml1.x == -INFINITY) ? 0.f : ex2_mufu(ml1.x - M);
      Lsum = ml0.y * w0 + ml1.y * w1;
      const float inv = 1.f / Lsum;
      f0 = w0 * inv;
      f1 = w1 * inv;
      const uint32_t o0 = tmem + lane_base + 256 + 64 * (2 * t) + 32 * h;
      const uint32_t o1 = tmem + lane_base + 256 + 64 * (2 * t + 1) + 32 * h;
      if (my_nkv > 0) {  // warp-uniform: tile t's count
        tmem_ld32(o0, a);
        tmem_ld32(o1, b);
        tmem_ld_wait();
      }
      if (!SPLIT && grow < N) {
        typename E::T* orow =
            reinterpret_cast<typename E::T*>(out) + ((size_t)bh * N + grow) * D + 32 * h;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack2_u32<BF16>(a[i] * f0 + b[i] * f1, a[i + 1] * f0 + b[i + 1] * f1);
          w.y = pack2_u32<BF16>(a[i + 2] * f0 + b[i + 2] * f1, a[i + 3] * f0 + b[i + 3] * f1);
          w.z = pack2_u32<BF16>(a[i + 4] * f0 + b[i + 4] * f1, a[i + 5] * f0 + b[i + 5] * f1);
          w.w = pack2_u32<BF16>(a[i + 6] * f0 + b[i + 6] * f1, a[i + 7] * f0 + b[i + 7] * f1);
          *reinterpret_cast<uint4*>(orow + i) = w;
        }
        if (h == 0 && lse != nullptr)
          lse[(size_t)bh * N + grow] = M * 0.69314718055994531f + logf(Lsum);
      }
    }
    if constexpr (SPLIT) {
      // This CTA's partial for the row: O normalised by its own sum, and (M, L),
      // written over the K/V ring once no UMMA reads it.  Every softmax thread
      // has waited for its own tile's last PV above (that barrier is at most one
      // phase behind; a wait on the other tile's barrier could match an older
      // phase of the same parity and return early); the named barrier, reached
      // by all softmax threads on every path, extends that to both tiles.
      tc_fence_before();
      named_barrier_sync(1, kSoftmaxWGs * 128);
      {
        // (-inf, 0, O = 0) where this rank's slice shows the row no key
        const bool seen = ok && my_nkv > 0 && M != -INFINITY;
        float* po = reinterpret_cast<float*>(sp + kOffPartO) + (t * BM + row) * kPartStride + 32 * h;
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(po + i) =
              seen ? make_float4(a[i] * f0 + b[i] * f1, a[i + 1] * f0 + b[i + 1] * f1,
                                 a[i + 2] * f0 + b[i + 2] * f1, a[i + 3] * f0 + b[i + 3] * f1)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
        if (h == 0)
          reinterpret_cast<float2*>(sp + kOffPartML)[t * BM + row] =
              seen ? make_float2(M, Lsum) : make_float2(-INFINITY, 0.f);
      }
      // merge the cluster's partials, this CTA taking rows [crank * rows_per, ...):
      //   M* = max_c M_c, W_c = L_c 2^(M_c - M*), O = sum_c W_c O_c / sum_c W_c,
      //   L = M* ln 2 + ln sum_c W_c
      __syncwarp();
      cluster_sync_all();  // every CTA's partials are written
      const int rows_per = kRowsPerCta / splits;
      const uint32_t po_base = sb + kOffPartO, pml_base = sb + kOffPartML;
      for (int it = threadIdx.x; it < rows_per * (D / 4); it += kSoftmaxWGs * 128) {
        const int r = (int)crank * rows_per + it / (D / 4);
        const int c4 = (it % (D / 4)) * 4;
        float mx = -INFINITY;
        for (int c = 0; c < splits; ++c)
          mx = fmaxf(mx, ld_dsmem_f2(mapa_shared(pml_base + r * 8, (uint32_t)c)).x);
        float lt = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < splits; ++c) {
          const float2 ml = ld_dsmem_f2(mapa_shared(pml_base + r * 8, (uint32_t)c));
          if (ml.x == -INFINITY) continue;  // an empty partial
          const float w = ml.y * ex2_mufu(ml.x - mx);
          const float4 o =
              ld_dsmem_f4(mapa_shared(po_base + (r * kPartStride + c4) * 4, (uint32_t)c));
          lt += w;
          acc.x += w * o.x;
          acc.y += w * o.y;
          acc.z += w * o.z;
          acc.w += w * o.w;
        }
        const int qrow = q0 + r;
        if (qrow < N) {
          // lt == 0 only when every rank aborted on a timed-out wait (error
          // bit 0 is set then): O = 0, L = -inf instead of inf / NaN
          const float inv = lt > 0.f ? 1.f / lt : 0.f;
          uint2 wv;
          wv.x = pack2_u32<BF16>(acc.x * inv, acc.y * inv);
          wv.y = pack2_u32<BF16>(acc.z * inv, acc.w * inv);
          *reinterpret_cast<uint2*>(reinterpret_cast<typename E::T*>(out) +
                                    ((size_t)bh * N + qrow) * D + c4) = wv;
          if (c4 == 0 && lse != nullptr)
            lse[(size_t)bh * N + qrow] =
                lt > 0.f ? mx * 0.69314718055994531f + logf(lt) : -INFINITY;
        }
      }
      cluster_sync_all();  // no CTA leaves while a peer still reads its partials
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill64

template <bool BF16, bool CAUSAL, bool SPLIT>
static int launch_prefill_d64(const void* q, const void* k, const void* v, void* o, float* lse,
                              int B, int H, int Hkv, int N, int Nk, float scale, int splits,
                              cudaStream_t stream) {
  using namespace prefill64;
  auto kern = prefill_d64_kernel<BF16, CAUSAL, SPLIT>;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(B2A_ERR_CUDA, "cudaGetDevice failed");
  if (!attr_done[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(prefill d64)");
    attr_done[dev] = true;
  }
  CUtensorMap tq, tk, tv;
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = make_tmap_3d(&tq, q, dt, D, N, (uint64_t)B * H, 64, BM, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tk, k, dt, D, Nk, (uint64_t)B * Hkv, 64, BN, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tv, v, dt, D, Nk, (uint64_t)B * Hkv, 64, BN, true);
  if (rc != B2A_OK) return rc;
  const unsigned blocks = (unsigned)((N + kRowsPerCta - 1) / kRowsPerCta);
  const float scale_log2 = scale * 1.4426950408889634f;
  cudaError_t e;
  if constexpr (SPLIT) {
    const int nkv = (Nk + BN - 1) / BN;
    const int per = (nkv + splits - 1) / splits;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * H * splits), blocks, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, o, lse, N, Nk, H, H / Hkv, scale_log2, splits,
                           per);
  } else {
    dim3 grid((unsigned)(B * H), blocks);
    kern<<<grid, kThreads, kSmemBytes, stream>>>(tq, tk, tv, o, lse, N, Nk, H, H / Hkv, scale_log2,
                                                 1, 0);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return set_cuda_error(e, "prefill d64 kernel launch");
  return B2A_OK;
}

// Split-KV factor: the largest power of two <= 8 whose clusters still fit in
// one wave on the device's SMs and give every rank at least one KV tile of the
// heaviest block; 1 (no split) when the plain grid already fills the GPU.
static int d64_splits(int B, int H, int N, int Nk) {
  static int sms[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 1;
  if (sms[dev] == 0 &&
      cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 1;
  const int64_t ctas = (int64_t)B * H * ((N + prefill64::kRowsPerCta - 1) / prefill64::kRowsPerCta);
  const int nkv = (Nk + prefill64::BN - 1) / prefill64::BN;
  for (int s = prefill64::kMaxSplits; s >= 2; s >>= 1) {
    if (ctas * s > sms[dev]) continue;
    const int per = (nkv + s - 1) / s;
    if ((s - 1) * per < nkv) return s;
  }
  return 1;
}

int prefill_d64_dispatch(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                         int H, int Hkv, int N, int Nk, int dtype, int causal, float scale,
                         cudaStream_t stream) {
  const bool bf = dtype == B2A_BF16;
  const int splits = d64_splits(B, H, N, Nk);
#define B2A_D64(BB, CC, SS)                                                                      \
  if (bf == BB && (causal != 0) == CC && (splits > 1) == SS)                                    \
    return launch_prefill_d64<BB, CC, SS>(q, k, v, o, lse, B, H, Hkv, N, Nk, scale, splits,   \
                                          stream);
  B2A_D64(false, false, false)
  B2A_D64(false, false, true)
  B2A_D64(false, true, false)
  B2A_D64(true, false, false)
  B2A_D64(true, false, true)
  B2A_D64(true, true, false)
  B2A_D64(false, true, true)
  B2A_D64(true, true, true)
#undef B2A_D64
  return set_error(B2A_ERR_UNSUPPORTED, "prefill d64: no kernel for this configuration");
}

B2A_DEFINE_ERROR_READER(prefill_d64)

}  // namespace b2a

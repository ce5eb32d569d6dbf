// backward_sm100.cu -- attention backward (dQ, dK, dV) on B200 (sm_100a).
//
// The reference computes the same gradients with three scalar FP32 kernels
// (cuda/flash_attn_kernel.cu:173-412): D_i = rowsum(dO * O), then dQ, then
// dK / dV, recomputing P = exp(S - L) from the saved logsumexp.  Here:
//
//   * bwd_prep_kernel: per query row D_i = rowsum(dO * O) and L_i log2(e), in
//     fp32 arrays padded to a multiple of 128 rows (padding rows: D = 0,
//     L = +inf, so that their P is exactly 0), and a zeroed fp32 dQ
//     accumulator;
//   * bwd_main_kernel: one CTA per (128-key block j, KV head).  K_j, V_j stay
//     in shared memory and dK_j, dV_j accumulate in TMEM while the CTA walks
//     every query head of the KV head (GQA group) and every query block i of
//     BQ rows that sees block j (causal: from the diagonal on).  BQ = 128 for
//     D = 64 and 64 for D = 128.  Per step, on the 5th-generation tensor cores
//     (tcgen05, cta_group::1):
//         S^T  = K_j Q_i^T                      (SS UMMA -> TMEM)
//         dP^T = V_j dO_i^T                     (SS UMMA -> TMEM)
//         P^T  = exp2(S^T scale log2e - L_i log2e)     (element-wise warps,
//         dS^T = P^T (dP^T - D_i)                       one key row per lane)
//         dV_j += P^T dO_i                      (TS UMMA: P^T from TMEM)
//         dK_j += dS^T Q_i                      (SS UMMA: dS^T from smem)
//         dQ_i  = dS K_j        (D = 64)        (SS UMMA: the dS^T tile read
//         dQ_i^T = K_j^T dS^T   (D = 128)        MN-major; M = 128 either way)
//     and four read-out warps move dQ_i (TMEM -> registers -> a 128-byte
//     swizzled fp32 staging tile) into the global fp32 dQ accumulator with
//     TMA bulk reduce-adds (no per-element atomics).  The dS^T tiles and the
//     staging tiles are double-buffered, so a step never waits for the
//     previous step's reduce to finish reading;
//   * bwd_dq_kernel: dQ accumulator (fp32, already scaled) -> dtype.
//
// Warp roles (512 threads): warps 0-7 element-wise (warp w owns TMEM lanes
// 32 (w % 4) .. +31 = key rows, and query columns W (w / 4) .. +W-1, W =
// BQ / 2); warps 8-11 dQ read-out; warp 12 TMA producer; warp 13 UMMA issuer
// and TMEM owner; warps 14-15 idle.
//
// TMEM columns: S^T [0,BQ) with P^T written over it as packed 16-bit pairs,
// dP^T [BQ,2BQ), dV [2BQ, 2BQ+D), dK [2BQ+D, 2BQ+2D), dQ (or dQ^T) from
// 2BQ+2D: 448 of 512 columns for both head dimensions.
#include <cstdio>

#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace bwd {

constexpr int BK = 128;  // keys per CTA (UMMA M of S^T, dV, dK)
constexpr int kThreads = 512;
constexpr int kReadoutWarp0 = 8;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
// Register split: launched at 128 per thread (512 threads), the element-wise
// warpgroups take 144, the read-out warpgroup 168 (a whole D = 128 dQ row) and
// the control warpgroup 56: 256 * 144 + 128 * 168 + 128 * 56 == 512 * 128.
constexpr uint32_t kRegsElem = 144;
constexpr uint32_t kRegsReadout = 168;
constexpr uint32_t kRegsCtrl = 56;
static_assert(256 * kRegsElem + 128 * kRegsReadout + 128 * kRegsCtrl == kThreads * 128,
              "register split must add up to the launch allocation");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kMaxSmem = 232448;    // 227 KB, the per-CTA limit
constexpr uint32_t kErrSmemAlign = 16u;  // device error bit: base alignment slack too small
constexpr int kPadRows = 128;            // L2 / D rows are padded to a multiple of this
// of every 4 consecutive (even, odd) score pairs, this many take the
// polynomial exp2 on the FMA pipe and the rest the MUFU ex2 (16 per clock
// per SM): half and half keeps both pipes equally busy
constexpr int kPolyPairsPer4 = 2;
constexpr int BQ = 128;  // query rows per step (UMMA N of S^T, M of dQ)

// Shared-memory plan per head dimension (both under 227 KB):
//   D = 64:  Q and dO share a 2-stage ring; 2 dS^T tiles; 2 fp32 staging
//            tiles; dQ has its own TMEM columns.
//   D = 128: Q in a 2-stage ring, dO single-buffered (reloaded as soon as dV
//            has read it); 1 dS^T tile; one 32 KB staging tile that the dQ
//            read-out fills in two 64-column rounds; dQ reuses the dP^T
//            columns (TMEM is full: S^T, dP^T, dV, dK = 4 x 128).
template <int D>
struct Cfg {
  static constexpr bool kWide = (D == 128);
  static constexpr int W = BQ / 2;                  // query columns per element-wise warp
  static constexpr int kBlocks = D / 64;            // 64-column (128-byte) blocks per row
  static constexpr int kDoStages = kWide ? 1 : 2;
  static constexpr int kDsBufs = kWide ? 1 : 2;
  static constexpr int kStBufs = kWide ? 1 : 2;     // staging tiles of BQ x 64 fp32
  static constexpr int kRounds = D / 64;            // staging rounds per step
  static constexpr uint32_t kTile = 128 * D * 2;    // K, V, Q or dO tile (128 rows)
  static constexpr uint32_t kBlk = 128 * 128;       // one 64-column block of a tile
  static constexpr uint32_t kDsTile = BK * BQ * 2;  // dS^T [128 keys][128 queries]
  static constexpr uint32_t kStBox = BQ * 128;      // staging box: BQ rows x 32 fp32
  static constexpr uint32_t kStTile = 2 * kStBox;   // 64 fp32 columns
  static constexpr uint32_t kVec = BQ * 8;          // {L2[BQ], D[BQ]}
  // TMEM columns
  static constexpr uint32_t kColS = 0, kColDP = BQ, kColDV = 2 * BQ, kColDK = 2 * BQ + D;
  static constexpr uint32_t kColDQ = kWide ? kColDP : 2 * BQ + 2 * D;
  static_assert((kWide ? kColDK + D : kColDQ + D) <= kTmemCols, "TMEM layout");
  // shared memory
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = kOffK + kTile;
  static constexpr uint32_t kOffQ = kOffV + kTile;                 // [2 stages]
  static constexpr uint32_t kOffDO = kOffQ + 2 * kTile;            // [kDoStages]
  static constexpr uint32_t kOffDS = kOffDO + kDoStages * kTile;   // [kDsBufs]
  static constexpr uint32_t kOffST = kOffDS + kDsBufs * kDsTile;   // [kStBufs]
  static constexpr uint32_t kOffVec = kOffST + kStBufs * kStTile;  // [2 stages]
  static constexpr uint32_t kOffBar = kOffVec + 2 * kVec;
  // kv_full, q_full[2], q_empty[2], s_full, dp_full, p_full, ds_full, dq_full,
  // dq_free, ds_empty[2], do_full, do_empty, fin
  static constexpr int kNumBars = 16;
  static constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
  static constexpr uint32_t kOffAbort = kOffTmemSlot + 8;
  static constexpr uint32_t kContent = kOffAbort + 8;
  // + slack to align the base to 1024 bytes (128-byte swizzle atoms); the
  // kernel checks at run time that the slack it needs fits
  static constexpr uint32_t kSmemBytes =
      kContent + 1024 <= kMaxSmem ? kContent + 1024 : kMaxSmem;
  static_assert(kContent <= kMaxSmem, "backward tiles exceed shared memory");
};

// Padded per-row arrays: L2 = L log2(e) (+inf past N) and D = rowsum(dO * O)
// (0 past N), [B*H][Npad]; the valid rows of the dQ accumulator zeroed.  One
// warp per padded row.
template <int D, bool BF16>
__global__ void bwd_prep_kernel(const void* __restrict__ o, const void* __restrict__ dout,
                                const float* __restrict__ lse, float* __restrict__ l2v,
                                float* __restrict__ dvec, float* __restrict__ dq_acc, int N,
                                int Npad, long long rows_pad) {
  using E = Elem<BF16>;
  const long long prow = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (prow >= rows_pad) return;
  const long long bh = prow / Npad;
  const int n = (int)(prow % Npad);
  if (n >= N) {
    if (lane == 0) {
      dvec[prow] = 0.f;
      l2v[prow] = INFINITY;
    }
    return;
  }
  const long long row = bh * N + n;
  constexpr int EPL = D / 32;  // elements per lane (2 or 4)
  const typename E::T* op = reinterpret_cast<const typename E::T*>(o) + row * D + lane * EPL;
  const typename E::T* dp = reinterpret_cast<const typename E::T*>(dout) + row * D + lane * EPL;
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; e += 2) {
    const float2 a = E::unpack(*reinterpret_cast<const typename E::T2*>(op + e));
    const float2 b = E::unpack(*reinterpret_cast<const typename E::T2*>(dp + e));
    acc = fmaf(a.x, b.x, fmaf(a.y, b.y, acc));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    dvec[prow] = acc;
    l2v[prow] = lse[row] * 1.4426950408889634f;
  }
  float* dqr = dq_acc + row * D + lane * EPL;
#pragma unroll
  for (int e = 0; e < EPL; ++e) dqr[e] = 0.f;
}

template <int D, bool BF16>
__global__ void bwd_dq_kernel(const float* __restrict__ dq_acc, void* __restrict__ dq, size_t n) {
  using E = Elem<BF16>;
  const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (i < n) {
    const float2 v = *reinterpret_cast<const float2*>(dq_acc + i);
    *reinterpret_cast<typename E::T2*>(reinterpret_cast<typename E::T*>(dq) + i) =
        E::pack(v.x, v.y);
  }
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128-byte
// swizzled tile of 128-byte rows (the layout TMA and UMMA use)
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Bounded wait whose result is the same for every lane of the warp (a wait
// that gave up on one lane stops the whole warp), so that the warp-collective
// tcgen05 loads / stores and __syncwarp after it never see a split warp.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}
// The same over the 128 threads of the read-out warps (named barrier 3).
__device__ __forceinline__ bool readout_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred P, Q;\n\tsetp.ne.u32 P, %1, 0;\n\t"
      "bar.red.and.pred Q, 3, 128, P;\n\tselp.u32 %0, 1, 0, Q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

template <int D, bool BF16, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_main_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmDQ, const float* __restrict__ l2v,
                    const float* __restrict__ dvec, void* __restrict__ dk, void* __restrict__ dv,
                    int N, int Nk, int Npad, int H, int Hkv, float scale) {
  using C = Cfg<D>;
  using E = Elem<BF16>;
  constexpr int W = C::W;
  const float scale_log2 = scale * 1.4426950408889634f;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  if ((sb - raw) + C::kContent > C::kSmemBytes) {  // uniform over the CTA
    if (threadIdx.x == 0) atomicOr(&g_error_flags, kErrSmemAlign);
    return;
  }
  uint8_t* sp = smem_raw + (sb - raw);
  const uint32_t sK = sb + C::kOffK, sV = sb + C::kOffV;
  const uint32_t sQ = sb + C::kOffQ, sDO = sb + C::kOffDO;
  const uint32_t sDS = sb + C::kOffDS, sST = sb + C::kOffST, sVec = sb + C::kOffVec;
  const uint32_t bar0 = sb + C::kOffBar;
  const uint32_t BAR_KV = bar0;
  auto BAR_QF = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_QE = [&](int s) { return bar0 + 8u * (3 + s); };
  const uint32_t BAR_S = bar0 + 8u * 5, BAR_DP = bar0 + 8u * 6, BAR_P = bar0 + 8u * 7;
  const uint32_t BAR_DS = bar0 + 8u * 8, BAR_DQ = bar0 + 8u * 9, BAR_DQF = bar0 + 8u * 10;
  auto BAR_DSE = [&](int s) { return bar0 + 8u * (11 + s); };
  const uint32_t BAR_DOF = bar0 + 8u * 13, BAR_DOE = bar0 + 8u * 14;  // single-buffered dO
  const uint32_t BAR_FIN = bar0 + 8u * 15;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sp + C::kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sp + C::kOffAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x;    // key block
  const int bhk = blockIdx.y;  // b * Hkv + hkv
  const int b = bhk / Hkv, hkv = bhk % Hkv;
  const int G = H / Hkv;
  const int kv0 = j * BK;
  const int koff = Nk - N;  // causal: query row r sees keys <= r + koff
  const int nq = (N + BQ - 1) / BQ;
  const int i0 = CAUSAL ? max(0, (kv0 - koff) / BQ) : 0;
  const int nqs = nq - i0;    // query blocks per query head (>= 1)
  const int steps = G * nqs;  // (query head, query block) pairs

  if (warp == kProducerWarp && lane == 0) {
    mbar_init(BAR_KV, 1u);
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR_QF(s), 1u);
      mbar_init(BAR_QE(s), 1u);
      mbar_init(BAR_DSE(s), 1u);
    }
    mbar_init(BAR_S, 1u);
    mbar_init(BAR_DP, 1u);
    mbar_init(BAR_P, 8u);
    mbar_init(BAR_DS, 8u);
    mbar_init(BAR_DQ, 1u);
    mbar_init(BAR_DQF, 4u);
    mbar_init(BAR_DOF, 1u);
    mbar_init(BAR_DOE, 1u);
    mbar_init(BAR_FIN, 1u);
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
  const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;

  if (warp >= kProducerWarp) {
    setmaxnreg_dec<kRegsCtrl>();
    if (warp == kProducerWarp) {
      // ------------------------------------------------------------ producer
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmDO);
        mbar_arrive_expect_tx(BAR_KV, 2 * C::kTile);
#pragma unroll
        for (int c = 0; c < C::kBlocks; ++c) {
          tma_load_3d(sK + c * C::kBlk, &tmK, BAR_KV, c * 64, kv0, bhk);
          tma_load_3d(sV + c * C::kBlk, &tmV, BAR_KV, c * 64, kv0, bhk);
        }
        for (int it = 0; it < steps; ++it) {
          const int st = it & 1;
          const int g = it / nqs, q0 = (i0 + it % nqs) * BQ;
          const int bh = b * H + hkv * G + g;
          if (it >= 2 && !mbar_wait(BAR_QE(st), ((it >> 1) - 1) & 1, abort_flag)) break;
          constexpr bool kDoInRing = C::kDoStages == 2;
          mbar_arrive_expect_tx(BAR_QF(st), (kDoInRing ? 2 : 1) * C::kTile + C::kVec);
#pragma unroll
          for (int c = 0; c < C::kBlocks; ++c) {
            tma_load_3d(sQ + st * C::kTile + c * C::kBlk, &tmQ, BAR_QF(st), c * 64, q0, bh);
            if (kDoInRing)
              tma_load_3d(sDO + st * C::kTile + c * C::kBlk, &tmDO, BAR_QF(st), c * 64, q0, bh);
          }
          bulk_load(sVec + st * C::kVec, l2v + (size_t)bh * Npad + q0, BQ * 4, BAR_QF(st));
          bulk_load(sVec + st * C::kVec + BQ * 4, dvec + (size_t)bh * Npad + q0, BQ * 4,
                    BAR_QF(st));
          if (!kDoInRing) {  // dO_it once dV_{it-1} has read dO_{it-1}
            if (it >= 1 && !mbar_wait(BAR_DOE, (it - 1) & 1, abort_flag)) break;
            mbar_arrive_expect_tx(BAR_DOF, C::kTile);
#pragma unroll
            for (int c = 0; c < C::kBlocks; ++c)
              tma_load_3d(sDO + c * C::kBlk, &tmDO, BAR_DOF, c * 64, q0, bh);
          }
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------------------ UMMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc_s = idesc_f16(128, BQ, BF16, false, false);
        constexpr uint32_t idesc_o = idesc_f16(128, D, BF16, false, true);
        constexpr uint32_t idesc_q = idesc_f16(BQ, D, BF16, true, true);  // dQ = dS K
        // Software-pipelined order: S^T(it+1) is issued right after dV(it), so
        // the element-wise warps form P^T(it+1) while dQ(it), dK(it) and
        // dP^T(it+1) run:
        //   S(0) dP(0) | dV(0) S(1) dQ(0) dK(0) dP(1) | dV(1) S(2) dQ(1) ...
        auto issue_s = [&](int it) {  // S^T = K Q^T (A = K, B = Q, both K-major)
          const uint32_t q_base = sQ + (it & 1) * C::kTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * C::kBlk + (kk & 3) * 32;
            umma_f16_ss(tmem + C::kColS, sdesc_sw128(sK + off, 16, 1024),
                        sdesc_sw128(q_base + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_S);
        };
        auto issue_dp = [&](int it) {  // dP^T = V dO^T (A = V, B = dO, both K-major)
          const uint32_t do_base = sDO + (C::kDoStages == 2 ? (it & 1) : 0) * C::kTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * C::kBlk + (kk & 3) * 32;
            umma_f16_ss(tmem + C::kColDP, sdesc_sw128(sV + off, 16, 1024),
                        sdesc_sw128(do_base + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_DP);
        };
        bool ok = mbar_wait(BAR_KV, 0, abort_flag) && mbar_wait(BAR_QF(0), 0, abort_flag) &&
                  (C::kDoStages == 2 || mbar_wait(BAR_DOF, 0, abort_flag));
        if (ok) {
          tc_fence_after();
          issue_s(0);
          issue_dp(0);
        }
        for (int it = 0; ok && it < steps; ++it) {
          const int st = it & 1;
          const uint32_t q_base = sQ + st * C::kTile;
          const uint32_t do_base = sDO + (C::kDoStages == 2 ? st : 0) * C::kTile;
          const int dsb = it % C::kDsBufs;
          const uint32_t ds_base = sDS + dsb * C::kDsTile;
          // dV += P^T dO (A = P^T from TMEM: warp half h packs queries hW..
          // from column hW; B = dO MN-major: rows = queries = K, 64-column
          // blocks of D = N)
          if (!mbar_wait(BAR_P, it & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16_ts(tmem + C::kColDV, tmem + C::kColS + (kk >> 2) * W + (kk & 3) * 8,
                        sdesc_sw128(do_base + kk * 2048, C::kBlk, 1024), idesc_o,
                        (it > 0 || kk > 0) ? 1u : 0u);
          if (C::kDoStages == 1) umma_commit(BAR_DOE);  // dO_it read
          // S^T(it+1) over P^T(it), which dV(it) above has already consumed
          if (it + 1 < steps) {
            if (!mbar_wait(BAR_QF((it + 1) & 1), ((it + 1) >> 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(it + 1);
          }
          if (!mbar_wait(BAR_DS, it & 1, abort_flag)) { ok = false; break; }
          // dQ_{it-1} must have left its own columns before dQ_it
          if (!C::kWide && it > 0 && !mbar_wait(BAR_DQF, (it - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // dQ = dS K: A = the dS^T tile read MN-major (rows = keys = K,
          // columns = queries = M); B = the K tile MN-major (rows = keys = K,
          // 64-column blocks of D = N).  At D = 128 it overwrites dP^T(it),
          // which the element-wise warps read before ds_full.
          auto issue_dq = [&]() {
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_f16_ss(tmem + C::kColDQ, sdesc_sw128(ds_base + kk * 2048, C::kBlk, 1024),
                          sdesc_sw128(sK + kk * 2048, C::kBlk, 1024), idesc_q, kk > 0 ? 1u : 0u);
            umma_commit(BAR_DQ);
          };
          // dK += dS^T Q (TS: A = dS^T packed over the dP^T columns by the
          // element-wise warps, like P^T over S^T; B = Q MN-major).  dK reads
          // those columns, so it goes before dQ, which overwrites them at D = 128.
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16_ts(tmem + C::kColDK, tmem + C::kColDP + (kk >> 2) * W + (kk & 3) * 8,
                        sdesc_sw128(q_base + kk * 2048, C::kBlk, 1024), idesc_o,
                        (it > 0 || kk > 0) ? 1u : 0u);
          issue_dq();
          umma_commit(BAR_QE(st));    // Q_it (and dO_it in the ring) read
          umma_commit(BAR_DSE(dsb));  // dS^T tile read
          // dP^T(it+1): at D = 128 into the dQ columns once dQ(it) has left them
          if (it + 1 < steps) {
            if (C::kWide && !mbar_wait(BAR_DQF, it & 1, abort_flag)) { ok = false; break; }
            if (C::kDoStages == 1 && !mbar_wait(BAR_DOF, (it + 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_dp(it + 1);
          }
        }
        umma_commit(BAR_FIN);  // dK / dV final (or the pipeline gave up)
      }
    }
  } else if (warp >= kReadoutWarp0) {
    setmaxnreg_inc<kRegsReadout>();
    // -------------------------------------------------------------- dQ read-out
    const int row = (warp & 3) * 32 + lane;  // query row of the block = TMEM lane
    const bool issuer = warp == kReadoutWarp0 && lane == 0;
    int rounds_done = 0;                     // staging rounds committed so far
    for (int it = 0; it < steps; ++it) {
      if (!readout_wait(BAR_DQ, it & 1, abort_flag)) break;
      tc_fence_after();
      const int g = it / nqs, q0 = (i0 + it % nqs) * BQ;
      const int bh = b * H + hkv * G + g;
      // the whole dQ row into registers first, so its TMEM columns free at once
      float v[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32(tmem + lane_base + C::kColDQ + c * 32, v + 32 * c);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_DQF);
#pragma unroll
      for (int r = 0; r < C::kRounds; ++r) {
        // the staging tile of this round was last read kStBufs rounds ago
        const int slot = rounds_done % C::kStBufs;
        if (rounds_done >= C::kStBufs) {
          if (issuer) bulk_wait_group_read<C::kStBufs - 1>();
          asm volatile("bar.sync 2, 128;" ::: "memory");
        }
        uint8_t* stg = sp + C::kOffST + slot * C::kStTile;
        // two 32-column boxes, 128-byte swizzled: [box][row][8 chunks of 4 floats]
        const float* vr = v + 64 * r;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<float4*>(stg + (c >> 3) * C::kStBox + sw128(row, c & 7)) =
              make_float4(vr[4 * c] * scale, vr[4 * c + 1] * scale, vr[4 * c + 2] * scale,
                          vr[4 * c + 3] * scale);
        fence_proxy_async_smem();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (issuer) {
          const uint32_t src = sST + slot * C::kStTile;
          tma_reduce_add_3d(&tmDQ, src, r * 64, q0, bh);
          tma_reduce_add_3d(&tmDQ, src + C::kStBox, r * 64 + 32, q0, bh);
          bulk_commit_group();
        }
        ++rounds_done;
      }
    }
    if (issuer) bulk_wait_group<0>();  // every dQ reduce has landed
  } else {
    setmaxnreg_inc<kRegsElem>();
    // ------------------------------------------------------------ element-wise
    const int krow = (warp & 3) * 32 + lane;  // key row of the block = TMEM lane
    const int key = kv0 + krow;
    const int h = warp >> 2;                  // query columns hW .. hW+W-1
    bool ok = true;
    for (int it = 0; it < steps; ++it) {
      const int st = it & 1;
      const int q0 = (i0 + it % nqs) * BQ;
      const float* vec = reinterpret_cast<const float*>(sp + C::kOffVec + st * C::kVec);
      const bool need_mask = (kv0 + BK > Nk) || (CAUSAL && kv0 + BK - 1 > q0 + koff);
      // valid iff key <= q + koff: columns c >= qmin of this warp's W
      const int qmin = key - koff - (q0 + W * h);
      // the L / D vectors arrived with Q_it (TMA): observe that barrier too
      if (!warp_wait(BAR_QF(st), (it >> 1) & 1, abort_flag)) { ok = false; break; }
      if (!warp_wait(BAR_S, it & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float p[W];
      tmem_ld32(tmem + lane_base + C::kColS + W * h, p);
      tmem_ld32(tmem + lane_base + C::kColS + W * h + 32, p + 32);
      tmem_ld_wait();
      const float4* l2 = reinterpret_cast<const float4*>(vec + W * h);
      const float2 sc2 = make_float2(scale_log2, scale_log2);
#pragma unroll
      for (int c = 0; c < W; c += 2) {
        const float4 l = l2[c >> 2];
        const float2 nl = (c & 2) ? make_float2(-l.z, -l.w) : make_float2(-l.x, -l.y);
        const float2 x = ffma2(make_float2(p[c], p[c + 1]), sc2, nl);
        float2 e;
        if (((c >> 1) & 3) < kPolyPairsPer4) {
          e = exp2_poly2(x);  // FMA pipe
        } else {
          e.x = ex2_mufu(x.x);  // MUFU pipe
          e.y = ex2_mufu(x.y);
        }
        p[c] = e.x;
        p[c + 1] = e.y;
      }
      if (need_mask) {
        const bool key_ok = key < Nk;
#pragma unroll
        for (int c = 0; c < W; ++c)
          if (!key_ok || (CAUSAL && c < qmin)) p[c] = 0.f;
      }
      {
        uint32_t pk[W / 2];
#pragma unroll
        for (int c = 0; c < W / 2; ++c) pk[c] = pack2_u32<BF16>(p[2 * c], p[2 * c + 1]);
        tmem_st32u(tmem + lane_base + C::kColS + W * h, pk);  // P^T over this warp's S^T
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_P);

      if (!warp_wait(BAR_DP, it & 1, abort_flag)) { ok = false; break; }
      // the dS^T tile was last read by the products of step it - kDsBufs
      const int dsb = it % C::kDsBufs;
      if (it >= C::kDsBufs &&
          !warp_wait(BAR_DSE(dsb), ((it / C::kDsBufs) - 1) & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float4* dd = reinterpret_cast<const float4*>(vec + BQ + W * h);
      // this warp's W queries = 8 16-byte chunks of row krow in block h,
      // formed and stored 32 queries (4 chunks) at a time
      uint8_t* dst = sp + C::kOffDS + dsb * C::kDsTile + h * C::kBlk;
#pragma unroll
      for (int half = 0; half < W / 32; ++half) {
        float dp[32];
        tmem_ld32(tmem + lane_base + C::kColDP + W * h + 32 * half, dp);
        tmem_ld_wait();
        uint32_t ds[16];
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 d4 = dd[(32 * half + c) >> 2];
          const int pc = 32 * half + c;
          const float2 a = fmul2(make_float2(p[pc], p[pc + 1]),
                                 fadd2(make_float2(dp[c], dp[c + 1]), make_float2(-d4.x, -d4.y)));
          const float2 bq = fmul2(make_float2(p[pc + 2], p[pc + 3]),
                                  fadd2(make_float2(dp[c + 2], dp[c + 3]), make_float2(-d4.z, -d4.w)));
          ds[c >> 1] = pack2_u32<BF16>(a.x, a.y);
          ds[(c >> 1) + 1] = pack2_u32<BF16>(bq.x, bq.y);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(dst + sw128(krow, 4 * half + u)) =
              make_uint4(ds[4 * u], ds[4 * u + 1], ds[4 * u + 2], ds[4 * u + 3]);
        // and packed over the dP^T columns just read (the A operand of dK)
        tmem_st16u(tmem + lane_base + C::kColDP + W * h + 16 * half, ds);
      }
      tmem_st_wait();
      // dP^T has been read (the dQ product may overwrite it after ds_full)
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_DS);
    }

    // ---- dV (warps 0-3) / dK (warps 4-7, scaled) of this key row
    if (ok && warp_wait(BAR_FIN, 0, abort_flag)) {
      tc_fence_after();
      using T = typename E::T;
      const uint32_t col = h ? C::kColDK : C::kColDV;
      const float mul = h ? scale : 1.f;
      T* out = reinterpret_cast<T*>(h ? dk : dv) + ((size_t)bhk * Nk + key) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_base + col + c * 32, v);
        tmem_ld_wait();
        if (key < Nk) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack2_u32<BF16>(v[i] * mul, v[i + 1] * mul);
            w.y = pack2_u32<BF16>(v[i + 2] * mul, v[i + 3] * mul);
            w.z = pack2_u32<BF16>(v[i + 4] * mul, v[i + 5] * mul);
            w.w = pack2_u32<BF16>(v[i + 6] * mul, v[i + 7] * mul);
            *reinterpret_cast<uint4*>(out + c * 32 + i) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace bwd

B2A_DEFINE_ERROR_READER(backward)

// Workspace (fp32): L2 [B*H][Npad], D [B*H][Npad], dQ accumulator [B*H*N*D];
// Npad = N rounded up to 128 (every region starts 512-byte aligned).
int64_t backward_workspace_floats(int B, int H, int N, int D) {
  const int64_t npad = ((int64_t)N + bwd::kPadRows - 1) / bwd::kPadRows * bwd::kPadRows;
  return 2 * (int64_t)B * H * npad + (int64_t)B * H * N * D;
}

template <int D, bool BF16, bool CAUSAL>
static int launch_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                      const float* lse, void* dq, void* dk, void* dv, float* ws, int B, int H,
                      int Hkv, int N, int Nk, float scale, cudaStream_t stream) {
  using namespace bwd;
  using C = Cfg<D>;
  auto kern = bwd_main_kernel<D, BF16, CAUSAL>;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(B2A_ERR_CUDA, "cudaGetDevice failed");
  if (!attr_done[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(backward)");
    attr_done[dev] = true;
  }
  const int npad = (N + kPadRows - 1) / kPadRows * kPadRows;
  const long long rows_pad = (long long)B * H * npad;
  float* l2v = ws;
  float* dvec = ws + rows_pad;
  float* dq_acc = ws + 2 * rows_pad;
  bwd_prep_kernel<D, BF16><<<(unsigned)((rows_pad + 7) / 8), 256, 0, stream>>>(
      o, dout, lse, l2v, dvec, dq_acc, N, npad, rows_pad);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward prep launch");
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tdo, tk, tv, tdq;
  int rc = make_tmap_3d(&tq, q, dt, D, N, (uint64_t)B * H, 64, BQ, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tdo, dout, dt, D, N, (uint64_t)B * H, 64, BQ, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tk, k, dt, D, Nk, (uint64_t)B * Hkv, 64, BK, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tv, v, dt, D, Nk, (uint64_t)B * Hkv, 64, BK, true);
  if (rc == B2A_OK)  // 32 fp32 = 128-byte boxes, swizzled like the staging tile
    rc = make_tmap_3d(&tdq, dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, D, N, (uint64_t)B * H, 32,
                      BQ, true, 4);
  if (rc != B2A_OK) return rc;
  dim3 grid((unsigned)((Nk + BK - 1) / BK), (unsigned)(B * Hkv));
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tq, tdo, tk, tv, tdq, l2v, dvec, dk, dv, N, Nk,
                                                   npad, H, Hkv, scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward kernel launch");
  const size_t n = (size_t)B * H * N * D;
  bwd_dq_kernel<D, BF16><<<(unsigned)((n / 2 + 255) / 256), 256, 0, stream>>>(dq_acc, dq, n);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward dQ launch");
  return B2A_OK;
}

int backward_dispatch(const void* q, const void* k, const void* v, const void* o, const void* dout,
                      const float* lse, void* dq, void* dk, void* dv, float* ws, int B, int H,
                      int Hkv, int N, int Nk, int D, int dtype, int causal, float scale,
                      cudaStream_t stream) {
  const bool bf = dtype == B2A_BF16;
#define B2A_BW(DD, BB, CC)                                                                   \
  if (D == DD && bf == BB && (causal != 0) == CC)                                            \
    return launch_bwd<DD, BB, CC>(q, k, v, o, dout, lse, dq, dk, dv, ws, B, H, Hkv, N, Nk, \
                                  scale, stream);
  B2A_BW(64, false, false)
  B2A_BW(64, false, true)
  B2A_BW(64, true, false)
  B2A_BW(64, true, true)
  B2A_BW(128, false, false)
  B2A_BW(128, false, true)
  B2A_BW(128, true, false)
  B2A_BW(128, true, true)
#undef B2A_BW
  return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
}

}  // namespace b2a

// prefill_sm100.cu -- attention prefill forward on B200 (sm_100a).
//
// O = softmax(Q K^T * scale [causal]) V and L = logsumexp(Q K^T * scale) per
// query row, the computation of fa3db_full_fwd_kernel in the reference
// (cuda/flash_attn_fa3_db_full.cu:87-344), re-designed for Blackwell:
//
//   * a CTA processes blocks of (256 query rows = two 128-row Q tiles, query
//     head); dense launches are persistent (one CTA per SM, blocks dealt out
//     by a static schedule, see kSched*) and load the next block's Q and issue
//     its first S while the softmax warps write the previous block's O;
//   * warp 8 (TMA producer): Q0/Q1 once, then K_j / V_j tiles (128 keys) into
//     a ring of kStages shared-memory stages, 128-byte swizzled (3-D tensor
//     maps {D, N, B*Hkv}: rows >= N read as zero);
//   * warp 9 (MMA issuer, TMEM owner): S_t = Q_t K_j^T (SS UMMA, M=128 N=128
//     K=D) into TMEM S_t, and O_t += P_t V_j (TS UMMA: P_t read from TMEM,
//     V_j from shared memory, M=128 N=D K=128) into TMEM O_t;
//   * warps 0-3 / 4-7 (softmax warpgroups for Q tile 0 / 1): thread r owns
//     query row r = TMEM lane r.  It loads its S row, applies the tail /
//     causal mask, keeps the running max in the log2 domain, rescales O_t in
//     TMEM only when the max grows by more than kRescaleThreshold (the
//     reference rescales every tile, cuda/flash_attn_fa3_db_full.cu:258-300),
//     and writes P = exp2(S - m) as packed 16-bit pairs back over S_t in TMEM
//     (the reference packs P into registers, :286-293).  At the end it
//     normalises O_t by the row sum and writes O and L = m ln2 + ln l (:340).
//
// VARLEN: sequences of different lengths packed token-major, q [total_q, H,
// D] and k/v [total_k, Hkv, D], sequence b owning tokens cu_q[b] ..
// cu_q[b+1]-1 (and cu_k[b] .. cu_k[b+1]-1 of the keys).  The tensor maps are
// then {D, heads, total} with box {64, 1, 128}: a box lands in shared memory
// as the same 128 rows x 128 bytes as a {D, N, B*H} box, so the rest of the
// kernel is unchanged.  A tile that runs past its sequence reads the next
// sequence's rows: keys there are masked like keys past Nk, query rows there
// are not stored.  The causal mask is aligned per sequence to its last key;
// a query row that sees no key gets O = 0 and L = -inf.
//
// The two Q tiles ping-pong: while one warpgroup runs its softmax the tensor
// core runs the other tile's PV and next S, so the MUFU/FMA work of the
// softmax and the UMMA work overlap.
#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {

namespace prefill {

constexpr int BM = 128;              // rows per Q tile (= UMMA M = TMEM lanes)
constexpr int BN = 128;              // keys per KV tile (= UMMA N of S)
constexpr int kQTiles = 2;           // Q tiles per CTA
constexpr int kRowsPerCta = BM * kQTiles;
constexpr int kThreads = 384;        // 2 softmax warpgroups + {producer, MMA, 2 idle}
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
// Register split: launched at kLaunchRegs per thread (the most 12 warps can
// have), the producer/MMA warpgroup gives registers to the softmax ones:
// 128 * kRegsCtrl + 256 * kRegsSoftmax <= 384 * kLaunchRegs.
constexpr uint32_t kLaunchRegs = 168;
constexpr uint32_t kRegsCtrl = 112;
constexpr uint32_t kRegsSoftmax = 192;
static_assert(128 * kRegsCtrl + 256 * kRegsSoftmax <= kThreads * kLaunchRegs,
              "register split must fit the launch allocation");
constexpr uint32_t kTmemCols = 512;  // S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D)
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8

template <int D>
struct Cfg {
  static constexpr int kStages = (D == 64) ? 4 : 2;
  static constexpr int kBlocks = D / 64;  // 64-element (128-byte) column blocks per row
  static constexpr uint32_t kQBytes = BM * D * 2;  // one Q tile
  static constexpr uint32_t kKVBytes = BN * D * 2;
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffK = kOffQ + kQTiles * kQBytes;
  static constexpr uint32_t kOffV = kOffK + kStages * kKVBytes;
  static constexpr uint32_t kOffBar = kOffV + kStages * kKVBytes;
  // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], pv_done[2], q_empty
  static constexpr int kNumBars = 1 + 3 * kStages + 7;
  static constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
  static constexpr uint32_t kOffAbort = kOffTmemSlot + 8;
  static constexpr uint32_t kSmemBytes = kOffAbort + 8 + 1024;  // + alignment slack
  static constexpr uint32_t kTmemO = 256;                         // O_t at kTmemO + t*D
};

// The blocks (query head, 256-row block) a CTA processes, in order.
//   * dense launches are persistent: gridDim.x = min(items, SMs) CTAs and CTA c
//     takes items c, c + gridDim.x, c + 2 gridDim.x, ...  Items are numbered
//     head-major, so the CTAs running at one time share the K/V of a few
//     heads in L2 instead of touching every head at once.
//   * under a causal mask an item pairs block j with block nqb-1-j of the same
//     head (heavier one first): their KV-tile counts add up to about the same
//     total for every item, so a static round-robin over items stays balanced
//     without any global counter.  Without a mask an item is one block.
//   * varlen launches keep one block per CTA: grid (B*H, blocks), grid.y
//     walked from the last block down.

// Block schedules of a dense launch (persistent: gridDim.x = min(items, SMs)
// CTAs, CTA c taking items c, c + gridDim.x, ...):
//   kSchedHeads  item = one block, numbered head-major (per = blocks per head);
//                every block costs the same without a causal mask.
//   kSchedPairs  causal: item j of a head = blocks (nqb-1-j, j), heavier first
//                (per = items per head).  Their KV-tile counts add up to about
//                the same for every item, so round-robin stays balanced with no
//                global counter, and items numbered head-major keep the CTAs
//                running at one time on the K/V of a few heads (L2 reuse).
//   kSchedSnake  causal with few items per CTA: single blocks sorted heaviest
//                first (per = heads), dealt boustrophedon -- round r left to
//                right, round r+1 right to left -- so the light blocks of the
//                last rounds even out the heavy ones of the first.
constexpr int kSchedHeads = 0;
constexpr int kSchedPairs = 1;
constexpr int kSchedSnake = 2;

template <int D, bool BF16, bool CAUSAL, bool VARLEN>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, void* __restrict__ out,
                       float* __restrict__ lse, int N, int Nk, int H, int group, float scale_log2,
                       const int* __restrict__ cu_q, const int* __restrict__ cu_k, int total_q,
                       int sched, int n_items, int per, int nqb) {
  using C = Cfg<D>;
  using E = Elem<BF16>;
  constexpr int S = C::kStages;
  // of every 8 consecutive (even, odd) score pairs, this many take the
  // polynomial exp2 on the FMA pipe and the rest the MUFU ex2, so that the two
  // pipes share the exponentials of a tile
  constexpr int kPolyPairsPer8 = (D == 64) ? 3 : 2;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;  // 1024-aligned: 128B-swizzle atoms
  uint8_t* sp = smem_raw + (sb - raw);

  const uint32_t sQ = sb + C::kOffQ;
  const uint32_t sK = sb + C::kOffK;
  const uint32_t sV = sb + C::kOffV;
  const uint32_t bar0 = sb + C::kOffBar;
  const uint32_t BAR_Q = bar0;
  auto BAR_KF = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_VF = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto BAR_KVE = [&](int s) { return bar0 + 8u * (1 + 2 * S + s); };
  auto BAR_SF = [&](int t) { return bar0 + 8u * (1 + 3 * S + t); };
  auto BAR_PF = [&](int t) { return bar0 + 8u * (3 + 3 * S + t); };
  auto BAR_PVD = [&](int t) { return bar0 + 8u * (5 + 3 * S + t); };
  const uint32_t BAR_QE = bar0 + 8u * (7 + 3 * S);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sp + C::kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sp + C::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // the CTA's position in its block sequence: item k, block `sub` of the item
  int it_k = VARLEN ? 0 : (int)blockIdx.x, it_sub = 0;
  if constexpr (VARLEN) {
    // a CTA whose block starts past its sequence has nothing to do
    const int b = (int)blockIdx.x / H;
    const int n_b = cu_q[b + 1] - cu_q[b];
    const int qb = (int)gridDim.y - 1 - (int)blockIdx.y;
    if (blockIdx.y == 0 && threadIdx.x == 0 &&
        (n_b > (int)gridDim.y * kRowsPerCta || n_b < 0 || cu_k[b + 1] - cu_k[b] < 0))
      atomicOr(&g_error_flags, 8u);  // sequence longer than max_seqlen_q, or bad cu_seqlens
    if (qb * kRowsPerCta >= n_b) return;
  }
  // Next block (bh, qb) of this CTA; false when it has no more (see kSched*).
  // Varlen: the one block (grid.x, grid.y walked from the last block down).
  auto next_block = [&](int& bh, int& qb) -> bool {
    if constexpr (VARLEN) {
      if (it_k > 0) return false;
      it_k = 1;
      bh = (int)blockIdx.x;
      qb = (int)gridDim.y - 1 - (int)blockIdx.y;
      return true;
    } else {
      if (sched == kSchedSnake) {
        // round r takes list entry r*G + c (even r) or r*G + G-1-c (odd r) of
        // the blocks sorted heaviest first (query block descending, heads inner)
        const int G = (int)gridDim.x, c = (int)blockIdx.x;
        const int rounds = (n_items + G - 1) / G;
        while (it_sub < rounds) {
          const int r = it_sub++;
          const int idx = r * G + ((r & 1) ? G - 1 - c : c);
          if (idx < n_items) {
            qb = nqb - 1 - idx / per;
            bh = idx % per;
            return true;
          }
        }
        return false;
      }
      if (it_k >= n_items) return false;
      const int j = it_k % per;
      bh = it_k / per;
      const bool pairs = CAUSAL && sched == kSchedPairs;
      qb = (pairs && it_sub == 0) ? nqb - 1 - j : j;
      const int ns = (pairs && 2 * j + 1 != nqb) ? 2 : 1;
      if (++it_sub >= ns) {
        it_sub = 0;
        it_k += (int)gridDim.x;
      }
      return true;
    }
  };

  // Per-block geometry, identical in every role.  Tensor-map coordinates
  // (row, head) of a Q tile / KV tile:
  //   dense  {D, N, B*H}:     y = row, z = b*H + h
  //   varlen {D, H, total}:   y = h,   z = first token of the sequence + row
  struct Geo {
    int bh, q0, Nb, Nkb, koff, q_first, k_first, q_head, k_head, nkv;
    int nkv_t[kQTiles];
  };
  auto geometry = [&](int bh, int qb) {
    Geo g;
    g.bh = bh;
    g.q0 = qb * kRowsPerCta;
    g.Nb = N;
    g.Nkb = Nk;
    g.q_first = 0;
    g.k_first = 0;
    g.q_head = bh;
    g.k_head = (bh / H) * (H / group) + (bh % H) / group;
    if constexpr (VARLEN) {
      const int b = bh / H;
      g.q_first = cu_q[b];
      g.k_first = cu_k[b];
      g.Nb = cu_q[b + 1] - g.q_first;
      g.Nkb = cu_k[b + 1] - g.k_first;
      g.q_head = bh % H;
      g.k_head = g.q_head / group;
    }
    // keys: Nk (>= N when causal); the causal mask is aligned to the bottom
    // right, query row r sees keys <= r + (Nk - N)
    g.koff = g.Nkb - g.Nb;
    const int nkv_all = (g.Nkb + BN - 1) / BN;
#pragma unroll
    for (int t = 0; t < kQTiles; ++t) {
      g.nkv_t[t] =
          CAUSAL ? min(nkv_all, (g.q0 + (t + 1) * BM + g.koff + BN - 1) / BN) : nkv_all;
      // varlen: a tile whose rows see no key (Nk == 0, or a causal offset below
      // zero) still runs one fully masked KV tile, so every role sees >= 1 tile
      if (VARLEN) g.nkv_t[t] = max(g.nkv_t[t], 1);
    }
    g.nkv = g.nkv_t[kQTiles - 1];
    return g;
  };
  auto tile_y = [&](int row, int head, int first) { return VARLEN ? head : row; };
  auto tile_z = [&](int row, int head, int first) { return VARLEN ? first + row : head; };

  if (warp == kProducerWarp && lane == 0) {
    for (int i = 0; i < C::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      // p_full collects one arrival per softmax warp, the rest one arrival
      // (expect_tx from the producer or a tcgen05.commit)
      const bool per_warp = bar == BAR_PF(0) || bar == BAR_PF(1);
      mbar_init(bar, per_warp ? 4u : 1u);
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

  if (warp >= 8) {
    setmaxnreg_dec<kRegsCtrl>();
    if (warp == kProducerWarp) {
      // ------------------------------------------------------------ producer
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        int kv = 0;  // K/V tiles loaded so far (ring position)
        bool ok = true;
        int bh, qb;
        for (int blk = 0; ok && next_block(bh, qb); ++blk) {
          const Geo g = geometry(bh, qb);
          // Q is reloaded once every S of the previous block has run
          if (blk > 0 && !mbar_wait(BAR_QE, (blk - 1) & 1, abort_flag)) break;
          mbar_arrive_expect_tx(BAR_Q, kQTiles * C::kQBytes);
#pragma unroll
          for (int t = 0; t < kQTiles; ++t)
#pragma unroll
            for (int c = 0; c < C::kBlocks; ++c)
              tma_load_3d(sQ + t * C::kQBytes + c * (BM * 128), &tmQ, BAR_Q, c * 64,
                          tile_y(g.q0 + t * BM, g.q_head, g.q_first),
                          tile_z(g.q0 + t * BM, g.q_head, g.q_first));
          for (int j = 0; j < g.nkv; ++j, ++kv) {
            const int st = kv % S;
            if (kv >= S && !mbar_wait(BAR_KVE(st), ((kv / S) - 1) & 1, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t k_dst = sK + st * C::kKVBytes;
            const uint32_t v_dst = sV + st * C::kKVBytes;
            mbar_arrive_expect_tx(BAR_KF(st), C::kKVBytes);
#pragma unroll
            for (int c = 0; c < C::kBlocks; ++c)
              tma_load_3d(k_dst + c * (BN * 128), &tmK, BAR_KF(st), c * 64,
                          tile_y(j * BN, g.k_head, g.k_first), tile_z(j * BN, g.k_head, g.k_first));
            mbar_arrive_expect_tx(BAR_VF(st), C::kKVBytes);
#pragma unroll
            for (int c = 0; c < C::kBlocks; ++c)
              tma_load_3d(v_dst + c * (BN * 128), &tmV, BAR_VF(st), c * 64,
                          tile_y(j * BN, g.k_head, g.k_first), tile_z(j * BN, g.k_head, g.k_first));
          }
        }
      }
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc_qk = idesc_f16(BM, BN, BF16, false, false);
        constexpr uint32_t idesc_pv = idesc_f16(BM, D, BF16, false, true);
        auto issue_s = [&](int t, int st) {
          const uint32_t q_base = sQ + t * C::kQBytes;
          const uint32_t k_base = sK + st * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            const uint64_t ad = sdesc_sw128(q_base + off, 16, 1024);
            const uint64_t bd = sdesc_sw128(k_base + off, 16, 1024);
            umma_f16_ss(tmem + t * 128, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
        };
        auto issue_pv = [&](int t, int st, bool first) {
          const uint32_t v_base = sV + st * C::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t bd = sdesc_sw128(v_base + kk * 2048, BN * 128, 1024);
            umma_f16_ts(tmem + C::kTmemO + t * D, tmem + t * 128 + kk * 8, bd, idesc_pv,
                        (!first || kk > 0) ? 1u : 0u);
          }
        };
        int kv = 0;             // K/V tiles consumed so far (ring position)
        int np[kQTiles] = {};   // P tiles consumed so far, per Q tile
        bool ok = true;
        int bh, qb;
        for (int blk = 0; ok && next_block(bh, qb); ++blk) {
          const Geo g = geometry(bh, qb);
          if (!mbar_wait(BAR_Q, blk & 1, abort_flag)) break;
          if (!mbar_wait(BAR_KF(kv % S), (kv / S) & 1, abort_flag)) break;
          tc_fence_after();
          // S_t(0) of this block: S_t's last reader, the previous block's last
          // PV_t, was issued earlier by this thread and runs first
          issue_s(0, kv % S);
          umma_commit(BAR_SF(0));
          issue_s(1, kv % S);
          umma_commit(BAR_SF(1));
          if (g.nkv == 1) umma_commit(BAR_QE);
          for (int j = 0; j < g.nkv; ++j, ++kv) {
            const int st = kv % S;
            if (!mbar_wait(BAR_VF(st), (kv / S) & 1, abort_flag)) { ok = false; break; }
            bool k_next_ready = false;
#pragma unroll
            for (int t = 0; t < kQTiles; ++t) {
              if (j >= g.nkv_t[t]) continue;
              if (!mbar_wait(BAR_PF(t), np[t] & 1, abort_flag)) { ok = false; break; }
              ++np[t];
              // The first PV of a block overwrites O_t.  Its p_full arrivals
              // come after the softmax warps' epilogue of the previous block has
              // read O_t out of TMEM (same threads, in program order, tcgen05.ld
              // waited), so no separate barrier guards O_t.
              tc_fence_after();
              issue_pv(t, st, j == 0);
              // PV_t(j) and S_t(j+1) share one commit point: every commit point
              // costs the tensor pipe a bubble of ~100 clocks
              const bool s_next = j + 1 < g.nkv_t[t];
              if (s_next) {
                if (!k_next_ready) {
                  if (!mbar_wait(BAR_KF((kv + 1) % S), ((kv + 1) / S) & 1, abort_flag)) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  k_next_ready = true;
                }
                issue_s(t, (kv + 1) % S);
              }
              umma_commit(BAR_PVD(t));
              if (s_next) umma_commit(BAR_SF(t));
              // the block's last S (tile 1, KV tile nkv-1) frees Q for the next block
              if (s_next && t == kQTiles - 1 && j + 2 == g.nkv) umma_commit(BAR_QE);
            }
            if (!ok) break;
            umma_commit(BAR_KVE(st));  // K_j / V_j free once every MMA above has run
          }
        }
      }
    }
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax warpgroups
    const int t = warp >> 2;           // Q tile of this warpgroup
    const int row = threadIdx.x & 127;  // TMEM lane
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_base + t * 128;
    const uint32_t t_o = tmem + lane_base + C::kTmemO + t * D;
    int n0 = 0;  // S / P / PV events of this Q tile before the current block
    bool ok = true;
    int bh, qb;
    while (ok && next_block(bh, qb)) {
      const Geo g = geometry(bh, qb);
      const int grow = g.q0 + t * BM + row;
      const int my_nkv = g.nkv_t[t];
      float m_run = -INFINITY;  // running max of scaled scores, log2 units
      float l_run = 0.f;

      for (int j = 0; j < my_nkv; ++j) {
        if (!mbar_wait(BAR_SF(t), (n0 + j) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(t_s + c * 32, s + c * 32);
        tmem_ld_wait();

        const int kv0 = j * BN;
        const bool need_mask =
            (kv0 + BN > g.Nkb) || (CAUSAL && kv0 + BN > g.q0 + t * BM + g.koff);
        if (need_mask) {
          const int lim = (CAUSAL ? min(g.Nkb, grow + 1 + g.koff) : g.Nkb) - kv0;  // first masked column
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (c >= lim) s[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(s[i], s[i + 8]);
#pragma unroll
        for (int c = 16; c < BN; c += 16)
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = fmax3(mx8[i], s[c + i], s[c + 8 + i]);
        const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                               fmaxf(mx8[6], mx8[7]));
        const float m_tile = mx * scale_log2;
        const float m_new = fmaxf(m_run, m_tile);
        const bool rescale = m_new > m_run + kRescaleThreshold;  // true on the first tile
        float alpha = 1.f;
        if (rescale) {
          alpha = ex2_mufu(m_run - m_new);  // 0 when m_run == -inf
          m_run = m_new;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 sc2 = make_float2(scale_log2, scale_log2);
        const float2 nm2 = make_float2(-m_use, -m_use);
        float2 rs[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) rs[i] = make_float2(0.f, 0.f);
        uint32_t pk[BN / 2];
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
          const float2 x = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
          float2 p;
          if (((c >> 1) & 7) < kPolyPairsPer8) {
            p = exp2_poly2(x);  // FMA pipe
          } else {
            p.x = ex2_mufu(x.x);  // MUFU pipe
            p.y = ex2_mufu(x.y);
          }
          rs[(c >> 1) & 3] = fadd2(rs[(c >> 1) & 3], p);
          pk[c >> 1] = pack2_u32<BF16>(p.x, p.y);
        }
        const float2 r01 = fadd2(fadd2(rs[0], rs[1]), fadd2(rs[2], rs[3]));
        l_run = l_run * alpha + (r01.x + r01.y);

        // O_t is still being accumulated by PV_{j-1}; rescale it once that is done
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          if (!mbar_wait(BAR_PVD(t), (n0 + j - 1) & 1, abort_flag)) { ok = false; break; }
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
        // P over S_t: 128 16-bit values = 64 packed columns
        tmem_st32u(t_s, pk);
        tmem_st32u(t_s + 32, pk + 32);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(BAR_PF(t));
      }

      // ---------------------------------------------------------- epilogue
      if (ok && mbar_wait(BAR_PVD(t), (n0 + my_nkv - 1) & 1, abort_flag)) {
        tc_fence_after();
        // a row that saw no key (varlen only) keeps m_run = -inf: O = 0, L = -inf
        const bool no_key = VARLEN && m_run == -INFINITY;
        const float inv_l = no_key ? 0.f : 1.f / l_run;
        const size_t orow_idx =
            VARLEN ? ((size_t)(g.q_first + grow) * H + g.q_head) : ((size_t)bh * g.Nb + grow);
        typename E::T* orow = reinterpret_cast<typename E::T*>(out) + orow_idx * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(t_o + c * 32, o);
          tmem_ld_wait();
          if (grow < g.Nb) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 w;
              w.x = pack2_u32<BF16>(o[i] * inv_l, o[i + 1] * inv_l);
              w.y = pack2_u32<BF16>(o[i + 2] * inv_l, o[i + 3] * inv_l);
              w.z = pack2_u32<BF16>(o[i + 4] * inv_l, o[i + 5] * inv_l);
              w.w = pack2_u32<BF16>(o[i + 6] * inv_l, o[i + 7] * inv_l);
              *reinterpret_cast<uint4*>(orow + c * 32 + i) = w;
            }
          }
        }
        if (lse != nullptr && grow < g.Nb) {
          // dense L [B, H, N]; varlen L [H, total_q]
          const size_t li = VARLEN ? ((size_t)g.q_head * total_q + g.q_first + grow)
                                   : ((size_t)bh * g.Nb + grow);
          // one explicit rounding (fma) so that every instantiation agrees bitwise
          lse[li] = no_key ? -INFINITY : __fmaf_rn(m_run, 0.69314718055994531f, logf(l_run));
        }
      } else {
        ok = false;
      }
      n0 += my_nkv;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace prefill

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
// Dense: N, Nk are the sequence lengths.  Varlen (cu_q != nullptr): N is
// max_seqlen_q (it sizes the grid), total_q / total_k the packed token counts.
template <int D, bool BF16, bool CAUSAL, bool VARLEN>
static int launch_prefill(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                          int H, int Hkv, int N, int Nk, float scale, const int* cu_q,
                          const int* cu_k, int total_q, int total_k, cudaStream_t stream) {
  using namespace prefill;
  using C = Cfg<D>;
  auto kern = prefill_fwd_kernel<D, BF16, CAUSAL, VARLEN>;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(B2A_ERR_CUDA, "cudaGetDevice failed");
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::kSmemBytes);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(prefill)");
    attr_done[dev] = true;
  }
  CUtensorMap tq, tk, tv;
  const CUtensorMapDataType dt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc;
  if (VARLEN) {
    rc = make_tmap_tokens(&tq, q, dt, D, H, total_q, 64, BM);
    if (rc != B2A_OK) return rc;
    rc = make_tmap_tokens(&tk, k, dt, D, Hkv, total_k, 64, BN);
    if (rc != B2A_OK) return rc;
    rc = make_tmap_tokens(&tv, v, dt, D, Hkv, total_k, 64, BN);
  } else {
    rc = make_tmap_3d(&tq, q, dt, D, N, (uint64_t)B * H, 64, BM, /*swizzle128=*/true);
    if (rc != B2A_OK) return rc;
    rc = make_tmap_3d(&tk, k, dt, D, Nk, (uint64_t)B * Hkv, 64, BN, true);
    if (rc != B2A_OK) return rc;
    rc = make_tmap_3d(&tv, v, dt, D, Nk, (uint64_t)B * Hkv, 64, BN, true);
  }
  if (rc != B2A_OK) return rc;
  const int nqb = (N + kRowsPerCta - 1) / kRowsPerCta;
  dim3 grid;
  int sched = kSchedHeads, n_items = 1, per = 1;
  if (VARLEN) {
    grid = dim3((unsigned)(B * H), (unsigned)nqb);
  } else {
    static int sms[kMaxDevices] = {};
    if (sms[dev] == 0) {
      cudaError_t e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return set_cuda_error(e, "cudaDeviceGetAttribute(SM count)");
    }
    const int64_t bh = (int64_t)B * H;
    if ((bh * nqb) > 0x7fffffff) return set_error(B2A_ERR_INVALID_ARG, "B*H*blocks too large");
    if (!CAUSAL) {
      sched = kSchedHeads;
      per = nqb;
      n_items = (int)(bh * nqb);
    } else if (bh * ((nqb + 1) / 2) >= 6LL * sms[dev]) {
      // six or more pair items per CTA: pairs balance to within ~1%
      sched = kSchedPairs;
      per = (nqb + 1) / 2;
      n_items = (int)(bh * per);
    } else {
      sched = kSchedSnake;
      per = (int)bh;
      n_items = (int)(bh * nqb);
    }
    grid = dim3((unsigned)(n_items < sms[dev] ? n_items : sms[dev]));
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tq, tk, tv, o, lse, N, Nk, H, H / Hkv, scale_log2,
                                                  cu_q, cu_k, total_q, sched, n_items, per,
                                                  nqb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "prefill kernel launch");
  return B2A_OK;
}

B2A_DEFINE_ERROR_READER(prefill)

int prefill_dispatch(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H,
                     int Hkv, int N, int Nk, int D, int dtype, int causal, float scale,
                     cudaStream_t stream) {
  const bool bf = dtype == B2A_BF16;
  // D = 64: the split-row kernel of prefill_d64_sm100.cu
  if (D == 64) return prefill_d64_dispatch(q, k, v, o, lse, B, H, Hkv, N, Nk, dtype, causal, scale, stream);
#define B2A_PF(DD, BB, CC) \
  if (D == DD && bf == BB && (causal != 0) == CC) \
    return launch_prefill<DD, BB, CC, false>(q, k, v, o, lse, B, H, Hkv, N, Nk, scale, nullptr, \
                                             nullptr, 0, 0, stream);
  B2A_PF(128, false, false)
  B2A_PF(128, false, true)
  B2A_PF(128, true, false)
  B2A_PF(128, true, true)
#undef B2A_PF
  return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
}

// Varlen prefill, D = 64 or 128 (D = 64 also runs this kernel: the split-row
// D = 64 kernel has no varlen form).
int prefill_varlen_dispatch(const void* q, const void* k, const void* v, void* o, float* lse,
                            const int* cu_q, const int* cu_k, int B, int H, int Hkv, int total_q,
                            int total_k, int max_seqlen_q, int D, int dtype, int causal,
                            float scale, cudaStream_t stream) {
  const bool bf = dtype == B2A_BF16;
#define B2A_PV(DD, BB, CC)                                                                   \
  if (D == DD && bf == BB && (causal != 0) == CC)                                            \
    return launch_prefill<DD, BB, CC, true>(q, k, v, o, lse, B, H, Hkv, max_seqlen_q, 0, scale, \
                                            cu_q, cu_k, total_q, total_k, stream);
  B2A_PV(64, false, false)
  B2A_PV(64, false, true)
  B2A_PV(64, true, false)
  B2A_PV(64, true, true)
  B2A_PV(128, false, false)
  B2A_PV(128, false, true)
  B2A_PV(128, true, false)
  B2A_PV(128, true, true)
#undef B2A_PV
  return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
}

}  // namespace b2a

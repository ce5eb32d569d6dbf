// prefill_sm100.cu -- attention prefill forward on B200 (sm_100a).
//
// O = softmax(Q K^T * scale [causal]) V and L = logsumexp(Q K^T * scale) per
// query row, the computation of fa3db_full_fwd_kernel in the reference
// (cuda/flash_attn_fa3_db_full.cu:87-344), re-designed for Blackwell:
//
//   * one CTA per (128 query rows, query head); grid.y walks query tiles from
//     the last (heaviest under the causal mask) to the first;
//   * warp 4  (TMA producer): Q once, then K_j / V_j tiles into a ring of
//     kStages shared-memory stages with 128-byte swizzle (3-D tensor maps
//     {D, N, B*Hkv}, so rows >= N read as zero);
//   * warp 5  (MMA issuer, TMEM owner): S_j = Q K_j^T (M=128, N=128, K=D) into
//     one of two TMEM S buffers, and O += P_j V_j (M=128, N=D, K=128) into the
//     TMEM O accumulator; completion is signalled by tcgen05.commit;
//   * warps 0-3 (softmax + correction + epilogue): thread r owns query row r =
//     TMEM lane r.  It loads its S row, applies the tail / causal mask, keeps
//     the running max in the log2 domain and rescales O in TMEM only when the
//     max grows by more than kRescaleThreshold (the reference rescales every
//     tile, cuda/flash_attn_fa3_db_full.cu:258-300), writes P = exp2(S - m) in
//     the input dtype into a swizzled shared-memory tile for the PV UMMA, and
//     finally normalises O by the row sum and writes O and L
//     (L = m ln2 + ln l, cuda/flash_attn_fa3_db_full.cu:340).
//
// Because the S buffers are double-buffered, S_{j+1} runs on the tensor core
// while the softmax warps work on S_j, and PV_j runs while they work on S_{j+1}.
#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {

namespace prefill {

constexpr int BM = 128;               // query rows per CTA (= UMMA M = TMEM lanes)
constexpr int BN = 128;               // keys per KV tile (= UMMA N of S)
constexpr int kThreads = 192;         // 4 softmax warps + producer + MMA
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 512;   // S0 [0,128) S1 [128,256) O [256,256+D)
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays <= 2^8

template <int D>
struct Cfg {
  static constexpr int kStages = (D == 64) ? 4 : 2;
  static constexpr int kBlocks = D / 64;  // 64-element (128-byte) column blocks per row
  static constexpr uint32_t kQBytes = BM * D * 2;
  static constexpr uint32_t kKVBytes = BN * D * 2;
  static constexpr uint32_t kPBytes = BM * BN * 2;
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffK = kOffQ + kQBytes;
  static constexpr uint32_t kOffV = kOffK + kStages * kKVBytes;
  static constexpr uint32_t kOffP = kOffV + kStages * kKVBytes;
  static constexpr uint32_t kOffBar = kOffP + kPBytes;
  static constexpr int kNumBars = 1 + 3 * kStages + 6;
  static constexpr uint32_t kOffTmemSlot = kOffBar + 8 * kNumBars;
  static constexpr uint32_t kOffAbort = kOffTmemSlot + 8;
  static constexpr uint32_t kSmemBytes = kOffAbort + 8 + 1024;  // + alignment slack
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D, bool BF16, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, void* __restrict__ out,
                       float* __restrict__ lse, int N, int H, int group, float scale_log2) {
  using C = Cfg<D>;
  using E = Elem<BF16>;
  constexpr int S = C::kStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;  // 1024-aligned: 128B-swizzle atoms
  uint8_t* sp = smem_raw + (sb - raw);

  const uint32_t sQ = sb + C::kOffQ;
  const uint32_t sK = sb + C::kOffK;
  const uint32_t sV = sb + C::kOffV;
  const uint32_t sP = sb + C::kOffP;
  const uint32_t bar0 = sb + C::kOffBar;
  auto BAR_Q = [&]() { return bar0; };
  auto BAR_KF = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_VF = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto BAR_KVE = [&](int s) { return bar0 + 8u * (1 + 2 * S + s); };
  auto BAR_SF = [&](int b) { return bar0 + 8u * (1 + 3 * S + b); };
  auto BAR_SE = [&](int b) { return bar0 + 8u * (3 + 3 * S + b); };
  const uint32_t BAR_PF = bar0 + 8u * (5 + 3 * S);
  const uint32_t BAR_PVD = bar0 + 8u * (6 + 3 * S);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(sp + C::kOffTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sp + C::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int bhk = (bh / H) * (H / group) + (bh % H) / group;  // KV head of this query head
  const int qt = (int)gridDim.y - 1 - (int)blockIdx.y;
  const int q0 = qt * BM;
  const int nkv_all = (N + BN - 1) / BN;
  const int nkv = CAUSAL ? min(nkv_all, (q0 + BM + BN - 1) / BN) : nkv_all;

  if (warp == kProducerWarp && lane == 0) {
    // s_empty / p_full collect one arrival per softmax warp, the rest one
    // arrival (expect_tx from the producer or a tcgen05.commit)
    for (int i = 0; i < C::kNumBars; ++i) {
      const uint32_t bar = bar0 + 8u * i;
      const bool per_warp = bar == BAR_SE(0) || bar == BAR_SE(1) || bar == BAR_PF;
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

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(BAR_Q(), C::kQBytes);
#pragma unroll
      for (int c = 0; c < C::kBlocks; ++c)
        tma_load_3d(sQ + c * (BM * 128), &tmQ, BAR_Q(), c * 64, q0, bh);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % S;
        if (j >= S && !mbar_wait(BAR_KVE(st), ((j / S) - 1) & 1, abort_flag)) break;
        const uint32_t k_dst = sK + st * C::kKVBytes;
        const uint32_t v_dst = sV + st * C::kKVBytes;
        mbar_arrive_expect_tx(BAR_KF(st), C::kKVBytes);
#pragma unroll
        for (int c = 0; c < C::kBlocks; ++c)
          tma_load_3d(k_dst + c * (BN * 128), &tmK, BAR_KF(st), c * 64, j * BN, bhk);
        mbar_arrive_expect_tx(BAR_VF(st), C::kKVBytes);
#pragma unroll
        for (int c = 0; c < C::kBlocks; ++c)
          tma_load_3d(v_dst + c * (BN * 128), &tmV, BAR_VF(st), c * 64, j * BN, bhk);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(BM, BN, BF16, false, false);
      constexpr uint32_t idesc_pv = idesc_f16(BM, D, BF16, false, true);
      const uint32_t t_o = tmem + 256;
      bool ok = mbar_wait(BAR_Q(), 0, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int st = j % S, b = j & 1;
        if (!mbar_wait(BAR_KF(st), (j / S) & 1, abort_flag)) return false;
        if (j >= 2 && !mbar_wait(BAR_SE(b), ((j >> 1) - 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_base = sK + st * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(sQ + off, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_base + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
          umma_f16_ss(tmem + b * 128, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(BAR_SF(b));
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j % S;
        if (!mbar_wait(BAR_VF(st), (j / S) & 1, abort_flag)) return false;
        if (!mbar_wait(BAR_PF, j & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t v_base = sV + st * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(sP + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_base + kk * 2048, BN * 128, 1024);
          umma_f16_ss(t_o, ad, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(BAR_PVD);
        umma_commit(BAR_KVE(st));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv) ok = issue_s(j + 1);
        if (ok) ok = issue_pv(j);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    const int grow = q0 + row;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t t_o = tmem + lane_base + 256;
    float m_run = -INFINITY;  // running max of scaled scores, log2 units
    float l_run = 0.f;
    bool ok = true;
    uint8_t* prow = sp + C::kOffP + row * 128;

    for (int j = 0; j < nkv && ok; ++j) {
      const int b = j & 1;
      if (!mbar_wait(BAR_SF(b), (j >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(tmem + lane_base + b * 128 + c * 32, s + c * 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_SE(b));

      const int kv0 = j * BN;
      const bool need_mask = (kv0 + BN > N) || (CAUSAL && kv0 + BN > q0);
      if (need_mask) {
        const int lim = CAUSAL ? min(N, grow + 1) : N;  // first masked key
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (kv0 + c >= lim) s[c] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < BN; ++c) mx = fmaxf(mx, s[c]);
      const float m_tile = mx * scale_log2;
      const float m_new = fmaxf(m_run, m_tile);
      const bool rescale = m_new > m_run + kRescaleThreshold;  // true on the first tile
      float alpha = 1.f;
      if (rescale) {
        alpha = ex2(m_run - m_new);  // 0 when m_run == -inf
        m_run = m_new;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        s[c] = ex2(fmaf(s[c], scale_log2, -m_use));
        s[c + 1] = ex2(fmaf(s[c + 1], scale_log2, -m_use));
        rs0 += s[c];
        rs1 += s[c + 1];
      }
      l_run = l_run * alpha + (rs0 + rs1);

      // O and the P tile are still in use by PV_{j-1}
      if (j > 0) {
        if (!mbar_wait(BAR_PVD, (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            tmem_ld32(t_o + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(t_o + c * 32, o);
          }
          tmem_st_wait();
        }
      }
      // P row -> K-major 128B-swizzled tile: 16-byte chunk k8 of a row goes to
      // chunk (k8 ^ (row & 7)) of that row's 128-byte line.
#pragma unroll
      for (int blk = 0; blk < BN / 64; ++blk) {
#pragma unroll
        for (int k8 = 0; k8 < 8; ++k8) {
          const float* pv = s + blk * 64 + k8 * 8;
          uint4 w;
          w.x = pack2_u32<BF16>(pv[0], pv[1]);
          w.y = pack2_u32<BF16>(pv[2], pv[3]);
          w.z = pack2_u32<BF16>(pv[4], pv[5]);
          w.w = pack2_u32<BF16>(pv[6], pv[7]);
          *reinterpret_cast<uint4*>(prow + blk * (BM * 128) + ((k8 ^ (row & 7)) << 4)) = w;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_PF);
    }

    // ---------------------------------------------------------- epilogue
    if (ok && mbar_wait(BAR_PVD, (nkv - 1) & 1, abort_flag)) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      typename E::T* orow = reinterpret_cast<typename E::T*>(out) + ((size_t)bh * N + grow) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float o[32];
        tmem_ld32(t_o + c * 32, o);
        tmem_ld_wait();
        if (grow < N) {
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
      if (lse != nullptr && grow < N)
        lse[(size_t)bh * N + grow] = m_run * 0.69314718055994531f + logf(l_run);
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
template <int D, bool BF16, bool CAUSAL>
static int launch_prefill(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                          int H, int Hkv, int N, float scale, cudaStream_t stream) {
  using namespace prefill;
  using C = Cfg<D>;
  auto kern = prefill_fwd_kernel<D, BF16, CAUSAL>;
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
  int rc = make_tmap_3d(&tq, q, dt, D, N, (uint64_t)B * H, 64, BM, /*swizzle128=*/true);
  if (rc != B2A_OK) return rc;
  rc = make_tmap_3d(&tk, k, dt, D, N, (uint64_t)B * Hkv, 64, BN, true);
  if (rc != B2A_OK) return rc;
  rc = make_tmap_3d(&tv, v, dt, D, N, (uint64_t)B * Hkv, 64, BN, true);
  if (rc != B2A_OK) return rc;
  dim3 grid((unsigned)(B * H), (unsigned)((N + BM - 1) / BM));
  const float scale_log2 = scale * 1.4426950408889634f;
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tq, tk, tv, o, lse, N, H, H / Hkv, scale_log2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "prefill kernel launch");
  return B2A_OK;
}

B2A_DEFINE_ERROR_READER(prefill)

int prefill_dispatch(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H,
                     int Hkv, int N, int D, int dtype, int causal, float scale,
                     cudaStream_t stream) {
  const bool bf = dtype == B2A_BF16;
#define B2A_PF(DD, BB, CC) \
  if (D == DD && bf == BB && (causal != 0) == CC) \
    return launch_prefill<DD, BB, CC>(q, k, v, o, lse, B, H, Hkv, N, scale, stream);
  B2A_PF(64, false, false)
  B2A_PF(64, false, true)
  B2A_PF(64, true, false)
  B2A_PF(64, true, true)
  B2A_PF(128, false, false)
  B2A_PF(128, false, true)
  B2A_PF(128, true, false)
  B2A_PF(128, true, true)
#undef B2A_PF
  return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
}

}  // namespace b2a

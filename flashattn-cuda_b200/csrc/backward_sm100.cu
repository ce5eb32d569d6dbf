// backward_sm100.cu -- attention backward (dQ, dK, dV) on B200 (sm_100a).
//
// The reference computes the same gradients with three scalar FP32 kernels
// (cuda/flash_attn_kernel.cu:173-412): D_i = rowsum(dO * O), then dQ, then
// dK / dV, recomputing P = exp(S - L) from the saved logsumexp.  Here:
//
//   * bwd_prep_kernel: D_i = rowsum(dO * O) in fp32 and a zeroed fp32 dQ
//     accumulator (workspace);
//   * bwd_main_kernel: one CTA per (64-key block j, KV head).  It keeps K_j,
//     V_j in shared memory and dK_j, dV_j in registers, and walks every query
//     head of the KV head (GQA group) and every 64-row query block i that sees
//     block j (causal: from the diagonal on).  Per block:
//         S^T = K_j Q_i^T            P^T = exp2(S^T scale log2e - L_i log2e)
//         dV_j += P^T dO_i           dP^T = V_j dO_i^T
//         dS^T = P^T (dP^T - D_i)    dK_j += dS^T Q_i
//         dQ_i += dS K_j * scale  -> staged in shared memory, then ONE TMA bulk
//                                     reduce-add of the 64 x D fp32 tile into
//                                     the dQ accumulator (no per-element atomics)
//     Q_i / dO_i arrive by TMA (128-byte swizzle) into a 2-stage ring fed by a
//     producer warp; the products run on the tensor cores (mma.m16n8k16, each
//     of the 4 consumer warps owning 16 of the 64 keys);
//   * bwd_dq_kernel: dQ accumulator (fp32, already scaled) -> dtype.
#include <cstdio>

#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace bwd {

constexpr int BQ = 64;  // query rows per step
constexpr int BK = 64;  // keys per CTA (16 per consumer warp)
constexpr int kConsumers = 4;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kProducerWarp = kConsumers;
constexpr int kStages = 2;
constexpr int kDsStride = BQ + 8;  // halves per row of the dS^T tile (pad: no bank conflicts)

template <int D>
struct Cfg {
  static constexpr int kBlocks = D / 64;
  static constexpr uint32_t kTile = 64 * D * 2;  // one 64-row K, V, Q or dO tile
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = kOffK + kTile;
  static constexpr uint32_t kOffQ = kOffV + kTile;                // [kStages]
  static constexpr uint32_t kOffDO = kOffQ + kStages * kTile;     // [kStages]
  static constexpr uint32_t kOffDQ = kOffDO + kStages * kTile;    // fp32 [2][BQ][D]
  static constexpr uint32_t kOffDS = kOffDQ + 2 * BQ * D * 4;     // [BK][kDsStride]
  static constexpr uint32_t kOffBar = kOffDS + BK * kDsStride * 2;
  // kv_full, full[S], empty[S]
  static constexpr int kNumBars = 1 + 2 * kStages;
  static constexpr uint32_t kOffAbort = kOffBar + 8 * kNumBars;
  static constexpr uint32_t kSmemBytes = kOffAbort + 16 + 1024;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
template <bool BF16>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// byte offset of element (row r, column c) of a 64-row tile written by TMA
// with 128-byte swizzle in 64-column blocks
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((c >> 6) * (64 * 128) + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) +
                    (c & 7) * 2);
}

// D_i = rowsum(dO * O) (fp32) and a zeroed dQ accumulator; one warp per row.
template <int D, bool BF16>
__global__ void bwd_prep_kernel(const void* __restrict__ o, const void* __restrict__ dout,
                                float* __restrict__ dvec, float* __restrict__ dq_acc, int rows) {
  using E = Elem<BF16>;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  constexpr int EPL = D / 32;  // elements per lane (2 or 4)
  const typename E::T* op = reinterpret_cast<const typename E::T*>(o) + (size_t)row * D + lane * EPL;
  const typename E::T* dp =
      reinterpret_cast<const typename E::T*>(dout) + (size_t)row * D + lane * EPL;
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; e += 2) {
    const float2 a = E::unpack(*reinterpret_cast<const typename E::T2*>(op + e));
    const float2 b = E::unpack(*reinterpret_cast<const typename E::T2*>(dp + e));
    acc = fmaf(a.x, b.x, fmaf(a.y, b.y, acc));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) dvec[row] = acc;
  float* dqr = dq_acc + (size_t)row * D + lane * EPL;
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

template <int D, bool BF16, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_main_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmDQ, const float* __restrict__ lse,
                    const float* __restrict__ dvec, void* __restrict__ dk, void* __restrict__ dv,
                    int N, int Nk, int H, int Hkv, float scale) {
  using C = Cfg<D>;
  using E = Elem<BF16>;
  constexpr int S = kStages;
  constexpr float kLog2e = 1.4426950408889634f;
  const float scale_log2 = scale * kLog2e;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw);
  const uint32_t sK = sb + C::kOffK, sV = sb + C::kOffV;
  const uint32_t sQ = sb + C::kOffQ, sDO = sb + C::kOffDO;
  const uint32_t sDQ = sb + C::kOffDQ, sDS = sb + C::kOffDS;
  const uint32_t bar0 = sb + C::kOffBar;
  const uint32_t BAR_KV = bar0;
  auto BAR_F = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_E = [&](int s) { return bar0 + 8u * (1 + S + s); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sp + C::kOffAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x;           // key block
  const int bhk = blockIdx.y;         // b * Hkv + hkv
  const int b = bhk / Hkv, hkv = bhk % Hkv;
  const int G = H / Hkv;
  const int kv0 = j * BK;
  const int koff = Nk - N;  // causal: query row r sees keys <= r + koff
  const int nq = (N + BQ - 1) / BQ;
  const int i0 = CAUSAL ? max(0, (kv0 - koff) / BQ) : 0;
  const int steps = G * max(0, nq - i0);  // (query head, query block) pairs

  if (threadIdx.x == kProducerWarp * 32) {
    mbar_init(BAR_KV, 1u);
    for (int s = 0; s < S; ++s) {
      mbar_init(BAR_F(s), 1u);
      mbar_init(BAR_E(s), kConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ producer
    if (lane == 0 && steps > 0) {
      mbar_arrive_expect_tx(BAR_KV, 2 * C::kTile);
#pragma unroll
      for (int c = 0; c < C::kBlocks; ++c) {
        tma_load_3d(sK + c * (64 * 128), &tmK, BAR_KV, c * 64, kv0, bhk);
        tma_load_3d(sV + c * (64 * 128), &tmV, BAR_KV, c * 64, kv0, bhk);
      }
      for (int it = 0; it < steps; ++it) {
        const int st = it % S;
        if (it >= S && !mbar_wait(BAR_E(st), ((it / S) - 1) & 1, abort_flag)) break;
        const int g = it / (nq - i0), qi = i0 + it % (nq - i0);
        const int bh = b * H + hkv * G + g;
        mbar_arrive_expect_tx(BAR_F(st), 2 * C::kTile);
#pragma unroll
        for (int c = 0; c < C::kBlocks; ++c) {
          tma_load_3d(sQ + st * C::kTile + c * (64 * 128), &tmQ, BAR_F(st), c * 64, qi * BQ, bh);
          tma_load_3d(sDO + st * C::kTile + c * (64 * 128), &tmDO, BAR_F(st), c * 64, qi * BQ, bh);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumers
  const int g4 = lane >> 2, t4 = lane & 3;
  const int r0 = warp * 16;  // this warp's first key row in the block
  float dK[D / 8][4], dV[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dK[n][e] = dV[n][e] = 0.f;
  bool ok = steps == 0 || mbar_wait(BAR_KV, 0, abort_flag);

  for (int it = 0; it < steps; ++it) {
    const int st = it % S;
    if (ok) ok = mbar_wait(BAR_F(st), (it / S) & 1, abort_flag);
    // all consumer warps leave together if any wait gave up
    {
      uint32_t r;
      asm volatile(
          "{\n\t.reg .pred P, Q;\n\tsetp.ne.u32 P, %1, 0;\n\t"
          "bar.red.and.pred Q, 1, 128, P;\n\tselp.u32 %0, 1, 0, Q;\n\t}"
          : "=r"(r)
          : "r"((uint32_t)ok)
          : "memory");
      if (!r) break;
    }
    const int g = it / (nq - i0), qi = i0 + it % (nq - i0);
    const int bh = b * H + hkv * G + g;
    const int q0 = qi * BQ;
    const uint32_t q_base = sQ + st * C::kTile, do_base = sDO + st * C::kTile;

    // per-column (query) constants of this lane: columns 8n + 2 t4 + {0, 1}
    float l2[16], dd[16];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int q = q0 + 8 * n + 2 * t4 + e;
        const bool in = q < N;
        l2[2 * n + e] = in ? lse[(size_t)bh * N + q] * kLog2e : INFINITY;
        dd[2 * n + e] = in ? dvec[(size_t)bh * N + q] : 0.f;
      }

    // ---- S^T = K Q^T and dP^T = V dO^T (16 keys x 64 queries per warp)
    float sT[8][4], dpT[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) sT[n][e] = dpT[n][e] = 0.f;
#pragma unroll
    for (int kp = 0; kp < D / 32; ++kp) {  // two 16-column k-steps per pass
      uint32_t ak0[4], ak1[4], av0[4], av1[4];
      const int ar = r0 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int ac = 32 * kp + 8 * (lane >> 4);
      ldsm_x4(sK + sw_off(ar, ac), ak0);
      ldsm_x4(sK + sw_off(ar, ac + 16), ak1);
      ldsm_x4(sV + sw_off(ar, ac), av0);
      ldsm_x4(sV + sw_off(ar, ac + 16), av1);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        // B = Q^T / dO^T: query rows 8n..8n+7, columns 32kp + {0, 8, 16, 24}
        uint32_t bq[4], bo[4];
        const int br = 8 * n + (lane & 7), bc = 32 * kp + 8 * (lane >> 3);
        ldsm_x4(q_base + sw_off(br, bc), bq);
        ldsm_x4(do_base + sw_off(br, bc), bo);
        mma16816<BF16>(sT[n], ak0, bq[0], bq[1]);
        mma16816<BF16>(sT[n], ak1, bq[2], bq[3]);
        mma16816<BF16>(dpT[n], av0, bo[0], bo[1]);
        mma16816<BF16>(dpT[n], av1, bo[2], bo[3]);
      }
    }

    // ---- P^T and dS^T = P^T (dP^T - D)
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kv0 + r0 + g4 + 8 * (e >> 1);
        const int q = q0 + 8 * n + 2 * t4 + (e & 1);
        const bool valid = key < Nk && (!CAUSAL || key <= q + koff);
        const float p = valid ? exp2f(fmaf(sT[n][e], scale_log2, -l2[2 * n + (e & 1)])) : 0.f;
        sT[n][e] = p;
        dpT[n][e] = p * (dpT[n][e] - dd[2 * n + (e & 1)]);
      }

    // ---- dV += P^T dO and dK += dS^T Q  (k = 64 queries, n = D)
#pragma unroll
    for (int kq = 0; kq < 4; ++kq) {
      uint32_t ap[4], ads[4];
      ap[0] = pack2_u32<BF16>(sT[2 * kq][0], sT[2 * kq][1]);
      ap[1] = pack2_u32<BF16>(sT[2 * kq][2], sT[2 * kq][3]);
      ap[2] = pack2_u32<BF16>(sT[2 * kq + 1][0], sT[2 * kq + 1][1]);
      ap[3] = pack2_u32<BF16>(sT[2 * kq + 1][2], sT[2 * kq + 1][3]);
      ads[0] = pack2_u32<BF16>(dpT[2 * kq][0], dpT[2 * kq][1]);
      ads[1] = pack2_u32<BF16>(dpT[2 * kq][2], dpT[2 * kq][3]);
      ads[2] = pack2_u32<BF16>(dpT[2 * kq + 1][0], dpT[2 * kq + 1][1]);
      ads[3] = pack2_u32<BF16>(dpT[2 * kq + 1][2], dpT[2 * kq + 1][3]);
      if (kq == 0) {
        // dS^T of this warp's 16 keys -> shared memory (read back for dQ)
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          uint8_t* row_lo = sp + C::kOffDS + (size_t)(r0 + g4) * kDsStride * 2;
          uint8_t* row_hi = row_lo + 8 * kDsStride * 2;
          *reinterpret_cast<uint32_t*>(row_lo + (8 * n + 2 * t4) * 2) =
              pack2_u32<BF16>(dpT[n][0], dpT[n][1]);
          *reinterpret_cast<uint32_t*>(row_hi + (8 * n + 2 * t4) * 2) =
              pack2_u32<BF16>(dpT[n][2], dpT[n][3]);
        }
      }
#pragma unroll
      for (int nd = 0; nd < D / 8; nd += 2) {
        // B = dO / Q rows 16kq.. (k), columns 8nd.. (n): transposed loads
        const int br = 16 * kq + (lane & 7) + 8 * ((lane >> 3) & 1), bc = 8 * nd + 8 * (lane >> 4);
        uint32_t bo[4], bq[4];
        ldsm_x4_t(do_base + sw_off(br, bc), bo);
        ldsm_x4_t(q_base + sw_off(br, bc), bq);
        mma16816<BF16>(dV[nd], ap, bo[0], bo[1]);
        mma16816<BF16>(dV[nd + 1], ap, bo[2], bo[3]);
        mma16816<BF16>(dK[nd], ads, bq[0], bq[1]);
        mma16816<BF16>(dK[nd + 1], ads, bq[2], bq[3]);
      }
    }

    // ---- dQ_i += dS K * scale (this warp: queries 16w..16w+15, all D columns)
    asm volatile("bar.sync 1, 128;" ::: "memory");  // dS^T tile complete
    const uint32_t dq_buf = sDQ + (it & 1) * (BQ * D * 4);
    if (it >= 2 && warp == 0 && lane == 0) bulk_wait_group_read<1>();  // buffer reused
    asm volatile("bar.sync 1, 128;" ::: "memory");
    {
      float acc[D / 8][4];
#pragma unroll
      for (int n = 0; n < D / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        // A = dS (m = queries, k = keys) from the dS^T tile [keys][queries]
        uint32_t a[4];
        const int ar = 16 * kk + (lane & 7) + 8 * (lane >> 4), ac = 16 * warp + 8 * ((lane >> 3) & 1);
        // blocks (k 0-7, m 0-7), (k 0-7, m 8-15), (k 8-15, m 0-7), (k 8-15, m 8-15)
        // transposed: exactly the A fragment a0..a3
        ldsm_x4_t(sDS + (uint32_t)(ar * kDsStride + ac) * 2, a);
        const uint32_t* af = a;
#pragma unroll
        for (int nd = 0; nd < D / 8; nd += 2) {
          const int br = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1), bc = 8 * nd + 8 * (lane >> 4);
          uint32_t bk[4];
          ldsm_x4_t(sK + sw_off(br, bc), bk);
          mma16816<BF16>(acc[nd], af, bk[0], bk[1]);
          mma16816<BF16>(acc[nd + 1], af, bk[2], bk[3]);
        }
      }
      // stage the scaled fp32 tile (row-major [BQ][D]) for the bulk reduce
      float* dqs = reinterpret_cast<float*>(sp + (dq_buf - sb));
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        const int row = 16 * warp + g4, col = 8 * n + 2 * t4;
        *reinterpret_cast<float2*>(dqs + row * D + col) =
            make_float2(acc[n][0] * scale, acc[n][1] * scale);
        *reinterpret_cast<float2*>(dqs + (row + 8) * D + col) =
            make_float2(acc[n][2] * scale, acc[n][3] * scale);
      }
    }
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (warp == 0 && lane == 0) {
      tma_reduce_add_3d(&tmDQ, dq_buf, 0, q0, bh);
      bulk_commit_group();
    }
    // release Q_i / dO_i
    __syncwarp();
    if (lane == 0) mbar_arrive(BAR_E(st));
  }
  if (warp == 0 && lane == 0) bulk_wait_group<0>();  // every dQ reduce has landed

  // ---- dK (scaled), dV of this warp's 16 keys
  if (ok) {
    using T = typename E::T;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int key = kv0 + r0 + g4 + 8 * hi;
        if (key >= Nk) continue;
        const size_t off = ((size_t)bhk * Nk + key) * D + 8 * n + 2 * t4;
        *reinterpret_cast<typename E::T2*>(reinterpret_cast<T*>(dk) + off) =
            E::pack(dK[n][2 * hi] * scale, dK[n][2 * hi + 1] * scale);
        *reinterpret_cast<typename E::T2*>(reinterpret_cast<T*>(dv) + off) =
            E::pack(dV[n][2 * hi], dV[n][2 * hi + 1]);
      }
  }
}

}  // namespace bwd

B2A_DEFINE_ERROR_READER(backward)

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
  const size_t rows = (size_t)B * H * N;
  float* dvec = ws;                 // [B*H*N]
  float* dq_acc = ws + ((rows + 63) / 64) * 64;  // [B*H*N*D], 256-byte aligned
  bwd_prep_kernel<D, BF16><<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(o, dout, dvec, dq_acc,
                                                                           (int)rows);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward prep launch");
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tq, tdo, tk, tv, tdq;
  int rc = make_tmap_3d(&tq, q, dt, D, N, (uint64_t)B * H, 64, BQ, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tdo, dout, dt, D, N, (uint64_t)B * H, 64, BQ, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tk, k, dt, D, Nk, (uint64_t)B * Hkv, 64, BK, true);
  if (rc == B2A_OK) rc = make_tmap_3d(&tv, v, dt, D, Nk, (uint64_t)B * Hkv, 64, BK, true);
  if (rc == B2A_OK)
    rc = make_tmap_3d(&tdq, dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, D, N, (uint64_t)B * H, D, BQ,
                      false, 4);
  if (rc != B2A_OK) return rc;
  dim3 grid((unsigned)((Nk + BK - 1) / BK), (unsigned)(B * Hkv));
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tq, tdo, tk, tv, tdq, lse, dvec, dk, dv, N, Nk,
                                                   H, Hkv, scale);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "backward kernel launch");
  const size_t n = rows * D;
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

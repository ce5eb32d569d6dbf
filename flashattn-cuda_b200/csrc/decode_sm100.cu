// decode_sm100.cu -- split-KV and paged-KV GQA decode (query length 1) and
// the LSE-weighted combine, for B200 (sm_100a).
//
// The reference has no decode path; the math is its online softmax
// (cuda/flash_attn_fa3_db_full.cu:250-300) applied to one query row per head,
// with each split of the KV sequence producing a partial (o, l) that
// combine_kernel merges with the rescale identity of :261-284 and :340.
//
// Design (HBM-bound: every K/V byte is read exactly once):
//   * one CTA per (split, KV head, batch row).  Its G = H/Hkv query heads share
//     every K/V byte it loads (GQA head packing);
//   * warp 4 (producer) streams 64-token K and V tiles with TMA (3-D tensor
//     maps, 128-byte swizzle) into a ring of kStages stages.  Paged KV is read
//     page by page through the block table, one TMA box per (page, 64-column
//     block), so every 16-token page is a single contiguous 2-4 KB read;
//   * warps 0-3 (consumers) each own 16 tokens of a tile.  S = q K^T and
//     O += P V run on the tensor cores (mma.m16n8k16, the G heads in rows
//     0..G-1 of the A operand), with the online softmax on the accumulator
//     fragments;  the four warps' (m, l, o) states merge through shared memory
//     at the end, and the CTA writes the split's normalised o and natural-log l.
#include <cstdio>
#include <mutex>

#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace decode {

constexpr int kTok = 64;  // tokens per tile, 16 per consumer warp
constexpr int kThreads = 160;
constexpr int kProducerWarp = 4;
constexpr int kMaxPagesPerSplit = 256;

template <int D>
struct Cfg {
  static constexpr int kBlocks = D / 64;
  static constexpr uint32_t kTileBytes = kTok * D * 2;  // one K or V tile
  static constexpr int kStages = (D == 128) ? 3 : 6;
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = kStages * kTileBytes;
  static constexpr uint32_t kOffBar = 2 * kStages * kTileBytes;
  static constexpr uint32_t kOffPages = kOffBar + 16 * kStages;
  static constexpr uint32_t kOffAbort = kOffPages + 4 * kMaxPagesPerSplit;
  static constexpr uint32_t kSmemBytes = kOffAbort + 16 + 1024;
  // merge scratch (aliases the K stages once the pipeline has drained)
  static constexpr uint32_t kMergeBytes = 4 * 8 * (D + 2) * 4;
  static_assert(kMergeBytes <= kOffBar, "merge scratch must fit in the stage area");
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// C[16x8] += A[16x16] B[16x8] with only A rows 0-7 (a0, a2) live; c0/c1 are the
// accumulators of row lane/4, columns 2*(lane%4) + {0,1}.
template <bool BF16>
__device__ __forceinline__ void mma_rows8(float& c0, float& c1, uint32_t a0, uint32_t a2,
                                          uint32_t b0, uint32_t b1) {
  float d2 = 0.f, d3 = 0.f;
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c0), "+f"(c1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c0), "+f"(c1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
}

// byte offset of (row r, 8-element chunk ch) inside a [64 rows x 128 B] block
// written by TMA with 128-byte swizzle
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4));
}

template <int D, int G, bool BF16, bool PAGED>
__global__ void __launch_bounds__(kThreads, 2)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const void* __restrict__ q, const int32_t* __restrict__ block_table,
                  const int32_t* __restrict__ kv_lens, float* __restrict__ o_part,
                  float* __restrict__ l_part, int H, int Hkv, int Lkv, int splits, int tps,
                  int page_size, int max_pages, int num_pages, float scale_log2) {
  using C = Cfg<D>;
  using T = typename Elem<BF16>::T;
  constexpr int S = C::kStages;
  constexpr int NT = D / 8;  // 8-column output tiles per head

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw);
  const uint32_t sK = sb + C::kOffK;
  const uint32_t sV = sb + C::kOffV;
  const uint32_t bar0 = sb + C::kOffBar;
  auto BAR_F = [&](int s) { return bar0 + 8u * s; };
  auto BAR_E = [&](int s) { return bar0 + 8u * (S + s); };
  int32_t* s_pages = reinterpret_cast<int32_t*>(sp + C::kOffPages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sp + C::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int hkv = blockIdx.y;
  const int b = blockIdx.z;

  int len = PAGED ? kv_lens[b] : Lkv;
  if (PAGED && (len < 0 || len > max_pages * page_size)) {
    // a length the block table cannot hold: flag it and keep to the table
    if (split == 0 && hkv == 0 && threadIdx.x == 0) atomicOr(&g_error_flags, 2u);
    len = min(max(len, 0), max_pages * page_size);
  }
  const int t_begin = split * tps;
  const int t_end = min(len, t_begin + tps);
  const int head0 = b * H + hkv * G;  // first query head (flattened b*H + h)

  if (t_begin >= t_end) {
    // no tokens: an empty partial (paged splits past the sequence are never read)
    if (!PAGED) {
      for (int i = threadIdx.x; i < G * D; i += kThreads)
        o_part[((size_t)(head0 + i / D) * splits + split) * D + (i % D)] = 0.f;
      if (threadIdx.x < G) l_part[(size_t)(head0 + threadIdx.x) * splits + split] = -INFINITY;
    }
    return;
  }
  const int ntiles = (t_end - t_begin + kTok - 1) / kTok;

  if (threadIdx.x == kProducerWarp * 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(BAR_F(s), 1u);
      mbar_init(BAR_E(s), 4u);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (PAGED && warp == kProducerWarp) {
    const int p0 = t_begin / page_size;
    const int np = (t_end - t_begin + page_size - 1) / page_size;
    for (int i = lane; i < np; i += 32) {
      int pid = block_table[(size_t)b * max_pages + p0 + i];
      if (pid < 0 || pid >= num_pages) {
        atomicOr(&g_error_flags, 2u);  // page id out of range: read page 0 instead
        pid = 0;
      }
      s_pages[i] = pid;
    }
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % S;
        if (i >= S && !mbar_wait(BAR_E(st), ((i / S) - 1) & 1, abort_flag)) break;
        const int t0 = t_begin + i * kTok;
        const uint32_t kd = sK + st * C::kTileBytes, vd = sV + st * C::kTileBytes;
        if constexpr (!PAGED) {
          mbar_arrive_expect_tx(BAR_F(st), 2 * C::kTileBytes);
          const int row_outer = b * Hkv + hkv;
#pragma unroll
          for (int c = 0; c < C::kBlocks; ++c) {
            tma_load_3d(kd + c * (kTok * 128), &tmK, BAR_F(st), c * 64, t0, row_outer);
            tma_load_3d(vd + c * (kTok * 128), &tmV, BAR_F(st), c * 64, t0, row_outer);
          }
        } else {
          const int ppt = kTok / page_size;  // pages per tile
          const int pl0 = (t0 - t_begin) / page_size;
          const int np_all = (t_end - t_begin + page_size - 1) / page_size;
          const int np = min(ppt, np_all - pl0);
          mbar_arrive_expect_tx(BAR_F(st), (uint32_t)(np * page_size * 128 * 2 * C::kBlocks));
          for (int p = 0; p < np; ++p) {
            const int outer = s_pages[pl0 + p] * Hkv + hkv;
#pragma unroll
            for (int c = 0; c < C::kBlocks; ++c) {
              const uint32_t off = c * (kTok * 128) + p * page_size * 128;
              tma_load_3d(kd + off, &tmK, BAR_F(st), c * 64, 0, outer);
              tma_load_3d(vd + off, &tmV, BAR_F(st), c * 64, 0, outer);
            }
          }
        }
      }
    }
    return;  // the producer takes no part in the merge
  }

  // ------------------------------------------------------------------ consumers
  // q as the A operand: row h = lane/4 (heads >= G are zero rows)
  const int hq = lane >> 2;
  const int qc = 2 * (lane & 3);
  uint32_t qa[D / 16][2];
  {
    const T* qp = reinterpret_cast<const T*>(q) + (size_t)(head0 + hq) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      if (hq < G) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(qp + ks * 16 + qc);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 8 + qc);
      } else {
        qa[ks][0] = qa[ks][1] = 0u;
      }
    }
  }
  float o[NT][2];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % S;
    if (!mbar_wait(BAR_F(st), (i / S) & 1, abort_flag)) { ok = false; break; }
    const uint32_t kd = sK + st * C::kTileBytes, vd = sV + st * C::kTileBytes;
    const int r0 = warp * 16;                       // first tile row of this warp
    const int tok0 = t_begin + i * kTok + r0;       // its token index
    const int nvalid = min(16, t_end - tok0);
    if (nvalid > 0) {
      if (nvalid < 16) {
        // rows past the end may hold stale or foreign data: zero their V
        for (int idx = lane; idx < (16 - nvalid) * 8 * C::kBlocks; idx += 32) {
          const int r = r0 + nvalid + idx / (8 * C::kBlocks);
          const int rem = idx % (8 * C::kBlocks);
          *reinterpret_cast<uint4*>(sp + (vd - sb) + (rem / 8) * (kTok * 128) + swz(r, rem % 8)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      // ---- S = q K^T for 16 tokens (two 8-token column tiles)
      float s[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = 0.f;
        const int r = r0 + nt * 8 + (lane & 7);
        const int mtx = lane >> 3;
#pragma unroll
        for (int ks = 0; ks < D / 16; ks += 2) {
          const int d = 16 * (ks + (mtx >> 1)) + 8 * (mtx & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kd + (d >> 6) * (kTok * 128) + swz(r, (d & 63) >> 3), b0, b1, b2, b3);
          mma_rows8<BF16>(s[nt][0], s[nt][1], qa[ks][0], qa[ks][1], b0, b1);
          mma_rows8<BF16>(s[nt][0], s[nt][1], qa[ks + 1][0], qa[ks + 1][1], b2, b3);
        }
      }
      // ---- online softmax on row hq (a quad of lanes holds its 16 scores)
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = nt * 8 + qc + e;
          s[nt][e] = (tk < nvalid) ? s[nt][e] * scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[nt][e]);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2(m_run - m_use);
      m_run = m_new;
      float ps = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[nt][e] = ex2(s[nt][e] - m_use);
          ps += s[nt][e];
        }
      l_run = l_run * alpha + ps;
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          o[n][0] *= alpha;
          o[n][1] *= alpha;
        }
      }
      const uint32_t pa0 = pack2_u32<BF16>(s[0][0], s[0][1]);
      const uint32_t pa2 = pack2_u32<BF16>(s[1][0], s[1][1]);
      // ---- O += P V over this warp's 16 tokens
      {
        const int mtx = lane >> 3;
        const int r = r0 + 8 * (mtx & 1) + (lane & 7);
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          const int d = 8 * (n + (mtx >> 1));
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vd + (d >> 6) * (kTok * 128) + swz(r, (d & 63) >> 3), b0, b1, b2, b3);
          mma_rows8<BF16>(o[n][0], o[n][1], pa0, pa2, b0, b1);
          mma_rows8<BF16>(o[n + 1][0], o[n + 1][1], pa0, pa2, b2, b3);
        }
      }
      if (nvalid < 16) fence_proxy_async_smem();  // zeroed rows precede the next TMA write
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(BAR_E(st));
  }

  // ---------------------------------------------------------------- merge warps
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  asm volatile("bar.sync 1, 128;" ::: "memory");  // all consumers are done with the stages
  float* mg = reinterpret_cast<float*>(sp);           // [4][8] m, [4][8] l, [4][8][D] o
  float* mg_m = mg;
  float* mg_l = mg + 32;
  float* mg_o = mg + 64;
  if (hq < G) {
    if ((lane & 3) == 0) {
      mg_m[warp * 8 + hq] = ok ? m_run : -INFINITY;
      mg_l[warp * 8 + hq] = ok ? l_run : 0.f;
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      mg_o[(warp * 8 + hq) * D + n * 8 + qc] = o[n][0];
      mg_o[(warp * 8 + hq) * D + n * 8 + qc + 1] = o[n][1];
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (int idx = threadIdx.x; idx < G * D; idx += 128) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mg_m[w * 8 + h]);
    float L = 0.f, acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = ex2(mg_m[w * 8 + h] - M);
        L += mg_l[w * 8 + h] * f;
        acc += mg_o[(w * 8 + h) * D + d] * f;
      }
    }
    const size_t row = (size_t)(head0 + h) * splits + split;
    o_part[row * D + d] = (L > 0.f) ? acc / L : 0.f;
    if (d == 0) l_part[row] = (L > 0.f) ? M * 0.69314718055994531f + logf(L) : -INFINITY;
  }
}

// One CTA per (batch row, query head).  The partials may come from several
// ranks (KV-sharded decode): rank r's block of [B,H,S,D] o / [B,H,S] l starts
// r * rank_stride floats after rank 0's, and rank r's splits follow rank r-1's
// in sequence order (one rank: R = 1).
// OUT: 0 fp16 O, 1 bf16 O, 2 fp32 O (a merged partial: o normalised by its
// own sum, lse = log sum exp over all splits -- the form of one split).
// kCombineThreads threads: the (rank, split) entries are spread over the
// threads for the max and the weights (one load each, all in flight at once),
// and every output column then sums its entries with eight loads in flight,
// so the latency of one partial's load is paid a few times, not once per split.
constexpr int kCombineThreads = 128;
constexpr int kCombineChunk = 1024;  // weights held in shared memory at a time

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5;
  __syncthreads();  // red may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int i = 1; i < kCombineThreads / 32; ++i) v = is_max ? fmaxf(v, red[i]) : v + red[i];
  return v;
}

template <int OUT>
__global__ void __launch_bounds__(kCombineThreads)
    combine_kernel(const float* __restrict__ o_part, const float* __restrict__ l_part,
                   void* __restrict__ out, float* __restrict__ lse, int H, int S, int D,
                   const int32_t* __restrict__ kv_lens, int tps, int R, long long rank_stride) {
  __shared__ float sw[kCombineChunk];
  __shared__ float red[kCombineThreads / 32];
  const int bh = blockIdx.x;
  int ns = S;  // splits per rank
  if (kv_lens != nullptr) ns = max(0, min(S, (kv_lens[bh / H] + tps - 1) / tps));
  const int n = R * ns;  // entries (rank r, split s) = r * ns + s
  auto lp = [&](int i) {
    return l_part + (i / ns) * rank_stride + (size_t)bh * S + (i % ns);
  };
  auto op = [&](int i) {
    return o_part + (i / ns) * rank_stride + ((size_t)bh * S + (i % ns)) * D;
  };
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += kCombineThreads) m = fmaxf(m, *lp(i));
  const float M = block_reduce(m, red, true);
  const int d = threadIdx.x;
  float psum = 0.f, acc = 0.f;
  for (int c0 = 0; c0 < n; c0 += kCombineChunk) {
    const int cn = min(kCombineChunk, n - c0);
    __syncthreads();  // the previous chunk's weights are consumed
    for (int i = threadIdx.x; i < cn; i += kCombineThreads) {
      const float l = *lp(c0 + i);
      const float w = (l == -INFINITY) ? 0.f : expf(l - M);
      sw[i] = w;
      psum += w;
    }
    __syncthreads();
    if (d < D) {
      // eight entries' loads in flight at a time
      for (int i0 = 0; i0 < cn; i0 += 8) {
        float ov[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) ov[i] = op(c0 + min(i0 + i, cn - 1))[d];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i0 + i < cn) acc += sw[i0 + i] * ov[i];
      }
    }
  }
  const float sum = block_reduce(psum, red, false);
  // no key at all (an empty sequence): O = 0, L = -inf
  if (d < D) {
    const float o = sum > 0.f ? acc / sum : 0.f;
    if constexpr (OUT == 2)
      reinterpret_cast<float*>(out)[(size_t)bh * D + d] = o;
    else
      reinterpret_cast<typename Elem<OUT == 1>::T*>(out)[(size_t)bh * D + d] =
          Elem<OUT == 1>::from(o);
  }
  if (lse != nullptr && d == 0) lse[bh] = sum > 0.f ? M + logf(sum) : -INFINITY;
}

}  // namespace decode

B2A_DEFINE_ERROR_READER(decode)

template <int D, int G, bool BF16, bool PAGED>
static int launch_decode(const void* q, const void* k, const void* v, const int32_t* block_table,
                         const int32_t* kv_lens, float* o_part, float* l_part, int B, int H,
                         int Hkv, int Lkv, int splits, int tps, int page_size, int max_pages,
                         int num_pages, float scale, cudaStream_t stream) {
  using namespace decode;
  using C = Cfg<D>;
  auto kern = decode_kernel<D, G, BF16, PAGED>;
  static bool attr_done[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(B2A_ERR_CUDA, "cudaGetDevice failed");
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::kSmemBytes);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaFuncSetAttribute(decode)");
    attr_done[dev] = true;
  }
  const CUtensorMapDataType dt =
      BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tk, tv;
  int rc;
  if (!PAGED) {
    rc = make_tmap_3d(&tk, k, dt, D, Lkv, (uint64_t)B * Hkv, 64, kTok, true);
    if (rc == B2A_OK) rc = make_tmap_3d(&tv, v, dt, D, Lkv, (uint64_t)B * Hkv, 64, kTok, true);
  } else {
    rc = make_tmap_3d(&tk, k, dt, D, page_size, (uint64_t)num_pages * Hkv, 64, page_size, true);
    if (rc == B2A_OK)
      rc = make_tmap_3d(&tv, v, dt, D, page_size, (uint64_t)num_pages * Hkv, 64, page_size, true);
  }
  if (rc != B2A_OK) return rc;
  dim3 grid((unsigned)splits, (unsigned)Hkv, (unsigned)B);
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tk, tv, q, block_table, kv_lens, o_part, l_part,
                                                   H, Hkv, Lkv, splits, tps, page_size, max_pages,
                                                   num_pages, scale * 1.4426950408889634f);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "decode kernel launch");
  return B2A_OK;
}

int decode_dispatch(const void* q, const void* k, const void* v, const int32_t* block_table,
                    const int32_t* kv_lens, float* o_part, float* l_part, int B, int H, int Hkv,
                    int Lkv, int D, int splits, int tps, int page_size, int max_pages,
                    int num_pages, int dtype, float scale, cudaStream_t stream) {
  const bool bf = dtype == B2A_BF16;
  const bool paged = block_table != nullptr;
  const int G = H / Hkv;
  if (paged && tps / page_size > decode::kMaxPagesPerSplit)
    return set_error(B2A_ERR_INVALID_ARG, "pages_per_split must be <= 256");
#define B2A_DC(DD, GG, BB, PP)                                                                  \
  if (D == DD && G == GG && bf == BB && paged == PP)                                            \
    return launch_decode<DD, GG, BB, PP>(q, k, v, block_table, kv_lens, o_part, l_part, B, H,   \
                                         Hkv, Lkv, splits, tps, page_size, max_pages, num_pages, \
                                         scale, stream);
#define B2A_DC_G(DD, BB, PP) \
  B2A_DC(DD, 1, BB, PP) B2A_DC(DD, 2, BB, PP) B2A_DC(DD, 4, BB, PP) B2A_DC(DD, 8, BB, PP)
  B2A_DC_G(64, false, false)
  B2A_DC_G(64, true, false)
  B2A_DC_G(128, false, false)
  B2A_DC_G(128, true, false)
  B2A_DC_G(64, false, true)
  B2A_DC_G(64, true, true)
  B2A_DC_G(128, false, true)
  B2A_DC_G(128, true, true)
#undef B2A_DC_G
#undef B2A_DC
  return set_error(B2A_ERR_UNSUPPORTED, "decode: unsupported (D, group, dtype)");
}

int combine_dispatch(const float* o_part, const float* l_part, void* o, float* lse, int B, int H,
                     int splits, int D, int dtype, const int32_t* kv_lens, int tps,
                     cudaStream_t stream, int ranks, long long rank_stride) {
  const unsigned threads = decode::kCombineThreads;  // >= D
  auto go = [&](auto kern) {
    kern<<<B * H, threads, 0, stream>>>(o_part, l_part, o, lse, H, splits, D, kv_lens, tps, ranks,
                                        rank_stride);
  };
  if (dtype == kCombineF32) go(decode::combine_kernel<2>);
  else if (dtype == B2A_BF16) go(decode::combine_kernel<1>);
  else go(decode::combine_kernel<0>);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "combine kernel launch");
  return B2A_OK;
}

// ---------------------------------------------------------------------------
// Scratch for b2a_decode_paged_noalloc.  Some callers cannot allocate device
// memory at the point where they decode: an allocator-free serving runtime
// that owns all of HBM up front, code running inside a memory pool that must
// not grow, or a plugin host that forbids cudaMalloc on its request path.
// For them the split partials live in this fixed array instead of a
// caller-provided buffer.  Every GPU that loads the library holds it (16 MiB)
// until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchFloats = 4u * 1024u * 1024u;  // 16 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Device address of g_noalloc_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device with cudaGetSymbolAddress (with that device current) and cached.
static int noalloc_scratch_ptr(float** out) {
  static float* ptrs[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(B2A_ERR_INVALID_ARG, "device index too large");
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    ptrs[dev] = static_cast<float*>(p);
  }
  *out = ptrs[dev];
  return B2A_OK;
}

}  // namespace b2a

extern "C" int b2a_decode_paged_noalloc(const void* q, const void* k_pool, const void* v_pool,
                                        const int32_t* block_table, const int32_t* kv_lens,
                                        void* o, float* lse, int B, int H, int Hkv, int D,
                                        int page_size, int max_pages, int num_pages,
                                        int pages_per_split, int dtype, float scale,
                                        void* stream) {
  using namespace b2a;
  // the device check comes first: the scratch address exists only on a
  // device that can run the kernels
  int rc = require_device(dtype);
  if (rc != B2A_OK) return rc;
  if (B <= 0 || H <= 0 || D <= 0 || max_pages <= 0 || pages_per_split <= 0)
    return set_error(B2A_ERR_INVALID_ARG,
                     "B, H, D, max_pages and pages_per_split must be > 0");
  const size_t splits = ((size_t)max_pages + pages_per_split - 1) / pages_per_split;
  const size_t rows = (size_t)B * H * splits;
  const size_t need = rows * (size_t)D + rows;
  if (need > kNoAllocScratchFloats) {
    char buf[256];
    snprintf(buf, sizeof buf,
             "decode_paged_noalloc: B*H*ceil(max_pages/pages_per_split)*(D+1) = %zu floats "
             "exceeds the fixed scratch of %zu floats (16 MiB); use b2a_decode_paged with a "
             "caller-provided scratch buffer or raise pages_per_split",
             need, kNoAllocScratchFloats);
    return set_error(B2A_ERR_INVALID_ARG, buf);
  }
  float* scratch = nullptr;
  rc = noalloc_scratch_ptr(&scratch);
  if (rc != B2A_OK) return rc;
  float* o_part = scratch;                       // [B, H, splits, D]
  float* l_part = scratch + rows * (size_t)D;    // [B, H, splits]; 16-byte aligned (D % 4 == 0)
  return b2a_decode_paged(q, k_pool, v_pool, block_table, kv_lens, o_part, l_part, o, lse, B, H,
                          Hkv, D, page_size, max_pages, num_pages, pages_per_split, dtype, scale,
                          stream);
}


// exchange_sm100.cu -- the exchange step of KV-sharded decode as ONE kernel
// over NVLink peer memory: merge of the rank's split partials, all-gather of
// the merged partials by peer stores, and the LSE-weighted combine.
//
// Each rank owns one exchange buffer, mapped into every other rank's address
// space (CUDA IPC over NVLink / NVSwitch).  For B*H rows, world W and head
// dim D its layout is
//   data  [2][W][B*H][D+1] of {value, call}  8-byte words: slot (parity,
//         source rank, row) holds o[0..D-1] then l, each tagged with the call
//         count it belongs to
//   seen  [B*H] u32   calls this rank has completed, per row
// One CTA per row (b, h):
//   1. merge the rank's S split partials (o_s, l_s) into one (o, l) -- the
//      online-softmax rescale of cuda/flash_attn_fa3_db_full.cu:261-284;
//   2. call = seen + 1, parity = call & 1; store {value, call} words into slot
//      (parity, this rank, row) of EVERY rank's buffer (peer stores);
//   3. poll (bounded) the W slots of the row in this rank's own buffer until
//      every word carries `call`, then combine them into O, L;
//   4. seen = call.
// An 8-byte aligned store is seen whole, so a word whose tag matches holds
// the matching value: no fence and no separate flag round trip are needed.
// Two parities suffice: a rank can be at most one call ahead of a slowest
// peer (finishing call n needs every peer's call-n words, which a peer sends
// only after it has finished call n-1 and its reads of the other parity).
// Tags only grow, so nothing is reset between calls.  No TMA or bulk copy
// touches peer memory; no multicast of any kind.
#include <cstring>

#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace exch {

constexpr int kThreads = 160;  // > D (64 or 128): the last thread carries l
constexpr int kMaxWorld = 64;
constexpr uint64_t kExchangeLimitNs = 1000000000ull;  // 1 s

// 8-byte {value, call} words of the data region
__host__ __device__ inline size_t data_words(int BH, int W, int D) {
  return (size_t)2 * W * BH * (D + 1);
}

__device__ __forceinline__ void st_tagged(uint2* dst, float v, uint32_t call) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(dst), "r"(__float_as_uint(v)),
               "r"(call)
               : "memory");
}
__device__ __forceinline__ uint2 ld_tagged(const uint2* src) {
  uint2 r;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(src)
               : "memory");
  return r;
}

template <int OUT>
__global__ void __launch_bounds__(kThreads)
    exchange_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ l_part,
                            const uint64_t* __restrict__ peers, int rank, int W, int BH, int S,
                            int D, void* __restrict__ out, float* __restrict__ lse) {
  __shared__ float red[kThreads / 32];
  __shared__ float s_l[kMaxWorld];
  __shared__ uint32_t s_call;
  __shared__ int s_timeout;
  const int bh = blockIdx.x;
  const int tid = threadIdx.x;
  uint2* local = reinterpret_cast<uint2*>(peers[rank]);
  uint32_t* seen = reinterpret_cast<uint32_t*>(local + data_words(BH, W, D));

  auto block_reduce = [&](float v, bool is_max) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, w) : v + w;
    }
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < kThreads / 32; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
    return r;
  };

  if (tid == 0) {
    s_call = *reinterpret_cast<volatile uint32_t*>(seen + bh) + 1u;
    s_timeout = 0;
  }
  // 1. merge this rank's S splits
  const float* lp = l_part + (size_t)bh * S;
  const float* op = o_part + (size_t)bh * S * D;
  float m = -INFINITY;
  for (int s = tid; s < S; s += kThreads) m = fmaxf(m, lp[s]);
  const float M = block_reduce(m, true);
  float psum = 0.f, acc = 0.f;
  for (int s = tid; s < S; s += kThreads) psum += (lp[s] == -INFINITY) ? 0.f : expf(lp[s] - M);
  if (tid < D) {
    // eight splits' loads in flight at a time (the partials sit in L2)
    for (int s0 = 0; s0 < S; s0 += 8) {
      float ov[8], lv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int s = min(s0 + i, S - 1);
        ov[i] = op[(size_t)s * D + tid];
        lv[i] = lp[s];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (s0 + i < S && lv[i] != -INFINITY) acc += expf(lv[i] - M) * ov[i];
    }
  }
  const float sum = block_reduce(psum, false);  // its barriers also publish s_call
  const float o_m = sum > 0.f ? acc / sum : 0.f;
  const float l_m = sum > 0.f ? M + logf(sum) : -INFINITY;

  // 2. deliver the tagged (o_m, l_m) words to every rank
  const uint32_t call = s_call;
  const int par = (int)(call & 1u);
  const size_t slot = (((size_t)par * W + rank) * BH + bh) * (D + 1);
  for (int p = 0; p < W; ++p) {
    uint2* dst = reinterpret_cast<uint2*>(peers[p]) + slot;
    if (tid < D) st_tagged(dst + tid, o_m, call);
    if (tid == 0) st_tagged(dst + D, l_m, call);
  }

  // 3. poll this rank's own slots of the row until every word carries `call`
  const uint2* base = local + (((size_t)par * W) * BH + bh) * (D + 1);
  const size_t rstride = (size_t)BH * (D + 1);
  const uint64_t t0 = globaltimer();
  float o_r[kMaxWorld];  // this thread's column of every rank's partial
  if (tid < D || tid == kThreads - 1) {
    const int col = tid < D ? tid : D;
    // eight ranks' words in flight per poll round
    for (int r0 = 0; r0 < W; r0 += 8) {
      const int nr = min(8, W - r0);
      uint32_t pending = (1u << nr) - 1u;
      while (pending != 0u) {
        uint2 w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if ((pending >> i) & 1u) w[i] = ld_tagged(base + (size_t)(r0 + i) * rstride + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (((pending >> i) & 1u) && w[i].y == call) {
            if (tid < D) o_r[r0 + i] = __uint_as_float(w[i].x);
            else s_l[r0 + i] = __uint_as_float(w[i].x);
            pending &= ~(1u << i);
          }
        }
        if (pending != 0u) {
          if (*reinterpret_cast<volatile int*>(&s_timeout)) break;
          if (globaltimer() - t0 > kExchangeLimitNs) {
            atomicOr(&g_error_flags, kErrWaitTimeout);
            s_timeout = 1;
            break;
          }
        }
      }
      if (pending != 0u) {  // timed out: this rank's words are missing; count them as empty
        for (int i = 0; i < nr; ++i)
          if ((pending >> i) & 1u) {
            if (tid < D) o_r[r0 + i] = 0.f;
            else s_l[r0 + i] = -INFINITY;
          }
      }
    }
  }
  __syncthreads();

  // combine the W delivered partials
  float M2 = -INFINITY;
  for (int r = 0; r < W; ++r) M2 = fmaxf(M2, s_l[r]);
  float sum2 = 0.f, acc2 = 0.f;
  for (int r = 0; r < W; ++r) {
    const float w = (s_l[r] == -INFINITY) ? 0.f : expf(s_l[r] - M2);
    sum2 += w;
    if (tid < D) acc2 += w * o_r[r];
  }
  if (tid < D) {
    const float o = sum2 > 0.f ? acc2 / sum2 : 0.f;
    reinterpret_cast<typename Elem<OUT == 1>::T*>(out)[(size_t)bh * D + tid] =
        Elem<OUT == 1>::from(o);
  }
  if (lse != nullptr && tid == 0) lse[bh] = sum2 > 0.f ? M2 + logf(sum2) : -INFINITY;
  // 4. this call is complete here (a timed-out call still advances, so the
  // ranks stay in step; its output is undefined and error bit 0 is set)
  if (tid == 0) seen[bh] = call;
}

}  // namespace exch

B2A_DEFINE_ERROR_READER(exchange)

}  // namespace b2a

using namespace b2a;

extern "C" {

int64_t b2a_exchange_bytes(int B, int H, int D, int world) {
  if (B <= 0 || H <= 0 || D <= 0 || world <= 0) return -1;
  const size_t BH = (size_t)B * H;
  const size_t bytes = exch::data_words((int)BH, world, D) * 8 + BH * 4;
  return (int64_t)((bytes + 255) / 256 * 256);
}

int b2a_exchange_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes <= 0 || ptr == nullptr || ipc_handle == nullptr)
    return set_error(B2A_ERR_INVALID_ARG, "bytes must be > 0 and ptr / ipc_handle non-null");
  int rc = require_device(B2A_F16);
  if (rc != B2A_OK) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaMalloc(exchange buffer)");
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_cuda_error(e, "exchange buffer set-up");
  }
  *ptr = p;
  return B2A_OK;
}

int b2a_exchange_open(const void* ipc_handle, void** ptr) {
  if (ipc_handle == nullptr || ptr == nullptr)
    return set_error(B2A_ERR_INVALID_ARG, "ipc_handle and ptr must be non-null");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof h);
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaIpcOpenMemHandle(peer exchange buffer)");
  return B2A_OK;
}

int b2a_exchange_close(void* peer_ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaIpcCloseMemHandle");
  return B2A_OK;
}

int b2a_exchange_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaFree(exchange buffer)");
  return B2A_OK;
}

int b2a_decode_exchange_combine(const float* o_part, const float* l_part, const uint64_t* peers,
                                int rank, int world, void* o, float* lse, int B, int H,
                                int splits, int D, int dtype, void* stream) {
  int rc = require_device(dtype);
  if (rc != B2A_OK) return rc;
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || H <= 0 || splits <= 0 || world <= 0 || world > exch::kMaxWorld || rank < 0 ||
      rank >= world)
    return set_error(B2A_ERR_INVALID_ARG,
                     "B, H, splits must be > 0, world in [1, 64] and 0 <= rank < world");
  if ((int64_t)B * H > 0x7fffffff) return set_error(B2A_ERR_INVALID_ARG, "B*H too large");
  if (o_part == nullptr || l_part == nullptr || peers == nullptr || o == nullptr)
    return set_error(B2A_ERR_INVALID_ARG, "o_part, l_part, peers and O must be non-null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kern) {
    kern<<<B * H, exch::kThreads, 0, s>>>(o_part, l_part, peers, rank, world, B * H, splits, D,
                                         o, lse);
  };
  if (dtype == B2A_BF16) go(exch::exchange_combine_kernel<1>);
  else go(exch::exchange_combine_kernel<0>);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "exchange kernel launch");
  return B2A_OK;
}

}  // extern "C"

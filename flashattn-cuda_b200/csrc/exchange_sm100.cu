// exchange_sm100.cu -- the exchange step of KV-sharded decode as ONE kernel
// over NVLink peer memory: merge of the rank's split partials, all-gather of
// the merged partials by peer stores, and the LSE-weighted combine.
//
// Each rank owns one exchange buffer, mapped into every other rank's address
// space (CUDA IPC over NVLink / NVSwitch).  For B*H rows, world W and head
// dim D its layout is
//   data  [2][W][B*H][D+1] fp32  slot (parity, source rank, row): o then l
//   flags [W][B*H]         u32   call count the source rank has delivered
//   seen  [B*H]            u32   calls this rank has completed, per row
// One CTA per row (b, h):
//   1. merge the rank's S split partials (o_s, l_s) into one (o, l) -- the
//      online-softmax rescale of cuda/flash_attn_fa3_db_full.cu:261-284;
//   2. target = seen + 1, parity = target & 1; store (o, l) into slot
//      (parity, this rank, row) of EVERY rank's buffer (peer stores), fence at
//      system scope, then store `target` into this rank's flag of the row in
//      every rank's buffer;
//   3. wait (bounded) until every rank's flag for the row here reaches
//      `target`, then combine the W slots from local memory into O, L;
//   4. seen = target.
// Two parities suffice: a rank can be at most one call ahead of a slowest
// peer (finishing call n needs every peer's call-n signal, which a peer sends
// only after it has finished call n-1 and its reads of the other parity).
// Flags only grow, so nothing is reset between calls.  No TMA or bulk copy
// touches peer memory; no multicast of any kind.
#include <cstring>

#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace exch {

constexpr int kThreads = 128;  // >= D (64 or 128) and >= W
constexpr int kMaxWorld = 64;
constexpr uint64_t kExchangeLimitNs = 1000000000ull;  // 1 s

__host__ __device__ inline size_t data_floats(int BH, int W, int D) {
  return (size_t)2 * W * BH * (D + 1);
}

template <int OUT>
__global__ void __launch_bounds__(kThreads)
    exchange_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ l_part,
                            const uint64_t* __restrict__ peers, int rank, int W, int BH, int S,
                            int D, void* __restrict__ out, float* __restrict__ lse) {
  __shared__ float red[kThreads / 32];
  __shared__ float s_w[kMaxWorld];
  __shared__ uint32_t s_target;
  const int bh = blockIdx.x;
  const int tid = threadIdx.x;
  float* local = reinterpret_cast<float*>(peers[rank]);
  uint32_t* flags = reinterpret_cast<uint32_t*>(local + data_floats(BH, W, D));
  uint32_t* seen = flags + (size_t)W * BH;

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

  // 1. merge this rank's S splits
  const float* lp = l_part + (size_t)bh * S;
  const float* op = o_part + (size_t)bh * S * D;
  float m = -INFINITY;
  for (int s = tid; s < S; s += kThreads) m = fmaxf(m, lp[s]);
  const float M = block_reduce(m, true);
  float psum = 0.f, acc = 0.f;
  for (int s = tid; s < S; s += kThreads) psum += (lp[s] == -INFINITY) ? 0.f : expf(lp[s] - M);
  if (tid < D) {
    float a0 = 0.f, a1 = 0.f;
    int s = 0;
    for (; s + 2 <= S; s += 2) {
      const float w0 = (lp[s] == -INFINITY) ? 0.f : expf(lp[s] - M);
      const float w1 = (lp[s + 1] == -INFINITY) ? 0.f : expf(lp[s + 1] - M);
      a0 += w0 * op[(size_t)s * D + tid];
      a1 += w1 * op[(size_t)(s + 1) * D + tid];
    }
    if (s < S) a0 += ((lp[s] == -INFINITY) ? 0.f : expf(lp[s] - M)) * op[(size_t)s * D + tid];
    acc = a0 + a1;
  }
  const float sum = block_reduce(psum, false);
  const float o_m = sum > 0.f ? acc / sum : 0.f;
  const float l_m = sum > 0.f ? M + logf(sum) : -INFINITY;

  // 2. deliver (o_m, l_m) to every rank, then signal
  if (tid == 0) s_target = *reinterpret_cast<volatile uint32_t*>(seen + bh) + 1u;
  __syncthreads();
  const uint32_t target = s_target;
  const int par = (int)(target & 1u);
  const size_t slot = (((size_t)par * W + rank) * BH + bh) * (D + 1);
  for (int p = 0; p < W; ++p) {
    float* dst = reinterpret_cast<float*>(peers[p]) + slot;
    if (tid < D) dst[tid] = o_m;
    if (tid == 0) dst[D] = l_m;
  }
  __threadfence_system();  // this thread's stores are visible before the signal
  __syncthreads();
  if (tid < W) {
    uint32_t* f = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(peers[tid]) +
                                              data_floats(BH, W, D)) +
                  (size_t)rank * BH + bh;
    *reinterpret_cast<volatile uint32_t*>(f) = target;
  }

  // 3. wait for every rank's delivery of this call, bounded
  if (tid < W) {
    volatile uint32_t* f = flags + (size_t)tid * BH + bh;
    if ((int)(*f - target) < 0) {
      const uint64_t t0 = globaltimer();
      while ((int)(*f - target) < 0) {
        if (globaltimer() - t0 > kExchangeLimitNs) {
          atomicOr(&g_error_flags, kErrWaitTimeout);
          break;
        }
      }
    }
  }
  __threadfence_system();
  __syncthreads();

  // combine the W delivered partials (local memory, written by the peers)
  const float* base = local + (((size_t)par * W) * BH + bh) * (D + 1);
  const size_t rstride = (size_t)BH * (D + 1);
  if (tid < W) s_w[tid] = __ldcg(base + tid * rstride + D);
  __syncthreads();
  float M2 = -INFINITY;
  for (int r = 0; r < W; ++r) M2 = fmaxf(M2, s_w[r]);
  float sum2 = 0.f, acc2 = 0.f;
  for (int r = 0; r < W; ++r) {
    const float w = (s_w[r] == -INFINITY) ? 0.f : expf(s_w[r] - M2);
    sum2 += w;
    if (tid < D) acc2 += w * __ldcg(base + r * rstride + tid);
  }
  if (tid < D) {
    const float o = sum2 > 0.f ? acc2 / sum2 : 0.f;
    reinterpret_cast<typename Elem<OUT == 1>::T*>(out)[(size_t)bh * D + tid] =
        Elem<OUT == 1>::from(o);
  }
  if (lse != nullptr && tid == 0) lse[bh] = sum2 > 0.f ? M2 + logf(sum2) : -INFINITY;
  // 4. this call is complete here (a timed-out call still advances, so the
  // ranks stay in step; its output is undefined and error bit 0 is set)
  if (tid == 0) seen[bh] = target;
}

}  // namespace exch

B2A_DEFINE_ERROR_READER(exchange)

}  // namespace b2a

using namespace b2a;

extern "C" {

int64_t b2a_exchange_bytes(int B, int H, int D, int world) {
  if (B <= 0 || H <= 0 || D <= 0 || world <= 0) return -1;
  const size_t BH = (size_t)B * H;
  const size_t bytes = exch::data_floats((int)BH, world, D) * 4 + ((size_t)world + 1) * BH * 4;
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

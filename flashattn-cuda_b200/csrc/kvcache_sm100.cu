// kvcache_sm100.cu -- the write path of the paged KV cache read by the paged
// decode kernel: append T new tokens per sequence into pages of a pool laid
// out [P, Hkv, page_size, D] (the layout decode_sm100.cu reads).
//
// Token t of sequence b lands at position kv_lens[b] + t, i.e. in page
// block_table[b, (kv_lens[b] + t) / page_size], slot (kv_lens[b] + t) %
// page_size.  The pages must already be assigned in the block table (the
// host-side allocator b200attn.kvcache.PagePool does that); optionally the
// kernel advances kv_lens[b] by T afterwards.  HBM-bound copy: each thread
// moves 16-byte vectors, a warp covers whole 128- or 256-byte rows.
#include "sm100_ptx.cuh"
#include "b2a_host.h"

namespace b2a {
namespace kvcache {

constexpr int kThreads = 256;

// One CTA per (token t, KV head, sequence b) group of rows: blockIdx.x walks
// the T tokens in chunks so that each thread copies one 16-byte vector of K and
// one of V.
template <int D>
__global__ void __launch_bounds__(kThreads)
    append_kernel(const uint4* __restrict__ k_new, const uint4* __restrict__ v_new,
                  uint4* __restrict__ k_pool, uint4* __restrict__ v_pool,
                  const int32_t* __restrict__ block_table, const int32_t* __restrict__ kv_lens,
                  int Hkv, int T, int page_size, int max_pages, int num_pages) {
  constexpr int VPR = D * 2 / 16;                // 16-byte vectors per row
  constexpr int ROWS = kThreads / VPR;           // token rows per CTA
  const int b = blockIdx.z, hkv = blockIdx.y;
  const int t = blockIdx.x * ROWS + threadIdx.x / VPR;
  const int vec = threadIdx.x % VPR;
  if (t >= T) return;
  // 64-bit position: kv_lens[b] + t must not wrap; a negative or too large
  // position has no block-table entry
  const long long pos64 = (long long)kv_lens[b] + t;
  const long long pidx64 = pos64 >= 0 ? pos64 / page_size : -1;
  int page = (pidx64 >= 0 && pidx64 < max_pages) ? block_table[(size_t)b * max_pages + pidx64] : -1;
  const int pos = (int)pos64;
  if (page < 0 || page >= num_pages) {
    atomicOr(&g_error_flags, 4u);  // no page assigned for this position: token dropped
    return;
  }
  const size_t src = (((size_t)b * Hkv + hkv) * T + t) * VPR + vec;
  const size_t dst = (((size_t)page * Hkv + hkv) * page_size + pos % page_size) * VPR + vec;
  k_pool[dst] = k_new[src];
  v_pool[dst] = v_new[src];
}

__global__ void advance_lens_kernel(int32_t* __restrict__ kv_lens, int B, int T) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) kv_lens[b] += T;
}

}  // namespace kvcache

B2A_DEFINE_ERROR_READER(kvcache)

int kv_append_dispatch(const void* k_new, const void* v_new, void* k_pool, void* v_pool,
                       const int32_t* block_table, int32_t* kv_lens, int B, int Hkv, int T, int D,
                       int page_size, int max_pages, int num_pages, int advance,
                       cudaStream_t stream) {
  using namespace kvcache;
  const int vpr = D * 2 / 16;
  const int rows = kThreads / vpr;
  dim3 grid((unsigned)((T + rows - 1) / rows), (unsigned)Hkv, (unsigned)B);
  auto args = [&](auto kern) {
    kern<<<grid, kThreads, 0, stream>>>(
        static_cast<const uint4*>(k_new), static_cast<const uint4*>(v_new),
        static_cast<uint4*>(k_pool), static_cast<uint4*>(v_pool), block_table, kv_lens, Hkv, T,
        page_size, max_pages, num_pages);
  };
  if (D == 64) args(append_kernel<64>);
  else args(append_kernel<128>);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "kv append kernel launch");
  if (advance) {
    advance_lens_kernel<<<(B + 255) / 256, 256, 0, stream>>>(kv_lens, B, T);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(e, "kv length update launch");
  }
  return B2A_OK;
}

}  // namespace b2a

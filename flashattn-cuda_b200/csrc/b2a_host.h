// b2a_host.h -- host-side helpers shared by the kernels' launchers:
// thread-local error messages, device checks and TMA tensor-map encoding.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200attn.h"

namespace b2a {

constexpr int kMaxDevices = 64;

// Record `msg` as this thread's last error and return `status`.
int set_error(int status, const char* msg);
// Record a CUDA runtime failure ("<what>: <cuda error string>").
int set_cuda_error(cudaError_t e, const char* what);

// 3-D tiled tensor map over a contiguous [outer, rows, inner] array of
// `elem_bytes`-byte elements: dims {inner, rows, outer}, box {box_inner,
// box_rows, 1}.  Rows past `rows` (per outer index) read as zero; stores and
// reductions there are dropped.
int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t rows, uint64_t outer, uint32_t box_inner, uint32_t box_rows,
                 bool swizzle128, uint32_t elem_bytes = 2);
// 3-D tiled tensor map over a packed token-major [tokens, heads, inner] array
// of 2-byte elements (the varlen layout): dims {inner, heads, tokens}, box
// {box_inner, 1, box_tokens}, 128-byte swizzle.  A box lands in shared memory
// as box_tokens rows of box_inner elements, like a make_tmap_3d box.
int make_tmap_tokens(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                     uint64_t heads, uint64_t tokens, uint32_t box_inner, uint32_t box_tokens);
// 2-D tiled tensor map over a contiguous [rows, inner] array of 2-byte elements.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t rows, uint32_t box_inner, uint32_t box_rows, bool swizzle128);

// B2A_OK when an sm_100 device is current and dtype is f16/bf16; otherwise
// B2A_ERR_NO_DEVICE / B2A_ERR_UNSUPPORTED with the message recorded.
int require_device(int dtype);

// Read-and-clear of each translation unit's device error word.
int take_error_flags_prefill(uint32_t* flags);
int take_error_flags_prefill_d64(uint32_t* flags);
int take_error_flags_kvcache(uint32_t* flags);
int take_error_flags_backward(uint32_t* flags);
int take_error_flags_decode(uint32_t* flags);
int take_error_flags_selftest(uint32_t* flags);
int take_error_flags_exchange(uint32_t* flags);

// Defines take_error_flags_<unit>() for the unit that expands it.
#define B2A_DEFINE_ERROR_READER(unit)                                          \
  int take_error_flags_##unit(uint32_t* flags) {                              \
    uint32_t v = 0, zero = 0;                                                 \
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_error_flags, sizeof v);        \
    if (e != cudaSuccess) return set_cuda_error(e, "read device error word"); \
    e = cudaMemcpyToSymbol(g_error_flags, &zero, sizeof zero);                \
    if (e != cudaSuccess) return set_cuda_error(e, "clear device error word");\
    *flags |= v;                                                              \
    return B2A_OK;                                                            \
  }

// Kernel dispatchers (defined next to their kernels).
int prefill_dispatch(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                     int H, int Hkv, int N, int Nk, int D, int dtype, int causal, float scale,
                     cudaStream_t stream);
int prefill_varlen_dispatch(const void* q, const void* k, const void* v, void* o, float* lse,
                            const int* cu_q, const int* cu_k, int B, int H, int Hkv, int total_q,
                            int total_k, int max_seqlen_q, int D, int dtype, int causal,
                            float scale, cudaStream_t stream);
int prefill_d64_dispatch(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                         int H, int Hkv, int N, int Nk, int dtype, int causal, float scale,
                         cudaStream_t stream);
int decode_dispatch(const void* q, const void* k, const void* v, const int32_t* block_table,
                    const int32_t* kv_lens, float* o_part, float* l_part, int B, int H, int Hkv,
                    int Lkv, int D, int splits, int tokens_per_split, int page_size, int max_pages,
                    int num_pages, int dtype, float scale, cudaStream_t stream);
// fp32 workspace size of the backward (padded L/D rows + the dQ accumulator).
int64_t backward_workspace_floats(int B, int H, int N, int D);
int backward_dispatch(const void* q, const void* k, const void* v, const void* o, const void* dout,
                      const float* lse, void* dq, void* dk, void* dv, float* workspace, int B,
                      int H, int Hkv, int N, int Nk, int D, int dtype, int causal, float scale,
                      cudaStream_t stream);
int kv_append_dispatch(const void* k_new, const void* v_new, void* k_pool, void* v_pool,
                       const int32_t* block_table, int32_t* kv_lens, int B, int Hkv, int T, int D,
                       int page_size, int max_pages, int num_pages, int advance,
                       cudaStream_t stream);
// combine_dispatch's dtype for an fp32 merged partial (o, lse) instead of O.
constexpr int kCombineF32 = 100;
// ranks > 1: partials of `ranks` ranks, rank r's o / l blocks `rank_stride`
// floats after rank r-1's (KV-sharded decode's gathered buffer).
int combine_dispatch(const float* o_part, const float* l_part, void* o, float* lse, int B, int H,
                     int splits, int D, int dtype, const int32_t* kv_lens, int tps,
                     cudaStream_t stream, int ranks = 1, long long rank_stride = 0);

}  // namespace b2a

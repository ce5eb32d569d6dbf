// capi.cu -- the extern "C" boundary of libb200attn.so (declared in
// include/b200attn.h): argument validation, device checks and dispatch to the
// kernels.  Validation mirrors the reference's host checks
// (cuda/flash_attn_fa3_db_full.cu:352-363) and reuses their wording where the
// condition is the same.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "b2a_host.h"

namespace b2a {

namespace {
thread_local char t_last_error[512] = "";

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 1 = sm_100 device current, 0 = not; cached per device.
int device_ok() {
  static int cache[kMaxDevices] = {};  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  if (cache[dev] == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return 0;
    cache[dev] = (major == 10) ? 1 : 2;
  }
  return cache[dev] == 1;
}

// A pointer the current device can address as device memory (the C-level
// counterpart of the reference's "must be CUDA tensors" / "same device").
int check_device_ptr(const void* p, const char* what, bool need16 = true) {
  if (p == nullptr) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s must not be null", what);
    return set_error(B2A_ERR_INVALID_ARG, buf);
  }
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_cuda_error(e, what);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s must be CUDA device memory (Q/K/V must be CUDA tensors)", what);
    return set_error(B2A_ERR_INVALID_ARG, buf);
  }
  if (attr.type == cudaMemoryTypeDevice && attr.device != dev) {
    return set_error(B2A_ERR_INVALID_ARG, "Q/K/V must be on the same device");
  }
  if (need16 && !aligned16(p)) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s must be 16-byte aligned", what);
    return set_error(B2A_ERR_MISALIGNED, buf);
  }
  return B2A_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

#define B2A_TRY(expr)              \
  do {                             \
    int rc__ = (expr);             \
    if (rc__ != B2A_OK) return rc__; \
  } while (0)

int common_checks(int dtype) {
  if (!device_ok())
    return set_error(B2A_ERR_NO_DEVICE, "b200attn requires a current sm_100 (B200) CUDA device");
  if (dtype != B2A_F16 && dtype != B2A_BF16)
    return set_error(B2A_ERR_UNSUPPORTED, "dtype must be float16 or bfloat16");
  return B2A_OK;
}
}  // namespace

int set_error(int status, const char* msg) {
  snprintf(t_last_error, sizeof t_last_error, "%s", msg);
  return status;
}

int require_device(int dtype) { return common_checks(dtype); }

int set_cuda_error(cudaError_t e, const char* what) {
  snprintf(t_last_error, sizeof t_last_error, "%s: %s", what, cudaGetErrorString(e));
  return B2A_ERR_CUDA;
}

// A tensor map is a pure function of its arguments, so a small per-thread
// cache of recent encodings (keyed by every argument) saves the host-side
// encode when a caller reuses its buffers (the usual case in a serving loop).
namespace {
struct TmapKey {
  const void* base;
  int dt, rank, swz;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof *this) == 0; }
};
constexpr int kTmapCacheSize = 16;
thread_local TmapKey t_tmap_keys[kTmapCacheSize];
thread_local CUtensorMap t_tmap_vals[kTmapCacheSize];
thread_local int t_tmap_count = 0, t_tmap_next = 0;
}  // namespace

static int make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int rank,
                     const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                     bool swizzle128) {
  TmapKey key;
  std::memset(&key, 0, sizeof key);
  key.base = base;
  key.dt = (int)dt;
  key.rank = rank;
  key.swz = swizzle128 ? 1 : 0;
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) key.strides[i] = strides[i];
  for (int i = 0; i < t_tmap_count; ++i)
    if (t_tmap_keys[i] == key) {
      *map = t_tmap_vals[i];
      return B2A_OK;
    }
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(B2A_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return set_error(B2A_ERR_INVALID_ARG, buf);
  }
  const int slot = t_tmap_next;
  t_tmap_next = (t_tmap_next + 1) % kTmapCacheSize;
  if (t_tmap_count < kTmapCacheSize) ++t_tmap_count;
  t_tmap_keys[slot] = key;
  t_tmap_vals[slot] = *map;
  return B2A_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t rows, uint64_t outer, uint32_t box_inner, uint32_t box_rows,
                 bool swizzle128, uint32_t elem_bytes) {
  cuuint64_t dims[3] = {inner, rows, outer};
  cuuint64_t strides[2] = {inner * elem_bytes, inner * rows * elem_bytes};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  return make_tmap(map, base, dt, 3, dims, strides, box, swizzle128);
}

int make_tmap_tokens(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                     uint64_t heads, uint64_t tokens, uint32_t box_inner, uint32_t box_tokens) {
  cuuint64_t dims[3] = {inner, heads, tokens};
  cuuint64_t strides[2] = {inner * 2, inner * heads * 2};
  cuuint32_t box[3] = {box_inner, 1, box_tokens};
  return make_tmap(map, base, dt, 3, dims, strides, box, true);
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner,
                 uint64_t rows, uint32_t box_inner, uint32_t box_rows, bool swizzle128) {
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {box_inner, box_rows};
  return make_tmap(map, base, dt, 2, dims, strides, box, swizzle128);
}

}  // namespace b2a

using namespace b2a;

extern "C" {

const char* b2a_status_string(int status) {
  switch (status) {
    case B2A_OK: return "ok";
    case B2A_ERR_INVALID_ARG: return "invalid argument";
    case B2A_ERR_UNSUPPORTED: return "unsupported configuration";
    case B2A_ERR_MISALIGNED: return "misaligned pointer";
    case B2A_ERR_CUDA: return "CUDA error";
    case B2A_ERR_TIMEOUT: return "device wait timed out";
    case B2A_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

const char* b2a_last_error(void) { return t_last_error; }

const char* b2a_version(void) { return "0.1.0"; }

int b2a_prefill_fwd_kv(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                       int H, int Hkv, int N, int Nk, int D, int dtype, int causal, float scale,
                       void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (N <= 0 || Nk <= 0) return set_error(B2A_ERR_INVALID_ARG, "N must be > 0");
  if (causal && Nk < N)
    return set_error(B2A_ERR_INVALID_ARG,
                     "causal attention needs Nk >= N (the mask is aligned to the last key)");
  if (B <= 0 || H <= 0 || Hkv <= 0) return set_error(B2A_ERR_INVALID_ARG, "B, H and Hkv must be > 0");
  if (H % Hkv != 0) return set_error(B2A_ERR_INVALID_ARG, "H must be a multiple of Hkv");
  if ((int64_t)B * H > 0x7fffffff) return set_error(B2A_ERR_INVALID_ARG, "B*H too large");
  if ((N + 255) / 256 > 65535) return set_error(B2A_ERR_INVALID_ARG, "N too large (grid.y limit)");
  if (!(scale > 0.f)) return set_error(B2A_ERR_INVALID_ARG, "scale must be > 0");
  B2A_TRY(check_device_ptr(q, "Q"));
  B2A_TRY(check_device_ptr(k, "K"));
  B2A_TRY(check_device_ptr(v, "V"));
  B2A_TRY(check_device_ptr(o, "O"));
  if (lse != nullptr) B2A_TRY(check_device_ptr(lse, "L"));
  return prefill_dispatch(q, k, v, o, lse, B, H, Hkv, N, Nk, D, dtype, causal, scale,
                          static_cast<cudaStream_t>(stream));
}

int b2a_prefill_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H,
                    int Hkv, int N, int D, int dtype, int causal, float scale, void* stream) {
  return b2a_prefill_fwd_kv(q, k, v, o, lse, B, H, Hkv, N, N, D, dtype, causal, scale, stream);
}

int b2a_prefill_fwd_varlen(const void* q, const void* k, const void* v, void* o, float* lse,
                           const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int B, int H,
                           int Hkv, int total_q, int total_k, int max_seqlen_q, int D, int dtype,
                           int causal, float scale, void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || H <= 0 || Hkv <= 0) return set_error(B2A_ERR_INVALID_ARG, "B, H and Hkv must be > 0");
  if (H % Hkv != 0) return set_error(B2A_ERR_INVALID_ARG, "H must be a multiple of Hkv");
  if (total_q <= 0 || total_k <= 0 || max_seqlen_q <= 0)
    return set_error(B2A_ERR_INVALID_ARG, "total_q, total_k and max_seqlen_q must be > 0");
  if (max_seqlen_q > total_q)
    return set_error(B2A_ERR_INVALID_ARG, "max_seqlen_q must be <= total_q");
  if ((int64_t)B * H > 0x7fffffff) return set_error(B2A_ERR_INVALID_ARG, "B*H too large");
  if ((max_seqlen_q + 255) / 256 > 65535)
    return set_error(B2A_ERR_INVALID_ARG, "max_seqlen_q too large (grid.y limit)");
  if ((int64_t)total_q * H > 0x7fffffff || (int64_t)total_k * Hkv > 0x7fffffff)
    return set_error(B2A_ERR_INVALID_ARG, "total tokens x heads too large");
  if (!(scale > 0.f)) return set_error(B2A_ERR_INVALID_ARG, "scale must be > 0");
  B2A_TRY(check_device_ptr(q, "Q"));
  B2A_TRY(check_device_ptr(k, "K"));
  B2A_TRY(check_device_ptr(v, "V"));
  B2A_TRY(check_device_ptr(o, "O"));
  if (lse != nullptr) B2A_TRY(check_device_ptr(lse, "L"));
  B2A_TRY(check_device_ptr(cu_seqlens_q, "cu_seqlens_q", false));
  B2A_TRY(check_device_ptr(cu_seqlens_k, "cu_seqlens_k", false));
  if ((reinterpret_cast<uintptr_t>(cu_seqlens_q) | reinterpret_cast<uintptr_t>(cu_seqlens_k)) & 3u)
    return set_error(B2A_ERR_MISALIGNED, "cu_seqlens must be 4-byte aligned");
  return prefill_varlen_dispatch(q, k, v, o, lse, cu_seqlens_q, cu_seqlens_k, B, H, Hkv, total_q,
                                 total_k, max_seqlen_q, D, dtype, causal, scale,
                                 static_cast<cudaStream_t>(stream));
}

int b2a_decode_splitkv(const void* q, const void* k, const void* v, float* o_part, float* l_part,
                       int B, int H, int Hkv, int Lkv, int D, int splits, int dtype, float scale,
                       void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || H <= 0 || Hkv <= 0 || Lkv <= 0 || splits <= 0)
    return set_error(B2A_ERR_INVALID_ARG, "B, H, Hkv, Lkv and splits must be > 0");
  if (H % Hkv != 0) return set_error(B2A_ERR_INVALID_ARG, "H must be a multiple of Hkv");
  const int G = H / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return set_error(B2A_ERR_UNSUPPORTED, "GQA group H/Hkv must be 1, 2, 4 or 8");
  if (splits > 65535 || B > 65535 || Hkv > 65535)
    return set_error(B2A_ERR_INVALID_ARG, "splits, B and Hkv must be <= 65535");
  if (!(scale > 0.f)) return set_error(B2A_ERR_INVALID_ARG, "scale must be > 0");
  B2A_TRY(check_device_ptr(q, "q"));
  B2A_TRY(check_device_ptr(k, "K"));
  B2A_TRY(check_device_ptr(v, "V"));
  B2A_TRY(check_device_ptr(o_part, "o_part"));
  B2A_TRY(check_device_ptr(l_part, "l_part"));
  const int tps = (Lkv + splits - 1) / splits;
  return decode_dispatch(q, k, v, nullptr, nullptr, o_part, l_part, B, H, Hkv, Lkv, D, splits, tps,
                         0, 0, 0, dtype, scale, static_cast<cudaStream_t>(stream));
}

int b2a_decode_combine(const float* o_part, const float* l_part, void* o, float* lse, int B, int H,
                       int splits, int D, int dtype, void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || H <= 0 || splits <= 0)
    return set_error(B2A_ERR_INVALID_ARG, "B, H and splits must be > 0");
  B2A_TRY(check_device_ptr(o_part, "o_part"));
  B2A_TRY(check_device_ptr(l_part, "l_part"));
  B2A_TRY(check_device_ptr(o, "O"));
  if (lse != nullptr) B2A_TRY(check_device_ptr(lse, "L"));
  return combine_dispatch(o_part, l_part, o, lse, B, H, splits, D, dtype, nullptr, 0,
                          static_cast<cudaStream_t>(stream));
}

int b2a_decode_combine_ranks(const float* o_part, const float* l_part, void* o, float* lse, int B,
                             int H, int splits, int ranks, int64_t rank_stride, int D, int dtype,
                             void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || H <= 0 || splits <= 0 || ranks <= 0)
    return set_error(B2A_ERR_INVALID_ARG, "B, H, splits and ranks must be > 0");
  const int64_t block = (int64_t)B * H * splits * D;
  if (ranks > 1 && rank_stride < block + (int64_t)B * H * splits)
    return set_error(B2A_ERR_INVALID_ARG,
                     "rank_stride must cover one rank's o and l partials (B*H*splits*(D+1) floats)");
  B2A_TRY(check_device_ptr(o_part, "o_part"));
  B2A_TRY(check_device_ptr(l_part, "l_part", false));
  if (reinterpret_cast<uintptr_t>(l_part) & 3u)
    return set_error(B2A_ERR_MISALIGNED, "l_part must be 4-byte aligned");
  B2A_TRY(check_device_ptr(o, "O"));
  if (lse != nullptr) B2A_TRY(check_device_ptr(lse, "L"));
  return combine_dispatch(o_part, l_part, o, lse, B, H, splits, D, dtype, nullptr, 0,
                          static_cast<cudaStream_t>(stream), ranks, (long long)rank_stride);
}

int b2a_decode_merge_splits(const float* o_part, const float* l_part, float* o_merged,
                            float* l_merged, int B, int H, int splits, int D, void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(B2A_F16));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || H <= 0 || splits <= 0)
    return set_error(B2A_ERR_INVALID_ARG, "B, H and splits must be > 0");
  B2A_TRY(check_device_ptr(o_part, "o_part"));
  B2A_TRY(check_device_ptr(l_part, "l_part"));
  B2A_TRY(check_device_ptr(o_merged, "o_merged"));
  B2A_TRY(check_device_ptr(l_merged, "l_merged", false));
  if (reinterpret_cast<uintptr_t>(l_merged) & 3u)
    return set_error(B2A_ERR_MISALIGNED, "l_merged must be 4-byte aligned");
  return combine_dispatch(o_part, l_part, o_merged, l_merged, B, H, splits, D, kCombineF32,
                          nullptr, 0, static_cast<cudaStream_t>(stream));
}

int b2a_decode_paged(const void* q, const void* k_pool, const void* v_pool,
                     const int32_t* block_table, const int32_t* kv_lens, float* o_part,
                     float* l_part, void* o, float* lse, int B, int H, int Hkv, int D,
                     int page_size, int max_pages, int num_pages, int pages_per_split, int dtype,
                     float scale, void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (page_size != 16 && page_size != 32 && page_size != 64)
    return set_error(B2A_ERR_UNSUPPORTED, "page_size must be 16, 32 or 64");
  if (B <= 0 || H <= 0 || Hkv <= 0 || max_pages <= 0 || num_pages <= 0 || pages_per_split <= 0)
    return set_error(B2A_ERR_INVALID_ARG,
                     "B, H, Hkv, max_pages, num_pages and pages_per_split must be > 0");
  if (pages_per_split > 256) return set_error(B2A_ERR_INVALID_ARG, "pages_per_split must be <= 256");
  if ((int64_t)num_pages * Hkv > 0x7fffffff)
    return set_error(B2A_ERR_INVALID_ARG, "num_pages * Hkv too large");
  if (H % Hkv != 0) return set_error(B2A_ERR_INVALID_ARG, "H must be a multiple of Hkv");
  const int G = H / Hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return set_error(B2A_ERR_UNSUPPORTED, "GQA group H/Hkv must be 1, 2, 4 or 8");
  if ((pages_per_split * page_size) % 64 != 0)
    return set_error(B2A_ERR_INVALID_ARG, "pages_per_split * page_size must be a multiple of 64");
  const int splits = (max_pages + pages_per_split - 1) / pages_per_split;
  if (splits > 65535 || B > 65535 || Hkv > 65535)
    return set_error(B2A_ERR_INVALID_ARG, "splits, B and Hkv must be <= 65535");
  if (!(scale > 0.f)) return set_error(B2A_ERR_INVALID_ARG, "scale must be > 0");
  B2A_TRY(check_device_ptr(q, "q"));
  B2A_TRY(check_device_ptr(k_pool, "k_pool"));
  B2A_TRY(check_device_ptr(v_pool, "v_pool"));
  B2A_TRY(check_device_ptr(block_table, "block_table"));
  B2A_TRY(check_device_ptr(kv_lens, "kv_lens"));
  B2A_TRY(check_device_ptr(o_part, "o_part"));
  B2A_TRY(check_device_ptr(l_part, "l_part"));
  B2A_TRY(check_device_ptr(o, "O"));
  if (lse != nullptr) B2A_TRY(check_device_ptr(lse, "L"));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tps = pages_per_split * page_size;
  B2A_TRY(decode_dispatch(q, k_pool, v_pool, block_table, kv_lens, o_part, l_part, B, H, Hkv, 0, D,
                          splits, tps, page_size, max_pages, num_pages, dtype, scale, s));
  return combine_dispatch(o_part, l_part, o, lse, B, H, splits, D, dtype, kv_lens, tps, s);
}

int b2a_backward(const void* q, const void* k, const void* v, const void* o, const void* dout,
                 const float* lse, void* dq, void* dk, void* dv, float* workspace, int B, int H,
                 int Hkv, int N, int Nk, int D, int dtype, int causal, float scale, void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (N <= 0 || Nk <= 0) return set_error(B2A_ERR_INVALID_ARG, "N must be > 0");
  if (causal && Nk < N)
    return set_error(B2A_ERR_INVALID_ARG,
                     "causal attention needs Nk >= N (the mask is aligned to the last key)");
  if (B <= 0 || H <= 0 || Hkv <= 0) return set_error(B2A_ERR_INVALID_ARG, "B, H and Hkv must be > 0");
  if (H % Hkv != 0) return set_error(B2A_ERR_INVALID_ARG, "H must be a multiple of Hkv");
  if ((int64_t)B * Hkv > 65535) return set_error(B2A_ERR_INVALID_ARG, "B*Hkv must be <= 65535");
  if (!(scale > 0.f)) return set_error(B2A_ERR_INVALID_ARG, "scale must be > 0");
  B2A_TRY(check_device_ptr(q, "Q"));
  B2A_TRY(check_device_ptr(k, "K"));
  B2A_TRY(check_device_ptr(v, "V"));
  B2A_TRY(check_device_ptr(o, "O"));
  B2A_TRY(check_device_ptr(dout, "dO"));
  B2A_TRY(check_device_ptr(lse, "L"));
  B2A_TRY(check_device_ptr(dq, "dQ"));
  B2A_TRY(check_device_ptr(dk, "dK"));
  B2A_TRY(check_device_ptr(dv, "dV"));
  B2A_TRY(check_device_ptr(workspace, "workspace"));
  return backward_dispatch(q, k, v, o, dout, lse, dq, dk, dv, workspace, B, H, Hkv, N, Nk, D,
                           dtype, causal, scale, static_cast<cudaStream_t>(stream));
}

int64_t b2a_backward_workspace_floats(int B, int H, int N, int D) {
  return backward_workspace_floats(B, H, N, D);
}

int b2a_kv_append_paged(const void* k_new, const void* v_new, void* k_pool, void* v_pool,
                        const int32_t* block_table, int32_t* kv_lens, int B, int Hkv, int T,
                        int D, int page_size, int max_pages, int num_pages, int dtype,
                        int advance_lens, void* stream) {
  t_last_error[0] = 0;
  B2A_TRY(common_checks(dtype));
  if (D != 64 && D != 128) return set_error(B2A_ERR_UNSUPPORTED, "Head dimension must be 64 or 128");
  if (B <= 0 || Hkv <= 0 || T <= 0 || page_size <= 0 || max_pages <= 0 || num_pages <= 0)
    return set_error(B2A_ERR_INVALID_ARG,
                     "B, Hkv, T, page_size, max_pages and num_pages must be > 0");
  if (B > 65535 || Hkv > 65535) return set_error(B2A_ERR_INVALID_ARG, "B and Hkv must be <= 65535");
  B2A_TRY(check_device_ptr(k_new, "k_new"));
  B2A_TRY(check_device_ptr(v_new, "v_new"));
  B2A_TRY(check_device_ptr(k_pool, "k_pool"));
  B2A_TRY(check_device_ptr(v_pool, "v_pool"));
  B2A_TRY(check_device_ptr(block_table, "block_table"));
  B2A_TRY(check_device_ptr(kv_lens, "kv_lens"));
  return kv_append_dispatch(k_new, v_new, k_pool, v_pool, block_table, kv_lens, B, Hkv, T, D,
                            page_size, max_pages, num_pages, advance_lens,
                            static_cast<cudaStream_t>(stream));
}

int b2a_device_error(uint32_t* flags) {
  t_last_error[0] = 0;
  if (flags == nullptr) return set_error(B2A_ERR_INVALID_ARG, "flags must not be null");
  if (!device_ok())
    return set_error(B2A_ERR_NO_DEVICE, "b200attn requires a current sm_100 (B200) CUDA device");
  uint32_t v = 0;
  B2A_TRY(take_error_flags_prefill(&v));
  B2A_TRY(take_error_flags_prefill_d64(&v));
  B2A_TRY(take_error_flags_kvcache(&v));
  B2A_TRY(take_error_flags_backward(&v));
  B2A_TRY(take_error_flags_decode(&v));
  B2A_TRY(take_error_flags_selftest(&v));
  B2A_TRY(take_error_flags_exchange(&v));
  *flags = v;
  if (v & 1u) {
    char buf[160];
    snprintf(buf, sizeof buf,
             "a device-side bounded wait timed out (error word 0x%x); outputs of the calls "
             "since the last check are undefined", v);
    return set_error(B2A_ERR_TIMEOUT, buf);
  }
  return B2A_OK;
}

}  // extern "C"

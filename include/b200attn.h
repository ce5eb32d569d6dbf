/*
 * b200attn.h -- C ABI of libb200attn.so, the B200 (sm_100a) attention library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed
 * as `void*`; nothing here names a torch or pybind type.  All buffers are owned
 * by the caller (no allocation, no ownership transfer).  Calls are asynchronous
 * on `stream` and return a status; a non-OK status leaves a human-readable
 * message in b2a_last_error() (thread-local).
 *
 * Layouts (row-major, contiguous, element strides implied by the shape):
 *   prefill    Q,O [B,H,N,D]; K,V [B,Hkv,N,D]; lse [B,H,N] fp32 (natural log)
 *   decode     q,o [B,H,D] (query length 1); K,V [B,Hkv,Lkv,D]
 *   partials   o_part [B,H,S,D] fp32 (each split normalised by its own sum),
 *              l_part [B,H,S] fp32 (natural-log sum of exp over the split)
 *   paged      k_pool,v_pool [P,Hkv,page_size,D]; block_table int32
 *              [B,max_pages]; kv_lens int32 [B]
 *
 * Reference interface being replaced (Bias92/flashattn-cuda):
 *   cuda/flash_attn_fa3_db_full.cu:349-403  fa3db_full_forward_impl
 *   cuda/flash_attn_fa3_db_full.cu:405-418  forward / forward_only bindings
 * The decode entry points have no function in the reference; they follow the
 * same conventions (fp32 natural-log L, scale D^-0.5 by default).
 */
#ifndef B200ATTN_H_
#define B200ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  B2A_OK = 0,
  B2A_ERR_INVALID_ARG = 1,   /* bad shape / null pointer / out-of-range size   */
  B2A_ERR_UNSUPPORTED = 2,   /* dtype, head dim or group size not built        */
  B2A_ERR_MISALIGNED = 3,    /* a pointer is not 16-byte aligned (TMA rule)     */
  B2A_ERR_CUDA = 4,          /* a CUDA runtime/driver call failed               */
  B2A_ERR_TIMEOUT = 5,       /* a device-side bounded wait gave up             */
  B2A_ERR_NO_DEVICE = 6      /* no sm_100 device is current                     */
} b2a_status;

typedef enum { B2A_F16 = 0, B2A_BF16 = 1 } b2a_dtype;

/* Human-readable name of a status code. */
const char* b2a_status_string(int status);
/* Message of the last failing call on this thread ("" if none). */
const char* b2a_last_error(void);
/* Library version, e.g. "0.1.0". */
const char* b2a_version(void);

/*
 * Prefill forward: O = softmax(Q K^T * scale [+ causal mask]) V and, when
 * lse != NULL, L = logsumexp of the scaled scores per query row.
 * lse == NULL is the O-only path (reference forward_only); O is bitwise equal
 * between the two paths.  H % Hkv == 0 (Hkv == H is the reference's case).
 * D in {64, 128}; dtype f16 or bf16 (the reference casts everything to f16).
 * Replaces: cuda/flash_attn_fa3_db_full.cu:349-403 (fa3db_full_forward_impl)
 * and the kernel fa3db_full_fwd_kernel (same file, 87-344).
 */
int b2a_prefill_fwd(const void* q, const void* k, const void* v, void* o,
                    float* lse, int B, int H, int Hkv, int N, int D,
                    int dtype, int causal, float scale, void* stream);

/*
 * Prefill forward with a key/value length Nk that may differ from the query
 * length N (cross-attention, or a chunk of N new queries over a cache of Nk
 * keys): Q,O [B,H,N,D], K,V [B,Hkv,Nk,D], lse [B,H,N].  With causal != 0 the
 * mask is aligned to the last key -- query row r sees keys 0 .. r + Nk - N --
 * and Nk >= N is required.  b2a_prefill_fwd is the Nk == N case.  The
 * reference requires K and V to have Q's shape
 * (cuda/flash_attn_fa3_db_full.cu:358-359); this lifts that restriction.
 */
int b2a_prefill_fwd_kv(const void* q, const void* k, const void* v, void* o,
                       float* lse, int B, int H, int Hkv, int N, int Nk, int D,
                       int dtype, int causal, float scale, void* stream);

/*
 * Variable-length prefill forward: B sequences packed token-major,
 * Q,O [total_q, H, D], K,V [total_k, Hkv, D]; sequence b owns query tokens
 * cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 and keys cu_seqlens_k[b] ..
 * cu_seqlens_k[b+1]-1 (int32 device arrays of B+1 prefix sums starting at 0).
 * lse is [H, total_q] (nullable).  max_seqlen_q bounds every query length (it
 * sizes the grid; a longer sequence sets bit 3 of the device error word and
 * its tail rows are not computed).  With causal != 0 the mask is aligned per
 * sequence to its last key; a query row that sees no key gets O = 0 and
 * lse = -inf.  The reference has no varlen form: it requires K and V to have
 * Q's shape (cuda/flash_attn_fa3_db_full.cu:358-359).
 */
int b2a_prefill_fwd_varlen(const void* q, const void* k, const void* v, void* o,
                           float* lse, const int32_t* cu_seqlens_q,
                           const int32_t* cu_seqlens_k, int B, int H, int Hkv,
                           int total_q, int total_k, int max_seqlen_q, int D,
                           int dtype, int causal, float scale, void* stream);

/*
 * Backward of the prefill forward: dQ [B,H,N,D], dK, dV [B,Hkv,Nk,D] (dtype)
 * from Q, K, V, the forward's O and lse (natural-log logsumexp, fp32) and the
 * upstream gradient dO [B,H,N,D]; causal and scale as in the forward.  For
 * GQA, dK/dV of a KV head sum over its query heads.  `workspace` is
 * caller-provided fp32 scratch of b2a_backward_workspace_floats(B,H,N,D)
 * floats (row statistics and the dQ accumulator).  Replaces the reference's
 * backward(Q, K, V, O, dO, L) -> [dQ, dK, dV]
 * (cuda/flash_attn_kernel.cu:417-502 with the kernels at :173-412).
 */
int b2a_backward(const void* q, const void* k, const void* v, const void* o,
                 const void* dout, const float* lse, void* dq, void* dk,
                 void* dv, float* workspace, int B, int H, int Hkv, int N,
                 int Nk, int D, int dtype, int causal, float scale,
                 void* stream);
/* Floats of workspace b2a_backward needs: 2*B*H*Npad (row statistics, Npad =
 * N rounded up to 128) + B*H*N*D (the fp32 dQ accumulator). */
int64_t b2a_backward_workspace_floats(int B, int H, int N, int D);

/*
 * Split-KV decode, first stage: for each (batch, query head, split) the
 * softmax-normalised partial output and its natural-log sum of exp.  The KV
 * sequence of length Lkv is cut into `splits` chunks of ceil(Lkv/splits)
 * tokens; empty chunks write l = -inf, o = 0.  GQA group G = H/Hkv in
 * {1,2,4,8}; D in {64,128}.  No counterpart in the reference (new entry point
 * in the style of cuda/flash_attn_fa3_db_full.cu:405-408).
 */
int b2a_decode_splitkv(const void* q, const void* k, const void* v,
                       float* o_part, float* l_part, int B, int H, int Hkv,
                       int Lkv, int D, int splits, int dtype, float scale,
                       void* stream);

/*
 * LSE-weighted combine of split partials: L = log sum_s exp(l_s),
 * O = sum_s exp(l_s - L) * o_s, written as dtype O [B,H,D] and fp32 lse [B,H]
 * (lse may be NULL).  The identity is the online-softmax rescale of
 * cuda/flash_attn_fa3_db_full.cu:261-284 and :340 applied across splits.
 */
int b2a_decode_combine(const float* o_part, const float* l_part, void* o,
                       float* lse, int B, int H, int splits, int D, int dtype,
                       void* stream);

/*
 * Merge of `splits` split partials into ONE partial of the same form, in fp32:
 * o_merged [B,H,D] = sum_s exp(l_s - L) o_s and l_merged [B,H] = L =
 * log sum_s exp(l_s).  A KV-sharded rank merges its own splits with this
 * before the exchange, so that it sends B*H*(D+1) floats instead of
 * B*H*splits*(D+1); b2a_decode_combine_ranks with splits = 1 then combines
 * the ranks.  Same identity as b2a_decode_combine
 * (cuda/flash_attn_fa3_db_full.cu:261-284, :340), fp32 output.
 */
int b2a_decode_merge_splits(const float* o_part, const float* l_part,
                            float* o_merged, float* l_merged, int B, int H,
                            int splits, int D, void* stream);

/*
 * LSE-weighted combine of partials gathered from `ranks` ranks (KV-sharded
 * decode): rank r's o block [B,H,splits,D] starts r*rank_stride floats after
 * o_part and its l block [B,H,splits] r*rank_stride floats after l_part, and
 * rank r's splits follow rank r-1's in sequence order.  This reads the buffer
 * an all-gather of per-rank [o | l] chunks of rank_stride floats produces,
 * without a reordering copy.  ranks == 1 is b2a_decode_combine.  Same identity
 * as b2a_decode_combine (cuda/flash_attn_fa3_db_full.cu:261-284, :340).
 */
int b2a_decode_combine_ranks(const float* o_part, const float* l_part, void* o,
                             float* lse, int B, int H, int splits, int ranks,
                             int64_t rank_stride, int D, int dtype, void* stream);

/*
 * KV-sharded decode's exchange step as ONE kernel over NVLink peer memory.
 * Each of `world` ranks (one GPU each, one process each) owns an exchange
 * buffer of b2a_exchange_bytes(B, H, D, world) bytes made by
 * b2a_exchange_alloc, which also fills a 64-byte CUDA IPC handle; the ranks
 * swap handles (any host channel) and map each other's buffers with
 * b2a_exchange_open.  `peers` is a device array of `world` uint64 addresses,
 * peers[r] = rank r's buffer as mapped here (peers[rank] = the own buffer).
 * A call merges this rank's split partials o_part [B,H,splits,D] / l_part
 * [B,H,splits] (from b2a_decode_splitkv on its contiguous KV slice), stores
 * the merged partial into every rank's buffer as 8-byte words tagged with
 * the call count, polls its own buffer (bounded, 1 s; bit 0 of the device
 * error word on timeout) until every rank's words of this call are there,
 * and writes O [B,H,D]
 * (dtype) and lse [B,H] (may be NULL) -- identical on every rank.  Every rank
 * must make the same sequence of calls with the same B, H, D; calls on one
 * rank must be ordered (one stream); nothing is reset between calls.  It
 * replaces the all-gather of partials plus combine: the combine identity is
 * the online-softmax rescale of cuda/flash_attn_fa3_db_full.cu:261-284 and
 * :340; the reference has no multi-GPU code.  b2a_exchange_close unmaps a
 * peer buffer and b2a_exchange_free frees the own one (after every peer has
 * stopped using it).
 */
int64_t b2a_exchange_bytes(int B, int H, int D, int world);
int b2a_exchange_alloc(int64_t bytes, void** ptr, void* ipc_handle);
int b2a_exchange_open(const void* ipc_handle, void** ptr);
int b2a_exchange_close(void* peer_ptr);
int b2a_exchange_free(void* ptr);
int b2a_decode_exchange_combine(const float* o_part, const float* l_part,
                                const uint64_t* peers, int rank, int world,
                                void* o, float* lse, int B, int H, int splits,
                                int D, int dtype, void* stream);

/*
 * Paged decode: as split-KV decode, but token t of sequence b lives in page
 * block_table[b, t / page_size] at slot t % page_size of k_pool/v_pool
 * ([P,Hkv,page_size,D]).  Sequence b has kv_lens[b] >= 1 tokens.  Each split
 * covers `pages_per_split` pages; o_part/l_part are scratch sized
 * [B,H,ceil(max_pages/pages_per_split),D] and [B,H,ceil(...)] that the caller
 * provides.  num_pages is the pool size P; a block-table entry outside
 * [0, P) sets bit 1 of the device error word and reads page 0 instead.
 * Writes O [B,H,D] (dtype) and lse [B,H] (may be NULL).  page_size in
 * {16, 32, 64}; pages_per_split * page_size a multiple of 64 and
 * pages_per_split <= 256.  No counterpart in the reference.
 */
int b2a_decode_paged(const void* q, const void* k_pool, const void* v_pool,
                     const int32_t* block_table, const int32_t* kv_lens,
                     float* o_part, float* l_part, void* o, float* lse, int B,
                     int H, int Hkv, int D, int page_size, int max_pages,
                     int num_pages, int pages_per_split, int dtype, float scale,
                     void* stream);

/*
 * Append T new tokens per sequence to a paged KV cache (the write path of
 * b2a_decode_paged): k_new, v_new [B,Hkv,T,D] go to positions kv_lens[b] + t
 * of sequence b, i.e. page block_table[b, pos / page_size], slot pos %
 * page_size of k_pool / v_pool [P,Hkv,page_size,D].  The block table must
 * already hold a page for every written position (a missing or out-of-range
 * entry sets bit 2 of the device error word and that token is not written).
 * With advance_lens != 0, kv_lens[b] += T afterwards (same stream).  No
 * counterpart in the reference.
 */
int b2a_kv_append_paged(const void* k_new, const void* v_new, void* k_pool,
                        void* v_pool, const int32_t* block_table,
                        int32_t* kv_lens, int B, int Hkv, int T, int D,
                        int page_size, int max_pages, int num_pages, int dtype,
                        int advance_lens, void* stream);

/*
 * Paged decode that allocates nothing and takes no scratch buffer: identical
 * arguments and results to b2a_decode_paged minus o_part/l_part.  It is for
 * callers that cannot call cudaMalloc where they decode (an allocator-free
 * serving runtime that reserves all device memory up front, a memory pool
 * that must not grow, a plugin host that forbids allocation on its request
 * path).  The split partials go to a fixed 16 MiB array inside the library
 * that every GPU loading the library holds until exit; a call needing more
 * than that, B*H*ceil(max_pages/pages_per_split)*(D+1) > 4,194,304 floats,
 * is rejected with B2A_ERR_INVALID_ARG.  The first call on each device looks
 * up that array's device address (make it before any stream capture).  All
 * calls on one device share that device's copy of the array, which keeps the
 * last call's contents (nothing in it has to start at zero: every entry a
 * call reads is written earlier in the same call).  Two calls that can run
 * at the same time on one device, e.g. on different streams, race on it and
 * must be ordered by the caller.  The looked-up address is kept for the life
 * of the process, so do not use the library across a cudaDeviceReset of a
 * device it has run on.  No counterpart in the reference.
 */
int b2a_decode_paged_noalloc(const void* q, const void* k_pool,
                             const void* v_pool, const int32_t* block_table,
                             const int32_t* kv_lens, void* o, float* lse,
                             int B, int H, int Hkv, int D, int page_size,
                             int max_pages, int num_pages, int pages_per_split,
                             int dtype, float scale, void* stream);

/*
 * Device error word written by the kernels (bit 0: a bounded pipeline wait
 * timed out; bit 1: a paged-decode block-table entry was out of range;
 * bit 2: a KV append found no page for a position; bit 3: a varlen sequence
 * was longer than max_seqlen_q or cu_seqlens was not non-decreasing; bit 4:
 * the backward kernel found too little shared memory to align its tiles and
 * did nothing; bit 0 is also set when b2a_decode_exchange_combine gave up
 * waiting for a peer).  Reads and clears the
 * word of the current device; this call synchronises the device.  *flags
 * receives the word.  Returns B2A_ERR_TIMEOUT when bit 0 is set (the outputs
 * of the calls since the previous check are then undefined), B2A_OK
 * otherwise (the other bits report bad inputs and leave the status OK).
 * The reference has no device-side status: it checks only the launch
 * (cuda/flash_attn_fa3_db_full.cu:399).
 */
int b2a_device_error(uint32_t* flags);

/*
 * Self-test of the bounded waits: launches one thread that waits, with a
 * limit of limit_us microseconds (1 .. 1,000,000), on an mbarrier nothing
 * arrives at, synchronises `stream` and returns what that wait reported --
 * B2A_ERR_TIMEOUT when it gave up as intended.  Nothing else is in flight in
 * that kernel, so the device stays usable afterwards.  It shows that a
 * pipeline wait that is never satisfied ends as a status on the host instead
 * of a hang.  No counterpart in the reference (its only checks are host-side,
 * cuda/flash_attn_fa3_db_full.cu:352-363 and :399).
 */
int b2a_selftest_wait_timeout(int limit_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200ATTN_H_ */

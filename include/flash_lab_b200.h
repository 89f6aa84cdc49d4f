/*
 * flash_lab_b200.h — C ABI of the B200 (sm_100a) attention library behind flash_lab's operators.
 *
 * This ABI replaces the reference's PyTorch-extension boundary (tfan2437/flash-attention-lab):
 * the op schemas of csrc/bindings.cpp:7-42 and the per-op host glue that checked inputs, built
 * parameter structs and launched kernels (csrc/common/attn_host.h:18-93,
 * csrc/prefill/mma_pipelined.cu:152-185, csrc/decode/decode_host.h:18-85,
 * csrc/decode/decode.cu:231-340). Python binds it with ctypes and registers the same
 * torch.library schemas on top (flash_lab/_capi.py and flash_lab/ops.py in this repository).
 *
 * Conventions
 *  - Plain C: raw device pointers, int64 element strides, int32 sizes. No torch types.
 *  - The caller owns every buffer (inputs, outputs, workspaces). Apart from the one entry point
 *    documented as allocation-free with static scratch, the library allocates nothing, never
 *    synchronises, and launches only on the stream it is given.
 *  - Every entry point returns an flb_status. Nothing throws or aborts across the ABI.
 *    flb_last_error() gives a message for the calling thread's most recent failure.
 *  - Reentrant: no mutable global state except one-time per-device kernel attribute set-up.
 *    That set-up (shared-memory opt-ins, the static scratch address) is cached per device for
 *    the life of the process, so the library must not be used on a device again after
 *    cudaDeviceReset there.
 *  - Optional `status` device word: kernels whose pipeline waits exceed their deadline write a
 *    nonzero code there (first writer wins) and return early instead of hanging. Pass NULL to
 *    skip.
 */
#ifndef FLASH_LAB_B200_H_
#define FLASH_LAB_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FLB_ABI_VERSION 3

/* Most ranks a peer exchange (cross-GPU decode merge over NVLink) connects. */
#define FLB_MAX_PEERS 8

/* Stream handle: the same object as cudaStream_t / CUstream (NULL = legacy default stream). */
typedef struct CUstream_st* flb_stream_t;

typedef enum {
  FLB_OK = 0,
  FLB_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, inconsistent shape */
  FLB_ERR_UNSUPPORTED = 2,      /* dtype / head_dim / group not compiled into this library */
  FLB_ERR_MISALIGNED = 3,       /* a pointer or stride breaks the 16-byte row rule */
  FLB_ERR_CUDA = 4,             /* CUDA runtime or driver error (see flb_last_error) */
  FLB_ERR_WORKSPACE = 5,        /* workspace missing or smaller than flb_decode_workspace_bytes */
  FLB_ERR_NO_DEVICE = 6         /* no sm_100 device current */
} flb_status;

/* FLB_FP32 is accepted by the decode entry points only (the reference's fp32 decode). */
typedef enum { FLB_BF16 = 0, FLB_FP16 = 1, FLB_FP32 = 2 } flb_dtype;

/*
 * Prefill problem. Mirrors AttnParams (csrc/common/params.h:9-27 of the reference).
 * q [B, S_q, H, D], k and v [B, S_k, H_kv, D], o [B, S_q, H, D] (input dtype), lse [B, H, S_q]
 * fp32 contiguous (natural-log log-sum-exp of each scaled score row, -inf for rows that see no
 * key). Strides are in elements; the head_dim stride must be 1, every other stride and every
 * base pointer a multiple of 16 bytes. Query head h reads KV head h / (H / H_kv).
 * Causal masking is aligned to the bottom-right corner: query i sees key j iff
 * j <= i + (S_k - S_q).
 */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int64_t q_batch_stride, q_seq_stride, q_head_stride;
  int64_t k_batch_stride, k_seq_stride, k_head_stride;
  int64_t v_batch_stride, v_seq_stride, v_head_stride;
  int64_t o_batch_stride, o_seq_stride, o_head_stride;
  int32_t batch, seqlen_q, seqlen_k, heads, heads_kv, head_dim;
  int32_t causal;        /* 0 or 1 */
  int32_t dtype;         /* flb_dtype */
  float softmax_scale;   /* > 0 */
  int32_t* status;       /* optional device status word */
} flb_attn_params;

/*
 * Decode problem (one query token per sequence). Mirrors DecodeParams
 * (csrc/common/params.h:31-53 of the reference).
 * q [B, H, D]; k_cache / v_cache [B, S_max, H_kv, D] read in place through their strides;
 * seq_lens [B] int32 on the device (values are clamped to [0, S_max] on the device, never read
 * on the host); o [B, H, D]; lse [B, H] fp32 contiguous.
 * num_splits: 0 lets the library choose from the shapes only (flb_decode_num_splits), which keeps
 * the call CUDA-graph safe; 1 runs without a merge step. workspace must hold
 * flb_decode_workspace_bytes(...) bytes of device memory when the split count is above 1.
 * With more than one split, flb_decode_fwd launches batch * num_splits CTAs per KV head. For
 * 16-bit caches and batch <= 128 their key ranges are length-balanced: the sequences' 64-key
 * chunks are shared evenly among those CTAs, so a long sequence gets more of them than a short
 * one (read from seq_lens on the device; still graph safe). Otherwise each sequence is cut into
 * num_splits equal ranges.
 */
typedef struct {
  const void* q;
  const void* k_cache;
  const void* v_cache;
  void* o;
  float* lse;
  const int32_t* seq_lens;
  int64_t q_batch_stride, q_head_stride;
  int64_t k_batch_stride, k_seq_stride, k_head_stride;
  int64_t v_batch_stride, v_seq_stride, v_head_stride;
  int64_t o_batch_stride, o_head_stride;
  int32_t batch, heads, heads_kv, head_dim, max_seqlen;
  int32_t num_splits;    /* 0 = choose */
  int32_t dtype;         /* flb_dtype */
  float softmax_scale;   /* > 0 */
  void* workspace;
  size_t workspace_bytes;
  int32_t* status;       /* optional device status word */
  /* Paged cache when block_tables is not NULL (the reference's paged layout, layouts.py:95-167):
   * k_cache / v_cache are [num_blocks, page_size, H_kv, D] with k_batch_stride the block stride
   * and k_seq_stride the row stride; key j of sequence b is row j % page_size of block
   * block_tables[b * block_table_stride + j / page_size]; max_seqlen = max_blocks * page_size.
   * page_size is 8, 16, 32 or a multiple of 64. Block ids outside [0, num_blocks) read as
   * zeros. */
  const int32_t* block_tables;
  int64_t block_table_stride;
  int32_t page_size;
  int32_t num_blocks;
} flb_decode_params;

/* ABI version (FLB_ABI_VERSION). No reference counterpart. */
int flb_version(void);

/* Static text for a status code. No reference counterpart (the reference raised c10 errors,
 * csrc/common/checks.h:6-25). */
const char* flb_status_string(int status);

/* Message describing the calling thread's most recent failure ("" if none). */
const char* flb_last_error(void);

/* Prefill forward: o, lse = attention(q, k, v). Replaces the attention_mma_pipelined op
 * (csrc/prefill/mma_pipelined.cu:162-185, schema csrc/bindings.cpp:20-21) and its launcher
 * (mma_pipelined.cu:152-158). bf16 or fp16, head_dim 128. */
int flb_prefill_fwd(const flb_attn_params* params, flb_stream_t stream);

/* Split count the decode picks when num_splits == 0, from shapes and the SM count only.
 * Replaces choose_num_splits (csrc/decode/decode.cu:272-280). */
int flb_decode_num_splits(int32_t batch, int32_t heads, int32_t heads_kv, int32_t head_dim,
                          int32_t max_seqlen, int32_t sm_count);

/* Bytes of device workspace flb_decode_fwd needs for this split count (0 when num_splits <= 1):
 * fp32 partials for batch * heads * (2 * num_splits + 1) slots, (head_dim + 2) floats each.
 * Replaces the per-call partial_o / partial_ml allocations (csrc/decode/decode.cu:303-311). */
size_t flb_decode_workspace_bytes(int32_t batch, int32_t heads, int32_t head_dim,
                                  int32_t num_splits);

/* Split-KV decode step. Replaces the decode_splitkv / decode_inplace ops
 * (csrc/decode/decode.cu:282-340, schemas csrc/bindings.cpp:30-37). bf16, fp16 or fp32 (the
 * reference's three decode dtypes), head_dim 64 or 128. */
int flb_decode_fwd(const flb_decode_params* params, flb_stream_t stream);

/*
 * Allocation-free decode step. No counterpart in the reference: this entry point is an
 * addition for callers that cannot allocate device memory when they decode. cudaMalloc may
 * synchronise the device and is not allowed during CUDA-graph stream capture, and a serving loop
 * that plans its memory up front may forbid allocation altogether. It computes exactly what
 * flb_decode_fwd computes (the same kernels, the same split count), but keeps the split partials
 * in a static device array of flb_decode_static_scratch_bytes() bytes (8 MiB) instead of a
 * caller workspace; params->workspace is ignored. Problems whose partials do not fit
 * (flb_decode_workspace_bytes: B * H * (2 * splits + 1) * (head_dim + 2) * 4 bytes, rounded) return
 * FLB_ERR_WORKSPACE without launching.
 * Every GPU that loads the library holds the array until exit. All calls on a device share it
 * and it keeps the last call's contents (nothing needs to start at zero), so calls that overlap
 * on the GPU race. The first call on a device looks up the array's address with that device
 * current; make it before any stream capture. It calls no cudaMalloc, cudaFree or other
 * allocating routine.
 */
int flb_decode_fwd_static(const flb_decode_params* params, flb_stream_t stream);

/* Capacity in bytes of the static scratch array of flb_decode_fwd_static. */
size_t flb_decode_static_scratch_bytes(void);

/*
 * Raw split partials for a cross-GPU merge: runs the decode kernel on this device's keys
 * [key_begin, key_end) of every sequence (clamped to its length), cut into `num_splits` ranges
 * of the same rounding as flb_decode_fwd. The cache holds a sequence's keys from key seq_offset
 * on (0 for a whole cache; a shard's first key otherwise), and seq_lens count keys from key 0,
 * so a sequence's length in this cache is clamp(seq_lens[b] - seq_offset, 0, max_seqlen). It
 * writes
 *   partial_o  [B, H, num_splits, D] fp32  unnormalised sum_j 2^(s_j - m) v_j
 *   partial_ml [B, H, num_splits, 2] fp32  (m, l), m the log2-domain reference (-inf if empty)
 * No counterpart in the reference (single GPU); it generalises the split stage of
 * csrc/decode/decode.cu:41-202.
 */
int flb_decode_partials(const flb_decode_params* params, int32_t key_begin, int32_t key_end,
                        int32_t seq_offset, float* partial_o, float* partial_ml,
                        flb_stream_t stream);

/*
 * Fixed-order log-sum-exp merge of `num_splits` partials per (b, h) laid out as above (the
 * global split order is the index order), writing o [B, H, D] (dtype) and lse [B, H].
 * Replaces merge_kernel (csrc/decode/decode.cu:204-228).
 */
int flb_decode_merge(const float* partial_o, const float* partial_ml, int32_t batch,
                     int32_t heads, int32_t head_dim, int32_t num_splits, int32_t dtype, void* o,
                     int64_t o_batch_stride, int64_t o_head_stride, float* lse,
                     flb_stream_t stream);

/*
 * Cross-GPU decode exchange over peer memory (one process per GPU, NVLink / NVSwitch). No
 * counterpart in the reference, which is single-GPU: these replace an all-gather of the split
 * partials (flb_decode_partials + a collective + flb_decode_merge) with stores straight into
 * every rank's buffer and a bounded wait on arrival counters.
 *
 * Each rank allocates one exchange buffer with flb_peer_alloc, sends the handle to the other
 * ranks (any host channel) and maps theirs with flb_peer_open. Buffer layout, for `world` ranks,
 * B sequences, H query heads, head_dim D and S splits per rank (W*S splits in global order):
 *   [0, 256 * ceil(8 (W + 3) / 256))  uint64 words, all starting at 0: one arrival counter per
 *                                    source rank, then the CTA counts of this rank's push and
 *                                    merge in progress, then n, the steps this rank has merged
 *   then two parity regions, each partial_o [B, H, W*S, D] fp32 (256-byte aligned) followed by
 *   partial_ml [B, H, W*S, 2] fp32 (the flb_decode_partials layout).
 * Step n (counted on the device) uses parity n % 2, so a rank one step ahead never overwrites
 * partials a slower rank is still merging. Nothing on the host counts steps, so a push + merge
 * pair can be captured in a CUDA graph and replayed.
 * Failure is sticky: once the status word a push or merge is given is nonzero (a wait that timed
 * out), pushes publish nothing and merges write NaN to o and lse without waiting, on this rank
 * and, through their own timeouts, on the others, until every rank has called
 * flb_peer_exchange_reset with no step in flight and cleared its status word.
 */
size_t flb_peer_handle_bytes(void);
/* cudaMalloc + zero-fill + CUDA IPC export of `bytes` of device memory on the current device. */
int flb_peer_alloc(size_t bytes, void** ptr, void* handle);
/* Maps another process's buffer (its handle) into this process. */
int flb_peer_open(const void* handle, void** ptr);
int flb_peer_close(void* ptr);
int flb_peer_free(void* ptr);

typedef struct {
  int32_t world;                   /* ranks, 1..FLB_MAX_PEERS */
  int32_t rank;                    /* this rank */
  void* buffers[FLB_MAX_PEERS];    /* every rank's exchange buffer as mapped here ([rank] = own) */
  int64_t timeout_ns;              /* bound on the wait for the other ranks (<= 0: 2 s) */
} flb_peer_exchange;

/* Bytes of one exchange buffer for these shapes (the same on every rank). */
size_t flb_peer_exchange_bytes(int32_t world, int32_t batch, int32_t heads, int32_t head_dim,
                               int32_t splits_per_rank);

/*
 * This rank's split stage (flb_decode_partials on keys [key_begin, key_end), seq_offset, with
 * params->num_splits splits) writing its partials at global split indices
 * [rank * S, rank * S + S) of parity region n % 2 (n: this rank's step count) in EVERY rank's
 * buffer. Once all its CTAs have written, the launch adds 1, with release semantics at system
 * scope, to counter [rank] of every buffer: after n pushes every counter a rank waits on reads
 * n. params->status is the exchange's status word (see the failure rule above).
 */
int flb_decode_partials_push(const flb_decode_params* params, int32_t key_begin,
                             int32_t key_end, int32_t seq_offset,
                             const flb_peer_exchange* exchange, flb_stream_t stream);

/*
 * Step n of this rank: waits until every source counter of this rank's buffer has reached n + 1
 * (bounded by exchange->timeout_ns; on expiry it writes code 2 to `status`, and o / lse get NaN),
 * merges the W*S partials of parity region n % 2 in global split order, exactly as
 * flb_decode_merge does, and advances n.
 */
int flb_decode_merge_peers(const flb_peer_exchange* exchange, int32_t batch, int32_t heads,
                           int32_t head_dim, int32_t splits_per_rank, int32_t dtype, void* o,
                           int64_t o_batch_stride, int64_t o_head_stride, float* lse,
                           int32_t* status, flb_stream_t stream);

/* Zeroes this rank's counter block (arrivals, CTA counts, step count) on `stream`. Collective in
 * effect: every rank resets, with no push or merge of any rank in flight, before the next step. */
int flb_peer_exchange_reset(const flb_peer_exchange* exchange, flb_stream_t stream);

/*
 * Unit test of the tcgen05 building blocks the prefill kernel uses (no reference counterpart;
 * the reference's equivalent is its mma.sync fragment test, csrc/prefill/mma_tile_test.cu).
 * a [128, 128], b [128, 128] and v [128, 128] bf16 row-major, p [128, 128] bf16 row-major.
 * Writes s = a b^T (fp32, through TMA + SW128 descriptors + TMEM) and o = p v (fp32, with p
 * staged in TMEM as the A operand and v as an MN-major B operand).
 */
int flb_selftest_umma(const void* a, const void* b, const void* p, const void* v, float* s_out,
                      float* o_out, int32_t* status, flb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_LAB_B200_H_ */

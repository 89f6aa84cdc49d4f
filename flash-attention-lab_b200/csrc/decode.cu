// Split-KV decode for sm_100a: one new query token per sequence against the first seq_lens[b]
// rows of a [B, S_max, H_kv, D] cache, read in place through its strides.
//
// Reference behaviour: csrc/decode/decode.cu:41-235 of tfan2437/flash-attention-lab (split-KV
// "flash-decoding" with a fixed-order log-sum-exp merge), DecodeParams in
// csrc/common/params.h:31-53.
//
// B200 design (not a port):
//  * One CTA = (KV head, <=16 query heads of its GQA group) and a range of keys: one sequence's
//    key split (uniform launch), or an equal share of the batch's 64-key chunks that may span
//    sequences (length-balanced launch, see balanced_prefix). Every query head that shares the
//    KV head is served by the same CTA, so GQA reads each K/V byte once.
//  * A producer warp streams 64-key K and V tiles with TMA (128-byte swizzled boxes of
//    [64 keys x 64 dims]) into an mbarrier ring (3 stages, or 4 when a launch has one CTA per
//    SM); the strided cache is described by a 4-D tensor map, so any row stride (native
//    [B,S,H,D] or the HF [B,H,S,D] static-cache view) is read in place.
//  * Four consumer warps each take 16 keys of every tile. The group's query heads are the M rows
//    of a 16x8x16 warp MMA (rows beyond the group are zero), so Q K^T and P V are tiny tensor-core
//    GEMMs and the fp32 online softmax (exp2 domain) stays in registers.
//  * Partial results of the four warps, and then of the splits (or, in a balanced launch, of the
//    CTAs that hold a sequence's chunks), are merged in a fixed order, so a given configuration
//    is bitwise reproducible.
//  * seq_lens is read on the device only and clamped to [0, S_max]; keys past a sequence's length
//    get probability 0 and their V values are masked out of the product (unused cache rows may
//    hold anything, NaN included).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "host_common.h"
#include "sm100.cuh"

namespace flb {
namespace {

constexpr int kDecodeBK = 64;                       // keys per tile
constexpr int kDecodeConsumerWarps = 4;             // 16 keys of each tile per warp
constexpr int kDecodeThreads = (kDecodeConsumerWarps + 1) * 32;   // fp32 kernel: one producer
// Threads of the 16-bit kernel with kProducers producer warps (2 for small pages: a K warp and a
// V warp).
constexpr int decode_threads(int producers) { return (kDecodeConsumerWarps + producers) * 32; }
constexpr int kMaxHeadsPerCta = 16;                 // M of the warp MMA
constexpr int kMaxSplits = 256;
constexpr int kMaxDest = FLB_MAX_PEERS;             // destinations of pushed partials
constexpr int kMaxBalancedBatch = 128;              // sequences a length-balanced launch takes
constexpr int kDecodeBarBytes = 256;                // mbarriers and the abort flag
// Length-balanced launches keep the chunk prefix sums [batch + 1] and lengths [batch] here.
constexpr int kDecodeAuxBytes = ((2 * kMaxBalancedBatch + 1) * 4 + 127) / 128 * 128;

struct DecodeArgs {
  const void* q;
  void* o;
  float* lse;
  const int* seq_lens;
  // Split partials go to n_dest copies of [B, H, splits_total, D] / [B, H, splits_total, 2]
  // (one unless they are pushed to every rank of a peer exchange). When arrive[0] is set, the
  // launch adds 1 to every *arrive[i] (release, system scope) once all its partials are written;
  // cta_done counts the CTAs that have finished (the last one publishes and resets it).
  int n_dest;
  float* partial_o[kMaxDest];
  float* partial_ml[kMaxDest];
  unsigned long long* arrive[kMaxDest];
  unsigned int* cta_done;
  // Peer push: this rank's completed-step count (in its own exchange buffer) selects the parity
  // region; partials of parity 1 sit region_o / region_ml floats after those of parity 0. Null
  // outside a push (region 0 only).
  const unsigned long long* step_word;
  int64_t region_o, region_ml;
  // Paged cache: block table [B, max_blocks] (row stride bt_stride), page_size rows per block,
  // and box_rows, the rows of one TMA box (a box never crosses a page). Null for a contiguous
  // cache, whose "block" is the sequence and whose box covers a whole tile.
  const int32_t* block_tables;
  int64_t bt_stride;
  int page_size, max_blocks, box_rows;
  // 1: the K / V maps are two-half 5-D maps (16-bit, head_dim 128): one box per part of a tile.
  int halves_map;
  // Producer warps of the 16-bit kernel: 2 (one per kind) for caches of small pages, else 1.
  int producers;
  int* status;
  int64_t q_batch_stride, q_head_stride;
  int64_t o_batch_stride, o_head_stride;
  int batch, heads, heads_kv, group, head_chunks, max_seqlen;
  int num_splits;         // splits of this launch's key window
  int split_offset;       // index of this launch's first split in the partial arrays
  int splits_total;       // split dimension of the partial arrays
  int key_begin, key_end; // absolute key window of this launch
  int len_offset;         // seq_lens count keys from this key on (a shard's first key)
  int write_partials;     // 0: write o / lse (num_splits must be 1); 1: write partials
  // 1: length-balanced key ranges (balanced_prefix), 16-bit kernel of flb_decode_fwd only, over
  // bal_ctas CTAs per (KV head, head chunk) column; the cross-warp merge then has its own
  // shared-memory area of merge_rows rows per warp.
  int balanced;
  int bal_ctas;
  int merge_rows;
  float scale_log2;
  TmaCoords kc, vc;
};

// kDeep: the ring of a launch with one CTA per SM, 128 KB instead of 96 KB (measured on B200 with
// balanced launches: 4 stages of [64 x 128] K and V tiles beat 3 by 2-7 % and 6 stages).
template <int D, bool kDeep = false>
struct DecodeCfg {
  static constexpr int kTileBytes = kDecodeBK * D * 2;   // one K or V tile
  static constexpr int kBoxes = D / 64;                  // 64-wide column boxes per tile
  static constexpr int kBoxBytes = kDecodeBK * 128;
  static constexpr int kStages = kDeep ? (D == 128 ? 4 : 8) : (D == 128 ? 3 : 6);
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kMergeBytes =
      kDecodeConsumerWarps * kMaxHeadsPerCta * (D + 2) * 4;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kDataBytes = kRingBytes > kMergeBytes ? kRingBytes : kMergeBytes;
  static constexpr int kAuxOffset = kDataBytes + kDecodeBarBytes;
  static constexpr int kMergeOffset = kAuxOffset + kDecodeAuxBytes;   // balanced launches
  // Dynamic shared memory of a launch: the ring (where a uniform launch also merges its warps),
  // barriers, the balanced prefix sums, 1024 bytes of alignment slack, and for a balanced launch
  // a merge area of merge_bytes(merge_rows).
  static constexpr int kSmemBytes = kMergeOffset + 1024;
  static constexpr int merge_bytes(int rows) { return kDecodeConsumerWarps * rows * (D + 2) * 4; }
  static_assert(kMergeBytes <= kRingBytes, "a uniform launch merges its warps in the ring");
};

__device__ __forceinline__ int tma_c(const TmaCoords& c, int slot, int s, int h, int b) {
  return c.pos_s == slot ? s : (c.pos_h == slot ? h : b);
}

// The producer warp of both split kernels: streams ntiles tiles of kTileKeys keys (K then V) of
// one (sequence b, KV head) starting at key k0 into the kStages ring. A tile is kTileKeys /
// box_rows parts of box_rows rows (one page at most); a part is kColBoxes column boxes of
// kColsPerBox columns (rows of kRowBytes), stored one after the other, so the tile's layout is
// [part][column box][row in part]. Lane i issues copy i of the tile, so one warp instruction
// issues them all (at most 32). The small-page form (kSmallPageForm) may read through two-half
// maps (a.halves_map: one copy moves a whole part, both column boxes) and may load one kind
// only (kind_only 0 = K, 1 = V, for two producer warps); otherwise one warp loads K and V with
// one copy per column box. For a paged cache each box's block comes from the block table:
// the warp holds two windows of 32 entries (lane i: pages base + i and base + 32 + i), loading
// the next window one window ahead, and each lane takes its box's entry by shuffle. Keys past
// the split's end are still loaded (zeros or other blocks' rows) and masked by the consumers.
// The ring position continues from t_base tiles (earlier segments of the same CTA); returns the
// ring position after the tiles it issued.
template <int kTileKeys, int kColBoxes, int kColsPerBox, int kColBoxBytes, int kRowBytes,
          int kStages, int kTileBytes, bool kSmallPageForm = false>
__device__ __forceinline__ int produce_kv(const DecodeArgs& a, const CUtensorMap* tmk,
                                          const CUtensorMap* tmv, uint8_t* ring,
                                          uint64_t* full_bar, uint64_t* empty_bar, int k0,
                                          int ntiles, int hkv, int b, int t_base,
                                          const WaitGuard& guard, int lane, int kind_only) {
  constexpr int kStageBytes = 2 * kTileBytes;
  if (ntiles <= 0) return t_base;
  const bool paged = a.block_tables != nullptr;
  const int box_rows = paged ? a.box_rows : kTileKeys;
  const int parts = kTileKeys / box_rows;               // boxes along the keys of one tile
  const bool halves = kSmallPageForm && a.halves_map != 0;
  const int per_part = halves ? 1 : kColBoxes;          // copies per part
  if (!kSmallPageForm) kind_only = -1;
  const int kinds = kind_only < 0 ? 2 : 1;              // K and V, or only kind_only
  const int boxes = kinds * parts * per_part;           // copies of one tile by this warp (<= 32)
  // This lane's copy: kind (0 = K, 1 = V), part j along the keys, column box cb.
  const int kind = kind_only < 0 ? lane / (parts * per_part) : kind_only;
  const int j = (lane / per_part) % parts;
  const int cb = lane % per_part;
  const int part_bytes = kColBoxes * box_rows * kRowBytes;
  const CUtensorMap* map = kind == 0 ? tmk : tmv;
  const TmaCoords& crd = kind == 0 ? a.kc : a.vc;
  const int64_t bt_row = static_cast<int64_t>(b) * a.bt_stride;
  int page_base = 0, cur = -1, next = -1;
  if (paged) {
    page_base = k0 / a.page_size;
    const int p0 = page_base + lane, p1 = page_base + 32 + lane;
    cur = p0 < a.max_blocks ? __ldg(a.block_tables + bt_row + p0) : -1;
    next = p1 < a.max_blocks ? __ldg(a.block_tables + bt_row + p1) : -1;
  }
  int issued = t_base;
  for (int t = 0; t < ntiles; ++t) {
    const int r = t_base + t;   // ring position
    const int s = r % kStages;
    bool ok = true;
    if (r >= kStages) ok = mbar_wait(&empty_bar[s], ((r / kStages) - 1) & 1, guard);
    if (!__all_sync(0xffffffffu, ok)) break;
    uint8_t* dst = ring + s * kStageBytes + kind * kTileBytes;
    const int key = k0 + t * kTileKeys + j * box_rows;
    int blk = b, row = key;
    if (paged) {
      // A tile spans at most 8 pages, so its pages lie in [page_base, page_base + 64).
      if ((k0 + t * kTileKeys) / a.page_size >= page_base + 32) {
        page_base += 32;
        cur = next;
        const int p1 = page_base + 32 + lane;
        next = p1 < a.max_blocks ? __ldg(a.block_tables + bt_row + p1) : -1;
      }
      const int page = key / a.page_size;
      const int idx = page - page_base;
      const int from_cur = __shfl_sync(0xffffffffu, cur, idx & 31);
      const int from_next = __shfl_sync(0xffffffffu, next, idx & 31);
      blk = idx < 32 ? from_cur : from_next;
      row = key - page * a.page_size;
    }
    if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], kinds * kTileBytes);
    __syncwarp();
    if (lane < boxes) {
      uint8_t* box_dst = dst + j * part_bytes + cb * box_rows * kRowBytes;
      if (halves) {
        tma_load_5d(box_dst, map, &full_bar[s], 0, row, 0, tma_c(crd, 3, row, hkv, blk),
                    tma_c(crd, 4, row, hkv, blk));
      } else {
        tma_load_4d(box_dst, map, &full_bar[s], cb * kColsPerBox, tma_c(crd, 1, row, hkv, blk),
                    tma_c(crd, 2, row, hkv, blk), tma_c(crd, 3, row, hkv, blk));
      }
    }
    issued = r + 1;
  }
  return issued;
}

// The producer lane's first step, before anything it waits for: fetch both tensor maps.
__device__ __forceinline__ void prefetch_maps(const CUtensorMap* tmk, const CUtensorMap* tmv) {
  tma_prefetch_desc(tmk);
  tma_prefetch_desc(tmv);
}

// The producer's last step: do not leave the CTA while copies are still landing in shared
// memory (the last kStages of the `issued` ring positions).
template <int kStages>
__device__ __forceinline__ void drain_kv(uint64_t* full_bar, int issued, const WaitGuard& guard,
                                         int lane) {
  if (lane == 0) {
    for (int t = issued > kStages ? issued - kStages : 0; t < issued; ++t) {
      if (!mbar_wait(&full_bar[t % kStages], (t / kStages) & 1, guard)) break;
    }
  }
}

// Length-balanced partition of a launch's keys (16-bit kernel of flb_decode_fwd). Sequence b
// holds n_b = ceil(L_b / 64) chunks of 64 keys, L_b its length clamped to [0, S_max]. The
// T CTAs of one (KV head, head chunk) column share the concatenated chunk list evenly: CTA c takes chunks [floor(c N / T), floor((c + 1) N / T)), N = sum of n_b, which
// may hold the end of one sequence and the start of the next. A CTA writes one partial per
// sequence it touches, in slot h (batch + T) + b + c of query head h, so the merge of (b, h)
// reads the slots of the CTAs from the one holding b's first chunk to the one holding its last.
// With equal lengths every CTA holds one sequence's 1/num_splits, as in a uniform launch.
//
// One warp writes pref[0..batch] (exclusive prefix sums of n_b) and lens[0..batch).
__device__ __forceinline__ void balanced_prefix(const int* seq_lens, int batch, int len_offset,
                                                int max_seqlen, int* pref, int* lens, int lane) {
  constexpr int kPerLane = kMaxBalancedBatch / 32;
  int n[kPerLane];
  int sum = 0;
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) {
    const int b = lane * kPerLane + j;
    int len = 0;
    if (b < batch) {
      len = min(max(seq_lens[b] - len_offset, 0), max_seqlen);
      lens[b] = len;
    }
    n[j] = (len + kDecodeBK - 1) / kDecodeBK;
    sum += n[j];
  }
  int incl = sum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  int run = incl - sum;
#pragma unroll
  for (int j = 0; j < kPerLane; ++j) {
    const int b = lane * kPerLane + j;
    if (b < batch) pref[b] = run;
    run += n[j];
  }
  if (lane == 31) pref[batch] = incl;
}

// The sequence that holds chunk x (x < N): the largest b < batch with pref[b] <= x (sequences
// without chunks share their start with the next one). For x >= N, batch - 1.
__device__ __forceinline__ int sequence_of_chunk(const int* pref, int batch, int64_t x) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pref[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// g(c) = floor(c N / T) for consecutive c without a division per step: start() divides once,
// step() moves to c + 1 and returns g(c + 1).
struct ChunkWalk {
  int64_t g, r, q_step, r_step, total;
  __device__ __forceinline__ void start(int c, int64_t n, int t) {
    total = t;
    const int64_t cn = static_cast<int64_t>(c) * n;
    g = cn / t;
    r = cn - g * t;
    q_step = n / t;
    r_step = n - q_step * t;
  }
  __device__ __forceinline__ int64_t step() {
    g += q_step;
    r += r_step;
    if (r >= total) {
      r -= total;
      ++g;
    }
    return g;
  }
};

// True on every one of the 128 consumer threads when pred holds on any of them (named barrier
// 1 with an OR reduction), so that all of them take the same branch after it.
__device__ __forceinline__ bool consumers_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(kDecodeConsumerWarps * 32)
      : "memory");
  return r != 0;
}

// Publishes a push once per launch (called by one thread per CTA after the CTA's partial stores,
// which a CTA barrier orders before it): each CTA fences at GPU scope and counts itself; the last
// CTA to finish, having observed every count, fences at system scope and adds one arrival
// (release, system scope) to every destination's counter, which makes all the launch's stores,
// local or over NVLink, visible to a rank that acquires the counter. It then resets the count
// for the next launch (launches on one stream do not overlap). A contended system-scope atomic
// per CTA cost tens of microseconds, a system-scope fence per CTA about ten.
// A push whose status word is already nonzero (an earlier step's wait timed out, or one of this
// launch's own pipeline waits) publishes nothing: the other ranks' merges then time out too, so
// every rank's exchange ends in the failed state instead of one of them merging stale partials.
__device__ __forceinline__ bool push_failed(const DecodeArgs& a) {
  return a.status != nullptr && *reinterpret_cast<volatile const int*>(a.status) != 0;
}

__device__ __forceinline__ void publish_push(const DecodeArgs& a) {
  __threadfence();
  const unsigned int total = gridDim.x * gridDim.y;
  if (atomicAdd(a.cta_done, 1u) == total - 1) {
    // One system-scope fence orders every CTA's partials before all the adds that follow
    // (a release add per destination would fence once per destination).
    __threadfence_system();
    *a.cta_done = 0u;
    if (!push_failed(a)) {
      for (int dst = 0; dst < a.n_dest; ++dst) red_relaxed_sys_add(a.arrive[dst], 1ull);
    }
  }
}

// One output element in the output dtype (round to nearest even for the 16-bit types).
template <typename T>
__device__ __forceinline__ void store_out(T* p, float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    *p = __float2bfloat16_rn(v);
  } else if constexpr (std::is_same<T, __half>::value) {
    *p = __float2half_rn(v);
  } else {
    *p = v;
  }
}

// The end of a split CTA's segment, shared by the 16-bit and the fp32 kernels: the consumer
// warps have left their per-warp (m, l, O) in shared memory (wm, wl [warps][mrows],
// wo [warps][mrows][D]). Merges the warps in a fixed order and writes either o / lse (one split)
// or the segment's partials to every destination (query head h in slot seg_slot + h h_stride),
// then publishes a push. Called by the 128 consumer threads.
template <typename T, int D>
__device__ __forceinline__ void finish_split(const DecodeArgs& a, const float* wm, const float* wl,
                                             const float* wo, int heads_here, int head0, int b,
                                             int64_t seg_slot, int64_t h_stride, int mrows) {
  const int tid = threadIdx.x;
  // A push writes the parity region of this rank's step count, and nothing once the exchange
  // has failed.
  int64_t off_o = 0, off_ml = 0;
  bool skip = false;
  if (a.step_word != nullptr) {
    if (*reinterpret_cast<volatile const unsigned long long*>(a.step_word) & 1ull) {
      off_o = a.region_o;
      off_ml = a.region_ml;
    }
    skip = push_failed(a);
  }
  for (int idx = skip ? heads_here * D : tid; idx < heads_here * D;
       idx += kDecodeConsumerWarps * 32) {
    const int row = idx / D;
    const int d = idx - row * D;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeConsumerWarps; ++w) m = fmaxf(m, wm[w * mrows + row]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeConsumerWarps; ++w) {
      const float mw = wm[w * mrows + row];
      if (mw != -INFINITY) {
        const float f = ex2(mw - m);
        num += wo[(w * mrows + row) * D + d] * f;
        den += wl[w * mrows + row] * f;
      }
    }
    const int h = head0 + row;
    if (!a.write_partials) {
      T* o = static_cast<T*>(a.o) + static_cast<int64_t>(b) * a.o_batch_stride +
             static_cast<int64_t>(h) * a.o_head_stride;
      store_out<T>(o + d, den > 0.f ? num / den : 0.f);
      if (d == 0) {
        a.lse[static_cast<int64_t>(b) * a.heads + h] =
            den > 0.f ? m * 0.69314718055994530942f + logf(den) : -INFINITY;
      }
    } else {
      const int64_t slot = seg_slot + h * h_stride;
      for (int dst = 0; dst < a.n_dest; ++dst) {
        a.partial_o[dst][off_o + slot * D + d] = num;
        if (d == 0) {
          a.partial_ml[dst][off_ml + 2 * slot] = m;
          a.partial_ml[dst][off_ml + 2 * slot + 1] = den;
        }
      }
    }
  }
  if (a.write_partials && a.arrive[0] != nullptr) {
    asm volatile("bar.sync 1, %0;" ::"n"(kDecodeConsumerWarps * 32) : "memory");
    if (tid == 0) publish_push(a);
  }
}


template <typename T, int D, bool kDeep, int kProducers>
__global__ void __launch_bounds__(decode_threads(kProducers), kProducers == 2 ? 2 : 0)
    decode_split_kernel(const __grid_constant__ DecodeArgs a,
                        const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv) {
  // The merge kernel, launched as a programmatic dependent, may be scheduled once every CTA of
  // this grid has started; it waits (griddepcontrol.wait) for this grid to finish and flush.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  using Cfg = DecodeCfg<D, kDeep>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kKSteps = D / 16;   // MMA k-steps over head_dim
  constexpr int kNTiles = D / 8;    // MMA n-tiles over head_dim in P V

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);
  uint64_t* empty_bar = full_bar + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty_bar + kStages);
  int* pref = reinterpret_cast<int*>(smem + Cfg::kAuxOffset);   // [batch + 1], balanced only
  int* lens = pref + kMaxBalancedBatch + 1;                       // [batch], balanced only

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == kDecodeConsumerWarps && lane == 0) prefetch_maps(&tmk, &tmv);

  // Work item. Uniform: blockIdx.x = split within this launch, blockIdx.y = (b, hkv, head
  // chunk). Balanced: blockIdx.x = the CTA's place c in its column, blockIdx.y = (hkv, chunk).
  const int split = a.balanced ? 0 : blockIdx.x;
  const int chunk = blockIdx.y % a.head_chunks;
  const int bk = blockIdx.y / a.head_chunks;
  const int hkv = a.balanced ? bk : bk % a.heads_kv;
  const int b = a.balanced ? 0 : bk / a.heads_kv;
  const int head0 = hkv * a.group + chunk * kMaxHeadsPerCta;
  const int heads_here = min(kMaxHeadsPerCta, a.group - chunk * kMaxHeadsPerCta);

  // Uniform launch: this split's key range, the window clamped to the sequence length and cut
  // into num_splits ranges that are whole numbers of tiles (the last one shorter).
  int k0u = 0, k1u = 0;
  if (!a.balanced) {
    int len = a.seq_lens[b] - a.len_offset;
    len = min(max(len, 0), a.max_seqlen);
    const int lo = max(a.key_begin, 0);
    const int hi = min(a.key_end, len);
    const int n = hi - lo;
    if (n > 0) {
      const int per = (n + a.num_splits - 1) / a.num_splits;
      const int per_split = (per + kDecodeBK - 1) / kDecodeBK * kDecodeBK;
      k0u = lo + split * per_split;
      k1u = min(hi, k0u + per_split);
    }
  }

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], kProducers);
      mbar_init(&empty_bar[s], kDecodeConsumerWarps);
    }
    fence_barrier_init();
  }
  if (a.balanced && warp == kDecodeConsumerWarps)
    balanced_prefix(a.seq_lens, a.batch, a.len_offset, a.max_seqlen, pref, lens, lane);
  __syncthreads();
  const WaitGuard guard{abort_flag, a.status};

  // Segments of this CTA: one per sequence it touches, sequences [sb_begin, sb_end) at most.
  // Uniform: sequence b only (its split may be empty and still writes its partial).
  const int total = a.bal_ctas;                  // CTAs per column (balanced)
  const int c = static_cast<int>(blockIdx.x);    // this CTA's place in its column (balanced)
  int64_t g0 = 0, g1 = 0;
  int sb_begin = b, sb_end = b + 1;
  if (a.balanced) {
    const int64_t n = pref[a.batch];
    g0 = static_cast<int64_t>(c) * n / total;
    g1 = static_cast<int64_t>(c + 1) * n / total;
    sb_begin = sequence_of_chunk(pref, a.batch, g0);
    sb_end = a.batch;
  }
  // Key range [k0, k1) of this CTA's part of sequence sb: 1 = run it, 0 = nothing of sb here,
  // -1 = no later sequence either.
  auto segment = [&](int sb, int& k0, int& k1) -> int {
    if (!a.balanced) {
      k0 = k0u;
      k1 = k1u;
      return 1;
    }
    if (pref[sb] >= g1) return -1;
    const int64_t lo = max(g0, static_cast<int64_t>(pref[sb]));
    const int64_t hi = min(g1, static_cast<int64_t>(pref[sb + 1]));
    if (lo >= hi) return 0;
    k0 = static_cast<int>(lo - pref[sb]) * kDecodeBK;
    k1 = min(static_cast<int>(hi - pref[sb]) * kDecodeBK, lens[sb]);
    return 1;
  };

  if (warp >= kDecodeConsumerWarps) {
    // ---------------- producer warps ----------------
    // One warp loads K and V; with small pages two warps, one per kind, halve the copies each
    // issues per tile (the copy issue rate bounds small pages). Both then arrive on each full
    // barrier with their own bytes and both wait on each empty one.
    const int kind = kProducers == 2 ? warp - kDecodeConsumerWarps : -1;
    int issued = 0;
    for (int sb = sb_begin; sb < sb_end; ++sb) {
      int k0 = 0, k1 = 0;
      const int st = segment(sb, k0, k1);
      if (st < 0) break;
      if (st == 0) continue;
      const int nt = k1 > k0 ? (k1 - k0 + kDecodeBK - 1) / kDecodeBK : 0;
      issued = produce_kv<kDecodeBK, Cfg::kBoxes, 64, Cfg::kBoxBytes, 128, kStages,
                          Cfg::kTileBytes, kProducers == 2>(a, &tmk, &tmv, smem, full_bar,
                                                            empty_bar, k0, nt, hkv,
                                           sb, issued, guard, lane, kind);
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
    }
    drain_kv<kStages>(full_bar, issued, guard, lane);
    return;
  }

  // ---------------- consumer warps ----------------
  const int g = lane >> 2;   // fragment row group
  const int t4 = lane & 3;   // thread in quad
  const uint32_t smem_base = smem_u32(smem);
  // ldmatrix row addresses (lane-dependent parts). A tile is [part][column box][row in part]
  // (produce_kv); within a column box, rows are 128 bytes with the 16-byte chunks swizzled by
  // the row's low 3 bits (sw128_offset; parts are multiples of 8 rows). Launches without small
  // pages have one part per tile, whose column boxes are then compile-time kBoxBytes apart.
  const uint32_t k_row = static_cast<uint32_t>(warp * 16 + (lane >> 4) * 8 + (lane & 7));
  const uint32_t k_chunk_lo = static_cast<uint32_t>((lane >> 3) & 1);
  const uint32_t v_row = static_cast<uint32_t>(warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7));
  const uint32_t v_chunk_lo = static_cast<uint32_t>(lane >> 4);
  const uint32_t part_rows = kProducers == 2 ? static_cast<uint32_t>(a.box_rows) : kDecodeBK;
  const uint32_t colbox_bytes = part_rows * 128u;          // one column box of one part
  auto row_base = [&](uint32_t r) {                         // row r's line in column box 0
    return (r / part_rows) * (Cfg::kBoxes * colbox_bytes) + (r % part_rows) * 128u;
  };
  const uint32_t k_line = row_base(k_row), v_line = row_base(v_row);
  // Cross-warp merge area: the ring once a uniform launch has consumed it; its own area in a
  // balanced launch, whose producer is already loading the next segment.
  const int mrows = a.merge_rows;
  float* wm = reinterpret_cast<float*>(smem + (a.balanced ? Cfg::kMergeOffset : 0));  // [warps][mrows]
  float* wl = wm + kDecodeConsumerWarps * mrows;                                      // [warps][mrows]
  float* wo = wl + kDecodeConsumerWarps * mrows;                                      // [warps][mrows][D]

  int t_base = 0;   // ring position of the segment's first tile
  for (int sb = sb_begin; sb < sb_end; ++sb) {
    int k0 = 0, k1 = 0;
    const int st = segment(sb, k0, k1);
    if (st < 0) break;
    if (st == 0) continue;
    const int ntiles = k1 > k0 ? (k1 - k0 + kDecodeBK - 1) / kDecodeBK : 0;

    // Q as the A operand: rows = query heads of the group (zero beyond heads_here).
    uint32_t qa[kKSteps][4];
    {
      const T* qb = static_cast<const T*>(a.q) + static_cast<int64_t>(sb) * a.q_batch_stride;
      const bool r0 = g < heads_here, r1 = g + 8 < heads_here;
      const T* q0 = qb + static_cast<int64_t>(head0 + g) * a.q_head_stride;
      const T* q1 = qb + static_cast<int64_t>(head0 + g + 8) * a.q_head_stride;
#pragma unroll
      for (int kk = 0; kk < kKSteps; ++kk) {
        const int col = kk * 16 + 2 * t4;
        qa[kk][0] = r0 ? *reinterpret_cast<const uint32_t*>(q0 + col) : 0u;
        qa[kk][1] = r1 ? *reinterpret_cast<const uint32_t*>(q1 + col) : 0u;
        qa[kk][2] = r0 ? *reinterpret_cast<const uint32_t*>(q0 + col + 8) : 0u;
        qa[kk][3] = r1 ? *reinterpret_cast<const uint32_t*>(q1 + col + 8) : 0u;
      }
    }

    float o_acc[kNTiles][4];
#pragma unroll
    for (int j = 0; j < kNTiles; ++j) o_acc[j][0] = o_acc[j][1] = o_acc[j][2] = o_acc[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY};  // log2-domain running max, rows g and g + 8
    float l_run[2] = {0.f, 0.f};              // this thread's share of the row sums

    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int r = t_base + t;
      const int s = r % kStages;
      if (!mbar_wait(&full_bar[s], (r / kStages) & 1, guard)) {
        ok = false;
        break;
      }
      const uint32_t kbase = smem_base + s * Cfg::kStageBytes;
      const uint32_t vbase = kbase + Cfg::kTileBytes;
      const int key_w = k0 + t * kDecodeBK + warp * 16;   // first key of this warp's slice
      const int valid = k1 - key_w;                       // keys of the slice before the end

      // S = Q K^T over this warp's 16 keys (two n-tiles of 8 keys).
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < kKSteps; ++kk) {
        const uint32_t ch = 2 * kk + k_chunk_lo;
        const uint32_t addr =
            kbase + k_line + (ch >> 3) * colbox_bytes + (((ch & 7) ^ (k_row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma_16816<T>(sc[0], qa[kk], b0, b1);
        mma_16816<T>(sc[1], qa[kk], b2, b3);
      }

      // Online softmax in the exp2 domain; keys at or past k1 are hidden.
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = nt * 8 + 2 * t4 + (e & 1);
          const float v = key < valid ? sc[nt][e] * a.scale_log2 : -INFINITY;
          sc[nt][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      }
      float ref[2], resc[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
        const float m_new = fmaxf(m_run[rr], mx[rr]);
        ref[rr] = m_new == -INFINITY ? 0.f : m_new;
        resc[rr] = ex2(m_run[rr] - ref[rr]);
        m_run[rr] = m_new;
      }
      float p[2][4];
      float psum[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          p[nt][e] = ex2(sc[nt][e] - ref[e >> 1]);
          psum[e >> 1] += p[nt][e];
        }
      }
      l_run[0] = l_run[0] * resc[0] + psum[0];
      l_run[1] = l_run[1] * resc[1] + psum[1];
#pragma unroll
      for (int j = 0; j < kNTiles; ++j) {
        o_acc[j][0] *= resc[0];
        o_acc[j][1] *= resc[0];
        o_acc[j][2] *= resc[1];
        o_acc[j][3] *= resc[1];
      }
      uint32_t pa[4];
      pa[0] = pack2<T>(p[0][0], p[0][1]);
      pa[1] = pack2<T>(p[0][2], p[0][3]);
      pa[2] = pack2<T>(p[1][0], p[1][1]);
      pa[3] = pack2<T>(p[1][2], p[1][3]);

      // V rows of hidden keys are masked to zero in the B fragments (0 * NaN would poison O).
      // Fragment keys: regs 0/2 hold keys 2*t4 + {0,1}, regs 1/3 keys 8 + 2*t4 + {0,1}.
      uint32_t vmask_lo = 0xffffffffu, vmask_hi = 0xffffffffu;
      if (valid < 16) {
        const int kl = 2 * t4, kh = 8 + 2 * t4;
        vmask_lo = (kl < valid ? 0x0000ffffu : 0u) | (kl + 1 < valid ? 0xffff0000u : 0u);
        vmask_hi = (kh < valid ? 0x0000ffffu : 0u) | (kh + 1 < valid ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int jp = 0; jp < kNTiles / 2; ++jp) {
        const uint32_t ch = 2 * jp + v_chunk_lo;
        const uint32_t addr =
            vbase + v_line + (ch >> 3) * colbox_bytes + (((ch & 7) ^ (v_row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(addr, b0, b1, b2, b3);
        mma_16816<T>(o_acc[2 * jp], pa, b0 & vmask_lo, b1 & vmask_hi);
        mma_16816<T>(o_acc[2 * jp + 1], pa, b2 & vmask_lo, b3 & vmask_hi);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }
    t_base += ntiles;

    // Full row sums of this warp.
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 1);
      l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 2);
    }

    // Every consumer thread is past this segment's tiles and past the previous segment's merge
    // reads; all of them take the same branch.
    if (consumers_any(!ok || *abort_flag != 0)) {
      // A CTA that gave up still counts itself in a push, so the counters stay consistent for
      // the next step; the status word already tells the host this step's outputs are invalid.
      if (a.write_partials && a.arrive[0] != nullptr && threadIdx.x == 0) publish_push(a);
      return;
    }
    if (t4 == 0) {
      if (g < heads_here) {
        wm[warp * mrows + g] = m_run[0];
        wl[warp * mrows + g] = l_run[0];
      }
      if (g + 8 < heads_here) {
        wm[warp * mrows + g + 8] = m_run[1];
        wl[warp * mrows + g + 8] = l_run[1];
      }
    }
#pragma unroll
    for (int j = 0; j < kNTiles; ++j) {
      const int col = j * 8 + 2 * t4;
      if (g < heads_here) {
        float* r0 = wo + (warp * mrows + g) * D + col;
        r0[0] = o_acc[j][0];
        r0[1] = o_acc[j][1];
      }
      if (g + 8 < heads_here) {
        float* r1 = wo + (warp * mrows + g + 8) * D + col;
        r1[0] = o_acc[j][2];
        r1[1] = o_acc[j][3];
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kDecodeConsumerWarps * 32) : "memory");

    const int64_t seg_slot =
        a.balanced ? static_cast<int64_t>(sb) + c
                   : static_cast<int64_t>(b) * a.heads * a.splits_total + a.split_offset + split;
    const int64_t h_stride = a.balanced ? a.batch + total : a.splits_total;
    finish_split<T, D>(a, wm, wl, wo, heads_here, head0, sb, seg_slot, h_stride, mrows);
  }
}

// ---------------------------------------------------------------------------------------------
// fp32 caches (the reference's fp32 decode): the same CTA layout and TMA producer, with fp32
// tiles of 32 keys and the dot products on the FMA pipe (fp32 end to end, no tensor cores).
// Each half-warp takes one key at a time: lane l owns dims {64 i + 4 (l % 16) .. + 3}, so a
// quarter-warp reads 128 contiguous bytes of a row; a dot product is reduced over the half-warp
// with four shuffles. kHeads (1, 2, 4 or 8) query heads of the GQA group share each K/V read.
// ---------------------------------------------------------------------------------------------
constexpr int kF32BK = 32;            // keys per fp32 tile
constexpr int kF32MaxHeads = 8;       // query heads per fp32 CTA

template <int D>
struct DecodeF32Cfg {
  static constexpr int kTileBytes = kF32BK * D * 4;    // one K or V tile: 16 KB at D = 128
  static constexpr int kStages = D == 128 ? 3 : 6;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kMergeBytes = kDecodeConsumerWarps * kMaxHeadsPerCta * (D + 2) * 4;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kDataBytes = kRingBytes > kMergeBytes ? kRingBytes : kMergeBytes;
  static constexpr int kSmemBytes = kDataBytes + 1024 + 256;
};

template <int D, int kHeads>
__global__ void __launch_bounds__(kDecodeThreads, 2)
    decode_split_f32_kernel(const __grid_constant__ DecodeArgs a,
                            const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  using Cfg = DecodeF32Cfg<D>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kDL = D / 16;       // dims per lane
  constexpr int kV4 = kDL / 4;      // float4 loads per row per lane

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kDataBytes);
  uint64_t* empty_bar = full_bar + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty_bar + kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == kDecodeConsumerWarps && lane == 0) prefetch_maps(&tmk, &tmv);

  const int split = blockIdx.x;
  const int chunk = blockIdx.y % a.head_chunks;
  const int bk = blockIdx.y / a.head_chunks;
  const int hkv = bk % a.heads_kv;
  const int b = bk / a.heads_kv;
  const int head0 = hkv * a.group + chunk * kF32MaxHeads;
  const int heads_here = min(kF32MaxHeads, a.group - chunk * kF32MaxHeads);

  int len = a.seq_lens[b] - a.len_offset;
  len = min(max(len, 0), a.max_seqlen);
  const int lo = max(a.key_begin, 0);
  const int hi = min(a.key_end, len);
  const int n = hi - lo;
  int k0 = 0, k1 = 0;
  if (n > 0) {
    const int per = (n + a.num_splits - 1) / a.num_splits;
    const int per_split = (per + kDecodeBK - 1) / kDecodeBK * kDecodeBK;
    k0 = lo + split * per_split;
    k1 = min(hi, k0 + per_split);
  }
  const int ntiles = k1 > k0 ? (k1 - k0 + kF32BK - 1) / kF32BK : 0;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kDecodeConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const WaitGuard guard{abort_flag, a.status};

  if (warp == kDecodeConsumerWarps) {
    // ---------------- producer warp: [32 keys x D] fp32 tiles ----------------
    const int issued = produce_kv<kF32BK, 1, D, Cfg::kTileBytes, D * 4, kStages, Cfg::kTileBytes>(
        a, &tmk, &tmv, smem, full_bar, empty_bar, k0, ntiles, hkv, b, 0, guard, lane, -1);
    drain_kv<kStages>(full_bar, issued, guard, lane);
    return;
  }

  // ---------------- consumer warps: 8 keys of every tile, 4 per half-warp ----------------
  const int half = lane >> 4;
  const int hl = lane & 15;
  float q[kHeads][kDL];
  {
    const float* qb = static_cast<const float*>(a.q) + static_cast<int64_t>(b) * a.q_batch_stride;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      const float* qh = qb + static_cast<int64_t>(head0 + h) * a.q_head_stride;
#pragma unroll
      for (int i = 0; i < kV4; ++i) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (h < heads_here) v = *reinterpret_cast<const float4*>(qh + i * 64 + hl * 4);
        q[h][4 * i + 0] = v.x * a.scale_log2;
        q[h][4 * i + 1] = v.y * a.scale_log2;
        q[h][4 * i + 2] = v.z * a.scale_log2;
        q[h][4 * i + 3] = v.w * a.scale_log2;
      }
    }
  }
  float o[kHeads][kDL];
  float m_run[kHeads], l_run[kHeads];
#pragma unroll
  for (int h = 0; h < kHeads; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int i = 0; i < kDL; ++i) o[h][i] = 0.f;
  }

  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages;
    if (!mbar_wait(&full_bar[s], (t / kStages) & 1, guard)) {
      ok = false;
      break;
    }
    const float* kt = reinterpret_cast<const float*>(smem + s * Cfg::kStageBytes);
    const float* vt = kt + kF32BK * D;
    const int row0 = warp * 8 + half * 4;              // this half's first key in the tile
    const int valid = k1 - (k0 + t * kF32BK + row0);   // its keys before the split's end

    float sc[4][kHeads];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      float kv[kDL];
      const float* krow = kt + (row0 + kk) * D + hl * 4;
#pragma unroll
      for (int i = 0; i < kV4; ++i) {
        const float4 v = *reinterpret_cast<const float4*>(krow + i * 64);
        kv[4 * i + 0] = v.x;
        kv[4 * i + 1] = v.y;
        kv[4 * i + 2] = v.z;
        kv[4 * i + 3] = v.w;
      }
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kDL; ++i) dot = fmaf(q[h][i], kv[i], dot);
        dot += __shfl_xor_sync(0xffffffffu, dot, 8);
        dot += __shfl_xor_sync(0xffffffffu, dot, 4);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        sc[kk][h] = kk < valid ? dot : -INFINITY;
      }
    }
    // Online softmax over the warp's 8 keys (exp2 domain; q carries the scale).
    float ref[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      float mt = fmaxf(fmaxf(sc[0][h], sc[1][h]), fmaxf(sc[2][h], sc[3][h]));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float m_new = fmaxf(m_run[h], mt);
      ref[h] = m_new == -INFINITY ? 0.f : m_new;
      const float resc = ex2(m_run[h] - ref[h]);
      m_run[h] = m_new;
      l_run[h] *= resc;
#pragma unroll
      for (int i = 0; i < kDL; ++i) o[h][i] *= resc;
    }
    // O += P V over this half's valid keys (V rows of hidden keys are never read: 0 * NaN).
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (kk < valid) {
        float vv[kDL];
        const float* vrow = vt + (row0 + kk) * D + hl * 4;
#pragma unroll
        for (int i = 0; i < kV4; ++i) {
          const float4 v = *reinterpret_cast<const float4*>(vrow + i * 64);
          vv[4 * i + 0] = v.x;
          vv[4 * i + 1] = v.y;
          vv[4 * i + 2] = v.z;
          vv[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          const float p = ex2(sc[kk][h] - ref[h]);
          l_run[h] += p;
#pragma unroll
          for (int i = 0; i < kDL; ++i) o[h][i] = fmaf(p, vv[i], o[h][i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }

  // The two halves saw different keys with the same reference point: add them up.
#pragma unroll
  for (int h = 0; h < kHeads; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 16);
#pragma unroll
    for (int i = 0; i < kDL; ++i) o[h][i] += __shfl_xor_sync(0xffffffffu, o[h][i], 16);
  }

  if (consumers_any(!ok || *abort_flag != 0)) {
    if (a.write_partials && a.arrive[0] != nullptr && threadIdx.x == 0) publish_push(a);
    return;
  }
  float* wm = reinterpret_cast<float*>(smem);                         // [warps][16]
  float* wl = wm + kDecodeConsumerWarps * kMaxHeadsPerCta;            // [warps][16]
  float* wo = wl + kDecodeConsumerWarps * kMaxHeadsPerCta;            // [warps][16][D]
  if (half == 0) {
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      if (hl == 0) {
        wm[warp * kMaxHeadsPerCta + h] = m_run[h];
        wl[warp * kMaxHeadsPerCta + h] = l_run[h];
      }
      float* row = wo + (warp * kMaxHeadsPerCta + h) * D + hl * 4;
#pragma unroll
      for (int i = 0; i < kV4; ++i) {
        *reinterpret_cast<float4*>(row + i * 64) =
            make_float4(o[h][4 * i], o[h][4 * i + 1], o[h][4 * i + 2], o[h][4 * i + 3]);
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kDecodeConsumerWarps * 32) : "memory");

  finish_split<float, D>(a, wm, wl, wo, heads_here, head0, b,
                         static_cast<int64_t>(b) * a.heads * a.splits_total + a.split_offset +
                             split,
                         a.splits_total, kMaxHeadsPerCta);
}

// A peer merge's view of this rank's exchange buffer (null counters = a plain merge): the
// arrival counters of every source rank, this rank's completed-step count n and the CTA count of
// the merge in progress. Step n merges parity region n % 2 (partials region_o / region_ml floats
// past those of region 0 when it is 1) once every counter has reached n + 1; the last CTA to
// finish then advances n. Both live in device memory, so a captured CUDA graph replays steps.
struct PeerWait {
  const unsigned long long* counters;
  unsigned long long* step_word;
  unsigned int* merge_done;
  int world;
  int64_t region_o, region_ml;
  int64_t timeout_ns;
  int* status;
};

// Fixed-order merge of the split partials of one (b, h): thread d owns output column d.
// m = max_s m_s; l = sum_s l_s 2^(m_s - m); o = sum_s o_s 2^(m_s - m) / l (empty splits skipped).
// kPeers: the partials are written by other GPUs; thread 0 first waits (bounded) for every
// source's arrival counter, and the partials are read through L2 (ld.global.cg). A wait that
// times out, or an exchange whose status word is already nonzero, writes NaN to o and lse (the
// exchange stays failed until the ranks reset it together).
template <typename T, bool kPeers>
__global__ void decode_merge_kernel(const float* __restrict__ partial_o,
                                    const float* __restrict__ partial_ml, int heads, int head_dim,
                                    int num_splits, T* o, int64_t o_batch_stride,
                                    int64_t o_head_stride, float* lse, PeerWait wait) {
  // Launched as a programmatic dependent of the split kernel: wait for its writes first (a no-op
  // when launched normally).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int bh = blockIdx.x;
  const int b = bh / heads;
  const int h = bh - b * heads;
  if constexpr (kPeers) {
    __shared__ int s_failed;
    __shared__ unsigned long long s_step;
    if (threadIdx.x == 0) {
      int failed = wait.status != nullptr && *reinterpret_cast<volatile int*>(wait.status) != 0;
      const unsigned long long n =
          *reinterpret_cast<volatile const unsigned long long*>(wait.step_word);
      const uint64_t start = global_timer_ns();
      for (int src = 0; src < wait.world && !failed; ++src) {
        uint32_t polls = 0;
        while (ld_relaxed_sys_u64(wait.counters + src) < n + 1) {
          if (((++polls) & 63u) == 0 &&
              global_timer_ns() - start > static_cast<uint64_t>(wait.timeout_ns)) {
            failed = 1;
            if (wait.status != nullptr) atomicCAS(wait.status, 0, kDevPeerTimeout);
            break;
          }
        }
      }
      fence_acq_rel_sys();   // the partials the counters announce are visible from here on
      s_failed = failed;
      s_step = n;
    }
    __syncthreads();
    const unsigned long long n = s_step;
    if (n & 1ull) {
      partial_o += wait.region_o;
      partial_ml += wait.region_ml;
    }
    if (s_failed) {
      T* out = o + static_cast<int64_t>(b) * o_batch_stride + static_cast<int64_t>(h) * o_head_stride;
      for (int d = threadIdx.x; d < head_dim; d += blockDim.x) store_out<T>(out + d, NAN);
      if (threadIdx.x == 0) lse[bh] = NAN;
    }
    // Every CTA has read n before the last one to count itself advances it.
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(wait.merge_done, 1u) == gridDim.x - 1) {
        *wait.merge_done = 0u;
        *wait.step_word = n + 1;
      }
    }
    if (s_failed) return;
  }
  auto load = [](const float* p) { return kPeers ? __ldcg(p) : *p; };
  const int64_t base = static_cast<int64_t>(bh) * num_splits;
  // Partials are read kMergeBatch at a time, a batch's loads issued before any is used, and
  // combined in split order.
  constexpr int kMergeBatch = 8;
  float m = -INFINITY;
  for (int s0 = 0; s0 < num_splits; s0 += kMergeBatch) {
    float mv[kMergeBatch];
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i)
      mv[i] = s0 + i < num_splits ? load(partial_ml + 2 * (base + s0 + i)) : -INFINITY;
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) m = fmaxf(m, mv[i]);
  }
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s0 = 0; s0 < num_splits; s0 += kMergeBatch) {
      float ms[kMergeBatch], ls[kMergeBatch], os[kMergeBatch];
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        const int64_t sl = base + s0 + i;
        const bool in = s0 + i < num_splits;
        ms[i] = in ? load(partial_ml + 2 * sl) : -INFINITY;
        ls[i] = in ? load(partial_ml + 2 * sl + 1) : 0.f;
        os[i] = in ? load(partial_o + sl * head_dim + d) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        if (ms[i] != -INFINITY) {
          const float f = ex2(ms[i] - m);
          num += os[i] * f;
          den += ls[i] * f;
        }
      }
    }
    T* out = o + static_cast<int64_t>(b) * o_batch_stride + static_cast<int64_t>(h) * o_head_stride;
    store_out<T>(out + d, den > 0.f ? num / den : 0.f);
    if (d == 0) lse[bh] = den > 0.f ? m * 0.69314718055994530942f + logf(den) : -INFINITY;
  }
}

// Merge of a length-balanced launch (balanced_prefix): the same fixed-order log-sum-exp merge as
// decode_merge_kernel, over the slots of the CTAs that hold a chunk of sequence b, in CTA order.
// The prefix sums are rebuilt from seq_lens before waiting for the split kernel.
template <typename T>
__global__ void decode_merge_balanced_kernel(const float* __restrict__ partial_o,
                                             const float* __restrict__ partial_ml,
                                             const int* __restrict__ seq_lens, int batch,
                                             int heads, int head_dim, int total,
                                             int max_seqlen, T* o, int64_t o_batch_stride,
                                             int64_t o_head_stride, float* lse) {
  __shared__ int pref[kMaxBalancedBatch + 1];
  __shared__ int lens[kMaxBalancedBatch];
  if (threadIdx.x < 32) balanced_prefix(seq_lens, batch, 0, max_seqlen, pref, lens, threadIdx.x);
  __syncthreads();
  // Everything that depends on the lengths only is done before waiting for the split kernel.
  const int bh = blockIdx.x;
  const int b = bh / heads;
  const int h = bh - b * heads;
  const int64_t n = pref[batch];
  const int64_t p0 = pref[b], p1 = pref[b + 1];
  // CTAs holding chunks p0 and p1 - 1: CTA c holds chunk x when c = floor(((x + 1) T - 1) / N).
  int c_first = 0, c_last = -1;
  ChunkWalk walk0{};
  if (p1 > p0) {
    c_first = static_cast<int>(((p0 + 1) * total - 1) / n);
    c_last = static_cast<int>((p1 * total - 1) / n);
    walk0.start(c_first, n, total);
  }
  const int64_t base = static_cast<int64_t>(h) * (batch + total) + b;   // + c: CTA c's slot
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // CTA c (chunks [g(c), g(c + 1))) holds part of sequence b when that range meets [p0, p1).
  // The holders' partials are read kMergeBatch at a time, all loads of a batch issued before
  // any is used (each is an L2 round trip), and combined in CTA order as before.
  constexpr int kMergeBatch = 8;
  float m = -INFINITY;
  {
    ChunkWalk w = walk0;
    for (int c0 = c_first; c0 <= c_last; c0 += kMergeBatch) {
      float mv[kMergeBatch];
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        const int c = c0 + i;
        mv[i] = -INFINITY;
        if (c <= c_last) {
          const int64_t g0 = w.g;
          const int64_t g1 = w.step();
          if (max(g0, p0) < min(g1, p1)) mv[i] = partial_ml[2 * (base + c)];
        }
      }
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) m = fmaxf(m, mv[i]);
    }
  }
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    ChunkWalk w = walk0;
    for (int c0 = c_first; c0 <= c_last; c0 += kMergeBatch) {
      float ms[kMergeBatch], ls[kMergeBatch], os[kMergeBatch];
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        const int c = c0 + i;
        ms[i] = -INFINITY;
        ls[i] = os[i] = 0.f;
        if (c <= c_last) {
          const int64_t g0 = w.g;
          const int64_t g1 = w.step();
          if (max(g0, p0) < min(g1, p1)) {
            ms[i] = partial_ml[2 * (base + c)];
            ls[i] = partial_ml[2 * (base + c) + 1];
            os[i] = partial_o[(base + c) * head_dim + d];
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        if (ms[i] != -INFINITY) {
          const float f = ex2(ms[i] - m);
          num += os[i] * f;
          den += ls[i] * f;
        }
      }
    }
    T* out = o + static_cast<int64_t>(b) * o_batch_stride + static_cast<int64_t>(h) * o_head_stride;
    store_out<T>(out + d, den > 0.f ? num / den : 0.f);
    if (d == 0) lse[bh] = den > 0.f ? m * 0.69314718055994530942f + logf(den) : -INFINITY;
  }
}

template <typename T, int D, bool kDeep, int kProducers>
int launch_split_p(const DecodeArgs& args, const CUtensorMap& tmk, const CUtensorMap& tmv,
                   int grid_x, int grid_y, cudaStream_t stream) {
  using Cfg = DecodeCfg<D, kDeep>;
  static thread_local int configured_device = -1;  // per-thread cache of the attribute set-up
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    if (int st = check_cuda(cudaFuncSetAttribute(decode_split_kernel<T, D, kDeep, kProducers>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 Cfg::kSmemBytes +
                                                     Cfg::merge_bytes(kMaxHeadsPerCta)),
                            "cudaFuncSetAttribute(decode)"))
      return st;
    configured_device = dev;
  }
  const int smem = Cfg::kSmemBytes + (args.balanced ? Cfg::merge_bytes(args.merge_rows) : 0);
  decode_split_kernel<T, D, kDeep, kProducers>
      <<<dim3(grid_x, grid_y), decode_threads(kProducers), smem, stream>>>(args, tmk, tmv);
  return check_cuda(cudaGetLastError(), "decode_split_kernel launch");
}

// Small pages (several parts per tile) run the two-producer form, everything else the
// one-producer form whose consumers address one-part tiles with compile-time offsets.
template <typename T, int D, bool kDeep>
int launch_split(const DecodeArgs& args, const CUtensorMap& tmk, const CUtensorMap& tmv,
                 int grid_x, int grid_y, cudaStream_t stream) {
  if (args.producers == 2)
    return launch_split_p<T, D, kDeep, 2>(args, tmk, tmv, grid_x, grid_y, stream);
  if (args.box_rows != kDecodeBK)
    return fail(FLB_ERR_UNSUPPORTED, "decode: pages under %d rows need the two-producer kernel",
                kDecodeBK);
  return launch_split_p<T, D, kDeep, 1>(args, tmk, tmv, grid_x, grid_y, stream);
}

template <typename T, bool kPeers = false>
int launch_merge(const float* po, const float* pml, int batch, int heads, int head_dim,
                 int splits, void* o, int64_t obs, int64_t ohs, float* lse, cudaStream_t stream,
                 PeerWait wait = PeerWait{}) {
  // Programmatic dependent launch: the merge grid is scheduled while the split kernel drains
  // and waits (griddepcontrol.wait) for its results, which hides the launch gap between them.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(batch * heads);
  cfg.blockDim = dim3(head_dim);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  T* out = static_cast<T*>(o);
  return check_cuda(cudaLaunchKernelEx(&cfg, decode_merge_kernel<T, kPeers>, po, pml, heads,
                                       head_dim, splits, out, obs, ohs, lse, wait),
                    "decode_merge_kernel launch");
}

// The merge of a length-balanced launch, for any output dtype (programmatic dependent launch).
int launch_merge_balanced(const flb_decode_params* p, const float* po, const float* pml,
                          int ctas, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p->batch * p->heads);
  cfg.blockDim = dim3(p->head_dim);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t err;
  if (p->dtype == FLB_BF16) {
    err = cudaLaunchKernelEx(&cfg, decode_merge_balanced_kernel<__nv_bfloat16>, po, pml,
                             p->seq_lens, p->batch, p->heads, p->head_dim, ctas, p->max_seqlen,
                             static_cast<__nv_bfloat16*>(p->o), p->o_batch_stride,
                             p->o_head_stride, p->lse);
  } else {
    err = cudaLaunchKernelEx(&cfg, decode_merge_balanced_kernel<__half>, po, pml, p->seq_lens,
                             p->batch, p->heads, p->head_dim, ctas, p->max_seqlen,
                             static_cast<__half*>(p->o), p->o_batch_stride, p->o_head_stride,
                             p->lse);
  }
  return check_cuda(err, "decode_merge_balanced_kernel launch");
}

int validate(const flb_decode_params* p) {
  if (p == nullptr) return fail(FLB_ERR_INVALID_ARGUMENT, "params is NULL");
  if (!p->q || !p->k_cache || !p->v_cache || !p->o || !p->lse || !p->seq_lens)
    return fail(FLB_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (p->batch <= 0 || p->heads <= 0 || p->heads_kv <= 0 || p->max_seqlen <= 0)
    return fail(FLB_ERR_INVALID_ARGUMENT, "empty input: batch %d heads %d heads_kv %d S_max %d",
                p->batch, p->heads, p->heads_kv, p->max_seqlen);
  if (p->heads % p->heads_kv != 0)
    return fail(FLB_ERR_INVALID_ARGUMENT,
                "the number of query heads (%d) must be a multiple of KV heads (%d)", p->heads,
                p->heads_kv);
  if (p->dtype != FLB_BF16 && p->dtype != FLB_FP16 && p->dtype != FLB_FP32)
    return fail(FLB_ERR_UNSUPPORTED, "decode takes bf16, fp16 or fp32 (dtype code %d)",
                p->dtype);
  if (p->head_dim != 64 && p->head_dim != 128)
    return fail(FLB_ERR_UNSUPPORTED, "unsupported head_dim %d (64 or 128)", p->head_dim);
  if (!(p->softmax_scale > 0.f))
    return fail(FLB_ERR_INVALID_ARGUMENT, "softmax_scale must be positive");
  if (p->num_splits < 0 || p->num_splits > kMaxSplits)
    return fail(FLB_ERR_INVALID_ARGUMENT, "num_splits must be in [0, %d]", kMaxSplits);
  if (p->block_tables != nullptr) {
    const int ps = p->page_size;
    // A 128-byte-swizzled box must start on a 1024-byte (8-row) boundary, and a box never
    // crosses a page: pages of 8, 16 or 32 rows, or whole multiples of the 64-key tile.
    if (ps <= 0 || !(ps == 8 || ps == 16 || ps == 32 || ps % 64 == 0))
      return fail(FLB_ERR_UNSUPPORTED,
                  "paged cache: page_size %d must be 8, 16, 32 or a multiple of 64", ps);
    if (p->num_blocks <= 0)
      return fail(FLB_ERR_INVALID_ARGUMENT, "paged cache: num_blocks must be positive");
    if (p->max_seqlen % ps != 0)
      return fail(FLB_ERR_INVALID_ARGUMENT,
                  "paged cache: max_seqlen %d must be max_blocks * page_size (page_size %d)",
                  p->max_seqlen, ps);
    if (p->batch > 1 && p->block_table_stride < p->max_seqlen / ps)
      return fail(FLB_ERR_INVALID_ARGUMENT, "paged cache: block_table_stride %lld < max_blocks %d",
                  static_cast<long long>(p->block_table_stride), p->max_seqlen / ps);
  }
  const int64_t esize = p->dtype == FLB_FP32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(p->q) % 16 != 0 ||
      (p->batch > 1 && (p->q_batch_stride * esize) % 16 != 0) ||
      (p->heads > 1 && (p->q_head_stride * esize) % 16 != 0))
    return fail(FLB_ERR_MISALIGNED, "q must have 16-byte aligned rows");
  return FLB_OK;
}

// Keys per tile of the kernel that runs p, and rows per TMA box (a box never crosses a page).
int tile_keys_for(const flb_decode_params* p) { return p->dtype == FLB_FP32 ? kF32BK : kDecodeBK; }

int box_rows_for(const flb_decode_params* p) {
  const int tile = tile_keys_for(p);
  return p->block_tables != nullptr ? std::min(tile, p->page_size) : tile;
}

// Caches of pages under one tile (8, 16 or 32 rows) need several TMA copies per tile, and the
// producers' copy issue rate bounds them. With 16-bit head_dim 128 they are read through
// two-half maps (one copy per page instead of one per 64-column box: 8 instead of 16 per 64-key
// tile at 16-row pages) by two producer warps. Measured on the ragged GQA configuration with
// 16-row pages: 121.9 -> 119.9 us. Contiguous caches keep one producer and 4-D maps, which
// measured 1-4 % faster for them (short contexts most).
bool has_small_pages(const flb_decode_params* p) {
  return p->block_tables != nullptr && p->page_size < kDecodeBK;
}
bool uses_halves_map(const flb_decode_params* p) {
  return p->dtype != FLB_FP32 && p->head_dim == 128 && has_small_pages(p);
}

int build_maps(const flb_decode_params* p, CUtensorMap* tmk, CUtensorMap* tmv, TmaCoords* kc,
               TmaCoords* vc) {
  const int esize = p->dtype == FLB_FP32 ? 4 : 2;
  // A paged cache is the same 4-D view with blocks in place of sequences and pages in place of
  // the sequence axis; its boxes are at most one page tall.
  const bool paged = p->block_tables != nullptr;
  const int64_t outer = paged ? p->num_blocks : p->batch;
  const int64_t rows = paged ? p->page_size : p->max_seqlen;
  View4 kv{p->k_cache,
           {outer, rows, p->heads_kv, p->head_dim},
           {p->k_batch_stride, p->k_seq_stride, p->k_head_stride, 1},
           esize};
  View4 vv{p->v_cache,
           {outer, rows, p->heads_kv, p->head_dim},
           {p->v_batch_stride, p->v_seq_stride, p->v_head_stride, 1},
           esize};
  if (!rows_16b_aligned(kv))
    return fail(FLB_ERR_MISALIGNED, "k_cache must have 16-byte aligned rows (data pointer and strides)");
  if (!rows_16b_aligned(vv))
    return fail(FLB_ERR_MISALIGNED, "v_cache must have 16-byte aligned rows (data pointer and strides)");
  const int box_rows = box_rows_for(p);
  if (p->dtype == FLB_FP32) {   // [box_rows x D] fp32 boxes, unswizzled
    if (int st = encode_rows_map(tmk, kc, kv, box_rows, p->head_dim, FLB_FP32, false)) return st;
    return encode_rows_map(tmv, vc, vv, box_rows, p->head_dim, FLB_FP32, false);
  }
  if (uses_halves_map(p)) {
    if (int st = encode_rows_x64x2_map(tmk, kc, kv, box_rows, p->dtype)) return st;
    return encode_rows_x64x2_map(tmv, vc, vv, box_rows, p->dtype);
  }
  if (int st = encode_rows_x64_map(tmk, kc, kv, box_rows, p->dtype)) return st;
  return encode_rows_x64_map(tmv, vc, vv, box_rows, p->dtype);
}

DecodeArgs make_args(const flb_decode_params* p) {
  DecodeArgs a{};
  a.q = p->q;
  a.o = p->o;
  a.lse = p->lse;
  a.seq_lens = p->seq_lens;
  a.status = p->status;
  a.q_batch_stride = p->q_batch_stride;
  a.q_head_stride = p->q_head_stride;
  a.o_batch_stride = p->o_batch_stride;
  a.o_head_stride = p->o_head_stride;
  a.batch = p->batch;
  a.heads = p->heads;
  a.heads_kv = p->heads_kv;
  a.group = p->heads / p->heads_kv;
  const int heads_per_cta = p->dtype == FLB_FP32 ? kF32MaxHeads : kMaxHeadsPerCta;
  a.head_chunks = (a.group + heads_per_cta - 1) / heads_per_cta;
  a.max_seqlen = p->max_seqlen;
  a.scale_log2 = static_cast<float>(static_cast<double>(p->softmax_scale) * 1.4426950408889634);
  a.key_begin = 0;
  a.key_end = p->max_seqlen;
  if (p->block_tables != nullptr) {
    a.block_tables = p->block_tables;
    a.bt_stride = p->block_table_stride;
    a.page_size = p->page_size;
    a.max_blocks = p->max_seqlen / p->page_size;
  }
  a.box_rows = box_rows_for(p);
  a.halves_map = uses_halves_map(p) ? 1 : 0;
  a.producers = p->dtype != FLB_FP32 && has_small_pages(p) ? 2 : 1;
  a.merge_rows = kMaxHeadsPerCta;
  return a;
}

template <int D, int kHeads>
int launch_split_f32(const DecodeArgs& args, const CUtensorMap& tmk, const CUtensorMap& tmv,
                     int grid_x, int grid_y, cudaStream_t stream) {
  using Cfg = DecodeF32Cfg<D>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    if (int st = check_cuda(cudaFuncSetAttribute(decode_split_f32_kernel<D, kHeads>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 Cfg::kSmemBytes),
                            "cudaFuncSetAttribute(decode f32)"))
      return st;
    configured_device = dev;
  }
  decode_split_f32_kernel<D, kHeads>
      <<<dim3(grid_x, grid_y), kDecodeThreads, Cfg::kSmemBytes, stream>>>(args, tmk, tmv);
  return check_cuda(cudaGetLastError(), "decode_split_f32_kernel launch");
}

template <int D>
int launch_split_f32_heads(const DecodeArgs& a, const CUtensorMap& tmk, const CUtensorMap& tmv,
                           int grid_x, int grid_y, cudaStream_t stream) {
  // Query heads a CTA holds in registers: the group (a power of two at least as large), at most 8.
  if (a.group >= 5) return launch_split_f32<D, 8>(a, tmk, tmv, grid_x, grid_y, stream);
  if (a.group >= 3) return launch_split_f32<D, 4>(a, tmk, tmv, grid_x, grid_y, stream);
  if (a.group == 2) return launch_split_f32<D, 2>(a, tmk, tmv, grid_x, grid_y, stream);
  return launch_split_f32<D, 1>(a, tmk, tmv, grid_x, grid_y, stream);
}

template <typename T, bool kDeep>
int launch_split_t(int head_dim, const DecodeArgs& a, const CUtensorMap& tmk,
                   const CUtensorMap& tmv, int grid_x, int grid_y, cudaStream_t stream) {
  if (head_dim == 128) return launch_split<T, 128, kDeep>(a, tmk, tmv, grid_x, grid_y, stream);
  return launch_split<T, 64, kDeep>(a, tmk, tmv, grid_x, grid_y, stream);
}

// The split kernel for any supported (dtype, head_dim); deep: the one-CTA-per-SM ring (16-bit).
int launch_split_any(int dtype, int head_dim, const DecodeArgs& a, const CUtensorMap& tmk,
                     const CUtensorMap& tmv, int grid_x, int grid_y, cudaStream_t stream,
                     bool deep = false) {
  if (dtype == FLB_FP32) {
    if (head_dim == 128) return launch_split_f32_heads<128>(a, tmk, tmv, grid_x, grid_y, stream);
    return launch_split_f32_heads<64>(a, tmk, tmv, grid_x, grid_y, stream);
  }
  if (dtype == FLB_BF16) {
    return deep ? launch_split_t<__nv_bfloat16, true>(head_dim, a, tmk, tmv, grid_x, grid_y, stream)
                : launch_split_t<__nv_bfloat16, false>(head_dim, a, tmk, tmv, grid_x, grid_y,
                                                       stream);
  }
  return deep ? launch_split_t<__half, true>(head_dim, a, tmk, tmv, grid_x, grid_y, stream)
              : launch_split_t<__half, false>(head_dim, a, tmk, tmv, grid_x, grid_y, stream);
}

// The merge kernel for any output dtype.
template <bool kPeers = false>
int launch_merge_any(int dtype, const float* po, const float* pml, int batch, int heads,
                     int head_dim, int splits, void* o, int64_t obs, int64_t ohs, float* lse,
                     cudaStream_t stream, PeerWait wait = PeerWait{}) {
  if (dtype == FLB_BF16)
    return launch_merge<__nv_bfloat16, kPeers>(po, pml, batch, heads, head_dim, splits, o, obs,
                                               ohs, lse, stream, wait);
  if (dtype == FLB_FP16)
    return launch_merge<__half, kPeers>(po, pml, batch, heads, head_dim, splits, o, obs, ohs, lse,
                                        stream, wait);
  if (dtype == FLB_FP32)
    return launch_merge<float, kPeers>(po, pml, batch, heads, head_dim, splits, o, obs, ohs, lse,
                                       stream, wait);
  return fail(FLB_ERR_UNSUPPORTED, "merge takes bf16, fp16 or fp32 (dtype code %d)", dtype);
}

// Split count from shapes only (so a captured CUDA graph stays valid for any lengths). Measured
// on B200 at 32K keys: about one CTA per SM is best (B=1 MHA: 4 splits 89 us against 107 us for
// 37; B=8 MHA: 1 split 606 us against 626 us for 8; B=8 GQA with ragged lengths: 3 splits
// 124 us against 132 us for 18), and splits shorter than 8 tiles (512 keys) lose to their fixed
// costs. More, shorter CTAs pay more prologues, more partials and a longer merge than the load
// balance they buy.
int splits_for(int batch, int heads, int heads_kv, int head_dim, int max_seqlen, int sm_count) {
  (void)head_dim;
  if (batch <= 0 || heads <= 0 || heads_kv <= 0 || heads % heads_kv != 0 || max_seqlen <= 0 ||
      sm_count <= 0)
    return 1;
  const int group = heads / heads_kv;
  const int chunks = (group + kMaxHeadsPerCta - 1) / kMaxHeadsPerCta;
  const int64_t ctas = static_cast<int64_t>(batch) * heads_kv * chunks;
  const int64_t by_sm = (sm_count + ctas - 1) / ctas;
  const int64_t by_len = std::max<int64_t>(1, max_seqlen / (8 * kDecodeBK));
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({by_sm, by_len, kMaxSplits})));
}

// A uniform launch of the 16-bit kernel (the sharded entry points) takes the deep ring when its
// grid fits on the SMs at one CTA per SM.
bool deep_fits(int grid_x, int grid_y, int sm_count) {
  return static_cast<int64_t>(grid_x) * grid_y <= sm_count;
}

// Dynamic shared memory of a balanced launch of the 16-bit kernel.
int balanced_smem(int head_dim, bool deep, int merge_rows) {
  if (head_dim == 128)
    return deep ? DecodeCfg<128, true>::kSmemBytes + DecodeCfg<128, true>::merge_bytes(merge_rows)
                : DecodeCfg<128>::kSmemBytes + DecodeCfg<128>::merge_bytes(merge_rows);
  return deep ? DecodeCfg<64, true>::kSmemBytes + DecodeCfg<64, true>::merge_bytes(merge_rows)
              : DecodeCfg<64>::kSmemBytes + DecodeCfg<64>::merge_bytes(merge_rows);
}

bool two_per_sm(int smem) {
  constexpr int kSmemPerSm = 228 * 1024, kReservedPerCta = 1024;
  return 2 * (smem + kReservedPerCta) <= kSmemPerSm;
}

// How flb_decode_fwd runs p with more than one split: length-balanced key ranges over `ctas` CTAs
// per (KV head, head chunk) column (16-bit caches, at most kMaxBalancedBatch sequences), or the
// uniform split (on = false).
struct BalancedPlan {
  bool on = false;
  bool deep = false;   // the one-CTA-per-SM ring
  int ctas = 0;
  int merge_rows = 0;
};

BalancedPlan plan_balanced(const flb_decode_params* p, int splits, int columns, int group,
                           int sm_count) {
  BalancedPlan plan;
  if (splits <= 1 || p->dtype == FLB_FP32 || p->batch > kMaxBalancedBatch) return plan;
  const int64_t chunks = (static_cast<int64_t>(p->max_seqlen) + kDecodeBK - 1) / kDecodeBK;
  if (static_cast<int64_t>(p->batch) * chunks >= (int64_t{1} << 31)) return plan;
  plan.merge_rows = std::min(group, kMaxHeadsPerCta);
  const int64_t smem2 = balanced_smem(p->head_dim, false, plan.merge_rows);
  if (p->num_splits > 0) {
    // An explicit split count: batch * num_splits CTAs per column with the default ring, while
    // two of them still fit on an SM or the grid fits on the SMs.
    plan.ctas = p->batch * splits;
    plan.on = two_per_sm(smem2) || static_cast<int64_t>(plan.ctas) * columns <= sm_count;
    return plan;
  }
  // Split count left to the library: every SM gets the same number of CTAs. One CTA per SM with
  // the deep ring, except for caches of small pages (under 64 rows), whose tiles are 8 to 16 TMA
  // boxes each: there one producer warp per SM cannot issue them fast enough (measured with
  // 16-row pages: 179 us with one CTA per SM, 157 us with more), so two CTAs share each SM.
  const int per_sm = has_small_pages(p) && two_per_sm(smem2) ? 2 : 1;
  plan.deep = per_sm == 1;
  plan.ctas = std::clamp(per_sm * sm_count / columns, p->batch, 2 * p->batch * splits);
  plan.on = true;
  return plan;
}

}  // namespace
}  // namespace flb

using namespace flb;

extern "C" int flb_decode_num_splits(int32_t batch, int32_t heads, int32_t heads_kv,
                                     int32_t head_dim, int32_t max_seqlen, int32_t sm_count) {
  return splits_for(batch, heads, heads_kv, head_dim, max_seqlen, sm_count);
}

namespace flb {
namespace {
// Partial slots of a flb_decode_fwd workspace: batch * heads * (2 num_splits + 1), the most a
// length-balanced launch writes (heads * (batch + T) for T <= 2 batch num_splits CTAs per
// column); a uniform launch uses the first batch * heads * num_splits.
size_t workspace_slots(int batch, int heads, int num_splits) {
  return static_cast<size_t>(batch) * heads * (2 * static_cast<size_t>(num_splits) + 1);
}
}  // namespace
}  // namespace flb

extern "C" size_t flb_decode_workspace_bytes(int32_t batch, int32_t heads, int32_t head_dim,
                                             int32_t num_splits) {
  if (num_splits <= 1 || batch <= 0 || heads <= 0 || head_dim <= 0) return 0;
  const size_t slots = workspace_slots(batch, heads, num_splits);
  const size_t o_bytes = (slots * head_dim * sizeof(float) + 255) / 256 * 256;
  return o_bytes + slots * 2 * sizeof(float);
}

extern "C" int flb_decode_fwd(const flb_decode_params* p, flb_stream_t stream_) {
  clear_error();
  if (int st = validate(p)) return st;
  int dev = 0, sm_count = 0;
  if (int st = current_device_info(&dev, &sm_count, nullptr, nullptr)) return st;
  CUtensorMap tmk, tmv;
  TmaCoords kc{}, vc{};
  if (int st = build_maps(p, &tmk, &tmv, &kc, &vc)) return st;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);

  DecodeArgs a = make_args(p);
  a.kc = kc;
  a.vc = vc;
  const int splits = p->num_splits > 0
                         ? p->num_splits
                         : splits_for(p->batch, p->heads, p->heads_kv, p->head_dim,
                                      p->max_seqlen, sm_count);
  const int grid_y = p->batch * p->heads_kv * a.head_chunks;
  if (grid_y > 65535)
    return fail(FLB_ERR_UNSUPPORTED, "batch * heads_kv * head chunks = %d exceeds 65535", grid_y);
  a.num_splits = splits;
  a.split_offset = 0;
  a.splits_total = splits;
  if (splits == 1) {
    a.write_partials = 0;
    return launch_split_any(p->dtype, p->head_dim, a, tmk, tmv, 1, grid_y, stream);
  }
  const size_t need = flb_decode_workspace_bytes(p->batch, p->heads, p->head_dim, splits);
  if (p->workspace == nullptr || p->workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "decode with %d splits needs %zu bytes of workspace, got %zu",
                splits, need, p->workspace == nullptr ? size_t(0) : p->workspace_bytes);
  if (reinterpret_cast<uintptr_t>(p->workspace) % 256 != 0)
    return fail(FLB_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  const size_t slots = workspace_slots(p->batch, p->heads, splits);
  a.n_dest = 1;
  a.partial_o[0] = static_cast<float*>(p->workspace);
  a.partial_ml[0] = reinterpret_cast<float*>(
      static_cast<char*>(p->workspace) + (slots * p->head_dim * sizeof(float) + 255) / 256 * 256);
  a.write_partials = 1;
  // A balanced launch runs plan.ctas CTAs per (KV head, head chunk) column. With the split
  // count left to the library every SM gets the same number of CTAs (CTAs that share an SM with
  // another finish measurably later than CTAs alone).
  const int columns = p->heads_kv * a.head_chunks;
  const BalancedPlan plan = plan_balanced(p, splits, columns, a.group, sm_count);
  if (plan.on) {
    a.balanced = 1;
    a.bal_ctas = plan.ctas;
    a.merge_rows = plan.merge_rows;
    if (int st = launch_split_any(p->dtype, p->head_dim, a, tmk, tmv, plan.ctas, columns, stream,
                                  plan.deep))
      return st;
    return launch_merge_balanced(p, a.partial_o[0], a.partial_ml[0], plan.ctas, stream);
  }
  if (int st = launch_split_any(p->dtype, p->head_dim, a, tmk, tmv, splits, grid_y, stream))
    return st;
  return launch_merge_any(p->dtype, a.partial_o[0], a.partial_ml[0], p->batch, p->heads,
                          p->head_dim, splits, p->o, p->o_batch_stride, p->o_head_stride, p->lse,
                          stream);
}

extern "C" int flb_decode_partials(const flb_decode_params* p, int32_t key_begin,
                                   int32_t key_end, int32_t seq_offset, float* partial_o,
                                   float* partial_ml, flb_stream_t stream_) {
  clear_error();
  if (p == nullptr) return fail(FLB_ERR_INVALID_ARGUMENT, "params is NULL");
  flb_decode_params q = *p;
  // o / lse are not written in this mode; accept NULL for them.
  static char dummy;
  if (q.o == nullptr) q.o = &dummy;
  if (q.lse == nullptr) q.lse = reinterpret_cast<float*>(&dummy);
  if (int st = validate(&q)) return st;
  if (!partial_o || !partial_ml) return fail(FLB_ERR_INVALID_ARGUMENT, "partials are NULL");
  if (key_begin < 0 || key_end < key_begin)
    return fail(FLB_ERR_INVALID_ARGUMENT, "bad key window [%d, %d)", key_begin, key_end);
  if (q.num_splits < 1) return fail(FLB_ERR_INVALID_ARGUMENT, "num_splits must be >= 1 here");
  if (q.block_tables != nullptr && key_begin % tile_keys_for(&q) != 0)
    return fail(FLB_ERR_UNSUPPORTED, "paged cache: key_begin %d must be a multiple of %d",
                key_begin, tile_keys_for(&q));
  int dev = 0, sm_count = 0;
  if (int st = current_device_info(&dev, &sm_count, nullptr, nullptr)) return st;
  CUtensorMap tmk, tmv;
  TmaCoords kc{}, vc{};
  if (int st = build_maps(&q, &tmk, &tmv, &kc, &vc)) return st;
  DecodeArgs a = make_args(&q);
  a.kc = kc;
  a.vc = vc;
  a.key_begin = key_begin;
  a.key_end = key_end;
  a.len_offset = seq_offset;
  a.num_splits = q.num_splits;
  a.split_offset = 0;
  a.splits_total = q.num_splits;
  a.write_partials = 1;
  a.n_dest = 1;
  a.partial_o[0] = partial_o;
  a.partial_ml[0] = partial_ml;
  const int grid_y = q.batch * q.heads_kv * a.head_chunks;
  if (grid_y > 65535)
    return fail(FLB_ERR_UNSUPPORTED, "batch * heads_kv * head chunks = %d exceeds 65535", grid_y);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  return launch_split_any(q.dtype, q.head_dim, a, tmk, tmv, q.num_splits, grid_y, stream,
                          deep_fits(q.num_splits, grid_y, sm_count));
}

extern "C" int flb_decode_merge(const float* partial_o, const float* partial_ml, int32_t batch,
                                int32_t heads, int32_t head_dim, int32_t num_splits,
                                int32_t dtype, void* o, int64_t o_batch_stride,
                                int64_t o_head_stride, float* lse, flb_stream_t stream_) {
  clear_error();
  if (!partial_o || !partial_ml || !o || !lse)
    return fail(FLB_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (batch <= 0 || heads <= 0 || num_splits <= 0 || (head_dim != 64 && head_dim != 128))
    return fail(FLB_ERR_INVALID_ARGUMENT, "bad merge shape");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  return launch_merge_any(dtype, partial_o, partial_ml, batch, heads, head_dim, num_splits, o,
                          o_batch_stride, o_head_stride, lse, stream);
}

// ---------------------------------------------------------------------------------------------
// Cross-GPU exchange over peer memory (layout in include/flash_lab_b200.h).
// ---------------------------------------------------------------------------------------------
namespace flb {
namespace {

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct ExchangeLayout {
  size_t counters;      // bytes of the counter block
  size_t po_bytes;      // partial_o of one parity region
  size_t region;        // one parity region
};

// Words of the counter block (uint64 each): [0, world) arrivals per source rank, then this
// rank's CTA count of the push in progress, the CTA count of the merge in progress and its
// completed-step count.
constexpr int kPushCtasWord = 0, kMergeCtasWord = 1, kStepWord = 2;   // after the arrivals

size_t counter_block_bytes(int world) {
  return align256(static_cast<size_t>(world + 3) * sizeof(unsigned long long));
}

ExchangeLayout exchange_layout(int world, int batch, int heads, int head_dim, int splits) {
  ExchangeLayout l;
  l.counters = counter_block_bytes(world);
  const size_t slots = static_cast<size_t>(batch) * heads * world * splits;
  l.po_bytes = align256(slots * head_dim * sizeof(float));
  l.region = align256(l.po_bytes + slots * 2 * sizeof(float));
  return l;
}

int check_exchange(const flb_peer_exchange* x) {
  if (x == nullptr) return fail(FLB_ERR_INVALID_ARGUMENT, "exchange is NULL");
  if (x->world < 1 || x->world > FLB_MAX_PEERS || x->rank < 0 || x->rank >= x->world)
    return fail(FLB_ERR_INVALID_ARGUMENT, "exchange: rank %d of world %d (at most %d ranks)",
                x->rank, x->world, FLB_MAX_PEERS);
  for (int r = 0; r < x->world; ++r) {
    if (x->buffers[r] == nullptr)
      return fail(FLB_ERR_INVALID_ARGUMENT, "exchange: buffer of rank %d is NULL", r);
    if (reinterpret_cast<uintptr_t>(x->buffers[r]) % 256 != 0)
      return fail(FLB_ERR_MISALIGNED, "exchange: buffer of rank %d is not 256-byte aligned", r);
  }
  return FLB_OK;
}

}  // namespace
}  // namespace flb

extern "C" size_t flb_peer_exchange_bytes(int32_t world, int32_t batch, int32_t heads,
                                          int32_t head_dim, int32_t splits_per_rank) {
  if (world < 1 || batch <= 0 || heads <= 0 || head_dim <= 0 || splits_per_rank <= 0) return 0;
  const ExchangeLayout l = exchange_layout(world, batch, heads, head_dim, splits_per_rank);
  return l.counters + 2 * l.region;
}

extern "C" int flb_decode_partials_push(const flb_decode_params* p, int32_t key_begin,
                                        int32_t key_end, int32_t seq_offset,
                                        const flb_peer_exchange* x, flb_stream_t stream_) {
  clear_error();
  if (p == nullptr) return fail(FLB_ERR_INVALID_ARGUMENT, "params is NULL");
  if (int st = check_exchange(x)) return st;
  flb_decode_params q = *p;
  static char dummy;
  if (q.o == nullptr) q.o = &dummy;
  if (q.lse == nullptr) q.lse = reinterpret_cast<float*>(&dummy);
  if (int st = validate(&q)) return st;
  if (key_begin < 0 || key_end < key_begin)
    return fail(FLB_ERR_INVALID_ARGUMENT, "bad key window [%d, %d)", key_begin, key_end);
  if (q.num_splits < 1) return fail(FLB_ERR_INVALID_ARGUMENT, "num_splits must be >= 1 here");
  if (q.block_tables != nullptr && key_begin % tile_keys_for(&q) != 0)
    return fail(FLB_ERR_UNSUPPORTED, "paged cache: key_begin %d must be a multiple of %d",
                key_begin, tile_keys_for(&q));
  int dev = 0, sm_count = 0;
  if (int st = current_device_info(&dev, &sm_count, nullptr, nullptr)) return st;
  CUtensorMap tmk, tmv;
  TmaCoords kc{}, vc{};
  if (int st = build_maps(&q, &tmk, &tmv, &kc, &vc)) return st;
  DecodeArgs a = make_args(&q);
  a.kc = kc;
  a.vc = vc;
  a.key_begin = key_begin;
  a.key_end = key_end;
  a.len_offset = seq_offset;
  a.num_splits = q.num_splits;
  a.split_offset = x->rank * q.num_splits;
  a.splits_total = x->world * q.num_splits;
  a.write_partials = 1;
  const ExchangeLayout l = exchange_layout(x->world, q.batch, q.heads, q.head_dim, q.num_splits);
  a.n_dest = x->world;
  for (int r = 0; r < x->world; ++r) {
    char* region = static_cast<char*>(x->buffers[r]) + l.counters;   // parity region 0
    a.partial_o[r] = reinterpret_cast<float*>(region);
    a.partial_ml[r] = reinterpret_cast<float*>(region + l.po_bytes);
    a.arrive[r] = static_cast<unsigned long long*>(x->buffers[r]) + x->rank;
  }
  unsigned long long* own = static_cast<unsigned long long*>(x->buffers[x->rank]);
  a.cta_done = reinterpret_cast<unsigned int*>(own + x->world + kPushCtasWord);
  a.step_word = own + x->world + kStepWord;
  a.region_o = static_cast<int64_t>(l.region / sizeof(float));
  a.region_ml = a.region_o;
  const int grid_y = q.batch * q.heads_kv * a.head_chunks;
  if (grid_y > 65535)
    return fail(FLB_ERR_UNSUPPORTED, "batch * heads_kv * head chunks = %d exceeds 65535", grid_y);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  return launch_split_any(q.dtype, q.head_dim, a, tmk, tmv, q.num_splits, grid_y, stream,
                          deep_fits(q.num_splits, grid_y, sm_count));
}

extern "C" int flb_decode_merge_peers(const flb_peer_exchange* x, int32_t batch, int32_t heads,
                                      int32_t head_dim, int32_t splits_per_rank, int32_t dtype,
                                      void* o, int64_t o_batch_stride, int64_t o_head_stride,
                                      float* lse, int32_t* status, flb_stream_t stream_) {
  clear_error();
  if (int st = check_exchange(x)) return st;
  if (!o || !lse) return fail(FLB_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (batch <= 0 || heads <= 0 || splits_per_rank <= 0 || (head_dim != 64 && head_dim != 128))
    return fail(FLB_ERR_INVALID_ARGUMENT, "bad merge shape");
  if (batch * heads > 0x7fffffff / 2) return fail(FLB_ERR_UNSUPPORTED, "merge grid too large");
  const ExchangeLayout l = exchange_layout(x->world, batch, heads, head_dim, splits_per_rank);
  const char* region = static_cast<const char*>(x->buffers[x->rank]) + l.counters;
  const float* po = reinterpret_cast<const float*>(region);
  const float* pml = reinterpret_cast<const float*>(region + l.po_bytes);
  unsigned long long* own = static_cast<unsigned long long*>(x->buffers[x->rank]);
  PeerWait wait;
  wait.counters = own;
  wait.step_word = own + x->world + kStepWord;
  wait.merge_done = reinterpret_cast<unsigned int*>(own + x->world + kMergeCtasWord);
  wait.world = x->world;
  wait.region_o = static_cast<int64_t>(l.region / sizeof(float));
  wait.region_ml = wait.region_o;
  wait.timeout_ns = x->timeout_ns > 0 ? x->timeout_ns : static_cast<int64_t>(kWaitTimeoutNs);
  wait.status = status;
  const int splits = x->world * splits_per_rank;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  return launch_merge_any<true>(dtype, po, pml, batch, heads, head_dim, splits, o,
                                o_batch_stride, o_head_stride, lse, stream, wait);
}

extern "C" int flb_peer_exchange_reset(const flb_peer_exchange* x, flb_stream_t stream_) {
  clear_error();
  if (int st = check_exchange(x)) return st;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  return check_cuda(cudaMemsetAsync(x->buffers[x->rank], 0, counter_block_bytes(x->world), stream),
                    "cudaMemsetAsync(exchange counters)");
}

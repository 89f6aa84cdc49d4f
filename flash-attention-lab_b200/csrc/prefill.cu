// Attention forward (prefill) for sm_100a with tcgen05 tensor cores, TMEM accumulators and TMA.
//
// Reference behaviour: the FlashAttention-2 forward of tfan2437/flash-attention-lab,
// csrc/prefill/mma_pipelined.cu:55-149 with the tile math of csrc/prefill/mma_tile.cuh:40-174
// (bottom-right causal mask, exp2-domain online softmax whose reference point is 0 for rows that
// have seen only masked keys, natural-log LSE = m * scale + ln l, -inf for rows without keys) and
// the host glue of csrc/common/attn_host.h:18-93.
//
// B200 design (not a port):
//  * CTA = 256 query rows of one (batch, head) as two 128-row Q tiles; one softmax warpgroup per
//    Q tile. Warp 8 is the TMA producer, warp 9 issues every tcgen05.mma from one thread.
//  * Q (once) and 128-key K / V tiles arrive by TMA in 128-byte-swizzled [128 x 64] boxes (two
//    per tile at head_dim 128, one at 64); K and V alternate through a 128 KB mbarrier ring.
//  * TMEM (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each (O uses head_dim of them).
//    S = Q K^T is an SS UMMA (M=128, N=128, K=16 steps). The softmax warpgroup reads its S row (thread = row = TMEM lane),
//    writes P as packed 16-bit pairs over the first 64 columns of the same S region, and O += P V
//    is a TS UMMA with P taken from TMEM and V as an MN-major shared-memory operand.
//  * The MMA thread interleaves the two Q tiles: PV0(j), S0(j+1), PV1(j), S1(j+1), so one tile's
//    softmax overlaps the other tile's GEMMs.
//  * Online softmax in the exp2 domain with a lazily updated reference point: the running max is
//    only moved (and O, l rescaled in TMEM) when a tile's max exceeds it by more than 2^8, so
//    probabilities stay <= 256 and the common case never touches O. The final O / l and the LSE
//    are exact for any reference point.
//  * Work items are 256 query rows of one (batch, head). Two launch forms of one kernel:
//    - one item per CTA (non-causal head_dim 128): the q-blocks of one (batch, head) are
//      adjacent in launch order, so the CTAs running together share K/V in L2 (causal launches
//      of this form run heaviest first across groups of 16 (batch, head) pairs). The epilogue
//      stages O / l in the Q tile's shared-memory buffer (free by then) and writes it with TMA
//      stores.
//    - persistent CTAs, one per SM, each running a fixed sequence of items (causal, and head_dim
//      64, where the per-item start and end weigh more against the work). Barrier phases continue
//      across items; the next item's Q tiles load as soon as the last Q K^T reading them
//      completes and its K/V tiles stream on through the same ring. Causal work comes in units
//      of two q-blocks of one head, the i-th heaviest with the i-th lightest, so every unit
//      costs the same and the static assignment stays balanced; when K and V fit about in L2,
//      single q-blocks are dealt out in cost order instead, back and forth over the CTAs, which
//      balances item counts that are not multiples of the CTA count. The Q buffers are not free
//      for staging here, so each softmax thread stores its O row directly.
//  * Tiles past the diagonal are never loaded; tiles crossing it are masked element-wise.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <type_traits>

#include "host_common.h"
#include "sm100.cuh"


namespace flb {
namespace {

constexpr int kBM = 128;                       // rows per Q tile
constexpr int kBN = 128;                       // keys per K/V tile
constexpr int kQTiles = 2;                     // Q tiles per CTA
constexpr int kRowsPerCta = kBM * kQTiles;
constexpr int kBoxBytes = kBM * 64 * 2;        // one swizzled [128 x 64] 16-bit box: 16 KB

// Per head dim: a [128 x D] tile is D / 64 boxes. The K/V ring holds 128 KB of tiles at either
// head dim (4 slots of 32 KB at D = 128, 8 of 16 KB at D = 64), so one CTA fills an SM.
template <int D>
struct Geometry {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static constexpr int kBoxes = D / 64;
  static constexpr int kTileBytes = kBM * D * 2;
  static constexpr int kSlots = D == 64 ? 8 : 4;
  static constexpr int kSmemData = (kQTiles + kSlots) * kTileBytes;
  static constexpr int kSmemBytes = kSmemData + 1024 + 256;
};
// Warps: softmax WG0 (0-3), WG1 (4-7), then WG2: producer (8), MMA issuer (9) and two warps with
// no role (10, 11), which make WG2 a whole warpgroup for the register split: the launch gives
// every thread 168 registers (384 x 168 = 64512 of the SM's 65536); WG2 then drops to
// kControl and the softmax warpgroups rise to kSoftmax (2 x 128 x 216 + 128 x 72 = 64512).
// Measured on B200: 208 / 88 spills less in the persistent form but runs slower there (head_dim
// 64: 712 -> 693 TFLOP/s), so both forms use 216 / 72.
constexpr int kThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kLaunchRegs = 168;
template <bool kPersistent>
struct RegSplit {
  static constexpr int kSoftmax = 216;
  static constexpr int kControl = 72;
  static_assert(2 * 128 * kSoftmax + 128 * kControl <= kThreads * kLaunchRegs,
                "the register split must fit in the launch's registers");
};
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;      // log2 units: p <= 2^8 between rescales
constexpr int kDefaultPolyPairs = 2;           // of every 8 score pairs, 2^x on the FMA pipe
#ifndef FLB_PREFILL_PERSISTENT_D128
#define FLB_PREFILL_PERSISTENT_D128 0   // non-causal head_dim 128 persistent too (measurement knob)
#endif
constexpr bool kPersistentD128 = FLB_PREFILL_PERSISTENT_D128 != 0;
// Causal persistent launches whose K and V fit about in L2 schedule single items in cost order
// (PrefillArgs::snake); larger ones keep heavy / light pairs of one head, whose CTAs share K/V
// in L2. Measured on one B200 at the per-GPU shapes of (4, 32, 32, 4096, 128) sharded over N
// GPUs (B x H = 128 / N heads; K+V 268 / 134 / 67 / 34 MB): pairs 492 / 276 / 151 / 81 us,
// single items in cost order 559 / 264 / 136-145 / 70-77 us.
constexpr int64_t kSnakeMaxKvBytes = int64_t{192} << 20;
#ifndef FLB_PREFILL_P_CHUNKS
#define FLB_PREFILL_P_CHUNKS 2
#endif
constexpr int kDefaultPChunks = FLB_PREFILL_P_CHUNKS;   // P published to the MMA warp in this
                                                        // many chunks (1 or 2)
static_assert(kDefaultPChunks == 1 || kDefaultPChunks == 2, "P is published in 1 or 2 chunks");
constexpr int kCausalGroup = 16;               // (batch, head) pairs ordered together (one item
                                               // per CTA, causal)

struct PrefillArgs {
  void* o;
  float* lse;
  int* status;
  int64_t o_batch_stride, o_seq_stride, o_head_stride;
  int batch, seqlen_q, seqlen_k, heads, heads_kv, group;
  int causal, causal_offset;
  int q_blocks;
  int snake;   // causal persistent: single items in cost order, boustrophedon over the CTAs
  float scale, scale_log2;
  TmaCoords qc, kc, vc, oc;
};

template <int kSlots>
struct SharedBarriers {
  uint64_t q_full[kQTiles];
  uint64_t q_free[kQTiles];      // the last Q K^T of an item that reads a Q buffer has completed
  uint64_t kv_full[kSlots];
  uint64_t kv_empty[kSlots];
  uint64_t s_full[kQTiles];
  uint64_t p_half[kQTiles][2];   // P columns 0-31 / 32-63 of a Q tile stored in TMEM
  uint64_t o_full[kQTiles];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ int tma_c(const TmaCoords& c, int slot, int s, int h, int b) {
  return c.pos_s == slot ? s : (c.pos_h == slot ? h : b);
}

// Loads a [128 rows x D dims] tile as D / 64 swizzled boxes.
template <int D>
__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map,
                                          const TmaCoords& c, uint64_t* bar, int row, int head,
                                          int b) {
#pragma unroll
  for (int box = 0; box < Geometry<D>::kBoxes; ++box) {
    tma_load_4d(dst + box * kBoxBytes, map, bar, box * 64, tma_c(c, 1, row, head, b),
                tma_c(c, 2, row, head, b), tma_c(c, 3, row, head, b));
  }
}

// Shared-memory operand descriptors, kept as their two 32-bit words. Within a tile, and from one
// tile of the K/V ring or the Q buffers to the next, only the start-address field changes (the
// address >> 4, bits 0-13 of the low word), and an add to it never carries out of the field
// because shared-memory addresses stay below 2^18 bytes. So the MMA issuer derives the
// descriptor of any k-step of any tile from one base descriptor with a single add: one UMMA
// every 64 clocks (a 128 x 128 x 16 step) leaves the issuing warp no room for the full
// descriptor arithmetic (measured on B200: SS and TS GEMMs of 128 x 128 x 128 issued
// alternately take 727 clocks each with per-step descriptor construction, 514 with this).
struct Desc {
  uint32_t lo, hi;
  __device__ __forceinline__ explicit Desc(uint64_t d)
      : lo(static_cast<uint32_t>(d)), hi(static_cast<uint32_t>(d >> 32)) {}
  __device__ __forceinline__ Desc(uint32_t l, uint32_t h) : lo(l), hi(h) {}
  // The descriptor `bytes` further on in shared memory (bytes a multiple of 16).
  __device__ __forceinline__ Desc at(uint32_t bytes) const { return Desc(lo + (bytes >> 4), hi); }
  __device__ __forceinline__ uint64_t u64() const {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
  }
};

// K-major SW128 operand (Q or K tile): the descriptor of k-step 0 of the tile at tile_addr, and
// the byte offset of k-step kk (16 elements) of a [128 x D] tile.
__device__ __forceinline__ Desc kmajor_desc(uint32_t tile_addr) {
  return Desc(umma_smem_desc_sw128(tile_addr, 16, 1024));
}
constexpr uint32_t kmajor_step(int kk) { return (kk >> 2) * kBoxBytes + (kk & 3) * 32; }

// MN-major SW128 operand (V tile, N = head_dim): k-step kk covers keys 16kk..16kk+15; the
// leading byte offset steps to the next 64 columns of N (unused at D = 64).
__device__ __forceinline__ Desc mnmajor_desc(uint32_t tile_addr) {
  return Desc(umma_smem_desc_sw128(tile_addr, kBoxBytes, 1024));
}
constexpr uint32_t mnmajor_step(int kk) { return kk * 2048; }

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* x, float scale) {
  uint4 r;
  r.x = pack2<T>(x[0] * scale, x[1] * scale);
  r.y = pack2<T>(x[2] * scale, x[3] * scale);
  r.z = pack2<T>(x[4] * scale, x[5] * scale);
  r.w = pack2<T>(x[6] * scale, x[7] * scale);
  return r;
}

// 2^(s * scale_log2 - ref) for one row of 128 scores, row sums in ps, P packed to 16 bits and
// stored to TMEM columns [0, 64) of the row's S region, published in kChunks chunks (each chunk's
// barrier completes when all 128 rows stored it). kPoly of every 8 pairs use the FMA-pipe
// polynomial; the rest use the SFU.
template <typename T, int kPoly, int kChunks, bool kPublish = true>
__device__ __forceinline__ void softmax_exp_store(const float* sf, float sl2, float nref,
                                                  float (&ps)[4], uint32_t taddr_s,
                                                  uint64_t* chunk_bars) {
  constexpr int kPairsPerChunk = 64 / kChunks;
#pragma unroll
  for (int ch = 0; ch < kChunks; ++ch) {
#pragma unroll
    for (int q = 0; q < kPairsPerChunk / 32; ++q) {
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int pair = ch * kPairsPerChunk + q * 32 + c;
        const int i = 2 * pair;
        float x0, x1, p0, p1;
        ffma2(x0, x1, sf[i], sf[i + 1], sl2, sl2, nref, nref);
        if ((pair & 7) < kPoly) {
          exp2_poly2(p0, p1, x0, x1);
        } else {
          p0 = ex2(x0);
          p1 = ex2(x1);
        }
        const int acc = (c & 1) * 2;
        fadd2(ps[acc], ps[acc + 1], ps[acc], ps[acc + 1], p0, p1);
        pk[c] = pack2<T>(p0, p1);
      }
      tmem_st32(taddr_s + ch * (kPairsPerChunk) + q * 32, pk);
    }
    if (kPublish) {
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&chunk_bars[ch]);
    }
  }
}

// Work item k of this CTA: a (batch * head, q-block) pair, or nothing past the end. Every role
// walks the same sequence.
//  One item per CTA: item 0 only. Non-causal in launch order (the q-blocks of one (batch, head)
//  adjacent: they share K/V in L2). Causal heaviest first across groups of kCausalGroup (batch,
//  head) pairs: all the group's last q-blocks, then the ones before, and so on; a group's K/V
//  (33 MB at S = 4096, D = 128) stays in L2 while it runs, and the longest CTAs start well
//  before the final wave.
//  Persistent: non-causal, CTA c takes items c, c + grid, ... in launch order. Causal, the unit
//  of work is a pair of q-blocks of one (batch, head), the i-th heaviest and the i-th lightest,
//  whose costs add up to the same total for every pair; CTA c takes units c, c + grid, ... and
//  runs the heavy item of each unit first.
struct Item {
  int bh, qb;
};

template <bool kPersistent>
__device__ __forceinline__ bool item_at(const PrefillArgs& a, int k, Item& it) {
  if (!kPersistent) {
    if (k > 0) return false;
    if (a.causal) {
      const int per_group = kCausalGroup * a.q_blocks;
      const int g = blockIdx.x / per_group;
      const int first = g * kCausalGroup;
      const int width = min(kCausalGroup, a.batch * a.heads - first);   // last group may be short
      const int r = blockIdx.x - g * per_group;
      it.bh = first + r % width;
      it.qb = a.q_blocks - 1 - r / width;
    } else {
      it.bh = blockIdx.x / a.q_blocks;
      it.qb = blockIdx.x - it.bh * a.q_blocks;
    }
    return true;
  }
  if (!a.causal) {
    const int64_t u = blockIdx.x + static_cast<int64_t>(k) * gridDim.x;
    if (u >= static_cast<int64_t>(a.batch) * a.heads * a.q_blocks) return false;
    it.bh = static_cast<int>(u / a.q_blocks);
    it.qb = static_cast<int>(u - static_cast<int64_t>(it.bh) * a.q_blocks);
    return true;
  }
  if (a.snake) {
    // Item i of the cost order (all heads' last q-block, then all heads' second-to-last, ...):
    // round k gives CTAs 0..G-1 items kG..kG+G-1 on even rounds and in reverse on odd ones,
    // so every CTA's total stays close to the mean.
    const int64_t total = static_cast<int64_t>(a.batch) * a.heads * a.q_blocks;
    const int64_t pos = (k & 1) ? gridDim.x - 1 - blockIdx.x : blockIdx.x;
    const int64_t i = static_cast<int64_t>(k) * gridDim.x + pos;
    if (i >= total) return false;
    const int64_t bhs = static_cast<int64_t>(a.batch) * a.heads;
    it.qb = a.q_blocks - 1 - static_cast<int>(i / bhs);
    it.bh = static_cast<int>(i - (i / bhs) * bhs);
    return true;
  }
  const int pairs = (a.q_blocks + 1) / 2;
  // Items per round: every CTA runs one unit per round, each unit 2 items (the middle q-block
  // of an odd count is a unit of 1, whose second item is skipped).
  const int round = k >> 1, sub = k & 1;
  const int64_t u = blockIdx.x + static_cast<int64_t>(round) * gridDim.x;
  if (u >= static_cast<int64_t>(a.batch) * a.heads * pairs) return false;
  it.bh = static_cast<int>(u / pairs);
  const int p = static_cast<int>(u - static_cast<int64_t>(it.bh) * pairs);
  it.qb = sub == 0 ? a.q_blocks - 1 - p : p;
  if (sub == 1 && it.qb == a.q_blocks - 1 - p) it.qb = -1;   // single-item unit
  return true;
}

// KV tiles each Q tile of an item needs: all of them, or up to the last key its last row sees
// (causal). The item streams the larger count; Q tile 0 of a causal item stops earlier.
__device__ __forceinline__ int kv_tiles_for(const PrefillArgs& a, int qb, int t) {
  const int kv_tiles_all = (a.seqlen_k + kBN - 1) / kBN;
  if (!a.causal) return kv_tiles_all;
  const int last_row = min(qb * kRowsPerCta + (t + 1) * kBM, a.seqlen_q) - 1;
  const int max_key = last_row + a.causal_offset;  // last key any row of the tile sees
  return max_key < 0 ? 0 : min(kv_tiles_all, max_key / kBN + 1);
}

template <typename T, int D, int kPolyPairs, int kPChunks, bool kPersistent>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ PrefillArgs a, const __grid_constant__ CUtensorMap tmq,
                   const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                   const __grid_constant__ CUtensorMap tmo) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kTileBytes = Geometry<D>::kTileBytes;
  constexpr int kSlots = Geometry<D>::kSlots;
  uint8_t* q_smem = smem;                               // kQTiles tiles
  uint8_t* ring = smem + kQTiles * kTileBytes;          // kSlots tiles
  auto* sb = reinterpret_cast<SharedBarriers<kSlots>*>(smem + Geometry<D>::kSmemData);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    sb->abort_flag = 0;
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sb->kv_full[i], 1);
      mbar_init(&sb->kv_empty[i], 1);
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(&sb->q_full[t], 1);
      mbar_init(&sb->q_free[t], 1);
      mbar_init(&sb->s_full[t], 1);
      mbar_init(&sb->p_half[t][0], kBM);
      mbar_init(&sb->p_half[t][1], kBM);
      mbar_init(&sb->o_full[t], 1);
    }
    mbar_init(&sb->mma_done, 1);
    fence_barrier_init();
  }
  if (warp == kProducerWarp) {
    tmem_alloc(&sb->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sb->tmem_base;
  const WaitGuard guard{reinterpret_cast<volatile int*>(&sb->abort_flag), a.status};

  // Barrier phases run on across items: each role counts the completions it has waited for.
  // Each role's branch starts with its side of the register split (every warp of a warpgroup
  // executes the same setmaxnreg).
  if (warp == kProducerWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<kPersistent>::kControl));
    // ------------------------------- TMA producer -------------------------------
    // Per item: Q tile 0, K_0, Q tile 1, V_0, K_1, V_1, ... (Q tile 0 and K_0 first, so tile 0's
    // first Q K^T waits for 64 KB). A Q buffer is reloaded for the next item as soon as the last
    // Q K^T of the previous item that reads it has completed (q_free), which is while that
    // item's last tiles still run. Q tiles without keys are not loaded.
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      if (!kPersistent) tma_prefetch_desc(&tmo);
      int issued = 0;                  // ring copies issued (K and V tiles, all items)
      int q_loads[kQTiles] = {};       // Q copies issued per buffer
      bool ok = true;
      Item it;
      for (int k = 0; ok && item_at<kPersistent>(a, k, it); ++k) {
        if (it.qb < 0) continue;
        const int b = it.bh / a.heads, h = it.bh - b * a.heads, hkv = h / a.group;
        const int q0 = it.qb * kRowsPerCta;
        int n_kv_tile[kQTiles];
#pragma unroll
        for (int t = 0; t < kQTiles; ++t) n_kv_tile[t] = kv_tiles_for(a, it.qb, t);
        const int n_kv = n_kv_tile[kQTiles - 1];
        if (n_kv == 0) continue;
        auto load_q = [&](int t) -> bool {
          if (n_kv_tile[t] == 0) return true;
          if (kPersistent && q_loads[t] > 0 &&
              !mbar_wait(&sb->q_free[t], (q_loads[t] - 1) & 1, guard))
            return false;
          mbar_arrive_expect_tx(&sb->q_full[t], kTileBytes);
          load_tile<D>(q_smem + t * kTileBytes, &tmq, a.qc, &sb->q_full[t], q0 + t * kBM, h, b);
          ++q_loads[t];
          return true;
        };
        ok = load_q(0);
        for (int j = 0; j < n_kv && ok; ++j) {
          for (int kind = 0; kind < 2 && ok; ++kind) {
            const int i = issued;
            const int slot = i % kSlots;
            if (i >= kSlots && !mbar_wait(&sb->kv_empty[slot], ((i / kSlots) - 1) & 1, guard)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&sb->kv_full[slot], kTileBytes);
            load_tile<D>(ring + slot * kTileBytes, kind == 0 ? &tmk : &tmv,
                         kind == 0 ? a.kc : a.vc, &sb->kv_full[slot], j * kBN, hkv, b);
            ++issued;
            if (j == 0 && kind == 0) {
              for (int t = 1; t < kQTiles && ok; ++t) ok = load_q(t);
            }
          }
        }
      }
      // Wait for the copies still landing before the CTA may exit.
      for (int t = 0; t < kQTiles; ++t) {
        if (q_loads[t] > 0) mbar_wait(&sb->q_full[t], (q_loads[t] - 1) & 1, guard);
      }
      for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i) {
        if (!mbar_wait(&sb->kv_full[i % kSlots], (i / kSlots) & 1, guard)) break;
      }
    }
  } else if (warp == kMmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<kPersistent>::kControl));
    // ------------------------------- MMA issuer -------------------------------
    // The whole warp runs this loop (waits stay warp-uniform); one lane, elected once, issues
    // every tcgen05.mma and commit, so each commit tracks all the MMAs before it. Descriptors
    // come from three base descriptors by one add each (Desc). Across items, Q K^T of an item's first
    // KV tile follows P V of the previous item's last one for the same Q tile: MMAs of one thread
    // run in issue order, so it cannot overwrite P before P V reads it. P V with accumulate = 0
    // overwrites O only after the softmax warpgroup has published the new item's first P, which
    // it does after reading the previous item's O.
    constexpr int kFmt = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
    constexpr uint32_t kIdescQK = umma_idesc_f16(kFmt, kBM, kBN, 0);
    constexpr uint32_t kIdescPV = umma_idesc_f16(kFmt, kBM, D, 1);
    const bool leader = elect_one();
    const Desc q_desc = kmajor_desc(smem_u32(q_smem));
    const Desc ring_k = kmajor_desc(smem_u32(ring));
    const Desc ring_v = mnmajor_desc(smem_u32(ring));
    auto commit = [&](uint64_t* bar) {
      if (leader) umma_commit(bar);
    };
    int consumed = 0;                 // ring index of the item's K_0
    int q_waits[kQTiles] = {};
    int p_waits[kQTiles] = {};
    bool ok = true;
    bool issued_any = false;
    auto wait_ring = [&](int i) {
      return __all_sync(0xffffffffu, mbar_wait(&sb->kv_full[i % kSlots], (i / kSlots) & 1, guard));
    };
    auto issue_qk = [&](int t, int k_slot) {
      if (leader) {
        const Desc qd = q_desc.at(t * kTileBytes);
        const Desc kd = ring_k.at(k_slot * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_ss(tmem + t * 128, qd.at(kmajor_step(kk)).u64(), kd.at(kmajor_step(kk)).u64(),
                  kIdescQK, kk > 0);
        }
        umma_commit(&sb->s_full[t]);
      }
    };
    Item it;
    for (int k = 0; ok && item_at<kPersistent>(a, k, it); ++k) {
      if (it.qb < 0) continue;
      int n_kv_tile[kQTiles];
#pragma unroll
      for (int t = 0; t < kQTiles; ++t) n_kv_tile[t] = kv_tiles_for(a, it.qb, t);
      const int n_kv = n_kv_tile[kQTiles - 1];
      if (n_kv == 0) continue;
      issued_any = true;
      const int kbase = consumed;     // K_j at kbase + 2j, V_j at kbase + 2j + 1
      ok = wait_ring(kbase);
      if (!ok) break;
#pragma unroll
      for (int t = 0; t < kQTiles; ++t) {
        if (n_kv_tile[t] == 0) continue;
        ok = __all_sync(0xffffffffu, mbar_wait(&sb->q_full[t], q_waits[t] & 1, guard));
        if (!ok) break;
        ++q_waits[t];
        tc_fence_after();
        issue_qk(t, kbase % kSlots);
        if (kPersistent && n_kv_tile[t] == 1) commit(&sb->q_free[t]);   // last Q K^T
      }
      if (!ok) break;
      commit(&sb->kv_empty[kbase % kSlots]);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int iv = kbase + 2 * j + 1;  // V_j ring index
        const int sv = iv % kSlots;
        const int ik = iv + 1;             // K_{j+1} ring index
        const int sk = ik % kSlots;
        ok = wait_ring(iv);
        if (!ok) break;
        bool k_ready = false;
#pragma unroll
        for (int t = 0; t < kQTiles; ++t) {
          if (j < n_kv_tile[t]) {
            // P arrives in kPChunks chunks of keys; each chunk's k-steps are issued as soon as
            // the softmax warpgroup has stored it.
#pragma unroll
            for (int ch = 0; ch < kPChunks; ++ch) {
              ok = __all_sync(0xffffffffu, mbar_wait(&sb->p_half[t][ch], p_waits[t] & 1, guard));
              if (!ok) break;
              tc_fence_after();
              if (leader) {
                const Desc vd = ring_v.at(sv * kTileBytes);
#pragma unroll
                for (int kq = 0; kq < kBN / 16 / kPChunks; ++kq) {
                  const int kk = ch * (kBN / 16 / kPChunks) + kq;
                  umma_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8,
                          vd.at(mnmajor_step(kk)).u64(), kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
                }
              }
            }
            if (!ok) break;
            ++p_waits[t];
          }
          // V_j is released once the last tile that uses it (always tile 1, whose range is the
          // item's) has its PV issued; K_{j+1} once tile 1's S for it is issued.
          if (t == kQTiles - 1) commit(&sb->kv_empty[sv]);
          if (j + 1 < n_kv_tile[t]) {
            if (!k_ready) {
              ok = wait_ring(ik);
              if (!ok) break;
              tc_fence_after();
              k_ready = true;
            }
            issue_qk(t, sk);
            if (kPersistent && j + 2 == n_kv_tile[t]) {
              commit(&sb->q_free[t]);   // its last Q K^T
            }
          } else if (j + 1 == n_kv_tile[t]) {
            commit(&sb->o_full[t]);
          }
          if (t == kQTiles - 1 && j + 1 < n_kv) commit(&sb->kv_empty[sk]);
        }
      }
      consumed = kbase + 2 * n_kv;
    }
    // Every MMA issued has completed before TMEM may be released.
    if (issued_any) {
      commit(&sb->mma_done);
      mbar_wait(&sb->mma_done, 0, guard);
    }
  } else if (warp < kProducerWarp) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(RegSplit<kPersistent>::kSoftmax));
    // ------------------------------- softmax warpgroups -------------------------------
    const int t = warp >> 2;                  // Q tile of this warpgroup
    const int quarter = warp & 3;             // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t taddr_s = tmem + t * 128 + lane_field;
    const uint32_t taddr_o = tmem + 256 + t * 128 + lane_field;
    const float sl2 = a.scale_log2;
    int s_waits = 0, o_waits = 0;
    bool ok = true;
    Item it;
    for (int k = 0; ok && item_at<kPersistent>(a, k, it); ++k) {
      if (it.qb < 0) continue;
      const int b = it.bh / a.heads, h = it.bh - b * a.heads;
      const int tile_row0 = it.qb * kRowsPerCta + t * kBM;   // first row of this Q tile
      const int row = tile_row0 + row_in_tile;
      const int n_kv_t = kv_tiles_for(a, it.qb, t);

      float m_ref = -INFINITY;  // log2-domain reference point of this row
      float l_sum = 0.f;
      for (int j = 0; j < n_kv_t; ++j) {
        if (!mbar_wait(&sb->s_full[t], s_waits & 1, guard)) {
          ok = false;
          break;
        }
        ++s_waits;
        tc_fence_after();
        uint32_t s[128];
        tmem_ld32(taddr_s + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tmem_ld32(taddr_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        tmem_ld32(taddr_s + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
        tmem_ld32(taddr_s + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
        tmem_ld_wait();
        float* sf = reinterpret_cast<float*>(s);

        const int k0 = j * kBN;
        const bool tile_needs_mask =
            (k0 + kBN > a.seqlen_k) || (a.causal && k0 + kBN - 1 > tile_row0 + a.causal_offset);
        if (tile_needs_mask) {
          const int limit = min(a.seqlen_k, a.causal ? row + a.causal_offset + 1 : a.seqlen_k);
          const int visible = limit - k0;  // keys [k0, k0 + visible) are visible to this row
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            if (c >= visible) sf[c] = -INFINITY;
          }
        }
        // Row max: 8 independent chains of 3-input maxima over columns 16..127, seeded by 0..15.
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = fmaxf(sf[i], sf[i + 8]);
#pragma unroll
        for (int c = 16; c < 128; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = fmax3(mx8[i], sf[c + 2 * i], sf[c + 2 * i + 1]);
        }
        const float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]),
                               fmaxf(fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float mt = mx == -INFINITY ? -INFINITY : mx * sl2;

        float m_new = m_ref;
        if (m_ref == -INFINITY || mt > m_ref + kRescaleThreshold) m_new = fmaxf(m_ref, mt);
        const bool rescale = (m_new != m_ref) && (m_ref != -INFINITY);
        const float factor = rescale ? ex2(m_ref - m_new) : 1.f;
        if (rescale) l_sum *= factor;
        m_ref = m_new;
        const float ref = m_ref == -INFINITY ? 0.f : m_ref;
        if (__any_sync(0xffffffffu, rescale)) {
          // Rare: the reference point moved by more than the threshold. O holds PV through tile
          // j-1 (its completion is covered by s_full) and PV of tile j waits for the first P
          // half, so O is rescaled in place here, 16 columns at a time.
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t ov[16];
            tmem_ld16(taddr_o + c * 16, ov);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              ov[e] = __float_as_uint(__uint_as_float(ov[e]) * factor);
            }
            tmem_st16(taddr_o + c * 16, ov);
          }
        }

        // x = s * scale_log2 - ref on pairs; 2^x on the SFU for most pairs and, in tiles without
        // masked scores, with the FMA-pipe polynomial for kPolyPairs of every 8 pairs (the
        // choice is made once per tile so the unrolled loop has no branches). P is published to
        // the MMA warp in kPChunks chunks as soon as each chunk is in TMEM.
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
        const float nref = -ref;
        if (tile_needs_mask) {
          softmax_exp_store<T, 0, kPChunks>(sf, sl2, nref, ps, taddr_s, sb->p_half[t]);
        } else {
          softmax_exp_store<T, kPolyPairs, kPChunks>(sf, sl2, nref, ps, taddr_s, sb->p_half[t]);
        }
        l_sum += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      }

      // Epilogue: O / l in the input dtype, and the natural-log LSE. Reading O (tcgen05.ld +
      // wait) happens before this warpgroup publishes the next item's first P, which the next
      // item's first P V (accumulate = 0) waits for.
      if (ok && n_kv_t > 0) {
        ok = mbar_wait(&sb->o_full[t], o_waits & 1, guard);
        ++o_waits;
      }
      if (kPersistent && !ok) break;   // (the one-item form must reach its barrier below)
      tc_fence_after();
      const bool row_ok = row < a.seqlen_q;
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      if constexpr (kPersistent) {
        // One 2 D-byte row per thread (the Q buffers already hold the next item's Q).
        T* orow = static_cast<T*>(a.o) + static_cast<int64_t>(b) * a.o_batch_stride +
                  static_cast<int64_t>(row) * a.o_seq_stride +
                  static_cast<int64_t>(h) * a.o_head_stride;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          if (n_kv_t > 0) {
            tmem_ld32(taddr_o + c * 32, ov);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = 0u;
          }
          if (row_ok) {
            const float* of = reinterpret_cast<const float*>(ov);
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) dst[v] = pack8<T>(of + 8 * v, inv);
          }
        }
      } else {
        // Staged in this Q tile's buffer (free: o_full follows every MMA of the tile, its Q K^T
        // included; a Q tile without keys was never loaded) in the Q tile's swizzled layout,
        // then written by TMA stores, which clip rows past S_q.
        // Every thread of the warpgroup reaches the barrier, whatever its waits returned.
        uint8_t* stage = q_smem + t * kTileBytes;
        if (ok) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t ov[32];
            if (n_kv_t > 0) {
              tmem_ld32(taddr_o + c * 32, ov);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) ov[e] = 0u;
            }
            const float* of = reinterpret_cast<const float*>(ov);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int chunk = c * 4 + v;    // 16-byte chunk of the row: 8 per 64-column box
              *reinterpret_cast<uint4*>(stage + (chunk >> 3) * kBoxBytes + sw128_offset(
                  static_cast<uint32_t>(row_in_tile), static_cast<uint32_t>(chunk & 7))) =
                  pack8<T>(of + 8 * v, inv);
            }
          }
          fence_proxy_async_shared();
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");   // this warpgroup only
        if (threadIdx.x % 128 == 0 && ok && !sb->abort_flag) {
#pragma unroll
          for (int box = 0; box < D / 64; ++box) {
            tma_store_4d(&tmo, stage + box * kBoxBytes, box * 64,
                         tma_c(a.oc, 1, tile_row0, h, b), tma_c(a.oc, 2, tile_row0, h, b),
                         tma_c(a.oc, 3, tile_row0, h, b));
          }
          tma_store_commit();
          tma_store_wait_read();   // the CTA may exit once the stores have read the stage
        }
      }
      if (!ok) break;
      if (row_ok) {
        a.lse[(static_cast<int64_t>(b) * a.heads + h) * a.seqlen_q + row] =
            l_sum > 0.f ? m_ref * 0.69314718055994530942f + logf(l_sum) : -INFINITY;
      }
      tc_fence_before();
    }
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(RegSplit<kPersistent>::kControl));   // warps 10, 11
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// The tensor maps of a launch: q, k and v loads and the o store (one-item form).
struct Maps {
  CUtensorMap q, k, v, o;
};

// One shared-memory opt-in per (kernel instantiation, device) and host thread.
template <typename T, int D, int kPoly, bool kPersistent>
int launch_variant(const PrefillArgs& a, const Maps& m, int grid, int dev, cudaStream_t stream) {
  constexpr int kSmemBytes = Geometry<D>::kSmemBytes;
  auto kernel = prefill_kernel<T, D, kPoly, kDefaultPChunks, kPersistent>;
  static thread_local int configured_device = -1;
  if (configured_device != dev) {
    if (int st = check_cuda(cudaFuncSetAttribute(kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kSmemBytes),
                            "cudaFuncSetAttribute(prefill)"))
      return st;
    // The register split (setmaxnreg) draws on the registers the CTA is launched with; a build
    // that launched with fewer than the split hands out would wait forever in setmaxnreg.inc.
    cudaFuncAttributes attr{};
    if (int st = check_cuda(cudaFuncGetAttributes(&attr, kernel), "cudaFuncGetAttributes(prefill)"))
      return st;
    if (attr.numRegs * kThreads <
        2 * 128 * RegSplit<kPersistent>::kSoftmax + 128 * RegSplit<kPersistent>::kControl)
      return fail(FLB_ERR_CUDA, "prefill kernel built with %d registers per thread, fewer than its "
                  "register split needs", attr.numRegs);
    configured_device = dev;
  }
  kernel<<<grid, kThreads, kSmemBytes, stream>>>(a, m.q, m.k, m.v, m.o);
  return check_cuda(cudaGetLastError(), "prefill_kernel launch");
}

// Tuning knob read once per process: FLASH_LAB_PREFILL_POLY_PAIRS=0|2|3|4, the pairs of every 8
// whose 2^x runs on the FMA pipe (head_dim 128; head_dim 64 runs the default).
int poly_pairs() {
  static const int value = [] {
    const char* env = std::getenv("FLASH_LAB_PREFILL_POLY_PAIRS");
    if (env == nullptr) return kDefaultPolyPairs;
    const int v = std::atoi(env);
    return (v == 0 || v == 2 || v == 3 || v == 4) ? v : kDefaultPolyPairs;
  }();
  return value;
}

// head_dim 128: one item per CTA when non-causal, persistent CTAs when causal; head_dim 64:
// persistent CTAs (each form measured faster where it is used).
template <typename T>
int launch_prefill(const PrefillArgs& a, const Maps& m, int head_dim, int sm_count, int dev,
                   cudaStream_t stream) {
  const int64_t items = static_cast<int64_t>(a.batch) * a.heads * a.q_blocks;
  if (head_dim == 64) {
    const int64_t units = static_cast<int64_t>(a.batch) * a.heads *
                          (a.causal && !a.snake ? (a.q_blocks + 1) / 2 : a.q_blocks);
    const int grid = static_cast<int>(std::min<int64_t>(units, sm_count));
    return launch_variant<T, 64, kDefaultPolyPairs, true>(a, m, grid, dev, stream);
  }
  if (a.causal || kPersistentD128) {
    // Causal at head_dim 128: persistent CTAs, whose paired heavy / light units also even out
    // the items' lengths (measured 1058 -> 1082 TFLOP/s at (4,32,32,4096,128); non-causal
    // stays one item per CTA, 1212 against 1206 persistent).
    const int64_t units = static_cast<int64_t>(a.batch) * a.heads *
                          (a.causal && !a.snake ? (a.q_blocks + 1) / 2 : a.q_blocks);
    const int grid = static_cast<int>(std::min<int64_t>(units, sm_count));
    return launch_variant<T, 128, kDefaultPolyPairs, true>(a, m, grid, dev, stream);
  }
  const int grid = static_cast<int>(items);
  switch (poly_pairs()) {
    case 0: return launch_variant<T, 128, 0, false>(a, m, grid, dev, stream);
    case 2: return launch_variant<T, 128, 2, false>(a, m, grid, dev, stream);
    case 3: return launch_variant<T, 128, 3, false>(a, m, grid, dev, stream);
    default: return launch_variant<T, 128, 4, false>(a, m, grid, dev, stream);
  }
}

int validate(const flb_attn_params* p) {
  if (p == nullptr) return fail(FLB_ERR_INVALID_ARGUMENT, "params is NULL");
  if (!p->q || !p->k || !p->v || !p->o || !p->lse)
    return fail(FLB_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (p->batch <= 0 || p->seqlen_q <= 0 || p->seqlen_k <= 0 || p->heads <= 0 ||
      p->heads_kv <= 0 || p->head_dim <= 0)
    return fail(FLB_ERR_INVALID_ARGUMENT, "empty input");
  if (p->heads % p->heads_kv != 0)
    return fail(FLB_ERR_INVALID_ARGUMENT,
                "the number of query heads (%d) must be a multiple of KV heads (%d)", p->heads,
                p->heads_kv);
  if (p->dtype != FLB_BF16 && p->dtype != FLB_FP16)
    return fail(FLB_ERR_UNSUPPORTED, "prefill takes bf16 or fp16 (dtype code %d)", p->dtype);
  if (p->head_dim != 64 && p->head_dim != 128)
    return fail(FLB_ERR_UNSUPPORTED, "unsupported head_dim %d (64 or 128)", p->head_dim);
  if (!(p->softmax_scale > 0.f))
    return fail(FLB_ERR_INVALID_ARGUMENT, "softmax_scale must be positive");
  const int64_t q_blocks = (p->seqlen_q + kRowsPerCta - 1) / kRowsPerCta;
  if (q_blocks * p->batch * p->heads > 0x7fffffffLL)
    return fail(FLB_ERR_UNSUPPORTED, "problem too large for one launch");
  if (reinterpret_cast<uintptr_t>(p->o) % 16 != 0 ||
      (p->batch > 1 && (p->o_batch_stride * 2) % 16 != 0) ||
      (p->seqlen_q > 1 && (p->o_seq_stride * 2) % 16 != 0) ||
      (p->heads > 1 && (p->o_head_stride * 2) % 16 != 0))
    return fail(FLB_ERR_MISALIGNED, "o must have 16-byte aligned rows");
  return FLB_OK;
}

}  // namespace
}  // namespace flb

using namespace flb;

extern "C" int flb_prefill_fwd(const flb_attn_params* p, flb_stream_t stream_) {
  clear_error();
  if (int st = validate(p)) return st;
  int dev = 0, sm_count = 0;
  if (int st = current_device_info(&dev, &sm_count, nullptr, nullptr)) return st;

  View4 qv{p->q, {p->batch, p->seqlen_q, p->heads, p->head_dim},
           {p->q_batch_stride, p->q_seq_stride, p->q_head_stride, 1}, 2};
  View4 kv{p->k, {p->batch, p->seqlen_k, p->heads_kv, p->head_dim},
           {p->k_batch_stride, p->k_seq_stride, p->k_head_stride, 1}, 2};
  View4 vv{p->v, {p->batch, p->seqlen_k, p->heads_kv, p->head_dim},
           {p->v_batch_stride, p->v_seq_stride, p->v_head_stride, 1}, 2};
  Maps m;
  PrefillArgs a{};
  if (!rows_16b_aligned(qv))
    return fail(FLB_ERR_MISALIGNED, "q must have 16-byte aligned rows (data pointer and strides)");
  if (!rows_16b_aligned(kv))
    return fail(FLB_ERR_MISALIGNED, "k must have 16-byte aligned rows (data pointer and strides)");
  if (!rows_16b_aligned(vv))
    return fail(FLB_ERR_MISALIGNED, "v must have 16-byte aligned rows (data pointer and strides)");
  if (int st = encode_rows_x64_map(&m.q, &a.qc, qv, kBM, p->dtype)) return st;
  if (int st = encode_rows_x64_map(&m.k, &a.kc, kv, kBN, p->dtype)) return st;
  if (int st = encode_rows_x64_map(&m.v, &a.vc, vv, kBN, p->dtype)) return st;
  View4 ov{p->o, {p->batch, p->seqlen_q, p->heads, p->head_dim},
           {p->o_batch_stride, p->o_seq_stride, p->o_head_stride, 1}, 2};
  if (int st = encode_rows_x64_map(&m.o, &a.oc, ov, kBM, p->dtype)) return st;

  a.o = p->o;
  a.lse = p->lse;
  a.status = p->status;
  a.o_batch_stride = p->o_batch_stride;
  a.o_seq_stride = p->o_seq_stride;
  a.o_head_stride = p->o_head_stride;
  a.batch = p->batch;
  a.seqlen_q = p->seqlen_q;
  a.seqlen_k = p->seqlen_k;
  a.heads = p->heads;
  a.heads_kv = p->heads_kv;
  a.group = p->heads / p->heads_kv;
  a.causal = p->causal ? 1 : 0;
  a.causal_offset = p->seqlen_k - p->seqlen_q;
  a.q_blocks = (p->seqlen_q + kRowsPerCta - 1) / kRowsPerCta;
  const int64_t kv_bytes = static_cast<int64_t>(p->batch) * p->heads_kv * p->seqlen_k *
                           p->head_dim * 2 * 2;
  a.snake = (p->causal && kv_bytes <= kSnakeMaxKvBytes) ? 1 : 0;
  a.scale = p->softmax_scale;
  a.scale_log2 = static_cast<float>(static_cast<double>(p->softmax_scale) * 1.4426950408889634);

  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (p->dtype == FLB_BF16)
    return launch_prefill<__nv_bfloat16>(a, m, p->head_dim, sm_count, dev, stream);
  return launch_prefill<__half>(a, m, p->head_dim, sm_count, dev, stream);
}

// Unit test of the tcgen05 building blocks used by prefill.cu, in isolation (one CTA):
//   s = a b^T   : TMA (SW128 boxes) -> K-major smem descriptors -> SS UMMA -> TMEM -> registers
//   o = p v     : p written into TMEM as packed 16-bit pairs (the A operand), v as an MN-major
//                 SW128 B operand -> TS UMMA -> TMEM -> registers
// The reference's counterpart is its mma.sync fragment test (csrc/prefill/mma_tile_test.cu).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "host_common.h"
#include "sm100.cuh"

namespace flb {
namespace {

constexpr int kN = 128;
constexpr int kTile = kN * kN * 2;
constexpr int kBox = kTile / 2;
constexpr int kSmem = 3 * kTile + 1024 + 128;

struct SelftestArgs {
  const __nv_bfloat16* p;
  float* s_out;
  float* o_out;
  int* status;
  TmaCoords ca, cb, cv;
};

__device__ __forceinline__ int tma_c(const TmaCoords& c, int slot, int s) {
  return c.pos_s == slot ? s : 0;
}

__global__ void __launch_bounds__(128, 1)
    selftest_kernel(const __grid_constant__ SelftestArgs args,
                    const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                    const __grid_constant__ CUtensorMap tv) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sbm = smem + kTile;
  uint8_t* sv = smem + 2 * kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 3 * kTile);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitGuard guard{abort_flag, args.status};

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[0], 3 * kTile);
    const CUtensorMap* maps[3] = {&ta, &tb, &tv};
    const TmaCoords cs[3] = {args.ca, args.cb, args.cv};
    uint8_t* dst[3] = {sa, sbm, sv};
    for (int m = 0; m < 3; ++m) {
      for (int box = 0; box < 2; ++box) {
        tma_load_4d(dst[m] + box * kBox, maps[m], &bars[0], box * 64, tma_c(cs[m], 1, 0),
                    tma_c(cs[m], 2, 0), tma_c(cs[m], 3, 0));
      }
    }
    if (mbar_wait(&bars[0], 0, guard)) {
      tc_fence_after();
      const uint32_t idesc = umma_idesc_f16(1, kN, kN, 0);
      for (int kk = 0; kk < kN / 16; ++kk) {
        const uint64_t da = umma_smem_desc_sw128(smem_u32(sa) + (kk >> 2) * kBox + (kk & 3) * 32,
                                                 16, 1024);
        const uint64_t db = umma_smem_desc_sw128(smem_u32(sbm) + (kk >> 2) * kBox + (kk & 3) * 32,
                                                 16, 1024);
        umma_ss(tmem, da, db, idesc, kk > 0);
      }
      umma_commit(&bars[1]);
    }
  }
  __syncwarp();
  const uint32_t lane_field = static_cast<uint32_t>(warp * 32) << 16;
  const int row = warp * 32 + lane;
  bool ok = mbar_wait(&bars[1], 0, guard);
  if (ok) {
    tc_fence_after();
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + lane_field + c * 32, r);
      tmem_ld_wait();
      for (int e = 0; e < 32; ++e) args.s_out[row * kN + c * 32 + e] = __uint_as_float(r[e]);
    }
    // p row -> TMEM columns 0..63 (two 16-bit values per column, lower key in the low half).
    const uint32_t* prow = reinterpret_cast<const uint32_t*>(args.p + row * kN);
    for (int c = 0; c < 2; ++c) {
      uint32_t r[32];
      for (int e = 0; e < 32; ++e) r[e] = prow[c * 32 + e];
      tmem_st32(tmem + lane_field + c * 32, r);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && ok && !*abort_flag) {
    tc_fence_after();
    const uint32_t idesc = umma_idesc_f16(1, kN, kN, 1);
    for (int kk = 0; kk < kN / 16; ++kk) {
      const uint64_t dv = umma_smem_desc_sw128(smem_u32(sv) + kk * 2048, kBox, 1024);
      umma_ts(tmem + 128, tmem + kk * 8, dv, idesc, kk > 0);
    }
    umma_commit(&bars[2]);
  }
  __syncwarp();
  if (ok && mbar_wait(&bars[2], 0, guard)) {
    tc_fence_after();
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + 128 + lane_field + c * 32, r);
      tmem_ld_wait();
      for (int e = 0; e < 32; ++e) args.o_out[row * kN + c * 32 + e] = __uint_as_float(r[e]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace
}  // namespace flb

using namespace flb;

extern "C" int flb_selftest_umma(const void* a, const void* b, const void* p, const void* v,
                                 float* s_out, float* o_out, int32_t* status,
                                 flb_stream_t stream_) {
  clear_error();
  if (!a || !b || !p || !v || !s_out || !o_out)
    return fail(FLB_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (int st = current_device_info(nullptr, nullptr, nullptr, nullptr)) return st;
  CUtensorMap ta, tb, tv;
  SelftestArgs args{};
  args.p = static_cast<const __nv_bfloat16*>(p);
  args.s_out = s_out;
  args.o_out = o_out;
  args.status = status;
  View4 va{a, {1, kN, 1, kN}, {kN * kN, kN, kN, 1}, 2};
  View4 vb{b, {1, kN, 1, kN}, {kN * kN, kN, kN, 1}, 2};
  View4 vv{v, {1, kN, 1, kN}, {kN * kN, kN, kN, 1}, 2};
  if (int st = encode_rows_x64_map(&ta, &args.ca, va, kN, FLB_BF16)) return st;
  if (int st = encode_rows_x64_map(&tb, &args.cb, vb, kN, FLB_BF16)) return st;
  if (int st = encode_rows_x64_map(&tv, &args.cv, vv, kN, FLB_BF16)) return st;
  if (int st = check_cuda(cudaFuncSetAttribute(selftest_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem),
                          "cudaFuncSetAttribute(selftest)"))
    return st;
  selftest_kernel<<<1, 128, kSmem, reinterpret_cast<cudaStream_t>(stream_)>>>(args, ta, tb, tv);
  return check_cuda(cudaGetLastError(), "selftest_kernel launch");
}

// Host-side helpers shared by the C-ABI entry points (see host_common.h).
#include "host_common.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

namespace flb {
namespace {

thread_local char g_last_error[512] = {0};

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

struct DeviceInfo {
  int sm_count = 0, major = 0, minor = 0;
  bool valid = false;
};
constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_devices_mutex;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return g_encode;
}

}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

void clear_error() { g_last_error[0] = '\0'; }

const char* g_last_error_message() { return g_last_error; }

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return FLB_OK;
  return fail(FLB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

int current_device_info(int* device, int* sm_count, int* cc_major, int* cc_minor) {
  int dev = 0;
  if (int st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  if (dev < 0 || dev >= kMaxDevices) return fail(FLB_ERR_NO_DEVICE, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_devices_mutex);
  DeviceInfo& info = g_devices[dev];
  if (!info.valid) {
    if (int st = check_cuda(
            cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount, dev),
            "cudaDeviceGetAttribute"))
      return st;
    if (int st = check_cuda(
            cudaDeviceGetAttribute(&info.major, cudaDevAttrComputeCapabilityMajor, dev),
            "cudaDeviceGetAttribute"))
      return st;
    if (int st = check_cuda(
            cudaDeviceGetAttribute(&info.minor, cudaDevAttrComputeCapabilityMinor, dev),
            "cudaDeviceGetAttribute"))
      return st;
    info.valid = true;
  }
  if (device) *device = dev;
  if (sm_count) *sm_count = info.sm_count;
  if (cc_major) *cc_major = info.major;
  if (cc_minor) *cc_minor = info.minor;
  if (info.major != 10) {
    return fail(FLB_ERR_NO_DEVICE, "this library is built for sm_100a; device %d is sm_%d%d",
                dev, info.major, info.minor);
  }
  return FLB_OK;
}

bool rows_16b_aligned(const View4& v) {
  if (reinterpret_cast<uintptr_t>(v.base) % 16 != 0) return false;
  if (v.stride[3] != 1 && v.size[3] != 1) return false;
  for (int i = 0; i < 3; ++i) {
    if (v.size[i] > 1 && (v.stride[i] * v.elem_bytes) % 16 != 0) return false;
  }
  return true;
}

int encode_rows_x64_map(CUtensorMap* map, TmaCoords* coords, const View4& v, int box_rows,
                        int dtype) {
  return encode_rows_map(map, coords, v, box_rows, 64, dtype, true);
}

int encode_rows_map(CUtensorMap* map, TmaCoords* coords, const View4& v, int box_rows,
                    int box_cols, int dtype, bool swizzle128) {
  if (!rows_16b_aligned(v)) {
    return fail(FLB_ERR_MISALIGNED,
                "tensor must have 16-byte aligned rows (data pointer and strides)");
  }
  auto encode = encoder();
  if (encode == nullptr) {
    return fail(FLB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  }
  // Outer logical dims S(1), H(2), B(0) ordered by stride; size-1 dims get a harmless stride.
  int order[3] = {1, 2, 0};
  int64_t eff_stride[4];
  for (int i = 0; i < 4; ++i) eff_stride[i] = v.stride[i];
  for (int i = 0; i < 3; ++i) {
    if (v.size[i] <= 1) eff_stride[i] = -1;  // placed last, stride fixed below
  }
  for (int a = 0; a < 3; ++a) {
    for (int b = a + 1; b < 3; ++b) {
      const int64_t sa = eff_stride[order[a]] < 0 ? INT64_MAX : eff_stride[order[a]];
      const int64_t sb = eff_stride[order[b]] < 0 ? INT64_MAX : eff_stride[order[b]];
      if (sb < sa) {
        int t = order[a];
        order[a] = order[b];
        order[b] = t;
      }
    }
  }
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  cuuint32_t box[4];
  cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  dims[0] = static_cast<cuuint64_t>(v.size[3]);
  box[0] = static_cast<cuuint32_t>(box_cols);
  int64_t prev_bytes = v.size[3] * v.elem_bytes;
  int8_t pos[3] = {0, 0, 0};
  for (int j = 0; j < 3; ++j) {
    const int logical = order[j];
    dims[j + 1] = static_cast<cuuint64_t>(v.size[logical]);
    int64_t bytes = eff_stride[logical] < 0 ? -1 : eff_stride[logical] * v.elem_bytes;
    if (bytes < 0) {
      // Size-1 dimension: any stride works; keep it 16-byte aligned and past the previous one.
      bytes = ((prev_bytes + 15) / 16) * 16;
      if (bytes == 0) bytes = 16;
    }
    strides[j] = static_cast<cuuint64_t>(bytes);
    prev_bytes = bytes * v.size[logical];
    box[j + 1] = logical == 1 ? static_cast<cuuint32_t>(box_rows) : 1u;
    pos[logical] = static_cast<int8_t>(j + 1);
  }
  coords->pos_b = pos[0];
  coords->pos_s = pos[1];
  coords->pos_h = pos[2];
  coords->pad = 0;
  const CUtensorMapDataType type =
      dtype == FLB_FP32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
      : dtype == FLB_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = encode(map, type, 4, const_cast<void*>(v.base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(FLB_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d): dims %llu,%llu,%llu,%llu strides "
                "%llu,%llu,%llu bytes",
                static_cast<int>(r), (unsigned long long)dims[0], (unsigned long long)dims[1],
                (unsigned long long)dims[2], (unsigned long long)dims[3],
                (unsigned long long)strides[0], (unsigned long long)strides[1],
                (unsigned long long)strides[2]);
  }
  return FLB_OK;
}

int encode_rows_x64x2_map(CUtensorMap* map, TmaCoords* coords, const View4& v, int box_rows,
                          int dtype) {
  if (!rows_16b_aligned(v)) {
    return fail(FLB_ERR_MISALIGNED,
                "tensor must have 16-byte aligned rows (data pointer and strides)");
  }
  if (v.size[3] != 128 || v.elem_bytes != 2 || dtype == FLB_FP32) {
    return fail(FLB_ERR_INVALID_ARGUMENT, "two-half tensor map needs 16-bit head_dim 128");
  }
  auto encode = encoder();
  if (encode == nullptr) {
    return fail(FLB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  }
  // H (2) and B (0) after the half dimension, by increasing stride; size-1 dims get a harmless
  // 16-byte multiple stride.
  int outer[2] = {2, 0};
  auto eff = [&](int i) -> int64_t { return v.size[i] <= 1 ? INT64_MAX : v.stride[i]; };
  if (eff(outer[1]) < eff(outer[0])) std::swap(outer[0], outer[1]);
  auto bytes_of = [&](int i, int64_t fallback) -> cuuint64_t {
    if (v.size[i] <= 1) return static_cast<cuuint64_t>(fallback);
    return static_cast<cuuint64_t>(v.stride[i] * v.elem_bytes);
  };
  const int64_t row_bytes = v.stride[1] * v.elem_bytes;
  const int64_t span = std::max<int64_t>(row_bytes * std::max<int64_t>(v.size[1], 1), 256);
  cuuint64_t dims[5] = {64, static_cast<cuuint64_t>(v.size[1]), 2,
                        static_cast<cuuint64_t>(v.size[outer[0]]),
                        static_cast<cuuint64_t>(v.size[outer[1]])};
  cuuint64_t strides[4];
  strides[0] = v.size[1] <= 1 ? 256 : static_cast<cuuint64_t>(row_bytes);
  strides[1] = 128;
  strides[2] = bytes_of(outer[0], ((span + 15) / 16) * 16);
  strides[3] = bytes_of(outer[1], ((static_cast<int64_t>(strides[2]) *
                                    std::max<int64_t>(v.size[outer[0]], 1) + 15) / 16) * 16);
  cuuint32_t box[5] = {64, static_cast<cuuint32_t>(box_rows), 2, 1, 1};
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  int8_t pos[3] = {0, 0, 0};
  pos[1] = 1;
  pos[outer[0]] = 3;
  pos[outer[1]] = 4;
  coords->pos_b = pos[0];
  coords->pos_s = pos[1];
  coords->pos_h = pos[2];
  coords->pad = 0;
  const CUtensorMapDataType type =
      dtype == FLB_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = encode(map, type, 5, const_cast<void*>(v.base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(FLB_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d): dims 64,%llu,2,%llu,%llu strides "
                "%llu,%llu,%llu,%llu bytes",
                static_cast<int>(r), (unsigned long long)dims[1], (unsigned long long)dims[3],
                (unsigned long long)dims[4], (unsigned long long)strides[0],
                (unsigned long long)strides[1], (unsigned long long)strides[2],
                (unsigned long long)strides[3]);
  }
  return FLB_OK;
}

}  // namespace flb

extern "C" const char* flb_last_error(void) { return flb::g_last_error_message(); }

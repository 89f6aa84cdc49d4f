// Host-side helpers shared by the C-ABI entry points: error reporting, device queries and TMA
// tensor-map encoding for strided [B, S, H, D] views.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "flash_lab_b200.h"

namespace flb {

// Records a printf-style message for flb_last_error() on this thread and returns `status`.
int fail(int status, const char* fmt, ...);
void clear_error();
const char* g_last_error_message();

// Returns FLB_OK or FLB_ERR_CUDA with the runtime's message recorded.
int check_cuda(cudaError_t err, const char* what);

// SM count and compute capability of the current device (cached per device).
int current_device_info(int* device, int* sm_count, int* cc_major, int* cc_minor);

// A [B, S, H, D] tensor view with element strides (the D stride must be 1).
struct View4 {
  const void* base;
  int64_t size[4];    // B, S, H, D
  int64_t stride[4];  // elements
  int elem_bytes;
};

// Where each logical coordinate goes in the 4-D TMA coordinate vector (slot 0 is always D).
struct TmaCoords {
  int8_t pos_s, pos_h, pos_b, pad;
};

// Encodes a tiled TMA map over `v` whose box is [box_rows along S] x [64 along D] (one head, one
// batch), 128-byte swizzled. Outer dimensions are ordered by increasing stride. Returns FLB_OK,
// FLB_ERR_MISALIGNED or FLB_ERR_CUDA.
int encode_rows_x64_map(CUtensorMap* map, TmaCoords* coords, const View4& v, int box_rows,
                        int dtype);

// The general form: a [box_rows along S] x [box_cols along D] box, 128-byte swizzled or not
// (box_cols * element size must be a multiple of 16 bytes; 64 columns of 16-bit elements when
// swizzled).
int encode_rows_map(CUtensorMap* map, TmaCoords* coords, const View4& v, int box_rows,
                    int box_cols, int dtype, bool swizzle128);

// A 5-D map over a 16-bit `v` with head_dim 128 whose box moves a whole [box_rows x 128] tile in
// one copy: dimensions [64 columns] x [S] x [2 column halves, stride 128 bytes] x [H, B ordered
// by stride]. The box [64 x box_rows x 2] lands in shared memory as two 128-byte-swizzled
// [box_rows x 64] halves, one after the other (the layout of two encode_rows_x64_map boxes).
// Coordinates: slot 0 and slot 2 (the half) are 0; coords gives the slots of S (always 1), H
// and B (3 and 4).
int encode_rows_x64x2_map(CUtensorMap* map, TmaCoords* coords, const View4& v, int box_rows,
                          int dtype);

// The 16-byte row rule every kernel here relies on: base pointer and every stride of a dimension
// longer than 1 are multiples of 16 bytes, and the head_dim stride is 1.
bool rows_16b_aligned(const View4& v);

}  // namespace flb

// Decode without any allocation: the split-KV partials live in a static device array.
//
// flb_decode_fwd needs a workspace the caller allocates. Some callers cannot allocate at the
// point where they decode. cudaMalloc may synchronise the device, so it cannot be called while a
// stream is being captured into a CUDA graph. And a serving loop that plans all of its device
// memory up front, or a host callback that runs while another allocator holds its lock, must
// not allocate at all. flb_decode_fwd_static serves those callers: the same kernels, with the
// partials in g_decode_scratch, a file-scope array loaded with this library.
//
// Limits and caveats (also in include/flash_lab_b200.h):
//  * capacity kStaticScratchBytes (8 MiB) per device, enough for B * H * (2 splits + 1) <= 16,131
//    (head_dim 128) or 31,775 (head_dim 64); larger problems get FLB_ERR_WORKSPACE and nothing
//    runs;
//  * every GPU that loads the library holds the array until the process exits;
//  * all calls on a device share the array and it keeps the last call's contents. Nothing has to
//    start at zero: every partial slot a launch reads is written earlier in the same launch.
//    Calls that overlap on the GPU (two streams at once) race on it;
//  * the first call on a device looks up the array's device address (cudaGetSymbolAddress, with
//    that device current) and caches it, so make that first call before any stream capture.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "host_common.h"

namespace flb {
namespace {

constexpr size_t kStaticScratchBytes = 8u << 20;
constexpr int kMaxScratchDevices = 64;

// The host-side name of this array is only a stand-in for it; kernels get the device address
// that cudaGetSymbolAddress returns below.
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

void* g_scratch_ptr[kMaxScratchDevices] = {};
std::mutex g_scratch_mutex;

// Device address of g_decode_scratch on the current device (looked up once per device).
int scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxScratchDevices)
    return fail(FLB_ERR_NO_DEVICE, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    if (int st = check_cuda(cudaGetSymbolAddress(&ptr, g_decode_scratch),
                            "cudaGetSymbolAddress(g_decode_scratch)"))
      return st;
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return FLB_OK;
}

}  // namespace
}  // namespace flb

using namespace flb;

extern "C" size_t flb_decode_static_scratch_bytes(void) { return kStaticScratchBytes; }

extern "C" int flb_decode_fwd_static(const flb_decode_params* p, flb_stream_t stream) {
  clear_error();
  if (p == nullptr) return fail(FLB_ERR_INVALID_ARGUMENT, "params is NULL");
  int dev = 0, sm_count = 0;
  if (int st = current_device_info(&dev, &sm_count, nullptr, nullptr)) return st;
  const int splits =
      p->num_splits > 0 ? p->num_splits
                        : flb_decode_num_splits(p->batch, p->heads, p->heads_kv, p->head_dim,
                                                p->max_seqlen, sm_count);
  const size_t need = flb_decode_workspace_bytes(p->batch, p->heads, p->head_dim, splits);
  if (need > kStaticScratchBytes)
    return fail(FLB_ERR_WORKSPACE,
                "flb_decode_fwd_static: B=%d H=%d head_dim=%d with %d splits needs %zu bytes of "
                "scratch; the static array holds %zu (use flb_decode_fwd with a workspace)",
                p->batch, p->heads, p->head_dim, splits, need, kStaticScratchBytes);
  // num_splits stays as the caller gave it: with 0, flb_decode_fwd makes the same choices as
  // for a workspace call (split count and, for a balanced launch, one CTA per SM), so both entry
  // points compute the same partials.
  flb_decode_params q = *p;
  q.workspace = nullptr;
  q.workspace_bytes = 0;
  if (need > 0) {
    void* scratch = nullptr;
    if (int st = scratch_address(dev, &scratch)) return st;
    q.workspace = scratch;
    q.workspace_bytes = kStaticScratchBytes;
  }
  return flb_decode_fwd(&q, stream);
}

// PyTorch binding of the C ABI for eager calls (flash_lab/ops.py calls it when it is built).
//
// The same work as the ctypes path of flash_lab/ops.py (_prefill / _decode): allocate o, lse and
// the decode workspace with ATen on the inputs' device, fill flb_attn_params /
// flb_decode_params, call flb_prefill_fwd / flb_decode_fwd on the device's current stream and
// turn a nonzero status into RuntimeError with the library's message. Calling through here
// instead of ctypes keeps an eager call's host cost near the reference's C++ extension
// (csrc/bindings.cpp there), which registers its ops the same way. No kernel code is here: the
// library behind include/flash_lab_b200.h does the work.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <optional>
#include <stdexcept>
#include <string>
#include <tuple>

#include "flash_lab_b200.h"

namespace {

int dtype_code(at::ScalarType t, bool allow_fp32) {
  switch (t) {
    case at::kBFloat16: return FLB_BF16;
    case at::kHalf: return FLB_FP16;
    case at::kFloat:
      if (allow_fp32) return FLB_FP32;
      [[fallthrough]];
    default: return -1;
  }
}

// The message flash_lab/ops.py raises for a failed call: "<what>: <status>: <detail>".
[[noreturn]] void raise_status(const char* what, int status) {
  std::string msg = std::string(what) + ": " + flb_status_string(status);
  const char* detail = flb_last_error();
  if (detail != nullptr && detail[0] != '\0') msg += std::string(": ") + detail;
  throw std::runtime_error(msg);
}

flb_stream_t current_stream(const at::Tensor& t) {
  return reinterpret_cast<flb_stream_t>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

std::tuple<at::Tensor, at::Tensor> prefill(const at::Tensor& q, const at::Tensor& k,
                                           const at::Tensor& v, bool causal, double scale,
                                           int64_t status) {
  const int code = dtype_code(q.scalar_type(), false);
  if (code < 0 || k.scalar_type() != q.scalar_type() || v.scalar_type() != q.scalar_type())
    throw std::runtime_error("prefill takes bf16 or fp16 tensors of one dtype, got " +
                             std::string(c10::toString(q.scalar_type())));
  if (q.stride(-1) != 1 || k.stride(-1) != 1 || v.stride(-1) != 1)
    throw std::runtime_error("q, k, v must be contiguous in head_dim");
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t batch = q.size(0), seqlen_q = q.size(1), heads = q.size(2), head_dim = q.size(3);
  at::Tensor o = at::empty({batch, seqlen_q, heads, head_dim}, q.options());
  at::Tensor lse = at::empty({batch, heads, seqlen_q}, q.options().dtype(at::kFloat));
  flb_attn_params p{};
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.o = o.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.q_batch_stride = q.stride(0);
  p.q_seq_stride = q.stride(1);
  p.q_head_stride = q.stride(2);
  p.k_batch_stride = k.stride(0);
  p.k_seq_stride = k.stride(1);
  p.k_head_stride = k.stride(2);
  p.v_batch_stride = v.stride(0);
  p.v_seq_stride = v.stride(1);
  p.v_head_stride = v.stride(2);
  p.o_batch_stride = o.stride(0);
  p.o_seq_stride = o.stride(1);
  p.o_head_stride = o.stride(2);
  p.batch = static_cast<int32_t>(batch);
  p.seqlen_q = static_cast<int32_t>(seqlen_q);
  p.seqlen_k = static_cast<int32_t>(k.size(1));
  p.heads = static_cast<int32_t>(heads);
  p.heads_kv = static_cast<int32_t>(k.size(2));
  p.head_dim = static_cast<int32_t>(head_dim);
  p.causal = causal ? 1 : 0;
  p.dtype = code;
  p.softmax_scale = static_cast<float>(scale);
  p.status = reinterpret_cast<int32_t*>(status);
  if (int st = flb_prefill_fwd(&p, current_stream(q))) raise_status("flb_prefill_fwd", st);
  return {o, lse};
}

std::tuple<at::Tensor, at::Tensor> decode(const at::Tensor& q, const at::Tensor& k_cache,
                                          const at::Tensor& v_cache, const at::Tensor& seq_lens,
                                          const std::optional<at::Tensor>& block_tables,
                                          double scale, int64_t num_splits, bool allow_splits,
                                          int64_t status, int64_t sm_count) {
  const int code = dtype_code(q.scalar_type(), true);
  if (code < 0)
    throw std::runtime_error("decode takes bf16, fp16 or fp32, got " +
                             std::string(c10::toString(q.scalar_type())));
  // q is [B, H, D], or [B, 1, H, D] (one query token per sequence), and o takes its shape.
  const bool q4 = q.dim() == 4 && q.size(1) == 1;
  if ((q.dim() != 3 && !q4) || k_cache.dim() != 4)
    throw std::runtime_error("q must be [B, H, D], caches [B, S_max, H_kv, D]");
  if (seq_lens.scalar_type() != at::kInt || !seq_lens.is_contiguous())
    throw std::runtime_error("seq_lens must be contiguous int32");
  const c10::cuda::CUDAGuard guard(q.device());
  const int hd = q4 ? 2 : 1;   // q's head dimension
  const int64_t batch = q.size(0), heads = q.size(hd), head_dim = q.size(hd + 1);
  const int64_t heads_kv = k_cache.size(2);
  flb_decode_params p{};
  int64_t max_seqlen = k_cache.size(1);
  if (block_tables.has_value()) {
    const at::Tensor& bt = *block_tables;
    if (bt.scalar_type() != at::kInt || bt.dim() != 2 || bt.stride(1) != 1)
      throw std::runtime_error("block_tables must be [B, max_blocks] int32 with unit column stride");
    max_seqlen = bt.size(1) * k_cache.size(1);
    p.block_tables = bt.data_ptr<int32_t>();
    p.block_table_stride = bt.stride(0);
    p.page_size = static_cast<int32_t>(k_cache.size(1));
    p.num_blocks = static_cast<int32_t>(k_cache.size(0));
  }
  // num_splits 0 lets the library choose (the count of flb_decode_num_splits, and one CTA per
  // SM for a length-balanced launch); the resolved count sizes the workspace.
  int32_t splits = 1, abi_splits = 1;
  if (allow_splits) {
    if (num_splits > 0) {
      splits = abi_splits = static_cast<int32_t>(num_splits);
    } else {
      abi_splits = 0;
      splits = flb_decode_num_splits(static_cast<int32_t>(batch), static_cast<int32_t>(heads),
                                     static_cast<int32_t>(heads_kv),
                                     static_cast<int32_t>(head_dim),
                                     static_cast<int32_t>(max_seqlen),
                                     static_cast<int32_t>(sm_count));
    }
  }
  const size_t ws_bytes = flb_decode_workspace_bytes(
      static_cast<int32_t>(batch), static_cast<int32_t>(heads), static_cast<int32_t>(head_dim),
      splits);
  at::Tensor workspace;
  if (ws_bytes > 0)
    workspace = at::empty({static_cast<int64_t>(ws_bytes)}, q.options().dtype(at::kByte));
  at::Tensor o = q4 ? at::empty({batch, 1, heads, head_dim}, q.options())
                    : at::empty({batch, heads, head_dim}, q.options());
  at::Tensor lse = at::empty({batch, heads}, q.options().dtype(at::kFloat));
  p.q = q.data_ptr();
  p.k_cache = k_cache.data_ptr();
  p.v_cache = v_cache.data_ptr();
  p.o = o.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.seq_lens = seq_lens.data_ptr<int32_t>();
  p.q_batch_stride = q.stride(0);
  p.q_head_stride = q.stride(hd);
  p.k_batch_stride = k_cache.stride(0);
  p.k_seq_stride = k_cache.stride(1);
  p.k_head_stride = k_cache.stride(2);
  p.v_batch_stride = v_cache.stride(0);
  p.v_seq_stride = v_cache.stride(1);
  p.v_head_stride = v_cache.stride(2);
  p.o_batch_stride = o.stride(0);
  p.o_head_stride = o.stride(hd);
  p.batch = static_cast<int32_t>(batch);
  p.heads = static_cast<int32_t>(heads);
  p.heads_kv = static_cast<int32_t>(heads_kv);
  p.head_dim = static_cast<int32_t>(head_dim);
  p.max_seqlen = static_cast<int32_t>(max_seqlen);
  p.num_splits = abi_splits;
  p.dtype = code;
  p.softmax_scale = static_cast<float>(scale);
  p.workspace = ws_bytes > 0 ? workspace.data_ptr() : nullptr;
  p.workspace_bytes = ws_bytes;
  p.status = reinterpret_cast<int32_t*>(status);
  if (int st = flb_decode_fwd(&p, current_stream(q))) raise_status("flb_decode_fwd", st);
  return {o, lse};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "flash_lab's eager ops: ATen allocation + the sm_100a library's C ABI";
  m.def("prefill", &prefill, "o, lse of one prefill call (flb_prefill_fwd)");
  m.def("decode", &decode, "o, lse of one decode call (flb_decode_fwd)");
  m.def("abi_version", &flb_version);
}

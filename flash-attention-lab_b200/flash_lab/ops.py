"""Public entry points: drop-in for flash_lab/ops.py of tfan2437/flash-attention-lab.

The ops keep the reference's torch.library schemas (csrc/bindings.cpp:12-38 there):
    flash_lab::attention_<impl>(Tensor q, Tensor k, Tensor v, bool causal, float softmax_scale)
        -> (Tensor, Tensor)
    flash_lab::decode_<impl>(Tensor q, Tensor k_cache, Tensor v_cache, Tensor seq_lens,
        float softmax_scale, int num_splits) -> (Tensor, Tensor)
with fake (shape-only) kernels, so they trace under torch.compile(fullgraph=True) and replay in
CUDA graphs. Each op allocates its outputs and workspace with PyTorch's allocator and calls the
sm_100a library through its C ABI (flash_lab._capi) on the current stream. There is no CPU
path: without the library, or on a non-CUDA tensor, the ops raise.

Implementations (impl=): "sm100" is the tcgen05 prefill; "mma_pipelined" is kept as a name for
the same kernel so callers of the reference's op keep working. Decode has "splitkv" (split-KV with
a fixed-order merge) and "decode_inplace" (one split).
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass

import torch
from torch.utils import _python_dispatch

from flash_lab import _capi
from flash_lab.layouts import AttnShape, DecodeShape, check_attention_inputs, check_decode_inputs

try:
    _LIB = _capi.load()
except (OSError, AttributeError) as exc:
    _LIB = None
    HAS_EXTENSION = False
    EXTENSION_ERROR = str(exc)
else:
    HAS_EXTENSION = True
    EXTENSION_ERROR = ""

# The PyTorch binding of the same C ABI (binding/torch_ops.cpp, built next to the library): it
# allocates with ATen and calls flb_prefill_fwd / flb_decode_fwd from C++, which takes the ctypes
# marshalling off an eager call. It links the in-tree library, so it is used only when that is the
# library loaded (FLASH_LAB_LIBRARY not pointing elsewhere); the ctypes path below is otherwise
# the one that runs, with the same semantics.
_NATIVE = None
if HAS_EXTENSION and os.path.realpath(os.environ.get("FLASH_LAB_LIBRARY", str(_capi.LIB_PATH))) \
        == os.path.realpath(_capi.LIB_PATH):
    try:
        from flash_lab import _flash_lab_torch as _NATIVE
    except ImportError:
        _NATIVE = None

_DTYPE_CODE = {torch.bfloat16: _capi.FLB_BF16, torch.float16: _capi.FLB_FP16}
# The decode kernels also take fp32 caches (the reference's fp32 decode); prefill does not.
_DECODE_DTYPE_CODE = {**_DTYPE_CODE, torch.float32: _capi.FLB_FP32}
DEBUG = os.environ.get("FLASH_LAB_DEBUG", "0") not in ("", "0")


@dataclass(frozen=True)
class PrefillImpl:
    op: str
    dtypes: tuple
    head_dims: tuple
    gqa: bool = True
    causal_unequal_lengths: bool = True  # causal with S_q != S_k (bottom-right aligned)

    def unsupported_reason(self, shape: AttnShape, dtype: torch.dtype, causal: bool) -> str | None:
        if dtype not in self.dtypes:
            return f"dtype {dtype} is not one of {self.dtypes}"
        if shape.head_dim not in self.head_dims:
            return f"head_dim {shape.head_dim} is not one of {self.head_dims}"
        if shape.group > 1 and not self.gqa:
            return "grouped-query attention (H_kv < H) is not supported"
        if causal and shape.seqlen_q != shape.seqlen_k and not self.causal_unequal_lengths:
            return "causal attention requires S_q == S_k"
        return None


@dataclass(frozen=True)
class DecodeImpl:
    op: str
    dtypes: tuple
    head_dims: tuple
    paged_op: str | None = None   # the op taking a block table (none: paged caches unsupported)
    in_auto: bool = True

    @property
    def paged(self) -> bool:
        return self.paged_op is not None

    def unsupported_reason(self, shape: DecodeShape, dtype: torch.dtype) -> str | None:
        if dtype not in self.dtypes:
            return f"dtype {dtype} is not one of {self.dtypes}"
        if shape.head_dim not in self.head_dims:
            return f"head_dim {shape.head_dim} is not one of {self.head_dims}"
        if shape.paged and not self.paged:
            return "paged KV caches are not supported"
        if shape.paged and not (shape.page_size in (8, 16, 32) or shape.page_size % 64 == 0):
            return f"page_size {shape.page_size} is not 8, 16, 32 or a multiple of 64"
        return None


_HALF = (torch.bfloat16, torch.float16)
_DECODE_DTYPES = (torch.bfloat16, torch.float16, torch.float32)
PREFILL_IMPLS: dict[str, PrefillImpl] = {
    "sm100": PrefillImpl(op="attention_sm100", dtypes=_HALF, head_dims=(64, 128)),
    "mma_pipelined": PrefillImpl(op="attention_mma_pipelined", dtypes=_HALF,
                                 head_dims=(64, 128)),
}
DECODE_IMPLS: dict[str, DecodeImpl] = {
    "splitkv": DecodeImpl(op="decode_splitkv", dtypes=_DECODE_DTYPES, head_dims=(64, 128),
                          paged_op="decode_splitkv_paged"),
    "decode_inplace": DecodeImpl(op="decode_inplace", dtypes=_DECODE_DTYPES,
                                 head_dims=(64, 128), paged_op="decode_inplace_paged"),
}

_PREFILL_SCHEMA = "(Tensor q, Tensor k, Tensor v, bool causal, float softmax_scale) -> (Tensor, Tensor)"
_DECODE_PAGED_SCHEMA = ("(Tensor q, Tensor k_cache, Tensor v_cache, Tensor seq_lens, "
                        "Tensor block_tables, float softmax_scale, int num_splits) "
                        "-> (Tensor, Tensor)")
_DECODE_SCHEMA = ("(Tensor q, Tensor k_cache, Tensor v_cache, Tensor seq_lens, float softmax_scale,"
                  " int num_splits) -> (Tensor, Tensor)")


# ------------------------------------------------------------------------------------------------
# Plumbing shared by the op implementations
# ------------------------------------------------------------------------------------------------

_status_words: dict[int, torch.Tensor] = {}
_sm_counts: dict[int, int] = {}


def _status_ptr(device: torch.device) -> int:
    """Device status word the kernels raise on a timed-out pipeline wait (0 = healthy)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    word = _status_words.get(idx)
    if word is None:
        if torch.cuda.is_current_stream_capturing():
            return 0
        word = torch.zeros(1, dtype=torch.int32, device=device)
        _status_words[idx] = word
    return word.data_ptr()


def device_status(device: torch.device | int | None = None) -> int:
    """Reads (and clears) the status word of a device: 0, or the code of a timed-out wait."""
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, int):
        idx = device
    else:
        idx = torch.device(device).index
        idx = torch.cuda.current_device() if idx is None else idx
    word = _status_words.get(idx)
    if word is None:
        return 0
    value = int(word.item())
    word.zero_()
    return value


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(idx)
    if n is None:
        n = torch.cuda.get_device_properties(idx).multi_processor_count
        _sm_counts[idx] = n
    return n


def _raw_stream(device: torch.device) -> int:
    """The current CUDA stream of `device` as a cudaStream_t value (without building a Stream
    object)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(idx)


def _require_library() -> ctypes.CDLL:
    if _LIB is None:
        raise RuntimeError(f"the sm_100a library did not load: {EXTENSION_ERROR}")
    return _LIB


def _check(status: int, what: str, device: torch.device) -> None:
    if status != _capi.FLB_OK:
        raise RuntimeError(f"{what}: {_capi.error_message(_LIB, status)}")
    if DEBUG:
        torch.cuda.synchronize(device)
        code = device_status(device)
        if code:
            raise RuntimeError(f"{what}: a kernel pipeline wait timed out (status {code})")


class _DeviceGuard:
    """Makes `device` current for the C-ABI call when it is not already."""

    def __init__(self, device: torch.device):
        self.idx = device.index
        self.prev = None

    def __enter__(self):
        if self.idx is not None:
            cur = torch.cuda.current_device()
            if cur != self.idx:
                self.prev = cur
                torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


# ------------------------------------------------------------------------------------------------
# Op implementations (CUDA dispatch key)
# ------------------------------------------------------------------------------------------------

def _prefill(q, k, v, causal: bool, softmax_scale: float):
    lib = _require_library()
    if _NATIVE is not None:
        o, lse = _NATIVE.prefill(q, k, v, bool(causal), float(softmax_scale),
                                 _status_ptr(q.device))
        if DEBUG:
            _check(_capi.FLB_OK, "flb_prefill_fwd", q.device)
        return o, lse
    if q.dtype not in _DTYPE_CODE or k.dtype != q.dtype or v.dtype != q.dtype:
        raise RuntimeError(f"prefill takes bf16 or fp16 tensors of one dtype, got {q.dtype}")
    batch, seqlen_q, heads, head_dim = q.shape
    seqlen_k, heads_kv = k.shape[1], k.shape[2]
    o = torch.empty((batch, seqlen_q, heads, head_dim), dtype=q.dtype, device=q.device)
    lse = torch.empty((batch, heads, seqlen_q), dtype=torch.float32, device=q.device)
    p = _capi.AttnParams(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
        q.stride(0), q.stride(1), q.stride(2),
        k.stride(0), k.stride(1), k.stride(2),
        v.stride(0), v.stride(1), v.stride(2),
        o.stride(0), o.stride(1), o.stride(2),
        batch, seqlen_q, seqlen_k, heads, heads_kv, head_dim,
        1 if causal else 0, _DTYPE_CODE[q.dtype], float(softmax_scale),
        _status_ptr(q.device),
    )
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise RuntimeError("q, k, v must be contiguous in head_dim")
    with _DeviceGuard(q.device):
        status = lib.flb_prefill_fwd(ctypes.byref(p), _raw_stream(q.device))
    _check(status, "flb_prefill_fwd", q.device)
    return o, lse


def _decode(q, k_cache, v_cache, seq_lens, softmax_scale: float, num_splits: int,
            allow_splits: bool, block_tables=None):
    lib = _require_library()
    if _NATIVE is not None:
        o, lse = _NATIVE.decode(q, k_cache, v_cache, seq_lens, block_tables,
                                float(softmax_scale), int(num_splits), bool(allow_splits),
                                _status_ptr(q.device), _sm_count(q.device))
        if DEBUG:
            _check(_capi.FLB_OK, "flb_decode_fwd", q.device)
        return o, lse
    if q.dtype not in _DECODE_DTYPE_CODE:
        raise RuntimeError(f"decode takes bf16, fp16 or fp32, got {q.dtype}")
    if q.dim() != 3 or k_cache.dim() != 4:
        raise RuntimeError("q must be [B, H, D], caches [B, S_max, H_kv, D]")
    if seq_lens.dtype != torch.int32 or not seq_lens.is_contiguous():
        raise RuntimeError("seq_lens must be contiguous int32")
    batch, heads, head_dim = q.shape
    heads_kv = k_cache.shape[2]
    if block_tables is None:
        max_seqlen = k_cache.shape[1]
        paged = (0, 0, 0, 0)
    else:
        # Paged: caches [num_blocks, page_size, H_kv, D], block_tables [B, max_blocks] int32.
        if block_tables.dtype != torch.int32 or block_tables.dim() != 2 \
                or block_tables.stride(1) != 1:
            raise RuntimeError("block_tables must be [B, max_blocks] int32 with unit column stride")
        max_seqlen = block_tables.shape[1] * k_cache.shape[1]
        paged = (block_tables.data_ptr(), block_tables.stride(0), k_cache.shape[1],
                 k_cache.shape[0])
    # abi_splits 0 lets the library choose (the same count as flb_decode_num_splits, and one CTA
    # per SM for a length-balanced launch); the resolved count sizes the workspace.
    if not allow_splits:
        splits = abi_splits = 1
    elif num_splits > 0:
        splits = abi_splits = int(num_splits)
    else:
        abi_splits = 0
        splits = lib.flb_decode_num_splits(batch, heads, heads_kv, head_dim, max_seqlen,
                                           _sm_count(q.device))
    ws_bytes = lib.flb_decode_workspace_bytes(batch, heads, head_dim, splits)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    o = torch.empty((batch, heads, head_dim), dtype=q.dtype, device=q.device)
    lse = torch.empty((batch, heads), dtype=torch.float32, device=q.device)
    p = _capi.DecodeParams(
        q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(), lse.data_ptr(),
        seq_lens.data_ptr(),
        q.stride(0), q.stride(1),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
        o.stride(0), o.stride(1),
        batch, heads, heads_kv, head_dim, max_seqlen, abi_splits, _DECODE_DTYPE_CODE[q.dtype],
        float(softmax_scale),
        0 if workspace is None else workspace.data_ptr(), ws_bytes,
        _status_ptr(q.device), *paged,
    )
    with _DeviceGuard(q.device):
        status = lib.flb_decode_fwd(ctypes.byref(p), _raw_stream(q.device))
    _check(status, "flb_decode_fwd", q.device)
    return o, lse


def _prefill_fake(q, k, v, causal, softmax_scale):
    batch, seqlen_q, heads, _ = q.shape
    return q.new_empty(q.shape), q.new_empty((batch, heads, seqlen_q), dtype=torch.float32)


def _decode_fake(q, k_cache, v_cache, seq_lens, softmax_scale, num_splits):
    return q.new_empty(q.shape), q.new_empty(q.shape[:2], dtype=torch.float32)


def _decode_paged_fake(q, k_cache, v_cache, seq_lens, block_tables, softmax_scale, num_splits):
    return q.new_empty(q.shape), q.new_empty(q.shape[:2], dtype=torch.float32)


_LIBRARIES: list = []  # keeps the torch.library fragments alive


# The Python implementation behind each registered op, for the eager fast path (_call_op).
_EAGER_IMPLS: dict[str, object] = {}


def _define(name: str, schema: str, impl, fake) -> None:
    _EAGER_IMPLS[name] = impl
    if hasattr(torch.ops.flash_lab, name):
        return
    lib = torch.library.Library("flash_lab", "FRAGMENT")
    lib.define(name + schema)
    lib.impl(name, impl, "CUDA")
    _LIBRARIES.append(lib)
    torch.library.register_fake(f"flash_lab::{name}", fake, lib=lib)


def _register_ops() -> None:
    for spec in PREFILL_IMPLS.values():
        _define(spec.op, _PREFILL_SCHEMA, _prefill, _prefill_fake)
    _define("decode_splitkv", _DECODE_SCHEMA,
            lambda q, kc, vc, sl, scale, ns: _decode(q, kc, vc, sl, scale, ns, True), _decode_fake)
    _define("decode_inplace", _DECODE_SCHEMA,
            lambda q, kc, vc, sl, scale, ns: _decode(q, kc, vc, sl, scale, ns, False),
            _decode_fake)
    # Paged-cache forms (no counterpart op in the reference, whose kernels reject block tables).
    _define("decode_splitkv_paged", _DECODE_PAGED_SCHEMA,
            lambda q, kc, vc, sl, bt, scale, ns: _decode(q, kc, vc, sl, scale, ns, True, bt),
            _decode_paged_fake)
    _define("decode_inplace_paged", _DECODE_PAGED_SCHEMA,
            lambda q, kc, vc, sl, bt, scale, ns: _decode(q, kc, vc, sl, scale, ns, False, bt),
            _decode_paged_fake)


if HAS_EXTENSION:
    _register_ops()

_BUILT_OPS = frozenset(
    spec.op for spec in (*PREFILL_IMPLS.values(), *DECODE_IMPLS.values())
    if HAS_EXTENSION and hasattr(torch.ops.flash_lab, spec.op)
)


def _plain_eager() -> bool:
    """Eager mode with no torch function or dispatch mode active and no profiler (which then
    records the flash_lab:: op by name)."""
    if torch.compiler.is_compiling() or torch._C._is_torch_function_mode_enabled():
        return False
    if torch.autograd._profiler_enabled():
        return False
    return _python_dispatch._get_current_dispatch_mode() is None


def _eager_ok(args) -> bool:
    """Plain tensors in plain eager mode (_plain_eager)."""
    return _plain_eager() and all(type(a) is torch.Tensor for a in args
                                  if isinstance(a, torch.Tensor))


def _call_op(name: str, *args):
    """Runs torch.ops.flash_lab.<name>. torch.compile, tensor subclasses and torch modes go
    through the registered op; plain eager calls run the same implementation directly, without
    the dispatcher's cost (about 4 us per call)."""
    if _eager_ok(args):
        return _EAGER_IMPLS[name](*args)
    return getattr(torch.ops.flash_lab, name)(*args)


_SELECTED: dict[tuple, object] = {}
# Plain eager decode calls (no block table) by input metadata: the binding's arguments after a
# call with the same metadata passed validation (see decode()).
_DECODE_CALLS: dict[tuple, tuple] = {}


def _select_cached(kind: str, table: dict, impl: str, device: torch.device, key: tuple,
                   describe, reason_of):
    """_select, memoised on (table, impl, device type, key) once it has succeeded (key holds
    every input of reason_of: the shape, the dtype and, for prefill, causal). Failures are not
    cached, so errors come from _select in its order. Under torch.compile the selection is
    traced as written (it folds to a constant)."""
    if torch.compiler.is_compiling():
        return _select(table, impl, device, describe, reason_of)
    full = (kind, impl, device.type, key)
    spec = _SELECTED.get(full)
    if spec is None:
        spec = _select(table, impl, device, describe, reason_of)
        if len(_SELECTED) >= 4096:   # many distinct shapes: start over rather than grow
            _SELECTED.clear()
        _SELECTED[full] = spec
    return spec


def available_impls() -> dict[str, list[str]]:
    """Implementations compiled into this build, by entry point."""
    return {
        "attention": [name for name, spec in PREFILL_IMPLS.items() if spec.op in _BUILT_OPS],
        "decode": [name for name, spec in DECODE_IMPLS.items() if spec.op in _BUILT_OPS],
    }


def _select(table: dict, impl: str, device: torch.device, describe, reason_of):
    """The implementation to run (same rules and messages as the reference's ops.py:139-159)."""
    if impl != "auto" and impl not in table:
        raise ValueError(f"unknown impl {impl!r}; choose from {['auto', *table]}")
    if device.type != "cuda":
        raise ValueError(f"flash_lab kernels take CUDA tensors, got device {device}")
    missing = "" if HAS_EXTENSION else f" (the CUDA extension did not load: {EXTENSION_ERROR})"
    if impl != "auto":
        spec = table[impl]
        reason = reason_of(spec)
        if reason is not None:
            raise ValueError(f"impl {impl!r} cannot run {describe()}: {reason}")
        if spec.op not in _BUILT_OPS:
            raise RuntimeError(f"impl {impl!r} is not available in this build{missing}")
        return spec
    for spec in table.values():
        if getattr(spec, "in_auto", True) and spec.op in _BUILT_OPS and reason_of(spec) is None:
            return spec
    raise ValueError(f"no available implementation supports {describe()}{missing}")


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              softmax_scale: float | None = None, impl: str = "auto", return_lse: bool = False):
    """Attention forward. q is [B, S_q, H, D]; k and v are [B, S_k, H_kv, D] with H % H_kv == 0.

    Returns o [B, S_q, H, D] in the input dtype and, with return_lse=True, the natural-log
    log-sum-exp of each score row as fp32 [B, H, S_q]. Causal masking with S_q != S_k is
    aligned to the bottom-right corner.
    """
    shape = check_attention_inputs(q, k, v)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(shape.head_dim)
    if not scale > 0:
        raise ValueError(f"softmax_scale must be positive, got {scale}")
    spec = _select_cached(
        "attention", PREFILL_IMPLS, impl, q.device, (shape, q.dtype, bool(causal)),
        lambda: (f"dtype={q.dtype}, head_dim={shape.head_dim}, heads={shape.heads}/"
                 f"{shape.heads_kv}, S_q={shape.seqlen_q}, S_k={shape.seqlen_k}, causal={causal}"),
        lambda s: s.unsupported_reason(shape, q.dtype, causal),
    )
    out, lse = _call_op(spec.op, q, k, v, causal, scale)
    return (out, lse) if return_lse else out


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, seq_lens: torch.Tensor,
           block_tables: torch.Tensor | None = None, softmax_scale: float | None = None,
           impl: str = "auto", num_splits: int | None = None, return_lse: bool = False):
    """One decode step: each sequence's single query token attends to its first seq_lens[b] keys.

    The cache is [B, S_max, H_kv, D], read in place through its strides, or paged:
    [num_blocks, page_size, H_kv, D] with block_tables [B, max_blocks] int32 (page_size 8, 16,
    32 or a multiple of 64). seq_lens values are not checked on the host (that would force a device
    sync); the kernel clamps them to [0, S_max].
    num_splits=None lets the library choose the split count from the shapes only.
    """
    fast_key = None
    if (_NATIVE is not None and block_tables is None and not DEBUG and type(q) is torch.Tensor
            and type(k_cache) is torch.Tensor and type(v_cache) is torch.Tensor
            and type(seq_lens) is torch.Tensor and _plain_eager()):
        fast_key = (q.shape, q.stride(), q.dtype, q.device, k_cache.shape, k_cache.stride(),
                    k_cache.dtype, k_cache.device, v_cache.shape, v_cache.stride(),
                    v_cache.dtype, v_cache.device, seq_lens.shape, seq_lens.stride(),
                    seq_lens.dtype, seq_lens.device, softmax_scale, num_splits, impl)
        hit = _DECODE_CALLS.get(fast_key)
        if hit is not None:
            out, lse = _NATIVE.decode(q, k_cache, v_cache, seq_lens, None, *hit)
            return (out, lse) if return_lse else out
    q3, shape = check_decode_inputs(q, k_cache, v_cache, seq_lens, block_tables)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(shape.head_dim)
    if num_splits is not None and num_splits < 1:
        raise ValueError(f"num_splits must be positive, got {num_splits}")
    spec = _select_cached(
        "decode", DECODE_IMPLS, impl, q.device, (shape, q.dtype),
        lambda: (f"dtype={q.dtype}, head_dim={shape.head_dim}, heads={shape.heads}/"
                 f"{shape.heads_kv}, paged={shape.paged}"),
        lambda s: s.unsupported_reason(shape, q.dtype),
    )
    if fast_key is not None:
        # Validation and the implementation choice depend only on what the key holds (shapes,
        # strides, dtypes, devices and the arguments), so later calls with the same key go
        # straight to the binding with the same arguments (a [B, 1, H, D] q is passed as is; the
        # binding returns o in its shape).
        if len(_DECODE_CALLS) >= 4096:
            _DECODE_CALLS.clear()
        _DECODE_CALLS[fast_key] = (float(scale), int(num_splits or 0),
                                   spec.op != "decode_inplace", _status_ptr(q.device),
                                   _sm_count(q.device))
    if block_tables is None:
        out, lse = _call_op(spec.op, q3, k_cache, v_cache, seq_lens, scale, num_splits or 0)
    else:
        out, lse = _call_op(spec.paged_op, q3, k_cache, v_cache, seq_lens, block_tables, scale,
                            num_splits or 0)
    if q.dim() == 4:
        out = out.unsqueeze(1)
    return (out, lse) if return_lse else out

"""Long-context decode with the KV sequence split across GPUs (one process per GPU).

Each rank holds one contiguous shard of every sequence's cache, keys [offset, offset + S_shard),
as a [B, S_shard, H_kv, D] tensor (any strides the decode kernel accepts). A step runs in three
phases:

  1. partials: every rank runs the split-KV decode kernel over its shard
     (flb_decode_partials). It writes fp32 (m, l, O) partials for `splits_per_rank` key ranges
     of each (sequence, head). The shard's valid length, clamp(seq_lens - offset, 0, S_shard), is
     computed on the device, so nothing is read back to the host.
  2. exchange: an all_gather over the process group (NCCL over NVLink) gives every rank the
     partials of all ranks, in rank order.
  3. merge: flb_decode_merge combines the N * splits_per_rank partials of each (b, h) in that
     fixed global order.

The result is the same on every rank. It is bitwise equal to a single-GPU run that cuts the same
global key ranges, because the split boundaries inside a shard depend only on the shard's valid
length and the split count, and the merge order is fixed. The exchange moves
B * H * splits_per_rank * (D + 2) * 4 bytes per rank: 16.6 KB at B=1, H=32, D=128, 1 split.
There is no CPU path: the kernels are the library's, and only the collective is torch's.

No counterpart in the reference, which is single-GPU (README.md:183 there); the merge follows
its split merge (csrc/decode/decode.cu:204-228).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from flash_lab import _capi


@dataclass(frozen=True)
class ShardSpec:
    """Which keys this rank holds: [offset, offset + length) of every sequence."""

    offset: int
    length: int

    @staticmethod
    def even(max_seqlen: int, world_size: int, rank: int) -> "ShardSpec":
        """Contiguous, nearly equal shards of [0, max_seqlen) (the first ranks get the extra)."""
        base, extra = divmod(max_seqlen, world_size)
        start = rank * base + min(rank, extra)
        return ShardSpec(start, base + (1 if rank < extra else 0))


def local_lengths(seq_lens: torch.Tensor, shard: ShardSpec) -> torch.Tensor:
    """Valid keys of each sequence inside the shard, computed on the device (no host sync)."""
    return (seq_lens - shard.offset).clamp_(0, shard.length).to(torch.int32).contiguous()


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _capi.FLB_BF16
    if dtype == torch.float16:
        return _capi.FLB_FP16
    raise ValueError(f"sharded decode takes bf16 or fp16, got {dtype}")


def shard_partials(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                   local_lens: torch.Tensor, splits: int, softmax_scale: float):
    """Phase 1 on this rank: partials [B, H, splits, D] and (m, l) [B, H, splits, 2], fp32."""
    lib = _capi.load()
    batch, heads, head_dim = q.shape
    po = torch.empty((batch, heads, splits, head_dim), device=q.device, dtype=torch.float32)
    pml = torch.empty((batch, heads, splits, 2), device=q.device, dtype=torch.float32)
    p = _capi.DecodeParams(
        q.data_ptr(), k_shard.data_ptr(), v_shard.data_ptr(), 0, 0, local_lens.data_ptr(),
        q.stride(0), q.stride(1),
        k_shard.stride(0), k_shard.stride(1), k_shard.stride(2),
        v_shard.stride(0), v_shard.stride(1), v_shard.stride(2),
        0, 0,
        batch, heads, k_shard.shape[2], head_dim, k_shard.shape[1], splits, _dtype_code(q.dtype),
        float(softmax_scale), 0, 0, 0,
    )
    rc = lib.flb_decode_partials(ctypes.byref(p), 0, k_shard.shape[1], po.data_ptr(),
                                 pml.data_ptr(), torch.cuda.current_stream(q.device).cuda_stream)
    if rc != _capi.FLB_OK:
        raise RuntimeError(f"flb_decode_partials: {_capi.error_message(lib, rc)}")
    return po, pml


def merge_partials(partial_o: torch.Tensor, partial_ml: torch.Tensor, dtype: torch.dtype):
    """Phase 3: fixed-order merge of [B, H, S, D] / [B, H, S, 2] partials -> o [B, H, D], lse."""
    lib = _capi.load()
    batch, heads, splits, head_dim = partial_o.shape
    o = torch.empty((batch, heads, head_dim), device=partial_o.device, dtype=dtype)
    lse = torch.empty((batch, heads), device=partial_o.device, dtype=torch.float32)
    rc = lib.flb_decode_merge(partial_o.data_ptr(), partial_ml.data_ptr(), batch, heads,
                              head_dim, splits, _dtype_code(dtype), o.data_ptr(), o.stride(0),
                              o.stride(1), lse.data_ptr(),
                              torch.cuda.current_stream(partial_o.device).cuda_stream)
    if rc != _capi.FLB_OK:
        raise RuntimeError(f"flb_decode_merge: {_capi.error_message(lib, rc)}")
    return o, lse


def gather_in_rank_order(po: torch.Tensor, pml: torch.Tensor, group=None):
    """Phase 2: every rank's partials, concatenated along the split axis in rank order."""
    world = dist.get_world_size(group)
    batch, heads, splits, head_dim = po.shape
    packed = torch.cat([po, pml], dim=-1).contiguous()            # [B, H, S, D + 2]
    out = torch.empty((world * batch, *packed.shape[1:]), device=packed.device,
                      dtype=packed.dtype)                          # rank-major along dim 0
    dist.all_gather_into_tensor(out, packed, group=group)
    out = out.view(world, batch, heads, splits, head_dim + 2)
    merged = out.permute(1, 2, 0, 3, 4).reshape(batch, heads, world * splits, head_dim + 2)
    return merged[..., :head_dim].contiguous(), merged[..., head_dim:].contiguous()


def decode_sharded(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                   seq_lens: torch.Tensor, shard: ShardSpec, splits_per_rank: int = 1,
                   softmax_scale: float | None = None, group=None, return_lse: bool = False,
                   _partials=shard_partials, _merge=merge_partials):
    """One decode step over a KV cache split along the sequence across the ranks of `group`.

    q [B, H, D] or [B, 1, H, D] (identical on every rank); k_shard / v_shard
    [B, S_shard, H_kv, D] hold keys [shard.offset, shard.offset + shard.length) of every
    sequence; seq_lens [B] int32 are the global lengths. Returns o (q's shape) and, with
    return_lse, the natural-log LSE [B, H], on every rank.
    """
    if splits_per_rank < 1:
        raise ValueError(f"splits_per_rank must be positive, got {splits_per_rank}")
    if k_shard.shape[1] != shard.length:
        raise ValueError(f"k_shard holds {k_shard.shape[1]} keys but the shard spec says "
                         f"{shard.length}")
    q3 = q[:, 0] if q.dim() == 4 else q
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q3.shape[-1])
    lens = local_lengths(seq_lens, shard)
    po, pml = _partials(q3, k_shard, v_shard, lens, splits_per_rank, scale)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        po, pml = gather_in_rank_order(po, pml, group)
    o, lse = _merge(po, pml, q3.dtype)
    if q.dim() == 4:
        o = o.unsqueeze(1)
    return (o, lse) if return_lse else o

"""Long-context decode with the KV sequence split across GPUs (one process per GPU).

Each rank holds one contiguous shard of every sequence's cache, keys [offset, offset + S_shard),
as a [B, S_shard, H_kv, D] tensor (any strides the decode kernel accepts). A step runs in three
phases:

  1. partials: every rank runs the split-KV decode kernel over its shard
     (flb_decode_partials). It writes fp32 (m, l, O) partials for `splits_per_rank` key ranges
     of each (sequence, head). The kernel takes the global seq_lens and the shard's first key
     and clamps each length to the shard on the device (clamp(seq_lens - offset, 0, S_shard)),
     so nothing is read back to the host and no extra kernel runs.
  2. exchange: an all_gather over the process group (NCCL over NVLink) gives every rank the
     partials of all ranks, in rank order.
  3. merge: flb_decode_merge combines the N * splits_per_rank partials of each (b, h) in that
     fixed global order.

The result is the same on every rank. It is bitwise equal to a single-GPU run that cuts the same
global key ranges, because the split boundaries inside a shard depend only on the shard's valid
length and the split count, and the merge order is fixed. The exchange moves
B * H * splits_per_rank * (D + 2) * 4 bytes per rank: 16.6 KB at B=1, H=32, D=128, 1 split.
There is no CPU path: the kernels are the library's, and only the collective is torch's.

With a PeerExchange, phases 1 and 2 are one kernel: each rank's split kernel stores its partials
straight into every rank's exchange buffer over NVLink (CUDA IPC peer mappings); its last CTA to
finish then adds one arrival to this rank's counter in every buffer (release, system scope). Phase 3 waits on the
device, bounded by a timeout, until every source's counter has reached the step's expected count,
and merges; no NCCL call is on the path. Buffers alternate by step parity, so a rank that runs one
step ahead cannot overwrite partials another rank is still merging. The result is bitwise equal
to the all-gather path (same partials, same merge order).

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
    """Valid keys of each sequence inside the shard (on the device, no host sync). The kernels
    apply the same clamp themselves; this is for callers and tests."""
    return (seq_lens - shard.offset).clamp_(0, shard.length).to(torch.int32).contiguous()


def default_splits_per_rank(batch: int, heads: int, heads_kv: int, shard_length: int,
                            sm_count: int) -> int:
    """Key splits per rank for decode_sharded: one CTA per SM (the sharded kernels then run
    their deeper K/V ring), and splits of at least 512 keys. A function of shapes only, so the
    same on every rank and valid inside a captured graph."""
    units = batch * heads_kv * -(-(heads // heads_kv) // 16)
    return max(1, min(sm_count // max(units, 1), shard_length // 512))


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _capi.FLB_BF16
    if dtype == torch.float16:
        return _capi.FLB_FP16
    if dtype == torch.float32:
        return _capi.FLB_FP32
    raise ValueError(f"sharded decode takes bf16, fp16 or fp32, got {dtype}")


def shard_partials(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                   seq_lens: torch.Tensor, seq_offset: int, splits: int, softmax_scale: float):
    """Phase 1 on this rank: partials [B, H, splits, D] and (m, l) [B, H, splits, 2], fp32.
    seq_lens are the global lengths; the shard holds keys from seq_offset on."""
    lib = _capi.load()
    batch, heads, head_dim = q.shape
    po = torch.empty((batch, heads, splits, head_dim), device=q.device, dtype=torch.float32)
    pml = torch.empty((batch, heads, splits, 2), device=q.device, dtype=torch.float32)
    p = _capi.DecodeParams(
        q.data_ptr(), k_shard.data_ptr(), v_shard.data_ptr(), 0, 0, seq_lens.data_ptr(),
        q.stride(0), q.stride(1),
        k_shard.stride(0), k_shard.stride(1), k_shard.stride(2),
        v_shard.stride(0), v_shard.stride(1), v_shard.stride(2),
        0, 0,
        batch, heads, k_shard.shape[2], head_dim, k_shard.shape[1], splits, _dtype_code(q.dtype),
        float(softmax_scale), 0, 0, 0,
    )
    rc = lib.flb_decode_partials(ctypes.byref(p), 0, k_shard.shape[1], int(seq_offset),
                                 po.data_ptr(), pml.data_ptr(),
                                 torch.cuda.current_stream(q.device).cuda_stream)
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


class PeerExchange:
    """Exchange buffers for decode_sharded over peer memory, one per (process group, shape).

    Collective: every rank of `group` constructs it with the same shapes, with its own GPU
    current. Each rank allocates one buffer (flb_peer_alloc), the CUDA IPC handles are
    all-gathered over the process group once, and every rank maps the others' buffers. Not for
    CUDA-graph capture: the expected arrival count is a host value that grows with every step.
    """

    def __init__(self, batch: int, heads: int, head_dim: int, splits_per_rank: int = 1,
                 group=None, timeout_s: float = 2.0):
        lib = _capi.load()
        self._lib = lib
        self.group = group
        multi = dist.is_initialized() and dist.get_world_size(group) > 1
        self.world = dist.get_world_size(group) if multi else 1
        self.rank = dist.get_rank(group) if multi else 0
        if self.world > _capi.FLB_MAX_PEERS:
            raise ValueError(f"a peer exchange connects at most {_capi.FLB_MAX_PEERS} ranks, "
                             f"got {self.world}")
        self.shape = (batch, heads, head_dim, splits_per_rank)
        self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = lib.flb_peer_exchange_bytes(self.world, batch, heads, head_dim, splits_per_rank)
        if nbytes == 0:
            raise ValueError(f"bad exchange shape {self.shape}")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * lib.flb_peer_handle_bytes())()
        rc = lib.flb_peer_alloc(nbytes, ctypes.byref(own), handle)
        if rc != _capi.FLB_OK:
            raise RuntimeError(f"flb_peer_alloc: {_capi.error_message(lib, rc)}")
        self._own = own.value
        handles = [bytes(handle)]
        if multi:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        x = _capi.PeerExchange()
        x.world, x.rank, x.timeout_ns = self.world, self.rank, int(timeout_s * 1e9)
        self._opened = []
        for r in range(self.world):
            if r == self.rank:
                x.buffers[r] = self._own
                continue
            ptr = ctypes.c_void_p()
            raw = (ctypes.c_ubyte * len(handles[r])).from_buffer_copy(handles[r])
            rc = lib.flb_peer_open(raw, ctypes.byref(ptr))
            if rc != _capi.FLB_OK:
                raise RuntimeError(f"flb_peer_open(rank {r}): {_capi.error_message(lib, rc)}")
            x.buffers[r] = ptr.value
            self._opened.append(ptr.value)
        self.x = x
        self.steps = 0       # decode steps taken (selects the parity region)
        self.expected = 0    # arrivals every source counter has reached after those steps
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def read_status(self) -> int:
        """Device status of the exchange waits (0, or 2 when a peer's partials timed out);
        synchronises and clears it."""
        code = int(self.status.item())
        self.status.zero_()
        return code

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's buffer."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)      # nobody still writes into a buffer being freed
        for ptr in self._opened:
            self._lib.flb_peer_close(ptr)
        if self.world > 1:
            dist.barrier(group=self.group)
        self._lib.flb_peer_free(self._own)
        self._own = None
        self._opened = []


def _decode_sharded_peer(q3, k_shard, v_shard, seq_lens, seq_offset, splits, scale,
                         exchange: PeerExchange):
    lib = exchange._lib
    batch, heads, head_dim = q3.shape
    if exchange.shape != (batch, heads, head_dim, splits):
        raise ValueError(f"the exchange was built for (batch, heads, head_dim, splits) = "
                         f"{exchange.shape}, got {(batch, heads, head_dim, splits)}")
    stream = torch.cuda.current_stream(q3.device).cuda_stream
    p = _capi.DecodeParams(
        q3.data_ptr(), k_shard.data_ptr(), v_shard.data_ptr(), 0, 0, seq_lens.data_ptr(),
        q3.stride(0), q3.stride(1),
        k_shard.stride(0), k_shard.stride(1), k_shard.stride(2),
        v_shard.stride(0), v_shard.stride(1), v_shard.stride(2),
        0, 0,
        batch, heads, k_shard.shape[2], head_dim, k_shard.shape[1], splits, _dtype_code(q3.dtype),
        float(scale), 0, 0, exchange.status.data_ptr(),
    )
    parity = exchange.steps & 1
    rc = lib.flb_decode_partials_push(ctypes.byref(p), 0, k_shard.shape[1], int(seq_offset),
                                      ctypes.byref(exchange.x), parity, stream)
    if rc != _capi.FLB_OK:
        raise RuntimeError(f"flb_decode_partials_push: {_capi.error_message(lib, rc)}")
    exchange.expected += 1
    exchange.steps += 1
    o = torch.empty((batch, heads, head_dim), device=q3.device, dtype=q3.dtype)
    lse = torch.empty((batch, heads), device=q3.device, dtype=torch.float32)
    rc = lib.flb_decode_merge_peers(ctypes.byref(exchange.x), parity, exchange.expected, batch,
                                    heads, head_dim, splits, _dtype_code(q3.dtype), o.data_ptr(),
                                    o.stride(0), o.stride(1), lse.data_ptr(),
                                    exchange.status.data_ptr(), stream)
    if rc != _capi.FLB_OK:
        raise RuntimeError(f"flb_decode_merge_peers: {_capi.error_message(lib, rc)}")
    return o, lse


def decode_sharded(q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
                   seq_lens: torch.Tensor, shard: ShardSpec, splits_per_rank: int = 1,
                   softmax_scale: float | None = None, group=None, return_lse: bool = False,
                   exchange: PeerExchange | None = None,
                   _partials=shard_partials, _merge=merge_partials):
    """One decode step over a KV cache split along the sequence across the ranks of `group`.

    q [B, H, D] or [B, 1, H, D] (identical on every rank); k_shard / v_shard
    [B, S_shard, H_kv, D] hold keys [shard.offset, shard.offset + shard.length) of every
    sequence; seq_lens [B] int32 are the global lengths. Returns o (q's shape) and, with
    return_lse, the natural-log LSE [B, H], on every rank. With `exchange`, the partials move
    over peer memory (one fused push kernel per rank) instead of an all_gather; a wait that
    times out leaves code 2 in exchange.status (exchange.read_status()).
    """
    if splits_per_rank < 1:
        raise ValueError(f"splits_per_rank must be positive, got {splits_per_rank}")
    if k_shard.shape[1] != shard.length:
        raise ValueError(f"k_shard holds {k_shard.shape[1]} keys but the shard spec says "
                         f"{shard.length}")
    q3 = q[:, 0] if q.dim() == 4 else q
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q3.shape[-1])
    if seq_lens.dtype != torch.int32 or not seq_lens.is_contiguous():
        raise ValueError("seq_lens must be contiguous int32")
    if exchange is not None:
        o, lse = _decode_sharded_peer(q3, k_shard, v_shard, seq_lens, shard.offset,
                                      splits_per_rank, scale, exchange)
        if q.dim() == 4:
            o = o.unsqueeze(1)
        return (o, lse) if return_lse else o
    po, pml = _partials(q3, k_shard, v_shard, seq_lens, shard.offset, splits_per_rank, scale)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        po, pml = gather_in_rank_order(po, pml, group)
    o, lse = _merge(po, pml, q3.dtype)
    if q.dim() == 4:
        o = o.unsqueeze(1)
    return (o, lse) if return_lse else o

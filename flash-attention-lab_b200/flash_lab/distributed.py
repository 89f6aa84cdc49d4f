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
finish then adds one arrival to this rank's counter in every buffer (release, system scope).
Phase 3 waits on the device, bounded by a timeout, until every source's counter has reached the
step's count, and merges; no NCCL call is on the path. Buffers alternate by step parity, so a rank
that runs one step ahead cannot overwrite partials another rank is still merging. The step count
lives in device memory (the merge advances it), so a decode step with an exchange can be captured
in a CUDA graph and replayed. The result is bitwise equal to the all-gather path (same partials,
same merge order).

Prefill shards over (batch, KV head) units with no communication (attention_sharded): rank r of N
takes units [r U / N, (r + 1) U / N) of the U = B * H_kv units in batch-major order, each unit a
KV head with its query heads, as at most three rectangular views of q, k and v. Every row of the
output depends only on its own (batch, head) inputs, so the shards' outputs are bitwise those of
one unsharded call.

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


class _DeviceWords:
    """A non-owning view of n int64 words of device memory (the exchange's counter block), for
    torch.as_tensor through the CUDA array interface."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i8", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """Exchange buffers for decode_sharded over peer memory, one per (process group, shape).

    Collective: every rank of `group` constructs it with the same shapes, with its own GPU
    current. Each rank allocates one buffer (flb_peer_alloc), the CUDA IPC handles are
    all-gathered over the process group once, and every rank maps the others' buffers.

    The step count, which selects the parity region and the arrival count to wait for, is kept
    in this rank's buffer on the device, so decode_sharded(..., exchange=...) can be captured in
    a CUDA graph; every replay is one step.

    Failure is sticky. When a wait times out (a rank did not push in time), `status` gets code 2
    and that step's o and lse are NaN; from then on this rank's pushes publish nothing and its
    merges return NaN at once, so the other ranks fail the same way rather than merging stale
    partials. reset() (collective) clears the failure.
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
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        # This rank's counter block: arrivals per source, push and merge CTA counts, step count.
        self._words = torch.as_tensor(_DeviceWords(self._own, self.world + 3), device=self.device)

    def read_status(self) -> int:
        """Device status of the exchange waits (0, or 2 when a peer's partials timed out);
        synchronises. The code stays set (the exchange stays failed) until reset()."""
        return int(self.status.item())

    def steps(self) -> int:
        """Decode steps this rank has merged (read from the device; synchronises)."""
        return int(self._words[self.world + 2].item())

    def reset(self) -> None:
        """Collective: clears a failure. Every rank waits for its own work, then all zero their
        counters and status words together, so the next step starts from step 0 everywhere."""
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)   # no rank still pushes into another's counters
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = self._lib.flb_peer_exchange_reset(ctypes.byref(self.x), stream)
        if rc != _capi.FLB_OK:
            raise RuntimeError(f"flb_peer_exchange_reset: {_capi.error_message(self._lib, rc)}")
        self.status.zero_()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's buffer."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        self._words = None
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
    rc = lib.flb_decode_partials_push(ctypes.byref(p), 0, k_shard.shape[1], int(seq_offset),
                                      ctypes.byref(exchange.x), stream)
    if rc != _capi.FLB_OK:
        raise RuntimeError(f"flb_decode_partials_push: {_capi.error_message(lib, rc)}")
    o = torch.empty((batch, heads, head_dim), device=q3.device, dtype=q3.dtype)
    lse = torch.empty((batch, heads), device=q3.device, dtype=torch.float32)
    rc = lib.flb_decode_merge_peers(ctypes.byref(exchange.x), batch,
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
    over peer memory (one fused push kernel per rank) instead of an all_gather, with no host
    synchronisation and no host-side step state (the call can be captured in a CUDA graph); a
    wait that times out leaves code 2 in exchange.status and NaN in o and lse, and the exchange
    stays failed until exchange.reset().
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


# ------------------------------------------------------------------------------------------------
# Prefill sharded over (batch, KV head) units
# ------------------------------------------------------------------------------------------------

@dataclass(frozen=True)
class PrefillPiece:
    """Batches [b0, b1) x KV heads [g0, g1) (with their query heads) of one prefill problem."""

    b0: int
    b1: int
    g0: int
    g1: int

    @property
    def units(self) -> int:
        return (self.b1 - self.b0) * (self.g1 - self.g0)


def prefill_pieces(batch: int, heads_kv: int, world_size: int, rank: int) -> list[PrefillPiece]:
    """The units [rank U / N, (rank + 1) U / N) of the U = batch * heads_kv (batch, KV head)
    units, batch-major, as rectangles: the tail of a first batch, whole batches, the head of a
    last batch (at most three pieces). A function of shapes only, the same on every rank."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} of world {world_size}")
    units = batch * heads_kv
    u, u1 = rank * units // world_size, (rank + 1) * units // world_size
    pieces = []
    while u < u1:
        b, g = divmod(u, heads_kv)
        if g == 0 and u1 - u >= heads_kv:
            nb = (u1 - u) // heads_kv
            pieces.append(PrefillPiece(b, b + nb, 0, heads_kv))
            u += nb * heads_kv
        else:
            g1 = min(heads_kv, g + (u1 - u))
            pieces.append(PrefillPiece(b, b + 1, g, g1))
            u += g1 - g
    return pieces


@dataclass
class ShardedPrefill:
    """This rank's part of a sharded prefill: per piece, o [b1-b0, S_q, (g1-g0) group, D] and lse
    [b1-b0, (g1-g0) group, S_q] (fp32)."""

    shape: tuple          # (B, S_q, H, H_kv, D) of the whole problem
    world_size: int
    rank: int
    pieces: list
    outputs: list         # [(o, lse)] per piece

    def gather(self, group=None):
        """Collective: the whole o [B, S_q, H, D] and lse [B, H, S_q] on every rank (one padded
        all_gather each for o and lse). Outside the sharded step: the step itself exchanges
        nothing."""
        batch, seqlen_q, heads, heads_kv, head_dim = self.shape
        grp = heads // heads_kv
        o0 = self.outputs[0][0] if self.outputs else None
        device = o0.device if o0 is not None else torch.device("cuda", torch.cuda.current_device())
        dtype = o0.dtype if o0 is not None else torch.bfloat16
        ldtype = self.outputs[0][1].dtype if self.outputs else torch.float32
        per_unit_o = seqlen_q * grp * head_dim
        per_unit_l = grp * seqlen_q
        cap = -(-batch * heads_kv // self.world_size)     # most units any rank holds
        flat_o = torch.zeros(cap * per_unit_o, device=device, dtype=dtype)
        flat_l = torch.zeros(cap * per_unit_l, device=device, dtype=ldtype)
        at = 0
        for piece, (o, lse) in zip(self.pieces, self.outputs):
            n = piece.units
            # units in (b, g) order: o [nb, S, ng*grp, D] -> [nb, ng, S, grp, D]
            ob = o.view(piece.b1 - piece.b0, seqlen_q, piece.g1 - piece.g0, grp, head_dim)
            flat_o[at * per_unit_o:(at + n) * per_unit_o].copy_(ob.transpose(1, 2).reshape(-1))
            flat_l[at * per_unit_l:(at + n) * per_unit_l].copy_(lse.reshape(-1))
            at += n
        if self.world_size > 1:
            all_o = torch.empty(self.world_size * flat_o.numel(), device=device, dtype=dtype)
            all_l = torch.empty(self.world_size * flat_l.numel(), device=device, dtype=ldtype)
            dist.all_gather_into_tensor(all_o, flat_o, group=group)
            dist.all_gather_into_tensor(all_l, flat_l, group=group)
        else:
            all_o, all_l = flat_o, flat_l
        out = torch.empty((batch, seqlen_q, heads, head_dim), device=device, dtype=dtype)
        lse_all = torch.empty((batch, heads, seqlen_q), device=device, dtype=ldtype)
        for r in range(self.world_size):
            at = 0
            for piece in prefill_pieces(batch, heads_kv, self.world_size, r):
                n = piece.units
                nb, ng = piece.b1 - piece.b0, piece.g1 - piece.g0
                src_o = all_o[(r * cap + at) * per_unit_o:(r * cap + at + n) * per_unit_o]
                src_l = all_l[(r * cap + at) * per_unit_l:(r * cap + at + n) * per_unit_l]
                h0, h1 = piece.g0 * grp, piece.g1 * grp
                out[piece.b0:piece.b1, :, h0:h1].copy_(
                    src_o.view(nb, ng, seqlen_q, grp, head_dim).transpose(1, 2)
                    .reshape(nb, seqlen_q, ng * grp, head_dim))
                lse_all[piece.b0:piece.b1, h0:h1].copy_(src_l.view(nb, ng * grp, seqlen_q))
                at += n
        return out, lse_all


def attention_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                      softmax_scale: float | None = None, group=None,
                      world_size: int | None = None, rank: int | None = None) -> ShardedPrefill:
    """This rank's share of flash_lab.attention(q, k, v) over the ranks of `group`.

    q [B, S_q, H, D], k / v [B, S_k, H_kv, D] are the whole problem (the same on every rank; only
    the views of this rank's pieces are read). Rank r computes the (batch, KV head) units
    prefill_pieces(B, H_kv, N, r) with one flash_lab.attention call per piece on zero-copy head /
    batch slices. No communication; ShardedPrefill.gather() assembles the whole output when a
    caller needs it. world_size / rank default to the process group's.
    """
    from flash_lab import ops

    if world_size is None:
        multi = dist.is_initialized()
        world_size = dist.get_world_size(group) if multi else 1
        rank = dist.get_rank(group) if multi else 0
    elif rank is None:
        raise ValueError("rank is required with world_size")
    batch, seqlen_q, heads, head_dim = q.shape
    heads_kv = k.shape[2]
    if heads % heads_kv != 0:
        raise ValueError(f"heads {heads} must be a multiple of heads_kv {heads_kv}")
    grp = heads // heads_kv
    pieces = prefill_pieces(batch, heads_kv, world_size, rank)
    outputs = []
    for pc in pieces:
        h0, h1 = pc.g0 * grp, pc.g1 * grp
        outputs.append(ops.attention(q[pc.b0:pc.b1, :, h0:h1], k[pc.b0:pc.b1, :, pc.g0:pc.g1],
                                     v[pc.b0:pc.b1, :, pc.g0:pc.g1], causal=causal,
                                     softmax_scale=softmax_scale, return_lse=True))
    return ShardedPrefill((batch, seqlen_q, heads, heads_kv, head_dim), world_size, rank, pieces,
                          outputs)

"""Long-context decode split along the KV sequence across ranks (flash_lab.distributed).

CPU part: two gloo ranks run decode_sharded end to end with the kernel steps replaced by numpy
restatements (the oracle's partials and merge, test infrastructure only), which checks the
plumbing: shard offsets, device-side local lengths, the all_gather in rank order and the merge
layout, against the oracle's unsplit decode.

GPU part (one GPU): the real kernels on emulated shards. Partials computed shard by shard and
merged are bitwise equal to partials of the same global key windows computed on the full cache,
and within tolerance of the oracle. A two-GPU NCCL test runs when two GPUs are visible.
"""

import ctypes
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import flash_lab
import oracle
from flash_lab import _capi
from flash_lab import reference
from flash_lab.distributed import (ShardedPrefill, ShardSpec, decode_sharded,
                                   default_splits_per_rank, local_lengths, merge_partials,
                                   prefill_pieces)

TILE = 64  # keys per decode tile: split ranges are whole numbers of tiles


def numpy_partials(q3, k_shard, v_shard, seq_lens, seq_offset, splits, scale):
    """Reference partials with the kernel's split boundaries (fp64 on the CPU)."""
    lens = (seq_lens - seq_offset).clamp(0, k_shard.shape[1])
    q = q3.double().numpy()
    k = k_shard.double().numpy()
    v = v_shard.double().numpy()
    batch, heads, head_dim = q.shape
    group = heads // k.shape[2]
    po = np.zeros((batch, heads, splits, head_dim))
    pml = np.zeros((batch, heads, splits, 2))
    pml[..., 0] = -np.inf
    for b in range(batch):
        n = int(lens[b])
        if n <= 0:
            continue
        per = -(-(-(-n // splits)) // TILE) * TILE
        for s in range(splits):
            k0, k1 = s * per, min(n, s * per + per)
            if k1 <= k0:
                continue
            for h in range(heads):
                x = (k[b, k0:k1, h // group] @ q[b, h]) * scale / math.log(2.0)
                m = x.max()
                p = np.exp2(x - m)
                po[b, h, s] = p @ v[b, k0:k1, h // group]
                pml[b, h, s] = (m, p.sum())
    return torch.from_numpy(po), torch.from_numpy(pml)


def numpy_merge(po, pml, dtype):
    o, lse = oracle.merge_partials(po.numpy(), pml[..., 0].numpy(), pml[..., 1].numpy())
    return torch.from_numpy(o), torch.from_numpy(lse)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_rank(rank, world, port, inputs, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kc, vc, lens = inputs
        shard = ShardSpec.even(kc.shape[1], world, rank)
        k_shard = kc[:, shard.offset:shard.offset + shard.length]
        v_shard = vc[:, shard.offset:shard.offset + shard.length]
        o, lse = decode_sharded(q, k_shard, v_shard, lens, shard, splits_per_rank=3,
                                return_lse=True, _partials=numpy_partials, _merge=numpy_merge)
        results[rank] = (o.numpy(), lse.numpy())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_the_oracle():
    gen = torch.Generator().manual_seed(0)
    batch, heads, heads_kv, smax, d = 2, 4, 2, 500, 16
    q = torch.randn(batch, heads, d, generator=gen, dtype=torch.float64)
    kc = torch.randn(batch, smax, heads_kv, d, generator=gen, dtype=torch.float64)
    vc = torch.randn(batch, smax, heads_kv, d, generator=gen, dtype=torch.float64)
    lens = torch.tensor([500, 203], dtype=torch.int32)   # the second ends inside shard 0
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_cpu_rank, args=(r, 2, port, (q, kc, vc, lens), results))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        out = dict(results)
    ref, ref_lse = oracle.decode(q.numpy(), kc.numpy(), vc.numpy(), lens.numpy(),
                                 return_lse=True)
    for rank in range(2):
        o, lse = out[rank]
        np.testing.assert_allclose(o, ref, rtol=0, atol=1e-12)
        np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=1e-12)


def test_shards_cover_the_sequence():
    for smax, world in [(32768, 8), (1000, 3), (5, 4)]:
        shards = [ShardSpec.even(smax, world, r) for r in range(world)]
        assert shards[0].offset == 0
        assert sum(s.length for s in shards) == smax
        for a, b in zip(shards, shards[1:]):
            assert a.offset + a.length == b.offset
    lens = torch.tensor([0, 10, 600, 1000], dtype=torch.int32)
    got = local_lengths(lens, ShardSpec(334, 333))
    assert got.tolist() == [0, 0, 266, 333]


def test_default_splits_per_rank():
    # One CTA per SM over batch * KV heads * head chunks, splits of at least 512 keys.
    assert default_splits_per_rank(1, 32, 32, 16384, 148) == 4
    assert default_splits_per_rank(1, 32, 32, 4096, 148) == 4
    assert default_splits_per_rank(1, 32, 32, 1000, 148) == 1
    assert default_splits_per_rank(8, 32, 8, 32768, 148) == 2
    assert default_splits_per_rank(1, 64, 2, 4096, 148) == 8     # group 32: two head chunks
    assert default_splits_per_rank(64, 32, 8, 32768, 148) == 1   # more units than SMs


def _window_partials(q3, kc, vc, lens, key_begin, key_end, splits, scale):
    """The library's partials of one global key window on the full cache (one GPU)."""
    lib = _capi.load()
    batch, heads, head_dim = q3.shape
    po = torch.empty((batch, heads, splits, head_dim), device="cuda", dtype=torch.float32)
    pml = torch.empty((batch, heads, splits, 2), device="cuda", dtype=torch.float32)
    p = _capi.DecodeParams(
        q3.data_ptr(), kc.data_ptr(), vc.data_ptr(), 0, 0, lens.data_ptr(),
        q3.stride(0), q3.stride(1), kc.stride(0), kc.stride(1), kc.stride(2),
        vc.stride(0), vc.stride(1), vc.stride(2), 0, 0,
        batch, heads, kc.shape[2], head_dim, kc.shape[1], splits, _capi.FLB_BF16, scale, 0, 0,
        0)
    rc = lib.flb_decode_partials(ctypes.byref(p), key_begin, key_end, 0, po.data_ptr(),
                                 pml.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _capi.error_message(lib, rc)
    return po, pml


@pytest.mark.gpu
@pytest.mark.parametrize("world,splits", [(2, 1), (4, 2), (8, 1)])
def test_emulated_shards_are_bitwise_equal_to_global_windows(world, splits):
    gen = torch.Generator(device="cuda").manual_seed(world)
    batch, heads, heads_kv, smax, d = 1, 32, 32, 32768, 128
    q = torch.randn(batch, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    kc = torch.randn(batch, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    vc = torch.randn(batch, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    lens = torch.tensor([smax - 1000], device="cuda", dtype=torch.int32)
    scale = 1.0 / math.sqrt(d)
    from flash_lab.distributed import shard_partials

    shard_po, shard_pml, win_po, win_pml = [], [], [], []
    for r in range(world):
        shard = ShardSpec.even(smax, world, r)
        ks = kc[:, shard.offset:shard.offset + shard.length].contiguous()
        vs = vc[:, shard.offset:shard.offset + shard.length].contiguous()
        po, pml = shard_partials(q, ks, vs, lens, shard.offset, splits, scale)
        shard_po.append(po)
        shard_pml.append(pml)
        po, pml = _window_partials(q, kc, vc, lens, shard.offset, shard.offset + shard.length,
                                   splits, scale)
        win_po.append(po)
        win_pml.append(pml)
    o_shards, lse_shards = merge_partials(torch.cat(shard_po, 2), torch.cat(shard_pml, 2),
                                          torch.bfloat16)
    o_win, lse_win = merge_partials(torch.cat(win_po, 2), torch.cat(win_pml, 2), torch.bfloat16)
    assert torch.equal(o_shards, o_win) and torch.equal(lse_shards, lse_win)
    ref, ref_lse = oracle.decode(q.double().cpu().numpy(), kc.double().cpu().numpy(),
                                 vc.double().cpu().numpy(), lens.cpu().numpy(), return_lse=True)
    err = np.abs(o_shards.double().cpu().numpy() - ref).max()
    rounding = np.abs(torch.from_numpy(ref).bfloat16().double().numpy() - ref).max()
    assert err <= 2 * rounding, (err, rounding)
    assert np.abs(lse_shards.double().cpu().numpy() - ref_lse).max() < 1e-3


def _nccl_rank(rank, world, port, seed):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator(device="cuda").manual_seed(seed)
        q = torch.randn(1, 32, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
        kc = torch.randn(1, 8192, 8, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
        vc = torch.randn(1, 8192, 8, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
        lens = torch.tensor([8000], device="cuda", dtype=torch.int32)
        shard = ShardSpec.even(8192, world, rank)
        o = decode_sharded(q, kc[:, shard.offset:shard.offset + shard.length],
                           vc[:, shard.offset:shard.offset + shard.length], lens, shard,
                           splits_per_rank=2)
        torch.cuda.synchronize()
        ref = oracle.decode(q.double().cpu().numpy(), kc.double().cpu().numpy(),
                            vc.double().cpu().numpy(), lens.cpu().numpy())
        err = np.abs(o.double().cpu().numpy() - ref).max()
        rounding = np.abs(torch.from_numpy(ref).bfloat16().double().numpy() - ref).max()
        assert err <= 2 * rounding, (rank, err, rounding)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpus_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, 5)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0


@pytest.mark.parametrize("batch,heads_kv,world", [(4, 32, 1), (4, 32, 2), (4, 32, 8),
                                                   (4, 32, 3), (3, 5, 7), (2, 8, 16), (1, 1, 2)])
def test_prefill_pieces_cover_every_unit_once(batch, heads_kv, world):
    seen = {}
    for rank in range(world):
        pieces = prefill_pieces(batch, heads_kv, world, rank)
        assert len(pieces) <= 3
        assert sum(p.units for p in pieces) == \
            (rank + 1) * batch * heads_kv // world - rank * batch * heads_kv // world
        for p in pieces:
            for b in range(p.b0, p.b1):
                for g in range(p.g0, p.g1):
                    seen[(b, g)] = seen.get((b, g), 0) + 1
    assert seen == {(b, g): 1 for b in range(batch) for g in range(heads_kv)}


def _sharded_prefill_rank(rank, world, port, results):
    # Each rank computes its pieces with the fp64 torch reference (no GPU) and the gather puts
    # the whole output together on every rank.
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(3)
        batch, seqlen, heads, heads_kv, d = 3, 20, 6, 3, 16
        q = torch.randn(batch, seqlen, heads, d, generator=gen, dtype=torch.float64)
        k = torch.randn(batch, seqlen, heads_kv, d, generator=gen, dtype=torch.float64)
        v = torch.randn(batch, seqlen, heads_kv, d, generator=gen, dtype=torch.float64)
        grp = heads // heads_kv
        pieces = prefill_pieces(batch, heads_kv, world, rank)
        outs = []
        for pc in pieces:
            h0, h1 = pc.g0 * grp, pc.g1 * grp
            outs.append(reference.attention(q[pc.b0:pc.b1, :, h0:h1], k[pc.b0:pc.b1, :, pc.g0:pc.g1],
                                            v[pc.b0:pc.b1, :, pc.g0:pc.g1], causal=True,
                                            return_lse=True))
        sp = ShardedPrefill((batch, seqlen, heads, heads_kv, d), world, rank, pieces, outs)
        o, lse = sp.gather()
        o_ref, lse_ref = reference.attention(q, k, v, causal=True, return_lse=True)
        results[rank] = bool(torch.allclose(o, o_ref, rtol=0, atol=1e-12)
                             and torch.allclose(lse, lse_ref, rtol=0, atol=1e-12))
    finally:
        dist.destroy_process_group()


def test_sharded_prefill_gather_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_sharded_prefill_rank, args=(r, 2, port, results))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        assert dict(results) == {0: True, 1: True}


@pytest.mark.gpu
@pytest.mark.parametrize("world", [3, 8])
def test_attention_sharded_pieces_equal_the_unsharded_call(world):
    # Emulated ranks on one GPU: every piece of every rank is bitwise the matching slice of one
    # unsharded call (rows depend only on their own (batch, head) inputs).
    from flash_lab.distributed import attention_sharded

    gen = torch.Generator(device="cuda").manual_seed(5)
    batch, seqlen, heads, heads_kv, d = 3, 600, 8, 4, 128
    q = torch.randn(batch, seqlen, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    k = torch.randn(batch, seqlen, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    v = torch.randn(batch, seqlen, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    for causal in (False, True):
        o_full, lse_full = flash_lab.attention(q, k, v, causal=causal, return_lse=True)
        covered = 0
        for rank in range(world):
            sp = attention_sharded(q, k, v, causal=causal, world_size=world, rank=rank)
            for pc, (o, lse) in zip(sp.pieces, sp.outputs):
                h0, h1 = pc.g0 * 2, pc.g1 * 2
                assert torch.equal(o, o_full[pc.b0:pc.b1, :, h0:h1]), (rank, pc)
                assert torch.equal(lse, lse_full[pc.b0:pc.b1, h0:h1]), (rank, pc)
                covered += pc.units
        assert covered == batch * heads_kv
    sp = attention_sharded(q, k, v, causal=True, world_size=1, rank=0)
    o, lse = sp.gather()
    assert torch.equal(o, o_full) and torch.equal(lse, lse_full)


@pytest.mark.gpu
def test_peer_exchange_single_rank_matches_all_gather_path():
    # World of one: the push kernel writes into this rank's own exchange buffer and the merge
    # waits on its own counters. Same partials and merge order as the all_gather path: bitwise.
    from flash_lab.distributed import PeerExchange

    gen = torch.Generator(device="cuda").manual_seed(11)
    batch, heads, heads_kv, smax, d, splits = 2, 32, 8, 4096, 128, 3
    kc = torch.randn(batch, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    vc = torch.randn(batch, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    lens = torch.tensor([4000, 1234], device="cuda", dtype=torch.int32)
    shard = ShardSpec(0, smax)
    ex = PeerExchange(batch, heads, d, splits_per_rank=splits)
    try:
        for step in range(3):   # parities 0, 1, 0
            q = torch.randn(batch, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
            o_ref, lse_ref = decode_sharded(q, kc, vc, lens, shard, splits_per_rank=splits,
                                            return_lse=True)
            o, lse = decode_sharded(q, kc, vc, lens, shard, splits_per_rank=splits,
                                    return_lse=True, exchange=ex)
            assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref), step
        assert ex.read_status() == 0
        assert ex.steps() == 3
    finally:
        ex.close()


@pytest.mark.gpu
def test_peer_exchange_step_replays_from_a_cuda_graph():
    # The step count lives on the device, so a captured push + merge replays as successive
    # steps (alternating parity regions); each replay equals the all-gather path bitwise.
    from flash_lab.distributed import PeerExchange

    gen = torch.Generator(device="cuda").manual_seed(12)
    batch, heads, heads_kv, smax, d, splits = 2, 16, 4, 2048, 128, 2
    kc = torch.randn(batch, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    vc = torch.randn(batch, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    lens = torch.tensor([2000, 700], device="cuda", dtype=torch.int32)
    q = torch.randn(batch, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    shard = ShardSpec(0, smax)
    ex = PeerExchange(batch, heads, d, splits_per_rank=splits)
    try:
        decode_sharded(q, kc, vc, lens, shard, splits_per_rank=splits, exchange=ex)  # warm-up
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o_g, lse_g = decode_sharded(q, kc, vc, lens, shard, splits_per_rank=splits,
                                        return_lse=True, exchange=ex)
        for step in range(4):
            q.copy_(torch.randn(batch, heads, d, device="cuda", dtype=torch.bfloat16,
                                generator=gen))
            lens.copy_(torch.tensor([2048 - 300 * step, 1 + 200 * step], device="cuda",
                                    dtype=torch.int32))
            graph.replay()
            o_ref, lse_ref = decode_sharded(q, kc, vc, lens, shard, splits_per_rank=splits,
                                            return_lse=True)
            torch.cuda.synchronize()
            assert torch.equal(o_g, o_ref) and torch.equal(lse_g, lse_ref), step
        assert ex.read_status() == 0
        assert ex.steps() == 5          # the warm-up and four replays (capture runs nothing)
        del graph
    finally:
        ex.close()


@pytest.mark.gpu
def test_peer_exchange_wait_times_out_with_a_status():
    # A merge whose expected arrivals never come: the device wait gives up after its timeout,
    # writes status 2 and returns; the GPU stays usable.
    from flash_lab.distributed import PeerExchange

    ex = PeerExchange(1, 8, 64, splits_per_rank=1, timeout_s=0.02)
    try:
        lib = _capi.load()

        def merge_only():
            o = torch.zeros(1, 8, 64, device="cuda", dtype=torch.bfloat16)
            lse = torch.zeros(1, 8, device="cuda")
            rc = lib.flb_decode_merge_peers(ctypes.byref(ex.x), 1, 8, 64, 1, _capi.FLB_BF16,
                                            o.data_ptr(), o.stride(0), o.stride(1),
                                            lse.data_ptr(), ex.status.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
            assert rc == 0
            torch.cuda.synchronize()
            return o, lse

        o, lse = merge_only()                   # no push came: the wait times out
        assert ex.read_status() == 2
        assert torch.isnan(o).all() and torch.isnan(lse).all()
        # Sticky: the next merge fails at once (no second timeout) and the status stays.
        o, lse = merge_only()
        assert torch.isnan(o).all() and ex.read_status() == 2

        q = torch.randn(1, 1, 8, 64, device="cuda", dtype=torch.bfloat16)
        kc = torch.randn(1, 128, 8, 64, device="cuda", dtype=torch.bfloat16)
        lens = torch.tensor([100], device="cuda", dtype=torch.int32)
        # A push on a failed exchange publishes nothing: its merge fails too.
        o = decode_sharded(q, kc, kc, lens, ShardSpec(0, 128), exchange=ex)
        torch.cuda.synchronize()
        assert torch.isnan(o).all() and ex.read_status() == 2

        ex.reset()                               # clears the failure: steps work again
        assert ex.read_status() == 0 and ex.steps() == 0
        o = decode_sharded(q, kc, kc, lens, ShardSpec(0, 128), exchange=ex)
        o_ref = decode_sharded(q, kc, kc, lens, ShardSpec(0, 128))
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and ex.read_status() == 0 and ex.steps() == 1
        import flash_lab

        flash_lab.decode(q, kc, kc, lens)       # the context still works
        torch.cuda.synchronize()
    finally:
        ex.close()


def _peer_rank(rank, world, port, seed):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime

    from flash_lab.distributed import PeerExchange

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        gen = torch.Generator(device="cuda").manual_seed(seed)
        heads, heads_kv, smax, d, splits = 32, 8, 8192, 128, 2
        kc = torch.randn(2, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
        vc = torch.randn(2, smax, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
        lens = torch.tensor([8000, 3000], device="cuda", dtype=torch.int32)  # 2nd: one shard only
        shard = ShardSpec.even(smax, world, rank)
        ks = kc[:, shard.offset:shard.offset + shard.length]
        vs = vc[:, shard.offset:shard.offset + shard.length]
        ex = PeerExchange(2, heads, d, splits_per_rank=splits)
        for step in range(4):
            q = torch.randn(2, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
            o_ref, lse_ref = decode_sharded(q, ks, vs, lens, shard, splits_per_rank=splits,
                                            return_lse=True)
            o, lse = decode_sharded(q, ks, vs, lens, shard, splits_per_rank=splits,
                                    return_lse=True, exchange=ex)
            torch.cuda.synchronize()
            assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref), (rank, step)
        assert ex.read_status() == 0
        # The same step captured in a CUDA graph on both ranks and replayed: each replay is one
        # exchange step, bitwise equal to the all-gather path.
        qg = q.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o_g, lse_g = decode_sharded(qg, ks, vs, lens, shard, splits_per_rank=splits,
                                        return_lse=True, exchange=ex)
        for step in range(3):
            qg.copy_(torch.randn(2, heads, d, device="cuda", dtype=torch.bfloat16,
                                 generator=gen))
            graph.replay()
            o_ref, lse_ref = decode_sharded(qg, ks, vs, lens, shard, splits_per_rank=splits,
                                            return_lse=True)
            torch.cuda.synchronize()
            assert torch.equal(o_g, o_ref) and torch.equal(lse_g, lse_ref), (rank, "graph", step)
        assert ex.read_status() == 0 and ex.steps() == 7
        q, o = qg.clone(), o_g.clone()      # the oracle check below: the last replay's step
        del graph
        ref = oracle.decode(q.double().cpu().numpy(), kc.double().cpu().numpy(),
                            vc.double().cpu().numpy(), lens.cpu().numpy())
        err = np.abs(o.double().cpu().numpy() - ref).max()
        rounding = np.abs(torch.from_numpy(ref).bfloat16().double().numpy() - ref).max()
        assert err <= 2 * rounding, (rank, err, rounding)
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpus_over_peer_memory():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_peer_rank, args=(r, 2, port, 7)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0


def _dropout_rank(rank, world, port, results):
    # Rank 1 fails on the host before the step (an exception in its own code); rank 0 enters
    # decode_sharded and must get an error from the process group's timeout, not hang.
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    try:
        if rank == 1:
            results[rank] = "raised"
            raise RuntimeError("injected failure on rank 1")
        gen = torch.Generator().manual_seed(0)
        q = torch.randn(1, 4, 16, generator=gen, dtype=torch.float64)
        kc = torch.randn(1, 64, 2, 16, generator=gen, dtype=torch.float64)
        lens = torch.tensor([64], dtype=torch.int32)
        shard = ShardSpec.even(64, world, rank)
        try:
            decode_sharded(q, kc[:, :shard.length], kc[:, :shard.length], lens, shard,
                           _partials=numpy_partials, _merge=numpy_merge)
            results[rank] = "returned"
        except Exception as exc:  # the collective's timeout or the peer's disconnect
            results[rank] = f"error: {type(exc).__name__}"
    except RuntimeError:
        pass
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_dropout_ends_the_step_with_an_error():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_dropout_rank, args=(r, 2, port, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode is not None, "a rank hung"
        out = dict(results)
    assert out[1] == "raised"
    assert out[0].startswith("error"), out

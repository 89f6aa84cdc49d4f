"""The split-KV decode kernel through flash_lab.decode (and so the C ABI) against the numpy oracle
and the reference's golden vectors. Cases follow the reference's tests/test_decode.py: ragged
lengths, length 1, GQA groups 4 and 8, random lengths, split counts with empty splits, strided
caches, rank-3 queries, determinism, rejections; plus poisoned unused cache rows, lengths outside
[1, S_max] (clamped on the device) and the benchmark's 32K configurations checked on slices."""

import numpy as np
import pytest
import torch

import flash_lab
import oracle
from checks import check_decode, host64
from golden_io import bf16_to_f32, load, names

pytestmark = pytest.mark.gpu

IMPLS = ["decode_inplace", "splitkv"]
DTYPES = [torch.bfloat16, torch.float16, torch.float32]   # the reference's decode dtypes

CASES = [
    # batch, heads, heads_kv, max_seqlen, head_dim, seq_lens
    (1, 8, 8, 64, 64, [64]),
    (4, 8, 1, 1100, 128, [1, 5, 1023, 1100]),
    (3, 32, 4, 4097, 128, [4097, 64, 1024]),
    (2, 6, 2, 300, 64, [300, 17]),
    (2, 32, 8, 700, 128, [700, 333]),
    (16, 8, 2, 512, 64, "random"),
    (2, 64, 2, 400, 128, [400, 399]),   # group 32: two head chunks per KV head
]


def make_case(case, dtype, gen):
    batch, heads, heads_kv, max_seqlen, head_dim, lens = case
    q = torch.randn(batch, 1, heads, head_dim, device="cuda", dtype=dtype, generator=gen)
    shape = (batch, max_seqlen, heads_kv, head_dim)
    k_cache = torch.randn(shape, device="cuda", dtype=dtype, generator=gen)
    v_cache = torch.randn(shape, device="cuda", dtype=dtype, generator=gen)
    if lens == "random":
        seq_lens = torch.randint(1, max_seqlen + 1, (batch,), device="cuda", generator=gen)
    else:
        seq_lens = torch.tensor(lens, device="cuda")
    return q, k_cache, v_cache, seq_lens.to(torch.int32)


def case_id(c):
    return f"B{c[0]}-H{c[1]}-Hkv{c[2]}-S{c[3]}-D{c[4]}"


@pytest.mark.parametrize("case", CASES, ids=case_id)
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("impl", IMPLS)
def test_matches_oracle(impl, dtype, case):
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k_cache, v_cache, seq_lens = make_case(case, dtype, gen)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl, return_lse=True)
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


@pytest.mark.parametrize("name", names("decode"))
def test_matches_reference_goldens(name):
    g = load(name)
    q = torch.from_numpy(bf16_to_f32(g["q"])).to("cuda", torch.bfloat16)
    kc = torch.from_numpy(bf16_to_f32(g["k_cache"])).to("cuda", torch.bfloat16)
    vc = torch.from_numpy(bf16_to_f32(g["v_cache"])).to("cuda", torch.bfloat16)
    lens = torch.from_numpy(g["seq_lens"]).to("cuda")
    for impl in IMPLS:
        out, lse = flash_lab.decode(q, kc, vc, lens, impl=impl, return_lse=True)
        ref = g["o"]
        err = np.abs(host64(out) - ref).max()
        rounding = np.abs(torch.from_numpy(ref).to(torch.bfloat16).double().numpy() - ref).max()
        assert err <= 2 * rounding, (name, impl, err, rounding)
        assert np.abs(host64(lse) - g["lse"]).max() < 1e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32],
                         ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("num_splits", [1, 2, 8, 64, None])
def test_split_counts(num_splits, dtype):
    # More splits than tiles leaves some splits empty; they must not disturb the merge.
    gen = torch.Generator(device="cuda").manual_seed(1)
    q, k_cache, v_cache, seq_lens = make_case((3, 16, 4, 2000, 128, [2000, 40, 777]), dtype,
                                              gen)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl="splitkv",
                                num_splits=num_splits, return_lse=True)
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


# Length-balanced key ranges (16-bit caches, more than one split): the sequences' 64-key chunks
# are shared evenly among batch * num_splits CTAs per KV head, so one CTA may hold the end of one
# sequence and the start of the next, or several short sequences whole, and some CTAs may hold
# nothing. Lengths of 0 and past S_max included.
BALANCED = [
    # batch, heads, heads_kv, max_seqlen, head_dim, seq_lens, num_splits
    (8, 32, 8, 4096, 128, [4096, 1, 2, 64, 65, 0, 130, 3000], 2),
    (8, 8, 8, 1000, 64, [1000, 999, 1, 0, 5000, 63, 64, 65], 3),
    (5, 16, 2, 3000, 128, [3000, 100, 2900, 50, 1500], 7),    # group 8
    (3, 32, 2, 2048, 128, [2048, 1, 1024], 4),                  # group 16
    (2, 64, 2, 700, 128, [700, 699], 5),                         # group 32: two head chunks
    (4, 8, 4, 200, 64, [1, 2, 3, 4], 16),                        # more CTAs than chunks
    (12, 32, 4, 8192, 128, "random", 3),
]


@pytest.mark.parametrize("auto", [False, True], ids=["explicit", "auto"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16],
                         ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("case", BALANCED, ids=lambda c: case_id(c) + f"-splits{c[6]}")
def test_balanced_key_ranges(case, dtype, auto):
    # auto: the library's split count, and with it one CTA per SM (the deep K/V ring).
    gen = torch.Generator(device="cuda").manual_seed(9)
    *shape, splits = case
    splits = None if auto else splits
    q, k_cache, v_cache, seq_lens = make_case(tuple(shape), dtype, gen)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl="splitkv",
                                num_splits=splits, return_lse=True)
    again = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl="splitkv", num_splits=splits)
    assert torch.equal(out, again)
    lens = seq_lens.clamp(0, k_cache.shape[1])
    empty = (lens == 0).nonzero().flatten()
    assert torch.all(out[empty] == 0) and torch.isneginf(lse[empty]).all()
    keep = (lens > 0).nonzero().flatten()
    check_decode(out[keep], lse[keep], q[keep], k_cache[keep], v_cache[keep], lens[keep])


@pytest.mark.parametrize("num_splits", [2, None], ids=["splits2", "auto"])
@pytest.mark.parametrize("batch", [128, 130])
def test_balanced_launch_batch_limit(batch, num_splits):
    # Up to 128 sequences take the length-balanced launch; more take the uniform split.
    gen = torch.Generator(device="cuda").manual_seed(10)
    q, k_cache, v_cache, seq_lens = make_case((batch, 8, 1, 2048, 64, "random"), torch.bfloat16,
                                              gen)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl="splitkv",
                                num_splits=num_splits, return_lse=True)
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32],
                         ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("impl", IMPLS)
def test_strided_cache_and_rank3_query(impl, dtype):
    # Caches carved out of a larger allocation (every other KV head), q given as [B, H, D].
    gen = torch.Generator(device="cuda").manual_seed(2)
    big = torch.randn(2, 600, 8, 128, device="cuda", dtype=dtype, generator=gen)
    k_cache, v_cache = big[:, :, 0::2], big[:, :, 1::2]
    q = torch.randn(2, 16, 128, device="cuda", dtype=dtype, generator=gen)
    seq_lens = torch.tensor([600, 123], device="cuda", dtype=torch.int32)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl, return_lse=True)
    assert out.shape == q.shape
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32],
                         ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("impl", IMPLS)
def test_head_major_static_cache_view(impl, dtype):
    # The Hugging Face static cache: [B, H_kv, L, D] storage read as [B, L, H_kv, D].
    gen = torch.Generator(device="cuda").manual_seed(6)
    kh = torch.randn(2, 4, 1000, 128, device="cuda", dtype=dtype, generator=gen)
    vh = torch.randn(2, 4, 1000, 128, device="cuda", dtype=dtype, generator=gen)
    q = torch.randn(2, 1, 16, 128, device="cuda", dtype=dtype, generator=gen)
    seq_lens = torch.tensor([1000, 517], device="cuda", dtype=torch.int32)
    out, lse = flash_lab.decode(q, kh.transpose(1, 2), vh.transpose(1, 2), seq_lens, impl=impl,
                                return_lse=True)
    check_decode(out, lse, q, kh.transpose(1, 2), vh.transpose(1, 2), seq_lens)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32],
                         ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("impl", IMPLS)
def test_unused_rows_are_never_read(impl, dtype):
    # NaN past each sequence's length must not reach the output (0 * NaN would).
    gen = torch.Generator(device="cuda").manual_seed(7)
    q, k_cache, v_cache, seq_lens = make_case((3, 8, 2, 333, 128, [333, 70, 1]), dtype, gen)
    for b, n in enumerate(seq_lens.tolist()):
        k_cache[b, n:] = float("nan")
        v_cache[b, n:] = float("nan")
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl, return_lse=True)
    assert torch.isfinite(out).all()
    clean_k, clean_v = k_cache.nan_to_num(0.0), v_cache.nan_to_num(0.0)
    check_decode(out, lse, q, clean_k, clean_v, seq_lens)


def test_lengths_outside_the_cache_are_clamped():
    """seq_lens is never read on the host; the kernel clamps it to [0, S_max]: a length past the
    cache attends to every row, a length of 0 gives zeros and an LSE of -inf."""
    gen = torch.Generator(device="cuda").manual_seed(8)
    q, k_cache, v_cache, _ = make_case((3, 8, 8, 200, 128, [1, 1, 1]), torch.bfloat16, gen)
    seq_lens = torch.tensor([500, 0, 50], device="cuda", dtype=torch.int32)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, return_lse=True)
    assert torch.all(out[1] == 0) and torch.isneginf(lse[1]).all()
    ref, ref_lse = oracle.decode(host64(q[[0, 2]]), host64(k_cache[[0, 2]]),
                                 host64(v_cache[[0, 2]]), np.array([200, 50]), return_lse=True)
    assert np.abs(host64(out[[0, 2]]) - ref).max() < 1e-2
    assert np.abs(host64(lse[[0, 2]]) - ref_lse).max() < 1e-3


@pytest.mark.parametrize("impl", IMPLS)
def test_deterministic(impl):
    gen = torch.Generator(device="cuda").manual_seed(3)
    q, k_cache, v_cache, seq_lens = make_case((4, 32, 8, 3000, 128, [3000, 1, 2048, 999]),
                                              torch.bfloat16, gen)
    first = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl)
    second = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl)
    assert torch.equal(first, second)


def test_auto_is_splitkv():
    gen = torch.Generator(device="cuda").manual_seed(4)
    q, k_cache, v_cache, seq_lens = make_case((2, 8, 8, 64, 64, [64, 3]), torch.bfloat16, gen)
    assert torch.equal(flash_lab.decode(q, k_cache, v_cache, seq_lens),
                       flash_lab.decode(q, k_cache, v_cache, seq_lens, impl="splitkv"))


@pytest.mark.parametrize("impl", IMPLS)
def test_rejects_unsupported(impl):
    q = torch.randn(1, 1, 4, 96, device="cuda", dtype=torch.bfloat16)
    cache = torch.randn(1, 8, 4, 96, device="cuda", dtype=torch.bfloat16)
    seq_lens = torch.tensor([8], device="cuda", dtype=torch.int32)
    with pytest.raises(ValueError, match="head_dim"):
        flash_lab.decode(q, cache, cache, seq_lens, impl=impl)
    q, cache = q[..., :64], torch.randn(4, 4, 4, 64, device="cuda", dtype=torch.bfloat16)
    tables = torch.zeros(1, 2, device="cuda", dtype=torch.int32)
    with pytest.raises(ValueError, match="page_size 4"):   # pages of 4 rows: too short here
        flash_lab.decode(q.contiguous(), cache, cache, seq_lens, block_tables=tables, impl=impl)
    q64 = torch.randn(1, 1, 4, 64, device="cuda", dtype=torch.float64)
    c64 = torch.randn(1, 8, 4, 64, device="cuda", dtype=torch.float64)
    with pytest.raises(ValueError, match="dtype"):
        flash_lab.decode(q64, c64, c64, seq_lens, impl=impl)


def _check_slices(out, lse, q, k_cache, v_cache, seq_lens, picks):
    """Oracle check of selected (b, kv head) slices of a full-size run."""
    group = q.shape[2] // k_cache.shape[2]
    for b, hkv in picks:
        hs = slice(hkv * group, (hkv + 1) * group)
        n = int(seq_lens[b])
        ref, ref_lse = oracle.decode(host64(q[b:b + 1, :, hs]),
                                     host64(k_cache[b:b + 1, :n, hkv:hkv + 1]),
                                     host64(v_cache[b:b + 1, :n, hkv:hkv + 1]), np.array([n]),
                                     return_lse=True)
        err = np.abs(host64(out[b:b + 1, :, hs]) - ref).max()
        rounding = np.abs(torch.from_numpy(ref).to(torch.bfloat16).double().numpy() - ref).max()
        assert err <= 2 * rounding, (b, hkv, err, rounding)
        assert np.abs(host64(lse[b:b + 1, hs]) - ref_lse).max() < 1e-3


def test_baseline_mha_32k():
    """The benchmark's MHA decode configuration: B=8, H=H_kv=32, D=128, S_max=32768, all 32768."""
    gen = torch.Generator(device="cuda").manual_seed(10)
    q, k_cache, v_cache, _ = make_case((8, 32, 32, 32768, 128, [1] * 8), torch.bfloat16, gen)
    seq_lens = torch.full((8,), 32768, device="cuda", dtype=torch.int32)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, return_lse=True)
    _check_slices(out, lse, q, k_cache, v_cache, seq_lens, [(0, 0), (3, 17), (7, 31)])


def test_baseline_gqa_32k_ragged():
    """The benchmark's GQA decode configuration: B=8, H=32, H_kv=8, lengths U[16384, 32768]."""
    gen = torch.Generator(device="cuda").manual_seed(11)
    q, k_cache, v_cache, _ = make_case((8, 32, 8, 32768, 128, [1] * 8), torch.bfloat16, gen)
    seq_lens = torch.randint(16384, 32769, (8,), generator=torch.Generator().manual_seed(0))
    seq_lens = seq_lens.to("cuda", torch.int32)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, return_lse=True)
    _check_slices(out, lse, q, k_cache, v_cache, seq_lens, [(0, 0), (4, 5), (7, 7)])


@pytest.mark.parametrize("group", [1, 2, 4, 8, 16])
def test_fp32_gqa_groups_8k(group):
    # fp32 caches at every register-tile size of the fp32 kernel (1, 2, 4, 8 heads per CTA; a
    # group of 16 takes two CTAs per KV head), checked in full.
    gen = torch.Generator(device="cuda").manual_seed(20 + group)
    heads_kv = 32 // group if group <= 32 else 1
    q, k_cache, v_cache, seq_lens = make_case((2, 32, heads_kv, 8192, 128, [8192, 5000]),
                                              torch.float32, gen)
    out, lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, return_lse=True)
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


def to_paged(cache, page, perm):
    """The same cache as a shuffled block pool [num_blocks, page, H_kv, D] (unused blocks NaN)."""
    batch, smax, heads_kv, d = cache.shape
    pool = torch.full((perm.numel() + 5, page, heads_kv, d), float("nan"), device=cache.device,
                      dtype=cache.dtype)
    pool[perm.reshape(-1)] = cache.reshape(batch * (smax // page), page, heads_kv, d)
    return pool


@pytest.mark.parametrize("page", [8, 16, 32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32],
                         ids=lambda d: str(d).removeprefix("torch."))
@pytest.mark.parametrize("impl", IMPLS)
def test_paged_cache_matches_contiguous(impl, dtype, page):
    # The reference's paged layout (layouts.py:95-167): block_tables [B, max_blocks] int32 into a
    # pool of pages; a shuffled pool gives bitwise the contiguous result (same keys, same splits).
    gen = torch.Generator(device="cuda").manual_seed(30 + page)
    q, k_cache, v_cache, seq_lens = make_case((3, 16, 4, 1024, 128, [1024, 37, 700]), dtype, gen)
    nb = 1024 // page
    perm = torch.randperm(3 * nb + 5, device="cuda", generator=gen)[:3 * nb].view(3, nb)
    tables = perm.to(torch.int32)
    kp, vp = to_paged(k_cache, page, perm), to_paged(v_cache, page, perm)
    # Entries past each sequence's pages point at a NaN block or out of the pool: never used.
    unused = sorted(set(range(kp.shape[0])) - set(perm.reshape(-1).tolist()))[0]
    for b, n in enumerate(seq_lens.tolist()):
        tables[b, -(-n // page):] = -1 if b % 2 else unused
    ref_o, ref_lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, impl=impl, return_lse=True)
    out, lse = flash_lab.decode(q, kp, vp, seq_lens, block_tables=tables, impl=impl,
                                return_lse=True)
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_lse)
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


@pytest.mark.parametrize("page", [8, 16, 32])
def test_paged_pool_head_major_strides(page):
    # A pool stored [num_blocks, H_kv, page, D] and passed as its [num_blocks, page, H_kv, D]
    # view: the small-page kernel's two-half tensor maps follow any strides that keep the
    # 16-byte rows, and give bitwise the contiguous-pool result.
    gen = torch.Generator(device="cuda").manual_seed(50 + page)
    q, k_cache, v_cache, seq_lens = make_case((2, 32, 8, 2048, 128, [2048, 1333]),
                                              torch.bfloat16, gen)
    nb = 2048 // page
    perm = torch.randperm(2 * nb, device="cuda", generator=gen).view(2, nb)
    tables = perm.to(torch.int32)
    kp, vp = to_paged(k_cache, page, perm), to_paged(v_cache, page, perm)
    kh = kp.transpose(1, 2).contiguous().transpose(1, 2)   # same values, head-major storage
    vh = vp.transpose(1, 2).contiguous().transpose(1, 2)
    assert kh.stride(1) == 128 and kh.stride(2) == page * 128
    ref_o, ref_lse = flash_lab.decode(q, kp, vp, seq_lens, block_tables=tables, return_lse=True)
    out, lse = flash_lab.decode(q, kh, vh, seq_lens, block_tables=tables, return_lse=True)
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_lse)
    check_decode(out, lse, q, k_cache, v_cache, seq_lens)


@pytest.mark.parametrize("page", [16, 64])
def test_paged_against_the_oracle_gqa_d64(page):
    # head_dim 64, GQA group 4, ragged lengths: the oracle reads the pool through the tables
    # (its gather_cache, pinned to the reference's paged golden case).
    gen = torch.Generator(device="cuda").manual_seed(40 + page)
    batch, heads, heads_kv, d, max_blocks = 4, 16, 4, 64, 2048 // page
    pool_k = torch.randn(batch * max_blocks + 7, page, heads_kv, d, device="cuda",
                         dtype=torch.bfloat16, generator=gen)
    pool_v = torch.randn_like(pool_k)
    tables = torch.randperm(pool_k.shape[0], device="cuda", generator=gen)[:batch * max_blocks]
    tables = tables.view(batch, max_blocks).to(torch.int32)
    q = torch.randn(batch, 1, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    seq_lens = torch.tensor([2048, 1, 1500, 999], device="cuda", dtype=torch.int32)
    out, lse = flash_lab.decode(q, pool_k, pool_v, seq_lens, block_tables=tables,
                                return_lse=True)
    ref, ref_lse = oracle.decode(host64(q), host64(pool_k), host64(pool_v),
                                 seq_lens.cpu().numpy(), block_tables=tables.cpu().numpy(),
                                 return_lse=True)
    err = np.abs(host64(out) - ref).max()
    rounding = np.abs(torch.from_numpy(ref).to(torch.bfloat16).double().numpy() - ref).max()
    assert err <= 2 * rounding, (err, rounding)
    assert np.abs(host64(lse) - ref_lse).max() < 1e-3


@pytest.mark.parametrize("fill", ["ones", "random"])
def test_balanced_decode_ignores_workspace_contents(fill):
    # Every partial slot a merge reads is written by the same call, so a workspace holding
    # anything (here all-ones bytes, or random bytes) gives the same bits as a fresh one, call
    # after call.
    import ctypes

    from flash_lab import _capi

    lib = _capi.load()
    gen = torch.Generator(device="cuda").manual_seed(22)
    q, k_cache, v_cache, seq_lens = make_case((6, 32, 8, 3000, 128, [3000, 1, 0, 2500, 64, 777]),
                                              torch.bfloat16, gen)
    ref_o, ref_lse = flash_lab.decode(q, k_cache, v_cache, seq_lens, return_lse=True)
    q3 = q[:, 0]
    batch, heads, d = q3.shape
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    splits = lib.flb_decode_num_splits(batch, heads, 8, d, k_cache.shape[1], sm)
    ws = torch.empty(lib.flb_decode_workspace_bytes(batch, heads, d, splits), device="cuda",
                     dtype=torch.uint8)
    if fill == "ones":
        ws.fill_(0xFF)
    else:
        ws.copy_(torch.randint(0, 256, ws.shape, device="cuda", generator=gen).to(torch.uint8))
    for _ in range(3):
        o = torch.empty_like(q3)
        lse = torch.empty(batch, heads, device="cuda", dtype=torch.float32)
        p = _capi.DecodeParams(
            q3.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), o.data_ptr(), lse.data_ptr(),
            seq_lens.data_ptr(), q3.stride(0), q3.stride(1),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
            o.stride(0), o.stride(1), batch, heads, 8, d, k_cache.shape[1], 0, _capi.FLB_BF16,
            1.0 / d ** 0.5, ws.data_ptr(), ws.numel(), 0)
        assert lib.flb_decode_fwd(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(o, ref_o[:, 0]) and torch.equal(lse, ref_lse)

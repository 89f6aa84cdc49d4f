"""The tcgen05 prefill kernel through flash_lab.attention (and so through the C ABI) against the
numpy oracle and the reference's golden vectors. Cases follow the reference's
tests/test_attention_fwd.py: ragged lengths, S_q != S_k with bottom-right causal masking, rows
without keys, GQA, large scores, strided packed-QKV views, determinism and rejections; plus the
benchmark's prefill configuration (4, 32, 32, 4096, 128) checked on sampled rows."""

import numpy as np
import pytest
import torch

import flash_lab
from checks import check_prefill
from golden_io import bf16_to_f32, load, manifest

pytestmark = pytest.mark.gpu

IMPLS = ["sm100", "mma_pipelined"]
DTYPES = [torch.bfloat16, torch.float16]

SHAPES = [
    # batch, seqlen_q, seqlen_k, heads, heads_kv, head_dim
    (1, 1, 1, 1, 1, 128),
    (1, 7, 7, 8, 8, 128),
    (1, 16, 16, 1, 1, 128),
    (3, 63, 63, 8, 2, 128),
    (3, 257, 257, 8, 8, 128),
    (2, 1024, 1024, 4, 4, 128),
    (2, 37, 101, 4, 2, 128),   # S_q < S_k
    (1, 101, 37, 4, 4, 128),   # S_q > S_k: causal rows without keys
    (2, 1, 300, 8, 2, 128),
    (1, 300, 300, 32, 4, 128),  # GQA group 8
    (1, 600, 129, 2, 1, 128),   # causal: whole CTAs without keys
]

# head_dim 64 (the reference's other prefill head dim; Llama-3.2-1B's attention)
SHAPES_D64 = [
    (1, 1, 1, 1, 1, 64),
    (3, 63, 63, 8, 2, 64),
    (3, 257, 257, 8, 8, 64),
    (2, 1024, 1024, 4, 4, 64),
    (2, 37, 101, 4, 2, 64),
    (1, 101, 37, 4, 4, 64),
    (1, 600, 129, 2, 1, 64),
    # more work units than SMs, so persistent CTAs run several items; causal rows < 700 see no keys
    (2, 1000, 300, 64, 8, 64),
]


def make_inputs(shape, dtype, scale=1.0, seed=0):
    batch, seqlen_q, seqlen_k, heads, heads_kv, head_dim = shape
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, seqlen_q, heads, head_dim, device="cuda", dtype=dtype,
                    generator=gen) * scale
    k = torch.randn(batch, seqlen_k, heads_kv, head_dim, device="cuda", dtype=dtype,
                    generator=gen) * scale
    v = torch.randn(batch, seqlen_k, heads_kv, head_dim, device="cuda", dtype=dtype,
                    generator=gen)
    return q, k, v


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("shape", SHAPES + SHAPES_D64, ids=str)
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d).removeprefix("torch."))
def test_matches_oracle(dtype, shape, causal):
    q, k, v = make_inputs(shape, dtype)
    out, lse = flash_lab.attention(q, k, v, causal=causal, impl="sm100", return_lse=True)
    check_prefill(out, lse, q, k, v, causal)


@pytest.mark.parametrize("impl", IMPLS)
def test_impl_names_run_the_same_kernel(impl):
    q, k, v = make_inputs((2, 200, 200, 4, 2, 128), torch.bfloat16)
    ref = flash_lab.attention(q, k, v, causal=True, impl="sm100")
    assert torch.equal(flash_lab.attention(q, k, v, causal=True, impl=impl), ref)
    assert torch.equal(flash_lab.attention(q, k, v, causal=True), ref)   # auto


GOLDEN_PREFILL = sorted(n for n, m in manifest().items() if m["kind"] == "prefill")


@pytest.mark.parametrize("name", GOLDEN_PREFILL)
def test_matches_reference_goldens(name):
    """The reference's own fp64 outputs on the committed inputs (bf16 bits)."""
    g = load(name)
    q, k, v = (torch.from_numpy(bf16_to_f32(g[x])).to("cuda", torch.bfloat16) for x in "qkv")
    for tag, causal in (("full", False), ("causal", True)):
        out, lse = flash_lab.attention(q, k, v, causal=causal, return_lse=True)
        ref = g[f"o_{tag}"]
        err = np.abs(out.double().cpu().numpy() - ref).max()
        rounding = np.abs(torch.from_numpy(ref).to(torch.bfloat16).double().numpy() - ref).max()
        assert err <= 2 * rounding, (name, tag, err, rounding)
        ref_lse = g[f"lse_{tag}"]
        got = lse.double().cpu().numpy()
        assert np.array_equal(np.isfinite(got), np.isfinite(ref_lse))
        fin = np.isfinite(ref_lse)
        if fin.any():
            assert np.abs(got[fin] - ref_lse[fin]).max() < 2e-3


@pytest.mark.parametrize("head_dim", [64, 128])
def test_large_scores(head_dim):
    # Scores of order 100 overflow exp() unless a running reference point is subtracted.
    q, k, v = make_inputs((2, 129, 129, 4, 2, head_dim), torch.bfloat16, scale=10.0)
    out, lse = flash_lab.attention(q, k, v, causal=True, return_lse=True)
    check_prefill(out, lse, q, k, v, causal=True)


@pytest.mark.parametrize("causal", [False, True])
def test_strided_inputs(causal):
    # q, k, v sliced out of one packed [B, S, 3, H, D] projection: no copies, unusual strides.
    gen = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn(2, 333, 3, 4, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    q, k, v = qkv.unbind(dim=2)
    assert not q.is_contiguous()
    out, lse = flash_lab.attention(q, k, v, causal=causal, return_lse=True)
    check_prefill(out, lse, q, k, v, causal=causal)


def test_head_major_views():
    # [B, H, S, D] storage seen as [B, S, H, D] (the Hugging Face layout).
    gen = torch.Generator(device="cuda").manual_seed(4)
    qh = torch.randn(2, 8, 190, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    kh = torch.randn(2, 2, 190, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    vh = torch.randn(2, 2, 190, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    q, k, v = qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2)
    out, lse = flash_lab.attention(q, k, v, causal=True, return_lse=True)
    check_prefill(out, lse, q, k, v, causal=True)


def test_deterministic():
    q, k, v = make_inputs((2, 300, 300, 8, 2, 128), torch.bfloat16)
    first = flash_lab.attention(q, k, v, causal=True)
    second = flash_lab.attention(q, k, v, causal=True)
    assert torch.equal(first, second)


def test_rejects_unsupported_inputs():
    q, k, v = make_inputs((1, 8, 8, 2, 2, 96), torch.bfloat16)
    with pytest.raises(ValueError, match="head_dim"):
        flash_lab.attention(q, k, v)
    q, k, v = make_inputs((1, 8, 8, 2, 2, 128), torch.float32)
    with pytest.raises(ValueError, match="dtype"):
        flash_lab.attention(q, k, v)
    q, k, v = make_inputs((1, 8, 8, 2, 2, 128), torch.bfloat16)
    with pytest.raises(RuntimeError, match="aligned"):
        torch.ops.flash_lab.attention_sm100(q, k, _misaligned(v), False, 0.1)


def _misaligned(x):
    """The same values one element off a 16-byte boundary."""
    buf = torch.empty(x.numel() + 8, device=x.device, dtype=x.dtype)
    y = buf[1:1 + x.numel()].view(x.shape)
    y.copy_(x)
    return y


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_baseline_config_sampled_rows(causal):
    """The benchmark's prefill configuration (B, H, H_kv, S, D) = (4, 32, 32, 4096, 128), on 256 rows
    (first, last and 254 random ones, as the reference's bench/run.py:75-80)."""
    q, k, v = make_inputs((4, 4096, 4096, 32, 32, 128), torch.bfloat16, seed=1)
    out, lse = flash_lab.attention(q, k, v, causal=causal, return_lse=True)
    gen = torch.Generator().manual_seed(5)
    middle = torch.randperm(4094, generator=gen)[:254] + 1
    rows = torch.cat([torch.tensor([0, 4095]), middle]).sort().values
    check_prefill(out, lse, q, k, v, causal, rows=rows)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_head_dim_64_long_gqa_sampled_rows(causal):
    """Llama-3.2-1B attention shape (H=32, H_kv=8, D=64) at 4096 tokens, on 256 sampled rows."""
    q, k, v = make_inputs((2, 4096, 4096, 32, 8, 64), torch.bfloat16, seed=2)
    out, lse = flash_lab.attention(q, k, v, causal=causal, return_lse=True)
    gen = torch.Generator().manual_seed(6)
    middle = torch.randperm(4094, generator=gen)[:254] + 1
    rows = torch.cat([torch.tensor([0, 4095]), middle]).sort().values
    check_prefill(out, lse, q, k, v, causal, rows=rows)


def test_causal_schedules_agree_bitwise():
    """Causal launches whose K/V exceed 192 MB run heavy/light q-block pairs per CTA, smaller ones
    single q-blocks dealt in cost order; the schedule only decides which CTA runs an item. The
    benchmark configuration (268 MB of K/V, pairs) must equal its two batch halves (134 MB each,
    cost order) bit for bit."""
    q, k, v = make_inputs((4, 4096, 4096, 32, 32, 128), torch.bfloat16, seed=3)
    out, lse = flash_lab.attention(q, k, v, causal=True, return_lse=True)
    for b0 in (0, 2):
        part, part_lse = flash_lab.attention(q[b0:b0 + 2], k[b0:b0 + 2], v[b0:b0 + 2],
                                             causal=True, return_lse=True)
        assert torch.equal(part, out[b0:b0 + 2])
        assert torch.equal(part_lse, lse[b0:b0 + 2])

"""Out-of-bounds write checks without a sanitizer (compute-sanitizer is not available here): the
shapes of the reference's tests/test_sanitize.py (ragged sequence lengths, masking, GQA, few
splits), run through the C ABI with every output embedded in a larger buffer filled with a
sentinel. After the launch the bytes around and between the outputs must be untouched, and the
outputs must equal the ones flash_lab returns for the same inputs."""

import ctypes

import pytest
import torch

import flash_lab
from flash_lab import _capi

pytestmark = pytest.mark.gpu

SENTINEL = -7.0   # exactly representable in bf16 / fp16 / fp32, never an attention output here


def _guarded(shape, dtype, pad_rows=2, pad_cols=64):
    """A [..., rows, heads, D] view inside a sentinel buffer with extra rows, heads and columns."""
    *lead, rows, heads, d = shape
    big = torch.full((*lead, rows + 2 * pad_rows, heads + 2, d + pad_cols), SENTINEL,
                     device="cuda", dtype=dtype)
    view = big[..., pad_rows:pad_rows + rows, 1:1 + heads, :d]
    return big, view


def _outside_untouched(big, view):
    """True when every element of `big` outside `view` (a view into it) still holds SENTINEL."""
    mask = torch.ones(big.numel(), dtype=torch.bool, device=big.device)
    idx = torch.arange(big.numel(), device=big.device)
    offs = torch.as_strided(idx, view.shape, view.stride(),
                            view.storage_offset() - big.storage_offset())
    mask[offs.reshape(-1)] = False
    return bool((big.reshape(-1)[mask] == SENTINEL).all())


def _lse_guarded(n):
    pad = 64
    buf = torch.full((n + 2 * pad,), SENTINEL, device="cuda", dtype=torch.float32)
    return buf, buf[pad:pad + n], pad


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("shape", [(2, 70, 70, 4, 2, 64), (1, 33, 65, 2, 1, 128)], ids=str)
def test_prefill_writes_only_its_outputs(shape, causal):
    lib = _capi.load()
    batch, sq, sk, heads, heads_kv, d = shape
    gen = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(batch, sq, heads, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    k = torch.randn(batch, sk, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    v = torch.randn(batch, sk, heads_kv, d, device="cuda", dtype=torch.bfloat16, generator=gen)
    big, o = _guarded((batch, sq, heads, d), torch.bfloat16)
    lse_buf, lse, pad = _lse_guarded(batch * heads * sq)
    p = _capi.AttnParams(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                         *q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *o.stride()[:3],
                         batch, sq, sk, heads, heads_kv, d, int(causal), _capi.FLB_BF16,
                         d ** -0.5, 0)
    assert lib.flb_prefill_fwd(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _outside_untouched(big, o)
    assert (lse_buf[:pad] == SENTINEL).all() and (lse_buf[pad + lse.numel():] == SENTINEL).all()
    ref_o, ref_lse = flash_lab.attention(q, k, v, causal=causal, return_lse=True)
    assert torch.equal(o, ref_o)
    assert torch.equal(lse.view(batch, heads, sq), ref_lse)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32],
                         ids=lambda t: str(t).removeprefix("torch."))
@pytest.mark.parametrize("num_splits", [1, 3, 0])
def test_decode_writes_only_its_outputs(num_splits, dtype):
    lib = _capi.load()
    gen = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(3, 8, 64, device="cuda", dtype=dtype, generator=gen)
    kc = torch.randn(3, 150, 2, 64, device="cuda", dtype=dtype, generator=gen)
    vc = torch.randn(3, 150, 2, 64, device="cuda", dtype=dtype, generator=gen)
    lens = torch.tensor([150, 1, 77], device="cuda", dtype=torch.int32)
    big = torch.full((3, 8 + 2, 64 + 64), SENTINEL, device="cuda", dtype=dtype)
    o = big[:, 1:9, :64]
    lse_buf, lse, pad = _lse_guarded(3 * 8)
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    splits = num_splits or lib.flb_decode_num_splits(3, 8, 2, 64, 150, sm)
    need = lib.flb_decode_workspace_bytes(3, 8, 64, splits)
    ws = torch.full((need // 4 + 256,), SENTINEL, device="cuda", dtype=torch.float32)
    code = {torch.bfloat16: _capi.FLB_BF16, torch.float32: _capi.FLB_FP32}[dtype]
    p = _capi.DecodeParams(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(),
                           lse.data_ptr(), lens.data_ptr(), q.stride(0), q.stride(1),
                           *kc.stride()[:3], *vc.stride()[:3], o.stride(0), o.stride(1),
                           3, 8, 2, 64, 150, splits, code, 0.125, ws.data_ptr(), need, 0)
    assert lib.flb_decode_fwd(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    mask = torch.ones_like(big, dtype=torch.bool)
    mask[:, 1:9, :64] = False
    assert (big.masked_select(mask) == SENTINEL).all()
    assert (lse_buf[:pad] == SENTINEL).all() and (lse_buf[pad + lse.numel():] == SENTINEL).all()
    assert (ws[need // 4:] == SENTINEL).all()          # nothing past the workspace it asked for
    ref_o, ref_lse = flash_lab.decode(q, kc, vc, lens, num_splits=splits, return_lse=True)
    assert torch.equal(o, ref_o) and torch.equal(lse, ref_lse.reshape(-1))

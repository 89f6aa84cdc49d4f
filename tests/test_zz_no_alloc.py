"""The allocation-free decode entry point, flb_decode_fwd_static, through the C ABI.

Some callers cannot allocate device memory at the moment they decode: cudaMalloc may synchronise
the device and is not allowed while a stream is being captured into a CUDA graph, and serving
loops that plan their memory up front forbid allocation on the step path. For them the library
keeps the decode's split partials in a static device array instead of a caller workspace.

This file checks that the static variant returns exactly what the workspace variant
(flb_decode_fwd) returns, on two calls in a row with different inputs (the array keeps the
previous call's contents), and that a problem too large for the array is refused before
anything runs. It is collected last so that a failure here never hides the other tests.
"""

import ctypes

import pytest
import torch

from flash_lab import _capi

pytestmark = pytest.mark.gpu


def _params(q, kc, vc, lens, o, lse, num_splits=0, workspace=None):
    batch, heads, head_dim = q.shape
    return _capi.DecodeParams(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), lse.data_ptr(),
        lens.data_ptr(),
        q.stride(0), q.stride(1),
        kc.stride(0), kc.stride(1), kc.stride(2),
        vc.stride(0), vc.stride(1), vc.stride(2),
        o.stride(0), o.stride(1),
        batch, heads, kc.shape[2], head_dim, kc.shape[1], num_splits, _capi.FLB_BF16,
        1.0 / head_dim ** 0.5,
        0 if workspace is None else workspace.data_ptr(),
        0 if workspace is None else workspace.numel(),
        0,
    )


def _inputs(seed, batch=4, heads=32, heads_kv=8, smax=8192, head_dim=128):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, heads, head_dim, device="cuda", dtype=torch.bfloat16, generator=gen)
    kc = torch.randn(batch, smax, heads_kv, head_dim, device="cuda", dtype=torch.bfloat16,
                     generator=gen)
    vc = torch.randn_like(kc)
    lens = torch.randint(1, smax + 1, (batch,), device="cuda", generator=gen).to(torch.int32)
    return q, kc, vc, lens


def _run(lib, fn_name, q, kc, vc, lens, workspace=None):
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:2], device="cuda", dtype=torch.float32)
    p = _params(q, kc, vc, lens, o, lse, workspace=workspace)
    rc = getattr(lib, fn_name)(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert rc == _capi.FLB_OK, _capi.error_message(lib, rc)
    return o, lse


def test_static_scratch_matches_the_workspace_entry_point():
    lib = _capi.load()
    assert lib.flb_decode_static_scratch_bytes() == 8 << 20
    for seed in (0, 1):  # two calls in a row: the second sees the first call's scratch contents
        q, kc, vc, lens = _inputs(seed)
        sm = torch.cuda.get_device_properties(0).multi_processor_count
        splits = lib.flb_decode_num_splits(q.shape[0], q.shape[1], kc.shape[2], q.shape[2],
                                           kc.shape[1], sm)
        assert splits > 1  # the case exercises the scratch
        ws = torch.empty(lib.flb_decode_workspace_bytes(q.shape[0], q.shape[1], q.shape[2],
                                                        splits), dtype=torch.uint8, device="cuda")
        o_ref, lse_ref = _run(lib, "flb_decode_fwd", q, kc, vc, lens, workspace=ws)
        o, lse = _run(lib, "flb_decode_fwd_static", q, kc, vc, lens)
        torch.cuda.synchronize()
        # Same kernels and split count: the results are identical, well inside the decode
        # tests' tolerance.
        assert torch.equal(o, o_ref)
        assert torch.equal(lse, lse_ref)


def test_problem_too_large_for_the_static_scratch_is_refused():
    lib = _capi.load()
    q, kc, vc, lens = _inputs(2, batch=64, heads=64, heads_kv=64, smax=256)
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:2], device="cuda", dtype=torch.float32)
    p = _params(q, kc, vc, lens, o, lse, num_splits=8)  # 64*64*8 slots * 520 B > 8 MiB
    rc = lib.flb_decode_fwd_static(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert rc == _capi.FLB_ERR_WORKSPACE
    assert b"static array holds" in lib.flb_last_error()

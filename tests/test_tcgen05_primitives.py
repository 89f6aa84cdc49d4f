"""The tcgen05 building blocks of the prefill kernel in isolation (flb_selftest_umma through the C
ABI): TMA into 128-byte-swizzled boxes, K-major and MN-major shared-memory descriptors, TMEM
accumulator and A-operand layouts. Identity and permutation operands make any layout mistake show
up as a visible permutation, as the reference's fragment test does for mma.sync
(tests/test_mma_primitives.py there)."""

import ctypes

import pytest
import torch

from flash_lab import _capi

pytestmark = pytest.mark.gpu


def run(a, b, p, v):
    lib = _capi.load()
    s = torch.full((128, 128), float("nan"), device="cuda")
    o = torch.full((128, 128), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.flb_selftest_umma(a.data_ptr(), b.data_ptr(), p.data_ptr(), v.data_ptr(),
                               s.data_ptr(), o.data_ptr(), status.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _capi.error_message(lib, rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return s, o


def test_identity_operands_reproduce_the_inputs():
    gen = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(128, 128, device="cuda", generator=gen).to(torch.bfloat16)
    v = torch.randn(128, 128, device="cuda", generator=gen).to(torch.bfloat16)
    eye = torch.eye(128, device="cuda", dtype=torch.bfloat16)
    s, o = run(a, eye, eye, v)
    torch.testing.assert_close(s, a.float(), rtol=0, atol=0)   # a @ I^T
    torch.testing.assert_close(o, v.float(), rtol=0, atol=0)   # I @ v


def test_permutations_are_not_scrambled():
    perm = torch.randperm(128, generator=torch.Generator().manual_seed(1)).cuda()
    eye = torch.eye(128, device="cuda", dtype=torch.bfloat16)
    pm = eye[perm]
    idx = torch.arange(128 * 128, device="cuda", dtype=torch.float32).view(128, 128) % 251
    a = idx.to(torch.bfloat16)
    s, o = run(a, pm, pm, a)
    torch.testing.assert_close(s, (a.float() @ pm.float().t()), rtol=0, atol=0)
    torch.testing.assert_close(o, (pm.float() @ a.float()), rtol=0, atol=0)


def test_random_products():
    gen = torch.Generator(device="cuda").manual_seed(2)
    a, b, v = (torch.randn(128, 128, device="cuda", generator=gen).to(torch.bfloat16)
               for _ in range(3))
    p = torch.rand(128, 128, device="cuda", generator=gen).to(torch.bfloat16)
    s, o = run(a, b, p, v)
    torch.testing.assert_close(s, a.float() @ b.float().t(), rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(o, p.float() @ v.float(), rtol=1e-4, atol=1e-3)

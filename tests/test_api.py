"""Input validation of the public API on CPU tensors: every error is raised before any kernel.
Mirrors the reference's tests/test_api.py (same error types and message fragments)."""

import pytest
import torch

import flash_lab


def qkv(batch=2, seqlen_q=8, seqlen_k=8, heads=4, heads_kv=4, head_dim=16, dtype=torch.float32):
    q = torch.randn(batch, seqlen_q, heads, head_dim, dtype=dtype)
    k = torch.randn(batch, seqlen_k, heads_kv, head_dim, dtype=dtype)
    v = torch.randn(batch, seqlen_k, heads_kv, head_dim, dtype=dtype)
    return q, k, v


def test_rejects_wrong_rank():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="4-D"):
        flash_lab.attention(q[0], k, v)


def test_rejects_non_tensors():
    _, k, v = qkv()
    with pytest.raises(TypeError, match="torch.Tensor"):
        flash_lab.attention([[1.0]], k, v)


def test_rejects_mixed_dtypes():
    q, k, v = qkv()
    with pytest.raises(TypeError, match="dtype"):
        flash_lab.attention(q, k.double(), v)


def test_rejects_mixed_devices():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="one device"):
        flash_lab.attention(q, k.to("meta"), v)


def test_rejects_heads_not_divisible_by_kv_heads():
    q, k, v = qkv(heads=6, heads_kv=4)
    with pytest.raises(ValueError, match="multiple of KV heads"):
        flash_lab.attention(q, k, v)


def test_rejects_mismatched_batch_and_head_dim():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="batch"):
        flash_lab.attention(q[:1], k, v)
    with pytest.raises(ValueError, match="head_dim"):
        flash_lab.attention(q[..., :8], k, v)
    with pytest.raises(ValueError, match="same shape"):
        flash_lab.attention(q, k, v[:, :4])


def test_requires_unit_stride_in_head_dim():
    _, k, v = qkv()
    strided = torch.randn(2, 8, 4, 32)[..., ::2]
    with pytest.raises(ValueError, match="last dimension"):
        flash_lab.attention(strided, k, v)


def test_rejects_unknown_impl():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="unknown impl"):
        flash_lab.attention(q, k, v, impl="does-not-exist")


def test_rejects_cpu_tensors():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="CUDA"):
        flash_lab.attention(q, k, v)


def test_rejects_non_positive_scale():
    q, k, v = qkv()
    with pytest.raises(ValueError, match="softmax_scale"):
        flash_lab.attention(q, k, v, softmax_scale=0.0)


def decode_inputs(batch=2, max_seqlen=16, heads=4, heads_kv=2, head_dim=16):
    q = torch.randn(batch, 1, heads, head_dim)
    k_cache = torch.randn(batch, max_seqlen, heads_kv, head_dim)
    v_cache = torch.randn(batch, max_seqlen, heads_kv, head_dim)
    seq_lens = torch.full((batch,), max_seqlen, dtype=torch.int32)
    return q, k_cache, v_cache, seq_lens


def test_decode_validation():
    q, k_cache, v_cache, seq_lens = decode_inputs()
    with pytest.raises(TypeError, match="int32"):
        flash_lab.decode(q, k_cache, v_cache, seq_lens.long())
    with pytest.raises(ValueError, match="seq_lens must have shape"):
        flash_lab.decode(q, k_cache, v_cache, seq_lens[:1])
    with pytest.raises(ValueError, match="seq_lens must be contiguous"):
        flash_lab.decode(q, k_cache, v_cache, seq_lens[:1].expand(2))
    with pytest.raises(ValueError, match="one query token"):
        flash_lab.decode(q.expand(2, 3, 4, 16), k_cache, v_cache, seq_lens)
    with pytest.raises(ValueError, match="same shape"):
        flash_lab.decode(q, k_cache, v_cache[:, :8], seq_lens)
    with pytest.raises(ValueError, match="num_splits"):
        flash_lab.decode(q, k_cache, v_cache, seq_lens, num_splits=0)
    with pytest.raises(ValueError, match="CUDA"):
        flash_lab.decode(q, k_cache, v_cache, seq_lens)


def test_decode_paged_validation():
    q, _, _, seq_lens = decode_inputs()
    pool = torch.randn(10, 4, 2, 16)
    tables = torch.zeros(2, 4, dtype=torch.int64)
    with pytest.raises(TypeError, match="block_tables must be int32"):
        flash_lab.decode(q, pool, pool, seq_lens, block_tables=tables)
    with pytest.raises(ValueError, match="block_tables must be"):
        flash_lab.decode(q, pool, pool, seq_lens, block_tables=tables[:1].int())


def test_available_impls_lists_both_entry_points():
    impls = flash_lab.available_impls()
    assert set(impls) == {"attention", "decode"}
    assert impls["attention"] == ["sm100", "mma_pipelined"]
    assert impls["decode"] == ["splitkv", "decode_inplace"]


def test_ops_keep_the_reference_schemas():
    ops = torch.ops.flash_lab
    prefill = "(Tensor q, Tensor k, Tensor v, bool causal, float softmax_scale) -> (Tensor, Tensor)"
    decode = ("(Tensor q, Tensor k_cache, Tensor v_cache, Tensor seq_lens, float softmax_scale, "
              "int num_splits) -> (Tensor, Tensor)")
    for name, schema in [("attention_mma_pipelined", prefill), ("attention_sm100", prefill),
                         ("decode_splitkv", decode), ("decode_inplace", decode)]:
        assert str(getattr(ops, name).default._schema) == f"flash_lab::{name}{schema}"


def test_fake_kernels_give_output_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(2, 5, 8, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(2, 7, 2, 128, dtype=torch.bfloat16, device="cuda")
        o, lse = torch.ops.flash_lab.attention_sm100(q, k, k, True, 0.1)
        assert o.shape == q.shape and lse.shape == (2, 8, 5) and lse.dtype == torch.float32
        q3 = torch.empty(2, 8, 128, dtype=torch.bfloat16, device="cuda")
        cache = torch.empty(2, 64, 2, 128, dtype=torch.bfloat16, device="cuda")
        lens = torch.empty(2, dtype=torch.int32, device="cuda")
        o, lse = torch.ops.flash_lab.decode_splitkv(q3, cache, cache, lens, 0.1, 0)
        assert o.shape == q3.shape and lse.shape == (2, 8)


def test_c_abi_error_status_becomes_runtime_error(monkeypatch):
    # An error status from the library (here a fake one) reaches Python as RuntimeError with the
    # library's message, as the reference's TORCH_CHECK failures did.
    from flash_lab import _capi, ops

    class FakeLib:
        def flb_last_error(self):
            return b"injected launch failure"

        def flb_status_string(self, status):
            return b"CUDA error"

    monkeypatch.setattr(ops, "_LIB", FakeLib())
    with pytest.raises(RuntimeError, match="flb_decode_fwd: CUDA error: injected launch failure"):
        ops._check(_capi.FLB_ERR_CUDA, "flb_decode_fwd", torch.device("cpu"))
    ops._check(_capi.FLB_OK, "flb_decode_fwd", torch.device("cpu"))   # OK passes silently


@pytest.mark.gpu
def test_eager_fast_path_matches_the_registered_ops():
    # Plain eager calls run the op's implementation directly; the registered op gives the same
    # bits, and a torch dispatch mode still sees the flash_lab:: ops by name.
    from torch.utils._python_dispatch import TorchDispatchMode

    gen = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(1, 300, 4, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    k = torch.randn(1, 300, 2, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    v = torch.randn(1, 300, 2, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    o, lse = flash_lab.attention(q, k, v, causal=True, return_lse=True)
    o_op, lse_op = torch.ops.flash_lab.attention_sm100(q, k, v, True, 128 ** -0.5)
    assert torch.equal(o, o_op) and torch.equal(lse, lse_op)

    qd = torch.randn(2, 8, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    kc = torch.randn(2, 3000, 2, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    vc = torch.randn(2, 3000, 2, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    lens = torch.tensor([3000, 1234], device="cuda", dtype=torch.int32)
    od, lsed = flash_lab.decode(qd, kc, vc, lens, return_lse=True)
    od_op, lsed_op = torch.ops.flash_lab.decode_splitkv(qd, kc, vc, lens, 128 ** -0.5, 0)
    assert torch.equal(od, od_op) and torch.equal(lsed, lsed_op)

    class Record(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.names = []

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            self.names.append(str(func))
            return func(*args, **(kwargs or {}))

    with Record() as rec:
        flash_lab.attention(q, k, v, causal=True)
        flash_lab.decode(qd, kc, vc, lens)
    assert any("flash_lab.attention_sm100" in n for n in rec.names), rec.names
    assert any("flash_lab.decode_splitkv" in n for n in rec.names), rec.names


def test_eager_fast_path_only_for_plain_eager_calls():
    # The direct call is taken for plain tensors only; torch modes and tensor subclasses (and
    # torch.compile, which traces flash_lab.attention / decode) go through the registered ops.
    from torch.overrides import TorchFunctionMode
    from torch.utils._python_dispatch import TorchDispatchMode

    from flash_lab import ops

    x = torch.zeros(2)
    assert ops._eager_ok((x, 1.0, 3))

    class Sub(torch.Tensor):
        pass

    assert not ops._eager_ok((x.as_subclass(Sub), 1.0))

    class Dispatch(TorchDispatchMode):
        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            return func(*args, **(kwargs or {}))

    with Dispatch():
        assert not ops._eager_ok((x,))

    class Function(TorchFunctionMode):
        def __torch_function__(self, func, types, args=(), kwargs=None):
            return func(*args, **(kwargs or {}))

    with Function():
        assert not ops._eager_ok((x,))
    assert ops._eager_ok((x,))


def test_ops_use_the_built_torch_binding():
    # When the PyTorch binding of the C ABI is built next to the library, the ops call it (the
    # ctypes path stays for a library taken from FLASH_LAB_LIBRARY).
    import os

    from flash_lab import _capi, ops

    binding = _capi.LIB_PATH.parent / "_flash_lab_torch.so"
    if not binding.exists() or not ops.HAS_EXTENSION or os.environ.get("FLASH_LAB_LIBRARY"):
        pytest.skip("the binding is not built here")
    assert ops._NATIVE is not None and ops._NATIVE.abi_version() == 3


@pytest.mark.gpu
def test_torch_binding_and_ctypes_paths_agree(monkeypatch):
    # The binding and the ctypes path fill the same parameter blocks: same bits, and a
    # rejection inside the library (rows not 16-byte aligned) gives the same message.
    from flash_lab import ops

    if ops._NATIVE is None:
        pytest.skip("the binding is not built here")
    gen = torch.Generator(device="cuda").manual_seed(6)
    q = torch.randn(2, 300, 8, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    k = torch.randn(2, 500, 2, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    qd = torch.randn(3, 1, 16, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    kc = torch.randn(3, 2048, 4, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    lens = torch.tensor([2048, 1, 900], device="cuda", dtype=torch.int32)
    bad_q = torch.empty(3, 8, 136, device="cuda", dtype=torch.bfloat16)[:, :, :128]
    bad_q = bad_q.as_strided((3, 8, 128), (8 * 136 - 8, 136 - 1, 1))   # rows 270 bytes apart
    results, messages = [], []
    for native in (ops._NATIVE, None):
        monkeypatch.setattr(ops, "_NATIVE", native)
        results.append((flash_lab.attention(q, k, k, causal=True, return_lse=True),
                        flash_lab.decode(qd, kc, kc, lens, return_lse=True)))
        with pytest.raises(RuntimeError) as err:
            ops._decode(bad_q, kc, kc, lens, 0.1, 0, True)
        messages.append(str(err.value))
    torch.cuda.synchronize()
    (pa, da), (pb, db) = results
    assert torch.equal(pa[0], pb[0]) and torch.equal(pa[1], pb[1])
    assert torch.equal(da[0], db[0]) and torch.equal(da[1], db[1])
    assert messages[0] == messages[1] and "16-byte aligned rows" in messages[0], messages


@pytest.mark.gpu
def test_repeated_eager_decode_calls_take_the_memoised_path():
    # A plain eager decode whose input metadata was seen before goes straight to the binding:
    # same bits and shapes as the first (validated) call, for [B, 1, H, D] and [B, H, D] queries,
    # and inputs with other metadata still get the reference's validation errors.
    from flash_lab import ops

    if ops._NATIVE is None:
        pytest.skip("the binding is not built here")
    gen = torch.Generator(device="cuda").manual_seed(7)
    q4 = torch.randn(2, 1, 8, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    kc = torch.randn(2, 3000, 2, 128, device="cuda", dtype=torch.bfloat16, generator=gen)
    lens = torch.tensor([3000, 1234], device="cuda", dtype=torch.int32)
    ops._DECODE_CALLS.clear()
    for q in (q4, q4[:, 0]):
        first = flash_lab.decode(q, kc, kc, lens, return_lse=True)
        second = flash_lab.decode(q, kc, kc, lens, return_lse=True)
        third = flash_lab.decode(q, kc, kc, lens, num_splits=1, return_lse=True)
        assert second[0].shape == q.shape == first[0].shape
        assert torch.equal(first[0], second[0]) and torch.equal(first[1], second[1])
        torch.testing.assert_close(third[0], first[0], atol=2e-2, rtol=0)
    assert len(ops._DECODE_CALLS) == 4
    with pytest.raises(TypeError, match="seq_lens must be int32"):
        flash_lab.decode(q4, kc, kc, lens.long())
    with pytest.raises(ValueError, match="num_splits must be positive"):
        flash_lab.decode(q4, kc, kc, lens, num_splits=0)

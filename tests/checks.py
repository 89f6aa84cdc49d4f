"""Tolerance rules for the GPU parity tests, with the numpy oracle as ground truth.

Two rules are applied to every bf16/fp16 output (fp32 decode outputs get the first, with the
reference's fp32 floors 1e-6 / 1e-5):
  * the reference's drop-in rule (tests/test_attention_fwd.py:114-138 and
    tests/test_decode.py:256-266 of tfan2437/flash-attention-lab):
        err <= 2 * err_torch + FLOOR   (err_torch: PyTorch's own computation at the input dtype)
        err <= GUARD * (1 + max|v|)    (prefill)
        lse_err <= 2 * lse_err_torch + LSE_FLOOR, and lse is -inf exactly where the oracle's is;
  * the stricter rounding rule of the benchmark's parity target:
        err <= 2 * max|round_dtype(ref64) - ref64|
    i.e. the kernel's output error is at most twice that of the fp64 reference rounded to the
    output dtype.
err = max |out - ref64| over all (or the sampled) rows, in fp64.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

import oracle

FLOOR = {torch.bfloat16: 1e-3, torch.float16: 1e-3, torch.float32: 1e-6}
GUARD = {torch.bfloat16: 2e-2, torch.float16: 1e-2}
LSE_FLOOR = {torch.bfloat16: 1e-3, torch.float16: 1e-3, torch.float32: 1e-5}


def host64(x: torch.Tensor) -> np.ndarray:
    return x.detach().double().cpu().numpy()


def rounding_error(ref: np.ndarray, dtype: torch.dtype) -> float:
    """max |round_dtype(ref) - ref|: the error of the fp64 reference stored in `dtype`."""
    t = torch.from_numpy(ref)
    return float((t.to(dtype).double() - t).abs().max())


def sdpa_rows_at_dtype(q, k, v, rows, causal, scale):
    """PyTorch's math backend at the input dtype for the given query rows (bottom-right mask)."""
    group = q.shape[2] // k.shape[2]
    k = k.repeat_interleave(group, dim=2)
    v = v.repeat_interleave(group, dim=2)
    mask = None
    if causal:
        cols = torch.arange(k.shape[1], device=q.device)[None, :]
        mask = cols <= rows.to(q.device)[:, None] + (k.shape[1] - q.shape[1])
    with sdpa_kernel(SDPBackend.MATH):
        out = F.scaled_dot_product_attention(q[:, rows].transpose(1, 2), k.transpose(1, 2),
                                             v.transpose(1, 2), attn_mask=mask, scale=scale)
    return out.transpose(1, 2)


def torch_lse_at_dtype(q, k, v, rows, causal, scale):
    """LSE computed with plain torch ops at the input dtype (the reference's lse_torch)."""
    group = q.shape[2] // k.shape[2]
    kk = k.repeat_interleave(group, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q[:, rows], kk) * scale
    if causal:
        cols = torch.arange(k.shape[1], device=q.device)[None, :]
        hidden = cols > rows.to(q.device)[:, None] + (k.shape[1] - q.shape[1])
        s = s.masked_fill(hidden, float("-inf"))
    return torch.logsumexp(s, dim=-1)


def check_prefill(out, lse, q, k, v, causal, scale=None, rows=None, baseline_rule=True):
    """Checks o [B, S_q, H, D] and lse [B, H, S_q] against the oracle on `rows` (all rows by
    default). Returns the measured errors."""
    dtype = q.dtype
    head_dim = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    seqlen_q = q.shape[1]
    if rows is None:
        rows = torch.arange(seqlen_q)
    assert out.shape == q.shape and out.dtype == dtype
    assert lse.shape == (q.shape[0], q.shape[2], seqlen_q) and lse.dtype == torch.float32
    o_rows = host64(out[:, rows.to(out.device)])
    assert np.isfinite(o_rows).all()
    ref, ref_lse = oracle.attention_rows(host64(q), host64(k), host64(v), rows.numpy(),
                                         causal=causal, softmax_scale=scale, return_lse=True)
    err = float(np.abs(o_rows - ref).max())
    torch_out = sdpa_rows_at_dtype(q, k, v, rows, causal, scale)
    err_torch = float(np.nan_to_num(np.abs(host64(torch_out) - ref), nan=0.0).max())
    vmax = float(v.abs().max())
    info = {"err": err, "err_torch": err_torch, "round": rounding_error(ref, dtype)}
    assert err <= 2 * err_torch + FLOOR[dtype], info
    assert err <= GUARD[dtype] * (1 + vmax), info
    if baseline_rule:
        assert err <= 2 * info["round"], info

    got_lse = host64(lse[:, :, rows.to(lse.device)])
    visible = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(got_lse), visible), "lse -inf pattern differs"
    assert np.all(np.isneginf(got_lse[~visible]))
    if visible.any():
        lse_t = host64(torch_lse_at_dtype(q, k, v, rows, causal, scale))
        lse_err = float(np.abs(got_lse[visible] - ref_lse[visible]).max())
        lse_err_torch = float(np.abs(lse_t[visible] - ref_lse[visible]).max())
        info.update(lse_err=lse_err, lse_err_torch=lse_err_torch)
        assert lse_err <= 2 * lse_err_torch + LSE_FLOOR[dtype], info
    return info


def plain_decode_at_dtype(q3, k_cache, v_cache, seq_lens, scale):
    """The reference's decode at the input dtype (reference.py:167-205 with dtype=q.dtype),
    written with torch ops: every intermediate stays in that dtype."""
    outs, lses = [], []
    for b, n in enumerate(seq_lens.tolist()):
        kk = k_cache[b, :n]
        vv = v_cache[b, :n]
        group = q3.shape[1] // kk.shape[1]
        kk = kk.repeat_interleave(group, dim=1)
        vv = vv.repeat_interleave(group, dim=1)
        s = torch.einsum("hd,khd->hk", q3[b], kk) * scale
        lse = torch.logsumexp(s, dim=-1)
        p = torch.exp(s - lse[:, None])
        outs.append(torch.einsum("hk,khd->hd", p, vv))
        lses.append(lse)
    return torch.stack(outs), torch.stack(lses)


def check_decode(out, lse, q, k_cache, v_cache, seq_lens, scale=None, baseline_rule=True):
    dtype = q.dtype
    q3 = q[:, 0] if q.dim() == 4 else q
    head_dim = q3.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
    assert out.shape == q.shape and out.dtype == dtype
    o = host64(out)
    assert np.isfinite(o).all()
    ref, ref_lse = oracle.decode(host64(q), host64(k_cache), host64(v_cache),
                                 seq_lens.cpu().numpy(), softmax_scale=scale, return_lse=True)
    err = float(np.abs(o - ref).max())
    plain, plain_lse = plain_decode_at_dtype(q3, k_cache, v_cache, seq_lens, scale)
    ref3 = ref[:, 0] if ref.ndim == 4 else ref
    err_plain = float(np.abs(host64(plain) - ref3).max())
    info = {"err": err, "err_plain": err_plain, "round": rounding_error(ref, dtype)}
    assert err <= 2 * err_plain + FLOOR[dtype], info
    if baseline_rule and dtype != torch.float32:
        assert err <= 2 * info["round"], info
    lse_err = float(np.abs(host64(lse) - ref_lse).max())
    lse_err_plain = float(np.abs(host64(plain_lse) - ref_lse).max())
    info.update(lse_err=lse_err, lse_err_plain=lse_err_plain)
    assert lse_err <= 2 * lse_err_plain + LSE_FLOOR[dtype], info
    return info

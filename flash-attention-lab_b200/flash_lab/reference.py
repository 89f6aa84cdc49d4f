"""Plain-PyTorch fp64 attention, kept for source compatibility with `flash_lab.reference` of the
reference package (flash_lab/reference.py:16-205 there), which user test code calls as ground
truth.

This module is a utility for callers. flash_lab.attention and flash_lab.decode never call it:
they only run the sm_100a kernels and raise when those are unavailable. Semantics: bottom-right
causal mask (query i sees key j iff j <= i + S_k - S_q), rows without keys give zeros and an LSE
of -inf, natural-log LSE of shape [B, H, S_q].
"""

from __future__ import annotations

import math

import torch

from flash_lab.layouts import check_attention_inputs, check_decode_inputs


def causal_mask(seqlen_q: int, seqlen_k: int, device=None) -> torch.Tensor:
    """[S_q, S_k] boolean mask, True where the key is hidden from the query."""
    rows = torch.arange(seqlen_q, device=device)[:, None]
    cols = torch.arange(seqlen_k, device=device)[None, :]
    return cols > rows + (seqlen_k - seqlen_q)


def _scale(head_dim: int, softmax_scale):
    return softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)


def _kv(x: torch.Tensor, group: int, dtype) -> torch.Tensor:
    x = x.to(dtype)
    return x.repeat_interleave(group, dim=2) if group > 1 else x


def _finish(scores: torch.Tensor, v_: torch.Tensor):
    lse = torch.logsumexp(scores, dim=-1)
    shift = torch.where(torch.isneginf(lse), torch.zeros_like(lse), lse)
    probs = torch.exp(scores - shift.unsqueeze(-1))
    return torch.einsum("bhqk,bkhd->bqhd", probs, v_), lse


def attention(q, k, v, causal: bool = False, softmax_scale=None, return_lse: bool = False,
              dtype: torch.dtype = torch.float64):
    """Materialises the scaled score matrix. Returns o [B, S_q, H, D] in `dtype` (and lse)."""
    shape = check_attention_inputs(q, k, v, require_unit_stride=False)
    scale = _scale(shape.head_dim, softmax_scale)
    scores = torch.einsum("bqhd,bkhd->bhqk", q.to(dtype), _kv(k, shape.group, dtype)) * scale
    if causal:
        scores = scores.masked_fill(causal_mask(shape.seqlen_q, shape.seqlen_k, q.device),
                                    float("-inf"))
    out, lse = _finish(scores, _kv(v, shape.group, dtype))
    return (out, lse) if return_lse else out


def attention_rows(q, k, v, rows: torch.Tensor, causal: bool = False, softmax_scale=None,
                   dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """attention() for the listed query rows only, [B, len(rows), H, D]; the causal mask uses
    each row's position in the full sequence."""
    shape = check_attention_inputs(q, k, v, require_unit_stride=False)
    scale = _scale(shape.head_dim, softmax_scale)
    qr = q[:, rows].to(dtype)
    scores = torch.einsum("bqhd,bkhd->bhqk", qr, _kv(k, shape.group, dtype)) * scale
    if causal:
        cols = torch.arange(shape.seqlen_k, device=q.device)[None, :]
        hidden = cols > rows.to(q.device)[:, None] + (shape.seqlen_k - shape.seqlen_q)
        scores = scores.masked_fill(hidden, float("-inf"))
    out, _ = _finish(scores, _kv(v, shape.group, dtype))
    return out


def attention_tiled(q, k, v, causal: bool = False, softmax_scale=None, return_lse: bool = False,
                    block_q: int = 64, block_k: int = 64, dtype: torch.dtype = torch.float64):
    """attention() computed block by block with the online softmax, never forming the full
    [S_q, S_k] score matrix (the reference's reference.py:90-152). Blocks wholly above the
    causal diagonal are skipped and blocks crossing it are masked; while a row has seen only
    masked keys its reference point is 0, so its exponentials are exactly 0. Returns o
    [B, S_q, H, D] in `dtype` (and lse [B, H, S_q])."""
    shape = check_attention_inputs(q, k, v, require_unit_stride=False)
    scale = _scale(shape.head_dim, softmax_scale)
    offset = shape.seqlen_k - shape.seqlen_q
    qh = q.to(dtype).transpose(1, 2)                        # [B, H, S_q, D]
    kh = _kv(k, shape.group, dtype).transpose(1, 2)         # [B, H, S_k, D]
    vh = _kv(v, shape.group, dtype).transpose(1, 2)
    out = torch.zeros_like(qh)
    lse = torch.full(qh.shape[:-1], float("-inf"), dtype=dtype, device=q.device)
    for q0 in range(0, shape.seqlen_q, block_q):
        q1 = min(q0 + block_q, shape.seqlen_q)
        m = torch.full((shape.batch, shape.heads, q1 - q0), float("-inf"), dtype=dtype,
                       device=q.device)
        l = torch.zeros_like(m)
        acc = torch.zeros((*m.shape, shape.head_dim), dtype=dtype, device=q.device)
        stop = min(shape.seqlen_k, q1 + offset) if causal else shape.seqlen_k
        for k0 in range(0, max(stop, 0), block_k):
            k1 = min(k0 + block_k, shape.seqlen_k)
            s = qh[:, :, q0:q1] @ kh[:, :, k0:k1].transpose(-1, -2) * scale
            if causal and k1 - 1 > q0 + offset:
                hidden = (torch.arange(k0, k1, device=q.device)[None, :]
                          > torch.arange(q0, q1, device=q.device)[:, None] + offset)
                s = s.masked_fill(hidden, float("-inf"))
            m_new = torch.maximum(m, s.amax(dim=-1))
            ref = torch.where(torch.isneginf(m_new), torch.zeros_like(m_new), m_new)
            alpha = torch.exp(m - ref)
            p = torch.exp(s - ref[..., None])
            l = alpha * l + p.sum(dim=-1)
            acc = alpha[..., None] * acc + p @ vh[:, :, k0:k1]
            m = m_new
        seen = l > 0
        denom = torch.where(seen, l, torch.ones_like(l))
        out[:, :, q0:q1] = acc / denom[..., None]
        lse[:, :, q0:q1] = torch.where(seen, m + torch.log(denom),
                                       torch.full_like(m, float("-inf")))
    out = out.transpose(1, 2)
    return (out, lse) if return_lse else out


def gather_cache(cache: torch.Tensor, block_tables, batch_idx: int, length: int) -> torch.Tensor:
    """Rows 0..length-1 of one sequence as [length, H_kv, D], contiguous or paged cache."""
    if block_tables is None:
        return cache[batch_idx, :length]
    page = cache.shape[1]
    pages = block_tables[batch_idx, : -(-length // page)].long()
    return cache[pages].reshape(-1, *cache.shape[2:])[:length]


def decode(q, k_cache, v_cache, seq_lens, block_tables=None, softmax_scale=None,
           return_lse: bool = False, dtype: torch.dtype = torch.float64):
    """One query token per sequence against its first seq_lens[b] cached keys. Returns o with
    q's rank and lse [B, H]."""
    q3, shape = check_decode_inputs(q, k_cache, v_cache, seq_lens, block_tables,
                                    require_unit_stride=False)
    scale = _scale(shape.head_dim, softmax_scale)
    outs, lses = [], []
    for b, length in enumerate(seq_lens.tolist()):
        if not 1 <= length <= shape.max_seqlen:
            raise ValueError(f"seq_lens[{b}] = {length} is outside [1, {shape.max_seqlen}]")
        keys = gather_cache(k_cache, block_tables, b, length)[None]
        values = gather_cache(v_cache, block_tables, b, length)[None]
        o_b, lse_b = attention(q3[b][None, None], keys, values, softmax_scale=scale,
                               return_lse=True, dtype=dtype)
        outs.append(o_b[0, 0])
        lses.append(lse_b[0, :, 0])
    out = torch.stack(outs)
    if q.dim() == 4:
        out = out.unsqueeze(1)
    lse = torch.stack(lses)
    return (out, lse) if return_lse else out

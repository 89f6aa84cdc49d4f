"""numpy fp64 restatement of the reference's attention ground truth (test infrastructure only).

Semantics follow flash_lab/reference.py of the reference:
  * tensors are [B, S, H, D]; K/V may have H_kv < H heads and query head h reads KV head
    h // (H // H_kv) (reference.py:23-25);
  * causal masks are aligned to the bottom-right corner: query i sees key j iff
    j <= i + (S_k - S_q) (reference.py:16-20);
  * a row that sees no key returns zeros and an LSE of -inf (reference.py:53-55);
  * the LSE is the natural-log log-sum-exp of the scaled scores, shape [B, H, S_q].

Inputs may be numpy arrays or anything np.asarray accepts (torch CPU tensors included). All math
runs in float64 unless `dtype` says otherwise; the result has that dtype.
"""

from __future__ import annotations

import math

import numpy as np

NEG_INF = -np.inf


def _as(x, dtype) -> np.ndarray:
    if hasattr(x, "detach"):  # a torch tensor: go through fp32/fp64 on the host
        x = x.detach().cpu()
        if str(x.dtype) in ("torch.bfloat16", "torch.float16"):
            x = x.float()
        x = x.numpy()
    return np.asarray(x, dtype=dtype)


def _default_scale(head_dim: int, softmax_scale: float | None) -> float:
    """reference.py:28-29: 1/sqrt(D) unless a scale is given."""
    return softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)


def _expand_kv(x: np.ndarray, group: int) -> np.ndarray:
    """[B, S, H_kv, D] -> [B, S, H, D] so query head h lines up with KV head h // group
    (reference.py:23-25)."""
    return np.repeat(x, group, axis=2) if group > 1 else x


def causal_mask(seqlen_q: int, seqlen_k: int) -> np.ndarray:
    """[S_q, S_k] bool, True where the key is hidden (reference.py:16-20)."""
    rows = np.arange(seqlen_q)[:, None]
    cols = np.arange(seqlen_k)[None, :]
    return cols > rows + (seqlen_k - seqlen_q)


def _softmax_rows(scores: np.ndarray):
    """Natural-log LSE of the last axis and exp(scores - lse), with rows of all -inf mapped to
    probability 0 and LSE -inf (reference.py:52-55)."""
    row_max = scores.max(axis=-1, keepdims=True)
    finite = np.isfinite(row_max)
    shift = np.where(finite, row_max, 0.0)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        e = np.exp(scores - shift)
        total = e.sum(axis=-1, keepdims=True)
        lse = np.where(total > 0, shift + np.log(np.where(total > 0, total, 1.0)), NEG_INF)
    lse_shift = np.where(np.isneginf(lse), 0.0, lse)
    probs = np.exp(scores - lse_shift)
    return probs, lse[..., 0]


def attention(q, k, v, causal: bool = False, softmax_scale: float | None = None,
              return_lse: bool = False, dtype=np.float64):
    """Materialises the scaled score matrix (reference.py:32-57). Returns o [B, S_q, H, D]
    (and lse [B, H, S_q])."""
    q_, k_, v_ = _as(q, dtype), _as(k, dtype), _as(v, dtype)
    batch, seqlen_q, heads, head_dim = q_.shape
    seqlen_k, heads_kv = k_.shape[1], k_.shape[2]
    group = heads // heads_kv
    scale = _default_scale(head_dim, softmax_scale)
    k_ = _expand_kv(k_, group)
    v_ = _expand_kv(v_, group)
    # [B, H, S_q, S_k] through BLAS: (B, H, S_q, D) @ (B, H, D, S_k)
    scores = np.matmul(q_.transpose(0, 2, 1, 3), k_.transpose(0, 2, 3, 1)) * dtype(scale)
    if causal:
        scores = np.where(causal_mask(seqlen_q, seqlen_k), NEG_INF, scores)
    probs, lse = _softmax_rows(scores)
    out = np.matmul(probs, v_.transpose(0, 2, 1, 3)).transpose(0, 2, 1, 3)
    out = np.ascontiguousarray(out, dtype=dtype)
    return (out, lse.astype(dtype)) if return_lse else out


def attention_rows(q, k, v, rows, causal: bool = False, softmax_scale: float | None = None,
                   dtype=np.float64, return_lse: bool = False):
    """attention() for the listed query rows only, [B, len(rows), H, D] (reference.py:60-87).
    The causal mask uses each row's position in the full sequence."""
    q_, k_, v_ = _as(q, dtype), _as(k, dtype), _as(v, dtype)
    rows = np.asarray(rows, dtype=np.int64)
    batch, seqlen_q, heads, head_dim = q_.shape
    seqlen_k, heads_kv = k_.shape[1], k_.shape[2]
    group = heads // heads_kv
    scale = _default_scale(head_dim, softmax_scale)
    qr = q_[:, rows]
    k_ = _expand_kv(k_, group)
    v_ = _expand_kv(v_, group)
    scores = np.matmul(qr.transpose(0, 2, 1, 3), k_.transpose(0, 2, 3, 1)) * dtype(scale)
    if causal:
        cols = np.arange(seqlen_k)[None, :]
        hidden = cols > rows[:, None] + (seqlen_k - seqlen_q)
        scores = np.where(hidden, NEG_INF, scores)
    probs, lse = _softmax_rows(scores)
    out = np.matmul(probs, v_.transpose(0, 2, 1, 3)).transpose(0, 2, 1, 3)
    out = np.ascontiguousarray(out, dtype=dtype)
    return (out, lse.astype(dtype)) if return_lse else out


def attention_tiled(q, k, v, causal: bool = False, softmax_scale: float | None = None,
                    return_lse: bool = False, block_q: int = 64, block_k: int = 64,
                    dtype=np.float64):
    """FlashAttention-2 forward with the online softmax, tile by tile (reference.py:90-152).

    Never forms the [S_q, S_k] matrix. Tiles that lie entirely above the causal diagonal are
    skipped, tiles that cross it are masked, and a row whose running max is still -inf uses 0 as
    its reference point so its exponentials are exactly 0 (reference.py:126-144).
    """
    q_, k_, v_ = _as(q, dtype), _as(k, dtype), _as(v, dtype)
    batch, seqlen_q, heads, head_dim = q_.shape
    seqlen_k, heads_kv = k_.shape[1], k_.shape[2]
    group = heads // heads_kv
    scale = _default_scale(head_dim, softmax_scale)
    offset = seqlen_k - seqlen_q
    qh = q_.transpose(0, 2, 1, 3)                       # [B, H, S_q, D]
    kh = _expand_kv(k_, group).transpose(0, 2, 1, 3)    # [B, H, S_k, D]
    vh = _expand_kv(v_, group).transpose(0, 2, 1, 3)
    out = np.zeros_like(qh)
    lse = np.full(qh.shape[:-1], NEG_INF, dtype=dtype)
    for q0 in range(0, seqlen_q, block_q):
        q1 = min(q0 + block_q, seqlen_q)
        shape = (batch, heads, q1 - q0)
        row_max = np.full(shape, NEG_INF, dtype=dtype)
        row_sum = np.zeros(shape, dtype=dtype)
        acc = np.zeros(shape + (head_dim,), dtype=dtype)
        k_end = min(seqlen_k, q1 + offset) if causal else seqlen_k
        for k0 in range(0, max(k_end, 0), block_k):
            k1 = min(k0 + block_k, seqlen_k)
            s = np.matmul(qh[:, :, q0:q1], kh[:, :, k0:k1].transpose(0, 1, 3, 2)) * dtype(scale)
            if causal and k1 - 1 > q0 + offset:
                r = np.arange(q0, q1)[:, None]
                c = np.arange(k0, k1)[None, :]
                s = np.where(c > r + offset, NEG_INF, s)
            new_max = np.maximum(row_max, s.max(axis=-1))
            ref = np.where(np.isneginf(new_max), 0.0, new_max)
            with np.errstate(invalid="ignore"):
                alpha = np.exp(row_max - ref)
            p = np.exp(s - ref[..., None])
            row_sum = alpha * row_sum + p.sum(axis=-1)
            acc = alpha[..., None] * acc + np.matmul(p, vh[:, :, k0:k1])
            row_max = new_max
        seen = row_sum > 0
        safe = np.where(seen, row_sum, 1.0)
        out[:, :, q0:q1] = acc / safe[..., None]
        lse[:, :, q0:q1] = np.where(seen, row_max + np.log(safe), NEG_INF)
    out = np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return (out, lse) if return_lse else out


def gather_cache(cache, block_tables, batch_idx: int, length: int) -> np.ndarray:
    """Rows 0..length-1 of one sequence as [length, H_kv, D], from a contiguous
    [B, S_max, H_kv, D] cache or a paged [num_blocks, page, H_kv, D] pool (reference.py:155-164)."""
    cache = np.asarray(cache)
    if block_tables is None:
        return cache[batch_idx, :length]
    tables = np.asarray(block_tables)
    page = cache.shape[1]
    pages = tables[batch_idx, : -(-length // page)].astype(np.int64)
    return cache[pages].reshape(-1, *cache.shape[2:])[:length]


def decode(q, k_cache, v_cache, seq_lens, block_tables=None, softmax_scale: float | None = None,
           return_lse: bool = False, dtype=np.float64):
    """One query token per sequence against its first seq_lens[b] cached keys
    (reference.py:167-205). q is [B, 1, H, D] or [B, H, D]; o has q's rank; lse is [B, H].
    Lengths outside [1, S_max] raise ValueError, as the reference does (reference.py:187-188)."""
    q_ = _as(q, dtype)
    q3 = q_[:, 0] if q_.ndim == 4 else q_
    kc, vc = _as(k_cache, dtype), _as(v_cache, dtype)
    lens = np.asarray(_as(seq_lens, np.int64)).reshape(-1)
    tables = None if block_tables is None else _as(block_tables, np.int64)
    head_dim = q3.shape[-1]
    scale = _default_scale(head_dim, softmax_scale)
    max_seqlen = kc.shape[1] if tables is None else tables.shape[1] * kc.shape[1]
    outs, lses = [], []
    for b, length in enumerate(lens.tolist()):
        if not 1 <= length <= max_seqlen:
            raise ValueError(f"seq_lens[{b}] = {length} is outside [1, {max_seqlen}]")
        keys = gather_cache(kc, tables, b, length)
        values = gather_cache(vc, tables, b, length)
        o_b, lse_b = attention(q3[b][None, None], keys[None], values[None], softmax_scale=scale,
                               return_lse=True, dtype=dtype)
        outs.append(o_b[0, 0])
        lses.append(lse_b[0, :, 0])
    out = np.stack(outs)
    if q_.ndim == 4:
        out = out[:, None]
    lse = np.stack(lses)
    return (out, lse) if return_lse else out


def merge_partials(partial_o, partial_m, partial_l):
    """Fixed-order log-sum-exp merge of split-KV partials (the merge of csrc/decode/decode.cu:
    204-228 in the reference), in fp64.

    partial_o [..., S, D] holds unnormalised outputs sum_j 2^(s_j - m_s) v_j, partial_m [..., S]
    the log2-domain reference point m_s (-inf for an empty split) and partial_l [..., S] the sum
    of 2^(s_j - m_s). Returns o [..., D] and the natural-log LSE [...]:
        m = max_s m_s, l = sum_s l_s 2^(m_s - m), o = sum_s o_s 2^(m_s - m) / l,
        lse = m ln 2 + ln l, or o = 0 and lse = -inf when every split is empty.
    """
    po = np.asarray(partial_o, dtype=np.float64)
    pm = np.asarray(partial_m, dtype=np.float64)
    pl = np.asarray(partial_l, dtype=np.float64)
    m = pm.max(axis=-1)
    ref = np.where(np.isneginf(m), 0.0, m)
    with np.errstate(invalid="ignore"):
        f = np.where(np.isneginf(pm), 0.0, np.exp2(pm - ref[..., None]))
    num = (po * f[..., None]).sum(axis=-2)
    den = (pl * f).sum(axis=-1)
    seen = den > 0
    o = np.where(seen[..., None], num / np.where(seen, den, 1.0)[..., None], 0.0)
    lse = np.where(seen, ref * math.log(2.0) + np.log(np.where(seen, den, 1.0)), -np.inf)
    return o, lse

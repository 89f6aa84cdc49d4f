"""Pins the numpy oracle to the reference: every function against the golden vectors the real
flash_lab.reference produced (tests/golden/make_golden.py), at the reference's own exactness
tolerance atol=1e-12 (tests/test_reference.py:202 of the reference). Also the closed-form checks
the reference applies to its oracle (tests/test_reference.py:234-283). CPU only."""

import numpy as np
import pytest

import oracle
from golden_io import bf16_to_f32, load, manifest, names

EXACT = dict(rtol=0.0, atol=1e-12)


def close(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape
    assert np.array_equal(np.isneginf(a), np.isneginf(b))
    fin = np.isfinite(b)
    np.testing.assert_allclose(a[fin], b[fin], **EXACT)


@pytest.mark.parametrize("name", names("prefill") + names("prefill_causal_only"))
def test_attention_matches_reference_goldens(name):
    g = load(name)
    meta = manifest()[name]
    q, k, v = (bf16_to_f32(g[x]) for x in "qkv")
    for tag, causal in (("full", False), ("causal", True)):
        if f"o_{tag}" not in g:
            continue
        o, lse = oracle.attention(q, k, v, causal=causal, softmax_scale=meta["scale"],
                                  return_lse=True)
        close(o, g[f"o_{tag}"])
        close(lse, g[f"lse_{tag}"])


def test_rows_and_tiled_match_reference_goldens():
    g = load("rows_tiled")
    q, k, v = (bf16_to_f32(g[x]) for x in "qkv")
    for tag, causal in (("full", False), ("causal", True)):
        close(oracle.attention_rows(q, k, v, g["rows"], causal=causal), g[f"rows_{tag}"])
        o, lse = oracle.attention_tiled(q, k, v, causal=causal, return_lse=True, block_q=16,
                                        block_k=8)
        close(o, g[f"tiled_o_{tag}"])
        close(lse, g[f"tiled_lse_{tag}"])


@pytest.mark.parametrize("name", names("decode"))
def test_decode_matches_reference_goldens(name):
    g = load(name)
    q = bf16_to_f32(g["q"])
    kc, vc = bf16_to_f32(g["k_cache"]), bf16_to_f32(g["v_cache"])
    o, lse = oracle.decode(q, kc, vc, g["seq_lens"], return_lse=True)
    close(o, g["o"])
    close(lse, g["lse"])


def test_paged_decode_matches_reference_goldens():
    g = load("decode_paged")
    q = bf16_to_f32(g["q"])
    o, lse = oracle.decode(q, bf16_to_f32(g["k_pool"]), bf16_to_f32(g["v_pool"]), g["seq_lens"],
                           block_tables=g["block_tables"], return_lse=True)
    close(o, g["o_paged"])
    close(lse, g["lse_paged"])
    contiguous = oracle.decode(q, bf16_to_f32(g["k_cache"]), bf16_to_f32(g["v_cache"]),
                               g["seq_lens"])
    close(contiguous, g["o_contig"])


def rand(rng, *shape, scale=1.0):
    return rng.standard_normal(shape) * scale


def test_single_key_returns_its_value():
    rng = np.random.default_rng(0)
    q, k, v = rand(rng, 2, 5, 4, 8), rand(rng, 2, 1, 2, 8), rand(rng, 2, 1, 2, 8)
    out, lse = oracle.attention(q, k, v, return_lse=True)
    np.testing.assert_allclose(out, np.broadcast_to(np.repeat(v, 2, axis=2), out.shape), **EXACT)
    scores = np.einsum("bqhd,bkhd->bhqk", q, np.repeat(k, 2, axis=2)) / np.sqrt(8)
    np.testing.assert_allclose(lse, scores[..., 0], **EXACT)


def test_identical_keys_average_the_values():
    rng = np.random.default_rng(1)
    q, k, v = rand(rng, 1, 4, 2, 8), rand(rng, 1, 6, 2, 8), rand(rng, 1, 6, 2, 8)
    k = np.broadcast_to(k[:, :1], k.shape)
    out = oracle.attention(q, k, v)
    np.testing.assert_allclose(out, np.broadcast_to(v.mean(axis=1, keepdims=True), out.shape),
                               **EXACT)


def test_gqa_equals_repeated_kv_heads():
    rng = np.random.default_rng(2)
    q, k, v = rand(rng, 2, 9, 8, 16), rand(rng, 2, 11, 2, 16), rand(rng, 2, 11, 2, 16)
    grouped = oracle.attention(q, k, v, causal=True)
    repeated = oracle.attention(q, np.repeat(k, 4, axis=2), np.repeat(v, 4, axis=2), causal=True)
    np.testing.assert_allclose(grouped, repeated, **EXACT)


def test_rows_without_visible_keys_are_zero():
    rng = np.random.default_rng(3)
    q, k, v = rand(rng, 2, 5, 2, 8), rand(rng, 2, 2, 1, 8), rand(rng, 2, 2, 1, 8)
    out, lse = oracle.attention(q, k, v, causal=True, return_lse=True)
    assert np.all(out[:, :3] == 0) and np.all(np.isneginf(lse[:, :, :3]))
    assert np.isfinite(out).all() and np.isfinite(lse[:, :, 3:]).all()


def test_large_scores_stay_finite_in_fp32():
    rng = np.random.default_rng(4)
    q, k, v = rand(rng, 1, 64, 2, 64, scale=10), rand(rng, 1, 64, 2, 64, scale=10), \
        rand(rng, 1, 64, 2, 64)
    out32 = oracle.attention(q, k, v, causal=True, dtype=np.float32)
    out64 = oracle.attention(q, k, v, causal=True)
    assert np.isfinite(out32).all()
    np.testing.assert_allclose(out32.astype(np.float64), out64, rtol=0, atol=1e-2)


def test_decode_rejects_lengths_outside_the_cache():
    rng = np.random.default_rng(5)
    kc, vc = rand(rng, 2, 8, 1, 8), rand(rng, 2, 8, 1, 8)
    q = rand(rng, 2, 1, 1, 8)
    for lens in ([3, 9], [0, 1]):
        with pytest.raises(ValueError, match="outside"):
            oracle.decode(q, kc, vc, np.array(lens, dtype=np.int32))


def test_merge_partials_equals_unsplit_attention():
    """The split-KV merge over any split boundaries reproduces the unsplit row exactly (fp64)."""
    rng = np.random.default_rng(6)
    d, n = 16, 37
    q, k, v = rand(rng, d), rand(rng, n, d), rand(rng, n, d)
    s = (k @ q) / np.sqrt(d) * np.log2(np.e)          # log2-domain scores
    bounds = [0, 5, 5, 20, 37]                        # includes an empty split
    po, pm, pl = [], [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        if a == b:
            po.append(np.zeros(d)); pm.append(-np.inf); pl.append(0.0)
            continue
        m = s[a:b].max()
        p = np.exp2(s[a:b] - m)
        po.append(p @ v[a:b]); pm.append(m); pl.append(p.sum())
    o, lse = oracle.merge_partials(np.array(po), np.array(pm), np.array(pl))
    ref, ref_lse = oracle.attention(q[None, None, None], k[None, :, None], v[None, :, None],
                                    return_lse=True)
    np.testing.assert_allclose(o, ref[0, 0, 0], **EXACT)
    np.testing.assert_allclose(lse, ref_lse[0, 0, 0], **EXACT)
    o0, lse0 = oracle.merge_partials(np.zeros((2, d)), np.array([-np.inf] * 2), np.zeros(2))
    assert np.all(o0 == 0) and np.isneginf(lse0)

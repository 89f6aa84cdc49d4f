"""flash_lab.reference (the torch fp64 utility kept for source compatibility) agrees with the
numpy oracle, which is itself pinned to the reference's golden vectors. CPU only."""

import numpy as np
import torch

import oracle
from flash_lab import reference
from golden_io import bf16_to_f32, load


def test_attention_matches_oracle():
    g = load("prefill_4")  # S_q < S_k, GQA
    q, k, v = (torch.from_numpy(bf16_to_f32(g[x])) for x in "qkv")
    for causal in (False, True):
        o, lse = reference.attention(q, k, v, causal=causal, return_lse=True)
        o2, lse2 = oracle.attention(q.numpy(), k.numpy(), v.numpy(), causal=causal,
                                    return_lse=True)
        np.testing.assert_allclose(o.numpy(), o2, rtol=0, atol=1e-12)
        np.testing.assert_allclose(lse.numpy(), lse2, rtol=0, atol=1e-12)
        rows = torch.tensor([0, 5, 36])
        part = reference.attention_rows(q, k, v, rows, causal=causal)
        np.testing.assert_allclose(part.numpy(), o2[:, rows.numpy()], rtol=0, atol=1e-12)


def test_decode_matches_oracle_contiguous_and_paged():
    g = load("decode_paged")
    q = torch.from_numpy(bf16_to_f32(g["q"]))
    lens = torch.from_numpy(g["seq_lens"])
    o = reference.decode(q, torch.from_numpy(bf16_to_f32(g["k_pool"])),
                         torch.from_numpy(bf16_to_f32(g["v_pool"])), lens,
                         block_tables=torch.from_numpy(g["block_tables"]))
    np.testing.assert_allclose(o.numpy(), g["o_paged"], rtol=0, atol=1e-12)


def test_attention_tiled_matches_the_reference_goldens():
    """reference.attention_tiled against the fixture the real reference's attention_tiled wrote
    (block_q=16, block_k=8; S_q=70 > S_k=50, GQA, so causal has rows without keys), and against
    the dense attention()."""
    g = load("rows_tiled")
    q, k, v = (torch.from_numpy(bf16_to_f32(g[x])) for x in "qkv")
    for tag, causal in (("full", False), ("causal", True)):
        o, lse = reference.attention_tiled(q, k, v, causal=causal, return_lse=True, block_q=16,
                                           block_k=8)
        np.testing.assert_allclose(o.numpy(), g[f"tiled_o_{tag}"], rtol=0, atol=1e-12)
        np.testing.assert_allclose(lse.numpy(), g[f"tiled_lse_{tag}"], rtol=0, atol=1e-12)
        dense, dense_lse = reference.attention(q, k, v, causal=causal, return_lse=True)
        np.testing.assert_allclose(o.numpy(), dense.numpy(), rtol=0, atol=1e-12)
        np.testing.assert_allclose(lse.numpy(), dense_lse.numpy(), rtol=0, atol=1e-12)

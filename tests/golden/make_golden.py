"""Writes the golden vectors that pin the oracle to the reference's own implementation.

Run once in a container that has the reference checked out (it imports the real
flash_lab.reference, pure PyTorch, on the CPU):

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py [case ...]

With case names, only those fixtures are rewritten (the manifest always lists every case).

For each case it draws seeded N(0, 1) inputs with torch's CPU generator, rounds them to bf16 (the
dtype the kernels run in), calls flash_lab.reference (attention, attention_rows, attention_tiled,
decode, paged decode) in fp64, and stores the inputs as raw bf16 bits plus the fp64 outputs in
tests/golden/<case>.npz. The fixtures are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import json
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent


def bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def rnd(gen, *shape, scale=1.0):
    return (torch.randn(*shape, generator=gen, dtype=torch.float64) * scale).to(torch.bfloat16)


def main() -> int:
    try:
        from flash_lab import reference
    except ImportError as exc:  # pragma: no cover
        print(f"needs the reference package on PYTHONPATH: {exc}", file=sys.stderr)
        return 1

    manifest = {}
    only = set(sys.argv[1:])

    def save(name, meta, **arrays):
        if not only or name in only:
            np.savez_compressed(HERE / f"{name}.npz", **arrays)
        manifest[name] = meta

    # C0, the benchmark's CPU-plumbing configuration: B=1, H=H_kv=4, S=256, D=64, scale 1/8.
    gen = torch.Generator().manual_seed(0)
    q, k, v = rnd(gen, 1, 256, 4, 64), rnd(gen, 1, 256, 4, 64), rnd(gen, 1, 256, 4, 64)
    outs = {}
    for causal in (False, True):
        o, lse = reference.attention(q, k, v, causal=causal, softmax_scale=0.125, return_lse=True)
        tag = "causal" if causal else "full"
        outs[f"o_{tag}"] = o.numpy()
        outs[f"lse_{tag}"] = lse.numpy()
    save("c0_prefill", {"kind": "prefill", "scale": 0.125, "shape": [1, 256, 256, 4, 4, 64]},
         q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v), **outs)

    # Prefill shapes of the reference's kernel tests (tests/test_attention_fwd.py:74-87),
    # the ones small enough to store: ragged, GQA, S_q < S_k, S_q > S_k, one query row.
    shapes = [
        (1, 1, 1, 1, 1, 64),
        (3, 7, 7, 8, 8, 64),
        (1, 16, 16, 1, 1, 128),
        (1, 63, 63, 4, 2, 128),
        (2, 37, 101, 4, 2, 64),
        (1, 101, 37, 4, 4, 128),
        (1, 1, 300, 8, 2, 128),
    ]
    for i, (b, sq, sk, h, hkv, d) in enumerate(shapes):
        gen = torch.Generator().manual_seed(100 + i)
        q, k, v = rnd(gen, b, sq, h, d), rnd(gen, b, sk, hkv, d), rnd(gen, b, sk, hkv, d)
        outs = {}
        for causal in (False, True):
            o, lse = reference.attention(q, k, v, causal=causal, return_lse=True)
            tag = "causal" if causal else "full"
            outs[f"o_{tag}"] = o.numpy()
            outs[f"lse_{tag}"] = lse.numpy()
        save(f"prefill_{i}", {"kind": "prefill", "scale": None, "shape": [b, sq, sk, h, hkv, d]},
             q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v), **outs)

    # Scores of order 100 (tests/test_attention_fwd.py:160-165): q and k scaled by 10.
    gen = torch.Generator().manual_seed(7)
    q, k, v = rnd(gen, 1, 129, 4, 64, scale=10.0), rnd(gen, 1, 129, 2, 64, scale=10.0), \
        rnd(gen, 1, 129, 2, 64)
    o, lse = reference.attention(q, k, v, causal=True, return_lse=True)
    save("large_scores", {"kind": "prefill_causal_only", "scale": None,
                          "shape": [1, 129, 129, 4, 2, 64]},
         q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v), o_causal=o.numpy(),
         lse_causal=lse.numpy())

    # attention_rows and attention_tiled on one ragged GQA problem (reference.py:60-152).
    gen = torch.Generator().manual_seed(11)
    q, k, v = rnd(gen, 2, 70, 4, 16), rnd(gen, 2, 50, 2, 16), rnd(gen, 2, 50, 2, 16)
    rows = torch.tensor([0, 7, 31, 69])
    extra = {}
    for causal in (False, True):
        tag = "causal" if causal else "full"
        extra[f"rows_{tag}"] = reference.attention_rows(q, k, v, rows, causal=causal).numpy()
        o_t, lse_t = reference.attention_tiled(q, k, v, causal=causal, return_lse=True,
                                               block_q=16, block_k=8)
        extra[f"tiled_o_{tag}"] = o_t.numpy()
        extra[f"tiled_lse_{tag}"] = lse_t.numpy()
    save("rows_tiled", {"kind": "rows_tiled", "shape": [2, 70, 50, 4, 2, 16]},
         q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v), rows=rows.numpy(), **extra)

    # Decode cases from tests/test_decode.py:232-240 (the small ones), a GQA-4 case, and a
    # ragged batch long enough for several splits (on B200 a length-balanced launch, whose CTAs
    # hold parts of several short sequences).
    decode_cases = [
        (1, 8, 8, 64, 64, [64]),
        (2, 6, 2, 300, 64, [300, 17]),
        (4, 8, 1, 260, 128, [1, 5, 129, 260]),
        (3, 16, 4, 120, 128, [120, 40, 77]),
        (6, 4, 1, 1100, 64, [1100, 1, 3, 64, 700, 65]),
    ]
    for i, (b, h, hkv, smax, d, lens) in enumerate(decode_cases):
        gen = torch.Generator().manual_seed(200 + i)
        q = rnd(gen, b, 1, h, d)
        kc, vc = rnd(gen, b, smax, hkv, d), rnd(gen, b, smax, hkv, d)
        seq_lens = torch.tensor(lens, dtype=torch.int32)
        o, lse = reference.decode(q, kc, vc, seq_lens, return_lse=True)
        save(f"decode_{i}", {"kind": "decode", "shape": [b, h, hkv, smax, d], "lens": lens},
             q=bf16_bits(q), k_cache=bf16_bits(kc), v_cache=bf16_bits(vc),
             seq_lens=seq_lens.numpy(), o=o.numpy(), lse=lse.numpy())

    # Paged decode (tests/test_reference.py:317-356): shuffled pages plus unused blocks.
    gen = torch.Generator().manual_seed(300)
    batch, smax, h, hkv, d, page = 3, 16, 4, 1, 8, 4
    kc, vc = rnd(gen, batch, smax, hkv, d), rnd(gen, batch, smax, hkv, d)
    pages_per_seq = smax // page
    num_blocks = batch * pages_per_seq + 3
    order = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(1))
    order = order[: batch * pages_per_seq]
    tables = order.view(batch, pages_per_seq).to(torch.int32)
    k_pool = torch.zeros(num_blocks, page, hkv, d, dtype=torch.bfloat16)
    v_pool = torch.zeros(num_blocks, page, hkv, d, dtype=torch.bfloat16)
    k_pool[order.long()] = kc.reshape(batch * pages_per_seq, page, hkv, d)
    v_pool[order.long()] = vc.reshape(batch * pages_per_seq, page, hkv, d)
    q = rnd(gen, batch, h, d)
    seq_lens = torch.tensor([5, 16, 9], dtype=torch.int32)
    o_paged, lse_paged = reference.decode(q, k_pool, v_pool, seq_lens, block_tables=tables,
                                          return_lse=True)
    o_contig = reference.decode(q, kc, vc, seq_lens)
    save("decode_paged", {"kind": "decode_paged", "page_size": page},
         q=bf16_bits(q), k_cache=bf16_bits(kc), v_cache=bf16_bits(vc),
         k_pool=bf16_bits(k_pool), v_pool=bf16_bits(v_pool), block_tables=tables.numpy(),
         seq_lens=seq_lens.numpy(), o_paged=o_paged.numpy(), lse_paged=lse_paged.numpy(),
         o_contig=o_contig.numpy())

    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(manifest)} fixtures to {HERE}")
    return 0


if __name__ == "__main__":
    sys.exit(main())

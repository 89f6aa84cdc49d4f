"""Hugging Face transformers integration: attn_implementation="flash_lab".

    import flash_lab.hf
    flash_lab.hf.register()
    model = AutoModelForCausalLM.from_pretrained(name, attn_implementation="flash_lab")

Same contract as flash_lab/hf.py of the reference (hf.py:27-88): prompt processing (several query
tokens) runs flash_lab.attention with causal masking on the valid cache rows; each generated
token (one query token) runs flash_lab.decode directly on the whole KV cache buffer of the layer,
read in place through the strides of the [B, H_kv, max_len, D] -> [B, max_len, H_kv, D] view, with
seq_lens from position_ids and no host sync, so generate() can compile and graph-capture the
decode step. transformers builds no mask for an unknown attention implementation, so batches must
be unpadded (every sequence starts at position 0 and all have the same length); prefill checks it.
"""

from __future__ import annotations

from functools import partial

import torch

from flash_lab.ops import attention, decode

NAME = "flash_lab"


def attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                      value: torch.Tensor, attention_mask: torch.Tensor | None,
                      scaling: float | None = None, dropout: float = 0.0, *,
                      prefill_impl: str = "auto", decode_impl: str = "auto", **kwargs):
    """transformers' attention-function signature: query is [B, H, S_q, D], key and value are
    [B, H_kv, S_k, D] (the whole buffer for a static cache); returns ([B, S_q, H, D], None)."""
    if dropout:
        raise ValueError("flash_lab attention has no dropout; call model.eval() first")
    if kwargs.get("sliding_window") is not None:
        raise NotImplementedError("flash_lab attention has no sliding-window masking")
    position_ids = kwargs.get("position_ids")
    if position_ids is None:
        raise ValueError("flash_lab attention needs position_ids to find the valid cache rows")

    batch, _, seqlen_q, _ = query.shape
    q, k, v = query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2)
    last = position_ids[:, -1]
    if seqlen_q == 1:
        # No host sync here: this is the step generate() compiles and replays.
        seq_lens = (last + 1).to(torch.int32).expand(batch).contiguous()
        return decode(q, k, v, seq_lens, softmax_scale=scaling, impl=decode_impl), None

    ends = set(last.tolist())
    if len(ends) != 1:
        raise ValueError("flash_lab attention supports unpadded batches only")
    seqlen_k = ends.pop() + 1
    if not seqlen_q <= seqlen_k <= k.shape[1]:
        raise ValueError(
            f"position_ids end at {seqlen_k - 1}, which does not fit {seqlen_q} new tokens "
            f"and a cache of {k.shape[1]} rows"
        )
    out = attention(q, k[:, :seqlen_k], v[:, :seqlen_k], causal=getattr(module, "is_causal", True),
                    softmax_scale=scaling, impl=prefill_impl)
    return out, None


def register(name: str = NAME, prefill_impl: str = "auto", decode_impl: str = "auto") -> str:
    """Registers attention_forward with transformers under `name` and returns the name to pass
    as attn_implementation."""
    from transformers import AttentionInterface

    AttentionInterface.register(
        name, partial(attention_forward, prefill_impl=prefill_impl, decode_impl=decode_impl)
    )
    return name

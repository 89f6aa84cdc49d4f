"""flash_lab as a transformers attention backend, end to end on a small random-init Llama
(reference tests/test_e2e_llama.py, without its checkpoint): logits against SDPA and an fp32
model, greedy generation with a static cache, and the compiled static-cache decode step.
Runs the sm_100a prefill and decode kernels through flash_lab.hf."""

import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")


def make_model(attn: str, dtype=torch.bfloat16, seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM

    import flash_lab.hf

    flash_lab.hf.register()
    cfg = LlamaConfig(vocab_size=1024, hidden_size=1024, intermediate_size=2048,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=128, max_position_embeddings=1024, rope_theta=500000.0)
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = LlamaForCausalLM(cfg)
    model = model.to(dtype).eval()
    model.config._attn_implementation = attn
    return model


def prompt(n=300, seed=1):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randint(0, 1024, (1, n), device="cuda", generator=gen)


@torch.no_grad()
def test_prefill_logits_match_sdpa_quality():
    ids = prompt()
    ref = make_model("sdpa", torch.float32)(ids).logits.double()
    ours = make_model("flash_lab")(ids).logits.double()
    sdpa = make_model("sdpa")(ids).logits.double()
    err = (ours - ref).abs().max().item()
    err_sdpa = (sdpa - ref).abs().max().item()
    # The reference's e2e rule: flash_lab's logit error is at most twice SDPA's at bf16.
    assert err <= 2 * err_sdpa, (err, err_sdpa)


@torch.no_grad()
def test_static_cache_greedy_generation_follows_sdpa():
    ids = prompt(200, seed=2)
    outs = {}
    for attn in ("sdpa", "flash_lab"):
        model = make_model(attn)
        out = model.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=24,
                             do_sample=False, cache_implementation="static", pad_token_id=0)
        outs[attn] = out[0, ids.shape[1]:]
    same = (outs["sdpa"] == outs["flash_lab"]).int()
    # bf16 rounding can flip a near-tie; the first several tokens must agree.
    assert same[:8].all(), (outs["sdpa"].tolist(), outs["flash_lab"].tolist())


@torch.no_grad()
def test_compiled_static_cache_decode():
    from transformers import CompileConfig

    torch._dynamo.reset()
    ids = prompt(120, seed=3)
    model = make_model("flash_lab")
    eager = model.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=12,
                           do_sample=False, cache_implementation="static", pad_token_id=0)
    model.generation_config.compile_config = CompileConfig(fullgraph=True)
    compiled = model.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=12,
                              do_sample=False, cache_implementation="static", pad_token_id=0,
                              compile_config=CompileConfig(fullgraph=True))
    assert torch.equal(eager, compiled)

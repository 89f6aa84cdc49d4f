"""flash_lab as a transformers attention backend, end to end on a small random-init Llama
(reference tests/test_e2e_llama.py, without its checkpoint): logits against SDPA and an fp32
model, greedy generation with a static cache, and the compiled static-cache decode step.
Runs the sm_100a prefill and decode kernels through flash_lab.hf."""

import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")


def make_model(attn: str, dtype=torch.bfloat16, seed=0, full_width=False):
    """A small random-init Llama: 2 layers of width 1024 (8 / 2 heads), or (full_width) one
    layer of the Llama-3.1-8B architecture's width (d_model 4096, 32 query / 8 KV heads of 128,
    MLP 14336), with a 1024-token vocabulary either way."""
    from transformers import LlamaConfig, LlamaForCausalLM

    import flash_lab.hf

    flash_lab.hf.register()
    if full_width:
        cfg = LlamaConfig(vocab_size=1024, hidden_size=4096, intermediate_size=14336,
                          num_hidden_layers=1, num_attention_heads=32, num_key_value_heads=8,
                          head_dim=128, max_position_embeddings=4096, rope_theta=500000.0)
    else:
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
def test_full_width_layer_logits_and_decode_match_sdpa_quality():
    # One layer at the Llama-3.1-8B width (GQA 32/8): prefill logits over a 1500-token prompt,
    # then a static-cache decode of 8 tokens, each against the fp32 SDPA model under the same
    # rule (at most twice the error of SDPA at bf16).
    ids = prompt(1500, seed=4)
    models = {name: make_model(attn, dtype, full_width=True)
              for name, attn, dtype in (("ref", "sdpa", torch.float32), ("ours", "flash_lab",
                                        torch.bfloat16), ("sdpa", "sdpa", torch.bfloat16))}
    logits = {name: m(ids).logits.double() for name, m in models.items()}
    err = (logits["ours"] - logits["ref"]).abs().max().item()
    err_sdpa = (logits["sdpa"] - logits["ref"]).abs().max().item()
    assert err <= 2 * err_sdpa, (err, err_sdpa)
    outs = {}
    for name in ("ours", "sdpa"):
        outs[name] = models[name].generate(ids, attention_mask=torch.ones_like(ids),
                                           max_new_tokens=8, do_sample=False,
                                           cache_implementation="static", pad_token_id=0,
                                           output_logits=True, return_dict_in_generate=True)
    assert torch.equal(outs["ours"].sequences[0, :ids.shape[1] + 1],
                       outs["sdpa"].sequences[0, :ids.shape[1] + 1])
    # The first decoded position's logits come from the decode kernel (one query token against
    # the 1500-entry static cache).
    step = torch.stack([x.double() for x in outs["ours"].logits[1:2]])
    step_sdpa = torch.stack([x.double() for x in outs["sdpa"].logits[1:2]])
    ref_step = models["ref"].generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=2,
                                      do_sample=False, cache_implementation="static",
                                      pad_token_id=0, output_logits=True,
                                      return_dict_in_generate=True)
    if torch.equal(ref_step.sequences[0, :ids.shape[1] + 1],
                   outs["ours"].sequences[0, :ids.shape[1] + 1]):
        ref_l = ref_step.logits[1].double()
        assert (step - ref_l).abs().max() <= 2 * (step_sdpa - ref_l).abs().max() + 1e-3


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

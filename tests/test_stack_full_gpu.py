"""Greedy-token match on the random-init Gemma-4-26B-A4B-shaped decoder at
its full shape: 30 layers (every sixth on full attention, the rest a 1024
sliding window), hidden 2816, 128 experts top-8, expert intermediate 704,
vocab 262144, weights N(0, 0.02), seed 0.

The product configuration (experts converted to NVFP4 on the GPU by the
checkpoint builder's expert step and run through ``Gemma4TextExpertsNVFP4``,
routers swapped for the fused kernel) prefills 2048 random token ids and
decodes 64 greedy tokens. The reference configuration runs the same model
with HF's own router and, in place of every swapped expert module, the
torch restatement of the reference forward (``oracle/torch_port.py``,
dequantize-then-matmul in f32 on the GPU, pinned to the numpy oracle by
``tests/test_torch_port.py``) over the same NVFP4 buffers. The greedy tokens
must be identical. (The reference's own gate, ``examples/parity_check.py``,
allows up to 5% of 50 tokens to differ.)

The dimensions BASELINE does not pin are the bench's choice: 16 query heads
and 8 KV heads of 256 (512 on full-attention layers), dense MLP 2112, no
per-layer input embedding.
"""
import pytest
import torch
import torch.nn as nn

from oracle import torch_port as TP

pytestmark = pytest.mark.gpu

PROMPT, NEW = 2048, 64
H, E, TOPK, I = 2816, 128, 8, 704


def stack_config(layers=30):
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    types_ = [("full_attention" if (i + 1) % 6 == 0 else "sliding_attention") for i in range(layers)]
    return Gemma4TextConfig(
        hidden_size=H, num_hidden_layers=layers, num_attention_heads=16, num_key_value_heads=8, head_dim=256,
        global_head_dim=512, intermediate_size=2112, moe_intermediate_size=I, num_experts=E, top_k_experts=TOPK,
        enable_moe_block=True, vocab_size=262144, vocab_size_per_layer_input=262144,
        hidden_size_per_layer_input=0, sliding_window=1024, layer_types=types_, max_position_embeddings=8192)


class TorchOracleExperts(nn.Module):
    """The reference forward restated in torch (f32 dequantize-then-matmul,
    every bf16 rounding point) over a converted module's NVFP4 buffers."""

    def __init__(self, m):
        super().__init__()
        self.m = TP.Experts(m.gate_up_proj, m.gate_up_proj_scale, m.gate_up_proj_scale_2.float(),
                            m.down_proj, m.down_proj_scale, m.down_proj_scale_2.float())
        self.calls = 0

    def forward(self, hidden_states, top_k_index, top_k_weights):
        self.calls += 1
        return TP.forward(self.m, hidden_states.to(torch.bfloat16), top_k_index, top_k_weights)


def greedy(model, ids, n):
    with torch.no_grad():
        out = model(ids, use_cache=True)
        pkv, nxt = out.past_key_values, out.logits[:, -1:].argmax(-1)
        last = out.logits[0, -1].float()
        toks = [int(nxt)]
        margins = []
        for _ in range(n - 1):
            out = model(nxt, past_key_values=pkv, use_cache=True)
            logits = out.logits[0, -1].float()
            top2 = torch.topk(logits, 2).values
            margins.append(float(top2[0] - top2[1]))
            pkv, nxt = out.past_key_values, out.logits[:, -1:].argmax(-1)
            toks.append(int(nxt))
    return toks, last, margins


def test_full_stack_greedy_tokens_match():
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM, Gemma4TextRouter
    from aeo_quant_b200.bridges.gemma4.loader import quantize_experts_to_nvfp4, swap_routers
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = Gemma4ForCausalLM(stack_config()).eval()
    torch.set_default_dtype(old)
    assert quantize_experts_to_nvfp4(model) == 30
    torch.cuda.empty_cache()
    ids = torch.randint(10, 262144, (1, PROMPT), generator=torch.Generator().manual_seed(1)).to(dev)

    # the layer-0 expert inputs of the prefill, to compare the two expert
    # implementations directly
    seen = {}

    def keep_first(mod, args, out):
        if "io" not in seen:
            seen["io"] = (tuple(a.clone() for a in args), out.clone())
    hook = model.model.layers[0].experts.register_forward_hook(keep_first)

    # product configuration: swapped experts and routers
    assert swap_routers(model) == 30
    ours, last_ours, _ = greedy(model, ids, NEW)
    hook.remove()
    (h0, i0, w0), y0 = seen["io"]
    assert h0.shape[0] == PROMPT
    oracle0 = TorchOracleExperts(model.model.layers[0].experts)
    with torch.no_grad():
        r0 = oracle0(h0, i0, w0).float()
    layer0_rel = float((y0.float() - r0).abs().max() / r0.abs().max())
    assert 0 < float(r0.abs().max()) and layer0_rel <= 2e-3, layer0_rel

    # reference configuration: HF's router, torch restatement of the experts
    swapped = []
    for layer in model.model.layers:
        layer.router.__class__ = Gemma4TextRouter
        swapped.append(layer.experts)
        layer.experts = TorchOracleExperts(layer.experts)
    ref, last_ref, margins = greedy(model, ids, NEW)
    assert all(layer.experts.calls == NEW for layer in model.model.layers)   # prefill + NEW - 1 decodes
    for layer, m in zip(model.model.layers, swapped):
        layer.experts = m

    rel = float((last_ours - last_ref).abs().max() / last_ref.abs().max())
    first = next((i for i, (a, b) in enumerate(zip(ours, ref)) if a != b), None)
    print(f"layer-0 prefill expert output vs the torch oracle: max rel diff {layer0_rel:.2e}; "
          f"prefill logits max rel diff {rel:.2e}; first differing step {first}; "
          f"smallest top-2 logit margin of the reference run {min(margins):.3e}")
    assert rel <= 2e-2
    assert ours == ref

"""A random-init Gemma-4 decoder stack with its experts converted to NVFP4
on the GPU (the checkpoint builder's expert step) and run through the
swapped ``Gemma4TextExpertsNVFP4``: prefill through the grouped path, greedy
decode through the one-token path. The same model with an oracle experts
module in place of every swapped module must produce the same greedy tokens
and prefill logits within tolerance."""
import numpy as np
import pytest
import torch
import torch.nn as nn

from helpers import TOL, bf16_to_np, max_rel_err
from oracle import moe as OM

pytestmark = pytest.mark.gpu

PROMPT, NEW = 48, 8


class OracleExperts(nn.Module):
    """The oracle restatement of ``Gemma4TextExpertsNVFP4.forward`` over the
    buffers of a converted module (runs on the host)."""

    def __init__(self, m):
        super().__init__()
        u8 = lambda t: t.detach().view(torch.uint8).cpu().numpy()
        self.om = OM.NVFP4Experts(u8(m.gate_up_proj), u8(m.gate_up_proj_scale), float(m.gate_up_proj_scale_2),
                                  u8(m.down_proj), u8(m.down_proj_scale), float(m.down_proj_scale_2))

    def forward(self, hidden_states, top_k_index, top_k_weights):
        y = OM.nvfp4_experts_forward(self.om, bf16_to_np(hidden_states), top_k_index.cpu().numpy(),
                                     bf16_to_np(top_k_weights))
        out = torch.from_numpy(np.ascontiguousarray(y, np.float32)).to(torch.bfloat16)
        return out.to(hidden_states.device)


def small_config():
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    return Gemma4TextConfig(
        hidden_size=512, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
        global_head_dim=128, intermediate_size=1024, moe_intermediate_size=256, num_experts=16, top_k_experts=8,
        enable_moe_block=True, vocab_size=4096, vocab_size_per_layer_input=4096, hidden_size_per_layer_input=0,
        sliding_window=32, layer_types=["sliding_attention", "full_attention"], initializer_range=0.1)


@pytest.fixture(scope="module")
def stack():
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    from aeo_quant_b200.bridges.gemma4.loader import quantize_experts_to_nvfp4
    from aeo_quant_b200.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4
    torch.manual_seed(0)
    model = Gemma4ForCausalLM(small_config()).to(device="cuda", dtype=torch.bfloat16).eval()
    # random-init router: give it a spread so that routing is not uniform
    for layer in model.model.layers:
        nn.init.normal_(layer.router.proj.weight, std=0.5)
    assert quantize_experts_to_nvfp4(model) == 2
    assert all(isinstance(l.experts, Gemma4TextExpertsNVFP4) for l in model.model.layers)
    return model


def _greedy(model, ids):
    """Greedy tokens and the logits of every generated position."""
    with torch.no_grad():
        out = model.generate(ids, max_new_tokens=NEW, do_sample=False, min_new_tokens=NEW,
                             output_logits=True, return_dict_in_generate=True)
    logits = torch.stack([l[0].float() for l in out.logits]).cpu()
    return out.sequences[0, ids.shape[1]:].cpu(), logits


def test_converted_buffer_layout(stack):
    m = stack.model.layers[0].experts
    assert m.gate_up_proj.dtype == torch.uint8 and m.gate_up_proj.shape == (16, 512, 256)
    assert m.down_proj_scale.dtype == torch.float8_e4m3fn and m.down_proj_scale.shape == (16, 512, 16)
    assert m.gate_up_proj_scale_2.dtype == torch.float32 and m.gate_up_proj_scale_2.dim() == 0


def test_greedy_matches_oracle_experts(stack):
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(10, 4096, (1, PROMPT), generator=g).cuda()
    tok, logits = _greedy(stack, ids)
    swapped = [l.experts for l in stack.model.layers]
    try:
        for l, m in zip(stack.model.layers, swapped):
            l.experts = OracleExperts(m)
        tok_ref, logits_ref = _greedy(stack, ids)
    finally:
        for l, m in zip(stack.model.layers, swapped):
            l.experts = m
    # The first generated position is the prefill (grouped path); the rest
    # are one-token decodes. Greedy tokens must agree; logits within 2e-2 of
    # their max (bf16 activations through the attention and MLP layers
    # amplify the experts' last-ulp differences).
    assert tok.tolist() == tok_ref.tolist()
    for i in range(NEW):
        err = float((logits[i] - logits_ref[i]).abs().max() / logits_ref[i].abs().max())
        assert err <= 2e-2, (i, err)


def test_every_expert_call_in_the_stack_vs_oracle(stack):
    """Each expert call the stack makes (HF's router output as routing;
    prefill and one-token decodes) against the oracle on the same inputs."""
    calls = []

    def record(mod, args, out):
        h, idx, w = args
        calls.append((mod, h.detach().clone(), idx.detach().clone(), w.detach().clone(), out.detach().clone()))

    hooks = [l.experts.register_forward_hook(record) for l in stack.model.layers]
    try:
        ids = torch.randint(10, 4096, (1, PROMPT), generator=torch.Generator().manual_seed(8)).cuda()
        _greedy(stack, ids)
    finally:
        for hk in hooks:
            hk.remove()
    assert len(calls) == 2 * NEW
    assert sum(1 for c in calls if c[1].shape[0] == 1) == 2 * (NEW - 1)
    oracles = {}
    for mod, h, idx, w, y in calls:
        om = oracles.setdefault(id(mod), OracleExperts(mod).om)
        ref = OM.nvfp4_experts_forward(om, bf16_to_np(h), idx.cpu().numpy(), bf16_to_np(w))
        assert max_rel_err(bf16_to_np(y), ref) <= TOL


def test_fused_router_in_stack(stack):
    """The stack with every router on the fused kernel generates the same
    greedy tokens as with HF's eager routers, logits within 2e-2."""
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextRouter
    from aeo_quant_b200.bridges.gemma4.loader import swap_routers
    ids = torch.randint(10, 4096, (1, PROMPT), generator=torch.Generator().manual_seed(9)).cuda()
    tok_ref, logits_ref = _greedy(stack, ids)
    try:
        assert swap_routers(stack) == 2
        tok, logits = _greedy(stack, ids)
    finally:
        for l in stack.model.layers:
            l.router.__class__ = Gemma4TextRouter
    assert tok.tolist() == tok_ref.tolist()
    for i in range(NEW):
        err = float((logits[i] - logits_ref[i]).abs().max() / logits_ref[i].abs().max())
        assert err <= 2e-2, (i, err)

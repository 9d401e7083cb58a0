"""The router oracle against HF transformers' own Gemma4TextRouter (the
reference implementation of the router, transformers 5.5.0), run on the
CPU in bfloat16."""
import numpy as np
import pytest
import torch

from helpers import bf16_to_np, check_router
from oracle import router as OR


def hf_router(H, E, k, seed, proj_std):
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextRouter
    cfg = Gemma4TextConfig(hidden_size=H, num_experts=E, top_k_experts=k, moe_intermediate_size=64,
                           enable_moe_block=True)
    torch.manual_seed(seed)
    r = Gemma4TextRouter(cfg)
    with torch.no_grad():
        r.proj.weight.normal_(0.0, proj_std)
        r.scale.uniform_(0.5, 1.5)
        r.per_expert_scale.uniform_(0.5, 2.0)
    return r.to(torch.bfloat16).eval()


def oracle_of(r, x):
    return OR.gemma4_router(bf16_to_np(x), bf16_to_np(r.scale.detach()), bf16_to_np(r.proj.weight.detach()),
                            bf16_to_np(r.per_expert_scale.detach()), r.config.top_k_experts, r.eps)


# proj std 0.02 (HF init) makes the probabilities nearly uniform: most of
# them tie in bf16 and the sets may differ wherever the order of equal
# values decides; check_router still requires every difference to be a tie.
@pytest.mark.parametrize("H,E,k,T,std,max_differ", [(2816, 128, 8, 16, 0.02, 16), (2816, 128, 8, 16, 0.5, 4),
                                                    (512, 16, 4, 9, 0.3, 2)])
def test_oracle_matches_hf_router(H, E, k, T, std, max_differ):
    r = hf_router(H, E, k, 3, std)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(4)) * 2.0).to(torch.bfloat16)
    with torch.no_grad():
        p, w, i = r(x)
    op, ow, oi = oracle_of(r, x)
    differ = check_router(op, ow, oi, bf16_to_np(p), bf16_to_np(w), i.numpy())
    assert differ <= max_differ

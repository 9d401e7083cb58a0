"""The NVFP4 checkpoint builder with the GPU quantizer, end to end: a bf16
Gemma-4 checkpoint is converted, the expert tensors are checked bit for bit
against the oracle quantizer, and the checkpoint loaded under the class swap
generates the same greedy tokens as the same weights converted in memory."""
import json

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import quant as OQ
from test_stack_gpu import small_config

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def source(tmp_path_factory):
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    root = tmp_path_factory.mktemp("ckpt_gpu")
    torch.manual_seed(0)
    model = Gemma4ForCausalLM(small_config()).to(torch.bfloat16).eval()
    for layer in model.model.layers:
        nn.init.normal_(layer.router.proj.weight, std=0.5)
    model.save_pretrained(root / "src")
    return model, root


def test_builder_bit_exact_and_generation(source):
    from safetensors import safe_open
    from aeo_quant_b200.bridges.gemma4.checkpoint import build_checkpoint_nvfp4, is_expert_key
    from aeo_quant_b200.bridges.gemma4.loader import load_gemma4_nvfp4, quantize_experts_to_nvfp4, swap_routers
    from aeo_quant_b200.bridges.gemma4.router import Gemma4TextRouterB200

    model, root = source
    counts = build_checkpoint_nvfp4(root / "src", root / "out", device="cuda", log=None)
    assert counts["quantized"] == 4
    with open(root / "out" / "model.safetensors.index.json") as f:
        wm = json.load(f)["weight_map"]
    sd = model.state_dict()
    checked = 0
    for key in wm:
        if not is_expert_key(key):
            continue
        w = sd[key].float().numpy()
        E, N, K = w.shape
        op, osf, ots = OQ.quantize_nvfp4(w.reshape(E * N, K))
        with safe_open(str(root / "out" / wm[key]), "pt") as f:
            p = f.get_tensor(key)
        with safe_open(str(root / "out" / wm[key + "_scale"]), "pt") as f:
            s = f.get_tensor(key + "_scale")
        with safe_open(str(root / "out" / wm[key + "_scale_2"]), "pt") as f:
            ts = f.get_tensor(key + "_scale_2")
        assert np.array_equal(p.numpy().reshape(E * N, K // 2), op), key
        assert np.array_equal(s.view(torch.uint8).numpy().reshape(E * N, K // 16), osf), key
        assert ts.dtype == torch.bfloat16 and float(ts) == float(np.asarray(ots).reshape(-1)[0]), key
        checked += 1
    assert checked == 4

    loaded = load_gemma4_nvfp4(str(root / "out"), device_map="cuda").eval()
    assert all(isinstance(l.router, Gemma4TextRouterB200) for l in loaded.model.layers)
    ref = model.to("cuda")
    assert quantize_experts_to_nvfp4(ref) == 2 and swap_routers(ref) == 2
    ids = torch.randint(10, 4096, (1, 40), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        a = loaded.generate(ids, max_new_tokens=6, min_new_tokens=6, do_sample=False)
        b = ref.generate(ids, max_new_tokens=6, min_new_tokens=6, do_sample=False)
    assert torch.equal(a, b)

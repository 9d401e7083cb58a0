"""Host logic of the NVFP4 checkpoint builder and of the checkpoint load
path, on the CPU: shard streaming and naming, the index, the config stamp,
the three tensors per expert projection, pass-through of every other tensor,
and loading the result under the class swap. The quantizer is a stand-in
here (the builder accepts one); the GPU test runs the real one."""
import json
import os

import pytest
import torch

from aeo_quant_b200.bridges.gemma4 import checkpoint as C


def tiny_config():
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    return Gemma4TextConfig(
        hidden_size=256, num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1, head_dim=64,
        global_head_dim=64, intermediate_size=128, moe_intermediate_size=64, num_experts=8, top_k_experts=2,
        enable_moe_block=True, vocab_size=512, vocab_size_per_layer_input=512, hidden_size_per_layer_input=0,
        sliding_window=16, layer_types=["sliding_attention", "full_attention"])


def stand_in_quantize(t):
    """Right shapes and dtypes, content derived from the input so that the
    test can tell the tensors apart."""
    E, N, K = t.shape
    packed = (t.float() * 1000).round().to(torch.int64).remainder(256).to(torch.uint8)[..., ::2].contiguous()
    sf = torch.full((E, N, K // 16), 0.5).to(torch.float8_e4m3fn)
    return packed, sf, t.abs().amax().to(torch.bfloat16)


def source_tensors(root):
    from safetensors import safe_open
    with safe_open(str(root / "src" / "model.safetensors"), "pt") as f:
        return {k: f.get_tensor(k) for k in f.keys()}


@pytest.fixture(scope="module")
def built(tmp_path_factory):
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM
    root = tmp_path_factory.mktemp("ckpt")
    torch.manual_seed(0)
    model = Gemma4ForCausalLM(tiny_config()).to(torch.bfloat16)
    model.save_pretrained(root / "src")
    counts = C.build_checkpoint_nvfp4(root / "src", root / "out", device="cpu", quantize=stand_in_quantize,
                                      shard_size_bytes=100_000, log=None)
    return model, root, counts


def test_counts_shards_and_index(built):
    model, root, counts = built
    out = root / "out"
    n_src = len(source_tensors(root))
    assert counts["quantized"] == 4 and counts["passthrough"] == n_src - 4
    with open(out / "model.safetensors.index.json") as f:
        wm = json.load(f)["weight_map"]
    files = sorted(set(wm.values()))
    assert len(files) == counts["shards"] > 1
    n = len(files)
    assert files == [f"model-{i:05d}-of-{n:05d}.safetensors" for i in range(1, n + 1)]
    assert not [p for p in os.listdir(out) if p.endswith(".tmp")]
    from safetensors import safe_open
    seen = {}
    for fn in files:
        size, count = 0, 0
        with safe_open(str(out / fn), "pt") as f:
            for k in f.keys():
                t = f.get_tensor(k)
                seen[k] = fn
                size += t.numel() * t.element_size()
                count += 1
        assert size <= 100_000 or count == 1       # a tensor above the limit gets a shard of its own
    assert seen == wm
    assert len(wm) == n_src + 2 * 4


def test_expert_tensors_and_passthrough(built):
    model, root, _ = built
    from safetensors import safe_open
    out = root / "out"
    with open(out / "model.safetensors.index.json") as f:
        wm = json.load(f)["weight_map"]
    get = lambda k: safe_open(str(out / wm[k]), "pt").get_tensor(k)
    for name, t in source_tensors(root).items():
        if C.is_expert_key(name):
            p, s, ts = stand_in_quantize(t)
            assert torch.equal(get(name), p)
            assert torch.equal(get(name + "_scale").view(torch.uint8), s.view(torch.uint8))
            g2 = get(name + "_scale_2")
            assert g2.dim() == 0 and g2.dtype == torch.bfloat16 and torch.equal(g2, ts)
        else:
            assert torch.equal(get(name), t), name


def test_config_stamp(built):
    _, root, _ = built
    with open(root / "out" / "config.json") as f:
        cfg = json.load(f)
    assert cfg["aeo_quantization"] == {"quant_algo": "NVFP4", "block_size": 16}
    assert C.is_nvfp4_checkpoint(root / "out") and not C.is_nvfp4_checkpoint(root / "src")
    assert (root / "out" / "generation_config.json").exists()


def test_load_under_class_swap(built):
    from aeo_quant_b200.bridges.gemma4.loader import load_gemma4_nvfp4
    from aeo_quant_b200.bridges.gemma4.modeling_nvfp4 import Gemma4TextExpertsNVFP4
    model, root, _ = built
    m2 = load_gemma4_nvfp4(str(root / "out"), device_map="cpu")
    for i, layer in enumerate(m2.model.layers):
        ex = layer.experts
        assert isinstance(ex, Gemma4TextExpertsNVFP4)
        for proj in ("gate_up_proj", "down_proj"):
            p, s, ts = stand_in_quantize(getattr(model.model.layers[i].experts, proj).detach())
            assert torch.equal(getattr(ex, proj), p)
            assert torch.equal(getattr(ex, proj + "_scale").view(torch.uint8), s.view(torch.uint8))
            s2 = getattr(ex, proj + "_scale_2")
            assert s2.dtype == torch.float32 and s2.dim() == 0 and float(s2) == float(ts)
    sd2 = m2.state_dict()
    for k, v in source_tensors(root).items():
        if not C.is_expert_key(k):
            assert torch.equal(sd2[k], v), k


def test_single_file_source_and_errors(tmp_path, built):
    _, root, _ = built
    with pytest.raises(ValueError, match="differ"):
        C.build_checkpoint_nvfp4(root / "src", root / "src", device="cpu", quantize=stand_in_quantize)
    with pytest.raises(FileNotFoundError):
        C.build_checkpoint_nvfp4(tmp_path, tmp_path / "o", device="cpu", quantize=stand_in_quantize)
    from safetensors.torch import save_file
    src = tmp_path / "bad"
    src.mkdir()
    save_file({"model.layers.0.experts.gate_up_proj": torch.zeros(4, 4, dtype=torch.bfloat16)},
              str(src / "model.safetensors"))
    with pytest.raises(ValueError, match="fused"):
        C.build_checkpoint_nvfp4(src, tmp_path / "o2", device="cpu", quantize=stand_in_quantize, log=None)


def test_expert_key_pattern():
    assert C.is_expert_key("model.layers.3.experts.gate_up_proj")
    assert C.is_expert_key("model.language_model.layers.29.experts.down_proj")
    assert not C.is_expert_key("model.layers.3.experts.down_proj_scale")
    assert not C.is_expert_key("model.layers.3.router.proj.weight")


def test_device_map_without_accelerate():
    pytest.importorskip("transformers")
    try:
        import accelerate  # noqa: F401
        pytest.skip("accelerate is installed")
    except ImportError:
        pass
    from aeo_quant_b200.bridges.gemma4.loader import load_gemma4_nvfp4
    with pytest.raises(ValueError, match="accelerate"):
        load_gemma4_nvfp4("/nonexistent", device_map="auto")


def test_router_swap_only_supported_shapes():
    import torch.nn as nn
    from test_router_oracle import hf_router
    from aeo_quant_b200.bridges.gemma4.loader import swap_routers
    from aeo_quant_b200.bridges.gemma4.router import Gemma4TextRouterB200, router_supported
    ok, odd, narrow = hf_router(2816, 128, 8, 1, 0.02), hf_router(2816, 12, 4, 1, 0.02), hf_router(256, 128, 8, 1, 0.02)
    assert router_supported(ok) and not router_supported(odd) and not router_supported(narrow)
    # a router loaded in another dtype keeps HF's forward
    f32 = hf_router(2816, 128, 8, 1, 0.02).float()
    assert not router_supported(f32)
    seq = nn.Sequential(ok, odd, narrow)
    assert swap_routers(seq, only_supported=True) == 1
    assert type(ok) is Gemma4TextRouterB200 and type(odd) is not Gemma4TextRouterB200
    assert swap_routers(seq) == 2          # an explicit swap takes every router

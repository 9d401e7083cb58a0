"""NVFP4 checkpoint builder: a bf16 Gemma-4 safetensors checkpoint in, the
NVFP4 checkpoint that ``load_gemma4_nvfp4`` reads out.

Same output format as aeo_quant ``examples/build_checkpoint_nvfp4.py``:

* every fused 3-D expert tensor ``...layers.<i>.experts.{gate_up_proj,down_proj}``
  (:59-61, matched with or without the multimodal ``language_model.``
  prefix) becomes three tensors (:140-151): ``<proj>`` packed E2M1 (u8, two
  per byte, high nibble = even k), ``<proj>_scale`` e4m3 block scales per 16
  values, ``<proj>_scale_2`` the 0-d bf16 tensor scale;
* every other tensor is copied unchanged (:153-156);
* shards of at most ``shard_size_bytes`` (5 GiB by default, :48) named
  ``model-<i>-of-<n>.safetensors`` with ``model.safetensors.index.json``
  (:100-191);
* ``config.json`` (and the generation / tokenizer / template files) copied
  with ``"aeo_quantization": {"quant_algo": "NVFP4", "block_size": 16}``
  added (:193-205).

The source is streamed one shard at a time, as in the reference. The
difference is where quantization runs: each expert tensor is moved to the
GPU and quantized there by ``quantize_3d_to_nvfp4`` (the sm_100a kernels),
then the packed result comes back to host memory for writing. One expert
tensor (about 1 GB in bf16 at the Gemma-4-26B-A4B shapes) is on the device
at a time.
"""
from __future__ import annotations

import json
import re
import shutil
from pathlib import Path

import torch

SHARD_SIZE_BYTES = 5 * 1024 ** 3
AEO_QUANTIZATION = {"quant_algo": "NVFP4", "block_size": 16}
_EXPERT_RE = re.compile(r"^model\.(?:language_model\.)?layers\.(\d+)\.experts\.(gate_up_proj|down_proj)$")
_COPIED = ("config.json", "generation_config.json", "tokenizer*.json", "processor_config.json",
           "chat_template.jinja")


def is_expert_key(key: str) -> bool:
    """True for a fused 3-D expert weight key that the builder quantizes."""
    return _EXPERT_RE.match(key) is not None


def _source_shards(src: Path):
    index = src / "model.safetensors.index.json"
    if index.exists():
        with open(index) as f:
            meta = json.load(f)
        return sorted(set(meta["weight_map"].values())), meta.get("metadata", {})
    single = src / "model.safetensors"
    if single.exists():
        return [single.name], {}
    raise FileNotFoundError(f"no model.safetensors.index.json or model.safetensors in {src}")


class _ShardWriter:
    """Collects tensors into shards of at most ``limit`` bytes (a tensor
    larger than the limit gets a shard of its own), written under temporary
    names and renamed to ``model-<i>-of-<n>`` once ``n`` is known."""

    def __init__(self, out: Path, limit: int):
        self.out, self.limit = out, limit
        self.pending: dict[str, torch.Tensor] = {}
        self.nbytes = 0
        self.files: list[tuple[str, list[str]]] = []

    def add(self, key: str, t: torch.Tensor):
        n = t.numel() * t.element_size()
        if self.pending and self.nbytes + n > self.limit:
            self.flush()
        self.pending[key] = t.contiguous()
        self.nbytes += n

    def flush(self):
        from safetensors.torch import save_file
        if not self.pending:
            return
        name = f"_shard-{len(self.files) + 1:05d}.safetensors.tmp"
        save_file(self.pending, str(self.out / name), metadata={"format": "pt"})
        self.files.append((name, list(self.pending)))
        self.pending, self.nbytes = {}, 0

    def finish(self) -> dict[str, str]:
        self.flush()
        n = len(self.files)
        weight_map = {}
        for i, (tmp, keys) in enumerate(self.files, start=1):
            final = f"model-{i:05d}-of-{n:05d}.safetensors"
            (self.out / tmp).rename(self.out / final)
            for k in keys:
                weight_map[k] = final
        return weight_map


@torch.no_grad()
def build_checkpoint_nvfp4(src_dir, out_dir, *, device="cuda", shard_size_bytes: int = SHARD_SIZE_BYTES,
                           quantize=None, log=print) -> dict:
    """Writes the NVFP4 checkpoint of the bf16 checkpoint in ``src_dir`` to
    ``out_dir``. ``quantize`` maps a bf16 (E, N, K) device tensor to
    ``(packed, block_scale, tensor_scale)`` and defaults to this library's
    ``quantize_3d_to_nvfp4``. Returns counts: ``quantized`` expert tensors,
    ``passthrough`` tensors, ``shards`` written."""
    from safetensors import safe_open

    if quantize is None:
        from ...gpu.quant import quantize_3d_to_nvfp4 as quantize
    src, out = Path(src_dir), Path(out_dir)
    if src.resolve() == out.resolve():
        raise ValueError("out_dir must differ from src_dir")
    out.mkdir(parents=True, exist_ok=True)
    shards, metadata = _source_shards(src)
    writer = _ShardWriter(out, int(shard_size_bytes))
    n_q = n_p = 0
    for shard in shards:
        with safe_open(str(src / shard), framework="pt", device="cpu") as f:
            for key in f.keys():  # noqa: SIM118 (safe_open has no __iter__)
                t = f.get_tensor(key)
                m = _EXPERT_RE.match(key)
                if m is None:
                    writer.add(key, t)
                    n_p += 1
                    continue
                if t.dim() != 3:
                    raise ValueError(f"{key}: expected a fused (E, N, K) expert tensor, got shape {tuple(t.shape)}")
                packed, block_scale, tensor_scale = quantize(t.to(device=device, dtype=torch.bfloat16))
                base = key.rsplit(".", 1)[0] + "." + m.group(2)
                writer.add(key, packed.cpu())
                writer.add(base + "_scale", block_scale.cpu())
                writer.add(base + "_scale_2", tensor_scale.cpu())
                del t, packed, block_scale, tensor_scale
                n_q += 1
                if log:
                    log(f"NVFP4: {key}")
    weight_map = writer.finish()
    with open(out / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": metadata, "weight_map": weight_map}, f, indent=2)
    for pattern in _COPIED:
        for p in src.glob(pattern):
            shutil.copy2(p, out / p.name)
    cfg_path = out / "config.json"
    if cfg_path.exists():
        with open(cfg_path) as f:
            cfg = json.load(f)
        cfg["aeo_quantization"] = dict(AEO_QUANTIZATION)
        with open(cfg_path, "w") as f:
            json.dump(cfg, f, indent=2)
    return {"quantized": n_q, "passthrough": n_p, "shards": len(set(weight_map.values()))}


def is_nvfp4_checkpoint(path) -> bool:
    """True if ``path/config.json`` carries the builder's NVFP4 stamp."""
    cfg_path = Path(path) / "config.json"
    if not cfg_path.exists():
        return False
    with open(cfg_path) as f:
        q = json.load(f).get("aeo_quantization") or {}
    return q.get("quant_algo") == "NVFP4"

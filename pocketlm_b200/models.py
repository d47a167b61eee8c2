"""Model-keyed access to resident MoE layers: what run_fp8_router /
run_fp8_moe (model_id, layer_index, hidden) need to find a layer.

The reference resolves a model id through its tensor catalog to a model
directory holding `config.json` and the checkpoint, reads the router config
from `config.json` (`_load_deepseek_route_config`,
core/runtime/fp8_source.py:5143-5155) and the layer's tensors from the FP8
pack when one exists, else from the safetensors shards
(`_read_packed_mlp_full_tensors`, :4709-4792; `_load_regular_tensor`).

Here a model id maps to a directory by `register_model`, else
$PCKETLM_MODELS_ROOT/<model_id>/original (or .../<model_id>); the layer is
read once -- from the FP8 pack ($PCKETLM_FP8_PACK_DIR or
<model_dir>/artifacts/fp8_pack) when its manifest exists, else from the
shards named by model.safetensors.index.json -- into HBM and kept as a
`DsMoELayerGPU` per (model, layer, device) until `evict_layers`.
"""

from __future__ import annotations

import json
import os
import threading
from pathlib import Path

import torch

from . import fp8_pack, native, synth
from .q4_artifact import safetensors_index

_REGISTRY: dict[str, Path] = {}
_LAYERS: dict[tuple[str, int, str], object] = {}
_LOCK = threading.Lock()


def register_model(model_id: str, model_dir: str | Path) -> None:
    """Make `model_id` resolve to `model_dir` (config.json + FP8 pack or
    safetensors shards).  Re-registering drops the model's resident layers."""
    evict_layers(model_id)
    _REGISTRY[str(model_id)] = Path(model_dir).resolve()


def model_dir(model_id: str) -> Path:
    if model_id in _REGISTRY:
        return _REGISTRY[model_id]
    root = os.environ.get("PCKETLM_MODELS_ROOT", "").strip()
    if root:
        for cand in (Path(root) / model_id / "original", Path(root) / model_id):
            if (cand / "config.json").exists():
                return cand.resolve()
    raise FileNotFoundError(f"Model {model_id!r} is not registered (register_model) and was not found under "
                            f"$PCKETLM_MODELS_ROOT.")


def _config_payload(model_id: str) -> dict:
    path = model_dir(model_id) / "config.json"
    return json.loads(path.read_text(encoding="utf-8")) if path.exists() else {}


def route_config(model_id: str) -> dict:
    """The router settings with the reference's keys, fallbacks and defaults
    (fp8_source.py:5143-5155: softmax when scoring_func is absent)."""
    p = _config_payload(model_id)
    return {
        "top_k": int(p.get("num_experts_per_tok", p.get("n_activated_experts", 1)) or 1),
        "n_groups": int(p.get("n_group", p.get("n_expert_groups", 1)) or 1),
        "topk_groups": int(p.get("topk_group", p.get("n_limited_groups", 1)) or 1),
        "scoring_func": str(p.get("scoring_func", p.get("score_func", "softmax"))),
        "route_scale": float(p.get("routed_scaling_factor", p.get("route_scale", 1.0)) or 1.0),
    }


def layer_config(model_id: str) -> synth.DsMoEConfig:
    """The MoE layer shape of a DeepSeek-V3-style config.json."""
    p = _config_payload(model_id)
    rc = route_config(model_id)
    try:
        hidden = int(p["hidden_size"])
        inter = int(p.get("moe_intermediate_size") or p["intermediate_size"])
        n_routed = int(p.get("n_routed_experts") or p["num_local_experts"])
    except KeyError as exc:
        raise ValueError(f"config.json of {model_id!r} lacks {exc.args[0]}") from exc
    return synth.DsMoEConfig(str(model_id), hidden=hidden, inter=inter, n_routed=n_routed, top_k=rc["top_k"],
                             n_group=rc["n_groups"], topk_group=rc["topk_groups"], route_scale=rc["route_scale"],
                             scoring_func=rc["scoring_func"])


class SafetensorsCheckpoint(fp8_pack.Fp8Pack):
    """A safetensors checkpoint (model.safetensors.index.json + shards) seen
    through the FP8 pack's lookup interface: each tensor is a byte range of
    its shard, each FP8 weight's block scales are `<weight>_scale_inv`."""

    def __init__(self, directory: str | Path):  # noqa: D107 -- no pack manifest to read
        self.pack_dir = Path(directory).resolve()
        index = self.pack_dir / "model.safetensors.index.json"
        if index.exists():
            shards = sorted(set(json.loads(index.read_text(encoding="utf-8")).get("weight_map", {}).values()))
        else:
            shards = sorted(p.name for p in self.pack_dir.glob("*.safetensors"))
        if not shards:
            raise FileNotFoundError(f"no safetensors checkpoint in {self.pack_dir}")
        self.shards = [self.pack_dir / s for s in shards]
        self.manifest = {"format": "safetensors"}
        self.tensors = {}
        for i, shard in enumerate(self.shards):
            for name, (dtype, shape, off, length) in safetensors_index(shard).items():
                self.tensors[name] = {"dtype": dtype, "shape": shape, "byte_offset": off, "byte_length": length,
                                      "pack_file_index": i}
        for name, entry in self.tensors.items():
            if f"{name}_scale_inv" in self.tensors:
                entry["scale_name"] = f"{name}_scale_inv"

    def entry(self, name: str) -> dict:
        try:
            return self.tensors[name]
        except KeyError as exc:
            raise KeyError(f"Tensor {name} is not present in the safetensors checkpoint.") from exc

    def path(self, pack_file_index: int) -> Path:
        return self.shards[int(pack_file_index)]


def checkpoint(model_id: str) -> fp8_pack.Fp8Pack:
    """The model's FP8 pack when its manifest exists, else its safetensors shards."""
    mdir = model_dir(model_id)
    pack_dir = fp8_pack.default_pack_dir(mdir)
    if (pack_dir / "pack_manifest.json").exists():
        return fp8_pack.Fp8Pack(pack_dir)
    return SafetensorsCheckpoint(mdir)


def resident_layer(model_id: str, layer_index: int, device: torch.device | str | None = None):
    """The layer's DsMoELayerGPU on `device` (current CUDA device by default),
    read into HBM on first use and kept."""
    from .runtime import DsMoELayerGPU

    if device is not None:
        dev = torch.device(device)
    elif torch.cuda.is_available():
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = None  # resolved after the model lookup, which reports a missing model first
    key = (str(model_id), int(layer_index), str(dev))
    with _LOCK:
        layer = _LAYERS.get(key)
        if layer is None:
            cfg = layer_config(model_id)
            dev = dev if dev is not None else native._device()
            host = fp8_pack.load_fp8_layer(checkpoint(model_id), int(layer_index), cfg, device=dev)
            layer = DsMoELayerGPU(host, int(layer_index))
            _LAYERS[key] = layer
    return layer


def evict_layers(model_id: str | None = None) -> int:
    """Drop resident layers (of one model, or all); returns how many."""
    with _LOCK:
        keys = [k for k in _LAYERS if model_id is None or k[0] == str(model_id)]
        for k in keys:
            del _LAYERS[k]
    return len(keys)


def resident_layers() -> list[tuple[str, int, str]]:
    with _LOCK:
        return sorted(_LAYERS)

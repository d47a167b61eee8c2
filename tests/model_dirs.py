"""Test helper: one-layer DeepSeek-V3-style model directories (config.json
with the reference's keys + safetensors shards, or + an FP8 pack) for the
model-keyed run_fp8_router / run_fp8_moe."""

import json
from pathlib import Path

import torch

from pocketlm_b200 import synth

PACK = Path(__file__).resolve().parent / "golden" / "fp8_pack_tiny"
PACK_EXPECTED = json.loads((PACK / "expected.json").read_text(encoding="utf-8"))
PACK_CFG = synth.DsMoEConfig("pack-tiny", hidden=PACK_EXPECTED["config"]["hidden"],
                             inter=PACK_EXPECTED["config"]["inter"], n_routed=PACK_EXPECTED["config"]["n_routed"],
                             top_k=2, n_group=2, topk_group=1, route_scale=2.5)


def write_config(model_dir: Path, cfg: synth.DsMoEConfig, **extra) -> Path:
    model_dir.mkdir(parents=True, exist_ok=True)
    payload = {"model_type": "deepseek_v3", "hidden_size": cfg.hidden, "moe_intermediate_size": cfg.inter,
               "n_routed_experts": cfg.n_routed, "n_shared_experts": 1, "num_experts_per_tok": cfg.top_k,
               "n_group": cfg.n_group, "topk_group": cfg.topk_group, "scoring_func": cfg.scoring_func,
               "routed_scaling_factor": cfg.route_scale}
    payload.update(extra)
    (model_dir / "config.json").write_text(json.dumps(payload), encoding="utf-8")
    return model_dir


def write_safetensors_layer(model_dir: Path, layer: synth.Fp8MoELayer, layer_index: int = 0,
                            shards: int = 2) -> Path:
    """Layer `layer_index` of a checkpoint in HF DeepSeek-V3 names, split
    over `shards` files, with model.safetensors.index.json."""
    from safetensors.torch import save_file

    cfg = layer.cfg
    prefix = f"model.layers.{layer_index}.mlp"
    tensors = {f"{prefix}.gate.weight": layer.router_weight.cpu().contiguous()}
    if layer.bias is not None:
        tensors[f"{prefix}.gate.e_score_correction_bias"] = layer.bias.cpu().float().contiguous()
    for e in range(cfg.n_routed + 1):
        name = f"{prefix}.experts.{e}" if e < cfg.n_routed else f"{prefix}.shared_experts"
        g, gs, u, us, d, ds = (t.cpu().contiguous() for t in layer.expert(e))
        for proj, w, s in (("gate_proj", g, gs), ("up_proj", u, us), ("down_proj", d, ds)):
            tensors[f"{name}.{proj}.weight"] = w.view(torch.float8_e4m3fn).clone()
            tensors[f"{name}.{proj}.weight_scale_inv"] = s.clone()
    names = list(tensors)
    weight_map = {}
    for i in range(shards):
        part = {n: tensors[n] for n in names[i::shards]}
        fname = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
        save_file(part, str(model_dir / fname))
        weight_map.update({n: fname for n in part})
    (model_dir / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}), encoding="utf-8")
    return model_dir

"""The model-keyed drop-in entry points on the GPU:
run_fp8_router(model_id, layer_index, hidden) and run_fp8_moe(model_id,
layer_index, hidden, *, dtype, router) with the reference's signatures
(fp8_source.py:1500-1576), the layer read by model id from the reference
writer's FP8 pack (tests/golden/fp8_pack_tiny) or from safetensors shards,
checked against the oracle and against the reference's own run_fp8_moe
output on config 1 (tests/golden/c1_tiny_T64.pt)."""

import pytest
import torch

import oracle
from pocketlm_b200 import models, synth
from pocketlm_b200.runtime import run_fp8_moe, run_fp8_router
from tests.model_dirs import PACK, PACK_CFG, PACK_EXPECTED, write_config, write_safetensors_layer
from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, id_mismatches, rel_l2

pytestmark = pytest.mark.gpu


def test_pack_model_router_and_moe_match_oracle(cuda_device, tmp_path, monkeypatch):
    monkeypatch.setenv("PCKETLM_FP8_PACK_DIR", str(PACK))
    models.register_model("gpu-pack-tiny", write_config(tmp_path / "pack-tiny", PACK_CFG))
    src = synth.make_fp8_layer(PACK_CFG, seed=PACK_EXPECTED["seed"])
    x = synth.make_hidden(24, PACK_CFG.hidden, seed=3)  # host tensors, as the reference's callers pass
    r = run_fp8_router("gpu-pack-tiny", 0, x)
    assert r.ready and r.model_id == "gpu-pack-tiny" and r.bias_loaded and r.scoring_func == "sigmoid"
    assert r.indices_tensor.device.type == "cpu" and r.weights_tensor.dtype == torch.bfloat16
    expected, route = oracle.ds_moe_layer(x, src)
    bad, excused = id_mismatches(r.indices_tensor, route)
    assert bad == excused
    m = run_fp8_moe("gpu-pack-tiny", 0, x)
    assert m.ready and m.output_tensor.device.type == "cpu" and m.output_tensor.dtype == torch.bfloat16
    assert rel_l2(m.output_tensor, expected) <= REL_L2_GATE and cos_dist(m.output_tensor, expected) <= COS_GATE
    # a router result passed in is used as it is: same routing, same output
    m2 = run_fp8_moe("gpu-pack-tiny", 0, x, router=r)
    assert m2.ready and m2.router is r and m2.router_elapsed_seconds == 0.0
    assert rel_l2(m2.output_tensor, m.output_tensor) <= 1e-3
    # the layer stays resident: the second call did not read the pack again
    assert ("gpu-pack-tiny", 0, str(torch.device("cuda", 0))) in models.resident_layers()
    assert models.evict_layers("gpu-pack-tiny") == 1


def test_safetensors_model_matches_reference_golden(cuda_device, golden_dir, tmp_path):
    g = torch.load(golden_dir / "c1_tiny_T64.pt", weights_only=False)
    cfg = synth.C1_TINY
    layer = synth.make_fp8_layer(cfg, seed=g["seed"])
    d = write_safetensors_layer(write_config(tmp_path / "c1", cfg), layer)
    models.register_model("gpu-c1", d)
    x = synth.make_hidden(g["tokens"], cfg.hidden, seed=g["seed"]).to("cuda")
    m = run_fp8_moe("gpu-c1", 0, x)
    assert m.ready and m.output_tensor.device.type == "cuda"
    assert torch.equal(torch.sort(m.router.indices_tensor.cpu(), 1).values, torch.sort(g["ids"], 1).values)
    assert rel_l2(m.output_tensor, g["out"]) <= REL_L2_GATE and cos_dist(m.output_tensor, g["out"]) <= COS_GATE
    r = run_fp8_router("gpu-c1", 0, x)
    assert torch.equal(torch.sort(r.indices_tensor.cpu(), 1).values, torch.sort(g["ids"], 1).values)
    # each token's weights, matched by expert id, equal the reference's (bf16 rounding aside)
    order_ours, order_ref = torch.argsort(r.indices_tensor.cpu(), 1), torch.argsort(g["ids"], 1)
    ours = r.weights_tensor.cpu().float().gather(1, order_ours)
    ref = g["weights"].float().gather(1, order_ref)
    assert (ours - ref).abs().max() <= 1e-2
    # the reference's own routing passed in as the router result
    r.indices_tensor, r.weights_tensor = g["ids"].to("cuda"), g["weights"].to("cuda")
    m2 = run_fp8_moe("gpu-c1", 0, x, router=r)
    assert rel_l2(m2.output_tensor, g["out"]) <= REL_L2_GATE and cos_dist(m2.output_tensor, g["out"]) <= COS_GATE
    models.evict_layers("gpu-c1")

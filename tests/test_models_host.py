"""Host side of the model-keyed entry points (pocketlm_b200.models): model
id resolution, config.json parsing with the reference's keys and defaults
(fp8_source.py:5143-5155), the safetensors and FP8-pack checkpoints read
byte for byte on the CPU, and blockers instead of exceptions for a model
that cannot be found (fp8_source.py:1500-1576)."""

import torch

from pocketlm_b200 import fp8_pack, models, runtime, synth
from tests.model_dirs import PACK, PACK_CFG, PACK_EXPECTED, write_config, write_safetensors_layer


def test_route_config_defaults_and_fallback_keys(tmp_path):
    d = tmp_path / "m"
    d.mkdir()
    (d / "config.json").write_text('{"hidden_size": 8}', encoding="utf-8")
    models.register_model("bare", d)
    assert models.route_config("bare") == {"top_k": 1, "n_groups": 1, "topk_groups": 1, "scoring_func": "softmax",
                                           "route_scale": 1.0}
    (d / "config.json").write_text('{"n_activated_experts": 6, "n_expert_groups": 8, "n_limited_groups": 3, '
                                   '"score_func": "sigmoid", "route_scale": 2.0}', encoding="utf-8")
    assert models.route_config("bare") == {"top_k": 6, "n_groups": 8, "topk_groups": 3, "scoring_func": "sigmoid",
                                           "route_scale": 2.0}


def test_layer_config_and_models_root(tmp_path, monkeypatch):
    write_config(tmp_path / "root" / "ds-tiny" / "original", synth.C1_TINY)
    monkeypatch.setenv("PCKETLM_MODELS_ROOT", str(tmp_path / "root"))
    assert models.model_dir("ds-tiny") == (tmp_path / "root" / "ds-tiny" / "original").resolve()
    cfg = models.layer_config("ds-tiny")
    c1 = synth.C1_TINY
    assert (cfg.hidden, cfg.inter, cfg.n_routed, cfg.top_k, cfg.n_group, cfg.topk_group, cfg.route_scale,
            cfg.scoring_func) == (c1.hidden, c1.inter, c1.n_routed, c1.top_k, c1.n_group, c1.topk_group,
                                  c1.route_scale, "sigmoid")


def test_safetensors_checkpoint_loads_byte_for_byte(tmp_path):
    cfg = synth.DsMoEConfig("st", hidden=256, inter=128, n_routed=3, top_k=2, n_group=1, topk_group=1,
                            route_scale=1.5)
    layer = synth.make_fp8_layer(cfg, seed=4)
    d = write_safetensors_layer(write_config(tmp_path / "st", cfg), layer, layer_index=2, shards=3)
    models.register_model("st", d)
    ck = models.checkpoint("st")
    assert isinstance(ck, models.SafetensorsCheckpoint)
    got = fp8_pack.load_fp8_layer(ck, 2, models.layer_config("st"), device="cpu")
    assert torch.equal(got.router_weight.view(torch.int16), layer.router_weight.view(torch.int16))
    assert torch.equal(got.bias, layer.bias)
    for name in ("w13", "s13", "w2", "s2"):
        assert torch.equal(getattr(got, name), getattr(layer, name)), name


def test_fp8_pack_is_preferred_when_present(tmp_path, monkeypatch):
    d = write_config(tmp_path / "pk", PACK_CFG)
    monkeypatch.setenv("PCKETLM_FP8_PACK_DIR", str(PACK))
    models.register_model("pack-tiny", d)
    ck = models.checkpoint("pack-tiny")
    assert isinstance(ck, fp8_pack.Fp8Pack) and not isinstance(ck, models.SafetensorsCheckpoint)
    got = fp8_pack.load_fp8_layer(ck, 0, models.layer_config("pack-tiny"), device="cpu")
    src = synth.make_fp8_layer(PACK_CFG, seed=PACK_EXPECTED["seed"])
    for name in ("w13", "s13", "w2", "s2"):
        assert torch.equal(getattr(got, name), getattr(src, name)), name


def test_unknown_model_reports_blockers(monkeypatch):
    monkeypatch.delenv("PCKETLM_MODELS_ROOT", raising=False)
    x = torch.zeros((2, 16), dtype=torch.bfloat16)
    r = runtime.run_fp8_router("no-such-model", 0, x)
    assert not r.ready and r.blockers and r.indices_tensor is None and r.model_id == "no-such-model"
    m = runtime.run_fp8_moe("no-such-model", 3, x)
    assert not m.ready and m.blockers and m.output_tensor is None and m.layer_index == 3
    assert set(m.to_dict()) >= {"model_id", "router", "blockers", "ready", "total_elapsed_seconds"}

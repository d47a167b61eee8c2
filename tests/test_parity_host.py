"""The checker's handling of routing ties, on the CPU (no GPU): a token whose
last top-k slot is an exact score tie may take either expert; its output is
checked against the experts actually picked, not the oracle's own pick."""

import torch

import oracle
from oracle.parity import REL_L2_GATE, fp8_layer_parity, rel_l2, tie_tokens
from oracle.router import route_deepseek, route_with_ids
from pocketlm_b200 import synth


def _tied_layer():
    """C1_TINY (16 experts in 4 groups, top-4 of the best 2 groups), no bias;
    token 0's logits: experts 0-2 high, experts 3 and 4 (identical router rows)
    tied for the fourth slot, groups 2-3 far below."""
    cfg = synth.C1_TINY
    layer = synth.make_fp8_layer(cfg, seed=5, device="cpu", bias_kind="none")
    gen = torch.Generator().manual_seed(6)
    x = torch.randn((3, cfg.hidden), generator=gen).to(torch.bfloat16)
    u = x[0].float() / x[0].float().norm() ** 2
    level = torch.full((cfg.n_routed,), -3.0)
    level[:3] = 3.0
    level[3] = level[4] = 0.5
    level[5:8] = -2.0
    rw = (level[:, None] * u[None, :]).to(torch.bfloat16)
    rw[4] = rw[3]
    layer.router_weight = rw
    return cfg, layer, x


def test_route_with_ids_reproduces_the_oracle_weights():
    cfg, layer, x = _tied_layer()
    r = route_deepseek(x, layer.router_weight, None, top_k=cfg.top_k, n_groups=cfg.n_group,
                       topk_groups=cfg.topk_group, route_scale=cfg.route_scale)
    again = route_with_ids(x, layer.router_weight, r.ids, route_scale=cfg.route_scale)
    assert torch.equal(again.weights, r.weights) and torch.equal(again.weights_f32, r.weights_f32)


def test_tied_token_is_checked_with_the_gpu_pick():
    cfg, layer, x = _tied_layer()
    r = route_deepseek(x, layer.router_weight, None, top_k=cfg.top_k, n_groups=cfg.n_group,
                       topk_groups=cfg.topk_group, route_scale=cfg.route_scale)
    picked = set(r.ids[0].tolist())
    assert {0, 1, 2} <= picked and len(picked & {3, 4}) == 1
    # the "GPU" takes the other expert of the tie for token 0
    gpu_ids = r.ids.clone()
    other = 4 if 3 in picked else 3
    gpu_ids[0][(gpu_ids[0] == 3) | (gpu_ids[0] == 4)] = other
    bad, excused = tie_tokens(gpu_ids, r)
    assert bad.tolist() == [True, False, False] and excused.tolist() == [True, False, False]
    gpu_route = route_with_ids(x, layer.router_weight, gpu_ids, route_scale=cfg.route_scale)
    out, _ = oracle.ds_moe_layer(x, layer, route=gpu_route)
    own, _ = oracle.ds_moe_layer(x, layer, route=r)
    assert rel_l2(out[:1], own[:1]) > REL_L2_GATE  # the pick matters: the two experts differ
    rep = fp8_layer_parity(layer, x, out, gpu_ids)
    assert rep["pass"] and rep["ties_excused"] == 1 and rep["ties_checked_with_gpu_pick"] == 1
    assert rep["rel_l2"] == 0.0
    # a mismatch that is not a tie still fails
    wrong = gpu_ids.clone()
    wrong[1][0] = 15 if 15 not in wrong[1].tolist() else 14
    assert not fp8_layer_parity(layer, x, out, wrong)["pass"]

"""Layer-level restatements -- TEST INFRASTRUCTURE ONLY, see oracle/__init__.py.

ds_moe_layer(): PocketLM's run_fp8_moe default flow
(src/pcketlm/core/runtime/fp8_source.py:1569-1884) as it runs when no FP8
pack file is present (the weighted-many branches need preloaded pack spans,
:1736-1738, so they are skipped):

  1. route (fp8_source.py:1500-1566, oracle/router.py);
  2. for each selected expert in ascending id order, gather its rows
     (torch.where, :1600-1605), run fp8_e4m3_block_mlp_f32 on them (via
     _run_fp8_native_mlp_full, :4842-4928) and round the result to bf16;
  3. combine in bf16: out[rows] += y_bf16 * w_bf16 (:1839-1847);
  4. add the shared expert, also rounded to bf16 (:1849-1862).

mixtral_q4_layer(): the Q4 decode/prefill flow of layer_bridge.py: softmax
top-2 router (:2682-2689), then q4_moe_selected_forward_u16 per token with the
experts in top-k order (_run_q4_moe_mlp_token_loop, :909-955), fp16 output
cast back to the hidden dtype.
"""

from __future__ import annotations

import torch

from . import kernels
from .router import RouteResult, route_deepseek, route_softmax_topk


def ds_moe_layer(hidden: torch.Tensor, layer, route: RouteResult | None = None, mlp_fn=None):
    """Return (out_bf16 [T, H], RouteResult).

    `layer` is a pocketlm_b200.synth.Fp8MoELayer (any device); the expert
    tensors of the selected experts are copied to the CPU as needed.
    `mlp_fn` replaces the expert kernel (default: the C restatement,
    oracle.kernels.fp8_mlp); bench.py passes the reference's own compiled
    fp8_e4m3_block_mlp_f32 (oracle.ref.fp8_mlp) to time the reference path.
    """
    mlp = mlp_fn or kernels.fp8_mlp
    cfg = layer.cfg
    flat = hidden.detach().cpu().reshape(-1, int(hidden.shape[-1]))
    if route is None:
        route = route_deepseek(
            flat, layer.router_weight, layer.bias, top_k=cfg.top_k, n_groups=cfg.n_group,
            topk_groups=cfg.topk_group, scoring_func=cfg.scoring_func, route_scale=cfg.route_scale,
        )
    ids = route.ids
    weights = route.weights.float()
    out = torch.zeros_like(flat, dtype=torch.bfloat16)
    for expert in sorted({int(v) for v in ids.reshape(-1).tolist()}):
        rows, slots = torch.where(ids == expert)
        tensors = [t.cpu() for t in layer.expert(expert)]
        y = mlp(*tensors, flat[rows].to(torch.bfloat16).float()).to(torch.bfloat16)
        w = weights[rows, slots].view(-1, 1).to(torch.bfloat16)
        out[rows] += y * w
    shared = [t.cpu() for t in layer.shared_expert()]
    shared_out = mlp(*shared, flat.to(torch.bfloat16).float()).to(torch.bfloat16)
    out = out + shared_out
    return out, route


def mixtral_q4_layer(hidden: torch.Tensor, layer, route: RouteResult | None = None):
    """Return (out [T, H] in hidden.dtype, RouteResult) for a Q4 Mixtral-shape layer
    (pocketlm_b200.synth.Q4MoELayer)."""
    cfg = layer.cfg
    flat = hidden.detach().cpu().reshape(-1, int(hidden.shape[-1]))
    if route is None:
        route = route_softmax_topk(flat, layer.router_weight, top_k=cfg.top_k, normalize=True)
    x16 = flat.to(torch.float16)
    rows = []
    for t in range(flat.shape[0]):
        experts = [[p.cpu() for p in layer.expert(int(e))] for e in route.ids[t].tolist()]
        rows.append(kernels.q4_moe_selected_forward(x16[t], experts, route.weights[t].float(),
                                                    cfg.hidden, cfg.inter))
    return torch.stack(rows).to(hidden.dtype), route

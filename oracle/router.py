"""Router restatements (torch CPU) -- TEST INFRASTRUCTURE ONLY, see oracle/__init__.py.

The DeepSeek-V3 router in PocketLM is Python/torch code, not native:
run_fp8_router (src/pcketlm/core/runtime/fp8_source.py:1500-1566) with the
group mask _mask_deepseek_route_groups (fp8_source.py:5125-5140).  The
Mixtral/Q4 router is the softmax top-k of layer_bridge.py:2682-2689 (also
_run_moe_mlp, layer_bridge.py:849-855).  Both are restated here with the same
sequence of fp32 torch CPU operations, so the ids and weights are those the
reference itself computes on the same inputs (tests/golden pins this against
the reference run in place).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class RouteResult:
    ids: torch.Tensor          # int64 [T, k]
    weights: torch.Tensor      # [T, k] in the hidden dtype (bf16 on the layer path)
    choice: torch.Tensor       # fp32 [T, E] selection scores after bias + group mask
    weights_f32: torch.Tensor  # fp32 [T, k] before the final dtype cast
    group_gap: torch.Tensor | None = None  # fp32 [T]: kept-group boundary margin (None: no groups)


def group_mask(choice: torch.Tensor, n_groups: int, topk_groups: int, use_bias: bool) -> torch.Tensor:
    """fp8_source.py:5125-5140: keep the `topk_groups` best groups of experts.

    A group's score is the sum of its two best members when a correction bias
    is present, otherwise its best member; every expert of a dropped group is
    set to -inf.
    """
    tokens = int(choice.shape[0])
    grouped = choice.view(tokens, int(n_groups), -1)
    if use_bias:
        group_score = grouped.topk(2, dim=-1)[0].sum(dim=-1)
    else:
        group_score = grouped.amax(dim=-1)
    keep = group_score.topk(max(1, min(int(topk_groups), int(n_groups))), dim=-1)[1]
    dropped = torch.ones((tokens, int(n_groups)), dtype=torch.bool).scatter_(1, keep, False)
    return grouped.masked_fill(dropped.unsqueeze(-1), float("-inf")).flatten(1)


def route_deepseek(
    hidden: torch.Tensor,
    router_weight: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    top_k: int,
    n_groups: int,
    topk_groups: int,
    scoring_func: str = "sigmoid",
    route_scale: float = 1.0,
) -> RouteResult:
    """fp8_source.py:1522-1547 on CPU tensors."""
    x = hidden.detach().cpu().reshape(-1, int(hidden.shape[-1])).float()
    logits = F.linear(x, router_weight.detach().cpu().float())
    if scoring_func == "softmax":
        probs = logits.softmax(dim=-1, dtype=torch.float32)
    else:
        probs = logits.sigmoid()
    bias_f = None if bias is None else bias.detach().cpu().float()
    choice = probs + bias_f if bias_f is not None else probs
    group_gap = None
    if n_groups > 1:
        group_gap = _group_boundary_gap(choice, n_groups, topk_groups, bias_f is not None)
        choice = group_mask(choice, n_groups, topk_groups, bias_f is not None)
    k = max(1, min(int(top_k), int(choice.shape[-1])))
    ids = torch.topk(choice, k, dim=-1)[1]
    picked = probs.gather(1, ids)
    if scoring_func == "sigmoid":
        picked = picked / picked.sum(dim=-1, keepdim=True).clamp_min(1e-12)
    scaled = picked * float(route_scale)
    return RouteResult(ids=ids, weights=scaled.to(dtype=hidden.dtype), choice=choice, weights_f32=scaled,
                       group_gap=group_gap)


def route_with_ids(
    hidden: torch.Tensor,
    router_weight: torch.Tensor,
    ids: torch.Tensor,
    *,
    scoring_func: str = "sigmoid",
    route_scale: float = 1.0,
) -> RouteResult:
    """The routing weights fp8_source.py:1540-1547 gives a fixed choice of
    experts `ids` [T, k]: the scores of those experts, renormalised (sigmoid
    scoring) and scaled.  The checker uses it for tokens whose selection is a
    score tie, to compute their outputs with the experts the GPU picked."""
    x = hidden.detach().cpu().reshape(-1, int(hidden.shape[-1])).float()
    logits = F.linear(x, router_weight.detach().cpu().float())
    probs = logits.softmax(dim=-1, dtype=torch.float32) if scoring_func == "softmax" else logits.sigmoid()
    ids = ids.detach().cpu().to(torch.int64)
    picked = probs.gather(1, ids)
    if scoring_func == "sigmoid":
        picked = picked / picked.sum(dim=-1, keepdim=True).clamp_min(1e-12)
    scaled = picked * float(route_scale)
    return RouteResult(ids=ids, weights=scaled.to(dtype=hidden.dtype), choice=probs, weights_f32=scaled)


def _group_boundary_gap(choice: torch.Tensor, n_groups: int, topk_groups: int, use_bias: bool) -> torch.Tensor:
    """Margin between the last kept group's score and the best dropped one."""
    grouped = choice.view(int(choice.shape[0]), int(n_groups), -1)
    score = grouped.topk(2, dim=-1)[0].sum(dim=-1) if use_bias else grouped.amax(dim=-1)
    kg = max(1, min(int(topk_groups), int(n_groups)))
    if kg >= n_groups:
        return torch.full((int(choice.shape[0]),), float("inf"))
    top = score.topk(kg + 1, dim=-1)[0]
    return top[:, kg - 1] - top[:, kg]


def route_softmax_topk(hidden: torch.Tensor, router_weight: torch.Tensor, *, top_k: int,
                       normalize: bool = True) -> RouteResult:
    """layer_bridge.py:2682-2689: softmax over fp32 logits, top-k, optional renorm."""
    x = hidden.detach().cpu().reshape(-1, int(hidden.shape[-1])).float()
    probs = torch.softmax(F.linear(x, router_weight.detach().cpu().float()), dim=-1)
    k = max(1, min(int(top_k), int(probs.shape[-1])))
    weights, ids = torch.topk(probs, k, dim=-1)
    if normalize:
        weights = weights / weights.sum(dim=-1, keepdim=True).clamp_min(1e-12)
    return RouteResult(ids=ids, weights=weights, choice=probs, weights_f32=weights)


def boundary_gap(choice: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """Per token: (k-th selected score) - (best unselected score).

    Used by the parity tests to excuse id mismatches that come from score
    ties: where the gap is below the tie tolerance, two implementations that
    sum the router dot products in a different order may legitimately pick a
    different expert at the boundary.
    """
    picked = choice.gather(1, ids)
    kth = picked.min(dim=1).values
    rest = choice.clone()
    rest.scatter_(1, ids, float("-inf"))
    best_rest = rest.max(dim=1).values
    return kth - best_rest

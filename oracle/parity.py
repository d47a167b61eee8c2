"""Parity metrics and checks -- TEST INFRASTRUCTURE ONLY (the checker).

Used by tests/ and by bench.py's parity leg, which runs after the timed
region on the timed batch; nothing here is measured or shipped.

The layer-level gate: relative L2 error <= 2e-2 and
cosine distance <= 1e-3 against the reference's CPU path; expert ids
bit-exact except where the selection boundary is a score tie within 1e-6.
"""

from __future__ import annotations

import torch

REL_L2_GATE = 2e-2
COS_GATE = 1e-3
TIE_TOL = 1e-6


def rel_l2(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a, e = actual.detach().double().cpu().reshape(-1), expected.detach().double().cpu().reshape(-1)
    return float((a - e).norm() / e.norm().clamp_min(1e-30))


def cos_dist(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a, e = actual.detach().double().cpu().reshape(-1), expected.detach().double().cpu().reshape(-1)
    return float(1.0 - torch.dot(a, e) / (a.norm() * e.norm()).clamp_min(1e-30))


def tie_tokens(ids: torch.Tensor, route, tol: float = TIE_TOL) -> tuple[torch.Tensor, torch.Tensor]:
    """Per token (bool [T] masks): the GPU's selection differs from the
    oracle's RouteResult as a set, and such a difference is excused because
    the oracle's expert boundary gap (k-th pick minus best other) or its
    group boundary gap is within `tol`."""
    from .router import boundary_gap

    a = torch.sort(ids.detach().cpu(), dim=1).values
    b = torch.sort(route.ids.detach().cpu(), dim=1).values
    bad = (a != b).any(dim=1)
    near = boundary_gap(route.choice, route.ids) <= tol
    if route.group_gap is not None:
        near = near | (route.group_gap <= tol)
    return bad, bad & near


def id_mismatches(ids: torch.Tensor, route, tol: float = TIE_TOL):
    """(mismatching tokens, of which excused as ties) against an oracle
    RouteResult (tie_tokens, counted)."""
    bad, excused = tie_tokens(ids, route, tol)
    return int(bad.sum()), int(excused.sum())


def slice_tokens(ids: torch.Tensor, n_spread: int = 64, n_heavy: int = 32) -> list[int]:
    """Tokens to check against the layer oracle in a large batch: every
    (T / n_spread)-th token, plus up to n_heavy tokens spread over the rows of
    the most loaded expert (its pairs fill many GEMM m-tiles).  Tokens are
    computed independently, so a slice checks the batch's kernels as run."""
    T = int(ids.shape[0])
    step = max(1, T // max(1, n_spread))
    picked = set(range(0, T, step))
    flat = ids.detach().cpu().reshape(T, -1)
    counts = torch.bincount(flat.reshape(-1).clamp_min(0))
    heavy = int(torch.argmax(counts))
    rows = torch.nonzero((flat == heavy).any(dim=1)).reshape(-1).tolist()
    if rows:
        stride = max(1, len(rows) // max(1, n_heavy))
        picked.update(rows[::stride][:n_heavy])
        picked.add(rows[-1])
    return sorted(picked)


def host_fp8_sublayer(layer, experts: list[int]):
    """A CPU copy of `layer` (pocketlm_b200.synth.Fp8MoELayer, any device)
    holding only `experts` (the shared expert id included when wanted)."""
    from pocketlm_b200 import synth

    idx = torch.tensor([e if layer.slots is None else layer.slots[e] for e in experts], device=layer.w13.device)
    parts = [t.index_select(0, idx).cpu() for t in (layer.w13, layer.s13, layer.w2, layer.s2)]
    bias = None if layer.bias is None else layer.bias.cpu()
    return synth.Fp8MoELayer(layer.cfg, layer.router_weight.cpu(), bias, *parts,
                             {e: i for i, e in enumerate(experts)})


def fp8_layer_parity(layer, x: torch.Tensor, out: torch.Tensor, ids: torch.Tensor,
                     tokens: list[int] | None = None) -> dict:
    """The GPU layer's routing of every token and its outputs on `tokens`
    (all when None) against the oracle's run_fp8_moe flow, with the layer's
    own weights copied to the host for the experts those tokens select."""
    from .layer import ds_moe_layer
    from .router import RouteResult, route_deepseek, route_with_ids

    cfg = layer.cfg
    xc = x.detach().cpu()
    route = route_deepseek(xc, layer.router_weight.cpu(), None if layer.bias is None else layer.bias.cpu(),
                           top_k=cfg.top_k, n_groups=cfg.n_group, topk_groups=cfg.topk_group,
                           scoring_func=cfg.scoring_func, route_scale=cfg.route_scale)
    bad_mask, tie_mask = tie_tokens(ids, route)
    bad, ties = int(bad_mask.sum()), int(tie_mask.sum())
    sel = list(range(int(xc.shape[0]))) if tokens is None else list(tokens)
    # a token whose selection is an excused tie is checked with the experts the GPU picked (either pick is
    # the reference's answer; its output follows the pick)
    use_ids = route.ids.clone()
    use_ids[tie_mask] = ids.detach().cpu().to(torch.int64)[tie_mask]
    if ties:
        route = route_with_ids(xc, layer.router_weight.cpu(), use_ids, scoring_func=cfg.scoring_func,
                               route_scale=cfg.route_scale)
    experts = sorted({int(v) for v in use_ids[sel].reshape(-1).tolist()}) + [cfg.n_routed]
    host = layer if layer.w13.device.type == "cpu" else host_fp8_sublayer(layer, experts)
    sub = RouteResult(ids=route.ids[sel], weights=route.weights[sel], choice=route.choice[sel],
                      weights_f32=route.weights_f32[sel])
    expected, _ = ds_moe_layer(xc[sel], host, route=sub)
    got = out.detach().cpu()[sel]
    rl, cd = rel_l2(got, expected), cos_dist(got, expected)
    return {"tokens_checked": len(sel), "tokens_routed": int(xc.shape[0]), "rel_l2": rl, "cos_dist": cd,
            "id_mismatches": bad, "ties_excused": ties, "ties_checked_with_gpu_pick": int(tie_mask[sel].sum()),
            "pass": bool(rl <= REL_L2_GATE and cd <= COS_GATE and bad == ties)}


def q4_layer_parity(layer, x: torch.Tensor, out: torch.Tensor, ids: torch.Tensor,
                    tokens: list[int] | None = None) -> dict:
    """The Q4 layer (pocketlm_b200.synth.Q4MoELayer, any device): routing of
    every token and outputs on `tokens` against the oracle's Q4 token loop."""
    from .layer import mixtral_q4_layer
    from .router import route_softmax_topk

    cfg = layer.cfg
    xc = x.detach().cpu()
    route = route_softmax_topk(xc, layer.router_weight.cpu(), top_k=cfg.top_k, normalize=True)
    bad, ties = id_mismatches(ids, route)
    sel = list(range(int(xc.shape[0]))) if tokens is None else list(tokens)
    host = layer.to("cpu")
    expected, _ = mixtral_q4_layer(xc[sel], host)
    got = out.detach().cpu()[sel]
    rl, cd = rel_l2(got, expected), cos_dist(got, expected)
    return {"tokens_checked": len(sel), "tokens_routed": int(xc.shape[0]), "rel_l2": rl, "cos_dist": cd,
            "id_mismatches": bad, "ties_excused": ties,
            "pass": bool(rl <= REL_L2_GATE and cd <= COS_GATE and bad == ties)}

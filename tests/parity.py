"""Parity metrics shared by the GPU tests and bench.py.

The layer-level gate: relative L2 error <= 2e-2 and
cosine distance <= 1e-3 against the reference's CPU path; expert ids
bit-exact except where the selection boundary is a score tie within 1e-6.
"""

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


def id_mismatches(ids: torch.Tensor, route, tol: float = TIE_TOL):
    """(mismatching tokens, of which excused as ties) against an oracle
    RouteResult.  Selections compare as sets; a differing set is excused when
    the oracle's expert boundary gap (k-th pick minus best other) or its group
    boundary gap is within `tol`."""
    from oracle.router import boundary_gap

    a = torch.sort(ids.detach().cpu(), dim=1).values
    b = torch.sort(route.ids.detach().cpu(), dim=1).values
    bad = (a != b).any(dim=1)
    near = boundary_gap(route.choice, route.ids) <= tol
    if route.group_gap is not None:
        near = near | (route.group_gap <= tol)
    excused = bad & near
    return int(bad.sum()), int(excused.sum())

"""Parity metrics shared by the GPU tests (defined in oracle/parity.py,
where bench.py's parity leg uses them too).

The layer-level gate: relative L2 error <= 2e-2 and
cosine distance <= 1e-3 against the reference's CPU path; expert ids
bit-exact except where the selection boundary is a score tie within 1e-6.
"""

from oracle.parity import COS_GATE, REL_L2_GATE, TIE_TOL, cos_dist, id_mismatches, rel_l2  # noqa: F401

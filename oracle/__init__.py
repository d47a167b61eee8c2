"""CPU oracle for PocketLM's MoE expert hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (pocketlm_b200/)
imports this package; only tests/, __graft_entry__.smoke() and the
cpu_baseline / `--impl reference` legs of bench.py do, and there only as the
checker or the timed CPU baseline -- never as the thing measured or shipped.

Contents
--------
moe_oracle.c / kernels.py
    C restatement (gcc, OpenMP) of the reference's native kernels on this
    path: fp8_linear.cpp, fp8_dequant.cpp, q4_dequant.cpp,
    fp16_packed_gemv.cpp, fp16_moe.cpp and the combine/router of
    ds_forward.cpp (paths under src/pcketlm/native/ of the reference).
router.py
    The DeepSeek-V3 sigmoid + bias + group-limited top-k router and the
    softmax top-k router, restated with the reference's torch CPU ops.
layer.py
    Layer-level flows: run_fp8_moe's default path and the Q4 token loop.
mla.py
    The one-token MLA attention (ds_forward.cpp:517-782) with the reference's
    per-position online softmax.
ref.py
    The reference's own kernels compiled from source into oracle/_ref/
    (Makefile target `ref`), used to pin the restatement and as the CPU
    baseline.

Pinning: tests/test_oracle_vs_reference.py checks kernels.py against ref.py
(bit-exact for the FP8 linear/MLP/dequant kernels, whose operation order is
restated exactly), and tests/test_golden.py checks the layer/router
restatements against golden vectors produced by the reference's own Python
runtime (tests/golden/make_golden.py).
"""

from . import kernels, layer, mla, ref, router  # noqa: F401
from .layer import ds_moe_layer, mixtral_q4_layer  # noqa: F401
from .router import RouteResult, boundary_gap, route_deepseek, route_softmax_topk  # noqa: F401

"""The decode prologue (decode_prologue_kernel: selection, dispatch, chunk
list, x staging and counter reset in one 256-thread launch) against the two
launches it replaces (route_dispatch_kernel + rows_to_f16_kernel,
moe_b200_decode_prologue(0)): the same routing, pair order and staged rows,
so the layer's outputs, ids and weights are the same bits.  Also the
staggered k-block walk (moe_b200_kb_rotate): the same sums in another
order."""

import pytest
import torch

from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import DsMoELayerGPU
from tests.parity import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _defaults_and_clean_error_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = native.load_library()
    lib.moe_b200_select_gemv(0)
    yield
    lib.moe_b200_decode_prologue(1)
    lib.moe_b200_router_stages_x(1)
    lib.moe_b200_kb_rotate(0)
    torch.cuda.synchronize()
    assert lib.moe_b200_device_error(None) == 0, "a bounded wait inside a kernel gave up"


def _run(gpu, x):
    T, k = int(x.shape[0]), gpu.cfg.top_k
    ids = torch.empty((T, k), dtype=torch.int64, device=x.device)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=x.device)
    out = gpu.forward(x, ids=ids, weights=w).clone()
    torch.cuda.synchronize()
    return out, ids, w


@pytest.mark.parametrize("cfg_name,tokens", [("c1", 1), ("c1", 7), ("c1", 64), ("c2", 1), ("c2", 4), ("c2", 8),
                                             ("c2", 33)])
def test_prologue_is_bit_identical_to_two_launches(cuda_device, cfg_name, tokens):
    cfg = synth.C1_TINY if cfg_name == "c1" else synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=300 + tokens, device="cuda")
    gpu = DsMoELayerGPU(layer)
    lib = native.load_library()
    for dtype in (torch.bfloat16, torch.float32):
        x = synth.make_hidden(tokens, cfg.hidden, seed=301 + tokens, device="cuda").to(dtype)
        lib.moe_b200_decode_prologue(1)
        a = _run(gpu, x)
        lib.moe_b200_decode_prologue(0)
        b = _run(gpu, x)
        for u, v in zip(a, b):
            assert torch.equal(u, v)
    # graph replay with the prologue: the same bits again
    lib.moe_b200_decode_prologue(1)
    x = synth.make_hidden(tokens, cfg.hidden, seed=301 + tokens, device="cuda")
    graphed = gpu.capture(tokens)
    assert torch.equal(graphed(x), _run(gpu, x)[0])


@pytest.mark.parametrize("tokens", [1, 16])
def test_rotated_kblock_walk_matches(cuda_device, tokens):
    cfg = synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=400, device="cuda")
    gpu = DsMoELayerGPU(layer)
    lib = native.load_library()
    x = synth.make_hidden(tokens, cfg.hidden, seed=401, device="cuda")
    plain = _run(gpu, x)[0]
    lib.moe_b200_kb_rotate(1)
    for fused in (0, 1):
        lib.moe_b200_fused_decode(fused)
        rotated = _run(gpu, x)[0]
        assert rel_l2(rotated, plain) <= 1e-3
    lib.moe_b200_fused_decode(0)


@pytest.mark.parametrize("cfg_name,tokens", [("c1", 1), ("c1", 9), ("c1", 200), ("c2", 1), ("c2", 16), ("c2", 64)])
def test_folded_staging_and_combine_are_bit_identical(cuda_device, cfg_name, tokens):
    """The activation staging folded into the gate/up launch and the combine
    into the down launch (moe_b200_fold_epilogues(1)) against their own
    launches (0, the default): the same bits, eager and graph-replayed."""
    cfg = synth.C1_TINY if cfg_name == "c1" else synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=700 + tokens, device="cuda")
    gpu = DsMoELayerGPU(layer)
    lib = native.load_library()
    x = synth.make_hidden(tokens, cfg.hidden, seed=701 + tokens, device="cuda")
    try:
        lib.moe_b200_fold_epilogues(1)
        a = _run(gpu, x)
        graphed = gpu.capture(tokens)
        replayed = graphed(x).clone()
        lib.moe_b200_fold_epilogues(0)
        b = _run(gpu, x)
    finally:
        lib.moe_b200_fold_epilogues(0)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    assert torch.equal(replayed, a[0])


@pytest.mark.parametrize("cfg_name,tokens", [("c1", 1), ("c1", 12), ("c2", 1), ("c2", 4), ("c2", 64)])
def test_shared_expert_side_stream(cuda_device, cfg_name, tokens):
    """The shared expert on the side stream (moe_b200_shared_side(1)) against
    the one-stream layer (0, the default): the same routing, outputs to
    bf16 rounding of a different k-split grouping; graph replay with the
    fork / join captured gives the eager bits; the oracle's gate holds."""
    import oracle
    from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, id_mismatches

    cfg = synth.C1_TINY if cfg_name == "c1" else synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=800 + tokens, device="cuda")
    gpu = DsMoELayerGPU(layer)
    lib = native.load_library()
    x = synth.make_hidden(tokens, cfg.hidden, seed=801 + tokens, device="cuda")
    try:
        lib.moe_b200_shared_side(1)
        side = _run(gpu, x)
        graphed = gpu.capture(tokens)
        replayed = [graphed(x).clone() for _ in range(2)]
        lib.moe_b200_shared_side(0)
        single = _run(gpu, x)
    finally:
        lib.moe_b200_shared_side(0)
    assert torch.equal(side[1], single[1]) and torch.equal(side[2], single[2])
    assert rel_l2(side[0], single[0]) <= 1e-3
    assert all(torch.equal(r, side[0]) for r in replayed)
    expected, route = oracle.ds_moe_layer(x.cpu(), layer)
    bad, excused = id_mismatches(side[1], route)
    assert bad == excused
    assert rel_l2(side[0], expected) <= REL_L2_GATE and cos_dist(side[0], expected) <= COS_GATE


@pytest.mark.parametrize("cfg_name,tokens", [("c1", 1), ("c1", 8), ("c2", 1), ("c2", 2), ("c2", 8)])
def test_router_staged_x_is_bit_identical(cuda_device, cfg_name, tokens):
    """x staged by the router launch's extra cluster (moe_b200_router_stages_x(1),
    the default) against the prologue's own staging (0): the same f16 rows and
    row scales, so the same bits out -- including a row scaled far up, one far
    down and an all-zero row (scale 1); eager and graph-replayed."""
    cfg = synth.C1_TINY if cfg_name == "c1" else synth.C2_DSV3
    layer = synth.make_fp8_layer(cfg, seed=900 + tokens, device="cuda")
    gpu = DsMoELayerGPU(layer)
    lib = native.load_library()
    x = synth.make_hidden(tokens, cfg.hidden, seed=901 + tokens, device="cuda").float()
    x[0] *= 3.0e4
    if tokens > 2:
        x[1] = 0.0
        x[2] *= 1.0e-6
    x = x.to(torch.bfloat16)
    try:
        lib.moe_b200_router_stages_x(1)
        a = _run(gpu, x)
        graphed = gpu.capture(tokens)
        replayed = graphed(x).clone()
        lib.moe_b200_router_stages_x(0)
        b = _run(gpu, x)
    finally:
        lib.moe_b200_router_stages_x(1)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    assert torch.equal(replayed, a[0])

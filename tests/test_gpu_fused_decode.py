"""The fused decode experts (decode_fused_kernel: gate/up + SwiGLU, the f16
staging of the activations and down in one persistent launch) against the
three-launch path it replaces (moe_b200_fused_decode(0)) and against the
oracle.  The two paths differ only in how each task's k-blocks are grouped
into partial sums, so they agree to fp32 rounding; the routing is the same
kernel.  Covers the DS-V3 decode sizes, the tiny config (4 and 2 k-blocks
per task: tasks split over up to five warps), a layer with absent experts,
repeat calls and CUDA-graph replay (bit-identical: the piece order is fixed)."""

import pytest
import torch

import oracle
from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import DsMoELayerGPU
from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, id_mismatches, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fused_on_and_clean_error_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = native.load_library()
    lib.moe_b200_select_gemv(0)
    lib.moe_b200_fused_decode(1)
    yield
    lib.moe_b200_fused_decode(0)
    torch.cuda.synchronize()
    assert lib.moe_b200_device_error(None) == 0, "a bounded wait inside a kernel gave up"


def _both(gpu: DsMoELayerGPU, x: torch.Tensor):
    lib = native.load_library()
    T, k = int(x.shape[0]), gpu.cfg.top_k
    ids_f = torch.empty((T, k), dtype=torch.int64, device=x.device)
    fused = gpu.forward(x, ids=ids_f).clone()
    lib.moe_b200_fused_decode(0)
    ids_u = torch.empty_like(ids_f)
    unfused = gpu.forward(x, ids=ids_u).clone()
    lib.moe_b200_fused_decode(1)
    torch.cuda.synchronize()
    assert torch.equal(ids_f, ids_u)
    return fused, unfused, ids_f


@pytest.fixture(scope="module")
def dsv3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    layer = synth.make_fp8_layer(synth.C2_DSV3, seed=31, device="cuda")
    gpu = DsMoELayerGPU(layer)
    yield layer, gpu
    del gpu, layer
    torch.cuda.empty_cache()


@pytest.mark.parametrize("tokens", [1, 2, 4, 16, 64, 200])
def test_fused_matches_three_launches_and_oracle_dsv3(dsv3, tokens):
    layer, gpu = dsv3
    x = synth.make_hidden(tokens, layer.cfg.hidden, seed=500 + tokens, device="cuda")
    fused, unfused, ids = _both(gpu, x)
    assert torch.isfinite(fused.float()).all()
    # bf16 outputs: a few elements one bf16 ulp apart
    assert rel_l2(fused, unfused) <= 1e-3 and cos_dist(fused, unfused) <= 1e-6
    expected, route = oracle.ds_moe_layer(x.cpu(), layer)
    bad, excused = id_mismatches(ids, route)
    assert bad == excused
    assert rel_l2(fused, expected) <= REL_L2_GATE and cos_dist(fused, expected) <= COS_GATE
    # the same batch again, and replayed from a CUDA graph: the same bits
    assert torch.equal(gpu.forward(x), fused)
    graphed = gpu.capture(tokens)
    for _ in range(2):
        assert torch.equal(graphed(x), fused)


@pytest.mark.parametrize("tokens", [1, 3, 8, 64, 300])
def test_fused_tiny_layer_many_pieces(cuda_device, tokens):
    cfg = synth.C1_TINY
    layer = synth.make_fp8_layer(cfg, seed=40 + tokens, device="cuda")
    gpu = DsMoELayerGPU(layer)
    x = synth.make_hidden(tokens, cfg.hidden, seed=41 + tokens, device="cuda")
    fused, unfused, ids = _both(gpu, x)
    assert rel_l2(fused, unfused) <= 1e-3
    expected, route = oracle.ds_moe_layer(x.cpu(), layer)
    bad, excused = id_mismatches(ids, route)
    assert bad == excused
    assert rel_l2(fused, expected) <= REL_L2_GATE and cos_dist(fused, expected) <= COS_GATE


def test_fused_absent_experts_match_three_launches(cuda_device):
    """A partial layer: absent experts' pieces stream nothing and their pairs'
    rows come out zero in both paths."""
    cfg = synth.DsMoEConfig("mid", hidden=1024, inter=512, n_routed=32, top_k=4, n_group=4, topk_group=2,
                            route_scale=2.5)
    resident = [e for e in range(cfg.n_routed) if e % 3 != 1] + [cfg.n_routed]
    layer = synth.make_fp8_layer(cfg, seed=55, device="cuda", experts=resident)
    gpu = DsMoELayerGPU(layer, allow_partial=True)
    x = synth.make_hidden(48, cfg.hidden, seed=56, device="cuda")
    fused, unfused, _ids = _both(gpu, x)
    assert torch.isfinite(fused.float()).all()
    assert rel_l2(fused, unfused) <= 1e-3

"""Prefill-sized batches (>= 512 tokens) on the tcgen05 grouped GEMM
(prefill_gemm.cu) against the oracle's run_fp8_moe flow and against the
decode GEMV path on the same layer.

The prefill GEMM folds each 128 x 128 block scale into the weights as it
converts them to fp16 (w * s rounded to fp16) and, in the whole layer,
rounds each expert's output row to bf16 before the combine (where the
reference rounds it too), so it agrees with the exact GEMV path, which keeps
fp32 rows, to about 1e-3 rather than bit for bit (checked at 4e-3)."""

GEMV_TOL = 4e-3

import pytest
import torch

import oracle
from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import DsMoELayerGPU
from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, id_mismatches, rel_l2

pytestmark = pytest.mark.gpu

C_MID = synth.DsMoEConfig("mid", hidden=1024, inter=512, n_routed=32, top_k=4, n_group=4, topk_group=2,
                          route_scale=2.5)


@pytest.fixture(autouse=True)
def _clean_error_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = native.load_library()
    lib.moe_b200_select_gemv(0)
    yield
    torch.cuda.synchronize()
    assert lib.moe_b200_device_error(None) == 0, "a bounded wait inside a kernel gave up"


def _run(cfg, tokens, seed, bias="uniform"):
    layer = synth.make_fp8_layer(cfg, seed=seed, device="cuda", bias_kind=bias)
    x = synth.make_hidden(tokens, cfg.hidden, seed=seed + 1, device="cuda")
    gpu = DsMoELayerGPU(layer)
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int64, device="cuda")
    out = gpu.forward(x, ids=ids).clone()
    gemv = DsMoELayerGPU(layer, tiled=False).forward(x).clone()  # row-major weights: the decode GEMV
    torch.cuda.synchronize()
    return layer, x, out, ids, gemv


@pytest.mark.parametrize("cfg,tokens", [(synth.C1_TINY, 512), (synth.C1_TINY, 2048), (C_MID, 1024)])
def test_prefill_matches_oracle_and_gemv(cuda_device, cfg, tokens):
    layer, x, out, ids, gemv = _run(cfg, tokens, seed=40 + tokens)
    assert rel_l2(out, gemv) <= GEMV_TOL and cos_dist(out, gemv) <= 1e-5
    expected, route = oracle.ds_moe_layer(x.cpu(), layer)
    bad, excused = id_mismatches(ids, route)
    assert bad == excused
    assert rel_l2(out, expected) <= REL_L2_GATE and cos_dist(out, expected) <= COS_GATE


def test_prefill_zipf_routing_uneven_experts(cuda_device):
    """Zipf-biased routing (config 3's distribution): a few experts take most
    pairs (many m-tiles), others none (empty segments)."""
    layer, x, out, ids, gemv = _run(C_MID, 1536, seed=77, bias="zipf")
    counts = torch.bincount(ids.reshape(-1).cpu(), minlength=C_MID.n_routed)
    assert counts.max() > 4 * counts.float().mean()
    assert rel_l2(out, gemv) <= GEMV_TOL


def test_prefill_dsv3_shape(cuda_device):
    cfg = synth.C2_DSV3
    layer, x, out, ids, gemv = _run(cfg, 512, seed=91)
    assert rel_l2(out, gemv) <= GEMV_TOL and cos_dist(out, gemv) <= 1e-5
    n = 48  # the oracle on a slice of the batch: every token is computed independently
    expected, route = oracle.ds_moe_layer(x[:n].cpu(), layer)
    bad, excused = id_mismatches(ids[:n], route)
    assert bad == excused
    assert rel_l2(out[:n], expected) <= REL_L2_GATE and cos_dist(out[:n], expected) <= COS_GATE


def test_prefill_skips_absent_experts_like_the_gemv(cuda_device):
    """A partial layer (some experts not resident, null table entries): the
    prefill GEMM skips their tiles in every role and writes their pairs'
    rows as zeros, as the GEMV path leaves them -- same output."""
    cfg = C_MID
    resident = [e for e in range(cfg.n_routed) if e % 3 != 1] + [cfg.n_routed]
    layer = synth.make_fp8_layer(cfg, seed=55, device="cuda", experts=resident)
    x = synth.make_hidden(1024, cfg.hidden, seed=56, device="cuda")
    out = DsMoELayerGPU(layer, allow_partial=True).forward(x).clone()
    gemv = DsMoELayerGPU(layer, allow_partial=True, tiled=False).forward(x).clone()
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert rel_l2(out, gemv) <= GEMV_TOL and cos_dist(out, gemv) <= 1e-5


def test_prefill_graph_replay_matches_eager(cuda_device):
    """A prefill-sized layer (the tcgen05 path) captured as a CUDA graph: every
    replay gives the eager forward's bits (the bench times prefill this way)."""
    layer = synth.make_fp8_layer(C_MID, seed=93, device="cuda", bias_kind="zipf")
    gpu = DsMoELayerGPU(layer)
    x = synth.make_hidden(1024, C_MID.hidden, seed=94, device="cuda")
    eager = gpu.forward(x).clone()
    graphed = gpu.capture(1024)
    for _ in range(2):
        assert torch.equal(graphed(x), eager)

"""Parity at the sizes bench.py reports, on the batches it times.

Config 3 (DS-V3 layer, Zipf-skewed router bias) at 2048, 8192 and 16384
tokens on the tcgen05 grouped GEMM, and config 4 (Mixtral-shape Q4 layer) at
4096 tokens, with bench.py's seeds.  Every token's expert ids are compared
with the oracle's router (ties within 1e-6 excused); outputs are compared
with the oracle's layer flow on a slice of the batch -- every T/64-th token
plus tokens spread over the rows of the most loaded expert, whose pairs fill
many m-tiles (tokens are computed independently, so the slice checks the
batch's kernels as they ran).  The 16384-token batch has 147,456 pairs, past
the 65,535-row launch limits the kernels loop over."""

import pytest
import torch

from oracle.parity import COS_GATE, REL_L2_GATE, fp8_layer_parity, q4_layer_parity, slice_tokens
from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import DsMoELayerGPU, Q4MoELayerGPU

pytestmark = pytest.mark.gpu

BENCH_SEED = 20  # bench.py --seed default


@pytest.fixture(autouse=True)
def _clean_error_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = native.load_library()
    lib.moe_b200_select_gemv(0)
    yield
    torch.cuda.synchronize()
    assert lib.moe_b200_device_error(None) == 0, "a bounded wait inside a kernel gave up"


@pytest.fixture(scope="module")
def c3_layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    layer = synth.make_fp8_layer(synth.C2_DSV3, seed=BENCH_SEED + 1, device="cuda", bias_kind="zipf")
    gpu = DsMoELayerGPU(layer)
    yield layer, gpu
    del gpu, layer
    torch.cuda.empty_cache()


@pytest.mark.parametrize("tokens", [2048, 8192, 16384])
def test_c3_prefill_zipf_matches_oracle(c3_layer, tokens):
    layer, gpu = c3_layer
    cfg = layer.cfg
    x = synth.make_hidden(tokens, cfg.hidden, seed=BENCH_SEED + tokens, device="cuda")
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int64, device="cuda")
    out = gpu.forward(x, ids=ids)
    torch.cuda.synchronize()
    counts = torch.bincount(ids.reshape(-1).cpu(), minlength=cfg.n_routed)
    assert counts.max() > 2 * counts.float().mean()  # the Zipf skew is there
    assert torch.isfinite(out.float()).all()
    rep = fp8_layer_parity(layer, x, out, ids, slice_tokens(ids))
    assert rep["id_mismatches"] == rep["ties_excused"], rep
    assert rep["rel_l2"] <= REL_L2_GATE and rep["cos_dist"] <= COS_GATE, rep
    # a second forward of the same batch is bit-identical (deterministic split and reduction order)
    again = gpu.forward(x)
    assert torch.equal(again, out)


def test_c4_q4_prefill_matches_oracle(cuda_device):
    cfg = synth.C4_MIXTRAL
    T = 4096
    layer = Q4MoELayerGPU(synth.make_q4_layer(cfg, seed=BENCH_SEED, device="cuda"))
    x = synth.make_hidden(T, cfg.hidden, seed=BENCH_SEED + 7 * T, device="cuda")
    ids = torch.empty((T, cfg.top_k), dtype=torch.int64, device="cuda")
    out = layer.forward(x, ids=ids)
    torch.cuda.synchronize()
    assert layer.tables_tiled is not None  # 4096 tokens run on the tcgen05 GEMM
    rep = q4_layer_parity(layer.layer, x, out, ids, slice_tokens(ids, n_spread=48, n_heavy=16))
    assert rep["id_mismatches"] == rep["ties_excused"], rep
    assert rep["rel_l2"] <= REL_L2_GATE and rep["cos_dist"] <= COS_GATE, rep

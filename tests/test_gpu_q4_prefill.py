"""Prefill-sized Q4 batches on the tcgen05 grouped GEMM (prefill_gemm.cu with
int4 weights in the Q4 tiled layout) against the warp-MMA GEMV path on the
same layer and against the oracle's token loop (q4_dequant.cpp:357-476).

The GEMM multiplies the exact int4 codes by the fp16-staged activations and
applies each weight row's fp16 scale to the fp32 sum, as the GEMV does; only
the order of the fp32 sums differs."""

import pytest
import torch

import oracle
from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import Q4MoELayerGPU
from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, id_mismatches, rel_l2

pytestmark = pytest.mark.gpu

Q4_SMALL = synth.MixtralQ4Config("q4-small", hidden=512, inter=768, n_experts=8, top_k=2)


@pytest.fixture(autouse=True)
def _clean_error_word():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = native.load_library()
    yield
    torch.cuda.synchronize()
    assert lib.moe_b200_device_error(None) == 0, "a bounded wait inside a kernel gave up"


def _both(cfg, tokens, seed, dtype):
    layer = synth.make_q4_layer(cfg, seed=seed, device="cuda")
    gpu = Q4MoELayerGPU(layer)
    assert gpu.tables_tiled is not None
    x = synth.make_hidden(tokens, cfg.hidden, seed=seed + 1, device="cuda").to(dtype)
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int64, device="cuda")
    gemm = gpu.forward(x, ids=ids, layout=1).clone()
    gemv = gpu.forward(x, layout=0).clone()
    torch.cuda.synchronize()
    return layer, x, ids, gemm, gemv


@pytest.mark.parametrize("tokens", [512, 700])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_q4_prefill_matches_gemv_and_oracle(cuda_device, tokens, dtype):
    layer, x, ids, gemm, gemv = _both(Q4_SMALL, tokens, seed=tokens, dtype=dtype)
    assert gemm.dtype == dtype
    assert rel_l2(gemm, gemv) <= 1e-3 and cos_dist(gemm, gemv) <= 1e-5
    n = 96  # the oracle's token loop on a slice: tokens are independent
    want, route = oracle.mixtral_q4_layer(x[:n].cpu(), layer)
    bad, excused = id_mismatches(ids[:n], route)
    assert bad == excused
    assert rel_l2(gemm[:n], want) <= REL_L2_GATE and cos_dist(gemm[:n], want) <= COS_GATE


def test_q4_prefill_mixtral_shape(cuda_device):
    cfg = synth.C4_MIXTRAL
    layer, x, ids, gemm, gemv = _both(cfg, 512, seed=9, dtype=torch.bfloat16)
    assert rel_l2(gemm, gemv) <= 1e-3 and cos_dist(gemm, gemv) <= 1e-5
    n = 8
    want, route = oracle.mixtral_q4_layer(x[:n].cpu(), layer)
    assert rel_l2(gemm[:n], want) <= REL_L2_GATE and cos_dist(gemm[:n], want) <= COS_GATE


def test_q4_tiled_layout_is_a_permutation(cuda_device):
    """The tiled copy holds the same bytes: 4 KiB runs of 128 rows x 32 bytes."""
    rows, cols = 200, 192
    packed = torch.randint(0, 256, (rows, cols // 2), dtype=torch.uint8, device="cuda")
    lib = native.load_library()
    nbytes = int(lib.moe_q4_tiled_bytes(rows, cols))
    assert nbytes == 256 * cols // 2
    tiled = torch.empty((nbytes,), dtype=torch.uint8, device="cuda")
    native._check(lib.moe_q4_tile_weights(native._ptr(packed), native._ptr(tiled), rows, cols, native._stream()),
                  "moe_q4_tile_weights")
    t = tiled.cpu().view(2, cols // 64, 128, 32)  # group, 64-column block, row, byte
    want = torch.zeros((256, cols // 2), dtype=torch.uint8)
    want[:rows] = packed.cpu()
    got = t.permute(0, 2, 1, 3).reshape(256, cols // 2)
    assert torch.equal(got, want)

"""Pin the C restatement (oracle/kernels.py) to the reference's own kernels
compiled from source (oracle/ref.py, `make -C oracle ref`).

Bit-exact where the reference's operation order is restated exactly (FP8
linear/MLP/many variants, FP8 and Q4 dequant, row8 packing, the fp32
combine); to a tight tolerance where the reference uses vector FMAs or a
different summation order (Q4 AVX2 dot products, row8 GEMV, fp16 MoE).
These mirror the reference's own tests (tests/test_native_fp8_linear.py,
test_native_fp8_dequant.py, test_native_ds_moe.py, test_native_ds_router.py,
test_q4_quantizer.py, test_native_fp16_packed_gemv.py).
"""

import pytest
import torch

from oracle import kernels as orc
from oracle import ref

pytestmark = pytest.mark.skipif(not ref.available(), reason="reference build (oracle/_ref) missing")


def _fp8(values: torch.Tensor) -> torch.Tensor:
    return values.to(torch.float8_e4m3fn).view(torch.uint8).contiguous()


def _expert(seed: int, hidden: int, inter: int, scale=(0.875, 1.125, 0.75), nan_codes=False):
    gen = torch.Generator().manual_seed(seed)
    gate = _fp8(torch.randn((inter, hidden), generator=gen) * 0.25)
    up = _fp8(torch.randn((inter, hidden), generator=gen) * 0.25)
    down = _fp8(torch.randn((hidden, inter), generator=gen) * 0.25)
    if nan_codes:
        gate.view(-1)[::97] = 0x7F
        down.view(-1)[5::89] = 0xFF
    gs = (inter + 127) // 128, (hidden + 127) // 128
    ds = (hidden + 127) // 128, (inter + 127) // 128
    g_s = torch.rand(gs, generator=gen) + scale[0]
    u_s = torch.rand(gs, generator=gen) + scale[1]
    d_s = torch.rand(ds, generator=gen) + scale[2]
    return gate, g_s, up, u_s, down, d_s


SHAPES = [(64, 32, 1), (128, 128, 4), (384, 130, 3), (300, 257, 2)]


@pytest.mark.parametrize("hidden,inter,batch", SHAPES)
def test_linear_bit_exact(hidden, inter, batch):
    g, gs, *_ = _expert(3, hidden, inter, nan_codes=True)
    x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(9))
    assert torch.equal(orc.fp8_linear(g, gs, x), ref.fp8_linear(g, gs, x))


@pytest.mark.parametrize("hidden,inter,batch", SHAPES)
def test_mlp_bit_exact(hidden, inter, batch):
    item = _expert(5, hidden, inter, nan_codes=True)
    x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(11)) * 0.5
    assert torch.equal(orc.fp8_mlp(*item, x), ref.fp8_mlp(*item, x))


def test_many_variants_bit_exact():
    hidden, inter, batch = 256, 160, 3
    items = [_expert(s, hidden, inter) for s in (21, 22, 23, 24)]
    x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(12)) * 0.5
    assert torch.equal(orc.fp8_mlp_many(items, x), ref.fp8_mlp_many(items, x))
    route = torch.tensor([0.31, 0.17, 0.29, 0.23])
    assert torch.equal(orc.fp8_mlp_many_weighted(items, x, route), ref.fp8_mlp_many_weighted(items, x, route))
    rows = torch.tensor([[0.6, 0.0, 0.4], [0.4, 0.5, 0.0], [0.0, 0.5, 0.35], [0.0, 0.0, 0.25]])
    assert torch.equal(orc.fp8_mlp_many_row_weighted(items, x, rows), ref.fp8_mlp_many_row_weighted(items, x, rows))
    pi, pr, pw = [], [], []
    for e in range(rows.shape[0]):
        for b in range(rows.shape[1]):
            if rows[e, b] != 0:
                pi.append(e)
                pr.append(b)
                pw.append(float(rows[e, b]))
    args = (torch.tensor(pi), torch.tensor(pr), torch.tensor(pw))
    assert torch.equal(orc.fp8_mlp_many_pair_weighted(items, x, *args), ref.fp8_mlp_many_pair_weighted(items, x, *args))


def test_avx512_twins_match_scalar_reference():
    """The reference's AVX-512 kernels are bit-exact to its scalar ones
    (fp8_linear_avx512.cpp:103-133); the oracle therefore covers both."""
    try:
        ref.lib("fp8_linear_avx512")
    except OSError:
        pytest.skip("AVX-512 reference build unavailable")
    if not ref.lib("fp8_linear_avx512").fp8_linear_avx512_cpu_has_avx512():
        pytest.skip("host has no AVX-512")
    item = _expert(31, 256, 384)
    x = torch.randn((2, 256), generator=torch.Generator().manual_seed(1)) * 0.25
    assert torch.equal(ref.fp8_mlp(*item, x, avx512=True), orc.fp8_mlp(*item, x))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dequant_bit_exact(dtype):
    codes = torch.arange(256, dtype=torch.uint8).repeat(3, 2)[:, :300].contiguous()
    codes = torch.cat([codes] * 50)[:150]
    s = torch.rand((2, 3), generator=torch.Generator().manual_seed(2)) * 4
    a, b = orc.fp8_dequant(codes, s, dtype), ref.fp8_dequant(codes, s, dtype)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_q4_dequant_bit_exact():
    gen = torch.Generator().manual_seed(7)
    packed = torch.randint(0, 256, (97 * 64 // 2,), generator=gen, dtype=torch.uint8)
    scales = (torch.rand((97,), generator=gen) * 0.01).to(torch.float16)
    a = orc.q4_dequant_to_fp16(packed, scales, 97, 64)
    b = ref.q4_dequant_to_fp16(packed, scales, 97, 64)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_q4_moe_close():
    from pocketlm_b200.synth import quantize_q4_rows

    gen = torch.Generator().manual_seed(8)
    hidden, inter = 128, 96
    experts = []
    for _ in range(2):
        item = []
        for shape in ((inter, hidden), (inter, hidden), (hidden, inter)):
            item.extend(quantize_q4_rows(torch.randn(shape, generator=gen) * 0.02))
        experts.append(item)
    x = torch.randn((hidden,), generator=gen).to(torch.float16)
    route = torch.tensor([0.7, 0.3])
    a = orc.q4_moe_selected_forward(x, experts, route, hidden, inter).float()
    b = ref.q4_moe_selected_forward(x, experts, route, hidden, inter).float()
    assert torch.allclose(a, b, atol=2e-4, rtol=2e-3)


@pytest.mark.parametrize("rows,cols", [(1, 7), (17, 31), (32, 64)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rows8(rows, cols, dtype):
    gen = torch.Generator().manual_seed(rows * 100 + cols)
    w = torch.randn((rows, cols), generator=gen).to(dtype)
    x = torch.randn((cols,), generator=gen).to(dtype)
    assert torch.equal(orc.pack_rows8(w.view(torch.int16)), ref.pack_rows8(w.view(torch.int16)))
    packed = ref.pack_rows8(w.view(torch.int16))
    a = orc.packed_gemv_rows8(x, packed, rows, cols)
    b = ref.packed_gemv_rows8(x, packed, rows, cols)
    assert torch.allclose(a, b, atol=1e-5, rtol=1e-5)


def test_softmax_router_matches():
    gen = torch.Generator().manual_seed(20260519)
    router = torch.randn((11, 16), generator=gen).mul(0.25).to(torch.float16)
    rows = torch.randn((5, 16), generator=gen).mul(0.5).to(torch.float16)
    for row in rows:
        ia, wa = orc.router_softmax_topk_u16(row, router, 4)
        ib, wb = ref.router_softmax_topk_u16(row, router, 4)
        assert torch.equal(ia, ib)
        assert torch.allclose(wa, wb, atol=1e-6, rtol=1e-6)


def test_fp16_moe_selected_close():
    gen = torch.Generator().manual_seed(5)
    seq, hidden, inter, sel = 3, 64, 48, 2
    x = torch.randn((seq, hidden), generator=gen).to(torch.bfloat16)
    g = (torch.randn((sel, inter, hidden), generator=gen) * 0.1).to(torch.bfloat16)
    u = (torch.randn((sel, inter, hidden), generator=gen) * 0.1).to(torch.bfloat16)
    d = (torch.randn((sel, hidden, inter), generator=gen) * 0.1).to(torch.bfloat16)
    r = torch.tensor([[0.6, 0.4], [0.5, 0.5], [0.9, 0.1]])
    a = orc.moe_selected_forward_u16(x, g, u, d, r).float()
    b = ref.moe_selected_forward_u16(x, g, u, d, r).float()
    assert torch.allclose(a, b, atol=1e-2, rtol=1e-2)

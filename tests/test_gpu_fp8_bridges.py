"""GPU parity of the reference-compatible FP8 bridges (pocketlm_b200.native)
against the CPU oracle (oracle/kernels.py, itself bit-exact to the reference's
fp8_linear.cpp / fp8_dequant.cpp).

Tolerances: the kernels compute in fp32 like the reference but sum in a
different order, so outputs agree to fp32 rounding: |gpu - oracle| <=
1e-5 * max|oracle| + 1e-6.  Dequantisation is bit-exact (all 256 codes,
including the NaN payloads).  Cases mirror tests/test_native_fp8_linear.py
and test_native_fp8_dequant.py of the reference.
"""

import pytest
import torch

from oracle import kernels as orc
from pocketlm_b200 import native

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["auto", "stream", "direct"])
def gemv_impl(request):
    """Run every case on each expert-GEMV kernel the bridges use: auto and
    the direct-load one (fp8_gemv.cu), the bulk-copy streaming one
    (fp8_stream.cu)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = native.load_library()
    assert lib.moe_b200_select_gemv({"auto": 0, "stream": 1, "direct": 2, "mma_tma": 4}[request.param]) == 0
    yield request.param
    torch.cuda.synchronize()
    assert lib.moe_b200_device_error(None) == 0, "a bounded wait inside a kernel gave up"
    lib.moe_b200_select_gemv(0)


def _fp8(values: torch.Tensor) -> torch.Tensor:
    return values.to(torch.float8_e4m3fn).view(torch.uint8).contiguous()


def _item(seed, hidden, inter, nan_codes=False):
    gen = torch.Generator().manual_seed(seed)
    gate = _fp8(torch.randn((inter, hidden), generator=gen) * 0.25)
    up = _fp8(torch.randn((inter, hidden), generator=gen) * 0.25)
    down = _fp8(torch.randn((hidden, inter), generator=gen) * 0.25)
    if nan_codes:
        gate.view(-1)[::97] = 0x7F
        down.view(-1)[5::89] = 0xFF
    gs = ((inter + 127) // 128, (hidden + 127) // 128)
    ds = ((hidden + 127) // 128, (inter + 127) // 128)
    return (gate, torch.rand(gs, generator=gen) + 0.5, up, torch.rand(gs, generator=gen) + 0.5,
            down, torch.rand(ds, generator=gen) + 0.5)


def _close(actual, expected, rel=1e-5):
    actual, expected = actual.detach().cpu().float(), expected.detach().cpu().float()
    scale = float(expected.abs().max()) if expected.numel() else 1.0
    err = float((actual - expected).abs().max()) if expected.numel() else 0.0
    assert err <= rel * scale + 1e-6, f"max abs err {err} vs scale {scale}"


SHAPES = [(64, 32, 1), (128, 128, 4), (256, 384, 2), (300, 257, 3), (7168, 2048, 1)]


@pytest.mark.parametrize("hidden,inter,batch", SHAPES)
def test_linear(cuda_device, hidden, inter, batch):
    w, s, *_ = _item(1, hidden, inter, nan_codes=True)
    x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(2))
    out = native.fp8_e4m3_block_linear_f32(w.cuda(), s.cuda(), x.cuda())
    assert out.is_cuda and out.shape == (batch, inter)
    _close(out, orc.fp8_linear(w, s, x))


def test_dual_linear(cuda_device):
    a, sa, b, sb, *_ = _item(3, 256, 130)
    x = torch.randn((5, 256), generator=torch.Generator().manual_seed(4))
    oa, ob = native.fp8_e4m3_block_dual_linear_f32(a, sa, b, sb, x)  # CPU tensors in, CPU out
    assert oa.device.type == "cpu"
    _close(oa, orc.fp8_linear(a, sa, x))
    _close(ob, orc.fp8_linear(b, sb, x))


@pytest.mark.parametrize("hidden,inter,batch", SHAPES)
def test_mlp(cuda_device, hidden, inter, batch):
    item = _item(5, hidden, inter, nan_codes=True)
    x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(6)) * 0.5
    out = native.fp8_e4m3_block_mlp_f32(*[t.cuda() for t in item], x.cuda())
    _close(out, orc.fp8_mlp(*item, x))
    out2 = native.fp8_e4m3_block_mlp_avx512_f32(*[t.cuda() for t in item], x.cuda())
    assert torch.equal(out, out2)


def test_many_and_weighted(cuda_device):
    hidden, inter, batch = 256, 160, 3
    items = [_item(s, hidden, inter) for s in (21, 22, 23, 24)]
    gpu_items = [tuple(t.cuda() for t in it) for it in items]
    x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(7)) * 0.5
    _close(native.fp8_e4m3_block_mlp_many_f32(gpu_items, x.cuda()), orc.fp8_mlp_many(items, x))
    route = torch.tensor([0.31, 0.17, 0.29, 0.23])
    expected = orc.fp8_mlp_many_weighted(items, x, route)
    _close(native.fp8_e4m3_block_mlp_many_weighted_f32(gpu_items, x.cuda(), route.cuda()), expected)
    _close(native.fp8_e4m3_block_mlp_many_weighted_avx512_f32(gpu_items, x.cuda(), route.cuda()), expected)


def test_row_and_pair_weighted(cuda_device):
    hidden, inter = 64, 32
    items = [_item(s, hidden, inter) for s in (5, 6, 7, 8)]
    x = torch.linspace(-0.5, 0.5, steps=3 * hidden).reshape(3, hidden)
    rows = torch.tensor([[0.6, 0.0, 0.4], [0.4, 0.5, 0.0], [0.0, 0.5, 0.35], [0.0, 0.0, 0.25]])
    expected = orc.fp8_mlp_many_row_weighted(items, x, rows)
    got = native.fp8_e4m3_block_mlp_many_row_weighted_f32(items, x, rows)
    _close(got, expected)
    pi, pr, pw = [], [], []
    for e in range(rows.shape[0]):
        for b in range(rows.shape[1]):
            if rows[e, b] != 0:
                pi.append(e)
                pr.append(b)
                pw.append(float(rows[e, b]))
    args = (torch.tensor(pi), torch.tensor(pr), torch.tensor(pw))
    pair = native.fp8_e4m3_block_mlp_many_pair_weighted_f32(items, x, *args)
    _close(pair, orc.fp8_mlp_many_pair_weighted(items, x, *args))
    _close(pair, got)


def test_pair_weighted_rejects_bad_index(cuda_device):
    items = [_item(9, 64, 32)]
    x = torch.zeros((2, 64))
    with pytest.raises(RuntimeError):
        native.fp8_e4m3_block_mlp_many_pair_weighted_f32(items, x, torch.tensor([0, 1]), torch.tensor([0, 1]),
                                                          torch.tensor([1.0, 1.0]))


def test_shape_errors_match_reference_messages(cuda_device):
    gate, gs, up, us, down, ds = _item(11, 64, 32)
    with pytest.raises(ValueError, match="128x128 block layout"):
        native.fp8_e4m3_dequant_to_fp16(torch.zeros((256, 256), dtype=torch.uint8), torch.ones((1, 1)))
    with pytest.raises(ValueError, match="down weight must have shape"):
        native.fp8_e4m3_block_mlp_f32(gate, gs, up, us, gate, ds, torch.zeros((1, 64)))
    with pytest.raises(ValueError, match="hidden input size"):
        native.fp8_e4m3_block_mlp_f32(gate, gs, up, us, down, ds, torch.zeros((1, 63)))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dequant_all_codes_bit_exact(cuda_device, dtype):
    codes = torch.arange(256, dtype=torch.uint8).reshape(16, 16)
    for scale in (torch.tensor([[1.0]]), torch.tensor([[0.75]])):
        fn = native.fp8_e4m3_dequant_to_bf16 if dtype == torch.bfloat16 else native.fp8_e4m3_dequant_to_fp16
        got = fn(codes.cuda(), scale.cuda())
        assert torch.equal(got.view(torch.int16).cpu(), orc.fp8_dequant(codes, scale, dtype).view(torch.int16))


def test_dequant_blocks_bit_exact(cuda_device):
    gen = torch.Generator().manual_seed(12)
    codes = torch.randint(0, 256, (300, 520), generator=gen, dtype=torch.uint8)
    scale = torch.rand((3, 5), generator=gen) * 3
    for dtype in (torch.float16, torch.bfloat16):
        fn = native.fp8_e4m3_dequant_to_bf16 if dtype == torch.bfloat16 else native.fp8_e4m3_dequant_to_fp16
        got = fn(codes.cuda(), scale.cuda())
        assert torch.equal(got.view(torch.int16).cpu(), orc.fp8_dequant(codes, scale, dtype).view(torch.int16))


def test_session_combine_and_counters(cuda_device):
    outputs = torch.tensor([[[1.0, 2.0, 3.0, 4.0]], [[10.0, 20.0, 30.0, 40.0]]])
    route = torch.tensor([0.75, 0.25])
    with native.DeepSeekNativeSession(num_layers=2, hidden_dim=4, num_experts=4, top_k=2) as session:
        got = native.ds_moe_layer_forward(session, outputs.cuda(), route.cuda())
        assert torch.equal(got.cpu(), orc.combine_f32(outputs, route))
        assert session.monolithic_call_count() == 1
        assert session.expert_invocation_count() == 2
        hidden = torch.tensor([[0.5, -0.25, 0.75, 1.0]])
        items = [_item(1, 4, 2), _item(2, 4, 2)]
        w = torch.tensor([0.6, 0.4])
        got = native.ds_moe_layer_forward_fp8(session, items, hidden, w)
        _close(got, orc.fp8_mlp_many_weighted(items, hidden, w))
        assert session.monolithic_call_count() == 2
        assert session.expert_invocation_count() == 4

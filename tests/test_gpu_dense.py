"""GPU parity of the Q4, row8 and 16-bit dense MoE entry points against the
oracle (a CPU restatement of q4_dequant.cpp, fp16_packed_gemv.cpp and
fp16_moe.cpp) and the reference's own outputs in tests/golden/.

Shapes cover both GPU paths: the warp-MMA kernel (hidden and intermediate
multiples of 128 for int4, of 32 for 16-bit weights) and the generic kernel
(any other shape, e.g. the golden Q4 case with hidden 96)."""

import pytest
import torch

import oracle
from oracle import kernels as orc
from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import Q4MoELayerGPU
from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, id_mismatches, rel_l2

pytestmark = pytest.mark.gpu

# fp32 sums in a different order than the reference, activations staged in
# fp16 between the projections: a few parts in 1e4 of the output norm
DENSE_REL_L2 = 3e-3


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _q4_expert(H, I, gen):
    mats = [torch.randn(shape, generator=gen) * 0.02 for shape in ((I, H), (I, H), (H, I))]
    out = []
    for m in mats:
        out.extend(synth.quantize_q4_rows(m))
    return out


def test_q4_dequant_matches_reference_golden(cuda_device, golden_dir):
    g = torch.load(golden_dir / "q4_moe.pt", weights_only=False)
    h, i = g["x"].numel(), g["experts"][0][1].numel()
    got = native.q4_dequant_to_fp16(g["experts"][0][0].cuda(), g["experts"][0][1].cuda(), i, h)
    assert torch.equal(got.cpu().view(torch.int16), g["dequant_gate0"].view(torch.int16))


@pytest.mark.parametrize("channels,size", [(1, 1), (3, 7), (17, 33), (64, 4096)])
def test_q4_dequant_bit_exact(cuda_device, channels, size):
    gen = _gen(channels * 1000 + size)
    codes = torch.randint(-8, 8, (channels * size,), generator=gen)
    packed = synth.pack_int4(codes)
    scales = (torch.rand((channels,), generator=gen) * 0.01 + 1e-4).to(torch.float16)
    want = orc.q4_dequant_to_fp16(packed, scales, channels, size)
    got = native.q4_dequant_to_fp16(packed.cuda(), scales.cuda(), channels, size)
    assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16))


def test_q4_dequant_many(cuda_device):
    gen = _gen(5)
    items, wants = [], []
    for channels, size in ((4, 16), (9, 5), (128, 256)):
        packed = synth.pack_int4(torch.randint(-8, 8, (channels * size,), generator=gen))
        scales = (torch.rand((channels,), generator=gen) * 0.01).to(torch.float16)
        items.append((packed.cuda(), scales.cuda(), channels, size))
        wants.append(orc.q4_dequant_to_fp16(packed, scales, channels, size))
    outs = native.q4_dequant_many_to_fp16(items)
    for got, want in zip(outs, wants):
        assert torch.equal(got.cpu().view(torch.int16), want.view(torch.int16))
    assert native.q4_dequant_many_to_fp16([]) == []


def test_q4_moe_selected_matches_reference_golden(cuda_device, golden_dir):
    g = torch.load(golden_dir / "q4_moe.pt", weights_only=False)
    h, i = g["x"].numel(), g["experts"][0][1].numel()
    experts = [[t.cuda() for t in item] for item in g["experts"]]
    got = native.q4_moe_selected_forward_u16(g["x"].cuda(), experts, g["route"].cuda(), hidden_size=h,
                                             intermediate_size=i)
    assert got.dtype == torch.float16 and got.shape == (h,)
    assert rel_l2(got, g["out"]) <= DENSE_REL_L2


@pytest.mark.parametrize("H,I,S", [(96, 160, 3), (256, 384, 2), (512, 1024, 4)])
def test_q4_moe_selected_matches_oracle(cuda_device, H, I, S):
    gen = _gen(H + I + S)
    experts = [_q4_expert(H, I, gen) for _ in range(S)]
    x = torch.randn((H,), generator=gen).to(torch.float16)
    route = torch.rand((S,), generator=gen)
    want = orc.q4_moe_selected_forward(x, experts, route, H, I)
    got = native.q4_moe_selected_forward_u16(x.cuda(), [[t.cuda() for t in e] for e in experts], route.cuda(),
                                             hidden_size=H, intermediate_size=I)
    assert rel_l2(got, want) <= DENSE_REL_L2 and cos_dist(got, want) <= COS_GATE


@pytest.mark.parametrize("tokens", [1, 3, 19])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_q4_layer_matches_oracle(cuda_device, tokens, dtype):
    cfg = synth.MixtralQ4Config("q4-small", hidden=512, inter=768, n_experts=8, top_k=2)
    layer = synth.make_q4_layer(cfg, seed=3)
    x = synth.make_hidden(tokens, cfg.hidden, seed=4).to(dtype)
    want, route = oracle.mixtral_q4_layer(x, layer)
    gpu = Q4MoELayerGPU(layer)
    ids = torch.empty((tokens, cfg.top_k), dtype=torch.int64, device="cuda")
    w = torch.empty((tokens, cfg.top_k), dtype=torch.float32, device="cuda")
    got = gpu.forward(x.cuda(), ids=ids, weights=w)
    assert got.dtype == dtype
    bad, excused = id_mismatches(ids, route)
    assert bad == excused
    assert rel_l2(got, want) <= REL_L2_GATE and cos_dist(got, want) <= COS_GATE
    same = (torch.sort(ids.cpu(), 1).values == torch.sort(route.ids, 1).values).all(dim=1)
    assert torch.allclose(w.cpu()[same].sort(1).values, route.weights.float()[same].sort(1).values, atol=1e-5)


def test_rows8_matches_reference_golden(cuda_device, golden_dir):
    for case in torch.load(golden_dir / "rows8.pt", weights_only=False):
        rows, cols = case["w"].shape
        packed = native.pack_weight_rows8(case["w"].cuda())
        assert torch.equal(packed.cpu().view(torch.int16), case["packed"])
        out = native.packed_gemv_rows8(case["x"].cuda(), packed, rows=rows, cols=cols)
        assert torch.allclose(out.cpu(), case["out"], atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("rows,cols", [(5, 3), (1000, 4096), (14336, 512)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rows8_matches_oracle(cuda_device, rows, cols, dtype):
    gen = _gen(rows * 7 + cols)
    w = (torch.randn((rows, cols), generator=gen) * 0.05).to(dtype)
    x = torch.randn((cols,), generator=gen).to(dtype)
    packed = native.pack_weight_rows8(w.cuda())
    assert torch.equal(packed.cpu().view(torch.int16), orc.pack_rows8(w.view(torch.int16)))
    got = native.packed_gemv_rows8(x.cuda(), packed, rows=rows, cols=cols)
    want = orc.packed_gemv_rows8(x, packed.cpu().view(torch.int16), rows, cols)
    assert got.shape == (rows,)
    assert torch.allclose(got.cpu(), want, atol=1e-4, rtol=1e-4)


def test_rows8_cache_counts(cuda_device, monkeypatch):
    monkeypatch.setenv("PCKETLM_PACKED_GEMV_CACHE_MB", "1")
    native.reset_packed_gemv_cache()
    w = torch.randn((16, 32)).to(torch.float16).cuda()
    a = native.cached_pack_weight_rows8("w", w)
    b = native.cached_pack_weight_rows8("w", w)
    assert a is b
    stats = native.packed_gemv_cache_stats()
    assert stats["hits"] == 1 and stats["misses"] == 1 and stats["stores"] == 1 and stats["resident_count"] == 1
    native.reset_packed_gemv_cache()


def _dense_weights(S, H, I, dtype, gen):
    g = (torch.randn((S, I, H), generator=gen) * 0.05).to(dtype)
    u = (torch.randn((S, I, H), generator=gen) * 0.05).to(dtype)
    d = (torch.randn((S, H, I), generator=gen) * 0.05).to(dtype)
    return g, u, d


@pytest.mark.parametrize("T,H,S,I", [(1, 40, 2, 24), (5, 256, 3, 128), (9, 512, 4, 1024)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_moe_selected_forward_matches_oracle(cuda_device, T, H, S, I, dtype):
    gen = _gen(T * H + S * I)
    g, u, d = _dense_weights(S, H, I, dtype, gen)
    x = torch.randn((T, H), generator=gen).to(dtype)
    route = torch.rand((T, S), generator=gen)
    want = orc.moe_selected_forward_u16(x, g, u, d, route)
    got = native.moe_selected_forward_u16(x.cuda(), g.cuda(), u.cuda(), d.cuda(), route.cuda())
    assert got.dtype == dtype and got.shape == (T, H)
    assert rel_l2(got, want) <= DENSE_REL_L2 and cos_dist(got, want) <= COS_GATE


def _fp16_moe_expected(x, router, g, u, d, k, normalize):
    probs = torch.softmax(x.float() @ router.float().t(), dim=-1)
    w, ids = torch.topk(probs, k, dim=-1)
    if normalize:
        w = w / w.sum(dim=-1, keepdim=True)
    rows = [orc.moe_selected_forward_u16(x[t:t + 1], g[ids[t]], u[ids[t]], d[ids[t]], w[t:t + 1])
            for t in range(x.shape[0])]
    return torch.cat(rows), ids, w, probs


@pytest.mark.parametrize("T,H,E,k,I", [(3, 64, 4, 2, 32), (7, 256, 8, 2, 384)])
@pytest.mark.parametrize("normalize", [True, False])
def test_moe_forward_fp16_matches_oracle(cuda_device, T, H, E, k, I, normalize):
    gen = _gen(T + H + E + k + I)
    g, u, d = _dense_weights(E, H, I, torch.float16, gen)
    router = (torch.randn((E, H), generator=gen) * 0.1).to(torch.float16)
    x = torch.randn((T, H), generator=gen).to(torch.float16)
    want, want_ids, want_w, probs = _fp16_moe_expected(x, router, g, u, d, k, normalize)
    out, ids, w = native.moe_forward_fp16(x.cuda(), router.cuda(), g.cuda(), u.cuda(), d.cuda(), top_k=k,
                                          normalize_topk=normalize)
    route = oracle.RouteResult(ids=want_ids, weights=want_w, choice=probs, weights_f32=want_w)
    bad, excused = id_mismatches(ids, route)
    assert bad == excused == 0
    assert torch.allclose(w.cpu(), want_w, atol=1e-5, rtol=1e-4)
    assert rel_l2(out, want) <= DENSE_REL_L2 and cos_dist(out, want) <= COS_GATE


def test_dense_entry_points_reject_bad_arguments(cuda_device):
    lib = native.load_library()
    assert lib.moe_q4_dequant_to_fp16(None, None, None, 1, 1, None) == 1
    assert lib.moe_pack_u16_rows8(None, None, 1, 1, None) == 1
    x = torch.zeros(4, dtype=torch.float16, device="cuda")
    assert lib.moe_packed_gemv_rows8(native._ptr(x), native._ptr(x), native._ptr(x), 1, 1, 7, None) == 2
    assert lib.moe_moe_selected_forward_u16(native._ptr(x), native._ptr(x), native._ptr(x), native._ptr(x),
                                            native._ptr(x), native._ptr(x), 1, 1, 1, 1, 5, None, 0, None) == 3
    assert lib.moe_moe_forward_fp16(native._ptr(x), native._ptr(x), native._ptr(x), native._ptr(x), native._ptr(x),
                                    native._ptr(x), None, None, 1, 4, 2, 3, 4, 1, None, 0, None) == 3

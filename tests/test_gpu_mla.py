"""MLA attention on the GPU (csrc/mla.cu) through the reference-shaped entry
points pocketlm_b200.native.ds_mla_attention_flash_forward /
ds_attention_block_forward (ds_forward.cpp:517-782): against the
reference's own outputs (tests/golden/mla.pt), against the oracle
restatement at the DeepSeek-V3 shapes (128 heads, kv_lora_rank 512, rope 64,
nope 128, v 128) for cache lengths that take 1 to 64 position splits, and
the in-place cache append of the C entry point.  fp32 against fp32: the
tolerance is summation order (rel-L2 1e-5; the reference's own test holds
its native block to atol = rtol = 1e-5 against torch)."""

import ctypes

import pytest
import torch

import oracle.mla as omla
from pocketlm_b200 import native

pytestmark = pytest.mark.gpu

TOL = 1e-5
DSV3 = dict(heads=128, nope=128, rope=64, R=512, v=128)


def _rel(a, b):
    return float((a.detach().cpu().float() - b.detach().cpu().float()).norm() / b.float().norm().clamp_min(1e-30))


def _block_args(inp):
    return (inp["hidden"], inp["q_a"], inp["q_b"], inp["kv_a"], inp["kv_b"], inp["o_w"], inp["q_norm"],
            inp["kv_norm"])


def test_golden_cases_match_reference(cuda_device, golden_dir):
    cases = torch.load(golden_dir / "mla.pt", weights_only=False)
    for tag, case in cases.items():
        inp = case["inputs"]
        if case["kind"] == "block":
            with native.DeepSeekNativeSession(num_layers=1, hidden_dim=inp["hidden"].numel(), num_experts=0,
                                              top_k=0) as session:
                out, (kv, pe) = native.ds_attention_block_forward(
                    session, *(t.cuda() for t in _block_args(inp)),
                    previous_kv_cache=None if inp["previous_kv"] is None else inp["previous_kv"].cuda(),
                    previous_pe_cache=None if inp["previous_pe"] is None else inp["previous_pe"].cuda(),
                    rope_cos=inp["cos"].cuda(), rope_sin=inp["sin"].cuda(), **case["dims"])
                assert session.fused_attention_invocation_count() == 1
                assert session.attention_invocation_count() == 1 and session.monolithic_call_count() == 1
            assert out.device.type == "cuda"
            assert _rel(out, case["out"]) <= TOL, tag
            assert torch.allclose(out.cpu(), case["out"], atol=1e-5, rtol=1e-5), tag
            assert torch.allclose(kv.cpu(), case["next_kv"], atol=1e-5, rtol=1e-5), tag
            assert torch.allclose(pe.cpu(), case["next_pe"], atol=1e-5, rtol=1e-5), tag
        else:
            # host tensors in, host tensor out, as the reference's callers pass them
            out = native.ds_mla_attention_flash_forward(inp["q_nope"], inp["q_pe"], inp["kv_cache"],
                                                        inp["pe_cache"], inp["wkv_b"],
                                                        softmax_scale=case["softmax_scale"])
            assert out.device.type == "cpu"
            assert _rel(out, case["out"]) <= TOL, tag


@pytest.mark.parametrize("L", [1, 16, 17, 1000, 4096])
def test_core_dsv3_shape_matches_oracle(cuda_device, L):
    d = DSV3
    g = torch.Generator(device="cuda").manual_seed(L)
    qn = torch.randn((d["heads"], d["nope"]), generator=g, device="cuda")
    qp = torch.randn((d["heads"], d["rope"]), generator=g, device="cuda")
    kv = torch.randn((L, d["R"]), generator=g, device="cuda") * 0.5
    pe = torch.randn((L, d["rope"]), generator=g, device="cuda") * 0.5
    w = torch.randn((d["heads"], d["nope"] + d["v"], d["R"]), generator=g, device="cuda") * 0.05
    scale = (d["nope"] + d["rope"]) ** -0.5
    out = native.ds_mla_attention_flash_forward(qn, qp, kv, pe, w, softmax_scale=scale)
    torch.cuda.synchronize()
    want = omla.mla_attention_flash(qn, qp, kv, pe, w, scale)
    assert _rel(out, want) <= TOL


@pytest.mark.parametrize("heads,L,nope,rope,R,v", [(20, 333, 16, 8, 40, 12), (3, 50, 7, 5, 33, 5),
                                                   (33, 129, 64, 32, 1024, 64)])
def test_core_odd_shapes_match_oracle(cuda_device, heads, L, nope, rope, R, v):
    g = torch.Generator(device="cuda").manual_seed(heads + L)
    qn, qp = torch.randn((heads, nope), generator=g, device="cuda"), torch.randn((heads, rope), generator=g, device="cuda")
    kv, pe = torch.randn((L, R), generator=g, device="cuda"), torch.randn((L, rope), generator=g, device="cuda")
    w = torch.randn((heads, nope + v, R), generator=g, device="cuda") * 0.1
    out = native.ds_mla_attention_flash_forward(qn, qp, kv, pe, w, softmax_scale=0.1)
    assert _rel(out, omla.mla_attention_flash(qn, qp, kv, pe, w, 0.1)) <= TOL


def test_core_without_rope_is_rejected_like_the_reference(cuda_device):
    # an empty q_pe has no address: the reference returns 1 (ds_forward.cpp:531-536) and its wrapper raises
    qn, kv, w = torch.randn(2, 3), torch.randn(4, 8), torch.randn(2, 5, 8)
    with pytest.raises(RuntimeError, match="code 1"):
        native.ds_mla_attention_flash_forward(qn, torch.zeros(2, 0), kv, torch.zeros(4, 0), w, softmax_scale=1.0)


def _dsv3_block(prev_len, seed, H=7168, q_rank=1536):
    d = DSV3
    g = torch.Generator(device="cuda").manual_seed(seed)

    def rnd(*shape, scale=1.0):
        return torch.randn(shape, generator=g, device="cuda") * scale

    inp = dict(hidden=rnd(H), q_a=rnd(q_rank, H, scale=H ** -0.5), q_b=rnd(d["heads"] * (d["nope"] + d["rope"]), q_rank,
                                                                           scale=q_rank ** -0.5),
               kv_a=rnd(d["R"] + d["rope"], H, scale=H ** -0.5), kv_b=rnd(d["heads"] * (d["nope"] + d["v"]), d["R"],
                                                                         scale=d["R"] ** -0.5),
               o_w=rnd(H, d["heads"] * d["v"], scale=(d["heads"] * d["v"]) ** -0.5), q_norm=1 + 0.1 * rnd(q_rank),
               kv_norm=1 + 0.1 * rnd(d["R"]), previous_kv=rnd(prev_len, d["R"]), previous_pe=rnd(prev_len, d["rope"]))
    angles = torch.arange(d["rope"] // 2, device="cuda", dtype=torch.float32) * (prev_len + 1) * 1e-3
    inp["cos"], inp["sin"] = angles.cos(), angles.sin()
    dims = dict(q_lora_rank=q_rank, kv_lora_rank=d["R"], num_heads=d["heads"], qk_nope_dim=d["nope"],
                qk_rope_dim=d["rope"], v_head_dim=d["v"], rms_eps=1e-6, softmax_scale=(d["nope"] + d["rope"]) ** -0.5)
    return inp, dims


def test_block_dsv3_shape_matches_oracle(cuda_device):
    inp, dims = _dsv3_block(prev_len=1023, seed=7)
    with native.DeepSeekNativeSession(num_layers=1, hidden_dim=7168, num_experts=0, top_k=0) as session:
        out, (kv, pe) = native.ds_attention_block_forward(
            session, *_block_args(inp), previous_kv_cache=inp["previous_kv"], previous_pe_cache=inp["previous_pe"],
            rope_cos=inp["cos"], rope_sin=inp["sin"], **dims)
    torch.cuda.synchronize()
    want, (wkv, wpe) = omla.attention_block(*_block_args(inp), inp["previous_kv"], inp["previous_pe"], inp["cos"],
                                            inp["sin"], **dims)
    assert _rel(out, want) <= TOL
    assert torch.equal(kv[:-1].cpu(), inp["previous_kv"].cpu()) and torch.equal(pe[:-1].cpu(), inp["previous_pe"].cpu())
    assert _rel(kv[-1], wkv[-1]) <= TOL and _rel(pe[-1], wpe[-1]) <= TOL


def test_block_appends_in_place(cuda_device):
    """next_*_cache == previous_*_cache with room for one more row: the C entry
    point appends without copying and gives the out-of-place result."""
    prev = 300
    inp, dims = _dsv3_block(prev_len=prev, seed=11, H=1024, q_rank=256)
    with native.DeepSeekNativeSession(num_layers=1, hidden_dim=1024, num_experts=0, top_k=0) as s:
        out_ref, (kv_ref, pe_ref) = native.ds_attention_block_forward(
            s, *_block_args(inp), previous_kv_cache=inp["previous_kv"], previous_pe_cache=inp["previous_pe"],
            rope_cos=inp["cos"], rope_sin=inp["sin"], **dims)
    lib = native.load_library()
    d = DSV3
    kv_buf = torch.zeros((prev + 1, d["R"]), device="cuda")
    pe_buf = torch.zeros((prev + 1, d["rope"]), device="cuda")
    kv_buf[:prev] = inp["previous_kv"]
    pe_buf[:prev] = inp["previous_pe"]
    out = torch.empty(1024, device="cuda")
    ws = torch.empty(int(lib.moe_ds_attention_block_workspace_bytes(1024, 256, d["R"], d["heads"], d["nope"],
                                                                      d["rope"], d["v"], prev)),
                     dtype=torch.uint8, device="cuda")
    session = lib.moe_ds_session_create(1, 1024, 0, 0)
    p = native._ptr
    try:
        code = lib.moe_ds_attention_block_forward_f32(
            ctypes.c_void_p(session), *(p(t) for t in _block_args(inp)), p(kv_buf), p(pe_buf), p(inp["cos"]),
            p(inp["sin"]), p(kv_buf), p(pe_buf), p(out), 1024, 256, d["R"], d["heads"], d["nope"], d["rope"], d["v"],
            prev, 1e-6, dims["softmax_scale"], p(ws), ws.numel(), native._stream())
        assert code == 0
        assert lib.moe_ds_fused_attention_invocation_count(ctypes.c_void_p(session)) == 1
    finally:
        lib.moe_ds_session_destroy(ctypes.c_void_p(session))
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref) and torch.equal(kv_buf, kv_ref) and torch.equal(pe_buf, pe_ref)


def test_kill_switches(monkeypatch):
    monkeypatch.setenv("PCKETLM_DISABLE_FUSED_DS_ATTENTION", "1")
    assert native.native_fused_ds_attention_available() is False
    monkeypatch.setenv("PCKETLM_DISABLE_NATIVE_FLASH_MLA", "1")
    assert native.native_flash_mla_available() is False

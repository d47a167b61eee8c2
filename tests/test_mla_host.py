"""MLA attention on the host: the oracle restatement (oracle/mla.py) against
the reference's own outputs (tests/golden/mla.pt, made by the reference's
pcketlm.native.ds_attention_block_forward / ds_mla_attention_flash_forward)
and against the reference compiled from ds_forward.cpp (oracle/_ref); the
C entry points' argument checks, which return before any device work, with
the reference's codes (1 null pointer, 2 bad dimensions, 3 missing previous
cache); the Python wrappers' shape errors."""

import ctypes

import pytest
import torch

import oracle.mla as omla
import oracle.ref as oref
from pocketlm_b200 import native

BLOCK_TOL = 2e-6  # rel-L2, fp32 against fp32 (summation order only)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def _golden(golden_dir):
    return torch.load(golden_dir / "mla.pt", weights_only=False)


def test_oracle_matches_reference_golden(golden_dir):
    for tag, case in _golden(golden_dir).items():
        inp = case["inputs"]
        if case["kind"] == "block":
            out, (kv, pe) = omla.attention_block(inp["hidden"], inp["q_a"], inp["q_b"], inp["kv_a"], inp["kv_b"],
                                                 inp["o_w"], inp["q_norm"], inp["kv_norm"], inp["previous_kv"],
                                                 inp["previous_pe"], inp["cos"], inp["sin"], **case["dims"])
            assert _rel(out, case["out"]) <= BLOCK_TOL, tag
            assert torch.allclose(kv, case["next_kv"], atol=1e-6, rtol=1e-6), tag
            assert torch.allclose(pe, case["next_pe"], atol=1e-6, rtol=1e-6), tag
        else:
            out = omla.mla_attention_flash(inp["q_nope"], inp["q_pe"], inp["kv_cache"], inp["pe_cache"],
                                           inp["wkv_b"], case["softmax_scale"])
            assert _rel(out, case["out"]) <= BLOCK_TOL, tag


@pytest.mark.skipif(not oref.available(), reason="reference build (oracle/_ref) missing")
@pytest.mark.parametrize("heads,L,nope,rope,R,v", [(8, 300, 128, 64, 512, 128), (20, 77, 16, 8, 40, 12),
                                                   (5, 4, 6, 5, 12, 3)])
def test_oracle_core_matches_compiled_reference(heads, L, nope, rope, R, v):
    g = torch.Generator().manual_seed(heads * 1000 + L)
    qn, qp = torch.randn((heads, nope), generator=g), torch.randn((heads, rope), generator=g)
    kv, pe = torch.randn((L, R), generator=g) * 0.5, torch.randn((L, rope), generator=g) * 0.5
    w = torch.randn((heads, nope + v, R), generator=g) * 0.1
    want = oref.mla_attention_flash(qn, qp, kv, pe, w, 0.3)
    assert _rel(omla.mla_attention_flash(qn, qp, kv, pe, w, 0.3), want) <= BLOCK_TOL


# --- C entry points: argument checks (no device work happens before them) ---

def _lib():
    try:
        return native.load_library()
    except Exception as exc:  # pragma: no cover - the library is built by the suite's build step
        pytest.skip(f"library not loadable: {exc}")


FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: every call below returns from its checks


def test_flash_entry_argument_codes():
    lib = _lib()
    f = lib.moe_mla_attention_flash_forward
    args = [FAKE] * 6 + [4, 10, 8, 4, 16, 8, 0.5, None, 0, None]
    assert f(*([None] + args[1:])) == 1
    bad = list(args)
    bad[7] = 0  # cache_len
    assert f(*bad) == 2
    bad = list(args)
    bad[9] = -1  # qk_rope_dim
    assert f(*bad) == 2
    big = list(args)
    big[10] = 2048  # kv_lora_rank beyond the kernels' 1024
    assert f(*big) == -5
    assert lib.moe_mla_attention_workspace_bytes(4, 10, 8, 4, 2048, 8) == -1
    assert lib.moe_mla_attention_workspace_bytes(128, 4096, 128, 64, 512, 128) > 128 * 512 * 4


def test_block_entry_argument_codes():
    lib = _lib()
    session = lib.moe_ds_session_create(1, 16, 0, 0)
    assert session
    try:
        f = lib.moe_ds_attention_block_forward_f32
        ptrs = [FAKE] * 9 + [None, None] + [FAKE] * 5  # previous caches null
        dims = [16, 6, 5, 4, 3, 4, 2, 0]
        tail = [1e-6, 0.25, None, 0, None]
        assert f(None, *ptrs[1:], *dims, *tail) == 1
        no_cos = list(ptrs)
        no_cos[11] = None
        assert f(ctypes.c_void_p(session), *no_cos[1:], *dims, *tail) == 1
        bad = list(dims)
        bad[6] = 0  # v_head_dim
        assert f(ctypes.c_void_p(session), *ptrs[1:], *bad, *tail) == 2
        prev = list(dims)
        prev[7] = 3  # previous_len without previous caches
        assert f(ctypes.c_void_p(session), *ptrs[1:], *prev, *tail) == 3
        # next caches partly overlapping the previous ones (not equal): rejected before any device work
        over = list(ptrs)
        over[9], over[10] = FAKE, FAKE  # previous caches
        over[13], over[14] = ctypes.c_void_p(0x1000 + 4), ctypes.c_void_p(0x1000 + 4)  # next = previous + 1 float
        assert f(ctypes.c_void_p(session), *over[1:], *prev, *tail) == -2
        huge = list(dims)
        huge[7] = 2 ** 31  # cache length beyond the kernels' 32-bit step counts
        assert f(ctypes.c_void_p(session), *over[1:9], FAKE, FAKE, *over[11:], *huge, *tail) == -5
        assert lib.moe_ds_attention_invocation_count(ctypes.c_void_p(session)) == 0
        assert lib.moe_ds_fused_attention_invocation_count(ctypes.c_void_p(session)) == 0
        assert lib.moe_ds_attention_invocation_count(None) == -1
        assert lib.moe_ds_attention_block_workspace_bytes(16, 6, 5, 4, 3, 4, 2, -1) == -1
    finally:
        lib.moe_ds_session_destroy(ctypes.c_void_p(session))


def test_wrapper_shape_errors():
    heads, nope, rope, R, v, L = 4, 3, 4, 5, 2, 6
    qn, qp = torch.zeros(heads, nope), torch.zeros(heads, rope)
    kv, pe, w = torch.zeros(L, R), torch.zeros(L, rope), torch.zeros(heads, nope + v, R)
    with pytest.raises(ValueError, match="head count mismatch"):
        native.ds_mla_attention_flash_forward(qn, torch.zeros(heads + 1, rope), kv, pe, w, softmax_scale=1.0)
    with pytest.raises(ValueError, match="pe_cache shape mismatch"):
        native.ds_mla_attention_flash_forward(qn, qp, kv, torch.zeros(L + 1, rope), w, softmax_scale=1.0)
    with pytest.raises(ValueError, match="wkv_b shape mismatch"):
        native.ds_mla_attention_flash_forward(qn, qp, kv, pe, torch.zeros(heads, nope, R), softmax_scale=1.0)
    H, qr = 16, 6
    kw = dict(previous_kv_cache=None, previous_pe_cache=None, rope_cos=torch.zeros(rope // 2),
              rope_sin=torch.zeros(rope // 2), q_lora_rank=qr, kv_lora_rank=R, num_heads=heads, qk_nope_dim=nope,
              qk_rope_dim=rope, v_head_dim=v, rms_eps=1e-6, softmax_scale=0.25)
    ws = [torch.zeros(qr, H), torch.zeros(heads * (nope + rope), qr), torch.zeros(R + rope, H),
          torch.zeros(heads * (nope + v), R), torch.zeros(H, heads * v), torch.ones(qr), torch.ones(R)]
    with pytest.raises(ValueError, match=r"q_a_weight must be \[q_lora_rank, hidden_dim\]"):
        native.ds_attention_block_forward(None, torch.zeros(H + 1), *ws, **kw)
    bad = dict(kw, rope_cos=torch.zeros(rope))
    with pytest.raises(ValueError, match="rope cos/sin sizes"):
        native.ds_attention_block_forward(None, torch.zeros(H), *ws, **bad)
    bad = dict(kw, previous_kv_cache=torch.zeros(3, R), previous_pe_cache=torch.zeros(2, rope))
    with pytest.raises(ValueError, match="previous KV and PE cache lengths must match"):
        native.ds_attention_block_forward(None, torch.zeros(H), *ws, **bad)


@pytest.mark.skipif(not oref.available(), reason="reference build (oracle/_ref) missing")
@pytest.mark.parametrize("H,qr,R,heads,nope,rope,v,prev", [(64, 16, 16, 4, 8, 8, 8, 32), (256, 96, 64, 6, 16, 8, 16, 0),
                                                           (128, 32, 24, 5, 8, 6, 8, 10), (96, 24, 20, 3, 4, 5, 6, 7)])
def test_oracle_block_matches_compiled_reference(H, qr, R, heads, nope, rope, v, prev):
    """The block restatement against ds_attention_block_forward_f32 compiled from the reference's source,
    an odd rope width (no rotation, as the reference) included."""
    g = torch.Generator().manual_seed(H + prev)

    def rnd(*shape, scale=1.0):
        return torch.randn(shape, generator=g) * scale

    args = (rnd(H), rnd(qr, H, scale=0.05), rnd(heads * (nope + rope), qr, scale=0.05), rnd(R + rope, H, scale=0.05),
            rnd(heads * (nope + v), R, scale=0.05), rnd(H, heads * v, scale=0.05), 1 + 0.1 * rnd(qr), 1 + 0.1 * rnd(R),
            rnd(prev, R, scale=0.5) if prev else None, rnd(prev, rope, scale=0.5) if prev else None)
    angles = torch.arange(rope // 2, dtype=torch.float32) * 0.37
    kw = dict(q_lora_rank=qr, kv_lora_rank=R, num_heads=heads, qk_nope_dim=nope, qk_rope_dim=rope, v_head_dim=v,
              rms_eps=1e-6, softmax_scale=0.2)
    out, (kv, pe) = omla.attention_block(*args, angles.cos(), angles.sin(), **kw)
    want, (wkv, wpe) = oref.attention_block(*args, angles.cos(), angles.sin(), **kw)
    assert _rel(out, want) <= BLOCK_TOL
    assert torch.allclose(kv, wkv, atol=1e-6, rtol=1e-6) and torch.allclose(pe, wpe, atol=1e-6, rtol=1e-6)

"""ctypes access to the reference's own CPU kernels, compiled from its sources
into oracle/_ref/ by `make -C oracle ref` -- TEST INFRASTRUCTURE ONLY.

Two uses: tests/test_oracle_vs_reference.py checks the C restatement against
these (bit for bit where the reference's operation order allows), and
bench.py's cpu_baseline / `--impl reference` legs time them on the host cores.
The call signatures are the reference's C ABI, as bound by
src/pcketlm/native/__init__.py.
"""

from __future__ import annotations

import ctypes
import json
import os
import subprocess
from pathlib import Path

import torch

from .kernels import _I64, _INT, _P, _Tables, _check, _f32, _ptr, _rows, _u8

REF_DIR = Path(__file__).resolve().parent / "_ref"
_LIBS: dict[str, ctypes.CDLL] = {}


def reference_root() -> Path | None:
    """The reference checkout: $PCKETLM_REFERENCE_ROOT, else BASELINE.json's
    `reference_path`; None when neither names an existing directory (a
    machine without the reference tree)."""
    text = os.environ.get("PCKETLM_REFERENCE_ROOT", "").strip()
    if not text:
        baseline = REF_DIR.parent.parent / "BASELINE.json"
        try:
            text = str(json.loads(baseline.read_text()).get("reference_path") or "")
        except (OSError, ValueError):
            text = ""
    return Path(text) if text and Path(text).is_dir() else None


def reference_sources() -> Path | None:
    root = reference_root()
    src = None if root is None else root / "src" / "pcketlm" / "native"
    return src if src is not None and src.is_dir() else None


def build() -> bool:
    """Compile the reference libraries when the reference tree is present.

    Returns True when oracle/_ref/ holds a usable build afterwards.  On a
    machine without the reference tree (the GPU box) the prebuilt files that
    travelled with the repository are used as they are.
    """
    src = reference_sources()
    if src is not None:
        subprocess.run(["make", "-s", "-C", str(REF_DIR.parent), "ref", f"REF={src}"], check=True)
    return available()


def available() -> bool:
    return (REF_DIR / "fp8_linear.so").exists()


def lib(name: str) -> ctypes.CDLL:
    if name not in _LIBS:
        path = REF_DIR / f"{name}.so"
        if not path.exists():
            raise FileNotFoundError(f"reference build missing: {path} (run `make -C oracle ref`)")
        handle = ctypes.CDLL(str(path))
        _LIBS[name] = handle
    return _LIBS[name]


def threads() -> int:
    return len(os.sched_getaffinity(0))


def fp8_linear(w, s, x):
    w, s, x = _u8(w), _f32(s), _rows(x)
    out = torch.empty((x.shape[0], w.shape[0]), dtype=torch.float32)
    f = lib("fp8_linear").fp8_e4m3_block_linear_f32
    f.restype = _INT
    _check(f(_ptr(w), _ptr(s), _ptr(x), _ptr(out), _I64(x.shape[0]), _I64(w.shape[0]),
             _I64(w.shape[1]), _I64(s.shape[1])), "ref fp8_linear")
    return out


def fp8_mlp(gate, gate_s, up, up_s, down, down_s, x, *, avx512: bool = False):
    gate, up, down = _u8(gate), _u8(up), _u8(down)
    gate_s, up_s, down_s, x = _f32(gate_s), _f32(up_s), _f32(down_s), _rows(x)
    inter, hidden = int(gate.shape[0]), int(gate.shape[1])
    out = torch.empty((x.shape[0], hidden), dtype=torch.float32)
    if avx512:
        f = lib("fp8_linear_avx512").fp8_e4m3_block_mlp_avx512_f32
    else:
        f = lib("fp8_linear").fp8_e4m3_block_mlp_f32
    f.restype = _INT
    _check(f(_ptr(gate), _ptr(gate_s), _ptr(up), _ptr(up_s), _ptr(down), _ptr(down_s), _ptr(x),
             _ptr(out), _I64(x.shape[0]), _I64(inter), _I64(hidden), _I64(gate_s.shape[1]),
             _I64(down_s.shape[1])), "ref fp8_mlp")
    return out


def fp8_mlp_many(items, x):
    t, x = _Tables(items), _rows(x)
    out = torch.zeros((len(items), x.shape[0], t.hidden), dtype=torch.float32)
    f = lib("fp8_linear").fp8_e4m3_block_mlp_many_f32
    f.restype = _INT
    _check(f(*t.args(), _ptr(x), _ptr(out), _I64(len(items)), _I64(x.shape[0]), _I64(t.inter),
             _I64(t.hidden), _I64(t.gsc), _I64(t.dsc)), "ref fp8_mlp_many")
    return out


def fp8_mlp_many_weighted(items, x, route, *, avx512: bool = False):
    t, x, route = _Tables(items), _rows(x), _f32(route.reshape(-1))
    out = torch.empty((x.shape[0], t.hidden), dtype=torch.float32)
    if avx512:
        f = lib("fp8_linear_avx512").fp8_e4m3_block_mlp_many_weighted_avx512_f32
    else:
        f = lib("fp8_linear").fp8_e4m3_block_mlp_many_weighted_f32
    f.restype = _INT
    _check(f(*t.args(), _ptr(x), _ptr(route), _ptr(out), _I64(len(items)), _I64(x.shape[0]),
             _I64(t.inter), _I64(t.hidden), _I64(t.gsc), _I64(t.dsc)), "ref fp8_mlp_many_weighted")
    return out


def fp8_mlp_many_row_weighted(items, x, route):
    t, x, route = _Tables(items), _rows(x), _f32(route)
    out = torch.empty((x.shape[0], t.hidden), dtype=torch.float32)
    f = lib("fp8_linear").fp8_e4m3_block_mlp_many_row_weighted_f32
    f.restype = _INT
    _check(f(*t.args(), _ptr(x), _ptr(route), _ptr(out), _I64(len(items)), _I64(x.shape[0]),
             _I64(t.inter), _I64(t.hidden), _I64(t.gsc), _I64(t.dsc)), "ref fp8_mlp_many_row_weighted")
    return out


def fp8_mlp_many_pair_weighted(items, x, pair_items, pair_rows, pair_weights):
    t, x = _Tables(items), _rows(x)
    pi = pair_items.detach().cpu().contiguous().reshape(-1).to(torch.int64)
    pr = pair_rows.detach().cpu().contiguous().reshape(-1).to(torch.int64)
    pw = _f32(pair_weights.reshape(-1))
    out = torch.empty((x.shape[0], t.hidden), dtype=torch.float32)
    f = lib("fp8_linear").fp8_e4m3_block_mlp_many_pair_weighted_f32
    f.restype = _INT
    _check(f(*t.args(), _ptr(x), _ptr(pi), _ptr(pr), _ptr(pw), _ptr(out), _I64(len(items)),
             _I64(pi.numel()), _I64(x.shape[0]), _I64(t.inter), _I64(t.hidden), _I64(t.gsc),
             _I64(t.dsc)), "ref fp8_mlp_many_pair_weighted")
    return out


def fp8_dequant(w, s, dtype):
    w, s = _u8(w), _f32(s)
    rows, cols = int(w.shape[0]), int(w.shape[1])
    out = torch.empty((rows, cols), dtype=torch.int16)
    name = "fp8_e4m3_dequant_to_bf16" if dtype == torch.bfloat16 else "fp8_e4m3_dequant_to_fp16"
    f = getattr(lib("fp8_dequant"), name)
    f.restype = _INT
    _check(f(_ptr(w), _ptr(s), _ptr(out), _I64(rows), _I64(cols), _I64(s.shape[1])), "ref dequant")
    return out.view(dtype)


def q4_dequant_to_fp16(packed, scales, channels: int, channel_size: int):
    packed = packed.detach().cpu().contiguous().to(torch.uint8)
    scales = scales.detach().cpu().contiguous().to(torch.float16)
    out = torch.empty((channels * channel_size,), dtype=torch.float16)
    f = lib("q4_dequant").q4_dequant_to_fp16
    f.restype = None
    f(_ptr(packed), _ptr(scales), _ptr(out), _I64(channels), _I64(channel_size))
    return out


def q4_moe_selected_forward(hidden, experts, route, hidden_size: int, intermediate_size: int):
    x = hidden.detach().cpu().contiguous().reshape(-1).to(torch.float16)
    r = _f32(route.reshape(-1))
    keep = []
    arrays = [(ctypes.c_void_p * len(experts))() for _ in range(6)]
    for i, item in enumerate(experts):
        conv = [t.detach().cpu().contiguous().to(torch.uint8 if j % 2 == 0 else torch.float16)
                for j, t in enumerate(item)]
        keep.append(conv)
        for j, t in enumerate(conv):
            arrays[j][i] = ctypes.c_void_p(int(t.data_ptr()))
    out = torch.empty((hidden_size,), dtype=torch.float16)
    f = lib("q4_dequant").q4_moe_selected_forward_u16
    f.restype = _INT
    _check(f(_ptr(x), *arrays, _ptr(r), _ptr(out), _I64(hidden_size), _I64(intermediate_size),
             _I64(len(experts))), "ref q4_moe_selected_forward")
    return out


def pack_rows8(weight):
    w = weight.detach().cpu().contiguous()
    rows, cols = int(w.shape[0]), int(w.shape[1])
    out = torch.empty((((rows + 7) // 8) * cols * 8,), dtype=torch.int16)
    f = lib("fp16_packed_gemv").native_pack_u16_rows8
    f.restype = _INT
    _check(f(_ptr(w), _ptr(out), _I64(rows), _I64(cols)), "ref pack_rows8")
    return out


def packed_gemv_rows8(hidden, packed, rows: int, cols: int):
    x = hidden.detach().cpu().contiguous().reshape(-1)
    p = packed.detach().cpu().contiguous()
    out = torch.empty((rows,), dtype=torch.float32)
    f = lib("fp16_packed_gemv").native_packed_gemv_rows8
    f.restype = _INT
    _check(f(_ptr(x), _ptr(p), _ptr(out), _I64(rows), _I64(cols),
             _INT(1 if x.dtype == torch.bfloat16 else 0)), "ref packed_gemv_rows8")
    return out


def moe_selected_forward_u16(hidden, gate, up, down, route):
    x = hidden.detach().cpu().contiguous()
    g, u, d = (t.detach().cpu().contiguous() for t in (gate, up, down))
    r = _f32(route)
    out = torch.empty(tuple(x.shape), dtype=hidden.dtype)
    f = lib("fp16_moe").native_moe_selected_forward_u16
    f.restype = _INT
    _check(f(_ptr(x), _ptr(g), _ptr(u), _ptr(d), _ptr(r), _ptr(out), _I64(x.shape[0]),
             _I64(x.shape[1]), _I64(g.shape[0]), _I64(g.shape[1]),
             _INT(1 if x.dtype == torch.bfloat16 else 0)), "ref moe_selected_forward_u16")
    return out


def router_softmax_topk_u16(hidden, router_weights, k: int):
    x = hidden.detach().cpu().contiguous().reshape(-1)
    if x.dtype not in (torch.float16, torch.bfloat16):
        x = x.to(torch.float16)
    w = router_weights.detach().cpu().contiguous().to(x.dtype)
    ids = torch.empty((k,), dtype=torch.int64)
    weights = torch.empty((k,), dtype=torch.float32)
    f = lib("ds_forward").ds_router_topk_u16
    f.restype = _INT
    _check(f(_ptr(x), _ptr(w), _I64(w.shape[1]), _I64(w.shape[0]), _I64(k),
             _I64(1 if x.dtype == torch.bfloat16 else 0), _ptr(ids), _ptr(weights)), "ref router")
    return ids, weights


def mla_attention_flash(q_nope, q_pe, kv_cache, pe_cache, wkv_b, softmax_scale: float):
    """ds_mla_attention_flash_forward (ds_forward.cpp:517) on the host cores."""
    qn, qp = q_nope.detach().cpu().contiguous().float(), q_pe.detach().cpu().contiguous().float()
    kv, pe = kv_cache.detach().cpu().contiguous().float(), pe_cache.detach().cpu().contiguous().float()
    w = wkv_b.detach().cpu().contiguous().float()
    heads, nope, rope = qn.shape[0], qn.shape[1], qp.shape[1]
    v_dim = w.shape[1] - nope
    out = torch.empty((heads, v_dim), dtype=torch.float32)
    f = lib("ds_forward").ds_mla_attention_flash_forward
    f.restype = _INT
    _check(f(_ptr(qn), _ptr(qp), _ptr(kv), _ptr(pe), _ptr(w), _ptr(out), _I64(heads), _I64(kv.shape[0]),
             _I64(nope), _I64(rope), _I64(kv.shape[1]), _I64(v_dim), ctypes.c_float(softmax_scale)),
           "ref mla attention")
    return out


def attention_block(hidden, q_a, q_b, kv_a, kv_b, o_w, q_norm, kv_norm, previous_kv, previous_pe, cos, sin, *,
                    q_lora_rank: int, kv_lora_rank: int, num_heads: int, qk_nope_dim: int, qk_rope_dim: int,
                    v_head_dim: int, rms_eps: float, softmax_scale: float):
    """ds_attention_block_forward_f32 (ds_forward.cpp:647) on the host cores,
    through a session of its own -> (hidden_out, (next_kv, next_pe))."""
    def f32(t):
        return t.detach().cpu().contiguous().reshape(-1).float()

    x = f32(hidden)
    H = x.numel()
    prev_len = 0 if previous_kv is None else previous_kv.numel() // kv_lora_rank
    next_kv = torch.empty((prev_len + 1, kv_lora_rank), dtype=torch.float32)
    next_pe = torch.empty((prev_len + 1, qk_rope_dim), dtype=torch.float32)
    out = torch.empty((H,), dtype=torch.float32)
    args = [f32(t) for t in (q_a, q_b, kv_a, kv_b, o_w, q_norm, kv_norm)]
    pk = f32(previous_kv) if prev_len else None
    pp = f32(previous_pe) if prev_len else None
    c, s = f32(cos), f32(sin)
    L = lib("ds_forward")
    L.ds_session_create.restype = _P
    L.ds_session_create.argtypes = [_I64, _I64, _I64, _I64, _P, _P]
    L.ds_session_destroy.argtypes = [_P]
    handle = L.ds_session_create(1, H, 0, 0, None, None)
    try:
        f = L.ds_attention_block_forward_f32
        f.restype = _INT
        _check(f(_P(handle), _ptr(x), *(_ptr(a) for a in args), _ptr(pk) if pk is not None else _P(0),
                 _ptr(pp) if pp is not None else _P(0), _ptr(c), _ptr(s),
                 _ptr(next_kv), _ptr(next_pe), _ptr(out), _I64(H), _I64(q_lora_rank), _I64(kv_lora_rank),
                 _I64(num_heads), _I64(qk_nope_dim), _I64(qk_rope_dim), _I64(v_head_dim), _I64(prev_len),
                 ctypes.c_float(rms_eps), ctypes.c_float(softmax_scale)), "ref attention block")
    finally:
        L.ds_session_destroy(_P(handle))
    return out, (next_kv, next_pe)

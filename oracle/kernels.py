"""ctypes wrappers over oracle/liboracle.so (the C restatement in moe_oracle.c).

TEST INFRASTRUCTURE ONLY -- see oracle/__init__.py.  Inputs and outputs are
CPU torch tensors; every wrapper mirrors the argument checks of the reference
bridge it stands in for (src/pcketlm/native/__init__.py) closely enough for
the tests, and raises RuntimeError on a nonzero return code.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_LIB: ctypes.CDLL | None = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int


def build() -> Path:
    """Compile liboracle.so (gcc, OpenMP) if it is missing or stale."""
    src = _HERE / "moe_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE), "all"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        build()
        handle = ctypes.CDLL(str(_LIB_PATH))
        for name in (
            "orc_fp8_linear_f32", "orc_fp8_dual_linear_f32", "orc_fp8_mlp_f32",
            "orc_fp8_mlp_many_f32", "orc_fp8_mlp_many_weighted_f32",
            "orc_fp8_mlp_many_row_weighted_f32", "orc_fp8_mlp_many_pair_weighted_f32",
            "orc_fp8_dequant", "orc_q4_dequant_to_fp16", "orc_q4_moe_selected_forward",
            "orc_pack_rows8", "orc_packed_gemv_rows8", "orc_moe_selected_forward_u16",
            "orc_router_softmax_topk_u16", "orc_combine_f32",
        ):
            getattr(handle, name).restype = _INT
        _LIB = handle
    return _LIB


def _ptr(t: torch.Tensor) -> _P:
    return _P(int(t.data_ptr()))


def _check(code: int, name: str) -> None:
    if code != 0:
        raise RuntimeError(f"oracle {name} failed with code {code}")


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().contiguous().to(torch.float32)


def _u8(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    return t.to(torch.uint8)


def _rows(hidden: torch.Tensor) -> torch.Tensor:
    return _f32(hidden.reshape(-1, int(hidden.shape[-1])))


def fp8_linear(w: torch.Tensor, s: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """fp8_e4m3_block_linear_f32 (fp8_linear.cpp:50-117)."""
    w, s, x = _u8(w), _f32(s), _rows(x)
    out = torch.empty((x.shape[0], w.shape[0]), dtype=torch.float32)
    code = lib().orc_fp8_linear_f32(_ptr(w), _ptr(s), _ptr(x), _ptr(out), _I64(x.shape[0]),
                                    _I64(w.shape[0]), _I64(w.shape[1]), _I64(s.shape[1]))
    _check(code, "fp8_linear")
    return out


def fp8_mlp(gate, gate_s, up, up_s, down, down_s, x: torch.Tensor) -> torch.Tensor:
    """fp8_e4m3_block_mlp_f32 (fp8_linear.cpp:212-362)."""
    gate, up, down = _u8(gate), _u8(up), _u8(down)
    gate_s, up_s, down_s, x = _f32(gate_s), _f32(up_s), _f32(down_s), _rows(x)
    inter, hidden = int(gate.shape[0]), int(gate.shape[1])
    out = torch.empty((x.shape[0], hidden), dtype=torch.float32)
    code = lib().orc_fp8_mlp_f32(_ptr(gate), _ptr(gate_s), _ptr(up), _ptr(up_s), _ptr(down),
                                 _ptr(down_s), _ptr(x), _ptr(out), _I64(x.shape[0]), _I64(inter),
                                 _I64(hidden), _I64(gate_s.shape[1]), _I64(down_s.shape[1]))
    _check(code, "fp8_mlp")
    return out


class _Tables:
    """uint64 host-pointer tables for a list of 6-tuples (gate, gs, up, us, down, ds)."""

    def __init__(self, items):
        self.keep = []
        cols = [[], [], [], [], [], []]
        for item in items:
            conv = (_u8(item[0]), _f32(item[1]), _u8(item[2]), _f32(item[3]), _u8(item[4]), _f32(item[5]))
            self.keep.append(conv)
            for j, t in enumerate(conv):
                cols[j].append(int(t.data_ptr()))
        self.tables = [torch.tensor(c, dtype=torch.int64) for c in cols]
        first = self.keep[0]
        self.inter, self.hidden = int(first[0].shape[0]), int(first[0].shape[1])
        self.gsc, self.dsc = int(first[1].shape[1]), int(first[5].shape[1])

    def args(self):
        return [_ptr(t) for t in self.tables]


def fp8_mlp_many(items, x: torch.Tensor) -> torch.Tensor:
    """fp8_e4m3_block_mlp_many_f32 (fp8_linear.cpp:364-473) -> [E, B, H]."""
    t, x = _Tables(items), _rows(x)
    out = torch.zeros((len(items), x.shape[0], t.hidden), dtype=torch.float32)
    code = lib().orc_fp8_mlp_many_f32(*t.args(), _ptr(x), _ptr(out), _I64(len(items)),
                                      _I64(x.shape[0]), _I64(t.inter), _I64(t.hidden),
                                      _I64(t.gsc), _I64(t.dsc))
    _check(code, "fp8_mlp_many")
    return out


def fp8_mlp_many_weighted(items, x: torch.Tensor, route: torch.Tensor) -> torch.Tensor:
    """fp8_e4m3_block_mlp_many_weighted_f32 (fp8_linear.cpp:475-589)."""
    t, x, route = _Tables(items), _rows(x), _f32(route.reshape(-1))
    out = torch.empty((x.shape[0], t.hidden), dtype=torch.float32)
    code = lib().orc_fp8_mlp_many_weighted_f32(*t.args(), _ptr(x), _ptr(route), _ptr(out),
                                               _I64(len(items)), _I64(x.shape[0]), _I64(t.inter),
                                               _I64(t.hidden), _I64(t.gsc), _I64(t.dsc))
    _check(code, "fp8_mlp_many_weighted")
    return out


def fp8_mlp_many_row_weighted(items, x: torch.Tensor, route: torch.Tensor) -> torch.Tensor:
    """fp8_e4m3_block_mlp_many_row_weighted_f32 (fp8_linear.cpp:591-831); route [E, B]."""
    t, x, route = _Tables(items), _rows(x), _f32(route)
    out = torch.empty((x.shape[0], t.hidden), dtype=torch.float32)
    code = lib().orc_fp8_mlp_many_row_weighted_f32(*t.args(), _ptr(x), _ptr(route), _ptr(out),
                                                   _I64(len(items)), _I64(x.shape[0]),
                                                   _I64(t.inter), _I64(t.hidden), _I64(t.gsc),
                                                   _I64(t.dsc))
    _check(code, "fp8_mlp_many_row_weighted")
    return out


def fp8_mlp_many_pair_weighted(items, x, pair_items, pair_rows, pair_weights) -> torch.Tensor:
    """fp8_e4m3_block_mlp_many_pair_weighted_f32 (fp8_linear.cpp:833-980)."""
    t, x = _Tables(items), _rows(x)
    pi = pair_items.detach().cpu().contiguous().reshape(-1).to(torch.int64)
    pr = pair_rows.detach().cpu().contiguous().reshape(-1).to(torch.int64)
    pw = _f32(pair_weights.reshape(-1))
    out = torch.empty((x.shape[0], t.hidden), dtype=torch.float32)
    code = lib().orc_fp8_mlp_many_pair_weighted_f32(*t.args(), _ptr(x), _ptr(pi), _ptr(pr),
                                                    _ptr(pw), _ptr(out), _I64(len(items)),
                                                    _I64(pi.numel()), _I64(x.shape[0]),
                                                    _I64(t.inter), _I64(t.hidden), _I64(t.gsc),
                                                    _I64(t.dsc))
    _check(code, "fp8_mlp_many_pair_weighted")
    return out


def fp8_dequant(w: torch.Tensor, s: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp8_e4m3_dequant_to_fp16 / _bf16 (fp8_dequant.cpp:119-204)."""
    w, s = _u8(w), _f32(s)
    rows, cols = int(w.shape[0]), int(w.shape[1])
    out = torch.empty((rows, cols), dtype=torch.int16)
    code = lib().orc_fp8_dequant(_ptr(w), _ptr(s), _ptr(out), _I64(rows), _I64(cols),
                                 _I64(s.shape[1]), _INT(1 if dtype == torch.bfloat16 else 0))
    _check(code, "fp8_dequant")
    return out.view(dtype)


def q4_dequant_to_fp16(packed: torch.Tensor, scales: torch.Tensor, channels: int, channel_size: int):
    """q4_dequant_to_fp16 (q4_dequant.cpp:154-208) -> flat fp16."""
    packed = packed.detach().cpu().contiguous().to(torch.uint8)
    scales = scales.detach().cpu().contiguous().to(torch.float16)
    out = torch.empty((channels * channel_size,), dtype=torch.float16)
    code = lib().orc_q4_dequant_to_fp16(_ptr(packed), _ptr(scales), _ptr(out), _I64(channels),
                                        _I64(channel_size))
    _check(code, "q4_dequant_to_fp16")
    return out


def q4_moe_selected_forward(hidden, experts, route, hidden_size: int, intermediate_size: int):
    """q4_moe_selected_forward_u16 (q4_dequant.cpp:357-476) -> fp16 [H]."""
    x = hidden.detach().cpu().contiguous().reshape(-1).to(torch.float16)
    r = _f32(route.reshape(-1))
    keep, cols = [], [[], [], [], [], [], []]
    for item in experts:
        conv = [t.detach().cpu().contiguous().to(torch.uint8 if j % 2 == 0 else torch.float16)
                for j, t in enumerate(item)]
        keep.append(conv)
        for j, t in enumerate(conv):
            cols[j].append(int(t.data_ptr()))
    tables = [torch.tensor(c, dtype=torch.int64) for c in cols]
    out = torch.empty((hidden_size,), dtype=torch.float16)
    code = lib().orc_q4_moe_selected_forward(_ptr(x), *[_ptr(t) for t in tables], _ptr(r), _ptr(out),
                                             _I64(hidden_size), _I64(intermediate_size),
                                             _I64(len(experts)))
    _check(code, "q4_moe_selected_forward")
    return out


def pack_rows8(weight: torch.Tensor) -> torch.Tensor:
    """native_pack_u16_rows8 (fp16_packed_gemv.cpp:52-77) -> flat uint16 storage (int16 view)."""
    w = weight.detach().cpu().contiguous()
    rows, cols = int(w.shape[0]), int(w.shape[1])
    out = torch.empty((((rows + 7) // 8) * cols * 8,), dtype=torch.int16)
    code = lib().orc_pack_rows8(_ptr(w), _ptr(out), _I64(rows), _I64(cols))
    _check(code, "pack_rows8")
    return out


def packed_gemv_rows8(hidden: torch.Tensor, packed: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """native_packed_gemv_rows8 (fp16_packed_gemv.cpp:79-116) -> f32 [rows]."""
    x = hidden.detach().cpu().contiguous().reshape(-1)
    code_dtype = 1 if x.dtype == torch.bfloat16 else 0
    p = packed.detach().cpu().contiguous()
    out = torch.empty((rows,), dtype=torch.float32)
    code = lib().orc_packed_gemv_rows8(_ptr(x), _ptr(p), _ptr(out), _I64(rows), _I64(cols),
                                       _INT(code_dtype))
    _check(code, "packed_gemv_rows8")
    return out


def moe_selected_forward_u16(hidden, gate, up, down, route) -> torch.Tensor:
    """native_moe_selected_forward_u16 (fp16_moe.cpp:199-267)."""
    dtype_code = 1 if hidden.dtype == torch.bfloat16 else 0
    x = hidden.detach().cpu().contiguous()
    g, u, d = (t.detach().cpu().contiguous() for t in (gate, up, down))
    r = _f32(route)
    seq, hid = int(x.shape[0]), int(x.shape[1])
    sel, inter = int(g.shape[0]), int(g.shape[1])
    out = torch.empty((seq, hid), dtype=hidden.dtype)
    code = lib().orc_moe_selected_forward_u16(_ptr(x), _ptr(g), _ptr(u), _ptr(d), _ptr(r), _ptr(out),
                                              _I64(seq), _I64(hid), _I64(sel), _I64(inter),
                                              _INT(dtype_code))
    _check(code, "moe_selected_forward_u16")
    return out


def router_softmax_topk_u16(hidden: torch.Tensor, router_weights: torch.Tensor, k: int):
    """ds_router_topk_u16 (ds_forward.cpp:879-955) for one token."""
    x = hidden.detach().cpu().contiguous().reshape(-1)
    if x.dtype not in (torch.float16, torch.bfloat16):
        x = x.to(torch.float16)
    w = router_weights.detach().cpu().contiguous().to(x.dtype)
    ids = torch.empty((k,), dtype=torch.int64)
    weights = torch.empty((k,), dtype=torch.float32)
    code = lib().orc_router_softmax_topk_u16(_ptr(x), _ptr(w), _I64(w.shape[1]), _I64(w.shape[0]),
                                             _I64(k), _INT(1 if x.dtype == torch.bfloat16 else 0),
                                             _ptr(ids), _ptr(weights))
    _check(code, "router_softmax_topk_u16")
    return ids, weights


def combine_f32(expert_outputs: torch.Tensor, route: torch.Tensor) -> torch.Tensor:
    """ds_moe_layer_forward_f32 combine (ds_forward.cpp:337-367)."""
    y = _f32(expert_outputs)
    if y.ndim == 2:
        y = y.unsqueeze(1)
    r = _f32(route.reshape(-1))
    out = torch.empty((y.shape[1], y.shape[2]), dtype=torch.float32)
    code = lib().orc_combine_f32(_ptr(y), _ptr(r), _I64(y.shape[0]), _I64(y.shape[1]),
                                 _I64(y.shape[2]), _ptr(out))
    _check(code, "combine_f32")
    return out

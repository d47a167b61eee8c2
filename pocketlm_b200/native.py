"""Drop-in replacement for the MoE entry points of PocketLM's native bridge.

Mirrors src/pcketlm/native/__init__.py of the reference: the same function
names, positional/keyword signatures, return dtypes and shapes, the same
ValueError messages for shape checks and RuntimeError on a nonzero return
code.  The computation always runs on the GPU through libmoe_b200.so
(include/moe_b200.h); there is no CPU path.  Inputs may live on the CPU (as
the reference's callers pass them) or on the GPU: CPU inputs are copied to
the current CUDA device and the result comes back on the device of `hidden`
(or of the weights for the dequant calls).

Kill switches: the reference's PCKETLM_DISABLE_NATIVE_* variables
(native/__init__.py:64-138) still mark an entry point unavailable, and a call
to it then raises RuntimeError -- it never silently computes elsewhere.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
_LIB_PATH = _PKG / "libmoe_b200.so"
_LIB: ctypes.CDLL | None = None
_LIB_ERROR: Exception | None = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
_F32 = ctypes.c_float

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2


def _flag(name: str) -> bool:
    return os.environ.get(name, "").strip().lower() in {"1", "true", "yes", "on"}


def _native_fp8_linear_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_FP8_LINEAR")


def _native_fp8_avx512_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_FP8_AVX512")


def _native_fp8_dequant_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_FP8_DEQUANT")


def _native_ds_router_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_DS_ROUTER")


def _native_ds_moe_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_DS_MOE")


def _native_flash_mla_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_FLASH_MLA")


def _native_fused_ds_attention_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_FUSED_DS_ATTENTION")


def _ds_monolithic_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_DS_MONOLITHIC")


def _native_disabled() -> bool:  # Q4 (the reference's name)
    return _flag("PCKETLM_DISABLE_NATIVE_Q4")


def _native_packed_gemv_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_PACKED_GEMV")


def _native_moe_disabled() -> bool:
    return _flag("PCKETLM_DISABLE_NATIVE_MOE")


_SIGNATURES: dict[str, tuple[list, object]] = {
    "moe_b200_abi_version": ([], _INT),
    "moe_b200_last_error": ([], ctypes.c_char_p),
    "moe_read_tensor_bytes": ([ctypes.c_char_p, ctypes.c_uint64, ctypes.c_uint64, _P], _INT),
    "moe_read_spans": ([ctypes.c_char_p, _I64, _P, _P, _P, _I64], _INT),
    "moe_fp8_e4m3_block_linear_f32": ([_P, _P, _P, _P, _I64, _I64, _I64, _I64, _P], _INT),
    "moe_fp8_e4m3_block_dual_linear_f32": ([_P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P], _INT),
    "moe_fp8_e4m3_block_mlp_f32": ([_P] * 8 + [_I64] * 5 + [_P, _I64, _P], _INT),
    "moe_fp8_e4m3_block_mlp_many_f32": ([_P] * 8 + [_I64] * 6 + [_P, _I64, _P], _INT),
    "moe_fp8_e4m3_block_mlp_many_weighted_f32": ([_P] * 9 + [_I64] * 6 + [_P, _I64, _P], _INT),
    "moe_fp8_e4m3_block_mlp_many_row_weighted_f32": ([_P] * 9 + [_I64] * 6 + [_P, _I64, _P], _INT),
    "moe_fp8_e4m3_block_mlp_many_pair_weighted_f32": ([_P] * 11 + [_I64] * 7 + [_P, _I64, _P], _INT),
    "moe_fp8_mlp_workspace_bytes": ([_I64] * 5, _I64),
    "moe_fp8_e4m3_block_mlp_f32_noalloc": ([_P] * 8 + [_I64] * 5 + [_P], _INT),
    "moe_fp8_e4m3_dequant_to_fp16": ([_P, _P, _P, _I64, _I64, _I64, _P], _INT),
    "moe_fp8_e4m3_dequant_to_bf16": ([_P, _P, _P, _I64, _I64, _I64, _P], _INT),
    "moe_ds_router_topk_u16": ([_P, _P, _I64, _I64, _I64, _I64, _P, _P, _P], _INT),
    "moe_route_topk": ([_P, _INT, _P, _INT, _P, _I64, _I64, _I64, _I64, _I64, _I64, _INT, _INT, _F32, _INT,
                        _P, _P, _P, _P, _I64, _P], _INT),
    "moe_route_topk_workspace_bytes": ([_I64, _I64], _I64),
    "moe_ds_moe_layer_fp8": ([_P, _INT, _I64, _I64, _I64, _P, _INT, _P, _I64, _I64, _I64, _I64, _INT, _F32, _P,
                              _INT, _P, _INT, _P, _P, _P, _P, _I64, _P], _INT),
    "moe_fp8_tiled_bytes": ([_I64, _I64], _I64),
    "moe_fp8_tile_weights": ([_P, _P, _I64, _I64, _P], _INT),
    "moe_fp8_nan_free_flags": ([_P, _I64, _I64, _I64, _P, _P], _INT),
    "moe_ds_moe_layer_workspace_bytes": ([_I64] * 5 + [_INT], _I64),
    "moe_ds_session_create": ([_I64] * 4, _P),
    "moe_ds_session_destroy": ([_P], None),
    "moe_ds_monolithic_call_counter": ([_P], _I64),
    "moe_ds_expert_invocation_count": ([_P], _I64),
    "moe_ds_layers_executed_count": ([_P], _I64),
    "moe_ds_attention_invocation_count": ([_P], _I64),
    "moe_ds_fused_attention_invocation_count": ([_P], _I64),
    "moe_mla_attention_workspace_bytes": ([_I64] * 6, _I64),
    "moe_mla_attention_flash_forward": ([_P] * 6 + [_I64] * 6 + [_F32, _P, _I64, _P], _INT),
    "moe_ds_attention_block_workspace_bytes": ([_I64] * 8, _I64),
    "moe_ds_attention_block_forward_f32": ([_P] * 16 + [_I64] * 8 + [_F32, _F32, _P, _I64, _P], _INT),
    "moe_ds_moe_layer_forward_f32": ([_P, _P, _P, _I64, _I64, _I64, _P, _P], _INT),
    "moe_ds_moe_layer_forward_fp8_f32": ([_P] * 9 + [_I64] * 6 + [_P, _P, _I64, _P], _INT),
    "moe_q4_dequant_to_fp16": ([_P, _P, _P, _I64, _I64, _P], _INT),
    "moe_q4_dequant_many_to_fp16": ([_P, _P, _P, _P, _P, _I64, _P], _INT),
    "moe_q4_moe_selected_forward_u16": ([_P] * 9 + [_I64] * 3 + [_P, _I64, _P], _INT),
    "moe_q4_moe_selected_workspace_bytes": ([_I64] * 3, _I64),
    "moe_q4_moe_layer_u16": ([_P, _INT, _I64, _I64, _I64, _P, _INT, _I64, _I64, _P, _INT, _P, _P, _P, _P, _I64, _P],
                             _INT),
    "moe_q4_tiled_bytes": ([_I64, _I64], _I64),
    "moe_q4_tile_weights": ([_P, _P, _I64, _I64, _P], _INT),
    "moe_q4_moe_layer_workspace_bytes": ([_I64] * 5, _I64),
    "moe_pack_u16_rows8": ([_P, _P, _I64, _I64, _P], _INT),
    "moe_packed_gemv_rows8": ([_P, _P, _P, _I64, _I64, _INT, _P], _INT),
    "moe_moe_selected_forward_u16": ([_P] * 6 + [_I64] * 4 + [_INT, _P, _I64, _P], _INT),
    "moe_moe_selected_forward_workspace_bytes": ([_I64] * 4 + [_INT], _I64),
    "moe_moe_forward_fp16": ([_P] * 8 + [_I64] * 5 + [_INT, _P, _I64, _P], _INT),
    "moe_moe_forward_fp16_workspace_bytes": ([_I64] * 5, _I64),
    "moe_ep_dispatch_pack": ([_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _P], _INT),
    "moe_ep_dispatch_workspace_bytes": ([_I64, _I64], _I64),
    "moe_ep_experts_fp8": ([_P, _P, _I64, _I64, _I64, _P, _I64, _P, _INT, _P, _P, _I64, _P], _INT),
    "moe_ep_experts_workspace_bytes": ([_I64] * 4, _I64),
    "moe_ep_combine": ([_P, _INT, _P, _P, _I64, _I64, _I64, _INT, _P, _P], _INT),
    "moe_ep_count_ranks": ([_P, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "moe_ep_barrier_p2p": ([_P, _I64, _I64, _P, _P, _I64, _P, _I64, _P], _INT),
    "moe_ep_route_dispatch_p2p_workspace_bytes": ([_I64, _I64], _I64),
    "moe_ep_route_dispatch_p2p": ([_P, _P, _INT, _P, _I64, _I64, _I64, _I64, _I64, _I64, _F32, _I64, _I64,
                                   _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _I64, _P], _INT),
    "moe_ep_dispatch_p2p": ([_P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P, _P, _I64, _P],
                            _INT),
    "moe_ep_dispatch_p2p_workspace_bytes": ([_I64, _I64, _I64], _I64),
    "moe_ep_return_p2p": ([_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _P], _INT),
    "moe_ep_experts_return_p2p": ([_P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _INT, _I64, _I64, _I64, _P,
                                   _P, _I64, _P], _INT),
    "moe_ep_experts_return_p2p_workspace_bytes": ([_I64] * 5 + [_INT], _I64),
    "moe_b200_fused_decode": ([_INT], _INT),
    "moe_b200_fused_decode_enabled": ([], _INT),
    "moe_b200_force_ksplit": ([_INT], _INT),
    "moe_b200_decode_prologue": ([_INT], _INT),
    "moe_b200_kb_rotate": ([_INT], _INT),
    "moe_b200_fold_epilogues": ([_INT], _INT),
    "moe_b200_router_stages_x": ([_INT], _INT),
    "moe_b200_shared_side": ([_INT], _INT),
    "moe_b200_stage_timing": ([_INT], _INT),
    "moe_b200_stage_times": ([_P, _INT], _INT),
    "moe_b200_select_gemv": ([_INT], _INT),
    "moe_b200_selected_gemv": ([], _INT),
    "moe_b200_device_error": ([_P], _INT),
}


def load_library() -> ctypes.CDLL:
    """Load libmoe_b200.so; raise RuntimeError (never fall back) when it is missing."""
    global _LIB, _LIB_ERROR
    if _LIB is not None:
        return _LIB
    if not _LIB_PATH.exists():
        _LIB_ERROR = FileNotFoundError(f"{_LIB_PATH} (build it with `python -m pocketlm_b200.build`)")
        raise RuntimeError(f"libmoe_b200 is unavailable: {_LIB_ERROR}")
    try:
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
    except Exception as exc:  # pragma: no cover - platform path
        _LIB_ERROR = exc
        raise RuntimeError(f"libmoe_b200 is unavailable: {exc}") from exc
    _LIB = lib
    _LIB_ERROR = None
    return lib


def library_symbols() -> list[str]:
    return list(_SIGNATURES)


def _lib_or_none() -> ctypes.CDLL | None:
    try:
        return load_library()
    except RuntimeError:
        return None


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("libmoe_b200 needs a CUDA device (sm_100a); none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def _stream() -> _P:
    return _P(torch.cuda.current_stream().cuda_stream)


def _gpu(t: torch.Tensor, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Contiguous copy/view of `t` on the current CUDA device (optionally cast)."""
    t = t.detach()
    if t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    if dtype is not None and t.dtype != dtype:
        if dtype == torch.uint8 and t.dtype == torch.int8:
            t = t.view(torch.uint8)
        else:
            t = t.to(dtype)
    dev = _device()
    if t.device != dev:
        t = t.to(dev, non_blocking=False)
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()  # the kernels' vector and bulk loads want 16-byte aligned rows
    return t


def _ptr(t: torch.Tensor | None) -> _P:
    return _P(0 if t is None else int(t.data_ptr()))


def native_read_tensor_bytes(path: str | Path, absolute_offset: int, nbytes: int, out: torch.Tensor) -> None:
    """Read nbytes at absolute_offset of `path` into the host tensor `out`
    (moe_read_tensor_bytes; the reference's checks and errors,
    native/__init__.py:3314-3331)."""
    lib = load_library()
    if out.device.type != "cpu":
        raise ValueError("native_read_tensor_bytes reads into host memory")
    if not out.is_contiguous():
        raise ValueError("native_read_tensor_bytes requires a contiguous output tensor")
    if out.nelement() * out.element_size() != int(nbytes):
        raise ValueError("output tensor byte size does not match requested native read size")
    code = lib.moe_read_tensor_bytes(str(Path(path)).encode("utf-8"), int(absolute_offset), int(nbytes),
                                     _P(int(out.data_ptr())))
    if code != 0:
        raise OSError(f"native_read_tensor_bytes failed with code {code} for {path}")


def read_spans(path: str | Path, spans: list[tuple[int, int]], outs: list[torch.Tensor], threads: int = 0) -> None:
    """Byte ranges (offset, length) of one file into contiguous host tensors of
    exactly those lengths, several threads at once (moe_read_spans)."""
    if len(spans) != len(outs):
        raise ValueError("one output tensor per span")
    for (_off, n), out in zip(spans, outs):
        if out.device.type != "cpu" or not out.is_contiguous() or out.nelement() * out.element_size() != int(n):
            raise ValueError("span outputs must be contiguous host tensors of the span's length")
    k = len(spans)
    offs = (ctypes.c_uint64 * max(k, 1))(*[int(o) for o, _ in spans])
    lens = (ctypes.c_uint64 * max(k, 1))(*[int(n) for _, n in spans])
    ptrs = (ctypes.c_void_p * max(k, 1))(*[int(t.data_ptr()) for t in outs])
    code = load_library().moe_read_spans(str(Path(path)).encode("utf-8"), k, ctypes.cast(offs, _P),
                                         ctypes.cast(lens, _P), ctypes.cast(ptrs, _P), int(threads))
    if code != 0:
        raise OSError(f"moe_read_spans failed with code {code} for {path}")


def _check(code: int, name: str) -> None:
    if code != 0:
        detail = load_library().moe_b200_last_error() or b""
        raise RuntimeError(f"{name} failed with code {code}: {detail.decode(errors='replace')}")


def _workspace(nbytes: int) -> torch.Tensor:
    return torch.empty((max(int(nbytes), 256),), dtype=torch.uint8, device=_device())


def _out_device(ref: torch.Tensor) -> torch.device:
    return ref.device


# ---------------------------------------------------------------------------
# availability predicates (native/__init__.py:302-310, 510-561, 746-850)
# ---------------------------------------------------------------------------

def native_fp8_linear_available() -> bool:
    return not _native_fp8_linear_disabled() and _lib_or_none() is not None and torch.cuda.is_available()


def native_fp8_linear_error() -> Exception | None:
    _lib_or_none()
    return _LIB_ERROR


def native_fp8_linear_avx512_error() -> Exception | None:
    return native_fp8_linear_error()


def native_fp8_dual_linear_available() -> bool:
    return native_fp8_linear_available()


def native_fp8_mlp_available() -> bool:
    return native_fp8_linear_available()


def native_fp8_mlp_avx512_available() -> bool:
    return native_fp8_linear_available() and not _native_fp8_avx512_disabled()


def native_fp8_mlp_many_available() -> bool:
    return native_fp8_linear_available()


def native_fp8_mlp_many_weighted_available() -> bool:
    return native_fp8_linear_available()


def native_fp8_mlp_many_row_weighted_available() -> bool:
    return native_fp8_linear_available()


def native_fp8_mlp_many_pair_weighted_available() -> bool:
    return native_fp8_linear_available()


def native_fp8_mlp_many_weighted_avx512_available() -> bool:
    return native_fp8_mlp_avx512_available()


def native_fp8_dequant_available() -> bool:
    return not _native_fp8_dequant_disabled() and _lib_or_none() is not None and torch.cuda.is_available()


def native_fp8_dequant_error() -> Exception | None:
    _lib_or_none()
    return _LIB_ERROR


def native_ds_forward_available() -> bool:
    return not _ds_monolithic_disabled() and _lib_or_none() is not None and torch.cuda.is_available()


def native_ds_router_available() -> bool:
    return native_ds_forward_available() and not _native_ds_router_disabled()


def native_ds_moe_available() -> bool:
    return native_ds_forward_available() and not _native_ds_moe_disabled()


def native_flash_mla_available() -> bool:
    return native_ds_forward_available() and not _native_flash_mla_disabled()


def native_fused_ds_attention_available() -> bool:
    return native_ds_forward_available() and not _native_fused_ds_attention_disabled()


def _require(available: bool, what: str, disabled: bool) -> None:
    if not available:
        reason = "disabled" if disabled else (_LIB_ERROR or "no CUDA device")
        raise RuntimeError(f"Native {what} is unavailable: {reason}")


# ---------------------------------------------------------------------------
# FP8 dequant (native/__init__.py:3378-3439)
# ---------------------------------------------------------------------------

def _dequant(fp8_weight: torch.Tensor, scale_inv: torch.Tensor, bf16: bool) -> torch.Tensor:
    _require(native_fp8_dequant_available(), "FP8 BF16 dequant" if bf16 else "FP8 dequant",
             _native_fp8_dequant_disabled())
    if fp8_weight.ndim != 2:
        raise ValueError("fp8_weight must have shape [rows, cols]")
    if scale_inv.ndim != 2:
        raise ValueError("scale_inv must have shape [scale_rows, scale_cols]")
    w = _gpu(fp8_weight, torch.uint8)
    s = _gpu(scale_inv, torch.float32)
    rows, cols = int(w.shape[0]), int(w.shape[1])
    expected = ((rows + 127) // 128, (cols + 127) // 128)
    if tuple(s.shape) != expected:
        raise ValueError("scale_inv shape does not match FP8 128x128 block layout")
    dtype = torch.bfloat16 if bf16 else torch.float16
    out = torch.empty((rows, cols), dtype=dtype, device=w.device)
    lib = load_library()
    fn = lib.moe_fp8_e4m3_dequant_to_bf16 if bf16 else lib.moe_fp8_e4m3_dequant_to_fp16
    code = fn(_ptr(w), _ptr(s), _ptr(out), rows, cols, expected[1], _stream())
    _check(code, "fp8_e4m3_dequant_to_bf16" if bf16 else "fp8_e4m3_dequant_to_fp16")
    return out.to(_out_device(fp8_weight))


def fp8_e4m3_dequant_to_fp16(fp8_weight: torch.Tensor, scale_inv: torch.Tensor) -> torch.Tensor:
    return _dequant(fp8_weight, scale_inv, bf16=False)


def fp8_e4m3_dequant_to_bf16(fp8_weight: torch.Tensor, scale_inv: torch.Tensor) -> torch.Tensor:
    return _dequant(fp8_weight, scale_inv, bf16=True)


# ---------------------------------------------------------------------------
# FP8 linears (native/__init__.py:3442-3531)
# ---------------------------------------------------------------------------

def _hidden_rows(hidden: torch.Tensor) -> torch.Tensor:
    return _gpu(hidden.reshape(-1, int(hidden.shape[-1])), torch.float32)


def fp8_e4m3_block_linear_f32(fp8_weight: torch.Tensor, scale_inv: torch.Tensor, hidden: torch.Tensor) -> torch.Tensor:
    _require(native_fp8_linear_available(), "FP8 linear", _native_fp8_linear_disabled())
    if fp8_weight.ndim != 2:
        raise ValueError("fp8_weight must have shape [out_rows, in_cols]")
    if scale_inv.ndim != 2:
        raise ValueError("scale_inv must have shape [scale_rows, scale_cols]")
    x = _hidden_rows(hidden)
    w = _gpu(fp8_weight, torch.uint8)
    s = _gpu(scale_inv, torch.float32)
    out_rows, in_cols = int(w.shape[0]), int(w.shape[1])
    if int(x.shape[1]) != in_cols:
        raise ValueError("hidden input size does not match FP8 weight columns")
    if tuple(s.shape) != ((out_rows + 127) // 128, (in_cols + 127) // 128):
        raise ValueError("scale_inv shape does not match FP8 128x128 block layout")
    out = torch.empty((int(x.shape[0]), out_rows), dtype=torch.float32, device=x.device)
    code = load_library().moe_fp8_e4m3_block_linear_f32(_ptr(w), _ptr(s), _ptr(x), _ptr(out), int(x.shape[0]),
                                                        out_rows, in_cols, int(s.shape[1]), _stream())
    _check(code, "fp8_e4m3_block_linear_f32")
    return out.to(_out_device(hidden))


def fp8_e4m3_block_dual_linear_f32(fp8_weight_a, scale_inv_a, fp8_weight_b, scale_inv_b, hidden):
    _require(native_fp8_dual_linear_available(), "FP8 dual linear", _native_fp8_linear_disabled())
    if fp8_weight_a.ndim != 2 or fp8_weight_b.ndim != 2:
        raise ValueError("fp8 weights must have shape [out_rows, in_cols]")
    wa, wb = _gpu(fp8_weight_a, torch.uint8), _gpu(fp8_weight_b, torch.uint8)
    if tuple(wa.shape) != tuple(wb.shape):
        raise ValueError("dual FP8 weights must have matching shapes")
    sa, sb = _gpu(scale_inv_a, torch.float32), _gpu(scale_inv_b, torch.float32)
    if tuple(sa.shape) != tuple(sb.shape):
        raise ValueError("dual FP8 scales must have matching shapes")
    x = _hidden_rows(hidden)
    out_rows, in_cols = int(wa.shape[0]), int(wa.shape[1])
    if int(x.shape[1]) != in_cols:
        raise ValueError("hidden input size does not match FP8 weight columns")
    if tuple(sa.shape) != ((out_rows + 127) // 128, (in_cols + 127) // 128):
        raise ValueError("scale_inv shape does not match FP8 128x128 block layout")
    out_a = torch.empty((int(x.shape[0]), out_rows), dtype=torch.float32, device=x.device)
    out_b = torch.empty_like(out_a)
    code = load_library().moe_fp8_e4m3_block_dual_linear_f32(
        _ptr(wa), _ptr(sa), _ptr(wb), _ptr(sb), _ptr(x), _ptr(out_a), _ptr(out_b), int(x.shape[0]), out_rows,
        in_cols, int(sa.shape[1]), _stream())
    _check(code, "fp8_e4m3_block_dual_linear_f32")
    dev = _out_device(hidden)
    return out_a.to(dev), out_b.to(dev)


# ---------------------------------------------------------------------------
# FP8 expert MLPs (native/__init__.py:3533-4022)
# ---------------------------------------------------------------------------

def _check_mlp_item(gate, gate_s, up, up_s, down, down_s):
    if gate.ndim != 2 or up.ndim != 2 or down.ndim != 2:
        raise ValueError("FP8 MLP weights must be 2D")
    if tuple(gate.shape) != tuple(up.shape):
        raise ValueError("FP8 MLP gate and up weights must have matching shapes")
    inter, hid = int(gate.shape[0]), int(gate.shape[1])
    if tuple(down.shape) != (hid, inter):
        raise ValueError("FP8 MLP down weight must have shape [hidden, intermediate]")
    if tuple(gate_s.shape) != tuple(up_s.shape):
        raise ValueError("FP8 MLP gate and up scales must have matching shapes")
    if tuple(gate_s.shape) != ((inter + 127) // 128, (hid + 127) // 128):
        raise ValueError("FP8 MLP gate scale shape does not match 128x128 block layout")
    if tuple(down_s.shape) != ((hid + 127) // 128, (inter + 127) // 128):
        raise ValueError("FP8 MLP down scale shape does not match 128x128 block layout")
    return inter, hid


def _mlp(gate, gate_scale_inv, up, up_scale_inv, down, down_scale_inv, hidden, what: str, avx512: bool):
    avail = native_fp8_mlp_avx512_available() if avx512 else native_fp8_mlp_available()
    _require(avail, what, _native_fp8_avx512_disabled() if avx512 else _native_fp8_linear_disabled())
    inter, hid = _check_mlp_item(gate, gate_scale_inv, up, up_scale_inv, down, down_scale_inv)
    x = _hidden_rows(hidden)
    if int(x.shape[1]) != hid:
        raise ValueError("hidden input size does not match FP8 MLP input size")
    t = [_gpu(gate, torch.uint8), _gpu(gate_scale_inv, torch.float32), _gpu(up, torch.uint8),
         _gpu(up_scale_inv, torch.float32), _gpu(down, torch.uint8), _gpu(down_scale_inv, torch.float32)]
    batch = int(x.shape[0])
    out = torch.empty((batch, hid), dtype=torch.float32, device=x.device)
    lib = load_library()
    ws = _workspace(lib.moe_fp8_mlp_workspace_bytes(batch, 1, batch, inter, hid))
    code = lib.moe_fp8_e4m3_block_mlp_f32(*[_ptr(v) for v in t], _ptr(x), _ptr(out), batch, inter, hid,
                                          (hid + 127) // 128, (inter + 127) // 128, _ptr(ws), ws.numel(),
                                          _stream())
    _check(code, "fp8_e4m3_block_mlp_avx512_f32" if avx512 else "fp8_e4m3_block_mlp_f32")
    return out.to(_out_device(hidden))


def fp8_e4m3_block_mlp_f32(gate_weight, gate_scale_inv, up_weight, up_scale_inv, down_weight, down_scale_inv,
                           hidden) -> torch.Tensor:
    return _mlp(gate_weight, gate_scale_inv, up_weight, up_scale_inv, down_weight, down_scale_inv, hidden,
                "FP8 MLP", avx512=False)


def fp8_e4m3_block_mlp_avx512_f32(gate_weight, gate_scale_inv, up_weight, up_scale_inv, down_weight,
                                  down_scale_inv, hidden) -> torch.Tensor:
    """The reference's AVX-512 twin is bit-exact to its scalar kernel
    (fp8_linear_avx512.cpp:103-133); on the GPU both are the same kernel."""
    return _mlp(gate_weight, gate_scale_inv, up_weight, up_scale_inv, down_weight, down_scale_inv, hidden,
                "FP8 AVX-512 MLP", avx512=True)


class ExpertTables:
    """Device uint64 tables of expert weight/scale addresses (the reference's
    int64 pointer tables, native/__init__.py:1372-1378, but device-resident).
    Keeps the tensors alive for as long as the tables are in use."""

    def __init__(self, items):
        if not items:
            raise ValueError("items must not be empty")
        first = items[0]
        self.inter, self.hidden = int(first[0].shape[0]), int(first[0].shape[1])
        self.tensors = []
        cols = [[] for _ in range(6)]
        for gate, gate_s, up, up_s, down, down_s in items:
            gate_t, up_t, down_t = (_gpu(v, torch.uint8) for v in (gate, up, down))
            if tuple(gate_t.shape) != (self.inter, self.hidden):
                raise ValueError("all gate weights must have matching shape")
            if tuple(up_t.shape) != (self.inter, self.hidden):
                raise ValueError("all up weights must have matching shape")
            if tuple(down_t.shape) != (self.hidden, self.inter):
                raise ValueError("all down weights must have matching shape")
            conv = (gate_t, _gpu(gate_s, torch.float32), up_t, _gpu(up_s, torch.float32), down_t,
                    _gpu(down_s, torch.float32))
            self.tensors.append(conv)
            for j, t in enumerate(conv):
                cols[j].append(int(t.data_ptr()))
        gsc = ((self.inter + 127) // 128, (self.hidden + 127) // 128)
        dsc = ((self.hidden + 127) // 128, (self.inter + 127) // 128)
        for conv in self.tensors:
            if tuple(conv[1].shape) != gsc or tuple(conv[3].shape) != gsc:
                raise ValueError("gate/up scale shapes do not match 128x128 block layout")
            if tuple(conv[5].shape) != dsc:
                raise ValueError("down scale shape does not match 128x128 block layout")
        self.table = torch.tensor(cols, dtype=torch.int64).to(_device())  # [6, E]
        self.count = len(self.tensors)
        self.gsc, self.dsc = gsc[1], dsc[1]

    def ptrs(self) -> list[_P]:
        base = int(self.table.data_ptr())
        return [_P(base + j * self.count * 8) for j in range(6)]


def _many_common(items, hidden, what, avail_fn, disabled):
    _require(avail_fn(), what, disabled)
    tables = ExpertTables(items)
    x = _hidden_rows(hidden)
    if int(x.shape[1]) != tables.hidden:
        raise ValueError("hidden input size does not match FP8 MLP input size")
    return tables, x


def fp8_e4m3_block_mlp_many_f32(items, hidden: torch.Tensor) -> torch.Tensor:
    tables, x = _many_common(items, hidden, "FP8 many-MLP", native_fp8_mlp_many_available,
                             _native_fp8_linear_disabled())
    E, B = tables.count, int(x.shape[0])
    out = torch.zeros((E, B, tables.hidden), dtype=torch.float32, device=x.device)
    lib = load_library()
    ws = _workspace(lib.moe_fp8_mlp_workspace_bytes(E * B, E, B, tables.inter, tables.hidden))
    code = lib.moe_fp8_e4m3_block_mlp_many_f32(*tables.ptrs(), _ptr(x), _ptr(out), E, B, tables.inter,
                                               tables.hidden, tables.gsc, tables.dsc, _ptr(ws), ws.numel(),
                                               _stream())
    _check(code, "fp8_e4m3_block_mlp_many_f32")
    return out.to(_out_device(hidden))


def _weighted(items, hidden, route_weights, avx512: bool):
    what = "FP8 AVX-512 weighted many-MLP" if avx512 else "FP8 weighted many-MLP"
    avail = native_fp8_mlp_many_weighted_avx512_available if avx512 else native_fp8_mlp_many_weighted_available
    tables, x = _many_common(items, hidden, what, avail,
                             _native_fp8_avx512_disabled() if avx512 else _native_fp8_linear_disabled())
    route = _gpu(route_weights.reshape(-1), torch.float32)
    if int(route.numel()) != tables.count:
        raise ValueError("route_weights length must match item count")
    E, B = tables.count, int(x.shape[0])
    out = torch.empty((B, tables.hidden), dtype=torch.float32, device=x.device)
    lib = load_library()
    ws = _workspace(lib.moe_fp8_mlp_workspace_bytes(E * B, E, B, tables.inter, tables.hidden))
    code = lib.moe_fp8_e4m3_block_mlp_many_weighted_f32(*tables.ptrs(), _ptr(x), _ptr(route), _ptr(out), E, B,
                                                        tables.inter, tables.hidden, tables.gsc, tables.dsc,
                                                        _ptr(ws), ws.numel(), _stream())
    _check(code, "fp8_e4m3_block_mlp_many_weighted_avx512_f32" if avx512 else "fp8_e4m3_block_mlp_many_weighted_f32")
    return out.to(_out_device(hidden))


def fp8_e4m3_block_mlp_many_weighted_f32(items, hidden: torch.Tensor, route_weights: torch.Tensor) -> torch.Tensor:
    return _weighted(items, hidden, route_weights, avx512=False)


def fp8_e4m3_block_mlp_many_weighted_avx512_f32(items, hidden: torch.Tensor, route_weights: torch.Tensor):
    return _weighted(items, hidden, route_weights, avx512=True)


def fp8_e4m3_block_mlp_many_row_weighted_f32(items, hidden: torch.Tensor, route_weights: torch.Tensor):
    tables, x = _many_common(items, hidden, "FP8 row-weighted many-MLP", native_fp8_mlp_many_row_weighted_available,
                             _native_fp8_linear_disabled())
    route = _gpu(route_weights, torch.float32)
    if tuple(route.shape) != (tables.count, int(x.shape[0])):
        raise ValueError("route_weights must have shape [expert_count, batch]")
    E, B = tables.count, int(x.shape[0])
    out = torch.empty((B, tables.hidden), dtype=torch.float32, device=x.device)
    lib = load_library()
    ws = _workspace(lib.moe_fp8_mlp_workspace_bytes(E * B, E, B, tables.inter, tables.hidden))
    code = lib.moe_fp8_e4m3_block_mlp_many_row_weighted_f32(*tables.ptrs(), _ptr(x), _ptr(route), _ptr(out), E,
                                                            B, tables.inter, tables.hidden, tables.gsc,
                                                            tables.dsc, _ptr(ws), ws.numel(), _stream())
    _check(code, "fp8_e4m3_block_mlp_many_row_weighted_f32")
    return out.to(_out_device(hidden))


def fp8_e4m3_block_mlp_many_pair_weighted_f32(items, hidden, pair_item_indices, pair_row_indices, pair_weights):
    tables, x = _many_common(items, hidden, "FP8 pair-weighted many-MLP",
                             native_fp8_mlp_many_pair_weighted_available, _native_fp8_linear_disabled())
    pi = _gpu(pair_item_indices.reshape(-1), torch.int64)
    pr = _gpu(pair_row_indices.reshape(-1), torch.int64)
    pw = _gpu(pair_weights.reshape(-1), torch.float32)
    if int(pi.numel()) != int(pr.numel()) or int(pi.numel()) != int(pw.numel()):
        raise ValueError("pair index and weight tensors must have matching length")
    E, B, P = tables.count, int(x.shape[0]), int(pi.numel())
    out = torch.empty((B, tables.hidden), dtype=torch.float32, device=x.device)
    lib = load_library()
    ws = _workspace(lib.moe_fp8_mlp_workspace_bytes(P, E, 1, tables.inter, tables.hidden) + 16 * (P + B + 64) + 4096)
    code = lib.moe_fp8_e4m3_block_mlp_many_pair_weighted_f32(*tables.ptrs(), _ptr(x), _ptr(pi), _ptr(pr), _ptr(pw),
                                                             _ptr(out), E, P, B, tables.inter, tables.hidden,
                                                             tables.gsc, tables.dsc, _ptr(ws), ws.numel(), _stream())
    _check(code, "fp8_e4m3_block_mlp_many_pair_weighted_f32")
    return out.to(_out_device(hidden))


# ---------------------------------------------------------------------------
# Routers (native/__init__.py:765-813)
# ---------------------------------------------------------------------------

def ds_router_topk(hidden: torch.Tensor, router_weights: torch.Tensor, *, k: int):
    """Softmax router top-k for one token (ds_forward.cpp:879-955), on the GPU."""
    if router_weights.ndim != 2:
        raise ValueError("router_weights must be rank-2 [num_experts, hidden_dim]")
    if hidden.reshape(-1).numel() != router_weights.shape[1]:
        raise ValueError("hidden size must match router weight columns")
    _require(native_ds_router_available(), "DS router", _native_ds_router_disabled() or _ds_monolithic_disabled())
    effective_k = max(1, min(int(k), int(router_weights.shape[0])))
    x = hidden.reshape(-1)
    if x.dtype not in {torch.float16, torch.bfloat16}:
        x = x.to(torch.float16)
    w = router_weights if router_weights.dtype == x.dtype else router_weights.to(x.dtype)
    x, w = _gpu(x), _gpu(w)
    ids = torch.empty((effective_k,), dtype=torch.int64, device=x.device)
    weights = torch.empty((effective_k,), dtype=torch.float32, device=x.device)
    code = load_library().moe_ds_router_topk_u16(_ptr(x), _ptr(w), int(w.shape[1]), int(w.shape[0]), effective_k,
                                                 1 if x.dtype == torch.bfloat16 else 0, _ptr(ids), _ptr(weights),
                                                 _stream())
    if code != 0:
        raise RuntimeError(f"ds_router_topk_u16 failed with code {code}")
    dev = _out_device(hidden)
    return ids.to(dev), weights.to(dev)


def _python_ds_router_topk(hidden: torch.Tensor, router_weights: torch.Tensor, k: int):
    """The reference's torch restatement of the softmax router
    (native/__init__.py:804-813), kept for callers and tests that compare
    against it; the product path never calls it."""
    scores = torch.nn.functional.linear(hidden.reshape(1, -1).float(), router_weights.float()).reshape(-1)
    probs = torch.softmax(scores, dim=-1)
    weights, ids = torch.topk(probs, int(k), dim=-1)
    weights = weights / weights.sum().clamp_min(1e-12)
    return ids.to(torch.int64).contiguous(), weights.to(torch.float32).contiguous()


def route_topk(hidden: torch.Tensor, router_weight: torch.Tensor, bias: torch.Tensor | None, *, top_k: int,
               n_group: int = 1, topk_group: int = 1, scoring_func: str = "sigmoid", route_scale: float = 1.0,
               renorm: bool = False, round_to_hidden_dtype: bool = True, weights_fp32: bool = False):
    """Batched router on the GPU: the math of run_fp8_router
    (fp8_source.py:1522-1547) or, with scoring_func="softmax" and renorm,
    the Mixtral router (layer_bridge.py:2682-2689).

    Returns (ids int64 [T, k], weights [T, k]) with weights in hidden.dtype
    when round_to_hidden_dtype (the reference casts them), else fp32;
    weights_fp32 returns them as fp32 values (rounded through the hidden
    dtype when round_to_hidden_dtype)."""
    x = _gpu(hidden.reshape(-1, int(hidden.shape[-1])))
    dt = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}
    if x.dtype not in dt:
        x = x.float()
    w = _gpu(router_weight)
    if w.dtype not in dt:
        w = w.float()
    b = None if bias is None else _gpu(bias, torch.float32)
    T, H = int(x.shape[0]), int(x.shape[1])
    E = int(w.shape[0])
    k = max(1, min(int(top_k), E))
    ids = torch.empty((T, k), dtype=torch.int64, device=x.device)
    wf = torch.empty((T, k), dtype=torch.float32, device=x.device)
    wb = torch.empty((T, k), dtype=torch.bfloat16, device=x.device) if x.dtype == torch.bfloat16 else None
    lib = load_library()
    ws = _workspace(lib.moe_route_topk_workspace_bytes(T, E))
    code = lib.moe_route_topk(_ptr(x), dt[x.dtype], _ptr(w), dt[w.dtype], _ptr(b), T, H, E, int(n_group),
                              int(topk_group), k, 1 if scoring_func == "softmax" else 0, 1 if renorm else 0,
                              float(route_scale), 1 if (round_to_hidden_dtype and wb is not None) else 0,
                              _ptr(ids), _ptr(wf), _ptr(wb), _ptr(ws), ws.numel(), _stream())
    _check(code, "moe_route_topk")
    if weights_fp32:
        weights = wf
    elif round_to_hidden_dtype:
        weights = wb if wb is not None else wf.to(hidden.dtype)
    else:
        weights = wf
    dev = _out_device(hidden)
    return ids.to(dev), weights.to(dev)


# ---------------------------------------------------------------------------
# DeepSeek session + MoE combine (native/__init__.py:1300-1520)
# ---------------------------------------------------------------------------

class DeepSeekNativeSession:
    """Opaque session with the reference's observable counters
    (ds_forward.cpp:192-335).  The fp8 pack / KV callbacks of the reference
    belong to its callback-driven layer loop and pack streaming, which this
    path does not have; the arguments are accepted and ignored."""

    def __init__(self, *, num_layers: int, hidden_dim: int, num_experts: int, top_k: int,
                 fp8_pack_callback: object | None = None, kv_session_handle: int | None = None):
        if not native_ds_forward_available():
            reason = "disabled" if _ds_monolithic_disabled() else (_LIB_ERROR or "no CUDA device")
            raise RuntimeError(f"DeepSeek native session is unavailable: {reason}")
        self._lib = load_library()
        handle = self._lib.moe_ds_session_create(int(num_layers), int(hidden_dim), int(num_experts), int(top_k))
        if not handle:
            raise RuntimeError("ds_session_create returned a null handle")
        self._handle = _P(handle)
        self._tensor_keepalive: list[object] = []

    def close(self) -> None:
        if getattr(self, "_handle", None):
            self._lib.moe_ds_session_destroy(self._handle)
            self._handle = None
            self._tensor_keepalive.clear()

    def __enter__(self) -> "DeepSeekNativeSession":
        return self

    def __exit__(self, *_exc: object) -> None:
        self.close()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def keep_tensor_alive(self, tensor: object) -> None:
        self._tensor_keepalive.append(tensor)

    def monolithic_call_count(self) -> int:
        return int(self._lib.moe_ds_monolithic_call_counter(self._handle))

    def expert_invocation_count(self) -> int:
        return int(self._lib.moe_ds_expert_invocation_count(self._handle))

    def layers_executed_count(self) -> int:
        return int(self._lib.moe_ds_layers_executed_count(self._handle))

    def attention_invocation_count(self) -> int:
        return int(self._lib.moe_ds_attention_invocation_count(self._handle))

    def fused_attention_invocation_count(self) -> int:
        return int(self._lib.moe_ds_fused_attention_invocation_count(self._handle))


def _python_ds_moe_layer_forward(expert_outputs: torch.Tensor, route_weights: torch.Tensor) -> torch.Tensor:
    """The reference's torch restatement of the combine (native/__init__.py:1403-1408)."""
    outputs = expert_outputs.detach().to(torch.float32)
    if outputs.ndim == 2:
        outputs = outputs.unsqueeze(1)
    weights = route_weights.detach().reshape(-1).to(device=outputs.device, dtype=torch.float32)
    return (outputs * weights.view(-1, 1, 1)).sum(dim=0)


def ds_moe_layer_forward(session: DeepSeekNativeSession, expert_outputs: torch.Tensor, route_weights: torch.Tensor):
    """Combine selected expert outputs (ds_forward.cpp:337-367) on the GPU."""
    outputs = _gpu(expert_outputs, torch.float32)
    if outputs.ndim == 2:
        outputs = outputs.unsqueeze(1).contiguous()
    if outputs.ndim != 3:
        raise ValueError("expert_outputs must be [selected, batch, hidden]")
    weights = _gpu(route_weights.reshape(-1), torch.float32)
    if int(weights.numel()) != int(outputs.shape[0]):
        raise ValueError("route weight count must match selected expert count")
    _require(native_ds_moe_available(), "DS MoE", _native_ds_moe_disabled())
    out = torch.empty((int(outputs.shape[1]), int(outputs.shape[2])), dtype=torch.float32, device=outputs.device)
    code = session._lib.moe_ds_moe_layer_forward_f32(session._handle, _ptr(outputs), _ptr(weights),
                                                     int(outputs.shape[0]), int(outputs.shape[1]),
                                                     int(outputs.shape[2]), _ptr(out), _stream())
    if code != 0:
        raise RuntimeError(f"ds_moe_layer_forward_f32 failed with code {code}")
    return out.to(_out_device(expert_outputs))


def ds_moe_layer_forward_fp8(session: DeepSeekNativeSession, items, hidden: torch.Tensor,
                             route_weights: torch.Tensor) -> torch.Tensor:
    """Selected FP8 expert MLPs + combine in one call (ds_forward.cpp:784-877)."""
    _require(native_ds_moe_available(), "DS MoE", _native_ds_moe_disabled())
    tables = ExpertTables(items)
    x = _hidden_rows(hidden)
    route = _gpu(route_weights.reshape(-1), torch.float32)
    if int(x.shape[1]) != tables.hidden:
        raise ValueError("hidden input size does not match FP8 MLP input size")
    if int(route.numel()) != tables.count:
        raise ValueError("route weight count must match selected experts")
    E, B = tables.count, int(x.shape[0])
    out = torch.empty((B, tables.hidden), dtype=torch.float32, device=x.device)
    lib = load_library()
    ws = _workspace(lib.moe_fp8_mlp_workspace_bytes(E * B, E, B, tables.inter, tables.hidden))
    code = lib.moe_ds_moe_layer_forward_fp8_f32(session._handle, *tables.ptrs(), _ptr(x), _ptr(route), E, B,
                                                tables.inter, tables.hidden, tables.gsc, tables.dsc, _ptr(out),
                                                _ptr(ws), ws.numel(), _stream())
    if code != 0:
        raise RuntimeError(f"ds_moe_layer_forward_fp8_f32 failed with code {code}")
    return out.to(_out_device(hidden))


# ---------------------------------------------------------------------------
# MLA attention (native/__init__.py:878-1075; ds_forward.cpp:517-782)
# ---------------------------------------------------------------------------

def ds_mla_attention_flash_forward(q_nope: torch.Tensor, q_pe: torch.Tensor, kv_cache: torch.Tensor,
                                   pe_cache: torch.Tensor, wkv_b: torch.Tensor, *,
                                   softmax_scale: float) -> torch.Tensor:
    """Compressed-KV MLA attention core for one query token on the GPU
    (ds_forward.cpp:517-597): q_nope [heads, nope], q_pe [heads, rope],
    kv_cache [cache_len, kv_lora_rank], pe_cache [cache_len, rope], wkv_b
    [heads, nope + v, kv_lora_rank] -> [heads, v] fp32 on q_nope's device.
    The shape checks and messages are the reference's (native/__init__.py:895-916)."""
    if q_nope.ndim != 2 or q_pe.ndim != 2:
        raise ValueError("q_nope and q_pe must be [heads, dim]")
    if kv_cache.ndim != 2 or pe_cache.ndim != 2:
        raise ValueError("kv_cache and pe_cache must be [cache_len, dim]")
    if wkv_b.ndim != 3:
        raise ValueError("wkv_b must be [heads, qk_nope + v_head_dim, kv_lora_rank]")
    heads, nope, rope = int(q_nope.shape[0]), int(q_nope.shape[1]), int(q_pe.shape[1])
    cache_len, rank = int(kv_cache.shape[0]), int(kv_cache.shape[1])
    if int(q_pe.shape[0]) != heads or int(wkv_b.shape[0]) != heads:
        raise ValueError("head count mismatch")
    if int(pe_cache.shape[0]) != cache_len or int(pe_cache.shape[1]) != rope:
        raise ValueError("pe_cache shape mismatch")
    if int(wkv_b.shape[2]) != rank or int(wkv_b.shape[1]) <= nope:
        raise ValueError("wkv_b shape mismatch")
    v_dim = int(wkv_b.shape[1]) - nope
    _require(native_flash_mla_available(), "flash MLA", _native_flash_mla_disabled())
    qn, qp = _gpu(q_nope, torch.float32), _gpu(q_pe, torch.float32)
    kv, pe, wkv = _gpu(kv_cache, torch.float32), _gpu(pe_cache, torch.float32), _gpu(wkv_b, torch.float32)
    lib = load_library()
    out = torch.empty((heads, v_dim), dtype=torch.float32, device=qn.device)
    ws = _workspace(lib.moe_mla_attention_workspace_bytes(heads, cache_len, nope, rope, rank, v_dim))
    code = lib.moe_mla_attention_flash_forward(_ptr(qn), _ptr(qp), _ptr(kv), _ptr(pe), _ptr(wkv), _ptr(out), heads,
                                               cache_len, nope, rope, rank, v_dim, float(softmax_scale), _ptr(ws),
                                               ws.numel(), _stream())
    _check(code, "ds_mla_attention_flash_forward")
    return out.to(_out_device(q_nope))


def ds_attention_block_forward(session: DeepSeekNativeSession, hidden: torch.Tensor, q_a_weight: torch.Tensor,
                               q_b_weight: torch.Tensor, kv_a_weight: torch.Tensor, kv_b_weight: torch.Tensor,
                               o_weight: torch.Tensor, q_norm_weight: torch.Tensor, kv_norm_weight: torch.Tensor, *,
                               previous_kv_cache: torch.Tensor | None, previous_pe_cache: torch.Tensor | None,
                               rope_cos: torch.Tensor, rope_sin: torch.Tensor, q_lora_rank: int, kv_lora_rank: int,
                               num_heads: int, qk_nope_dim: int, qk_rope_dim: int, v_head_dim: int, rms_eps: float,
                               softmax_scale: float) -> tuple[torch.Tensor, tuple[torch.Tensor, torch.Tensor]]:
    """A one-token DeepSeek attention block as one call (ds_forward.cpp:647-782)
    on the GPU: returns hidden_out [hidden_dim] and the new caches
    ([previous_len + 1, kv_lora_rank], [previous_len + 1, qk_rope_dim]), fp32 on
    hidden's device.  The shape checks and messages are the reference's
    (native/__init__.py:969-1005); weights stay where they are when they are
    already fp32 on the GPU (one upload per call otherwise)."""
    H = int(hidden.numel())
    if H <= 0:
        raise ValueError("hidden must not be empty")
    q_rank, rank, heads = int(q_lora_rank), int(kv_lora_rank), int(num_heads)
    nope, rope, v_dim = int(qk_nope_dim), int(qk_rope_dim), int(v_head_dim)
    if tuple(q_a_weight.shape) != (q_rank, H):
        raise ValueError("q_a_weight must be [q_lora_rank, hidden_dim]")
    if tuple(q_b_weight.shape) != (heads * (nope + rope), q_rank):
        raise ValueError("q_b_weight shape does not match DeepSeek attention config")
    if tuple(kv_a_weight.shape) != (rank + rope, H):
        raise ValueError("kv_a_weight shape does not match DeepSeek attention config")
    if tuple(kv_b_weight.shape) != (heads * (nope + v_dim), rank):
        raise ValueError("kv_b_weight shape does not match DeepSeek attention config")
    if tuple(o_weight.shape) != (H, heads * v_dim):
        raise ValueError("o_weight shape does not match DeepSeek attention config")
    if int(q_norm_weight.numel()) != q_rank or int(kv_norm_weight.numel()) != rank:
        raise ValueError("norm weight sizes do not match ranks")
    if int(rope_cos.numel()) != max(0, rope // 2) or int(rope_sin.numel()) != max(0, rope // 2):
        raise ValueError("rope cos/sin sizes must be qk_rope_dim / 2")
    prev_len = 0 if previous_kv_cache is None else int(previous_kv_cache.numel()) // max(rank, 1)
    prev_pe_len = 0 if previous_pe_cache is None else int(previous_pe_cache.numel()) // max(rope, 1)
    if previous_pe_cache is not None and rope == 0:
        prev_pe_len = prev_len if int(previous_pe_cache.numel()) == 0 else -1
    if prev_pe_len != prev_len:
        raise ValueError("previous KV and PE cache lengths must match")
    _require(native_fused_ds_attention_available(), "fused DeepSeek attention", _native_fused_ds_attention_disabled())
    x = _gpu(hidden, torch.float32).reshape(-1)
    q_a, q_b = _gpu(q_a_weight, torch.float32), _gpu(q_b_weight, torch.float32)
    kv_a, kv_b, o_w = _gpu(kv_a_weight, torch.float32), _gpu(kv_b_weight, torch.float32), _gpu(o_weight, torch.float32)
    q_norm = _gpu(q_norm_weight, torch.float32).reshape(-1)
    kv_norm = _gpu(kv_norm_weight, torch.float32).reshape(-1)
    cos, sin = _gpu(rope_cos, torch.float32).reshape(-1), _gpu(rope_sin, torch.float32).reshape(-1)
    prev_kv = None if not prev_len else _gpu(previous_kv_cache, torch.float32).reshape(-1, rank)
    prev_pe = None if not prev_len else _gpu(previous_pe_cache, torch.float32).reshape(-1, rope)
    lib = load_library()
    next_kv = torch.empty((prev_len + 1, rank), dtype=torch.float32, device=x.device)
    next_pe = torch.empty((prev_len + 1, rope), dtype=torch.float32, device=x.device)
    out = torch.empty((H,), dtype=torch.float32, device=x.device)
    # a zero-size cos/sin still needs an address (the reference requires non-null pointers)
    if cos.numel() == 0:
        cos = torch.zeros((1,), dtype=torch.float32, device=x.device)
        sin = torch.zeros((1,), dtype=torch.float32, device=x.device)
    ws = _workspace(lib.moe_ds_attention_block_workspace_bytes(H, q_rank, rank, heads, nope, rope, v_dim, prev_len))
    code = lib.moe_ds_attention_block_forward_f32(
        session._handle, _ptr(x), _ptr(q_a), _ptr(q_b), _ptr(kv_a), _ptr(kv_b), _ptr(o_w), _ptr(q_norm),
        _ptr(kv_norm), _ptr(prev_kv), _ptr(prev_pe), _ptr(cos),
        _ptr(sin), _ptr(next_kv), _ptr(next_pe), _ptr(out), H, q_rank, rank, heads, nope, rope, v_dim, prev_len,
        float(rms_eps), float(softmax_scale), _ptr(ws), ws.numel(), _stream())
    _check(code, "ds_attention_block_forward_f32")
    dev = _out_device(hidden)
    return out.to(dev), (next_kv.to(dev), next_pe.to(dev))


# ---------------------------------------------------------------------------
# Q4 (native/__init__.py:204-215, 4025-4155)
# ---------------------------------------------------------------------------

def native_q4_available() -> bool:
    return not _native_disabled() and _lib_or_none() is not None and torch.cuda.is_available()


def native_q4_load_error() -> Exception | None:
    _lib_or_none()
    return _LIB_ERROR


def q4_dequant_to_fp16(packed: torch.Tensor, scales: torch.Tensor, num_channels: int,
                       channel_size: int) -> torch.Tensor:
    _require(native_q4_available(), "Q4 dequant", _native_disabled())
    pk = _gpu(packed.reshape(-1), torch.uint8)
    sc = _gpu(scales.reshape(-1), torch.float16)
    n = int(num_channels) * int(channel_size)
    if pk.numel() * 2 < n or sc.numel() < int(num_channels):
        raise ValueError("packed / scales are too small for num_channels x channel_size")
    out = torch.empty((n,), dtype=torch.float16, device=pk.device)
    code = load_library().moe_q4_dequant_to_fp16(_ptr(pk), _ptr(sc), _ptr(out), int(num_channels),
                                                 int(channel_size), _stream())
    _check(code, "q4_dequant_to_fp16")
    return out.to(_out_device(packed))


def q4_dequant_many_to_fp16(items: list[tuple[torch.Tensor, torch.Tensor, int, int]]) -> list[torch.Tensor]:
    _require(native_q4_available(), "Q4 batch dequant", _native_disabled())
    if not items:
        return []
    keep, outs = [], []
    n = len(items)
    pk_ptrs, sc_ptrs, out_ptrs = (_P * n)(), (_P * n)(), (_P * n)()
    channels, sizes = (_I64 * n)(), (_I64 * n)()
    for i, (packed, scales, num_channels, channel_size) in enumerate(items):
        pk = _gpu(packed.reshape(-1), torch.uint8)
        sc = _gpu(scales.reshape(-1), torch.float16)
        elems = int(num_channels) * int(channel_size)
        if pk.numel() * 2 < elems or sc.numel() < int(num_channels):
            raise ValueError("packed / scales are too small for num_channels x channel_size")
        out = torch.empty((elems,), dtype=torch.float16, device=pk.device)
        keep += [pk, sc]
        outs.append(out)
        pk_ptrs[i], sc_ptrs[i], out_ptrs[i] = _ptr(pk), _ptr(sc), _ptr(out)
        channels[i], sizes[i] = int(num_channels), int(channel_size)
    code = load_library().moe_q4_dequant_many_to_fp16(pk_ptrs, sc_ptrs, out_ptrs, channels, sizes, n, _stream())
    if code != 0:
        raise RuntimeError(f"Native Q4 batch dequant failed with code {code}")
    return [o.to(_out_device(items[i][0])) for i, o in enumerate(outs)]


def q4_moe_selected_forward_u16(hidden: torch.Tensor, experts: list, route_weights: torch.Tensor, *,
                                hidden_size: int, intermediate_size: int) -> torch.Tensor:
    _require(native_q4_available(), "Q4 MoE selected forward", _native_disabled())
    if not experts:
        raise ValueError("experts must not be empty")
    x = _gpu(hidden.reshape(-1), torch.float16)
    if x.numel() != int(hidden_size):
        raise ValueError("hidden size mismatch")
    route = _gpu(route_weights.reshape(-1), torch.float32)
    if route.numel() != len(experts):
        raise ValueError("route weight count must match selected experts")
    dtypes = (torch.uint8, torch.float16) * 3
    tensors = [[_gpu(t.reshape(-1), dt) for t, dt in zip(item, dtypes)] for item in experts]
    table = torch.tensor([[int(item[j].data_ptr()) for item in tensors] for j in range(6)], dtype=torch.int64,
                         device=x.device)
    S = len(experts)
    out = torch.empty((int(hidden_size),), dtype=torch.float16, device=x.device)
    cols = [_P(int(table.data_ptr()) + 8 * S * j) for j in range(6)]
    code = load_library().moe_q4_moe_selected_forward_u16(_ptr(x), *cols, _ptr(route), _ptr(out), int(hidden_size),
                                                          int(intermediate_size), S, None, 0, _stream())
    if code != 0:
        raise RuntimeError(f"Native Q4 MoE selected forward failed with code {code}")
    return out.to(_out_device(hidden))


# ---------------------------------------------------------------------------
# row8 packed GEMV (native/__init__.py:1658-1668, 2108-2223)
# ---------------------------------------------------------------------------
_U16_STORAGE_CODES = {torch.float16: 0, torch.bfloat16: 1}


class _Row8PackCache:
    """Device-resident row8 packs keyed by the caller's cache key, bounded
    by PCKETLM_PACKED_GEMV_CACHE_MB (unset, unparsable or <= 0: no caching;
    PCKETLM_DISABLE_PACKED_GEMV_CACHE: no caching).  The least recently used
    packs leave first when a new pack would exceed the budget; a pack larger
    than the whole budget is returned without being kept.  The statistics
    keys are the ones the reference's callers read
    (native/__init__.py:2110-2193)."""

    def __init__(self) -> None:
        self._packs: dict[str, tuple[torch.Tensor, int, int]] = {}  # key -> (pack, bytes, last use)
        self._clock = 0
        self._bytes = 0
        self.counts = dict.fromkeys(("hits", "misses", "stores", "evictions"), 0)

    @staticmethod
    def budget() -> int:
        try:
            return max(0, int(os.environ.get("PCKETLM_PACKED_GEMV_CACHE_MB", ""))) << 20
        except ValueError:
            return 0

    def clear(self) -> None:
        self._packs.clear()
        self._bytes = 0
        self.counts = dict.fromkeys(self.counts, 0)

    def stats(self) -> dict[str, int | float]:
        return {**self.counts, "resident_count": len(self._packs), "resident_bytes": self._bytes,
                "resident_mb": round(self._bytes / (1 << 20), 4), "budget_bytes": self.budget()}

    def get(self, key: str, weight: torch.Tensor) -> torch.Tensor:
        self._clock += 1
        limit = 0 if _flag("PCKETLM_DISABLE_PACKED_GEMV_CACHE") else self.budget()
        entry = self._packs.get(key) if limit else None
        if entry is not None:
            self.counts["hits"] += 1
            self._packs[key] = (entry[0], entry[1], self._clock)
            return entry[0]
        self.counts["misses"] += 1
        packed = pack_weight_rows8(weight)
        size = packed.numel() * packed.element_size()
        if not limit or size > limit:
            return packed
        while self._packs and self._bytes + size > limit:
            stalest = min(self._packs, key=lambda k: self._packs[k][2])
            self._bytes -= self._packs.pop(stalest)[1]
            self.counts["evictions"] += 1
        self._packs[key] = (packed, size, self._clock)
        self._bytes += size
        self.counts["stores"] += 1
        return packed


_ROW8_CACHE = _Row8PackCache()


def native_fp16_packed_gemv_available() -> bool:
    return not _native_packed_gemv_disabled() and _lib_or_none() is not None and torch.cuda.is_available()


def reset_packed_gemv_cache() -> None:
    _ROW8_CACHE.clear()


def packed_gemv_cache_stats() -> dict[str, int | float]:
    return _ROW8_CACHE.stats()


def _u16_storage_dtype_code(dtype: torch.dtype) -> int:
    if dtype not in _U16_STORAGE_CODES:
        raise TypeError("native KV kernels require torch.float16 or torch.bfloat16 tensors")
    return _U16_STORAGE_CODES[dtype]


def pack_weight_rows8(weight: torch.Tensor) -> torch.Tensor:
    """[rows, cols] fp16/bf16 -> flat uint16 row8 layout [ceil(rows/8) * cols * 8],
    packed on the GPU and kept there (device of the result: the current CUDA device)."""
    _require(native_fp16_packed_gemv_available(), "packed GEMV", _native_packed_gemv_disabled())
    if weight.dtype not in {torch.float16, torch.bfloat16}:
        raise TypeError("pack_weight_rows8 requires torch.float16 or torch.bfloat16 weight")
    if weight.ndim != 2:
        raise ValueError("weight must have shape [rows, cols]")
    w = _gpu(weight).view(torch.uint16)
    rows, cols = int(w.shape[0]), int(w.shape[1])
    packed = torch.empty((((rows + 7) // 8) * cols * 8,), dtype=torch.uint16, device=w.device)
    code = load_library().moe_pack_u16_rows8(_ptr(w), _ptr(packed), rows, cols, _stream())
    if code != 0:
        raise RuntimeError(f"native_pack_u16_rows8 failed with code {code}")
    return packed


def cached_pack_weight_rows8(cache_key: str, weight: torch.Tensor) -> torch.Tensor:
    """pack_weight_rows8 through the process-wide LRU of device packs."""
    return _ROW8_CACHE.get(str(cache_key), weight)


def packed_gemv_rows8(hidden: torch.Tensor, packed_weight: torch.Tensor, *, rows: int, cols: int) -> torch.Tensor:
    _require(native_fp16_packed_gemv_available(), "packed GEMV", _native_packed_gemv_disabled())
    if hidden.dtype not in {torch.float16, torch.bfloat16}:
        raise TypeError("packed_gemv_rows8 requires torch.float16 or torch.bfloat16 hidden")
    if packed_weight.dtype != torch.uint16:
        raise TypeError("packed_weight must be a torch.uint16 tensor from pack_weight_rows8")
    x = _gpu(hidden.reshape(-1))
    if x.numel() != int(cols):
        raise ValueError("hidden length does not match packed weight column count")
    pk = _gpu(packed_weight)
    if pk.numel() != ((int(rows) + 7) // 8) * int(cols) * 8:
        raise ValueError("packed weight length does not match rows/cols")
    out = torch.empty((int(rows),), dtype=torch.float32, device=x.device)
    code = load_library().moe_packed_gemv_rows8(_ptr(x.view(torch.uint16)), _ptr(pk), _ptr(out), int(rows), int(cols),
                                                _u16_storage_dtype_code(x.dtype), _stream())
    if code != 0:
        raise RuntimeError(f"native_packed_gemv_rows8 failed with code {code}")
    return out.to(_out_device(hidden))


# ---------------------------------------------------------------------------
# 16-bit dense MoE (native/__init__.py:2465-2574)
# ---------------------------------------------------------------------------

def native_fp16_moe_available() -> bool:
    return not _native_moe_disabled() and _lib_or_none() is not None and torch.cuda.is_available()


def native_fp16_moe_error() -> Exception | None:
    _lib_or_none()
    return _LIB_ERROR


def moe_forward_fp16(hidden: torch.Tensor, router_weight: torch.Tensor, gate_weight: torch.Tensor,
                     up_weight: torch.Tensor, down_weight: torch.Tensor, *, top_k: int,
                     normalize_topk: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    _require(native_fp16_moe_available(), "fp16 MoE", _native_moe_disabled())
    tensors = [hidden, router_weight, gate_weight, up_weight, down_weight]
    if any(t.dtype != torch.float16 for t in tensors):
        raise TypeError("moe_forward_fp16 requires torch.float16 tensors")
    if hidden.ndim != 2:
        raise ValueError("hidden must have shape [seq_len, hidden_size]")
    if gate_weight.ndim != 3 or up_weight.ndim != 3 or down_weight.ndim != 3:
        raise ValueError("expert weights must be rank-3 [num_experts, rows, cols]")
    x, rw, g, u, d = (_gpu(t) for t in tensors)
    T, H = int(x.shape[0]), int(x.shape[1])
    E, I, k = int(rw.shape[0]), int(g.shape[1]), int(top_k)
    out = torch.empty((T, H), dtype=torch.float16, device=x.device)
    ids = torch.empty((T, k), dtype=torch.int64, device=x.device)
    wts = torch.empty((T, k), dtype=torch.float32, device=x.device)
    u16 = lambda t: _ptr(t.view(torch.uint16))  # noqa: E731
    code = load_library().moe_moe_forward_fp16(u16(x), u16(rw), u16(g), u16(u), u16(d), u16(out), _ptr(ids),
                                               _ptr(wts), T, H, E, k, I, 1 if normalize_topk else 0, None, 0,
                                               _stream())
    if code != 0:
        raise RuntimeError(f"native_moe_forward_fp16 failed with code {code}")
    dev = _out_device(hidden)
    return out.to(dev), ids.to(dev), wts.to(dev)


def moe_selected_forward_u16(hidden: torch.Tensor, gate_weight: torch.Tensor, up_weight: torch.Tensor,
                             down_weight: torch.Tensor, route_weights: torch.Tensor) -> torch.Tensor:
    _require(native_fp16_moe_available(), "fp16 MoE", _native_moe_disabled())
    dtype_code = _u16_storage_dtype_code(hidden.dtype)
    tensors = [hidden, gate_weight, up_weight, down_weight]
    if any(t.dtype != hidden.dtype for t in tensors):
        raise TypeError(f"moe_selected_forward_u16 requires all model tensors to share dtype {hidden.dtype}")
    if hidden.ndim != 2:
        raise ValueError("hidden must have shape [seq_len, hidden_size]")
    if gate_weight.ndim != 3 or up_weight.ndim != 3 or down_weight.ndim != 3:
        raise ValueError("selected expert weights must be rank-3")
    T, H = int(hidden.shape[0]), int(hidden.shape[1])
    S, I = int(gate_weight.shape[0]), int(gate_weight.shape[1])
    if route_weights.shape != (T, S):
        raise ValueError("route_weights must have shape [seq_len, selected_count]")
    x, g, u, d = (_gpu(t) for t in tensors)
    route = _gpu(route_weights, torch.float32)
    out = torch.empty((T, H), dtype=hidden.dtype, device=x.device)
    u16 = lambda t: _ptr(t.view(torch.uint16))  # noqa: E731
    code = load_library().moe_moe_selected_forward_u16(u16(x), u16(g), u16(u), u16(d), _ptr(route), u16(out), T, H,
                                                       S, I, dtype_code, None, 0, _stream())
    if code != 0:
        raise RuntimeError(f"native_moe_selected_forward_u16 failed with code {code}")
    return out.to(_out_device(hidden))

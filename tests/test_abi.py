"""The C-ABI library loads on the CPU and exports every symbol that
include/*.h declares; the Python bridge binds exactly those symbols.
No compute calls (no GPU here)."""

import ctypes
import re
from pathlib import Path

from pocketlm_b200 import native

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(moe_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    from pocketlm_b200 import build

    build.build()
    lib = ctypes.CDLL(str(native._LIB_PATH))
    declared = _declared()
    assert len(declared) >= 25
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_bridge_binds_the_declared_symbols():
    assert set(native.library_symbols()) == _declared()
    lib = native.load_library()
    assert lib.moe_b200_abi_version() == 1


def test_bridge_refuses_to_run_without_a_gpu(monkeypatch):
    import pytest
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    assert native.native_fp8_linear_available() is False
    with pytest.raises(RuntimeError, match="unavailable"):
        native.fp8_e4m3_block_linear_f32(torch.zeros((4, 4), dtype=torch.uint8), torch.ones((1, 1)),
                                         torch.zeros((1, 4)))


def test_kill_switch_marks_unavailable(monkeypatch):
    monkeypatch.setenv("PCKETLM_DISABLE_NATIVE_FP8_LINEAR", "1")
    assert native.native_fp8_linear_available() is False
    monkeypatch.setenv("PCKETLM_DISABLE_NATIVE_DS_ROUTER", "1")
    assert native.native_ds_router_available() is False

"""Row8 packed-GEMV artifacts (pocketlm_b200/row8_artifact.py) on an artifact
written by the reference's own packer (tests/golden/row8_artifact, made by
tests/golden/make_golden.py with tools/pack_weights_row8.py)."""

import json
import shutil
from pathlib import Path

import pytest
import torch

from pocketlm_b200 import native
from pocketlm_b200.row8_artifact import ROW8_FORMAT, Row8Artifact, row8_packed_elements

ART = Path(__file__).resolve().parent / "golden" / "row8_artifact"


def source_tensors() -> dict[str, torch.Tensor]:
    """The fixture's matrices, regenerated as make_golden.py's row8_source_tensors() draws them."""
    gen = torch.Generator().manual_seed(808)
    return {
        "model.layers.0.mlp.experts.0.gate_proj.weight": (torch.randn((20, 48), generator=gen) * 0.5).half(),
        "model.layers.0.mlp.experts.0.down_proj.weight": (torch.randn((13, 40), generator=gen) * 0.5).bfloat16(),
        "model.layers.0.self_attn.o_proj.weight": (torch.randn((8, 16), generator=gen)).half(),
    }


def unpack(packed: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Row8 layout [ceil(rows/8)][cols][8] back to [rows, cols] uint16."""
    blocks = packed.cpu().reshape(-1, cols, 8)
    return blocks.permute(0, 2, 1).reshape(-1, cols)[:rows]


def test_artifact_loads_the_packed_layout():
    art = Row8Artifact(ART)
    src = source_tensors()
    got = art.load(list(src), device="cpu")
    assert set(got) == set(src)
    for name, w in src.items():
        packed, entry = got[name]
        rows, cols = w.shape
        assert packed.dtype == torch.uint16 and packed.numel() == row8_packed_elements(rows, cols)
        assert entry["dtype"] == ("BF16" if w.dtype == torch.bfloat16 else "F16")
        assert torch.equal(unpack(packed, rows, cols), w.view(torch.uint16))
        # the padding rows of the last block are zero
        assert not packed.reshape(-1, cols, 8)[-1, :, rows % 8 or 8:].to(torch.int32).any()
    one, _ = art.load_one("model.layers.0.self_attn.o_proj.weight", device="cpu")
    assert torch.equal(one, got["model.layers.0.self_attn.o_proj.weight"][0])


def test_artifact_checks(tmp_path):
    with pytest.raises(FileNotFoundError):
        Row8Artifact(tmp_path)
    with pytest.raises(KeyError):
        Row8Artifact(ART).entry("model.layers.0.input_layernorm.weight")  # 1-D: the packer skipped it
    bad = tmp_path / "bad"
    shutil.copytree(ART, bad)
    manifest = json.loads((bad / "row8_manifest.json").read_text(encoding="utf-8"))
    manifest["format"] = "other"
    (bad / "row8_manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="unsupported row8 artifact format"):
        Row8Artifact(bad)
    manifest["format"] = ROW8_FORMAT
    name = "model.layers.0.self_attn.o_proj.weight"
    manifest["tensors"][name]["nbytes"] = 2
    (bad / "row8_manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="expected"):
        Row8Artifact(bad).entry(name)


@pytest.mark.gpu
def test_artifact_feeds_the_packed_gemv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    src = source_tensors()
    got = Row8Artifact(ART).load(list(src), device="cuda")
    for name, w in src.items():
        packed, _entry = got[name]
        assert packed.is_cuda
        rows, cols = w.shape
        x = torch.randn((cols,), generator=torch.Generator().manual_seed(rows)).to(w.dtype)
        out = native.packed_gemv_rows8(x.cuda(), packed, rows=rows, cols=cols)
        want = w.float() @ x.float()
        assert torch.allclose(out.cpu(), want, rtol=1e-4, atol=1e-4)
        # the same bytes this library's own GPU packer writes
        assert torch.equal(native.pack_weight_rows8(w.cuda()).cpu(), packed.cpu())

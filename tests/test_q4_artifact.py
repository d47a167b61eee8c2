"""Q4 artifacts (pocketlm_b200/q4_artifact.py) on an artifact written by the
reference's own converter (tests/golden/q4_artifact, made by
tests/golden/make_golden.py with core/model_import/q4_quantize.py)."""

import json
import shutil
from pathlib import Path

import pytest
import torch

from pocketlm_b200 import synth
from pocketlm_b200.q4_artifact import Q4_FORMAT, Q4Artifact, load_q4_layer, safetensors_index

ART = Path(__file__).resolve().parent / "golden" / "q4_artifact"
CFG = synth.MixtralQ4Config("q4-tiny", hidden=128, inter=256, n_experts=4, top_k=2)


def source_tensors() -> dict[str, torch.Tensor]:
    """The fixture's checkpoint, regenerated as make_golden.py's q4_source_tensors() draws it."""
    gen = torch.Generator().manual_seed(4444)
    t = {"model.layers.0.block_sparse_moe.gate.weight":
         (torch.randn((CFG.n_experts, CFG.hidden), generator=gen) * 0.02).bfloat16()}
    for e in range(CFG.n_experts):
        for w, shape in (("w1", (CFG.inter, CFG.hidden)), ("w2", (CFG.hidden, CFG.inter)),
                         ("w3", (CFG.inter, CFG.hidden))):
            t[f"model.layers.0.block_sparse_moe.experts.{e}.{w}.weight"] = (
                torch.randn(shape, generator=gen) * 0.02).bfloat16()
    return t


def _check_layer(got, src):
    for e in range(CFG.n_experts):
        for w, packed, scales in (("w1", got.gate_p, got.gate_s), ("w3", got.up_p, got.up_s),
                                  ("w2", got.down_p, got.down_s)):
            want_p, want_s = synth.quantize_q4_rows(src[f"model.layers.0.block_sparse_moe.experts.{e}.{w}.weight"])
            assert torch.equal(packed[e].cpu(), want_p), (e, w)
            assert torch.equal(scales[e].cpu().view(torch.int16), want_s.view(torch.int16)), (e, w)


def test_layer_loads_the_reference_codes():
    src = source_tensors()
    got = load_q4_layer(Q4Artifact(ART), 0, CFG, device="cpu")
    _check_layer(got, src)
    # the router comes back dequantized to fp16, as the reference's loader returns it
    p, s = synth.quantize_q4_rows(src["model.layers.0.block_sparse_moe.gate.weight"])
    codes = torch.stack([p.to(torch.int16) & 0x0F, p.to(torch.int16) >> 4], 1).reshape(-1)
    codes = torch.where(codes >= 8, codes - 16, codes).float().reshape(CFG.n_experts, CFG.hidden)
    want = (codes * s.float()[:, None]).to(torch.float16)
    assert got.router_weight.dtype == torch.float16
    assert torch.equal(got.router_weight.view(torch.int16), want.view(torch.int16))


def test_safetensors_index_and_manifest():
    art = Q4Artifact(ART)
    name = "model.layers.0.block_sparse_moe.experts.2.w2.weight"
    (cpath, coff, clen), (spath, soff, slen) = art.locate(name)
    assert cpath.name.endswith(".q4.safetensors") and spath.name.endswith(".scales.safetensors")
    assert clen == CFG.hidden * CFG.inter // 2 and slen == 2 * CFG.hidden
    idx = safetensors_index(cpath)
    assert idx[name][2] == coff and idx[name][0] == "U8"
    with open(cpath, "rb") as f:
        f.seek(coff)
        raw = f.read(clen)
    want, _ = synth.quantize_q4_rows(source_tensors()[name])
    assert raw == bytes(want.numpy().tobytes())


def test_artifact_checks(tmp_path):
    with pytest.raises(FileNotFoundError):
        Q4Artifact(tmp_path)
    with pytest.raises(KeyError):
        Q4Artifact(ART).entry("model.layers.1.block_sparse_moe.gate.weight")
    bad = tmp_path / "bad"
    shutil.copytree(ART, bad)
    manifest = json.loads((bad / "q4_manifest.json").read_text(encoding="utf-8"))
    manifest["format"] = "other"
    (bad / "q4_manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="unsupported Q4 artifact format"):
        Q4Artifact(bad)
    assert Q4_FORMAT == "pcketlm-q4"
    wrong = synth.MixtralQ4Config("wrong", hidden=CFG.hidden, inter=2 * CFG.inter, n_experts=CFG.n_experts, top_k=2)
    with pytest.raises(ValueError, match="expected"):
        load_q4_layer(Q4Artifact(ART), 0, wrong, device="cpu")


@pytest.mark.gpu
def test_layer_uploads_to_the_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    got = load_q4_layer(Q4Artifact(ART), 0, CFG, device="cuda")
    assert got.gate_p.is_cuda and got.router_weight.is_cuda
    _check_layer(got, source_tensors())

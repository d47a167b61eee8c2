"""The FP8 pack loader (pocketlm_b200/fp8_pack.py) on a pack written by the
reference's own writer (tests/golden/fp8_pack_tiny, made by
tests/golden/make_golden.py with tools/pack_fp8.py and 96 KiB pack files, so
every expert's down projection sits in the next file), and the native
pack-file reader (moe_read_spans / moe_read_tensor_bytes)."""

import hashlib
import json
import shutil
from pathlib import Path

import pytest
import torch

from pocketlm_b200 import native, synth
from pocketlm_b200.fp8_pack import FORMAT, Fp8Pack, default_pack_dir, load_fp8_layer

PACK = Path(__file__).resolve().parent / "golden" / "fp8_pack_tiny"
EXPECTED = json.loads((PACK / "expected.json").read_text(encoding="utf-8"))
CFG = synth.DsMoEConfig("pack-tiny", hidden=EXPECTED["config"]["hidden"], inter=EXPECTED["config"]["inter"],
                        n_routed=EXPECTED["config"]["n_routed"], top_k=2, n_group=2, topk_group=1, route_scale=2.5)


def _sha(*tensors):
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().cpu().contiguous()
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.uint8 else t.numpy().tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def source():
    layer = synth.make_fp8_layer(CFG, seed=EXPECTED["seed"])
    assert _sha(layer.router_weight, layer.bias, layer.w13, layer.s13, layer.w2, layer.s2) == EXPECTED["sha_layer"], \
        "the synthetic generator changed; regenerate tests/golden/fp8_pack_tiny"
    return layer


def test_layer_loads_byte_for_byte(source):
    got = load_fp8_layer(Fp8Pack(PACK), 0, CFG, device="cpu")
    assert got.is_full
    assert torch.equal(got.router_weight.view(torch.int16), source.router_weight.view(torch.int16))
    assert torch.equal(got.bias, source.bias)
    for name in ("w13", "s13", "w2", "s2"):
        assert torch.equal(getattr(got, name), getattr(source, name)), name


def test_partial_layer_holds_the_named_experts(source):
    got = load_fp8_layer(Fp8Pack(PACK), 0, CFG, experts=[3, 1], device="cpu")
    assert got.slots == {3: 0, 1: 1, CFG.n_routed: 2}
    for e in (3, 1, CFG.n_routed):
        for a, b in zip(got.expert(e), source.expert(e)):
            assert torch.equal(a, b)


def test_expert_ranges_follow_the_writer_order():
    pack = Fp8Pack(PACK)
    names = pack.expert_tensor_names(0, 2, CFG.n_routed)
    assert names == [f"model.layers.0.mlp.experts.2.{p}.weight{s}" for p in ("gate_proj", "up_proj", "down_proj")
                     for s in ("", "_scale_inv")]
    ranges = pack.ranges(names)
    assert len(ranges) == 2  # gate and up (+ scales) in one file, down (+ scale) in the next
    gate, gate_s = ranges[0].tensor_slices[names[0]], ranges[0].tensor_slices[names[1]]
    assert gate == (0, CFG.inter * CFG.hidden) and gate_s[0] == gate[1]
    assert ranges[1].tensor_slices[names[4]][0] == 0
    shared = pack.expert_tensor_names(0, CFG.n_routed, CFG.n_routed)
    assert shared[0] == "model.layers.0.mlp.shared_experts.gate_proj.weight"


def test_native_reads_match_file_reads(tmp_path):
    data = bytes(range(256)) * 40000  # ~10 MB: more than one 8 MiB piece
    f = tmp_path / "blob.bin"
    f.write_bytes(data)
    spans = [(0, 17), (3, 9 << 20), (len(data) - 5, 5), (100, 0)]
    outs = [torch.empty((n,), dtype=torch.uint8) for _o, n in spans]
    native.read_spans(f, spans, outs, threads=3)
    for (o, n), out in zip(spans, outs):
        assert bytes(out.numpy().tobytes()) == data[o:o + n]
    one = torch.empty((1000,), dtype=torch.uint8)
    native.native_read_tensor_bytes(f, 12345, 1000, one)
    assert bytes(one.numpy().tobytes()) == data[12345:13345]


def test_native_reader_errors(tmp_path):
    f = tmp_path / "small.bin"
    f.write_bytes(b"x" * 64)
    lib = native.load_library()
    buf = torch.empty((128,), dtype=torch.uint8)
    ptr = native._P(int(buf.data_ptr()))
    assert lib.moe_read_tensor_bytes(None, 0, 1, ptr) == 1
    assert lib.moe_read_tensor_bytes(str(tmp_path / "missing.bin").encode(), 0, 1, ptr) == 2
    assert lib.moe_read_tensor_bytes(str(f).encode(), 60, 8, ptr) == 3  # ends past the file
    with pytest.raises(OSError):
        native.native_read_tensor_bytes(f, 0, 128, buf)
    with pytest.raises(ValueError, match="byte size"):
        native.native_read_tensor_bytes(f, 0, 8, buf)


def test_manifest_checks(tmp_path, monkeypatch):
    with pytest.raises(FileNotFoundError, match="manifest not found"):
        Fp8Pack(tmp_path)
    bad = tmp_path / "bad"
    shutil.copytree(PACK, bad)
    manifest = json.loads((bad / "pack_manifest.json").read_text(encoding="utf-8"))
    manifest["format"] = "something-else"
    (bad / "pack_manifest.json").write_text(json.dumps(manifest), encoding="utf-8")
    with pytest.raises(ValueError, match="unsupported FP8 pack format"):
        Fp8Pack(bad)
    assert FORMAT == "pcketlm-fp8-pack-v1"
    with pytest.raises(KeyError, match="not present in FP8 pack manifest"):
        Fp8Pack(PACK).entry("model.layers.9.mlp.gate.weight")
    wrong = synth.DsMoEConfig("wrong", hidden=CFG.hidden, inter=2 * CFG.inter, n_routed=CFG.n_routed, top_k=2,
                              n_group=2, topk_group=1, route_scale=2.5)
    with pytest.raises(ValueError, match="expected"):
        load_fp8_layer(Fp8Pack(PACK), 0, wrong, device="cpu")
    monkeypatch.setenv("PCKETLM_FP8_PACK_DIR", str(PACK))
    assert default_pack_dir(tmp_path) == PACK.resolve()
    monkeypatch.delenv("PCKETLM_FP8_PACK_DIR")
    assert default_pack_dir(tmp_path) == (tmp_path / "artifacts" / "fp8_pack").resolve()


@pytest.mark.gpu
def test_layer_uploads_to_the_gpu_byte_for_byte(source):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    got = load_fp8_layer(Fp8Pack(PACK), 0, CFG, experts=[0, 2, 3], device="cuda")
    assert got.w13.is_cuda
    for e in (0, 2, 3, CFG.n_routed):
        for a, b in zip(got.expert(e), source.expert(e)):
            assert torch.equal(a.cpu(), b)

"""DeepSeek-V3 MoE layers from the reference's lossless FP8 pack, straight into HBM.

The pack ("pcketlm-fp8-pack-v1") is the reference's on-disk form of an FP8
checkpoint: `pack_manifest.json` plus `pack_NNNN.bin` files that hold the
safetensors payloads byte for byte, ordered by (layer, group, expert,
projection, tensor, weight before scale) (writer tools/pack_fp8.py:277-283,
manifest entries :316-336; reader src/pcketlm/core/runtime/fp8_pack.py:57-243).
One expert's six tensors -- gate, up and down e4m3 codes, each followed by
its 128x128 fp32 block scales -- are therefore adjacent, and the expert
path's caller reads them as one span (`_read_packed_mlp_full_tensors`,
core/runtime/fp8_source.py:4709-4792) into host tensors.

`load_fp8_layer` reads every expert of a layer the same way -- one byte
range per pack file, pread by several threads (`moe_read_spans`) into a
pinned staging buffer -- copies each range to the device once (two staging
buffers, so the next expert is read while the last one is in flight) and
places the six tensors into the layer's expert-major HBM tensors with device
copies.  The result is the `synth.Fp8MoELayer` container that
`DsMoELayerGPU` and `ExpertParallelLayer` take (a partial layer when
`experts` names a subset: an expert-parallel rank reads only its own).
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from pathlib import Path

import torch

from pocketlm_b200 import native, synth

FORMAT = "pcketlm-fp8-pack-v1"

_FP8 = {"F8_E4M3", "F8_E4M3FN"}
_WIDTH = {"F8_E4M3": 1, "F8_E4M3FN": 1, "U8": 1, "BF16": 2, "F16": 2, "F32": 4}
_TORCH = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}
_PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def default_pack_dir(model_dir: str | Path) -> Path:
    """The pack directory of a model directory: $PCKETLM_FP8_PACK_DIR when set,
    else <model_dir>/artifacts/fp8_pack (fp8_pack.py:319-324)."""
    override = os.environ.get("PCKETLM_FP8_PACK_DIR", "").strip()
    if override:
        return Path(override).resolve()
    return Path(model_dir).resolve() / "artifacts" / "fp8_pack"


@dataclass(frozen=True)
class PackRange:
    """One contiguous byte range of a pack file and the tensors inside it
    (name -> (offset within the range, byte length))."""

    path: Path
    byte_offset: int
    byte_length: int
    tensor_slices: dict[str, tuple[int, int]]


class Fp8Pack:
    """A pack's manifest, with the reference reader's lookup rules."""

    def __init__(self, pack_dir: str | Path):
        self.pack_dir = Path(pack_dir).resolve()
        manifest_path = self.pack_dir / "pack_manifest.json"
        if not manifest_path.exists():
            raise FileNotFoundError(f"FP8 pack manifest not found: {manifest_path}")
        self.manifest = json.loads(manifest_path.read_text(encoding="utf-8"))
        fmt = self.manifest.get("format")
        if fmt != FORMAT:
            raise ValueError(f"unsupported FP8 pack format {fmt!r} (expected {FORMAT!r})")
        self.tensors: dict[str, dict] = dict(self.manifest.get("tensors") or {})

    @classmethod
    def for_model_dir(cls, model_dir: str | Path) -> "Fp8Pack":
        return cls(default_pack_dir(model_dir))

    def entry(self, name: str) -> dict:
        try:
            return self.tensors[name]
        except KeyError as exc:
            raise KeyError(f"Tensor {name} is not present in FP8 pack manifest.") from exc

    def path(self, pack_file_index: int) -> Path:
        return self.pack_dir / f"pack_{int(pack_file_index):04d}.bin"

    def expert_tensor_names(self, layer: int, expert: int, n_routed: int) -> list[str]:
        """gate, gate scale, up, up scale, down, down scale of one expert
        (expert == n_routed: the shared expert)."""
        prefix = (f"model.layers.{int(layer)}.mlp.experts.{int(expert)}" if expert < n_routed
                  else f"model.layers.{int(layer)}.mlp.shared_experts")
        names = []
        for proj in _PROJECTIONS:
            weight = f"{prefix}.{proj}.weight"
            scale = self.entry(weight).get("scale_name")
            if not scale:
                raise ValueError(f"{weight} has no block-scale companion in the FP8 pack")
            names += [weight, str(scale)]
        return names

    def ranges(self, names: list[str]) -> list[PackRange]:
        """The tensors grouped by pack file, one range per file from the first
        tensor's start to the last one's end (the writer keeps an expert's
        tensors adjacent; a range that also covers other bytes reads them too)."""
        if not names:
            raise ValueError("Packed tensor span requires at least one tensor name.")
        by_file: dict[int, list[tuple[str, dict]]] = {}
        for name in names:
            e = self.entry(name)
            by_file.setdefault(int(e["pack_file_index"]), []).append((name, e))
        out = []
        for index in sorted(by_file):
            group = by_file[index]
            start = min(int(e["byte_offset"]) for _n, e in group)
            end = max(int(e["byte_offset"]) + int(e["byte_length"]) for _n, e in group)
            out.append(PackRange(self.path(index), start, end - start,
                                 {n: (int(e["byte_offset"]) - start, int(e["byte_length"])) for n, e in group}))
        return out

    def read_host(self, names: list[str], *, pin: bool = False,
                  buffer: torch.Tensor | None = None) -> tuple[torch.Tensor, dict[str, tuple[int, int]]]:
        """The tensors' bytes in one host buffer (`buffer` when large enough;
        pinned when `pin`), plus name -> (offset, length) in it."""
        ranges = self.ranges(names)
        total = sum(r.byte_length for r in ranges)
        if buffer is None or buffer.numel() < total:
            buffer = torch.empty((max(total, 1),), dtype=torch.uint8, pin_memory=pin)
        slices: dict[str, tuple[int, int]] = {}
        base = 0
        by_path: dict[Path, tuple[list, list]] = {}
        for r in ranges:
            spans, outs = by_path.setdefault(r.path, ([], []))
            spans.append((r.byte_offset, r.byte_length))
            outs.append(buffer[base:base + r.byte_length])
            for n, (off, ln) in r.tensor_slices.items():
                slices[n] = (base + off, ln)
            base += r.byte_length
        for path, (spans, outs) in by_path.items():
            native.read_spans(path, spans, outs)
        return buffer, slices

    def read_tensor(self, name: str) -> torch.Tensor:
        """One tensor as a host tensor of its manifest dtype and shape."""
        e = self.entry(name)
        buf, slices = self.read_host([name])
        off, ln = slices[name]
        return _typed(buf[off:off + ln], str(e["dtype"]), [int(v) for v in e.get("shape", [])], name)


def _typed(raw: torch.Tensor, dtype: str, shape: list[int], name: str) -> torch.Tensor:
    if dtype in _FP8 or dtype == "U8":
        t = raw
    elif dtype in _TORCH:
        if raw.storage_offset() % _WIDTH[dtype]:
            raw = raw.clone()  # a payload that starts off its element alignment in the staging buffer
        t = raw.view(_TORCH[dtype])
    else:
        raise ValueError(f"{name}: unsupported dtype {dtype} in the FP8 pack")
    return t.reshape(shape)


def _check_entry(pack: Fp8Pack, name: str, dtypes: set[str], shape: tuple[int, ...]) -> dict:
    e = pack.entry(name)
    dtype = str(e["dtype"])
    got = tuple(int(v) for v in e.get("shape", []))
    if dtype not in dtypes or got != shape:
        raise ValueError(f"{name}: {dtype} {list(got)} in the FP8 pack, expected one of {sorted(dtypes)} "
                         f"{list(shape)}")
    width = _WIDTH[dtype]
    n = 1
    for v in shape:
        n *= v
    if int(e["byte_length"]) != n * width:
        raise ValueError(f"{name}: {e['byte_length']} bytes in the FP8 pack, expected {n * width}")
    return e


def load_fp8_layer(pack: Fp8Pack, layer: int, cfg: synth.DsMoEConfig, *, experts: list[int] | None = None,
                   device: torch.device | str | None = None) -> synth.Fp8MoELayer:
    """Layer `layer` of the pack -- router, routed experts (`experts`, all by
    default) and the shared expert -- as a synth.Fp8MoELayer on `device`,
    every byte as the pack holds it (scales as fp32).  Shapes and dtypes are
    checked against `cfg`; a missing tensor raises KeyError."""
    device = torch.device(device if device is not None else native._device())
    H, I = cfg.hidden, cfg.inter
    gs, ds = cfg.gate_scale_shape, cfg.down_scale_shape
    routed = list(range(cfg.n_routed)) if experts is None else [int(e) for e in experts]
    if any(e < 0 or e >= cfg.n_routed for e in routed) or len(set(routed)) != len(routed):
        raise ValueError("experts must be distinct routed expert ids")
    ids = routed + [cfg.n_routed]
    prefix = f"model.layers.{int(layer)}.mlp.gate"
    _check_entry(pack, f"{prefix}.weight", {"BF16", "F16", "F32"}, (cfg.n_routed, H))
    router_weight = pack.read_tensor(f"{prefix}.weight").to(device)
    bias = None
    if f"{prefix}.e_score_correction_bias" in pack.tensors:
        _check_entry(pack, f"{prefix}.e_score_correction_bias", {"BF16", "F16", "F32"}, (cfg.n_routed,))
        bias = pack.read_tensor(f"{prefix}.e_score_correction_bias").float().to(device)
    E1 = len(ids)
    w13 = torch.empty((E1, 2, I, H), dtype=torch.uint8, device=device)
    s13 = torch.empty((E1, 2, *gs), dtype=torch.float32, device=device)
    w2 = torch.empty((E1, H, I), dtype=torch.uint8, device=device)
    s2 = torch.empty((E1, *ds), dtype=torch.float32, device=device)
    cuda = device.type == "cuda"
    host = [None, None]           # two pinned staging buffers (cuda) ...
    staged = [None, None]         # ... their device copies
    done = [None, None]           # and the events after which a buffer may be refilled
    stream = torch.cuda.current_stream(device) if cuda else None
    for slot, e in enumerate(ids):
        names = pack.expert_tensor_names(layer, e, cfg.n_routed)
        shapes = [(I, H), gs, (I, H), gs, (H, I), ds]
        dtypes = [_FP8, {"F32", "BF16", "F16"}] * 3
        entries = [_check_entry(pack, n, dt, sh) for n, dt, sh in zip(names, dtypes, shapes)]
        b = slot % 2
        if cuda and done[b] is not None:
            done[b].synchronize()  # the copy out of this staging buffer has finished
        buf, slices = pack.read_host(names, pin=cuda, buffer=host[b])
        host[b] = buf
        used = max(off + ln for off, ln in slices.values())
        if cuda:
            if staged[b] is None or staged[b].numel() < used:
                staged[b] = torch.empty((buf.numel(),), dtype=torch.uint8, device=device)
            staged[b][:used].copy_(buf[:used], non_blocking=True)
            src = staged[b]
        else:
            src = buf
        views = [_typed(src[off:off + ln], str(ent["dtype"]), list(sh), n)
                 for n, ent, sh in zip(names, entries, shapes) for off, ln in [slices[n]]]
        w13[slot, 0].copy_(views[0].reshape(I, H))
        s13[slot, 0].copy_(views[1].float())
        w13[slot, 1].copy_(views[2].reshape(I, H))
        s13[slot, 1].copy_(views[3].float())
        w2[slot].copy_(views[4].reshape(H, I))
        s2[slot].copy_(views[5].float())
        if cuda:
            ev = torch.cuda.Event()
            ev.record(stream)
            done[b] = ev
    if cuda:
        torch.cuda.current_stream(device).synchronize()
    slots = None if experts is None else {e: i for i, e in enumerate(ids)}
    return synth.Fp8MoELayer(cfg, router_weight, bias, w13, s13, w2, s2, slots)

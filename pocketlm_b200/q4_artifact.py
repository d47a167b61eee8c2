"""Q4 streaming artifacts read straight into HBM as a Mixtral-shape Q4 layer.

The reference converts a checkpoint's floating tensors to its Q4 scheme
("per-channel-symmetric-v1": signed int4 codes two per byte, even index in
the low nibble, one fp16 scale amax/7 per output row) and writes, per source
shard, `<shard>.q4.safetensors` (the packed codes) and
`<shard>.scales.safetensors` (the scales) plus `q4_manifest.json` (format
"pcketlm-q4"; writer core/model_import/q4_quantize.py:94-174, quantizer
:47-75).  Its runtime finds a tensor through the manifest and reads both
payloads from the shards (core/runtime/tensor_loader.py:362-409, 631-700),
dequantizing the non-expert tensors (the router among them) to fp16
(:571-598).

`load_q4_layer` reads one layer's experts the same way -- the byte ranges
from the shards' safetensors headers, pread by several threads
(`moe_read_spans`) into pinned memory, one upload per expert -- into the
expert-major tensors of `synth.Q4MoELayer`, which `Q4MoELayerGPU` takes as
they are (the bytes are the reference's, unchanged).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import torch

from pocketlm_b200 import native, synth

Q4_FORMAT = "pcketlm-q4"
Q4_MANIFEST_NAME = "q4_manifest.json"

# Mixtral (HF) names: w1 = gate, w3 = up, w2 = down
_EXPERT = "model.layers.{layer}.block_sparse_moe.experts.{expert}.{w}.weight"
_ROUTER = "model.layers.{layer}.block_sparse_moe.gate.weight"


def _unpack_int4(packed: torch.Tensor, count: int) -> torch.Tensor:
    """Bytes -> `count` signed int4 codes (even index in the low nibble)."""
    b = packed.reshape(-1).to(torch.int16)
    codes = torch.stack([b & 0x0F, b >> 4], dim=1).reshape(-1)[:count]
    return torch.where(codes >= 8, codes - 16, codes).to(torch.int8)


def safetensors_index(path: str | Path) -> dict[str, tuple[str, list[int], int, int]]:
    """name -> (dtype, shape, absolute byte offset, byte length) from a
    safetensors file's header (8-byte little-endian header size, JSON header,
    payload offsets relative to its end)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n).decode("utf-8"))
    base = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        start, end = (int(v) for v in meta["data_offsets"])
        out[name] = (str(meta["dtype"]), [int(v) for v in meta["shape"]], base + start, end - start)
    return out


class Q4Artifact:
    """One Q4 artifact directory (manifest, code shards, scale shards)."""

    def __init__(self, artifact_dir: str | Path):
        self.artifact_dir = Path(artifact_dir).resolve()
        path = self.artifact_dir / Q4_MANIFEST_NAME
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.manifest = json.loads(path.read_text(encoding="utf-8"))
        fmt = self.manifest.get("format")
        if fmt != Q4_FORMAT:
            raise ValueError(f"unsupported Q4 artifact format {fmt!r} (expected {Q4_FORMAT!r})")
        self.tensors: dict[str, dict] = dict(self.manifest.get("tensors") or {})
        self._index: dict[str, dict] = {}

    def entry(self, name: str) -> dict:
        if name not in self.tensors:
            raise KeyError(name)
        return self.tensors[name]

    def _shard(self, shard: str) -> dict:
        if shard not in self._index:
            self._index[shard] = safetensors_index(self.artifact_dir / shard)
        return self._index[shard]

    def locate(self, name: str) -> tuple[tuple[Path, int, int], tuple[Path, int, int]]:
        """((code shard, offset, length), (scale shard, offset, length)) of one tensor."""
        e = self.entry(name)
        out = []
        for key, want in (("q4_shard", ("U8",)), ("scale_shard", ("F16",))):
            shard = str(e[key])
            if name not in self._shard(shard):
                raise KeyError(f"{name} is missing from {shard}")
            dtype, _shape, off, nbytes = self._shard(shard)[name]
            if dtype not in want:
                raise ValueError(f"{name}: {dtype} in {shard}, expected {want[0]}")
            out.append((self.artifact_dir / shard, off, nbytes))
        return out[0], out[1]

    def read(self, names: list[str], *, pin: bool = False,
             buffer: torch.Tensor | None = None) -> tuple[torch.Tensor, dict[str, tuple[tuple[int, int], tuple[int, int]]]]:
        """Codes and scales of the tensors in one host buffer, plus name ->
        ((code offset, length), (scale offset, length)) in it."""
        parts = {n: self.locate(n) for n in names}
        total = sum(c[2] + s[2] for c, s in parts.values())
        if buffer is None or buffer.numel() < total:
            buffer = torch.empty((max(total, 1),), dtype=torch.uint8, pin_memory=pin)
        by_path: dict[Path, tuple[list, list]] = {}
        where = {}
        base = 0
        for n, (c, s) in parts.items():
            slots = []
            for path, off, nbytes in (c, s):
                spans, outs = by_path.setdefault(path, ([], []))
                spans.append((off, nbytes))
                outs.append(buffer[base:base + nbytes])
                slots.append((base, nbytes))
                base += nbytes
            where[n] = (slots[0], slots[1])
        for path, (spans, outs) in by_path.items():
            native.read_spans(path, spans, outs)
        return buffer, where

    def dequantize(self, name: str) -> torch.Tensor:
        """A Q4 tensor back to fp16 on the host, as the reference's loader does
        (codes x fp32(scale), rounded to fp16; tensor_loader.py:571-581)."""
        e = self.entry(name)
        shape = [int(v) for v in e["shape"]]
        buf, where = self.read([name])
        (co, cn), (so, sn) = where[name]
        rows = shape[0] if shape else 1
        count = 1
        for v in shape:
            count *= v
        codes = _unpack_int4(buf[co:co + cn], count).to(torch.float32).reshape(rows, -1)
        scales = buf[so:so + sn].clone().view(torch.float16).float().reshape(-1, 1)
        return (codes * scales).reshape(shape).to(torch.float16)


def load_q4_layer(art: Q4Artifact, layer: int, cfg: synth.MixtralQ4Config, *,
                  device: torch.device | str | None = None) -> synth.Q4MoELayer:
    """Layer `layer`'s router (dequantized to fp16) and experts as a
    synth.Q4MoELayer on `device`; shapes are checked against `cfg`."""
    device = torch.device(device if device is not None else native._device())
    E, H, I = cfg.n_experts, cfg.hidden, cfg.inter
    router_name = _ROUTER.format(layer=int(layer))
    if [int(v) for v in art.entry(router_name)["shape"]] != [E, H]:
        raise ValueError(f"{router_name}: shape {art.entry(router_name)['shape']}, expected {[E, H]}")
    router_weight = art.dequantize(router_name).to(device)
    gate_p = torch.empty((E, I * H // 2), dtype=torch.uint8, device=device)
    up_p = torch.empty_like(gate_p)
    down_p = torch.empty((E, H * I // 2), dtype=torch.uint8, device=device)
    gate_s = torch.empty((E, I), dtype=torch.float16, device=device)
    up_s = torch.empty_like(gate_s)
    down_s = torch.empty((E, H), dtype=torch.float16, device=device)
    cuda = device.type == "cuda"
    host, staged, done = [None, None], [None, None], [None, None]
    for e in range(E):
        names = [_EXPERT.format(layer=int(layer), expert=e, w=w) for w in ("w1", "w3", "w2")]
        for n, shape in zip(names, ([I, H], [I, H], [H, I])):
            if [int(v) for v in art.entry(n)["shape"]] != shape:
                raise ValueError(f"{n}: shape {art.entry(n)['shape']}, expected {shape}")
        b = e % 2
        if cuda and done[b] is not None:
            done[b].synchronize()
        buf, where = art.read(names, pin=cuda, buffer=host[b])
        host[b] = buf
        used = max(o + ln for pair in where.values() for o, ln in pair)
        if cuda:
            if staged[b] is None or staged[b].numel() < used:
                staged[b] = torch.empty((buf.numel(),), dtype=torch.uint8, device=device)
            staged[b][:used].copy_(buf[:used], non_blocking=True)
            src = staged[b]
        else:
            src = buf
        for n, packed, scales, rows in ((names[0], gate_p, gate_s, I), (names[1], up_p, up_s, I),
                                        (names[2], down_p, down_s, H)):
            (co, cn), (so, sn) = where[n]
            if cn != packed.shape[1] or sn != 2 * rows:
                raise ValueError(f"{n}: {cn} code and {sn} scale bytes, expected {packed.shape[1]} and {2 * rows}")
            packed[e].copy_(src[co:co + cn])
            scale_bytes = src[so:so + sn]
            if scale_bytes.storage_offset() % 2:
                scale_bytes = scale_bytes.clone()
            scales[e].copy_(scale_bytes.view(torch.float16))
        if cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(device))
            done[b] = ev
    if cuda:
        torch.cuda.current_stream(device).synchronize()
    return synth.Q4MoELayer(cfg, router_weight, gate_p, gate_s, up_p, up_s, down_p, down_s)

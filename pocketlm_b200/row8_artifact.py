"""Row8 packed-GEMV artifacts read straight into device memory.

The reference packs fp16/bf16 matrices offline into the row8 layout its
packed GEMV reads (`[ceil(rows/8)][cols][8]` uint16, rows padded with zeros):
one data file plus `row8_manifest.json` (format "pcketlm-row8-packed-gemv",
per tensor dtype, shape, byte offset and length; writer
tools/pack_weights_row8.py:86-142).  Its runtime reads a tensor's bytes into
host memory (core/runtime/packed_artifact_loader.py:61-87, or the native
cache native/row8_artifact_cache.cpp:20-67) for every call.

`Row8Artifact.load` reads the named tensors' ranges with `moe_read_spans`
(threaded pread) into one pinned buffer, copies it to the device once and
hands back flat uint16 device tensors that `native.packed_gemv_rows8` takes
as they are -- the same layout this library's `pack_weight_rows8` builds on
the GPU -- so an artifact is read from disk once and stays resident in HBM.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from pocketlm_b200 import native

ROW8_FORMAT = "pcketlm-row8-packed-gemv"
ROW8_MANIFEST_NAME = "row8_manifest.json"
ROW_BLOCK = 8


def row8_packed_elements(rows: int, cols: int) -> int:
    return (int(rows) + ROW_BLOCK - 1) // ROW_BLOCK * int(cols) * ROW_BLOCK


class Row8Artifact:
    """One row8 artifact directory (its manifest and data file)."""

    def __init__(self, artifact_dir: str | Path):
        self.artifact_dir = Path(artifact_dir).resolve()
        path = self.artifact_dir / ROW8_MANIFEST_NAME
        if not path.exists():
            raise FileNotFoundError(str(path))
        self.manifest = json.loads(path.read_text(encoding="utf-8"))
        fmt = self.manifest.get("format")
        if fmt != ROW8_FORMAT:
            raise ValueError(f"unsupported row8 artifact format {fmt!r} (expected {ROW8_FORMAT!r})")
        if int(self.manifest.get("row_block", ROW_BLOCK)) != ROW_BLOCK:
            raise ValueError(f"row8 artifact with row_block {self.manifest.get('row_block')}")
        self.data_file = self.artifact_dir / str(self.manifest["data_file"])
        self.tensors: dict[str, dict] = dict(self.manifest.get("tensors") or {})

    def entry(self, name: str) -> dict:
        if name not in self.tensors:
            raise KeyError(name)
        e = dict(self.tensors[name])
        rows, cols = (int(v) for v in e["shape"])
        if str(e["dtype"]).upper() not in ("F16", "BF16"):
            raise ValueError(f"{name}: row8 dtype {e['dtype']} (expected F16 or BF16)")
        if int(e["nbytes"]) != 2 * row8_packed_elements(rows, cols):
            raise ValueError(f"{name}: {e['nbytes']} bytes, expected {2 * row8_packed_elements(rows, cols)} "
                             f"for shape {[rows, cols]}")
        return e

    def load(self, names: list[str], device: torch.device | str | None = None) -> dict[str, tuple[torch.Tensor, dict]]:
        """name -> (flat uint16 row8 tensor on `device`, manifest entry)."""
        device = torch.device(device if device is not None else native._device())
        entries = {n: self.entry(n) for n in dict.fromkeys(names)}
        if not entries:
            return {}
        total = sum(int(e["nbytes"]) for e in entries.values())
        cuda = device.type == "cuda"
        host = torch.empty((total,), dtype=torch.uint8, pin_memory=cuda)
        spans, outs, where = [], [], {}
        base = 0
        for n, e in sorted(entries.items(), key=lambda kv: int(kv[1]["offset"])):
            nb = int(e["nbytes"])
            spans.append((int(e["offset"]), nb))
            outs.append(host[base:base + nb])
            where[n] = (base, nb)
            base += nb
        native.read_spans(self.data_file, spans, outs)
        dev = host.to(device, non_blocking=cuda) if cuda else host
        if cuda:
            torch.cuda.current_stream(device).synchronize()  # the pinned buffer is released on return
        out = {}
        for n, e in entries.items():
            off, nb = where[n]
            out[n] = (dev[off:off + nb].view(torch.uint16), e)
        return out

    def load_one(self, name: str, device: torch.device | str | None = None) -> tuple[torch.Tensor, dict]:
        return self.load([name], device)[name]

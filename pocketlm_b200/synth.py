"""Seeded synthetic MoE layers in the reference's weight formats.

There is no checkpoint on this machine, so every benchmark and parity case
runs on random weights with the distributions the benchmark configs name:

* DeepSeek-V3 FP8 layers (configs 1-3, 5): expert weights ~N(0, 0.02)
  quantised to e4m3 with one fp32 scale per 128x128 block, scale = amax/448
  (the `weight_scale_inv` convention read by fp8_source.py:812-858); router
  weight ~N(0, 0.02) in bf16; correction bias ~U(-0.01, 0.01) or a Zipf-like
  skew for the prefill config; activations ~N(0, 1) in bf16.
* Mixtral-shape Q4 layers (config 4): weights ~N(0, 0.02) quantised with the
  per-output-row symmetric int4 scheme of
  src/pcketlm/core/model_import/q4_quantize.py:21-71 (scale = amax/7 stored
  as fp16, codes clamped to [-7, 7], two codes per byte, low nibble first).

Each expert draws from its own generator seeded from (seed, expert), so any
subset of experts can be regenerated on any device without the others.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

FP8_BLOCK = 128
E4M3_MAX = 448.0


@dataclass(frozen=True)
class DsMoEConfig:
    name: str
    hidden: int
    inter: int
    n_routed: int
    top_k: int
    n_group: int
    topk_group: int
    route_scale: float
    scoring_func: str = "sigmoid"

    @property
    def gate_scale_shape(self) -> tuple[int, int]:
        return (_ceil(self.inter), _ceil(self.hidden))

    @property
    def down_scale_shape(self) -> tuple[int, int]:
        return (_ceil(self.hidden), _ceil(self.inter))

    @property
    def expert_bytes(self) -> int:
        """FP8 weight + fp32 scale bytes of one expert (gate, up, down)."""
        w = 3 * self.hidden * self.inter
        gs, ds = self.gate_scale_shape, self.down_scale_shape
        return w + 4 * (2 * gs[0] * gs[1] + ds[0] * ds[1])


@dataclass(frozen=True)
class MixtralQ4Config:
    name: str
    hidden: int
    inter: int
    n_experts: int
    top_k: int

    @property
    def expert_bytes(self) -> int:
        """Packed int4 + fp16 row-scale bytes of one expert."""
        return 3 * self.hidden * self.inter // 2 + 2 * (2 * self.inter + self.hidden)


# BASELINE configs (the names follow the benchmark's numbering).
C1_TINY = DsMoEConfig("c1-tiny", hidden=512, inter=256, n_routed=16, top_k=4, n_group=4,
                      topk_group=2, route_scale=2.5)
C2_DSV3 = DsMoEConfig("c2-dsv3", hidden=7168, inter=2048, n_routed=256, top_k=8, n_group=8,
                      topk_group=4, route_scale=2.5)
C4_MIXTRAL = MixtralQ4Config("c4-mixtral-q4", hidden=4096, inter=14336, n_experts=8, top_k=2)


def _ceil(n: int) -> int:
    return (n + FP8_BLOCK - 1) // FP8_BLOCK


def _generator(device: torch.device | str, seed: int) -> torch.Generator:
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed) & 0x7FFF_FFFF_FFFF_FFFF)
    return gen


def _expert_seed(seed: int, expert: int, role: int) -> int:
    return (seed * 1_000_003 + expert * 7_919 + role * 104_729 + 17) % (2**61 - 1)


def quantize_fp8_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 [R, C] -> (e4m3 bytes uint8 [R, C], fp32 scale_inv [ceil(R/128), ceil(C/128)]).

    One scale per 128x128 block, scale = amax/448 (1.0 for an all-zero
    block), so dequantisation is byte_value * scale.  The all-ones codes
    0x7F/0xFF (NaN in e4m3fn) never occur: |w/scale| <= 448 rounds to at
    most 0x7E.
    """
    rows, cols = int(w.shape[0]), int(w.shape[1])
    br, bc = _ceil(rows), _ceil(cols)
    padded = torch.zeros((br * FP8_BLOCK, bc * FP8_BLOCK), dtype=torch.float32, device=w.device)
    padded[:rows, :cols] = w.float()
    blocks = padded.view(br, FP8_BLOCK, bc, FP8_BLOCK)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = (blocks / scale[:, None, :, None]).view(br * FP8_BLOCK, bc * FP8_BLOCK)[:rows, :cols]
    codes = q.contiguous().to(torch.float8_e4m3fn).view(torch.uint8)
    return codes, scale.contiguous()


def pack_int4(values: torch.Tensor) -> torch.Tensor:
    """Signed int4 codes in [-8, 7] -> bytes, two per byte, even index in the
    low nibble (the layout of q4_quantize.py:21-33)."""
    flat = values.reshape(-1).to(torch.int16)
    nibbles = torch.bitwise_and(flat, 0xF).to(torch.uint8)
    if nibbles.numel() % 2:
        nibbles = torch.cat([nibbles, nibbles.new_zeros(1)])
    return (nibbles[0::2] | (nibbles[1::2] << 4)).contiguous()


def quantize_q4_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-row symmetric int4 (q4_quantize.py:48-71):
    scale = amax/7 (1 for a zero row), code = clamp(round(w/scale), -7, 7).
    Returns (packed uint8 [R*C/2], fp16 scales [R])."""
    m = w.float().reshape(w.shape[0], -1)
    amax = m.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 7.0, torch.ones_like(amax))
    codes = torch.round(m / scale[:, None]).clamp(-7, 7).to(torch.int8)
    return pack_int4(codes), scale.to(torch.float16).contiguous()


class Fp8MoELayer:
    """One DeepSeek-V3 MoE layer: router + routed experts + one shared expert.

    HBM layout (expert index n_routed is the shared expert):
      w13 uint8 [E+1, 2, I, H]   gate (0) and up (1) projections
      s13 fp32  [E+1, 2, ceil(I/128), ceil(H/128)]
      w2  uint8 [E+1, H, I]      down projection
      s2  fp32  [E+1, ceil(H/128), ceil(I/128)]
    """

    def __init__(self, cfg: DsMoEConfig, router_weight, bias, w13, s13, w2, s2,
                 slots: dict[int, int] | None = None):
        self.cfg = cfg
        self.router_weight = router_weight
        self.bias = bias
        self.w13, self.s13, self.w2, self.s2 = w13, s13, w2, s2
        # expert id -> slot in the stacked tensors; None means slot == id (a full layer)
        self.slots = slots

    @property
    def device(self) -> torch.device:
        return self.w13.device

    @property
    def is_full(self) -> bool:
        return self.slots is None

    def expert(self, e: int):
        """(gate, gate_s, up, up_s, down, down_s) views of expert `e`."""
        i = e if self.slots is None else self.slots[e]
        return (self.w13[i, 0], self.s13[i, 0], self.w13[i, 1], self.s13[i, 1], self.w2[i], self.s2[i])

    def shared_expert(self):
        return self.expert(self.cfg.n_routed)

    def to(self, device) -> "Fp8MoELayer":
        mv = lambda t: None if t is None else t.to(device)  # noqa: E731
        return Fp8MoELayer(self.cfg, mv(self.router_weight), mv(self.bias), mv(self.w13),
                           mv(self.s13), mv(self.w2), mv(self.s2), self.slots)


def make_router_bias(cfg: DsMoEConfig, seed: int, device, kind: str = "uniform") -> torch.Tensor | None:
    """Correction bias: 'uniform' ~U(-0.01, 0.01); 'zipf' = 0.25 * rank^-1.1
    over a seeded random permutation of ranks 1..E (skews routing towards a
    few experts, as the prefill config asks); 'none' -> None."""
    if kind == "none":
        return None
    gen = _generator("cpu", _expert_seed(seed, 0, 11))
    if kind == "uniform":
        bias = torch.rand((cfg.n_routed,), generator=gen) * 0.02 - 0.01
    elif kind == "zipf":
        ranks = torch.randperm(cfg.n_routed, generator=gen).to(torch.float64) + 1.0
        bias = (0.25 * ranks.pow(-1.1)).to(torch.float32)
    else:
        raise ValueError(f"unknown bias kind {kind!r}")
    return bias.to(device)


def make_fp8_layer(cfg: DsMoEConfig, seed: int = 0, device="cpu", bias_kind: str = "uniform",
                   experts: list[int] | None = None, threads: int = 1) -> Fp8MoELayer:
    """Generate a layer.  `experts` (ids; the shared expert is id
    cfg.n_routed) limits which experts are generated and stored: such a
    partial layer holds only those, in the order given.  `threads` > 1
    generates CPU experts concurrently (same values: each expert has its
    own generator)."""
    device = torch.device(device)
    H, I = cfg.hidden, cfg.inter
    ids = list(range(cfg.n_routed + 1)) if experts is None else list(experts)
    E1 = len(ids)
    gen_r = _generator(device, _expert_seed(seed, 0, 1))
    router_weight = (torch.randn((cfg.n_routed, H), generator=gen_r, device=device) * 0.02).to(torch.bfloat16)
    bias = make_router_bias(cfg, seed, device, bias_kind)
    w13 = torch.zeros((E1, 2, I, H), dtype=torch.uint8, device=device)
    s13 = torch.ones((E1, 2, *cfg.gate_scale_shape), dtype=torch.float32, device=device)
    w2 = torch.zeros((E1, H, I), dtype=torch.uint8, device=device)
    s2 = torch.ones((E1, *cfg.down_scale_shape), dtype=torch.float32, device=device)

    def fill(slot: int, e: int) -> None:
        for proj in range(3):
            gen = _generator(device, _expert_seed(seed, e + 1, 2 + proj))
            shape = (H, I) if proj == 2 else (I, H)
            w = torch.randn(shape, generator=gen, device=device) * 0.02
            q, s = quantize_fp8_blocks(w)
            if proj == 2:
                w2[slot].copy_(q)
                s2[slot].copy_(s)
            else:
                w13[slot, proj].copy_(q)
                s13[slot, proj].copy_(s)
            del w, q, s

    if threads > 1 and device.type == "cpu":
        from concurrent.futures import ThreadPoolExecutor

        intra = torch.get_num_threads()
        torch.set_num_threads(1)  # one expert per thread; torch's own threads would oversubscribe the cores
        try:
            with ThreadPoolExecutor(max_workers=threads) as pool:
                list(pool.map(lambda se: fill(*se), enumerate(ids)))
        finally:
            torch.set_num_threads(intra)
    else:
        for slot, e in enumerate(ids):
            fill(slot, e)
    slots = None if experts is None else {e: i for i, e in enumerate(ids)}
    return Fp8MoELayer(cfg, router_weight, bias, w13, s13, w2, s2, slots)


def make_hidden(tokens: int, hidden: int, seed: int = 0, device="cpu",
                dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Activations ~N(0, 1), rounded to `dtype`."""
    gen = _generator(device, _expert_seed(seed, 0, 31))
    return torch.randn((tokens, hidden), generator=gen, device=device).to(dtype)


class Q4MoELayer:
    """Mixtral-shape MoE layer in the reference's Q4 format.

      gate/up packed uint8 [E, I*H/2], scales fp16 [E, I]
      down    packed uint8 [E, H*I/2], scales fp16 [E, H]
    """

    def __init__(self, cfg: MixtralQ4Config, router_weight, gate_p, gate_s, up_p, up_s, down_p, down_s):
        self.cfg = cfg
        self.router_weight = router_weight
        self.gate_p, self.gate_s, self.up_p, self.up_s = gate_p, gate_s, up_p, up_s
        self.down_p, self.down_s = down_p, down_s

    def expert(self, e: int):
        return (self.gate_p[e], self.gate_s[e], self.up_p[e], self.up_s[e], self.down_p[e], self.down_s[e])

    def to(self, device) -> "Q4MoELayer":
        return Q4MoELayer(self.cfg, *(t.to(device) for t in (
            self.router_weight, self.gate_p, self.gate_s, self.up_p, self.up_s, self.down_p, self.down_s)))


def make_q4_layer(cfg: MixtralQ4Config, seed: int = 0, device="cpu") -> Q4MoELayer:
    device = torch.device(device)
    E, H, I = cfg.n_experts, cfg.hidden, cfg.inter
    gen_r = _generator(device, _expert_seed(seed, 0, 1))
    router_weight = (torch.randn((E, H), generator=gen_r, device=device) * 0.02).to(torch.bfloat16)
    gate_p = torch.empty((E, I * H // 2), dtype=torch.uint8, device=device)
    up_p = torch.empty_like(gate_p)
    down_p = torch.empty((E, H * I // 2), dtype=torch.uint8, device=device)
    gate_s = torch.empty((E, I), dtype=torch.float16, device=device)
    up_s = torch.empty_like(gate_s)
    down_s = torch.empty((E, H), dtype=torch.float16, device=device)
    for e in range(E):
        for proj, (pk, sc) in enumerate(((gate_p, gate_s), (up_p, up_s), (down_p, down_s))):
            gen = _generator(device, _expert_seed(seed, e + 1, 2 + proj))
            shape = (H, I) if proj == 2 else (I, H)
            w = torch.randn(shape, generator=gen, device=device) * 0.02
            packed, scales = quantize_q4_rows(w)
            pk[e].copy_(packed)
            sc[e].copy_(scales)
            del w, packed, scales
    return Q4MoELayer(cfg, router_weight, gate_p, gate_s, up_p, up_s, down_p, down_s)

"""Layer-level entry points: the GPU counterparts of run_fp8_router and
run_fp8_moe (src/pcketlm/core/runtime/fp8_source.py:1500-1884).

`run_fp8_router(model_id, layer_index, hidden)` and
`run_fp8_moe(model_id, layer_index, hidden, *, dtype, router)` keep the
reference's signatures and result types: the layer is found by model id
(pocketlm_b200.models: config.json + FP8 pack or safetensors shards) and
kept resident in HBM, so a caller swaps one import for the other.
`route_resident_layer` / `moe_resident_layer` take an HBM-resident layer
object directly (DsMoELayerGPU, or a synth.Fp8MoELayer for the router).
Results carry the fields of the reference's FP8RouterResult /
FP8MoEResult; problems finding the layer are reported as blockers with
ready=False, as the reference does.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch

from . import native
from .synth import Fp8MoELayer


@dataclass
class FP8RouterResult:
    model_id: str
    layer_index: int
    hidden_shape: list[int]
    weights_shape: list[int]
    indices_shape: list[int]
    selected_experts: list[int]
    scoring_func: str
    route_scale: float
    n_groups: int
    topk_groups: int
    bias_loaded: bool
    weights_tensor: torch.Tensor | None = None
    indices_tensor: torch.Tensor | None = None
    blockers: list[str] = field(default_factory=list)
    ready: bool = False

    def to_dict(self) -> dict:
        return {"model_id": self.model_id, "layer_index": self.layer_index, "hidden_shape": list(self.hidden_shape),
                "weights_shape": list(self.weights_shape), "indices_shape": list(self.indices_shape),
                "selected_experts": list(self.selected_experts), "scoring_func": self.scoring_func,
                "route_scale": self.route_scale, "n_groups": self.n_groups, "topk_groups": self.topk_groups,
                "bias_loaded": self.bias_loaded, "weights_materialized": self.weights_tensor is not None,
                "indices_materialized": self.indices_tensor is not None, "blockers": list(self.blockers),
                "ready": self.ready}


@dataclass
class FP8MoEResult:
    model_id: str
    layer_index: int
    hidden_shape: list[int]
    output_shape: list[int]
    selected_experts: list[int]
    routed_weight_bytes: int
    shared_weight_bytes: int
    dequantized_weight_bytes: int = 0
    router: FP8RouterResult | None = None
    output_tensor: torch.Tensor | None = None
    router_elapsed_seconds: float = 0.0
    preload_elapsed_seconds: float = 0.0
    routed_elapsed_seconds: float = 0.0
    shared_elapsed_seconds: float = 0.0
    total_elapsed_seconds: float = 0.0
    blockers: list[str] = field(default_factory=list)
    ready: bool = False

    def to_dict(self) -> dict:
        return {"model_id": self.model_id, "layer_index": self.layer_index, "hidden_shape": list(self.hidden_shape),
                "output_shape": list(self.output_shape), "selected_experts": list(self.selected_experts),
                "routed_weight_bytes": self.routed_weight_bytes, "shared_weight_bytes": self.shared_weight_bytes,
                "dequantized_weight_bytes": self.dequantized_weight_bytes,
                "router": None if self.router is None else self.router.to_dict(),
                "output_materialized": self.output_tensor is not None,
                "router_elapsed_seconds": float(self.router_elapsed_seconds),
                "preload_elapsed_seconds": float(self.preload_elapsed_seconds),
                "routed_elapsed_seconds": float(self.routed_elapsed_seconds),
                "shared_elapsed_seconds": float(self.shared_elapsed_seconds),
                "total_elapsed_seconds": float(self.total_elapsed_seconds), "blockers": list(self.blockers),
                "ready": self.ready}


class DsMoELayerGPU:
    """An FP8 DeepSeek-V3 MoE layer resident in HBM, ready for the fused path.

    Holds the [6, E+1] device table of expert addresses (gate, gate scale,
    up, up scale, down, down scale; the shared expert last) that
    moe_ds_moe_layer_fp8 walks, and a reusable workspace."""

    def __init__(self, layer: Fp8MoELayer, layer_index: int = 0, *, allow_partial: bool = False,
                 tiled: bool = True):
        """allow_partial: accept a layer holding only some experts; the absent
        ones get null table entries, which the kernels skip (they contribute
        nothing), so outputs are only right for tokens routed to resident
        experts.  For small profiling cases; a full layer is the product path.

        tiled: also keep the expert weights in the decode GEMV's
        fragment-native layout (moe_fp8_tile_weights; same bytes, one
        contiguous stream per warp), used whenever the default GEMV runs."""
        if not layer.is_full and not allow_partial:
            raise ValueError("the fused layer path needs every expert resident (a full layer)")
        if layer.device.type != "cuda":
            layer = layer.to(native._device())
        self.layer = layer
        self.cfg = layer.cfg
        self.layer_index = int(layer_index)
        n = self.cfg.n_routed + 1
        cols = [[0] * n for _ in range(6)]
        for e in range(n):
            if not layer.is_full and e not in layer.slots:
                continue
            for j, t in enumerate(layer.expert(e)):
                cols[j][e] = int(t.data_ptr())
        self.tables = torch.tensor(cols, dtype=torch.int64, device=layer.device)
        # experts with no 0x7F/0xFF byte skip the decoder's NaN-code fix-up (computed once)
        self.nan_free = torch.zeros((n,), dtype=torch.uint8, device=layer.device)
        native._check(native.load_library().moe_fp8_nan_free_flags(
            native._ptr(self.tables), n, self.cfg.inter, self.cfg.hidden, native._ptr(self.nan_free),
            native._stream()), "moe_fp8_nan_free_flags")
        self.tables_tiled = None
        cfg = self.cfg
        lib = native.load_library()
        if tiled and cfg.hidden % 128 == 0 and cfg.inter % 128 == 0:
            tb13 = int(lib.moe_fp8_tiled_bytes(cfg.inter, cfg.hidden))
            tb2 = int(lib.moe_fp8_tiled_bytes(cfg.hidden, cfg.inter))
            self._tiled13 = torch.empty((n, 2, tb13), dtype=torch.uint8, device=layer.device)
            self._tiled2 = torch.empty((n, tb2), dtype=torch.uint8, device=layer.device)
            tcols = [list(c) for c in cols]
            for e in range(n):
                if cols[0][e] == 0:
                    continue
                g, _gs, u, _us, d, _ds = layer.expert(e)
                for src, dst, rows, k in ((g, self._tiled13[e, 0], cfg.inter, cfg.hidden),
                                          (u, self._tiled13[e, 1], cfg.inter, cfg.hidden),
                                          (d, self._tiled2[e], cfg.hidden, cfg.inter)):
                    native._check(lib.moe_fp8_tile_weights(native._ptr(src), native._ptr(dst), rows, k,
                                                           native._stream()), "moe_fp8_tile_weights")
                tcols[0][e] = int(self._tiled13[e, 0].data_ptr())
                tcols[2][e] = int(self._tiled13[e, 1].data_ptr())
                tcols[4][e] = int(self._tiled2[e].data_ptr())
            self.tables_tiled = torch.tensor(tcols, dtype=torch.int64, device=layer.device)
        self._workspace = torch.empty((0,), dtype=torch.uint8, device=layer.device)

    def workspace_for(self, tokens: int) -> torch.Tensor:
        lib = native.load_library()
        need = int(lib.moe_ds_moe_layer_workspace_bytes(tokens, self.cfg.hidden, self.cfg.inter,
                                                        self.cfg.n_routed, self.cfg.top_k, 1))
        if self._workspace.numel() < need:
            self._workspace = torch.empty((need,), dtype=torch.uint8, device=self.layer.device)
        return self._workspace

    def forward(self, hidden: torch.Tensor, *, out: torch.Tensor | None = None,
                ids: torch.Tensor | None = None, weights: torch.Tensor | None = None) -> torch.Tensor:
        """hidden [T, H] bf16 on the layer's device -> out [T, H] bf16.

        `ids` (int64 [T, k]) and `weights` (bf16 [T, k]) receive the routing
        when given.  Everything is enqueued on the current stream."""
        cfg = self.cfg
        x = hidden.reshape(-1, cfg.hidden)
        if x.device != self.layer.device:
            raise ValueError("hidden must be on the layer's device")
        if x.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("hidden must be bf16 or fp32")
        x = x.contiguous()
        T = int(x.shape[0])
        if out is None:
            out = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=x.device)
        ws = self.workspace_for(T)
        rw = self.layer.router_weight
        rdt = {torch.float32: native.DTYPE_F32, torch.bfloat16: native.DTYPE_BF16, torch.float16: native.DTYPE_F16}
        lib = native.load_library()
        # the tiled copy serves the default GEMV; the other selections read row-major weights
        layout = 1 if self.tables_tiled is not None and lib.moe_b200_selected_gemv() == 0 else 0
        tables = self.tables_tiled if layout else self.tables
        code = lib.moe_ds_moe_layer_fp8(
            native._ptr(x), native.DTYPE_BF16 if x.dtype == torch.bfloat16 else native.DTYPE_F32, T, cfg.hidden,
            cfg.inter, native._ptr(rw), rdt[rw.dtype], native._ptr(self.layer.bias), cfg.n_routed, cfg.n_group,
            cfg.topk_group, cfg.top_k, 1 if cfg.scoring_func == "softmax" else 0, float(cfg.route_scale),
            native._ptr(tables), 1, native._ptr(self.nan_free), layout, native._ptr(out), native._ptr(ids),
            native._ptr(weights),
            native._ptr(ws), ws.numel(), native._stream())
        native._check(code, "moe_ds_moe_layer_fp8")
        return out


    def forward_routed(self, hidden: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, *,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """The layer for a routing the caller already has (a router result
        passed to run_fp8_moe): ids int64 [T, k], weights [T, k] (any float
        dtype; used as fp32).  Rows are bucketed per expert, the routed
        experts and the shared expert run as one grouped launch, and the
        combine adds them in slot order, then the shared expert, rounding
        once to bf16 -- the fused layer's arithmetic for the same routing."""
        cfg = self.cfg
        x = hidden.reshape(-1, cfg.hidden).to(torch.bfloat16).contiguous()
        T, k, H = int(x.shape[0]), int(ids.shape[-1]), cfg.hidden
        dev = x.device
        ids = ids.reshape(T, k).to(device=dev, dtype=torch.int64).contiguous()
        if T and (int(ids.min()) < 0 or int(ids.max()) >= cfg.n_routed):
            raise ValueError("router indices must be routed expert ids")
        w = weights.reshape(T, k).to(device=dev, dtype=torch.float32).contiguous()
        if out is None:
            out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        if T == 0:
            return out
        lib = native.load_library()
        n = T * k
        rows = torch.empty((n + T, H), dtype=torch.bfloat16, device=dev)
        row_expert = torch.empty((n + T,), dtype=torch.int32, device=dev)
        offsets = torch.empty((2,), dtype=torch.int32, device=dev)
        entry_pos = torch.empty((n,), dtype=torch.int32, device=dev)
        pos_weight = torch.empty((n,), dtype=torch.float32, device=dev)
        ws = torch.empty((int(lib.moe_ep_dispatch_workspace_bytes(T, k)),), dtype=torch.uint8, device=dev)
        native._check(lib.moe_ep_dispatch_pack(
            native._ptr(ids), native._ptr(w), native._ptr(x), T, H, k, cfg.n_routed, 1, native._ptr(rows),
            native._ptr(row_expert), native._ptr(offsets), native._ptr(entry_pos), native._ptr(pos_weight),
            native._ptr(ws), ws.numel(), native._stream()), "moe_ep_dispatch_pack")
        rows[n:].copy_(x)
        row_expert[n:].fill_(cfg.n_routed)  # the shared expert, last in the tables
        R, S = n + T, cfg.n_routed + 1
        y = torch.empty((R, H), dtype=torch.float32, device=dev)
        layout = 1 if self.tables_tiled is not None and lib.moe_b200_selected_gemv() == 0 else 0
        tables = self.tables_tiled if layout else self.tables
        ws = torch.empty((int(lib.moe_ep_experts_workspace_bytes(R, H, cfg.inter, S)),), dtype=torch.uint8,
                         device=dev)
        native._check(lib.moe_ep_experts_fp8(
            native._ptr(rows), native._ptr(row_expert), R, H, cfg.inter, native._ptr(tables), S,
            native._ptr(self.nan_free), layout, native._ptr(y), native._ptr(ws), ws.numel(), native._stream()),
            "moe_ep_experts_fp8")
        # fp32 rows: the fused layer's arithmetic for the same routing
        native._check(lib.moe_ep_combine(native._ptr(y), native.DTYPE_F32, native._ptr(entry_pos),
                                         native._ptr(pos_weight), T, k, H, 1, native._ptr(out), native._stream()),
                      "moe_ep_combine")
        return out

    def capture(self, tokens: int, *, input_dtype: torch.dtype = torch.bfloat16) -> "GraphedDsMoELayer":
        """Record the whole layer (7 kernels) for a fixed token count into a
        CUDA graph; replaying it removes the per-kernel host launch cost,
        which at decode sizes is comparable to the kernels themselves."""
        return GraphedDsMoELayer(self, tokens, input_dtype)


class GraphedDsMoELayer:
    """A DsMoELayerGPU forward for one token count, captured as a CUDA graph.

    Write the activations into `.input` (or pass them to __call__), replay,
    read `.output`; `.ids` / `.weights` hold the routing of the last replay."""

    def __init__(self, layer: DsMoELayerGPU, tokens: int, input_dtype: torch.dtype):
        cfg = layer.cfg
        dev = layer.layer.device
        self.layer = layer
        self.tokens = int(tokens)
        self.input = torch.zeros((tokens, cfg.hidden), dtype=input_dtype, device=dev)
        self.output = torch.empty((tokens, cfg.hidden), dtype=torch.bfloat16, device=dev)
        self.ids = torch.empty((tokens, cfg.top_k), dtype=torch.int64, device=dev)
        self.weights = torch.empty((tokens, cfg.top_k), dtype=torch.bfloat16, device=dev)
        layer.workspace_for(tokens)
        # warm up outside the capture (kernel attributes, lazy module loading)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            layer.forward(self.input, out=self.output, ids=self.ids, weights=self.weights)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            layer.forward(self.input, out=self.output, ids=self.ids, weights=self.weights)
        torch.cuda.synchronize(dev)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.output

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        self.input.copy_(hidden.reshape(self.input.shape), non_blocking=True)
        return self.replay()


def _router_result(model_id: str, layer_index: int, hidden: torch.Tensor, cfg, bias_loaded: bool, ids, weights,
                   blockers: list[str] | None = None) -> FP8RouterResult:
    selected = [] if ids is None else sorted({int(v) for v in ids.reshape(-1).tolist()})
    blockers = list(blockers or [])
    return FP8RouterResult(
        model_id=str(model_id), layer_index=int(layer_index), hidden_shape=[int(v) for v in hidden.shape],
        weights_shape=[] if weights is None else [int(v) for v in weights.shape],
        indices_shape=[] if ids is None else [int(v) for v in ids.shape], selected_experts=selected,
        scoring_func=cfg.scoring_func if cfg else "", route_scale=float(cfg.route_scale) if cfg else 0.0,
        n_groups=int(cfg.n_group) if cfg else 0, topk_groups=int(cfg.topk_group) if cfg else 0,
        bias_loaded=bool(bias_loaded), weights_tensor=weights, indices_tensor=ids, blockers=blockers,
        ready=not blockers and ids is not None and weights is not None)


def route_resident_layer(layer: Fp8MoELayer | DsMoELayerGPU, hidden: torch.Tensor, layer_index: int | None = None,
                         *, model_id: str = "") -> FP8RouterResult:
    """The router of fp8_source.py:1500-1566 on the GPU for a resident layer:
    ids int64 [T, k] and weights [T, k] in hidden's dtype, on hidden's device."""
    base = layer.layer if isinstance(layer, DsMoELayerGPU) else layer
    if layer_index is None:
        layer_index = layer.layer_index if isinstance(layer, DsMoELayerGPU) else 0
    cfg = base.cfg
    ids, weights = native.route_topk(hidden, base.router_weight, base.bias, top_k=cfg.top_k, n_group=cfg.n_group,
                                     topk_group=cfg.topk_group, scoring_func=cfg.scoring_func,
                                     route_scale=cfg.route_scale, round_to_hidden_dtype=True)
    return _router_result(model_id, layer_index, hidden, cfg, base.bias is not None, ids.to(hidden.device),
                          weights.to(hidden.device))


def moe_resident_layer(layer: DsMoELayerGPU, hidden: torch.Tensor, *, dtype: torch.dtype = torch.bfloat16,
                       router: FP8RouterResult | None = None, layer_index: int | None = None,
                       model_id: str = "") -> FP8MoEResult:
    """One MoE layer (routed experts + shared expert) on the GPU for a
    resident layer, the counterpart of fp8_source.py:1569-1884.  Without
    `router` the fused path routes, dispatches, runs the experts and combines
    in one launch sequence; with it, its indices and weights are used.  The
    combine rounds once to bf16; another `dtype` is a cast of that result."""
    start = time.perf_counter()
    cfg = layer.cfg
    dev = layer.layer.device
    index = int(layer.layer_index if layer_index is None else layer_index)
    flat = hidden.reshape(-1, cfg.hidden)
    x = flat.to(dev).to(torch.bfloat16) if flat.dtype != torch.float32 else flat.to(dev)
    T = int(x.shape[0])
    if router is not None:
        if router.indices_tensor is None or router.weights_tensor is None:
            return FP8MoEResult(
                model_id=str(model_id), layer_index=index, hidden_shape=[int(v) for v in hidden.shape],
                output_shape=[], selected_experts=[], routed_weight_bytes=0, shared_weight_bytes=0, router=router,
                blockers=list(router.blockers) + ["Router did not produce selected experts and route weights."])
        r0 = time.perf_counter()
        out = layer.forward_routed(x, router.indices_tensor, router.weights_tensor)
        router_result, router_s = router, 0.0
        ids = router.indices_tensor
    else:
        ids = torch.empty((T, cfg.top_k), dtype=torch.int64, device=dev)
        weights = torch.empty((T, cfg.top_k), dtype=torch.bfloat16, device=dev)
        r0 = time.perf_counter()
        out = layer.forward(x, ids=ids, weights=weights)
        router_s = 0.0
        w_out = weights if hidden.dtype == torch.bfloat16 else weights.to(hidden.dtype)
        router_result = _router_result(model_id, index, hidden, cfg, layer.layer.bias is not None,
                                       ids.to(hidden.device), w_out.to(hidden.device))
    output = out.reshape(hidden.shape).to(device=hidden.device, dtype=dtype)
    routed_s = time.perf_counter() - r0
    selected = sorted({int(v) for v in ids.reshape(-1).tolist()})
    return FP8MoEResult(
        model_id=str(model_id), layer_index=index, hidden_shape=[int(v) for v in hidden.shape],
        output_shape=[int(v) for v in output.shape], selected_experts=selected,
        routed_weight_bytes=len(selected) * cfg.expert_bytes, shared_weight_bytes=cfg.expert_bytes,
        dequantized_weight_bytes=0, router=router_result, output_tensor=output, router_elapsed_seconds=router_s,
        routed_elapsed_seconds=routed_s, total_elapsed_seconds=time.perf_counter() - start, ready=True)


def run_fp8_router(model_id: str, layer_index: int, hidden: torch.Tensor) -> FP8RouterResult:
    """DeepSeek-V3 sigmoid (or softmax) group-limited top-k routing for one
    layer of `model_id` (fp8_source.py:1500-1566), on the GPU."""
    from . import models

    try:
        layer = models.resident_layer(model_id, layer_index)
    except (FileNotFoundError, KeyError, ValueError) as exc:
        return _router_result(model_id, layer_index, hidden, None, False, None, None, [str(exc)])
    return route_resident_layer(layer, hidden, layer_index, model_id=model_id)


def run_fp8_moe(model_id: str, layer_index: int, hidden: torch.Tensor, *, dtype: torch.dtype = torch.bfloat16,
                router: FP8RouterResult | None = None) -> FP8MoEResult:
    """Routed experts plus the shared expert for one MoE layer of `model_id`
    (fp8_source.py:1569-1884), on the GPU; `router` reuses a routing result."""
    from . import models

    start = time.perf_counter()
    try:
        layer = models.resident_layer(model_id, layer_index)
    except (FileNotFoundError, KeyError, ValueError) as exc:
        return FP8MoEResult(model_id=str(model_id), layer_index=int(layer_index),
                            hidden_shape=[int(v) for v in hidden.shape], output_shape=[], selected_experts=[],
                            routed_weight_bytes=0, shared_weight_bytes=0, router=router, blockers=[str(exc)])
    preload = time.perf_counter() - start
    res = moe_resident_layer(layer, hidden, dtype=dtype, router=router, layer_index=layer_index, model_id=model_id)
    res.preload_elapsed_seconds = preload
    res.total_elapsed_seconds = time.perf_counter() - start
    return res


class Q4MoELayerGPU:
    """A Mixtral-shape Q4 MoE layer (pocketlm_b200.synth.Q4MoELayer) resident
    in HBM for moe_q4_moe_layer_u16: softmax top-k router, then every token
    through its experts with q4_moe_selected_forward_u16's arithmetic (the
    batch form of layer_bridge.py:909-955).

    tiled: also keep the codes in the Q4 tiled layout (moe_q4_tile_weights,
    +1x the packed bytes) so that batches of at least `prefill_pairs`
    (token, expert) pairs per expert run on the tcgen05 grouped GEMM; smaller
    batches stream the row-major codes through the warp-MMA GEMV."""

    prefill_pairs = 32

    def __init__(self, layer, *, tiled: bool = True):
        if layer.gate_p.device.type != "cuda":
            layer = layer.to(native._device())
        self.layer = layer
        self.cfg = layer.cfg
        E = self.cfg.n_experts
        cols = [[int(t.data_ptr()) for t in (layer.gate_p[e], layer.gate_s[e], layer.up_p[e], layer.up_s[e],
                                             layer.down_p[e], layer.down_s[e])] for e in range(E)]
        self.tables = torch.tensor(cols, dtype=torch.int64, device=layer.gate_p.device).t().contiguous()
        self.tables_tiled = None
        cfg = self.cfg
        if tiled and cfg.hidden % 256 == 0 and cfg.inter % 128 == 0:
            lib = native.load_library()
            dev = layer.gate_p.device
            tb13 = int(lib.moe_q4_tiled_bytes(cfg.inter, cfg.hidden))
            tb2 = int(lib.moe_q4_tiled_bytes(cfg.hidden, cfg.inter))
            self._tiled13 = torch.empty((E, 2, tb13), dtype=torch.uint8, device=dev)
            self._tiled2 = torch.empty((E, tb2), dtype=torch.uint8, device=dev)
            tcols = [list(c) for c in cols]
            for e in range(E):
                for src, dst, rows, k in ((layer.gate_p[e], self._tiled13[e, 0], cfg.inter, cfg.hidden),
                                          (layer.up_p[e], self._tiled13[e, 1], cfg.inter, cfg.hidden),
                                          (layer.down_p[e], self._tiled2[e], cfg.hidden, cfg.inter)):
                    native._check(lib.moe_q4_tile_weights(native._ptr(src), native._ptr(dst), rows, k,
                                                          native._stream()), "moe_q4_tile_weights")
                tcols[e][0] = int(self._tiled13[e, 0].data_ptr())
                tcols[e][2] = int(self._tiled13[e, 1].data_ptr())
                tcols[e][4] = int(self._tiled2[e].data_ptr())
            self.tables_tiled = torch.tensor(tcols, dtype=torch.int64, device=dev).t().contiguous()
        self._workspace = torch.empty((0,), dtype=torch.uint8, device=layer.gate_p.device)

    def workspace_for(self, tokens: int) -> torch.Tensor:
        cfg = self.cfg
        need = int(native.load_library().moe_q4_moe_layer_workspace_bytes(tokens, cfg.hidden, cfg.inter,
                                                                          cfg.n_experts, cfg.top_k))
        if self._workspace.numel() < need:
            self._workspace = torch.empty((need,), dtype=torch.uint8, device=self.tables.device)
        return self._workspace

    def forward(self, hidden: torch.Tensor, *, out: torch.Tensor | None = None, ids: torch.Tensor | None = None,
                weights: torch.Tensor | None = None, layout: int | None = None) -> torch.Tensor:
        """hidden [T, H] bf16 or fp16 on the layer's device -> out [T, H] same dtype.

        layout: 0 (GEMV, row-major codes) or 1 (tcgen05 GEMM, tiled codes);
        by default 1 from prefill_pairs pairs per expert on, when tiled."""
        cfg = self.cfg
        x = hidden.reshape(-1, cfg.hidden).contiguous()
        if x.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("hidden must be bf16 or fp16")
        T = int(x.shape[0])
        if layout is None:
            layout = int(self.tables_tiled is not None and T * cfg.top_k >= self.prefill_pairs * cfg.n_experts)
        if layout == 1 and self.tables_tiled is None:
            raise ValueError("layout 1 needs the tiled copy (tiled=True and hidden % 256, intermediate % 128 == 0)")
        tables = self.tables_tiled if layout == 1 else self.tables
        if out is None:
            out = torch.empty((T, cfg.hidden), dtype=x.dtype, device=x.device)
        ws = self.workspace_for(T)
        rw = self.layer.router_weight
        rdt = {torch.float32: native.DTYPE_F32, torch.bfloat16: native.DTYPE_BF16, torch.float16: native.DTYPE_F16}
        code = native.load_library().moe_q4_moe_layer_u16(
            native._ptr(x), rdt[x.dtype], T, cfg.hidden, cfg.inter, native._ptr(rw), rdt[rw.dtype], cfg.n_experts,
            cfg.top_k, native._ptr(tables), int(layout), native._ptr(out), native._ptr(ids), native._ptr(weights),
            native._ptr(ws), ws.numel(), native._stream())
        native._check(code, "moe_q4_moe_layer_u16")
        return out

"""Expert-parallel DeepSeek-V3 MoE layer: one process per GPU, experts
partitioned over the ranks, tokens exchanged with all-to-all collectives.

Rank r of N owns routed experts [r * E / N, (r + 1) * E / N); the router and
the shared expert are replicated.  A layer step on each rank, for that rank's
own tokens (the reference's run_fp8_moe flow, fp8_source.py:1569-1884, with
the per-expert loop spread over the ranks):

  1. route (sigmoid + bias, group-limited top-k; weights rounded through the
     hidden dtype as fp8_source.py:1547 does);
  2. pack the (token, slot) entries by destination rank -- token rows, the
     expert id local to that rank, and where each entry went;
  3. all-to-all of the per-rank counts, then of the rows and expert ids;
  4. grouped FP8 experts over the received rows, plus the shared expert over
     the rank's own rows in the same launch;
  5. reverse all-to-all of the fp32 expert outputs;
  6. combine at home in top-k slot order, then the shared expert, one bf16
     rounding -- the order of the single-GPU layer.

The counts exchange needs the sizes on the host (NCCL collectives take host
counts), so a step synchronises once.  The compute steps go through an ops
object: CudaEPOps calls libmoe_b200's kernels; tests substitute a CPU
implementation to check the exchange logic with gloo ranks.

On GPUs the default exchange (PeerExchange) has no host synchronisation and
no collective on the data path: receive and return buffers live in torch
symmetric memory, the dispatch kernel writes each row straight into its
destination rank's buffer over NVLink and the return kernel writes each
output row back into its source rank's buffer; only the [world] entry counts
go through an NCCL all-gather, and two one-element NCCL all-reduces order
the steps across ranks (no device-side waiting of our own).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import native, synth


@dataclass
class Packed:
    send_rows: torch.Tensor     # bf16 [T*k, H], grouped by destination rank
    send_expert: torch.Tensor   # int32 [T*k], expert id local to the destination
    send_offsets: torch.Tensor  # int32 [N + 1]
    entry_pos: torch.Tensor     # int32 [T*k]: send position of entry t*k + slot
    pos_weight: torch.Tensor    # fp32 [T*k]: routing weight at each send position


class CudaEPOps:
    """The compute steps on the GPU (libmoe_b200)."""

    def __init__(self, layer: "ExpertParallelLayer"):
        self.layer = layer
        self.lib = native.load_library()
        self._ws = torch.empty((0,), dtype=torch.uint8, device=layer.device)

    def _workspace(self, nbytes: int) -> torch.Tensor:
        if self._ws.numel() < nbytes:
            self._ws = torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=self.layer.device)
        return self._ws

    def route(self, x: torch.Tensor):
        L = self.layer
        cfg = L.cfg
        return native.route_topk(x, L.router_weight, L.bias, top_k=cfg.top_k, n_group=cfg.n_group,
                                 topk_group=cfg.topk_group, scoring_func=cfg.scoring_func,
                                 route_scale=cfg.route_scale, round_to_hidden_dtype=True, weights_fp32=True)

    def pack(self, ids: torch.Tensor, w: torch.Tensor, x: torch.Tensor) -> Packed:
        L = self.layer
        T, k, H = int(ids.shape[0]), int(ids.shape[1]), L.cfg.hidden
        dev = x.device
        p = Packed(torch.empty((T * k, H), dtype=torch.bfloat16, device=dev),
                   torch.empty((T * k,), dtype=torch.int32, device=dev),
                   torch.empty((L.world + 1,), dtype=torch.int32, device=dev),
                   torch.empty((T * k,), dtype=torch.int32, device=dev),
                   torch.empty((T * k,), dtype=torch.float32, device=dev))
        ws = self._workspace(int(self.lib.moe_ep_dispatch_workspace_bytes(T, k)))
        code = self.lib.moe_ep_dispatch_pack(
            native._ptr(ids), native._ptr(w), native._ptr(x), T, H, k, L.cfg.n_routed, L.world,
            native._ptr(p.send_rows), native._ptr(p.send_expert), native._ptr(p.send_offsets),
            native._ptr(p.entry_pos), native._ptr(p.pos_weight), native._ptr(ws), ws.numel(), native._stream())
        native._check(code, "moe_ep_dispatch_pack")
        return p

    def experts(self, rows: torch.Tensor, row_expert: torch.Tensor) -> torch.Tensor:
        L = self.layer
        R = int(rows.shape[0])
        out = torch.empty((R, L.cfg.hidden), dtype=torch.float32, device=rows.device)
        ws = self._workspace(int(self.lib.moe_ep_experts_workspace_bytes(R, L.cfg.hidden, L.cfg.inter, L.n_local + 1)))
        layout = 1 if L.tables_tiled is not None and self.lib.moe_b200_selected_gemv() == 0 else 0
        tables = L.tables_tiled if layout else L.tables
        code = self.lib.moe_ep_experts_fp8(
            native._ptr(rows), native._ptr(row_expert), R, L.cfg.hidden, L.cfg.inter, native._ptr(tables),
            L.n_local + 1, native._ptr(L.nan_free), layout, native._ptr(out), native._ptr(ws), ws.numel(),
            native._stream())
        native._check(code, "moe_ep_experts_fp8")
        return out

    def experts_home(self, rows: torch.Tensor, row_expert: torch.Tensor, row_src: torch.Tensor, src_stride: int,
                     peer_yback: torch.Tensor, valid_rows: int = 0, home_rows: int | None = None) -> None:
        """experts() with each output row written into its source rank's
        return buffer (moe_ep_experts_return_p2p); valid_rows: the rows
        expected to carry a local expert (picks the kernel; 0 = all);
        home_rows: the rows of every rank's return buffer (default
        src_stride) -- a src code pointing outside them is not stored."""
        L = self.layer
        R = int(rows.shape[0])
        layout = 1 if L.tables_tiled is not None and self.lib.moe_b200_selected_gemv() == 0 else 0
        ws = self._workspace(int(self.lib.moe_ep_experts_return_p2p_workspace_bytes(
            R, valid_rows, L.cfg.hidden, L.cfg.inter, L.n_local + 1, layout)))
        tables = L.tables_tiled if layout else L.tables
        code = self.lib.moe_ep_experts_return_p2p(
            native._ptr(rows), native._ptr(row_expert), native._ptr(row_src), R, valid_rows, L.cfg.hidden,
            L.cfg.inter,
            native._ptr(tables), L.n_local + 1, native._ptr(L.nan_free), layout, src_stride, L.world,
            src_stride if home_rows is None else int(home_rows), native._ptr(peer_yback),
            native._ptr(ws), ws.numel(), native._stream())
        native._check(code, "moe_ep_experts_return_p2p")

    def combine(self, y: torch.Tensor, p: Packed, T: int) -> torch.Tensor:
        """y: the expert output rows in bf16 (rounded once, as the reference rounds them)."""
        L = self.layer
        k = L.cfg.top_k
        if y.dtype != torch.bfloat16:
            y = y.to(torch.bfloat16)
        out = torch.empty((T, L.cfg.hidden), dtype=torch.bfloat16, device=y.device)
        code = self.lib.moe_ep_combine(native._ptr(y), native.DTYPE_BF16, native._ptr(p.entry_pos),
                                       native._ptr(p.pos_weight), T, k,
                                       L.cfg.hidden, 1, native._ptr(out), native._stream())
        native._check(code, "moe_ep_combine")
        return out


class PeerExchange:
    """Symmetric-memory buffers for a layer's peer-to-peer exchange, sized for
    up to `max_tokens` tokens per rank and step.

    sync: how the ranks order a step's three phases (counts exchanged, rows
    landed, outputs home) -- "p2p" (default): moe_ep_barrier_p2p, a one-CTA
    kernel that signals every peer through its symmetric signal buffer and
    waits (bounded) for theirs, carrying the counts row for the all-gather;
    "nccl": an NCCL all-gather and two one-element all-reduces."""

    BARRIER_LIMIT_US = 10_000_000  # a peer 10 s late is an error (code 256), not a hang

    def __init__(self, layer: "ExpertParallelLayer", max_tokens: int, sync: str = "p2p"):
        import torch.distributed._symmetric_memory as symm

        if sync not in ("p2p", "nccl"):
            raise ValueError("sync must be p2p or nccl")
        self.sync = sync

        L = layer
        cfg = L.cfg
        dev = L.device
        self.max_tokens = int(max_tokens)
        self.stride = self.max_tokens * cfg.top_k            # routed entries of one rank
        self.src_stride = self.stride + self.max_tokens       # return rows of one rank (src encoding)
        self.capacity = L.world * self.stride                 # rows one rank can receive
        H = cfg.hidden
        group = L.group if L.group is not None else dist.group.WORLD
        self.rows = symm.empty((self.capacity + self.max_tokens, H), dtype=torch.bfloat16, device=dev)
        self.expert = symm.empty((self.capacity + self.max_tokens,), dtype=torch.int32, device=dev)
        self.src = symm.empty((self.capacity + self.max_tokens,), dtype=torch.int32, device=dev)
        # return rows in bf16: each expert output is rounded there, as the reference rounds it
        self.yback = symm.empty((self.stride + self.max_tokens, H), dtype=torch.bfloat16, device=dev)
        # the [world][world] counts (row = source rank) and the barrier's signal slots, peer-written too
        self.matrix = symm.empty((L.world * L.world,), dtype=torch.int32, device=dev)
        self.sig = symm.empty((L.world,), dtype=torch.int32, device=dev)
        self.handles = [symm.rendezvous(t, group) for t in (self.rows, self.expert, self.src, self.yback,
                                                            self.matrix, self.sig)]
        self.peers = [torch.tensor([int(p) for p in h.buffer_ptrs], dtype=torch.int64, device=dev)
                      for h in self.handles]
        self.flag = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.counts = torch.empty((L.world,), dtype=torch.int32, device=dev)
        self.sig.zero_()
        self.epoch = torch.zeros((1,), dtype=torch.int32, device=dev)  # this rank's barrier count
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)  # every rank's signal slots are zero before the first barrier
        self.identity = torch.arange(self.stride, dtype=torch.int32, device=dev)
        self._shared_src = {}  # tokens -> src codes of this rank's shared-expert rows
        self.lib = native.load_library()
        self._ws = torch.empty((0,), dtype=torch.uint8, device=dev)

    def _barrier(self, L: "ExpertParallelLayer", payload: torch.Tensor | None = None) -> None:
        """Every rank reaches this point before any goes on; with payload (this
        rank's [world] counts), the counts matrix is all-gathered too."""
        if self.sync == "nccl":
            if payload is not None:
                dist.all_gather_into_tensor(self.matrix, payload, group=L.group)
            else:
                dist.all_reduce(self.flag, group=L.group)
            return
        has = payload is not None
        native._check(self.lib.moe_ep_barrier_p2p(
            native._ptr(self.peers[5]), L.world, L.rank, native._ptr(self.epoch),
            native._ptr(payload) if has else None, L.world if has else 0, native._ptr(self.peers[4]) if has else None,
            self.BARRIER_LIMIT_US, native._stream()), "moe_ep_barrier_p2p")

    FUSED_SEND_MAX_ROWS = 128  # routed rows per rank the one-CTA send moves (more: the multi-CTA scatter)

    def _fused_send(self, L: "ExpertParallelLayer", x: torch.Tensor) -> bool:
        """Whether this step's send side runs as moe_ep_route_dispatch_p2p (the
        router logits, then one CTA for selection, dispatch and both barriers).
        Small decode batches only: one CTA stores every routed row over NVLink,
        which for 128 rows of 14 KB (16 tokens of DS-V3) is about 1.8 MB."""
        cfg = L.cfg
        return (self.sync == "p2p" and isinstance(L.ops, CudaEPOps) and x.dtype == torch.bfloat16
                and cfg.scoring_func == "sigmoid" and L.bias is not None
                and L.router_weight.dtype in (torch.bfloat16, torch.float16)
                and self.max_tokens * cfg.top_k <= self.FUSED_SEND_MAX_ROWS and cfg.n_routed <= 256
                and L.world <= 32 and cfg.hidden % 8 == 0)

    def forward(self, L: "ExpertParallelLayer", x: torch.Tensor):
        cfg, lib = L.cfg, self.lib
        T, k, H = int(x.shape[0]), cfg.top_k, cfg.hidden
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange's {self.max_tokens}")
        if self._fused_send(L, x):
            return self._forward_fused(L, x)
        if T == 0:  # nothing to send; this rank still takes every step (it may receive rows)
            ids, w = L._no_routes(x)
            self.counts.zero_()
        else:
            ids, w = L.ops.route(x)
            native._check(lib.moe_ep_count_ranks(native._ptr(ids), T, k, cfg.n_routed, L.world,
                                                 native._ptr(self.counts), native._stream()), "moe_ep_count_ranks")
        # empty receive slots; peers write only after the counts' all-gather, which this rank joins after the reset
        self.expert.fill_(-1)
        self._barrier(L, payload=self.counts)
        if T > 0:
            need = int(lib.moe_ep_dispatch_p2p_workspace_bytes(T, k, L.world))
            if self._ws.numel() < need:
                self._ws = torch.empty((need,), dtype=torch.uint8, device=x.device)
            native._check(lib.moe_ep_dispatch_p2p(
                native._ptr(ids), native._ptr(x), T, H, k, cfg.n_routed, L.world, L.rank,
                native._ptr(self.matrix), self.capacity, self.src_stride, native._ptr(self.peers[0]),
                native._ptr(self.peers[1]), native._ptr(self.peers[2]), native._ptr(self._ws), self._ws.numel(),
                native._stream()), "moe_ep_dispatch_p2p")
        self._barrier(L)  # every rank's rows have landed
        C = self.capacity
        self.rows[C:C + T].copy_(x)
        self.expert[C:C + T].fill_(L.n_local)      # the shared expert, last in the local tables
        if T not in self._shared_src:              # its outputs go to this rank's return rows T*k + t
            self._shared_src[T] = (torch.arange(T, dtype=torch.int32, device=x.device)
                                   + (L.rank * self.src_stride + T * k))
        self.src[C:C + T].copy_(self._shared_src[T])
        # the local experts; every output row is stored straight into its source rank's return buffer.
        # Rows expected: T * k routed (a rank receives about what it sends) + T shared
        L.ops.experts_home(self.rows[:C + T], self.expert[:C + T], self.src[:C + T], self.src_stride,
                           self.peers[3], valid_rows=max(T, 1) * (k + 1))
        self._barrier(L)  # every output row is home
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        if T == 0:
            return out, ids, w
        w_flat = w.reshape(-1).contiguous()  # referenced until the launch (a temporary could be freed first)
        native._check(lib.moe_ep_combine(native._ptr(self.yback), native.DTYPE_BF16, native._ptr(self.identity),
                                         native._ptr(w_flat), T, k, H, 1, native._ptr(out), native._stream()),
                      "moe_ep_combine")
        return out, ids, w


    def _forward_fused(self, L: "ExpertParallelLayer", x: torch.Tensor):
        """A decode step with the send side fused (moe_ep_route_dispatch_p2p):
        the same rows, slots, codes and barriers as forward()'s launches, so the
        same bits."""
        cfg, lib = L.cfg, self.lib
        T, k, H = int(x.shape[0]), cfg.top_k, cfg.hidden
        dev = x.device
        ids = torch.empty((T, k), dtype=torch.int64, device=dev)
        w = torch.empty((T, k), dtype=torch.float32, device=dev)
        need = int(lib.moe_ep_route_dispatch_p2p_workspace_bytes(T, cfg.n_routed))
        if self._ws.numel() < need:
            self._ws = torch.empty((need,), dtype=torch.uint8, device=dev)
        rw_dtype = native.DTYPE_BF16 if L.router_weight.dtype == torch.bfloat16 else native.DTYPE_F16
        native._check(lib.moe_ep_route_dispatch_p2p(
            native._ptr(x) if T else None, native._ptr(L.router_weight), rw_dtype, native._ptr(L.bias), T, H,
            cfg.n_routed, cfg.n_group, cfg.topk_group, k, float(cfg.route_scale), L.world, L.rank, self.capacity,
            self.src_stride, native._ptr(self.peers[0]), native._ptr(self.peers[1]), native._ptr(self.peers[2]),
            native._ptr(self.peers[4]), native._ptr(self.peers[5]), native._ptr(self.epoch), self.BARRIER_LIMIT_US,
            native._ptr(ids) if T else None, native._ptr(w) if T else None, native._ptr(self._ws),
            self._ws.numel(), native._stream()), "moe_ep_route_dispatch_p2p")
        C = self.capacity
        L.ops.experts_home(self.rows[:C + T], self.expert[:C + T], self.src[:C + T], self.src_stride,
                           self.peers[3], valid_rows=max(T, 1) * (k + 1))
        self._barrier(L)  # every output row is home
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        if T == 0:
            return out, ids, w
        w_flat = w.reshape(-1)  # referenced until the launch
        native._check(lib.moe_ep_combine(native._ptr(self.yback), native.DTYPE_BF16, native._ptr(self.identity),
                                         native._ptr(w_flat), T, k, H, 1, native._ptr(out), native._stream()),
                      "moe_ep_combine")
        return out, ids, w


class GraphedExpertParallelLayer:
    """An ExpertParallelLayer step with the peer exchange for one token count,
    captured as a CUDA graph (its kernels, memsets and the exchange's barriers:
    peer-memory kernels, or NCCL collectives with sync="nccl").  Every rank captures and replays in step.  Write the tokens
    into `.input` (or pass them to __call__), replay, read `.output`.
    Release it (del) before destroying the process group."""

    def __init__(self, layer: "ExpertParallelLayer", tokens: int):
        if layer.peer is None:
            raise ValueError("graph capture needs the peer exchange (no host-synchronised counts)")
        cfg, dev = layer.cfg, layer.device
        self.input = torch.zeros((tokens, cfg.hidden), dtype=torch.bfloat16, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):  # kernel attributes, workspaces, NCCL set-up outside the capture
                layer.forward(self.input)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.output, self.ids, self.weights = layer.forward(self.input)
        torch.cuda.synchronize(dev)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.output

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        self.input.copy_(hidden.reshape(self.input.shape), non_blocking=True)
        return self.replay()


class ExpertParallelLayer:
    """This rank's share of one expert-parallel DS-V3 MoE layer.

    `layer` may be a full or partial synth.Fp8MoELayer holding at least the
    router, this rank's experts and the shared expert; by default they are
    generated from `seed` (identical on every rank)."""

    def __init__(self, cfg: synth.DsMoEConfig, rank: int, world: int, *, group=None, seed: int = 20,
                 device: torch.device | str | None = None, layer: synth.Fp8MoELayer | None = None, ops=None,
                 exchange: str = "auto", max_tokens: int = 64, peer: "PeerExchange | None" = None,
                 row_major: bool = True, peer_sync: str = "p2p"):
        if cfg.n_routed % world:
            raise ValueError("the routed experts must split evenly over the ranks")
        self.cfg, self.rank, self.world, self.group = cfg, int(rank), int(world), group
        self.n_local = cfg.n_routed // world
        self.first = self.rank * self.n_local
        local = list(range(self.first, self.first + self.n_local)) + [cfg.n_routed]
        if device is None:
            device = native._device()
        self.device = torch.device(device)
        if layer is None:
            layer = synth.make_fp8_layer(cfg, seed=seed, device=self.device, experts=local)
        self.layer = layer
        self.router_weight = layer.router_weight.to(self.device)
        self.bias = layer.bias.to(self.device)
        # local tables [6][n_local + 1]: this rank's experts, then the shared expert
        self.local_experts = [[t.to(self.device) for t in layer.expert(e)] for e in local]
        self.tables = torch.tensor([[int(ex[j].data_ptr()) for ex in self.local_experts] for j in range(6)],
                                   dtype=torch.int64, device=self.device) if self.device.type == "cuda" else None
        self.nan_free = None
        self.tables_tiled = None
        if self.device.type == "cuda":
            lib = native.load_library()
            n = self.n_local + 1
            self.nan_free = torch.zeros((n,), dtype=torch.uint8, device=self.device)
            native._check(lib.moe_fp8_nan_free_flags(
                native._ptr(self.tables), n, cfg.inter, cfg.hidden, native._ptr(self.nan_free),
                native._stream()), "moe_fp8_nan_free_flags")
            if cfg.hidden % 128 == 0 and cfg.inter % 128 == 0:
                # the decode GEMV's fragment-native copy of the local experts (moe_fp8_tile_weights)
                tb13 = int(lib.moe_fp8_tiled_bytes(cfg.inter, cfg.hidden))
                tb2 = int(lib.moe_fp8_tiled_bytes(cfg.hidden, cfg.inter))
                self._tiled13 = torch.empty((n, 2, tb13), dtype=torch.uint8, device=self.device)
                self._tiled2 = torch.empty((n, tb2), dtype=torch.uint8, device=self.device)
                cols = [[int(ex[j].data_ptr()) for ex in self.local_experts] for j in range(6)]
                for i, (g, _gs, u, _us, d, _ds) in enumerate(self.local_experts):
                    for src, dst, rows, k in ((g, self._tiled13[i, 0], cfg.inter, cfg.hidden),
                                              (u, self._tiled13[i, 1], cfg.inter, cfg.hidden),
                                              (d, self._tiled2[i], cfg.hidden, cfg.inter)):
                        native._check(lib.moe_fp8_tile_weights(native._ptr(src), native._ptr(dst), rows, k,
                                                               native._stream()), "moe_fp8_tile_weights")
                    cols[0][i] = int(self._tiled13[i, 0].data_ptr())
                    cols[2][i] = int(self._tiled13[i, 1].data_ptr())
                    cols[4][i] = int(self._tiled2[i].data_ptr())
                self.tables_tiled = torch.tensor(cols, dtype=torch.int64, device=self.device)
        self.ops = ops(self) if ops is not None else CudaEPOps(self)
        # "p2p": PeerExchange (GPUs, NCCL group); "nccl": all-to-alls with host counts; "auto": p2p when possible
        if exchange not in ("auto", "p2p", "nccl"):
            raise ValueError("exchange must be auto, p2p or nccl")
        if not row_major:
            # keep only the tiled copy the default GEMV and the GEMM read (half the memory): drop the
            # row-major codes and the source layer; the scales stay
            if self.tables_tiled is None:
                raise ValueError("row_major=False needs the tiled copy (CUDA, hidden and intermediate % 128 == 0)")
            self.local_experts = [[None, ex[1], None, ex[3], None, ex[5]] for ex in self.local_experts]
            self.tables = None
            self.layer = layer = None
        use_p2p = exchange == "p2p" or (exchange == "auto" and ops is None and self.device.type == "cuda"
                                        and dist.is_initialized() and dist.get_backend(group) == "nccl")
        if peer is not None:  # layers run one after another, so one set of exchange buffers serves them all
            if not use_p2p:
                raise ValueError("a shared peer exchange needs exchange='p2p' or 'auto' on an NCCL group")
            self.peer = peer
        else:
            self.peer = PeerExchange(self, max_tokens, sync=peer_sync) if use_p2p else None

    def capture(self, tokens: int) -> GraphedExpertParallelLayer:
        """A CUDA graph of one step for `tokens` tokens per rank (peer exchange only)."""
        return GraphedExpertParallelLayer(self, tokens)

    def forward(self, x: torch.Tensor):
        """x [T, H] bf16 (this rank's tokens) -> (out [T, H] bf16, ids [T, k], weights fp32 [T, k])."""
        cfg, ops = self.cfg, self.ops
        x = x.reshape(-1, cfg.hidden).contiguous()
        if self.peer is not None:
            return self.peer.forward(self, x)
        T, k, H = int(x.shape[0]), cfg.top_k, cfg.hidden
        if T == 0:  # nothing to route; this rank still exchanges (it may receive rows) in step with the others
            ids, w = self._no_routes(x)
            p = Packed(torch.empty((0, H), dtype=torch.bfloat16, device=x.device),
                       torch.empty((0,), dtype=torch.int32, device=x.device),
                       torch.zeros((self.world + 1,), dtype=torch.int32, device=x.device),
                       torch.empty((0,), dtype=torch.int32, device=x.device),
                       torch.empty((0,), dtype=torch.float32, device=x.device))
        else:
            ids, w = ops.route(x)
            p = ops.pack(ids, w, x)
        send_counts = (p.send_offsets[1:] - p.send_offsets[:-1]).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts]).cpu()  # the step's one host synchronisation
        sc, rc = counts[0].tolist(), counts[1].tolist()
        R = int(sum(rc))
        rows = torch.empty((R + T, H), dtype=torch.bfloat16, device=x.device)
        row_expert = torch.empty((R + T,), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(rows[:R], p.send_rows, rc, sc, group=self.group)
        dist.all_to_all_single(row_expert[:R], p.send_expert, rc, sc, group=self.group)
        rows[R:].copy_(x)
        row_expert[R:].fill_(self.n_local)  # the shared expert, last in the local tables
        y = ops.experts(rows, row_expert) if R + T > 0 else torch.empty((0, H), dtype=torch.float32,
                                                                        device=x.device)
        # the outputs rounded to bf16 (round to nearest even, as the peer exchange's kernels round them)
        y16 = y.to(torch.bfloat16)
        y_back = torch.empty((T * k + T, H), dtype=torch.bfloat16, device=x.device)
        dist.all_to_all_single(y_back[:T * k], y16[:R], sc, rc, group=self.group)
        y_back[T * k:].copy_(y16[R:])
        if T == 0:
            return torch.empty((0, H), dtype=torch.bfloat16, device=x.device), ids, w
        return ops.combine(y_back, p, T), ids, w

    def _no_routes(self, x: torch.Tensor):
        k = self.cfg.top_k
        return (torch.empty((0, k), dtype=torch.int64, device=x.device),
                torch.empty((0, k), dtype=torch.float32, device=x.device))


class ExpertParallelStack:
    """A stack of expert-parallel DS-V3 MoE layers with the attention blocks
    replaced by the identity: h <- h + moe_l(h) for l = 0 .. n_layers - 1, in
    bf16 (the routed-expert stack of a decode step).  Layer l is generated
    from seed + l unless `layers` gives it; every layer keeps only the tiled
    copy of its experts on GPUs (row_major=False), and the layers share one
    peer exchange, whose buffers serve one layer after the other."""

    def __init__(self, cfg: synth.DsMoEConfig, rank: int, world: int, n_layers: int, *, group=None,
                 seed: int = 20, device: torch.device | str | None = None,
                 layers: list[synth.Fp8MoELayer] | None = None, ops=None, exchange: str = "auto",
                 max_tokens: int = 64, row_major: bool | None = None, peer_sync: str = "p2p"):
        if n_layers < 1 or (layers is not None and len(layers) != n_layers):
            raise ValueError("n_layers must be >= 1 and match `layers`")
        self.cfg, self.world = cfg, int(world)
        self.layers: list[ExpertParallelLayer] = []
        peer = None
        for li in range(n_layers):
            given = layers[li] if layers is not None else None
            keep = row_major if row_major is not None else (ops is not None or torch.device(
                device if device is not None else native._device()).type != "cuda")
            ep = ExpertParallelLayer(cfg, rank, world, group=group, seed=seed + li, device=device, layer=given,
                                     ops=ops, exchange=exchange, max_tokens=max_tokens, peer=peer, row_major=keep,
                                     peer_sync=peer_sync)
            peer = ep.peer
            self.layers.append(ep)
            del given, ep
        self.device = self.layers[0].device
        self.peer = peer

    def forward(self, x: torch.Tensor, ids_out: list | None = None) -> torch.Tensor:
        """x [T, H] bf16 (this rank's tokens, T may be 0) -> h [T, H] bf16 after
        every layer; ids_out, when given, receives each layer's expert ids."""
        h = x.reshape(-1, self.cfg.hidden).to(torch.bfloat16)
        for ep in self.layers:
            out, ids, _w = ep.forward(h)
            if ids_out is not None:
                ids_out.append(ids)
            h = h + out
        return h

    def capture(self, tokens: int) -> "GraphedExpertParallelStack":
        """One CUDA graph of the whole stack for `tokens` tokens on this rank (peer exchange only)."""
        return GraphedExpertParallelStack(self, tokens)


class GraphedExpertParallelStack:
    """ExpertParallelStack.forward for one token count captured as one CUDA
    graph (every layer's kernels, memsets, residual adds and NCCL calls).
    Every rank captures and replays in step; release it (del) before
    destroying the process group."""

    def __init__(self, stack: ExpertParallelStack, tokens: int):
        if stack.peer is None:
            raise ValueError("graph capture needs the peer exchange (no host-synchronised counts)")
        dev = stack.device
        self.input = torch.zeros((tokens, stack.cfg.hidden), dtype=torch.bfloat16, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):  # kernel attributes, workspaces, NCCL set-up outside the capture
                stack.forward(self.input)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.output = stack.forward(self.input)
        torch.cuda.synchronize(dev)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.output

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        self.input.copy_(hidden.reshape(self.input.shape), non_blocking=True)
        return self.replay()

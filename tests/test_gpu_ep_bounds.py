"""Range checks of the expert-parallel peer kernels, on one GPU with local
buffers only.

The peer kernels store into addresses built from values other ranks wrote
(src codes, exchanged counts).  Each test declares a buffer smaller than its
real allocation (and, for the rank check, a device table with one more entry
than the declared world, that entry pointing at this GPU's buffer too), then
feeds codes just past the declared bounds.  A store that a broken check let
through would still land in memory this process owns, so the test cannot
fault; it expects the error code (64) from moe_b200_device_error and the
memory past the declared bounds untouched."""

import pytest
import torch

from pocketlm_b200 import native, synth
from pocketlm_b200.runtime import DsMoELayerGPU

pytestmark = pytest.mark.gpu

SENTINEL = -7.0
EP_RANGE_ERROR = 64


def _lib():
    return native.load_library()


def _device_error() -> int:
    return int(_lib().moe_b200_device_error(native._stream()))


def _table(*tensors) -> torch.Tensor:
    return torch.tensor([int(t.data_ptr()) for t in tensors], dtype=torch.int64, device="cuda")


def test_return_p2p_skips_out_of_range_src(cuda_device):
    assert _device_error() == 0
    H, src_stride, home_rows = 64, 8, 6
    big = torch.full((32, H), SENTINEL, dtype=torch.float32, device=cuda_device)
    base = big[16:]  # 16 owned rows on either side of the declared return buffer
    peers = _table(base, base)  # declared world 1; entry 1 exists only so a missed rank check stays local
    y = torch.randn((6, H), device=cuda_device)
    expert = torch.tensor([0, 0, 0, 0, 0, -1], dtype=torch.int32, device=cuda_device)
    # rows 0 and 5 in range; 6 = home_rows; 9 = rank 1 of a world of 1; -3 negative; the last row has no expert
    src = torch.tensor([0, 5, 6, 9, -3, 2], dtype=torch.int32, device=cuda_device)
    code = _lib().moe_ep_return_p2p(native._ptr(y), 6, native._ptr(expert), native._ptr(src), H, src_stride, 1,
                                    home_rows, native._ptr(peers), native._stream())
    native._check(code, "moe_ep_return_p2p")
    assert _device_error() == EP_RANGE_ERROR
    assert torch.equal(base[0], y[0]) and torch.equal(base[5], y[1])
    untouched = torch.ones(32, dtype=torch.bool)
    untouched[16 + 0] = untouched[16 + 5] = False
    assert (big[untouched] == SENTINEL).all()
    assert _device_error() == 0  # the word was cleared by the read


def test_dispatch_p2p_skips_slots_past_capacity(cuda_device):
    assert _device_error() == 0
    T, k, H, E, world, rank, capacity, src_stride = 3, 2, 64, 16, 2, 1, 5, 8
    ids = torch.tensor([[1, 9], [2, 3], [10, 11]], dtype=torch.int64, device=cuda_device)
    x = torch.randn((T, H), device=cuda_device).to(torch.bfloat16)
    # rank 0 sent 2 rows to rank 0 and 4 to rank 1: this rank's slots are 2, 3, 4 there and 4, 5, 6 here
    matrix = torch.tensor([2, 4, 0, 0], dtype=torch.int32, device=cuda_device)
    rows = [torch.zeros((12, H), dtype=torch.bfloat16, device=cuda_device) for _ in range(world)]
    expert = [torch.full((12,), -5, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    srcs = [torch.full((12,), -5, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    need = int(_lib().moe_ep_dispatch_p2p_workspace_bytes(T, k, world))
    ws = torch.empty((need,), dtype=torch.uint8, device=cuda_device)
    # the device tables stay referenced until the kernel has run (a freed one could be reused by the next)
    peer_rows, peer_expert, peer_src = _table(*rows), _table(*expert), _table(*srcs)
    code = _lib().moe_ep_dispatch_p2p(
        native._ptr(ids), native._ptr(x), T, H, k, E, world, rank, native._ptr(matrix), capacity, src_stride,
        native._ptr(peer_rows), native._ptr(peer_expert), native._ptr(peer_src), native._ptr(ws),
        ws.numel(), native._stream())
    native._check(code, "moe_ep_dispatch_p2p")
    assert _device_error() == EP_RANGE_ERROR
    # destination 0: entries (token 0 slot 0), (1, 0), (1, 1) -> slots 2, 3, 4
    assert torch.equal(rows[0][2:5], x[[0, 1, 1]])
    assert expert[0][2:5].tolist() == [1, 2, 3]
    assert srcs[0][2:5].tolist() == [rank * src_stride + e for e in (0, 2, 3)]
    # destination 1: entry (0, 1) -> slot 4 stored; (2, 0), (2, 1) -> slots 5, 6 >= capacity, not stored
    assert torch.equal(rows[1][4], x[0]) and expert[1][4].item() == 1 and srcs[1][4].item() == rank * src_stride + 1
    assert (rows[1][5:] == 0).all() and (expert[1][5:] == -5).all() and (srcs[1][5:] == -5).all()
    assert (rows[0][5:] == 0).all() and (expert[0][:2] == -5).all() and (expert[1][:4] == -5).all()


@pytest.mark.parametrize("n_rows", [8, 640])
def test_experts_return_p2p_keeps_bad_homes_local(cuda_device, n_rows):
    """8 rows run the warp-MMA experts and a copy kernel, 640 rows the
    tcgen05 GEMM whose epilogue stores the rows home; rows with a bad home
    are computed into the caller's own workspace and never stored."""
    assert _device_error() == 0
    cfg = synth.C1_TINY
    layer = DsMoELayerGPU(synth.make_fp8_layer(cfg, seed=5, device=cuda_device))
    H, S = cfg.hidden, cfg.n_routed + 1
    gen = torch.Generator(device="cpu").manual_seed(11)
    rows = (torch.randn((n_rows, H), generator=gen)).to(torch.bfloat16).to(cuda_device)
    row_expert = torch.randint(0, S, (n_rows,), generator=gen, dtype=torch.int32).to(cuda_device)
    lib = _lib()
    layout = 1 if n_rows >= 512 else 0
    tables = layer.tables_tiled if layout else layer.tables
    want = torch.empty((n_rows, H), dtype=torch.float32, device=cuda_device)
    ws = torch.empty((int(lib.moe_ep_experts_workspace_bytes(n_rows, H, cfg.inter, S)),), dtype=torch.uint8,
                     device=cuda_device)
    native._check(lib.moe_ep_experts_fp8(native._ptr(rows), native._ptr(row_expert), n_rows, H, cfg.inter,
                                         native._ptr(tables), S, native._ptr(layer.nan_free), layout,
                                         native._ptr(want), native._ptr(ws), ws.numel(), native._stream()),
                  "moe_ep_experts_fp8")
    src_stride = n_rows + 8
    home_rows = n_rows  # declared; the real buffer has 16 more rows on each side
    margin = 16
    big = torch.full((src_stride + 2 * margin, H), SENTINEL, dtype=torch.float32, device=cuda_device)
    base = big[margin:]
    peers = _table(base, base)
    src = torch.randperm(n_rows, generator=gen).to(torch.int32)
    bad = {1: home_rows, 3: src_stride - 1, 4: src_stride + 2, 6: -2}  # row, past the rows, rank 1, negative
    for j, code in bad.items():
        src[j] = code
    src = src.to(cuda_device)
    need = int(lib.moe_ep_experts_return_p2p_workspace_bytes(n_rows, 0, H, cfg.inter, S, layout))
    ws = torch.empty((need,), dtype=torch.uint8, device=cuda_device)
    code = lib.moe_ep_experts_return_p2p(
        native._ptr(rows), native._ptr(row_expert), native._ptr(src), n_rows, 0, H, cfg.inter, native._ptr(tables), S,
        native._ptr(layer.nan_free), layout, src_stride, 1, home_rows, native._ptr(peers), native._ptr(ws),
        ws.numel(), native._stream())
    native._check(code, "moe_ep_experts_return_p2p")
    assert _device_error() == EP_RANGE_ERROR
    good = [j for j in range(n_rows) if j not in bad]
    src_cpu = src.cpu()
    homes = torch.tensor([int(src_cpu[j]) for j in good])
    assert torch.equal(base[homes.to(cuda_device)], want[good])
    untouched = torch.ones(big.shape[0], dtype=torch.bool)
    untouched[homes + margin] = False
    assert (big[untouched.to(cuda_device)] == SENTINEL).all()

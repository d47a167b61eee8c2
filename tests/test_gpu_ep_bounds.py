"""Range checks of the expert-parallel peer kernels and the bounded wait of
the peer-memory barrier, on one GPU with local buffers only.

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
    big = torch.full((32, H), SENTINEL, dtype=torch.bfloat16, device=cuda_device)  # bf16 return rows
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
    assert torch.equal(base[0], y[0].to(torch.bfloat16)) and torch.equal(base[5], y[1].to(torch.bfloat16))
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
    big = torch.full((src_stride + 2 * margin, H), SENTINEL, dtype=torch.bfloat16, device=cuda_device)
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
    assert torch.equal(base[homes.to(cuda_device)], want[good].to(torch.bfloat16))  # rounded once, to nearest
    untouched = torch.ones(big.shape[0], dtype=torch.bool)
    untouched[homes + margin] = False
    assert (big[untouched.to(cuda_device)] == SENTINEL).all()


EP_WAIT_ERROR = 256


def test_barrier_single_rank_and_payload(cuda_device):
    """World 1: the rank signals its own slot and passes at once; the payload
    lands in its own counts row; the epoch counts barriers."""
    assert _device_error() == 0
    sig = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    matrix = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
    epoch = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    payload = torch.tensor([7], dtype=torch.int32, device=cuda_device)
    peers_sig, peers_mat = _table(sig), _table(matrix)
    lib = _lib()
    for i in range(3):
        has = i == 1
        code = lib.moe_ep_barrier_p2p(native._ptr(peers_sig), 1, 0, native._ptr(epoch),
                                      native._ptr(payload) if has else None, 1 if has else 0,
                                      native._ptr(peers_mat) if has else None, 1_000_000, native._stream())
        native._check(code, "moe_ep_barrier_p2p")
    assert epoch.item() == 3 and sig.item() == 3 and matrix.item() == 7
    assert _device_error() == 0


def test_barrier_wait_runs_out_and_reports(cuda_device):
    """World 2 with no second rank: this rank's signal to "rank 1" lands in a
    local stand-in buffer, and nothing ever writes rank 1's slot here, so the
    wait runs out after its limit (50 ms), sets code 256 and returns; while the
    code is set a second barrier does not wait; reading the code clears it."""
    assert _device_error() == 0
    sig = torch.zeros((2,), dtype=torch.int32, device=cuda_device)
    stand_in = torch.zeros((2,), dtype=torch.int32, device=cuda_device)
    epoch = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    payload = torch.tensor([3, 4], dtype=torch.int32, device=cuda_device)
    matrix = torch.zeros((4,), dtype=torch.int32, device=cuda_device)
    matrix_stand_in = torch.zeros((4,), dtype=torch.int32, device=cuda_device)
    peers_sig, peers_mat = _table(sig, stand_in), _table(matrix, matrix_stand_in)
    lib = _lib()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    native._check(lib.moe_ep_barrier_p2p(native._ptr(peers_sig), 2, 0, native._ptr(epoch), native._ptr(payload), 2,
                                         native._ptr(peers_mat), 50_000, native._stream()), "moe_ep_barrier_p2p")
    end.record()
    torch.cuda.synchronize()
    assert start.elapsed_time(end) >= 45.0
    # the payload and the signal reached both "ranks" (row 0 of each counts buffer, slot 0 of each signal buffer)
    assert matrix[:2].tolist() == [3, 4] and matrix_stand_in[:2].tolist() == [3, 4]
    assert sig.tolist() == [1, 0] and stand_in.tolist() == [1, 0] and epoch.item() == 1
    # a second barrier while the code is set: no wait
    start.record()
    native._check(lib.moe_ep_barrier_p2p(native._ptr(peers_sig), 2, 0, native._ptr(epoch), None, 0, None, 50_000,
                                         native._stream()), "moe_ep_barrier_p2p")
    end.record()
    torch.cuda.synchronize()
    assert start.elapsed_time(end) < 40.0 and epoch.item() == 2
    assert _device_error() == EP_WAIT_ERROR
    assert _device_error() == 0

"""Host-side behaviour of the expert-parallel experts entry points
(include/moe_b200.h): argument checks and the workspace each kernel choice
needs.  Pure host arithmetic and early returns -- no device work."""

from pocketlm_b200 import native

H, I = 7168, 2048


def test_workspace_follows_the_kernel_choice():
    lib = native.load_library()
    S = 256 // 8 + 1                       # one of 8 ranks: 32 routed experts + the shared one
    T = 8192
    R = 8 * T * 8 + T                      # receive buffer sized for every rank's worst case
    lean = lib.moe_ep_experts_return_p2p_workspace_bytes(R, T * 9, H, I, S, 1)     # grouped GEMM
    gemv = lib.moe_ep_experts_return_p2p_workspace_bytes(R, 16 * 9, H, I, S, 1)    # ~4 rows per expert
    rowmajor = lib.moe_ep_experts_return_p2p_workspace_bytes(R, T * 9, H, I, S, 0)  # untiled: no GEMM
    assert 0 < lean < gemv
    assert rowmajor == gemv
    # 64 tokens per rank at 8 ranks: 576 rows, ~16 per local expert -- the GEMM's threshold
    assert lib.moe_ep_experts_return_p2p_workspace_bytes(R, 64 * 9, H, I, S, 1) == lean
    # the GEMM path keeps no warp-MMA buffers and no pair-order outputs: well under half
    assert lean < gemv // 2
    # valid_rows 0 means every row, and more than rows is clamped
    assert lib.moe_ep_experts_return_p2p_workspace_bytes(R, 0, H, I, S, 1) == lean
    assert lib.moe_ep_experts_return_p2p_workspace_bytes(R, 10 * R, H, I, S, 1) == lean


def test_workspace_rejects_bad_sizes():
    lib = native.load_library()
    for args in ((0, 0, H, I, 9), (100, 0, 0, I, 9), (100, 0, H, 0, 9), (100, 0, H, I, 0)):
        assert lib.moe_ep_experts_return_p2p_workspace_bytes(*args, 1) == -1
    assert lib.moe_ep_experts_workspace_bytes(0, H, I, 9) == -1


def test_entry_points_check_pointers_before_any_device_work():
    lib = native.load_library()
    code = lib.moe_ep_experts_return_p2p(None, None, None, 16, 0, H, I, None, 9, None, 1, 16, 2, 16, None, None, 0,
                                         None)
    assert code == -1 and b"null" in lib.moe_b200_last_error()
    code = lib.moe_ep_return_p2p(None, 16, None, None, H, 16, 2, 16, None, None)
    assert code == -1 and b"null" in lib.moe_b200_last_error()


def test_peer_entry_points_check_world_and_return_rows():
    """The return buffer's rows must lie within src_stride and the world in
    range; both are checked on the host before anything is launched."""
    import ctypes

    lib = native.load_library()
    fake = ctypes.c_void_p(16)  # never dereferenced: the calls return before any launch
    for world, home_rows in ((0, 16), (2, 0), (2, 17), (4096, 16)):
        code = lib.moe_ep_return_p2p(fake, 16, fake, fake, H, 16, world, home_rows, fake, None)
        assert code == -2, (world, home_rows)
        code = lib.moe_ep_experts_return_p2p(fake, fake, fake, 16, 0, H, I, fake, 9, fake, 1, 16, world, home_rows,
                                             fake, None, 0, None)
        assert code == -2, (world, home_rows)
    code = lib.moe_ep_experts_fp8(None, None, 16, H, I, None, 9, None, 1, None, None, 0, None)
    assert code == -1 and b"null" in lib.moe_b200_last_error()


def test_barrier_checks_its_arguments_before_launching():
    """moe_ep_barrier_p2p: tables, world, rank, limit and the payload pair are
    checked on the host; nothing is launched when they are wrong."""
    import ctypes

    lib = native.load_library()
    fake = ctypes.c_void_p(16)  # never dereferenced: the calls return before any launch
    assert lib.moe_ep_barrier_p2p(None, 2, 0, fake, None, 0, None, 1000, None) == -1
    assert lib.moe_ep_barrier_p2p(fake, 2, 0, None, None, 0, None, 1000, None) == -1
    for world, rank, limit in ((0, 0, 1000), (2, 2, 1000), (2, -1, 1000), (2048, 0, 1000), (2, 0, 0)):
        assert lib.moe_ep_barrier_p2p(fake, world, rank, fake, None, 0, None, limit, None) == -2, (world, rank)
    # a payload needs its peer buffers and a length, and the other way round
    assert lib.moe_ep_barrier_p2p(fake, 2, 0, fake, fake, 2, None, 1000, None) == -2
    assert lib.moe_ep_barrier_p2p(fake, 2, 0, fake, None, 0, fake, 1000, None) == -2
    assert lib.moe_ep_barrier_p2p(fake, 2, 0, fake, fake, 0, fake, 1000, None) == -2


def test_fused_send_checks_its_arguments_before_launching():
    """moe_ep_route_dispatch_p2p: pointers, dimensions (experts split evenly,
    room for every source entry) and its one-CTA limits (128 tokens, 1024
    entries, 256 experts, 32 ranks, aligned rows) are checked on the host."""
    import ctypes

    lib = native.load_library()
    fake = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(258)

    def call(x=fake, rw=fake, T=4, E=256, ng=8, tg=4, k=8, world=8, rank=0, cap=8 * 64, stride=None, sig=fake):
        stride = T * (k + 1) if stride is None else stride
        return lib.moe_ep_route_dispatch_p2p(x, rw, 1, fake, T, H, E, ng, tg, k, 2.5, world, rank, cap, stride,
                                             fake, fake, fake, fake, sig, fake, 1000, fake, fake, fake, 1 << 20, None)

    assert call(rw=None) == -1 and call(sig=None) == -1 and call(x=None) == -1
    assert call(E=250) == -2                 # 250 experts do not split over 8 ranks
    assert call(stride=4 * 8) == -2          # no room for the ranks' own shared-expert rows
    assert call(rank=8) == -2 and call(world=0) == -2
    assert call(T=129, cap=129 * 64, stride=129 * 9) == -5   # more tokens than one CTA selects
    assert call(E=512, ng=8, world=8) == -5  # selection scratch holds 256 experts
    assert call(world=64, E=256, cap=64 * 64) == -5
    assert call(x=odd) == -5                 # rows must be 16-byte aligned
    assert lib.moe_ep_route_dispatch_p2p_workspace_bytes(4, 256) >= 4 * 256 * 4


def test_combine_checks_row_dtype_and_pointers():
    """moe_ep_combine takes the output rows as bf16 (y_dtype 1, the exchanges' rows) or fp32 (0); anything
    else, or a missing pointer, is refused before any launch."""
    import ctypes

    lib = native.load_library()
    fake = ctypes.c_void_p(256)
    assert lib.moe_ep_combine(None, 1, fake, fake, 2, 8, H, 1, fake, None) == -1
    assert lib.moe_ep_combine(fake, 2, fake, fake, 2, 8, H, 1, fake, None) == -5   # f16 rows: not a layout it reads
    assert lib.moe_ep_combine(fake, 1, fake, fake, 0, 8, H, 1, fake, None) == -2

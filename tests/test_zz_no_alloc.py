"""The allocation-free expert MLP entry point (moe_fp8_e4m3_block_mlp_f32_noalloc).

It exists for callers that cannot allocate device memory themselves or let
the library do it -- a serving process whose GPU memory is all reserved by its
own arena, a hot path that must avoid the CUDA allocator, a binding that only
owns the pointers it passes -- and keeps its scratch in a static device array
shared by all calls.  This test calls it through the C ABI twice in a row (so
the second call runs on the scratch the first one left behind) and checks each
result against the allocating entry point, moe_fp8_e4m3_block_mlp_f32, with the
tolerance the other FP8 bridge tests use.  The file name sorts last so that a
run stopping at the first failure has run every other test before this one.
"""

import ctypes

import pytest
import torch

from pocketlm_b200 import native

pytestmark = pytest.mark.gpu


def _fp8(values):
    return values.to(torch.float8_e4m3fn).view(torch.uint8).contiguous()


def _expert(seed, hidden, inter):
    gen = torch.Generator().manual_seed(seed)
    gate = _fp8(torch.randn((inter, hidden), generator=gen) * 0.25)
    up = _fp8(torch.randn((inter, hidden), generator=gen) * 0.25)
    down = _fp8(torch.randn((hidden, inter), generator=gen) * 0.25)
    gs = ((inter + 127) // 128, (hidden + 127) // 128)
    ds = ((hidden + 127) // 128, (inter + 127) // 128)
    tensors = (gate, torch.rand(gs, generator=gen) + 0.5, up, torch.rand(gs, generator=gen) + 0.5, down,
               torch.rand(ds, generator=gen) + 0.5)
    return [t.cuda() for t in tensors]


def _noalloc(lib, item, x):
    batch, hidden = int(x.shape[0]), int(x.shape[1])
    inter = int(item[0].shape[0])
    out = torch.full((batch, hidden), float("nan"), device="cuda")
    code = lib.moe_fp8_e4m3_block_mlp_f32_noalloc(
        *[ctypes.c_void_p(t.data_ptr()) for t in item], ctypes.c_void_p(x.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), batch, inter, hidden, (hidden + 127) // 128, (inter + 127) // 128,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == 0, lib.moe_b200_last_error()
    return out


def _close(actual, expected, rel=1e-5):
    scale = float(expected.abs().max())
    err = float((actual - expected).abs().max())
    assert err <= rel * scale + 1e-6, f"max abs err {err} vs scale {scale}"


# growing and shrinking batches (a smaller call after a larger one runs on the chunk list and activations
# the larger one left in the shared scratch), and 1000 columns, which are not a multiple of 16 (scalar loads)
@pytest.mark.parametrize("hidden,inter,batches", [(1024, 512, (3, 5)), (7168, 2048, (1, 2)),
                                                  (1024, 512, (5, 3, 1)), (1000, 384, (4, 2))])
def test_noalloc_mlp_matches_allocating_entry_point_twice(cuda_device, hidden, inter, batches):
    lib = native.load_library()
    for call, batch in enumerate(batches):
        item = _expert(100 + call, hidden, inter)
        x = torch.randn((batch, hidden), generator=torch.Generator().manual_seed(200 + call)).cuda()
        got = _noalloc(lib, item, x)
        want = native.fp8_e4m3_block_mlp_f32(*item, x)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        _close(got, want)


def test_noalloc_call_takes_no_device_memory(cuda_device):
    """After a first call (which loads the kernels), further calls change
    neither the device's free memory nor torch's allocator."""
    lib = native.load_library()
    item = _expert(300, 1024, 512)
    x = torch.randn((4, 1024), generator=torch.Generator().manual_seed(301)).cuda()
    out = torch.empty((4, 1024), device="cuda")
    args = [ctypes.c_void_p(t.data_ptr()) for t in item] + [ctypes.c_void_p(x.data_ptr()),
                                                             ctypes.c_void_p(out.data_ptr())]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.moe_fp8_e4m3_block_mlp_f32_noalloc(*args, 4, 512, 1024, 8, 4, stream) == 0
    torch.cuda.synchronize()
    free0, torch0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for _ in range(3):
        assert lib.moe_fp8_e4m3_block_mlp_f32_noalloc(*args, 4, 512, 1024, 8, 4, stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0 and torch.cuda.memory_allocated() == torch0


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    lib = native.load_library()
    hidden, inter, batch = 256, 2048, 1024  # needs 8 MiB of activations > 4 MiB
    item = _expert(7, hidden, inter)
    x = torch.zeros((batch, hidden), device="cuda")
    out = torch.zeros((batch, hidden), device="cuda")
    code = lib.moe_fp8_e4m3_block_mlp_f32_noalloc(
        *[ctypes.c_void_p(t.data_ptr()) for t in item], ctypes.c_void_p(x.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), batch, inter, hidden, 2, 16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == -3
    assert b"static limit" in lib.moe_b200_last_error()
    # a batch whose activations alone overflow any size product is refused the same way
    code = lib.moe_fp8_e4m3_block_mlp_f32_noalloc(
        *[ctypes.c_void_p(t.data_ptr()) for t in item], ctypes.c_void_p(x.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), 1 << 62, inter, hidden, 2, 16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == -3

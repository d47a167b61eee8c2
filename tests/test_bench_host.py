"""Host arithmetic of bench.py's expert-parallel stack mode (config 5):
how a decode batch is spread over the ranks and which weight bytes lie on
the stack's critical path.  No GPU."""

import torch

import bench


def test_stack_share_spreads_a_batch_over_the_ranks():
    assert [bench.stack_share(1, r, 8) for r in range(8)] == [1, 0, 0, 0, 0, 0, 0, 0]
    assert [bench.stack_share(2, r, 8) for r in range(8)] == [1, 1, 0, 0, 0, 0, 0, 0]
    assert [bench.stack_share(32, r, 8) for r in range(8)] == [4] * 8
    assert sum(bench.stack_share(13, r, 4) for r in range(4)) == 13


def test_stack_critical_bytes_takes_the_busiest_rank_per_layer():
    per_rank, eb, rb = 4, 100, 7  # 2 ranks x 4 routed experts
    empty = torch.empty((0, 2), dtype=torch.int64)
    # layer 0: rank 0's token hits experts 1 and 5 (one on each rank); rank 1 has no tokens
    # layer 1: the token hits experts 4 and 6 (both on rank 1)
    ids = [[torch.tensor([[1, 5]]), torch.tensor([[4, 6]])], [empty, empty]]
    got = bench.stack_critical_bytes(ids, per_rank, eb, rb)
    # layer 0: rank 0 = 1 routed + shared + router = 207, rank 1 = 1 routed = 100
    # layer 1: rank 0 = 0 routed + shared + router = 107, rank 1 = 2 routed = 200
    assert got == 207 + 200

"""Expert-parallel exchange logic (pocketlm_b200/ep.py) with gloo ranks on CPU.

The compute steps are the oracle's (CPU); what runs for real is the
partitioning, the count / row / expert-id all-to-alls, the reverse exchange
of the expert outputs and the home combine.  Each rank checks that the
world-2 layer gives bit-for-bit the output of the same layer run on one rank
(a singleton group), and that both match the oracle's whole-layer flow."""

import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from oracle import kernels as orc
from pocketlm_b200 import synth
from pocketlm_b200.ep import ExpertParallelLayer, Packed
from tests.parity import COS_GATE, REL_L2_GATE, cos_dist, rel_l2


class OracleEPOps:
    """The EP compute steps on the CPU with the oracle's arithmetic."""

    def __init__(self, layer: ExpertParallelLayer):
        self.L = layer

    def route(self, x):
        cfg = self.L.cfg
        r = oracle.route_deepseek(x, self.L.router_weight, self.L.bias, top_k=cfg.top_k, n_groups=cfg.n_group,
                                  topk_groups=cfg.topk_group, route_scale=cfg.route_scale)
        return r.ids, r.weights.float()

    def pack(self, ids, w, x):
        L = self.L
        T, k = ids.shape
        flat = ids.reshape(-1)
        dst = flat // L.n_local
        order = torch.sort(dst, stable=True).indices          # entries grouped by rank, entry order kept
        entry_pos = torch.empty_like(order)
        entry_pos[order] = torch.arange(order.numel())
        offsets = torch.zeros(L.world + 1, dtype=torch.int32)
        offsets[1:] = torch.cumsum(torch.bincount(dst, minlength=L.world), 0).to(torch.int32)
        return Packed(send_rows=x[order // k].to(torch.bfloat16).contiguous(),
                      send_expert=(flat[order] - dst[order] * L.n_local).to(torch.int32),
                      send_offsets=offsets, entry_pos=entry_pos.to(torch.int32),
                      pos_weight=w.reshape(-1)[order].float().contiguous())

    def experts(self, rows, row_expert):
        out = torch.zeros((rows.shape[0], self.L.cfg.hidden), dtype=torch.float32)
        for i in range(rows.shape[0]):
            g, gs, u, us, d, ds = self.L.local_experts[int(row_expert[i])]
            out[i] = orc.fp8_mlp(g, gs, u, us, d, ds, rows[i:i + 1].float())[0]
        return out

    def combine(self, y, p, T):
        k = self.L.cfg.top_k
        out = torch.zeros((T, self.L.cfg.hidden), dtype=torch.float32)
        for t in range(T):
            for s in range(k):
                pos = int(p.entry_pos[t * k + s])
                out[t] += p.pos_weight[pos] * y[pos]
            out[t] += y[T * k + t]
        return out.to(torch.bfloat16)


def _rank_main(rank, world, port, tokens, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = synth.C1_TINY
        full = synth.make_fp8_layer(cfg, seed=9)
        x = synth.make_hidden(tokens[rank], cfg.hidden, seed=50 + rank)
        ep = ExpertParallelLayer(cfg, rank, world, layer=full, device="cpu", ops=OracleEPOps)
        out, ids, _w = ep.forward(x)
        solo_groups = [dist.new_group([r]) for r in range(world)]  # every rank creates every group, in order
        solo = ExpertParallelLayer(cfg, 0, 1, group=solo_groups[rank], layer=full, device="cpu", ops=OracleEPOps)
        ref, ref_ids, _ = solo.forward(x)
        if x.shape[0]:
            expected, _route = oracle.ds_moe_layer(x, full)
        else:  # a rank with no tokens this step still takes part in the exchange
            expected = torch.empty((0, cfg.hidden), dtype=torch.bfloat16)
        torch.save({"out": out, "ref": ref, "ids": ids, "ref_ids": ref_ids, "expected": expected},
                   os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("tokens", [(8, 8), (5, 11), (0, 7), (3, 0, 5, 2)])
def test_ep_world2_matches_one_rank_and_oracle(tokens):
    """World 2, and world 4 (each rank exchanging with three peers, one of
    them empty) against one rank and the oracle."""
    world = len(tokens)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), tokens, d), nprocs=world, join=True,
                           start_method="spawn")
        for rank in range(world):
            r = torch.load(os.path.join(d, f"rank{rank}.pt"))
            assert torch.equal(r["ids"], r["ref_ids"])
            assert r["out"].shape == (tokens[rank], synth.C1_TINY.hidden)
            assert torch.equal(r["out"].view(torch.int16), r["ref"].view(torch.int16))
            if tokens[rank] == 0:
                continue
            assert rel_l2(r["out"], r["expected"]) <= REL_L2_GATE
            assert cos_dist(r["out"], r["expected"]) <= COS_GATE


def _stack_main(rank, world, port, tokens, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from pocketlm_b200.ep import ExpertParallelStack

        cfg = synth.C1_TINY
        layers = [synth.make_fp8_layer(cfg, seed=30 + li) for li in range(3)]
        x = synth.make_hidden(tokens[rank], cfg.hidden, seed=80 + rank)
        stack = ExpertParallelStack(cfg, rank, world, 3, layers=layers, device="cpu", ops=OracleEPOps)
        out = stack.forward(x)
        solo_groups = [dist.new_group([r]) for r in range(world)]
        solo = ExpertParallelStack(cfg, 0, 1, 3, group=solo_groups[rank], layers=layers, device="cpu",
                                   ops=OracleEPOps)
        ref = solo.forward(x)
        h = x.clone()
        for layer in layers:  # the oracle's layer flow, layer after layer, residual in bf16
            if h.shape[0]:
                h = h + oracle.ds_moe_layer(h, layer)[0]
        torch.save({"out": out, "ref": ref, "expected": h}, os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens", [(4, 5), (3, 0)])
def test_ep_stack_world2_matches_one_rank_and_oracle(tokens):
    """Three layers with residuals (the routed-expert stack of a decode step),
    a rank with no tokens included."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_stack_main, args=(2, _free_port(), tokens, d), nprocs=2, join=True, start_method="spawn")
        for rank in range(2):
            r = torch.load(os.path.join(d, f"rank{rank}.pt"))
            assert r["out"].shape == (tokens[rank], synth.C1_TINY.hidden) and r["out"].dtype == torch.bfloat16
            assert torch.equal(r["out"].view(torch.int16), r["ref"].view(torch.int16))
            if tokens[rank]:
                assert rel_l2(r["out"], r["expected"]) <= REL_L2_GATE
                assert cos_dist(r["out"], r["expected"]) <= COS_GATE

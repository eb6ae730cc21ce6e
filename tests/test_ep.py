"""Expert parallelism, host side: ownership and the exchange of ExpertParallelMoe over a 2-rank gloo
group on CPU. The backend here is a small torch model with the engine's EP contract (routing of every
token on every rank, owned pairs' outputs at their bucket index, combine that takes each pair from
its owner's slice in rank order), so the test checks what the exchange must deliver: the single-rank
result, bit for bit."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hearth_b200.ep import ExpertParallelMoe, owned_experts

D, E, K, L = 32, 12, 3, 2


def test_owned_experts_partition():
    for world in (1, 2, 3, 4, 8):
        parts = [owned_experts(E, r, world) for r in range(world)]
        assert sorted(sum(parts, [])) == list(range(E))
        for r, p in enumerate(parts):
            assert all(e % world == r for e in p)


class TorchEpBackend:
    """A tiny MoE with the engine's expert-parallel contract, in torch on CPU."""

    def __init__(self, ep_size, ep_rank, max_tokens, seed=5):
        g = torch.Generator().manual_seed(seed)
        self.router = [torch.randn(E, D, generator=g) for _ in range(L)]
        self.w = [[torch.randn(D, D, generator=g) * 0.2 for _ in range(E)] for _ in range(L)]
        self.ep_size, self.ep_rank, self.K, self.D, self.n_layers = ep_size, ep_rank, K, D, L

        class Cfg:
            pass
        self.cfg = Cfg()
        self.cfg.max_tokens, self.cfg.device = max_tokens, 0
        self._route = None

    def _routing(self, layer, h):
        logits = h @ self.router[layer].T
        w, ids = torch.topk(torch.softmax(logits, -1), K, dim=-1)
        # buckets: experts ascending, tokens ascending; pair_of[t, j] = bucket position of (t, j)
        pairs = sorted(((int(ids[t, j]), t, j) for t in range(h.shape[0]) for j in range(K)))
        pair_of = torch.zeros_like(ids)
        for p, (e, t, j) in enumerate(pairs):
            pair_of[t, j] = p
        return ids, w, pair_of

    def ep_layer_dev(self, layer, h, T, y, stream=None):
        ids, w, pair_of = self._routing(layer, h[:T])
        self._route = (ids, w, pair_of)
        for t in range(T):
            for j in range(K):
                e = int(ids[t, j])
                if e % self.ep_size == self.ep_rank:
                    y[int(pair_of[t, j])] = torch.tanh(h[t] @ self.w[layer][e])

    def ep_combine_dev(self, layer, y_all, T, h, stream=None):
        ids, w, pair_of = self._route
        ya = y_all.view(self.ep_size, T * K, D)
        for t in range(T):
            o = torch.zeros(D)
            for j in range(K):
                o = o + w[t, j] * ya[int(ids[t, j]) % self.ep_size, int(pair_of[t, j])]
            h[t] = h[t] + o


def _rank_main(rank, world, port, T, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        be = TorchEpBackend(world, rank, max_tokens=T)
        ep = ExpertParallelMoe(be, device="cpu")
        h = torch.randn(T, D, generator=torch.Generator().manual_seed(9))
        ep.forward_dev(h, T)
        out[rank] = h.clone()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("T", [1, 5])
def test_exchange_over_gloo_equals_single_rank(T):
    mgr = mp.get_context("spawn").Manager()
    got = mgr.dict()
    mp.spawn(_rank_main, args=(2, _free_port(), T, got), nprocs=2, join=True)
    ref = mgr.dict()
    mp.spawn(_rank_main, args=(1, _free_port(), T, ref), nprocs=1, join=True)
    for r in range(2):
        assert torch.equal(got[r].view(torch.int32), ref[0].view(torch.int32)), f"rank {r}"

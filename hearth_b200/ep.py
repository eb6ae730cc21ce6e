"""Expert parallelism: one MoE stack over the GPUs of a torch.distributed process group.

Rank r (one process per GPU) holds the experts e with e % world == r of every layer; the router,
norms and any shared expert are replicated. Per layer every rank routes every token (the routing is
deterministic, so it is identical everywhere), computes the outputs of its own (token, rank) pairs,
the ranks all-gather those outputs (NCCL over NVLink on B200), and every rank forms the rank-order
sum taking each pair from its owner. The result equals the single-GPU result bit for bit, for any
number of ranks, and every rank ends the layer with the same h.

Single tokens on handles the persistent decode kernel takes: one launch per token on every rank for
every layer, the owners storing their (token, rank) outputs straight into every GPU's memory over
NVLink (CUDA IPC mappings exchanged once at start); no collective per layer. Batches: per layer, the
routing and the owned pairs, an NCCL all-gather, the combine.

The reference evaluates the whole layer in one process (engine/src/model.c:986-1131 moe_layer,
904-923 moe_sum_range); the exchange is this backend's addition.
"""
from __future__ import annotations

from .moe import MoeBackend


def owned_experts(n_experts: int, rank: int, world: int) -> list:
    """The experts rank `rank` holds: e % world == rank."""
    return [e for e in range(n_experts) if e % world == rank]


class ExpertParallelMoe:
    """One rank's share of an expert-parallel MoE stack.

    backend: an open MoeBackend with ep_size == world and ep_rank == rank (see `open`).
    group: the torch.distributed process group (NCCL for GPUs; any backend that implements
    all_gather_into_tensor on the buffers' device).
    """

    def __init__(self, backend, group=None, max_tokens: int | None = None, device=None):
        import torch
        import torch.distributed as dist
        self.be = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if backend.ep_size != self.world or backend.ep_rank != self.rank:
            raise ValueError(f"backend holds rank {backend.ep_rank} of {backend.ep_size}, "
                             f"the group is rank {self.rank} of {self.world}")
        T = max_tokens or backend.cfg.max_tokens
        dev = torch.device(device) if device is not None else torch.device("cuda", backend.cfg.device)
        self._y = torch.zeros((T * backend.K, backend.D), dtype=torch.float32, device=dev)
        self._y_all = torch.zeros((self.world * T * backend.K * backend.D,), dtype=torch.float32, device=dev)
        self.connected = False
        decode_path = getattr(backend, "decode_path", None)
        if dev.type == "cuda" and decode_path is not None and decode_path() == "persistent":
            self._connect(dev)

    def _connect(self, dev) -> None:
        """Every rank maps the other ranks' y-word buffers (CUDA IPC handles, all-gathered)."""
        import numpy as np
        import torch
        import torch.distributed as dist
        from ._lib import check, lib
        mine = np.zeros(64, np.uint8)
        check(lib().hxb_moe_ep_ipc_handle(self.be.h, mine.ctypes.data), "hxb_moe_ep_ipc_handle")
        t = torch.from_numpy(mine).to(dev)
        every = torch.empty(self.world * 64, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(every, t, group=self.group)
        allh = np.ascontiguousarray(every.cpu().numpy())
        check(lib().hxb_moe_ep_connect(self.be.h, allh.ctypes.data), "hxb_moe_ep_connect")
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)   # no rank launches before every rank has mapped the others
        self.connected = True

    @classmethod
    def open(cls, group=None, **cfg) -> "ExpertParallelMoe":
        """Opens this rank's MoeBackend (ep_size / ep_rank from the group) and wraps it."""
        import torch.distributed as dist
        be = MoeBackend(ep_size=dist.get_world_size(group), ep_rank=dist.get_rank(group), **cfg)
        return cls(be, group)

    def layer_dev(self, layer: int, h, T: int, stream=None) -> None:
        """One MoE layer in place on h [T, D] (a CUDA tensor, the same on every rank)."""
        import torch
        import torch.distributed as dist
        cuda = h.device.type == "cuda"
        s = stream if stream is not None or not cuda else torch.cuda.current_stream(h.device)
        n = T * self.be.K
        y = self._y[:n]                                                   # [T*K, D], this rank's pairs
        y_all = self._y_all[: self.world * n * self.be.D].view(self.world * n, self.be.D)   # [world][T*K][D]
        self.be.ep_layer_dev(layer, h, T, y, stream=s)
        if cuda:   # the collective on the stream of the layer's kernels
            with torch.cuda.stream(s):
                dist.all_gather_into_tensor(y_all, y, group=self.group)
        else:
            dist.all_gather_into_tensor(y_all, y, group=self.group)
        self.be.ep_combine_dev(layer, y_all, T, h, stream=s)

    def forward_dev(self, h, T: int, layer0: int = 0, n_layers: int | None = None, stream=None) -> None:
        """Layers [layer0, layer0 + n_layers) in place on h [T, D]."""
        n_layers = self.be.n_layers - layer0 if n_layers is None else n_layers
        if self.connected and T == 1:   # one persistent launch for every layer, exchange over NVLink
            self.be.forward_dev(h, 1, layer0, n_layers, stream=stream)
            return
        for l in range(layer0, layer0 + n_layers):
            self.layer_dev(l, h, T, stream=stream)

"""Expert parallelism through the C ABI on one GPU: G handles (ranks 0..G-1, disjoint experts)
emulate G GPUs, the gather is a stack of their outputs, and every rank's combine must give the
single-handle result bit for bit (which itself equals the oracle). The same path over NCCL runs when
two or more GPUs are visible."""
import numpy as np
import pytest

from moe_util import bits, build_pair

CASES = {
    "softmax": dict(),
    "sigmoid_group_bias": dict(score_fn=1, score_bias=1, n_group=4, topk_group=2, routed_scale=2.5),
    "shared_gated": dict(Fs=128, shared_gate=True, residual_scale=0.5),
}


@pytest.mark.gpu
@pytest.mark.parametrize("G", [2, 3])
@pytest.mark.parametrize("T", [1, 6])
@pytest.mark.parametrize("case", sorted(CASES))
def test_ep_emulated_equals_single_handle(gpu, case, T, G):
    import torch
    model, be, eps = build_pair(61, L=2, D=256, F=128, E=16, K=4, max_tokens=8, ep_size=G, **CASES[case])
    s = torch.cuda.current_stream()
    rng = np.random.default_rng(3)
    h0 = rng.standard_normal((T, 256)).astype(np.float32)
    ref = torch.from_numpy(h0.copy()).cuda()
    be.forward_dev(ref, T, stream=s)
    hs = [torch.from_numpy(h0.copy()).cuda() for _ in range(G)]   # every rank's copy of h
    for l in range(2):
        ys = []
        for r, b in enumerate(eps):
            y = torch.full((T * 4, 256), float("nan"), device="cuda")   # untouched rows stay NaN
            b.ep_layer_dev(l, hs[r], T, y, stream=s)
            ys.append(y)
        y_all = torch.stack(ys).contiguous()
        for r, b in enumerate(eps):
            b.ep_combine_dev(l, y_all, T, hs[r], stream=s)
    torch.cuda.synchronize()
    for b in eps:
        b.sync()
    want = model.forward(h0)
    assert np.array_equal(bits(ref.cpu().numpy()), bits(want))
    for r in range(G):
        assert np.array_equal(bits(hs[r].cpu().numpy()), bits(want)), f"rank {r}"
    for b in eps + [be]:
        b.close()


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["softmax", "sigmoid_group_bias"])
def test_ep_emulated_staged_tensor_core(gpu, case):
    """Expert parallelism on the staged tensor-core kernels (a batch of 40 tokens, D 512): each rank's
    store holds only its experts, its jobs are its own buckets; every rank ends with the
    single-handle h bit for bit."""
    import torch
    G, T, D = 2, 40, 512
    model, be, eps = build_pair(63, L=2, D=D, F=256, E=16, K=4, max_tokens=T, ep_size=G, **CASES[case])
    s = torch.cuda.current_stream()
    h0 = np.random.default_rng(4).standard_normal((T, D)).astype(np.float32)
    ref = torch.from_numpy(h0.copy()).cuda()
    be.forward_dev(ref, T, stream=s)
    hs = [torch.from_numpy(h0.copy()).cuda() for _ in range(G)]
    for l in range(2):
        ys = []
        for r, b in enumerate(eps):
            y = torch.full((T * 4, D), float("nan"), device="cuda")
            b.ep_layer_dev(l, hs[r], T, y, stream=s)
            ys.append(y)
        y_all = torch.stack(ys).contiguous()
        for r, b in enumerate(eps):
            b.ep_combine_dev(l, y_all, T, hs[r], stream=s)
    torch.cuda.synchronize()
    for b in eps:
        b.sync()
    want = model.forward(h0)
    assert np.array_equal(bits(ref.cpu().numpy()), bits(want))
    for r in range(G):
        assert np.array_equal(bits(hs[r].cpu().numpy()), bits(want)), f"rank {r}"
    for b in eps + [be]:
        b.close()


@pytest.mark.gpu
def test_ep_handle_rejects_whole_stack_calls(gpu):
    model, be, eps = build_pair(62, L=1, D=256, F=128, E=16, K=4, max_tokens=2, ep_size=2)
    h = np.zeros((1, 256), np.float32)
    with pytest.raises(Exception, match="expert-parallel"):
        eps[0].forward(h)
    assert eps[0].decode_path() == "layers"
    st = eps[1].stats()
    assert st["n_slots"] == 8   # one layer, the 8 experts of rank 1
    for b in eps + [be]:
        b.close()


def _nccl_rank(rank, world, port, T, out):
    import datetime
    import os

    import torch
    import torch.distributed as dist

    import hearth_b200 as hb
    from hearth_b200.ep import ExpertParallelMoe
    from moe_util import backend_kwargs, load_weights, make_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        kw = dict(L=3, D=256, F=128, E=16, K=4, max_tokens=8, Fs=128, shared_gate=True)
        be = hb.MoeBackend(ep_size=world, ep_rank=rank, device=rank, **backend_kwargs(**kw))
        load_weights(be, make_weights(71, **kw))
        ep = ExpertParallelMoe(be)
        h0 = np.random.default_rng(4).standard_normal((T, 256)).astype(np.float32)
        h = torch.from_numpy(h0).cuda()
        ep.forward_dev(h, T)
        torch.cuda.synchronize()
        be.sync()
        out[rank] = h.cpu().numpy()
        be.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 5])
def test_ep_over_nccl_equals_oracle(gpu, T):
    """Two ranks on two GPUs exchange their pairs' outputs with an NCCL all-gather (NVLink); both end
    with the oracle's h bit for bit."""
    import socket

    import torch
    import torch.multiprocessing as mp

    from moe_util import make_weights, oracle_model

    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs two GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    got = mp.get_context("spawn").Manager().dict()
    mp.spawn(_nccl_rank, args=(world, port, T, got), nprocs=world, join=True)
    kw = dict(L=3, D=256, F=128, E=16, K=4, Fs=128, shared_gate=True)
    want = oracle_model(make_weights(71, **kw), **kw).forward(
        np.random.default_rng(4).standard_normal((T, 256)).astype(np.float32))
    for r in range(world):
        assert np.array_equal(bits(got[r]), bits(want)), f"rank {r}"


def _persistent_rank(rank, world, port, steps, out):
    import datetime
    import os

    import torch
    import torch.distributed as dist

    import hearth_b200 as hb
    from hearth_b200.ep import ExpertParallelMoe
    from moe_util import backend_kwargs, load_weights, make_weights

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        kw = dict(L=3, D=512, F=256, E=32, K=4, max_tokens=1, residual_scale=0.7)
        be = hb.MoeBackend(ep_size=world, ep_rank=rank, device=rank, **backend_kwargs(**kw))
        load_weights(be, make_weights(81, **kw))
        ep = ExpertParallelMoe(be)
        assert be.decode_path() == "persistent" and ep.connected
        rng = np.random.default_rng(6)
        res = []
        for _ in range(steps):   # the same tokens on every rank; one launch per token and rank
            h = torch.from_numpy(rng.standard_normal((1, 512)).astype(np.float32)).cuda()
            ep.forward_dev(h, 1)
            be.sync()
            res.append(h.cpu().numpy())
        out[rank] = np.concatenate(res)
        torch.cuda.synchronize()
        dist.barrier()
        be.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_ep_persistent_decode_over_nvlink_equals_oracle(gpu):
    """Expert parallelism inside the persistent decode kernel on every GPU of the box (2 to 8): each
    rank computes the experts it owns and stores their y rows into every GPU's memory (peer stores
    over NVLink, tagged words); all ranks end every token with the oracle's h bit for bit."""
    import socket

    import torch
    import torch.multiprocessing as mp

    from moe_util import make_weights, oracle_model

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    steps = 6
    got = mp.get_context("spawn").Manager().dict()
    mp.spawn(_persistent_rank, args=(world, port, steps, got), nprocs=world, join=True)
    kw = dict(L=3, D=512, F=256, E=32, K=4, residual_scale=0.7)
    model = oracle_model(make_weights(81, **kw), **kw)
    rng = np.random.default_rng(6)
    want = np.concatenate([model.forward(rng.standard_normal((1, 512)).astype(np.float32)) for _ in range(steps)])
    for r in range(world):
        assert np.array_equal(bits(got[r]), bits(want)), f"rank {r}"

"""The multi-GPU partitions on the GPU, over NCCL: column-parallel linear (all_gather), head-sharded
inference attention (all_reduce(MAX) of eq, ek) and head-sharded training attention (plus the dO exponent
exchange of the backward). Each rank's results must equal the matching slice of the unsharded call on
the same GPU. With one GPU the partitions run as a world of one (the collectives are identities, the code
path is the same); with two or more GPUs, as two ranks on two GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _check_rank(rank, world):
    """Runs on every rank after init_process_group; returns a dict of failures (empty when all pass)."""
    import inputs
    from tbf16 import autograd, attention, ops, shard
    from helpers import ulp_distance
    dev = torch.device("cuda", torch.cuda.current_device())
    bad = {}
    # column-parallel linear: N split over ranks, y gathered
    x = inputs.gemm_x(1024, 2048, seed=31, device=dev)
    w16, ws = ops.prepare_weight(inputs.gemm_w(4096, 2048, seed=32, device=dev))
    full = ops.scaled_linear(x, w16, ws)
    y = shard.linear_column_parallel(x, *shard.shard_weight(w16, ws, None, rank, world))
    if int(ulp_distance(y, full).max()) > 1:
        bad["column_parallel"] = int(ulp_distance(y, full).max())
    # the two-phase sharded prepare (local exponents, all_reduce, global scale) equals the slice of the
    # unsharded prepare_qkv: GQA 8/4, a head dim (100) the kernels pad to 104, rank 1's q heads hotter
    q2, k2, v2 = inputs.attention_qkv(2, 8, 300, 100, seed=34, device=dev, Hkv=4)
    q2[:, 4:] *= 64
    g0, g1 = shard.shard_range(4, rank, world)
    got = shard.prepare_qkv_sharded(q2[:, 2 * g0:2 * g1], k2[:, g0:g1], v2[:, g0:g1], v_exp=13)
    want = attention.prepare_qkv(q2, k2, v2, v_exp=13)
    want = (want[0][:, 2 * g0:2 * g1, ..., :100], want[1][:, g0:g1, ..., :100], want[2][:, g0:g1, ..., :100],
            want[3], want[4][:, g0:g1])
    for name, g, w in zip(("q16", "k16", "v16", "a", "ev"), got, want):
        if g.shape != w.shape or not torch.equal(g, w):
            bad[f"prepare_qkv_sharded {name}"] = (tuple(g.shape), tuple(w.shape))
    # head-sharded attention (inference): rank 1's heads are hotter, so the exchange matters
    q, k, v = inputs.attention_qkv(1, 8, 512, 128, seed=33, device=dev)
    q[:, 4:] *= 64
    h0, h1 = shard.shard_range(8, rank, world)
    out = shard.sdpa_heads(q[:, h0:h1], k[:, h0:h1], v[:, h0:h1], is_causal=True)
    ref = attention.sdpa(q, k, v, is_causal=True)[:, h0:h1]
    if not torch.equal(out.view(torch.int16), ref.view(torch.int16)):
        bad["sdpa_heads"] = int(ulp_distance(out, ref).max())
    # head-sharded training attention: forward and gradients equal the unsharded call's slices
    do = (torch.randn(1, 8, 512, 128, device=dev) * 2.0 ** -20).bfloat16()
    do[:, 4:] *= 2.0 ** 9

    def grads(fn, ins, g):
        ins = [t.detach().clone().requires_grad_() for t in ins]
        o = fn(*ins)
        o.backward(g)
        return [o.detach()] + [t.grad for t in ins]

    got = grads(lambda a, b, c: shard.sdpa_heads_train(a, b, c, is_causal=True),
                [q[:, h0:h1], k[:, h0:h1], v[:, h0:h1]], do[:, h0:h1])
    want = grads(lambda a, b, c: autograd.sdpa(a, b, c, is_causal=True), [q, k, v], do)
    for name, g, w in zip(("o", "dq", "dk", "dv"), got, want):
        if not torch.equal(g.view(torch.int16), w[:, h0:h1].view(torch.int16)):
            bad[f"train_{name}"] = int(ulp_distance(g, w[:, h0:h1]).max())
    return bad


def _worker(rank, world, port, results):
    import pathlib
    import sys
    root = pathlib.Path(__file__).resolve().parents[1]
    for p in (root / "tests" / "golden", root / "tests", root, root / "turing-bf16_b200"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        results[rank] = _check_rank(rank, world)
    finally:
        dist.destroy_process_group()


def test_partitions_world_of_one():
    import datetime
    port = _free_port()
    store = dist.TCPStore("127.0.0.1", port, 1, True, timeout=datetime.timedelta(seconds=30))
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        bad = _check_rank(0, 1)
    finally:
        dist.destroy_process_group()
    assert not bad, bad


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_partitions_two_gpus():
    world = 2
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, start_method="spawn", join=True)
    assert len(results) == world
    for rank in range(world):
        assert not results[rank], (rank, results[rank])

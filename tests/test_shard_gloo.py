"""Host logic of the multi-GPU partitions, on CPU with 2 gloo ranks: the column-parallel all-gather
reassembles exactly the unsharded linear, the head-sharded exponent exchange gives every rank the
unsharded call's (a, ev, fp16 operands), and the backward's dO exponent exchange gives the unsharded
G. The compute ops are the CPU oracle's (the GPU kernels are covered by the -m gpu tests); only the
exchange and partition logic is under test here."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    import sys
    import pathlib
    root = pathlib.Path(__file__).resolve().parents[1]
    for p in (root / "tests" / "golden", root, root / "turing-bf16_b200"):
        sys.path.insert(0, str(p))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import inputs
        from oracle import oracle as orc
        from tbf16 import shard

        def cpu_linear(x, w16, ws, bias):
            return orc.linear_fused(x, w16, ws, bias)[0]

        # column-parallel linear
        x = inputs.gemm_x(48, 256, seed=3)
        w16, ws = orc.prepare_weight(inputs.gemm_w(128, 256, seed=4))
        bias = (torch.randn(128, generator=torch.Generator().manual_seed(5)) * 0.1).bfloat16()
        ws16, wss, bs = shard.shard_weight(w16, ws, bias, rank, world)
        y = shard.linear_column_parallel(x, ws16, wss, bs, linear=cpu_linear)
        full = cpu_linear(x, w16, ws, bias)
        col_ok = torch.equal(y.view(torch.int16), full.view(torch.int16))

        # row-sharded linear: this rank's rows equal the matching rows of the unsharded result
        a0, a1 = shard.shard_range(48, rank, world)
        rows_ok = torch.equal(shard.linear_rows(x[a0:a1], w16, ws, bias, linear=cpu_linear).view(torch.int16),
                              full[a0:a1].view(torch.int16))

        # head-sharded attention exponents: rank r holds heads [h0, h1); rank 1's heads are hotter
        q, k, v = inputs.attention_qkv(1, 4, 64, 64, seed=9, Hkv=4)
        q[:, 2:] *= 64
        k[:, 3:] *= 0.25
        h0, h1 = shard.shard_range(4, rank, world)
        q16, k16, v16, a, ev = shard.prepare_qkv_sharded(q[:, h0:h1], k[:, h0:h1], v[:, h0:h1], v_exp=13,
                                                         head_exp=orc.head_exp, head_scale=orc.head_scale)
        rq, rk, rv, ra, rev = orc.prepare_qkv(q, k, v, 13)
        att_ok = (int(a) == int(ra) and torch.equal(ev, rev[:, h0:h1])
                  and torch.equal(q16.view(torch.int16), rq[:, h0:h1].view(torch.int16))
                  and torch.equal(k16.view(torch.int16), rk[:, h0:h1].view(torch.int16))
                  and torch.equal(v16.view(torch.int16), rv[:, h0:h1].view(torch.int16)))
        # without the exchange, rank 0 alone would pick a different a
        local_a = orc.prepare_qkv(q[:, h0:h1], k[:, h0:h1], v[:, h0:h1], 13)[3]

        # training backward: the dO exponent G of the sharded call equals the unsharded call's
        # (reference autograd.py:173-178); rank 1's heads carry the larger dO, so rank 0 needs the exchange
        do = torch.randn(1, 4, 64, 64, generator=torch.Generator().manual_seed(12)).bfloat16()
        do[:, 2:] *= 2.0 ** 9
        _, _, _, _, ev_t = orc.prepare_qkv(q, k, v, 0)
        e_local, e_global = shard.global_dout_exponent(do[:, h0:h1], ev_t[:, h0:h1], head_exp=orc.head_exp)
        t_do = 12 - 6  # 12 - ceil(log2 64)
        G_full = orc.sdpa_bwd(q, k, v, do)["G"]
        offset = int(e_global) - int(e_local)
        # the kernel derives G from its own heads with the lowered target: (t_do - offset) - e_local
        g_ok = (t_do - int(e_global) == G_full) and ((t_do - offset) - int(e_local) == G_full)
        g_mattered = offset > 0 if rank == 0 else offset == 0
        results[rank] = (col_ok, rows_ok, att_ok, int(local_a) != int(ra) or rank == 1, g_ok, g_mattered)
    finally:
        dist.destroy_process_group()


def test_shard_exchange_gloo_world2():
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, start_method="spawn", join=True)
    assert len(results) == world
    for rank in range(world):
        col_ok, rows_ok, att_ok, exchange_mattered, g_ok, g_mattered = results[rank]
        assert col_ok, f"column-parallel gather differs on rank {rank}"
        assert rows_ok, f"row-sharded linear differs on rank {rank}"
        assert att_ok, f"head-sharded exponents differ on rank {rank}"
        assert exchange_mattered
        assert g_ok, f"head-sharded backward exponent G differs on rank {rank}"
        assert g_mattered


def test_shard_range_partitions():
    from tbf16.shard import shard_range
    for n, world, mult in ((100, 3, 1), (1024, 8, 8), (7, 4, 1), (64, 8, 8)):
        spans = [shard_range(n, r, world, mult) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
        assert all((b - a) % mult == 0 or b == n for a, b in spans)

"""Row sharding on CPU ranks (gloo, world size 2): the partition, the dBias all-reduce and the
output all-gather give exactly the unsharded results. The per-rank compute is the CPU oracle
here (the B200 kernels need a GPU); the product path passes the kernels and NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from colabfold_legacy_kernels import distributed as cd


def test_row_range_covers_rows_once():
    for total in (0, 1, 7, 512, 513, 2048):
        for world in (1, 2, 3, 4, 8):
            got = [cd.row_range(total, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == total
            for (a0, a1), (b0, b1) in zip(got, got[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        cd.row_range(10, 2, 2)


def _oracle_fwd(q, k, v, bias, kmask, *, scale, block_q, block_k):
    from oracle import attention as oa
    out, lse = oa.attention_forward(q.numpy(), k.numpy(), v.numpy(), bias.numpy(),
                                    kmask.numpy(), scale)
    return torch.tensor(out), torch.tensor(lse)


def _oracle_bwd(q, k, v, bias, kmask, out, dout, lse, *, scale):
    from oracle import attention as oa
    g = oa.attention_grads(q.numpy(), k.numpy(), v.numpy(), bias.numpy(), kmask.numpy(),
                           dout.numpy(), scale)
    return tuple(torch.tensor(x) for x in g[2:])


def _oracle_packed(p, bias, kmask, gate_bias, lims, *, scale, block_q, block_k, column):
    from oracle import attention as oa
    out = oa.packed_forward(p.numpy(), bias.numpy(), kmask.numpy(), gate_bias.numpy(), scale,
                            column, None if lims is None else lims.numpy())
    return torch.tensor(out)


def _inputs():
    rng = np.random.default_rng(0)
    n, h, s, d = 6, 2, 20, 8
    q, k, v, dout = (torch.tensor(rng.standard_normal((n, h, s, d))) for _ in range(4))
    bias = torch.tensor(rng.standard_normal((h, s, s)))
    km = torch.tensor((rng.random((n, s)) > 0.2).astype(np.uint8))
    km[3] = 0
    X, Y, H, D = 6, 11, 2, 8
    p = torch.tensor(rng.standard_normal((X, Y, 4, H, D)))
    pb = torch.tensor(rng.standard_normal((H, Y, Y)))
    pkm = torch.tensor((rng.random((X, Y)) > 0.3).astype(np.uint8))
    pkm[:, 7:] = 0
    pkm[-1] = 0
    gb = torch.tensor(rng.standard_normal((H, D)) * 0.1)
    return (q, k, v, bias, km, dout), (p, pb, pkm, gb)


def _rank_main(rank, world, port, results):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=__import__('datetime').timedelta(seconds=60))
    try:
        (q, k, v, bias, km, dout), (p, pb, pkm, gb) = _inputs()
        a, b = cd.row_range(q.shape[0], world, rank)
        res = cd.attention_fwd_bwd(q[a:b], k[a:b], v[a:b], bias, km[a:b], dout[a:b], scale=0.35,
                                   fwd=_oracle_fwd, bwd=_oracle_bwd)
        from oracle import attention as oa
        lims = torch.tensor(oa.trim_limits(pkm.numpy()))
        a2, b2 = cd.row_range(p.shape[0], world, rank)
        local_lims = torch.cat([lims[a2:b2], lims[-1:]])
        full = cd.packed_forward_gathered(p[a2:b2], pb, pkm[a2:b2], gb, local_lims, scale=0.35,
                                          fwd=_oracle_packed)
        results[rank] = ([t.numpy() for t in res], full.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_two_ranks_match_unsharded():
    world = 2
    manager = mp.get_context('spawn').Manager()
    results = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), results), nprocs=world,
                       join=True, start_method='spawn')
    from oracle import attention as oa
    (q, k, v, bias, km, dout), (p, pb, pkm, gb) = _inputs()
    want = oa.attention_grads(q.numpy(), k.numpy(), v.numpy(), bias.numpy(), km.numpy(),
                              dout.numpy(), 0.35)
    lims = oa.trim_limits(pkm.numpy())
    want_p = oa.packed_forward(p.numpy(), pb.numpy(), pkm.numpy(), gb.numpy(), 0.35, False, lims)
    for rank in range(world):
        (out, lse, dq, dk, dv, dbias), full = results[rank]
        a, b = cd.row_range(q.shape[0], world, rank)
        np.testing.assert_allclose(out, want[0][a:b], atol=1e-12)
        np.testing.assert_allclose(lse, want[1][a:b], atol=1e-12)
        for got, w in zip((dq, dk, dv), want[2:5]):
            np.testing.assert_allclose(got, w[a:b], atol=1e-12)
        np.testing.assert_allclose(dbias, want[5], atol=1e-12)   # the all-reduced sum
        np.testing.assert_allclose(full, want_p, atol=1e-12)     # the all-gathered output

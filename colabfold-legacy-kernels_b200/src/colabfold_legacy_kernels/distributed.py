"""Row sharding of the hot path across GPUs (one process per GPU, torch.distributed).

The batch axis of pair-biased attention (triangle-attention rows, MSA sequences) and the rows of
the pair-stack fusions are independent, so each rank computes a contiguous slice of them. The
only exchanges are the two the path has:

  * the dBias all-reduce after the backward: every rank's dBias [H, Sq, Sk] is the sum over its
    rows, and the bias is shared by all rows, so the ranks' partials are summed (NCCL over
    NVLink; gloo in the CPU tests);
  * the output all-gather after an inference forward, when a rank needs the whole output.

The fusions need no exchange (weights are replicated, rows independent).

The compute functions default to the B200 kernels (colabfold_legacy_kernels.b200); they are
parameters so that the partitioning and exchange logic can be exercised on CPU ranks.
"""
import torch
import torch.distributed as dist


def row_range(total, world, rank):
    """[start, stop) of rank's rows: an even split, the first total % world ranks one longer."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError('rank %d of world %d' % (rank, world))
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def attention_fwd_bwd(q, k, v, bias, kmask, dout, *, scale, group=None, fwd=None, bwd=None,
                      block_q=64, block_k=32):
    """Forward (with lse) and backward of this rank's rows, dBias summed over all ranks.

    q, k, v, dout [n_local, H, S, D] and kmask [n_local, S] are this rank's rows; bias [H, S, S]
    is replicated. Returns (out, lse, dq, dk, dv, dbias) with dbias the all-rank sum.
    """
    if fwd is None or bwd is None:
        from . import b200
        fwd = fwd or b200.volta_mma
        bwd = bwd or b200.volta_mma_bwd
    out, lse = fwd(q, k, v, bias, kmask, scale=scale, block_q=block_q, block_k=block_k)
    dq, dk, dv, dbias = bwd(q, k, v, bias, kmask, out, dout, lse, scale=scale)
    world, _ = _world(group)
    if world > 1:
        dist.all_reduce(dbias, op=dist.ReduceOp.SUM, group=group)
    return out, lse, dq, dk, dv, dbias


def packed_forward_gathered(p, bias, kmask, gate_bias, lims=None, *, scale, group=None,
                            fwd=None, gather=True, block_q=64, block_k=32):
    """Row-attention inference on this rank's rows of p [X_local, Y, G, H, D], then (gather)
    the all-gather of out into the whole [X, Y, H, D] on every rank.

    Every rank must hold the same number of rows (pad X to a multiple of the world size).
    kmask [X_local, Y] is this rank's rows; lims (if given) is this rank's entries of the
    global trim limits followed by the global last entry (every row's maximum), so that the
    sharded result equals the unsharded one.
    """
    if fwd is None:
        from . import b200
        fwd = b200.volta_mma_packed
    out = fwd(p, bias, kmask, gate_bias, lims, scale=scale, block_q=block_q, block_k=block_k,
              column=False)
    world, _ = _world(group)
    if world == 1 or not gather:
        return out
    full = torch.empty((world * out.shape[0],) + tuple(out.shape[1:]), dtype=out.dtype,
                       device=out.device)
    dist.all_gather_into_tensor(full, out.contiguous(), group=group)
    return full

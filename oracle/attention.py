"""CPU oracle for pair-biased attention -- TEST INFRASTRUCTURE, never the product path.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
import this module, and only as the checker (or as the timed CPU baseline). The library itself
never calls it.

What it restates (colabfold-legacy-kernels):
  * attention_grads: the reference's float64 closed form `reference_grads`
    (tests/test_attn_bwd.py:82-101): a masked key takes the logit -1e4 (NEG, :20;
    cuda/volta_attn.h:11), the softmax of a fully masked row is therefore uniform over its Sk
    keys, lse is in the log2 domain (m + log2 l, cuda/volta_mma_attn.cu:431-445), dS is zero on
    masked keys (:98; cuda/volta_mma_attn_bwd.cu:223-229) while P still carries dV, and dBias is
    dS summed over the batch, unscaled (cuda/volta_mma_attn_bwd.cu:230-235).
  * packed_forward: the gated, packed forward VoltaMmaPacked[Trim]
    (cuda/volta_mma_attn.cu:544-623; AttnLayout::packed and apply_gate, cuda/volta_attn.h:27-53):
    q/k/v/gate read in place from p [X, Y, G, H, D]; rows attend along Y, columns along X;
    out = attention * sigmoid(gate + gate_bias[h, c]) when G == 4. Trim (lims [N+1],
    tests/test_packed_attention.py:53-57): a row with lims[n] == 0 is zero; keys at or past
    lims[n] are masked keys anyway, so skipping them changes nothing.

Parity is pinned: tests/golden/make_golden.py runs the reference's own numpy functions
(`reference_grads`, `inputs`, packed `reference`, `trim_limits`, read from the reference test
files) and commits their outputs; tests/test_oracle.py checks this module against them.

The float32 entry points (attention_grads_f32) are the same math in float32 through numpy's
BLAS: the "port" CPU baseline that bench.py times.
"""
import numpy as np

NEG = -1.0e4          # masked-key logit, natural units (cuda/volta_attn.h:11)
LOG2E = 1.4426950408889634


def _masked_logits(q, k, bias, kmask, scale):
    """scale * q.k + bias where the key is live, NEG where it is masked; [N,H,Sq,Sk]."""
    m = np.asarray(kmask)[:, None, None, :] != 0
    logits = scale * np.einsum('nhqd,nhkd->nhqk', q, k) + bias[None]
    return np.where(m, logits, NEG), m


def attention_forward(q, k, v, bias, kmask, scale):
    """out [N,H,Sq,D] and the log2-domain lse [N,H,Sq], float64."""
    q, k, v, bias = (np.asarray(x, np.float64) for x in (q, k, v, bias))
    logits, _ = _masked_logits(q, k, bias, kmask, scale)
    mx = logits.max(-1, keepdims=True)
    e = np.exp(logits - mx)
    l = e.sum(-1, keepdims=True)
    p = e / l
    out = np.einsum('nhqk,nhkd->nhqd', p, v)
    lse2 = (np.log(l) + mx)[..., 0] * LOG2E
    return out, lse2


def attention_grads(q, k, v, bias, kmask, dout, scale):
    """(out, lse2, dq, dk, dv, dbias) in float64; dbias [H,Sq,Sk] summed over the batch.

    Follows tests/test_attn_bwd.py:82-101 step by step.
    """
    q, k, v = (np.asarray(x, np.float64) for x in (q, k, v))
    bias, dout = np.asarray(bias, np.float64), np.asarray(dout, np.float64)
    logits, m = _masked_logits(q, k, bias, kmask, scale)
    mx = logits.max(-1, keepdims=True)
    e = np.exp(logits - mx)
    l = e.sum(-1, keepdims=True)
    p = e / l
    out = np.einsum('nhqk,nhkd->nhqd', p, v)
    lse2 = (np.log(l) + mx)[..., 0] * LOG2E
    dv = np.einsum('nhqk,nhqd->nhkd', p, dout)
    dp = np.einsum('nhqd,nhkd->nhqk', dout, v)
    ds = p * (dp - (p * dp).sum(-1, keepdims=True))
    ds = np.where(m, ds, 0.0)
    dq = np.einsum('nhqk,nhkd->nhqd', ds, k) * scale
    dk = np.einsum('nhqk,nhqd->nhkd', ds, q) * scale
    return out, lse2, dq, dk, dv, ds.sum(0)


def attention_grads_f32(q, k, v, bias, kmask, dout, scale):
    """The same closed form in float32 with batched matmuls (BLAS, all host threads).

    This is the CPU baseline that bench.py times; it is not used for parity.
    """
    f = np.float32
    q, k, v, bias, dout = (np.asarray(x, f) for x in (q, k, v, bias, dout))
    live = (np.asarray(kmask) != 0)[:, None, None, :]
    logits = np.matmul(q, np.swapaxes(k, -1, -2)) * f(scale) + bias[None]
    logits = np.where(live, logits, f(NEG))
    mx = logits.max(-1, keepdims=True)
    p = np.exp(logits - mx)
    l = p.sum(-1, keepdims=True)
    p /= l
    out = np.matmul(p, v)
    lse2 = (np.log(l) + mx)[..., 0] * f(LOG2E)
    dv = np.matmul(np.swapaxes(p, -1, -2), dout)
    dp = np.matmul(dout, np.swapaxes(v, -1, -2))
    delta = (out * dout).sum(-1, keepdims=True)
    ds = p * (dp - delta)
    ds = np.where(live, ds, f(0))
    dq = np.matmul(ds, k) * f(scale)
    dk = np.matmul(np.swapaxes(ds, -1, -2), q) * f(scale)
    return out, lse2, dq, dk, dv, ds.sum(0)


def attention_forward_f32(q, k, v, bias, kmask, scale):
    """The forward alone (out, log2-domain lse) in float32 with batched matmuls: the CPU baseline
    of the inference workload."""
    f = np.float32
    q, k, v, bias = (np.asarray(x, f) for x in (q, k, v, bias))
    live = (np.asarray(kmask) != 0)[:, None, None, :]
    logits = np.matmul(q, np.swapaxes(k, -1, -2)) * f(scale) + bias[None]
    logits = np.where(live, logits, f(NEG))
    mx = logits.max(-1, keepdims=True)
    p = np.exp(logits - mx)
    l = p.sum(-1, keepdims=True)
    p /= l
    return np.matmul(p, v), (np.log(l) + mx)[..., 0] * f(LOG2E)


def gated_attention_grads(q, k, v, gate, gate_bias, bias, kmask, dy, scale):
    """The gated attention y = o * sigmoid(gate + gate_bias[h]) (o = the attention output,
    gate [N,H,Sq,D], gate_bias [H,D]) and its gradients, float64: (y, lse2, dq, dk, dv, dgate,
    dgate_bias [H,D], dbias [H,Sq,Sk]).

    The reference composes this from VoltaMma (o, lse), an XLA gate and VoltaMmaBwd
    (cuda/volta_mma_attn.cu:544-575 applies the same gate in its forward-only packed targets);
    this is the autodiff of that composition: dO = dy * s with s = sigmoid(gate + gate_bias),
    the attention gradients from attention_grads with dout = dO, dgate = dy * o * s * (1 - s),
    dgate_bias = dgate summed over the batch and the queries.
    """
    g = np.asarray(gate, np.float64) + np.asarray(gate_bias, np.float64)[None, :, None, :]
    s = 1.0 / (1.0 + np.exp(-g))
    dy = np.asarray(dy, np.float64)
    o, lse2, dq, dk, dv, dbias = attention_grads(q, k, v, bias, kmask, dy * s, scale)
    dgate = dy * o * s * (1.0 - s)
    return o * s, lse2, dq, dk, dv, dgate, dgate.sum(axis=(0, 2)), dbias


def trim_limits(kmask):
    """lims [N+1]: each batch row's last live key + 1, then their maximum
    (tests/test_packed_attention.py:53-57)."""
    kmask = np.asarray(kmask) != 0
    s = kmask.shape[1]
    last = np.where(kmask.any(axis=1), s - np.argmax(kmask[:, ::-1], axis=1), 0)
    return np.concatenate([last, [last.max() if last.size else 0]]).astype(np.int32)


def unpack(p, column):
    """q, k, v and (G == 4) gate as [N, H, S, D] float64 views of p [X, Y, G, H, D]."""
    p = np.asarray(p, np.float64)
    if column:
        p = np.transpose(p, (1, 0, 2, 3, 4))
    # now [N, S, G, H, D]
    parts = [np.transpose(p[:, :, i], (0, 2, 1, 3)) for i in range(p.shape[2])]
    return parts


def packed_forward(p, bias, kmask, gate_bias, scale, column, lims=None):
    """out [X, Y, H, D] float64, the kernel's semantics for VoltaMmaPacked / VoltaMmaPackedTrim.

    Masked keys take the logit NEG, so a row with no live key averages its keys uniformly; with
    lims, such a row (lims[n] == 0) is zero instead.
    """
    parts = unpack(p, column)
    q, k, v = parts[:3]
    out, _ = attention_forward(q, k, v, bias, kmask, scale)   # [N, H, S, D]
    if len(parts) == 4:
        g = parts[3] + np.asarray(gate_bias, np.float64)[None, :, None, :]
        out = out / (1.0 + np.exp(-g))
    if lims is not None:
        dead = np.asarray(lims)[:-1] == 0
        out[dead] = 0.0
    out = np.transpose(out, (0, 2, 1, 3))          # [N, S, H, D]
    if column:
        out = np.transpose(out, (1, 0, 2, 3))      # [X, Y, H, D]
    return out


def attention_flops(n, h, sq, sk, d, backward=True):
    """Algorithmic FLOPs: 4.N.H.Sq.Sk.D forward (QK^T and PV), 10.N.H.Sq.Sk.D backward."""
    f = 4 * n * h * sq * sk * d
    return f + (10 * n * h * sq * sk * d if backward else 0)

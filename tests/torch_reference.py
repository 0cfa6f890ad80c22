"""Float32 torch restatement of the attention closed form -- TEST INFRASTRUCTURE only.

The same math as oracle/attention.py's `attention_grads` (the reference's float64 closed form,
tests/test_attn_bwd.py:82-101 of colabfold-legacy-kernels): a masked key takes the logit -1e4,
lse in the log2 domain, dS zero on masked keys, dBias summed over the batch. It runs in float32
on whatever device its inputs are on (IEEE float32 matmuls, TF32 off), a chunk of batch rows at
a time, so that the GPU tests can check the kernels at the BASELINE configs' full sizes, where
the float64 numpy oracle would take minutes. tests/test_torch_reference.py pins it to the oracle
and the golden fixtures on the CPU; the GPU tests also check sampled batch rows against the
float64 oracle directly.
"""
import contextlib
import math

import torch

NEG = -1.0e4
LOG2E = 1.0 / math.log(2.0)


@contextlib.contextmanager
def ieee_fp32():
    """Matmuls in IEEE float32 (no TF32) for the duration."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def forward(q, k, v, bias, kmask, scale, chunk=16):
    """out [N,H,Sq,D] and log2-domain lse [N,H,Sq], float32."""
    outs, lses = [], []
    b = bias.float()
    with ieee_fp32():
        for n0 in range(0, q.shape[0], chunk):
            sl = slice(n0, n0 + chunk)
            qq, kk, vv = q[sl].float(), k[sl].float(), v[sl].float()
            live = (kmask[sl] != 0)[:, None, None, :]
            logits = torch.where(live, scale * qq @ kk.transpose(-1, -2) + b[None],
                                 torch.tensor(NEG, device=q.device))
            mx = logits.amax(-1, keepdim=True)
            e = torch.exp(logits - mx)
            l = e.sum(-1, keepdim=True)
            outs.append((e / l) @ vv)
            lses.append(((torch.log(l) + mx)[..., 0]) * LOG2E)
    return torch.cat(outs), torch.cat(lses)


def grads(q, k, v, bias, kmask, dout, scale, chunk=16):
    """(out, lse2, dq, dk, dv, dbias), float32; dbias [H,Sq,Sk] summed over the batch."""
    outs, lses, dqs, dks, dvs = [], [], [], [], []
    dbias = torch.zeros(bias.shape, dtype=torch.float32, device=bias.device)
    b = bias.float()
    with ieee_fp32():
        for n0 in range(0, q.shape[0], chunk):
            sl = slice(n0, n0 + chunk)
            qq, kk, vv, do = q[sl].float(), k[sl].float(), v[sl].float(), dout[sl].float()
            live = (kmask[sl] != 0)[:, None, None, :]
            logits = torch.where(live, scale * qq @ kk.transpose(-1, -2) + b[None],
                                 torch.tensor(NEG, device=q.device))
            mx = logits.amax(-1, keepdim=True)
            e = torch.exp(logits - mx)
            l = e.sum(-1, keepdim=True)
            p = e / l
            outs.append(p @ vv)
            lses.append(((torch.log(l) + mx)[..., 0]) * LOG2E)
            dvs.append(p.transpose(-1, -2) @ do)
            dp = do @ vv.transpose(-1, -2)
            ds = p * (dp - (p * dp).sum(-1, keepdim=True))
            ds = torch.where(live, ds, torch.zeros((), device=q.device))
            dqs.append((ds @ kk) * scale)
            dks.append((ds.transpose(-1, -2) @ qq) * scale)
            dbias += ds.sum(0)
    return (torch.cat(outs), torch.cat(lses), torch.cat(dqs), torch.cat(dks), torch.cat(dvs),
            dbias)


def gated_grads(q, k, v, gate, gate_bias, bias, kmask, dy, scale, chunk=16):
    """The gated attention y = o * sigmoid(gate + gate_bias[h]) and its gradients in float32:
    (y, lse2, dq, dk, dv, dgate, dgate_bias [H,D], dbias), the autodiff of the composition the
    reference's callers build from VoltaMma, an elementwise gate and VoltaMmaBwd."""
    s = torch.sigmoid(gate.float() + gate_bias.float()[None, :, None, :])
    dyf = dy.float()
    o, lse, dq, dk, dv, dbias = grads(q, k, v, bias, kmask, dyf * s, scale, chunk)
    dgate = dyf * o * s * (1.0 - s)
    return o * s, lse, dq, dk, dv, dgate, dgate.sum(dim=(0, 2)), dbias

"""The gated attention oracle (oracle/attention.py gated_attention_grads) against float64 torch
autograd of the composition it restates (attention, then the gate o * sigmoid(gate + gate_bias),
as the reference's callers compose VoltaMma, an XLA gate and VoltaMmaBwd), on the CPU; and the
float32 torch restatement (tests/torch_reference.py gated_grads) against the oracle."""
import numpy as np
import torch

import torch_reference as tr
from oracle import attention as oa
from oracle.numerics import rel_max


def _case(seed=0, n=3, h=2, sq=17, sk=19, d=8):
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal((n, h, s, d)) * 0.7 for s in (sq, sk, sk))
    gate, dy = (rng.standard_normal((n, h, sq, d)) for _ in range(2))
    gb = rng.standard_normal((h, d)) * 0.5 + 1.0
    bias = rng.standard_normal((h, sq, sk))
    km = (rng.random((n, sk)) > 0.25).astype(np.uint8)
    km[1] = 0
    return q, k, v, gate, gb, bias, km, dy


def test_gated_oracle_matches_autograd():
    q, k, v, gate, gb, bias, km, dy = _case()
    scale = 0.4
    got = oa.gated_attention_grads(q, k, v, gate, gb, bias, km, dy, scale)
    tq, tk, tv, tg, tgb, tb = (torch.tensor(x, dtype=torch.float64, requires_grad=True)
                               for x in (q, k, v, gate, gb, bias))
    live = torch.tensor(km)[:, None, None, :] != 0
    logits = torch.where(live, scale * tq @ tk.transpose(-1, -2) + tb[None],
                         torch.tensor(-1e4, dtype=torch.float64))
    y = (torch.softmax(logits, -1) @ tv) * torch.sigmoid(tg + tgb[None, :, None, :])
    (y * torch.tensor(dy)).sum().backward()
    want = [y.detach(), None, tq.grad, tk.grad, tv.grad, tg.grad, tgb.grad, tb.grad]
    for i, (g, w) in enumerate(zip(got, want)):
        if w is None:
            continue
        assert rel_max(g, w.numpy()) < 1e-10, i


def test_torch_gated_reference_matches_oracle():
    q, k, v, gate, gb, bias, km, dy = _case(1)
    want = oa.gated_attention_grads(q, k, v, gate, gb, bias, km, dy, 0.3)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.float32)
    got = tr.gated_grads(t(q), t(k), t(v), t(gate), t(gb), t(bias), torch.tensor(km), t(dy), 0.3,
                         chunk=2)
    for i, (g, w) in enumerate(zip(got, want)):
        if i == 1:
            assert np.abs(g.double().numpy() - w).max() < 1e-3
        else:
            assert rel_max(g.double().numpy(), w) < 1e-4, i

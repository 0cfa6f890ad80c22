"""The gated attention training path (cflk_volta_mma_gated + cflk_volta_mma_gated_bwd) against
the float64 oracle of the composition the reference's callers build (VoltaMma, an elementwise
gate o * sigmoid(gate + gate_bias[h]) and VoltaMmaBwd; oracle/attention.py
gated_attention_grads, pinned to autodiff by tests/test_gated_oracle.py), and at the BASELINE
configs' sizes (configs[2], gate bias 1.0; configs[1]) against the float32 torch restatement.
Tolerances as the plain attention tests: the reference's rel-max below 0.05, relative L2 below
1e-2, lse within 1e-3; dgate_bias (a float32 sum over the batch and queries) relative L2 1e-2.
"""
import numpy as np
import pytest
import torch

import bench
import torch_reference as tr
from oracle import attention as oa
from oracle.numerics import rel_l2, rel_max, round_to
from test_attention_fwd_gpu import assert_lse, b200, host, inputs, to_dev

pytestmark = pytest.mark.gpu

NAMES = ('y', 'lse', 'dq', 'dk', 'dv', 'dgate', 'dgate_bias', 'dbias')


def run_gated(q, k, v, gate, gb, bias, km, dy, dt, dev):
    m = b200()
    t = [to_dev(x, dt, dev) for x in (q, k, v, gate, gb, bias, dy)]
    kmask = torch.tensor(km, device=dev)
    scale = q.shape[-1] ** -0.5
    y, lse = m.volta_mma_gated(t[0], t[1], t[2], t[3], t[4], t[5], kmask, scale=scale)
    grads = m.volta_mma_gated_bwd(t[0], t[1], t[2], t[3], t[4], t[5], kmask, y, t[6], lse,
                                  scale=scale)
    assert m.device_status() == 0
    return (y, lse) + tuple(grads)


def check_all(got, want, tag, tol=0.05):
    for nm, g, w in zip(NAMES, got, want):
        g = host(g) if torch.is_tensor(g) else g
        w = host(w) if torch.is_tensor(w) else np.asarray(w, np.float64)
        if nm == 'lse':
            assert_lse(g, w)
            continue
        r, e = rel_max(g, w), rel_l2(g, w)
        assert r < tol and e < 1e-2, '%s %s: rel_max %.3e rel_l2 %.3e' % (tag, nm, r, e)


def gated_inputs(n, h, sq, sk, d, seed, dt, gate_mean=0.0):
    q, k, v, bias, km, dy = inputs(n, h, sq, sk, d, seed, dt)
    rng = np.random.default_rng(seed + 100)
    gate = round_to(rng.standard_normal((n, h, sq, d)), dt)
    gb = round_to(rng.standard_normal((h, d)) * 0.5 + gate_mean, dt)
    return q, k, v, gate, gb, bias, km, dy


SHAPES = [(3, 4, 96, 96, 32), (2, 4, 70, 83, 16), (2, 2, 130, 130, 64), (1, 8, 300, 260, 32),
          (2, 2, 7, 13, 8), (2, 2, 130, 130, 24), (1, 2, 130, 130, 96), (2, 2, 64, 64, 48)]


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('shape', SHAPES, ids=['x'.join(map(str, s)) for s in SHAPES])
def test_gated_against_oracle(shape, dt, cuda_device):
    n, h, sq, sk, d = shape
    args = gated_inputs(n, h, sq, sk, d, 0, dt, gate_mean=1.0)
    want = oa.gated_attention_grads(*args, d ** -0.5)
    got = run_gated(*args, dt, cuda_device)
    check_all(got, want, str(shape))


def test_gated_forward_matches_ungated_times_gate(cuda_device):
    """y is the plain forward's output times the gate, and lse is the plain forward's lse."""
    m = b200()
    q, k, v, gate, gb, bias, km, dy = gated_inputs(2, 4, 96, 96, 32, 3, 'bf16')
    t = [to_dev(x, 'bf16', cuda_device) for x in (q, k, v, gate, gb, bias)]
    kmask = torch.tensor(km, device=cuda_device)
    y, lse = m.volta_mma_gated(*t[:5], t[5], kmask, scale=32 ** -0.5)
    o, lse0 = m.volta_mma(t[0], t[1], t[2], t[5], kmask, scale=32 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(lse, lse0)
    want = o.float() * torch.sigmoid(t[3].float() + t[4].float()[None, :, None, :])
    assert rel_max(host(y), host(want)) < 0.02


def test_gated_fully_masked_row_and_determinism(cuda_device):
    args = list(gated_inputs(3, 2, 96, 96, 32, 5, 'bf16'))
    args[6][:] = 1
    args[6][2] = 0
    want = oa.gated_attention_grads(*args, 32 ** -0.5)
    a = run_gated(*args, 'bf16', cuda_device)
    b = run_gated(*args, 'bf16', cuda_device)
    check_all(a, want, 'masked row')
    assert torch.equal(a[3], b[3]) and torch.equal(a[4], b[4])   # dk, dv bitwise
    assert torch.equal(a[5], b[5])                                # dgate elementwise
    assert rel_max(host(a[6]), host(b[6])) < 1e-3


def test_gated_config3_full_size(cuda_device):
    """configs[2] with its gate (gate bias 1.0): the MSA inputs bench.py times plus a gate."""
    q, k, v, bias, kmask, dy = bench.make_inputs(torch, cuda_device, 0, 1)
    gate, gb = bench.make_gate(torch, cuda_device, q.shape)
    m = b200()
    scale = 32 ** -0.5
    y, lse = m.volta_mma_gated(q, k, v, gate, gb, bias, kmask, scale=scale)
    grads = m.volta_mma_gated_bwd(q, k, v, gate, gb, bias, kmask, y, dy, lse, scale=scale)
    torch.cuda.synchronize()
    assert m.device_status() == 0
    want = tr.gated_grads(q, k, v, gate, gb, bias, kmask, dy, scale)
    check_all((y, lse) + tuple(grads), want, 'config3 gated')

"""The float32 torch restatement (tests/torch_reference.py) against the float64 oracle and the
golden fixtures, on the CPU: the GPU tests use it as the full-size reference at the BASELINE
configs' shapes, so it is pinned here first."""
import numpy as np
import pytest
import torch

import torch_reference as tr
from conftest import golden
from oracle import attention as oa
from oracle.numerics import rel_l2, rel_max


def _t(a, dt=torch.float32):
    return torch.tensor(np.asarray(a), dtype=dt)


FIXTURES = golden('attn_*.npz')


@pytest.mark.parametrize('name,z', FIXTURES, ids=[n for n, _ in FIXTURES])
def test_torch_reference_matches_golden(name, z):
    d = z['q'].shape[-1]
    got = tr.grads(_t(z['q']), _t(z['k']), _t(z['v']), _t(z['bias']),
                   _t(z['kmask'], torch.uint8), _t(z['dout']), d ** -0.5, chunk=2)
    want = (z['out'], z['lse2'], z['dq'], z['dk'], z['dv'], z['dbias'])
    for nm, g, w in zip(('out', 'lse', 'dq', 'dk', 'dv', 'dbias'), got, want):
        g = g.double().numpy()
        if nm == 'lse':
            fin = np.isfinite(w)
            assert np.abs(g[fin] - w[fin]).max(initial=0) < 1e-3, nm
            continue
        assert rel_max(g, w) < 1e-4 and rel_l2(g, w) < 1e-5, (name, nm)


def test_torch_reference_matches_oracle_masked_and_chunked():
    rng = np.random.default_rng(3)
    n, h, sq, sk, d = 5, 3, 40, 37, 16
    q, k, v, dout = (rng.standard_normal((n, h, s, d)) for s in (sq, sk, sk, sq))
    bias = rng.standard_normal((h, sq, sk))
    km = (rng.random((n, sk)) > 0.3).astype(np.uint8)
    km[2] = 0
    want = oa.attention_grads(q, k, v, bias, km, dout, 0.3)
    got = tr.grads(_t(q), _t(k), _t(v), _t(bias), _t(km, torch.uint8), _t(dout), 0.3, chunk=2)
    for i, (g, w) in enumerate(zip(got, want)):
        assert rel_max(g.double().numpy(), w) < 1e-4, i
    fo, fl = tr.forward(_t(q), _t(k), _t(v), _t(bias), _t(km, torch.uint8), 0.3, chunk=3)
    assert rel_max(fo.double().numpy(), want[0]) < 1e-4
    assert np.abs(fl.double().numpy() - want[1]).max() < 1e-3

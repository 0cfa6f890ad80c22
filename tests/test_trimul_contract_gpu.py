"""The triangle multiplication's contraction (cflk_trimul_contract) on the B200 against the CPU
oracle, and the whole fused triangle multiplication chained as the reference's
tests/test_fused.py:125-139 chains it: ln_gdp -> einsum('cik,cjk->cij') -> trimul_epilogue.

Sizes: pairs of 59 and 260 residues (the reference's; rows not 16-byte multiples, so the
CUDA-core tile kernel), 128, 200 and 384 (the tcgen05 tile GEMM), a non-square case with partial
tiles, both edge directions, f16 and bf16; and the BASELINE configs[3] pair (768 x 768, 128
channels) with 8 sampled channels checked. Tolerance of the contraction: float32 sums against
float64 ones, relative L2 below 1e-5 and max |got - want| / max |want| below 1e-4; the chain:
the reference's rel-max 0.03 (tests/test_fused.py:139).
"""
import numpy as np
import pytest
import torch

from oracle import fused as of
from oracle.numerics import rel_l2, rel_max, round_to

pytestmark = pytest.mark.gpu

TD = {'f16': torch.float16, 'bf16': torch.bfloat16}


def b200():
    from colabfold_legacy_kernels import b200 as m
    return m


def run(a, b, incoming, dt, d):
    ta = torch.tensor(np.asarray(a, np.float32), dtype=TD[dt], device=d)
    tb = torch.tensor(np.asarray(b, np.float32), dtype=TD[dt], device=d)
    got = b200().trimul_contract(ta, tb, incoming=incoming)
    assert b200().device_status() == 0
    return got.double().cpu().numpy()


def close(name, got, want, rmax=1e-4, rl2=1e-5):
    r, e = rel_max(got, want), rel_l2(got, want)
    assert np.isfinite(got).all() and r < rmax and e < rl2, \
        '%s: rel_max %.3e rel_l2 %.3e' % (name, r, e)


def shapes(C, I, J, K, incoming):
    return ((C, K, I), (C, K, J)) if incoming else ((C, I, K), (C, J, K))


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('incoming', [False, True])
@pytest.mark.parametrize('C,I,J,K', [(4, 59, 59, 59), (2, 260, 260, 260), (3, 128, 128, 128),
                                     (2, 200, 200, 200), (2, 384, 384, 384), (3, 136, 72, 48),
                                     (1, 8, 264, 520), (5, 1, 1, 1)])
def test_trimul_contract(C, I, J, K, incoming, dt, cuda_device):
    rng = np.random.default_rng(C * 1000 + I + K)
    sa, sb = shapes(C, I, J, K, incoming)
    a = round_to(rng.standard_normal(sa), dt)
    b = round_to(rng.standard_normal(sb), dt)
    close('contract %s' % ((C, I, J, K, incoming),), run(a, b, incoming, dt, cuda_device),
          of.trimul_contract(a, b, incoming))


def test_trimul_contract_k0_and_empty(cuda_device):
    m = b200()
    d = cuda_device
    a = torch.zeros(3, 5, 0, dtype=torch.float16, device=d)
    b = torch.zeros(3, 7, 0, dtype=torch.float16, device=d)
    out = torch.full((3, 5, 7), 7.0, device=d)
    m.trimul_contract(a, b, out=out)
    assert (out == 0).all()
    assert m.trimul_contract(torch.zeros(0, 5, 4, dtype=torch.float16, device=d),
                             torch.zeros(0, 7, 4, dtype=torch.float16, device=d)).shape == (0, 5, 7)
    with pytest.raises(ValueError, match='share K'):
        m.trimul_contract(torch.zeros(1, 5, 4, dtype=torch.float16, device=d),
                          torch.zeros(1, 7, 8, dtype=torch.float16, device=d))


@pytest.mark.parametrize('incoming', [False, True])
def test_trimul_contract_config_size(incoming, cuda_device):
    """a 768 x 768 pair, 128 channels, bf16 left/right of unit scale; all
    channels run, 8 sampled channels are checked against float64 sums."""
    C, n = 128, 768
    rng = np.random.default_rng(7)
    d = cuda_device
    sa, sb = shapes(C, n, n, n, incoming)
    ta = torch.randn(sa, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(d)
    tb = torch.randn(sb, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).to(d)
    got = b200().trimul_contract(ta, tb, incoming=incoming)
    assert b200().device_status() == 0
    for c in sorted(rng.choice(C, 8, replace=False)):
        a = ta[c:c + 1].double().cpu().numpy()
        b = tb[c:c + 1].double().cpu().numpy()
        close('channel %d' % c, got[c:c + 1].double().cpu().numpy(),
              of.trimul_contract(a, b, incoming))


@pytest.mark.parametrize('a,ci', [(128, 128), (64, 64)])
@pytest.mark.parametrize('n', [59, 260, 128])
def test_fused_triangle_multiplication_chain(a, ci, n, cuda_device):
    """ln_gdp -> contraction -> trimul_epilogue (add_input) on the GPU against the same chain of
    oracles, the reference's whole-chain check (tests/test_fused.py:125-139)."""
    d, dt = cuda_device, 'f16'
    rng = np.random.default_rng(n + a)
    h = lambda *s, sc=1., mean=0.: round_to(rng.standard_normal(s) * sc + mean, dt)
    f32 = lambda *s, sc=1., mean=0.: (rng.standard_normal(s) * sc + mean).astype(np.float32)
    M = n * n
    x = h(M, a, sc=2.)
    mask = round_to((rng.uniform(size=M) > .1).astype(np.float64), dt)
    isc, iof = f32(a, sc=.1, mean=1.), f32(a, sc=.1)
    wpT, wgT = h(2 * ci, a, sc=.1), h(2 * ci, a, sc=.1)
    bp, bg = h(2 * ci, sc=.1), h(2 * ci, sc=.1)
    lsc, lof = f32(ci, sc=.1, mean=1.), f32(ci, sc=.1)
    woT, bo, wgoT, bgo = h(a, ci, sc=.1), h(a, sc=.1), h(a, a, sc=.1), h(a, sc=.1)

    left, right = of.ln_gdp(x, isc, iof, wpT, bp, wgT, bg, mask, 1e-5, dt, 128)
    x_cm = of.trimul_contract(left.reshape(ci, n, n), right.reshape(ci, n, n), False)
    want = of.trimul_epilogue(x_cm.reshape(ci, M).astype(np.float32), x, isc, iof, lsc, lof, woT,
                              bo, wgoT, bgo, None, 1e-5, True, dt, 128,
                              before=np.zeros((M, a)))

    m = b200()
    t16 = lambda v: torch.tensor(np.asarray(v, np.float32), dtype=torch.float16, device=d)
    t32 = lambda v: torch.tensor(np.asarray(v, np.float32), device=d)
    tx = t16(x)
    gl, gr = m.volta_ln_gdp(tx, t32(isc), t32(iof), t16(wpT), t16(bp), t16(wgT), t16(bg),
                            t16(mask), eps=1e-5)
    tri = m.trimul_contract(gl.view(ci, n, n), gr.view(ci, n, n))
    got = m.volta_trimul_epilogue(tri.view(ci, M), tx, t32(isc), t32(iof), t32(lsc), t32(lof),
                                  t16(woT), t16(bo), t16(wgoT), t16(bgo),
                                  torch.zeros(1, dtype=torch.float16, device=d), eps=1e-5,
                                  add_input=True, has_keep=False)
    assert m.device_status() == 0
    r = rel_max(got.double().cpu().numpy(), want)
    assert r < 0.03, 'chain a=%d ci=%d n=%d: rel_max %.3e' % (a, ci, n, r)

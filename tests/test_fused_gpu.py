"""The LayerNorm-folded fusions on the B200 against the CPU oracle (oracle/fused.py).

Shapes and input recipes follow the reference's tests/test_fused.py (rows 1, 59, 4101 and a
260 x 260 pair; widths (128, 128), (64, 64), (128, 64); x ~ 2 N(0,1), LN scale ~ 1 + 0.1 N,
weights ~ 0.1 N) and tests/test_keep.py (a padded pair and an MSA with keep: real rows identical
with and without keep, padding zero or untouched where the output aliases its input, tiles with
keep below zero not written). Tolerance: the reference's rel-max below 0.02 (its test tolerance,
tests/test_fused.py:51) and relative L2 below 1e-2. Row tiles here are 128 rows.
"""
import numpy as np
import pytest
import torch

from oracle import fused as of
from oracle.numerics import rel_l2, rel_max, round_to

pytestmark = pytest.mark.gpu

TILE = 128
TD = {'f16': torch.float16, 'bf16': torch.bfloat16}
ROWS = (1, 59, 4101, 260 * 260)
WIDTHS = ((128, 128), (64, 64), (128, 64))


def b200():
    from colabfold_legacy_kernels import b200 as m
    return m


class Gen:
    def __init__(self, seed, dt):
        self.rng = np.random.default_rng(seed)
        self.dt = dt

    def h(self, *shape, s=0.5, mean=0.0):
        """A 16-bit tensor's values (float64, already rounded)."""
        return round_to(self.rng.standard_normal(shape) * s + mean, self.dt)

    def f(self, *shape, s=0.5, mean=0.0):
        return (self.rng.standard_normal(shape) * s + mean).astype(np.float32).astype(np.float64)


def dev16(a, dt, d):
    return torch.tensor(np.asarray(a, np.float32), dtype=TD[dt], device=d)


def dev32(a, d):
    return torch.tensor(np.asarray(a, np.float32), device=d)


def host(t):
    return t.float().cpu().numpy().astype(np.float64)


def close(name, got, want, tol=0.02):
    r, e = rel_max(got, want), rel_l2(got, want)
    assert r < tol and e < 1e-2, '%s: rel_max %.3e rel_l2 %.3e' % (name, r, e)


# ---- layer_norm (VoltaLayerNorm) --------------------------------------------------------------

@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('C', [128, 64, 256, 8, 96, 100])
def test_layer_norm(C, M, dt, cuda_device):
    """Vector path (C / 8 a power of two up to 32) and the row path (96, 100), against the
    one-pass oracle; rows with a large common offset check the statistics' accumulation."""
    g = Gen(7, dt)
    x = g.h(M, C, s=2., mean=0.5)
    sc, off = g.f(C, s=.1, mean=1.), g.f(C, s=.1)
    want = of.layer_norm_one_pass(x, sc, off, 1e-5, dt)
    got = b200().volta_layer_norm(dev16(x, dt, cuda_device), dev32(sc, cuda_device),
                                  dev32(off, cuda_device), eps=1e-5)
    close('layer_norm', host(got), want)


def test_layer_norm_in_place_and_empty(cuda_device):
    g = Gen(8, 'bf16')
    x = g.h(1000, 128, s=3.)
    sc, off = g.f(128, s=.1, mean=1.), g.f(128, s=.1)
    want = of.layer_norm_one_pass(x, sc, off, 1e-5, 'bf16')
    t = dev16(x, 'bf16', cuda_device)
    out = b200().volta_layer_norm(t, dev32(sc, cuda_device), dev32(off, cuda_device), eps=1e-5,
                                  out=t)
    assert out.data_ptr() == t.data_ptr()
    close('layer_norm in place', host(t), want)
    e = torch.empty(0, 128, dtype=torch.bfloat16, device=cuda_device)
    assert b200().volta_layer_norm(e, dev32(sc, cuda_device), dev32(off, cuda_device),
                                   eps=1e-5).shape == (0, 128)
    with pytest.raises(ValueError, match=r'x must be \[M,C\]'):
        b200().volta_layer_norm(t.view(10, 100, 128), dev32(sc, cuda_device),
                                dev32(off, cuda_device), eps=1e-5)


# ---- gated_dual_proj (VoltaGdp) ---------------------------------------------------------------

@pytest.mark.parametrize('act', [0, 1])
@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('K,N', [(128, 128), (64, 64), (128, 64), (64, 128)])
def test_gdp(K, N, M, dt, act, cuda_device):
    """The unfused gated dual projection against its oracle, sigmoid and swish gates, a row
    mask with zeros, negatives and fractions (applied unclamped)."""
    g = Gen(11, dt)
    x = g.h(M, K, s=1.)
    wp, wg = g.h(K, N, s=.1), g.h(K, N, s=.1)
    bp, bg = g.h(N, s=.1), g.h(N, s=.1)
    mask = round_to(np.resize(np.array([1.0, 0.0, -1.0, 0.5, 2.0]), M), dt)
    want = of.gdp(x, wp, bp, wg, bg, mask, act, dt)
    d = cuda_device
    got = b200().volta_gdp(dev16(x, dt, d), dev16(wp, dt, d), dev16(bp, dt, d), dev16(wg, dt, d),
                           dev16(bg, dt, d), dev16(mask, dt, d), activation=act)
    assert b200().device_status() == 0
    close('gdp', host(got), want)


def test_gdp_refusals(cuda_device):
    d = cuda_device
    x = torch.zeros(10, 128, dtype=torch.bfloat16, device=d)
    w = torch.zeros(128, 128, dtype=torch.bfloat16, device=d)
    b = torch.zeros(128, dtype=torch.bfloat16, device=d)
    m = torch.ones(10, dtype=torch.bfloat16, device=d)
    with pytest.raises(ValueError, match='activation is 0'):
        b200().volta_gdp(x, w, b, w, b, m, activation=2)
    w3 = torch.zeros(128, 100, dtype=torch.bfloat16, device=d)
    b3 = torch.zeros(100, dtype=torch.bfloat16, device=d)
    with pytest.raises(ValueError, match='N must be a multiple of 8'):
        b200().volta_gdp(x, w3, b3, w3, b3, m)


@pytest.mark.parametrize('act', [0, 1])
@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', (1, 59, 4101))
@pytest.mark.parametrize('K,N', [(256, 256), (32, 8), (96, 200), (512, 136), (8, 64), (100, 96),
                                 (3, 16), (130, 256)])
def test_gdp_general_widths(K, N, M, dt, act, cuda_device):
    """VoltaGdp at widths outside 64/128 (any K, N a multiple of 8, as the reference takes): the
    tcgen05 tile GEMM for K % 8 == 0 (partial K slices, N tiles and row tiles clipped), the
    CUDA-core tile kernel for K % 8 != 0."""
    g = Gen(12, dt)
    x = g.h(M, K, s=1.)
    wp, wg = g.h(K, N, s=K ** -.5), g.h(K, N, s=K ** -.5)
    bp, bg = g.h(N, s=.1), g.h(N, s=.1)
    mask = round_to(np.resize(np.array([1.0, 0.0, -1.0, 0.5, 2.0]), M), dt)
    want = of.gdp(x, wp, bp, wg, bg, mask, act, dt)
    d = cuda_device
    got = b200().volta_gdp(dev16(x, dt, d), dev16(wp, dt, d), dev16(bp, dt, d), dev16(wg, dt, d),
                           dev16(bg, dt, d), dev16(mask, dt, d), activation=act)
    assert b200().device_status() == 0
    close('gdp %dx%d' % (K, N), host(got), want)


# ---- ln_gated_dual_proj ---------------------------------------------------------------------

def ln_gdp_case(K, CI, M, dt, d, mask=None, seed=0):
    g = Gen(seed, dt)
    x = g.h(M, K, s=2.)
    if mask is None:
        mask = round_to((g.rng.uniform(size=M) > .1).astype(np.float64), dt)
    sc, off = g.f(K, s=.1, mean=1.), g.f(K, s=.1)
    wpT, wgT = g.h(2 * CI, K, s=.1), g.h(2 * CI, K, s=.1)
    bp, bg = g.h(2 * CI, s=.1), g.h(2 * CI, s=.1)
    want = of.ln_gdp(x, sc, off, wpT, bp, wgT, bg, mask, 1e-5, dt, TILE)
    m = b200()
    left, right = m.volta_ln_gdp(dev16(x, dt, d), dev32(sc, d), dev32(off, d), dev16(wpT, dt, d),
                                 dev16(bp, dt, d), dev16(wgT, dt, d), dev16(bg, dt, d),
                                 dev16(mask, dt, d), eps=1e-5)
    assert m.device_status() == 0
    return (host(left), host(right)), want


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('K,CI', WIDTHS)
def test_ln_gdp(K, CI, M, dt, cuda_device):
    got, want = ln_gdp_case(K, CI, M, dt, cuda_device)
    close('left', got[0], want[0])
    close('right', got[1], want[1])


# ---- ln_projection / output_projection ----------------------------------------------------

def ln_proj_case(K, n, heads, M, dt, d, keep=None, seed=0):
    g = Gen(seed, dt)
    x = g.h(M, K, s=2.)
    sc, off = g.f(K, s=.1, mean=1.), g.f(K, s=.1)
    wT = g.h(n, K, s=.1) if n else None
    wbT = g.h(heads, K, s=.1) if heads else None
    want = of.ln_projection(x, sc, off, wT, wbT, keep, 1e-5, dt, TILE)
    m = b200()
    z = torch.zeros(1, dtype=TD[dt], device=d)
    p, bias = m.volta_ln_proj(dev16(x, dt, d), dev32(sc, d), dev32(off, d),
                              dev16(wT, dt, d) if n else z, dev16(wbT, dt, d) if heads else z,
                              dev16(keep, dt, d) if keep is not None else z, eps=1e-5, n=n,
                              heads=heads, has_keep=keep is not None)
    assert m.device_status() == 0
    return (host(p) if n else None, host(bias) if heads else None), want


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('K,nn', WIDTHS)
@pytest.mark.parametrize('slots,heads', [(4, 4), (3, 8)])
def test_ln_projection(K, nn, slots, heads, M, dt, cuda_device):
    got, want = ln_proj_case(K, slots * nn, heads, M, dt, cuda_device)
    close('p', got[0], want[0])
    close('bias', got[1], want[1])


@pytest.mark.parametrize('K', [64, 128])
def test_ln_projection_bias_only_and_wide(K, cuda_device):
    got, want = ln_proj_case(K, 0, 8, 4101, 'bf16', cuda_device)
    assert got[0] is None
    close('bias only', got[1], want[1])
    got, want = ln_proj_case(K, 1152, 2, 1000, 'bf16', cuda_device)   # three passes
    close('p wide', got[0], want[0])
    close('bias wide', got[1], want[1])


def out_proj_case(K, N, M, dt, d, residual=True, keep=None, seed=0, alias=False):
    g = Gen(seed, dt)
    o, wT, b = g.h(M, K), g.h(N, K, s=.1), g.h(N, s=.1)
    r = g.h(M, N, s=2.) if residual else None
    before = r if (alias and residual) else np.zeros((M, N))
    want = of.output_projection(o, wT, b, r, keep, dt, TILE, before=before)
    m = b200()
    z = torch.zeros(1, dtype=TD[dt], device=d)
    res = dev16(r, dt, d) if residual else z
    out = m.volta_out_proj(dev16(o, dt, d), dev16(wT, dt, d), dev16(b, dt, d), res,
                           dev16(keep, dt, d) if keep is not None else z,
                           has_residual=residual, has_keep=keep is not None,
                           out=res if (alias and residual) else None)
    assert m.device_status() == 0
    return host(out), want


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('K,N', [(128, 128), (64, 64), (128, 64), (64, 128)])
def test_output_projection(K, N, M, dt, cuda_device):
    got, want = out_proj_case(K, N, M, dt, cuda_device)
    close('with residual', got, want)
    got, want = out_proj_case(K, N, M, dt, cuda_device, residual=False)
    close('no residual', got, want)


def test_output_projection_in_place(cuda_device):
    """The output may alias the residual, as XLA aliases it."""
    got, want = out_proj_case(128, 128, 4101, 'bf16', cuda_device, alias=True)
    close('aliased', got, want)


# ---- keep ---------------------------------------------------------------------------------------

def pair_keep(S, n):
    tok = np.arange(S) < n
    return (tok[:, None] & tok[None, :]).reshape(-1).astype(np.float64)


KEEP_CASES = [('pair', 256, 200), ('pair', 256, 129), ('pair', 192, 65), ('msa', 508, 37)]


def keep_vector(kind, a, b):
    if kind == 'pair':
        return pair_keep(a, b)
    X, live = a, b
    return np.broadcast_to((np.arange(X) < live)[:, None], (X, 200)).reshape(-1).astype(float)


@pytest.mark.parametrize('case', KEEP_CASES, ids=['%s_%d_%d' % c for c in KEEP_CASES])
def test_keep_projections(case, cuda_device):
    """Real rows are bit-identical with and without keep; padding is zero (or the residual,
    where the output aliases it); everything matches the oracle's tile semantics."""
    keep = keep_vector(*case)
    M = keep.size
    got_k, want_k = ln_proj_case(128, 512, 4, M, 'bf16', cuda_device, keep=keep)
    got, _ = ln_proj_case(128, 512, 4, M, 'bf16', cuda_device)
    live = keep > 0
    assert np.array_equal(got_k[0][live], got[0][live])
    assert np.array_equal(got_k[1][:, live], got[1][:, live])
    assert np.array_equal(got_k[0], want_k[0]) or rel_max(got_k[0], want_k[0]) < 0.02
    pad = ~live
    assert np.all((got_k[0][pad] == got[0][pad]) | (got_k[0][pad] == 0))
    got_k, want_k = out_proj_case(128, 128, M, 'bf16', cuda_device, keep=keep, alias=True)
    close('out_proj keep aliased', got_k, want_k)


def test_keep_below_zero_not_written(cuda_device):
    """Tiles whose keep is all below zero keep the output buffer's previous contents."""
    m = b200()
    d = cuda_device
    S, n = 384, 129
    R = -(-n // TILE) * TILE
    tok, ins = np.arange(S) < n, np.arange(S) < R
    mask = (tok[:, None] & tok[None, :]).astype(np.float64)
    region = np.where(ins[:, None] & ins[None, :], mask, -1.0).reshape(-1)
    M = S * S
    g = Gen(3, 'bf16')
    o, wT, b = g.h(M, 128), g.h(128, 128, s=.1), g.h(128, s=.1)
    sentinel = torch.full((M, 128), 3.0, dtype=torch.bfloat16, device=d)
    out = m.volta_out_proj(dev16(o, 'bf16', d), dev16(wT, 'bf16', d), dev16(b, 'bf16', d),
                           torch.zeros(1, dtype=torch.bfloat16, device=d),
                           dev16(region, 'bf16', d), has_residual=False, has_keep=True,
                           out=sentinel)
    assert m.device_status() == 0
    want = of.output_projection(o, wT, b, None, region, 'bf16', TILE,
                                before=np.full((M, 128), 3.0))
    got = host(out)
    work = of.tile_work(region, M, TILE, -1.0)
    for t, w in enumerate(work):
        rows = slice(t * TILE, min(M, (t + 1) * TILE))
        if w == 'skip':
            assert np.all(got[rows] == 3.0)
        elif w == 'padding':
            assert np.all(got[rows] == 0.0)
    close('keep below zero', got, want)


def test_ln_gdp_mask_is_keep(cuda_device):
    """ln_gdp's mask is its keep (other 0): padded pairs exactly zero, tiles below zero left."""
    S, n = 256, 129
    mask = pair_keep(S, n)
    got, want = ln_gdp_case(128, 128, S * S, 'bf16', cuda_device, mask=mask)
    for gg, w in zip(got, want):
        close('ln_gdp keep', gg, w)
        assert np.abs(gg[:, mask == 0]).max(initial=0) == 0


def test_rejects_unsupported_widths(cuda_device):
    m = b200()
    d = cuda_device
    x = torch.zeros(8, 256, dtype=torch.bfloat16, device=d)
    f = torch.ones(256, device=d)
    w = torch.zeros(256, 256, dtype=torch.bfloat16, device=d)
    with pytest.raises(ValueError, match='64 or 128'):
        m.volta_ln_gdp(x, f, f, w, w[0], w, w[0], x[:, 0].contiguous(), eps=1e-5)
    with pytest.raises(ValueError, match='multiple of 64'):
        m.volta_ln_proj(x[:, :128].contiguous(), f[:128], f[:128], w[:32, :128].contiguous(),
                        w[:4, :128].contiguous(), f, eps=1e-5, n=32, heads=4, has_keep=False)


# ---- trimul_epilogue ------------------------------------------------------------------------

def trimul_case(CA, C, M, dt, d, add, amp=50., mean=0., keep=None, seed=0, alias=False):
    g = Gen(seed, dt)
    O = CA
    x = g.h(M, CA, s=2.)
    x_cm = g.f(C, M, s=amp, mean=mean)
    isc, iof = g.f(CA, s=.1, mean=1.), g.f(CA, s=.1)
    lsc, lof = g.f(C, s=.1, mean=1.), g.f(C, s=.1)
    woT, bo, wgT, bg = g.h(O, C, s=.1), g.h(O, s=.1), g.h(O, CA, s=.1), g.h(O, s=.1)
    before = x if alias else np.zeros((M, O))
    want = of.trimul_epilogue(x_cm, x, isc, iof, lsc, lof, woT, bo, wgT, bg, keep, 1e-5, add, dt,
                              TILE, before=before)
    m = b200()
    z = torch.zeros(1, dtype=TD[dt], device=d)
    tx = dev16(x, dt, d)
    out = m.volta_trimul_epilogue(
        dev32(x_cm, d), tx, dev32(isc, d), dev32(iof, d), dev32(lsc, d), dev32(lof, d),
        dev16(woT, dt, d), dev16(bo, dt, d), dev16(wgT, dt, d), dev16(bg, dt, d),
        dev16(keep, dt, d) if keep is not None else z, eps=1e-5, add_input=add,
        has_keep=keep is not None, out=tx if alias else None)
    assert m.device_status() == 0
    return host(out), want


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('CA,C', WIDTHS)
def test_trimul_epilogue(CA, C, M, dt, cuda_device):
    # the triangle product is float32 and wide; one case sits far from zero (two-pass stats)
    for amp, mean in ((50., 0.), (5., 1e3)):
        for add in (False, True):
            got, want = trimul_case(CA, C, M, dt, cuda_device, add, amp, mean)
            close('trimul amp %g mean %g add %s' % (amp, mean, add), got, want)


@pytest.mark.parametrize('case', KEEP_CASES[:3], ids=['%s_%d_%d' % c for c in KEEP_CASES[:3]])
def test_trimul_keep_aliased(case, cuda_device):
    keep = keep_vector(*case)
    M = keep.size
    got, want = trimul_case(128, 128, M, 'bf16', cuda_device, True, 20., 0., keep=keep,
                            alias=True)
    close('trimul keep aliased', got, want)
    got0, _ = trimul_case(128, 128, M, 'bf16', cuda_device, True, 20., 0., alias=True)
    live = keep > 0
    assert np.array_equal(got[live], got0[live])


# ---- transition ---------------------------------------------------------------------------

def trans_tile(C):
    return 256 if C <= 128 else 128


def transition_case(C, factor, M, dt, d, add, keep=None, seed=0, alias=False):
    g = Gen(seed, dt)
    H = factor * C
    x = g.h(M, C, s=2.)
    sc, off = g.f(C, s=.1, mean=1.), g.f(C, s=.1)
    w1T, b1 = g.h(H, C, s=C ** -.5), g.h(H, s=.1)
    w2 = g.h(H, C, s=H ** -.5)
    w2T = of.chunk_w2(w2)
    b2 = g.h(C, s=.1)
    before = x if alias else np.zeros((M, C))
    want = of.transition(x, sc, off, w1T, b1, w2T, b2, keep, 1e-5, add, dt, trans_tile(C),
                         before=before)
    m = b200()
    z = torch.zeros(1, dtype=TD[dt], device=d)
    tx = dev16(x, dt, d)
    out = m.volta_transition(tx, dev32(sc, d), dev32(off, d), dev16(w1T, dt, d),
                             dev16(b1, dt, d), dev16(w2T, dt, d), dev16(b2, dt, d),
                             dev16(keep, dt, d) if keep is not None else z, eps=1e-5,
                             add_input=add, has_keep=keep is not None,
                             out=tx if alias else None)
    assert m.device_status() == 0
    return host(out), want


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('M', ROWS)
@pytest.mark.parametrize('C,factor', [(128, 4), (64, 2), (64, 4), (256, 4), (128, 2),
                                      (256, 2)])
def test_transition(C, factor, M, dt, cuda_device):
    for add in (False, True):
        got, want = transition_case(C, factor, M, dt, cuda_device, add)
        close('transition add %s' % add, got, want)


@pytest.mark.parametrize('case', KEEP_CASES, ids=['%s_%d_%d' % c for c in KEEP_CASES])
@pytest.mark.parametrize('C', [128, 256])
def test_transition_keep(case, C, cuda_device):
    keep = keep_vector(*case)
    M = keep.size
    got, want = transition_case(C, 4, M, 'bf16', cuda_device, False, keep=keep)
    close('transition keep', got, want)
    got0, _ = transition_case(C, 4, M, 'bf16', cuda_device, False)
    live = keep > 0
    assert np.array_equal(got[live], got0[live])
    assert np.all((got[~live] == got0[~live]) | (got[~live] == 0))
    got, want = transition_case(C, 4, M, 'bf16', cuda_device, True, keep=keep, alias=True)
    close('transition keep aliased', got, want)

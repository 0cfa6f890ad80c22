"""VoltaOpmUpdate and VoltaOpmOuter on the B200 (the tcgen05 tile GEMMs) against the CPU oracle
(oracle/fused.py opm_update, opm_outer).

The grid and recipe follow the reference's tests/test_opm.py: B 1, 37 and 260, D 4, 64 and 260,
K 32, 64 and 512, F 128 and 64 (here also 16 and 32), lhs ~ N(0,1), t ~ N(0,1) K^-1/2, bias ~ 0.1
N(0,1), the norm a count of MSA rows in [1, K/32] (AF2's mask sum), the residual ~ 2 N(0,1), with
and without the residual; and the residual aliased to the output. Tolerance: the reference's
rel-max 2e-3 for f16 (tests/test_opm.py:46, max |got - want| / max |want|), 8e-3 for bf16 (its
rounding step is 8x coarser), and relative L2 below 1e-3.
"""
import numpy as np
import pytest
import torch

from oracle import fused as of
from oracle.numerics import rel_l2, rel_max, round_to

pytestmark = pytest.mark.gpu

TD = {'f16': torch.float16, 'bf16': torch.bfloat16}
TOL = {'f16': 2e-3, 'bf16': 8e-3}


def b200():
    from colabfold_legacy_kernels import b200 as m
    return m


def case(B, D, K, F, dt, seed, residual):
    rng = np.random.default_rng(seed)
    lhs = round_to(rng.standard_normal((B, K)), dt)
    t = round_to(rng.standard_normal((K, D, F)) * max(K, 1) ** -.5, dt)
    bias = rng.standard_normal(F).astype(np.float32) * np.float32(.1)
    norm = rng.integers(1, max(K // 32, 1) + 1, size=(B, D)).astype(np.float32)
    res = round_to(rng.standard_normal((B, D, F)) * 2., dt) if residual else None
    return lhs, t, bias, norm, res


def run(lhs, t, bias, norm, res, dt, d, eps=1e-3, out=None):
    h = lambda a: torch.tensor(np.asarray(a, np.float32), dtype=TD[dt], device=d)
    f = lambda a: torch.tensor(np.asarray(a, np.float32), device=d)
    got = b200().volta_opm_update(h(lhs), h(t), f(bias), f(norm),
                                  None if res is None else h(res), eps=eps, out=out)
    assert b200().device_status() == 0
    return got.float().cpu().numpy().astype(np.float64)


def close(name, got, want, dt):
    r, e = rel_max(got, want), rel_l2(got, want)
    assert np.isfinite(got).all() and r < TOL[dt] and e < 1e-3, \
        '%s: rel_max %.3e rel_l2 %.3e' % (name, r, e)


@pytest.mark.parametrize('residual', [False, True])
@pytest.mark.parametrize('F', [128, 64])
@pytest.mark.parametrize('K', [32, 64, 512])
@pytest.mark.parametrize('B,D', [(1, 4), (37, 64), (260, 260), (1, 260), (260, 4), (37, 4)])
def test_opm_update_f16(B, D, K, F, residual, cuda_device):
    lhs, t, bias, norm, res = case(B, D, K, F, 'f16', B * 7 + D + K + F, residual)
    want = of.opm_update(lhs, t, bias, norm, res, 1e-3, 'f16')
    close('opm_update B=%d D=%d K=%d F=%d' % (B, D, K, F),
          run(lhs, t, bias, norm, res, 'f16', cuda_device), want.reshape(B, D, F), 'f16')


@pytest.mark.parametrize('F', [16, 32, 64, 128])
@pytest.mark.parametrize('B,D,K', [(37, 64, 64), (300, 130, 512), (129, 33, 96)])
def test_opm_update_bf16_and_narrow_f(B, D, K, F, cuda_device):
    """bf16, and the F = 16 / 32 widths (a 32-column epilogue chunk spans two d for F = 16)."""
    lhs, t, bias, norm, res = case(B, D, K, F, 'bf16', 5 + F + K, True)
    want = of.opm_update(lhs, t, bias, norm, res, 1e-3, 'bf16')
    close('opm_update bf16 F=%d' % F, run(lhs, t, bias, norm, res, 'bf16', cuda_device),
          want.reshape(B, D, F), 'bf16')


def test_opm_update_residual_aliased_to_out(cuda_device):
    """The output may be the residual's own buffer (the reference aliases them inside its call)."""
    d = cuda_device
    lhs, t, bias, norm, res = case(37, 64, 64, 128, 'f16', 1, True)
    want = of.opm_update(lhs, t, bias, norm, res, 1e-3, 'f16')
    r = torch.tensor(np.asarray(res, np.float32), dtype=torch.float16, device=d)
    h = lambda a: torch.tensor(np.asarray(a, np.float32), dtype=torch.float16, device=d)
    f = lambda a: torch.tensor(np.asarray(a, np.float32), device=d)
    got = b200().volta_opm_update(h(lhs), h(t), f(bias), f(norm), r, eps=1e-3, out=r)
    assert got.data_ptr() == r.data_ptr()
    close('opm_update aliased', r.float().cpu().numpy().astype(np.float64), want, 'f16')


def test_opm_update_k0_and_empty(cuda_device):
    """K = 0: no product, bias / (eps + norm) (+ residual); B = 0 or D = 0: nothing launched."""
    lhs, t, bias, norm, res = case(5, 3, 0, 16, 'f16', 2, True)
    want = of.opm_update(lhs, t, bias, norm, res, 1e-3, 'f16')
    close('opm_update K=0', run(lhs, t, bias, norm, res, 'f16', cuda_device), want, 'f16')
    lhs, t, bias, norm, _ = case(0, 3, 32, 16, 'f16', 2, False)
    assert run(lhs, t, bias, norm, None, 'f16', cuda_device).shape == (0, 3, 16)


def test_opm_update_refusals(cuda_device):
    d = cuda_device
    z = lambda *s: torch.zeros(s, dtype=torch.float16, device=d)
    f = lambda *s: torch.ones(s, device=d)
    with pytest.raises(ValueError, match='K must be a multiple of 32'):
        b200().volta_opm_update(z(4, 48), z(48, 3, 16), f(16), f(4, 3), eps=1e-3)
    with pytest.raises(ValueError, match='K must be a multiple of 32'):
        b200().volta_opm_update(z(4, 32), z(32, 3, 48), f(48), f(4, 3), eps=1e-3)
    with pytest.raises(ValueError, match='shapes do not match'):
        b200().volta_opm_update(z(4, 32), z(32, 3, 16), f(16), f(4, 4), eps=1e-3)
    with pytest.raises(ValueError, match='must be float32'):
        b200().volta_opm_update(z(4, 32), z(32, 3, 16), z(16), f(4, 3), eps=1e-3)


# ---- opm_outer (VoltaOpmOuter) ----------------------------------------------------------------

def outer_case(B, D, C, F, dt, seed):
    rng = np.random.default_rng(seed)
    left = round_to(rng.standard_normal((16, B, C)), dt)
    right = round_to(rng.standard_normal((16, D, 32)), dt)
    wT = round_to(rng.standard_normal((F, C * 32)) * (C * 32) ** -.5, dt)
    return left, right, wT


def run_outer(left, right, wT, dt, d, workspace=None):
    h = lambda a: torch.tensor(np.asarray(a, np.float32), dtype=TD[dt], device=d)
    got = b200().volta_opm_outer(h(left), h(right), h(wT), workspace=workspace)
    assert b200().device_status() == 0
    return got.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize('F', [128, 64])
@pytest.mark.parametrize('B,D', [(1, 4), (37, 64), (260, 260), (1, 260), (260, 4)])
def test_opm_outer_f16(B, D, F, cuda_device):
    """The reference's grid (tests/test_opm.py:112-125): B and D of 1/37/260 and 4/64/260 on 16
    rows with AF2's 32 channels, against the outer product rounded to f16 then contracted in
    float32 (its outer_f32), rel-max 2e-3."""
    left, right, wT = outer_case(B, D, 32, F, 'f16', B + D + F)
    want = of.opm_outer(left, right, wT, 'f16')
    close('opm_outer B=%d D=%d F=%d' % (B, D, F), run_outer(left, right, wT, 'f16', cuda_device),
          want, 'f16')


@pytest.mark.parametrize('C', [16, 64, 128, 48])
@pytest.mark.parametrize('F', [16, 32, 128])
def test_opm_outer_channels_bf16(C, F, cuda_device):
    """Other channel counts (C = 48 does not divide 128: the CUDA-core first product) and F, bf16."""
    left, right, wT = outer_case(45, 36, C, F, 'bf16', C + F)
    want = of.opm_outer(left, right, wT, 'bf16')
    close('opm_outer C=%d F=%d' % (C, F), run_outer(left, right, wT, 'bf16', cuda_device), want,
          'bf16')


def test_opm_outer_chunked_workspace(cuda_device):
    """C = 64 (the two-GEMM path): a workspace of one chunk (128 / C rows of b) runs the batch in
    many chunks, the same result."""
    left, right, wT = outer_case(70, 68, 64, 128, 'f16', 3)
    want = of.opm_outer(left, right, wT, 'f16')
    ws = torch.empty(2 * 68 * 64 * 32 * 2, dtype=torch.uint8, device=cuda_device)
    close('opm_outer chunked', run_outer(left, right, wT, 'f16', cuda_device, ws), want, 'f16')
    with pytest.raises(ValueError, match='workspace below one chunk'):
        run_outer(left, right, wT, 'f16', cuda_device, ws[:2 * 68 * 64 * 32 * 2 - 16])


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('B,D,F', [(768, 768, 128), (300, 36, 16), (17, 100, 32), (64, 64, 64)])
def test_opm_outer_fused_sizes(B, D, F, dt, cuda_device):
    """The fused C = 32 kernel at AF2's pair size (768^2, F = c_z = 128, sampled rows checked) and
    at sizes with partial 16 x 16 tiles and narrow F."""
    left, right, wT = outer_case(B, D, 32, F, dt, B + D)
    if B * D > 100000:
        rows = np.random.default_rng(1).choice(B, 24, replace=False)
        got = run_outer(left, right, wT, dt, cuda_device)[rows]
        want = of.opm_outer(left[:, rows], right, wT, dt)
    else:
        got = run_outer(left, right, wT, dt, cuda_device)
        want = of.opm_outer(left, right, wT, dt)
    close('opm_outer fused B=%d D=%d F=%d' % (B, D, F), got, want, dt)


def test_opm_outer_refusals(cuda_device):
    d = cuda_device
    z = lambda *s: torch.zeros(s, dtype=torch.float16, device=d)
    with pytest.raises(ValueError, match='C a multiple of 16'):
        b200().volta_opm_outer(z(16, 4, 24), z(16, 4, 32), z(16, 24 * 32))
    with pytest.raises(ValueError, match='D a multiple of 4'):
        b200().volta_opm_outer(z(16, 4, 32), z(16, 6, 32), z(16, 32 * 32))
    with pytest.raises(ValueError, match='left must be'):
        b200().volta_opm_outer(z(8, 4, 32), z(16, 4, 32), z(16, 32 * 32))

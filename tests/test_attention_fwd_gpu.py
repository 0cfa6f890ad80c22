"""VoltaMma / VoltaMmaPacked[Trim] on the B200 against the CPU oracle and the golden fixtures.

Cases follow the reference's tests/test_attn_bwd.py (shapes, ragged and tiny lengths, every head
dim, a fully masked batch row, large amplitudes, want_lse) and tests/test_packed_attention.py
(rows and columns, gate, trim). Tolerances: the reference's own rel-max metric below 0.05 (its
test tolerance, tests/test_attn_bwd.py:166), relative L2 below 1e-2, and lse within 1e-3 (or
1e-3 relative where |lse| > 1, the float32 spacing near a fully masked row's -1.4e4).
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import attention as oa
from oracle.numerics import rel_l2, rel_max, round_to

pytestmark = pytest.mark.gpu

TD = {'f16': torch.float16, 'bf16': torch.bfloat16}


def b200():
    from colabfold_legacy_kernels import b200 as m
    return m


def to_dev(a, dt, dev):
    return torch.tensor(np.asarray(a, np.float32), dtype=TD[dt], device=dev)


def host(t):
    return t.float().cpu().numpy().astype(np.float64)


def assert_close(name, got, want, max_rel=0.05, l2=1e-2):
    r, e = rel_max(got, want), rel_l2(got, want)
    assert r < max_rel and e < l2, '%s: rel_max %.3e rel_l2 %.3e' % (name, r, e)


def assert_lse(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    assert np.isfinite(got[np.isfinite(want)]).all()
    assert err[np.isfinite(want)].max(initial=0) < 1e-3


def inputs(n, h, sq, sk, d, seed, dt, masked=0.15, qk_amp=0.5, vo_amp=0.5):
    """The reference's input recipe (tests/test_attn_bwd.py:114-125), rounded to dt."""
    rng = np.random.default_rng(seed)
    q = round_to(rng.standard_normal((n, h, sq, d)) * qk_amp, dt)
    k = round_to(rng.standard_normal((n, h, sk, d)) * qk_amp, dt)
    v = round_to(rng.standard_normal((n, h, sk, d)) * vo_amp, dt)
    bias = round_to(rng.standard_normal((h, sq, sk)) * qk_amp, dt)
    km = (rng.random((n, sk)) > masked).astype(np.uint8)
    dout = round_to(rng.standard_normal((n, h, sq, d)) * vo_amp, dt)
    return q, k, v, bias, km, dout


def run_fwd(q, k, v, bias, km, dt, dev, bq=64, bk=32, want_lse=True):
    m = b200()
    out, lse = m.volta_mma(to_dev(q, dt, dev), to_dev(k, dt, dev), to_dev(v, dt, dev),
                           to_dev(bias, dt, dev), torch.tensor(km, device=dev),
                           scale=q.shape[-1] ** -0.5, block_q=bq, block_k=bk, want_lse=want_lse)
    assert m.device_status() == 0
    return host(out), lse.cpu().numpy()


FIXTURES = golden('attn_*.npz')


@pytest.mark.parametrize('name,z', FIXTURES, ids=[n for n, _ in FIXTURES])
def test_forward_matches_golden(name, z, cuda_device):
    """f16, exactly the reference's inputs, against the reference oracle's own outputs."""
    d = z['q'].shape[-1]
    bq, bk = {8: (64, 64), 16: (64, 32), 32: (64, 32), 64: (64, 64)}[d]
    out, lse = run_fwd(z['q'], z['k'], z['v'], z['bias'], z['kmask'], 'f16', cuda_device, bq, bk)
    assert_close(name + ' out', out, z['out'])
    assert_lse(lse, z['lse2'])


SHAPES = [
    # n, h, sq, sk, d
    (3, 4, 96, 96, 32), (2, 4, 70, 83, 16), (1, 1, 128, 32, 8), (2, 2, 130, 130, 24),
    (2, 2, 130, 130, 48), (1, 2, 130, 130, 96), (2, 2, 64, 64, 64), (1, 8, 300, 260, 32),
    (2, 2, 1, 1, 16), (2, 2, 1, 4, 16), (2, 2, 7, 13, 16), (2, 2, 33, 1, 32), (2, 2, 3, 96, 8),
    (1, 1, 257, 513, 32),
]
TILE_FOR_D = {8: (64, 64), 16: (64, 32), 24: (64, 32), 32: (64, 32), 48: (64, 32),
              64: (64, 64), 96: (64, 32)}


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('shape', SHAPES, ids=['x'.join(map(str, s)) for s in SHAPES])
def test_forward_shapes(shape, dt, cuda_device):
    n, h, sq, sk, d = shape
    q, k, v, bias, km, _ = inputs(n, h, sq, sk, d, 0, dt)
    want, wlse = oa.attention_forward(q, k, v, bias, km, d ** -0.5)
    out, lse = run_fwd(q, k, v, bias, km, dt, cuda_device, *TILE_FOR_D[d])
    assert_close('out', out, want)
    assert_lse(lse, wlse)


def test_fully_masked_row_is_uniform(cuda_device):
    q, k, v, bias, km, _ = inputs(3, 4, 96, 96, 32, 0, 'bf16')
    km[:] = 1
    km[1] = 0
    out, lse = run_fwd(q, k, v, bias, km, 'bf16', cuda_device)
    want, wlse = oa.attention_forward(q, k, v, bias, km, 32 ** -0.5)
    assert_close('out', out, want)
    np.testing.assert_allclose(out[1], np.broadcast_to(v[1].mean(1, keepdims=True), out[1].shape),
                               atol=2e-2)
    assert_lse(lse, wlse)


@pytest.mark.parametrize('qk,vo', [(0.5, 32.0), (0.5, 90.0), (16.0, 0.5), (32.0, 0.5)])
def test_large_amplitudes(qk, vo, cuda_device):
    q, k, v, bias, km, _ = inputs(2, 2, 96, 96, 64, 0, 'f16', qk_amp=qk, vo_amp=vo)
    want, wlse = oa.attention_forward(q, k, v, bias, km, 64 ** -0.5)
    out, lse = run_fwd(q, k, v, bias, km, 'f16', cuda_device, 64, 64)
    assert_close('out', out, want)
    assert_lse(lse, wlse)


def test_want_lse_off_leaves_buffer_and_output(cuda_device):
    m = b200()
    q, k, v, bias, km, _ = inputs(2, 2, 96, 96, 32, 0, 'bf16')
    args = [to_dev(x, 'bf16', cuda_device) for x in (q, k, v, bias)]
    kmask = torch.tensor(km, device=cuda_device)
    out_on, _ = m.volta_mma(*args, kmask, scale=32 ** -0.5)
    one = torch.full((1,), 123.0, device=cuda_device)
    out_off, lse_off = m.volta_mma(*args, kmask, scale=32 ** -0.5, want_lse=False, lse=one)
    torch.cuda.synchronize()
    assert torch.equal(out_on, out_off)
    assert lse_off.item() == 123.0


def test_output_guard_band_untouched(cuda_device):
    """Canary-guarded output: the kernel writes exactly the output's elements."""
    m = b200()
    q, k, v, bias, km, _ = inputs(1, 2, 70, 83, 16, 0, 'bf16')
    args = [to_dev(x, 'bf16', cuda_device) for x in (q, k, v, bias)]
    n_out = q.size
    guard = 4096
    buf = torch.full((n_out + guard,), -7.0, dtype=torch.bfloat16, device=cuda_device)
    lse_buf = torch.full((1 * 2 * 70 + guard,), -7.0, device=cuda_device)
    out = buf[:n_out].view(q.shape)
    lse = lse_buf[:140].view(1, 2, 70)
    m.volta_mma(*args, torch.tensor(km, device=cuda_device), scale=0.25, out=out, lse=lse)
    torch.cuda.synchronize()
    assert (buf[n_out:] == -7.0).all()
    assert (lse_buf[140:] == -7.0).all()


def test_rejects_unsupported_tile_and_head_dim(cuda_device):
    m = b200()
    q = torch.zeros(1, 1, 8, 32, dtype=torch.float16, device=cuda_device)
    km = torch.ones(1, 8, dtype=torch.uint8, device=cuda_device)
    b = torch.zeros(1, 8, 8, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match='unsupported'):
        m.volta_mma(q, q, q, b, km, scale=1.0, block_q=64, block_k=128)
    q40 = torch.zeros(1, 1, 8, 40, dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match='unsupported'):
        m.volta_mma(q40, q40, q40, b, km, scale=1.0, block_q=64, block_k=32)


# ---- packed, gated, trimmed -----------------------------------------------------------------

PACKED = golden('packed_*.npz')


def run_packed(p, bias, km, gb, column, dt, dev, lims=None):
    m = b200()
    D = p.shape[-1]
    out = m.volta_mma_packed(to_dev(p, dt, dev), to_dev(bias, dt, dev),
                             torch.tensor(km.astype(np.uint8), device=dev), to_dev(gb, dt, dev),
                             None if lims is None else torch.tensor(lims, device=dev),
                             scale=D ** -0.5, block_q=64, block_k=64 if D == 64 else 32,
                             column=column)
    assert m.device_status() == 0
    return host(out)


@pytest.mark.parametrize('name,z', PACKED, ids=[n for n, _ in PACKED])
def test_packed_matches_golden(name, z, cuda_device):
    """tests/test_packed_attention.py's check: live rows within 0.03; with trim, live keys as
    the reference, padded queries as without trim or zero, dead rows exactly zero."""
    column = bool(z['column'])
    live = int(z['live'])
    to_bs = (lambda o: np.transpose(o, (1, 0, 2, 3))) if column else (lambda o: o)
    o = to_bs(run_packed(z['p'], z['bias'], z['kmask'], z['gate_bias'], column, 'f16',
                         cuda_device))
    r = z['out'].astype(np.float64)
    rows = z['kmask'].any(axis=1)
    assert np.abs(o[rows] - r[rows]).max(initial=0) < 0.03
    t = to_bs(run_packed(z['p'], z['bias'], z['kmask'], z['gate_bias'], column, 'f16',
                         cuda_device, z['lims']))
    assert np.abs(t[rows][:, :live] - r[rows][:, :live]).max(initial=0) < 0.03
    pad = t[rows][:, live:]
    assert np.minimum(np.abs(pad - o[rows][:, live:]), np.abs(pad)).max(initial=0) == 0
    assert np.abs(t[~rows]).max(initial=0) == 0


PACKED_CASES = [
    # X, Y, H, D, column, masked fraction, live (tests/test_packed_attention.py:89-93)
    (384, 384, 4, 32, False, 0.01, 384), (96, 384, 8, 32, True, 0.01, 96),
    (64, 256, 8, 8, False, 0.05, 256), (256, 64, 8, 8, True, 0.05, 64),
    (16, 128, 4, 16, False, 0.3, 128), (12, 200, 4, 64, False, 0.01, 200),
    (1, 261, 8, 32, True, 0.0, 1), (261, 1, 8, 32, False, 0.0, 1), (3, 37, 4, 32, True, 0.2, 3),
    (4, 264, 4, 32, False, 0.05, 264), (5, 129, 4, 32, True, 0.5, 5),
    (6, 256, 4, 32, False, 0.05, 200), (256, 6, 4, 32, True, 0.05, 200),
    (4, 128, 8, 8, False, 0.05, 72), (4, 261, 4, 32, False, 0.05, 200),
]


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('case', PACKED_CASES, ids=['_'.join(map(str, c)) for c in PACKED_CASES])
def test_packed_cases(case, dt, cuda_device):
    X, Y, H, D, column, frac, live = case
    rng = np.random.default_rng(0)
    p = round_to(rng.normal(size=(X, Y, 4, H, D)), dt)
    N, S = (Y, X) if column else (X, Y)
    bias = round_to(rng.normal(size=(H, S, S)), dt)
    gb = round_to(rng.normal(size=(H, D)) * .1, dt)
    km = rng.random((N, S)) >= frac
    if live < S:
        km[:, live:] = False
        km[-1] = False
    want = oa.packed_forward(p, bias, km, gb, D ** -0.5, column)
    got = run_packed(p, bias, km, gb, column, dt, cuda_device)
    assert_close('packed', got, want)
    lims = oa.trim_limits(km)
    want_t = oa.packed_forward(p, bias, km, gb, D ** -0.5, column, lims)
    got_t = run_packed(p, bias, km, gb, column, dt, cuda_device, lims)
    to_bs = (lambda o: np.transpose(o, (1, 0, 2, 3))) if column else (lambda o: o)
    rows = km.any(axis=1)
    gt, wt = to_bs(got_t), to_bs(want_t)
    assert np.abs(gt[~rows]).max(initial=0) == 0
    if rows.any():
        assert_close('trim live', gt[rows][:, :live], wt[rows][:, :live])


def test_packed_without_gate(cuda_device):
    """G == 3: no gate, the slot-3 pointer and gate_bias are not read."""
    rng = np.random.default_rng(3)
    X, Y, H, D = 8, 70, 4, 32
    p = round_to(rng.normal(size=(X, Y, 3, H, D)), 'bf16')
    bias = round_to(rng.normal(size=(H, Y, Y)), 'bf16')
    km = rng.random((X, Y)) > 0.1
    want = oa.packed_forward(p, bias, km, None, D ** -0.5, False)
    got = run_packed(p, bias, km, np.zeros((1,)), False, 'bf16', cuda_device)
    assert_close('packed G=3', got, want)

"""VoltaMmaBwd on the B200 against the CPU oracle, the golden fixtures and torch fp32 autograd.

Cases follow the reference's tests/test_attn_bwd.py: basic and ragged shapes, every head dim,
a fully masked batch row, large amplitudes, shapes below one tile, the batch sizes around its
grid-order threshold (63, 64, 96), repeated calls (dK and dV bitwise equal, dQ and dBias within
1e-3), want_dbias off (dK, dV unchanged, dBias exactly zero) and the custom-vjp composition.
"""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import attention as oa
from oracle.numerics import rel_l2, rel_max
from test_attention_fwd_gpu import TILE_FOR_D, b200, host, inputs, to_dev

pytestmark = pytest.mark.gpu

NAMES = ('dq', 'dk', 'dv', 'dbias')


def run_both(q, k, v, bias, km, dout, dt, dev, want_dbias=True, bq=None, bk=None):
    m = b200()
    d = q.shape[-1]
    bq, bk = (bq, bk) if bq else TILE_FOR_D[d]
    tq, tk, tv, tb = (to_dev(x, dt, dev) for x in (q, k, v, bias))
    kmask = torch.tensor(km, device=dev)
    scale = d ** -0.5
    out, lse = m.volta_mma(tq, tk, tv, tb, kmask, scale=scale, block_q=bq, block_k=bk)
    grads = m.volta_mma_bwd(tq, tk, tv, tb, kmask, out, to_dev(dout, dt, dev), lse, scale=scale,
                            want_dbias=want_dbias)
    assert m.device_status() == 0
    return out, lse, grads


def check_grads(got, want, tag=''):
    for name, g, w in zip(NAMES, got, want):
        g = host(g)
        r, e = rel_max(g, w), rel_l2(g, w)
        assert r < 0.05 and e < 1e-2, '%s %s: rel_max %.3e rel_l2 %.3e' % (tag, name, r, e)


FIXTURES = golden('attn_*.npz')


@pytest.mark.parametrize('name,z', FIXTURES, ids=[n for n, _ in FIXTURES])
def test_backward_matches_golden(name, z, cuda_device):
    _, _, grads = run_both(z['q'], z['k'], z['v'], z['bias'], z['kmask'], z['dout'], 'f16',
                           cuda_device)
    check_grads(grads, [z[n] for n in NAMES], name)


SHAPES = [
    (3, 4, 96, 96, 32), (2, 4, 70, 83, 16), (1, 1, 128, 32, 8), (2, 2, 130, 130, 24),
    (2, 2, 130, 130, 48), (1, 2, 130, 130, 96), (2, 2, 64, 64, 64), (1, 8, 300, 260, 32),
    (2, 2, 1, 1, 16), (2, 2, 1, 4, 16), (2, 2, 7, 13, 16), (2, 2, 33, 1, 32), (2, 2, 3, 96, 8),
    (1, 1, 257, 513, 32),
]


@pytest.mark.parametrize('dt', ['bf16', 'f16'])
@pytest.mark.parametrize('shape', SHAPES, ids=['x'.join(map(str, s)) for s in SHAPES])
def test_backward_shapes(shape, dt, cuda_device):
    n, h, sq, sk, d = shape
    q, k, v, bias, km, dout = inputs(n, h, sq, sk, d, 0, dt)
    want = oa.attention_grads(q, k, v, bias, km, dout, d ** -0.5)
    _, _, grads = run_both(q, k, v, bias, km, dout, dt, cuda_device)
    check_grads(grads, want[2:], str(shape))


def test_fully_masked_row(cuda_device):
    q, k, v, bias, km, dout = inputs(3, 4, 96, 96, 32, 0, 'bf16')
    km[:] = 1
    km[1] = 0
    want = oa.attention_grads(q, k, v, bias, km, dout, 32 ** -0.5)
    _, _, grads = run_both(q, k, v, bias, km, dout, 'bf16', cuda_device)
    check_grads(grads, want[2:])
    # a constant logit has no gradient: dQ and dK of the dead row are zero, dV is not
    assert float(grads[0][1].abs().max()) == 0.0
    assert float(grads[1][1].abs().max()) == 0.0
    assert float(grads[2][1].abs().max()) > 0.0


@pytest.mark.parametrize('qk,vo', [(0.5, 32.0), (0.5, 90.0), (16.0, 0.5), (32.0, 0.5)])
def test_large_amplitudes(qk, vo, cuda_device):
    q, k, v, bias, km, dout = inputs(2, 2, 96, 96, 64, 0, 'f16', qk_amp=qk, vo_amp=vo)
    want = oa.attention_grads(q, k, v, bias, km, dout, 64 ** -0.5)
    _, _, grads = run_both(q, k, v, bias, km, dout, 'f16', cuda_device)
    check_grads(grads, want[2:])


@pytest.mark.parametrize('n', [63, 64, 96])
def test_batch_sizes_around_grid_threshold(n, cuda_device):
    q, k, v, bias, km, dout = inputs(n, 2, 64, 64, 32, 0, 'bf16')
    want = oa.attention_grads(q, k, v, bias, km, dout, 32 ** -0.5)
    _, _, grads = run_both(q, k, v, bias, km, dout, 'bf16', cuda_device)
    check_grads(grads, want[2:])


def test_repeated_calls(cuda_device):
    m = b200()
    q, k, v, bias, km, dout = inputs(3, 4, 96, 96, 32, 0, 'bf16')
    tq, tk, tv, tb, td = (to_dev(x, 'bf16', cuda_device) for x in (q, k, v, bias, dout))
    kmask = torch.tensor(km, device=cuda_device)
    out, lse = m.volta_mma(tq, tk, tv, tb, kmask, scale=32 ** -0.5)
    a = m.volta_mma_bwd(tq, tk, tv, tb, kmask, out, td, lse, scale=32 ** -0.5)
    b = m.volta_mma_bwd(tq, tk, tv, tb, kmask, out, td, lse, scale=32 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
    assert rel_max(host(a[0]), host(b[0])) < 1e-3
    assert rel_max(host(a[3]), host(b[3])) < 1e-3


def test_want_dbias_off(cuda_device):
    m = b200()
    q, k, v, bias, km, dout = inputs(2, 2, 96, 96, 32, 0, 'f16')
    tq, tk, tv, tb, td = (to_dev(x, 'f16', cuda_device) for x in (q, k, v, bias, dout))
    kmask = torch.tensor(km, device=cuda_device)
    out, lse = m.volta_mma(tq, tk, tv, tb, kmask, scale=32 ** -0.5)
    on = m.volta_mma_bwd(tq, tk, tv, tb, kmask, out, td, lse, scale=32 ** -0.5)
    off = m.volta_mma_bwd(tq, tk, tv, tb, kmask, out, td, lse, scale=32 ** -0.5,
                          want_dbias=False)
    torch.cuda.synchronize()
    assert torch.equal(on[1], off[1]) and torch.equal(on[2], off[2])
    assert rel_max(host(on[0]), host(off[0])) < 1e-3
    assert float(off[3].abs().max()) == 0.0


def test_against_torch_autograd(cuda_device):
    """The kernels composed as a vjp against torch fp32 autograd of the same attention
    (the reference's vjp_case, tests/test_attn_bwd.py:262-293)."""
    q, k, v, bias, km, dout = inputs(2, 4, 96, 96, 32, 0, 'bf16')
    scale = 32 ** -0.5
    _, _, grads = run_both(q, k, v, bias, km, dout, 'bf16', cuda_device)
    tq, tk, tv, tb = (torch.tensor(x, dtype=torch.float32, device=cuda_device,
                                   requires_grad=True) for x in (q, k, v, bias))
    live = torch.tensor(km, device=cuda_device)[:, None, None, :] != 0
    logits = torch.where(live, scale * tq @ tk.transpose(-1, -2) + tb[None],
                         torch.tensor(-1e4, device=cuda_device))
    out = torch.softmax(logits, -1) @ tv
    (out * torch.tensor(dout, dtype=torch.float32, device=cuda_device)).sum().backward()
    want = [t.grad.double().cpu().numpy() for t in (tq, tk, tv, tb)]
    check_grads(grads, want, 'torch')


def test_guard_bands(cuda_device):
    """Canary-guarded results: the backward writes exactly its outputs."""
    m = b200()
    q, k, v, bias, km, dout = inputs(1, 2, 70, 83, 16, 0, 'bf16')
    tq, tk, tv, tb, td = (to_dev(x, 'bf16', cuda_device) for x in (q, k, v, bias, dout))
    kmask = torch.tensor(km, device=cuda_device)
    out, lse = m.volta_mma(tq, tk, tv, tb, kmask, scale=0.25)
    G = 4096
    lib = m.lib()
    bufs = [torch.full((t.numel() + G,), -7.0, dtype=dt, device=cuda_device)
            for t, dt in ((tq, torch.bfloat16), (tk, torch.bfloat16), (tv, torch.bfloat16),
                          (tb, torch.float32))]
    ws = torch.empty(m.volta_mma_bwd_workspace(1, 2, 70, 83, 16), dtype=torch.uint8,
                     device=cuda_device)
    import ctypes
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = lib.cflk_volta_mma_bwd(m._stream(), 1, P(tq), P(tk), P(tv), P(tb), P(kmask), P(out),
                                P(td), P(lse), P(bufs[0]), P(bufs[1]), P(bufs[2]), P(bufs[3]),
                                P(ws), ws.numel(), 1, 2, 70, 83, 16, 0.25, 1)
    assert rc == 0
    torch.cuda.synchronize()
    for t, b in zip((tq, tk, tv, tb), bufs):
        assert (b[t.numel():] == -7.0).all()


def test_rejects_bad_workspace_and_head_dim(cuda_device):
    m = b200()
    lib = m.lib()
    import ctypes
    z = ctypes.c_void_p(0)
    rc = lib.cflk_volta_mma_bwd(m._stream(), 0, z, z, z, z, z, z, z, z, z, z, z, z, z, 0, 1, 1,
                                8, 8, 40, 1.0, 1)
    assert rc == 1 and b'head dim' in lib.cflk_last_error()
    rc = lib.cflk_volta_mma_bwd(m._stream(), 0, z, z, z, z, z, z, z, z, z, z, z, z, z, 0, 1, 1,
                                8, 8, 32, 1.0, 1)
    assert rc == 2 and b'scratch' in lib.cflk_last_error()


def test_bf16_bias_beyond_f16_range(cuda_device):
    """A bf16 bias above f16's range (|b| > 65504) gives the backward the same P as the forward:
    the bias keeps its own 16-bit type through the backward's transpose."""
    q, k, v, bias, km, dout = inputs(2, 2, 96, 96, 32, 3, 'bf16')
    rng = np.random.default_rng(7)
    # about one key a row at +7e4 (bf16 69888 or 70144): it takes most of the row's softmax,
    # which a bias clamped to 65504 in the backward alone would move to the other keys; float32
    # resolves logits near 7e4 to 2^-7, so P keeps about 0.5% error in both passes
    big = rng.random(bias.shape) < 0.01
    bias = np.where(big, 7.0e4, bias)
    bias = oa_round(bias)
    want = oa.attention_grads(q, k, v, bias, km, dout, 32 ** -0.5)
    out, lse, grads = run_both(q, k, v, bias, km, dout, 'bf16', cuda_device)
    assert rel_max(host(out), want[0]) < 0.05
    check_grads(grads, want[2:], 'bf16 big bias')


def oa_round(x):
    from oracle.numerics import round_to
    return round_to(x, 'bf16')

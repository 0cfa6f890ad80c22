"""Parity at the BASELINE configs' own sizes: exactly the inputs bench.py times, through the same
entry points, checked with the north star's tolerances.

* configs[2] (the headline), MSA row attention: N_seq=512, N_res=512, H=8, d=32, bf16; forward
  with lse and backward with dBias summed over the 512 sequences.
* configs[1], triangle attention (starting node): pair 384 x 384, H=4, d=32, the last 38
  residues masked as keys, dBias over the 384 rows.
* configs[4], large-protein inference: pair 2048 x 2048, H=4, d=32, the last 5% masked, forward
  only with want_lse off and a one-element lse buffer (checked untouched); and the same rows
  through the packed, gated, trimmed target at that size.
* configs[3], the pair fusions on M = 768^2 = 589,824 rows.

References. The full outputs are compared with the float32 torch restatement of the reference's
closed form (tests/torch_reference.py, run on the GPU; pinned to the float64 oracle and the
golden fixtures by tests/test_torch_reference.py). Sampled batch rows are also compared with the
float64 oracle itself (oracle/attention.py); batch rows are independent, so a sampled row's out,
lse, dQ, dK and dV are exact checks of that row, and the torch reference's dBias over the same
rows is pinned to the oracle's. The fusions are compared with the fusion oracle
(oracle/fused.py) on sampled 128-row tiles: the first and last tiles, the tiles around the
persistent schedule's first wave boundary (148 CTAs) and 24 seeded random ones; rows are
independent, so each sampled tile is an exact check of those rows.

Tolerances (north star): max-abs 2e-2 (or one bfloat16 ulp of the reference where the output's
own rounding step is larger) and relative L2 1e-2 for the 16-bit outputs, relative L2 1e-2 for
dBias, lse within 1e-3; plus the reference's own rel-max metric below 0.05 (attention,
tests/test_attn_bwd.py:166) or 0.02 (fusions, tests/test_fused.py:51).
"""
import numpy as np
import pytest
import torch

import bench
import torch_reference as tr
from oracle import attention as oa
from oracle import fused as of
from oracle.numerics import max_abs, rel_l2, rel_max

pytestmark = pytest.mark.gpu


def b200():
    from colabfold_legacy_kernels import b200 as m
    return m


def host(t):
    return t.float().cpu().numpy().astype(np.float64)


def bf16_ulp(w):
    """One unit in the last place of bfloat16 at |w| (8 significant bits)."""
    m = np.maximum(np.abs(w), 1e-30)
    return np.exp2(np.floor(np.log2(m)) - 7)


def check(name, got, want, max_rel=0.05, l2=1e-2, absolute=2e-2):
    """rel-max and relative L2 bounds; and |got - want| <= 2e-2 (north star's max-abs) for every
    element, or one bfloat16 ulp of the reference where that is larger (an output with |w| >= 4
    is stored with a step of 2^-5 = 0.031, so a result one rounding step away is as close as the
    16-bit output can be)."""
    g, w = host(got) if torch.is_tensor(got) else got, host(want) if torch.is_tensor(want) else want
    r, e = rel_max(g, w), rel_l2(g, w)
    a = max_abs(g, w) if absolute is not None else 0.0
    msg = '%s: rel_max %.3e rel_l2 %.3e max_abs %.3e' % (name, r, e, a)
    assert r < max_rel and e < l2, msg
    if absolute is not None:
        over = np.abs(g - w) - np.maximum(absolute, bf16_ulp(w))
        assert over.max(initial=0.0) <= 0.0, msg


def check_lse(got, want):
    g, w = host(got), host(want) if torch.is_tensor(want) else np.asarray(want, np.float64)
    fin = np.isfinite(w)
    assert np.isfinite(g[fin]).all()
    assert np.abs(g[fin] - w[fin]).max(initial=0) < 1e-3
    assert (g[~fin] == w[~fin]).all()


def fwd_bwd_full(q, k, v, bias, kmask, dout):
    m = b200()
    scale = q.shape[-1] ** -0.5
    out, lse = m.volta_mma(q, k, v, bias, kmask, scale=scale)
    grads = m.volta_mma_bwd(q, k, v, bias, kmask, out, dout, lse, scale=scale)
    torch.cuda.synchronize()
    assert m.device_status() == 0
    return (out, lse) + tuple(grads)


def check_attention(got, q, k, v, bias, kmask, dout, sample):
    """Full outputs against the torch float32 reference; `sample` batch rows against the
    float64 oracle, which also pins the reference's dBias over those rows."""
    scale = q.shape[-1] ** -0.5
    want = tr.grads(q, k, v, bias, kmask, dout, scale, chunk=16)
    names = ('out', 'lse', 'dq', 'dk', 'dv', 'dbias')
    for nm, g, w in zip(names, got, want):
        if nm == 'lse':
            check_lse(g, w)
        elif nm == 'dbias':
            check(nm, g, w, absolute=None)
        else:
            check(nm, g, w)
    idx = torch.tensor(sample, device=q.device)
    hs = [host(t.index_select(0, idx)) for t in (q, k, v, dout)]
    km = kmask.index_select(0, idx).cpu().numpy()
    o64 = oa.attention_grads(hs[0], hs[1], hs[2], host(bias), km, hs[3], scale)
    for nm, g, w in zip(names[:5], got[:5], o64[:5]):
        gs = g.index_select(0, idx)
        if nm == 'lse':
            check_lse(gs, w)
        else:
            check(nm + ' (f64 oracle, sampled rows)', host(gs), w)
    sub = tr.grads(*(t.index_select(0, idx) for t in (q, k, v)), bias,
                   kmask.index_select(0, idx), dout.index_select(0, idx), scale)
    assert rel_l2(host(sub[5]), o64[5]) < 1e-5


def test_config3_msa_row_attention_full_size(cuda_device):
    q, k, v, bias, kmask, dout = bench.make_inputs(torch, cuda_device, 0, 1)
    assert tuple(q.shape) == (512, 8, 512, 32) and q.dtype == torch.bfloat16
    got = fwd_bwd_full(q, k, v, bias, kmask, dout)
    check_attention(got, q, k, v, bias, kmask, dout, sample=[0, 147, 300, 511])


def test_config2_triangle_attention_full_size(cuda_device):
    q, k, v, bias, kmask, dout = bench.make_triangle_inputs(torch, cuda_device, 0, 1)
    assert tuple(q.shape) == (384, 4, 384, 32) and int(kmask[:, -38:].sum()) == 0
    got = fwd_bwd_full(q, k, v, bias, kmask, dout)
    check_attention(got, q, k, v, bias, kmask, dout, sample=[0, 191, 345, 383])


def test_config2_sharded_rows_sum_to_the_whole(cuda_device):
    """The rows of each of 4 ranks run alone: their outputs are the whole run's rows, and their
    dBias partials sum to the whole run's dBias (the NCCL all-reduce adds exactly these)."""
    whole = bench.make_triangle_inputs(torch, cuda_device, 0, 1)
    ref = fwd_bwd_full(*whole)
    dbias = torch.zeros_like(ref[5])
    for r in range(4):
        part = bench.make_triangle_inputs(torch, cuda_device, r, 4)
        got = fwd_bwd_full(*part)
        a = r * 96
        check('out shard %d' % r, got[0], ref[0][a:a + 96], absolute=1e-2)
        assert torch.equal(got[3], ref[3][a:a + 96]) and torch.equal(got[4], ref[4][a:a + 96])
        dbias += got[5]
    check('dbias sum of shards', dbias, ref[5], absolute=None, l2=1e-5, max_rel=1e-4)


def test_config5_inference_full_size(cuda_device):
    m = b200()
    q, k, v, bias, kmask = bench.make_inference_inputs(torch, cuda_device, 0, 1)
    assert tuple(q.shape) == (2048, 4, 2048, 32)
    sentinel = torch.full((1,), 123.25, device=cuda_device)
    out, lse = m.volta_mma(q, k, v, bias, kmask, scale=32 ** -0.5, want_lse=False, lse=sentinel)
    torch.cuda.synchronize()
    assert m.device_status() == 0
    assert lse.data_ptr() == sentinel.data_ptr() and float(sentinel.item()) == 123.25
    assert bool(torch.isfinite(out).all())
    rows = list(range(0, 16)) + list(range(1016, 1032)) + list(range(2032, 2048))
    idx = torch.tensor(rows, device=cuda_device)
    sub = [t.index_select(0, idx) for t in (q, k, v, kmask)]
    want, _ = tr.forward(sub[0], sub[1], sub[2], bias, sub[3], 32 ** -0.5, chunk=8)
    check('out (torch fp32, 48 rows)', out.index_select(0, idx), want)
    pick = torch.tensor([5, 2047], device=cuda_device)
    o64, _ = oa.attention_forward(*(host(t.index_select(0, pick)) for t in (q, k, v)),
                                  host(bias), kmask.index_select(0, pick).cpu().numpy(),
                                  32 ** -0.5)
    check('out (f64 oracle, 2 rows)', host(out.index_select(0, pick)), o64)


def test_config5_packed_gated_trimmed_full_size(cuda_device):
    """The inference rows through VoltaMmaPackedTrim at full size: p [2048, 2048, 4, 4, 32]
    built from the same q, k, v and a gate, lims from the key mask."""
    m = b200()
    q, k, v, bias, kmask = bench.make_inference_inputs(torch, cuda_device, 0, 1)
    g = torch.Generator(device=cuda_device)
    g.manual_seed(9)
    gate = torch.randn(q.shape, generator=g, device=cuda_device).to(torch.bfloat16)
    gate_bias = torch.randn(4, 32, generator=g, device=cuda_device).to(torch.bfloat16)
    p = torch.stack([t.permute(0, 2, 1, 3) for t in (q, k, v, gate)], dim=2).contiguous()
    del gate
    lims = torch.tensor(oa.trim_limits(kmask.cpu().numpy()), device=cuda_device)
    out = m.volta_mma_packed(p, bias, kmask, gate_bias, lims, scale=32 ** -0.5)
    torch.cuda.synchronize()
    assert m.device_status() == 0 and tuple(out.shape) == (2048, 2048, 4, 32)
    rows = [0, 1023, 2047]
    idx = torch.tensor(rows, device=cuda_device)
    want = oa.packed_forward(host(p.index_select(0, idx)), host(bias),
                             kmask.index_select(0, idx).cpu().numpy(), host(gate_bias),
                             32 ** -0.5, False, lims=None)
    check('packed out (f64 oracle, 3 rows)', host(out.index_select(0, idx)), want)


# ---- the pair fusions at M = 589,824 ----------------------------------------------

M_PAIR = bench.PAIR * bench.PAIR
TILES = M_PAIR // 128


def sampled_rows():
    rng = np.random.default_rng(11)
    tiles = {0, 1, 146, 147, 148, 149, 295, 296, TILES // 2, TILES - 2, TILES - 1}
    tiles |= set(int(t) for t in rng.choice(TILES, 24, replace=False))
    tiles = sorted(tiles)
    return np.concatenate([np.arange(t * 128, (t + 1) * 128) for t in tiles])


class Pair:
    """Seeded bf16 inputs of the fusions (configs[3] distributions) on the device."""

    def __init__(self, dev):
        self.dev = dev
        self.g = torch.Generator(device=dev)
        self.g.manual_seed(21)
        self.x = self.rn(M_PAIR, 128)
        self.rows = sampled_rows()
        self.idx = torch.tensor(self.rows, device=dev)

    def rn(self, *shape, s=1.0, dt=torch.bfloat16):
        return (torch.randn(*shape, generator=self.g, device=self.dev) * s).to(dt)

    def f32(self, *shape, s=0.1, mean=0.0):
        return torch.randn(*shape, generator=self.g, device=self.dev) * s + mean

    def rows_of(self, t, axis=0):
        return host(t.index_select(axis, self.idx))


@pytest.fixture(scope='module')
def pair(cuda_device):
    return Pair(cuda_device)


def close_rows(name, got, want):
    check(name, got, want, max_rel=0.02)


@pytest.mark.parametrize('ci', [64, 128])
def test_config4_ln_gdp_full_size(ci, pair):
    P = pair
    sc, off = P.f32(128, mean=1.0), P.f32(128)
    wpT, wgT = P.rn(2 * ci, 128, s=128 ** -0.5), P.rn(2 * ci, 128, s=128 ** -0.5)
    bp, bg = P.rn(2 * ci, s=0.1), P.rn(2 * ci, s=0.1) + 1.0
    mask = (torch.rand(M_PAIR, generator=P.g, device=P.dev) > 0.1).to(torch.bfloat16)
    left, right = b200().volta_ln_gdp(P.x, sc, off, wpT, bp, wgT, bg, mask, eps=1e-5)
    assert b200().device_status() == 0
    wl, wr = of.ln_gdp(P.rows_of(P.x), host(sc), host(off), host(wpT), host(bp), host(wgT),
                       host(bg), P.rows_of(mask), 1e-5, 'bf16', 128)
    close_rows('left', P.rows_of(left, 1), wl)
    close_rows('right', P.rows_of(right, 1), wr)


@pytest.mark.parametrize('c', [64, 128])
def test_config4_trimul_epilogue_full_size(c, pair):
    P = pair
    x_cm = P.rn(c, M_PAIR, dt=torch.float32)
    isc, ioff, lsc, lof = P.f32(128, mean=1.0), P.f32(128), P.f32(c, mean=1.0), P.f32(c)
    woT, wgT = P.rn(128, c, s=c ** -0.5), P.rn(128, 128, s=128 ** -0.5)
    bo, bg = P.rn(128, s=0.1), P.rn(128, s=0.1)
    out = b200().volta_trimul_epilogue(x_cm, P.x, isc, ioff, lsc, lof, woT, bo, wgT, bg,
                                       torch.ones(1, dtype=torch.bfloat16, device=P.dev),
                                       eps=1e-5, add_input=True, has_keep=False)
    assert b200().device_status() == 0
    want = of.trimul_epilogue(P.rows_of(x_cm, 1), P.rows_of(P.x), host(isc), host(ioff),
                              host(lsc), host(lof), host(woT), host(bo), host(wgT), host(bg),
                              None, 1e-5, True, 'bf16', 128)
    close_rows('trimul C=%d' % c, P.rows_of(out), want)


def test_config4_ln_projection_full_size(pair):
    P = pair
    sc, off = P.f32(128, mean=1.0), P.f32(128)
    wT, wbT = P.rn(512, 128, s=128 ** -0.5), P.rn(4, 128, s=128 ** -0.5)
    p, bias = b200().volta_ln_proj(P.x, sc, off, wT, wbT, None, eps=1e-5, n=512, heads=4,
                                   has_keep=False)
    assert b200().device_status() == 0
    wp, wb = of.ln_projection(P.rows_of(P.x), host(sc), host(off), host(wT), host(wbT), None,
                              1e-5, 'bf16', 128)
    close_rows('p', P.rows_of(p), wp)
    close_rows('bias', P.rows_of(bias, 1), wb)


def test_config4_output_projection_full_size(pair):
    P = pair
    o, woT, bo, res = P.rn(M_PAIR, 128), P.rn(128, 128, s=128 ** -0.5), P.rn(128, s=0.1), \
        P.rn(M_PAIR, 128)
    out = b200().volta_out_proj(o, woT, bo, res, None, has_residual=True, has_keep=False)
    assert b200().device_status() == 0
    want = of.output_projection(P.rows_of(o), host(woT), host(bo), P.rows_of(res), None, 'bf16',
                                128)
    close_rows('out_proj', P.rows_of(out), want)


def test_config4_transition_full_size(pair):
    P = pair
    sc, off = P.f32(128, mean=1.0), P.f32(128)
    w1T, b1 = P.rn(512, 128, s=128 ** -0.5), P.rn(512, s=0.1)
    w2T, b2 = P.rn(512 * 128, s=512 ** -0.5), P.rn(128, s=0.1)
    out = b200().volta_transition(P.x, sc, off, w1T, b1, w2T, b2, None, eps=1e-5,
                                  add_input=True, has_keep=False)
    assert b200().device_status() == 0
    want = of.transition(P.rows_of(P.x), host(sc), host(off), host(w1T), host(b1), host(w2T),
                         host(b2), None, 1e-5, True, 'bf16', 128)
    close_rows('transition', P.rows_of(out), want)


def test_config4_layer_norm_and_gdp_full_size(pair):
    P = pair
    sc, off = P.f32(128, mean=1.0), P.f32(128)
    ln = b200().volta_layer_norm(P.x, sc, off, eps=1e-5)
    close_rows('layer_norm', P.rows_of(ln),
               of.layer_norm_one_pass(P.rows_of(P.x), host(sc), host(off), 1e-5, 'bf16'))
    wp, wg = P.rn(128, 128, s=128 ** -0.5), P.rn(128, 128, s=128 ** -0.5)
    bp, bg = P.rn(128, s=0.1), P.rn(128, s=0.1)
    mask = P.rn(M_PAIR, s=1.0)
    out = b200().volta_gdp(P.x, wp, bp, wg, bg, mask, activation=0)
    assert b200().device_status() == 0
    close_rows('gdp', P.rows_of(out),
               of.gdp(P.rows_of(P.x), host(wp), host(bp), host(wg), host(bg), P.rows_of(mask), 0,
                      'bf16'))

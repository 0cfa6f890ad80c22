"""The CPU oracle against the golden fixtures made by the reference's own oracle code
(tests/golden/make_golden.py runs colabfold-legacy-kernels' reference_grads and packed
reference). This pins the oracle before it is trusted as the checker of the CUDA path."""
import numpy as np
import pytest

from conftest import golden
from oracle import attention as oa
from oracle import fused as of
from oracle.numerics import rel_max, round_bf16, round_to

ATTN = golden('attn_*.npz')
PACKED = golden('packed_*.npz')


def test_fixtures_present():
    assert len(ATTN) >= 8 and len(PACKED) >= 4


@pytest.mark.parametrize('name,z', ATTN, ids=[n for n, _ in ATTN])
def test_attention_grads_match_reference_oracle(name, z):
    got = oa.attention_grads(z['q'], z['k'], z['v'], z['bias'], z['kmask'], z['dout'],
                             float(z['scale']))
    for key, g in zip(('out', 'lse2', 'dq', 'dk', 'dv', 'dbias'), got):
        want = z[key].astype(np.float64)
        err = np.abs(g - want).max() if want.size else 0.0
        # the fixtures hold float32 copies of float64 results
        assert err <= 1e-6 * max(1.0, np.abs(want).max()), (name, key, err)


@pytest.mark.parametrize('name,z', ATTN, ids=[n for n, _ in ATTN])
def test_float32_port_close_to_truth(name, z):
    got = oa.attention_grads_f32(z['q'], z['k'], z['v'], z['bias'], z['kmask'], z['dout'],
                                 float(z['scale']))
    for key, g in zip(('out', 'lse2', 'dq', 'dk', 'dv', 'dbias'), got):
        assert rel_max(g, z[key]) < 1e-3, (name, key)


@pytest.mark.parametrize('name,z', PACKED, ids=[n for n, _ in PACKED])
def test_packed_forward_matches_reference(name, z):
    """Rows with a live key match the reference's float32 packed oracle; the reference masks
    with -1e9 where the kernel uses -1e4, which only matters for rows with no live key."""
    column = bool(z['column'])
    X, Y, G, H, D = z['p'].shape
    out = oa.packed_forward(z['p'], z['bias'], z['kmask'], z['gate_bias'], D ** -0.5, column)
    rows = z['kmask'].any(axis=1)
    to_bs = (lambda o: np.transpose(o, (1, 0, 2, 3))) if column else (lambda o: o)
    # the reference returns [batch, sequence, H, D]; the kernel layout is [X, Y, H, D]
    o, r = to_bs(out), z['out'].astype(np.float64)
    assert np.abs(o[rows] - r[rows]).max() < 1e-5
    lims = oa.trim_limits(z['kmask'])
    np.testing.assert_array_equal(lims, z['lims'])
    t = to_bs(oa.packed_forward(z['p'], z['bias'], z['kmask'], z['gate_bias'], D ** -0.5,
                                column, lims))
    assert np.abs(t[~rows]).max(initial=0) == 0
    np.testing.assert_array_equal(t[rows], o[rows])


def test_dead_row_is_uniform_average():
    """A batch row with every key masked averages its keys (masked logit -1e4, not -inf)."""
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((2, 1, 5, 8)) for _ in range(3))
    bias = rng.standard_normal((1, 5, 7))[:, :, :5]
    km = np.ones((2, 5), np.uint8)
    km[1] = 0
    out, lse = oa.attention_forward(q, k, v, bias, km, 0.3)
    np.testing.assert_allclose(out[1, 0], np.broadcast_to(v[1, 0].mean(0), (5, 8)), atol=1e-12)
    np.testing.assert_allclose(lse[1], (-1e4 + np.log(5)) * oa.LOG2E, rtol=1e-12)


def test_bf16_rounding():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.14159, 65504.0, 1e-30], np.float32)
    r = round_bf16(x)
    import torch
    want = torch.tensor(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r, want)
    np.testing.assert_array_equal(round_to(x, 'f16'), x.astype(np.float16).astype(np.float64))


def test_layer_norm_two_pass():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((7, 64)) * 5 + 1e3
    y = of.layer_norm(x, np.ones(64), np.zeros(64), 1e-5)
    np.testing.assert_allclose(y.mean(-1), 0, atol=1e-3)
    np.testing.assert_allclose(y.std(-1), 1, atol=1e-3)


def test_layer_norm_one_pass():
    """VoltaLayerNorm's one-pass statistics: close to a float64 LayerNorm for centred rows, the
    variance clamped at zero (a constant row gives offset, not NaN)."""
    rng = np.random.default_rng(3)
    x = round_to(rng.standard_normal((9, 96)) * 2, 'f16')
    sc, off = rng.standard_normal(96) * 0.1 + 1, rng.standard_normal(96) * 0.1
    y = of.layer_norm_one_pass(x, sc, off, 1e-5, 'f32')
    m, v = x.mean(-1, keepdims=True), x.var(-1, keepdims=True)
    want = (x - m) / np.sqrt(v + 1e-5) * sc + off
    np.testing.assert_allclose(y, want, atol=1e-4)
    const = np.full((2, 32), 3.0)
    y = of.layer_norm_one_pass(const, np.ones(32), np.full(32, 0.25), 1e-5, 'f16')
    np.testing.assert_array_equal(y, np.full((2, 32), 0.25))


def test_gdp_activations():
    """VoltaGdp's restatement: sigmoid and swish gates, the row mask applied unclamped."""
    rng = np.random.default_rng(4)
    M, K, N = 5, 16, 8
    x = round_to(rng.standard_normal((M, K)), 'f16')
    wp, wg = rng.standard_normal((K, N)) * 0.3, rng.standard_normal((K, N)) * 0.3
    bp, bg = rng.standard_normal(N) * 0.1, rng.standard_normal(N) * 0.1
    mask = np.array([1.0, 0.0, -1.0, 0.5, 2.0])
    p, g = x @ wp + bp, x @ wg + bg
    s = 1 / (1 + np.exp(-g))
    for act, gate in ((0, s), (1, g * s)):
        got = of.gdp(x, wp, bp, wg, bg, mask, act, 'f32')
        np.testing.assert_allclose(got, mask[:, None] * p * gate, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError, match='activation'):
        of.gdp(x, wp, bp, wg, bg, mask, 2, 'f16')


def test_opm_update_and_outer():
    """The outer-product-mean restatements against plain float64 loops on small shapes."""
    rng = np.random.default_rng(5)
    B, K, D, F = 3, 32, 2, 16
    lhs = round_to(rng.standard_normal((B, K)), 'f16')
    t = round_to(rng.standard_normal((K, D, F)) * 0.2, 'f16')
    bias, norm = rng.standard_normal(F), np.abs(rng.standard_normal((B, D))) + 1
    res = round_to(rng.standard_normal((B, D, F)), 'f16')
    want = np.zeros((B, D, F))
    for b in range(B):
        for d in range(D):
            want[b, d] = (lhs[b] @ t[:, d, :] + bias) / (1e-3 + norm[b, d]) + res[b, d]
    got = of.opm_update(lhs, t, bias, norm, res, 1e-3, 'f32')
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    C, E = 2, 32
    left = round_to(rng.standard_normal((16, B, C)), 'f16')
    right = round_to(rng.standard_normal((16, D, E)), 'f16')
    wT = round_to(rng.standard_normal((F, C * E)) * 0.1, 'f16')
    want = np.zeros((B, D, F))
    for b in range(B):
        for d in range(D):
            g = np.einsum('ac,ae->ce', left[:, b, :], right[:, d, :]).reshape(C * E)
            want[b, d] = g @ wT.T
    got = of.opm_outer(left, right, wT, 'f32')
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)


def test_trimul_contract_directions():
    """The triangle contraction restatement against plain loops: outgoing sums over the shared
    last index (a[c,i,k] b[c,j,k]), incoming over the shared first (a[c,k,i] b[c,k,j])."""
    rng = np.random.default_rng(9)
    C, I, J, K = 2, 3, 4, 5
    a = rng.standard_normal((C, I, K))
    b = rng.standard_normal((C, J, K))
    want = np.zeros((C, I, J))
    for c in range(C):
        for i in range(I):
            for j in range(J):
                want[c, i, j] = sum(a[c, i, k] * b[c, j, k] for k in range(K))
    np.testing.assert_allclose(of.trimul_contract(a, b, False), want, rtol=1e-12)
    np.testing.assert_allclose(of.trimul_contract(a.transpose(0, 2, 1), b.transpose(0, 2, 1),
                                                  True), want, rtol=1e-12)


def test_tile_work():
    keep = np.array([1, 0, -1, -1, 0, 0, -1, -1, -1, -1], np.float32)
    assert of.tile_work(keep, 10, 2, -1.0) == ['compute', 'skip', 'padding', 'skip', 'skip']
    assert of.tile_work(keep, 10, 4, 0.0) == ['compute', 'padding', 'padding']
    assert of.tile_work(None, 10, 4, 0.0) == ['compute'] * 3


def test_transition_chunking_round_trip():
    w2 = np.arange(128 * 64, dtype=np.float64).reshape(128, 64)
    c = of.chunk_w2(w2)
    assert c.shape == (2, 64, 64)
    assert c[1, 5, 7] == w2[64 + 7, 5]
    np.testing.assert_array_equal(of.unchunk_w2(c), w2)

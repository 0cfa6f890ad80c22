"""CPU oracle for the LayerNorm-folded pair-stack fusions -- TEST INFRASTRUCTURE only.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may
import this module. The library never calls it.

PARITY UNPINNED against the reference's own oracles: colabfold-legacy-kernels checks these
kernels against float32 references in the sibling package `colabfold_kernels`
(tri_mul.ref_ln_gdp, tri_mul.ref_trimul_epilogue_ln, packed_attn.ref_ln_projection,
packed_attn.ref_output_projection, transition.ref_transition; tests/test_fused.py:19-22), which
is not vendored, has no pinned version and is absent here. This module restates the math from
the reference's handler contracts and kernels instead:

  * VoltaLayerNorm (the standalone op): one-pass float32 sum and sum of squares, the variance
    clamped at zero (cuda/volta_ops.cu:27-60).
  * VoltaGdp: mask * (x wp + bp) * sigmoid or swish (x wg + bg), the row mask unclamped
    (cuda/volta_ops.cu:108-205, cuda/volta_gdp.h:10-19).
  * VoltaOpmUpdate / VoltaOpmOuter (no cc=100 kernels yet): the outer-product-mean update and
    the 16-row outer product with its inner product rounded to 16 bits
    (cuda/volta_fused_ffi.h:261-335, cuda/volta_ops.cu:647-787).
  * LayerNorm: two-pass float32 statistics, eps inside the rsqrt, result rounded to the 16-bit
    compute type before the GEMM (ln_rows, cuda/volta_gdp.h:208-240; ln_columns over the
    channel-major float32 x_cm, :244-286).
  * keep: per row tile, compute when any keep > 0, write padding (zeros, or nothing where the
    output aliases its input) when the tile is all zero, write nothing when it is all below zero
    (tile_work, cuda/volta_gdp.h:114-136). Rows past M count as `other`.
  * ln_gdp: left/right [P/2, M] = max(mask, 0) * (y wp + bp) * sigmoid(y wg + bg), channel
    major; the mask is the keep with other = 0 (cuda/volta_fused_ffi.h:42-43,
    cuda/volta_ops.cu:349-393).
  * trimul_epilogue: out = (LN(x_cm^T) wo + bo) * sigmoid(LN_in(x) wg + bg) (+ x)
    (cuda/volta_fused_ffi.h:91, cuda/volta_ops.cu:408-466).
  * ln_projection: p = LN(x) w, bias[h, m] = (LN(x) wb)^T, no bias vector
    (cuda/volta_fused_ffi.h:135-136, cuda/volta_ops.cu:480-542, head_bias cuda/volta_gdp.h:290-332).
  * output_projection: out = o w + b (+ residual) (cuda/volta_fused_ffi.h:178).
  * transition: out = relu(LN(x) w1 + b1) w2 + b2 (+ x), the hidden activation rounded to the
    compute type; w2T holds w2 [H, C] as [H/64][C][64] chunks (cuda/volta_fused_ffi.h:216-217,
    cuda/volta_ops.cu:562-635).

Outputs are float64 arrays holding values rounded to the compute type, except where a tile is
skipped (the `before` contents are kept).
"""
import numpy as np

from .numerics import round_to

HIDDEN_CHUNK = 64


def layer_norm(x, scale, offset, eps):
    """Two-pass LayerNorm over the last axis in float32, as ln_rows does; float64 out."""
    v = np.asarray(x, np.float32)
    mean = v.sum(-1, keepdims=True, dtype=np.float32) * np.float32(1.0 / v.shape[-1])
    d = v - mean
    var = (d * d).sum(-1, keepdims=True, dtype=np.float32) * np.float32(1.0 / v.shape[-1])
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    y = d * rstd * np.asarray(scale, np.float32) + np.asarray(offset, np.float32)
    return y.astype(np.float64)


def layer_norm_one_pass(x, scale, offset, eps, dtype):
    """VoltaLayerNorm (cuda/volta_ops.cu:27-60): float32 sum and sum of squares over the last
    axis, mean = sum / C, var = max(sqsum / C - mean^2, 0), rstd = 1 / sqrt(var + eps),
    out = (x - mean) * rstd * scale + offset rounded to `dtype`; float64 out."""
    v = np.asarray(x, np.float32)
    inv = np.float32(1.0 / v.shape[-1])
    mean = v.sum(-1, keepdims=True, dtype=np.float32) * inv
    sq = (v * v).sum(-1, keepdims=True, dtype=np.float32) * inv
    var = np.maximum(sq - mean * mean, np.float32(0))
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    y = (v - mean) * rstd * np.asarray(scale, np.float32) + np.asarray(offset, np.float32)
    return round_to(y.astype(np.float64), dtype)


def sigmoid(g):
    return 1.0 / (1.0 + np.exp(-g))


def opm_update(lhs, t, bias, norm, residual, eps, dtype):
    """VoltaOpmUpdate (cuda/volta_fused_ffi.h:261-298, kernel cuda/volta_ops.cu:647-699):
    out [B, D, F] = (lhs @ t[:, d, :] + bias) / (eps + norm[b, d]) (+ residual), lhs [B, K],
    t [K, D, F], bias [F] and norm [B, D] float32; products in float32, the result rounded to
    `dtype`; float64 out."""
    l32 = np.asarray(lhs, np.float32)
    t32 = np.asarray(t, np.float32)
    K, D, F = t32.shape
    prod = (l32 @ t32.reshape(K, D * F)).reshape(-1, D, F)
    den = np.float32(eps) + np.asarray(norm, np.float32)[:, :, None]
    out = (prod + np.asarray(bias, np.float32)) / den
    if residual is not None:
        out = out + np.asarray(residual, np.float32)
    return round_to(out.astype(np.float64), dtype)


def trimul_contract(a, b, incoming):
    """The triangle multiplication's contraction (tests/test_fused.py:135 of the reference, an
    XLA einsum with preferred_element_type float32): outgoing einsum('cik,cjk->cij'), incoming
    einsum('cki,ckj->cij'); float64 sums of the 16-bit inputs, float64 out."""
    a64 = np.asarray(a, np.float64)
    b64 = np.asarray(b, np.float64)
    if incoming:
        return np.einsum('cki,ckj->cij', a64, b64, optimize=True)
    return np.einsum('cik,cjk->cij', a64, b64, optimize=True)


def opm_outer(left, right, wT, dtype):
    """VoltaOpmOuter (cuda/volta_fused_ffi.h:300-335, kernel cuda/volta_ops.cu:710-787): on 16
    MSA rows a, out [B, D, F] = sum over c, e of h(sum_a left[a, b, c] right[a, d, e]) w[c E + e, f]
    with h the rounding of the float32 inner product to the 16-bit type (the kernel rounds it in
    registers before the second product), left [16, B, C], right [16, D, E], wT [F, C E];
    accumulated in float32, the result rounded to `dtype`; float64 out."""
    l32 = np.asarray(left, np.float32)
    r32 = np.asarray(right, np.float32)
    g = np.einsum('abc,ade->bdce', l32, r32).astype(np.float32)
    g = round_to(g, dtype).astype(np.float32)
    B, D, C, E = g.shape
    w = np.asarray(wT, np.float32).T  # [C E, F]
    out = g.reshape(B, D, C * E) @ w
    return round_to(out.astype(np.float64), dtype)


def gdp(x, wp, bp, wg, bg, mask, activation, dtype):
    """VoltaGdp, the unfused gated dual projection (cuda/volta_ops.cu:108-205, its activation
    cuda/volta_gdp.h:10-19): out [M, N] = mask[m] * (x wp + bp) * act(x wg + bg), wp and wg
    [K, N] row-major, the row mask as given (not clamped), act = sigmoid (activation 0) or
    swish g * sigmoid(g) (activation 1); products accumulated in float32, the result rounded to
    `dtype`; float64 out."""
    if activation not in (0, 1):
        raise ValueError('gdp: activation is 0 (sigmoid) or 1 (swish), got %r' % (activation,))
    x32 = np.asarray(x, np.float32)
    p = x32 @ np.asarray(wp, np.float32) + np.asarray(bp, np.float32)
    g = x32 @ np.asarray(wg, np.float32) + np.asarray(bg, np.float32)
    s = sigmoid(g.astype(np.float64))
    act = s if activation == 0 else g * s
    out = np.asarray(mask, np.float64)[:, None] * p * act
    return round_to(out, dtype)


def tile_work(keep, M, tile, other):
    """'compute', 'padding' or 'skip' per row tile of `tile` rows (None keep: all compute)."""
    n_tiles = -(-M // tile)
    if keep is None:
        return ['compute'] * n_tiles
    k = np.full(n_tiles * tile, float(other))
    k[:M] = np.asarray(keep, np.float64)
    k = k.reshape(n_tiles, tile)
    work = []
    for row in k:
        if (row > 0).any():
            work.append('compute')
        elif (row == 0).any():
            work.append('padding')
        else:
            work.append('skip')
    return work


def _apply_tiles(M, tile, work, computed, padded, before, row_axis):
    """Assemble an output: computed rows in compute tiles, `padded` (or before) in padding
    tiles, before in skip tiles. row_axis: the axis that indexes rows (0, or 1 channel-major)."""
    out = np.array(before, np.float64, copy=True)
    for t, w in enumerate(work):
        sl = slice(t * tile, min(M, (t + 1) * tile))
        idx = (sl,) if row_axis == 0 else (slice(None), sl)
        if w == 'compute':
            out[idx] = computed[idx]
        elif w == 'padding' and padded is not None:
            out[idx] = padded[idx]
    return out


def ln_gdp(x, scale, offset, wpT, bp, wgT, bg, mask, eps, dtype, tile, before=None):
    """(left, right), each [P/2, M]."""
    M = x.shape[0]
    P = wpT.shape[0]
    y = round_to(layer_norm(x, scale, offset, eps), dtype)
    pp = y @ np.asarray(wpT, np.float64).T + np.asarray(bp, np.float64)
    gg = y @ np.asarray(wgT, np.float64).T + np.asarray(bg, np.float64)
    mv = np.maximum(np.asarray(mask, np.float64), 0.0)[:, None]
    val = round_to(mv * pp * sigmoid(gg), dtype).T            # [P, M]
    if before is None:
        before = np.zeros((P, M))
    else:
        before = np.concatenate([np.asarray(b, np.float64) for b in before], 0)
    work = tile_work(mask, M, tile, 0.0)
    full = _apply_tiles(M, tile, work, val, np.zeros_like(val), before, row_axis=1)
    return full[:P // 2], full[P // 2:]


def trimul_epilogue(x_cm, x, in_scale, in_offset, ln_scale, ln_offset, woT, bo, wgT, bg, keep,
                    eps, add_input, dtype, tile, before=None):
    """out [M, O]."""
    M = x.shape[0]
    O = woT.shape[0]
    y = round_to(layer_norm(np.asarray(x_cm, np.float32).T, ln_scale, ln_offset, eps), dtype)
    a = round_to(layer_norm(x, in_scale, in_offset, eps), dtype)
    o = y @ np.asarray(woT, np.float64).T + np.asarray(bo, np.float64)
    g = a @ np.asarray(wgT, np.float64).T + np.asarray(bg, np.float64)
    val = o * sigmoid(g)
    if add_input:
        val = val + np.asarray(x, np.float64)
    val = round_to(val, dtype)
    if before is None:
        before = np.zeros((M, O))
    work = tile_work(keep, M, tile, -1.0)
    padded = None if add_input else np.zeros_like(val)
    return _apply_tiles(M, tile, work, val, padded, before, row_axis=0)


def ln_projection(x, scale, offset, wT, wbT, keep, eps, dtype, tile, before=(None, None)):
    """(p [M, n] or None, bias [heads, M] or None)."""
    M = x.shape[0]
    y = round_to(layer_norm(x, scale, offset, eps), dtype)
    work = tile_work(keep, M, tile, -1.0)
    p = bias = None
    if wT is not None and wT.shape[0]:
        val = round_to(y @ np.asarray(wT, np.float64).T, dtype)
        b0 = np.zeros_like(val) if before[0] is None else before[0]
        p = _apply_tiles(M, tile, work, val, np.zeros_like(val), b0, row_axis=0)
    if wbT is not None and wbT.shape[0]:
        val = round_to((y @ np.asarray(wbT, np.float64).T).T, dtype)
        b1 = np.zeros_like(val) if before[1] is None else before[1]
        bias = _apply_tiles(M, tile, work, val, np.zeros_like(val), b1, row_axis=1)
    return p, bias


def output_projection(o, wT, b, residual, keep, dtype, tile, before=None):
    """out [M, N] = o w + b (+ residual)."""
    M = o.shape[0]
    val = np.asarray(o, np.float64) @ np.asarray(wT, np.float64).T + np.asarray(b, np.float64)
    if residual is not None:
        val = val + np.asarray(residual, np.float64)
    val = round_to(val, dtype)
    if before is None:
        before = np.zeros_like(val)
    work = tile_work(keep, M, tile, -1.0)
    padded = None if residual is not None else np.zeros_like(val)
    return _apply_tiles(M, tile, work, val, padded, before, row_axis=0)


def chunk_w2(w2):
    """w2 [H, C] -> w2T [H/64, C, 64], the layout VoltaTransition takes."""
    H, C = w2.shape
    return np.ascontiguousarray(np.asarray(w2).reshape(H // HIDDEN_CHUNK, HIDDEN_CHUNK, C)
                                .transpose(0, 2, 1))


def unchunk_w2(w2T):
    """Inverse of chunk_w2: [H/64, C, 64] -> [H, C]."""
    n, C, j = w2T.shape
    return np.asarray(w2T).transpose(0, 2, 1).reshape(n * j, C)


def transition(x, scale, offset, w1T, b1, w2T, b2, keep, eps, add_input, dtype, tile,
               before=None):
    """out [M, C] = relu(LN(x) w1 + b1) w2 + b2 (+ x); w2T chunked [H/64, C, 64]."""
    M, C = x.shape
    y = round_to(layer_norm(x, scale, offset, eps), dtype)
    hid = np.maximum(y @ np.asarray(w1T, np.float64).T + np.asarray(b1, np.float64), 0.0)
    hid = round_to(hid, dtype)
    w2 = unchunk_w2(np.asarray(w2T, np.float64).reshape(-1, C, HIDDEN_CHUNK))
    val = hid @ w2 + np.asarray(b2, np.float64)
    if add_input:
        val = val + np.asarray(x, np.float64)
    val = round_to(val, dtype)
    if before is None:
        before = np.zeros_like(val)
    work = tile_work(keep, M, tile, -1.0)
    padded = None if add_input else np.zeros_like(val)
    return _apply_tiles(M, tile, work, val, padded, before, row_axis=0)

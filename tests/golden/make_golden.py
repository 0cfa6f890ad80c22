"""Generate the golden attention fixtures by running the reference's own oracle code.

  python tests/golden/make_golden.py REFERENCE_ROOT

REFERENCE_ROOT is a checkout of colabfold-legacy-kernels (or set CFLK_REFERENCE_ROOT). Its test
files import jax, which this environment does not have, so the script does not import them:
it parses each file, takes the functions named below out of its syntax tree and executes them
against numpy, with a small numpy stand-in for the few jax.numpy / jax.nn calls they make.
Nothing of the reference is copied into this repository; only the arrays they produce are.

  tests/test_attn_bwd.py          inputs(), reference_grads()       -> attn_*.npz
  tests/test_packed_attention.py  reference(), trim_limits()        -> packed_*.npz

Inputs are stored as float16 (as the reference's `inputs` makes them), results as float32.
"""
import ast
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _jax_shim():
    """The subset of jax / jax.numpy the extracted functions call, on numpy."""
    jnp = types.SimpleNamespace(
        float16=np.float16, float32=np.float32, int32=np.int32, uint8=np.uint8,
        asarray=lambda x, dtype=None: np.asarray(x, dtype),
        where=np.where, transpose=np.transpose, concatenate=np.concatenate,
        einsum=lambda spec, *ops, precision=None: np.einsum(
            spec, *[np.asarray(o, np.float64) for o in ops]).astype(np.float32),
    )

    def softmax(x, axis=-1):
        x = np.asarray(x, np.float64)
        e = np.exp(x - x.max(axis=axis, keepdims=True))
        return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)

    def sigmoid(x):
        return (1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))).astype(np.float32)

    jax = types.SimpleNamespace(
        nn=types.SimpleNamespace(softmax=softmax, sigmoid=sigmoid),
        lax=types.SimpleNamespace(Precision=types.SimpleNamespace(HIGHEST=None)),
    )
    return jax, jnp


def load_functions(path, names, constants=()):
    """Execute the named top-level functions (and constant assignments) of a Python file."""
    tree = ast.parse(open(path).read(), path)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id in constants for t in node.targets):
            keep.append(node)
    module = ast.Module(body=keep, type_ignores=[])
    jax, jnp = _jax_shim()
    ns = {'np': np, 'jax': jax, 'jnp': jnp}
    exec(compile(module, path, 'exec'), ns)
    missing = [n for n in names if n not in ns]
    if missing:
        raise RuntimeError('%s: functions not found: %s' % (path, missing))
    return ns


# (n, h, sq, sk, d, seed, masked-batch-row): shapes from the reference's own case list
ATTN_CASES = (
    ('basic', 2, 2, 96, 96, 32, 0, None),           # tests/test_attn_bwd.py:379
    ('ragged', 2, 4, 70, 83, 16, 0, None),          # :382 (ragged, both axes)
    ('d8', 1, 1, 128, 32, 8, 0, None),              # :383
    ('allmasked', 3, 2, 64, 64, 32, 0, 1),          # :175-181
    ('tiny_1_1', 2, 2, 1, 1, 16, 0, None),          # :228
    ('tiny_7_13', 2, 2, 7, 13, 16, 0, None),        # :228
    ('tiny_33_1', 2, 2, 33, 1, 32, 0, None),        # :228
    ('d64', 1, 2, 64, 64, 64, 0, None),             # :381
)

# X, Y, H, D, column, masked fraction, live length: the patterns of
# tests/test_packed_attention.py:89-93 (rows and columns, D 8-32, S not a multiple of 8, trim),
# at sizes that keep the fixtures small
PACKED_CASES = (
    (3, 37, 4, 32, True, 0.2, 3),
    (4, 72, 4, 8, False, 0.05, 40),
    (5, 67, 2, 32, True, 0.5, 5),
    (6, 64, 2, 16, False, 0.3, 64),
)


def main(ref_root):
    attn = load_functions(os.path.join(ref_root, 'tests', 'test_attn_bwd.py'),
                          ('inputs', 'reference_grads'), constants=('NEG',))
    packed = load_functions(os.path.join(ref_root, 'tests', 'test_packed_attention.py'),
                            ('reference', 'trim_limits'), constants=('NEG',))

    for name, n, h, sq, sk, d, seed, dead in ATTN_CASES:
        q, k, v, bias, km, dout = attn['inputs'](n, h, sq, sk, d, seed)
        km = np.asarray(km)
        if dead is not None:
            km = np.ones((n, sk), np.uint8)
            km[dead, :] = 0
        scale = float(d) ** -0.5
        out, lse2, dq, dk, dv, dbias = attn['reference_grads'](q, k, v, bias, km, dout, scale)
        f32 = lambda a: np.asarray(a, np.float32)
        np.savez_compressed(
            os.path.join(HERE, 'attn_%s.npz' % name),
            q=np.asarray(q, np.float16), k=np.asarray(k, np.float16),
            v=np.asarray(v, np.float16), bias=np.asarray(bias, np.float16),
            kmask=km.astype(np.uint8), dout=np.asarray(dout, np.float16),
            scale=np.float32(scale), out=f32(out), lse2=f32(lse2), dq=f32(dq), dk=f32(dk),
            dv=f32(dv), dbias=f32(dbias))
        print('attn_%s.npz' % name)

    for X, Y, H, D, column, frac, live in PACKED_CASES:
        rng = np.random.default_rng(0)              # as tests/test_packed_attention.py:62-70
        p = np.asarray(rng.normal(size=(X, Y, 4, H, D)), np.float16)
        N, S = (Y, X) if column else (X, Y)
        bias = np.asarray(rng.normal(size=(H, S, S)), np.float16)
        gb = np.asarray(rng.normal(size=(H, D)) * .1, np.float16)
        km = rng.random((N, S)) >= frac
        if live < S:
            km[:, live:] = False
            km[-1] = False
        r = packed['reference'](p, bias, km, gb, column)
        lims = np.asarray(packed['trim_limits'](km), np.int32)
        tag = 'packed_%d_%d_%d_%d_%s' % (X, Y, H, D, 'col' if column else 'row')
        np.savez_compressed(os.path.join(HERE, tag + '.npz'), p=p, bias=bias, gate_bias=gb,
                            kmask=km.astype(np.uint8), lims=lims, column=np.bool_(column),
                            live=np.int32(live), out=np.asarray(r, np.float32))
        print(tag + '.npz')


if __name__ == '__main__':
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('CFLK_REFERENCE_ROOT')
    if not root:
        sys.exit('usage: make_golden.py REFERENCE_ROOT (a colabfold-legacy-kernels checkout)')
    main(root)

"""CPU-side checks of the drop-in boundary: the library loads and exports every entry point that
include/*.h declares, invalid arguments are refused before anything is launched, and the resolver
mirrors the reference's Python surface with compute capability 100 added
(src/colabfold_legacy_kernels/__init__.py:69-126 of the reference; its CI smoke test,
.github/workflows/build-and-publish.yml:72-89, asserts sm_80 is unavailable)."""
import ctypes
import os

import pytest

import colabfold_legacy_kernels as clk
from conftest import ROOT

import __graft_entry__ as ge


def lib():
    try:
        path = clk.library_path('attention', 100)
    except FileNotFoundError:
        pytest.fail('libcflk_sm100.so is not built (run __graft_entry__.build())')
    return ctypes.CDLL(path)


def test_library_exports_every_declared_symbol():
    names = ge.declared_symbols()
    assert 'cflk_volta_mma' in names and 'cflk_volta_transition' in names
    l = lib()
    missing = [n for n in names if not hasattr(l, n)]
    assert not missing


def test_every_cc100_target_has_a_declared_entry_point_and_binding():
    """Each cc=100 FFI target maps to a C entry point that include/*.h declares, and the torch
    binding carries its prototype."""
    from colabfold_legacy_kernels import b200
    names = set(ge.declared_symbols())
    for k in clk.KERNELS:
        if not clk.available(100, k):
            continue
        sym = clk.c_symbol(k, 100)
        assert sym in names, (k, sym)
        assert sym in b200._SIGS, (k, sym)


def test_layer_norm_refuses_bad_shapes_without_gpu():
    l = lib()
    l.cflk_last_error.restype = ctypes.c_char_p
    f = l.cflk_volta_layer_norm
    f.argtypes = [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 4 + [
        ctypes.c_int64, ctypes.c_int64, ctypes.c_float]
    assert f(None, 0, None, None, None, None, -1, 128, 1e-5) == 1
    assert b'[M,C]' in l.cflk_last_error()
    assert f(None, 5, None, None, None, None, 4, 128, 1e-5) == 1
    assert f(None, 0, None, None, None, None, 0, 128, 1e-5) == 0  # M = 0: nothing to do


def test_version_and_error_reporting_without_gpu():
    l = lib()
    l.cflk_last_error.restype = ctypes.c_char_p
    assert l.cflk_version() == 100
    z = ctypes.c_void_p(0)
    i64 = ctypes.c_int64
    # unsupported widths are refused before any CUDA call
    rc = l.cflk_volta_ln_gdp(z, 0, z, z, z, z, z, z, z, z, z, z, i64(10), i64(256), i64(512),
                             ctypes.c_float(1e-5))
    assert rc == 1 and b'64 or 128' in l.cflk_last_error()
    rc = l.cflk_volta_transition(z, 0, z, z, z, z, z, z, z, z, z, i64(10), i64(128), i64(384),
                                 ctypes.c_float(1e-5), 0)
    assert rc == 1 and b'H 2C or 4C' in l.cflk_last_error()
    rc = l.cflk_volta_mma(z, 0, z, z, z, z, z, z, z, i64(1), i64(1), i64(8), i64(8), i64(32),
                          ctypes.c_float(1.0), i64(64), i64(128), 1)
    assert rc == 1 and b'unsupported (D, bq, bk)' in l.cflk_last_error()
    rc = l.cflk_volta_mma(z, 5, z, z, z, z, z, z, z, i64(1), i64(1), i64(8), i64(8), i64(32),
                          ctypes.c_float(1.0), i64(64), i64(32), 1)
    assert rc == 1 and b'dtype' in l.cflk_last_error()
    # M == 0 succeeds without a launch, as the reference's handlers do
    rc = l.cflk_volta_out_proj(z, 0, z, z, z, z, z, z, i64(0), i64(128), i64(128))
    assert rc == 0 and l.cflk_last_error() == b''


def test_workspace_size():
    l = lib()
    n = ctypes.c_size_t(0)
    assert l.cflk_volta_mma_bwd_workspace_size(ctypes.c_int64(2), ctypes.c_int64(3),
                                               ctypes.c_int64(10), ctypes.c_int64(7),
                                               ctypes.c_int64(32), ctypes.byref(n)) == 0
    rows = 2 * 3 * 10
    align = lambda x: (x + 255) // 256 * 256
    # dQ accumulator, the two negated row statistics (-delta, -lse), f16 bias^T with the
    # queries padded to a multiple of 8
    assert n.value == (align(rows * 32 * 4) + 2 * align(rows * 4) + align(3 * 7 * 16 * 2))


def test_workspace_size_refuses_overflowing_sizes():
    """Sizes whose byte counts overflow 64 bits are refused, not wrapped; the no-allocation
    backward refuses them before it touches the GPU (its scratch size check relies on this)."""
    l = lib()
    l.cflk_last_error.restype = ctypes.c_char_p
    n = ctypes.c_size_t(0)
    i64 = ctypes.c_int64
    big = i64(1 << 40)
    assert l.cflk_volta_mma_bwd_workspace_size(big, big, i64(1 << 20), i64(8), i64(32),
                                               ctypes.byref(n)) == 1
    assert b'overflow' in l.cflk_last_error()
    assert l.cflk_volta_mma_bwd_workspace_size(i64(1), big, i64(8), big, i64(32),
                                               ctypes.byref(n)) == 1
    f = l.cflk_volta_mma_bwd_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 12 + [ctypes.c_int64] * 5 \
        + [ctypes.c_float, ctypes.c_int]
    z = None
    assert f(z, 1, *([z] * 12), 1 << 40, 1 << 40, 1 << 20, 8, 32, 0.17, 1) == 1
    assert f(z, 1, *([z] * 12), 4096, 8, 512, 512, 32, 0.17, 1) == 1
    assert b'static scratch' in l.cflk_last_error()


def test_opm_outer_workspace_size():
    """One chunk of G2 [b][d][c][e] (16-bit), whole multiples of 128 / C rows of b, about 64 MB
    (or the whole problem when smaller); at C = 32 (the fused kernel) wT's 256 KB; refusals
    before any CUDA call."""
    l = lib()
    n = ctypes.c_size_t(0)
    i64 = ctypes.c_int64
    per_b = 512 * 64 * 32 * 2
    assert l.cflk_volta_opm_outer_workspace_size(i64(512), i64(64), i64(512), i64(32),
                                                 ctypes.byref(n)) == 0
    assert n.value == (64 << 20) // per_b // 2 * 2 * per_b
    assert l.cflk_volta_opm_outer_workspace_size(i64(3), i64(64), i64(8), i64(32),
                                                 ctypes.byref(n)) == 0
    assert n.value == 3 * 8 * 64 * 32 * 2
    # C = 32: the fused kernel, whose workspace is wT laid out chunk by chunk (F <= 128)
    assert l.cflk_volta_opm_outer_workspace_size(i64(512), i64(32), i64(512), i64(32),
                                                 ctypes.byref(n)) == 0
    assert n.value == 128 * 32 * 32 * 2
    assert l.cflk_volta_opm_outer_workspace_size(i64(3), i64(32), i64(8), i64(16),
                                                 ctypes.byref(n)) == 1


def test_resolver_capabilities():
    assert clk.supported_capabilities() == (70, 75, 100)
    for k in ('attention', 'attention_bwd', 'ln_gated_dual_proj', 'trimul_epilogue',
              'ln_projection', 'output_projection', 'transition', 'layer_norm',
              'gated_dual_proj', 'opm_update', 'opm_outer'):
        assert clk.available(100, k)
        assert clk.library_path(k, 100).endswith('sm100/libcflk_sm100.so')
    assert clk.symbol('attention', 100) == 'VoltaMma'
    assert clk.symbol('attention_bwd', 100) == 'VoltaMmaBwd'
    assert clk.symbol('transition', 100) == 'VoltaTransition'
    assert clk.c_symbol('attention', 100) == 'cflk_volta_mma'
    # the reference's own names for its families are unchanged
    assert clk.symbol('attention', 75) == 'VoltaMma'
    assert clk.symbol('attention', 70) == 'VoltaWmma'
    assert clk.symbol('transition', 70) == 'VoltaTransitionWmma'
    # every kernel has a cc=100 entry; sm_80 has none
    assert clk.available(100)
    assert not clk.available(80)
    assert clk.symbol('layer_norm', 100) == 'VoltaLayerNorm'
    assert clk.c_symbol('layer_norm', 100) == 'cflk_volta_layer_norm'
    assert clk.symbol('gated_dual_proj', 100) == 'VoltaGdp'
    assert clk.symbol('opm_update', 100) == 'VoltaOpmUpdate'
    assert clk.c_symbol('opm_update', 100) == 'cflk_volta_opm_update'
    assert clk.c_symbol('opm_outer', 100) == 'cflk_volta_opm_outer'
    with pytest.raises(KeyError):
        clk.library_path('nonexistent', 100)
    assert clk.kernel_dir(100).endswith('sm100')


def test_no_oracle_in_product_path():
    """The library and its Python binding never import or call the CPU oracle."""
    pkg = os.path.join(ROOT, 'colabfold-legacy-kernels_b200')
    for dirpath, _, files in os.walk(pkg):
        for fn in files:
            if fn.endswith(('.py', '.cu', '.cuh', '.cpp', '.h')):
                text = open(os.path.join(dirpath, fn)).read()
                assert 'oracle' not in text.replace('colabfold', ''), fn

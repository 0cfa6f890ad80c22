"""ColabFold CUDA kernels: library resolver, extended with the B200 (sm_100a) library.

Same public surface as colabfold-legacy-kernels' resolver
(src/colabfold_legacy_kernels/__init__.py:5-12,69-126): `available`, `library_path`, `symbol`,
`kernel_dir`, `supported_capabilities` and `KERNELS`, with compute capability 100 added.

For cc=100 every kernel built so far lives in one library, libcflk_sm100.so, built from this
repository's sm_100a sources. That library exports plain C-ABI entry points
(include/cflk_b200.h), not XLA FFI handlers: `c_symbol(kernel, 100)` names the entry point, and
`symbol(kernel, 100)` names the XLA FFI target that a JAX caller registers for the kernel (the
reference's own target name). The handler behind that target is a thin shim over the C entry
point, compiled against XLA's FFI headers by the caller's build; this package does not ship it,
because the headers are not part of this build's toolchain. The outer-product
mean's outer kernel (opm_outer) has no cc=100 entry yet, so `available(100)` without a kernel is
False while `available(100, 'attention')` is True once the library is built.
"""

from pathlib import Path

__all__ = [
    "KERNELS",
    "available",
    "c_symbol",
    "kernel_dir",
    "library_path",
    "supported_capabilities",
    "symbol",
]

__version__ = "0.6.0+sm100"

_KERNEL_DIR = Path(__file__).resolve().parent / "kernels"

_CAPABILITIES = (70, 75, 100)

_SM100_LIB = "libcflk_sm100.so"

# kernel -> entries (min_cc, library, XLA FFI target), highest capability first. The sm_70 and
# sm_75 libraries are the reference's own wheel's; this package ships the sm100 one.
_TABLE = {
    "attention": (
        (100, _SM100_LIB, "VoltaMma"),
        (75, "libvolta_mma.so", "VoltaMma"),
        (70, "libvolta_wmma.so", "VoltaWmma"),
    ),
    "attention_bwd": (
        (100, _SM100_LIB, "VoltaMmaBwd"),
        (75, "libvolta_mma_bwd.so", "VoltaMmaBwd"),
        (70, "libvolta_wmma_bwd.so", "VoltaWmmaBwd"),
    ),
    "layer_norm": (
        (100, _SM100_LIB, "VoltaLayerNorm"),
        (70, "libvolta_ops.so", "VoltaLayerNorm"),
    ),
    "gated_dual_proj": (
        (100, _SM100_LIB, "VoltaGdp"),
        (75, "libvolta_ops.so", "VoltaGdp"),
        (70, "libvolta_gdp_wmma.so", "VoltaGdpWmma"),
    ),
    "ln_gated_dual_proj": (
        (100, _SM100_LIB, "VoltaLnGdp"),
        (75, "libvolta_ops.so", "VoltaLnGdp"),
        (70, "libvolta_gdp_wmma.so", "VoltaLnGdpWmma"),
    ),
    "trimul_epilogue": (
        (100, _SM100_LIB, "VoltaTrimulEpilogue"),
        (75, "libvolta_ops.so", "VoltaTrimulEpilogue"),
        (70, "libvolta_gdp_wmma.so", "VoltaTrimulEpilogueWmma"),
    ),
    "ln_projection": (
        (100, _SM100_LIB, "VoltaLnProj"),
        (75, "libvolta_ops.so", "VoltaLnProj"),
        (70, "libvolta_gdp_wmma.so", "VoltaLnProjWmma"),
    ),
    "output_projection": (
        (100, _SM100_LIB, "VoltaOutProj"),
        (75, "libvolta_ops.so", "VoltaOutProj"),
        (70, "libvolta_gdp_wmma.so", "VoltaOutProjWmma"),
    ),
    "transition": (
        (100, _SM100_LIB, "VoltaTransition"),
        (75, "libvolta_ops.so", "VoltaTransition"),
        (70, "libvolta_gdp_wmma.so", "VoltaTransitionWmma"),
    ),
    "opm_update": (
        (100, _SM100_LIB, "VoltaOpmUpdate"),
        (75, "libvolta_ops.so", "VoltaOpmUpdate"),
        (70, "libvolta_gdp_wmma.so", "VoltaOpmUpdateWmma"),
    ),
    "opm_outer": (
        (100, _SM100_LIB, "VoltaOpmOuter"),
        (75, "libvolta_ops.so", "VoltaOpmOuter"),
        (70, "libvolta_gdp_wmma.so", "VoltaOpmOuterWmma"),
    ),
}

# the C-ABI entry point behind each cc=100 target
_C_SYMBOLS = {
    "VoltaMma": "cflk_volta_mma",
    "VoltaMmaBwd": "cflk_volta_mma_bwd",
    "VoltaLnGdp": "cflk_volta_ln_gdp",
    "VoltaTrimulEpilogue": "cflk_volta_trimul_epilogue",
    "VoltaLnProj": "cflk_volta_ln_proj",
    "VoltaOutProj": "cflk_volta_out_proj",
    "VoltaTransition": "cflk_volta_transition",
    "VoltaLayerNorm": "cflk_volta_layer_norm",
    "VoltaGdp": "cflk_volta_gdp",
    "VoltaOpmUpdate": "cflk_volta_opm_update",
    "VoltaOpmOuter": "cflk_volta_opm_outer",
}

KERNELS = tuple(_TABLE)


def supported_capabilities():
    """Give the compute capabilities that this package knows."""
    return _CAPABILITIES


def _resolve(kernel, cc):
    """Find the library and the FFI symbol for one kernel and one capability."""
    if kernel not in _TABLE:
        raise KeyError(
            "unknown kernel %r, expected one of %s" % (kernel, ", ".join(KERNELS)))
    cc = int(cc)
    if cc not in _CAPABILITIES:
        return cc, None, None
    for min_cc, lib, sym in _TABLE[kernel]:
        # an sm100 library serves cc 100 only; the older families serve their range up to 99
        if cc >= min_cc and (min_cc == 100) == (cc >= 100):
            return cc, lib, sym
    return cc, None, None


def kernel_dir(cc):
    """Give the directory of the libraries for one capability."""
    cc, _, _ = _resolve("attention", cc)
    return str(_KERNEL_DIR / ("sm%d" % cc))


def library_path(kernel, cc):
    """Give the path of the library that supplies one kernel."""
    cc, lib, _ = _resolve(kernel, cc)
    if lib is None:
        raise FileNotFoundError(
            "no %s kernel for compute capability %d" % (kernel, cc))
    path = _KERNEL_DIR / ("sm%d" % cc) / lib
    if not path.is_file():
        raise FileNotFoundError("%s is not in this package" % path)
    return str(path)


def symbol(kernel, cc):
    """Give the XLA FFI target name of one kernel. The sm_70/sm_75 libraries export it; for
    cc=100 it is the name an FFI shim over c_symbol(kernel, 100) registers."""
    cc, lib, sym = _resolve(kernel, cc)
    if sym is None:
        raise FileNotFoundError(
            "no %s kernel for compute capability %d" % (kernel, cc))
    return sym


def c_symbol(kernel, cc=100):
    """Give the C-ABI entry point (include/cflk_b200.h) behind a cc=100 kernel."""
    sym = symbol(kernel, cc)
    if int(cc) != 100 or sym not in _C_SYMBOLS:
        raise FileNotFoundError("no C-ABI entry for %s at compute capability %d" % (kernel, cc))
    return _C_SYMBOLS[sym]


def available(cc, kernel=None):
    """Tell if the kernels are present. With kernel=None, test all of them."""
    names = KERNELS if kernel is None else (kernel,)
    for name in names:
        try:
            library_path(name, cc)
        except (FileNotFoundError, KeyError):
            return False
    return True

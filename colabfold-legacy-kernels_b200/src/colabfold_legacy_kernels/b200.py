"""The cc=100 kernels called from PyTorch, one function per XLA FFI target of the reference.

Each function takes the target's arguments in their bound order and its attributes as keyword
arguments (cuda/volta_mma_attn.cu:594-640, cuda/volta_mma_attn_bwd.cu:455-473,
cuda/volta_fused_ffi.h:337-418), allocates the results as XLA would, runs the sm_100a kernel
through the C ABI (include/cflk_b200.h) on the current CUDA stream, and returns the results.
An InvalidArgument from the library raises ValueError with the reference's message, an Internal
error RuntimeError. 16-bit tensors may be float16 (the reference's type) or bfloat16.

There is no fallback: if libcflk_sm100.so is missing or cannot be loaded, every call raises.
"""
import ctypes

import torch

from . import library_path

_C = ctypes
_p = _C.c_void_p
_i64 = _C.c_int64
_f32 = _C.c_float
_int = _C.c_int

_SIGS = {
    'cflk_volta_mma': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f32,
                       _i64, _i64, _int],
    'cflk_volta_mma_packed': [_p, _int, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                              _i64, _i64, _i64, _f32, _i64, _i64, _int],
    'cflk_volta_mma_bwd_workspace_size': [_i64, _i64, _i64, _i64, _i64, _C.POINTER(_C.c_size_t)],
    'cflk_volta_mma_bwd': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                           _C.c_size_t, _i64, _i64, _i64, _i64, _i64, _f32, _int],
    'cflk_volta_mma_gated': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                             _i64, _i64, _f32, _int],
    'cflk_volta_mma_gated_bwd_workspace_size': [_i64, _i64, _i64, _i64, _i64,
                                                _C.POINTER(_C.c_size_t)],
    'cflk_volta_mma_gated_bwd': [_p, _int] + [_p] * 17 + [_C.c_size_t, _i64, _i64, _i64, _i64,
                                                          _i64, _f32, _int],
    'cflk_volta_ln_gdp': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                          _f32],
    'cflk_volta_trimul_epilogue': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                   _i64, _i64, _i64, _i64, _f32, _int],
    'cflk_volta_ln_proj': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                           _f32],
    'cflk_volta_out_proj': [_p, _int, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64],
    'cflk_volta_transition': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                              _f32, _int],
    'cflk_volta_layer_norm': [_p, _int, _p, _p, _p, _p, _i64, _i64, _f32],
    'cflk_volta_gdp': [_p, _int, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64],
    'cflk_volta_opm_update': [_p, _int, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32],
    'cflk_trimul_contract': [_p, _int, _p, _p, _p, _i64, _i64, _i64, _i64, _int],
    'cflk_volta_opm_outer_workspace_size': [_i64, _i64, _i64, _i64, _C.POINTER(_C.c_size_t)],
    'cflk_volta_opm_outer': [_p, _int, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p,
                             _C.c_size_t],
}

_lib = None


def lib():
    """The loaded library (raises if it is not built: there is no other implementation)."""
    global _lib
    if _lib is None:
        path = library_path('attention', 100)
        handle = _C.CDLL(path)
        handle.cflk_last_error.restype = _C.c_char_p
        handle.cflk_device_status.restype = _C.c_uint
        for name, args in _SIGS.items():
            fn = getattr(handle, name, None)
            if fn is not None:
                fn.argtypes = args
                fn.restype = _int
        _lib = handle
    return _lib


def device_status():
    """Bit codes of bounded waits that gave up since the last read (0: none); synchronises."""
    torch.cuda.synchronize()
    return int(lib().cflk_device_status())


def _check(rc, who):
    if rc == 0:
        return
    msg = lib().cflk_last_error().decode()
    if rc == 1:
        raise ValueError(msg or who + ': invalid argument')
    raise RuntimeError(msg or who + ': internal error')


def _dtype_code(*ts):
    dt = ts[0].dtype
    for t in ts:
        if t.dtype != dt:
            raise ValueError('16-bit buffers must share one dtype, got %s and %s' % (dt, t.dtype))
    if dt == torch.float16:
        return 0
    if dt == torch.bfloat16:
        return 1
    raise ValueError('16-bit buffers must be float16 or bfloat16, got %s' % dt)


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError('tensors must be on a CUDA device')
    if not t.is_contiguous():
        raise ValueError('tensors must be contiguous')
    return _C.c_void_p(t.data_ptr())


def _stream():
    return _C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _f32_ptr(t, name, who):
    if t.dtype != torch.float32:
        raise ValueError('%s: %s must be float32' % (who, name))
    return _ptr(t)


# ---- attention ----------------------------------------------------------------------------

def volta_mma(q, k, v, bias, kmask, *, scale, block_q=64, block_k=32, want_lse=True, out=None,
              lse=None):
    """VoltaMma: (out [N,H,Sq,D], lse [N,H,Sq] float32, or a one-element buffer).

    out / lse may be given, as XLA passes pre-allocated results."""
    if q.dim() != 4:
        raise ValueError('q must be [N,H,S,D]')
    N, H, Sq, D = q.shape
    Sk = k.shape[2]
    dt = _dtype_code(q, k, v, bias)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((N, H, Sq) if want_lse else (1,), dtype=torch.float32, device=q.device)
    rc = lib().cflk_volta_mma(_stream(), dt, _ptr(q), _ptr(k), _ptr(v), _ptr(bias), _ptr(kmask),
                              _ptr(out), _ptr(lse), N, H, Sq, Sk, D, float(scale), int(block_q),
                              int(block_k), int(bool(want_lse)))
    _check(rc, 'volta_mma')
    return out, lse


def volta_mma_packed(p, bias, kmask, gate_bias, lims=None, *, scale, block_q=64, block_k=32,
                     column=False, out=None):
    """VoltaMmaPacked (lims None) / VoltaMmaPackedTrim: out [X,Y,H,D]."""
    if p.dim() != 5 or p.shape[2] not in (3, 4):
        raise ValueError('p must be [X,Y,3 or 4,H,D]')
    X, Y, G, H, D = p.shape
    dt = _dtype_code(p, bias, gate_bias)
    if out is None:
        out = torch.empty((X, Y, H, D), dtype=p.dtype, device=p.device)
    if lims is not None and lims.dtype != torch.int32:
        raise ValueError('lims must be int32')
    rc = lib().cflk_volta_mma_packed(_stream(), dt, _ptr(p), _ptr(bias), _ptr(kmask),
                                     _ptr(gate_bias), _ptr(lims), _ptr(out), X, Y, G, H, D,
                                     bias.numel(), kmask.numel(), gate_bias.numel(),
                                     float(scale), int(block_q), int(block_k), int(bool(column)))
    _check(rc, 'volta_mma_packed')
    return out


def volta_mma_bwd_workspace(N, H, Sq, Sk, D):
    n = _C.c_size_t(0)
    _check(lib().cflk_volta_mma_bwd_workspace_size(N, H, Sq, Sk, D, _C.byref(n)),
           'volta_mma_bwd')
    return n.value


def volta_mma_bwd(q, k, v, bias, kmask, out, dout, lse, *, scale, want_dbias=True):
    """VoltaMmaBwd: (dq, dk, dv, dbias [H,Sq,Sk] float32)."""
    if q.dim() != 4:
        raise ValueError('q must be [N,H,S,D]')
    N, H, Sq, D = q.shape
    Sk = k.shape[2]
    if v.shape != k.shape or dout.shape != q.shape:
        raise ValueError('volta_mma_bwd: v must match k, dout must match q')
    if tuple(lse.shape) != (N, H, Sq):
        raise ValueError('volta_mma_bwd: lse must be [N,H,Sq]')
    if out.shape != q.shape:
        raise ValueError('volta_mma_bwd: out must match q')
    if tuple(bias.shape) != (H, Sq, Sk):
        raise ValueError('volta_mma_bwd: bias and dbias must be [H,Sq,Sk]')
    dt = _dtype_code(q, k, v, bias, out, dout)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dbias = torch.empty((H, Sq, Sk), dtype=torch.float32, device=q.device)
    ws_bytes = volta_mma_bwd_workspace(N, H, Sq, Sk, D)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    rc = lib().cflk_volta_mma_bwd(_stream(), dt, _ptr(q), _ptr(k), _ptr(v), _ptr(bias),
                                  _ptr(kmask), _ptr(out), _ptr(dout),
                                  _f32_ptr(lse, 'lse', 'volta_mma_bwd'), _ptr(dq), _ptr(dk),
                                  _ptr(dv), _ptr(dbias), _ptr(ws), ws_bytes, N, H, Sq, Sk, D,
                                  float(scale), int(bool(want_dbias)))
    _check(rc, 'volta_mma_bwd')
    return dq, dk, dv, dbias


def volta_mma_gated(q, k, v, gate, gate_bias, bias, kmask, *, scale, want_lse=True, out=None,
                    lse=None):
    """Gated attention: (y [N,H,Sq,D] = attention * sigmoid(gate + gate_bias[h]), lse)."""
    if q.dim() != 4 or gate.shape != q.shape:
        raise ValueError('q and gate must be [N,H,S,D]')
    N, H, Sq, D = q.shape
    Sk = k.shape[2]
    if tuple(gate_bias.shape) != (H, D):
        raise ValueError('volta_mma_gated: gate_bias must be [H,D]')
    dt = _dtype_code(q, k, v, gate, gate_bias, bias)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((N, H, Sq) if want_lse else (1,), dtype=torch.float32, device=q.device)
    rc = lib().cflk_volta_mma_gated(_stream(), dt, _ptr(q), _ptr(k), _ptr(v), _ptr(gate),
                                    _ptr(gate_bias), _ptr(bias), _ptr(kmask), _ptr(out), _ptr(lse),
                                    N, H, Sq, Sk, D, float(scale), int(bool(want_lse)))
    _check(rc, 'volta_mma_gated')
    return out, lse


def volta_mma_gated_bwd(q, k, v, gate, gate_bias, bias, kmask, y, dy, lse, *, scale,
                        want_dbias=True):
    """Gradients of volta_mma_gated: (dq, dk, dv, dgate, dgate_bias [H,D] float32,
    dbias [H,Sq,Sk] float32)."""
    if q.dim() != 4 or gate.shape != q.shape or y.shape != q.shape or dy.shape != q.shape:
        raise ValueError('volta_mma_gated_bwd: q, gate, y and dy must be [N,H,Sq,D]')
    N, H, Sq, D = q.shape
    Sk = k.shape[2]
    if v.shape != k.shape or tuple(lse.shape) != (N, H, Sq) or tuple(bias.shape) != (H, Sq, Sk):
        raise ValueError('volta_mma_gated_bwd: shapes do not match')
    if tuple(gate_bias.shape) != (H, D):
        raise ValueError('volta_mma_gated_bwd: gate_bias must be [H,D]')
    dt = _dtype_code(q, k, v, gate, gate_bias, bias, y, dy)
    dq, dk, dv, dgate = (torch.empty_like(t) for t in (q, k, v, gate))
    dgate_bias = torch.empty((H, D), dtype=torch.float32, device=q.device)
    dbias = torch.empty((H, Sq, Sk), dtype=torch.float32, device=q.device)
    n = _C.c_size_t(0)
    _check(lib().cflk_volta_mma_gated_bwd_workspace_size(N, H, Sq, Sk, D, _C.byref(n)),
           'volta_mma_gated_bwd')
    ws = torch.empty(max(n.value, 1), dtype=torch.uint8, device=q.device)
    rc = lib().cflk_volta_mma_gated_bwd(
        _stream(), dt, _ptr(q), _ptr(k), _ptr(v), _ptr(gate), _ptr(gate_bias), _ptr(bias),
        _ptr(kmask), _ptr(y), _ptr(dy), _f32_ptr(lse, 'lse', 'volta_mma_gated_bwd'), _ptr(dq),
        _ptr(dk), _ptr(dv), _ptr(dgate), _ptr(dgate_bias), _ptr(dbias), _ptr(ws), n.value, N, H,
        Sq, Sk, D, float(scale), int(bool(want_dbias)))
    _check(rc, 'volta_mma_gated_bwd')
    return dq, dk, dv, dgate, dgate_bias, dbias


# ---- fused pair-stack ops -------------------------------------------------------------------

def volta_gdp(x, wp, bp, wg, bg, mask, *, activation=0, out=None):
    """VoltaGdp: out [M,N] = mask * (x wp + bp) * act(x wg + bg); wp, wg [K,N]; activation 0
    (sigmoid) or 1 (swish)."""
    who = 'gdp'
    if x.dim() != 2:
        raise ValueError('x must be [M,K]')
    M, K = x.shape
    if wp.dim() != 2 or wp.shape[0] != K or wg.shape != wp.shape:
        raise ValueError('gdp: wp and wg must be [K,N]')
    N = wp.shape[1]
    if bp.numel() != N or bg.numel() != N or mask.numel() != M:
        raise ValueError('gdp: shapes do not match')
    dt = _dtype_code(x, wp, bp, wg, bg, mask)
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    if M == 0:
        return out
    rc = lib().cflk_volta_gdp(_stream(), dt, _ptr(x), _ptr(wp), _ptr(bp), _ptr(wg), _ptr(bg),
                              _ptr(mask), _ptr(out), M, K, N, int(activation))
    _check(rc, who)
    return out


def volta_opm_update(lhs, t, bias, norm, residual=None, *, eps, out=None):
    """VoltaOpmUpdate: out [B,D,F] = (lhs @ t[:, d, :] + bias) / (eps + norm[b, d]) (+ residual);
    lhs [B,K], t [K,D,F], bias [F] and norm [B,D] float32, residual [B,D,F] or None."""
    who = 'opm_update'
    if lhs.dim() != 2 or t.dim() != 3 or t.shape[0] != lhs.shape[1]:
        raise ValueError('opm_update: lhs must be [B,K] and t [K,D,F]')
    B, K = lhs.shape
    _, D, F = t.shape
    if K % 32 or F not in (16, 32, 64, 128) or D > 65535:
        raise ValueError(
            'opm_update: K must be a multiple of 32, F 16, 32, 64 or 128, D at most 65535')
    if (bias.numel() != F or norm.numel() != B * D or
            (residual is not None and residual.numel() != B * D * F)):
        raise ValueError('opm_update: shapes do not match')
    dt = _dtype_code(lhs, t, *(() if residual is None else (residual,)))
    if out is None:
        out = torch.empty((B, D, F), dtype=lhs.dtype, device=lhs.device)
    if out.numel() != B * D * F or out.dtype != lhs.dtype:
        raise ValueError('opm_update: shapes do not match')
    if B == 0 or D == 0:
        return out
    rc = lib().cflk_volta_opm_update(_stream(), dt, _ptr(lhs), _ptr(t),
                                     _f32_ptr(bias, 'bias', who), _f32_ptr(norm, 'norm', who),
                                     _ptr(residual), _ptr(out), B, K, D, F, float(eps))
    _check(rc, who)
    return out


def opm_outer_workspace_size(B, C, D, E=32):
    """Bytes of VoltaOpmOuter's recommended workspace (one chunk of its rounded outer products)."""
    n = _C.c_size_t(0)
    _check(lib().cflk_volta_opm_outer_workspace_size(B, C, D, E, _C.byref(n)), 'opm_outer')
    return n.value


def volta_opm_outer(left, right, wT, *, out=None, workspace=None):
    """VoltaOpmOuter on 16 MSA rows: out [B,D,F] = sum_{c,e} h(sum_a left[a,b,c] right[a,d,e])
    wT[f, c*E+e]; left [16,B,C], right [16,D,E], wT [F,C*E]. `workspace` (uint8, on the device)
    defaults to cflk_volta_opm_outer_workspace_size bytes."""
    who = 'opm_outer'
    if (left.dim() != 3 or right.dim() != 3 or wT.dim() != 2 or left.shape[0] != 16 or
            right.shape[0] != 16):
        raise ValueError('opm_outer: left must be [16,B,C], right [16,D,E], wT [F,C*E]')
    _, B, C = left.shape
    _, D, E = right.shape
    F = wT.shape[0]
    if C % 16 or E != 32 or D % 4 or D // 4 > 65535 or wT.shape[1] != C * E or \
            F not in (16, 32, 64, 128):
        raise ValueError(
            'opm_outer: C a multiple of 16, E 32, D a multiple of 4, F 16, 32, 64 or 128')
    dt = _dtype_code(left, right, wT)
    if out is None:
        out = torch.empty((B, D, F), dtype=left.dtype, device=left.device)
    if out.numel() != B * D * F or out.dtype != left.dtype:
        raise ValueError('opm_outer: shapes do not match')
    if B == 0 or D == 0 or C == 0:
        return out
    if workspace is None:
        workspace = torch.empty(max(opm_outer_workspace_size(B, C, D, E), 16), dtype=torch.uint8,
                                device=left.device)
    rc = lib().cflk_volta_opm_outer(_stream(), dt, _ptr(left), _ptr(right), _ptr(wT), _ptr(out),
                                    B, C, D, E, F, _ptr(workspace), workspace.numel())
    _check(rc, who)
    return out


def trimul_contract(a, b, *, incoming=False, out=None):
    """The triangle multiplication's contraction, float32 out [C,I,J]: outgoing
    out[c,i,j] = sum_k a[c,i,k] b[c,j,k] (a [C,I,K], b [C,J,K]); incoming
    out[c,i,j] = sum_k a[c,k,i] b[c,k,j] (a [C,K,I], b [C,K,J])."""
    who = 'trimul_contract'
    if a.dim() != 3 or b.dim() != 3 or a.shape[0] != b.shape[0]:
        raise ValueError('trimul_contract: a and b must be [C,*,*] with the same C')
    if incoming:
        C, K, I = a.shape
        if b.shape[1] != K:
            raise ValueError('trimul_contract: a [C,K,I] and b [C,K,J] must share K')
        J = b.shape[2]
    else:
        C, I, K = a.shape
        if b.shape[2] != K:
            raise ValueError('trimul_contract: a [C,I,K] and b [C,J,K] must share K')
        J = b.shape[1]
    dt = _dtype_code(a, b)
    if out is None:
        out = torch.empty((C, I, J), dtype=torch.float32, device=a.device)
    if out.dtype != torch.float32 or out.numel() != C * I * J:
        raise ValueError('trimul_contract: out must be float32 [C,I,J]')
    if C == 0 or I == 0 or J == 0:
        return out
    rc = lib().cflk_trimul_contract(_stream(), dt, _ptr(a), _ptr(b), _ptr(out), C, I, J, K,
                                    int(bool(incoming)))
    _check(rc, who)
    return out


def volta_layer_norm(x, scale, offset, *, eps, out=None):
    """VoltaLayerNorm: out [M,C] (one-pass float32 statistics). `out` may be given (and may be
    x)."""
    who = 'layer_norm'
    if x.dim() != 2:
        raise ValueError('x must be [M,C]')
    M, C = x.shape
    if scale.numel() != C or offset.numel() != C:
        raise ValueError('layer_norm: scale and offset must be [C]')
    dt = _dtype_code(x)
    if out is None:
        out = torch.empty_like(x)
    if out.shape != x.shape or out.dtype != x.dtype:
        raise ValueError('layer_norm: out must match x')
    if M == 0:
        return out
    rc = lib().cflk_volta_layer_norm(_stream(), dt, _ptr(x), _f32_ptr(scale, 'scale', who),
                                     _f32_ptr(offset, 'offset', who), _ptr(out), M, C,
                                     float(eps))
    _check(rc, who)
    return out


def _keep(keep, has_keep, M, who):
    if not has_keep:
        return None
    if keep.numel() != M:
        raise ValueError('%s: shapes do not match' % who)
    return keep


def volta_ln_gdp(x, scale, offset, wpT, bp, wgT, bg, mask, *, eps):
    """VoltaLnGdp: (left [P/2,M], right [P/2,M])."""
    if x.dim() != 2 or wpT.dim() != 2 or wpT.shape[1] != x.shape[1]:
        raise ValueError('ln_gdp: x must be [M,K] and wpT [P,K]')
    M, K = x.shape
    P = wpT.shape[0]
    if K not in (64, 128) or P % 2 or P // 2 not in (64, 128):
        raise ValueError('ln_gdp: K and P/2 must be 64 or 128')
    if (wgT.numel() != P * K or bp.numel() != P or bg.numel() != P or mask.numel() != M
            or scale.numel() != K or offset.numel() != K):
        raise ValueError('ln_gdp: shapes do not match x [M,K], wpT [P,K]')
    dt = _dtype_code(x, wpT, bp, wgT, bg, mask)
    left = torch.empty((P // 2, M), dtype=x.dtype, device=x.device)
    right = torch.empty((P // 2, M), dtype=x.dtype, device=x.device)
    if M == 0:
        return left, right
    rc = lib().cflk_volta_ln_gdp(_stream(), dt, _ptr(x), _f32_ptr(scale, 'scale', 'ln_gdp'),
                                 _f32_ptr(offset, 'offset', 'ln_gdp'), _ptr(wpT), _ptr(bp),
                                 _ptr(wgT), _ptr(bg), _ptr(mask), _ptr(left), _ptr(right), M, K, P,
                                 float(eps))
    _check(rc, 'ln_gdp')
    return left, right


def volta_trimul_epilogue(x_cm, x, in_scale, in_offset, ln_scale, ln_offset, woT, bo, wgT, bg,
                          keep, *, eps, add_input, has_keep, out=None):
    """VoltaTrimulEpilogue: out [M,O]. `out` may be given (and may be x, as XLA aliases it)."""
    who = 'trimul_epilogue'
    if (x_cm.dim() != 2 or x.dim() != 2 or woT.dim() != 2 or x.shape[0] != x_cm.shape[1]
            or woT.shape[1] != x_cm.shape[0]):
        raise ValueError('trimul_epilogue: x_cm [C,M], x [M,CA], woT [O,C]')
    C, M = x_cm.shape
    CA, O = x.shape[1], woT.shape[0]
    if C not in (64, 128) or CA not in (64, 128) or O not in (64, 128) or (add_input and O != CA):
        raise ValueError('trimul_epilogue: C, CA and O must be 64 or 128, O == CA with add_input')
    if (wgT.numel() != O * CA or bo.numel() != O or bg.numel() != O or in_scale.numel() != CA
            or in_offset.numel() != CA or ln_scale.numel() != C or ln_offset.numel() != C):
        raise ValueError('trimul_epilogue: shapes do not match')
    kp = _keep(keep, has_keep, M, who)
    dt = _dtype_code(x, woT, bo, wgT, bg, *([kp] if kp is not None else []))
    if out is None:
        out = torch.empty((M, O), dtype=x.dtype, device=x.device)
    if out.numel() != M * O:
        raise ValueError('trimul_epilogue: shapes do not match')
    if M == 0:
        return out
    rc = lib().cflk_volta_trimul_epilogue(
        _stream(), dt, _f32_ptr(x_cm, 'x_cm', who), _ptr(x), _f32_ptr(in_scale, 'in_scale', who),
        _f32_ptr(in_offset, 'in_offset', who), _f32_ptr(ln_scale, 'ln_scale', who),
        _f32_ptr(ln_offset, 'ln_offset', who), _ptr(woT), _ptr(bo), _ptr(wgT), _ptr(bg),
        _ptr(kp), _ptr(out), M, C, CA, O, float(eps), int(bool(add_input)))
    _check(rc, who)
    return out


def volta_ln_proj(x, scale, offset, wT, wbT, keep, *, eps, n, heads, has_keep):
    """VoltaLnProj: (p [M,n], bias [heads,M]); a zero n or heads gives a one-element result."""
    who = 'ln_projection'
    if x.dim() != 2:
        raise ValueError('ln_projection: x must be [M,K]')
    M, K = x.shape
    if K not in (64, 128) or n < 0 or n % 64 or heads < 0 or heads > 8:
        raise ValueError(
            'ln_projection: K must be 64 or 128, n a multiple of 64, at most 8 heads')
    if (scale.numel() != K or offset.numel() != K or (n and wT.numel() != n * K)
            or (heads and wbT.numel() != heads * K)):
        raise ValueError('ln_projection: shapes do not match')
    kp = _keep(keep, has_keep, M, who)
    dt = _dtype_code(x, *[t for t in (wT if n else None, wbT if heads else None, kp)
                          if t is not None])
    p = torch.empty((M, n) if n else (1,), dtype=x.dtype, device=x.device)
    bias = torch.empty((heads, M) if heads else (1,), dtype=x.dtype, device=x.device)
    if M == 0:
        return p, bias
    rc = lib().cflk_volta_ln_proj(_stream(), dt, _ptr(x), _f32_ptr(scale, 'scale', who),
                                  _f32_ptr(offset, 'offset', who), _ptr(wT) if n else None,
                                  _ptr(wbT) if heads else None, _ptr(kp),
                                  _ptr(p) if n else None, _ptr(bias) if heads else None, M, K, n,
                                  heads, float(eps))
    _check(rc, who)
    return p, bias


def volta_out_proj(o, wT, b, residual, keep, *, has_residual, has_keep, out=None):
    """VoltaOutProj: out [M,N]. `out` may be given (and may be the residual)."""
    who = 'output_projection'
    if o.dim() != 2 or wT.dim() != 2 or wT.shape[1] != o.shape[1]:
        raise ValueError('output_projection: o must be [M,K] and wT [N,K]')
    M, K = o.shape
    N = wT.shape[0]
    if K not in (64, 128) or N not in (64, 128):
        raise ValueError('output_projection: K and N must be 64 or 128')
    if b.numel() != N or (has_residual and residual.numel() != M * N):
        raise ValueError('output_projection: shapes do not match')
    kp = _keep(keep, has_keep, M, who)
    res = residual if has_residual else None
    dt = _dtype_code(o, wT, b, *[t for t in (res, kp) if t is not None])
    if out is None:
        out = torch.empty((M, N), dtype=o.dtype, device=o.device)
    if out.numel() != M * N:
        raise ValueError('output_projection: shapes do not match')
    if M == 0:
        return out
    rc = lib().cflk_volta_out_proj(_stream(), dt, _ptr(o), _ptr(wT), _ptr(b), _ptr(res),
                                   _ptr(kp), _ptr(out), M, K, N)
    _check(rc, who)
    return out


def volta_transition(x, scale, offset, w1T, b1, w2T, b2, keep, *, eps, add_input, has_keep,
                     out=None):
    """VoltaTransition: out [M,C]. `out` may be given (and may be x)."""
    who = 'transition'
    if x.dim() != 2 or w1T.dim() != 2 or w1T.shape[1] != x.shape[1]:
        raise ValueError('transition: x must be [M,C] and w1T [H,C]')
    M, C = x.shape
    H = w1T.shape[0]
    if C not in (64, 128, 256) or H not in (2 * C, 4 * C):
        raise ValueError('transition: C must be 64, 128 or 256, H 2C or 4C')
    if (scale.numel() != C or offset.numel() != C or b1.numel() != H or w2T.numel() != H * C
            or b2.numel() != C):
        raise ValueError('transition: shapes do not match')
    kp = _keep(keep, has_keep, M, who)
    dt = _dtype_code(x, w1T, b1, w2T, b2, *([kp] if kp is not None else []))
    if out is None:
        out = torch.empty((M, C), dtype=x.dtype, device=x.device)
    if out.numel() != M * C:
        raise ValueError('transition: shapes do not match')
    if M == 0:
        return out
    rc = lib().cflk_volta_transition(_stream(), dt, _ptr(x), _f32_ptr(scale, 'scale', who),
                                     _f32_ptr(offset, 'offset', who), _ptr(w1T), _ptr(b1),
                                     _ptr(w2T), _ptr(b2), _ptr(kp), _ptr(out), M, C, H,
                                     float(eps), int(bool(add_input)))
    _check(rc, who)
    return out

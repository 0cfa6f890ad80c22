"""cflk_volta_mma_bwd_noalloc: the backward for callers that cannot allocate device memory.

Hosts that own every device allocation, or code that must not call cudaMalloc, cannot hand the
backward a workspace; this entry point keeps its scratch in a static device array instead. The
test calls it through the C ABI twice in a row and checks each result against the workspace
entry point's, with the tolerances of the repeated-call test (dK and dV bitwise, dQ and dBias
within 1e-3, since those two arrive by atomic adds); it checks that those two calls leave both
torch's allocator and the device's free memory unchanged, and that a problem larger than the
array is refused. It lives in its own file, collected last, and passes on its own in a fresh
process as well as after the other tests.
"""
import ctypes

import pytest
import torch

from oracle.numerics import rel_max
from test_attention_fwd_gpu import b200, host, inputs, to_dev

pytestmark = pytest.mark.gpu

_SIG = [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 12 + [ctypes.c_int64] * 5 + [
    ctypes.c_float, ctypes.c_int]


def noalloc_lib():
    lib = b200().lib()
    lib.cflk_volta_mma_bwd_noalloc.argtypes = _SIG
    lib.cflk_volta_mma_bwd_noalloc.restype = ctypes.c_int
    lib.cflk_volta_mma_bwd_noalloc_max_scratch.restype = ctypes.c_size_t
    return lib


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_entry_point(cuda_device):
    m = b200()
    lib = noalloc_lib()
    n, h, s, d = 3, 4, 96, 32
    q, k, v, bias, km, dout = inputs(n, h, s, s, d, 0, 'bf16')
    tq, tk, tv, tb, td = (to_dev(x, 'bf16', cuda_device) for x in (q, k, v, bias, dout))
    kmask = torch.tensor(km, device=cuda_device)
    scale = d ** -0.5
    out, lse = m.volta_mma(tq, tk, tv, tb, kmask, scale=scale)
    want = m.volta_mma_bwd(tq, tk, tv, tb, kmask, out, td, lse, scale=scale)
    outs = [(torch.empty_like(tq), torch.empty_like(tk), torch.empty_like(tv),
             torch.full((h, s, s), 7.0, device=cuda_device)) for _ in range(3)]

    def call(dq, dk, dv, dbias):
        rc = lib.cflk_volta_mma_bwd_noalloc(m._stream(), 1, P(tq), P(tk), P(tv), P(tb), P(kmask),
                                            P(out), P(td), P(lse), P(dq), P(dk), P(dv), P(dbias),
                                            n, h, s, s, d, scale, 1)
        assert rc == 0, lib.cflk_last_error()

    # one call first, so that loading the library's kernels (which the driver may do lazily, on
    # first use) is not counted; then the two checked calls must not change either figure
    call(*outs[0])
    torch.cuda.synchronize()
    torch_bytes = torch.cuda.memory_allocated(cuda_device)
    free_bytes = torch.cuda.mem_get_info(cuda_device)[0]
    for dq, dk, dv, dbias in outs[1:]:
        call(dq, dk, dv, dbias)
        torch.cuda.synchronize()
        assert m.device_status() == 0
        assert torch.cuda.memory_allocated(cuda_device) == torch_bytes
        assert torch.cuda.mem_get_info(cuda_device)[0] == free_bytes
        assert torch.equal(dk, want[1]) and torch.equal(dv, want[2])
        assert rel_max(host(dq), host(want[0])) < 1e-3
        assert rel_max(host(dbias), host(want[3])) < 1e-3


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    m = b200()
    lib = noalloc_lib()
    cap = lib.cflk_volta_mma_bwd_noalloc_max_scratch()
    assert cap == 32 << 20
    z = ctypes.c_void_p(0)
    # 4*N*H*Sq*(D+2) bytes alone: 4 * 4096 * 8 * 512 * 34 is far beyond 32 MiB; nothing is
    # launched
    rc = lib.cflk_volta_mma_bwd_noalloc(m._stream(), 1, *([z] * 12), 4096, 8, 512, 512, 32,
                                        0.17, 1)
    assert rc == 1
    assert b'static scratch' in lib.cflk_last_error()

"""Two building blocks of the kernels checked on their own, through the diagnostic entry points.

* The FMA-pipe exponential that the attention softmax uses for part of its exponentials
  (ex2_fma: rint range reduction and a cubic for 2^f on [-1/2, 1/2]) against exp2 in float64,
  over the inputs the kernels give it: [-125, 8] (below -125 it clamps to 2^-125, which stands in
  for 0). Bound: relative error 1e-4, under the 16-bit rounding of P (bf16: 3.9e-3, f16: 4.9e-4).
* The bounded mbarrier wait that every pipeline wait of the library uses: a CTA waits on a
  barrier nobody arrives on; after the limit it records status bit 4 and the kernel returns. No
  GPU is hung or faulted: the wait ends by its own limit.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def lib():
    from colabfold_legacy_kernels import b200
    l = b200.lib()
    l.cflk_diag_ex2_fma.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64]
    l.cflk_diag_ex2_fma.restype = ctypes.c_int
    l.cflk_diag_bounded_wait.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p,
                                         ctypes.c_void_p]
    l.cflk_diag_bounded_wait.restype = ctypes.c_int
    return b200, l


def test_ex2_fma_error_bound(cuda_device):
    b200, l = lib()
    x = torch.linspace(-125.0, 8.0, 1 << 20, device=cuda_device)
    x = torch.cat([x, torch.tensor([-0.5, 0.5, -0.4999, 0.4999, 0.0, 1.0, -1.0, 7.5],
                                   device=cuda_device)])
    fma_out, mufu_out = torch.empty_like(x), torch.empty_like(x)
    rc = l.cflk_diag_ex2_fma(b200._stream(), x.data_ptr(), fma_out.data_ptr(),
                             mufu_out.data_ptr(), x.numel())
    assert rc == 0
    torch.cuda.synchronize()
    xs = x.cpu().numpy().astype(np.float64)
    want = np.exp2(xs)
    got = fma_out.cpu().numpy().astype(np.float64)
    rel = np.abs(got - want) / want
    assert np.isfinite(got).all()
    assert rel.max() < 1e-4, rel.max()
    hw = mufu_out.cpu().numpy().astype(np.float64)
    assert (np.abs(hw - want) / want).max() < 1e-5


def test_ex2_fma_clamps_below_minus_125(cuda_device):
    b200, l = lib()
    x = torch.tensor([-126.0, -200.0, -1e4, -float('inf')], device=cuda_device)
    fma_out, mufu_out = torch.empty_like(x), torch.empty_like(x)
    assert l.cflk_diag_ex2_fma(b200._stream(), x.data_ptr(), fma_out.data_ptr(),
                               mufu_out.data_ptr(), x.numel()) == 0
    torch.cuda.synchronize()
    got = fma_out.cpu().numpy().astype(np.float64)
    assert np.allclose(got, 2.0 ** -125, rtol=1e-4)


@pytest.mark.parametrize('limit_ms', [20, 200])
def test_bounded_wait_runs_out_and_reports(limit_ms, cuda_device):
    b200, l = lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    elapsed = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    rc = l.cflk_diag_bounded_wait(b200._stream(), limit_ms * 1000000, status.data_ptr(),
                                  elapsed.data_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 4       # the wait gave up, and nothing arrived
    ns = int(elapsed.item())
    assert limit_ms * 1e6 <= ns < limit_ms * 1e6 + 5e8
    # the context is still usable
    assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0
    assert b200.device_status() == 0     # the library's own status words are untouched


def test_bounded_wait_refuses_limits_beyond_two_seconds(cuda_device):
    b200, l = lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = l.cflk_diag_bounded_wait(b200._stream(), 3 * 10 ** 9, status.data_ptr(),
                                  status.data_ptr())
    assert rc == 1

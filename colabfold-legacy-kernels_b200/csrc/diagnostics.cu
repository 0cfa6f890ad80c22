// Diagnostic entry points: no counterpart in the reference. They expose two building blocks of
// the kernels so that tests can check them on their own:
//
//   * cflk_diag_ex2_fma evaluates the FMA-pipe exponential (ex2_fma, sm100.cuh) that the
//     attention kernels use for part of their softmax, next to the hardware ex2.approx, so that
//     its error can be measured against exp2 over the inputs the kernels give it;
//   * cflk_diag_bounded_wait runs one CTA that waits on an mbarrier nobody arrives on, with a
//     caller-chosen limit: the wait gives up after the limit, records its code in a status word
//     and the kernel returns. This is the mechanism that keeps every pipeline wait of the library
//     from hanging a GPU; the test shows that it ends and reports.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "capi_internal.h"
#include "cflk_b200.h"
#include "sm100.cuh"

namespace cflk {
namespace {

__global__ void ex2_fma_kernel(const float* __restrict__ x, float* __restrict__ fma_out,
                               float* __restrict__ mufu_out, long long n) {
    for (long long i = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < n;
         i += 2ll * gridDim.x * blockDim.x) {
        const float a0 = x[i], a1 = i + 1 < n ? x[i + 1] : 0.f;
        const float2 e = ex2_fma(a0, a1);
        fma_out[i] = e.x;
        mufu_out[i] = ex2(a0);
        if (i + 1 < n) {
            fma_out[i + 1] = e.y;
            mufu_out[i + 1] = ex2(a1);
        }
    }
}

// One thread initialises an mbarrier that expects one arrival and waits on it for limit_ns.
// Nothing arrives, so the wait runs out: status[0] gets kStatusSyncWait, status[1] the elapsed
// nanoseconds (so the test can see that the limit, not a hang or an early exit, ended it).
__global__ void bounded_wait_kernel(unsigned long long limit_ns, unsigned* status,
                                    unsigned long long* elapsed) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long t0 = globaltimer();
        const bool ok = mbar_wait(&bar, 0, status, kStatusSyncWait, &abort_flag, limit_ns);
        *elapsed = globaltimer() - t0;
        if (ok) {
            atomicOr(status, 0x80000000u);  // cannot happen: nothing arrived
        }
    }
}

}  // namespace
}  // namespace cflk

using namespace cflk;

extern "C" int cflk_diag_ex2_fma(void* stream, const float* x, float* fma_out, float* mufu_out,
                                 int64_t n) {
    clear_error();
    if (n < 0 || (n > 0 && (x == nullptr || fma_out == nullptr || mufu_out == nullptr))) {
        return fail(kInvalidArgument, "diag_ex2_fma: bad arguments");
    }
    if (n == 0) {
        return kOk;
    }
    const long long pairs = (n + 1) / 2;
    const unsigned blocks = (unsigned)std::min<long long>((pairs + 255) / 256, 148 * 8);
    ex2_fma_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, fma_out, mufu_out, n);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess
               ? kOk
               : fail(kInternal, std::string("diag_ex2_fma launch: ") + cudaGetErrorString(e));
}

extern "C" int cflk_diag_bounded_wait(void* stream, uint64_t limit_ns, unsigned* status,
                                      unsigned long long* elapsed_ns) {
    clear_error();
    if (status == nullptr || elapsed_ns == nullptr || limit_ns == 0 ||
        limit_ns > kWaitLimitNs) {
        return fail(kInvalidArgument, "diag_bounded_wait: limit must be in (0, 2 s]");
    }
    bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, status,
                                                                         elapsed_ns);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess
               ? kOk
               : fail(kInternal, std::string("diag_bounded_wait launch: ") + cudaGetErrorString(e));
}

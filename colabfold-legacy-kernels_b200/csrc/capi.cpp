// Error reporting and status of the C-ABI (include/cflk_b200.h).
#include <cuda_runtime.h>

#include <string>

#include "capi_internal.h"
#include "cflk_b200.h"

namespace cflk {

namespace {
thread_local std::string t_last_error;
}

// translation units that are not linked in report a clear status
__attribute__((weak)) unsigned read_and_clear_status_bwd() {
    return 0;
}
__attribute__((weak)) unsigned read_and_clear_status_fused() {
    return 0;
}
__attribute__((weak)) unsigned read_and_clear_status_gemm() {
    return 0;
}
__attribute__((weak)) unsigned read_and_clear_status_opm() {
    return 0;
}

int fail(int code, const std::string& msg) {
    t_last_error = msg;
    return code;
}

void clear_error() {
    t_last_error.clear();
}

}  // namespace cflk

extern "C" const char* cflk_last_error(void) {
    return cflk::t_last_error.c_str();
}

extern "C" int cflk_version(void) {
    return 100;  // compute capability the library is built for
}

extern "C" unsigned cflk_device_status(void) {
    return cflk::read_and_clear_status_fwd() | cflk::read_and_clear_status_bwd() |
           cflk::read_and_clear_status_fused() | cflk::read_and_clear_status_gemm() |
           cflk::read_and_clear_status_opm();
}

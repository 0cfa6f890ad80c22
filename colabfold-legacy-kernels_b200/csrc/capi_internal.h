// Status codes, dtype codes and the last-error message shared by the C-ABI entry points.
#pragma once

#include <cstdint>
#include <string>

namespace cflk {

// return codes of every entry point (the XLA FFI handler maps them to ffi::Error kinds)
enum Status : int { kOk = 0, kInvalidArgument = 1, kInternal = 2 };
// element type of the 16-bit buffers
enum DType : int { kF16 = 0, kBF16 = 1 };

constexpr int kMaxDevices = 64;

// record msg as this thread's last error and return code
int fail(int code, const std::string& msg);
void clear_error();

// each translation unit's device status word (bounded waits that gave up), read and cleared
unsigned read_and_clear_status_fwd();
unsigned read_and_clear_status_bwd();
unsigned read_and_clear_status_fused();
unsigned read_and_clear_status_gemm();
unsigned read_and_clear_status_opm();

// VoltaOpmOuter fused at C = E = 32 (the caller has validated the sizes); the workspace holds
// wT laid out chunk by chunk (F * 2 KB)
int opm_outer_fused(void* stream, int dtype, const void* left, const void* right, const void* wT,
                    void* out, int64_t B, int64_t D, int64_t F, void* workspace,
                    size_t ws_bytes);

// VoltaGdp through the tile GEMM (widths the resident-weight row-tile kernel does not take)
int gdp_general(void* stream, int dtype, const void* x, const void* wp, const void* bp,
                const void* wg, const void* bg, const void* mask, void* out, int64_t M,
                int64_t K, int64_t N, int64_t activation);

}  // namespace cflk

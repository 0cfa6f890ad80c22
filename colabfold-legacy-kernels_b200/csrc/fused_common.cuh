// The persistent row-tile pipeline shared by the LayerNorm-folded pair-stack fusions.
//
// A CTA walks 128-row tiles of the input (tile = blockIdx.x, + gridDim.x, ...). Warp 8 is the
// producer: lane 0 loads the op's weights once (TMA, resident in shared memory for the whole
// CTA), streams x tiles two stages deep (one where a stage is large), and issues the tcgen05
// MMAs of each tile into tensor memory. Warps 0-7 are two warpgroups of workers; worker (g, t)
// owns row t of the tile (TMEM lane t) and either half g of its columns or, for ops that run
// the warpgroups ping-pong, the whole row of every other tile: it runs the op's prologue
// (LayerNorm in place on the swizzled tile) and epilogue (accumulators from TMEM, bias,
// gating, residual, stores).
//
// Row tiles follow the reference's keep rule (tile_work, colabfold-legacy-kernels
// cuda/volta_gdp.h:114-136): a tile is computed when a row's keep is above zero, written as
// padding when all are zero, and left alone when all are below zero; rows past M count as the
// op's `other`. Every warp classifies a tile itself, so producer and workers agree on which
// tiles enter the pipeline without talking to each other.
#pragma once

#include "sm100.cuh"

namespace cflk {
namespace fused {

constexpr int BM = 128;            // rows per tile = TMEM lanes
constexpr int kWorkers = 256;      // two warpgroups
constexpr int kThreads = kWorkers + 32;
constexpr int kProducerWarp = 8;
constexpr int ATOM = BM * 128;     // one 64-column, 128-byte-swizzled atom of a 128-row tile

enum Work : int { kCompute = 0, kPadding = 1, kSkip = 2 };

// Byte offset of element (row r, column c) in a K-major tile of 128 rows stored as 64-column
// atoms with the 128-byte swizzle (TMA's and the MMA's layout); c a multiple of 8 gives a
// 16-byte chunk.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)((c >> 6) * ATOM + r * 128 + ((((c >> 3) & 7) ^ (r & 7)) << 4) + (c & 7) * 2);
}

// The same for a weight matrix [rows][K] staged as 64-column atoms of `rows` rows each.
__device__ __forceinline__ uint32_t sw128_rows(int rows, int r, int c) {
    return (uint32_t)((c >> 6) * rows * 128 + r * 128 + ((((c >> 3) & 7) ^ (r & 7)) << 4) +
                      (c & 7) * 2);
}

// keep classification of rows [m0, m0 + BM), by one whole warp (every lane gets the result)
template <typename T>
__device__ __forceinline__ int tile_work(const T* keep, int M, int m0, float other) {
    if (keep == nullptr) {
        return kCompute;
    }
    const int lane = threadIdx.x & 31;
    bool live = false, zero = false;
#pragma unroll
    for (int i = 0; i < BM / 32; ++i) {
        const int r = m0 + lane + 32 * i;
        const float k = r < M ? Elem<T>::to_f(keep[r]) : other;
        live |= k > 0.f;
        zero |= k == 0.f;
    }
    if (__any_sync(0xffffffffu, live)) {
        return kCompute;
    }
    return __any_sync(0xffffffffu, zero) ? kPadding : kSkip;
}

// The keep values of rows m0 + lane + 32i (i < 4) for tile_work_of, loaded by volatile
// instructions so that the compiler keeps them where they are written (ahead of the waits that
// follow), which lets a worker load the next tile's values a whole tile early.
template <typename T>
__device__ __forceinline__ void keep_load(const T* keep, int M, int m0, float other,
                                          float (&v)[BM / 32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < BM / 32; ++i) {
        const int r = m0 + lane + 32 * i;
        unsigned short bits = 0;
        if (keep != nullptr && r < M) {
            asm volatile("ld.global.nc.u16 %0, [%1];"
                         : "=h"(bits)
                         : "l"(reinterpret_cast<const unsigned short*>(keep) + r));
            v[i] = Elem<T>::to_f(*reinterpret_cast<const T*>(&bits));
        } else {
            v[i] = keep == nullptr ? 1.f : other;
        }
    }
}

// tile_work from values keep_load fetched (the same rule)
__device__ __forceinline__ int tile_work_of(const float (&v)[BM / 32]) {
    bool live = false, zero = false;
#pragma unroll
    for (int i = 0; i < BM / 32; ++i) {
        live |= v[i] > 0.f;
        zero |= v[i] == 0.f;
    }
    if (__any_sync(0xffffffffu, live)) {
        return kCompute;
    }
    return __any_sync(0xffffffffu, zero) ? kPadding : kSkip;
}

// One 32-byte store (sm_100's 256-bit vector store): half the store instructions, and half the
// separate segments a warp's row-strided stores put through the memory pipeline
__device__ __forceinline__ void st_global_v8(void* p, const uint4& lo, const uint4& hi) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(lo.x),
                 "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
                 : "memory");
}

// Output tiles leave through TMA stores (shared memory to L2, no pass through L1): a worker warp
// writes its 32 rows' chunk into a staging buffer, fences it for the async proxy, and lane 0
// stores the box and commits it as one bulk group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0,
                                             int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            map),
        "r"(src), "r"(c0), "r"(c1)
        : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// until at most N of this thread's committed bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_reads() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// until every bulk group this thread committed has completed (writes included)
__device__ __forceinline__ void bulk_wait_done() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// 16-byte shared-memory store
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

// Per-warp staging of 32 rows x 64 bytes (32 columns of 16-bit values) for a TMA box {32, 32}
// with the 64-byte swizzle, in NB buffers of 2 KB: row r's 16-byte quarter k sits at
// 64r + 16(k ^ bits 1-2 of r), which keeps a quarter-warp's eight 16-byte stores on distinct
// banks. With NB = 1 the buffer is reused once the previous store has read it.
template <int NB>
struct RowChunkStager {
    static constexpr int BYTES = NB * 2048;
    uint32_t base;  // shared address of the warp's NB 2 KB buffers, 1024-byte aligned
    int n;          // chunks issued so far

    // the next buffer, once the store that last used it has read it (whole warp)
    __device__ __forceinline__ uint32_t acquire(int lane) {
        const uint32_t b = base + (NB == 1 ? 0 : (n % NB) * 2048);
        if (n >= NB) {
            if (lane == 0) {
                bulk_wait_reads<NB - 1>();
            }
            __syncwarp();
        }
        return b;
    }
    // lane's row, 16-byte quarter k (columns 8k .. 8k + 7) of buffer b
    __device__ __forceinline__ void write(uint32_t b, int lane, int k, uint32_t w0, uint32_t w1,
                                          uint32_t w2, uint32_t w3) {
        st_shared_v4(b + 64 * lane + 16 * (k ^ ((lane >> 1) & 3)), w0, w1, w2, w3);
    }
    // buffer b (every lane's four quarters written) as one box store of rows [row0, row0 + 32),
    // columns [col0, col0 + 32) of map; TMA clips rows and columns past the map (whole warp)
    __device__ __forceinline__ void issue(const CUtensorMap* map, uint32_t b, int lane, int col0,
                                          int row0) {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(map, b, col0, row0);
        }
        ++n;
    }
    // lane's row: 16 packed pairs (32 columns) through the next buffer
    __device__ __forceinline__ void put(const CUtensorMap* map, int lane, const uint32_t (&w)[16],
                                        int col0, int row0) {
        const uint32_t b = acquire(lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            write(b, lane, k, w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        }
        issue(map, b, lane, col0, row0);
    }
    __device__ __forceinline__ void finish(int lane) {
        if (lane == 0) {
            bulk_wait_done();
        }
        __syncwarp();
    }
};

// Barrier among the 256 workers (id 1).
__device__ __forceinline__ void workers_sync() {
    named_sync(1, kWorkers);
}

// K-major operand descriptor for the 128-byte-swizzled layout: 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_k128(uint32_t saddr) {
    return smem_desc(saddr, 16, 1024, kSwizzle128B);
}

// LayerNorm of row t in place on a swizzled tile: worker half g holds columns
// [g*K/2, (g+1)*K/2). Two-pass float32 statistics exchanged through red[2][2][BM]; the result
// is rounded to T, as the reference rounds LN(x) before its GEMM. raw (optional) receives the
// half row as it was, packed 2 per word.
template <typename T, int K>
__device__ __forceinline__ void ln_rows_half(uint8_t* tile, int t, int g, const float* scale,
                                             const float* offset, float eps, float* red,
                                             uint32_t* raw, float* y_out) {
    using E = Elem<T>;
    constexpr int KH = K / 2;
    float v[KH];
#pragma unroll
    for (int ch = 0; ch < KH / 8; ++ch) {
        const uint4 w = *reinterpret_cast<const uint4*>(tile + sw128(t, g * KH + 8 * ch));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (raw != nullptr) {
                raw[4 * ch + e] = ww[e];
            }
            const float2 f = E::unpack(ww[e]);
            v[8 * ch + 2 * e] = f.x;
            v[8 * ch + 2 * e + 1] = f.y;
        }
    }
    // sums in four paired partial accumulators (short dependency chains)
    uint64_t acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[i] = pk2(v[2 * i], v[2 * i + 1]);
    }
#pragma unroll
    for (int i = 8; i < KH; i += 2) {
        acc[(i >> 1) & 3] = add2(acc[(i >> 1) & 3], pk2(v[i], v[i + 1]));
    }
    float2 sp2 = upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])));
    red[(0 * 2 + g) * BM + t] = sp2.x + sp2.y;
    workers_sync();
    const float mean = (red[0 * BM + t] + red[1 * BM + t]) * (1.f / K);
    const uint64_t nm2 = pk2(-mean, -mean);
#pragma unroll
    for (int i = 0; i < KH; i += 2) {
        const float2 d = upk2(add2(pk2(v[i], v[i + 1]), nm2));
        v[i] = d.x;
        v[i + 1] = d.y;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint64_t d = pk2(v[2 * i], v[2 * i + 1]);
        acc[i] = mul2(d, d);
    }
#pragma unroll
    for (int i = 8; i < KH; i += 2) {
        const uint64_t d = pk2(v[i], v[i + 1]);
        acc[(i >> 1) & 3] = fma2(d, d, acc[(i >> 1) & 3]);
    }
    sp2 = upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])));
    red[(2 + g) * BM + t] = sp2.x + sp2.y;
    workers_sync();
    const float rstd = rsqrtf((red[2 * BM + t] + red[3 * BM + t]) * (1.f / K) + eps);
    const uint64_t r2 = pk2(rstd, rstd);
#pragma unroll
    for (int ch = 0; ch < KH / 8; ++ch) {
        const int c0 = g * KH + 8 * ch;
        // this 8-column chunk's scale and offset, 16-byte loads (broadcast across the warp)
        const float4 s0 = *reinterpret_cast<const float4*>(scale + c0);
        const float4 s1 = *reinterpret_cast<const float4*>(scale + c0 + 4);
        const float4 o0 = *reinterpret_cast<const float4*>(offset + c0);
        const float4 o1 = *reinterpret_cast<const float4*>(offset + c0 + 4);
        const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float of[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = 8 * ch + 2 * e;
            const uint64_t y = fma2(mul2(pk2(v[i], v[i + 1]), r2),
                                    pk2(sc[2 * e], sc[2 * e + 1]), pk2(of[2 * e], of[2 * e + 1]));
            const float2 yf = upk2(y);
            w[e] = E::pack(yf.x, yf.y);
            if (y_out != nullptr) {
                const float2 r = E::unpack(w[e]);
                y_out[i] = r.x;
                y_out[i + 1] = r.y;
            }
        }
        *reinterpret_cast<uint4*>(tile + sw128(t, c0)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// LayerNorm of row t in place on a swizzled tile, the whole row by one thread, with the row
// held in registers (K <= 128: one pass of 16-byte reads, the centred second moment from the
// registers, then the normalised row rounded to T written back): a third of ln_row_full's
// shared-memory reads, the same arithmetic.
template <typename T, int K>
__device__ __forceinline__ void ln_row_regs(uint8_t* tile, int t, const float* scale,
                                            const float* offset, float eps) {
    static_assert(K <= 128, "row in registers");
    using E = Elem<T>;
    uint4 w[K / 8];
#pragma unroll
    for (int ch = 0; ch < K / 8; ++ch) {
        w[ch] = *reinterpret_cast<const uint4*>(tile + sw128(t, 8 * ch));
    }
    uint64_t acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[i] = pk2(0.f, 0.f);
    }
#pragma unroll
    for (int ch = 0; ch < K / 8; ++ch) {
        const uint32_t ww[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(ww[e]);
            acc[e] = add2(acc[e], pk2(f.x, f.y));
        }
    }
    float2 r = upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])));
    const float mean = (r.x + r.y) * (1.f / K);
    const uint64_t nm2 = pk2(-mean, -mean);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[i] = pk2(0.f, 0.f);
    }
#pragma unroll
    for (int ch = 0; ch < K / 8; ++ch) {
        const uint32_t ww[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(ww[e]);
            const uint64_t d = add2(pk2(f.x, f.y), nm2);
            acc[e] = fma2(d, d, acc[e]);
        }
    }
    r = upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])));
    const float rstd = rsqrtf((r.x + r.y) * (1.f / K) + eps);
    const uint64_t r2 = pk2(rstd, rstd);
#pragma unroll
    for (int ch = 0; ch < K / 8; ++ch) {
        const uint32_t ww[4] = {w[ch].x, w[ch].y, w[ch].z, w[ch].w};
        const float4 s0 = *reinterpret_cast<const float4*>(scale + 8 * ch);
        const float4 s1 = *reinterpret_cast<const float4*>(scale + 8 * ch + 4);
        const float4 o0 = *reinterpret_cast<const float4*>(offset + 8 * ch);
        const float4 o1 = *reinterpret_cast<const float4*>(offset + 8 * ch + 4);
        const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float of[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(ww[e]);
            const float2 yf = upk2(fma2(mul2(add2(pk2(f.x, f.y), nm2), r2),
                                        pk2(sc[2 * e], sc[2 * e + 1]),
                                        pk2(of[2 * e], of[2 * e + 1])));
            o[e] = E::pack(yf.x, yf.y);
        }
        *reinterpret_cast<uint4*>(tile + sw128(t, 8 * ch)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// LayerNorm of row t in place on a swizzled tile, the whole row by one thread (no exchange, no
// barrier): three passes over the row in shared memory (sum, centred sum of squares, then the
// normalised row rounded to T and written back), so the row never sits in registers.
template <typename T, int K>
__device__ __forceinline__ void ln_row_full(uint8_t* tile, int t, const float* scale,
                                            const float* offset, float eps) {
    using E = Elem<T>;
    uint64_t acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[i] = pk2(0.f, 0.f);
    }
#pragma unroll 4
    for (int ch = 0; ch < K / 8; ++ch) {
        const uint4 w = *reinterpret_cast<const uint4*>(tile + sw128(t, 8 * ch));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(ww[e]);
            acc[e] = add2(acc[e], pk2(f.x, f.y));
        }
    }
    float2 r = upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])));
    const float mean = (r.x + r.y) * (1.f / K);
    const uint64_t nm2 = pk2(-mean, -mean);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[i] = pk2(0.f, 0.f);
    }
#pragma unroll 4
    for (int ch = 0; ch < K / 8; ++ch) {
        const uint4 w = *reinterpret_cast<const uint4*>(tile + sw128(t, 8 * ch));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(ww[e]);
            const uint64_t d = add2(pk2(f.x, f.y), nm2);
            acc[e] = fma2(d, d, acc[e]);
        }
    }
    r = upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])));
    const float rstd = rsqrtf((r.x + r.y) * (1.f / K) + eps);
    const uint64_t r2 = pk2(rstd, rstd);
#pragma unroll 4
    for (int ch = 0; ch < K / 8; ++ch) {
        uint8_t* p = tile + sw128(t, 8 * ch);
        const uint4 w = *reinterpret_cast<const uint4*>(p);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        const float4 s0 = *reinterpret_cast<const float4*>(scale + 8 * ch);
        const float4 s1 = *reinterpret_cast<const float4*>(scale + 8 * ch + 4);
        const float4 o0 = *reinterpret_cast<const float4*>(offset + 8 * ch);
        const float4 o1 = *reinterpret_cast<const float4*>(offset + 8 * ch + 4);
        const float sc[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const float of[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = E::unpack(ww[e]);
            const uint64_t y = fma2(mul2(add2(pk2(f.x, f.y), nm2), r2),
                                    pk2(sc[2 * e], sc[2 * e + 1]), pk2(of[2 * e], of[2 * e + 1]));
            const float2 yf = upk2(y);
            o[e] = E::pack(yf.x, yf.y);
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// sigmoid(g) = (1 + tanh(g/2)) / 2: one MUFU operation (tanh.approx, relative error ~2^-11)
// instead of an exponential and a reciprocal
__device__ __forceinline__ float sigmoid_fast(float g) {
    float th;
    asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(0.5f * g));
    return fmaf(0.5f, th, 0.5f);
}

}  // namespace fused
}  // namespace cflk

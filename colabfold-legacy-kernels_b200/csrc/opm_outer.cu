// VoltaOpmOuter fused for AF2's widths (C = E = 32) on sm_100a: out [B,D,F] = sum over c, e of
// h(sum_a left[a,b,c] right[a,d,e]) wT[f, 32 c + e] on 16 MSA rows a, h the rounding to the 16-bit
// type (colabfold-legacy-kernels cuda/volta_fused_ffi.h:300-335, kernel cuda/volta_ops.cu:710-787).
//
// A CTA tile is 16 b x 16 d (256 output rows (b, d)) and all F columns. Its K = C E = 1024 runs in
// 16 chunks of 8 c x 8 e, and each chunk chains two tensor-core products through tensor memory
// and shared memory, so the rounded outer products never leave the SM:
//   * first product, one tcgen05.mma (M = 128, N = 128, K = 16): rows (b, c) of left for the
//     tile's 16 b and the chunk's 8 c, columns (d, e) of right for the tile's 16 d and the chunk's
//     8 e, both MN-major in the unswizzled (interleaved) layout: TMA boxes [16 b][16 a][8 c] and
//     [16 d][16 a][8 e] whose 128-byte core matrices are 8 rows a of one b (or d); the result
//     G[b, c, d, e] lands in one of two 128-column TMEM buffers;
//   * two converter warpgroups (thread = lane = (b, c), one warpgroup a half of the d) read
//     8 d x 8 e each, round them to the 16-bit type and write them as rows (b, d) of a K-major
//     [256 rows][8 c x 8 e] tile (the second product's A operand, two of them in shared memory);
//   * second product: two M = 128 MMAs (b 0-7 and b 8-15) of that tile against the chunk's
//     slice of wT, accumulating out [256 rows][F] in TMEM over the 16 chunks; the slices are
//     first laid out chunk by chunk ([16 chunks][F][8 c x 8 e], in the workspace) so that each
//     arrives as one K-major 128-byte-swizzled box;
//   * an epilogue warpgroup rounds the accumulators and writes each 128-row half with TMA
//     stores of [8 b][16 d][64 f] boxes (rows and columns past B, D, F clip).
// Warp 0 streams the tile's left/right blocks (one tile ahead) and the wT slices (a ring of
// three); warp 1 issues every MMA, the first product two chunks ahead of the second.
// All waits are bounded; a wait that gives up ends the loads and the MMAs, and the drains at the
// end leave no copy or MMA in flight.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "capi_internal.h"
#include "cflk_b200.h"
#include "sm100.cuh"
#include "tmap.h"

namespace cflk {
namespace {

__device__ unsigned g_status;

constexpr int kTB = 16, kTD = 16;          // b and d of a tile
constexpr int kChunks = (32 / 8) * (32 / 8);  // 8 c x 8 e chunks of K = 1024
// warp 0 TMA, warp 1 MMA, warps 2-9 two converter warpgroups (d 0-7 and d 8-15 of a chunk),
// warps 10-13 the epilogue; a warp reaches TMEM lanes 32 (warp % 4) ..
constexpr int kThreads = 448;
constexpr int kConvWarp0 = 2, kEpiWarp0 = 10;
constexpr unsigned long long kDrain = 200000000ull;

// Every TMA box below has 16-byte rows and no swizzle (a swizzled box wants rows as wide as the
// swizzle span); the MMA reads them in the interleaved layout of 8-row x 16-byte core matrices.
constexpr int kBox = 16 * 16 * 8 * 2;      // one [16 b or d][16 a][8 c or e] box: 4 KB
constexpr int A1_BYTES = 4 * kBox;         // left: 4 c-blocks
constexpr int AB_BYTES = 8 * kBox;         // left then right (4 e-blocks)
constexpr int W_BYTES = 128 * 128;         // [128 f][8 c x 8 e], 128-byte swizzle
constexpr int kWStages = 3;
constexpr int G_BYTES = 2 * 128 * 128;     // two 128-row halves of [rows][128 bytes]
constexpr int OUT_BOX = 128 * 128;         // [8 b][16 d][64 f]
constexpr int SM_AB = 0;
constexpr int SM_W = SM_AB + 2 * AB_BYTES;
constexpr int SM_G = SM_W + kWStages * W_BYTES;
constexpr int SM_OUT = SM_G + 2 * G_BYTES;
constexpr int SMEM = SM_OUT + 2 * OUT_BOX + 1024;
static_assert(SMEM <= 227 * 1024, "shared memory");
// tensor memory: the second product's two halves (128 columns each), then the first product's
// two buffers
constexpr uint32_t T_ACC = 0, T_S1 = 256, kAlloc = 512;

struct OuterArgs {
    int B, D, F;
};

__device__ __forceinline__ void tma_store_3d_out(const CUtensorMap* map, uint32_t src, int c0,
                                                 int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::
            "l"(map),
        "r"(src), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_done_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    opm_outer_kernel(const __grid_constant__ CUtensorMap tl, const __grid_constant__ CUtensorMap tr,
                     const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap to,
                     const OuterArgs a) {
    using E = Elem<T>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t ab_full[2], ab_empty[2], w_full[kWStages], w_empty[kWStages], s1_full[2],
        g_full[2], g_empty[2], acc_full, acc_empty, drain;
    __shared__ uint32_t tmem_sh;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nbt = (a.B + kTB - 1) / kTB, ndt = (a.D + kTD - 1) / kTD;
    const int ntiles = nbt * ndt;

    if (warp == 1) {
        if (lane == 0) {
            for (int i = 0; i < 2; ++i) {
                mbar_init(&ab_full[i], 1);
                mbar_init(&ab_empty[i], 1);
                mbar_init(&s1_full[i], 1);
                mbar_init(&g_full[i], 256);  // both converter warpgroups
                mbar_init(&g_empty[i], 1);
            }
            for (int i = 0; i < kWStages; ++i) {
                mbar_init(&w_full[i], 1);
                mbar_init(&w_empty[i], 1);
            }
            mbar_init(&acc_full, 1);
            mbar_init(&acc_empty, 128);
            mbar_init(&drain, 1);
            abort_flag = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&tmem_sh, kAlloc);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;
    const auto origin = [&](int tile, int& b0, int& d0) {
        b0 = (tile % nbt) * kTB;
        d0 = (tile / nbt) * kTD;
    };

    if (warp == 0 && lane == 0) {
        // loads: a tile's left and right blocks one tile ahead, as 4 KB boxes [16 b][16 a][8 c]
        // (one per c-block) and [16 d][16 a][8 e] (one per e-block); the wT slices of every
        // chunk through a ring of three
        const auto load_ab = [&](int tile, int lt) -> bool {
            const int p = lt & 1;
            if (lt >= 2 && !mbar_wait(&ab_empty[p], ((lt - 2) >> 1) & 1, &g_status,
                                      kStatusMmaWait, &abort_flag)) {
                return false;
            }
            int b0, d0;
            origin(tile, b0, d0);
            uint8_t* dst = smem + SM_AB + p * AB_BYTES;
            mbar_arrive_expect_tx(&ab_full[p], AB_BYTES);
            for (int blk = 0; blk < 4; ++blk) {
                tma_load_3d(dst + blk * kBox, &tl, &ab_full[p], 8 * blk, 0, b0);
                tma_load_3d(dst + A1_BYTES + blk * kBox, &tr, &ab_full[p], 8 * blk, 0, d0);
            }
            return true;
        };
        int lt = 0, wq = 0, ab_issued = 0;
        bool ok = blockIdx.x < ntiles && load_ab(blockIdx.x, 0);
        ab_issued = ok ? 1 : 0;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++lt) {
            for (int k = 0; k < kChunks; ++k, ++wq) {
                // the next tile's blocks once this tile's MMAs have started (the buffer they
                // overwrite was released by the tile before this one)
                if (k == 4 && tile + (int)gridDim.x < ntiles) {
                    if (!load_ab(tile + gridDim.x, lt + 1)) {
                        ok = false;
                        break;
                    }
                    ++ab_issued;
                }
                const int s = wq % kWStages;
                if (wq >= kWStages &&
                    !mbar_wait(&w_empty[s], ((wq - kWStages) / kWStages) & 1, &g_status,
                               kStatusMmaWait, &abort_flag)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&w_full[s], W_BYTES);
                tma_load_3d(smem + SM_W + s * W_BYTES, &tw, &w_full[s], 0, 0, k);
            }
        }
        // the last copies land before the CTA can exit
        for (int h = ab_issued > 2 ? ab_issued - 2 : 0; h < ab_issued; ++h) {
            mbar_wait(&ab_full[h & 1], (h >> 1) & 1, &g_status, kStatusTmaWait, nullptr, kDrain);
        }
        for (int h = wq > kWStages ? wq - kWStages : 0; h < wq; ++h) {
            mbar_wait(&w_full[h % kWStages], (h / kWStages) & 1, &g_status, kStatusTmaWait,
                      nullptr, kDrain);
        }
    } else if (warp == 1 && lane == 0) {
        // MMAs. First product: A = left rows (b, c) and B = right columns (d, e), MN-major and
        // interleaved: core matrices [8 a][8 c or e], the next 8 of M or N (the next b or d) 256
        // bytes on, the second 8 rows a 128 bytes on. Second product: A = the converted chunk,
        // B = the wT slice (both K-major, 128-byte swizzle). Global chunk q is chunk q % 16 of
        // local tile q / 16; its first product runs two chunks ahead of its second.
        const bool bf = E::kBf16;
        const uint32_t id1 = idesc_f16(bf, 128, 128, true, true);
        const uint32_t id2 = idesc_f16(bf, 128, a.F, false, false);
        const uint32_t ab_base = smem_u32(smem + SM_AB), w_base = smem_u32(smem + SM_W),
                       g_base = smem_u32(smem + SM_G);
        const int total = ((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) *
                          kChunks;
        int ab_ready = -1;  // the last local tile whose blocks were waited for
        const auto need_ab = [&](int lt) -> bool {
            if (lt > ab_ready) {
                if (!mbar_wait(&ab_full[lt & 1], (lt >> 1) & 1, &g_status, kStatusTmaWait,
                               &abort_flag)) {
                    return false;
                }
                tc_fence_after();
                ab_ready = lt;
            }
            return true;
        };
        // chunk k: c-block k >> 2, e-block k & 3; its TMEM buffer was last read for chunk q - 2,
        // whose conversion was waited for before that chunk's second product
        const auto first = [&](int qq) {
            const int k = qq % kChunks;
            const uint32_t ab = ab_base + ((qq / kChunks) & 1) * AB_BYTES;
            mma_ss(tmem + T_S1 + (qq & 1) * 128,
                   smem_desc(ab + (k >> 2) * kBox, 128, 256, kSwizzleNone),
                   smem_desc(ab + A1_BYTES + (k & 3) * kBox, 128, 256, kSwizzleNone), id1, 0u);
            mma_commit(&s1_full[qq & 1]);
        };
        bool ok = total > 0 && need_ab(0);
        if (ok) {
            first(0);
            first(1);
        }
        for (int q = 0; ok && q < total; ++q) {
            const int lt = q / kChunks, k = q % kChunks, gb = q & 1, s = q % kWStages;
            if (!mbar_wait(&g_full[gb], (q >> 1) & 1, &g_status, kStatusSyncWait, &abort_flag) ||
                !mbar_wait(&w_full[s], (q / kWStages) & 1, &g_status, kStatusTmaWait,
                           &abort_flag) ||
                (k == 0 && lt >= 1 &&
                 !mbar_wait(&acc_empty, (lt - 1) & 1, &g_status, kStatusSyncWait, &abort_flag))) {
                break;
            }
            tc_fence_after();
            const uint32_t ga = g_base + gb * G_BYTES, wa = w_base + s * W_BYTES;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    mma_ss(tmem + T_ACC + h * 128,
                           smem_desc(ga + h * (128 * 128) + 32 * ks, 16, 1024, kSwizzle128B),
                           smem_desc(wa + 32 * ks, 16, 1024, kSwizzle128B), id2,
                           (k > 0 || ks > 0) ? 1u : 0u);
                }
            }
            mma_commit(&g_empty[gb]);
            mma_commit(&w_empty[s]);
            if (k == kChunks - 1) {
                mma_commit(&ab_empty[lt & 1]);
                mma_commit(&acc_full);
            }
            if (q + 2 < total) {
                if (!need_ab((q + 2) / kChunks)) {
                    break;
                }
                first(q + 2);
            }
        }
        mma_commit(&drain);
        mbar_wait(&drain, 0, &g_status, kStatusMmaWait, nullptr, kDrain);
    } else if (warp >= kConvWarp0 && warp < kEpiWarp0) {
        // converters: thread = lane m = (b, c) = (m / 8, m % 8) of the first product; warpgroup
        // cg takes d 8 cg .. 8 cg + 7 (TMEM columns 64 cg ..), whose 8 e values go to rows (b, d)
        // of the chunk tile, 16 bytes at piece c ^ (d % 8) of the row (128-byte swizzle), half
        // b / 8
        const int cg = (warp - kConvWarp0) >> 2;
        const int m = ((warp & 3) << 5) | lane;
        const int bl = m >> 3, cl = m & 7;
        const uint32_t lane_base = tmem_lane_base(warp);
        uint8_t* g_rows = smem + SM_G + (bl >> 3) * (128 * 128) + (bl & 7) * 16 * 128;
        const int total = ((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) *
                          kChunks;
        for (int q = 0; q < total && blockIdx.x < ntiles; ++q) {
            const int gb = q & 1;
            mbar_wait(&s1_full[gb], (q >> 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            const uint32_t src = tmem + T_S1 + gb * 128 + 64 * cg + lane_base;
            uint32_t v0[32], v1[32];
            tmem_ld32(src, v0);
            tmem_ld32(src + 32, v1);
            tmem_wait_ld();
            if (q >= 2) {
                mbar_wait(&g_empty[gb], ((q - 2) >> 1) & 1, &g_status, kStatusMmaWait,
                          &abort_flag);
            }
            uint8_t* rows = g_rows + gb * G_BYTES;
            // columns 0..63: d 0..7; 64..127: d 8..15 (8 e each)
            const auto put = [&](const uint32_t (&v)[32], int dbase) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int d = dbase + j;
                    uint4 w;
                    w.x = E::pack(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1]));
                    w.y = E::pack(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
                    w.z = E::pack(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
                    w.w = E::pack(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
                    *reinterpret_cast<uint4*>(rows + d * 128 + ((cl ^ (d & 7)) << 4)) = w;
                }
            };
            put(v0, 8 * cg);
            put(v1, 8 * cg + 4);
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(&g_full[gb]);
        }
    } else if (warp >= kEpiWarp0) {
        // epilogue: half h's lane r is row (b, d) = (8 h + r / 16, r % 16); F columns as boxes of
        // 64 [8 b][16 d][64 f] (row r, pieces c ^ (r % 8))
        const int r = ((warp & 3) << 5) | lane;
        const bool leader = threadIdx.x == kEpiWarp0 * 32;
        const uint32_t lane_base = tmem_lane_base(warp);
        uint8_t* stage = smem + SM_OUT;
        const int nbox = (a.F + 63) / 64;
        int lt = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
            int b0, d0;
            origin(tile, b0, d0);
            mbar_wait(&acc_full, lt & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            for (int h = 0; h < 2; ++h) {
                if (leader) {
                    bulk_wait_read_all();
                }
                named_sync(2, 128);
                for (int c32 = 0; c32 < (a.F + 31) / 32; ++c32) {
                    uint32_t v[32];
                    tmem_ld32(tmem + T_ACC + h * 128 + lane_base + 32 * c32, v);
                    tmem_wait_ld();
                    uint8_t* row = stage + (c32 >> 1) * OUT_BOX + r * 128;
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        const int c = 4 * (c32 & 1) + qq;
                        uint4 w;
                        w.x = E::pack(__uint_as_float(v[8 * qq]), __uint_as_float(v[8 * qq + 1]));
                        w.y = E::pack(__uint_as_float(v[8 * qq + 2]),
                                      __uint_as_float(v[8 * qq + 3]));
                        w.z = E::pack(__uint_as_float(v[8 * qq + 4]),
                                      __uint_as_float(v[8 * qq + 5]));
                        w.w = E::pack(__uint_as_float(v[8 * qq + 6]),
                                      __uint_as_float(v[8 * qq + 7]));
                        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = w;
                    }
                }
                if (h == 1) {
                    tc_fence_before();
                    mbar_arrive(&acc_empty);
                }
                fence_async_smem();
                named_sync(2, 128);
                if (leader) {
                    for (int j = 0; j < nbox; ++j) {
                        tma_store_3d_out(&to, smem_u32(stage + j * OUT_BOX), 64 * j, d0,
                                         b0 + 8 * h);
                    }
                    bulk_commit_group();
                }
            }
        }
        if (leader) {
            bulk_wait_done_all();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kAlloc);
    }
}

// wT [F][32 c][32 e] -> wr [16 chunks][F][8 c x 8 e], chunk k = (c-block k / 4, e-block k % 4):
// one 16-byte run of 8 e a thread
template <typename T>
__global__ void opm_w_layout_kernel(const T* wT, T* wr, int F) {
    const int n = 16 * F * 8;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int cl = i & 7, f = (i >> 3) % F, k = (i >> 3) / F;
        const int c = 8 * (k >> 2) + cl, e0 = 8 * (k & 3);
        reinterpret_cast<uint4*>(wr)[i] =
            *reinterpret_cast<const uint4*>(wT + (long long)f * 1024 + c * 32 + e0);
    }
}

}  // namespace

unsigned read_and_clear_status_opm() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    return v;
}

// VoltaOpmOuter at C = E = 32 (validated by the caller); the workspace takes wT laid out chunk by
// chunk (F * 2 KB)
int opm_outer_fused(void* stream, int dtype, const void* left, const void* right, const void* wT,
                    void* out, int64_t B, int64_t D, int64_t F, void* workspace,
                    size_t ws_bytes) {
    if (workspace == nullptr || ws_bytes < (size_t)F * 2048) {
        return fail(kInvalidArgument,
                    "opm_outer: workspace below one chunk (cflk_volta_opm_outer_workspace_size)");
    }
    const CUtensorMapDataType tdt =
        dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tl, tr, tw, to;
    // left [16 a][B][32 c] as dims (c, a, b) and right [16 a][D][32 e] as (e, a, d): boxes
    // [16 b][16 a][8 c] and [16 d][16 a][8 e]
    const uint64_t dl[3] = {32, 16, (uint64_t)B}, sl[2] = {(uint64_t)B * 32, 32};
    const uint64_t dr[3] = {32, 16, (uint64_t)D}, sr[2] = {(uint64_t)D * 32, 32};
    const uint32_t box8[3] = {8, 16, 16};
    // the laid-out wT [16][F][64]: boxes [128 f][64] (rows past F read as zero)
    const uint64_t dw[3] = {64, (uint64_t)F, 16}, sw[2] = {64, (uint64_t)F * 64};
    const uint32_t boxw[3] = {64, 128, 1};
    // out [B][D][F]: boxes [8 b][16 d][64 f]
    const uint64_t dout[3] = {(uint64_t)F, (uint64_t)D, (uint64_t)B},
                   sout[2] = {(uint64_t)F, (uint64_t)D * F};
    const uint32_t boxo[3] = {64, 16, 8};
    if (!encode_tiled(&tl, tdt, 2, 3, left, dl, sl, box8, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_tiled(&tr, tdt, 2, 3, right, dr, sr, box8, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_tiled(&tw, tdt, 2, 3, workspace, dw, sw, boxw, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&to, tdt, 2, 3, out, dout, sout, boxo, CU_TENSOR_MAP_SWIZZLE_128B)) {
        return fail(kInvalidArgument, "opm_outer: TMA descriptor rejected");
    }
    const OuterArgs args{(int)B, (int)D, (int)F};
    int dev = 0;
    cudaGetDevice(&dev);
    static bool attr[kMaxDevices][2] = {};
    static int sms[kMaxDevices] = {};
    const int ti = dtype == kBF16 ? 1 : 0;
    const auto kern = dtype == kBF16 ? opm_outer_kernel<__nv_bfloat16> : opm_outer_kernel<__half>;
    if (dev < kMaxDevices && !attr[dev][ti]) {
        const cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) {
            return fail(kInternal, std::string("opm_outer: ") + cudaGetErrorString(e));
        }
        attr[dev][ti] = true;
    }
    if (dev < kMaxDevices && sms[dev] == 0) {
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    const int nsm = dev < kMaxDevices && sms[dev] > 0 ? sms[dev] : 148;
    const long long tiles = ((B + kTB - 1) / kTB) * ((D + kTD - 1) / kTD);
    const dim3 grid((unsigned)std::min<long long>(tiles, nsm));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int nvec = (int)(16 * F * 8);
    if (dtype == kBF16) {
        opm_w_layout_kernel<__nv_bfloat16><<<(nvec + 255) / 256, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(wT), static_cast<__nv_bfloat16*>(workspace),
            (int)F);
    } else {
        opm_w_layout_kernel<__half><<<(nvec + 255) / 256, 256, 0, st>>>(
            static_cast<const __half*>(wT), static_cast<__half*>(workspace), (int)F);
    }
    kern<<<grid, kThreads, SMEM, st>>>(tl, tr, tw, to, args);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("opm_outer launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

}  // namespace cflk

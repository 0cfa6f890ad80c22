// Tile GEMMs with fused epilogues for sm_100a: VoltaOpmUpdate, and VoltaGdp at widths the
// resident-weight row-tile kernel does not cover (colabfold-legacy-kernels cuda/volta_ops.cu:
// 108-265 and 643-699, handlers cuda/volta_fused_ffi.h:261-298).
//
//   * out [M, N] = epilogue(A [M, K] @ B [K, N]) with A row-major (K contiguous, the K-major A
//     operand) and B row-major (N contiguous, the N-major B operand), 16-bit in, float32
//     accumulators in tensor memory; Gdp multiplies A by two B matrices at once (wp and wg);
//   * persistent CTAs walk 128 x 128 output tiles (rows fastest, so the CTAs running at once
//     share a B tile in L2); warp 0 streams 64-deep K slices of A and B through a ring of shared
//     memory stages by TMA, warp 1 issues the tcgen05 MMAs into one of two accumulator buffers,
//     the warpgroup of warps 4-7 (thread = row = tensor-memory lane) applies the epilogue to the
//     other buffer and writes the tile through swizzled shared memory with TMA stores (rows and
//     columns past M and N clip);
//   * VoltaOpmUpdate: out [B, D*F] = (lhs @ t[K, D*F] + bias[f]) / (eps + norm[b, d]) (+ residual)
//     with n = d F + f; VoltaGdp: out = mask[m] (x wp + bp) act(x wg + bg), act sigmoid or swish.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "capi_internal.h"
#include "cflk_b200.h"
#include "fused_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace cflk {
namespace {

__device__ unsigned g_status;

constexpr int GBM = 128, GBK = 64;
constexpr int kGemmThreads = 384;  // TMA warp, MMA warp, two idle, two epilogue warpgroups
constexpr int kEpiWarp0 = 4;
// a wait for copies or MMAs already issued, at the end of a CTA (the pipeline's own waits give up
// after 2 s and set the abort flag; these then bound the drain)
constexpr unsigned long long kDrainLimitNs = 200000000ull;

// kOpmOuterG / kPlain: the two products of VoltaOpmOuter. kOpmOuterG: G [(b,c), (d,e)] =
// left^T right over the 16 MSA rows, rounded to the 16-bit type and written as G2 [b][d][c][e]
// (a 4-D box store: a tile's 128 rows are 128/C whole b, its 128 columns 4 whole d); kPlain:
// out = A B rounded, no epilogue arithmetic (G2 as [B*D][C*E] times wT).
enum GemmKind : int { kOpmUpdate = 0, kGdpDual = 1, kContract = 2, kOpmOuterG = 3, kPlain = 4 };

struct GemmArgs {
    int M, N, K;
    int batch;  // independent products (kContract: the channels), each [M, N]
    int opm_c;  // kOpmOuterG: C (16, 32, 64 or 128), the rows of one b
    long long lda;  // A's row stride in elements when it is not the default (0)
    // VoltaOpmUpdate: bias [F] float32, norm [M, D] float32, residual [M, N] (or null)
    const float* bias_f;
    const float* norm;
    const void* residual;
    int F, D;
    float eps;
    // VoltaGdp: bp, bg [N] and the row mask [M] (16-bit), activation 0 sigmoid / 1 swish
    const void* bp;
    const void* bg;
    const void* mask;
    int act;
};

template <int KIND>
struct GemmCfg {
    static constexpr int NB = KIND == kGdpDual ? 2 : 1;   // B matrices
    // output tile 128 x BN: the contraction and VoltaOpmUpdate take 256 columns, halving their A
    // re-reads from L2 (and the shared-memory bytes an MMA reads per FLOP)
    static constexpr int BN = KIND == kContract || KIND == kOpmUpdate ? 256 : 128;
    static constexpr int A_BYTES = GBM * GBK * 2;          // [128 rows][64 k] or two [64 k][64 m]
    static constexpr int B_BYTES = GBK * BN * 2;           // [BN rows][64 k] or BN/64 [64 k][64 n]
    static constexpr int STAGE_BYTES = A_BYTES + NB * B_BYTES;
    static constexpr int STAGES = NB == 1 && BN == 128 ? 4 : 3;
    static constexpr int OUT_ELEM = KIND == kContract ? 4 : 2;
    // output staging in boxes of 128 rows x 128 bytes (64 16-bit or 32 float32 columns): one
    // tile's boxes (VoltaOpmUpdate's residual lands in them first), the contraction a ring of
    // four
    static constexpr int BOX_BYTES = GBM * 128;
    static constexpr int BOX_COLS = 128 / OUT_ELEM;
    static constexpr int BOXES = BN / BOX_COLS;
    static constexpr int STAGE_BOXES = KIND == kOpmUpdate || KIND == kContract ? 4 : 2;
    static constexpr int OUT_OFF = STAGES * STAGE_BYTES;
    static constexpr int SMEM = OUT_OFF + STAGE_BOXES * BOX_BYTES + 1024;
    static constexpr int ACC_COLS = NB * BN;               // one accumulator buffer
    static constexpr uint32_t ALLOC = 2 * ACC_COLS <= 256 ? 256 : 512;
    static_assert(2 * ACC_COLS <= 512, "tensor memory");
    static_assert(KIND != kContract || BOXES == BN / 32, "one float32 box per 32 columns");
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::
            "l"(map),
        "r"(src), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], "
        "[%1];" ::"l"(map),
        "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// until at most N of this thread's committed bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// A_MN: A is stored M-major ([K][M], M contiguous) instead of K-major ([M][K]); B_MN: B is
// stored N-major ([K][N]) instead of K-major ([N][K]). Every map is 3-D, the outer dimension the
// batch. tb1 is VoltaGdp's second B and VoltaOpmUpdate's residual (a map shaped as the output).
template <typename T, int KIND, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb0,
                const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap to,
                const GemmArgs a) {
    using C = GemmCfg<KIND>;
    using E = Elem<T>;
    constexpr int BN = C::BN;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[C::STAGES], empty[C::STAGES], acc_full[2], acc_empty[2], drain,
        res_full[2][2];
    __shared__ uint32_t tmem_sh;
    __shared__ int abort_flag;
    // per-column epilogue constants: VoltaOpmUpdate's bias [F] (F <= 128); VoltaGdp's bp and bg
    // of each epilogue warpgroup's 64 columns of the tile
    __shared__ __align__(16) float bias_sh[128];
    __shared__ __align__(16) float colv[2][2][64];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntm = (a.M + GBM - 1) / GBM, ntn = (a.N + BN - 1) / BN;
    const int per_batch = ntm * ntn;
    const int ntiles = per_batch * a.batch;
    const int nk = (a.K + GBK - 1) / GBK;

    if (warp == 1) {
        if (lane == 0) {
            for (int i = 0; i < C::STAGES; ++i) {
                mbar_init(&full[i], 1);
                mbar_init(&empty[i], 1);
            }
            for (int i = 0; i < 2; ++i) {
                mbar_init(&acc_full[i], 1);
                mbar_init(&acc_empty[i], 256);  // both epilogue warpgroups
                mbar_init(&res_full[0][i], 1);
                mbar_init(&res_full[1][i], 1);
            }
            mbar_init(&drain, 1);
            abort_flag = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&tmem_sh, C::ALLOC);
        tmem_relinquish();
    } else if (warp >= kEpiWarp0 && KIND == kOpmUpdate) {
        const int i = threadIdx.x - kEpiWarp0 * 32;
        if (i < a.F) {
            bias_sh[i] = a.bias_f[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;

    if (warp == 0 && lane == 0) {
        // TMA: per tile, the K slices of A and the B matrices through the stage ring (a stage is
        // refilled only once the MMAs that read it are done; a wait that gives up ends the loop)
        int g = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int bt = tile / per_batch, rem = tile - bt * per_batch;
            const int m0 = (rem % ntm) * GBM, n0 = (rem / ntm) * BN;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = g % C::STAGES;
                if (g >= C::STAGES &&
                    !mbar_wait(&empty[s], ((g - C::STAGES) / C::STAGES) & 1, &g_status,
                               kStatusMmaWait, &abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + s * C::STAGE_BYTES;
                const int k0 = kb * GBK;
                mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
                if constexpr (A_MN) {
                    // two 64-row atoms of [64 k][64 m]
                    tma_load_3d(st, &ta, &full[s], m0, k0, bt);
                    tma_load_3d(st + C::A_BYTES / 2, &ta, &full[s], m0 + 64, k0, bt);
                } else {
                    tma_load_3d(st, &ta, &full[s], k0, m0, bt);
                }
                uint8_t* b = st + C::A_BYTES;
#pragma unroll
                for (int j = 0; j < C::NB; ++j) {
                    const CUtensorMap* tb = j == 0 ? &tb0 : &tb1;
                    uint8_t* bj = b + j * C::B_BYTES;
                    if constexpr (B_MN) {
#pragma unroll
                        for (int h = 0; h < BN / 64; ++h) {
                            tma_load_3d(bj + h * (64 * 128), tb, &full[s], n0 + 64 * h, k0, bt);
                        }
                    } else {
                        tma_load_3d(bj, tb, &full[s], k0, n0, bt);
                    }
                }
            }
        }
        // the last loads (one per stage at most) land before the CTA can exit
        for (int h = g > C::STAGES ? g - C::STAGES : 0; h < g; ++h) {
            mbar_wait(&full[h % C::STAGES], (h / C::STAGES) & 1, &g_status, kStatusTmaWait,
                      nullptr, kDrainLimitNs);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA: M = 128, N = BN, K = 16 per instruction
        const uint32_t idesc = idesc_f16(E::kBf16, GBM, BN, A_MN, B_MN);
        // K-major operand: rows of 128 bytes (8-row groups 1 KB apart), a K step of 16 is 32
        // bytes along the row; MN-major: 64-wide atoms 8 KB apart, K steps of 16 rows 2 KB apart
        const auto desc = [](uint32_t base, int ks, bool mn) -> uint64_t {
            return mn ? smem_desc(base + ks * 16 * 128, 64 * 128, 1024, kSwizzle128B)
                      : smem_desc(base + 32 * ks, 16, 1024, kSwizzle128B);
        };
        int g = 0, lt = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++lt) {
            const int buf = lt & 1;
            if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt - 2) >> 1) & 1, &g_status,
                                      kStatusSyncWait, &abort_flag)) {
                break;
            }
            tc_fence_after();
            const uint32_t acc = tmem + buf * C::ACC_COLS;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int s = g % C::STAGES;
                if (!mbar_wait(&full[s], (g / C::STAGES) & 1, &g_status, kStatusTmaWait,
                               &abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                const uint32_t sb = sa + C::A_BYTES;
                // K steps past K (zero-filled) are skipped: VoltaOpmOuter's first product has K 16
                const int ksteps = min(GBK / 16, (a.K - kb * GBK + 15) / 16);
#pragma unroll
                for (int ks = 0; ks < GBK / 16; ++ks) {
                    if (ks >= ksteps) {
                        break;
                    }
                    const uint64_t ad = desc(sa, ks, A_MN);
                    const uint32_t acc_on = (kb > 0 || ks > 0) ? 1u : 0u;
                    mma_ss(acc, ad, desc(sb, ks, B_MN), idesc, acc_on);
                    if constexpr (C::NB == 2) {
                        mma_ss(acc + BN, ad, desc(sb + C::B_BYTES, ks, B_MN), idesc, acc_on);
                    }
                }
                mma_commit(&empty[s]);
            }
            if (ok) {
                mma_commit(&acc_full[buf]);
            }
        }
        // every MMA issued is complete before tensor memory is freed
        mma_commit(&drain);
        mbar_wait(&drain, 0, &g_status, kStatusMmaWait, nullptr, kDrainLimitNs);
    } else if (warp >= kEpiWarp0) {
        // epilogue: two warpgroups, each over all 128 rows (thread r = row r = tensor-memory
        // lane r) and half of the tile's columns: warpgroup g takes the 32-column chunks
        // [g NCH/2, (g+1) NCH/2), its own staging boxes, named barrier 1 + g and leader thread
        constexpr int NCH = BN / 32, HCH = NCH / 2;
        const int g = (warp - kEpiWarp0) >> 2;
        const int r = ((warp & 3) << 5) | lane;
        const bool leader = lane == 0 && (warp & 3) == 0;
        const uint32_t lane_base = tmem_lane_base(warp);
        uint8_t* ostage = smem + C::OUT_OFF;
        [[maybe_unused]] const bool has_res = KIND == kOpmUpdate && a.residual != nullptr;
        const auto tile_origin = [&](int tile, int& bt, int& m0, int& n0) {
            bt = tile / per_batch;
            const int rem = tile - bt * per_batch;
            m0 = (rem % ntm) * GBM;
            n0 = (rem / ntm) * BN;
        };
        // 16-bit kinds: warpgroup g's BN / 2 columns are BN / 128 boxes (j), boxes g BN/128 + j
        // of the staging; their first column
        constexpr int WB = BN / 128;
        const auto box16 = [&](int j) -> uint8_t* {
            return ostage + (g * WB + j) * C::BOX_BYTES;
        };
        // VoltaOpmUpdate: this warpgroup's residual boxes of the tile by TMA, issued as soon as
        // the previous tile's stores have read the staging, so the copy overlaps the tile's MMAs
        // (columns or rows past the ends read as zero)
        int res_issued = 0;  // the leader's count
        const auto load_res = [&](int n0, int m0, int bt) {
            ++res_issued;
            mbar_arrive_expect_tx(&res_full[g][0], WB * C::BOX_BYTES);
#pragma unroll
            for (int j = 0; j < WB; ++j) {
                tma_load_3d(box16(j), &tb1, &res_full[g][0], n0 + (BN / 2) * g + 64 * j, m0, bt);
            }
        };
        int lt = 0, box = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
            const int buf = lt & 1;
            int bt, m0, n0;
            tile_origin(tile, bt, m0, n0);
            const int m = m0 + r;
            // the previous tile's stores have read their staging (not for the contraction,
            // whose ring is released box by box)
            if constexpr (KIND != kContract) {
                if (leader) {
                    bulk_wait_read<0>();
                    if constexpr (KIND == kOpmUpdate) {
                        if (has_res) {
                            load_res(n0, m0, bt);
                        }
                    }
                }
            }
            if constexpr (KIND == kGdpDual) {
                // this warpgroup's 64 columns of bp and bg
                if (r < 64) {
                    const int n = n0 + 64 * g + r;
                    colv[g][0][r] = n < a.N ? E::to_f(static_cast<const T*>(a.bp)[n]) : 0.f;
                    colv[g][1][r] = n < a.N ? E::to_f(static_cast<const T*>(a.bg)[n]) : 0.f;
                }
            }
            named_sync(1 + g, 128);
            [[maybe_unused]] float mval = 0.f;
            [[maybe_unused]] float rden[8];
            if constexpr (KIND == kGdpDual) {
                mval = m < a.M ? E::to_f(static_cast<const T*>(a.mask)[m]) : 0.f;
            }
            if constexpr (KIND == kOpmUpdate) {
                // 1 / (eps + norm[m, d]) for the warpgroup's (BN / 2) / F values of d (at most 8)
                const int d0 = (n0 + (BN / 2) * g) / a.F, nd = (BN / 2) / a.F;
                const float* nrow = a.norm + (long long)m * a.D;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    rden[i] = (i < nd && m < a.M && d0 + i < a.D)
                                  ? __frcp_rn(a.eps + __ldg(nrow + d0 + i))
                                  : 0.f;
                }
                if (has_res) {
                    mbar_wait(&res_full[g][0], lt & 1, &g_status, kStatusTmaWait, &abort_flag);
                }
            }
            mbar_wait(&acc_full[buf], (lt >> 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            const uint32_t acc = tmem + buf * C::ACC_COLS + lane_base;
#pragma unroll
            for (int hc = 0; hc < HCH; ++hc) {
                const int ch = g * HCH + hc;  // the chunk of the tile's columns
                uint32_t r0[32];
                [[maybe_unused]] uint32_t r1[32];
                tmem_ld32(acc + 32 * ch, r0);
                if constexpr (KIND == kGdpDual) {
                    tmem_ld32(acc + BN + 32 * ch, r1);
                }
                tmem_wait_ld();
                if constexpr (KIND == kContract) {
                    // the float32 products as they are: the warpgroup's boxes alternate between
                    // its two ring slots (2g, 2g + 1), row r, 8 pieces of 4 floats at piece
                    // (p ^ (r % 8)); a slot is free once the store of the box two before it has
                    // read it
                    if (leader) {
                        bulk_wait_read<1>();
                    }
                    named_sync(1 + g, 128);
                    uint8_t* slot = ostage + (2 * g + (box & 1)) * C::BOX_BYTES;
                    uint8_t* row = slot + r * 128;
#pragma unroll
                    for (int p = 0; p < 8; ++p) {
                        *reinterpret_cast<uint4*>(row + ((p ^ (r & 7)) << 4)) =
                            make_uint4(r0[4 * p], r0[4 * p + 1], r0[4 * p + 2], r0[4 * p + 3]);
                    }
                    if (hc == HCH - 1) {
                        // every column of this warpgroup is in staging: its share of the
                        // buffer is free
                        tc_fence_before();
                        mbar_arrive(&acc_empty[buf]);
                    }
                    fence_async_smem();
                    named_sync(1 + g, 128);
                    if (leader) {
                        if (n0 + 32 * ch < a.N) {
                            tma_store_3d(&to, smem_u32(slot), n0 + 32 * ch, m0, bt);
                        }
                        bulk_commit();
                    }
                    ++box;
                } else if constexpr (KIND == kOpmOuterG) {
                    // row r = (b_l, c), chunk ch = d_l (e 0..31): 64 bytes at [b_l][d_l - 2g][c]
                    // of the warpgroup's [128/C][2][C][32] box (plain layout, a warp's 32 rows
                    // are 32 consecutive 64-byte runs)
                    const int bl = r / a.opm_c, cl = r - bl * a.opm_c;
                    uint8_t* dst = ostage + g * C::BOX_BYTES + (((bl * 2 + hc) * a.opm_c) + cl) * 64;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 w;
                        w.x = E::pack(__uint_as_float(r0[8 * q]), __uint_as_float(r0[8 * q + 1]));
                        w.y = E::pack(__uint_as_float(r0[8 * q + 2]),
                                      __uint_as_float(r0[8 * q + 3]));
                        w.z = E::pack(__uint_as_float(r0[8 * q + 4]),
                                      __uint_as_float(r0[8 * q + 5]));
                        w.w = E::pack(__uint_as_float(r0[8 * q + 6]),
                                      __uint_as_float(r0[8 * q + 7]));
                        *reinterpret_cast<uint4*>(dst + 16 * q) = w;
                    }
                } else {
                    const int nb = n0 + 32 * ch;
                    float v[32];
                    // staging pieces of these 32 columns: the warpgroup's box hc / 2, row r,
                    // pieces 4 (hc % 2) + q at (c ^ (r % 8))
                    uint8_t* row = box16(hc >> 1) + r * 128;
                    if constexpr (KIND == kOpmUpdate) {
                        // (acc + bias[f]) / (eps + norm[m, d]) (+ residual), n = d F + f: the 32
                        // columns span at most two d (F = 16)
                        const int i0 = (32 * hc) / a.F, i1 = (32 * hc + 16) / a.F;
                        float rd0 = 0.f, rd1 = 0.f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {  // selects, not a local-memory index
                            rd0 = i == i0 ? rden[i] : rd0;
                            rd1 = i == i1 ? rden[i] : rd1;
                        }
                        const float* bias = &bias_sh[nb & (a.F - 1)];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int c = 4 * (hc & 1) + q;
                            uint4 res = make_uint4(0, 0, 0, 0);
                            if (has_res) {
                                res = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) << 4));
                            }
                            const uint32_t w4[4] = {res.x, res.y, res.z, res.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int i = 8 * q + 2 * e;
                                // F = 16: columns 16-31 take bias[0..15] again
                                const float b0 = bias[i & (a.F - 1)], b1 = bias[(i + 1) & (a.F - 1)];
                                const float rd = i < 16 ? rd0 : rd1;
                                const float2 rr = E::unpack(w4[e]);
                                v[i] = fmaf(__uint_as_float(r0[i]) + b0, rd, rr.x);
                                v[i + 1] = fmaf(__uint_as_float(r0[i + 1]) + b1, rd, rr.y);
                            }
                        }
                    } else if constexpr (KIND == kPlain) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            v[i] = __uint_as_float(r0[i]);
                        }
                    } else {
                        // mask * (p + bp) * act(g + bg)
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const float p = __uint_as_float(r0[i]) + colv[g][0][32 * hc + i];
                            const float gt = __uint_as_float(r1[i]) + colv[g][1][32 * hc + i];
                            const float sg = fused::sigmoid_fast(gt);
                            v[i] = mval * p * (a.act == 0 ? sg : gt * sg);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int c = 4 * (hc & 1) + q;
                        uint4 w;
                        w.x = E::pack(v[8 * q], v[8 * q + 1]);
                        w.y = E::pack(v[8 * q + 2], v[8 * q + 3]);
                        w.z = E::pack(v[8 * q + 4], v[8 * q + 5]);
                        w.w = E::pack(v[8 * q + 6], v[8 * q + 7]);
                        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = w;
                    }
                }
            }
            if constexpr (KIND != kContract) {
                // this warpgroup's share of the accumulator buffer is free; its staged box goes
                // out by TMA
                tc_fence_before();
                mbar_arrive(&acc_empty[buf]);
                fence_async_smem();
                named_sync(1 + g, 128);
                if (leader) {
                    if constexpr (KIND == kOpmOuterG) {
                        // d 2g, 2g + 1 of the tile as one [128/C b][2 d][C c][32 e] box of G2
                        if (n0 + 64 * g < a.N) {
                            tma_store_4d(&to, smem_u32(ostage + g * C::BOX_BYTES), 0, 0,
                                         n0 / 32 + 2 * g, m0 / a.opm_c);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < WB; ++j) {
                            const int col = n0 + (BN / 2) * g + 64 * j;
                            if (col < a.N) {
                                tma_store_3d(&to, smem_u32(box16(j)), col, m0, bt);
                            }
                        }
                    }
                    bulk_commit();
                }
            }
        }
        if (leader) {
            bulk_wait_all();
            // every residual load has landed before the CTA exits (after an abort a wait may
            // have given up on one still in flight)
            if constexpr (KIND == kOpmUpdate) {
                if (res_issued > 0) {
                    mbar_wait(&res_full[g][0], (res_issued - 1) & 1, &g_status, kStatusTmaWait,
                              nullptr, kDrainLimitNs);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::ALLOC);
    }
}

template <typename T, int KIND, bool A_MN, bool B_MN>
cudaError_t launch_gemm(cudaStream_t stream, int dtype, const void* A, const void* B0,
                        const void* B1, void* out, const GemmArgs& a, bool& map_ok) {
    using C = GemmCfg<KIND>;
    const CUtensorMapDataType tdt =
        dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t M = a.M, N = a.N, K = a.K, Bt = a.batch;
    CUtensorMap ta, tb0, tb1, to;
    // A: [batch][M][K] (box 64 k x 128 m) or [batch][K][M] (box 64 m x 64 k)
    const uint64_t lda = a.lda > 0 ? (uint64_t)a.lda : (A_MN ? M : K);
    const uint64_t da[3] = {A_MN ? M : K, A_MN ? K : M, Bt}, sa[2] = {lda, lda * (A_MN ? K : M)};
    const uint32_t boxa[3] = {64, A_MN ? 64u : (uint32_t)GBM, 1};
    // B: [batch][N][K] (box 64 k x BN n) or [batch][K][N] (box 64 n x 64 k)
    const uint64_t db[3] = {B_MN ? N : K, B_MN ? K : N, Bt}, sb[2] = {B_MN ? N : K, N * K};
    const uint32_t boxb[3] = {64, B_MN ? 64u : (uint32_t)C::BN, 1};
    // out (and VoltaOpmUpdate's residual): [batch][M][N], boxes of 128 bytes a row
    const uint64_t dout[3] = {N, M, Bt}, sout[2] = {N, M * N};
    const uint32_t boxo[3] = {(uint32_t)C::BOX_COLS, GBM, 1};
    const CUtensorMapDataType odt = KIND == kContract ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : tdt;
    map_ok = encode_tiled(&ta, tdt, 2, 3, A, da, sa, boxa, CU_TENSOR_MAP_SWIZZLE_128B) &&
             encode_tiled(&tb0, tdt, 2, 3, B0, db, sb, boxb, CU_TENSOR_MAP_SWIZZLE_128B);
    if (map_ok && KIND == kOpmOuterG) {
        // G2 [b][d][c][e]: M = B C rows (b, c), N = D 32 columns (d, e)
        const uint64_t Cc = a.opm_c, D = N / 32, Bb = M / Cc;
        const uint64_t dg[4] = {32, Cc, D, Bb}, sg[3] = {32, 32 * Cc, 32 * Cc * D};
        const uint32_t boxg[4] = {32, (uint32_t)Cc, 2, (uint32_t)(GBM / Cc)};
        map_ok = encode_tiled(&to, tdt, 2, 4, out, dg, sg, boxg, CU_TENSOR_MAP_SWIZZLE_NONE);
    } else if (map_ok) {
        map_ok = encode_tiled(&to, odt, C::OUT_ELEM, 3, out, dout, sout, boxo,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    }
    tb1 = tb0;
    if (map_ok && KIND == kGdpDual) {
        map_ok = encode_tiled(&tb1, tdt, 2, 3, B1, db, sb, boxb, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (map_ok && KIND == kOpmUpdate && a.residual != nullptr) {
        map_ok = encode_tiled(&tb1, tdt, 2, 3, a.residual, dout, sout, boxo,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (!map_ok) {
        return cudaSuccess;
    }
    auto kern = gemm_kernel<T, KIND, A_MN, B_MN>;
    static bool attr_done[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < kMaxDevices && !attr_done[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) {
            return e;
        }
        attr_done[dev] = true;
    }
    static int sms[kMaxDevices] = {};
    if (dev < kMaxDevices && sms[dev] == 0) {
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    const int nsm = dev < kMaxDevices && sms[dev] > 0 ? sms[dev] : 148;
    const long long tiles =
        (long long)((a.M + GBM - 1) / GBM) * ((a.N + C::BN - 1) / C::BN) * a.batch;
    const dim3 grid((unsigned)std::min<long long>(tiles, nsm));
    kern<<<grid, kGemmThreads, C::SMEM, stream>>>(ta, tb0, tb1, to, a);
    return cudaGetLastError();
}

// VoltaOpmUpdate with K = 0: no product, out = bias[f] / (eps + norm[b, d]) (+ residual)
template <typename T>
__global__ void opm_update_k0_kernel(const float* bias, const float* norm, const T* residual,
                                     T* out, long long total, int N, int F, float eps) {
    using E = Elem<T>;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long b = i / N;
        const int n = (int)(i - b * N);
        float v = bias[n % F] / (eps + norm[b * (N / F) + n / F]);
        if (residual != nullptr) {
            v += E::to_f(residual[i]);
        }
        out[i] = E::from_f(v);
    }
}

// VoltaGdp with K not a multiple of 8 (rows not 16-byte aligned, out of TMA's reach): 64 x 64
// output tiles on the CUDA cores, 16-deep K slices of x, wp and wg staged in shared memory,
// float32 accumulators, each thread 4 rows x 4 columns
template <typename T>
__global__ void __launch_bounds__(256) gdp_simt_kernel(const T* x, const T* wp, const T* bp,
                                                       const T* wg, const T* bg, const T* mask,
                                                       T* out, int M, int K, int N, int act) {
    using E = Elem<T>;
    __shared__ float xs[16][64 + 1], ps[16][64], gs[16][64];
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int tr = threadIdx.x / 16, tc = threadIdx.x % 16;
    float accp[4][4] = {}, accg[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            const int kk = e % 16, mm = e / 16;
            const int m = m0 + mm, k = k0 + kk;
            xs[kk][mm] = (m < M && k < K) ? E::to_f(x[(long long)m * K + k]) : 0.f;
            const int nn = e % 64, kr = e / 64;
            const int n = n0 + nn, k2 = k0 + kr;
            const bool ok = n < N && k2 < K;
            ps[kr][nn] = ok ? E::to_f(wp[(long long)k2 * N + n]) : 0.f;
            gs[kr][nn] = ok ? E::to_f(wg[(long long)k2 * N + n]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float xv[4], pv[4], gv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xv[i] = xs[kk][tr + 16 * i];
                pv[i] = ps[kk][tc + 16 * i];
                gv[i] = gs[kk][tc + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    accp[i][j] = fmaf(xv[i], pv[j], accp[i][j]);
                    accg[i][j] = fmaf(xv[i], gv[j], accg[i][j]);
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + tr + 16 * i;
        if (m >= M) {
            continue;
        }
        const float mv = E::to_f(mask[m]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tc + 16 * j;
            if (n < N) {
                const float p = accp[i][j] + E::to_f(bp[n]);
                const float g = accg[i][j] + E::to_f(bg[n]);
                const float sg = fused::sigmoid_fast(g);
                out[(long long)m * N + n] = E::from_f(mv * p * (act == 0 ? sg : g * sg));
            }
        }
    }
}

// The triangle contraction on the CUDA cores, for sizes whose rows are not 16-byte multiples
// (out of TMA's reach): out[c] (64 x 64 tiles) from 16-deep k slices of A(i, k) and B(k, j) in
// shared memory, float32 accumulators, each thread 4 x 4 outputs. INCOMING: A(i, k) = a[c, k, i]
// and B(k, j) = b[c, k, j]; else A(i, k) = a[c, i, k] and B(k, j) = b[c, j, k].
template <typename T, bool INCOMING>
__global__ void __launch_bounds__(256) contract_simt_kernel(const T* a, const T* b, float* out,
                                                            int I, int J, int K) {
    using E = Elem<T>;
    __shared__ float as[16][64 + 1], bs[16][64 + 1];
    const long long c = blockIdx.z;
    const T* ac = a + c * I * (long long)K;
    const T* bc = b + c * J * (long long)K;
    const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
    const int tr = threadIdx.x / 16, tc = threadIdx.x % 16;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            // the contiguous index fastest, for coalesced reads
            int kk, x;
            if (INCOMING) {
                kk = e / 64;
                x = e % 64;
            } else {
                kk = e % 16;
                x = e / 16;
            }
            const int k = k0 + kk, i = i0 + x, j = j0 + x;
            float av = 0.f, bv = 0.f;
            if (k < K && i < I) {
                av = E::to_f(INCOMING ? ac[(long long)k * I + i] : ac[(long long)i * K + k]);
            }
            if (k < K && j < J) {
                bv = E::to_f(INCOMING ? bc[(long long)k * J + j] : bc[(long long)j * K + k]);
            }
            as[kk][x] = av;
            bs[kk][x] = bv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                av[u] = as[kk][tr + 16 * u];
                bv[u] = bs[kk][tc + 16 * u];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    acc[u][w] = fmaf(av[u], bv[w], acc[u][w]);
                }
            }
        }
        __syncthreads();
    }
    float* oc = out + c * I * (long long)J;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = i0 + tr + 16 * u;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int j = j0 + tc + 16 * w;
            if (i < I && j < J) {
                oc[(long long)i * J + j] = acc[u][w];
            }
        }
    }
}

// VoltaOpmOuter's first product on the CUDA cores, for C that does not divide 128: one block a
// (d, b) pair, G2[b][d][c][e] = h(sum_a left[a, b0 + b, c] right[a, d, e]) for every (c, e)
template <typename T>
__global__ void __launch_bounds__(256) opm_outer_g_simt_kernel(const T* left, const T* right,
                                                               T* g2, int Bfull, int C, int D,
                                                               int b0) {
    using E = Elem<T>;
    extern __shared__ float sh[];  // left rows [16][C], right rows [16][32]
    float* ls = sh;
    float* rs = sh + 16 * C;
    const int d = blockIdx.x, b = blockIdx.y;
    for (int i = threadIdx.x; i < 16 * C; i += blockDim.x) {
        const int arow = i / C, c = i - arow * C;
        ls[i] = E::to_f(left[((long long)arow * Bfull + b0 + b) * C + c]);
    }
    for (int i = threadIdx.x; i < 16 * 32; i += blockDim.x) {
        const int arow = i / 32, e = i - arow * 32;
        rs[i] = E::to_f(right[((long long)arow * D + d) * 32 + e]);
    }
    __syncthreads();
    T* dst = g2 + ((long long)b * D + d) * C * 32;
    for (int i = threadIdx.x; i < C * 32; i += blockDim.x) {
        const int c = i / 32, e = i - c * 32;
        float acc = 0.f;
#pragma unroll
        for (int arow = 0; arow < 16; ++arow) {
            acc = fmaf(ls[arow * C + c], rs[arow * 32 + e], acc);
        }
        dst[i] = E::from_f(acc);
    }
}

bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

}  // namespace

unsigned read_and_clear_status_gemm() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    return v;
}

// VoltaGdp at widths outside the resident-weight kernel's: K and N multiples of 8 (16-byte rows
// for TMA); the caller has validated the rest
int gdp_general(void* stream_, int dtype, const void* x, const void* wp, const void* bp,
                const void* wg, const void* bg, const void* mask, void* out, int64_t M, int64_t K,
                int64_t N, int64_t activation) {
    if (M >= (int64_t(1) << 31) || K >= (int64_t(1) << 31) || N >= (int64_t(1) << 31)) {
        return fail(kInvalidArgument, "gdp: sizes must be below 2^31");
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (K % 8) {
        // x rows are not 16-byte aligned: the CUDA-core tile kernel
        const dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64));
        if (grid.y > 65535u) {
            return fail(kInvalidArgument, "gdp: M must be below 4194240 when K is not a multiple of 8");
        }
        if (dtype == kBF16) {
            using T = __nv_bfloat16;
            gdp_simt_kernel<T><<<grid, 256, 0, stream>>>(
                static_cast<const T*>(x), static_cast<const T*>(wp), static_cast<const T*>(bp),
                static_cast<const T*>(wg), static_cast<const T*>(bg),
                static_cast<const T*>(mask), static_cast<T*>(out), (int)M, (int)K, (int)N,
                (int)activation);
        } else {
            using T = __half;
            gdp_simt_kernel<T><<<grid, 256, 0, stream>>>(
                static_cast<const T*>(x), static_cast<const T*>(wp), static_cast<const T*>(bp),
                static_cast<const T*>(wg), static_cast<const T*>(bg),
                static_cast<const T*>(mask), static_cast<T*>(out), (int)M, (int)K, (int)N,
                (int)activation);
        }
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? kOk : fail(kInternal, std::string("gdp launch: ") + cudaGetErrorString(e));
    }
    if (((M + GBM - 1) / GBM) * ((N + 127) / 128) >= (int64_t(1) << 31)) {
        return fail(kInvalidArgument, "gdp: too many output tiles");
    }
    GemmArgs a{};
    a.batch = 1;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.bp = bp;
    a.bg = bg;
    a.mask = mask;
    a.act = (int)activation;
    bool ok = true;
    const cudaError_t e =
        dtype == kBF16 ? launch_gemm<__nv_bfloat16, kGdpDual, false, true>(stream, dtype, x, wp, wg, out, a, ok)
                       : launch_gemm<__half, kGdpDual, false, true>(stream, dtype, x, wp, wg, out, a, ok);
    if (!ok) {
        return fail(kInvalidArgument, "gdp: TMA descriptor rejected");
    }
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("gdp launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

}  // namespace cflk

using namespace cflk;

extern "C" int cflk_volta_opm_update(void* stream, int dtype, const void* lhs, const void* t,
                                     const float* bias, const float* norm, const void* residual,
                                     void* out, int64_t B, int64_t K, int64_t D, int64_t F,
                                     float eps) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "opm_update: dtype must be f16 or bf16");
    }
    if (B < 0 || K < 0 || D < 0 || F < 0) {
        return fail(kInvalidArgument, "opm_update: lhs must be [B,K] and t [K,D,F]");
    }
    if (K % 32 || (F != 16 && F != 32 && F != 64 && F != 128) || D > 65535) {
        return fail(kInvalidArgument,
                    "opm_update: K must be a multiple of 32, F 16, 32, 64 or 128, D at most 65535");
    }
    if (B == 0 || D == 0) {
        return kOk;
    }
    if (B >= (int64_t(1) << 31) || K >= (int64_t(1) << 31) || D * F >= (int64_t(1) << 31)) {
        return fail(kInvalidArgument, "opm_update: sizes must be below 2^31");
    }
    if (!aligned16(lhs) || !aligned16(t) || !aligned16(out) ||
        (residual != nullptr && !aligned16(residual)) || bias == nullptr || norm == nullptr) {
        return fail(kInvalidArgument, "opm_update: buffers must be 16-byte aligned");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (K == 0) {
        const long long total = B * D * F;
        const unsigned grid = (unsigned)std::min<long long>((total + 255) / 256, 148 * 8);
        if (dtype == kBF16) {
            using T = __nv_bfloat16;
            opm_update_k0_kernel<T><<<grid, 256, 0, s>>>(bias, norm, static_cast<const T*>(residual),
                                                         static_cast<T*>(out), total, (int)(D * F),
                                                         (int)F, eps);
        } else {
            using T = __half;
            opm_update_k0_kernel<T><<<grid, 256, 0, s>>>(bias, norm, static_cast<const T*>(residual),
                                                         static_cast<T*>(out), total, (int)(D * F),
                                                         (int)F, eps);
        }
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? kOk
                                : fail(kInternal, std::string("opm_update launch: ") + cudaGetErrorString(e));
    }
    if (((B + GBM - 1) / GBM) * ((D * F + 127) / 128) >= (int64_t(1) << 31)) {
        return fail(kInvalidArgument, "opm_update: too many output tiles");
    }
    GemmArgs a{};
    a.batch = 1;
    a.M = (int)B;
    a.N = (int)(D * F);
    a.K = (int)K;
    a.bias_f = bias;
    a.norm = norm;
    a.residual = residual;
    a.F = (int)F;
    a.D = (int)D;
    a.eps = eps;
    bool ok = true;
    const cudaError_t e =
        dtype == kBF16 ? launch_gemm<__nv_bfloat16, kOpmUpdate, false, true>(s, dtype, lhs, t, nullptr, out, a, ok)
                       : launch_gemm<__half, kOpmUpdate, false, true>(s, dtype, lhs, t, nullptr, out, a, ok);
    if (!ok) {
        return fail(kInvalidArgument, "opm_update: TMA descriptor rejected");
    }
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("opm_update launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

extern "C" int cflk_trimul_contract(void* stream, int dtype, const void* a, const void* b,
                                    float* out, int64_t C, int64_t I, int64_t J, int64_t K,
                                    int incoming) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "trimul_contract: dtype must be f16 or bf16");
    }
    if (C < 0 || I < 0 || J < 0 || K < 0) {
        return fail(kInvalidArgument, "trimul_contract: sizes must be non-negative");
    }
    if (incoming != 0 && incoming != 1) {
        return fail(kInvalidArgument, "trimul_contract: incoming is 0 or 1");
    }
    if (C == 0 || I == 0 || J == 0) {
        return kOk;
    }
    if (C > 65535 || I >= (int64_t(1) << 31) || J >= (int64_t(1) << 31) ||
        K >= (int64_t(1) << 31)) {
        return fail(kInvalidArgument,
                    "trimul_contract: C at most 65535, I, J and K below 2^31");
    }
    if (out == nullptr || (K > 0 && (a == nullptr || b == nullptr))) {
        return fail(kInvalidArgument, "trimul_contract: null buffer");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (K == 0) {
        const cudaError_t e = cudaMemsetAsync(out, 0, (size_t)(C * I * J) * sizeof(float), s);
        return e == cudaSuccess ? kOk
                                : fail(kInternal, std::string("trimul_contract: ") +
                                                      cudaGetErrorString(e));
    }
    // TMA wants 16-byte rows: the k-major rows (outgoing) or the i and j rows (incoming) a
    // multiple of 8 elements, the float32 output rows of 4
    const bool rows16 = incoming ? (I % 8 == 0 && J % 8 == 0) : (K % 8 == 0);
    const bool tma = rows16 && J % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out) &&
                     ((I + GBM - 1) / GBM) * ((J + 255) / 256) * C < (int64_t(1) << 31);
    cudaError_t e = cudaSuccess;
    if (tma) {
        GemmArgs g{};
        g.batch = (int)C;
        g.M = (int)I;
        g.N = (int)J;
        g.K = (int)K;
        bool ok = true;
        if (dtype == kBF16) {
            using T = __nv_bfloat16;
            e = incoming ? launch_gemm<T, kContract, true, true>(s, dtype, a, b, nullptr, out, g, ok)
                         : launch_gemm<T, kContract, false, false>(s, dtype, a, b, nullptr, out, g,
                                                                   ok);
        } else {
            using T = __half;
            e = incoming ? launch_gemm<T, kContract, true, true>(s, dtype, a, b, nullptr, out, g, ok)
                         : launch_gemm<T, kContract, false, false>(s, dtype, a, b, nullptr, out, g,
                                                                   ok);
        }
        if (!ok) {
            return fail(kInvalidArgument, "trimul_contract: TMA descriptor rejected");
        }
    } else {
        const dim3 grid((unsigned)((J + 63) / 64), (unsigned)((I + 63) / 64), (unsigned)C);
        if (grid.y > 65535u) {
            return fail(kInvalidArgument,
                        "trimul_contract: I must be below 4194240 when rows are not 16-byte "
                        "multiples");
        }
#define CFLK_CONTRACT_SIMT(T)                                                                   \
    (incoming ? contract_simt_kernel<T, true><<<grid, 256, 0, s>>>(                             \
                    static_cast<const T*>(a), static_cast<const T*>(b), out, (int)I, (int)J,   \
                    (int)K)                                                                    \
              : contract_simt_kernel<T, false><<<grid, 256, 0, s>>>(                            \
                    static_cast<const T*>(a), static_cast<const T*>(b), out, (int)I, (int)J,   \
                    (int)K))
        if (dtype == kBF16) {
            CFLK_CONTRACT_SIMT(__nv_bfloat16);
        } else {
            CFLK_CONTRACT_SIMT(__half);
        }
#undef CFLK_CONTRACT_SIMT
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("trimul_contract launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

namespace {

constexpr size_t kOpmOuterChunkBytes = size_t(64) << 20;  // G2 per chunk: stays in L2

// b rows a chunk must hold whole: a stage-1 tile covers 128 / C values of b
int64_t opm_outer_block(int64_t C) {
    return (C == 16 || C == 32 || C == 64 || C == 128) ? 128 / C : 1;
}

}  // namespace

extern "C" int cflk_volta_opm_outer_workspace_size(int64_t B, int64_t C, int64_t D, int64_t E,
                                                   size_t* bytes) {
    clear_error();
    if (bytes == nullptr || B < 0 || C < 0 || D < 0 || E != 32) {
        return fail(kInvalidArgument, "opm_outer: left must be [16,B,C], right [16,D,E], E 32");
    }
    int64_t per_b = 0;
    if (__builtin_mul_overflow(D, C * E * 2, &per_b)) {
        return fail(kInvalidArgument, "opm_outer: workspace size overflows");
    }
    if (C == 32) {
        *bytes = size_t(128) * 32 * 32 * 2;  // the fused kernel: wT laid out (F at most 128)
        return kOk;
    }
    if (per_b == 0 || B == 0) {
        *bytes = 0;
        return kOk;
    }
    const int64_t blk = opm_outer_block(C);
    int64_t bc = (int64_t)(kOpmOuterChunkBytes / (size_t)per_b) / blk * blk;
    bc = std::max(bc, blk);
    bc = std::min(bc, B);
    int64_t total = 0;
    if (__builtin_mul_overflow(bc, per_b, &total)) {
        return fail(kInvalidArgument, "opm_outer: workspace size overflows");
    }
    *bytes = (size_t)total;
    return kOk;
}

extern "C" int cflk_volta_opm_outer(void* stream, int dtype, const void* left, const void* right,
                                    const void* wT, void* out, int64_t B, int64_t C, int64_t D,
                                    int64_t E, int64_t F, void* workspace, size_t ws_bytes) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "opm_outer: dtype must be f16 or bf16");
    }
    if (B < 0 || C < 0 || D < 0 || E < 0 || F < 0) {
        return fail(kInvalidArgument,
                    "opm_outer: left must be [16,B,C], right [16,D,E], wT [F,C*E]");
    }
    if (C % 16 || E != 32 || D % 4 || D / 4 > 65535 ||
        (F != 16 && F != 32 && F != 64 && F != 128)) {
        return fail(kInvalidArgument,
                    "opm_outer: C a multiple of 16, E 32, D a multiple of 4, F 16, 32, 64 or 128");
    }
    if (B == 0 || D == 0 || C == 0) {
        return kOk;
    }
    const int64_t blk = opm_outer_block(C);
    if (blk == 1 && C > 512) {
        return fail(kInvalidArgument, "opm_outer: C above 512 must be 16, 32, 64 or 128");
    }
    if (B * C >= (int64_t(1) << 31) || B * D >= (int64_t(1) << 31) ||
        D * 32 >= (int64_t(1) << 31)) {
        return fail(kInvalidArgument, "opm_outer: sizes must be below 2^31");
    }
    if (!aligned16(left) || !aligned16(right) || !aligned16(wT) || !aligned16(out) ||
        !aligned16(workspace)) {
        return fail(kInvalidArgument, "opm_outer: buffers must be 16-byte aligned");
    }
    if (C == 32) {
        return opm_outer_fused(stream, dtype, left, right, wT, out, B, D, F, workspace, ws_bytes);
    }
    const int64_t per_b = D * C * 64;  // G2 bytes of one b
    // b rows a chunk: all of them, or whole multiples of 128 / C
    int64_t bc = (int64_t)(ws_bytes / (size_t)per_b);
    bc = bc >= B ? B : bc / blk * blk;
    if (bc <= 0) {
        return fail(kInvalidArgument,
                    "opm_outer: workspace below one chunk (cflk_volta_opm_outer_workspace_size)");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const auto run = [&](auto tag) -> cudaError_t {
        using T = decltype(tag);
        for (int64_t b0 = 0; b0 < B; b0 += bc) {
            const int64_t nb = std::min(bc, B - b0);
            bool ok = true;
            cudaError_t e = cudaSuccess;
            if (blk > 1) {
                GemmArgs g{};
                g.batch = 1;
                g.M = (int)(nb * C);
                g.N = (int)(D * 32);
                g.K = 16;
                g.opm_c = (int)C;
                g.lda = B * C;
                e = launch_gemm<T, kOpmOuterG, true, true>(
                    s, dtype, static_cast<const T*>(left) + b0 * C, right, nullptr, workspace, g,
                    ok);
            } else {
                const dim3 grid((unsigned)D, (unsigned)nb);
                opm_outer_g_simt_kernel<T><<<grid, 256, (size_t)(16 * C + 512) * sizeof(float),
                                             s>>>(static_cast<const T*>(left),
                                                  static_cast<const T*>(right),
                                                  static_cast<T*>(workspace), (int)B, (int)C,
                                                  (int)D, (int)b0);
                e = cudaGetLastError();
            }
            if (!ok) {
                return cudaErrorInvalidValue;
            }
            if (e != cudaSuccess) {
                return e;
            }
            GemmArgs g2{};
            g2.batch = 1;
            g2.M = (int)(nb * D);
            g2.N = (int)F;
            g2.K = (int)(C * 32);
            e = launch_gemm<T, kPlain, false, false>(s, dtype, workspace, wT, nullptr,
                                                    static_cast<T*>(out) + b0 * D * F, g2, ok);
            if (!ok) {
                return cudaErrorInvalidValue;
            }
            if (e != cudaSuccess) {
                return e;
            }
        }
        return cudaSuccess;
    };
    const cudaError_t e = dtype == kBF16 ? run(__nv_bfloat16{}) : run(__half{});
    if (e == cudaErrorInvalidValue) {
        return fail(kInvalidArgument, "opm_outer: TMA descriptor rejected");
    }
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("opm_outer launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

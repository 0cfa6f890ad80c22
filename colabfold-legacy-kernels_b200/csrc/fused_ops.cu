// LayerNorm-folded pair-stack fusions for sm_100a: VoltaLnGdp, VoltaLnProj, VoltaOutProj,
// VoltaTrimulEpilogue, VoltaTransition (colabfold-legacy-kernels cuda/volta_fused_ffi.h:42-259,
// kernels cuda/volta_ops.cu:330-641). All run on the persistent row-tile pipeline of
// fused_common.cuh: TMA-fed 128-row tiles, resident weights, tcgen05 MMAs into tensor memory,
// LayerNorm prologue and epilogue in two worker warpgroups.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "capi_internal.h"
#include "cflk_b200.h"
#include "fused_common.cuh"
#include "tmap.h"

namespace cflk {
namespace {

__device__ unsigned g_status;

using namespace fused;

// ---------------------------------------------------------------------------------------------
// the pipeline
// ---------------------------------------------------------------------------------------------
// The accumulators live in a ring of Op::kSlots blocks of Op::kSlotCols tensor-memory columns: the MMA
// warp fills block j+1.. while the workers drain block j, so neither side waits for a whole
// tile. With Op::kPingPong the Op::kWorkerGroups worker warpgroups (two or three) take the
// tiles in turn (tile c to warpgroup c % kWorkerGroups, in x stage c % kStages), each doing a
// tile's whole prologue and epilogue, so one tile's LayerNorm overlaps another's epilogue;
// otherwise two warpgroups split every tile.
// Op supplies: T, Args (M, w_bytes, param_floats, eps), keep(), kOther, X_BYTES,
// RED_FLOATS, STORE_BYTES, nblocks(), load_params, load_weights, load_x, issue_block, prologue,
// epilogue_block, prefetch_block, padding, Regs, bind, finish, kPingPong, kWorkerGroups,
// kSlots, kSlotCols.
// STORE_BYTES of 1024-byte-aligned shared memory after the others are the op's output staging
// (TMA stores through the map `to`), handed to Op::bind with the map.

// Worker warpgroups and threads of an op's launch; the producer warp follows the workers. With
// three worker warpgroups (416 threads) a thread has at most 128 registers: an SM sub-partition
// holds four of the thirteen warps.
template <class Op>
struct Crew {
    static constexpr int kGroups = Op::kWorkerGroups;
    static constexpr int kWorkerThreads = 128 * kGroups;
    static constexpr int kProducer = 4 * kGroups;
    static constexpr int kThreads = kWorkerThreads + 32;
    static_assert(kGroups == 2 || (kGroups == 3 && Op::kPingPong), "worker warpgroups");
    // ping-pong: every stage serves one warpgroup only, so no waiter on a stage's barriers can
    // run a phase ahead (a warpgroup meets its stages in its own order)
    static_assert(!Op::kPingPong || Op::kStages % kGroups == 0, "stages per warpgroup");
};

template <class Op>
__global__ void __launch_bounds__(Crew<Op>::kThreads, 1)
    row_tile_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw0,
                    const __grid_constant__ CUtensorMap tw1,
                    const __grid_constant__ CUtensorMap to,
                    const __grid_constant__ CUtensorMap to1, const typename Op::Args a) {
    constexpr int kSlots = Op::kSlots, kSlotCols = Op::kSlotCols;
    // x stages: tile c in stage c % kStages; three where shared memory leaves room (the load of
    // tile c + 3 starts as soon as tile c's MMAs are done, a whole tile before a worker needs
    // it), two, or one where a stage is too large for two
    constexpr int kStages = Op::kStages;
    static_assert(kStages == 2 || kStages == 3 || (kStages == 1 && !Op::kPingPong), "stages");
    constexpr int kStageBars = kStages > 2 ? kStages : 2;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xs0 = smem;
    uint8_t* ws = smem + kStages * Op::X_BYTES;
    float* sp = reinterpret_cast<float*>(ws + a.w_bytes);
    float* red = sp + a.param_floats;  // [Op::RED_FLOATS]
    uint8_t* stb = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(red + Op::RED_FLOATS) + 1023) & ~uintptr_t(1023));
    // accumulator slot barriers per warpgroup that consumes the slot's block (both ping-pong
    // warpgroups pass blocks through the same slots; one barrier each keeps every barrier's
    // phases in one consumer's order, so no waiter can be two phases ahead)
    constexpr int kTeams = Op::kPingPong ? Crew<Op>::kGroups : 1;
    constexpr int kProducerWarp = Crew<Op>::kProducer;
    __shared__ uint64_t x_full[kStageBars], x_empty[kStageBars], a_ready[kStageBars],
        acc_full[kTeams][kSlots],
        acc_empty[kTeams][kSlots], w_full;
    __shared__ uint32_t tmem_sh;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (a.M + BM - 1) / BM;
    const int nb = Op::nblocks(a);
    if (warp == kProducerWarp) {
        if (lane == 0) {
            // ping-pong ops: one worker warpgroup per tile (the two take the tiles in turn)
            constexpr int kTeam = Op::kPingPong ? 128 : Crew<Op>::kWorkerThreads;
            for (int i = 0; i < kStageBars; ++i) {
                mbar_init(&x_full[i], 1);
                mbar_init(&x_empty[i], 1);
                mbar_init(&a_ready[i], kTeam);
            }
            for (int tm = 0; tm < kTeams; ++tm) {
                for (int i = 0; i < kSlots; ++i) {
                    mbar_init(&acc_full[tm][i], 1);
                    mbar_init(&acc_empty[tm][i], kTeam);
                }
            }
            mbar_init(&w_full, 1);
            abort_flag = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&tmem_sh, kSlots * kSlotCols);
        tmem_relinquish();
    } else if (warp < kProducerWarp) {
        Op::load_params(a, sp, ws, threadIdx.x);
        fence_async_smem();  // weight rows the workers wrote, read by the MMA
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;

    if (warp == kProducerWarp) {
        const auto next = [&](int& cursor) -> int {
            while (cursor < ntiles) {
                const int m0 = cursor * BM;
                cursor += gridDim.x;
                if (tile_work(Op::keep(a), a.M, m0, Op::kOther) == kCompute) {
                    return m0;
                }
            }
            return -1;
        };
        int cur = blockIdx.x, pcur = blockIdx.x, c = 0, q = 0;
        // parity of the acc_empty phases waited for, one bit per (team, slot): a register, not
        // a dynamically indexed array (which would live in local memory)
        uint32_t empty_par = 0;
        if (lane == 0) {
            Op::load_weights(a, &tw0, &tw1, ws, &w_full);
        }
        for (int k = 0; k < kStages; ++k) {
            const int m = next(pcur);
            if (m < 0) {
                break;
            }
            if (lane == 0) {
                Op::load_x(a, &tx, &to1, xs0 + k * Op::X_BYTES, &x_full[k], m);
            }
        }
        bool weights_ready = false;
        while (true) {
            const int m = next(cur);
            if (m < 0) {
                break;
            }
            const int s = c % kStages, sph = (c / kStages) & 1;
            if (lane == 0) {
                if (!weights_ready) {
                    mbar_wait(&w_full, 0, &g_status, kStatusTmaWait, &abort_flag);
                    weights_ready = true;
                }
                mbar_wait(&a_ready[s], sph, &g_status, kStatusSyncWait, &abort_flag);
                tc_fence_after();
                const int team = c % kTeams;
                for (int j = 0; j < nb; ++j, ++q) {
                    const int slot = q % kSlots;
                    if (q >= kSlots) {
                        // the slot's previous block: consumed by its warpgroup (the n-th of that
                        // warpgroup's blocks in this slot completes the barrier's n-th phase)
                        const int pt = ((q - kSlots) / nb) % kTeams;
                        const int bit = pt * kSlots + slot;
                        mbar_wait(&acc_empty[pt][slot], (empty_par >> bit) & 1, &g_status,
                                  kStatusSyncWait, &abort_flag);
                        empty_par ^= 1u << bit;
                        tc_fence_after();
                    }
                    Op::issue_block(a, smem_u32(xs0 + s * Op::X_BYTES), smem_u32(ws),
                                    tmem + slot * kSlotCols, j);
                    mma_commit(&acc_full[team][slot]);
                }
                mma_commit(&x_empty[s]);
            } else {
                q += nb;
            }
            __syncwarp();
            const int m2 = next(pcur);
            if (m2 >= 0) {
                if (lane == 0) {
                    mbar_wait(&x_empty[s], sph, &g_status, kStatusMmaWait, &abort_flag);
                    Op::load_x(a, &tx, &to1, xs0 + s * Op::X_BYTES, &x_full[s], m2);
                }
            }
            __syncwarp();
            ++c;
        }
    } else if (warp < kProducerWarp) {
        const int g = warp >> 2, t = ((warp & 3) << 5) | lane;
        const uint32_t lane_base = tmem_lane_base(warp);
        typename Op::Regs regs{};
        Op::bind(regs, stb, warp);
        int c = 0, q = 0;
        uint32_t full_par = 0;  // parity of the acc_full phases this warpgroup waited for, per slot
        // the keep values of the worker's next tile load a tile ahead (the classification's
        // global loads would otherwise stall every tile); a worker's own row value is also
        // handed to the op (ln_gdp's row mask)
        float kv[BM / 32];
        keep_load(Op::keep(a), a.M, blockIdx.x * BM, Op::kOther, kv);
        for (int cursor = blockIdx.x; cursor < ntiles; cursor += gridDim.x) {
            const int m0 = cursor * BM;
            const int work = tile_work_of(kv);
            Op::row_keep(regs, kv[warp & 3]);
            keep_load(Op::keep(a), a.M, m0 + gridDim.x * BM, Op::kOther, kv);
            if (work == kPadding) {
                Op::padding(a, m0, t, g);
                continue;
            }
            if (work == kSkip) {
                continue;
            }
            const int s = c % kStages, sph = (c / kStages) & 1;
            if constexpr (Op::kPingPong) {
                if (c % kTeams != g) {  // another warpgroup's tile
                    q += nb;
                    ++c;
                    continue;
                }
            }
            uint8_t* stage = xs0 + s * Op::X_BYTES;
            mbar_wait(&x_full[s], sph, &g_status, kStatusTmaWait, &abort_flag);
            Op::prologue(a, stage, sp, red, t, g, m0, regs);
            fence_async_smem();
            mbar_arrive(&a_ready[s]);
            const int team = kTeams > 1 ? g : 0;
            for (int j = 0; j < nb; ++j, ++q) {
                const int slot = q % kSlots;
                // global inputs of the block's epilogue start loading before the MMA wait
                Op::prefetch_block(a, t, g, m0, j, regs);
                // this warpgroup's blocks in the slot so far, modulo 2
                mbar_wait(&acc_full[team][slot], (full_par >> slot) & 1, &g_status, kStatusMmaWait,
                          &abort_flag);
                full_par ^= 1u << slot;
                tc_fence_after();
                Op::epilogue_block(a, tmem + slot * kSlotCols + lane_base, sp, t, g, m0, j, regs,
                                   &to, &to1);
                tc_fence_before();
                mbar_arrive(&acc_empty[team][slot]);
            }
            ++c;
        }
        Op::finish(regs, lane);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kProducerWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kSlots * kSlotCols);
    }
}

// TMA of the K columns of rows [m0, m0+128) of a row-major [M][K] map as 64-column atoms
__device__ __forceinline__ void load_rows_tile(const CUtensorMap* map, uint8_t* dst,
                                               uint64_t* bar, int K, int m0) {
    mbar_arrive_expect_tx(bar, (uint32_t)(K * BM * 2));
    for (int a = 0; a < K / 64; ++a) {
        tma_load_2d(dst + a * ATOM, map, bar, a * 64, m0);
    }
}

// Rows of one TMA box of a weight matrix: the largest of 256, 128, 64 that divides rows (a
// multiple of 64), so that boxes tile the matrix exactly.
__host__ __device__ __forceinline__ int weight_box(int rows) {
    return rows % 256 == 0 ? 256 : rows % 128 == 0 ? 128 : 64;
}

// TMA of a whole weight matrix [rows][K] (row-major) into 64-column atoms of `rows` rows
__device__ __forceinline__ void load_weight(const CUtensorMap* map, uint8_t* dst, uint64_t* bar,
                                            int rows, int K) {
    const int box = weight_box(rows);
    for (int a = 0; a < K / 64; ++a) {
        for (int r0 = 0; r0 < rows; r0 += box) {
            tma_load_2d(dst + a * rows * 128 + r0 * 128, map, bar, a * 64, r0);
        }
    }
}

// D[128 x N] (+)= A[128 x K] W^T for W [rows][K] staged by load_weight, output columns
// [n0, n0 + N), N <= 256 and a multiple of 16
__device__ __forceinline__ void mma_rows(uint32_t d, uint32_t a_base, uint32_t w_base, int rows,
                                         int K, int n0, int N, bool bf16, bool accumulate) {
    const uint32_t id = idesc_f16(bf16, 128, N, false, false);
    for (int k = 0; k < K / 16; ++k) {
        const int at = k >> 2, off = (k & 3) * 32;
        mma_ss(d, desc_k128(a_base + at * ATOM + off),
               desc_k128(w_base + at * rows * 128 + n0 * 128 + off), id,
               (accumulate || k > 0) ? 1u : 0u);
    }
}

// D[128 x 128] = W[c0, c0 + 128) A^T for W [rows][K] staged by load_weight and the row tile A:
// the transposed product, TMEM lanes are output channels and columns are the tile's rows
__device__ __forceinline__ void mma_cols(uint32_t d, uint32_t w_base, int rows, int c0,
                                         uint32_t a_base, int K, bool bf16) {
    const uint32_t id = idesc_f16(bf16, 128, 128, false, false);
    for (int k = 0; k < K / 16; ++k) {
        const int at = k >> 2, off = (k & 3) * 32;
        mma_ss(d, desc_k128(w_base + at * rows * 128 + c0 * 128 + off),
               desc_k128(a_base + at * ATOM + off), id, k > 0 ? 1u : 0u);
    }
}

// ---------------------------------------------------------------------------------------------
// VoltaLnGdp: left/right [CI, M] = max(mask, 0) * (y wp + bp) * sigmoid(y wg + bg), y = LN(x)
// ---------------------------------------------------------------------------------------------
template <typename T_, int K, int CI>
struct LnGdpOp {
    using T = T_;
    using E = Elem<T>;
    static constexpr int P = 2 * CI;
    // three x stages where the weights leave room (CI = 64: 64 KB of weights)
    static constexpr int kStages = CI <= 64 ? 3 : 2;
    static constexpr int X_BYTES = K * BM * 2;
    static constexpr float kOther = 0.f;
    static constexpr bool kPingPong = true;
    // with three stages, three warpgroups take the tiles in turn: twelve worker warps keep more
    // of the LayerNorm's and the epilogue's latency covered than eight
    static constexpr int kWorkerGroups = kStages;
    // the tile's row mask max(mask, 0): per warpgroup two buffers (its tile parity)
    static constexpr int RED_FLOATS = 2 * kWorkerGroups * BM;
    // the outputs are channel major, so the product is computed transposed (lanes = channels):
    // a block is 128 channels, the projection in the slot's columns [0, 128) and the gate in
    // [128, 256), one column per row of the tile
    static constexpr int kSlots = 2, kSlotCols = 256;
    // output staging when M % 8 == 0 (TMA row strides): per worker warp one 2 KB box buffer
    // for CI = 128 (its weights fill shared memory), two for CI = 64
    using Stager = RowChunkStager<CI <= 64 ? 2 : 1>;
    static constexpr int STORE_BYTES = 4 * kWorkerGroups * Stager::BYTES;
    struct Args {
        const T *x, *wpT, *bp, *wgT, *bg, *mask;
        const float *scale, *offset;
        T *left, *right;
        int M, w_bytes, param_floats, vec_store;
        int tma_out;  // outputs through the staging buffers and TMA stores (maps to, to1)
        float eps;
    };
    struct Regs {
        const float* maskv;  // this tile's row mask (shared memory)
        int parity;
        float row_mask;      // this worker's row of the mask, from the tile classification
        Stager st;
    };
    static __device__ void bind(Regs& r, uint8_t* stb, int warp) {
        r.st.base = smem_u32(stb) + warp * Stager::BYTES;
        r.st.n = 0;
    }
    static __device__ void finish(Regs& r, int lane) { r.st.finish(lane); }
    static __device__ void row_keep(Regs& r, float v) { r.row_mask = v; }
    static __device__ const T* keep(const Args& a) { return a.mask; }
    // scale [K], offset [K], bp [P], bg [P]
    static __device__ void load_params(const Args& a, float* sp, uint8_t*, int tid) {
        for (int i = tid; i < K; i += kWorkers) {
            sp[i] = a.scale[i];
            sp[K + i] = a.offset[i];
        }
        for (int i = tid; i < P; i += kWorkers) {
            sp[2 * K + i] = E::to_f(a.bp[i]);
            sp[2 * K + P + i] = E::to_f(a.bg[i]);
        }
    }
    static __device__ void load_weights(const Args& a, const CUtensorMap* tw0,
                                        const CUtensorMap* tw1, uint8_t* ws, uint64_t* bar) {
        mbar_arrive_expect_tx(bar, (uint32_t)(2 * P * K * 2));
        load_weight(tw0, ws, bar, P, K);
        load_weight(tw1, ws + P * K * 2, bar, P, K);
    }
    static __device__ void load_x(const Args& a, const CUtensorMap* tx, const CUtensorMap*,
                                  uint8_t* dst, uint64_t* bar, int m0) {
        load_rows_tile(tx, dst, bar, K, m0);
    }
    // block j: output channels [128j, 128j + 128) of the P
    static __device__ int nblocks(const Args&) { return P / 128; }
    static __device__ void issue_block(const Args& a, uint32_t xa, uint32_t wa, uint32_t acc,
                                       int j) {
        mma_cols(acc, wa, P, 128 * j, xa, K, E::kBf16);
        mma_cols(acc + 128, wa + P * K * 2, P, 128 * j, xa, K, E::kBf16);
    }
    // warpgroup g's tile: LayerNorm of row t (the whole row), the row mask into shared memory
    // (two buffers a warpgroup: its previous tile's epilogue may still read the other one),
    // then a barrier of the warpgroup, whose epilogue threads read every row's mask
    static __device__ void prologue(const Args& a, uint8_t* stage, const float* sp, float* red,
                                    int t, int g, int m0, Regs& regs) {
        float* mv = red + (2 * g + regs.parity) * BM;
        mv[t] = m0 + t < a.M ? fmaxf(regs.row_mask, 0.f) : 0.f;
        regs.maskv = mv;
        regs.parity ^= 1;
        if constexpr (kWorkerGroups == 3) {
            // three passes over the row in shared memory: the row held in registers would not
            // fit the 128 registers a thread of three worker warpgroups has
            ln_row_full<T, K>(stage, t, sp, sp + K, a.eps);
        } else {
            ln_row_regs<T, K>(stage, t, sp, sp + K, a.eps);
        }
        named_sync(2 + g, 128);
    }
    static __device__ void prefetch_block(const Args&, int, int, int, int, Regs&) {}
    // worker t of the tile's warpgroup: channel 128j + t (TMEM lane t), the tile's 128 rows in
    // four runs of 32, each stored as 64 contiguous bytes of the channel-major output
    static __device__ void epilogue_block(const Args& a, uint32_t acc, const float* sp, int t,
                                          int g, int m0, int j, Regs& regs,
                                          const CUtensorMap* to, const CUtensorMap* to1) {
        const int ch = 128 * j + t;
        const float bpv = sp[2 * K + ch], bgv = sp[2 * K + P + ch];
        T* out = ch < CI ? a.left + (long long)ch * a.M : a.right + (long long)(ch - CI) * a.M;
        // two rows an instruction (paired fp32): mask * (p + bp) * sigmoid(g + bg) with
        // sigmoid(x) = (1 + tanh(x / 2)) / 2, for 16 rows from r0
        const uint64_t bp2 = pk2(bpv, bpv), hbg2 = pk2(0.5f * bgv, 0.5f * bgv);
        const uint64_t half2 = pk2(0.5f, 0.5f);
        const auto rows16 = [&](const uint32_t (&pr)[16], const uint32_t (&gr)[16], int r0,
                                uint32_t* w) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 mk = *reinterpret_cast<const float4*>(regs.maskv + r0 + 4 * q);
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                    const int i = 4 * q + e;
                    const uint64_t pv =
                        add2(pk2(__uint_as_float(pr[i]), __uint_as_float(pr[i + 1])), bp2);
                    const float2 hg = upk2(fma2(
                        pk2(__uint_as_float(gr[i]), __uint_as_float(gr[i + 1])), half2, hbg2));
                    float t0, t1;
                    asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(hg.x));
                    asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(hg.y));
                    const uint64_t sg = fma2(pk2(t0, t1), half2, half2);
                    const uint64_t mm = e == 0 ? pk2(mk.x, mk.y) : pk2(mk.z, mk.w);
                    const float2 o = upk2(mul2(mul2(mm, pv), sg));
                    w[2 * q + e / 2] = E::pack(o.x, o.y);
                }
            }
        };
        // the tile's rows in four runs of 32, each read as two halves of 16 whose tensor-memory
        // loads run one half ahead of the arithmetic (a load is issued right after the wait for
        // the previous one)
        uint32_t pa[16], ga[16], pb[16], gb[16];
        tmem_ld16(acc, pa);
        tmem_ld16(acc + 128, ga);
        tmem_wait_ld();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
            const int r0 = 32 * cc;
            tmem_ld16(acc + r0 + 16, pb);
            tmem_ld16(acc + 128 + r0 + 16, gb);
            uint32_t w[16];
            rows16(pa, ga, r0, w);
            tmem_wait_ld();
            if (cc < 3) {
                tmem_ld16(acc + r0 + 32, pa);
                tmem_ld16(acc + 128 + r0 + 32, ga);
            }
            rows16(pb, gb, r0 + 16, w + 8);
            if (cc < 3) {
                tmem_wait_ld();
            }
            const int m = m0 + r0;
            if (m >= a.M) {
                continue;
            }
            if (a.tma_out) {
                // the warp's 32 channels x these 32 rows as one box of left or right
                const int chw = 128 * j + (t & ~31);
                regs.st.put(chw < CI ? to : to1, t & 31, w, m, chw < CI ? chw : chw - CI);
            } else if (a.vec_store == 2 && m + 32 <= a.M) {
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    st_global_v8(out + m + 16 * q,
                                 make_uint4(w[8 * q], w[8 * q + 1], w[8 * q + 2], w[8 * q + 3]),
                                 make_uint4(w[8 * q + 4], w[8 * q + 5], w[8 * q + 6], w[8 * q + 7]));
                }
            } else if (a.vec_store == 1 && m + 32 <= a.M) {
                uint4* dst = reinterpret_cast<uint4*>(out + m);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    dst[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                }
            } else {
                for (int i = 0; i < 32 && m + i < a.M; ++i) {
                    const uint32_t ww = w[i >> 1];
                    const uint16_t hv = (i & 1) ? (uint16_t)(ww >> 16) : (uint16_t)(ww & 0xffffu);
                    reinterpret_cast<uint16_t*>(out)[m + i] = hv;
                }
            }
        }
    }
    static __device__ void padding(const Args& a, int m0, int t, int g) {
        const int m = m0 + t;
        if (m >= a.M || g > 1) {  // warpgroup 0 zeroes left, 1 right
            return;
        }
        T* out = g == 0 ? a.left : a.right;
        for (int c = 0; c < CI; ++c) {
            out[(long long)c * a.M + m] = E::from_f(0.f);
        }
    }
};

// ---------------------------------------------------------------------------------------------
// VoltaGdp: out [M, N] = mask * (x wp + bp) * act(x wg + bg), act = sigmoid or swish
// g sigmoid(g), the row mask as given (cuda/volta_ops.cu:108-205; cuda/volta_gdp.h:10-19). wp and
// wg are [K, N] row-major, so they are the MMA's B operand N-major: each 64-column atom holds K
// rows of 128 bytes. Warpgroups ping-pong over tiles; a block is the whole N of both products.
// ---------------------------------------------------------------------------------------------
template <typename T_, int K>
struct GdpOp {
    using T = T_;
    using E = Elem<T>;
    static constexpr int kSlots = 2, kSlotCols = 256;
    static constexpr bool kPingPong = true;
    // three x stages (at most 64 KB of weights: K, N <= 128) and three warpgroups taking the
    // tiles in turn
    static constexpr int kStages = 3;
    static constexpr int kWorkerGroups = 3;
    static constexpr int X_BYTES = K * BM * 2;
    static constexpr float kOther = 0.f;
    static constexpr int RED_FLOATS = 4;  // unused
    using Stager = RowChunkStager<2>;
    static constexpr int STORE_BYTES = 4 * kWorkerGroups * Stager::BYTES;
    struct Args {
        const T *x, *wp, *bp, *wg, *bg, *mask;
        T* out;
        int M, N, act;  // act: 0 sigmoid, 1 swish
        int w_bytes, param_floats;
        float eps;  // unused
    };
    struct Regs {
        float mv;  // this worker's row of the mask
        Stager st;
    };
    static __device__ void bind(Regs& r, uint8_t* stb, int warp) {
        r.st.base = smem_u32(stb) + warp * Stager::BYTES;
        r.st.n = 0;
    }
    static __device__ void finish(Regs& r, int lane) { r.st.finish(lane); }
    static __device__ void row_keep(Regs&, float) {}
    static __device__ const T* keep(const Args&) { return nullptr; }
    // bp [N], bg [N]
    static __device__ void load_params(const Args& a, float* sp, uint8_t*, int tid) {
        for (int i = tid; i < a.N; i += kWorkers) {
            sp[i] = E::to_f(a.bp[i]);
            sp[a.N + i] = E::to_f(a.bg[i]);
        }
    }
    // wp then wg, each N/64 atoms of [K rows][64 columns] (box {64, K})
    static __device__ void load_weights(const Args& a, const CUtensorMap* tw0,
                                        const CUtensorMap* tw1, uint8_t* ws, uint64_t* bar) {
        mbar_arrive_expect_tx(bar, (uint32_t)(2 * K * a.N * 2));
        for (int at = 0; at < a.N / 64; ++at) {
            tma_load_2d(ws + at * K * 128, tw0, bar, at * 64, 0);
            tma_load_2d(ws + K * a.N * 2 + at * K * 128, tw1, bar, at * 64, 0);
        }
    }
    static __device__ void load_x(const Args& a, const CUtensorMap* tx, const CUtensorMap*,
                                  uint8_t* dst, uint64_t* bar, int m0) {
        load_rows_tile(tx, dst, bar, K, m0);
    }
    static __device__ int nblocks(const Args&) { return 1; }
    // x wp into the slot's columns [0, N), x wg into [N, 2N)
    static __device__ void issue_block(const Args& a, uint32_t xa, uint32_t wa, uint32_t acc,
                                       int) {
        const uint32_t id = idesc_f16(E::kBf16, 128, a.N, false, true);
        const uint32_t wg = wa + K * a.N * 2;
        for (int k = 0; k < K / 16; ++k) {
            const uint64_t ad = desc_k128(xa + (k >> 2) * ATOM + (k & 3) * 32);
            // N-major B: K steps 16 rows (2 KB) apart, 8-row groups 1024 bytes apart, the next
            // 64 columns one atom (K rows of 128 bytes) on
            mma_ss(acc, ad, smem_desc(wa + k * 16 * 128, K * 128, 1024, kSwizzle128B), id,
                   k > 0 ? 1u : 0u);
            mma_ss(acc + a.N, ad, smem_desc(wg + k * 16 * 128, K * 128, 1024, kSwizzle128B), id,
                   k > 0 ? 1u : 0u);
        }
    }
    static __device__ void prologue(const Args& a, uint8_t*, const float*, float*, int t, int,
                                    int m0, Regs& regs) {
        const int m = m0 + t;
        regs.mv = m < a.M ? E::to_f(a.mask[m]) : 0.f;
    }
    static __device__ void prefetch_block(const Args&, int, int, int, int, Regs&) {}
    // worker t: row t, 32 columns a TMEM wait and a store
    static __device__ void epilogue_block(const Args& a, uint32_t acc, const float* sp, int t,
                                          int, int m0, int, Regs& regs, const CUtensorMap* to,
                                          const CUtensorMap*) {
        const int lane = t & 31, row0 = m0 + (t & ~31);
        for (int c0 = 0; c0 < a.N; c0 += 32) {
            uint32_t rp[32], rg[32];
            tmem_ld32(acc + c0, rp);
            tmem_ld32(acc + a.N + c0, rg);
            tmem_wait_ld();
            if (row0 >= a.M) {
                continue;
            }
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                float o[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = c0 + 2 * e + h;
                    const float pv = __uint_as_float(rp[2 * e + h]) + sp[c];
                    const float gv = __uint_as_float(rg[2 * e + h]) + sp[a.N + c];
                    const float sg = sigmoid_fast(gv);
                    o[h] = regs.mv * pv * (a.act ? gv * sg : sg);
                }
                w[e] = E::pack(o[0], o[1]);
            }
            regs.st.put(to, lane, w, c0, row0);
        }
    }
    static __device__ void padding(const Args&, int, int, int) {}
};

// ---------------------------------------------------------------------------------------------
// VoltaLnProj (LN = true): p [M, n] = LN(x) w, bias [heads, M] = (LN(x) wb)^T
// VoltaOutProj (LN = false): out [M, n] = o w + b (+ residual)
// One launch covers output columns [0, n) of a pass, n <= 512, p's row stride ldp. G worker
// warpgroups take the tiles in turn, with as many x stages (two: three measured slower for the
// output projection, whose residual registers then spill).
// ---------------------------------------------------------------------------------------------
template <typename T_, int K, bool LN, int G = 2>
struct ProjOp {
    using T = T_;
    using E = Elem<T>;
    static constexpr int kSlots = 4, kSlotCols = 128;
    static constexpr bool kPingPong = true;
    static constexpr int kWorkerGroups = G;
    static constexpr int kStages = G;
    static constexpr int X_BYTES = K * BM * 2;
    static constexpr float kOther = -1.f;
    static constexpr int RED_FLOATS = 4;  // unused: a row's LayerNorm is one thread's
    // output staging: per worker warp one 2 KB box buffer for ln_projection (its weights fill
    // shared memory), two for output_projection
    using Stager = RowChunkStager<LN ? 1 : 2>;
    static constexpr int STORE_BYTES = 4 * G * Stager::BYTES;
    struct Args {
        const T *x, *wT, *b, *residual, *wbT, *keep;
        const float *scale, *offset;
        T *out, *bias;
        int M, n, ldp, heads;
        int hp;  // weight rows of the head bias after the n projection rows: 16 with heads, else 0
        int w_bytes, param_floats;
        float eps;
    };
    struct Regs {
        uint4 res[8];  // the residual part of the next block (up to 64 columns)
        Stager st;
    };
    static __device__ void bind(Regs& r, uint8_t* stb, int warp) {
        r.st.base = smem_u32(stb) + warp * Stager::BYTES;
        r.st.n = 0;
    }
    static __device__ void finish(Regs& r, int lane) { r.st.finish(lane); }
    static __device__ void row_keep(Regs&, float) {}
    static __device__ const T* keep(const Args& a) { return a.keep; }
    // scale [K], offset [K], b [n]; with heads, the head weights wb [heads][K] as weight rows
    // [n, n + 16) of every 64-column atom (rows past heads zero), so the MMA computes the
    // per-head bias of the rounded LN(x) as 16 more output columns
    static __device__ void load_params(const Args& a, float* sp, uint8_t* ws, int tid) {
        for (int i = tid; i < K; i += kWorkers) {
            sp[i] = LN ? a.scale[i] : 0.f;
            sp[K + i] = LN ? a.offset[i] : 0.f;
        }
        for (int i = tid; i < a.n; i += kWorkers) {
            sp[2 * K + i] = a.b != nullptr ? E::to_f(a.b[i]) : 0.f;
        }
        if (a.hp > 0) {
            const int rows = a.n + a.hp;
            const uint16_t* wb = reinterpret_cast<const uint16_t*>(a.wbT);
            for (int i = tid; i < 16 * K; i += kWorkers) {
                const int r = i / K, c = i % K;
                *reinterpret_cast<uint16_t*>(ws + sw128_rows(rows, a.n + r, c)) =
                    r < a.heads ? wb[(long long)r * K + c] : (uint16_t)0;
            }
        }
    }
    static __device__ void load_weights(const Args& a, const CUtensorMap* tw0,
                                        const CUtensorMap*, uint8_t* ws, uint64_t* bar) {
        mbar_arrive_expect_tx(bar, (uint32_t)(a.n * K * 2));
        if (a.n > 0) {
            const int rows = a.n + a.hp, box = weight_box(a.n);
            for (int at = 0; at < K / 64; ++at) {
                for (int r0 = 0; r0 < a.n; r0 += box) {
                    tma_load_2d(ws + at * rows * 128 + r0 * 128, tw0, bar, at * 64, r0);
                }
            }
        }
    }
    static __device__ void load_x(const Args& a, const CUtensorMap* tx, const CUtensorMap*,
                                  uint8_t* dst, uint64_t* bar, int m0) {
        load_rows_tile(tx, dst, bar, K, m0);
    }
    // block j < nb: output columns [128j, 128j + 128) (the last one 64 wide when n % 128 == 64);
    // with heads, block nb is the 16 head-bias columns
    static __device__ int nmain(const Args& a) { return (a.n + 127) / 128; }
    static __device__ int nblocks(const Args& a) { return nmain(a) + (a.hp > 0 ? 1 : 0); }
    static __device__ void issue_block(const Args& a, uint32_t xa, uint32_t wa, uint32_t acc,
                                       int j) {
        const int rows = a.n + a.hp;
        if (j == nmain(a)) {
            mma_rows(acc, xa, wa, rows, K, a.n, 16, E::kBf16, false);
            return;
        }
        const int n0 = 128 * j, N = a.n - n0 < 128 ? a.n - n0 : 128;
        mma_rows(acc, xa, wa, rows, K, n0, N, E::kBf16, false);
    }
    // warpgroup g's tile: LayerNorm of row t (the whole row), written back rounded to T
    static __device__ void prologue(const Args& a, uint8_t* stage, const float* sp, float* red,
                                    int t, int g, int m0, Regs&) {
        if constexpr (LN) {
            // the row held in registers (fits the 168 registers of two worker warpgroups)
            ln_row_regs<T, K>(stage, t, sp, sp + K, a.eps);
        }
    }
    // the residual of row t's first 64 columns of block j, loaded ahead of the MMA wait
    static __device__ void prefetch_block(const Args& a, int t, int g, int m0, int j,
                                          Regs& regs) {
        if constexpr (!LN) {
            const int m = m0 + t;
            if (a.residual == nullptr || m >= a.M || j >= nmain(a)) {
                return;
            }
            const int width = a.n - 128 * j < 128 ? a.n - 128 * j : 128;
            const uint4* rr =
                reinterpret_cast<const uint4*>(a.residual + (long long)m * a.ldp + 128 * j);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (8 * i < width) {
                    regs.res[i] = rr[i];
                }
            }
        }
    }
    // worker t of the tile's warpgroup: row t, every column 128j + [0, w) of the block's width
    // w, 32 columns at a time through the warp's staging buffer and TMA stores
    static __device__ void epilogue_block(const Args& a, uint32_t acc, const float* sp, int t,
                                          int g, int m0, int j, Regs& regs,
                                          const CUtensorMap* to, const CUtensorMap* to1) {
        const int m = m0 + t, lane = t & 31;
        if (j == nmain(a)) {
            // the head bias: columns h < heads, bias [heads, M] (a warp's 32 rows contiguous)
            uint32_t r[16];
            tmem_ld16(acc, r);
            tmem_wait_ld();
            if (m < a.M) {
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    if (h < a.heads) {
                        a.bias[(long long)h * a.M + m] = E::from_f(__uint_as_float(r[h]));
                    }
                }
            }
            return;
        }
        const int width = a.n - 128 * j < 128 ? a.n - 128 * j : 128;
        const float* b = sp + 2 * K + 128 * j;
        const int row0 = m0 + (t & ~31);
        // the residual of columns [64, 128) loads while the first 64 are done
        uint4 res2[8];
        if constexpr (!LN) {
            if (a.residual != nullptr && m < a.M && width > 64) {
                const uint4* rr = reinterpret_cast<const uint4*>(
                    a.residual + (long long)m * a.ldp + 128 * j + 64);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    res2[i] = rr[i];
                }
            }
        }
        // 32 columns a TMEM wait and a store
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            const int c0 = 32 * gi;
            if (c0 >= width) {
                break;
            }
            uint32_t r[32];
            tmem_ld32(acc + c0, r);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 bb = *reinterpret_cast<const float4*>(b + c0 + 4 * q);
                v[4 * q] = __uint_as_float(r[4 * q]) + bb.x;
                v[4 * q + 1] = __uint_as_float(r[4 * q + 1]) + bb.y;
                v[4 * q + 2] = __uint_as_float(r[4 * q + 2]) + bb.z;
                v[4 * q + 3] = __uint_as_float(r[4 * q + 3]) + bb.w;
            }
            if constexpr (!LN) {
                if (a.residual != nullptr) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint4 qq = gi < 2 ? regs.res[4 * gi + u] : res2[4 * gi - 8 + u];
                        const uint32_t qw[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = E::unpack(qw[e]);
                            v[8 * u + 2 * e] += f.x;
                            v[8 * u + 2 * e + 1] += f.y;
                        }
                    }
                }
            }
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                w[e] = E::pack(v[2 * e], v[2 * e + 1]);
            }
            // rows past M hold garbage; the store clips them (a warp wholly past M stores nothing)
            if (row0 < a.M) {
                regs.st.put(to, lane, w, 128 * j + c0, row0);
            }
        }
    }
    static __device__ void padding(const Args& a, int m0, int t, int g) {
        const int m = m0 + t;
        if (m >= a.M) {
            return;
        }
        // with a residual the output aliases it, which it keeps
        if (a.n > 0 && a.residual == nullptr) {
            // warpgroup g zeroes its share of the row, in 8-column pieces
            const int share = (a.n + 8 * G - 1) / (8 * G) * 8;
            const int c1 = min(a.n, (g + 1) * share);
            T* orow = a.out + (long long)m * a.ldp;
            for (int c = g * share; c < c1; c += 8) {
                *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
            }
        }
        if (g == 0) {
            for (int h = 0; h < a.heads; ++h) {
                a.bias[(long long)h * a.M + m] = E::from_f(0.f);
            }
        }
    }
};

// ---------------------------------------------------------------------------------------------
// VoltaTrimulEpilogue: out [M, O] = (LN(x_cm^T) wo + bo) * sigmoid(LN_in(x) wg + bg) (+ x)
// A tile stage holds Y = LN(x_cm^T) (C columns, written by the workers from the float32
// channel-major triangle product) and then x (CA columns, TMA), normalised in place.
// ---------------------------------------------------------------------------------------------
template <typename T_, int C, int CA, int O, bool ADD>
struct TrimulOp {
    using T = T_;
    using E = Elem<T>;
    static constexpr int kWorkerGroups = 2;
    static constexpr int kSlots = 4, kSlotCols = 128;
    // A stage starts with the tile's float32 x_cm columns ([C][128], by TMA with x when
    // M % 4 == 0), over whose first half the workers write Y; then x's atoms. At C = 128 such a
    // stage (96 KB) leaves room for one only.
    static constexpr int kStages = C <= 64 ? 2 : 1;
    // with two stages the warpgroups take the tiles in turn, a thread a whole row (both
    // LayerNorms without a barrier between warpgroups, one tile's LayerNorms overlapping the
    // other's epilogue); with one, both split every tile
    static constexpr bool kPingPong = kStages == 2;
    static constexpr int X_BYTES = (C * 4 + CA * 2) * BM;
    static constexpr int XOFF = C * BM * 4;  // x's atoms after the x_cm / Y region
    static constexpr float kOther = -1.f;
    static constexpr int RED_FLOATS = 8 * BM;
    // the output leaves through per-warp staging (two 2 KB box buffers a worker warp) and TMA
    // stores
    using Stager = RowChunkStager<2>;
    static constexpr int STORE_BYTES = (kWorkers / 32) * Stager::BYTES;
    struct Args {
        const float* x_cm;
        const T *x, *woT, *bo, *wgT, *bg, *keep;
        const float *in_scale, *in_offset, *ln_scale, *ln_offset;
        T* out;
        int M, w_bytes, param_floats;
        int xcm_tma;  // x_cm arrives in the stage (map tm1)
        float eps;
    };
    struct Regs {
        // x of the next block's channels (add_input): the block's 64 (ping-pong) or worker
        // half g's 32
        uint4 res[kPingPong ? 8 : 4];
        Stager st;
    };
    static __device__ void bind(Regs& r, uint8_t* stb, int warp) {
        r.st.base = smem_u32(stb) + warp * Stager::BYTES;
        r.st.n = 0;
    }
    static __device__ void finish(Regs& r, int lane) { r.st.finish(lane); }
    static __device__ void row_keep(Regs&, float) {}
    static __device__ const T* keep(const Args& a) { return a.keep; }
    // in_scale [CA], in_offset [CA], ln_scale [C], ln_offset [C], bo [O], bg [O]
    static __device__ void load_params(const Args& a, float* sp, uint8_t*, int tid) {
        for (int i = tid; i < CA; i += kWorkers) {
            sp[i] = a.in_scale[i];
            sp[CA + i] = a.in_offset[i];
        }
        for (int i = tid; i < C; i += kWorkers) {
            sp[2 * CA + i] = a.ln_scale[i];
            sp[2 * CA + C + i] = a.ln_offset[i];
        }
        for (int i = tid; i < O; i += kWorkers) {
            sp[2 * CA + 2 * C + i] = E::to_f(a.bo[i]);
            sp[2 * CA + 2 * C + O + i] = E::to_f(a.bg[i]);
        }
    }
    static __device__ void load_weights(const Args& a, const CUtensorMap* tw0,
                                        const CUtensorMap* tw1, uint8_t* ws, uint64_t* bar) {
        mbar_arrive_expect_tx(bar, (uint32_t)((O * C + O * CA) * 2));
        load_weight(tw0, ws, bar, O, C);
        load_weight(tw1, ws + O * C * 2, bar, O, CA);
    }
    static __device__ void load_x(const Args& a, const CUtensorMap* tx, const CUtensorMap* txc,
                                  uint8_t* dst, uint64_t* bar, int m0) {
        if (a.xcm_tma) {
            mbar_arrive_expect_tx(bar, (uint32_t)((CA * 2 + C * 4) * BM));
            for (int at = 0; at < CA / 64; ++at) {
                tma_load_2d(dst + XOFF + at * ATOM, tx, bar, at * 64, m0);
            }
            // x_cm [C][M] float32: rows [m0, m0 + 128) of every channel, [C][128] in the stage
            tma_load_2d(dst, txc, bar, m0, 0);
        } else {
            load_rows_tile(tx, dst + XOFF, bar, CA, m0);
        }
    }
    // block j: output channels [64j, 64j+64); LN(x_cm^T) wo in the slot's columns [0, 64),
    // LN_in(x) wg in [64, 128)
    static __device__ int nblocks(const Args&) { return O / 64; }
    static __device__ void issue_block(const Args& a, uint32_t xa, uint32_t wa, uint32_t acc,
                                       int j) {
        mma_rows(acc, xa, wa, O, C, 64 * j, 64, E::kBf16, false);
        mma_rows(acc + 64, xa + XOFF, wa + O * C * 2, O, CA, 64 * j, 64, E::kBf16, false);
    }
    static __device__ void prologue(const Args& a, uint8_t* stage, const float* sp, float* red,
                                    int t, int g, int m0, Regs& regs) {
        if constexpr (kPingPong) {
            prologue_row(a, stage, sp, t, g, m0);
        } else {
            prologue_split(a, stage, sp, red, t, g, m0);
        }
    }
    // ping-pong: thread t of warpgroup g normalises column m = m0 + t of x_cm over all C
    // channels (two-pass float32 from registers) into row t of Y, then row t of x in place
    static __device__ void prologue_row(const Args& a, uint8_t* stage, const float* sp, int t,
                                        int g, int m0) {
        const int m = m0 + t;
        const bool in = m < a.M;
        float v[C];
        if (a.xcm_tma) {
            const float* xc = reinterpret_cast<const float*>(stage) + t;
#pragma unroll
            for (int i = 0; i < C; ++i) {
                v[i] = xc[i * BM];
            }
        } else {
#pragma unroll
            for (int i = 0; i < C; ++i) {
                v[i] = in ? a.x_cm[(long long)i * a.M + m] : 0.f;
            }
        }
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < C; i += 2) {
            s0 += v[i];
            s1 += v[i + 1];
        }
        const float mean = (s0 + s1) * (1.f / C);
        float q0 = 0.f, q1 = 0.f;
#pragma unroll
        for (int i = 0; i < C; i += 2) {
            v[i] -= mean;
            v[i + 1] -= mean;
            q0 += v[i] * v[i];
            q1 += v[i + 1] * v[i + 1];
        }
        const float rstd = rsqrtf((q0 + q1) * (1.f / C) + a.eps);
        const float* ls = sp + 2 * CA;
        const float* lo = sp + 2 * CA + C;
        // Y overwrites the x_cm columns of other rows: all of the warpgroup's reads come first
        named_sync(2 + g, 128);
#pragma unroll
        for (int ch = 0; ch < C / 8; ++ch) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = 8 * ch + 2 * e;
                w[e] = E::pack(v[c] * rstd * ls[c] + lo[c], v[c + 1] * rstd * ls[c + 1] + lo[c + 1]);
            }
            *reinterpret_cast<uint4*>(stage + sw128(t, 8 * ch)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        ln_row_full<T, CA>(stage + XOFF, t, sp, sp + CA, a.eps);
    }
    // split: worker half g takes channels [g C/2, (g+1) C/2) of both LayerNorms, the statistics
    // exchanged through red
    static __device__ void prologue_split(const Args& a, uint8_t* stage, const float* sp,
                                          float* red, int t, int g, int m0) {
        // LN over the C channels of column m of the channel-major float32 x_cm
        constexpr int CH = C / 2;
        const int m = m0 + t;
        const bool in = m < a.M;
        float v[CH];
        if (a.xcm_tma) {
            // from the stage (zeros past M); Y overwrites it only after the second barrier
            const float* xc = reinterpret_cast<const float*>(stage) + g * CH * BM + t;
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                v[i] = xc[i * BM];
            }
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i) {
                v[i] = in ? a.x_cm[(long long)(g * CH + i) * a.M + m] : 0.f;
            }
        }
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < CH; ++i) {
            s += v[i];
        }
        float* r2 = red + 4 * BM;
        r2[g * BM + t] = s;
        workers_sync();
        const float mean = (r2[t] + r2[BM + t]) * (1.f / C);
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < CH; ++i) {
            v[i] -= mean;
            q += v[i] * v[i];
        }
        r2[(2 + g) * BM + t] = q;
        workers_sync();
        const float rstd = rsqrtf((r2[2 * BM + t] + r2[3 * BM + t]) * (1.f / C) + a.eps);
        const float* ls = sp + 2 * CA;
        const float* lo = sp + 2 * CA + C;
#pragma unroll
        for (int ch = 0; ch < CH / 8; ++ch) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = g * CH + 8 * ch + 2 * e;
                w[e] = E::pack(v[8 * ch + 2 * e] * rstd * ls[c] + lo[c],
                               v[8 * ch + 2 * e + 1] * rstd * ls[c + 1] + lo[c + 1]);
            }
            *reinterpret_cast<uint4*>(stage + sw128(t, g * CH + 8 * ch)) =
                make_uint4(w[0], w[1], w[2], w[3]);
        }
        // then LN_in(x) in place on the TMA-loaded x atoms
        ln_rows_half<T, CA>(stage + XOFF, t, g, sp, sp + CA, a.eps, red, nullptr, nullptr);
    }
    // x of worker half g's channels of block j (add_input), loaded ahead of the MMA wait; with
    // the first block, the next tile's x_cm lines of this worker's channels are prefetched into
    // L2, so that the next prologue's loads do not wait for DRAM
    static __device__ void prefetch_block(const Args& a, int t, int g, int m0, int j,
                                          Regs& regs) {
        const int m = m0 + t;
        if (j == 0 && !a.xcm_tma) {
            // this warpgroup's next tile (ping-pong: two tiles on, if none is skipped)
            const int mn = m + (kPingPong ? 2 : 1) * (int)gridDim.x * BM;
            if (mn < a.M) {
                constexpr int NC = kPingPong ? C : C / 2;
                const float* xc = a.x_cm + (long long)(kPingPong ? 0 : g * NC) * a.M + mn;
#pragma unroll 8
                for (int i = 0; i < NC; ++i) {
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(xc + (long long)i * a.M));
                }
            }
        }
        if constexpr (ADD) {
            if (m < a.M) {
                constexpr int NR = kPingPong ? 8 : 4;
                const uint4* xr = reinterpret_cast<const uint4*>(
                    a.x + (long long)m * CA + 64 * j + (kPingPong ? 0 : 32 * g));
#pragma unroll
                for (int i = 0; i < NR; ++i) {
                    regs.res[i] = xr[i];
                }
            }
        }
    }
    // worker half g: channels 64j + 32g + [0, 32)
    // (ping-pong: all 64 channels of block j, in two halves of 32)
    static __device__ void epilogue_block(const Args& a, uint32_t acc, const float* sp, int t,
                                          int g, int m0, int j, Regs& regs,
                                          const CUtensorMap* to, const CUtensorMap* to1) {
        if constexpr (kPingPong) {
            epilogue_staged(a, acc, sp, t, 0, m0, j, regs, to);
            epilogue_staged(a, acc, sp, t, 1, m0, j, regs, to);
        } else {
            epilogue_staged(a, acc, sp, t, g, m0, j, regs, to);
        }
    }
    // channels 64j + 32h + [0, 32) of row t
    static __device__ void epilogue_staged(const Args& a, uint32_t acc, const float* sp, int t,
                                           int h, int m0, int j, Regs& regs,
                                           const CUtensorMap* to) {
        const int lane = t & 31, row0 = m0 + (t & ~31), c0 = 32 * h;
        // this half's residual registers (ping-pong: the block's 64 channels, split mode: the
        // worker half's 32)
        const int rb = kPingPong ? 4 * h : 0;
        const float* bo = sp + 2 * CA + 2 * C + 64 * j + c0;
        const float* bg = bo + O;
        // rows past M would compute garbage that the store clips: a warp wholly past M skips
        if (row0 >= a.M) {
            return;
        }
        const uint32_t sb = regs.st.acquire(lane);
        // the 32 columns in two halves of 16 (one TMEM wait each), stored as one box
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            uint32_t ro[16], rg[16];
            tmem_ld16(acc + c0 + 16 * hh, ro);
            tmem_ld16(acc + 64 + c0 + 16 * hh, rg);
            tmem_wait_ld();
            uint32_t w[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 b0 = *reinterpret_cast<const float4*>(bo + 16 * hh + 4 * q);
                const float4 b1 = *reinterpret_cast<const float4*>(bg + 16 * hh + 4 * q);
                float v[4] = {(__uint_as_float(ro[4 * q]) + b0.x) *
                                  sigmoid_fast(__uint_as_float(rg[4 * q]) + b1.x),
                              (__uint_as_float(ro[4 * q + 1]) + b0.y) *
                                  sigmoid_fast(__uint_as_float(rg[4 * q + 1]) + b1.y),
                              (__uint_as_float(ro[4 * q + 2]) + b0.z) *
                                  sigmoid_fast(__uint_as_float(rg[4 * q + 2]) + b1.z),
                              (__uint_as_float(ro[4 * q + 3]) + b0.w) *
                                  sigmoid_fast(__uint_as_float(rg[4 * q + 3]) + b1.w)};
                if constexpr (ADD) {
                    const uint4 qq = regs.res[rb + 2 * hh + (q >> 1)];
                    const float2 f0 = E::unpack((q & 1) ? qq.z : qq.x);
                    const float2 f1 = E::unpack((q & 1) ? qq.w : qq.y);
                    v[0] += f0.x;
                    v[1] += f0.y;
                    v[2] += f1.x;
                    v[3] += f1.y;
                }
                w[2 * q] = E::pack(v[0], v[1]);
                w[2 * q + 1] = E::pack(v[2], v[3]);
            }
            regs.st.write(sb, lane, 2 * hh, w[0], w[1], w[2], w[3]);
            regs.st.write(sb, lane, 2 * hh + 1, w[4], w[5], w[6], w[7]);
        }
        regs.st.issue(to, sb, lane, 64 * j + c0, row0);
    }
    static __device__ void padding(const Args& a, int m0, int t, int g) {
        const int m = m0 + t;
        if (ADD || m >= a.M) {  // with add_input the output aliases x, which it keeps
            return;
        }
        T* orow = a.out + (long long)m * O;
        for (int c = g * (O / 2); c < (g + 1) * (O / 2); c += 8) {
            *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
        }
    }
};

// ---------------------------------------------------------------------------------------------
// VoltaTransition: out [M, C] = relu(LN(x) w1 + b1) w2 + b2 (+ x)
//
// A CTA tile is SUB*128 rows (SUB = 2 for C <= 128, so that every weight chunk serves 256 rows;
// 1 for C = 256). The hidden dimension is walked in 64-wide chunks j: GEMM1 writes
// acc1[s][j%2] = LN(x)_s w1[:, chunk] into tensor memory; the workers add b1, apply the ReLU and
// write the 16-bit result back over the same columns; GEMM2 accumulates acc2[s] += hidden_s
// w2[chunk, :] with its A operand read from tensor memory. Weight chunks (w1's 64 rows and w2T's
// chunk, [C][64], exactly the reference's chunked layout) stream through a shared-memory ring
// filled by a loader warp (warp 9); warp 8 issues the MMAs.
// ---------------------------------------------------------------------------------------------
template <int C>
struct TransCfg {
    static constexpr int SUB = C <= 128 ? 2 : 1;
    static constexpr int ROWS = SUB * BM;
    static constexpr int X_BYTES = ROWS * C * 2;           // one stage
    // hidden chunk width: 128 for the two-sub-tile case (one accumulator buffer a sub-tile, the
    // two sub-tiles' chains interleaved on the tensor pipe; fewer, wider GEMM1 MMAs), 64 with
    // two buffers for C = 256
    static constexpr int HC = SUB == 2 ? 128 : 64;
    static constexpr int SLOT = 4 * C * HC;                // w1 chunk [HC][C] + w2 chunk [C][HC]
    static constexpr int NSLOT = C == 64 ? 5 : 2;
    static constexpr int ACC2 = 0;                         // acc2[s] at s * C
    // SUB = 2: acc1[s] at ACC1 + s * HC; SUB = 1: acc1[b] at ACC1 + b * 64
    static constexpr int ACC1 = SUB * C;
    static constexpr int COLS = ACC1 + 2 * 64 * (SUB == 2 ? 2 : 1);
    static constexpr int ALLOC = COLS <= 256 ? 256 : 512;
    static constexpr int THREADS = kWorkers + 64;          // + MMA warp + loader warp
};

template <typename T>
struct TransArgs {
    const T *x, *w1T, *b1, *w2T, *b2, *keep;
    const float *scale, *offset;
    T* out;
    int M, H;
    float eps;
    bool add;
    int v8;  // 32-byte output stores allowed
};

template <typename T, int C>
__global__ void __launch_bounds__(TransCfg<C>::THREADS, 1)
    transition_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw1,
                      const __grid_constant__ CUtensorMap tw2, const TransArgs<T> a) {
    using G = TransCfg<C>;
    using E = Elem<T>;
    constexpr int SUB = G::SUB, ROWS = G::ROWS, NSLOT = G::NSLOT;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* xs = smem;                       // [SUB][C/64 atoms][128 rows][128 B]
    uint8_t* ring = smem + G::X_BYTES;        // NSLOT x (w1 chunk [C/64][HC][128B], w2 chunk)
    float* sp = reinterpret_cast<float*>(ring + NSLOT * G::SLOT);  // scale, offset, b2, b1
    float* red = sp + 3 * C + a.H;            // [4][BM]
    __shared__ uint64_t x_full, x_empty, a_ready, acc1_full[2], hid_ready[2], g2_done[2],
        acc2_full, acc2_empty, w_full[NSLOT], w_empty[NSLOT];
    __shared__ uint32_t tmem_sh;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int HC = G::HC;
    const int NH = a.H / HC;
    const int ntiles = (a.M + ROWS - 1) / ROWS;
    if (warp == kProducerWarp) {
        if (lane == 0) {
            mbar_init(&x_full, 1);
            mbar_init(&x_empty, 1);
            mbar_init(&a_ready, kWorkers);
            for (int i = 0; i < 2; ++i) {
                mbar_init(&acc1_full[i], 1);
                // SUB = 2: one barrier a sub-tile, its warpgroup's 128 workers
                mbar_init(&hid_ready[i], SUB == 2 ? kWorkers / 2 : kWorkers);
                mbar_init(&g2_done[i], 1);
            }
            mbar_init(&acc2_full, 1);
            mbar_init(&acc2_empty, kWorkers);
            for (int i = 0; i < NSLOT; ++i) {
                mbar_init(&w_full[i], 1);
                mbar_init(&w_empty[i], 1);
            }
            abort_flag = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&tmem_sh, G::ALLOC);
        tmem_relinquish();
    } else if (warp < kProducerWarp) {
        for (int i = threadIdx.x; i < C; i += kWorkers) {
            sp[i] = a.scale[i];
            sp[C + i] = a.offset[i];
            sp[2 * C + i] = E::to_f(a.b2[i]);
        }
        for (int i = threadIdx.x; i < a.H; i += kWorkers) {
            sp[3 * C + i] = E::to_f(a.b1[i]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_sh;
    const auto work_of = [&](int tile) {
        // a CTA tile is SUB row tiles; it is computed when any of them is
        int w = kSkip;
        for (int s = 0; s < SUB; ++s) {
            w = min(w, tile_work(a.keep, a.M, tile * ROWS + s * BM, -1.f));
        }
        return w;
    };

    if (warp == kProducerWarp + 1) {
        // loader: the weight chunks of every computed tile, in order
        int q = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            if (work_of(tile) != kCompute) {
                continue;
            }
            for (int j = 0; j < NH; ++j, ++q) {
                const int slot = q % NSLOT;
                if (lane == 0) {
                    if (q >= NSLOT) {
                        mbar_wait(&w_empty[slot], ((q - NSLOT) / NSLOT) & 1, &g_status,
                                  kStatusMmaWait, &abort_flag);
                    }
                    uint8_t* dst = ring + slot * G::SLOT;
                    mbar_arrive_expect_tx(&w_full[slot], G::SLOT);
                    // w1 rows [HC j, HC j + HC) as C/64 atoms of HC rows
                    for (int at = 0; at < C / 64; ++at) {
                        tma_load_2d(dst + at * HC * 128, &tw1, &w_full[slot], at * 64, j * HC);
                    }
                    // w2T's 64-wide chunks HC/64 j + u: [C][64] rows (HC/64 j + u) C .. + C of
                    // the [H/64 * C][64] view, one K atom each
                    for (int u = 0; u < HC / 64; ++u) {
                        for (int r0 = 0; r0 < C; r0 += 128) {
                            tma_load_2d(dst + C * HC * 2 + u * C * 128 + r0 * 128, &tw2,
                                        &w_full[slot], 0, ((HC / 64) * j + u) * C + r0);
                        }
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == kProducerWarp) {
        // MMA issue
        int q = 0, c = 0;
        int cursor = blockIdx.x;
        const auto next = [&]() -> int {
            while (cursor < ntiles) {
                const int tile = cursor;
                cursor += gridDim.x;
                if (work_of(tile) == kCompute) {
                    return tile;
                }
            }
            return -1;
        };
        int tile = next();
        if (tile >= 0 && lane == 0) {
            mbar_arrive_expect_tx(&x_full, G::X_BYTES);
            for (int s = 0; s < SUB; ++s) {
                for (int at = 0; at < C / 64; ++at) {
                    tma_load_2d(xs + s * BM * C * 2 + at * ATOM, &tx, &x_full, at * 64,
                                tile * ROWS + s * BM);
                }
            }
        }
        const uint32_t id1 = idesc_f16(E::kBf16, 128, 64, false, false);
        const uint32_t id2 = idesc_f16(E::kBf16, 128, C, false, false);
        // the next tile's x, once this tile's GEMM1s no longer read the stage (the workers
        // normalise it before they store this tile)
        const auto load_next_x = [&](int ntile) {
            mbar_wait(&x_empty, c & 1, &g_status, kStatusMmaWait, &abort_flag);
            mbar_arrive_expect_tx(&x_full, G::X_BYTES);
            for (int s = 0; s < SUB; ++s) {
                for (int at = 0; at < C / 64; ++at) {
                    tma_load_2d(xs + s * BM * C * 2 + at * ATOM, &tx, &x_full, at * 64,
                                ntile * ROWS + s * BM);
                }
            }
        };
        while (tile >= 0) {
            const int ntile = next();
            if constexpr (SUB == 2) {
                // two chains, one a sub-tile s: GEMM1(s, j) -> acc1[s] -> the warpgroup's
                // bias + ReLU -> GEMM2(s, j) -> GEMM1(s, j + 1) once GEMM2(s, j) has read acc1[s];
                // the chains interleave on the tensor pipe
                if (lane == 0) {
                    mbar_wait(&a_ready, c & 1, &g_status, kStatusSyncWait, &abort_flag);
                    tc_fence_after();
                    const auto gemm1 = [&](int sb, int j) {
                        const int hq = q + j, slot = hq % NSLOT;
                        if (sb == 0) {
                            mbar_wait(&w_full[slot], (hq / NSLOT) & 1, &g_status,
                                      kStatusTmaWait, &abort_flag);
                        }
                        if (hq >= 1) {
                            // GEMM2(sb, hq - 1) has read acc1[sb]
                            mbar_wait(&g2_done[sb], (hq - 1) & 1, &g_status, kStatusMmaWait,
                                      &abort_flag);
                        }
                        tc_fence_after();
                        mma_rows(tmem + G::ACC1 + sb * HC, smem_u32(xs + sb * BM * C * 2),
                                 smem_u32(ring + slot * G::SLOT), HC, C, 0, HC, E::kBf16, false);
                        mma_commit(&acc1_full[sb]);
                        if (sb == SUB - 1 && j == NH - 1) {
                            mma_commit(&x_empty);
                        }
                    };
                    gemm1(0, 0);
                    gemm1(1, 0);
                    for (int j = 0; j < NH; ++j) {
                        const int hq = q + j, slot = hq % NSLOT;
                        if (j == NH - 1 && ntile >= 0) {
                            load_next_x(ntile);
                        }
                        const uint32_t w2 = smem_u32(ring + slot * G::SLOT + C * HC * 2);
                        for (int sb = 0; sb < SUB; ++sb) {
                            mbar_wait(&hid_ready[sb], hq & 1, &g_status, kStatusSyncWait,
                                      &abort_flag);
                            if (j == 0 && sb == 0 && c > 0) {
                                mbar_wait(&acc2_empty, (c - 1) & 1, &g_status, kStatusSyncWait,
                                          &abort_flag);
                            }
                            tc_fence_after();
                            for (int k = 0; k < HC / 16; ++k) {
                                mma_ts(tmem + G::ACC2 + sb * C,
                                       tmem + G::ACC1 + sb * HC + 64 * (k >> 2) + (k & 3) * 8,
                                       desc_k128(w2 + (k >> 2) * C * 128 + (k & 3) * 32), id2,
                                       (j > 0 || k > 0) ? 1u : 0u);
                            }
                            mma_commit(&g2_done[sb]);
                            if (sb == SUB - 1) {
                                mma_commit(&w_empty[slot]);
                            }
                            if (j + 1 < NH) {
                                gemm1(sb, j + 1);
                            }
                        }
                    }
                    mma_commit(&acc2_full);
                }
                __syncwarp();
                q += NH;
                ++c;
                tile = ntile;
                continue;
            }
            if (lane == 0) {
                mbar_wait(&a_ready, c & 1, &g_status, kStatusSyncWait, &abort_flag);
                tc_fence_after();
                const auto gemm2 = [&](int jj) {
                    const int hq = q + jj, b = hq & 1, slot = hq % NSLOT;
                    mbar_wait(&hid_ready[b], (hq >> 1) & 1, &g_status, kStatusSyncWait,
                              &abort_flag);
                    if (jj == 0 && c > 0) {
                        mbar_wait(&acc2_empty, (c - 1) & 1, &g_status, kStatusSyncWait,
                                  &abort_flag);
                    }
                    tc_fence_after();
                    const uint32_t w2 = smem_u32(ring + slot * G::SLOT + C * 128);
                    for (int s = 0; s < SUB; ++s) {
                        for (int k = 0; k < 4; ++k) {
                            mma_ts(tmem + G::ACC2 + s * C,
                                   tmem + G::ACC1 + (b * SUB + s) * 64 + k * 8,
                                   desc_k128(w2 + k * 32), id2, (jj > 0 || k > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit(&g2_done[b]);
                    mma_commit(&w_empty[slot]);
                };
                for (int j = 0; j < NH; ++j) {
                    const int hq = q + j, b = hq & 1, slot = hq % NSLOT;
                    mbar_wait(&w_full[slot], (hq / NSLOT) & 1, &g_status, kStatusTmaWait,
                              &abort_flag);
                    if (hq >= 2) {
                        mbar_wait(&g2_done[b], ((hq - 2) >> 1) & 1, &g_status, kStatusMmaWait,
                                  &abort_flag);
                    }
                    tc_fence_after();
                    const uint32_t w1 = smem_u32(ring + slot * G::SLOT);
                    for (int s = 0; s < SUB; ++s) {
                        mma_rows(tmem + G::ACC1 + (b * SUB + s) * 64, smem_u32(xs + s * BM * C * 2),
                                 w1, 64, C, 0, 64, E::kBf16, false);
                    }
                    mma_commit(&acc1_full[b]);
                    if (j == NH - 1) {
                        mma_commit(&x_empty);
                    }
                    if (j >= 1) {
                        gemm2(j - 1);
                    }
                }
                if (ntile >= 0) {
                    load_next_x(ntile);
                }
                gemm2(NH - 1);
                mma_commit(&acc2_full);
            }
            __syncwarp();
            q += NH;
            ++c;
            tile = ntile;
        }
    } else {
        // workers: (g, t) = sub-tile g, row t (SUB = 2), or column half g of row t (SUB = 1).
        // A tile's order: hidden chunks; then the next computed tile's LayerNorm (its x arrives
        // while the last chunks run), so that the MMA warp starts the next tile's first GEMMs
        // while this tile's output is stored; then the output.
        const int g = warp >> 2, t = ((warp & 3) << 5) | lane;
        const uint32_t lane_base = tmem_lane_base(warp);
        const int s = SUB == 2 ? g : 0;
        // the next computed tile from `from` on, writing the padding tiles passed over
        const auto advance = [&](int from) -> int {
            for (int tl = from; tl < ntiles; tl += gridDim.x) {
                const int w = work_of(tl);
                if (w == kCompute) {
                    return tl;
                }
                const int mp = tl * ROWS + s * BM + t;
                if (w == kPadding && !a.add && mp < a.M) {
                    T* orow = a.out + (long long)mp * C;
                    const int c0 = SUB == 2 ? 0 : g * (C / 2), c1 = SUB == 2 ? C : c0 + C / 2;
                    for (int cc = c0; cc < c1; cc += 8) {
                        *reinterpret_cast<uint4*>(orow + cc) = make_uint4(0, 0, 0, 0);
                    }
                }
            }
            return -1;
        };
        // LayerNorm of the stage (tile number c of this CTA's computed tiles)
        const auto normalise = [&](int cn) {
            mbar_wait(&x_full, cn & 1, &g_status, kStatusTmaWait, &abort_flag);
            uint8_t* tile_s = xs + s * BM * C * 2;
            if constexpr (SUB == 2) {
                // a full row per worker, no exchange
                ln_row_full<T, C>(tile_s, t, sp, sp + C, a.eps);
            } else {
                ln_rows_half<T, C>(tile_s, t, g, sp, sp + C, a.eps, red, nullptr, nullptr);
            }
            fence_async_smem();
            mbar_arrive(&a_ready);
        };
        int q = 0, c = 0;
        int tile = advance(blockIdx.x);
        if (tile >= 0) {
            normalise(0);
        }
        while (tile >= 0) {
            const int m = tile * ROWS + s * BM + t;
            // the residual (x as it came in) of this worker's columns (up to 128 columns, 16 x 16
            // bytes), loaded a few 16-byte pieces a hidden chunk so that the loads spread over
            // the chunks instead of queueing at once before the second GEMM's wait
            constexpr int RC = SUB == 2 ? C : C / 2;   // columns a worker stores
            // of them: the first 64 prefetched during the hidden chunks (all of them held across
            // the chunks would not leave the chunks' registers), the rest loaded where used
            constexpr int RPRE = RC <= 128 && C <= 128 ? (RC < 64 ? RC : 64) : 0;
            // pieces a chunk: all of them by chunk 4 (128-wide chunks) or 8 (64-wide)
            constexpr int PER = (RPRE / 8 + 512 / HC / 2 - 1) / (512 / HC / 2);
            uint4 res[RPRE / 8 > 0 ? RPRE / 8 : 1];
            const uint4* xres = reinterpret_cast<const uint4*>(
                a.x + (long long)m * C + (SUB == 2 ? 0 : g * (C / 2)));
            // hidden chunks: bias, ReLU, 16-bit pairs back over the accumulator's columns (in
            // runs of 8, unrolled, so that the first run's residual pieces have fixed indices)
            for (int jb = 0; jb < NH; jb += 8) {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const int j = jb + jj;
                if (j >= NH) {
                    break;
                }
                if constexpr (RPRE > 0) {
                    if (jb == 0 && a.add && m < a.M) {
#pragma unroll
                        for (int u = 0; u < PER; ++u) {
                            if (jj * PER + u < RPRE / 8) {
                                res[jj * PER + u] = xres[jj * PER + u];
                            }
                        }
                    }
                }
                const int hq = q + j, b = hq & 1;
                if constexpr (SUB == 2) {
                    // sub-tile s's chunk j: acc1[s] (HC columns) in quarters of 32, quarter q
                    // written back as 16 columns of 16-bit pairs at 64 (q / 2) + 16 (q % 2) (the
                    // A layout of GEMM2's K steps), over columns already read; each quarter's
                    // tensor-memory load is issued before the previous quarter's arithmetic
                    mbar_wait(&acc1_full[s], hq & 1, &g_status, kStatusMmaWait, &abort_flag);
                    tc_fence_after();
                    const uint32_t base = tmem + G::ACC1 + s * HC + lane_base;
                    const float* b1 = sp + 3 * C + j * HC;
                    const auto relu_pack = [&](const uint32_t (&r)[32], int qq) {
                        uint32_t pk[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            pk[i] = E::pack(
                                fmaxf(__uint_as_float(r[2 * i]) + b1[32 * qq + 2 * i], 0.f),
                                fmaxf(__uint_as_float(r[2 * i + 1]) + b1[32 * qq + 2 * i + 1],
                                      0.f));
                        }
                        tmem_st16(base + 64 * (qq >> 1) + 16 * (qq & 1), pk);
                    };
                    static_assert(HC == 128, "four quarters");
                    uint32_t ra[32], rb[32];
                    tmem_ld32(base, ra);
                    tmem_wait_ld();
                    tmem_ld32(base + 32, rb);
                    relu_pack(ra, 0);
                    tmem_wait_ld();
                    tmem_ld32(base + 64, ra);
                    relu_pack(rb, 1);
                    tmem_wait_ld();
                    tmem_ld32(base + 96, rb);
                    relu_pack(ra, 2);
                    tmem_wait_ld();
                    relu_pack(rb, 3);
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(&hid_ready[s]);
                    continue;
                }
                mbar_wait(&acc1_full[b], (hq >> 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
                tc_fence_after();
                const uint32_t base = tmem + G::ACC1 + (b * SUB + s) * 64 + lane_base;
                const float* b1 = sp + 3 * C + j * 64;
                {
                    // column half g: hidden columns [32g, 32g+32) -> packed columns [16g, 16g+16)
                    uint32_t r0[32];
                    tmem_ld32(base + 32 * g, r0);
                    tmem_wait_ld();
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        pk[i] = E::pack(
                            fmaxf(__uint_as_float(r0[2 * i]) + b1[32 * g + 2 * i], 0.f),
                            fmaxf(__uint_as_float(r0[2 * i + 1]) + b1[32 * g + 2 * i + 1], 0.f));
                    }
                    // both halves must have read the fp32 columns before either overwrites them
                    workers_sync();
                    tmem_st16(base + 16 * g, pk);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&hid_ready[b]);
            }
            }
            // pieces the chunks did not cover (hidden widths below 512)
            if constexpr (RPRE > 0) {
                if (a.add && m < a.M) {
#pragma unroll
                    for (int idx = 0; idx < RPRE / 8; ++idx) {
                        if (idx >= (NH < 8 ? NH : 8) * PER) {
                            res[idx] = xres[idx];
                        }
                    }
                }
            }
            const int ntile = advance(tile + gridDim.x);
            if (ntile >= 0) {
                normalise(c + 1);
            }
            mbar_wait(&acc2_full, c & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            {
                const uint32_t acc = tmem + G::ACC2 + s * C + lane_base;
                const int c0 = SUB == 2 ? 0 : g * (C / 2);
                T* orow = a.out + (long long)m * C;
#pragma unroll
                for (int ci = 0; ci < RC / 16; ++ci) {
                    const int cc = c0 + 16 * ci;
                    uint32_t r[16];
                    tmem_ld16(acc + cc, r);
                    tmem_wait_ld();
                    if (m < a.M) {
                        float v[16];
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            const float4 bb =
                                *reinterpret_cast<const float4*>(sp + 2 * C + cc + 4 * q4);
                            v[4 * q4] = __uint_as_float(r[4 * q4]) + bb.x;
                            v[4 * q4 + 1] = __uint_as_float(r[4 * q4 + 1]) + bb.y;
                            v[4 * q4 + 2] = __uint_as_float(r[4 * q4 + 2]) + bb.z;
                            v[4 * q4 + 3] = __uint_as_float(r[4 * q4 + 3]) + bb.w;
                        }
                        if (a.add) {
                            uint4 q0, q1;
                            if (16 * ci < RPRE) {
                                q0 = res[2 * ci];
                                q1 = res[2 * ci + 1];
                            } else {
                                const uint4* xr =
                                    reinterpret_cast<const uint4*>(a.x + (long long)m * C + cc);
                                q0 = xr[0];
                                q1 = xr[1];
                            }
                            const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w,
                                                    q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const float2 f = E::unpack(qw[e]);
                                v[2 * e] += f.x;
                                v[2 * e + 1] += f.y;
                            }
                        }
                        uint32_t ww[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            ww[e] = E::pack(v[2 * e], v[2 * e + 1]);
                        }
                        if (a.v8) {
                            st_global_v8(orow + cc, make_uint4(ww[0], ww[1], ww[2], ww[3]),
                                         make_uint4(ww[4], ww[5], ww[6], ww[7]));
                        } else {
                            *reinterpret_cast<uint4*>(orow + cc) =
                                make_uint4(ww[0], ww[1], ww[2], ww[3]);
                            *reinterpret_cast<uint4*>(orow + cc + 8) =
                                make_uint4(ww[4], ww[5], ww[6], ww[7]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc2_empty);
            q += NH;
            ++c;
            tile = ntile;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kProducerWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, G::ALLOC);
    }
}

// ---------------------------------------------------------------------------------------------
// VoltaLayerNorm: out [M, C] = (x - mean) rstd scale + offset over the last axis, with the
// reference's one-pass statistics: fp32 sum and sum of squares, var = max(E[x^2] - mean^2, 0),
// rstd = rsqrt(var + eps), the result rounded to the 16-bit type (cuda/volta_ops.cu:27-60).
// No tensor-core work: a bandwidth kernel, every row read once and written once.
// ---------------------------------------------------------------------------------------------
constexpr int kLnRows = 4;  // rows a thread group has in flight

// C = 8G, G a power of two <= 32: G consecutive lanes take a row, 8 columns (one 16-byte load
// and store) each; a warp takes 32/G rows per pass, kLnRows passes at once (all loads issued
// before any arithmetic). Warp-uniform loop bounds keep every lane in the shuffles.
template <typename T, int G>
__global__ void __launch_bounds__(256) layer_norm_vec_kernel(const T* __restrict__ x,
                                                             const float* __restrict__ scale,
                                                             const float* __restrict__ offset,
                                                             T* __restrict__ out, long long M,
                                                             float eps) {
    using E = Elem<T>;
    constexpr int C = 8 * G, RPW = 32 / G;  // columns, rows a warp-pass
    const int lane = threadIdx.x & 31, sub = lane & (G - 1);
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    float sc[8], of[8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float4 s4 = *reinterpret_cast<const float4*>(scale + 8 * sub + 4 * h);
        const float4 o4 = *reinterpret_cast<const float4*>(offset + 8 * sub + 4 * h);
        sc[4 * h] = s4.x, sc[4 * h + 1] = s4.y, sc[4 * h + 2] = s4.z, sc[4 * h + 3] = s4.w;
        of[4 * h] = o4.x, of[4 * h + 1] = o4.y, of[4 * h + 2] = o4.z, of[4 * h + 3] = o4.w;
    }
    const float inv = 1.0f / (float)C;
    for (long long r0 = warp * RPW * kLnRows; r0 < M; r0 += nwarps * RPW * kLnRows) {
        uint4 v[kLnRows];
#pragma unroll
        for (int i = 0; i < kLnRows; ++i) {
            const long long row = r0 + i * RPW + lane / G;
            v[i] = row < M ? *reinterpret_cast<const uint4*>(x + row * C + 8 * sub)
                           : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < kLnRows; ++i) {
            const long long row = r0 + i * RPW + lane / G;
            const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
            float f[8];
            float sum = 0.f, sq = 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 p = E::unpack(w[e]);
                f[2 * e] = p.x;
                f[2 * e + 1] = p.y;
                sum += p.x + p.y;
                sq = fmaf(p.x, p.x, fmaf(p.y, p.y, sq));
            }
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) {
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
                sq += __shfl_xor_sync(0xffffffffu, sq, o);
            }
            const float mean = sum * inv;
            const float var = fmaxf(sq * inv - mean * mean, 0.f);
            const float rstd = rsqrtf(var + eps);
            uint32_t o4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                o4[e] = E::pack(fmaf((f[2 * e] - mean) * rstd, sc[2 * e], of[2 * e]),
                                fmaf((f[2 * e + 1] - mean) * rstd, sc[2 * e + 1], of[2 * e + 1]));
            }
            if (row < M) {
                *reinterpret_cast<uint4*>(out + row * C + 8 * sub) =
                    make_uint4(o4[0], o4[1], o4[2], o4[3]);
            }
        }
    }
}

// Any C (and unaligned buffers): a warp a row, lane-strided elements, as the reference does.
template <typename T>
__global__ void __launch_bounds__(256) layer_norm_row_kernel(const T* __restrict__ x,
                                                             const float* __restrict__ scale,
                                                             const float* __restrict__ offset,
                                                             T* __restrict__ out, long long M,
                                                             int C, float eps) {
    using E = Elem<T>;
    const int lane = threadIdx.x & 31;
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    const float inv = 1.0f / (float)C;
    for (long long row = warp; row < M; row += nwarps) {
        const T* xr = x + row * C;
        float sum = 0.f, sq = 0.f;
        for (int c = lane; c < C; c += 32) {
            const float v = E::to_f(xr[c]);
            sum += v;
            sq = fmaf(v, v, sq);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
        }
        const float mean = sum * inv;
        const float rstd = rsqrtf(fmaxf(sq * inv - mean * mean, 0.f) + eps);
        T* orow = out + row * C;
        for (int c = lane; c < C; c += 32) {
            orow[c] = E::from_f(fmaf((E::to_f(xr[c]) - mean) * rstd, scale[c], offset[c]));
        }
    }
}

// ---------------------------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------------------------
int sm_count() {
    static int cache[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) {
        return 148;
    }
    if (cache[dev] == 0) {
        cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
        if (cache[dev] <= 0) {
            cache[dev] = 148;
        }
    }
    return cache[dev];
}

bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

CUtensorMapDataType tdt(int dtype) {
    return dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// row-major [rows][cols] 16-bit matrix, boxes of 64 columns x box_rows rows, 128-byte swizzle
bool map_rows(CUtensorMap* m, int dtype, const void* base, long long rows, long long cols,
              long long ld, int box_rows) {
    const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)(rows > 0 ? rows : 1)};
    const uint64_t strides[1] = {(uint64_t)ld};
    const uint32_t box[2] = {64, (uint32_t)box_rows};
    return encode_tiled(m, tdt(dtype), 2, 2, base, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
}

template <class Op>
cudaError_t launch_op(cudaStream_t stream, const CUtensorMap& tx, const CUtensorMap& tw0,
                      const CUtensorMap& tw1, const CUtensorMap& to, const CUtensorMap& to1,
                      const typename Op::Args& a) {
    auto kern = row_tile_kernel<Op>;
    const int smem = Op::kStages * Op::X_BYTES + a.w_bytes +
                     (a.param_floats + Op::RED_FLOATS) * 4 + 1024 +
                     (Op::STORE_BYTES > 0 ? Op::STORE_BYTES + 1024 : 0);
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
        return e;
    }
    const int ntiles = (a.M + BM - 1) / BM;
    const int grid = std::min(ntiles, sm_count());
    kern<<<grid, Crew<Op>::kThreads, smem, stream>>>(tx, tw0, tw1, to, to1, a);
    return cudaGetLastError();
}

int launch_status(cudaError_t e, const char* who) {
    if (e != cudaSuccess) {
        return fail(kInternal, std::string(who) + " launch: " + cudaGetErrorString(e));
    }
    return kOk;
}

template <typename T, int K, int CI>
cudaError_t ln_gdp_typed(cudaStream_t stream, int dtype, const void* x, const float* scale,
                         const float* offset, const void* wpT, const void* bp, const void* wgT,
                         const void* bg, const void* mask, void* left, void* right, int M,
                         float eps) {
    using Op = LnGdpOp<T, K, CI>;
    CUtensorMap tx, tw0, tw1;
    if (!map_rows(&tx, dtype, x, M, K, K, BM) ||
        !map_rows(&tw0, dtype, wpT, 2 * CI, K, K, weight_box(2 * CI)) ||
        !map_rows(&tw1, dtype, wgT, 2 * CI, K, K, weight_box(2 * CI))) {
        return cudaErrorInvalidValue;
    }
    typename Op::Args a;
    a.x = static_cast<const T*>(x);
    a.wpT = static_cast<const T*>(wpT);
    a.bp = static_cast<const T*>(bp);
    a.wgT = static_cast<const T*>(wgT);
    a.bg = static_cast<const T*>(bg);
    a.mask = static_cast<const T*>(mask);
    a.scale = scale;
    a.offset = offset;
    a.left = static_cast<T*>(left);
    a.right = static_cast<T*>(right);
    a.M = M;
    a.w_bytes = 2 * Op::P * K * 2;
    a.param_floats = 2 * K + 2 * Op::P;
    // 2: 32-byte stores, 1: 16-byte stores, 0: element stores
    const uintptr_t lr = reinterpret_cast<uintptr_t>(left) | reinterpret_cast<uintptr_t>(right);
    a.vec_store = M % 16 == 0 && (lr & 31) == 0 ? 2 : M % 8 == 0 && (lr & 15) == 0 ? 1 : 0;
    a.eps = eps;
    // channel-major outputs leave in boxes of 32 rows x 32 channels (64-byte swizzle) when the
    // channel stride (M elements) is a multiple of 16 bytes
    CUtensorMap to0 = tx, to1 = tx;
    a.tma_out = 0;
    if (M % 8 == 0 && (lr & 15) == 0) {
        const uint64_t dims[2] = {(uint64_t)M, (uint64_t)CI};
        const uint64_t strides[1] = {(uint64_t)M};
        const uint32_t box[2] = {32, 32};
        if (!encode_tiled(&to0, tdt(dtype), 2, 2, left, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_64B) ||
            !encode_tiled(&to1, tdt(dtype), 2, 2, right, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_64B)) {
            return cudaErrorInvalidValue;
        }
        a.tma_out = 1;
    }
    return launch_op<Op>(stream, tx, tw0, tw1, to0, to1, a);
}

template <typename T, int K>
cudaError_t gdp_typed(cudaStream_t stream, int dtype, const void* x, const void* wp,
                      const void* bp, const void* wg, const void* bg, const void* mask,
                      void* out, int M, int N, int act) {
    using Op = GdpOp<T, K>;
    CUtensorMap tx, twp, twg, to;
    // weights [K, N] row-major: boxes of 64 columns x K rows (128-byte swizzle)
    const uint64_t wdims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t wstrides[1] = {(uint64_t)N};
    const uint32_t wbox[2] = {64, (uint32_t)K};
    // the output in boxes of 32 columns x 32 rows (64-byte swizzle)
    const uint64_t odims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t ostrides[1] = {(uint64_t)N};
    const uint32_t obox[2] = {32, 32};
    if (!map_rows(&tx, dtype, x, M, K, K, BM) ||
        !encode_tiled(&twp, tdt(dtype), 2, 2, wp, wdims, wstrides, wbox,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&twg, tdt(dtype), 2, 2, wg, wdims, wstrides, wbox,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tiled(&to, tdt(dtype), 2, 2, out, odims, ostrides, obox,
                      CU_TENSOR_MAP_SWIZZLE_64B)) {
        return cudaErrorInvalidValue;
    }
    typename Op::Args a;
    a.x = static_cast<const T*>(x);
    a.wp = static_cast<const T*>(wp);
    a.bp = static_cast<const T*>(bp);
    a.wg = static_cast<const T*>(wg);
    a.bg = static_cast<const T*>(bg);
    a.mask = static_cast<const T*>(mask);
    a.out = static_cast<T*>(out);
    a.M = M;
    a.N = N;
    a.act = act;
    a.w_bytes = 2 * K * N * 2;
    a.param_floats = 2 * N;
    a.eps = 0.f;
    return launch_op<Op>(stream, tx, twp, twg, to, to, a);
}

template <typename T, int K, bool LN>
cudaError_t proj_typed(cudaStream_t stream, int dtype, const void* x, const float* scale,
                       const float* offset, const void* wT, const void* b, const void* residual,
                       const void* wbT, const void* keep, void* out, void* bias, int M, int n,
                       int ldp, int heads, float eps) {
    using Op = ProjOp<T, K, LN>;
    CUtensorMap tx, tw0, to;
    if (!map_rows(&tx, dtype, x, M, K, K, BM)) {
        return cudaErrorInvalidValue;
    }
    if (n > 0) {
        // the output leaves in boxes of 32 columns x 32 rows (64-byte swizzle), one per worker
        // warp and 32 columns
        const uint64_t dims[2] = {(uint64_t)n, (uint64_t)M};
        const uint64_t strides[1] = {(uint64_t)ldp};
        const uint32_t box[2] = {32, 32};
        if (!map_rows(&tw0, dtype, wT, n, K, K, weight_box(n)) ||
            !encode_tiled(&to, tdt(dtype), 2, 2, out, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_64B)) {
            return cudaErrorInvalidValue;
        }
    } else {
        tw0 = tx;
        to = tx;
    }
    typename Op::Args a;
    a.x = static_cast<const T*>(x);
    a.wT = static_cast<const T*>(wT);
    a.b = static_cast<const T*>(b);
    a.residual = static_cast<const T*>(residual);
    a.wbT = static_cast<const T*>(wbT);
    a.keep = static_cast<const T*>(keep);
    a.scale = scale;
    a.offset = offset;
    a.out = static_cast<T*>(out);
    a.bias = static_cast<T*>(bias);
    a.M = M;
    a.n = n;
    a.ldp = ldp;
    a.heads = heads;
    a.hp = heads > 0 ? 16 : 0;
    a.w_bytes = (n + a.hp) * K * 2;
    a.param_floats = 2 * K + n;
    a.eps = eps;
    return launch_op<Op>(stream, tx, tw0, tw0, to, to, a);
}



template <typename T, int C, int CA, int O, bool ADD>
cudaError_t trimul_typed(cudaStream_t stream, int dtype, const float* x_cm, const void* x,
                         const float* in_scale, const float* in_offset, const float* ln_scale,
                         const float* ln_offset, const void* woT, const void* bo, const void* wgT,
                         const void* bg, const void* keep, void* out, int M, float eps) {
    using Op = TrimulOp<T, C, CA, O, ADD>;
    CUtensorMap tx, tw0, tw1, to;
    // the output leaves in boxes of 32 columns x 32 rows (64-byte swizzle)
    const uint64_t dims[2] = {(uint64_t)O, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)O};
    const uint32_t box[2] = {32, 32};
    if (!map_rows(&tx, dtype, x, M, CA, CA, BM) ||
        !map_rows(&tw0, dtype, woT, O, C, C, weight_box(O)) ||
        !map_rows(&tw1, dtype, wgT, O, CA, CA, weight_box(O))) {
        return cudaErrorInvalidValue;
    }
    if (!encode_tiled(&to, tdt(dtype), 2, 2, out, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B)) {
        return cudaErrorInvalidValue;
    }
    // x_cm [C][M] float32 into the stage with x (row stride M * 4 bytes a multiple of 16)
    CUtensorMap txc = tx;
    const bool xcm_tma =
        M % 4 == 0 && (reinterpret_cast<uintptr_t>(x_cm) & 15) == 0;
    if (xcm_tma) {
        const uint64_t cdims[2] = {(uint64_t)M, (uint64_t)C};
        const uint64_t cstrides[1] = {(uint64_t)M};
        const uint32_t cbox[2] = {(uint32_t)BM, (uint32_t)C};
        if (!encode_tiled(&txc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 2, x_cm, cdims, cstrides,
                          cbox, CU_TENSOR_MAP_SWIZZLE_NONE)) {
            return cudaErrorInvalidValue;
        }
    }
    typename Op::Args a;
    a.x_cm = x_cm;
    a.x = static_cast<const T*>(x);
    a.woT = static_cast<const T*>(woT);
    a.bo = static_cast<const T*>(bo);
    a.wgT = static_cast<const T*>(wgT);
    a.bg = static_cast<const T*>(bg);
    a.keep = static_cast<const T*>(keep);
    a.in_scale = in_scale;
    a.in_offset = in_offset;
    a.ln_scale = ln_scale;
    a.ln_offset = ln_offset;
    a.out = static_cast<T*>(out);
    a.M = M;
    a.xcm_tma = xcm_tma ? 1 : 0;
    a.w_bytes = (O * C + O * CA) * 2;
    a.param_floats = 2 * CA + 2 * C + 2 * O;
    a.eps = eps;
    return launch_op<Op>(stream, tx, tw0, tw1, to, txc, a);
}

template <typename T, int C, int CA>
cudaError_t trimul_o(cudaStream_t s, int dtype, int O, bool add, const float* x_cm,
                     const void* x, const float* is, const float* io, const float* ls,
                     const float* lo, const void* woT, const void* bo, const void* wgT,
                     const void* bg, const void* keep, void* out, int M, float eps) {
    if (add) {  // O == CA
        return trimul_typed<T, C, CA, CA, true>(s, dtype, x_cm, x, is, io, ls, lo, woT, bo, wgT,
                                                bg, keep, out, M, eps);
    }
    return O == 64 ? trimul_typed<T, C, CA, 64, false>(s, dtype, x_cm, x, is, io, ls, lo, woT,
                                                       bo, wgT, bg, keep, out, M, eps)
                   : trimul_typed<T, C, CA, 128, false>(s, dtype, x_cm, x, is, io, ls, lo, woT,
                                                        bo, wgT, bg, keep, out, M, eps);
}

template <typename T>
cudaError_t trimul_dispatch(cudaStream_t s, int dtype, int C, int CA, int O, bool add,
                            const float* x_cm, const void* x, const float* is, const float* io,
                            const float* ls, const float* lo, const void* woT, const void* bo,
                            const void* wgT, const void* bg, const void* keep, void* out, int M,
                            float eps) {
    if (C == 64) {
        return CA == 64 ? trimul_o<T, 64, 64>(s, dtype, O, add, x_cm, x, is, io, ls, lo, woT, bo,
                                              wgT, bg, keep, out, M, eps)
                        : trimul_o<T, 64, 128>(s, dtype, O, add, x_cm, x, is, io, ls, lo, woT,
                                               bo, wgT, bg, keep, out, M, eps);
    }
    return CA == 64 ? trimul_o<T, 128, 64>(s, dtype, O, add, x_cm, x, is, io, ls, lo, woT, bo,
                                           wgT, bg, keep, out, M, eps)
                    : trimul_o<T, 128, 128>(s, dtype, O, add, x_cm, x, is, io, ls, lo, woT, bo,
                                            wgT, bg, keep, out, M, eps);
}


template <typename T, int C>
cudaError_t transition_typed(cudaStream_t stream, int dtype, const void* x, const float* scale,
                             const float* offset, const void* w1T, const void* b1,
                             const void* w2T, const void* b2, const void* keep, void* out, int M,
                             int H, float eps, bool add) {
    using G = TransCfg<C>;
    CUtensorMap tx, tw1, tw2;
    // w2T [H/64][C][64] viewed as [H/64 * C] rows of 64
    if (!map_rows(&tx, dtype, x, M, C, C, BM) || !map_rows(&tw1, dtype, w1T, H, C, C, G::HC) ||
        !map_rows(&tw2, dtype, w2T, (long long)(H / 64) * C, 64, 64, std::min(C, 128))) {
        return cudaErrorInvalidValue;
    }
    TransArgs<T> a;
    a.x = static_cast<const T*>(x);
    a.w1T = static_cast<const T*>(w1T);
    a.b1 = static_cast<const T*>(b1);
    a.w2T = static_cast<const T*>(w2T);
    a.b2 = static_cast<const T*>(b2);
    a.keep = static_cast<const T*>(keep);
    a.scale = scale;
    a.offset = offset;
    a.out = static_cast<T*>(out);
    a.M = M;
    a.H = H;
    a.eps = eps;
    a.add = add;
    a.v8 = (reinterpret_cast<uintptr_t>(out) & 31) == 0;
    auto kern = transition_kernel<T, C>;
    const int smem = G::X_BYTES + G::NSLOT * G::SLOT + (3 * C + H + 4 * BM) * 4 + 1024;
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
        return e;
    }
    const int ntiles = (M + G::ROWS - 1) / G::ROWS;
    kern<<<std::min(ntiles, sm_count()), G::THREADS, smem, stream>>>(tx, tw1, tw2, a);
    return cudaGetLastError();
}

// blocks of 256 threads the GPU holds at once (a persistent grid of one wave)
long long one_wave(const void* kern) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0) != cudaSuccess ||
        per_sm < 1) {
        per_sm = 1;
    }
    return (long long)sm_count() * per_sm;
}

template <typename T, int G>
cudaError_t layer_norm_vec_launch(cudaStream_t stream, const T* x, const float* scale,
                                  const float* offset, T* out, long long M, float eps) {
    auto kern = layer_norm_vec_kernel<T, G>;
    const long long rows_per_block = 8LL * (32 / G) * kLnRows;  // 8 warps a block
    const long long blocks =
        std::min(one_wave((const void*)kern), (M + rows_per_block - 1) / rows_per_block);
    kern<<<(unsigned)blocks, 256, 0, stream>>>(x, scale, offset, out, M, eps);
    return cudaGetLastError();
}

template <typename T>
cudaError_t layer_norm_typed(cudaStream_t stream, const void* x, const float* scale,
                             const float* offset, void* out, long long M, int C, float eps) {
    const T* xp = static_cast<const T*>(x);
    T* op = static_cast<T*>(out);
    const bool vec = C % 8 == 0 && C / 8 <= 32 && ((C / 8) & (C / 8 - 1)) == 0 &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                       reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(offset)) &
                      15) == 0;
    if (vec) {
        switch (C / 8) {
        case 1: return layer_norm_vec_launch<T, 1>(stream, xp, scale, offset, op, M, eps);
        case 2: return layer_norm_vec_launch<T, 2>(stream, xp, scale, offset, op, M, eps);
        case 4: return layer_norm_vec_launch<T, 4>(stream, xp, scale, offset, op, M, eps);
        case 8: return layer_norm_vec_launch<T, 8>(stream, xp, scale, offset, op, M, eps);
        case 16: return layer_norm_vec_launch<T, 16>(stream, xp, scale, offset, op, M, eps);
        default: return layer_norm_vec_launch<T, 32>(stream, xp, scale, offset, op, M, eps);
        }
    }
    auto kern = layer_norm_row_kernel<T>;
    const long long blocks = std::min(one_wave((const void*)kern), (M + 7) / 8);
    kern<<<(unsigned)blocks, 256, 0, stream>>>(xp, scale, offset, op, M, C, eps);
    return cudaGetLastError();
}

}  // namespace

unsigned read_and_clear_status_fused() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    return v;
}

}  // namespace cflk

using namespace cflk;

extern "C" int cflk_volta_ln_gdp(void* stream, int dtype, const void* x, const float* scale,
                                 const float* offset, const void* wpT, const void* bp,
                                 const void* wgT, const void* bg, const void* mask, void* left,
                                 void* right, int64_t M, int64_t K, int64_t P, float eps) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "ln_gdp: dtype must be f16 or bf16");
    }
    if ((K != 64 && K != 128) || P % 2 || (P / 2 != 64 && P / 2 != 128) || M < 0) {
        return fail(kInvalidArgument, "ln_gdp: K and P/2 must be 64 or 128");
    }
    if (M == 0) {
        return kOk;
    }
    if (!aligned16(x) || !aligned16(wpT) || !aligned16(wgT)) {
        return fail(kInvalidArgument, "ln_gdp: buffers must be 16-byte aligned");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int m = (int)M, ci = (int)(P / 2);
    cudaError_t e;
#define CFLK_GDP(T)                                                                              \
    (K == 64 ? (ci == 64 ? ln_gdp_typed<T, 64, 64>(s, dtype, x, scale, offset, wpT, bp, wgT, bg, \
                                                   mask, left, right, m, eps)                    \
                         : ln_gdp_typed<T, 64, 128>(s, dtype, x, scale, offset, wpT, bp, wgT,    \
                                                    bg, mask, left, right, m, eps))              \
             : (ci == 64 ? ln_gdp_typed<T, 128, 64>(s, dtype, x, scale, offset, wpT, bp, wgT,    \
                                                    bg, mask, left, right, m, eps)               \
                         : ln_gdp_typed<T, 128, 128>(s, dtype, x, scale, offset, wpT, bp, wgT,   \
                                                     bg, mask, left, right, m, eps)))
    e = dtype == kBF16 ? CFLK_GDP(__nv_bfloat16) : CFLK_GDP(__half);
#undef CFLK_GDP
    return launch_status(e, "ln_gdp");
}

extern "C" int cflk_volta_ln_proj(void* stream, int dtype, const void* x, const float* scale,
                                  const float* offset, const void* wT, const void* wbT,
                                  const void* keep, void* p, void* bias, int64_t M, int64_t K,
                                  int64_t n, int64_t heads, float eps) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "ln_projection: dtype must be f16 or bf16");
    }
    if ((K != 64 && K != 128) || n < 0 || n % 64 || heads < 0 || heads > 8 || M < 0) {
        return fail(kInvalidArgument,
                    "ln_projection: K must be 64 or 128, n a multiple of 64, at most 8 heads");
    }
    if (M == 0 || (n == 0 && heads == 0)) {
        return kOk;
    }
    if (!aligned16(x) || (n > 0 && (!aligned16(wT) || !aligned16(p)))) {
        return fail(kInvalidArgument, "ln_projection: buffers must be 16-byte aligned");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int esz = 2;
    // passes of at most 512 output columns over the same rows; the head bias in the first
    for (int64_t n0 = 0; n0 < n || (n0 == 0 && n == 0); n0 += 512) {
        const int np = (int)std::min<int64_t>(512, n - n0);
        const void* w = n > 0 ? static_cast<const uint8_t*>(wT) + n0 * K * esz : nullptr;
        void* po = n > 0 ? static_cast<uint8_t*>(p) + n0 * esz : nullptr;
        const int hp = n0 == 0 ? (int)heads : 0;
        cudaError_t e;
        if (dtype == kBF16) {
            e = K == 64 ? proj_typed<__nv_bfloat16, 64, true>(s, dtype, x, scale, offset, w,
                                                              nullptr, nullptr, wbT, keep, po,
                                                              bias, (int)M, np, (int)n, hp, eps)
                        : proj_typed<__nv_bfloat16, 128, true>(s, dtype, x, scale, offset, w,
                                                               nullptr, nullptr, wbT, keep, po,
                                                               bias, (int)M, np, (int)n, hp, eps);
        } else {
            e = K == 64 ? proj_typed<__half, 64, true>(s, dtype, x, scale, offset, w, nullptr,
                                                       nullptr, wbT, keep, po, bias, (int)M, np,
                                                       (int)n, hp, eps)
                        : proj_typed<__half, 128, true>(s, dtype, x, scale, offset, w, nullptr,
                                                        nullptr, wbT, keep, po, bias, (int)M, np,
                                                        (int)n, hp, eps);
        }
        if (e != cudaSuccess) {
            return launch_status(e, "ln_projection");
        }
        if (n == 0) {
            break;
        }
    }
    return kOk;
}

extern "C" int cflk_volta_out_proj(void* stream, int dtype, const void* o, const void* wT,
                                   const void* b, const void* residual, const void* keep,
                                   void* out, int64_t M, int64_t K, int64_t N) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "output_projection: dtype must be f16 or bf16");
    }
    if ((K != 64 && K != 128) || (N != 64 && N != 128) || M < 0) {
        return fail(kInvalidArgument, "output_projection: K and N must be 64 or 128");
    }
    if (M == 0) {
        return kOk;
    }
    if (!aligned16(o) || !aligned16(wT) || !aligned16(out) ||
        (residual != nullptr && !aligned16(residual))) {
        return fail(kInvalidArgument, "output_projection: buffers must be 16-byte aligned");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (dtype == kBF16) {
        e = K == 64 ? proj_typed<__nv_bfloat16, 64, false>(s, dtype, o, nullptr, nullptr, wT, b,
                                                           residual, nullptr, keep, out, nullptr,
                                                           (int)M, (int)N, (int)N, 0, 0.f)
                    : proj_typed<__nv_bfloat16, 128, false>(s, dtype, o, nullptr, nullptr, wT, b,
                                                            residual, nullptr, keep, out,
                                                            nullptr, (int)M, (int)N, (int)N, 0,
                                                            0.f);
    } else {
        e = K == 64 ? proj_typed<__half, 64, false>(s, dtype, o, nullptr, nullptr, wT, b,
                                                    residual, nullptr, keep, out, nullptr,
                                                    (int)M, (int)N, (int)N, 0, 0.f)
                    : proj_typed<__half, 128, false>(s, dtype, o, nullptr, nullptr, wT, b,
                                                     residual, nullptr, keep, out, nullptr,
                                                     (int)M, (int)N, (int)N, 0, 0.f);
    }
    return launch_status(e, "output_projection");
}

extern "C" int cflk_volta_trimul_epilogue(void* stream, int dtype, const float* x_cm,
                                          const void* x, const float* in_scale,
                                          const float* in_offset, const float* ln_scale,
                                          const float* ln_offset, const void* woT, const void* bo,
                                          const void* wgT, const void* bg, const void* keep,
                                          void* out, int64_t M, int64_t C, int64_t CA, int64_t O,
                                          float eps, int add_input) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "trimul_epilogue: dtype must be f16 or bf16");
    }
    const auto w = [](int64_t c) { return c == 64 || c == 128; };
    if (!w(C) || !w(CA) || !w(O) || (add_input && O != CA) || M < 0) {
        return fail(kInvalidArgument,
                    "trimul_epilogue: C, CA and O must be 64 or 128, O == CA with add_input");
    }
    if (M == 0) {
        return kOk;
    }
    if (!aligned16(x) || !aligned16(woT) || !aligned16(wgT) || !aligned16(out)) {
        return fail(kInvalidArgument, "trimul_epilogue: buffers must be 16-byte aligned");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e =
        dtype == kBF16
            ? trimul_dispatch<__nv_bfloat16>(s, dtype, (int)C, (int)CA, (int)O, add_input != 0,
                                             x_cm, x, in_scale, in_offset, ln_scale, ln_offset,
                                             woT, bo, wgT, bg, keep, out, (int)M, eps)
            : trimul_dispatch<__half>(s, dtype, (int)C, (int)CA, (int)O, add_input != 0, x_cm, x,
                                      in_scale, in_offset, ln_scale, ln_offset, woT, bo, wgT, bg,
                                      keep, out, (int)M, eps);
    return launch_status(e, "trimul_epilogue");
}

extern "C" int cflk_volta_transition(void* stream, int dtype, const void* x, const float* scale,
                                     const float* offset, const void* w1T, const void* b1,
                                     const void* w2T, const void* b2, const void* keep, void* out,
                                     int64_t M, int64_t C, int64_t H, float eps, int add_input) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "transition: dtype must be f16 or bf16");
    }
    if ((C != 64 && C != 128 && C != 256) || (H != 2 * C && H != 4 * C) || M < 0) {
        return fail(kInvalidArgument, "transition: C must be 64, 128 or 256, H 2C or 4C");
    }
    if (M == 0) {
        return kOk;
    }
    if (!aligned16(x) || !aligned16(w1T) || !aligned16(w2T) || !aligned16(out)) {
        return fail(kInvalidArgument, "transition: buffers must be 16-byte aligned");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
#define CFLK_TR(T)                                                                              \
    (C == 64    ? transition_typed<T, 64>(s, dtype, x, scale, offset, w1T, b1, w2T, b2, keep,   \
                                          out, (int)M, (int)H, eps, add_input != 0)             \
     : C == 128 ? transition_typed<T, 128>(s, dtype, x, scale, offset, w1T, b1, w2T, b2, keep,  \
                                           out, (int)M, (int)H, eps, add_input != 0)            \
                : transition_typed<T, 256>(s, dtype, x, scale, offset, w1T, b1, w2T, b2, keep,  \
                                           out, (int)M, (int)H, eps, add_input != 0))
    e = dtype == kBF16 ? CFLK_TR(__nv_bfloat16) : CFLK_TR(__half);
#undef CFLK_TR
    return launch_status(e, "transition");
}

extern "C" int cflk_volta_layer_norm(void* stream, int dtype, const void* x, const float* scale,
                                     const float* offset, void* out, int64_t M, int64_t C,
                                     float eps) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "layer_norm: dtype must be f16 or bf16");
    }
    if (M < 0 || C < 1 || C > (1 << 20)) {
        return fail(kInvalidArgument, "x must be [M,C]");
    }
    if (M == 0) {
        return kOk;
    }
    if (x == nullptr || scale == nullptr || offset == nullptr || out == nullptr) {
        return fail(kInvalidArgument, "layer_norm: null buffer");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e =
        dtype == kBF16
            ? layer_norm_typed<__nv_bfloat16>(s, x, scale, offset, out, M, (int)C, eps)
            : layer_norm_typed<__half>(s, x, scale, offset, out, M, (int)C, eps);
    return launch_status(e, "layer_norm");
}

extern "C" int cflk_volta_gdp(void* stream, int dtype, const void* x, const void* wp,
                              const void* bp, const void* wg, const void* bg, const void* mask,
                              void* out, int64_t M, int64_t K, int64_t N, int64_t activation) {
    clear_error();
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "gdp: dtype must be f16 or bf16");
    }
    if (activation != 0 && activation != 1) {
        return fail(kInvalidArgument, "gdp: activation is 0 (sigmoid) or 1 (swish), got " +
                                          std::to_string(activation));
    }
    if (M < 0 || K < 1 || N < 1) {
        return fail(kInvalidArgument, "x must be [M,K]");
    }
    if (N % 8) {
        return fail(kInvalidArgument, "gdp: N must be a multiple of 8");
    }
    if (M == 0) {
        return kOk;
    }
    if (!aligned16(x) || !aligned16(wp) || !aligned16(wg) || !aligned16(out) || bp == nullptr ||
        bg == nullptr || mask == nullptr) {
        return fail(kInvalidArgument, "gdp: buffers must be 16-byte aligned");
    }
    if ((K != 64 && K != 128) || (N != 64 && N != 128)) {
        // other widths: the tile GEMM (K a multiple of 8, N of 8)
        return gdp_general(stream, dtype, x, wp, bp, wg, bg, mask, out, M, K, N, activation);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (dtype == kBF16) {
        e = K == 64 ? gdp_typed<__nv_bfloat16, 64>(s, dtype, x, wp, bp, wg, bg, mask, out, (int)M,
                                                   (int)N, (int)activation)
                    : gdp_typed<__nv_bfloat16, 128>(s, dtype, x, wp, bp, wg, bg, mask, out,
                                                    (int)M, (int)N, (int)activation);
    } else {
        e = K == 64 ? gdp_typed<__half, 64>(s, dtype, x, wp, bp, wg, bg, mask, out, (int)M,
                                            (int)N, (int)activation)
                    : gdp_typed<__half, 128>(s, dtype, x, wp, bp, wg, bg, mask, out, (int)M,
                                             (int)N, (int)activation);
    }
    return launch_status(e, "gdp");
}

// Pair-biased flash attention backward for sm_100a: VoltaMmaBwd.
//
// Given q, k, v, bias, the key mask, the forward's out and log2-domain lse, and dout:
//   P   = exp2(scale*log2e * q.k + log2e * bias - lse)    (a masked key: exp2(-1e4 log2e - lse))
//   dS  = P (dP - delta), dP = dout v^T, delta = rowsum(out * dout); zero on masked keys
//   dV  = P^T dout,  dK = scale dS^T q,  dQ = scale dS k,  dBias = sum over the batch of dS
// as colabfold-legacy-kernels computes them (cuda/volta_mma_attn_bwd.cu:84-383, where P still
// carries dV through a masked key but dS does not). The design is this file's own:
//
//   * one CTA owns a 128-key tile of one (n, h): K and V stay in shared memory, dK and dV
//     accumulate in tensor memory over every query, so both come out bitwise deterministic;
//   * warp roles: a TMA warp streams the 64-query steps (q, dout and the bias tile) two or
//     three stages deep; an MMA warp issues every tcgen05 MMA; two softmax warpgroups take the
//     steps alternately (ping-pong), each with its own S^T/dP^T columns in tensor memory and
//     its own dS buffer, so one group's exponentials overlap the other group's MMAs;
//   * S^T = K Q^T and dP^T = V dout^T (M=128 keys, N=64 queries); worker t owns key t = TMEM
//     lane t, forms P^T and dS^T and writes them back over S^T and dP^T as 16-bit pairs, the
//     A operands of dV += P^T dout and dK += dS^T q (A read from tensor memory);
//   * dS also goes MN-major into swizzled shared memory for dQ = dS k (M=64), whose fp32 tile
//     is added into the workspace accumulator with 16-byte vector atomics;
//   * the bias is transposed once per call into the workspace as f16 [H][Sk][Sq'] (exact for
//     f16 input; bf16 values are kept exactly within f16's range and clamped to +-65504 beyond
//     it), so a key's bias values arrive by TMA as one contiguous 128-byte row;
//   * dBias: each group stages its step's fp32 dS tile [64 queries][128 keys] in shared memory
//     and one thread hands it to TMA as a single bulk reduce-add into dBias (full-line L2
//     reductions); where the dBias rows are not 16-byte multiples (Sk % 4 != 0) the workers add
//     dS with coalesced fp32 reductions instead (a warp covers 32 consecutive keys of a row).
// Around it: the row statistic (delta), the bias transpose, the zero fills, the dQ conversion.
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

constexpr int kBK = 128;  // keys per CTA (= TMEM lanes)
constexpr int kBQ = 64;   // queries per step
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMaskedLogit = -1.0e4f;

struct BwdParams {
    const uint8_t* kmask;
    const float* lse;
    const float* delta;
    float* dq_acc;  // [N,H,Sq,D] fp32, zeroed
    void* dk;
    void* dv;
    float* dbias;   // [H,Sq,Sk] fp32, zeroed
    int N, H, Sq, Sk, D;
    float scale;
};

template <int DP>
struct BGeom {
    static constexpr int AE = DP == 96 ? 32 : DP;
    static constexpr int NA = DP / AE;
    static constexpr int ROWB = AE * 2;
    static constexpr uint32_t LAYOUT = ROWB >= 128 ? kSwizzle128B : ROWB >= 64 ? kSwizzle64B
                                                                               : kSwizzle32B;
    static constexpr int KATOM = kBK * ROWB;  // one atom of a 128-row (key) tile
    static constexpr int QATOM = kBQ * ROWB;  // one atom of a 64-row (query) tile
    static constexpr int KTILE = NA * KATOM;
    static constexpr int QTILE = NA * QATOM;
    static constexpr int BT = kBQ * kBK * 2;  // bias^T tile: [128 keys][64 queries] f16
    static constexpr int DS = kBK * 128;      // dS, MN-major: 128 key rows of 64 queries
    static constexpr int DN = DP;
    static constexpr int NWG = DN <= 32 ? 2 : 1;  // softmax warpgroups (ping-pong)
    static constexpr int NS = NWG == 2 ? 4 : 3;   // query-step stages
    static constexpr int THREADS = NWG * 128 + 64;
    // TMEM columns: group w's S^T at 128w, dP^T at 128w + 64; then dV, dK, one dQ per group
    static constexpr int T_DV = NWG * 128;
    static constexpr int T_DK = T_DV + DN;
    static constexpr int T_DQ = T_DK + DN;
    static constexpr int COLS = T_DQ + NWG * DN;
    static constexpr uint32_t ALLOC = COLS <= 256 ? 256 : 512;
    static_assert(COLS <= 512, "tensor memory");
};

template <int DP>
struct BSmem {
    using G = BGeom<DP>;
    static constexpr int K = 0;
    static constexpr int V = K + G::KTILE;
    static constexpr int STAGE = V + G::KTILE;               // NS x (Q, dO, bias^T)
    static constexpr int STAGE_BYTES = 2 * G::QTILE + G::BT;
    static constexpr int DSB = STAGE + G::NS * STAGE_BYTES;  // NWG dS buffers
    static constexpr int RED = DSB + G::NWG * G::DS;         // NWG fp32 dS tiles [64][128]
    static constexpr int STAT = RED + G::NWG * kBQ * kBK * 4;  // [NWG][2][lse, delta][64] fp32
    static constexpr int END = STAT + G::NWG * 2 * 2 * kBQ * 4;
    static constexpr int BYTES = END + 1024;
    static_assert(BYTES + 256 <= 227 * 1024, "shared memory (dynamic + the static barriers)");
};

// dBias modes
enum DbiasMode : int { kDbiasNone = 0, kDbiasRed = 1, kDbiasTma = 2 };

__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int c0,
                                                  int c1, int c2) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], "
        "[%1];" ::"l"(map),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// until every bulk operation this thread committed has finished reading shared memory
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// A fire-and-forget fp32 add (the result is unused, so it compiles to a reduction); unlike an
// asm statement with a memory clobber it lets the compiler overlap it with neighbouring loads.
__device__ __forceinline__ void red_add_f32(float* p, float v) {
    atomicAdd(p, v);
}

template <typename T, int DP, int DBIAS>
__global__ void __launch_bounds__(BGeom<DP>::THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                    const __grid_constant__ CUtensorMap tbt, const __grid_constant__ CUtensorMap tdb,
                    const BwdParams p) {
    using G = BGeom<DP>;
    using L = BSmem<DP>;
    using E = Elem<T>;
    constexpr int NWG = G::NWG, NS = G::NS;
    constexpr int MMA_WARP = 4 * NWG, TMA_WARP = MMA_WARP + 1;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t kv_full, q_full[NS], q_empty[NS], s_full[2], p_ready[2], mma_done[2];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // key tiles and heads vary fastest, so the CTAs in flight at once reduce into many different
    // dBias tiles rather than all into the same one
    const int k0 = blockIdx.x * kBK, h = blockIdx.y, n = blockIdx.z;
    const int D = p.D;
    const int DN = (D + 15) & ~15;
    const int nqt = (p.Sq + kBQ - 1) / kBQ;
    const long long rowbase = ((long long)n * p.H + h) * p.Sq;

    if (warp == MMA_WARP) {
        if (lane == 0) {
            mbar_init(&kv_full, 1);
            for (int i = 0; i < NS; ++i) {
                mbar_init(&q_full[i], 1);
                mbar_init(&q_empty[i], 1);
            }
            for (int i = 0; i < 2; ++i) {
                mbar_init(&s_full[i], 1);
                mbar_init(&p_ready[i], 128);
                mbar_init(&mma_done[i], 1);
            }
            abort_flag = 0;
            fence_mbar_init();
        }
        __syncwarp();
        tmem_alloc(&tmem_base_sh, G::ALLOC);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;

    if (warp == TMA_WARP) {
        if (lane == 0) {
            mbar_arrive_expect_tx(&kv_full, 2 * G::KTILE);
            for (int a = 0; a < G::NA; ++a) {
                tma_load_4d(smem + L::K + a * G::KATOM, &tk, &kv_full, a * G::AE, h, k0, n);
                tma_load_4d(smem + L::V + a * G::KATOM, &tv, &kv_full, a * G::AE, h, k0, n);
            }
            for (int i = 0; i < nqt; ++i) {
                const int s = i % NS, q0 = i * kBQ;
                if (i >= NS) {
                    mbar_wait(&q_empty[s], ((i - NS) / NS) & 1, &g_status, kStatusMmaWait,
                              &abort_flag);
                }
                uint8_t* st = smem + L::STAGE + s * L::STAGE_BYTES;
                mbar_arrive_expect_tx(&q_full[s], L::STAGE_BYTES);
                for (int a = 0; a < G::NA; ++a) {
                    tma_load_4d(st + a * G::QATOM, &tq, &q_full[s], a * G::AE, h, q0, n);
                    tma_load_4d(st + G::QTILE + a * G::QATOM, &tdo, &q_full[s], a * G::AE, h, q0,
                                n);
                }
                uint8_t* bt = st + 2 * G::QTILE;
                tma_load_3d(bt, &tbt, &q_full[s], q0, k0, h);
            }
        }
    } else if (warp == MMA_WARP) {
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16(E::kBf16, 128, kBQ, false, false);
            const uint32_t idesc_acc = idesc_f16(E::kBf16, 128, DN, false, true);
            const uint32_t idesc_dq = idesc_f16(E::kBf16, 64, DN, true, true);
            const uint32_t k_base = smem_u32(smem + L::K), v_base = smem_u32(smem + L::V);
            mbar_wait(&kv_full, 0, &g_status, kStatusTmaWait, &abort_flag);
            // S^T and dP^T of step i into group (i % NWG)'s columns
            const auto first_half = [&](int i) {
                const int w = i % NWG, s = i % NS;
                mbar_wait(&q_full[s], (i / NS) & 1, &g_status, kStatusTmaWait, &abort_flag);
                if (i >= NWG) {
                    mbar_wait(&mma_done[w], ((i - NWG) / NWG) & 1, &g_status, kStatusMmaWait,
                              &abort_flag);
                }
                tc_fence_after();
                const uint32_t st = smem_u32(smem + L::STAGE + s * L::STAGE_BYTES);
#pragma unroll
                for (int ks = 0; ks < DP / 16; ++ks) {
                    const int a = (ks * 16) / G::AE, off = ((ks * 16) % G::AE) * 2;
                    const uint64_t kd =
                        smem_desc(k_base + a * G::KATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                    const uint64_t vd =
                        smem_desc(v_base + a * G::KATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                    const uint64_t qd =
                        smem_desc(st + a * G::QATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                    const uint64_t od =
                        smem_desc(st + G::QTILE + a * G::QATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                    mma_ss(tmem + 128 * w, kd, qd, idesc_s, ks > 0);
                    mma_ss(tmem + 128 * w + 64, vd, od, idesc_s, ks > 0);
                }
                mma_commit(&s_full[w]);
            };
            // dV, dK and dQ of step j once its group has written P^T, dS^T and dS
            const auto second_half = [&](int j) {
                const int w = j % NWG, s = j % NS;
                mbar_wait(&p_ready[w], (j / NWG) & 1, &g_status, kStatusSyncWait, &abort_flag);
                tc_fence_after();
                const uint32_t st = smem_u32(smem + L::STAGE + s * L::STAGE_BYTES);
#pragma unroll
                for (int ks = 0; ks < kBQ / 16; ++ks) {
                    const uint64_t od = smem_desc(st + G::QTILE + ks * 16 * G::ROWB, G::QATOM,
                                                  8 * G::ROWB, G::LAYOUT);
                    const uint64_t qd =
                        smem_desc(st + ks * 16 * G::ROWB, G::QATOM, 8 * G::ROWB, G::LAYOUT);
                    mma_ts(tmem + G::T_DV, tmem + 128 * w + ks * 8, od, idesc_acc,
                           (j > 0 || ks > 0) ? 1u : 0u);
                    mma_ts(tmem + G::T_DK, tmem + 128 * w + 64 + ks * 8, qd, idesc_acc,
                           (j > 0 || ks > 0) ? 1u : 0u);
                }
                const uint32_t ds_base = smem_u32(smem + L::DSB + w * G::DS);
#pragma unroll
                for (int ks = 0; ks < kBK / 16; ++ks) {
                    const uint64_t ad =
                        smem_desc(ds_base + ks * 16 * 128, G::DS, 1024, kSwizzle128B);
                    const uint64_t bd =
                        smem_desc(k_base + ks * 16 * G::ROWB, G::KATOM, 8 * G::ROWB, G::LAYOUT);
                    mma_ss(tmem + G::T_DQ + w * G::DN, ad, bd, idesc_dq, ks > 0 ? 1u : 0u);
                }
                mma_commit(&mma_done[w]);
                mma_commit(&q_empty[s]);
            };
            for (int i = 0; i <= nqt; ++i) {
                if constexpr (NWG == 2) {
                    // the next step's S^T and dP^T go ahead of this step's accumulations
                    if (i < nqt) {
                        first_half(i);
                    }
                    if (i >= 1) {
                        second_half(i - 1);
                    }
                } else {
                    // one group: its columns are free only after the previous step's MMAs
                    if (i >= 1) {
                        second_half(i - 1);
                    }
                    if (i < nqt) {
                        first_half(i);
                    }
                }
            }
        }
    } else {
        // softmax warpgroups: worker (wg, t) owns key k0 + t = TMEM lane t
        const int wg = warp >> 2, t = ((warp & 3) << 5) | lane;
        const int key = k0 + t;
        const uint32_t lane_base = tmem_lane_base(warp);
        const bool live = key < p.Sk && p.kmask[(long long)n * p.Sk + key] != 0;
        const bool warp_live = __all_sync(0xffffffffu, live);
        const float qk_scale = p.scale * kLog2e;
        const float masked = kMaskedLogit * kLog2e;
        float* stat = reinterpret_cast<float*>(smem + L::STAT) + wg * (2 * 2 * kBQ);
        float* rbuf = reinterpret_cast<float*>(smem + L::RED) + wg * (kBQ * kBK);
        float* dbias_col = p.dbias + (long long)h * p.Sq * p.Sk + key;
        uint8_t* ds_row = smem + L::DSB + wg * G::DS + t * 128;
        const uint32_t t_dq = tmem + G::T_DQ + wg * G::DN;
        const uint32_t t_st = tmem + 128 * wg + lane_base, t_dp = t_st + 64;

        // dQ of a step: lanes 32w + r (r < 16) hold query row 16w + r (M=64 layout)
        const auto flush_dq = [&](int i) {
            const int q = i * kBQ + 16 * (warp & 3) + lane;
            for (int c = 0; c < DN; c += 16) {
                uint32_t r[16];
                tmem_ld16(t_dq + lane_base + c, r);
                tmem_wait_ld();
                if (lane < 16 && q < p.Sq) {
                    float* dst = p.dq_acc + (rowbase + q) * D + c;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        if (c + 4 * g < D) {
                            atomicAdd(reinterpret_cast<float4*>(dst + 4 * g),
                                      make_float4(__uint_as_float(r[4 * g]) * p.scale,
                                                  __uint_as_float(r[4 * g + 1]) * p.scale,
                                                  __uint_as_float(r[4 * g + 2]) * p.scale,
                                                  __uint_as_float(r[4 * g + 3]) * p.scale));
                        }
                    }
                }
            }
        };

        // one 32-query half of a step: P^T, dS^T (TMEM), dS (shared), dBias (global)
        const auto half_step = [&](auto fast, const uint8_t* brow, const float* lsh,
                                   const float* dlh, int half, int q0, int jn) {
            uint32_t sr[32], dr[32];
            tmem_ld32(t_st + 32 * half, sr);
            tmem_ld32(t_dp + 32 * half, dr);
            tmem_wait_ld();
            uint32_t pw[16], dw[16];
            float* drow = dbias_col + (long long)(q0 + 32 * half) * p.Sk;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                // queries 32 half + 4c .. +4: half of 16-byte chunk 4 half + c/2 of the key's row
                const uint2 b2 = *reinterpret_cast<const uint2*>(
                    brow + (((4 * half + (c >> 1)) ^ (t & 7)) << 4) + (c & 1) * 8);
                const float2 b01 = __half22float2(*reinterpret_cast<const __half2*>(&b2.x));
                const float2 b23 = __half22float2(*reinterpret_cast<const __half2*>(&b2.y));
                const float4 l4 = *reinterpret_cast<const float4*>(lsh + 4 * c);
                const float4 d4 = *reinterpret_cast<const float4*>(dlh + 4 * c);
                const float bb[4] = {b01.x * kLog2e, b01.y * kLog2e, b23.x * kLog2e,
                                     b23.y * kLog2e};
                const float ll[4] = {l4.x, l4.y, l4.z, l4.w};
                const float dd[4] = {d4.x, d4.y, d4.z, d4.w};
                float pv[4], gv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 4 * c + e;
                    if constexpr (decltype(fast)::value) {
                        pv[e] = ex2(fmaf(__uint_as_float(sr[j]), qk_scale, bb[e]) - ll[e]);
                        gv[e] = pv[e] * (__uint_as_float(dr[j]) - dd[e]);
                    } else {
                        const float l2 =
                            live ? fmaf(__uint_as_float(sr[j]), qk_scale, bb[e]) : masked;
                        pv[e] = ex2(l2 - ll[e]);
                        gv[e] = live ? pv[e] * (__uint_as_float(dr[j]) - dd[e]) : 0.f;
                    }
                }
                pw[2 * c] = E::pack(pv[0], pv[1]);
                pw[2 * c + 1] = E::pack(pv[2], pv[3]);
                dw[2 * c] = E::pack(gv[0], gv[1]);
                dw[2 * c + 1] = E::pack(gv[2], gv[3]);
                if constexpr (DBIAS == kDbiasTma) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        rbuf[(32 * half + 4 * c + e) * kBK + t] = gv[e];
                    }
                } else if constexpr (DBIAS == kDbiasRed) {
                    if (key < p.Sk) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (4 * c + e < jn) {
                                red_add_f32(drow + (long long)(4 * c + e) * p.Sk, gv[e]);
                            }
                        }
                    }
                }
            }
            tmem_st16(t_st + 16 * half, pw);
            tmem_st16(t_dp + 16 * half, dw);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int chunk = 4 * half + c;
                *reinterpret_cast<uint4*>(ds_row + ((chunk ^ (t & 7)) << 4)) =
                    make_uint4(dw[4 * c], dw[4 * c + 1], dw[4 * c + 2], dw[4 * c + 3]);
            }
        };

        // row statistics of a step: thread t < 64 holds lse of query t, t >= 64 delta of t - 64;
        // loaded one step ahead so that their latency hides behind the current step
        const auto load_stat = [&](int i) {
            const int q = i * kBQ + (t & 63);
            if (i >= nqt || q >= p.Sq) {
                return t < 64 ? INFINITY : 0.f;
            }
            return t < 64 ? p.lse[rowbase + q] : p.delta[rowbase + q];
        };
        float stat_next = load_stat(wg);
        int k = 0;
        for (int i = wg; i < nqt; i += NWG, ++k) {
            const int s = i % NS, q0 = i * kBQ, b = k & 1;
            // this step's row statistics into the group's buffer b
            float* ls = stat + b * (2 * kBQ);
            float* dl = ls + kBQ;
            stat[b * (2 * kBQ) + t] = stat_next;
            if constexpr (DBIAS == kDbiasTma) {
                if (t == 0 && k >= 1) {
                    bulk_wait_read();  // the previous step's reduce has read the dS tile
                }
            }
            named_sync(2 + wg, 128);
            stat_next = load_stat(i + NWG);
            if (k >= 1) {
                // this group's previous step: dQ out of tensor memory before it is reused
                mbar_wait(&mma_done[wg], (k - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
                tc_fence_after();
                flush_dq(i - NWG);
            }
            mbar_wait(&q_full[s], (i / NS) & 1, &g_status, kStatusTmaWait, &abort_flag);
            mbar_wait(&s_full[wg], k & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            const uint8_t* bt = smem + L::STAGE + s * L::STAGE_BYTES + 2 * G::QTILE;
            const int nq = min(kBQ, p.Sq - q0);
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                const uint8_t* brow = bt + t * 128;
                const int jn = min(32, nq - 32 * half);
                if (warp_live) {
                    half_step(std::true_type{}, brow, ls + 32 * half, dl + 32 * half, half, q0, jn);
                } else {
                    half_step(std::false_type{}, brow, ls + 32 * half, dl + 32 * half, half, q0,
                              jn);
                }
            }
            tmem_wait_st();
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(&p_ready[wg]);
            if constexpr (DBIAS == kDbiasTma) {
                // the whole fp32 dS tile in one bulk reduce-add (rows past Sq, keys past Sk clip)
                named_sync(2 + wg, 128);
                if (t == 0) {
                    tma_reduce_add_3d(&tdb, rbuf, k0, q0, h);
                }
            }
        }
        if constexpr (DBIAS == kDbiasTma) {
            if (t == 0) {
                bulk_wait_all();
            }
        }
        if (k >= 1) {
            mbar_wait(&mma_done[wg], (k - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            flush_dq(wg + (k - 1) * NWG);
        }
        // dK (scaled) and dV once the last step's accumulations are done
        const int last = nqt - 1;
        mbar_wait(&mma_done[last % NWG], (last / NWG) & 1, &g_status, kStatusMmaWait,
                  &abort_flag);
        tc_fence_after();
        const long long krow = ((long long)n * p.H + h) * p.Sk + key;
        for (int which = 0; which < 2; ++which) {
            if (NWG == 2 && which != wg) {
                continue;
            }
            const uint32_t acc = tmem + (which == 0 ? G::T_DK : G::T_DV) + lane_base;
            T* dst = reinterpret_cast<T*>(which == 0 ? p.dk : p.dv) + krow * D;
            const float mul = which == 0 ? p.scale : 1.f;
            for (int c = 0; c < DN; c += 16) {
                uint32_t r[16];
                tmem_ld16(acc + c, r);
                tmem_wait_ld();
                if (key < p.Sk) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int c8 = c + 8 * hh;
                        if (c8 < D) {
                            uint4 w;
                            uint32_t* pw = &w.x;
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                pw[e] = E::pack(__uint_as_float(r[8 * hh + 2 * e]) * mul,
                                                __uint_as_float(r[8 * hh + 2 * e + 1]) * mul);
                            }
                            *reinterpret_cast<uint4*>(dst + c8) = w;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, G::ALLOC);
    }
}

// delta[row] = sum_c out[row][c] * dout[row][c], one thread per row, 16-byte loads
template <typename T>
__global__ void row_delta_kernel(const T* __restrict__ out, const T* __restrict__ dout,
                                 float* __restrict__ delta, long long rows, int D) {
    using E = Elem<T>;
    const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) {
        return;
    }
    const uint4* o = reinterpret_cast<const uint4*>(out + r * D);
    const uint4* g = reinterpret_cast<const uint4*>(dout + r * D);
    float s = 0.f;
    for (int c = 0; c < D / 8; ++c) {
        const uint4 a = o[c], b = g[c];
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 x = E::unpack(aw[e]), y = E::unpack(bw[e]);
            s = fmaf(x.x, y.x, s);
            s = fmaf(x.y, y.y, s);
        }
    }
    delta[r] = s;
}

// bt[h][k][q] = log2e * bias[h][q][k] in fp32, queries padded to Sqp with zeros; 32x32 tiles
template <typename T>
__global__ void bias_transpose_kernel(const T* __restrict__ bias, __half* __restrict__ bt, int Sq,
                                      int Sk, int Sqp) {
    __shared__ float tile[32][33];
    const int h = blockIdx.z, q0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const T* src = bias + (long long)h * Sq * Sk;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int q = q0 + r, k = k0 + threadIdx.x;
        tile[r][threadIdx.x] =
            (q < Sq && k < Sk) ? Elem<T>::to_f(src[(long long)q * Sk + k]) : 0.f;
    }
    __syncthreads();
    __half* dst = bt + (long long)h * Sk * Sqp;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, q = q0 + threadIdx.x;
        if (k < Sk && q < Sqp) {
            dst[(long long)k * Sqp + q] =
                __float2half_rn(fminf(fmaxf(tile[threadIdx.x][r], -65504.f), 65504.f));
        }
    }
}

// dq = dq_acc rounded to 16 bits, 8 elements a thread
template <typename T>
__global__ void dq_convert_kernel(const float* __restrict__ acc, T* __restrict__ dq,
                                  long long n8) {
    using E = Elem<T>;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 a = reinterpret_cast<const float4*>(acc)[2 * i];
        const float4 b = reinterpret_cast<const float4*>(acc)[2 * i + 1];
        uint4 w;
        w.x = E::pack(a.x, a.y);
        w.y = E::pack(a.z, a.w);
        w.z = E::pack(b.x, b.y);
        w.w = E::pack(b.z, b.w);
        reinterpret_cast<uint4*>(dq)[i] = w;
    }
}

size_t align256(size_t x) {
    return (x + 255) & ~size_t(255);
}

int padded_dim(int D) {
    return D <= 16 ? 16 : D <= 32 ? 32 : D <= 64 ? 64 : 96;
}

bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// Workspace: dQ accumulator | row statistic | bias^T (f16, queries padded to a multiple of 8),
// each 256-byte aligned
struct Workspace {
    size_t dq, delta, bt, total;
    static Workspace of(size_t N, size_t H, size_t Sq, size_t Sk, size_t D) {
        Workspace w;
        const size_t rows = N * H * Sq, sqp = (Sq + 7) & ~size_t(7);
        w.dq = 0;
        w.delta = align256(rows * D * sizeof(float));
        w.bt = w.delta + align256(rows * sizeof(float));
        w.total = w.bt + align256(H * Sk * sqp * sizeof(__half));
        return w;
    }
};

template <typename T, int DP, int DB>
cudaError_t launch_main(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p) {
    auto kern = attn_bwd_kernel<T, DP, DB>;
    const int smem = BSmem<DP>::BYTES;
    static bool attr_done[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < kMaxDevices && !attr_done[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) {
            return e;
        }
        attr_done[dev] = true;
    }
    const dim3 grid((p.Sk + kBK - 1) / kBK, p.H, p.N);
    kern<<<grid, BGeom<DP>::THREADS, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], maps[4],
                                                     maps[5], p);
    return cudaGetLastError();
}

template <typename T, int DP>
cudaError_t launch_dp(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p, int db) {
    return db == kDbiasTma   ? launch_main<T, DP, kDbiasTma>(stream, maps, p)
           : db == kDbiasRed ? launch_main<T, DP, kDbiasRed>(stream, maps, p)
                             : launch_main<T, DP, kDbiasNone>(stream, maps, p);
}

template <typename T>
cudaError_t run_backward(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p,
                         const void* bias, __half* bt, int Sqp, const void* out, const void* dout,
                         float* delta, void* dq, int dbias_mode) {
    const long long rows = (long long)p.N * p.H * p.Sq;
    cudaError_t e;
    if ((e = cudaMemsetAsync(p.dbias, 0, sizeof(float) * (size_t)p.H * p.Sq * p.Sk, stream)) !=
        cudaSuccess) {
        return e;
    }
    if ((e = cudaMemsetAsync(p.dq_acc, 0, sizeof(float) * (size_t)rows * p.D, stream)) !=
        cudaSuccess) {
        return e;
    }
    row_delta_kernel<T><<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(
        static_cast<const T*>(out), static_cast<const T*>(dout), delta, rows, p.D);
    const dim3 tgrid((Sqp + 31) / 32, (p.Sk + 31) / 32, p.H);
    bias_transpose_kernel<T><<<tgrid, dim3(32, 8), 0, stream>>>(static_cast<const T*>(bias), bt,
                                                                 p.Sq, p.Sk, Sqp);
    if ((e = cudaGetLastError()) != cudaSuccess) {
        return e;
    }
    const int DP = padded_dim(p.D);
    e = DP == 16   ? launch_dp<T, 16>(stream, maps, p, dbias_mode)
        : DP == 32 ? launch_dp<T, 32>(stream, maps, p, dbias_mode)
        : DP == 64 ? launch_dp<T, 64>(stream, maps, p, dbias_mode)
                   : launch_dp<T, 96>(stream, maps, p, dbias_mode);
    if (e != cudaSuccess) {
        return e;
    }
    const long long n8 = rows * p.D / 8;
    dq_convert_kernel<T><<<(unsigned)std::min<long long>((n8 + 255) / 256, 148 * 16), 256, 0,
                           stream>>>(p.dq_acc, static_cast<T*>(dq), n8);
    return cudaGetLastError();
}

}  // namespace

unsigned read_and_clear_status_bwd() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    return v;
}

}  // namespace cflk

using namespace cflk;

extern "C" int cflk_volta_mma_bwd_workspace_size(int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                                                 int64_t D, size_t* bytes) {
    clear_error();
    if (N < 0 || H < 0 || Sq < 0 || Sk < 0 || D < 0 || bytes == nullptr) {
        return fail(kInvalidArgument, "volta_mma_bwd: bad sizes");
    }
    *bytes = Workspace::of(N, H, Sq, Sk, D).total;
    return kOk;
}

extern "C" int cflk_volta_mma_bwd(void* stream_, int dtype, const void* q, const void* k,
                                  const void* v, const void* bias, const uint8_t* kmask,
                                  const void* out, const void* dout, const float* lse, void* dq,
                                  void* dk, void* dv, float* dbias, void* workspace,
                                  size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq,
                                  int64_t Sk, int64_t D, float scale, int want_dbias) {
    clear_error();
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, "volta_mma_bwd: dtype must be f16 or bf16");
    }
    if (N < 0 || H < 0 || Sq < 0 || Sk < 0) {
        return fail(kInvalidArgument, "q must be [N,H,S,D]");
    }
    if (D != 8 && D != 16 && D != 24 && D != 32 && D != 48 && D != 64 && D != 96) {
        return fail(kInvalidArgument, "volta_mma_bwd: unsupported head dim");
    }
    const Workspace ws = Workspace::of(N, H, Sq, Sk, D);
    if (workspace_bytes < ws.total || (ws.total > 0 && workspace == nullptr) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255) != 0) {
        return fail(kInternal, "volta_mma_bwd: no scratch for the dQ accumulator");
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(dout) ||
        !aligned16(dq) || !aligned16(dk) || !aligned16(dv)) {
        return fail(kInvalidArgument, "volta_mma_bwd: buffers must be 16-byte aligned");
    }
    const size_t rows = (size_t)N * H * Sq;
    uint8_t* wsb = static_cast<uint8_t*>(workspace);
    float* dq_acc = reinterpret_cast<float*>(wsb + ws.dq);
    float* delta = reinterpret_cast<float*>(wsb + ws.delta);
    __half* bt = reinterpret_cast<__half*>(wsb + ws.bt);
    const int Sqp = (int)((Sq + 7) & ~int64_t(7));
    if (H == 0 || Sq == 0 || Sk == 0 || N == 0) {
        // nothing to differentiate: zero what exists
        if (H > 0 && Sq > 0 && Sk > 0) {
            cudaMemsetAsync(dbias, 0, sizeof(float) * (size_t)H * Sq * Sk, stream);
        }
        if (rows > 0) {
            cudaMemsetAsync(dq, 0, rows * D * 2, stream);
        }
        if (N * H * Sk > 0) {
            cudaMemsetAsync(dk, 0, (size_t)N * H * Sk * D * 2, stream);
            cudaMemsetAsync(dv, 0, (size_t)N * H * Sk * D * 2, stream);
        }
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? kOk
                                : fail(kInternal, std::string("volta_mma_bwd launch: ") +
                                                      cudaGetErrorString(e));
    }
    const CUtensorMapDataType tdt =
        dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int DP = padded_dim((int)D);
    const int AE = DP == 96 ? 32 : DP;
    CUtensorMap maps[6];
    {
        const uint64_t dq4[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)Sq, (uint64_t)N};
        const uint64_t sq4[3] = {(uint64_t)(Sq * D), (uint64_t)D, (uint64_t)(H * Sq * D)};
        const uint64_t dk4[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)Sk, (uint64_t)N};
        const uint64_t sk4[3] = {(uint64_t)(Sk * D), (uint64_t)D, (uint64_t)(H * Sk * D)};
        const uint32_t boxq[4] = {(uint32_t)AE, 1, (uint32_t)kBQ, 1};
        const uint32_t boxk[4] = {(uint32_t)AE, 1, (uint32_t)kBK, 1};
        const CUtensorMapSwizzle sw = swizzle_for_row(AE * 2);
        const uint64_t dbt[3] = {(uint64_t)Sqp, (uint64_t)Sk, (uint64_t)H};
        const uint64_t sbt[2] = {(uint64_t)Sqp, (uint64_t)Sk * (uint64_t)Sqp};
        const uint32_t boxbt[3] = {(uint32_t)kBQ, (uint32_t)kBK, 1};
        if (!encode_tiled(&maps[0], tdt, 2, 4, q, dq4, sq4, boxq, sw) ||
            !encode_tiled(&maps[1], tdt, 2, 4, k, dk4, sk4, boxk, sw) ||
            !encode_tiled(&maps[2], tdt, 2, 4, v, dk4, sk4, boxk, sw) ||
            !encode_tiled(&maps[3], tdt, 2, 4, dout, dq4, sq4, boxq, sw) ||
            !encode_tiled(&maps[4], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 3, bt, dbt, sbt, boxbt,
                          CU_TENSOR_MAP_SWIZZLE_128B)) {
            return fail(kInvalidArgument, "volta_mma_bwd: TMA descriptor rejected");
        }
    }
    // dBias by TMA bulk reduce where its rows are 16-byte multiples, else by fp32 reductions
    int dbias_mode = want_dbias ? kDbiasRed : kDbiasNone;
    maps[5] = maps[4];
    if (want_dbias && Sk % 4 == 0 && (reinterpret_cast<uintptr_t>(dbias) & 15) == 0) {
        const uint64_t ddb[3] = {(uint64_t)Sk, (uint64_t)Sq, (uint64_t)H};
        const uint64_t sdb[2] = {(uint64_t)Sk, (uint64_t)Sq * (uint64_t)Sk};
        const uint32_t boxdb[3] = {(uint32_t)kBK, (uint32_t)kBQ, 1};
        if (encode_tiled(&maps[5], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 3, dbias, ddb, sdb, boxdb,
                         CU_TENSOR_MAP_SWIZZLE_NONE)) {
            dbias_mode = kDbiasTma;
        }
    }
    BwdParams p;
    p.kmask = kmask;
    p.lse = lse;
    p.delta = delta;
    p.dq_acc = dq_acc;
    p.dk = dk;
    p.dv = dv;
    p.dbias = dbias;
    p.N = (int)N;
    p.H = (int)H;
    p.Sq = (int)Sq;
    p.Sk = (int)Sk;
    p.D = (int)D;
    p.scale = scale;
    const cudaError_t e =
        dtype == kBF16 ? run_backward<__nv_bfloat16>(stream, maps, p, bias, bt, Sqp, out, dout,
                                                     delta, dq, dbias_mode)
                       : run_backward<__half>(stream, maps, p, bias, bt, Sqp, out, dout, delta,
                                              dq, dbias_mode);
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("volta_mma_bwd launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

// ---------------------------------------------------------------------------------------------
// The backward without caller-provided workspace.
//
// Some callers of this library cannot allocate device memory: a plugin host that owns every
// device allocation and hands a kernel only its inputs and outputs (no scratch allocator), or
// latency-critical code that must not call cudaMalloc because it may synchronise the device.
// For them the backward's scratch (the float32 dQ accumulator, the row statistic and the
// transposed bias) lives in this file-scope array instead, kNoAllocScratchBytes long. Every GPU
// that loads the library holds the array until the process exits. All calls on a device share
// it and it keeps the last call's contents: the backward rewrites or zero-fills every part of it
// on every call, and calls whose kernels overlap on the GPU (different streams, no ordering)
// race on it.
// ---------------------------------------------------------------------------------------------
static constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The array's device address on the current device, looked up once per device. The host-side
// name g_noalloc_scratch is only a stand-in for the symbol, never a device pointer.
static int noalloc_scratch(void** out) {
    static void* addr[cflk::kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        return cflk::fail(cflk::kInternal, std::string("volta_mma_bwd_noalloc: ") +
                                               cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= cflk::kMaxDevices) {
        return cflk::fail(cflk::kInternal, "volta_mma_bwd_noalloc: device ordinal out of range");
    }
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            return cflk::fail(cflk::kInternal,
                              std::string("volta_mma_bwd_noalloc: scratch address: ") +
                                  cudaGetErrorString(e));
        }
        addr[dev] = p;
    }
    *out = addr[dev];
    return cflk::kOk;
}

extern "C" size_t cflk_volta_mma_bwd_noalloc_max_scratch(void) {
    return kNoAllocScratchBytes;
}

extern "C" int cflk_volta_mma_bwd_noalloc(void* stream, int dtype, const void* q, const void* k,
                                          const void* v, const void* bias, const uint8_t* kmask,
                                          const void* out, const void* dout, const float* lse,
                                          void* dq, void* dk, void* dv, float* dbias, int64_t N,
                                          int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                          float scale, int want_dbias) {
    cflk::clear_error();
    size_t need = 0;
    int rc = cflk_volta_mma_bwd_workspace_size(N, H, Sq, Sk, D, &need);
    if (rc != cflk::kOk) {
        return rc;
    }
    if (need > kNoAllocScratchBytes) {
        return cflk::fail(cflk::kInvalidArgument,
                          "volta_mma_bwd_noalloc: needs " + std::to_string(need) +
                              " bytes of scratch, the static scratch holds " +
                              std::to_string(kNoAllocScratchBytes) +
                              " (cflk_volta_mma_bwd_workspace_size: about 4*N*H*Sq*(D+1) + "
                              "2*H*Sk*Sq bytes); use cflk_volta_mma_bwd with a workspace");
    }
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc != cflk::kOk) {
        return rc;
    }
    return cflk_volta_mma_bwd(stream, dtype, q, k, v, bias, kmask, out, dout, lse, dq, dk, dv,
                              dbias, scratch, kNoAllocScratchBytes, N, H, Sq, Sk, D, scale,
                              want_dbias);
}

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
//     accumulate in tensor memory, so both come out bitwise deterministic;
//   * it walks the queries 64 at a time; TMA brings Q, dout and the bias tile two stages deep;
//   * S^T = K Q^T and dP^T = V dout^T are tcgen05 MMAs (M=128 keys, N=64 queries); thread t owns
//     key t = TMEM lane t, forms P^T and dS^T in registers and writes them back over S^T and
//     dP^T as 16-bit pairs, the A operands of dV += P^T dout and dK += dS^T q (A from TMEM);
//   * dS is also stored MN-major in swizzled shared memory for dQ = dS k (M=64), whose fp32
//     tile is added into a workspace accumulator with 16-byte vector atomics;
//   * dBias gets dS by coalesced fp32 reductions (a warp covers 32 consecutive keys of a row).
// Around it: a row-statistic kernel (delta), the zero fills, and the dQ conversion.
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
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMaskedLogit = -1.0e4f;

struct BwdParams {
    const void* bias;
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
    static constexpr int BIAS = kBQ * kBK * 2;  // two 64-key regions of 64 rows, 128B swizzle
    static constexpr int DS = kBK * 128;        // dS, MN-major: 128 key rows of 64 queries
    // TMEM columns: S^T [0,64), dP^T [64,128), dV, dK, dQ after them
    static constexpr int DN = DP == 96 ? 96 : DP;
    static constexpr uint32_t COLS_USED = 128 + 3 * DN;
    static constexpr uint32_t TMEM_COLS = COLS_USED <= 256 ? 256 : 512;
};

template <int DP, bool BIAS_TMA>
struct BSmem {
    using G = BGeom<DP>;
    static constexpr int K = 0;
    static constexpr int V = K + G::KTILE;
    static constexpr int Q0 = V + G::KTILE;            // 2 stages
    static constexpr int O0 = Q0 + 2 * G::QTILE;       // dout, 2 stages
    static constexpr int DSB = O0 + 2 * G::QTILE;      // dS
    static constexpr int B0 = DSB + G::DS;             // bias, 2 stages
    static constexpr int STAT = B0 + (BIAS_TMA ? 2 * G::BIAS : 0);  // lse, delta: 2 stages
    static constexpr int END = STAT + 2 * 2 * kBQ * 4;
    static constexpr int BYTES = END + 1024;
};

template <typename T, int DP, bool BIAS_TMA, bool WANT_DBIAS>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                    const __grid_constant__ CUtensorMap tb, const BwdParams p) {
    using G = BGeom<DP>;
    using L = BSmem<DP, BIAS_TMA>;
    using E = Elem<T>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t bar_kv, bar_full[2], bar_s, bar_mma;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = blockIdx.x, h = blockIdx.y, k0 = blockIdx.z * kBK;
    const int key = k0 + tid;
    const int D = p.D;
    const int DN = (D + 15) & ~15;
    const int nqt = (p.Sq + kBQ - 1) / kBQ;
    float* lse_s = reinterpret_cast<float*>(smem + L::STAT);          // [2][64]
    float* delta_s = lse_s + 2 * kBQ;                                  // [2][64]
    const long long rowbase = ((long long)n * p.H + h) * p.Sq;

    if (tid == 0) {
        mbar_init(&bar_kv, 1);
        mbar_init(&bar_full[0], 1);
        mbar_init(&bar_full[1], 1);
        mbar_init(&bar_s, 1);
        mbar_init(&bar_mma, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base_sh, G::TMEM_COLS);
        tmem_relinquish();
    }
    const auto load_stats = [&](int i) {
        const int s = i & 1, q = i * kBQ + (tid & 63);
        if (tid < 64) {
            lse_s[s * kBQ + (tid & 63)] = q < p.Sq ? p.lse[rowbase + q] : INFINITY;
        } else {
            delta_s[s * kBQ + (tid & 63)] = q < p.Sq ? p.delta[rowbase + q] : 0.f;
        }
    };
    load_stats(0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t t_st = tmem, t_dpt = tmem + 64;
    const uint32_t t_dv = tmem + 128, t_dk = t_dv + G::DN, t_dq = t_dk + G::DN;
    const uint32_t lane_base = tmem_lane_base(warp);

    constexpr uint32_t STAGE_TX = 2 * G::QTILE + (BIAS_TMA ? G::BIAS : 0);
    const auto load_tile = [&](int i) {
        const int s = i & 1, q0 = i * kBQ;
        mbar_arrive_expect_tx(&bar_full[s], STAGE_TX);
        for (int a = 0; a < G::NA; ++a) {
            tma_load_4d(smem + L::Q0 + s * G::QTILE + a * G::QATOM, &tq, &bar_full[s], a * G::AE,
                        h, q0, n);
            tma_load_4d(smem + L::O0 + s * G::QTILE + a * G::QATOM, &tdo, &bar_full[s],
                        a * G::AE, h, q0, n);
        }
        if constexpr (BIAS_TMA) {
            uint8_t* b = smem + L::B0 + s * G::BIAS;
            tma_load_3d(b, &tb, &bar_full[s], k0, q0, h);
            tma_load_3d(b + kBQ * 128, &tb, &bar_full[s], k0 + 64, q0, h);
        }
    };
    if (tid == 0) {
        mbar_arrive_expect_tx(&bar_kv, 2 * G::KTILE);
        for (int a = 0; a < G::NA; ++a) {
            tma_load_4d(smem + L::K + a * G::KATOM, &tk, &bar_kv, a * G::AE, h, k0, n);
            tma_load_4d(smem + L::V + a * G::KATOM, &tv, &bar_kv, a * G::AE, h, k0, n);
        }
        load_tile(0);
    }

    const bool live = key < p.Sk && p.kmask[(long long)n * p.Sk + key] != 0;
    const float qk_scale = p.scale * kLog2e;
    const float masked = kMaskedLogit * kLog2e;
    const uint32_t idesc_s = idesc_f16(E::kBf16, 128, kBQ, false, false);
    const uint32_t idesc_acc = idesc_f16(E::kBf16, 128, DN, false, true);
    const uint32_t idesc_dq = idesc_f16(E::kBf16, 64, DN, true, true);
    const uint32_t k_base = smem_u32(smem + L::K), v_base = smem_u32(smem + L::V);
    const uint32_t ds_base = smem_u32(smem + L::DSB);
    const T* bias_g = reinterpret_cast<const T*>(p.bias) + (long long)h * p.Sq * p.Sk;

    // dQ of step i: lanes 32w + r (r < 16) hold query row 16w + r (M=64 accumulator layout)
    const auto flush_dq = [&](int i) {
        const int q = i * kBQ + 16 * warp + lane;
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

    for (int i = 0; i < nqt; ++i) {
        const int s = i & 1, q0 = i * kBQ;
        if (tid == 0) {
            if (i > 0) {
                mbar_wait(&bar_mma, (i - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            }
            if (i + 1 < nqt) {
                load_tile(i + 1);
            }
            if (i == 0) {
                mbar_wait(&bar_kv, 0, &g_status, kStatusTmaWait, &abort_flag);
            }
            mbar_wait(&bar_full[s], (i >> 1) & 1, &g_status, kStatusTmaWait, &abort_flag);
            tc_fence_after();
            const uint32_t q_base = smem_u32(smem + L::Q0 + s * G::QTILE);
            const uint32_t o_base = smem_u32(smem + L::O0 + s * G::QTILE);
#pragma unroll
            for (int ks = 0; ks < DP / 16; ++ks) {
                const int a = (ks * 16) / G::AE, off = ((ks * 16) % G::AE) * 2;
                const uint64_t kd = smem_desc(k_base + a * G::KATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                const uint64_t vd = smem_desc(v_base + a * G::KATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                const uint64_t qd = smem_desc(q_base + a * G::QATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                const uint64_t od = smem_desc(o_base + a * G::QATOM + off, 16, 8 * G::ROWB, G::LAYOUT);
                mma_ss(t_st, kd, qd, idesc_s, ks > 0);
                mma_ss(t_dpt, vd, od, idesc_s, ks > 0);
            }
            mma_commit(&bar_s);
        }
        __syncwarp();
        if (i > 0) {
            // dQ of the previous step, before this step's dQ MMA reuses its columns
            mbar_wait(&bar_mma, (i - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            flush_dq(i - 1);
        }
        if (i + 1 < nqt) {
            load_stats(i + 1);  // read after this step's barrier
        }
        mbar_wait(&bar_s, i & 1, &g_status, kStatusMmaWait, &abort_flag);
        tc_fence_after();

        float st[kBQ], dpt[kBQ];
        {
            uint32_t r[32];
            tmem_ld32(t_st + lane_base, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) st[j] = __uint_as_float(r[j]);
            tmem_ld32(t_st + lane_base + 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) st[32 + j] = __uint_as_float(r[j]);
            tmem_ld32(t_dpt + lane_base, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) dpt[j] = __uint_as_float(r[j]);
            tmem_ld32(t_dpt + lane_base + 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) dpt[32 + j] = __uint_as_float(r[j]);
        }
        const float* ls = lse_s + s * kBQ;
        const float* dl = delta_s + s * kBQ;
        const uint8_t* bstage = smem + L::B0 + s * G::BIAS;
        const int kk = tid & 63;
        const uint8_t* bregion = bstage + (tid >> 6) * (kBQ * 128);
        uint8_t* ds_row = smem + L::DSB + tid * 128;
        float* dbias_col = p.dbias + (long long)h * p.Sq * p.Sk + key;

#pragma unroll
        for (int c = 0; c < kBQ / 16; ++c) {
            uint32_t pw[8], dw[8];
#pragma unroll
            for (int jj = 0; jj < 16; jj += 2) {
                float pv[2], dv[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int j = 16 * c + jj + e;
                    float b;
                    if constexpr (BIAS_TMA) {
                        const int phys = (kk >> 3) ^ (j & 7);
                        b = E::to_f(*reinterpret_cast<const T*>(bregion + j * 128 + (phys << 4) +
                                                                 (kk & 7) * 2));
                    } else {
                        const int q = q0 + j;
                        b = (q < p.Sq && key < p.Sk) ? E::to_f(bias_g[(long long)q * p.Sk + key])
                                                     : 0.f;
                    }
                    const float l2 = live ? fmaf(st[j], qk_scale, b * kLog2e) : masked;
                    const float pp = ex2(l2 - ls[j]);
                    const float g = live ? pp * (dpt[j] - dl[j]) : 0.f;
                    pv[e] = pp;
                    dv[e] = g;
                    if constexpr (WANT_DBIAS) {
                        if (g != 0.f) {
                            atomicAdd(dbias_col + (long long)(q0 + j) * p.Sk, g);
                        }
                    }
                }
                pw[jj >> 1] = E::pack(pv[0], pv[1]);
                dw[jj >> 1] = E::pack(dv[0], dv[1]);
            }
            tmem_st8(t_st + lane_base + 8 * c, pw);
            tmem_st8(t_dpt + lane_base + 8 * c, dw);
            // dS row (this key): queries 16c..16c+15 are chunks 2c, 2c+1 of the 128-byte row
            *reinterpret_cast<uint4*>(ds_row + (((2 * c) ^ (tid & 7)) << 4)) =
                make_uint4(dw[0], dw[1], dw[2], dw[3]);
            *reinterpret_cast<uint4*>(ds_row + (((2 * c + 1) ^ (tid & 7)) << 4)) =
                make_uint4(dw[4], dw[5], dw[6], dw[7]);
        }
        tmem_wait_st();
        fence_async_smem();
        tc_fence_before();
        __syncthreads();

        if (tid == 0) {
            tc_fence_after();
            const uint32_t q_base = smem_u32(smem + L::Q0 + s * G::QTILE);
            const uint32_t o_base = smem_u32(smem + L::O0 + s * G::QTILE);
#pragma unroll
            for (int ks = 0; ks < kBQ / 16; ++ks) {
                const uint64_t od =
                    smem_desc(o_base + ks * 16 * G::ROWB, G::QATOM, 8 * G::ROWB, G::LAYOUT);
                const uint64_t qd =
                    smem_desc(q_base + ks * 16 * G::ROWB, G::QATOM, 8 * G::ROWB, G::LAYOUT);
                mma_ts(t_dv, t_st + ks * 8, od, idesc_acc, (i > 0 || ks > 0) ? 1u : 0u);
                mma_ts(t_dk, t_dpt + ks * 8, qd, idesc_acc, (i > 0 || ks > 0) ? 1u : 0u);
            }
#pragma unroll
            for (int ks = 0; ks < kBK / 16; ++ks) {
                const uint64_t ad =
                    smem_desc(ds_base + ks * 16 * 128, G::DS, 1024, kSwizzle128B);
                const uint64_t bd =
                    smem_desc(k_base + ks * 16 * G::ROWB, G::KATOM, 8 * G::ROWB, G::LAYOUT);
                mma_ss(t_dq, ad, bd, idesc_dq, ks > 0 ? 1u : 0u);
            }
            mma_commit(&bar_mma);
        }
    }

    __syncwarp();
    mbar_wait(&bar_mma, (nqt - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
    tc_fence_after();
    flush_dq(nqt - 1);
    // dK (scaled) and dV rows of this key tile
    T* dk_row = reinterpret_cast<T*>(p.dk) + (rowbase / p.Sq * p.Sk + key) * (long long)D;
    T* dv_row = reinterpret_cast<T*>(p.dv) + (rowbase / p.Sq * p.Sk + key) * (long long)D;
    for (int c = 0; c < DN; c += 16) {
        uint32_t rk[16], rv[16];
        tmem_ld16(t_dk + lane_base + c, rk);
        tmem_ld16(t_dv + lane_base + c, rv);
        tmem_wait_ld();
        if (key < p.Sk) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int c8 = c + 8 * half;
                if (c8 < D) {
                    uint4 wk, wv;
                    uint32_t* pk = &wk.x;
                    uint32_t* pv = &wv.x;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        pk[e] = E::pack(__uint_as_float(rk[8 * half + 2 * e]) * p.scale,
                                        __uint_as_float(rk[8 * half + 2 * e + 1]) * p.scale);
                        pv[e] = E::pack(__uint_as_float(rv[8 * half + 2 * e]),
                                        __uint_as_float(rv[8 * half + 2 * e + 1]));
                    }
                    *reinterpret_cast<uint4*>(dk_row + c8) = wk;
                    *reinterpret_cast<uint4*>(dv_row + c8) = wv;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tmem_dealloc(tmem, G::TMEM_COLS);
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

template <typename T, int DP, bool BT, bool DB>
cudaError_t launch_main(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p) {
    auto kern = attn_bwd_kernel<T, DP, BT, DB>;
    const int smem = BSmem<DP, BT>::BYTES;
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
    const dim3 grid(p.N, p.H, (p.Sk + kBK - 1) / kBK);
    kern<<<grid, kThreads, smem, stream>>>(maps[0], maps[1], maps[2], maps[3], maps[4], p);
    return cudaGetLastError();
}

template <typename T, int DP>
cudaError_t launch_dp(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p, bool bt,
                      bool db) {
    if (bt) {
        return db ? launch_main<T, DP, true, true>(stream, maps, p)
                  : launch_main<T, DP, true, false>(stream, maps, p);
    }
    return db ? launch_main<T, DP, false, true>(stream, maps, p)
              : launch_main<T, DP, false, false>(stream, maps, p);
}

template <typename T>
cudaError_t run_backward(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p,
                         const void* out, const void* dout, float* delta, void* dq,
                         bool bias_tma, bool want_dbias) {
    const long long rows = (long long)p.N * p.H * p.Sq;
    cudaError_t e;
    if ((e = cudaMemsetAsync(p.dbias, 0, sizeof(float) * (size_t)p.H * p.Sq * p.Sk, stream)) !=
        cudaSuccess) {
        return e;
    }
    if (rows == 0) {
        return cudaSuccess;
    }
    if ((e = cudaMemsetAsync(p.dq_acc, 0, sizeof(float) * (size_t)rows * p.D, stream)) !=
        cudaSuccess) {
        return e;
    }
    row_delta_kernel<T><<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(
        static_cast<const T*>(out), static_cast<const T*>(dout), delta, rows, p.D);
    if ((e = cudaGetLastError()) != cudaSuccess) {
        return e;
    }
    if (p.Sk > 0) {
        const int DP = padded_dim(p.D);
        e = DP == 16   ? launch_dp<T, 16>(stream, maps, p, bias_tma, want_dbias)
            : DP == 32 ? launch_dp<T, 32>(stream, maps, p, bias_tma, want_dbias)
            : DP == 64 ? launch_dp<T, 64>(stream, maps, p, bias_tma, want_dbias)
                       : launch_dp<T, 96>(stream, maps, p, bias_tma, want_dbias);
        if (e != cudaSuccess) {
            return e;
        }
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
    const size_t rows = (size_t)N * H * Sq;
    *bytes = align256(rows * D * sizeof(float)) + align256(rows * sizeof(float));
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
    size_t need = 0;
    cflk_volta_mma_bwd_workspace_size(N, H, Sq, Sk, D, &need);
    if (workspace_bytes < need || (need > 0 && workspace == nullptr) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255) != 0) {
        return fail(kInternal, "volta_mma_bwd: no scratch for the dQ accumulator");
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(dout) ||
        !aligned16(dq) || !aligned16(dk) || !aligned16(dv)) {
        return fail(kInvalidArgument, "volta_mma_bwd: buffers must be 16-byte aligned");
    }
    const size_t rows = (size_t)N * H * Sq;
    float* dq_acc = static_cast<float*>(workspace);
    float* delta = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                            align256(rows * D * sizeof(float)));
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
    CUtensorMap maps[5];
    {
        const uint64_t dq4[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)Sq, (uint64_t)N};
        const uint64_t sq4[3] = {(uint64_t)(Sq * D), (uint64_t)D, (uint64_t)(H * Sq * D)};
        const uint64_t dk4[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)Sk, (uint64_t)N};
        const uint64_t sk4[3] = {(uint64_t)(Sk * D), (uint64_t)D, (uint64_t)(H * Sk * D)};
        const uint32_t boxq[4] = {(uint32_t)AE, 1, (uint32_t)kBQ, 1};
        const uint32_t boxk[4] = {(uint32_t)AE, 1, (uint32_t)kBK, 1};
        const CUtensorMapSwizzle sw = swizzle_for_row(AE * 2);
        if (!encode_tiled(&maps[0], tdt, 2, 4, q, dq4, sq4, boxq, sw) ||
            !encode_tiled(&maps[1], tdt, 2, 4, k, dk4, sk4, boxk, sw) ||
            !encode_tiled(&maps[2], tdt, 2, 4, v, dk4, sk4, boxk, sw) ||
            !encode_tiled(&maps[3], tdt, 2, 4, dout, dq4, sq4, boxq, sw)) {
            return fail(kInvalidArgument, "volta_mma_bwd: TMA descriptor rejected");
        }
    }
    const bool bias_tma = Sk % 8 == 0 && aligned16(bias);
    maps[4] = maps[0];
    if (bias_tma) {
        const uint64_t db[3] = {(uint64_t)Sk, (uint64_t)Sq, (uint64_t)H};
        const uint64_t sb[2] = {(uint64_t)Sk, (uint64_t)(Sq * Sk)};
        const uint32_t box[3] = {64, (uint32_t)kBQ, 1};
        if (!encode_tiled(&maps[4], tdt, 2, 3, bias, db, sb, box, CU_TENSOR_MAP_SWIZZLE_128B)) {
            return fail(kInvalidArgument, "volta_mma_bwd: TMA descriptor rejected (bias)");
        }
    }
    BwdParams p;
    p.bias = bias;
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
        dtype == kBF16
            ? run_backward<__nv_bfloat16>(stream, maps, p, out, dout, delta, dq, bias_tma,
                                          want_dbias != 0)
            : run_backward<__half>(stream, maps, p, out, dout, delta, dq, bias_tma,
                                   want_dbias != 0);
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
// For them the backward's scratch (the float32 dQ accumulator and the row statistic) lives in
// this file-scope array instead, kNoAllocScratchBytes long. Every GPU that loads the library
// holds the array until the process exits. All calls on a device share it and it keeps the last
// call's contents: the backward zero-fills the accumulator itself on every call, and calls whose
// kernels overlap on the GPU (different streams, no ordering) race on it.
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
                              " (N*H*Sq*(D+1)*4 bytes plus alignment); use cflk_volta_mma_bwd "
                              "with a workspace");
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

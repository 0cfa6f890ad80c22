// Pair-biased flash attention forward for sm_100a: VoltaMma, VoltaMmaPacked, VoltaMmaPackedTrim.
//
// out = softmax(scale * q k^T + bias[h] ; key mask) v, optionally times sigmoid(gate + gate_bias),
// with the row statistic lse = m + log2(l) in the log2 domain (-inf for an empty row). A masked
// key takes the logit -1e4 (so a row with no live key averages its keys), a key past Sk takes
// -inf. Semantics follow colabfold-legacy-kernels cuda/volta_mma_attn.cu:117-465 and
// cuda/volta_attn.h:9-53; the design is this file's own:
//
//   * one CTA owns 128 query rows of one (n, h) and loops over 128-key tiles;
//   * TMA brings Q once and K, V and the bias tile per key tile, two stages deep;
//   * S = Q K^T is a tcgen05 MMA (M=128, N=128) into tensor memory; thread t of the CTA owns
//     query row t = TMEM lane t, reads its 128 logits with tcgen05.ld, adds bias and mask in
//     registers, keeps the running max lazily (rescale only when it grows by more than 2^8),
//     and writes P = exp2(S - m) as 16-bit pairs over S's own columns;
//   * O += P V is a tcgen05 MMA with P read straight from tensor memory;
//   * the epilogue divides by l, applies the gate and stores rows with 16-byte stores.
// Two CTAs share an SM, so one's softmax overlaps the other's MMAs and loads.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "capi_internal.h"
#include "cflk_b200.h"
#include "sm100.cuh"
#include "tmap.h"

namespace cflk {
namespace {

__device__ unsigned g_status;

constexpr int kBQ = 128;   // query rows per CTA (= TMEM lanes)
constexpr int kBK = 128;   // keys per tile
constexpr int kThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMaskedLogit = -1.0e4f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P stays below 2^8 between rescales
constexpr uint32_t kTmemCols = 256;        // S: [0, 128), O: [128, 128 + D)

struct FwdParams {
    const void* bias;
    const uint8_t* kmask;
    const void* gate;       // null: no gate
    const void* gate_bias;  // [H, D]
    const int* lims;        // null: no trim
    void* out;
    float* lse;
    long long qn, qh, qs;   // element strides of q and the gate
    long long on, oh, os;   // of out
    int N, H, Sq, Sk, D;
    float scale;
};

template <int DP>
struct Geometry {
    // K-major atoms of AE elements along the head dim: 64-byte swizzle rows of 32 elements for
    // the 96-wide head, one atom of the padded width otherwise
    static constexpr int AE = DP == 96 ? 32 : DP;
    static constexpr int NA = DP / AE;
    static constexpr int ROWB = AE * 2;
    static constexpr uint32_t LAYOUT = ROWB >= 128 ? kSwizzle128B : ROWB >= 64 ? kSwizzle64B
                                                                               : kSwizzle32B;
    static constexpr int ATOM_BYTES = 128 * ROWB;      // one atom of a 128-row tile
    static constexpr int TILE_BYTES = NA * ATOM_BYTES; // Q, K or V tile
    static constexpr int BIAS_BYTES = kBQ * kBK * 2;   // two 64-key regions, 128-byte swizzle
};

template <int DP, bool BIAS_TMA>
struct Smem {
    using G = Geometry<DP>;
    static constexpr int Q = 0;
    static constexpr int K0 = Q + G::TILE_BYTES;
    static constexpr int V0 = K0 + 2 * G::TILE_BYTES;
    static constexpr int B0 = V0 + 2 * G::TILE_BYTES;
    static constexpr int END = B0 + (BIAS_TMA ? 2 * G::BIAS_BYTES : 0);
    static constexpr int BYTES = END + 1024;  // slack for the 1024-byte alignment
};

// 8 consecutive 16-bit values of the bias tile row r, keys [8i, 8i+8): region i/8, chunk i%8
__device__ __forceinline__ uint4 bias_chunk(const uint8_t* stage, int r, int i) {
    const uint8_t* region = stage + (i >> 3) * (kBQ * 128);
    const int phys = (i & 7) ^ (r & 7);
    return *reinterpret_cast<const uint4*>(region + r * 128 + (phys << 4));
}

template <typename T, int DP, bool BIAS_TMA, bool WANT_LSE>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tb,
                    const FwdParams p) {
    using G = Geometry<DP>;
    using L = Smem<DP, BIAS_TMA>;
    using E = Elem<T>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t bar_q, bar_full[2], bar_s, bar_o;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * kBQ, h = blockIdx.y, n = blockIdx.z;
    const int row = q0 + tid;
    const int D = p.D;

    // trim: a row with no live key, or a query tile past every row's live keys, is zeros
    int k_end = p.Sk;
    bool zero_tile = false;
    if (p.lims != nullptr) {
        k_end = p.lims[n];
        zero_tile = k_end <= 0 || q0 >= p.lims[p.N];
    }
    const int ntiles = zero_tile ? 0 : (k_end + kBK - 1) / kBK;
    T* out_row = reinterpret_cast<T*>(p.out) + n * p.on + h * p.oh + (long long)row * p.os;
    if (ntiles == 0) {
        if (row < p.Sq) {
            for (int c = 0; c < D; c += 8) {
                *reinterpret_cast<uint4*>(out_row + c) = make_uint4(0, 0, 0, 0);
            }
            if constexpr (WANT_LSE) {
                p.lse[((long long)n * p.H + h) * p.Sq + row] = -INFINITY;
            }
        }
        return;
    }

    if (tid == 0) {
        mbar_init(&bar_q, 1);
        mbar_init(&bar_full[0], 1);
        mbar_init(&bar_full[1], 1);
        mbar_init(&bar_s, 1);
        mbar_init(&bar_o, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_base_sh, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t t_s = tmem, t_o = tmem + 128;
    const uint32_t lane_base = tmem_lane_base(warp);

    constexpr uint32_t STAGE_TX = 2 * G::TILE_BYTES + (BIAS_TMA ? G::BIAS_BYTES : 0);
    const auto load_tile = [&](int j) {
        const int s = j & 1, k0 = j * kBK;
        mbar_arrive_expect_tx(&bar_full[s], STAGE_TX);
        for (int a = 0; a < G::NA; ++a) {
            tma_load_4d(smem + L::K0 + s * G::TILE_BYTES + a * G::ATOM_BYTES, &tk, &bar_full[s],
                        a * G::AE, h, k0, n);
            tma_load_4d(smem + L::V0 + s * G::TILE_BYTES + a * G::ATOM_BYTES, &tv, &bar_full[s],
                        a * G::AE, h, k0, n);
        }
        if constexpr (BIAS_TMA) {
            uint8_t* b = smem + L::B0 + s * G::BIAS_BYTES;
            tma_load_3d(b, &tb, &bar_full[s], k0, q0, h);
            tma_load_3d(b + kBQ * 128, &tb, &bar_full[s], k0 + 64, q0, h);
        }
    };

    if (tid == 0) {
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tk);
        tma_prefetch_desc(&tv);
        mbar_arrive_expect_tx(&bar_q, G::TILE_BYTES);
        for (int a = 0; a < G::NA; ++a) {
            tma_load_4d(smem + L::Q + a * G::ATOM_BYTES, &tq, &bar_q, a * G::AE, h, q0, n);
        }
        load_tile(0);
    }

    const float qk_scale = p.scale * kLog2e;
    const T* bias_row = reinterpret_cast<const T*>(p.bias) +
                        ((long long)h * p.Sq + (row < p.Sq ? row : 0)) * p.Sk;
    const uint8_t* km = p.kmask + (long long)n * p.Sk;
    const uint32_t idesc_s = idesc_f16(E::kBf16, 128, 128, false, false);
    const int DN = (D + 15) & ~15;  // the PV MMA's N: D rounded up to 16
    const uint32_t idesc_o = idesc_f16(E::kBf16, 128, DN, false, true);

    float m_run = -INFINITY, l_run = 0.f;

    for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1, k0 = j * kBK;
        if (tid == 0) {
            if (j > 0) {
                // PV(j-1) done: S's columns and the other stage are free again
                mbar_wait(&bar_o, (j - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            }
            if (j + 1 < ntiles) {
                load_tile(j + 1);
            }
            if (j == 0) {
                mbar_wait(&bar_q, 0, &g_status, kStatusTmaWait, &abort_flag);
            }
            mbar_wait(&bar_full[s], (j >> 1) & 1, &g_status, kStatusTmaWait, &abort_flag);
            tc_fence_after();
            const uint32_t q_base = smem_u32(smem + L::Q);
            const uint32_t k_base = smem_u32(smem + L::K0 + s * G::TILE_BYTES);
#pragma unroll
            for (int ks = 0; ks < DP / 16; ++ks) {
                const int a = (ks * 16) / G::AE, off = ((ks * 16) % G::AE) * 2;
                const uint64_t ad =
                    smem_desc(q_base + a * G::ATOM_BYTES + off, 16, 8 * G::ROWB, G::LAYOUT);
                const uint64_t bd =
                    smem_desc(k_base + a * G::ATOM_BYTES + off, 16, 8 * G::ROWB, G::LAYOUT);
                mma_ss(t_s, ad, bd, idesc_s, ks > 0);
            }
            mma_commit(&bar_s);
        }

        // this tile's key-mask bits, the same in every lane: bit i of word w is key 32w + i live
        uint32_t live[4];
        bool all_live = true;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const int col = k0 + 32 * w + lane;
            const bool ok = col < p.Sk && km[col] != 0;
            live[w] = __ballot_sync(0xffffffffu, ok);
            all_live = all_live && live[w] == 0xffffffffu;
        }
        const int n_in = min(kBK, p.Sk - k0);  // keys of the tile inside Sk

        __syncwarp();
        mbar_wait(&bar_s, j & 1, &g_status, kStatusMmaWait, &abort_flag);
        tc_fence_after();

        // logits of this row in the log2 domain
        float sv[kBK];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(t_s + lane_base + 32 * c, r);
            tmem_wait_ld();
            uint32_t bw[16];
            if constexpr (BIAS_TMA) {
                const uint8_t* stage = smem + L::B0 + s * G::BIAS_BYTES;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 v = bias_chunk(stage, tid, 4 * c + i);
                    bw[4 * i + 0] = v.x;
                    bw[4 * i + 1] = v.y;
                    bw[4 * i + 2] = v.z;
                    bw[4 * i + 3] = v.w;
                }
            } else {
                const unsigned short* br =
                    reinterpret_cast<const unsigned short*>(bias_row) + k0 + 32 * c;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int col = k0 + 32 * c + 2 * i;
                    const uint32_t lo = (row < p.Sq && col < p.Sk) ? br[2 * i] : 0u;
                    const uint32_t hi = (row < p.Sq && col + 1 < p.Sk) ? br[2 * i + 1] : 0u;
                    bw[i] = lo | (hi << 16);
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float2 b = E::unpack(bw[i]);
                sv[32 * c + 2 * i] = fmaf(__uint_as_float(r[2 * i]), qk_scale, b.x * kLog2e);
                sv[32 * c + 2 * i + 1] =
                    fmaf(__uint_as_float(r[2 * i + 1]), qk_scale, b.y * kLog2e);
            }
        }
        if (!all_live) {
#pragma unroll
            for (int i = 0; i < kBK; ++i) {
                const bool lv = (live[i >> 5] >> (i & 31)) & 1u;
                sv[i] = lv ? sv[i] : (i < n_in ? kMaskedLogit * kLog2e : -INFINITY);
            }
        }
        float m_tile = sv[0];
#pragma unroll
        for (int i = 1; i < kBK; ++i) {
            m_tile = fmaxf(m_tile, sv[i]);
        }

        // lazy rescale, decided per warp (tcgen05.ld/st of O are warp-wide)
        const bool need = m_tile > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
            const float m_new = fmaxf(m_run, m_tile);
            const float alpha = ex2(m_run - m_new);  // 0 on the first tile
            l_run *= alpha;
            m_run = m_new;
            if (j > 0) {
                __syncwarp();
                mbar_wait(&bar_o, (j - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
                tc_fence_after();
                for (int c = 0; c < DN; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(t_o + lane_base + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                    }
                    tmem_st16(t_o + lane_base + c, r);
                }
            }
        }

        // P = exp2(S - m) as 16-bit pairs over S's first 64 columns
        float l_tile = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t pw[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float e0 = ex2(sv[32 * c + 2 * i] - m_run);
                const float e1 = ex2(sv[32 * c + 2 * i + 1] - m_run);
                l_tile += e0 + e1;
                pw[i] = E::pack(e0, e1);
            }
            tmem_st16(t_s + lane_base + 16 * c, pw);
        }
        l_run += l_tile;
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();

        if (tid == 0) {
            tc_fence_after();
            const uint32_t v_base = smem_u32(smem + L::V0 + s * G::TILE_BYTES);
#pragma unroll
            for (int ks = 0; ks < kBK / 16; ++ks) {
                const uint64_t bd =
                    smem_desc(v_base + ks * 16 * G::ROWB, G::ATOM_BYTES, 8 * G::ROWB, G::LAYOUT);
                mma_ts(t_o, t_s + ks * 8, bd, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
            }
            mma_commit(&bar_o);
        }
    }

    // epilogue: O / l, the gate, 16-byte stores
    __syncwarp();
    mbar_wait(&bar_o, (ntiles - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
    tc_fence_after();
    const float inv = 1.f / fmaxf(l_run, 1e-30f);
    const T* gate_row = p.gate == nullptr
                            ? nullptr
                            : reinterpret_cast<const T*>(p.gate) + n * p.qn + h * p.qh +
                                  (long long)(row < p.Sq ? row : 0) * p.qs;
    const T* gb = reinterpret_cast<const T*>(p.gate_bias) + (long long)h * D;
    for (int c = 0; c < DN; c += 16) {
        uint32_t r[16];
        tmem_ld16(t_o + lane_base + c, r);
        tmem_wait_ld();
        if (row < p.Sq) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int c8 = c + 8 * half;
                if (c8 < D) {
                    float o[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        o[i] = __uint_as_float(r[8 * half + i]) * inv;
                    }
                    if (gate_row != nullptr) {
                        const uint4 gv = *reinterpret_cast<const uint4*>(gate_row + c8);
                        const uint4 bv = *reinterpret_cast<const uint4*>(gb + c8);
                        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
                        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 g = E::unpack(gw[i]), b = E::unpack(bw[i]);
                            o[2 * i] = __fdividef(o[2 * i], 1.f + ex2(-kLog2e * (g.x + b.x)));
                            o[2 * i + 1] =
                                __fdividef(o[2 * i + 1], 1.f + ex2(-kLog2e * (g.y + b.y)));
                        }
                    }
                    uint4 w;
                    w.x = E::pack(o[0], o[1]);
                    w.y = E::pack(o[2], o[3]);
                    w.z = E::pack(o[4], o[5]);
                    w.w = E::pack(o[6], o[7]);
                    *reinterpret_cast<uint4*>(out_row + c8) = w;
                }
            }
        }
    }
    if constexpr (WANT_LSE) {
        if (row < p.Sq) {
            p.lse[((long long)n * p.H + h) * p.Sq + row] =
                l_run > 0.f ? m_run + __log2f(l_run) : -INFINITY;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
struct Layout4 {
    long long qn, qh, qs, kn, kh, ks, on, oh, os;
};

// the (D, block_q, block_k) tuples the reference dispatches (cuda/volta_mma_attn.cu:508-517);
// on B200 they are accepted as hints and the tile is this kernel's own
bool reference_tile_ok(int D, long long bq, long long bk) {
    static const int tuples[][3] = {
        {8, 64, 64},   {8, 64, 32},   {8, 32, 32},  {8, 128, 64},  {8, 32, 64},  {32, 64, 64},
        {32, 64, 32},  {32, 32, 64},  {32, 32, 32}, {32, 128, 64}, {32, 16, 64}, {16, 64, 64},
        {16, 32, 32},  {16, 64, 32},  {64, 64, 64}, {64, 32, 32},  {24, 64, 32}, {24, 32, 32},
        {48, 64, 32},  {48, 32, 32},  {96, 64, 32}, {96, 32, 32}};
    for (const auto& t : tuples) {
        if (t[0] == D && t[1] == bq && t[2] == bk) {
            return true;
        }
    }
    return false;
}

int padded_dim(int D) {
    return D <= 16 ? 16 : D <= 32 ? 32 : D <= 64 ? 64 : 96;
}

template <typename T, int DP, bool BT, bool LSE>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& tq, const CUtensorMap& tk,
                         const CUtensorMap& tv, const CUtensorMap& tb, const FwdParams& p) {
    auto kern = attn_fwd_kernel<T, DP, BT, LSE>;
    const int smem = Smem<DP, BT>::BYTES;
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
    const dim3 grid((p.Sq + kBQ - 1) / kBQ, p.H, p.N);
    kern<<<grid, kThreads, smem, stream>>>(tq, tk, tv, tb, p);
    return cudaGetLastError();
}

template <typename T, int DP>
cudaError_t launch_dp(cudaStream_t stream, const CUtensorMap& tq, const CUtensorMap& tk,
                      const CUtensorMap& tv, const CUtensorMap& tb, const FwdParams& p,
                      bool bias_tma, bool want_lse) {
    if (bias_tma) {
        return want_lse ? launch_typed<T, DP, true, true>(stream, tq, tk, tv, tb, p)
                        : launch_typed<T, DP, true, false>(stream, tq, tk, tv, tb, p);
    }
    return want_lse ? launch_typed<T, DP, false, true>(stream, tq, tk, tv, tb, p)
                    : launch_typed<T, DP, false, false>(stream, tq, tk, tv, tb, p);
}

bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// Shared by the contiguous and packed entry points. q, k, v, gate: element pointers with the
// strides of lay; N batch rows, H heads, S_q / S_k sequence lengths, D head dim.
int attn_forward(cudaStream_t stream, int dtype, const void* q, const void* k, const void* v,
                 const void* gate, const void* gate_bias, const int* lims, const void* bias,
                 const uint8_t* kmask, void* out, float* lse, const Layout4& lay, int N, int H,
                 int Sq, int Sk, int D, float scale, bool want_lse, const char* who) {
    if (dtype != kF16 && dtype != kBF16) {
        return fail(kInvalidArgument, std::string(who) + ": dtype must be f16 or bf16");
    }
    if (D < 8 || D > 96 || D % 8 != 0) {
        return fail(kInvalidArgument, std::string(who) + ": unsupported head dim");
    }
    if (N == 0 || H == 0 || Sq == 0) {
        return kOk;
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
        (gate != nullptr && (!aligned16(gate) || !aligned16(gate_bias)))) {
        return fail(kInvalidArgument, std::string(who) + ": buffers must be 16-byte aligned");
    }
    const CUtensorMapDataType tdt =
        dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int DP = padded_dim(D);
    const int AE = DP == 96 ? 32 : DP;
    CUtensorMap tq, tk, tv, tb;
    {
        const uint64_t dq[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)Sq, (uint64_t)N};
        const uint64_t sq[3] = {(uint64_t)lay.qh, (uint64_t)lay.qs, (uint64_t)lay.qn};
        const uint64_t dk[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)(Sk > 0 ? Sk : 1),
                                (uint64_t)N};
        const uint64_t sk[3] = {(uint64_t)lay.kh, (uint64_t)lay.ks, (uint64_t)lay.kn};
        const uint32_t box[4] = {(uint32_t)AE, 1, 128, 1};
        const CUtensorMapSwizzle sw = swizzle_for_row(AE * 2);
        if (!encode_tiled(&tq, tdt, 2, 4, q, dq, sq, box, sw) ||
            !encode_tiled(&tk, tdt, 2, 4, k, dk, sk, box, sw) ||
            !encode_tiled(&tv, tdt, 2, 4, v, dk, sk, box, sw)) {
            return fail(kInvalidArgument, std::string(who) + ": TMA descriptor rejected");
        }
    }
    const bool bias_tma = Sk % 8 == 0 && aligned16(bias);
    tb = tq;  // unused unless bias_tma
    if (bias_tma) {
        const uint64_t db[3] = {(uint64_t)Sk, (uint64_t)Sq, (uint64_t)H};
        const uint64_t sb[2] = {(uint64_t)Sk, (uint64_t)Sq * (uint64_t)Sk};
        const uint32_t box[3] = {64, 128, 1};
        if (!encode_tiled(&tb, tdt, 2, 3, bias, db, sb, box, CU_TENSOR_MAP_SWIZZLE_128B)) {
            return fail(kInvalidArgument, std::string(who) + ": TMA descriptor rejected (bias)");
        }
    }
    FwdParams p;
    p.bias = bias;
    p.kmask = kmask;
    p.gate = gate;
    p.gate_bias = gate_bias;
    p.lims = lims;
    p.out = out;
    p.lse = lse;
    p.qn = lay.qn;
    p.qh = lay.qh;
    p.qs = lay.qs;
    p.on = lay.on;
    p.oh = lay.oh;
    p.os = lay.os;
    p.N = N;
    p.H = H;
    p.Sq = Sq;
    p.Sk = Sk;
    p.D = D;
    p.scale = scale;
    cudaError_t err;
    const bool lse_on = want_lse && lse != nullptr;
#define CFLK_DP(T)                                                                          \
    (DP == 16   ? launch_dp<T, 16>(stream, tq, tk, tv, tb, p, bias_tma, lse_on)           \
     : DP == 32 ? launch_dp<T, 32>(stream, tq, tk, tv, tb, p, bias_tma, lse_on)           \
     : DP == 64 ? launch_dp<T, 64>(stream, tq, tk, tv, tb, p, bias_tma, lse_on)           \
                : launch_dp<T, 96>(stream, tq, tk, tv, tb, p, bias_tma, lse_on))
    err = dtype == kBF16 ? CFLK_DP(__nv_bfloat16) : CFLK_DP(__half);
#undef CFLK_DP
    if (err != cudaSuccess) {
        return fail(kInternal, std::string(who) + " launch: " + cudaGetErrorString(err));
    }
    return kOk;
}

}  // namespace

unsigned read_and_clear_status_fwd() {
    unsigned v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
    cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    return v;
}

}  // namespace cflk

using namespace cflk;

extern "C" int cflk_volta_mma(void* stream, int dtype, const void* q, const void* k,
                              const void* v, const void* bias, const uint8_t* kmask, void* out,
                              float* lse, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                              float scale, int64_t block_q, int64_t block_k, int want_lse) {
    clear_error();
    if (N < 0 || H < 0 || Sq < 0 || Sk < 0 || D < 0) {
        return fail(kInvalidArgument, "q must be [N,H,S,D]");
    }
    if (!reference_tile_ok((int)D, block_q, block_k)) {
        return fail(kInvalidArgument, "volta_mma: unsupported (D, bq, bk)");
    }
    const Layout4 lay{H * Sq * D, Sq * D, D, H * Sk * D, Sk * D, D, H * Sq * D, Sq * D, D};
    return attn_forward(static_cast<cudaStream_t>(stream), dtype, q, k, v, nullptr, nullptr,
                        nullptr, bias, kmask, out, want_lse ? lse : nullptr, lay, (int)N, (int)H,
                        (int)Sq, (int)Sk, (int)D, scale, want_lse != 0, "volta_mma");
}

extern "C" int cflk_volta_mma_packed(void* stream, int dtype, const void* p, const void* bias,
                                     const uint8_t* kmask, const void* gate_bias,
                                     const int32_t* lims, void* out, int64_t X, int64_t Y,
                                     int64_t G, int64_t H, int64_t D, int64_t bias_elems,
                                     int64_t kmask_elems, int64_t gate_bias_elems, float scale,
                                     int64_t block_q, int64_t block_k, int column) {
    clear_error();
    if (X < 0 || Y < 0 || H < 0 || D < 0 || (G != 3 && G != 4)) {
        return fail(kInvalidArgument, "p must be [X,Y,3 or 4,H,D]");
    }
    const int64_t N = column ? Y : X, S = column ? X : Y;
    if (bias_elems != H * S * S || kmask_elems != N * S || (G == 4 && gate_bias_elems != H * D)) {
        return fail(kInvalidArgument, "bias must be [H,S,S], kmask [N,S], gate_bias [H,D]");
    }
    if (!reference_tile_ok((int)D, block_q, block_k)) {
        return fail(kInvalidArgument, "volta_mma: unsupported (D, bq, bk)");
    }
    // rows attend along Y (batch X); a column attends along X (batch Y)
    const long long pn = G * H * D, pr = Y * pn, on = H * D, orow = Y * on;
    const Layout4 lay = column ? Layout4{pn, D, pr, pn, D, pr, on, D, orow}
                               : Layout4{pr, D, pn, pr, D, pn, orow, D, on};
    const int esz = 2;
    const uint8_t* base = static_cast<const uint8_t*>(p);
    const void* gate = G == 4 ? base + 3 * H * D * esz : nullptr;
    return attn_forward(static_cast<cudaStream_t>(stream), dtype, base, base + H * D * esz,
                        base + 2 * H * D * esz, gate, G == 4 ? gate_bias : nullptr, lims, bias,
                        kmask, out, nullptr, lay, (int)N, (int)H, (int)S, (int)S, (int)D, scale,
                        false, lims ? "volta_mma_packed_trim" : "volta_mma_packed");
}

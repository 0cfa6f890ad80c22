// Pair-biased flash attention forward for sm_100a: VoltaMma, VoltaMmaPacked, VoltaMmaPackedTrim.
//
// out = softmax(scale * q k^T + bias[h] ; key mask) v, optionally times sigmoid(gate + gate_bias),
// with the row statistic lse = m + log2(l) in the log2 domain (-inf for an empty row). A masked
// key takes the logit -1e4 (so a row with no live key averages its keys), a key past Sk takes
// -inf. Semantics follow colabfold-legacy-kernels cuda/volta_mma_attn.cu:117-465 and
// cuda/volta_attn.h:9-53; the design is this file's own:
//
//   * persistent CTAs, one per SM, loop over work items: the same 128 query rows of two
//     consecutive sequences (n, n+1) of one head, which share the bias tile; an item loops
//     over 128-key tiles;
//   * warp roles: a TMA warp brings an item's Q tiles (two buffers, so the next item's load
//     early) and, in a ring of two or three stages that runs on across items, both sequences'
//     K and V tiles plus the one bias tile and the tile's key-mask words; one MMA warp per sequence (each issuing thread has
//     its own MMA pipeline, so the two overlap); one softmax warpgroup per sequence, so one
//     sequence's exponentials overlap the other's MMAs; the MMA/TMA warpgroup hands most of
//     its registers to the softmax warpgroups (setmaxnreg);
//   * S = Q K^T is a tcgen05 MMA (M=128, N=128) into tensor memory; thread t of a softmax
//     warpgroup owns query row t = TMEM lane t, reads its 128 logits with tcgen05.ld, adds bias
//     and mask in registers, keeps the running max lazily (rescale only when it grows by more
//     than 2^8), and writes P = exp2(S - m) as 16-bit pairs over S's own columns;
//   * O += P V is a tcgen05 MMA with P read straight from tensor memory, into one of two O
//     buffers per sequence, so an item's epilogue overlaps the next item's MMAs;
//   * the epilogue divides by l, applies the gate and stores rows with 16-byte stores.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
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
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kMaskedLogit = -1.0e4f;
// log2 units: O and l are rescaled only when a tile raises the row max by more than this, so P
// stays below 2^8 between rescales
constexpr float kRescaleThreshold = 8.0f;
// one exponential pair in kFmaExpEvery is computed on the FMA pipe, the rest on the MUFU
constexpr int kFmaExpEvery = 4;

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
    // sequences per CTA: the same 128 query rows of NSEQ consecutive sequences, which share the
    // bias tile; one softmax warpgroup and one MMA warp each
    static constexpr int NSEQ = DP == 96 ? 1 : 2;
    static constexpr int MMA_WARP0 = 4 * NSEQ;
    static constexpr int TMA_WARP = MMA_WARP0 + NSEQ;
    // with two sequences the MMA and TMA warps form a third warpgroup (one warp idle) that
    // hands registers to the softmax warpgroups: 384 threads x 168 = 2 x 128 x 224 + 128 x 56
    static constexpr int THREADS = NSEQ == 2 ? 384 : 32 * (TMA_WARP + 1);
    static constexpr uint32_t SOFTMAX_REGS = 224, OTHER_REGS = 56;
    static_assert(NSEQ == 1 || THREADS * 168 >= 2 * 128 * SOFTMAX_REGS + 128 * OTHER_REGS,
                  "register split");
    // Q buffers in shared memory (two where they fit, so the next item's Q loads early) and
    // stages of the key-tile ring (three where they fit: a stage's loads take about as long as
    // a tile's softmax)
    static constexpr int QB = DP == 64 ? 1 : 2;
    static constexpr int NST = DP <= 32 ? 3 : 2;
    // TMEM per sequence w: S (128 columns) at 192 w, P (128 keys as 16-bit pairs) at
    // 192 w + 128, so the next S can be computed while P is still being read; O at
    // 192 NSEQ + DP w
    static constexpr int T_O = 192 * NSEQ;
    static constexpr int COLS = T_O + NSEQ * DP;
    static constexpr uint32_t ALLOC = COLS <= 256 ? 256 : 512;
};

template <int DP, bool BIAS_TMA>
struct Smem {
    using G = Geometry<DP>;
    static constexpr int Q = 0;                                       // QB x NSEQ Q tiles
    static constexpr int STAGE = Q + G::QB * G::NSEQ * G::TILE_BYTES;  // 2 x (NSEQ x (K, V), bias)
    static constexpr int KV_BYTES = G::NSEQ * 2 * G::TILE_BYTES;
    static constexpr int STAGE_BYTES = KV_BYTES + (BIAS_TMA ? G::BIAS_BYTES : 0);
    static constexpr int END = STAGE + G::NST * STAGE_BYTES;
    static constexpr int BYTES = END + 1024;  // slack for the 1024-byte alignment
    static_assert(BYTES + 256 <= 227 * 1024, "shared memory");
};

// 8 consecutive 16-bit values of the bias tile row r, keys [8i, 8i+8): region i/8, chunk i%8
__device__ __forceinline__ uint4 bias_chunk(const uint8_t* stage, int r, int i) {
    const uint8_t* region = stage + (i >> 3) * (kBQ * 128);
    const int phys = (i & 7) ^ (r & 7);
    return *reinterpret_cast<const uint4*>(region + r * 128 + (phys << 4));
}

// A work item: the 128 query rows [q0, q0 + 128) of head h of the sequences n0 .. n0+NSEQ-1.
// Items run query tiles fastest (they share K and V in L2), then heads, then sequence groups; a
// persistent CTA takes items blockIdx.x, blockIdx.x + gridDim.x, ...
struct FwdItem {
    int q0, h, n0, nt_max;
    int ntiles[2];  // key tiles per sequence; 0: no output (past N) or zeros (trim)
    // sequence w's key tiles, chosen without indexing by a run-time w (which would put the
    // item in local memory)
    __device__ __forceinline__ int nt(int w) const { return w == 0 ? ntiles[0] : ntiles[1]; }
};

template <int NSEQ>
__device__ __forceinline__ FwdItem fwd_item(const FwdParams& p, int nqt, int u) {
    FwdItem it;
    const int rest = u / nqt;
    it.q0 = (u - rest * nqt) * kBQ;
    it.h = rest % p.H;
    it.n0 = (rest / p.H) * NSEQ;
    it.nt_max = 0;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        // trim: a sequence with no live key, or a query tile past every row's live keys, gives
        // zeros
        int k_end = p.Sk;
        bool zero = w >= NSEQ || it.n0 + w >= p.N;
        if (!zero && p.lims != nullptr) {
            k_end = p.lims[it.n0 + w];
            zero = k_end <= 0 || it.q0 >= p.lims[p.N];
        }
        it.ntiles[w] = zero ? 0 : (k_end + kBK - 1) / kBK;
        it.nt_max = max(it.nt_max, it.ntiles[w]);
    }
    return it;
}

// How many arrivals sequence w owes a barrier that expects one per sequence, when only the
// sequences with ntiles > j take part: the lowest one taking part also arrives for the others.
template <int NSEQ>
__device__ __forceinline__ int arrivals_for(const FwdItem& it, int w, int j) {
    int na = 0, first = -1;
#pragma unroll
    for (int v = 0; v < NSEQ; ++v) {
        if (j < it.ntiles[v]) {
            na += 1;
            first = first < 0 ? v : first;
        }
    }
    return w == first ? NSEQ - na + 1 : 1;
}

struct FwdBars {
    uint64_t q_full[2], q_empty[2], kv_full[3], kv_empty[3], s_full[2], s_free[2], p_ready[2],
        o_done[2];
    // key-mask words of each stage's tile: bit i of word c of sequence w is key 32c + i live
    uint32_t live[3][2][4];
};

// The key tiles of one sequence slot over a CTA's items, in order: item u (blockIdx.x,
// blockIdx.x + gridDim.x, ...), tile j of it; gbase counts the key tiles (stages) of the items
// before, qi their Q loads (items with no tile at all load nothing)
template <int NSEQ>
struct SlotTiles {
    int u, j, gbase, qi;
    FwdItem it;
    __device__ __forceinline__ void next_item(const FwdParams& p, int nqt, int nitems) {
        if (it.nt_max > 0) {
            gbase += it.nt_max;
            ++qi;
        }
        u += gridDim.x;
        if (u < nitems) {
            it = fwd_item<NSEQ>(p, nqt, u);
        }
        j = 0;
    }
    __device__ __forceinline__ void start(const FwdParams& p, int nqt, int nitems, int w) {
        u = blockIdx.x;
        j = 0;
        gbase = 0;
        qi = 0;
        it.nt_max = 0;
        if (u < nitems) {
            it = fwd_item<NSEQ>(p, nqt, u);
        }
        while (u < nitems && j >= it.nt(w)) {
            next_item(p, nqt, nitems);
        }
    }
    __device__ __forceinline__ void advance(const FwdParams& p, int nqt, int nitems, int w) {
        ++j;
        while (u < nitems && j >= it.nt(w)) {
            next_item(p, nqt, nitems);
        }
    }
    __device__ __forceinline__ bool valid(int nitems) const { return u < nitems; }
};

// TMA warp: per item, the Q tiles of its sequences (QB buffers); per key tile, every running
// sequence's K and V tiles and the shared bias tile, in a ring of NST stages that runs on across
// items, plus the tile's key-mask words (the whole warp reads the mask bytes; lane 0 issues
// the copies and publishes the words with the stage's barrier)
template <typename G, typename L, bool BIAS_TMA>
__device__ __forceinline__ void fwd_producer(const FwdParams& p, const CUtensorMap* tq,
                                             const CUtensorMap* tk, const CUtensorMap* tv,
                                             const CUtensorMap* tb, uint8_t* smem, FwdBars& bar,
                                             int nqt, int nitems, int* abort_flag) {
    constexpr int NSEQ = G::NSEQ, QB = G::QB;
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
        tma_prefetch_desc(tq);
        tma_prefetch_desc(tk);
        tma_prefetch_desc(tv);
    }
    int g = 0, qi = 0;  // key tiles and Q loads so far
    for (int u = blockIdx.x; u < nitems; u += gridDim.x) {
        const FwdItem it = fwd_item<NSEQ>(p, nqt, u);
        if (it.nt_max == 0) {
            continue;
        }
        const int qb = qi % QB;
        if (qi >= QB) {
            mbar_wait(&bar.q_empty[qb], ((qi - QB) / QB) & 1, &g_status, kStatusMmaWait,
                      abort_flag);
        }
        int nq = 0;
        for (int w = 0; w < NSEQ; ++w) {
            nq += it.ntiles[w] > 0;
        }
        if (lane == 0) {
            mbar_arrive_expect_tx(&bar.q_full[qb], nq * G::TILE_BYTES);
        }
        for (int w = 0; w < NSEQ && lane == 0; ++w) {
            if (it.ntiles[w] > 0) {
                for (int a = 0; a < G::NA; ++a) {
                    tma_load_4d(smem + L::Q + (qb * NSEQ + w) * G::TILE_BYTES + a * G::ATOM_BYTES,
                                tq, &bar.q_full[qb], a * G::AE, it.h, it.q0, it.n0 + w);
                }
            }
        }
        ++qi;
        for (int j = 0; j < it.nt_max; ++j, ++g) {
            const int st = g % G::NST, k0 = j * kBK;
            if (g >= G::NST) {
                mbar_wait(&bar.kv_empty[st], ((g - G::NST) / G::NST) & 1, &g_status, kStatusMmaWait,
                          abort_flag);
            }
            int na = 0;
            for (int w = 0; w < NSEQ; ++w) {
                na += j < it.ntiles[w];
                if (j < it.ntiles[w]) {
                    const uint8_t* kmr = p.kmask + (long long)(it.n0 + w) * p.Sk;
                    uint32_t words[4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const int col = k0 + 32 * c + lane;
                        words[c] = __ballot_sync(0xffffffffu, col < p.Sk && kmr[col] != 0);
                    }
                    if (lane == 0) {
                        *reinterpret_cast<uint4*>(bar.live[st][w]) =
                            make_uint4(words[0], words[1], words[2], words[3]);
                    }
                }
            }
            if (lane != 0) {
                continue;
            }
            uint8_t* stage = smem + L::STAGE + st * L::STAGE_BYTES;
            mbar_arrive_expect_tx(&bar.kv_full[st],
                                  na * 2 * G::TILE_BYTES + (BIAS_TMA ? G::BIAS_BYTES : 0));
            for (int w = 0; w < NSEQ; ++w) {
                if (j < it.ntiles[w]) {
                    uint8_t* kv = stage + w * 2 * G::TILE_BYTES;
                    for (int a = 0; a < G::NA; ++a) {
                        tma_load_4d(kv + a * G::ATOM_BYTES, tk, &bar.kv_full[st], a * G::AE,
                                    it.h, k0, it.n0 + w);
                        tma_load_4d(kv + G::TILE_BYTES + a * G::ATOM_BYTES, tv, &bar.kv_full[st],
                                    a * G::AE, it.h, k0, it.n0 + w);
                    }
                }
            }
            if constexpr (BIAS_TMA) {
                uint8_t* b = stage + L::KV_BYTES;
                tma_load_3d(b, tb, &bar.kv_full[st], k0, it.q0, it.h);
                tma_load_3d(b + kBQ * 128, tb, &bar.kv_full[st], k0 + 64, it.q0, it.h);
            }
        }
    }
}

// MMA warp of sequence slot w. S = Q K^T of the next tile goes out as soon as the softmax
// warpgroup has read the current S out of tensor memory, ahead of the current O += P V, which
// waits for P in its own columns (read from tensor memory).
template <typename G, typename L>
__device__ __forceinline__ void fwd_mma(const FwdParams& p, uint8_t* smem, uint32_t tmem, int w,
                                        bool bf16, FwdBars& bar, int nqt, int nitems,
                                        int* abort_flag) {
    constexpr int NSEQ = G::NSEQ, QB = G::QB, DP = G::AE * G::NA;
    const uint32_t idesc_s = idesc_f16(bf16, 128, 128, false, false);
    const int DN = (p.D + 15) & ~15;  // the PV MMA's N: D rounded up to 16
    const uint32_t idesc_o = idesc_f16(bf16, 128, DN, false, true);
    const uint32_t t_s = tmem + 192 * w, t_p = t_s + 128, t_o = tmem + G::T_O + DP * w;
    const auto issue_s = [&](const SlotTiles<NSEQ>& c, int k) {
        const int g = c.gbase + c.j, st = g % G::NST, qb = c.qi % QB;
        if (c.j == 0) {
            mbar_wait(&bar.q_full[qb], (c.qi / QB) & 1, &g_status, kStatusTmaWait, abort_flag);
        }
        mbar_wait(&bar.kv_full[st], (g / G::NST) & 1, &g_status, kStatusTmaWait, abort_flag);
        if (k > 0) {
            // the softmax warpgroup has read the previous S
            mbar_wait(&bar.s_free[w], (k - 1) & 1, &g_status, kStatusSyncWait, abort_flag);
        }
        tc_fence_after();
        const uint32_t q_base = smem_u32(smem + L::Q + (qb * NSEQ + w) * G::TILE_BYTES);
        const uint32_t k_base =
            smem_u32(smem + L::STAGE + st * L::STAGE_BYTES + w * 2 * G::TILE_BYTES);
#pragma unroll
        for (int ks = 0; ks < DP / 16; ++ks) {
            const int a = (ks * 16) / G::AE, off = ((ks * 16) % G::AE) * 2;
            const uint64_t ad =
                smem_desc(q_base + a * G::ATOM_BYTES + off, 16, 8 * G::ROWB, G::LAYOUT);
            const uint64_t bd =
                smem_desc(k_base + a * G::ATOM_BYTES + off, 16, 8 * G::ROWB, G::LAYOUT);
            mma_ss(t_s, ad, bd, idesc_s, ks > 0);
        }
        mma_commit(&bar.s_full[w]);
        if (c.j == c.it.nt(w) - 1) {
            // the item's Q tiles are free once every sequence's last S is done
            for (int r = arrivals_for<NSEQ>(c.it, w, 0); r > 0; --r) {
                mma_commit(&bar.q_empty[qb]);
            }
        }
    };
    const auto issue_pv = [&](const SlotTiles<NSEQ>& c, int k) {
        const int g = c.gbase + c.j, st = g % G::NST;
        mbar_wait(&bar.p_ready[w], k & 1, &g_status, kStatusSyncWait, abort_flag);
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + L::STAGE + st * L::STAGE_BYTES +
                                         w * 2 * G::TILE_BYTES + G::TILE_BYTES);
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
            const uint64_t bd =
                smem_desc(v_base + ks * 16 * G::ROWB, G::ATOM_BYTES, 8 * G::ROWB, G::LAYOUT);
            mma_ts(t_o, t_p + ks * 8, bd, idesc_o, (c.j > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit(&bar.o_done[w]);
        // the stage is free once every sequence reading it is done
        for (int r = arrivals_for<NSEQ>(c.it, w, c.j); r > 0; --r) {
            mma_commit(&bar.kv_empty[st]);
        }
    };
    SlotTiles<NSEQ> cs, cp;  // the next S to issue, the next PV to issue
    cs.start(p, nqt, nitems, w);
    cp = cs;
    int ks = 0, kp = 0;
    if (cs.valid(nitems)) {
        issue_s(cs, ks++);
        cs.advance(p, nqt, nitems, w);
    }
    while (cp.valid(nitems)) {
        if (cs.valid(nitems)) {
            issue_s(cs, ks++);
            cs.advance(p, nqt, nitems, w);
        }
        issue_pv(cp, kp++);
        cp.advance(p, nqt, nitems, w);
    }
}

template <typename T, int DP, bool BIAS_TMA, bool WANT_LSE>
__global__ void __launch_bounds__(Geometry<DP>::THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tb,
                    const FwdParams p) {
    using G = Geometry<DP>;
    using L = Smem<DP, BIAS_TMA>;
    using E = Elem<T>;
    constexpr int NSEQ = G::NSEQ;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ FwdBars bar;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = p.D;
    const int nqt = (p.Sq + kBQ - 1) / kBQ;
    const int nitems = nqt * p.H * ((p.N + NSEQ - 1) / NSEQ);

    if (warp == G::MMA_WARP0) {
        if (lane == 0) {
            for (int i = 0; i < G::NST; ++i) {
                mbar_init(&bar.kv_full[i], 1);
                mbar_init(&bar.kv_empty[i], NSEQ);
            }
            for (int i = 0; i < 2; ++i) {
                mbar_init(&bar.q_full[i], 1);
                mbar_init(&bar.q_empty[i], NSEQ);
                mbar_init(&bar.s_full[i], 1);
                mbar_init(&bar.s_free[i], 128);
                mbar_init(&bar.p_ready[i], 128);
                mbar_init(&bar.o_done[i], 1);
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

    if (warp >= G::MMA_WARP0) {
        // the MMA and TMA warps (with two sequences, one whole warpgroup)
        if constexpr (NSEQ == 2) {
            regs_decrease<G::OTHER_REGS>();
        }
        if (warp == G::TMA_WARP) {
            fwd_producer<G, L, BIAS_TMA>(p, &tq, &tk, &tv, &tb, smem, bar, nqt, nitems,
                                         &abort_flag);
        } else if (warp < G::TMA_WARP) {
            if (lane == 0) {
                fwd_mma<G, L>(p, smem, tmem, warp - G::MMA_WARP0, E::kBf16, bar, nqt, nitems,
                              &abort_flag);
            }
        }
    } else {
        if constexpr (NSEQ == 2) {
            regs_increase<G::SOFTMAX_REGS>();
        }
        // softmax warpgroup w: thread t owns query row q0 + t of sequence n0 + w = TMEM lane t
        const int w = warp >> 2, t = ((warp & 3) << 5) | lane;
        const uint32_t lane_base = tmem_lane_base(warp);
        const uint32_t t_s = tmem + 192 * w + lane_base, t_p = t_s + 128;
        const uint32_t t_o = tmem + G::T_O + DP * w + lane_base;
        const uint64_t scale2 = pk2(p.scale, p.scale), log2e2 = pk2(kLog2e, kLog2e);
        const int DN = (D + 15) & ~15;
        int g = 0, c = 0;  // key tiles, this slot's tiles
        for (int u = blockIdx.x; u < nitems; u += gridDim.x) {
            const FwdItem it = fwd_item<NSEQ>(p, nqt, u);
            const int n = it.n0 + w, row = it.q0 + t, h = it.h, nt = it.nt(w);
            const int g0 = g;
            g += it.nt_max;
            if (n >= p.N) {
                continue;  // no sequence in this slot
            }
            T* out_row = reinterpret_cast<T*>(p.out) + (long long)n * p.on + h * p.oh +
                         (long long)row * p.os;
            if (nt == 0) {
                if (row < p.Sq) {
                    for (int cc = 0; cc < D; cc += 8) {
                        *reinterpret_cast<uint4*>(out_row + cc) = make_uint4(0, 0, 0, 0);
                    }
                    if constexpr (WANT_LSE) {
                        p.lse[((long long)n * p.H + h) * p.Sq + row] = -INFINITY;
                    }
                }
                continue;
            }
            const T* bias_row = reinterpret_cast<const T*>(p.bias) +
                                ((long long)h * p.Sq + (row < p.Sq ? row : 0)) * p.Sk;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < nt; ++j, ++c) {
                const int st = (g0 + j) % G::NST, k0 = j * kBK;
                const int n_in = min(kBK, p.Sk - k0);  // keys of the tile inside Sk
                mbar_wait(&bar.s_full[w], c & 1, &g_status, kStatusMmaWait, &abort_flag);
                // the stage (bias tile, key-mask words) is complete: S was computed from it
                mbar_wait(&bar.kv_full[st], ((g0 + j) / G::NST) & 1, &g_status, kStatusTmaWait,
                          &abort_flag);
                tc_fence_after();
                // this tile's key-mask bits: bit i of word cc is key 32 cc + i live
                const uint4 lw = *reinterpret_cast<const uint4*>(bar.live[st][w]);
                const uint32_t live[4] = {lw.x, lw.y, lw.z, lw.w};
                const bool all_live = (lw.x & lw.y & lw.z & lw.w) == 0xffffffffu;

                // logits of this row, scale q.k + bias (natural units; log2e is applied with
                // the max subtracted), computed two at a time over the loaded S in place
                float sv[kBK];
                {
                    uint32_t* sr = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        tmem_ld32(t_s + 32 * cc,
                                  *reinterpret_cast<uint32_t(*)[32]>(sr + 32 * cc));
                    }
                    tmem_wait_ld();
                    // all of S is in registers: the next S may overwrite it
                    tc_fence_before();
                    mbar_arrive(&bar.s_free[w]);
                }
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t bw[16];
                    if constexpr (BIAS_TMA) {
                        const uint8_t* stage = smem + L::STAGE + st * L::STAGE_BYTES + L::KV_BYTES;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint4 v = bias_chunk(stage, t, 4 * cc + i);
                            bw[4 * i + 0] = v.x;
                            bw[4 * i + 1] = v.y;
                            bw[4 * i + 2] = v.z;
                            bw[4 * i + 3] = v.w;
                        }
                    } else {
                        const unsigned short* br =
                            reinterpret_cast<const unsigned short*>(bias_row) + k0 + 32 * cc;
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int col = k0 + 32 * cc + 2 * i;
                            const uint32_t lo = (row < p.Sq && col < p.Sk) ? br[2 * i] : 0u;
                            const uint32_t hi =
                                (row < p.Sq && col + 1 < p.Sk) ? br[2 * i + 1] : 0u;
                            bw[i] = lo | (hi << 16);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 b = E::unpack(bw[i]);
                        const float2 y = upk2(fma2(pk2(sv[32 * cc + 2 * i], sv[32 * cc + 2 * i + 1]),
                                                   scale2, pk2(b.x, b.y)));
                        sv[32 * cc + 2 * i] = y.x;
                        sv[32 * cc + 2 * i + 1] = y.y;
                    }
                }
                if (!all_live) {
#pragma unroll
                    for (int i = 0; i < kBK; ++i) {
                        const bool lv = (live[i >> 5] >> (i & 31)) & 1u;
                        sv[i] = lv ? sv[i] : (i < n_in ? kMaskedLogit : -INFINITY);
                    }
                }
                // row max in a tree of eight partial maxima (short dependency chains)
                float mp[8];
#pragma unroll
                for (int a = 0; a < 8; ++a) {
                    mp[a] = max3(sv[16 * a], sv[16 * a + 1], sv[16 * a + 2]);
#pragma unroll
                    for (int i = 3; i < 15; i += 2) {
                        mp[a] = max3(mp[a], sv[16 * a + i], sv[16 * a + i + 1]);
                    }
                    mp[a] = fmaxf(mp[a], sv[16 * a + 15]);
                }
                const float m_tile =
                    max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7])) *
                    kLog2e;  // log2 units

                if (c > 0) {
                    // the previous PV is done: P's columns are free and O is final
                    mbar_wait(&bar.o_done[w], (c - 1) & 1, &g_status, kStatusMmaWait,
                              &abort_flag);
                    tc_fence_after();
                }
                // lazy rescale, decided per warp (tcgen05.ld/st of O are warp-wide)
                const bool need = m_tile > m_run + kRescaleThreshold;
                if (__any_sync(0xffffffffu, need)) {
                    const float m_new = fmaxf(m_run, m_tile);
                    const float alpha = ex2(m_run - m_new);  // 0 on the first tile
                    l_run *= alpha;
                    m_run = m_new;
                    if (j > 0) {
                        for (int cc = 0; cc < DN; cc += 16) {
                            uint32_t r[16];
                            tmem_ld16(t_o + cc, r);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                            }
                            tmem_st16(t_o + cc, r);
                        }
                    }
                }

                // P = exp2(log2e y - m) as 16-bit pairs in P's columns
                const uint64_t neg_m2 = pk2(-m_run, -m_run);
                uint64_t l2[4];  // four partial sums (short dependency chains)
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t pw[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 a = upk2(fma2(
                            pk2(sv[32 * cc + 2 * i], sv[32 * cc + 2 * i + 1]), log2e2, neg_m2));
                        // one pair in kFmaExpEvery on the FMA pipe, the rest on the MUFU
                        float e0, e1;
                        if (i % kFmaExpEvery == kFmaExpEvery - 1) {
                            const float2 e = ex2_fma(a.x, a.y);
                            e0 = e.x;
                            e1 = e.y;
                        } else {
                            e0 = ex2(a.x);
                            e1 = ex2(a.y);
                        }
                        l2[i & 3] = cc == 0 && i < 4 ? pk2(e0, e1) : add2(l2[i & 3], pk2(e0, e1));
                        pw[i] = E::pack(e0, e1);
                    }
                    tmem_st16(t_p + 16 * cc, pw);
                }
                const float2 lt = upk2(add2(add2(l2[0], l2[1]), add2(l2[2], l2[3])));
                l_run += lt.x + lt.y;
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bar.p_ready[w]);
            }

            // epilogue: O / l, the gate, 16-byte stores; then the O buffer is free again
            mbar_wait(&bar.o_done[w], (c - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            const float inv = 1.f / fmaxf(l_run, 1e-30f);
            const T* gate_row = p.gate == nullptr
                                    ? nullptr
                                    : reinterpret_cast<const T*>(p.gate) + (long long)n * p.qn +
                                          h * p.qh + (long long)(row < p.Sq ? row : 0) * p.qs;
            const T* gb = reinterpret_cast<const T*>(p.gate_bias) + (long long)h * D;
            for (int cc = 0; cc < DN; cc += 16) {
                uint32_t r[16];
                tmem_ld16(t_o + cc, r);
                tmem_wait_ld();
                if (row < p.Sq) {
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int c8 = cc + 8 * half;
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
                                    const float2 gg = E::unpack(gw[i]), b = E::unpack(bw[i]);
                                    o[2 * i] =
                                        __fdividef(o[2 * i], 1.f + ex2(-kLog2e * (gg.x + b.x)));
                                    o[2 * i + 1] = __fdividef(o[2 * i + 1],
                                                              1.f + ex2(-kLog2e * (gg.y + b.y)));
                                }
                            }
                            uint4 wv;
                            wv.x = E::pack(o[0], o[1]);
                            wv.y = E::pack(o[2], o[3]);
                            wv.z = E::pack(o[4], o[5]);
                            wv.w = E::pack(o[6], o[7]);
                            *reinterpret_cast<uint4*>(out_row + c8) = wv;
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
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == G::MMA_WARP0) {
        tc_fence_after();
        tmem_dealloc(tmem, G::ALLOC);
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
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) {
            return e;
        }
        // the warpgroups' register hand-off must fit what the kernel is launched with, or a
        // setmaxnreg.inc would wait for registers that never come: refuse instead
        using G = Geometry<DP>;
        if constexpr (G::NSEQ == 2) {
            cudaFuncAttributes fa;
            if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) {
                return e;
            }
            if (fa.numRegs * G::THREADS < (int)(2 * 128 * G::SOFTMAX_REGS + 128 * G::OTHER_REGS)) {
                return cudaErrorInvalidConfiguration;
            }
        }
        attr_done[dev] = true;
    }
    constexpr int NSEQ = Geometry<DP>::NSEQ;
    // persistent: one CTA per SM, each looping over work items
    static int sms[kMaxDevices] = {};
    if (dev < kMaxDevices && sms[dev] == 0) {
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    const int nsm = dev < kMaxDevices && sms[dev] > 0 ? sms[dev] : 148;
    const long long items =
        (long long)((p.Sq + kBQ - 1) / kBQ) * p.H * ((p.N + NSEQ - 1) / NSEQ);
    const dim3 grid((unsigned)std::min<long long>(items, nsm));
    kern<<<grid, Geometry<DP>::THREADS, smem, stream>>>(tq, tk, tv, tb, p);
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

extern "C" int cflk_volta_mma_gated(void* stream, int dtype, const void* q, const void* k,
                                    const void* v, const void* gate, const void* gate_bias,
                                    const void* bias, const uint8_t* kmask, void* out, float* lse,
                                    int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                    float scale, int want_lse) {
    clear_error();
    if (N < 0 || H < 0 || Sq < 0 || Sk < 0 || D < 0) {
        return fail(kInvalidArgument, "q must be [N,H,S,D]");
    }
    if (gate == nullptr || gate_bias == nullptr) {
        return fail(kInvalidArgument, "volta_mma_gated: gate [N,H,Sq,D] and gate_bias [H,D]");
    }
    // the gate shares q's layout [N,H,Sq,D]
    const Layout4 lay{H * Sq * D, Sq * D, D, H * Sk * D, Sk * D, D, H * Sq * D, Sq * D, D};
    return attn_forward(static_cast<cudaStream_t>(stream), dtype, q, k, v, gate, gate_bias,
                        nullptr, bias, kmask, out, want_lse ? lse : nullptr, lay, (int)N, (int)H,
                        (int)Sq, (int)Sk, (int)D, scale, want_lse != 0, "volta_mma_gated");
}

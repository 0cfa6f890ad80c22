// Pair-biased flash attention backward for sm_100a: VoltaMmaBwd.
//
// Given q, k, v, bias, the key mask, the forward's out and log2-domain lse, and dout:
//   P   = exp2(scale*log2e * q.k + log2e * bias - lse)    (a masked key: exp2(-1e4 log2e - lse))
//   dS  = P (dP - delta), dP = dout v^T, delta = rowsum(out * dout); zero on masked keys
//   dV  = P^T dout,  dK = scale dS^T q,  dQ = scale dS k,  dBias = sum over the batch of dS
// as colabfold-legacy-kernels computes them (cuda/volta_mma_attn_bwd.cu:84-383, where P still
// carries dV through a masked key but dS does not). The design is this file's own:
//
//   * persistent CTAs, one per SM, each looping over work items (a 128-key tile of one (n, h)):
//     K and V of an item stay in shared memory (two buffers, so the next item's tiles load
//     while this one runs) and dK, dV accumulate in tensor memory over every query (two sets,
//     so one item's are stored while the next accumulates); both come out bitwise
//     deterministic;
//   * warp roles: a TMA warp streams the 64-query steps (q, dout and the bias tile) three
//     stages deep; MMA warp A issues S^T and dP^T, MMA warp B dQ, dV and dK (each issuing
//     thread has its own MMA pipeline, so the two overlap); softmax warpgroups in step sets
//     that take the steps alternately (ping-pong), each set with its own S^T/dP^T columns in
//     tensor memory and its own dS buffer, so one set's exponentials overlap the other set's
//     MMAs; the two warpgroups of a set take the two 32-query halves of its step;
//   * S^T = K Q^T and dP^T = V dout^T (M=128 keys, N=64 queries); worker t owns key t = TMEM
//     lane t, forms P^T and dS^T and writes them back over its own S^T and dP^T columns as
//     16-bit pairs, the A operands of dV += P^T dout and dK += dS^T q (A read from TMEM);
//   * dS also goes MN-major into swizzled shared memory for dQ = dS k (M=64); a CTA runs the
//     key tiles of each (n, h) it owns in order, so the first key tile stores a query step's
//     fp32 dQ tile into the workspace accumulator and the later ones add theirs with 16-byte
//     vector atomics (no zero fill of the accumulator); a conversion pass rounds it to dQ;
//   * the bias is transposed once per call into the workspace in its own 16-bit type
//     [H][Sk][Sq'] (exact), so a key's bias values arrive by TMA as one contiguous 128-byte row;
//   * dBias: each warpgroup stages its half-step's fp32 dS rows [32 queries][128 keys] in
//     shared memory and one thread hands them to TMA as a single bulk reduce-add into dBias
//     (full-line L2 reductions); an item's query steps start at a step that depends on its
//     sequence, so concurrent items reduce into different rows. Where the dBias rows are not
//     16-byte multiples (Sk % 4 != 0) the workers add dS with coalesced fp32 reductions
//     instead (a warp covers 32 consecutive keys of a row).
// Around it: the row statistic (delta), the bias transpose, the dBias zero fill, the dQ
// conversion.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
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
    const float* nlse;   // -lse, [N,H,Sq]
    const float* ndelta; // -delta
    float* dq_acc;  // [N,H,Sq,D] fp32: with contig stored by the first key tile, added to by
                    // the later ones; otherwise zeroed before the kernel, added to by all
    int contig;     // CTAs own contiguous runs of (n, h) pairs (the schedule below)
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
    static constexpr int BT = kBQ * kBK * 2;  // bias^T tile: [128 keys][64 queries], 16-bit
    static constexpr int DS = kBK * 128;      // dS, MN-major: 128 key rows of 64 queries
    static constexpr int DN = DP;
    // Step sets: consecutive 64-query steps alternate between NP sets (ping-pong). A set is two
    // softmax warpgroups, one per 32-query half of its step.
    static constexpr int NP = DN <= 32 ? 2 : 1;
    static constexpr int NWG = 2 * NP;
    static constexpr int MMA_A = 4 * NWG;    // warp issuing S^T and dP^T
    static constexpr int MMA_B = MMA_A + 1;  // warp issuing dQ, dV and dK
    static constexpr int TMA_WARP = MMA_A + 2;
    static constexpr int THREADS = NWG * 128 + 96;
    // K/V buffers in shared memory and dK/dV accumulator sets in tensor memory: two of each, so
    // that a CTA loads its next key tile and starts its MMAs while it stores the previous one
    static constexpr int KVB = DP == 96 ? 1 : 2;
    static constexpr int NB = DP == 96 ? 1 : 2;
    static constexpr int NS = NP == 2 ? 3 : DP == 96 ? 2 : 3;  // query-step stages
    // TMEM columns: set w's S^T at 128w, dP^T at 128w + 64; then NB x (dV, dK); one dQ per set
    static constexpr int T_ACC = NP * 128;
    static constexpr int T_DQ = T_ACC + NB * 2 * DN;
    static constexpr int COLS = T_DQ + NP * DN;
    static constexpr uint32_t ALLOC = COLS <= 256 ? 256 : 512;
    static_assert(COLS <= 512, "tensor memory");
};

template <int DP>
struct BSmem {
    using G = BGeom<DP>;
    static constexpr int KV = 0;                             // KVB x (K, V)
    static constexpr int STAGE = KV + G::KVB * 2 * G::KTILE;  // NS x (Q, dO, bias^T)
    // a stage: Q, dO, bias^T, then the step's negated row statistics (-lse[64], -delta[64])
    static constexpr int STAT_OFF = 2 * G::QTILE + G::BT;
    // a multiple of 1024 bytes: every stage's 128-byte-swizzled tiles, and the dS buffers after
    // the stages, need 1024-byte-aligned bases (the swizzle follows the address bits)
    static constexpr int STAGE_BYTES = (STAT_OFF + 2 * kBQ * 4 + 1023) / 1024 * 1024;
    static constexpr int STAGE_TX = STAT_OFF;  // bytes the TMA copies bring
    static constexpr int DSB = STAGE + G::NS * STAGE_BYTES;  // one dS buffer per set
    // fp32 dS staged for the dBias reduce: per set, per warp of its two warpgroups, the warp's
    // 32 keys of its warpgroup's 32 queries, [32 queries][32 keys]
    static constexpr int RED = DSB + G::NP * G::DS;
    static constexpr int END = RED + G::NP * kBQ * kBK * 4;
    static constexpr int BYTES = END + 1024;
    static_assert(BYTES + 512 <= 227 * 1024, "shared memory (dynamic + the static barriers)");
    static_assert(STAGE % 1024 == 0 && STAGE_BYTES % 1024 == 0 && DSB % 1024 == 0 &&
                      RED % 1024 == 0,
                  "1024-byte-aligned swizzled tiles");
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

// Where global step gi of a CTA lies: its work item (key tile, head, sequence) and query step.
// Items are numbered key tiles fastest, then heads, then sequences. With p.contig, CTA b owns
// the (n, h) pairs [b P / G, (b + 1) P / G) of the P = N H pairs (G CTAs), i.e. a contiguous run
// of items whose key tiles of one (n, h) follow one another; otherwise (where whole pairs would
// balance the CTAs badly, P / G small) it takes items b, b + G, b + 2G, ... It runs every item's
// nqs query steps in turn. With p.contig nqs is nqt (the steps that hold queries) rounded up to
// a multiple of the step sets, so that step i of every item falls to the same set (whose
// threads then handle the same dQ elements at every key tile); a step past nqt has no queries
// (all its rows lie past Sq: zero tiles, no outputs). The query steps of an item start at one that depends on its
// sequence, so the CTAs of different sequences running at once reduce into different dBias
// rows.
struct StepPos {
    int k0, h, n, q0;
    int rot;            // n mod (query steps holding queries): the item's first step
    long long rowbase;  // (n * H + h) * Sq
};

// The CTA's schedule: key tiles, query steps holding queries, steps per item, its first item
// and the stride between its items
struct Sched {
    int nkt, nqt, nqs, item0, istride;
};

// The first item of this CTA, the stride to its next, and how many it owns
__device__ __forceinline__ void cta_items(const BwdParams& p, int nkt, Sched& sc, int& count) {
    const long long b = blockIdx.x, g = gridDim.x;
    if (p.contig) {
        const long long pairs = (long long)p.N * p.H;
        const long long p0 = b * pairs / g, p1 = (b + 1) * pairs / g;
        sc.item0 = (int)(p0 * nkt);
        sc.istride = 1;
        count = (int)((p1 - p0) * nkt);
    } else {
        const long long items = (long long)nkt * p.H * p.N;
        sc.item0 = (int)b;
        sc.istride = (int)g;
        count = items > b ? (int)((items - 1 - b) / g + 1) : 0;
    }
}

// The position of the CTA's item j (divisions: once per item)
__device__ __forceinline__ StepPos item_pos(const BwdParams& p, const Sched& sc, int j) {
    const int nkt = sc.nkt;
    const int u = sc.item0 + j * sc.istride;
    const int rest = u / nkt;
    StepPos s;
    s.k0 = (u - rest * nkt) * kBK;
    s.h = rest % p.H;
    s.n = rest / p.H;
    s.q0 = 0;
    s.rot = s.n % ((p.Sq + kBQ - 1) / kBQ);
    s.rowbase = ((long long)s.n * p.H + s.h) * p.Sq;
    return s;
}

__device__ __forceinline__ int rotated_q0(const StepPos& s, int nqt, int i) {
    if (i >= nqt) {
        return nqt * kBQ;  // a padding step: every row past Sq
    }
    const int r = s.rot;
    return (i + r < nqt ? i + r : i + r - nqt) * kBQ;
}

// A walk over global steps gi = j * nqs + i in strides of `by` (by <= nqs is not required)
struct StepCursor {
    int gi, j, i;
    StepPos pos;
    __device__ __forceinline__ void start(const BwdParams& p, const Sched& sc, int g) {
        gi = g;
        j = g / sc.nqs;
        i = g - j * sc.nqs;
        pos = item_pos(p, sc, j);
        pos.q0 = rotated_q0(pos, sc.nqt, i);
    }
    __device__ __forceinline__ void advance(const BwdParams& p, const Sched& sc, int by) {
        gi += by;
        i += by;
        if (i >= sc.nqs) {
            const int dj = i / sc.nqs;
            j += dj;
            i -= dj * sc.nqs;
            pos = item_pos(p, sc, j);
        }
        pos.q0 = rotated_q0(pos, sc.nqt, i);
    }
};

template <typename T, int DP, int DBIAS>
__global__ void __launch_bounds__(BGeom<DP>::THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                    const __grid_constant__ CUtensorMap tbt, const __grid_constant__ CUtensorMap tdb,
                    const BwdParams p) {
    using G = BGeom<DP>;
    using L = BSmem<DP>;
    using E = Elem<T>;
    constexpr int NP = G::NP, NS = G::NS, KVB = G::KVB, NB = G::NB;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t kv_full[KVB], kv_empty[KVB], q_full[NS], q_empty[NS], s_full[NP],
        p_ready[NP], ts_done[NP], dq_done[NP], acc_full[NB], acc_empty[NB];
    __shared__ uint32_t tmem_base_sh;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = p.D;
    const int DN = (D + 15) & ~15;
    const int nkt = (p.Sk + kBK - 1) / kBK;
    const int nqt = (p.Sq + kBQ - 1) / kBQ;
    // the host keeps items * nqs below 2^31
    const int nqs = p.contig ? (nqt + NP - 1) / NP * NP : nqt;
    Sched sc;
    int J;  // this CTA's items
    sc.nkt = nkt;
    cta_items(p, nkt, sc, J);
    sc.nqt = nqt;
    sc.nqs = nqs;
    const int total = J * nqs;  // this CTA's query steps

    if (warp == G::MMA_A) {
        if (lane == 0) {
            for (int i = 0; i < KVB; ++i) {
                mbar_init(&kv_full[i], 1);
                mbar_init(&kv_empty[i], 1);
            }
            for (int i = 0; i < NS; ++i) {
                mbar_init(&q_full[i], 32);  // the TMA warp's 32 lanes (statistics, copies)
                mbar_init(&q_empty[i], 2);  // both MMA warps read a stage
            }
            for (int i = 0; i < NP; ++i) {
                mbar_init(&s_full[i], 1);
                mbar_init(&p_ready[i], 256);
                mbar_init(&ts_done[i], 1);
                mbar_init(&dq_done[i], 1);
            }
            for (int i = 0; i < NB; ++i) {
                mbar_init(&acc_full[i], 1);
                mbar_init(&acc_empty[i], G::NWG * 128);
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

    if (warp == G::TMA_WARP) {
        // the whole warp: lane 0 issues the copies, every lane stages two of the step's row
        // statistics and arrives on the stage's barrier (released with its own stores)
        {
            for (int j = 0; j < J; ++j) {
                const StepPos it = item_pos(p, sc, j);
                const int kb = j % KVB;
                if (lane == 0) {
                    if (j >= KVB) {
                        mbar_wait(&kv_empty[kb], ((j - KVB) / KVB) & 1, &g_status,
                                  kStatusMmaWait, &abort_flag);
                    }
                    uint8_t* kv = smem + L::KV + kb * 2 * G::KTILE;
                    mbar_arrive_expect_tx(&kv_full[kb], 2 * G::KTILE);
                    for (int a = 0; a < G::NA; ++a) {
                        tma_load_4d(kv + a * G::KATOM, &tk, &kv_full[kb], a * G::AE, it.h, it.k0,
                                    it.n);
                        tma_load_4d(kv + G::KTILE + a * G::KATOM, &tv, &kv_full[kb], a * G::AE,
                                    it.h, it.k0, it.n);
                    }
                }
                for (int i = 0; i < nqs; ++i) {
                    const int gi = j * nqs + i;
                    StepPos sp = it;
                    sp.q0 = rotated_q0(it, nqt, i);
                    const int s = gi % NS;
                    // the statistics load ahead of the wait for the stage
                    float sv[4];
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const int q = sp.q0 + 32 * r + lane;
                        const bool in = q < p.Sq;
                        sv[2 * r] = in ? p.nlse[sp.rowbase + q] : -INFINITY;  // P = 0 past Sq
                        sv[2 * r + 1] = in ? p.ndelta[sp.rowbase + q] : 0.f;
                    }
                    if (gi >= NS) {
                        mbar_wait(&q_empty[s], ((gi - NS) / NS) & 1, &g_status, kStatusMmaWait,
                                  &abort_flag);
                    }
                    uint8_t* st = smem + L::STAGE + s * L::STAGE_BYTES;
                    float* stat = reinterpret_cast<float*>(st + L::STAT_OFF);
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        stat[32 * r + lane] = sv[2 * r];
                        stat[kBQ + 32 * r + lane] = sv[2 * r + 1];
                    }
                    if (lane != 0) {
                        mbar_arrive(&q_full[s]);
                        continue;
                    }
                    mbar_arrive_expect_tx(&q_full[s], L::STAGE_TX);
                    for (int a = 0; a < G::NA; ++a) {
                        tma_load_4d(st + a * G::QATOM, &tq, &q_full[s], a * G::AE, sp.h, sp.q0,
                                    sp.n);
                        tma_load_4d(st + G::QTILE + a * G::QATOM, &tdo, &q_full[s], a * G::AE,
                                    sp.h, sp.q0, sp.n);
                    }
                    tma_load_3d(st + 2 * G::QTILE, &tbt, &q_full[s], sp.q0, sp.k0, sp.h);
                }
            }
        }
    } else if (warp == G::MMA_A) {
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16(E::kBf16, 128, kBQ, false, false);
            // S^T = K Q^T and dP^T = V dO^T of step gi into set (gi % NP)'s columns, once the dV
            // and dK MMAs of that set's previous step have read its P^T and dS^T
            const auto issue_s = [&](int gi, int j, int i) {
                const int w = gi % NP, s = gi % NS, kb = j % KVB;
                if (i == 0) {
                    mbar_wait(&kv_full[kb], (j / KVB) & 1, &g_status, kStatusTmaWait,
                              &abort_flag);
                }
                mbar_wait(&q_full[s], (gi / NS) & 1, &g_status, kStatusTmaWait, &abort_flag);
                if (gi >= NP) {
                    mbar_wait(&ts_done[w], ((gi - NP) / NP) & 1, &g_status, kStatusMmaWait,
                              &abort_flag);
                }
                tc_fence_after();
                const uint32_t k_base = smem_u32(smem + L::KV + kb * 2 * G::KTILE);
                const uint32_t v_base = k_base + G::KTILE;
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
                mma_commit(&q_empty[s]);
            };
            for (int j = 0, gi = 0; j < J; ++j) {
                for (int i = 0; i < nqs; ++i, ++gi) {
                    issue_s(gi, j, i);
                }
            }
        }
    } else if (warp == G::MMA_B) {
        if (lane == 0) {
            // dV += P^T dO and dK += dS^T Q, A read from tensor memory: the 16-bit P^T (dS^T) of
            // queries [32 hf, 32 hf + 32) sits in columns [32 hf, 32 hf + 16) of S^T (dP^T)
            const uint32_t idesc_acc = idesc_f16(E::kBf16, 128, DN, false, true);
            const uint32_t idesc_dq = idesc_f16(E::kBf16, 64, DN, true, true);
            for (int gi = 0, j = 0, i = 0; gi < total; ++gi) {
                const int w = gi % NP, s = gi % NS, db = j % NB;
                if (i == 0 && j >= NB) {
                    // the accumulators of item j - NB have been stored
                    mbar_wait(&acc_empty[db], ((j - NB) / NB) & 1, &g_status, kStatusSyncWait,
                              &abort_flag);
                }
                mbar_wait(&q_full[s], (gi / NS) & 1, &g_status, kStatusTmaWait, &abort_flag);
                mbar_wait(&p_ready[w], (gi / NP) & 1, &g_status, kStatusSyncWait, &abort_flag);
                tc_fence_after();
                // dQ = dS K (M = 64 queries) first, the MMA its set flushes next; the item's
                // last one releases the K/V buffer (the item's S^T/dP^T MMAs finished before
                // its last dS existed)
                {
                    const int kb = j % KVB;
                    const uint32_t k_base = smem_u32(smem + L::KV + kb * 2 * G::KTILE);
                    const uint32_t ds_base = smem_u32(smem + L::DSB + w * G::DS);
#pragma unroll
                    for (int ks = 0; ks < kBK / 16; ++ks) {
                        const uint64_t ad =
                            smem_desc(ds_base + ks * 16 * 128, G::DS, 1024, kSwizzle128B);
                        const uint64_t bd = smem_desc(k_base + ks * 16 * G::ROWB, G::KATOM,
                                                      8 * G::ROWB, G::LAYOUT);
                        mma_ss(tmem + G::T_DQ + w * G::DN, ad, bd, idesc_dq, ks > 0 ? 1u : 0u);
                    }
                    mma_commit(&dq_done[w]);
                    if (i == nqs - 1) {
                        mma_commit(&kv_empty[kb]);
                    }
                }
                const uint32_t st = smem_u32(smem + L::STAGE + s * L::STAGE_BYTES);
                const uint32_t t_dv = tmem + G::T_ACC + db * 2 * G::DN, t_dk = t_dv + G::DN;
#pragma unroll
                for (int ks = 0; ks < kBQ / 16; ++ks) {
                    const uint32_t acol = 8 * ks + 16 * (ks >> 1);
                    const uint64_t od = smem_desc(st + G::QTILE + ks * 16 * G::ROWB, G::QATOM,
                                                  8 * G::ROWB, G::LAYOUT);
                    const uint64_t qd =
                        smem_desc(st + ks * 16 * G::ROWB, G::QATOM, 8 * G::ROWB, G::LAYOUT);
                    mma_ts(t_dv, tmem + 128 * w + acol, od, idesc_acc, (i > 0 || ks > 0) ? 1u : 0u);
                    mma_ts(t_dk, tmem + 128 * w + 64 + acol, qd, idesc_acc,
                           (i > 0 || ks > 0) ? 1u : 0u);
                }
                mma_commit(&ts_done[w]);
                mma_commit(&q_empty[s]);
                if (i == nqs - 1) {
                    mma_commit(&acc_full[db]);
                }
                if (++i == nqs) {
                    i = 0;
                    ++j;
                }
            }
        }
    } else {
        // softmax warpgroups: worker (wg, t) owns key k0 + t = TMEM lane t, for the queries
        // [32 hf, 32 hf + 32) of the steps of set `set`
        const int wg = warp >> 2, set = wg >> 1, hf = wg & 1, t = ((warp & 3) << 5) | lane;
        const uint32_t lane_base = tmem_lane_base(warp);
        const float qk_scale = p.scale * kLog2e;
        const float masked = kMaskedLogit * kLog2e;
        const uint64_t qk2 = pk2(qk_scale, qk_scale), log2e2 = pk2(kLog2e, kLog2e);
        // this warp's fp32 dS staging for the dBias reduce: [32 queries][its 32 keys]
        float* rbuf = reinterpret_cast<float*>(smem + L::RED) + set * (kBQ * kBK) +
                      (4 * hf + (warp & 3)) * (32 * 32);
        uint8_t* ds_row = smem + L::DSB + set * G::DS + t * 128;
        const uint32_t t_dq = tmem + G::T_DQ + set * G::DN;
        const uint32_t t_st = tmem + 128 * set + lane_base + 32 * hf, t_dp = t_st + 64;

        // dQ of a step: lanes 32w + r (r < 16) hold query row 16w + r (M=64 layout); the two
        // warpgroups of the set take alternate 16-column chunks. The same thread handles these
        // dQ elements at this step of every key tile of the (n, h), in key-tile order: the first
        // stores its tile, the later ones add to it (after that store: program order).
        const auto flush_dq = [&](const StepPos& sp) {
            const int q = sp.q0 + 16 * (warp & 3) + lane;
            const bool first = p.contig && sp.k0 == 0;
            for (int c = 16 * hf; c < DN; c += 32) {
                uint32_t r[16];
                tmem_ld16(t_dq + lane_base + c, r);
                tmem_wait_ld();
                if (lane < 16 && q < p.Sq) {
                    float* dst = p.dq_acc + (sp.rowbase + q) * D + c;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        if (c + 4 * g < D) {
                            const float4 v = make_float4(__uint_as_float(r[4 * g]) * p.scale,
                                                         __uint_as_float(r[4 * g + 1]) * p.scale,
                                                         __uint_as_float(r[4 * g + 2]) * p.scale,
                                                         __uint_as_float(r[4 * g + 3]) * p.scale);
                            if (first) {
                                *reinterpret_cast<float4*>(dst + 4 * g) = v;
                            } else {
                                atomicAdd(reinterpret_cast<float4*>(dst + 4 * g), v);
                            }
                        }
                    }
                }
            }
        };

        // dK (scaled) and dV of item e out of accumulator set e % NB: warpgroup wg takes dK
        // (even) or dV (odd) and every NP-th 16-column chunk of it
        const auto store_acc = [&](int e) {
            const int db = e % NB;
            mbar_wait(&acc_full[db], (e / NB) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            const StepPos it = item_pos(p, sc, e);
            const int key = it.k0 + t;
            const long long krow = ((long long)it.n * p.H + it.h) * p.Sk + key;
            const int which = wg & 1;
            const uint32_t acc = tmem + G::T_ACC + db * 2 * G::DN + (which == 0 ? G::DN : 0) +
                                 lane_base;
            T* dst = reinterpret_cast<T*>(which == 0 ? p.dk : p.dv) + krow * D;
            const float mul = which == 0 ? p.scale : 1.f;
            for (int c = 16 * (wg >> 1); c < DN; c += 16 * NP) {
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
                            for (int e2 = 0; e2 < 4; ++e2) {
                                pw[e2] = E::pack(__uint_as_float(r[8 * hh + 2 * e2]) * mul,
                                                 __uint_as_float(r[8 * hh + 2 * e2 + 1]) * mul);
                            }
                            *reinterpret_cast<uint4*>(dst + c8) = w;
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[db]);
        };

        // per-item state of this worker's key
        int cur_item = -1;
        bool live = false, warp_live = false;
        float* dbias_col = nullptr;

        // this warpgroup's 32 queries of a step, in two chunks of 16: P^T, dS^T (TMEM, packed
        // over the chunk's own S^T/dP^T columns), dS (shared), dBias
        const auto half_step = [&](auto fast, const uint8_t* brow, const float* lsh,
                                   const float* dlh, int q0, int jn, int key) {
            // this half's first dBias row (the per-element reduction mode only)
            [[maybe_unused]] float* drow = dbias_col + (long long)(q0 + 32 * hf) * p.Sk;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                uint32_t sr[16], dr[16];
                tmem_ld16(t_st + 16 * cc, sr);
                tmem_ld16(t_dp + 16 * cc, dr);
                tmem_wait_ld();
                uint32_t pw[8], dw[8];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int qc = 16 * cc + 4 * c;  // query offset within the half
                    // queries 32 hf + qc .. +4: half of 16-byte chunk 4 hf + qc/8 of the key's row
                    const uint2 b2 = *reinterpret_cast<const uint2*>(
                        brow + (((4 * hf + (qc >> 3)) ^ (t & 7)) << 4) + (c & 1) * 8);
                    const float2 b01 = E::unpack(b2.x);
                    const float2 b23 = E::unpack(b2.y);
                    // the statistics are stored negated: -lse and -delta
                    const float4 l4 = *reinterpret_cast<const float4*>(lsh + qc);
                    const float4 d4 = *reinterpret_cast<const float4*>(dlh + qc);
                    float pv[4], gv[4];
                    if constexpr (decltype(fast)::value) {
                        // two queries an instruction (paired fp32): log2e bias - lse,
                        // + scale log2e s, exp2, dS = P (dP - delta)
#pragma unroll
                        for (int e = 0; e < 4; e += 2) {
                            const int j = 4 * c + e;
                            const float2 bb = e == 0 ? b01 : b23;
                            const uint64_t nl = e == 0 ? pk2(l4.x, l4.y) : pk2(l4.z, l4.w);
                            const uint64_t nd = e == 0 ? pk2(d4.x, d4.y) : pk2(d4.z, d4.w);
                            const uint64_t bl = fma2(pk2(bb.x, bb.y), log2e2, nl);
                            const float2 x = upk2(fma2(
                                pk2(__uint_as_float(sr[j]), __uint_as_float(sr[j + 1])), qk2, bl));
                            float2 pp;
                            if (c == 3 && e == 2) {
                                pp = ex2_fma(x.x, x.y);  // one pair in eight on the FMA pipe
                            } else {
                                pp = make_float2(ex2(x.x), ex2(x.y));
                            }
                            const float2 gg = upk2(mul2(
                                pk2(pp.x, pp.y),
                                add2(pk2(__uint_as_float(dr[j]), __uint_as_float(dr[j + 1])), nd)));
                            pv[e] = pp.x;
                            pv[e + 1] = pp.y;
                            gv[e] = gg.x;
                            gv[e + 1] = gg.y;
                        }
                    } else {
                        const float bl[4] = {fmaf(b01.x, kLog2e, l4.x), fmaf(b01.y, kLog2e, l4.y),
                                             fmaf(b23.x, kLog2e, l4.z), fmaf(b23.y, kLog2e, l4.w)};
                        const float nl[4] = {l4.x, l4.y, l4.z, l4.w};
                        const float nd[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int j = 4 * c + e;
                            const float l2 = live ? fmaf(__uint_as_float(sr[j]), qk_scale, bl[e])
                                                  : masked + nl[e];
                            pv[e] = ex2(l2);
                            gv[e] = live ? pv[e] * (__uint_as_float(dr[j]) + nd[e]) : 0.f;
                        }
                    }
                    pw[2 * c] = E::pack(pv[0], pv[1]);
                    pw[2 * c + 1] = E::pack(pv[2], pv[3]);
                    dw[2 * c] = E::pack(gv[0], gv[1]);
                    dw[2 * c + 1] = E::pack(gv[2], gv[3]);
                    if constexpr (DBIAS == kDbiasTma) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            rbuf[(qc + e) * 32 + lane] = gv[e];
                        }
                    } else if constexpr (DBIAS == kDbiasRed) {
                        if (key < p.Sk) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (qc + e < jn) {
                                    red_add_f32(drow + (long long)(qc + e) * p.Sk, gv[e]);
                                }
                            }
                        }
                    }
                }
                tmem_st8(t_st + 8 * cc, pw);
                tmem_st8(t_dp + 8 * cc, dw);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int chunk = 4 * hf + 2 * cc + c;
                    *reinterpret_cast<uint4*>(ds_row + ((chunk ^ (t & 7)) << 4)) =
                        make_uint4(dw[4 * c], dw[4 * c + 1], dw[4 * c + 2], dw[4 * c + 3]);
                }
            }
        };

        // cur: this step; nxt: this set's next step; prev: the set's previous step (its dQ is
        // flushed at the start of this one)
        StepCursor cur, nxt;
        cur.start(p, sc, set);
        nxt = cur;
        nxt.advance(p, sc, NP);
        StepPos prev = cur.pos;
        int k = 0, stored = 0;  // this set's steps so far; items whose dK/dV this group stored
        for (; cur.gi < total; ++k) {
            const int gi = cur.gi, s = gi % NS, j = cur.j;
            const StepPos sp = cur.pos;
            if constexpr (DBIAS == kDbiasTma) {
                if (lane == 0 && k >= 1) {
                    bulk_wait_read();  // this warp's previous reduce has read its dS rows
                }
                __syncwarp();
            }
            if (k >= 1) {
                // this set's previous step: dQ out of tensor memory before it is reused
                mbar_wait(&dq_done[set], (k - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
                tc_fence_after();
                flush_dq(prev);
            }
            if (j != cur_item) {
                cur_item = j;
                const int key = sp.k0 + t;
                live = key < p.Sk && p.kmask[(long long)sp.n * p.Sk + key] != 0;
                warp_live = __all_sync(0xffffffffu, live);
                dbias_col = p.dbias + (long long)sp.h * p.Sq * p.Sk + key;
            }
            mbar_wait(&q_full[s], (gi / NS) & 1, &g_status, kStatusTmaWait, &abort_flag);
            mbar_wait(&s_full[set], k & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            const uint8_t* stage = smem + L::STAGE + s * L::STAGE_BYTES;
            const uint8_t* brow = stage + 2 * G::QTILE + t * 128;
            // the step's negated row statistics, staged by the TMA warp
            const float* ls = reinterpret_cast<const float*>(stage + L::STAT_OFF) + 32 * hf;
            const float* dl = ls + kBQ;
            const int jn = min(32, p.Sq - sp.q0 - 32 * hf);
            if (warp_live) {
                half_step(std::true_type{}, brow, ls, dl, sp.q0, jn, sp.k0 + t);
            } else {
                half_step(std::false_type{}, brow, ls, dl, sp.q0, jn, sp.k0 + t);
            }
            tmem_wait_st();
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(&p_ready[set]);
            if constexpr (DBIAS == kDbiasTma) {
                // this warp's 32 queries x 32 keys of fp32 dS in one bulk reduce-add (rows past
                // Sq and keys past Sk clip)
                __syncwarp();
                if (lane == 0 && jn > 0 && sp.k0 + 32 * (warp & 3) < p.Sk) {
                    tma_reduce_add_3d(&tdb, rbuf, sp.k0 + 32 * (warp & 3), sp.q0 + 32 * hf, sp.h);
                }
            }
            // the accumulators of the items before this one: their last MMAs were issued a
            // step ago, so they are done or nearly so
            while (stored < j) {
                store_acc(stored++);
            }
            prev = sp;
            cur = nxt;
            nxt.advance(p, sc, NP);
        }
        if constexpr (DBIAS == kDbiasTma) {
            if (lane == 0) {
                bulk_wait_all();
            }
        }
        if (k >= 1) {
            mbar_wait(&dq_done[set], (k - 1) & 1, &g_status, kStatusMmaWait, &abort_flag);
            tc_fence_after();
            flush_dq(prev);
        }
        while (stored < J) {
            store_acc(stored++);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == G::MMA_A) {
        tc_fence_after();
        tmem_dealloc(tmem, G::ALLOC);
    }
}

// The backward's row statistics, negated: ndelta[row] = -sum_c out[row][c] * dout[row][c] and
// nlse[row] = -lse[row]; one thread per row, 16-byte loads. With dq_zero the row of the float32
// dQ accumulator is zeroed in the same pass.
template <typename T>
__global__ void row_delta_kernel(const T* __restrict__ out, const T* __restrict__ dout,
                                 const float* __restrict__ lse, float* __restrict__ ndelta,
                                 float* __restrict__ nlse, float* __restrict__ dq_zero,
                                 long long rows, int D) {
    using E = Elem<T>;
    const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) {
        return;
    }
    if (dq_zero != nullptr) {
        float4* z = reinterpret_cast<float4*>(dq_zero + r * D);
        for (int c = 0; c < D / 4; ++c) {
            z[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
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
    ndelta[r] = -s;
    nlse[r] = -lse[r];
}

// The gated backward's prologue (the attention output is y = o * s, s = sigmoid(gate + gate_bias)):
// dO = dy * s, the attention gradient the main kernel differentiates; dgate = dy * o * s (1 - s)
// = dy * y * (1 - s); the row statistic delta = sum_c o dO = sum_c y dy; and dgate_bias summed
// over the block's 64 queries in a fixed order, then added into [H, D] with one float atomic a
// column. Grid (ceil(Sq / 64), H, N); a block is 64 queries x D/8 threads, a thread 8 columns.
template <typename T>
__global__ void gate_prologue_kernel(const T* __restrict__ y, const T* __restrict__ dy,
                                     const T* __restrict__ gate, const T* __restrict__ gate_bias,
                                     const float* __restrict__ lse, T* __restrict__ dog,
                                     T* __restrict__ dgate, float* __restrict__ dgate_bias,
                                     float* __restrict__ ndelta, float* __restrict__ nlse,
                                     float* __restrict__ dq_zero, int H, int Sq, int D) {
    using E = Elem<T>;
    extern __shared__ float gsh[];  // [64][D] dgate (float32), then [64][D/8] partial deltas
    const int cpr = D >> 3;
    const int tid = threadIdx.x, rloc = tid / cpr, chunk = tid - rloc * cpr, c8 = chunk * 8;
    const int h = blockIdx.y, n = blockIdx.z, s = blockIdx.x * 64 + rloc;
    float dg[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float part = 0.f;
    if (s < Sq) {
        const long long off = (((long long)n * H + h) * Sq + s) * D + c8;
        const uint4 yv = *reinterpret_cast<const uint4*>(y + off);
        const uint4 dv = *reinterpret_cast<const uint4*>(dy + off);
        const uint4 gv = *reinterpret_cast<const uint4*>(gate + off);
        const uint4 bv = *reinterpret_cast<const uint4*>(gate_bias + (long long)h * D + c8);
        const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t ow[4], qw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 yy = E::unpack(yw[i]), dd = E::unpack(dw[i]), gg = E::unpack(gw[i]),
                         bb = E::unpack(bw[i]);
            // the forward's sigmoid: 1 / (1 + 2^(-log2e (g + gb)))
            const float s0 = __fdividef(1.f, 1.f + ex2(-kLog2e * (gg.x + bb.x)));
            const float s1 = __fdividef(1.f, 1.f + ex2(-kLog2e * (gg.y + bb.y)));
            ow[i] = E::pack(dd.x * s0, dd.y * s1);
            dg[2 * i] = dd.x * yy.x * (1.f - s0);
            dg[2 * i + 1] = dd.y * yy.y * (1.f - s1);
            qw[i] = E::pack(dg[2 * i], dg[2 * i + 1]);
            part = fmaf(yy.x, dd.x, part);
            part = fmaf(yy.y, dd.y, part);
        }
        *reinterpret_cast<uint4*>(dog + off) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        *reinterpret_cast<uint4*>(dgate + off) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
        if (dq_zero != nullptr) {  // this thread's 8 columns of the float32 dQ accumulator
            float4* z = reinterpret_cast<float4*>(dq_zero + off);
            z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
            z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        gsh[rloc * D + c8 + i] = dg[i];
    }
    float* psh = gsh + 64 * D;
    psh[rloc * cpr + chunk] = part;
    __syncthreads();
    if (tid < 64) {
        const int s2 = blockIdx.x * 64 + tid;
        if (s2 < Sq) {
            float d = 0.f;
            for (int c = 0; c < cpr; ++c) {
                d += psh[tid * cpr + c];
            }
            const long long row = ((long long)n * H + h) * Sq + s2;
            ndelta[row] = -d;
            nlse[row] = -lse[row];
        }
    }
    if (tid < D) {
        float acc = 0.f;
        for (int r = 0; r < 64; ++r) {
            acc += gsh[r * D + tid];
        }
        atomicAdd(dgate_bias + (long long)h * D + tid, acc);
    }
}

// bt[h][k][q] = bias[h][q][k] in the bias's own 16-bit type (exact), queries padded to Sqp with
// zeros; 32x32 tiles
template <typename T>
__global__ void bias_transpose_kernel(const T* __restrict__ bias, T* __restrict__ bt, int Sq,
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
    T* dst = bt + (long long)h * Sk * Sqp;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, q = q0 + threadIdx.x;
        if (k < Sk && q < Sqp) {
            dst[(long long)k * Sqp + q] = Elem<T>::from_f(tile[threadIdx.x][r]);
        }
    }
}

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

// The same transpose with 16-byte accesses (Sk % 8 == 0, a 16-byte-aligned bias): a block moves
// a 64 x 64 tile, each thread two 8-key pieces of bias rows in and two 8-query pieces of bt rows
// out, through a shared tile padded so that the column reads spread over the banks. With
// dbias_zero (16-byte aligned) the block also zeroes the same tile of dBias [H, Sq, Sk].
template <typename T>
__global__ void __launch_bounds__(256) bias_transpose_vec_kernel(const T* __restrict__ bias,
                                                                 T* __restrict__ bt, int Sq,
                                                                 int Sk, int Sqp,
                                                                 float* __restrict__ dbias_zero) {
    __shared__ __align__(16) uint16_t tile[64][64 + 2];
    const int h = blockIdx.z, q0 = blockIdx.x * 64, k0 = blockIdx.y * 64, tid = threadIdx.x;
    const uint16_t* src = reinterpret_cast<const uint16_t*>(bias) + (long long)h * Sq * Sk;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int piece = tid + 256 * r, qr = piece >> 3, kc = (piece & 7) * 8;
        const int q = q0 + qr, k = k0 + kc;
        uint4 w = make_uint4(0, 0, 0, 0);
        if (q < Sq && k < Sk) {  // Sk % 8 == 0: the piece is whole
            w = *reinterpret_cast<const uint4*>(src + (long long)q * Sk + k);
        }
        // rows of 132 bytes: every pair of keys starts on a 4-byte boundary
        uint32_t* row = reinterpret_cast<uint32_t*>(&tile[qr][kc]);
        row[0] = w.x;
        row[1] = w.y;
        row[2] = w.z;
        row[3] = w.w;
    }
    if (dbias_zero != nullptr) {
        float* zb = dbias_zero + (long long)h * Sq * Sk;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int piece = tid + 256 * r, qr = piece >> 4, kc = (piece & 15) * 4;
            const int q = q0 + qr, k = k0 + kc;
            if (q < Sq && k < Sk) {  // Sk % 8 == 0: the 4 floats are whole
                *reinterpret_cast<float4*>(zb + (long long)q * Sk + k) =
                    make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    __syncthreads();
    uint16_t* dst = reinterpret_cast<uint16_t*>(bt) + (long long)h * Sk * Sqp;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int piece = tid + 256 * r, kr = piece >> 3, qc = (piece & 7) * 8;
        const int k = k0 + kr, q = q0 + qc;
        if (k < Sk && q < Sqp) {  // Sqp % 8 == 0: the piece is whole (zeros past Sq)
            uint32_t ww[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ww[e] = (uint32_t)tile[qc + 2 * e][kr] | ((uint32_t)tile[qc + 2 * e + 1][kr] << 16);
            }
            *reinterpret_cast<uint4*>(dst + (long long)k * Sqp + q) =
                make_uint4(ww[0], ww[1], ww[2], ww[3]);
        }
    }
}

// SMs of device dev (cached)
int sm_count_of(int dev) {
    static int sms[kMaxDevices] = {};
    if (dev >= 0 && dev < kMaxDevices && sms[dev] == 0) {
        cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    }
    return dev >= 0 && dev < kMaxDevices && sms[dev] > 0 ? sms[dev] : 148;
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

// Workspace: dQ partial sums | -delta | -lse | bias^T (16-bit, queries padded to a multiple of
// 8) | (gated backward only) dO = dy * sigmoid(gate + gate_bias), 16-bit [N,H,Sq,D]; each part
// 256-byte aligned. `ok` is false when a size product overflows 64 bits.
struct Workspace {
    size_t dq = 0, delta = 0, nlse = 0, bt = 0, dog = 0, total = 0;
    bool ok = false;
    static Workspace of(uint64_t N, uint64_t H, uint64_t Sq, uint64_t Sk, uint64_t D,
                        bool gated = false) {
        Workspace w;
        uint64_t rows, dqb, btb;
        const uint64_t sqp = (Sq + 7) & ~uint64_t(7);
        if (Sq > (uint64_t(1) << 40) || __builtin_mul_overflow(N, H, &rows) ||
            __builtin_mul_overflow(rows, Sq, &rows) || __builtin_mul_overflow(rows, D, &dqb) ||
            __builtin_mul_overflow(dqb, uint64_t(4), &dqb) || rows > (uint64_t(1) << 60) ||
            __builtin_mul_overflow(H, Sk, &btb) || __builtin_mul_overflow(btb, sqp, &btb) ||
            __builtin_mul_overflow(btb, uint64_t(2), &btb) || dqb > (uint64_t(1) << 60) ||
            btb > (uint64_t(1) << 60)) {
            return w;
        }
        w.dq = 0;
        w.delta = align256(dqb);
        w.nlse = w.delta + align256(rows * sizeof(float));
        w.bt = w.nlse + align256(rows * sizeof(float));
        w.dog = w.bt + align256(btb);
        w.total = w.dog + (gated ? align256(dqb / 2) : 0);
        w.ok = true;
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
    // persistent: one CTA per SM, each looping over work items (with p.contig every CTA owns at
    // least one (n, h) pair and all of its key tiles)
    const long long pairs = (long long)p.N * p.H;
    const long long units = p.contig ? pairs : pairs * ((p.Sk + kBK - 1) / kBK);
    const dim3 grid((unsigned)std::min<long long>(units, sm_count_of(dev)));
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

// The gated backward's extra buffers (all null for the plain backward)
struct GateIO {
    const void* gate = nullptr;       // [N,H,Sq,D]
    const void* gate_bias = nullptr;  // [H,D]
    void* dgate = nullptr;            // [N,H,Sq,D]
    float* dgate_bias = nullptr;      // [H,D] float32
    void* dog = nullptr;              // workspace: dO = dy * sigmoid(gate + gate_bias)
};

template <typename T>
cudaError_t run_backward(cudaStream_t stream, const CUtensorMap* maps, const BwdParams& p,
                         const void* bias, void* bt, int Sqp, const void* out, const void* dout,
                         const float* lse, float* ndelta, float* nlse, void* dq, int dbias_mode,
                         const GateIO* g) {
    const long long rows = (long long)p.N * p.H * p.Sq;
    cudaError_t e;
    // dBias is zeroed by the vectorised transpose where it can (16-byte aligned), else here
    const bool vec_transpose = p.Sk % 8 == 0 && aligned16(bias);
    const bool zero_in_transpose = vec_transpose && aligned16(p.dbias);
    if (!zero_in_transpose &&
        (e = cudaMemsetAsync(p.dbias, 0, sizeof(float) * (size_t)p.H * p.Sq * p.Sk, stream)) !=
            cudaSuccess) {
        return e;
    }
    // the strided schedule adds every key tile's dQ into the accumulator, which the row
    // statistic's pass zeroes
    float* dq_zero = p.contig ? nullptr : p.dq_acc;
    if (g == nullptr) {
        row_delta_kernel<T><<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(
            static_cast<const T*>(out), static_cast<const T*>(dout), lse, ndelta, nlse, dq_zero,
            rows, p.D);
    } else {
        if ((e = cudaMemsetAsync(g->dgate_bias, 0, sizeof(float) * (size_t)p.H * p.D, stream)) !=
            cudaSuccess) {
            return e;
        }
        const int cpr = p.D / 8;
        const dim3 ggrid((p.Sq + 63) / 64, p.H, p.N);
        gate_prologue_kernel<T><<<ggrid, 64 * cpr, (size_t)64 * (p.D + cpr) * sizeof(float),
                                  stream>>>(
            static_cast<const T*>(out), static_cast<const T*>(dout),
            static_cast<const T*>(g->gate), static_cast<const T*>(g->gate_bias), lse,
            static_cast<T*>(g->dog), static_cast<T*>(g->dgate), g->dgate_bias, ndelta, nlse,
            dq_zero, p.H, p.Sq, p.D);
    }
    if (vec_transpose) {
        const dim3 tgrid((Sqp + 63) / 64, (p.Sk + 63) / 64, p.H);
        bias_transpose_vec_kernel<T><<<tgrid, 256, 0, stream>>>(
            static_cast<const T*>(bias), static_cast<T*>(bt), p.Sq, p.Sk, Sqp,
            zero_in_transpose ? p.dbias : nullptr);
    } else {
        const dim3 tgrid((Sqp + 31) / 32, (p.Sk + 31) / 32, p.H);
        bias_transpose_kernel<T><<<tgrid, dim3(32, 8), 0, stream>>>(static_cast<const T*>(bias),
                                                                     static_cast<T*>(bt), p.Sq,
                                                                     p.Sk, Sqp);
    }
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
    const Workspace ws = Workspace::of(N, H, Sq, Sk, D);
    if (!ws.ok) {
        return fail(kInvalidArgument, "volta_mma_bwd: sizes overflow the workspace size");
    }
    *bytes = ws.total;
    return kOk;
}

namespace cflk {
namespace {

// VoltaMmaBwd, and with g the gated backward: out is then the gated output y, dout dy.
int backward(void* stream_, int dtype, const void* q, const void* k, const void* v,
             const void* bias, const uint8_t* kmask, const void* out, const void* dout,
             const float* lse, void* dq, void* dk, void* dv, float* dbias, void* workspace,
             size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
             float scale, int want_dbias, GateIO* g) {
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
    {
        // (key tile, query step) pairs, each factor below 2^31 so that no product wraps
        int64_t pairs = 0;
        if (N >= (int64_t(1) << 31) || H >= (int64_t(1) << 31) || Sq >= (int64_t(1) << 31) ||
            Sk >= (int64_t(1) << 31) ||
            __builtin_mul_overflow((Sk + kBK - 1) / kBK, H, &pairs) ||
            __builtin_mul_overflow(pairs, N, &pairs) ||
            __builtin_mul_overflow(pairs, ((Sq + kBQ - 1) / kBQ + 1) & ~int64_t(1), &pairs) ||
            pairs >= (int64_t(1) << 31)) {
            return fail(kInvalidArgument,
                        "volta_mma_bwd: more than 2^31 (key tile, query step) pairs");
        }
    }
    const Workspace ws = Workspace::of(N, H, Sq, Sk, D, g != nullptr);
    if (!ws.ok) {
        return fail(kInvalidArgument, "volta_mma_bwd: sizes overflow the workspace size");
    }
    if (g != nullptr &&
        (!aligned16(g->gate) || !aligned16(g->gate_bias) || !aligned16(g->dgate) ||
         g->dgate_bias == nullptr)) {
        return fail(kInvalidArgument, "volta_mma_gated_bwd: gate buffers must be 16-byte aligned");
    }
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
    float* ndelta = reinterpret_cast<float*>(wsb + ws.delta);
    float* nlse = reinterpret_cast<float*>(wsb + ws.nlse);
    void* bt = wsb + ws.bt;
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
        if (g != nullptr) {
            if (rows > 0) {
                cudaMemsetAsync(g->dgate, 0, rows * D * 2, stream);
            }
            if (H > 0) {
                cudaMemsetAsync(g->dgate_bias, 0, sizeof(float) * (size_t)H * D, stream);
            }
        }
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? kOk
                                : fail(kInternal, std::string("volta_mma_bwd launch: ") +
                                                      cudaGetErrorString(e));
    }
    if (g != nullptr) {
        g->dog = wsb + ws.dog;
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
            !encode_tiled(&maps[3], tdt, 2, 4, g != nullptr ? g->dog : dout, dq4, sq4, boxq, sw) ||
            !encode_tiled(&maps[4], tdt, 2, 3, bt, dbt, sbt, boxbt, CU_TENSOR_MAP_SWIZZLE_128B)) {
            return fail(kInvalidArgument, "volta_mma_bwd: TMA descriptor rejected");
        }
    }
    // dBias by TMA bulk reduce where its rows are 16-byte multiples, else by fp32 reductions
    int dbias_mode = want_dbias ? kDbiasRed : kDbiasNone;
    maps[5] = maps[4];
    if (want_dbias && Sk % 4 == 0 && (reinterpret_cast<uintptr_t>(dbias) & 15) == 0) {
        const uint64_t ddb[3] = {(uint64_t)Sk, (uint64_t)Sq, (uint64_t)H};
        const uint64_t sdb[2] = {(uint64_t)Sk, (uint64_t)Sq * (uint64_t)Sk};
        const uint32_t boxdb[3] = {32, 32, 1};  // one warp's keys x one warpgroup's queries
        if (encode_tiled(&maps[5], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 3, dbias, ddb, sdb, boxdb,
                         CU_TENSOR_MAP_SWIZZLE_NONE)) {
            dbias_mode = kDbiasTma;
        }
    }
    BwdParams p;
    p.kmask = kmask;
    p.nlse = nlse;
    p.ndelta = ndelta;
    p.dq_acc = dq_acc;
    {
        // contiguous (n, h) runs when whole pairs balance the CTAs about as well as single
        // items do (the busiest CTA within 2% of the strided schedule's), else strided
        int dev = 0;
        cudaGetDevice(&dev);
        const long long g = sm_count_of(dev), pairs = N * H, nkt = (Sk + kBK - 1) / kBK;
        const long long most_contig = (pairs + g - 1) / g * nkt;
        const long long most_strided = (pairs * nkt + g - 1) / g;
        p.contig = 100 * most_contig <= 102 * most_strided ? 1 : 0;
    }
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
                                                     lse, ndelta, nlse, dq, dbias_mode, g)
                       : run_backward<__half>(stream, maps, p, bias, bt, Sqp, out, dout, lse,
                                              ndelta, nlse, dq, dbias_mode, g);
    if (e != cudaSuccess) {
        return fail(kInternal, std::string("volta_mma_bwd launch: ") + cudaGetErrorString(e));
    }
    return kOk;
}

}  // namespace
}  // namespace cflk

extern "C" int cflk_volta_mma_bwd(void* stream, int dtype, const void* q, const void* k,
                                  const void* v, const void* bias, const uint8_t* kmask,
                                  const void* out, const void* dout, const float* lse, void* dq,
                                  void* dk, void* dv, float* dbias, void* workspace,
                                  size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq,
                                  int64_t Sk, int64_t D, float scale, int want_dbias) {
    clear_error();
    return backward(stream, dtype, q, k, v, bias, kmask, out, dout, lse, dq, dk, dv, dbias,
                    workspace, workspace_bytes, N, H, Sq, Sk, D, scale, want_dbias, nullptr);
}

extern "C" int cflk_volta_mma_gated_bwd_workspace_size(int64_t N, int64_t H, int64_t Sq,
                                                       int64_t Sk, int64_t D, size_t* bytes) {
    clear_error();
    if (N < 0 || H < 0 || Sq < 0 || Sk < 0 || D < 0 || bytes == nullptr) {
        return fail(kInvalidArgument, "volta_mma_gated_bwd: bad sizes");
    }
    const Workspace ws = Workspace::of(N, H, Sq, Sk, D, true);
    if (!ws.ok) {
        return fail(kInvalidArgument, "volta_mma_gated_bwd: sizes overflow the workspace size");
    }
    *bytes = ws.total;
    return kOk;
}

extern "C" int cflk_volta_mma_gated_bwd(void* stream, int dtype, const void* q, const void* k,
                                        const void* v, const void* gate, const void* gate_bias,
                                        const void* bias, const uint8_t* kmask, const void* y,
                                        const void* dy, const float* lse, void* dq, void* dk,
                                        void* dv, void* dgate, float* dgate_bias, float* dbias,
                                        void* workspace, size_t workspace_bytes, int64_t N,
                                        int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                        float scale, int want_dbias) {
    clear_error();
    GateIO g;
    g.gate = gate;
    g.gate_bias = gate_bias;
    g.dgate = dgate;
    g.dgate_bias = dgate_bias;
    return backward(stream, dtype, q, k, v, bias, kmask, y, dy, lse, dq, dk, dv, dbias,
                    workspace, workspace_bytes, N, H, Sq, Sk, D, scale, want_dbias, &g);
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

// The array's device address on the current device, looked up on the first call on each device
// and kept in an atomic slot (two host threads making that first call at once both look it up
// and store the same value). The host-side name g_noalloc_scratch is only a stand-in for the
// symbol, never a device pointer. A cudaDeviceReset unloads the module; the cached address is
// then stale, so the library must not be used on that device after a reset.
static int noalloc_scratch(void** out) {
    static std::atomic<void*> addr[cflk::kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        return cflk::fail(cflk::kInternal, std::string("volta_mma_bwd_noalloc: ") +
                                               cudaGetErrorString(e));
    }
    if (dev < 0 || dev >= cflk::kMaxDevices) {
        return cflk::fail(cflk::kInternal, "volta_mma_bwd_noalloc: device ordinal out of range");
    }
    void* a = addr[dev].load(std::memory_order_acquire);
    if (a == nullptr) {
        e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
        if (e != cudaSuccess || a == nullptr) {
            return cflk::fail(cflk::kInternal,
                              std::string("volta_mma_bwd_noalloc: scratch address: ") +
                                  cudaGetErrorString(e));
        }
        addr[dev].store(a, std::memory_order_release);
    }
    *out = a;
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
                              " (cflk_volta_mma_bwd_workspace_size: about 4*N*H*Sq*(D+2) + "
                              "2*H*Sk*Sq8 bytes, Sq8 = Sq rounded up to 8); use "
                              "cflk_volta_mma_bwd with a workspace");
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

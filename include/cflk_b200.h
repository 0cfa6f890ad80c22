/* C ABI of the B200 (sm_100a) library that takes over colabfold-legacy-kernels' hot path for
 * compute capability 100: libcflk_sm100.so.
 *
 * Every entry point takes plain device pointers, sizes and attributes, launches asynchronously
 * on the given CUDA stream (a cudaStream_t, NULL for the legacy default stream) on the current
 * device, does no host synchronisation and allocates nothing. Each one replaces one XLA FFI
 * target of the reference (named below with its file:line); an XLA FFI handler, where the XLA
 * headers exist, is a thin shim over these functions.
 *
 * 16-bit buffers hold `dtype` elements: CFLK_F16 (the reference's F16, bit-compatible) or
 * CFLK_BF16 (an extension). float buffers are float32. Pointers to 16-bit data must be 16-byte
 * aligned. Returns CFLK_OK, CFLK_INVALID_ARGUMENT (nothing launched; message from
 * cflk_last_error) or CFLK_INTERNAL (a launch failed).
 */
#ifndef CFLK_B200_H
#define CFLK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CFLK_API __attribute__((visibility("default")))
#else
#define CFLK_API
#endif

#define CFLK_OK 0
#define CFLK_INVALID_ARGUMENT 1
#define CFLK_INTERNAL 2

#define CFLK_F16 0
#define CFLK_BF16 1

/* Message of this thread's last failed call ("" after a successful one). */
CFLK_API const char* cflk_last_error(void);

/* 100: the compute capability the library is built for. */
CFLK_API int cflk_version(void);

/* OR of the bit codes that kernels record when a bounded wait gave up (1: a TMA load,
 * 2: an MMA, 4: a thread-group barrier), cleared by the read. Call after synchronising. */
CFLK_API unsigned cflk_device_status(void);

/* ---- attention ------------------------------------------------------------------------- */

/* VoltaMma: out = softmax(scale * q k^T + bias[h]; kmask) v, and the log2-domain row statistic.
 * q [N,H,Sq,D], k and v [N,H,Sk,D], bias [H,Sq,Sk] (16-bit); kmask [N,Sk] u8 (0 masks a key);
 * out [N,H,Sq,D]; lse [N,H,Sq] float32, left untouched when want_lse is 0 (a one-element buffer
 * is then enough, or NULL). D in {8,16,24,32,48,64,96}; (D, block_q, block_k) must be a tuple
 * the reference accepts, taken as a hint only.
 * Replaces VoltaMma, cuda/volta_mma_attn.cu:524-542,625-640. */
CFLK_API int cflk_volta_mma(void* stream, int dtype, const void* q, const void* k, const void* v,
                            const void* bias, const uint8_t* kmask, void* out, float* lse,
                            int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale,
                            int64_t block_q, int64_t block_k, int want_lse);

/* VoltaMmaPacked / VoltaMmaPackedTrim: q, k, v (and the gate when G == 4) read in place from
 * p [X,Y,G,H,D]; out [X,Y,H,D] = attention * sigmoid(gate + gate_bias[h,c]). Rows attend along
 * Y (batch X); with column set, columns attend along X (batch Y). bias [H,S,S], kmask [N,S],
 * gate_bias [H,D]; the *_elems arguments are those buffers' element counts, checked as the
 * reference checks them. lims [N+1] int32 or NULL: with lims, batch row n's keys end at
 * lims[n], and a row with lims[n] == 0 or a query tile past lims[N] is written as zeros.
 * Replaces VoltaMmaPacked and VoltaMmaPackedTrim, cuda/volta_mma_attn.cu:544-623. */
CFLK_API int cflk_volta_mma_packed(void* stream, int dtype, const void* p, const void* bias,
                                   const uint8_t* kmask, const void* gate_bias,
                                   const int32_t* lims, void* out, int64_t X, int64_t Y,
                                   int64_t G, int64_t H, int64_t D, int64_t bias_elems,
                                   int64_t kmask_elems, int64_t gate_bias_elems, float scale,
                                   int64_t block_q, int64_t block_k, int column);

/* Bytes of device workspace cflk_volta_mma_bwd needs for these sizes: a float32 dQ accumulator,
 * the negated row statistics (-delta, -lse) and the bias transposed in its own 16-bit type
 * [H][Sk][Sq rounded up to 8] (the reference
 * takes its dQ accumulator and row statistic from XLA's ScratchAllocator,
 * cuda/volta_mma_attn_bwd.cu:346-361). */
CFLK_API int cflk_volta_mma_bwd_workspace_size(int64_t N, int64_t H, int64_t Sq, int64_t Sk,
                                               int64_t D, size_t* bytes);

/* VoltaMmaBwd: dq, dk, dv [as q, k, v] and dbias [H,Sq,Sk] float32 = dS summed over the batch
 * (unscaled). out and lse are the forward's; dout [N,H,Sq,D]. dbias is always zero-filled and
 * only accumulated when want_dbias is set. dk and dv are bitwise deterministic.
 * workspace: at least cflk_volta_mma_bwd_workspace_size bytes, 256-byte aligned.
 * Replaces VoltaMmaBwd, cuda/volta_mma_attn_bwd.cu:385-473. */
CFLK_API int cflk_volta_mma_bwd(void* stream, int dtype, const void* q, const void* k,
                                const void* v, const void* bias, const uint8_t* kmask,
                                const void* out, const void* dout, const float* lse, void* dq,
                                void* dk, void* dv, float* dbias, void* workspace,
                                size_t workspace_bytes, int64_t N, int64_t H, int64_t Sq,
                                int64_t Sk, int64_t D, float scale, int want_dbias);

/* VoltaMmaBwd for callers that cannot allocate device memory: the same computation and
 * arguments as cflk_volta_mma_bwd without the workspace. This entry point has no counterpart in
 * the reference; it exists for hosts that own every device allocation and give a kernel only its
 * inputs and outputs, and for code that must not call cudaMalloc (which may synchronise the
 * device). Its scratch is a static device array of cflk_volta_mma_bwd_noalloc_max_scratch()
 * bytes (32 MiB) that every GPU loading the library holds until exit; a problem needing more
 * (cflk_volta_mma_bwd_workspace_size) is rejected with CFLK_INVALID_ARGUMENT. The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress) for the current device,
 * so make that first call before any stream capture. All calls on a device share the array:
 * calls whose kernels overlap on the GPU race on it; calls ordered on one stream do not. Every
 * call writes the part of the array it uses before reading it (the float32 dQ accumulator is
 * stored by the first key tile or zeroed first), so nothing carries over from the previous call.
 * Nothing is allocated. */
CFLK_API size_t cflk_volta_mma_bwd_noalloc_max_scratch(void);
CFLK_API int cflk_volta_mma_bwd_noalloc(void* stream, int dtype, const void* q, const void* k,
                                        const void* v, const void* bias, const uint8_t* kmask,
                                        const void* out, const void* dout, const float* lse,
                                        void* dq, void* dk, void* dv, float* dbias, int64_t N,
                                        int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                        float scale, int want_dbias);

/* ---- gated attention training path (no counterpart in the reference) ------------------ */
/* The reference applies the gate of gated attention only in its forward-only packed targets;
 * for training it composes VoltaMma, an elementwise gate in XLA and VoltaMmaBwd
 * (cuda/volta_mma_attn.cu:544-575 for the gate's form). These two entry points fuse the gate.
 *
 * cflk_volta_mma_gated: y = attention(q, k, v, bias, kmask) * sigmoid(gate + gate_bias[h, c]),
 * with the log2-domain lse of the attention as cflk_volta_mma returns it (want_lse as there).
 * gate [N,H,Sq,D] (q's layout), gate_bias [H,D], both 16-bit; other arguments as cflk_volta_mma
 * (no tile hints). */
CFLK_API int cflk_volta_mma_gated(void* stream, int dtype, const void* q, const void* k,
                                  const void* v, const void* gate, const void* gate_bias,
                                  const void* bias, const uint8_t* kmask, void* out, float* lse,
                                  int64_t N, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                  float scale, int want_lse);

/* Workspace bytes of cflk_volta_mma_gated_bwd: that of cflk_volta_mma_bwd plus a 16-bit
 * [N,H,Sq,D] buffer for dy * sigmoid(gate + gate_bias). */
CFLK_API int cflk_volta_mma_gated_bwd_workspace_size(int64_t N, int64_t H, int64_t Sq,
                                                     int64_t Sk, int64_t D, size_t* bytes);

/* The gradients of cflk_volta_mma_gated: given y (its output), dy and lse, dq, dk, dv and dbias
 * as cflk_volta_mma_bwd gives them for the attention, dgate [N,H,Sq,D] (16-bit) =
 * dy * y * (1 - sigmoid(gate + gate_bias)) and dgate_bias [H,D] float32 = dgate summed over the
 * batch and the queries (accumulated with float atomics: like dq and dbias, equal run to run
 * within float rounding; dk and dv are bitwise deterministic). */
CFLK_API int cflk_volta_mma_gated_bwd(void* stream, int dtype, const void* q, const void* k,
                                      const void* v, const void* gate, const void* gate_bias,
                                      const void* bias, const uint8_t* kmask, const void* y,
                                      const void* dy, const float* lse, void* dq, void* dk,
                                      void* dv, void* dgate, float* dgate_bias, float* dbias,
                                      void* workspace, size_t workspace_bytes, int64_t N,
                                      int64_t H, int64_t Sq, int64_t Sk, int64_t D, float scale,
                                      int want_dbias);

/* ---- LayerNorm-folded pair-stack fusions ------------------------------------------------ */
/* keep [M] (16-bit) or NULL: per row tile, compute when a row of keep is above zero, write
 * padding (zeros, or nothing where the output aliases its input) when the tile is all zero,
 * nothing when it is all below zero (tile_work, cuda/volta_gdp.h:114-136). M == 0 launches
 * nothing. */

/* VoltaLnGdp: left, right [P/2, M] = the two halves of max(mask,0) * (y wp + bp) *
 * sigmoid(y wg + bg), channel major, y = LayerNorm(x). x [M,K]; scale, offset [K] float32;
 * wpT, wgT [P,K]; bp, bg [P]; mask [M] (also the keep, rows past M reading 0). K and P/2 in
 * {64, 128}. Replaces VoltaLnGdp, cuda/volta_fused_ffi.h:42-80,337-351. */
CFLK_API int cflk_volta_ln_gdp(void* stream, int dtype, const void* x, const float* scale,
                               const float* offset, const void* wpT, const void* bp,
                               const void* wgT, const void* bg, const void* mask, void* left,
                               void* right, int64_t M, int64_t K, int64_t P, float eps);

/* VoltaTrimulEpilogue: out [M,O] = (LN(x_cm^T) wo + bo) * sigmoid(LN_in(x) wg + bg), + x with
 * add_input (then O == CA, and out may alias x). x_cm [C,M] float32; x [M,CA]; in_scale,
 * in_offset [CA] and ln_scale, ln_offset [C] float32; woT [O,C], bo [O], wgT [O,CA], bg [O].
 * C, CA, O in {64, 128}. Replaces VoltaTrimulEpilogue, cuda/volta_fused_ffi.h:82-133,353-371. */
CFLK_API int cflk_volta_trimul_epilogue(void* stream, int dtype, const float* x_cm,
                                        const void* x, const float* in_scale,
                                        const float* in_offset, const float* ln_scale,
                                        const float* ln_offset, const void* woT, const void* bo,
                                        const void* wgT, const void* bg, const void* keep,
                                        void* out, int64_t M, int64_t C, int64_t CA, int64_t O,
                                        float eps, int add_input);

/* VoltaLnProj: p [M,n] = LN(x) w and bias [heads,M] = (LN(x) wb)^T. x [M,K]; scale, offset [K]
 * float32; wT [n,K]; wbT [heads,K]. K in {64, 128}, n a multiple of 64 (0: p untouched),
 * heads <= 8 (0: bias untouched). Replaces VoltaLnProj, cuda/volta_fused_ffi.h:135-176,373-388. */
CFLK_API int cflk_volta_ln_proj(void* stream, int dtype, const void* x, const float* scale,
                                const float* offset, const void* wT, const void* wbT,
                                const void* keep, void* p, void* bias, int64_t M, int64_t K,
                                int64_t n, int64_t heads, float eps);

/* VoltaOutProj: out [M,N] = o w + b, + residual when residual is not NULL (out may alias it).
 * o [M,K]; wT [N,K]; b [N]. K, N in {64, 128}.
 * Replaces VoltaOutProj, cuda/volta_fused_ffi.h:178-214,390-401. */
CFLK_API int cflk_volta_out_proj(void* stream, int dtype, const void* o, const void* wT,
                                 const void* b, const void* residual, const void* keep,
                                 void* out, int64_t M, int64_t K, int64_t N);

/* VoltaTransition: out [M,C] = relu(LN(x) w1 + b1) w2 + b2, + x with add_input (out may alias
 * x). x [M,C]; scale, offset [C] float32; w1T [H,C]; b1 [H]; w2T = w2 [H,C] as [H/64][C][64]
 * chunks, each transposed; b2 [C]. C in {64, 128, 256}, H in {2C, 4C}.
 * Replaces VoltaTransition, cuda/volta_fused_ffi.h:216-259,403-418. */
CFLK_API int cflk_volta_transition(void* stream, int dtype, const void* x, const float* scale,
                                   const float* offset, const void* w1T, const void* b1,
                                   const void* w2T, const void* b2, const void* keep, void* out,
                                   int64_t M, int64_t C, int64_t H, float eps, int add_input);

/* VoltaLayerNorm: out [M,C] = (x - mean) * rsqrt(var + eps) * scale + offset over the last
 * axis, the statistics in float32 in one pass (var = max(E[x^2] - mean^2, 0)). x, out [M,C]
 * (out may alias x); scale, offset [C] float32; any C >= 1 (vector path when C / 8 is a power of
 * two up to 32 and the buffers are 16-byte aligned). Replaces VoltaLayerNorm,
 * cuda/volta_ops.cu:27-91. */
CFLK_API int cflk_volta_layer_norm(void* stream, int dtype, const void* x, const float* scale,
                                   const float* offset, void* out, int64_t M, int64_t C,
                                   float eps);

/* VoltaGdp: out [M,N] = mask * (x wp + bp) * act(x wg + bg), act = sigmoid (activation 0) or
 * swish g * sigmoid(g) (1), the row mask unclamped. x [M,K]; wp, wg [K,N] row-major; bp, bg
 * [N]; mask [M]. Any K >= 1 and N % 8 == 0, as the reference: K and N of 64 or 128 run the
 * resident-weight row-tile kernel, other widths the persistent tcgen05 tile GEMM with both
 * products in one pass (K % 8 == 0) or, for K % 8 != 0, a CUDA-core tile kernel. x, wp, wg and
 * out 16-byte aligned. Replaces VoltaGdp, cuda/volta_ops.cu:108-205,212-265. */
CFLK_API int cflk_volta_gdp(void* stream, int dtype, const void* x, const void* wp,
                            const void* bp, const void* wg, const void* bg, const void* mask,
                            void* out, int64_t M, int64_t K, int64_t N, int64_t activation);

/* VoltaOpmUpdate: out [B,D,F] = (lhs @ t[:, d, :] + bias) / (eps + norm[b, d]) (+ residual when
 * residual is not NULL). lhs [B,K] and t [K,D,F] 16-bit, bias [F] and norm [B,D] float32,
 * residual and out [B,D,F] 16-bit (out may be the residual's buffer). K a multiple of 32, F 16, 32, 64 or 128, D at most 65535 (the
 * reference's limits); lhs, t, residual and out 16-byte aligned. One persistent tcgen05 tile GEMM
 * (128 x 128 output tiles, the epilogue fused). Replaces VoltaOpmUpdate,
 * cuda/volta_fused_ffi.h:261-298, kernel cuda/volta_ops.cu:647-699. */
CFLK_API int cflk_volta_opm_update(void* stream, int dtype, const void* lhs, const void* t,
                                   const float* bias, const float* norm, const void* residual,
                                   void* out, int64_t B, int64_t K, int64_t D, int64_t F,
                                   float eps);

/* VoltaOpmOuter on 16 MSA rows: out [B,D,F] = sum over c, e of h(sum_a left[a,b,c] right[a,d,e])
 * wT[f, c*E + e], h the rounding of the float32 inner product to the 16-bit type (AF2's order).
 * left [16,B,C], right [16,D,E], wT [F,C*E], out [B,D,F], all 16-bit. The reference's limits: C a
 * multiple of 16, E 32, D a multiple of 4 with D/4 at most 65535, F 16, 32, 64 or 128. At
 * AF2's C = 32 one fused kernel: per 16 b x 16 d tile and chunk of 8 c x 8 e, a tcgen05 MMA of
 * the outer products into tensor memory, rounded by a converter warpgroup into shared memory as
 * the A operand of the MMAs against wT laid out chunk by chunk in the workspace (F * 2 KB;
 * the size function gives 256 KB, enough for any F). Other C: two persistent
 * tile GEMMs per chunk of b, the outer products (K = 16, rounded, written as G2 [b][d][c][e]
 * into the workspace; a CUDA-core kernel when C does not divide 128) and G2 [b*D, C*E] times
 * wT; the workspace holds one chunk of G2 (whole multiples of 128/C rows of b, about 64 MB):
 * cflk_volta_opm_outer_workspace_size gives the recommended size; a smaller workspace (at least
 * one chunk of 128/C rows) runs more chunks. Buffers 16-byte aligned. Replaces VoltaOpmOuter,
 * cuda/volta_fused_ffi.h:300-335, kernel cuda/volta_ops.cu:710-787 (whose handler takes no
 * scratch: an FFI shim takes the workspace from XLA's scratch allocator). */
CFLK_API int cflk_volta_opm_outer_workspace_size(int64_t B, int64_t C, int64_t D, int64_t E,
                                                 size_t* bytes);
CFLK_API int cflk_volta_opm_outer(void* stream, int dtype, const void* left, const void* right,
                                  const void* wT, void* out, int64_t B, int64_t C, int64_t D,
                                  int64_t E, int64_t F, void* workspace, size_t ws_bytes);

/* The triangle multiplication's contraction between VoltaLnGdp and VoltaTrimulEpilogue (in the
 * reference an XLA einsum with a float32 result, tests/test_fused.py:135): for each channel c,
 *   incoming = 0 (AF2's outgoing edges): out[c,i,j] = sum_k a[c,i,k] b[c,j,k], a [C,I,K], b [C,J,K];
 *   incoming = 1 (incoming edges):       out[c,i,j] = sum_k a[c,k,i] b[c,k,j], a [C,K,I], b [C,K,J]
 * (AF2's incoming form passes its right projection as a and its left as b). a and b 16-bit
 * (the channel-major left/right that VoltaLnGdp writes), out [C,I,J] float32 (the x_cm that
 * VoltaTrimulEpilogue reads). Products accumulate in float32. The persistent tcgen05 tile GEMM
 * (128 x 128 tiles of one channel, K- or MN-major operands through TMA) runs when the rows are
 * 16-byte multiples (K % 8 == 0, or I % 8 == 0 and J % 8 == 0 for incoming; J % 4 == 0) and the
 * buffers 16-byte aligned; other sizes run a CUDA-core tile kernel. C at most 65535. No reference
 * kernel: the reference's callers run this einsum in XLA. */
CFLK_API int cflk_trimul_contract(void* stream, int dtype, const void* a, const void* b,
                                  float* out, int64_t C, int64_t I, int64_t J, int64_t K,
                                  int incoming);

/* ---- diagnostics (no counterpart in the reference) ------------------------------------- */

/* Evaluates, for n float32 inputs x on the device, the FMA-pipe exponential 2^x that the attention
 * kernels compute for part of their softmax (into fma_out) and the hardware ex2.approx (into
 * mufu_out), so that a test can bound its error. */
CFLK_API int cflk_diag_ex2_fma(void* stream, const float* x, float* fma_out, float* mufu_out,
                               int64_t n);

/* Runs one CTA that waits on an mbarrier nothing arrives on, for at most limit_ns (0 < limit_ns
 * <= 2 s), the bounded wait every pipeline of the library uses. The wait gives up, ORs the code 4
 * into *status and writes the nanoseconds it waited into *elapsed_ns (device pointers). */
CFLK_API int cflk_diag_bounded_wait(void* stream, uint64_t limit_ns, unsigned* status,
                                    unsigned long long* elapsed_ns);

#ifdef __cplusplus
}
#endif

#endif /* CFLK_B200_H */

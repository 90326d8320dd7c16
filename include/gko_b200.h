/*
 * gko_b200.h — C ABI of the B200 (sm_100a) fused-operator library.
 *
 * One shared library, libgko_b200.so, exports the entry points below. They take
 * plain device pointers, sizes and element strides (never framework types),
 * launch on the given CUDA stream (NULL = legacy default stream) and return
 * GKO_OK or an error code; gko_last_error() then holds a message naming the
 * violated constraint. Nothing here falls back to another implementation: an
 * input the kernels do not support is rejected.
 *
 * Every kernel bounds each of its internal waits. If one expires, the kernel
 * ORs a GKO_STATUS_* bit into *status (a caller-owned device word; may be NULL),
 * drains its own tensor-core work, frees its tensor memory and returns, so the
 * CUDA context stays usable. The host reads the word after synchronising.
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the EvoCompile repository).
 */
#ifndef GKO_B200_H
#define GKO_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define GKO_F16 1
#define GKO_BF16 2
#define GKO_F32 3

/* GEMM epilogue activations */
#define GKO_ACT_NONE 0
#define GKO_ACT_GELU 1 /* exact erf GELU: 0.5 x (1 + erf(x / sqrt 2)) */
#define GKO_ACT_RELU 2

/* attention bias layouts */
#define GKO_BIAS_NONE 0
#define GKO_BIAS_KEYPAD 1 /* additive [z, sk] row per batch (key padding) */
#define GKO_BIAS_FULL 2   /* additive [z, h, sq, sk] with broadcast (stride 0) allowed */

/* return codes */
#define GKO_OK 0
#define GKO_ERR_INVALID 1     /* bad sizes, strides, pointers */
#define GKO_ERR_UNSUPPORTED 2 /* valid input outside what the kernels implement */
#define GKO_ERR_CUDA 3        /* CUDA runtime / driver error */

/* status-word bits written by kernels */
#define GKO_STATUS_TIMEOUT_PRODUCER 0x1u
#define GKO_STATUS_TIMEOUT_MMA 0x2u
#define GKO_STATUS_TIMEOUT_EPILOGUE 0x4u
#define GKO_STATUS_TIMEOUT_SOFTMAX 0x8u
#define GKO_STATUS_TIMEOUT_DRAIN 0x10u

/* Message for the last error returned on this host thread ("" if none). */
const char* gko_last_error(void);

/* Library ABI version (major * 100 + minor). */
int gko_version(void);

/*
 * D[m, n] = act(sum_k A[m, k] * B[k, n] + bias[n])
 *
 * Replaces ext.addmm_epilogue(bias, mat1, mat2, act)
 * (eval/kernels/cutlass_fmha/gko_cutlass_attn.cu:552-586, binding :588-591) and the
 * Triton launch _triton_addmm_gelu (eval/kernels/addmm_gelu.py:87-118) behind
 * gko::addmm_gelu (eval/kernels/addmm_gelu.py:192-223).
 *
 * A (mat1) is [m, k] with element strides (a_sm, a_sk); B (mat2) is the
 * logical [k, n] operand with strides (b_sk, b_sn) — a transposed weight view
 * (b_sk == 1) is read in place. bias is NULL or a length-n vector of
 * bias_dtype. D is [m, n] with row stride ldd, same dtype as A.
 * f16/bf16 run on tcgen05 tensor cores (f32 accumulate) and need
 * a_sk == 1 and (b_sk == 1 or b_sn == 1), 16-byte aligned bases and row
 * strides that are multiples of 8 elements. With act == GKO_ACT_NONE, A may
 * also be a transposed view (a_sm == 1, a_sk a multiple of 8): the weight
 * gradient dW = dZ^T X of a Linear, read in place as an MN-major operand.
 * f32 runs exact fp32 FMA on any strides.
 */
int gko_addmm_act(int dtype, int act, int64_t m, int64_t n, int64_t k, const void* a, int64_t a_sm,
                  int64_t a_sk, const void* b, int64_t b_sk, int64_t b_sn, const void* bias,
                  int bias_dtype, void* d, int64_t ldd, unsigned int* status, void* stream);

/*
 * out[m, h] = silu(sum_k x[m, k] Wg[h, k]) * (sum_k x[m, k] Wu[h, k]),  W = [Wg; Wu] is [2h, k]
 *
 * Replaces ext.linear_swiglu(x, weight)
 * (eval/kernels/cutlass_fmha/gko_cutlass_swiglu.cu:287-326, binding :330-335) and the
 * Triton launch _triton_gemm_swiglu (eval/kernels/gemm_swiglu.py:112-144) behind
 * gko::gemm_swiglu (eval/kernels/gemm_swiglu.py:147-169,208-232). One kernel: the
 * [m, 2h] gate/up intermediate never reaches memory.
 *
 * x is [m, k] with strides (x_sm, x_sk); W is [2h, k] with strides (w_sn, w_sk)
 * (w_sk == 1 is the F.linear layout; w_sn == 1 is read as a transposed view).
 * out is [m, h] with row stride ldo, same dtype as x.
 */
int gko_linear_swiglu(int dtype, int64_t m, int64_t h, int64_t k, const void* x, int64_t x_sm,
                      int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, void* out,
                      int64_t ldo, unsigned int* status, void* stream);

/*
 * Fused multi-head attention forward (dense batch).
 *   out = softmax(mask(softcap(scale * Q K^T + bias))) V,  lse = m + ln(l) per row
 *
 * Replaces ext.fmha_fwd(q, k, v, bias, scale, causal, window, softcap)
 * (eval/kernels/cutlass_fmha/gko_cutlass_attn.cu:371-461, binding :588) and the
 * Triton launch _triton_fwd (eval/kernels/fused_sdpa.py:614-665) behind
 * gko::fused_sdpa_pair / gko::cutlass_fmha_pair (eval/kernels/fused_sdpa.py:912-943,
 * eval/kernels/cutlass_gemm_attn.py:81-121).
 *
 * q is logical [z, hq, sq, d], k and v are [z, hkv, sk, d] (hq % hkv == 0:
 * grouped-query heads h use kv head h / (hq / hkv)). *_strides give element
 * strides for (z, h, s, d); the d stride must be 1, the others multiples of 8,
 * so [z, s, h, d] storage viewed as [z, h, s, d] is read in place.
 * bias: GKO_BIAS_NONE, GKO_BIAS_KEYPAD (bias_strides[0] = z stride,
 * bias_strides[3] = key stride) or GKO_BIAS_FULL (strides for z, h, q, key;
 * 0 broadcasts). The bias holds bias_batch batches (dividing z); batch b of
 * q reads bias batch b % bias_batch (a shifted-window mask [nW, h, sq, sk]). causal keeps key <= query (top-left aligned); window > 0 keeps
 * |key - query| <= window; softcap > 0 applies softcap * tanh(x / softcap)
 * (x clamped to +-15 softcap first). Masked scores never contribute; a row
 * with every key masked yields zeros and lse = -inf.
 * out is [z, hq, sq, d] (same dtype as q): contiguous when out_strides is NULL,
 * else with element strides out_strides (z, h, s, d; d stride 1, others
 * multiples of 8 — e.g. [z, s, h, d] storage for a following projection).
 * lse is f32 [z * hq, sq].
 * dtype: GKO_F16 or GKO_BF16; d in {64, 128}.
 */
int gko_fmha_fwd(int dtype, int64_t z, int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int64_t d,
                 const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                 const void* v, const int64_t* v_strides, const void* bias, int bias_mode,
                 int bias_dtype, const int64_t* bias_strides, int64_t bias_batch,
                 const int64_t* out_strides, float scale, int causal, int window, float softcap,
                 void* out, float* lse, unsigned int* status, void* stream);

/*
 * Fused multi-head attention forward over packed variable-length sequences.
 *
 * New entry point (no reference counterpart: the reference's attention takes
 * only dense [z, h, s, d] batches, eval/kernels/fused_sdpa.py:535-543); it
 * backs gko::fmha_varlen_fwd. Sequence i owns query rows
 * [cu_seqlens_q[i], cu_seqlens_q[i+1]) and key rows [cu_seqlens_k[i], cu_seqlens_k[i+1]).
 * q is [tq, hq, d], k and v are [tk, hkv, d], with element strides (token, head)
 * (d stride 1). cu_seqlens_* are device int32 arrays of b + 1 entries;
 * max_seqlen_q bounds every query length. out is contiguous [tq, hq, d],
 * lse is f32 [hq, tq]. Masks and GQA as for gko_fmha_fwd (no bias).
 */
int gko_fmha_varlen_fwd(int dtype, int64_t b, int64_t hq, int64_t hkv, int64_t d, int64_t tq,
                        int64_t tk, int64_t max_seqlen_q, const void* q, int64_t q_st,
                        int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh, const void* v,
                        int64_t v_st, int64_t v_sh, const int32_t* cu_seqlens_q,
                        const int32_t* cu_seqlens_k, float scale, int causal, int window,
                        float softcap, void* out, float* lse, unsigned int* status, void* stream);

/*
 * Bytes of device workspace gko_fmha_bwd (varlen = 0: batch z, per-batch query
 * length sq_or_tq) or gko_fmha_varlen_bwd (varlen = 1: batch = sequences, sq_or_tq =
 * total query tokens) needs for head dim d; -1 for invalid sizes. The workspace holds
 * the fp32 dq accumulator and two f32 per query row.
 */
int64_t gko_fmha_bwd_workspace_size(int64_t batch, int64_t hq, int64_t sq_or_tq, int64_t d, int varlen);

/*
 * Fused multi-head attention backward: dq, dk, dv of gko_fmha_fwd's function.
 *
 * Replaces the Triton launches of _triton_bwd (eval/kernels/fused_sdpa.py:668-770:
 * _flash_bwd_pre, _flash_bwd_dq, _flash_bwd_dkdv at :159-496) behind
 * gko::fused_sdpa_bwd (eval/kernels/fused_sdpa.py:945-967). Arguments as for
 * gko_fmha_fwd, plus the forward output `out`, its lse (f32 [z * hq, sq]) and
 * dout, each [z, h, s, d] with element strides (d stride 1, others multiples of 8).
 * dq [z, hq, sq, d], dk and dv [z, hkv, sk, d] are written (any strides of the same
 * rules); with GQA dk/dv sum over each kv head's query group. `workspace` is
 * device memory of at least gko_fmha_bwd_workspace_size(z, hq, sq, d, 0) bytes,
 * 16-byte aligned; the call overwrites it. Three kernels on `stream`.
 */
int gko_fmha_bwd(int dtype, int64_t z, int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int64_t d,
                 const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                 const void* v, const int64_t* v_strides, const void* bias, int bias_mode,
                 int bias_dtype, const int64_t* bias_strides, int64_t bias_batch, const void* out,
                 const int64_t* out_strides, const void* dout, const int64_t* dout_strides,
                 const float* lse, float scale, int causal, int window, float softcap, void* dq,
                 const int64_t* dq_strides, void* dk, const int64_t* dk_strides, void* dv,
                 const int64_t* dv_strides, void* workspace, int64_t workspace_bytes,
                 unsigned int* status, void* stream);

/*
 * gko_fmha_bwd for callers that cannot allocate device memory: no workspace
 * argument, and no cudaMalloc / cudaFree or other allocating call inside.
 *
 * No counterpart in the reference. It exists for callers that cannot supply
 * gko_fmha_bwd's workspace: a host program whose device memory is reserved by
 * another runtime's pool, or code that must not pay the implicit device-wide
 * synchronisation of cudaMalloc / cudaFree, or a plain C caller with no allocator
 * of its own. The workspace comes instead from a fixed 32 MiB array in the
 * library's device image, which every GPU that loads the library holds until the
 * process exits. Limit: gko_fmha_bwd_workspace_size(z, hq, sq, d, 0) <= 32 MiB,
 * i.e. z * hq * ceil(sq / 64) <= 1008 blocks at d = 128 (1985 at d = 64); larger
 * problems are rejected with GKO_ERR_UNSUPPORTED. The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress), so make that first
 * call before any stream capture. All calls share the one array (each call clears
 * the parts it uses): calls that overlap on the GPU, on any stream, race and give
 * wrong results. Arguments and results as for gko_fmha_bwd.
 */
int gko_fmha_bwd_noalloc(int dtype, int64_t z, int64_t hq, int64_t hkv, int64_t sq, int64_t sk,
                         int64_t d, const void* q, const int64_t* q_strides, const void* k,
                         const int64_t* k_strides, const void* v, const int64_t* v_strides,
                         const void* bias, int bias_mode, int bias_dtype,
                         const int64_t* bias_strides, int64_t bias_batch, const void* out,
                         const int64_t* out_strides, const void* dout, const int64_t* dout_strides,
                         const float* lse, float scale, int causal, int window, float softcap,
                         void* dq, const int64_t* dq_strides, void* dk, const int64_t* dk_strides,
                         void* dv, const int64_t* dv_strides, unsigned int* status, void* stream);

/*
 * Backward of gko_fmha_varlen_fwd (no reference counterpart, like the forward).
 * Packed tensors [tokens, heads, d] with element strides (token, head): q, out, dout,
 * dq over tq query tokens and hq heads; k, v, dk, dv over tk key tokens and hkv heads.
 * lse is f32 [hq, tq]; max_seqlen_q / max_seqlen_k bound the sequence lengths.
 * workspace: gko_fmha_bwd_workspace_size(b, hq, tq, d, 1) bytes.
 */
int gko_fmha_varlen_bwd(int dtype, int64_t b, int64_t hq, int64_t hkv, int64_t d, int64_t tq,
                        int64_t tk, int64_t max_seqlen_q, int64_t max_seqlen_k, const void* q,
                        int64_t q_st, int64_t q_sh, const void* k, int64_t k_st, int64_t k_sh,
                        const void* v, int64_t v_st, int64_t v_sh, const void* out, int64_t o_st,
                        int64_t o_sh, const void* dout, int64_t do_st, int64_t do_sh,
                        const float* lse, const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                        float scale, int causal, int window, float softcap, void* dq,
                        int64_t dq_st, int64_t dq_sh, void* dk, int64_t dk_st, int64_t dk_sh,
                        void* dv, int64_t dv_st, int64_t dv_sh, void* workspace,
                        int64_t workspace_bytes, unsigned int* status, void* stream);

/*
 * Training forms of gko_addmm_act and gko_linear_swiglu that also write what the backward
 * needs, so it recomputes no GEMM (the reference backward re-runs the forward GEMM,
 * eval/kernels/addmm_gelu.py:175-185, eval/kernels/gemm_swiglu.py:177-200).
 * gko_addmm_act_aux: as gko_addmm_act, plus z[m, n] (row stride ldz) = the pre-activation
 * mat1 @ mat2 + bias. gko_linear_swiglu_aux: as gko_linear_swiglu, plus gate_up[m, 2h]
 * (row stride ldg) = [x Wg^T | x Wu^T]. bf16 / f16 only (tensor-core path).
 */
int gko_addmm_act_aux(int dtype, int act, int64_t m, int64_t n, int64_t k, const void* a, int64_t a_sm,
                      int64_t a_sk, const void* b, int64_t b_sk, int64_t b_sn, const void* bias,
                      int bias_dtype, void* d, int64_t ldd, void* z, int64_t ldz, unsigned int* status,
                      void* stream);
int gko_linear_swiglu_aux(int dtype, int64_t m, int64_t h, int64_t k, const void* x, int64_t x_sm,
                          int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, void* out,
                          int64_t ldo, void* gate_up, int64_t ldg, unsigned int* status, void* stream);

/*
 * out[m, n] = x[m, k] @ w[n, k]^T + resid[m, n]: a linear layer with the residual add fused into
 * its epilogue (one rounding to the output dtype). out may be resid (in place). Row-major x and w;
 * row strides x_sm, resid_sm, ldo in elements (multiples of 8, 16-byte aligned bases); bf16 / f16.
 * No reference counterpart. The reference's MLP rewrite ends in a plain projection
 * (eval/rewrites/simple_gpt_silu_mul.py:18, c_proj) whose output the enclosing transformer block
 * adds to its residual stream in a separate elementwise op; this entry does both in one kernel
 * (used by the tensor-parallel block's down projection on one rank).
 */
int gko_linear_residual(int dtype, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm, int64_t x_sk,
                        const void* w, int64_t w_sn, int64_t w_sk, const void* resid, int64_t resid_sm, void* out,
                        int64_t ldo, unsigned int* status, void* stream);

/*
 * SwiGLU backward from the saved pre-activations: with s = sigmoid(g) and dy[rows, h],
 * d_gate_up[:, :h] = dy u s (1 + g (1 - s)) and d_gate_up[:, h:] = dy g s, where
 * gate_up = [g | u] is [rows, 2h]. Row strides in elements; bf16 / f16; h and strides
 * multiples of 8. Replaces the elementwise part of the reference backward
 * (eval/kernels/gemm_swiglu.py:177-200).
 */
int gko_swiglu_bwd(int dtype, int64_t rows, int64_t h, const void* dy, int64_t ld_dy, const void* gate_up,
                   int64_t ld_gu, void* d_gate_up, int64_t ld_dgu, unsigned int* status, void* stream);

/*
 * Row-parallel linear with the tensor-parallel all-reduce inside the GEMM:
 * out_r += x @ w^T on every rank r of the group, where x is this rank's [m, k] input
 * slice (row stride x_sm, x_sk == 1) and w its [n, k] weight slice (row stride w_sn,
 * w_sk == 1). The epilogue adds each finished bf16/f16 output chunk into every rank's out
 * (row stride ldo): through `out_multicast`, an NVLink multicast address bound to all
 * ranks' out buffers (one in-switch reduction), or, when that is NULL, through
 * `out_peers`, a device array of the `world` ranks' mapped out pointers (one reduction
 * per rank). Every rank's out must be zero before any rank starts and the caller waits
 * for all ranks to finish before reading (group barriers around the call).
 *
 * No reference counterpart (the reference has no tensor-parallel path); it replaces the
 * GEMM + NCCL all-reduce pair of the Llama-3-70B block's o- and down-projections.
 */
int gko_linear_allreduce(int dtype, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm,
                         int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, void* out,
                         int64_t ldo, void* out_multicast, void* const* out_peers, int world,
                         unsigned int* status, void* stream);

/*
 * out[i] = silu(x[i]) * y[i] over n contiguous elements (dtype f16, bf16 or f32).
 *
 * Replaces the Triton launch _triton (eval/kernels/silu_mul.py:33-43) behind
 * gko::silu_mul (eval/kernels/silu_mul.py:66-88). Buffers 16-byte aligned.
 */
int gko_silu_mul(int dtype, int64_t n, const void* x, const void* y, void* out,
                 unsigned int* status, void* stream);

/*
 * RMSNorm folded into the following GEMM. gko_rms_stats writes inv[row] = 1 / sqrt(mean(v^2) + eps)
 * of v = x + residual (residual may be NULL; sum_out, when not NULL, receives v) and nothing
 * else; gko_linear_rowscale then computes out = (inv[row] * (x @ w^T)) with the RMSNorm weight
 * folded into w beforehand (w'[n, j] = w[n, j] * g[j]), which equals rmsnorm(x) * g @ w^T. With
 * swiglu != 0, w is [2n, k] = [Wg; Wu] and out[m, n] = silu(inv x Wg^T) * (inv x Wu^T). Row-major
 * x and w, bf16 / f16, strides in elements (multiples of 8), inv fp32 on the device.
 *
 * No reference counterpart: the block's RMSNorm prologue (the reference has no transformer block
 * on its kernel path); this skips writing the normalised activations to HBM.
 */
int gko_rms_stats(int dtype, int64_t rows, int64_t cols, const void* x, const void* residual, float eps,
                  void* sum_out, float* inv_out, int64_t ld, unsigned int* status, void* stream);
int gko_linear_rowscale(int dtype, int swiglu, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm,
                        int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, const float* row_scale, void* out,
                        int64_t ldo, unsigned int* status, void* stream);

/*
 * gko_linear_rowscale (swiglu = 0) whose epilogue also applies rotate-half RoPE to output columns
 * [0, rope_cols): heads of 128 columns, pair (i, i + 64) of a head at row r rotated by the angle
 * (r % seq_len) * theta^(-2i/128), computed on the fp32 accumulator before the one rounding to
 * bf16 / f16. The QKV projection of a Llama block (q heads, then k heads, then v heads) passes
 * rope_cols = (q heads + k heads) * 128 and writes q and k already rotated.
 *
 * No reference counterpart (the block's RoPE; the reference has no transformer block on its kernel
 * path): it replaces the block's separate in-place gko_rope launch over the q and k heads.
 */
int gko_linear_rowscale_rope(int dtype, int64_t m, int64_t n, int64_t k, const void* x, int64_t x_sm,
                             int64_t x_sk, const void* w, int64_t w_sn, int64_t w_sk, const float* row_scale,
                             void* out, int64_t ldo, int64_t rope_cols, int64_t seq_len, float theta,
                             unsigned int* status, void* stream);

/*
 * Caps the CTAs a tensor-core GEMM launch occupies at `ctas` SMs (0: every SM, the default) for
 * every GEMM launched after the call, from any host thread. Returns the previous cap, or -1
 * (with gko_last_error set) when ctas < 0. The persistent
 * GEMM otherwise holds every SM, so a collective launched on another stream (the tensor-parallel
 * block's NCCL all-reduce of one token chunk while the next chunk's GEMMs run) would wait for it.
 *
 * No reference counterpart (the reference has no tensor parallelism).
 */
int gko_set_gemm_ctas(int ctas);

/*
 * Row-slice all-reduce of a tensor-parallel row-parallel projection over NVLink multicast, fused
 * with the residual add and the RMSNorm statistics that follow it. Every rank has written its
 * partial [rows, cols] (row stride ld) into its copy of a symmetric buffer whose multicast address
 * is partial_mc, and the group has passed a barrier. This rank then sums rows [row0, row1) over the
 * ranks (multimem.ld_reduce, fp32 accumulation in the switch), adds resid (local, same row stride;
 * NULL: none), and writes the rounded rows to every rank's copy of the output buffer (out_mc) and,
 * when inv_mc is not NULL, 1 / sqrt(mean(v^2) + eps) of each row to every rank's fp32 [rows]
 * buffer. A barrier after the call completes the all-reduce on every rank. bf16 / f16, cols and
 * ld multiples of 8, cols <= 16384.
 *
 * No reference counterpart (the reference has no tensor parallelism): it replaces the NCCL
 * all-reduce after the block's o- and down projections, and the residual / statistics pass.
 */
int gko_allreduce_residual_nvls(int dtype, int64_t rows, int64_t cols, int64_t ld, int64_t row0, int64_t row1,
                                const void* partial_mc, const void* resid, void* out_mc, void* inv_mc, float eps,
                                unsigned int* status, void* stream);

/*
 * y = rmsnorm(x + residual) * weight over rows of `cols` elements (row stride ld),
 * rmsnorm(v) = v / sqrt(mean(v^2) + eps). residual may be NULL; when sum_out is
 * not NULL it receives x + residual (the updated residual stream). bf16/f16,
 * cols <= 16384, cols and ld multiples of 8.
 *
 * No reference counterpart: the RMSNorm of the Llama-3-70B block configuration
 * (the reference has no transformer block on its kernel path).
 */
int gko_rmsnorm(int dtype, int64_t rows, int64_t cols, const void* x, const void* residual,
                const void* weight, float eps, void* out, void* sum_out, int64_t ld,
                unsigned int* status, void* stream);

/*
 * Rotary position embedding, applied in place to `heads` heads of head_dim
 * elements for each of `tokens` tokens (element strides st_token, st_head),
 * rotate-half convention: for i < head_dim/2 and f_i = theta^(-2i/head_dim),
 * (x_i, x_{i+D/2}) <- (x_i cos(p f_i) - x_{i+D/2} sin(p f_i), x_{i+D/2} cos(p f_i) + x_i sin(p f_i)).
 * The position p of token t is positions[t] (device int32) or, when positions
 * is NULL, t % seq_len.
 *
 * No reference counterpart: the RoPE of the Llama-3-70B block configuration.
 */
int gko_rope(int dtype, int64_t tokens, int64_t heads, int64_t head_dim, void* x, int64_t st_token,
             int64_t st_head, const int32_t* positions, int64_t seq_len, float theta,
             unsigned int* status, void* stream);

/*
 * Self-test of the failure path (no reference counterpart): launches one CTA
 * that waits, through the operators' bounded wait, on a barrier nothing
 * arrives on; after limit_ns (<= 2 s) it ORs GKO_STATUS_TIMEOUT_PRODUCER into
 * *status and returns. Used by the tests to show that a stalled wait ends with
 * a status bit instead of a hang.
 */
int gko_selftest_wait_timeout(unsigned int* status, long long limit_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GKO_B200_H */

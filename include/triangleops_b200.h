/*
 * triangleops_b200.h — C ABI of libtriangleops_b200.so, the B200 (sm_100a)
 * implementation of TriangleOps' three Pairformer primitives.
 *
 * Conventions
 *   - Every pointer is a device pointer (16-byte aligned) unless noted; every
 *     launch goes on `stream` (a cudaStream_t passed as void*), asynchronously.
 *   - The library never allocates device memory: intermediates are caller-owned
 *     workspaces whose shapes are given below (elements of the IO dtype unless
 *     marked fp32). Np = N rounded up to a multiple of 8.
 *   - dtype: TOPS_F16 (0) or TOPS_BF16 (1) for the tensor-core paths.
 *   - Return value: TOPS_OK (0) or a negative status (status.h):
 *       TOPS_ERR_SHAPE  -1  shape mismatch            (reference: AssertionError)
 *       TOPS_ERR_DTYPE  -2  unsupported IO dtype      (reference: ValueError, _common/dtype.py:19)
 *       TOPS_ERR_ARG    -3  bad enum, e.g. direction  (reference: ValueError, triangle_mul/module.py:76)
 *       TOPS_ERR_ALIGN  -4  misaligned pointer/stride
 *       TOPS_ERR_TMAP   -5  TMA tensor-map encode failed
 *       TOPS_ERR_CUDA   -6  CUDA launch error
 *       TOPS_ERR_TIMEOUT -7 a bounded device-side wait gave up (see tops_device_error)
 *       TOPS_ERR_CAPACITY -8 size beyond a fixed-capacity entry point
 *   - Weights are "K-major rows": a projection y = x W (matmul convention) is passed
 *     as W^T, i.e. (out, in) row-major, the nn.Linear layout.
 *
 * Reference citations are paths inside youngchan2/TriangleOps.
 */
#ifndef TRIANGLEOPS_B200_H
#define TRIANGLEOPS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TOPS_F16 0
#define TOPS_BF16 1
#define TOPS_F32 2

/* Library version (100 = 0.1.0; reference triangle_ops/__init__.py:22). */
int tops_version(void);
/* Human-readable text of a status code. */
const char* tops_status_string(int code);
/* Synchronises `stream`, returns TOPS_ERR_TIMEOUT (and the wait-site id in *site)
 * if any device-side bounded wait gave up since the last call, then clears it. */
int tops_device_error(void* stream, int* site);

/* Single-tile check of one tcgen05 operand mode (0..3) against the host:
 * d (fp32) = A B^T in the layout of that mode. Library self-test. */
int tops_selftest_umma(int mode, const void* a, const void* b, float* d, void* stream);
/* 2^x of n f16 values (x_f16) by the two paths of the attention softmax: the FMA-pipe
 * polynomial (poly_f16) and the MUFU ex2.approx.f16x2 (mufu_f16). Library self-test;
 * no counterpart in the reference (whose Triton kernels use exp2 in fp32). */
int tops_selftest_ex2(const void* x_f16, void* poly_f16, void* mufu_f16, int64_t n, void* stream);

/* ---------------------------------------------------------------------------
 * triangle attention (starting node)
 * Replaces triangle_attn/kernel.py:256-374 (triangle_attn_forward: bias_proj_kernel
 * + triangle_attn_kernel) and, with apply_ln=1, the F.layer_norm of
 * triangle_attn/module.py:73-79.
 *   x        [N][N][C]          raw x (apply_ln=1) or x~ = LN(x) (apply_ln=0)
 *   ln_w/b   [C] fp32           LayerNorm affine (apply_ln=1)
 *   w_qkvz   [3C+16][C]         rows WQ^T | WK^T | WV^T | W_proj_z^T (H rows) | zero
 *   bz       [H] fp32           bias-projection bias
 *   mask     [N][N] uint8 or NULL (0 = masked key, per row; broadcast over heads/queries)
 *   xln_ws   [N*N][C]           receives x~ (apply_ln=1; else may be NULL)
 *   q_ws,k_ws [N][H][N][D] f16, vt_ws [N][H][D][Np] f16, maskf_ws [N][Np] f16, bias_ws [H][N][Np] f16
 *   o_out    [N][N][H*D]        attention output (pre-gate)
 * Supported (C,H,D): (128,4,32), (64,4,16). Rows whose key mask is all zero
 * produce non-finite values (the Python layer patches them to the reference's
 * uniform-softmax result). */
int tops_triangle_attn_forward(int dtype, int64_t N, int64_t C, int64_t H, int64_t D, const void* x, int apply_ln,
                               const float* ln_w, const float* ln_b, const void* w_qkvz, const float* bz,
                               const uint8_t* mask, float scale, float eps, void* xln_ws, void* q_ws, void* k_ws,
                               void* vt_ws, void* maskf_ws, void* bias_ws, void* o_out, void* stream);

/* The two halves of tops_triangle_attn_forward, for row-slab sharding:
 * project R pair rows (x [R][N][C], mask [R][N]) -> q/k [R][H][N][D], vt [R][H][D][Np],
 * maskf [R][Np], bias rows bias_ws [H][R][Np] (bias_proj_kernel, triangle_attn/kernel.py:36-98,
 * restricted to the rows); then attend R rows against the full shared bias [H][N][Np]
 * (triangle_attn_kernel, triangle_attn/kernel.py:110-253) into o_out [R][N][H*D]. */
int tops_triangle_attn_project(int dtype, int64_t R, int64_t N, int64_t C, int64_t H, int64_t D, const void* x,
                               int apply_ln, const float* ln_w, const float* ln_b, const void* w_qkvz,
                               const float* bz, const uint8_t* mask, float scale, float eps, void* xln_ws,
                               void* q_ws, void* k_ws, void* vt_ws, void* maskf_ws, void* bias_ws, void* stream);

/* tops_triangle_attn_project for the ending node without a transposed copy: pair
 * row i of the problem is column i of a square x, token (i, k) at x[(k*N + i)*C]
 * (x points at column r0 of the full [N][N][C] tensor for a slab of R columns).
 * mask [R][N] is the transposed mask's rows. N % 8 == 0. The reference's caller
 * passes X.transpose(0, 1).contiguous() instead (triangle_attn/module.py:53-121 takes
 * no direction); xln_ws, q/k/vt/maskf/bias are written in the transposed problem's order. */
int tops_triangle_attn_project_transposed(int dtype, int64_t R, int64_t N, int64_t C, int64_t H, int64_t D,
                                          const void* x, int apply_ln, const float* ln_w, const float* ln_b,
                                          const void* w_qkvz, const float* bz, const uint8_t* mask, float scale,
                                          float eps, void* xln_ws, void* q_ws, void* k_ws, void* vt_ws,
                                          void* maskf_ws, void* bias_ws, void* stream);
int tops_triangle_attn_attend(int dtype, int64_t R, int64_t N, int64_t H, int64_t D, const void* q_ws,
                              const void* k_ws, const void* vt_ws, const void* maskf_ws, const void* bias_ws,
                              void* o_out, void* stream);

/* out[t] = (o[t] * sigmoid(gin[t] wg^T + bg)) wo^T + bo over T tokens of width C.
 * Replaces triangle_attn/kernel.py:438-470 (fused_gate_forward; bg = bo = NULL) and
 * attn_pair_bias/module.py:65-66 (gate on raw X, with biases).
 *   o, gin, out [T][C]; wg, wo [C][C] (out,in); bg, bo [C] fp32 or NULL. C in {64,128}. */
int tops_fused_gate_forward(int dtype, int64_t T, int64_t C, const void* o, const void* gin, const void* wg,
                            const void* wo, const float* bg, const float* bo, void* out, void* stream);

/* tops_fused_gate_forward plus the Pairformer residual (no counterpart in the reference,
 * whose caller adds x + op(x) in torch): out[r(t)] = residual[r(t)] + gate result of token
 * t, where r(t) = t, or, with trans_n = n > 0, r(i*n + k) = k*n + i (the ending-node
 * result stored back in the untransposed layout). residual may be NULL or alias out. */
int tops_fused_gate_residual(int dtype, int64_t T, int64_t C, const void* o, const void* gin, const void* wg,
                             const void* wo, const float* bg, const float* bo, const void* residual, void* out,
                             int64_t trans_n, void* stream);

/* ---------------------------------------------------------------------------
 * triangle multiplicative update
 * Input phase — replaces triangle_mul/kernel.py:235-279 (input_phase):
 *   ab_out[k][m] = mask[m] * sigmoid(LN(x) g_in^T)[m,k] * (LN(x) p_in^T)[m,k], k < 2C, D-major.
 *   x [M][C]; mask [M] int8 multiplier or NULL; w_in [4C][C] = p_in_c | g_in_c (LN-folded);
 *   sum_in, b_in [4C] fp32 (folded column sums / biases); ab_out [2C][M]. C in {64,128}; M % 8 == 0. */
int tops_trimul_input_phase(int dtype, int64_t M, int64_t C, const void* x, const uint8_t* mask, const void* w_in,
                            const float* sum_in, const float* b_in, float eps, void* ab_out, void* stream);
/* Triangular contraction — replaces the torch.einsum of triangle_mul/module.py:70-76.
 *   direction 0 (outgoing): y[n][i][j] = sum_k a[n][i][k] b[n][j][k]
 *   direction 1 (incoming): y[n][i][j] = sum_k a[n][k][i] b[n][k][j]
 *   a, b, y [nb][L][L]; L % 8 == 0. */
int tops_trimul_contract(int dtype, int direction, int64_t nb, int64_t L, const void* a, const void* b, void* y,
                         void* stream);
/* Row-slab contraction for sharded runs (no counterpart in the single-device reference;
 * the einsum of triangle_mul/module.py:70-76 restricted to Mi output rows):
 *   a [nb][Mi][L] (outgoing) or [nb][L][Mi] (incoming) — this rank's rows i;
 *   b = P rank-major chunks as all_gather_into_tensor lays them out:
 *       [P][nb][L/P][L] (outgoing: rows j, K = k) or [P][nb][L][L/P] (incoming: M = j);
 *   y [nb][Mi][L]. L % P == 0 and (L/P) % 128 == 0 when P > 1; Mi % 8 == 0. */
int tops_trimul_contract_slab(int dtype, int direction, int64_t nb, int64_t Mi, int64_t L, int64_t P, const void* a,
                              const void* b, void* y, void* stream);
/* The row-slab contraction restricted to output columns [j_begin, j_begin + j_count) (no
 * counterpart in the reference): a sharded caller contracts each chunk of b as the
 * collective delivers it. j_begin % 256 == 0; j_count % 256 == 0 unless the range ends
 * at L. b is the full chunk buffer; only the chunks covering the range are read. */
int tops_trimul_contract_slab_cols(int dtype, int direction, int64_t nb, int64_t Mi, int64_t L, int64_t P,
                                   int64_t j_begin, int64_t j_count, const void* a, const void* b, void* y,
                                   void* stream);
/* Output phase — replaces triangle_mul/kernel.py:282-326 (output_phase):
 *   out[m][c] = sigmoid(LN_in(x) g_out^T)[m,c] * (LN_out(y) p_out^T)[m,c]
 *   y [C][M] (D-major), x [M][C]; w_out [2C][C] = p_out_c | g_out_c; sum_out, b_out [2C] fp32;
 *   out [M][C]; M % 8 == 0. */
int tops_trimul_output_phase(int dtype, int64_t M, int64_t C, const void* y, const void* x, const void* w_out,
                             const float* sum_out, const float* b_out, float eps, void* out, void* stream);

/* tops_trimul_output_phase with the Pairformer residual added in the epilogue (no
 * counterpart in the reference): out = residual + update; residual may alias out and x
 * (the in-place x += triangle_multiplicative_update(x)). */
int tops_trimul_output_phase_residual(int dtype, int64_t M, int64_t C, const void* y, const void* x,
                                      const void* w_out, const float* sum_out, const float* b_out, float eps,
                                      const void* residual, void* out, void* stream);
/* The whole op (triangle_mul/module.py:55-88 forward): input phase -> contraction ->
 * output phase. x [B][L][L][C] (L % 8 == 0), mask [B*L*L] int8 or NULL,
 * ab_ws [2C][B*L*L], y_ws [C][B*L*L], out [B][L][L][C]. */
int tops_trimul_forward(int dtype, int direction, int64_t B, int64_t L, int64_t C, const void* x, const uint8_t* mask,
                        const void* w_in, const float* sum_in, const float* b_in, const void* w_out,
                        const float* sum_out, const float* b_out, float eps, void* ab_ws, void* y_ws, void* out,
                        void* stream);

/* ---------------------------------------------------------------------------
 * attention with pair bias
 * Replaces attn_pair_bias/kernel.py:205-257 (apb_forward / _apb_kernel): writes the
 * pre-gate attention output og_out [M][H*D].
 *   x [M][C]; w_qkv [3C][C] rows WQ^T | WK^T | WV^T; z [M][M][Cz] raw pair tensor;
 *   wc [H][Cz] fp32, sum_w [H] fp32, b_const [H] fp32 (LN(z) folded into the bias
 *   projection, attn_pair_bias/module.py:29-35); key_mask [M] uint8 or NULL (extension);
 *   workspaces q_ws, k_ws [H][M][D] f16, vt_ws [H][D][Mp] f16, maskf_ws [Mp] f16, bias_ws [H][M][Mp] fp32.
 * Supported: Cz = 128, (C,H,D) in {(128,4,32), (64,4,16)}. */
int tops_apb_forward(int dtype, int64_t M, int64_t C, int64_t Cz, int64_t H, int64_t D, const void* x,
                     const void* w_qkv, const void* z, const float* wc, const float* sum_w, const float* b_const,
                     const uint8_t* key_mask, float scale, float eps, void* q_ws, void* k_ws, void* vt_ws,
                     void* maskf_ws, void* bias_ws, void* og_out, void* stream);

/* Query rows [q0, q0 + Mq) of tops_apb_forward (row-sharded pair-bias attention; the
 * reference is single-device, its kernel tiles queries the same way, attn_pair_bias/kernel.py:229).
 * x [M][C] is the whole sequence (K/V need every key); z_rows [Mq][M][Cz] are the pair rows
 * of those queries; bias_ws [H][Mq][Mp] fp32; og_rows [Mq][H*D]; q_ws/k_ws/vt_ws/maskf_ws
 * as for tops_apb_forward (full M). tops_apb_forward is q0 = 0, Mq = M. */
int tops_apb_forward_rows(int dtype, int64_t M, int64_t q0, int64_t Mq, int64_t C, int64_t Cz, int64_t H, int64_t D,
                          const void* x, const void* w_qkv, const void* z_rows, const float* wc, const float* sum_w,
                          const float* b_const, const uint8_t* key_mask, float scale, float eps, void* q_ws,
                          void* k_ws, void* vt_ws, void* maskf_ws, void* bias_ws, void* og_rows, void* stream);

/* No counterpart in the reference. tops_apb_forward for callers that cannot
 * allocate device memory (a serving runtime or embedding framework that owns a
 * fixed device-memory budget and forbids allocation after start-up): same
 * arguments minus the five workspaces, which live in one library-owned static
 * device array of about 2.5 MB per GPU, held until process exit. Limits: M <= 512,
 * C = 128, H = 4, D = 32, Cz = 128; M > 512 returns TOPS_ERR_CAPACITY. The array
 * is shared by all calls on a device — calls that overlap on the GPU race. The
 * first call on a device looks up the array's address; make it before any stream
 * capture. */
int tops_apb_forward_noalloc(int dtype, int64_t M, int64_t C, int64_t Cz, int64_t H, int64_t D, const void* x,
                             const void* w_qkv, const void* z, const float* wc, const float* sum_w,
                             const float* b_const, const uint8_t* key_mask, float scale, float eps, void* og_out,
                             void* stream);

/* ---------------------------------------------------------------------------
 * Workspace sizes (host-only, no device work; no counterpart in the reference,
 * whose temporaries torch allocates inside
 * triangle_attn/kernel.py:300-301,326). Each writes byte counts in the order listed
 * and validates the shape like the entry point that takes the workspaces. */

/* bytes[6] = xln, q, k, vt, maskf, bias for R projected rows of an N x N problem. */
int tops_triangle_attn_workspace_bytes(int dtype, int64_t R, int64_t N, int64_t C, int64_t H, int64_t D,
                                       int64_t* bytes);
/* bytes[2] = ab [2C][B*L*L], y [C][B*L*L]. */
int tops_trimul_workspace_bytes(int dtype, int64_t B, int64_t L, int64_t C, int64_t* bytes);
/* bytes[5] = q, k, vt, maskf, bias for query rows Mq of M tokens. */
int tops_apb_workspace_bytes(int64_t M, int64_t Mq, int64_t H, int64_t D, int64_t* bytes);

/* ---------------------------------------------------------------------------
 * fp32 IO path (CUDA cores). The reference admits fp32 IO for all three ops
 * (_common/dtype.py:7-19) and then runs its Triton kernels in fp32; these four
 * generic kernels are what the package composes each op's fp32 forward from
 * (triangleops_b200/_f32.py). All pointers fp32 unless noted. */

/* y[t][c] = LN(x[t])[c] * w[c] + b[c] over rows of width C; w, b may be NULL. */
int tops_f32_layernorm(int64_t T, int64_t C, const float* x, const float* w, const float* b, float eps, float* y,
                       void* stream);

/* Batched strided C(b,m,n) = sum_k A(b,m,k) B(b,n,k) + bias[n] (bias may be NULL).
 * strides[9] = {A: b, m, k; B: b, n, k; C: b, m, n} in elements. */
int tops_f32_gemm(int64_t batch, int64_t M, int64_t N, int64_t K, const float* A, const float* B, const float* bias,
                  float* C, const int64_t* strides, void* stream);

/* O[r][q][h*D+d] = softmax_k(scale * q.k + bias[h][q][k]) v, 1 <= D <= 128.
 * q/k/v element (r,h,n,d) at r*sr + h*sh + n*sn + d; mask [R][Nk] uint8 or NULL;
 * mask_mode 0: masked keys get -1e9 added (triangle attention); 1: masked keys dropped. */
int tops_f32_attention(int64_t R, int64_t H, int64_t Nq, int64_t Nk, int64_t D, const float* q, const float* k,
                       const float* v, int64_t sr, int64_t sh, int64_t sn, const float* bias, const uint8_t* mask,
                       float scale, int mask_mode, float* out, void* stream);

/* y[r][c] = a[r][c] * sigmoid(g[r][c] + bg[c]) * mask[r]; bg, mask (0/1 bytes) may be NULL. */
int tops_f32_gated_mul(int64_t rows, int64_t cols, const float* a, int64_t lda, const float* g, int64_t ldg,
                       const float* bg, const uint8_t* mask, float* y, int64_t ldy, void* stream);

/* ---------------------------------------------------------------------------
 * Pairformer pair transition (no counterpart in the reference, which ships only the
 * triangle ops; the AlphaFold-3 transition layer): over M tokens of C = 128 channels
 *   out = x + ( silu(LN(x) W1^T) * (LN(x) W2^T) ) W3^T,   hidden width 4C,
 * with the LN affine folded on the host: w12 [(4C/64) * 128][C] holds, per 64-wide
 * hidden chunk h, the rows W1[h]*gamma then W2[h]*gamma (IO dtype); b12 [(4C/64)][128]
 * fp32 the matching W1[h] beta | W2[h] beta; w3 [C][4C] (IO dtype). out may alias x. */
int tops_transition_forward(int dtype, int64_t M, int64_t C, const void* x, const void* w12, const void* w3,
                            const float* b12, float eps, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIANGLEOPS_B200_H */

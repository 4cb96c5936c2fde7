/* libbasal200: the C ABI of basal's quantised-linear hot path on B200 (sm_100a).
 *
 * Every entry point takes device pointers, sizes and a cudaStream_t (passed as void*; NULL = the legacy default
 * stream), enqueues its kernels on that stream and returns a status code. None allocates memory, synchronises the
 * stream or reads device data on the host, so a CUDA graph can capture any of them. Buffers are dense row-major
 * ("contiguous"); the 16-byte alignment of every base pointer is checked.
 *
 * Citations are to the reference, rkinas/basal 2.8.1 (path:line within that project).
 */
#ifndef BASAL200_H
#define BASAL200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
enum {
  BASAL200_OK = 0,
  BASAL200_ERR_ARG = 1,     /* a NULL pointer or a negative size */
  BASAL200_ERR_SHAPE = 2,   /* a size the format cannot take, e.g. N % 128 != 0 (basal/blockquant.py:38-39) */
  BASAL200_ERR_ALIGN = 3,   /* a base pointer not 16-byte aligned */
  BASAL200_ERR_DTYPE = 4,   /* an unsupported dtype code */
  BASAL200_ERR_ARCH = 5,    /* the current device is not compute capability 10.0 (sm_100a) */
  BASAL200_ERR_LAUNCH = 6,  /* a CUDA error at launch */
  BASAL200_ERR_TMAP = 7,    /* cuTensorMapEncodeTiled refused a TMA descriptor */
  BASAL200_ERR_LIMIT = 8    /* a size beyond what the entry point was built for */
};

/* Element type codes of activations, outputs and biases. */
enum { BASAL200_BF16 = 0, BASAL200_F16 = 1, BASAL200_F32 = 2 };

/* ---- FP8-block / INT8-block (128 x 128 weight blocks, 1 x 128 activation groups, fp32 scales) ---- */

/* x [M, K] (x_dtype) -> q [M, K] e4m3 codes, s [M, K/128] fp32. K % 128 == 0. Bit-exact to
 * BlockFormat.act_quant_ops of the FP8 format (basal/blockquant.py:118-123, :137-144; fp8block.py:30-31). */
int basal200_fp8_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, uint8_t* q, float* s, void* stream);

/* The INT8 format (int8block.py:43-44): q int8, round half to even, +-127. */
int basal200_int8_act_quant(const void* x, int x_dtype, int64_t M, int64_t K, int8_t* q, float* s, void* stream);

/* w [N, K] (w_dtype) -> q [N, K] e4m3, s [N/128, K/128] fp32. Bit-exact to BlockFormat.quantize
 * (basal/blockquant.py:126-135) of the FP8 format. N % 128 == 0, K % 128 == 0. */
int basal200_fp8_block_quantize(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* q, float* s,
                                void* stream);

/* The INT8 format of the same (int8block.py:43-44). */
int basal200_int8_block_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int8_t* q, float* s,
                                 void* stream);

/* Workspace bytes with which the block GEMMs and linears below spread a few-rows GEMM (M <= 64) over every SM; 0 for
 * a shape that never takes it (M > 64, or weights of enough 128-row tiles to fill the GPU). Pure: no device call. */
int64_t basal200_block_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* C [M, N] (c_dtype) = sum over 128-deep K slices of (q_kb . w_kb^T) * s[m, kb] * ws[n/128, kb], fp32 accumulation,
 * then + bias[n] (c_dtype, may be NULL) rounded as torch adds a bias to the cast output. Replaces the torch op
 * basal::fp8_block_gemm (basal/blockquant.py:151-159, kernel :63-106). N % 128 == 0, K % 128 == 0; M may be 0.
 * workspace (16-byte aligned, may be NULL): when it holds basal200_block_gemm_workspace_bytes(M, N, K) > 0 bytes, a
 * few-rows GEMM writes each 128-deep slice's product there and sums them in a second kernel, in the same order and
 * with the same roundings as without it: the output bits do not change, only which SMs stream the weights. */
int basal200_fp8_block_gemm(const uint8_t* q, const float* s, const uint8_t* w, const float* ws, const void* bias,
                            void* c, int c_dtype, int64_t M, int64_t N, int64_t K, void* workspace,
                            int64_t workspace_bytes, void* stream);

/* One rank's column shard of a column-parallel FP8 block linear (a tensor-parallel model's N-sharded linears; the
 * reference keeps whole weights on every GPU, so there is no reference function: this replaces the pair
 * "fp8_block_gemm of the shard, then all-gather of the outputs"): the shard's [M, N] result (its weight rows are the
 * linear's rows col_off .. col_off + N - 1) is stored into each of the npeers buffers outs[r] ([M, n_total], c_dtype
 * bf16 or fp16, row-major, peer-mapped device memory of every rank), at columns col_off .. col_off + N - 1, by the
 * GEMM's own stores. The caller synchronises the ranks afterwards. N, col_off multiples of 128; npeers <= 8.
 * barrier_pad: this rank's pad of basal200_peer_barrier (4-byte aligned), or NULL. When the pad's status word says
 * that a barrier gave up, the GEMM stores nothing at all, so a rank that missed a barrier never writes into a peer's
 * output while that peer may still be reading it. */
int basal200_fp8_block_gemm_gather(const uint8_t* q, const float* s, const uint8_t* w, const float* ws,
                                   void* const* outs, int npeers, int64_t col_off, int64_t n_total, int c_dtype,
                                   int64_t M, int64_t N, int64_t K, const uint32_t* barrier_pad, void* stream);

/* Word of a barrier pad that holds its sticky status: 0 while every barrier completed; non-zero once a wait of this
 * rank gave up, or a peer's did (a rank whose status is set writes it into every peer's pad at each barrier). The
 * host reads it to raise an error; it stays set until the caller zeroes it with every rank idle. */
#define BASAL200_PAD_STATUS_WORD 9

/* A barrier of the `world` ranks that share peer-mapped signal pads (pads[r]: rank r's pad, at least 10 uint32 words,
 * zero before the first call, used by nothing else): enqueued on `stream`, it returns (on the device) once every rank
 * has reached the same call, with each rank's stream work before it visible to the others' work after it. A wait
 * for a rank gives up after timeout_ns: the kernel records BASAL200_FAULT_TIMEOUT_PEER, sets the pad's status word
 * (BASAL200_PAD_STATUS_WORD) and ends (no trap). The call count lives in the pad, so a captured CUDA graph may replay
 * the barrier. world <= 8. */
int basal200_peer_barrier(uint32_t* const* pads, int world, int rank, int64_t timeout_ns, void* stream);

/* basal::int8_block_gemm (basal/blockquant.py:95-96, int8block.py:43): each slice's product exact in int32. */
int basal200_int8_block_gemm(const int8_t* q, const float* s, const int8_t* w, const float* ws, const void* bias,
                             void* c, int c_dtype, int64_t M, int64_t N, int64_t K, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* The whole linear: act_quant of x into the caller's scratch (q_scratch [M, K] bytes, s_scratch [M, K/128] fp32),
 * then the block GEMM into y [M, N] (y_dtype = x_dtype), + bias; workspace as for basal200_fp8_block_gemm. When the
 * workspace makes the GEMM split and x is bf16 or fp16, the quantiser runs inside the GEMM kernel instead (one launch
 * fewer; q_scratch is then not written, s_scratch is, and every bit of y and s_scratch is the same). Replaces
 * fp8block.linear / BlockFormat.linear (basal/fp8block.py:74-85, basal/blockquant.py:175-183) and the op
 * basal::fp8_block_linear_sm90 (fp8block.py:61-71). */
int basal200_fp8_block_linear(const void* x, int x_dtype, const uint8_t* w, const float* ws, const void* bias,
                              void* y, int64_t M, int64_t N, int64_t K, uint8_t* q_scratch, float* s_scratch,
                              void* workspace, int64_t workspace_bytes, void* stream);

/* int8block.linear (int8block.py:44 = BlockFormat.linear, basal/blockquant.py:175-183). */
int basal200_int8_block_linear(const void* x, int x_dtype, const int8_t* w, const float* ws, const void* bias,
                               void* y, int64_t M, int64_t N, int64_t K, int8_t* q_scratch, float* s_scratch,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* Activations of the gated linears. */
enum { BASAL200_ACT_SILU = 1, BASAL200_ACT_GELU_TANH = 2 };

/* The gated MLP input of a SwiGLU / GeGLU layer in one call: y [M, I] = act(x W_gate^T) * (x W_up^T) for a merged
 * block-quantised weight w [2I, K] = [gate; up] (the layout of blockquant.fuse, basal/blockquant.py:43-51, with the
 * scales ws [2I/128, K/128]), x [M, K] bf16 or fp16, y in x's type. act = BASAL200_ACT_SILU (Qwen,
 * basal/gdn_graph.py:127-128) or BASAL200_ACT_GELU_TANH (Gemma, basal/gemma4_graph.py:193-197). Replaces the pair
 * "linear of the merged gate/up weight, then act(gate) * up" with the same roundings (each linear output cast to
 * x's type, act(.) cast, the product cast): the activation quantiser into the scratch (as basal200_fp8_block_linear),
 * then one GEMM whose epilogue pairs gate and up columns, so the [M, 2I] intermediate is never written (few rows
 * with a workspace: see basal200_block_linear_glu_workspace_bytes). I % 128 == 0, K % 128 == 0. */
int basal200_fp8_block_linear_glu(const void* x, int x_dtype, const uint8_t* w, const float* ws, void* y, int64_t M,
                                  int64_t I, int64_t K, int act, uint8_t* q_scratch, float* s_scratch, void* workspace,
                                  int64_t workspace_bytes, void* stream);

/* The INT8 format of the same (int8block.py:43-44). */
int basal200_int8_block_linear_glu(const void* x, int x_dtype, const int8_t* w, const float* ws, void* y, int64_t M,
                                   int64_t I, int64_t K, int act, int8_t* q_scratch, float* s_scratch,
                                   void* workspace, int64_t workspace_bytes, void* stream);

/* Workspace bytes (16-byte aligned) with which the gated linears above run few rows (M <= 64) as the few-rows linear
 * of the merged weight into a [M, 2I] temporary, then the activation: the same bits as without it, faster. 0 for
 * M > 64. Pure: no device call. */
int64_t basal200_block_linear_glu_workspace_bytes(int64_t M, int64_t I, int64_t K);

/* A linear whose output is added to the residual stream in the same kernel: y [M, N] = residual [M, N] + (x W^T
 * (+ bias)), x, residual and y of x_dtype (bf16 or fp16), with torch's roundings (the linear's output cast, + bias,
 * the sum cast) -- the pair "linear, then h + out" of a pre-norm decoder layer's output projections (the Qwen 3.5
 * graph's MLP down, linear-attention out and attention o projections, basal/gdn_graph.py:128, :439, :466), which
 * the reference runs as two kernels. y may be the residual itself (in place).
 * The activation quantiser goes to the scratch as for basal200_fp8_block_linear; few rows (M <= 64) with
 * basal200_block_linear_residual_workspace_bytes(M, N, K) of workspace run the few-rows linear into a temporary,
 * then the addition (the same bits). N % 128 == 0, K % 128 == 0. No counterpart in the reference. */
int basal200_fp8_block_linear_residual(const void* x, int x_dtype, const uint8_t* w, const float* ws,
                                       const void* bias, const void* residual, void* y, int64_t M, int64_t N,
                                       int64_t K, uint8_t* q_scratch, float* s_scratch, void* workspace,
                                       int64_t workspace_bytes, void* stream);

/* The INT8 format of the same (int8block.py:43-44). */
int basal200_int8_block_linear_residual(const void* x, int x_dtype, const int8_t* w, const float* ws,
                                        const void* bias, const void* residual, void* y, int64_t M, int64_t N,
                                        int64_t K, int8_t* q_scratch, float* s_scratch, void* workspace,
                                        int64_t workspace_bytes, void* stream);

/* Workspace bytes (16-byte aligned) for the few-rows path of the residual linears; 0 for M > 64. Pure. */
int64_t basal200_block_linear_residual_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* The gated linear of basal200_fp8_block_linear_glu from activation codes and scales already quantised (q [M, K]
 * e4m3, s [M, K/128] fp32, e.g. by basal200_rms_norm_fp8_quant, which fuses the quantiser into the norm before it):
 * y [M, I] (y_dtype bf16 or fp16) = act(gate) * up with the same roundings. workspace as for the gated linear. No
 * counterpart in the reference, whose gated MLP input is the merged linear then act(g) * u (basal/gdn_graph.py:127). */
int basal200_fp8_block_gemm_glu(const uint8_t* q, const float* s, const uint8_t* w, const float* ws, void* y,
                                int y_dtype, int64_t M, int64_t I, int64_t K, int act, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* The residual linear of basal200_fp8_block_linear_residual from activation codes and scales already quantised (e.g.
 * by basal200_gdn_gate_fp8_quant): y [M, N] = residual + (q, s) . w^T (+ bias), y_dtype bf16 or fp16, y may be the
 * residual. The output projections of basal/gdn_graph.py:128, :439, :466. */
int basal200_fp8_block_gemm_residual(const uint8_t* q, const float* s, const uint8_t* w, const float* ws,
                                     const void* bias, const void* residual, void* y, int y_dtype, int64_t M,
                                     int64_t N, int64_t K, void* workspace, int64_t workspace_bytes, void* stream);

/* ---- The config-5 hybrid decoder's steps around its linears (a Qwen 3.5 layer, basal/gdn_graph.py:122-140, :432-439)
 * ---- */

/* Qwen3_5RMSNorm of each row of x [M, D] (x_dtype bf16 or fp16, weight w [D] of that type applied as 1 + w, fp32
 * inside, basal/gdn_graph.py:122-126) fused with the FP8 activation quantiser: q [M, D] e4m3 and s [M, D/128] fp32
 * are the codes of the normed row rounded to x_dtype, bit-exact to basal200_fp8_act_quant of that row; y [M, D] (may
 * be NULL) receives the normed row. D % 128 == 0. */
int basal200_rms_norm_fp8_quant(const void* x, int x_dtype, const void* w, float eps, int64_t M, int64_t D, void* y,
                                uint8_t* q, float* s, void* stream);

/* The Gated DeltaNet's input steps (basal/gdn_graph.py:131-140, :559-576, with transformers' Qwen3_5GatedDeltaNet):
 * over rows of T tokens (proj [rows * T, ld] of `dtype`, the merged input projection's output: the convolution's
 * channels [q (Hk heads) | k (Hk) | v (Hv)] of 128 from column 0, b and a (Hv each) at columns b_off and a_off), the
 * causal depthwise convolution of kw taps (conv [C, kw], C = (2 Hk + Hv) * 128; tail [tail_rows, kw - 1, C] the inputs
 * before token 0, tail_rows 1 (shared) or rows, or NULL for zeros) and SiLU, rounded to `dtype`; the l2 norms of q and
 * k (eps 1e-6; q also times 128^-1/2); beta = sigmoid(b) rounded; g = -exp(A_log) * softplus(a + dt_bias) in fp32.
 * Outputs are head-major: q, k [rows, Hk, T, 128] fp32 (one per key head), v [rows, Hv, T, 128] in `dtype` (its
 * values are `dtype` values already), beta, g [rows, Hv, T] fp32. */
int basal200_gdn_prep(const void* proj, int dtype, int64_t ld, const void* tail, int tail_rows, const void* conv,
                      int kw, const float* A_log, const void* dt_bias, int b_off, int a_off, int rows, int T, int Hk,
                      int Hv, float* q, float* k, void* v, float* beta, float* g, void* stream);

/* The Gated DeltaNet's output steps (basal/gdn_graph.py:432-438, Qwen3_5RMSNormGated) fused with the FP8 quantiser of
 * the output projection's input: o [rows, Hv, Tp, 128] (the recurrence's output, Tp >= T; o_dtype fp32 or `dtype`,
 * the same bits when basal200_gdn_chunk_rule wrote it in `dtype` as when in fp32), z in a [rows * T, ld]
 * matrix of `dtype` from column z_off (Hv * 128 values a token), gw [128]: each head's values rounded to `dtype`,
 * RMS-normed (eps), times gw, times silu(z), rounded -> y [rows * T, Hv * 128] (may be NULL), and quantised with one
 * scale per head: q [rows * T, Hv * 128] e4m3, s [rows * T, Hv] fp32 (bit-exact to basal200_fp8_act_quant of y). */
int basal200_gdn_gate_fp8_quant(const void* o, int o_dtype, int Tp, const void* z, int dtype, int64_t ld, int z_off,
                                const void* gw, float eps, int rows, int T, int Hv, void* y, uint8_t* q, float* s,
                                void* stream);

/* The attention layers' input steps (basal/gdn_graph.py:452-460, Qwen 3.5 full attention with a gated output) over
 * rows of T tokens of the merged projection qkv [rows * T, ld] (`dtype`; per token H heads of (128 q, 128 gate), then
 * Hk heads of 128 k, then Hk of 128 v): q and k Qwen3_5RMSNorm'ed with q_norm / k_norm [128] (eps), rounded to
 * `dtype`, then rotated in their first rot dimensions (rot % 8 == 0, rot <= 128; cos / sin [rows or 1, T, rot] with
 * cs_row elements between rows, 0 when shared) by x1 cos - x2 sin, x2 cos + x1 sin with torch's roundings. q ->
 * q_out [rows, H, T, 128]; k and v -> k_out / v_out [rows, Hk, kv_len, 128] at positions kv_off .. kv_off + T - 1
 * (after a prefix's keys and values already there). A norm's sum of squares is in this kernel's own order, so a
 * normed value may differ from torch's by one unit in the last place. */
int basal200_attn_prep(const void* qkv, int dtype, int64_t ld, int rows, int T, int H, int Hk, const void* q_norm,
                       const void* k_norm, float eps, const void* cos, const void* sin, int64_t cs_row, int rot,
                       void* q_out, void* k_out, void* v_out, int64_t kv_len, int64_t kv_off, void* stream);

/* The attention's output gate (basal/gdn_graph.py:464-466) fused with the FP8 quantiser of the output projection's
 * input: o [rows, H, T, 128] (`dtype`), the gates in qkv as for basal200_attn_prep: a = o * sigmoid(gate) with
 * torch's 16-bit roundings, quantised with one scale per head: q [rows * T, H * 128] e4m3, s [rows * T, H] fp32
 * (bit-exact to basal200_fp8_act_quant of a). */
int basal200_attn_gate_fp8_quant(const void* o, int dtype, const void* qkv, int64_t ld, int rows, int T, int H,
                                 uint8_t* q, float* s, void* stream);

/* The gated delta rule of the Gated DeltaNet layers (transformers' torch_chunk_gated_delta_rule / fla's
 * chunk_gated_delta_rule, called by basal/gdn_graph.py:81-87, :492-493), fp32: per row r and value head h, from the
 * state s0 [s0_rows, H, 128, 128] (s0_rows 1: shared by every row; NULL: zeros), over T tokens of q, k
 * [rows, Hk, T, 128] fp32 (value head h reads key head h / (H / Hk); l2-normed, q scaled, as basal200_gdn_prep leaves
 * them), v [rows, H, T, 128] (v_dtype fp32, bf16 or fp16), g, beta [rows, H, T] fp32:
 * S_t = e^{g_t} S_{t-1} + k_t (beta_t (v_t - e^{g_t} S_{t-1}^T k_t))^T, o_t = S_t^T q_t -> o [rows, H, T, 128]
 * (o_dtype fp32, or v_dtype when that is 16-bit: each fp32 value rounded to nearest once), and the final state into
 * s_out [rows, H, 128, 128] fp32 (may be NULL). Computed over chunks of 64 tokens. */
int basal200_gdn_chunk_rule(const float* q, const float* k, const void* v, int v_dtype, const float* g,
                            const float* beta, const float* s0, int s0_rows, void* o, int o_dtype, float* s_out,
                            int rows, int Hk, int H, int T, void* stream);

/* Size limit of basal200_fp8_block_linear_noalloc: at most this many activation values (M * K) a call. */
#define BASAL200_NOALLOC_MAX_ELEMS (1 << 24)

/* basal200_fp8_block_linear without caller scratch, for callers that cannot allocate device memory: a runtime whose
 * device memory is planned up front in a fixed arena, a host language that holds no device allocator of its own, a
 * caller that must not let cudaMalloc synchronise the device mid-request. The activation codes and scales go to an
 * array inside the library (16 MiB + 512 KiB, BASAL200_NOALLOC_MAX_ELEMS values), which every GPU that loads the
 * library holds until the process exits. M * K above that limit returns BASAL200_ERR_LIMIT before any work. The
 * call allocates nothing. Its first call on a device looks up the array's address on that device (with the device
 * current) and keeps it for the life of the process: make that first call before any stream capture, and do not
 * call it on a device after cudaDeviceReset (the kept address would then name memory of the destroyed context). All calls on a device share the array, so calls that
 * overlap on the GPU (other streams, other threads) race on it; serialise them. No counterpart in the reference. */
int basal200_fp8_block_linear_noalloc(const void* x, int x_dtype, const uint8_t* w, const float* ws,
                                      const void* bias, void* y, int64_t M, int64_t N, int64_t K, void* stream);

/* ---- NVFP4 (e2m1 values, e4m3 scales per 16 features in the 128 x 4 swizzle, fp32 global scales) ---- */

/* x [M, K] -> q [Mp, K/2] packed e2m1 (even feature in the low nibble), s [Mp * K/16] swizzled e4m3 scales,
 * Mp = M rounded up to 128, padding rows zero; inv_g [1] fp32 on the device. K % 64 == 0. Bit-exact to the
 * reference's quantiser (basal/nvfp4.py:115-158; its maths nvfp4.py:106-112). */
int basal200_nvfp4_act_quant(const void* x, int x_dtype, const float* inv_g, int64_t M, int64_t K, uint8_t* q,
                             uint8_t* s, void* stream);

/* y [M, N] (y_dtype) = alpha[0] * (dequantised q [Mp, K/2] . dequantised w [N, K/2]^T), + bias. The scales s and ws
 * in the 128 x 4 swizzle, ws covering ceil(N/128)*128 rows. Replaces nvfp4._mm (basal/nvfp4.py:167-180, cuBLAS
 * through F.scaled_mm). K % 64 == 0, N % 16 == 0. */
int basal200_nvfp4_gemm(const uint8_t* q, const uint8_t* s, const uint8_t* w, const uint8_t* ws, const float* alpha,
                        const void* bias, void* y, int y_dtype, int64_t M, int64_t N, int64_t K, void* stream);

/* The op basal::nvfp4_linear (basal/nvfp4.py:183-189): act_quant into the scratch (q_scratch [Mp, K/2],
 * s_scratch [Mp * K/16]) then the GEMM into y [M, N] (y_dtype = x_dtype), + bias. */
int basal200_nvfp4_linear(const void* x, int x_dtype, const uint8_t* w, const uint8_t* ws, const float* alpha,
                          const float* inv_g, const void* bias, void* y, int64_t M, int64_t N, int64_t K,
                          uint8_t* q_scratch, uint8_t* s_scratch, void* stream);

/* w [N, K] -> codes [N, K/2], swizzled scales [ceil(N/128)*128 * ceil(K/64)*4] (zero padded), g [1] fp32 global
 * scale. Bit-exact to nvfp4.quantize (basal/nvfp4.py:75-97): 8 candidate scales per 16-block by least squares.
 * Any N; K % 16 == 0 (the GEMM itself needs K % 64 == 0 and N % 16 == 0, nvfp4.fits). */
int basal200_nvfp4_quantize(const void* w, int w_dtype, int64_t N, int64_t K, uint8_t* codes, uint8_t* scales,
                            float* g, void* stream);

/* ---- Option-code readout ---- */

/* z [R, U] fp32 = h [R, D] (h_dtype, row stride ldh elements) . head[ids[u], :]^T (+ bias[ids[u]]), then
 * softcap * tanh(z / softcap) when softcap > 0. head [V, D] bf16, fp16 or fp32 (row stride ldw), ids [U] int64
 * into it, bias [V] (bias_dtype) or NULL. An id outside [0, V) reads nothing: its logits are NaN and the fault bit
 * BASAL200_FAULT_BAD_ID is set. Replaces CodeReadout.rows + .logits (basal/readout.py:57-74): the option rows are
 * read straight from the head, never copied. */
int basal200_code_logits(const void* h, int h_dtype, int64_t R, int64_t D, int64_t ldh, const void* head,
                         int head_dtype, int64_t V, int64_t ldw, const int64_t* ids, int64_t U, const void* bias,
                         int bias_dtype, float softcap, float* z, void* stream);

/* p [R, Kmax] fp32 = softmax over j of z[r, idx[r, j]] with -inf where pad[r, j] != 0 (the padding gets 0).
 * Replaces CodeReadout.probs_of (basal/readout.py:76-79). Kmax <= 1024. The kernel may start while the library
 * kernel ahead of it in the stream (code_logits) runs, and reads idx and pad before it waits for that kernel: they
 * must not be outputs of the library kernel directly ahead (z may be). */
int basal200_code_probs(const float* z, int64_t R, int64_t U, const int64_t* idx, const uint8_t* pad, int64_t Kmax,
                        float* p, void* stream);


/* ---- Diagnostics ---- */

/* Fault bits (basal200_device_faults): a bounded wait of a GEMM gave up (producer, MMA issuer, epilogue, drain), a
 * readout id was out of range, or a peer barrier's wait for another rank gave up. */
enum {
  BASAL200_FAULT_TIMEOUT_PRODUCER = 1,
  BASAL200_FAULT_TIMEOUT_MMA = 2,
  BASAL200_FAULT_TIMEOUT_EPILOGUE = 4,
  BASAL200_FAULT_TIMEOUT_DRAIN = 8,
  BASAL200_FAULT_BAD_ID = 16,
  BASAL200_FAULT_TIMEOUT_PEER = 32
};

/* The fault bits kernels on `device` recorded when a bounded wait gave up (0: none); clear != 0 resets them.
 * Synchronises the device: for tests and error paths, not for the hot path. */
unsigned basal200_device_faults(int device, int clear);

const char* basal200_status_string(int status);
int basal200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* BASAL200_H */

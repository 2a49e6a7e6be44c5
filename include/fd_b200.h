/*
 * futudiffu_b200 C ABI.
 *
 * One shared library (futudiffu_b200/libfd_b200.so) exports these entry
 * points.  Every function takes plain device pointers, sizes and a
 * cudaStream_t passed as void*, launches asynchronously on that stream and
 * returns an FD_* status code.  No function allocates device memory: the
 * caller owns every buffer (the reference's Python wrappers allocate all
 * outputs with torch before launching, and so does the Python layer here).
 *
 * Layouts and formulas follow the reference operator API of sqcu/futudiffu
 * (cited per function as file:line in that project).  Tensors are
 * row-major and contiguous unless a stride argument says otherwise.
 *
 * dtype codes follow the reference's custom-op encoding
 * (src/futudiffu/fp8_kernels.py:1772-1776): 0 bf16, 1 f16, 2 f32, 3 e4m3.
 */
#ifndef FD_B200_H
#define FD_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- status codes -------------------------------------------------------- */
#define FD_OK 0
#define FD_ERR_ARG 1         /* bad shape / alignment / null pointer          */
#define FD_ERR_CUDA 2        /* a CUDA runtime or driver call failed          */
#define FD_ERR_TIMEOUT 3     /* a device-side bounded wait expired            */
#define FD_ERR_UNSUPPORTED 4 /* combination of options not built               */

/* bits of the device-wide status word (fd_get_status) */
#define FD_STATUS_TIMEOUT 1u
#define FD_STATUS_BOUNDS 2u

/* ---- dtype codes ---------------------------------------------------------- */
#define FD_DT_BF16 0
#define FD_DT_F16 1
#define FD_DT_F32 2
#define FD_DT_E4M3 3
#define FD_DT_I8 4

/* ---- attention option codes ------------------------------------------------ */
#define FD_QK_INT8 0 /* INT8 codes, truncation toward zero (sage_kernels.py:632-639) */
#define FD_QK_FP8 1  /* e4m3 codes, RNE (sage_kernels.py:151-155)                  */
#define FD_GRAN_TOKEN 0 /* one scale per row (reference)                            */
#define FD_GRAN_BLOCK 1 /* one scale per 128 Q rows / 64 K rows                      */
#define FD_PV_BF16 0 /* bf16 P x bf16 V (sage_kernels.py:681-684)                     */
#define FD_PV_FP8 1  /* e4m3 P (static scale) x e4m3 V (per-channel scale)            */
/* FD_PV_FP8_TILE: the reference's FP8 PV (sage_kernels.py:1135-1154): per 64-key
 * tile, e4m3 P per row (scaled by its absmax in the tile) and e4m3 V per column
 * (scaled by its absmax over the tile's 64 rows, fd_attn_quant_v_tile).          */
#define FD_PV_FP8_TILE 2

/* Library version string and the last host-side error message (thread-local). */
const char* fd_version(void);
const char* fd_last_error(void);

/* Read (and optionally clear) the device status word on the current device.
 * Synchronises the device.  Returns FD_OK or FD_ERR_CUDA. */
int fd_get_status(unsigned int* out, int clear);

/* Numerics hook; no counterpart in the reference.  out[i] = a[i] / b[i] with the
 * f32 divide every quantiser here uses: PTX div.full.f32, which is what the
 * reference's Triton kernels compile `/` to (measured bit-identical on the B200).
 * Parity tests evaluate the CPU oracle's scale arithmetic with it. */
int fd_div_full_f32(const float* a, const float* b, float* out, int64_t n, void* stream);

/* TMEM load-throughput microbenchmark (no counterpart in the reference): one CTA
 * per SM allocates the 512 TMEM columns; `warps` warps read them with tcgen05.ld
 * 32x32b loads of `width` (16 / 32 / 64) columns, `per_wait` loads per
 * tcgen05.wait::ld, `iters` rounds of 128 columns per warp; with `fma` != 0 every
 * loaded value is accumulated as the FP8 GEMM's per-slice promotion does.
 * cycles (num_SMs x 12) int64: each warp's clock64 duration (unused slots are not
 * written).  Measures the bound of the GEMM's promotion (bench.py --workload
 * tmem_probe). */
int fd_probe_tmem_ld(int width, int per_wait, int warps, int fma, int iters, long long* cycles, float* sink,
                     void* stream);

/* G1 -- fp8_act_quant (src/futudiffu/fp8_kernels.py:54-90).
 * x (M, K) in x_dtype (bf16/f16/f32), K % block == 0, block == 128.
 * y (M, K) e4m3; s (M, K/block) f32 with s = max(amax/448, 1e-12),
 * y = e4m3_rne(clamp(x * (448 / max(amax, 1e-12)), -448, 448)). */
int fd_fp8_act_quant(const void* x, int x_dtype, void* y, float* s, int64_t M, int64_t K,
                     int block, void* stream);

/* G6 -- quantize_fp8_blockwise (src/futudiffu/fp8.py:337-371).
 * w (N, K) in w_dtype, N % block == 0, K % block == 0; y (N, K) e4m3;
 * s (N/block, K/block) f32 holding 1 / (448 / max(amax, 1e-12)). */
int fd_fp8_weight_quant(const void* w, int w_dtype, void* y, float* s, int64_t N, int64_t K,
                        int block, void* stream);

/* G6 -- dequantize_fp8_blockwise (src/futudiffu/fp8.py:452-480).
 * out (N, K) in out_dtype = float(code) * s[n/block, k/block]. */
int fd_fp8_dequant_blockwise(const void* w, const float* s, void* out, int out_dtype, int64_t N,
                             int64_t K, int block, void* stream);

/* G2 -- fp8_gemm_blockwise / fp8_addmm_blockwise / fp8_gemm_v1t
 * (src/futudiffu/fp8_kernels.py:125-343, :1417-1699; op :1814-1841).
 * a (M, K) e4m3, a_s (M, K/128) f32.
 * b_layout 0: b (N, K) e4m3, b_s (ceil(N/128), K/128)   [fp8_gemm_blockwise]
 * b_layout 1: b (K, N) e4m3, b_s (K/128, ceil(N/128))   [fp8_gemm_v1t]
 * b_layout 2: b (N, K) e4m3, b_s (N,) per-row, applied after the K loop
 *             [fp8_gemm_rowwise, fp8_kernels.py:349-414]
 * c (M, N) in c_dtype (bf16/f16/f32) =
 *   sum_k dot128(a, b)[m, n] * a_s[m, k] * b_s[n/128, k] (+ bias[n]).
 * bias may be NULL; bias_dtype in {bf16, f16, f32}.  K % 128 == 0,
 * N % 16 == 0.  Accumulation is fp32 with one promotion per 128-K slice. */
int fd_fp8_gemm_blockwise(const void* a, const float* a_s, const void* b, const float* b_s,
                          const void* bias, int bias_dtype, void* c, int c_dtype, int64_t M,
                          int64_t N, int64_t K, int b_layout, void* stream);

/* G4 -- fp8_silu_gate_quant (src/futudiffu/fp8_kernels.py:842-978).
 * x (M, 2N) bf16 = [w1 | w3]; y (M, N) e4m3 = quant(silu(w1) * w3) per 1 x block,
 * s (M, N/block) f32.  N % block == 0, block == 128. */
/* FP8 block GEMM (B stored (N, K)) plus a multi-LoRA delta in the same fp32
 * accumulator: C = A8 B8^T (block-scaled, as fd_fp8_gemm_blockwise) + lora_a lora_b^T
 * (+ bias), one rounding to c_dtype.  lora_a (M, lora_k) bf16 holds the per-token
 * scaled mid activations s_j (x A_j^T) of every adapter j side by side, lora_b
 * (N, lora_k) bf16 the adapters' B_j side by side; lora_k a positive multiple of 64
 * (zero-padded).  K may be 0 (delta only).  Replaces the base linear + the adapter
 * loop of MultiLoRALinear (src_ii/multi_lora.py:231-325) and the Triton
 * _multi_lora_kernel (src/futudiffu/lora_kernels.py:55-157). */
int fd_fp8_gemm_blockwise_lora(const void* a, const float* a_s, const void* b, const float* b_s,
                               const void* bias, int bias_dtype, void* c, int c_dtype, int64_t M,
                               int64_t N, int64_t K, const void* lora_a, const void* lora_b,
                               int64_t lora_k, void* stream);

/* GEMM with a quantising epilogue: c (M, N) e4m3 codes and c_s (M, N/128) fp32
 * dequant scales, 1 x 128 groups, from A (M, K) e4m3 + a_s and B e4m3 (K-major) + b_s
 * (128 x 128 blocks), optional bias (added in fp32).  N and K multiples of 128.
 *   act FD_ACT_NONE:      requantise the fp32 accumulator; replaces fp8_gemm_quant
 *                         (src/futudiffu/fp8_kernels.py:573-709).
 *   act FD_ACT_GELU_TANH: bf16(acc) -> GELU(tanh) -> quantise; replaces
 *                         fp8_addmm_blockwise followed by the GELU-tanh quantiser.
 *   act FD_ACT_SILU_GATE: B = [w1; w3] of shape (2 N, K), b_s (2 N/128, K/128), bias 2 N;
 *                         silu(bf16(w1 acc)) * bf16(w3 acc) -> quantise; replaces the FFN
 *                         chain head fp8_addmm -> fp8_silu_gate_quant
 *                         (src_ii/transformer.py:536-545, fp8_kernels.py:842-978).
 * Codes and scales equal those of the replaced kernel pair. */
#define FD_ACT_NONE 0
#define FD_ACT_GELU_TANH 1
#define FD_ACT_SILU_GATE 2
int fd_fp8_gemm_quant(const void* a, const float* a_s, const void* b, const float* b_s,
                      const void* bias, int bias_dtype, void* c, float* c_s, int64_t M, int64_t N,
                      int64_t K, int act, void* stream);
/* Two FP8 block GEMMs with the same epilogue in one persistent launch (each
 * problem C = A B^T as fd_fp8_gemm_blockwise with b_layout 0, or quantised as
 * fd_fp8_gemm_quant): the tiles of both are scheduled together, so a small
 * problem (the text stream of a double-stream block, M = 512 per sample) does
 * not leave most SMs idle.  act: FD_GEMM_STORE_BF16 (bf16 C) or FD_ACT_*
 * (1 x 128 e4m3 C + c_s).  bias: both or neither, bf16.  No counterpart in the
 * reference (one GEMM launch per linear). */
#define FD_GEMM_STORE_BF16 (-1)
typedef struct fd_gemm_problem {
  const void* a;     /* (M, K) e4m3 */
  const float* a_s;  /* (M, K / 128) */
  const void* b;     /* (N, K) e4m3 ((2 N, K) for FD_ACT_SILU_GATE) */
  const float* b_s;  /* (N / 128, K / 128) */
  const void* bias;  /* (N,) bf16 or NULL */
  void* c;           /* (M, N) bf16, or e4m3 codes */
  float* c_s;        /* (M, N / 128) when quantising */
  int64_t M, N, K;
} fd_gemm_problem;
int fd_fp8_gemm_grouped2(const fd_gemm_problem* p0, const fd_gemm_problem* p1, int bias_dtype, int act,
                         void* stream);

/* fd_fp8_gemm_quant writing into a column window of wider rows: output row m
 * starts at c + m * ldc (codes, ldc a multiple of 16) and c_s + m * ldcs. */
int fd_fp8_gemm_quant_ld(const void* a, const float* a_s, const void* b, const float* b_s,
                         const void* bias, int bias_dtype, void* c, float* c_s, int64_t M, int64_t N,
                         int64_t K, int act, int64_t ldc, int64_t ldcs, void* stream);

int fd_fp8_silu_gate_quant(const void* x, void* y, float* s, int64_t M, int64_t N, int block,
                           void* stream);

/* GELU(tanh approximation) + 1 x block fp8 quantisation of a bf16 tensor
 * (the MMDiT MLP activation; same quantiser formula as G1). */
int fd_fp8_gelu_tanh_quant(const void* x, void* y, float* s, int64_t M, int64_t N, int block,
                           void* stream);

/* fp8_gelu (src/futudiffu/fp8_kernels.py:716-833): dequant -> erf-GELU -> requant.
 * x (M, N) e4m3 with sx (M, N/block); y (M, N) e4m3 with sy (M, N/block). */
int fd_fp8_gelu_requant(const void* x, const float* sx, void* y, float* sy, int64_t M, int64_t N,
                        int block, void* stream);

/* P1 -- fused_rms_norm_modulate (src/futudiffu/fused_kernels.py:43-86, :155-197).
 * x (B, S, dim) bf16; w (dim) in w_dtype; scale (B, dim) in scale_dtype;
 * out (B, S, dim) bf16 = rmsnorm(x) * w * (1 + scale[b]). */
int fd_rms_norm_modulate(const void* x, const void* w, int w_dtype, const void* scale,
                         int scale_dtype, void* out, int64_t B, int64_t S, int64_t dim, float eps,
                         void* stream);

/* RMSNorm-modulate (as fd_rms_norm_modulate) with the 1 x 128 e4m3 activation
 * quantiser fused into the same pass: y (B, S, dim) e4m3 codes, y_s (B, S, dim/128)
 * fp32 dequant scales, equal to fd_rms_norm_modulate followed by fd_fp8_act_quant
 * code for code.  No single counterpart in the reference (it runs the pair
 * fused_rms_norm_modulate -> fp8_act_quant, fused_kernels.py:43-86 and
 * fp8_kernels.py:54-90); dim a multiple of 128. */
int fd_rms_norm_modulate_quant(const void* x, const void* w, int w_dtype, const void* scale,
                               int scale_dtype, void* y, float* y_s, int64_t B, int64_t S,
                               int64_t dim, float eps, void* stream);

/* P2 -- fused_rms_norm_gate_residual (src/futudiffu/fused_kernels.py:99-148, :200-247).
 * out = residual + tanh(gate[b]) * rmsnorm(x) * w. */
int fd_rms_norm_gate_residual(const void* x, const void* w, int w_dtype, const void* gate,
                              int gate_dtype, const void* residual, void* out, int64_t B,
                              int64_t S, int64_t dim, float eps, void* stream);

/* P1 / P1 + G1 / P2 for a packed multi-image sequence with per-image adaLN
 * (P4: the per-token path of JointTransformerBlock.forward,
 * src_ii/transformer.py:656-677, whose per-token scale / gate rows are the
 * per-image rows scattered by document_id, src_ii/zimage_model.py:496-512).
 * x, residual, out: (rows, dim); scale / gate: (n_params, dim).  Rows
 * [range_rows[i], range_rows[i + 1]) use parameter row range_param[i];
 * range_rows (n_ranges + 1) and range_param (n_ranges) are int32 device arrays.
 * Ranges that leave [0, rows) or name a row outside [0, n_params) are skipped;
 * rows covered by no range are not written.  The reference runs this path
 * unfused in torch bf16. */
int fd_rms_norm_modulate_ranges(const void* x, const void* w, int w_dtype, const void* scale,
                                int scale_dtype, void* out, int64_t rows, int64_t dim, float eps,
                                const int32_t* range_rows, const int32_t* range_param,
                                int64_t n_ranges, int64_t n_params, void* stream);
int fd_rms_norm_modulate_quant_ranges(const void* x, const void* w, int w_dtype, const void* scale,
                                      int scale_dtype, void* y, float* y_s, int64_t rows, int64_t dim,
                                      float eps, const int32_t* range_rows, const int32_t* range_param,
                                      int64_t n_ranges, int64_t n_params, void* stream);
int fd_rms_norm_gate_residual_ranges(const void* x, const void* w, int w_dtype, const void* gate,
                                     int gate_dtype, const void* residual, void* out, int64_t rows,
                                     int64_t dim, float eps, const int32_t* range_rows,
                                     const int32_t* range_param, int64_t n_ranges, int64_t n_params,
                                     void* stream);

/* P3 -- fused_qkv_postprocess (src/futudiffu/fused_kernels.py:270-471).
 * qkv (B*S, 3*H*hd) bf16; qw, kw (hd) f32; freqs (B*S, hd/2, 2, 2) f32;
 * oq, ok, ov (B, H, S, hd) bf16.  hd == 128. */
int fd_qkv_postprocess(const void* qkv, const float* qw, const float* kw, const float* freqs,
                       void* oq, void* ok, void* ov, int64_t B, int64_t S, int64_t H, int64_t hd,
                       float eps, void* stream);
/* fd_qkv_postprocess writing Q, K, V rows [s_off, s_off + S) of (B, H, S_out, 128)
 * buffers, so the streams of a joint attention land in one buffer without a copy.
 * No counterpart in the reference. */
int fd_qkv_postprocess_into(const void* qkv, const float* qw, const float* kw, const float* freqs,
                            void* oq, void* ok, void* ov, int64_t B, int64_t S, int64_t H,
                            int64_t hd, float eps, int64_t S_out, int64_t s_off, void* stream);

/* A1..A4 -- attention quantisation prologue.
 * Replaces _smooth_k (src/futudiffu/sage_attention.py:63-71) and the in-kernel
 * Q/K quantisation of the attention kernels (sage_kernels.py:632-639,
 * :656-663 int8; :151-155, :176-179 fp8) plus V quantisation (:1146-1151).
 * q, k, v: (BH, N, 128) bf16.
 *  smooth_k: subtract the bf16-rounded per-(bh, d) mean over N from K,
 *            rounding the difference to bf16 (torch bf16 semantics).
 *  qk_kind:  FD_QK_INT8 / FD_QK_FP8.
 *  q_gran / k_gran: FD_GRAN_TOKEN (per row) or FD_GRAN_BLOCK (128 Q rows,
 *            64 K rows).
 *  pv_kind:  FD_PV_BF16 (v_codes/v_desc unused) or FD_PV_FP8 (V -> e4m3 with
 *            one scale per (bh, d) over the whole sequence).
 * Outputs: q_codes/k_codes (BH, N, 128) int8|e4m3; q_desc (BH, nq) f32 with
 * sm_scale_log2e folded in (nq = N or ceil(N/128)); k_desc (BH, nk) f32
 * (nk = N or ceil(N/64)); v_codes (BH, N, 128) e4m3; v_desc (BH, 128) f32;
 * k_mean (BH, 128) f32 (the bf16-rounded mean, for inspection; may be NULL).
 * workspace: f32 scratch of fd_attn_quant_workspace_floats(BH, N) elements. */
int64_t fd_attn_quant_workspace_floats(int64_t BH, int64_t N);
int fd_attn_quant(const void* q, const void* k, const void* v, int64_t BH, int64_t N,
                  int smooth_k, int qk_kind, int q_gran, int k_gran, int pv_kind,
                  float sm_scale_log2e, void* q_codes, float* q_desc, void* k_codes,
                  float* k_desc, void* v_codes, float* v_desc, float* k_mean, float* workspace,
                  void* stream);

/* P3 fused with the attention prologue, for (joint) attention inputs straight
 * from the QKV linear.  No single counterpart in the reference, which runs
 * fused_qkv_postprocess (fused_kernels.py:270-471) and then quantises Q/K/V
 * inside every attention kernel (sage_kernels.py:632-663 and siblings); the
 * codes and scales equal fd_qkv_postprocess_into followed by fd_attn_quant
 * (the K smoothing mean is summed in another order, so it may differ from
 * fd_attn_quant's by one bf16 rounding in rare columns).
 *  fd_qkv_postprocess_quant, once per stream: qkv (B, S, 3 H 128) bf16 ->
 *    Q codes (B H, N, 128) + q_desc (as fd_attn_quant's), K and V bf16 into
 *    rows [s_off, s_off + S) of the joint (B, H, N, 128) buffers, and this
 *    stream's K column sums / V column absmax (V only for FD_PV_FP8) into the
 *    workspace.  s_off must be a multiple of 128 and every stream but the one
 *    ending at N must hold a multiple of 128 rows.
 *  fd_attn_quant_kv, once after every stream: K smoothing mean, K codes +
 *    k_desc, and for FD_PV_FP8 the e4m3 V codes + v_desc (as fd_attn_quant).
 * workspace: fd_qkv_quant_workspace_floats(B H, N) floats shared by both. */
int64_t fd_qkv_quant_workspace_floats(int64_t BH, int64_t N);
int fd_qkv_postprocess_quant(const void* qkv, const float* qw, const float* kw, const float* freqs, int64_t B,
                             int64_t S, int64_t H, float eps, int64_t N, int64_t s_off, int qk_kind, int q_gran,
                             int pv_kind, float sm_scale_log2e, void* q_codes, float* q_desc, void* k_out,
                             void* v_out, float* workspace, void* stream);
int fd_attn_quant_kv(const void* k, const void* v, int64_t BH, int64_t N, int smooth_k, int qk_kind, int k_gran,
                     int pv_kind, void* k_codes, float* k_desc, void* v_codes, float* v_desc, float* k_mean,
                     float* workspace, void* stream);

/* The QKV linear(s) of a joint attention with P3 and fd_qkv_postprocess_quant in
 * the GEMM's epilogue: the bf16 Q/K/V never go to HBM before the prologue reads
 * them.  No counterpart in the reference (fp8_gemm_blockwise, fused_qkv_postprocess
 * and the attention kernels' quantisation, fp8_kernels.py:195-227,
 * fused_kernels.py:270-471, sage_kernels.py:632-663).  Equal, code for code, to
 * fd_fp8_gemm_blockwise (bf16 output) followed by fd_qkv_postprocess_quant for
 * each stream; run fd_attn_quant_kv after it.  One problem per stream (p1 / s1
 * NULL for a single stream, else the two run as one launch): a (B S, K) e4m3,
 * b = the stream's QKV weight (3 H 128, K) e4m3 (rows [Q heads | K heads | V
 * heads]), bias bf16 or NULL on both; c / c_s unused.  S and s_off multiples of
 * 128, H even; outputs and workspace as fd_qkv_postprocess_quant's. */
typedef struct fd_qkv_stream {
  const float* q_norm;  /* (128,) f32 */
  const float* k_norm;  /* (128,) f32 */
  const float* freqs;   /* (B S, 64, 2, 2) f32 RoPE rotations of the stream's rows */
  int64_t S;            /* rows per sample */
  int64_t s_off;        /* first joint row of the stream */
  float eps;
} fd_qkv_stream;
int fd_fp8_gemm_qkv_quant(const fd_gemm_problem* p0, const fd_qkv_stream* s0, const fd_gemm_problem* p1,
                          const fd_qkv_stream* s1, int bias_dtype, int64_t B, int64_t H, int64_t N, int qk_kind,
                          int q_gran, int pv_kind, float sm_scale_log2e, void* q_codes, float* q_desc, void* k_out,
                          void* v_out, float* workspace, void* stream);

/* V for FD_PV_FP8_TILE (reference _sage_attn_fwd_fp8qk_fp8pv_lse,
 * src/futudiffu/sage_kernels.py:1142-1148): v (BH, N, 128) bf16 -> v_codes
 * (BH, N, 128) e4m3 and v_desc (BH, ceil(N/64), 128) f32, per 64-row tile and
 * column: v_desc = amax / 448, code = e4m3(v * (448 / max(amax, 1e-12))); rows
 * past N count as 0. */
int fd_attn_quant_v_tile(const void* v, int64_t BH, int64_t N, void* v_codes, float* v_desc, void* stream);

/* No counterpart in the reference.  fd_attn_quant with no workspace argument:
 * the scratch lives in a fixed device array inside the library (one per GPU
 * that loads it, FD_NOALLOC_WS_FLOATS floats = 4 MiB, held until exit), so
 * this entry point allocates nothing.  Meant for callers that cannot allocate
 * device memory (hosts that pass only their planned input/output buffers, or
 * paths where cudaMalloc's synchronisation is not allowed).  Rejects shapes
 * whose scratch, 2 * BH * ceil(N/256) * 128 floats, exceeds the array
 * (FD_ERR_ARG), as it rejects N >= 2^30 or BH > 65535.  The first call in a
 * CUDA context (the device's primary context, or one the caller made current)
 * looks up the array's device address for that context; make it before any
 * stream capture.  Calls share the array: calls that overlap on one GPU race.
 * fd_attn_quant_noalloc_max_floats() returns the array size. */
#define FD_NOALLOC_WS_FLOATS 1048576
int64_t fd_attn_quant_noalloc_max_floats(void);
int fd_attn_quant_noalloc(const void* q, const void* k, const void* v, int64_t BH, int64_t N,
                          int smooth_k, int qk_kind, int q_gran, int k_gran, int pv_kind,
                          float sm_scale_log2e, void* q_codes, float* q_desc, void* k_codes,
                          float* k_desc, void* v_codes, float* v_desc, float* k_mean,
                          void* stream);

/* A5/A6 -- quantized attention forward
 * (production kernel _sage_attn_fwd_int8qk_bf16pv_masked_lse,
 *  src/futudiffu/sage_kernels.py:1379-1477, and its unmasked / fp8 siblings).
 * Consumes the prologue outputs.  v is bf16 (BH, N, 128) when pv_kind ==
 * FD_PV_BF16, else the e4m3 codes with v_desc.  block_mask: uint8
 * (ceil(N/128), ceil(N/64)) per head at mask_bh_stride bytes (0 = broadcast),
 * or NULL.  out (BH, N, 128) bf16; lse (BH, N) f32 in log2 units (may be NULL). */
int fd_sage_attn_fwd(const void* q_codes, const float* q_desc, const void* k_codes,
                     const float* k_desc, const void* v, const float* v_desc,
                     const uint8_t* block_mask, int64_t mask_bh_stride, void* out, float* lse,
                     int64_t BH, int64_t N, int qk_kind, int q_gran, int k_gran, int pv_kind,
                     void* stream);
/* fd_sage_attn_fwd with out laid out (BH / H, N, H, 128), i.e. (B, N, H * 128): the
 * input layout of the output projection, so no transpose follows the kernel.
 * No counterpart in the reference. */
int fd_sage_attn_fwd_bnhd(const void* q_codes, const float* q_desc, const void* k_codes,
                          const float* k_desc, const void* v, const float* v_desc,
                          const uint8_t* block_mask, int64_t mask_bh_stride, void* out, float* lse,
                          int64_t BH, int64_t N, int64_t H, int qk_kind, int q_gran, int k_gran,
                          int pv_kind, void* stream);

/* fd_sage_attn_fwd_bnhd whose output is the output linear's quantised input:
 * every (token row, head) of the (B, N, H * 128) output is one 1 x 128 group,
 * written as e4m3 codes + an fp32 dequant scale, equal to fd_fp8_act_quant of
 * the bf16 output code for code.  Rows n < split go to region 0, rows n >= split
 * to region 1 (e.g. the text and image streams of a joint attention); region r
 * holds its rows of every sample consecutively, row stride code_stride_r bytes
 * (a multiple of 16, >= H * 128) and scale_stride_r floats (>= H).  split == N
 * leaves region 1 unused.  Replaces sage_attn_masked_op -> reshape ->
 * fp8_act_quant (src_ii/transformer.py:462-470, fp8.py:64); no counterpart
 * kernel in the reference. */
int fd_sage_attn_fwd_quant_out(const void* q_codes, const float* q_desc, const void* k_codes,
                               const float* k_desc, const void* v, const float* v_desc,
                               const uint8_t* block_mask, int64_t mask_bh_stride, float* lse, int64_t BH,
                               int64_t N, int64_t H, int qk_kind, int q_gran, int k_gran, int pv_kind,
                               void* codes0, float* scales0, int64_t code_stride0, int64_t scale_stride0,
                               void* codes1, float* scales1, int64_t code_stride1, int64_t scale_stride1,
                               int64_t split, void* stream);

/* A7 -- attention backward, Delta pre-pass (sage_kernels.py:322-349):
 * delta (BH, N) f32 = rowsum(dO * O). */
int fd_sage_attn_bwd_prepass(const void* dout, const void* out, float* delta, int64_t BH,
                             int64_t N, void* stream);

/* A7 -- attention backward on the tensor cores (sage_kernels.py:805-1015 int8,
 * :1491-1722 masked int8, :356-567 fp8).  Recomputes P = exp2((S q_desc) k_desc - lse)
 * from the same per-token Q/K codes the forward used (per-block scales expanded to
 * per-token arrays, row stride round_up(N, 128)), then dV = P^T dO,
 * dS = P (dO V^T - delta), dK = sm_scale dS^T Q, dQ = sm_scale dS K with bf16
 * operands and fp32 accumulation in TMEM: a dK / dV kernel (one CTA per 128-key
 * tile over 64-query steps) and a dQ kernel (one CTA per 128-query tile over
 * 64-key steps); masked (128 x 64) tiles are skipped.  q, k (smoothed), v, dout,
 * dq, dk, dv: (BH, N, 128) bf16, 16-byte aligned; any N. */
int fd_sage_attn_bwd(const void* q, const void* k, const void* v, const void* dout,
                     const float* lse, const float* delta, const void* q_codes,
                     const float* q_desc, const void* k_codes, const float* k_desc,
                     const uint8_t* block_mask, int64_t mask_bh_stride, void* dq, void* dk,
                     void* dv, int64_t BH, int64_t N, int qk_kind, float sm_scale, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* FD_B200_H */

/*
 * intcrush_b200 -- C ABI of the B200 (sm_100a) quantized-linear forward path.
 *
 * Every entry point takes raw device pointers, sizes, strides (in elements
 * unless the name says bytes) and a cudaStream_t (passed as void*; NULL =
 * legacy default stream).  Nothing is allocated, nothing synchronises the
 * host: each call only enqueues kernels on `stream`, so all of them can be
 * captured into a CUDA graph.  Each returns IC_OK or an IC_ERR_* code; the
 * matching message is available from ic_last_error() on the calling thread.
 *
 * The reference interface that each entry point replaces is cited as
 * path:line inside the ComfyUI-INT-Crush project.
 */
#ifndef INTCRUSH_B200_H_
#define INTCRUSH_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define IC_OK 0
#define IC_ERR_ARG 1          /* bad shape / stride / pointer / alignment  */
#define IC_ERR_UNSUPPORTED 2  /* valid request outside what is built      */
#define IC_ERR_CUDA 3         /* a CUDA runtime or driver call failed     */

/* device-side error word (ic_read_device_error) */
#define IC_DEV_ERR_NONE 0
#define IC_DEV_ERR_TIMEOUT 1  /* a bounded mbarrier wait expired          */

/* element type codes */
#define IC_DTYPE_F16 0
#define IC_DTYPE_BF16 1
#define IC_DTYPE_F32 2

/* weight kinds for ic_gemm_a8 */
#define IC_W_INT8 0           /* int8  [N, K], row stride ldw bytes         */
#define IC_W_INT4 1           /* uint8 [N, K/2] two signed nibbles per byte,
                                 low nibble = even k (two's complement)     */
#define IC_W_INT4R 2          /* same shape, ic_repack_int4 layout 0        */

/* Library version, (major << 16) | minor. */
int ic_version(void);

/* Message for the last error returned on this host thread ("" if none). */
const char* ic_last_error(void);

/* Read (and optionally clear) the device error word of the current device.
 * Synchronises the device: test/diagnostic use only. */
int ic_read_device_error(int clear, int* code_out);

/*
 * (a1) Activation prep + dynamic per-token INT8 quantisation, one HBM pass.
 *
 * Replaces Linear._prep_activation (_ops.py:337-365), rotate_activations
 * (_quant_utils.py:117-147), the INT8 smooth divide (_ops.py:529-533) and
 * dynamic_quantize_activation (kernels/triton_quantize.py:151-198).
 *
 *   x         [M, K] f16/bf16, row stride ldx              (read)
 *   smoothrot [K] fp32 or NULL: x /= fp16(smoothrot) before the rotation
 *   rot_size  0 (no rotation) or a power of two in [2, 4096]; powers of 4 use
 *             the regular Hadamard kron(H4/2), others the Sylvester one
 *   w_in      output width; the rotated row (K rounded up to rot_size) is
 *             zero-padded to w_in (w_in >= that width)
 *   perm      [w_in] int32 or NULL: out[:, j] = padded[:, perm[j]]
 *   smooth    [w_in] fp32 or NULL: out /= fp16(smooth) after the gather
 *   x_int8    [M, ldq] int8 or NULL (ldq >= w_in, ldq % 16 == 0); columns
 *             [w_in, ldq) are written with zeros
 *   s_a       [M] fp32 (required when x_int8 is given): max(amax,1e-8)/127
 *   x_prep    [M, w_in] in x's dtype or NULL: the prepped activations
 *   rowsum    [M] fp32 or NULL: sum of the prepped row (zero-point term)
 * Quantisation is q = clamp(rint(x / s), -128, 127) with IEEE division, i.e.
 * the CPU form kernels/triton_quantize.py:43-54 (round half to even).
 */
int ic_prep_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                  const float* smoothrot, int rot_size, int64_t w_in, const int32_t* perm,
                  const float* smooth, int8_t* x_int8, int64_t ldq, float* s_a,
                  void* x_prep, float* rowsum, void* stream);

/* ic_prep_quant preceded by a row normalisation, in the same pass:
 *   norm 1 (LayerNorm): x' = (x - mean) * rstd * gamma + beta (beta may be NULL)
 *   norm 2 (RMSNorm):   x' = x / sqrt(mean(x^2) + eps) * gamma
 * with fp32 row statistics, x' rounded once to x's dtype, then SmoothRot,
 * rotation (rot_size 0 or 16..256), padding, gather and quantisation as in
 * ic_prep_quant (no SmoothQuant factors).  norm 0 is ic_prep_quant.
 * Replaces fused_layernorm_quantize / fused_rmsnorm_quantize
 * (kernels/triton_quantize.py:208-451; rot_size 0, no perm), following their
 * CPU form (normalised values cast to the activation dtype, then
 * kernels/triton_quantize.py:43-54), and extends them with the layer's prep.
 * gamma, beta: fp32 [K]. */
int ic_prep_quant_norm(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int norm,
                       const float* gamma, const float* beta, float eps, const float* smoothrot,
                       int rot_size, int64_t w_in, const int32_t* perm, int8_t* x_int8, int64_t ldq,
                       float* s_a, void* x_prep, float* rowsum, void* stream);

/* dynamic_quantize_activation (kernels/triton_quantize.py:151-198): the
 * special case of ic_prep_quant with no smoothing, rotation or gather. */
int ic_dynamic_quantize(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                        int8_t* x_int8, int64_t ldq, float* s_a, void* stream);

/*
 * (a2, a3) INT8-activation GEMM with fused dequant on tcgen05 (kind::i8):
 *
 *   out[m, n] = s_a[m] * sum_g s_w[n, g] * (sum_{k in g} xq[m, k] * w[n, k])
 *               + bias[n] - rowsum[m] * zp_corr[n]
 *
 * Replaces fused_int8_gemm_dequant (kernels/triton_int8_gemm.py:135-205),
 * fused_w4a8_gemm_dequant (kernels/triton_w4a8_gemm.py:111-169) together
 * with unpack_int4_to_int8 (kernels/triton_int4_to_int8_unpack.py:55-81):
 * INT4 weights are unpacked inside the kernel, never materialised.
 *
 *   xq      [M, K] int8, row stride ldq bytes (ldq % 16 == 0)
 *   w       IC_W_INT8: int8 [N, K] (ldw % 16 == 0, K % 16 == 0)
 *           IC_W_INT4: uint8 [N, ceil(K/2)] (ldw % 16 == 0, K % 32 == 0)
 *           IC_W_INT4R: as IC_W_INT4 in ic_repack_int4 layout 0 (faster)
 *   s_w     fp32 [N, G] row-major; G == 1 is per-channel, G > 1 groups of
 *           group_size consecutive k (group_size % 128 == 0); the group form
 *           follows _quant_utils.py:255-270
 *   s_a     fp32 [M]
 *   bias    [N] in bias_dtype or NULL
 *   rowsum, zp_corr  fp32 [M], fp32 [N] or both NULL (zero-point term of
 *           _ops.py:459-461)
 *   out     [M, N] in out_dtype (f16/bf16/f32), row stride ldo
 */
int ic_gemm_a8(const int8_t* xq, int64_t M, int64_t K, int64_t ldq,
               const void* w, int w_kind, int64_t N, int64_t ldw,
               const float* s_w, int64_t G, int64_t group_size, const float* s_a,
               const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr,
               void* out, int out_dtype, int64_t ldo, void* stream);

/* Split-K form of ic_gemm_a8 for few output tiles (small M): the K range is
 * cut into `splits` equal parts (ceil(K/128) % splits == 0; with group scales
 * also K % group_size == 0 and G % splits == 0), each (tile, part) pair runs
 * as its own work unit and writes fp32 partials (scaled by s_a and s_w) to
 * `workspace` ([splits, M, N], at least splits*M*N floats, caller-owned,
 * contents need not be initialised); a second kernel sums the parts and adds
 * bias and the zero-point term.  Same result as ic_gemm_a8 up to fp32
 * summation order.  splits in [1, 16].  Extends fused_int8_gemm_dequant /
 * fused_w4a8_gemm_dequant (kernels/triton_int8_gemm.py:135-205,
 * kernels/triton_w4a8_gemm.py:111-169), which have no split-K form. */
int ic_gemm_a8_splitk(const int8_t* xq, int64_t M, int64_t K, int64_t ldq,
                      const void* w, int w_kind, int64_t N, int64_t ldw,
                      const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                      const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr,
                      void* out, int out_dtype, int64_t ldo, int splits,
                      float* workspace, int64_t workspace_elems, void* stream);

/* ic_gemm_a8_splitk with the optional epilogue of fused_int8_gemm_dequant
 * (kernels/triton_int8_gemm.py:119-129, :135-205): after dequantisation,
 * bias and zero-point term,
 *   activation 0 none, 1 SiLU x*sigmoid(x), 2 GELU 0.5x(1+erf(x/sqrt 2)),
 *              3 GELU with the tanh approximation (Flux-class MLPs),
 * then + residual[m, n] (residual_dtype f16/bf16/f32, row stride ldr; NULL
 * for none).  splits 1 needs no workspace. */
int ic_gemm_a8_ex(const int8_t* xq, int64_t M, int64_t K, int64_t ldq,
                  const void* w, int w_kind, int64_t N, int64_t ldw,
                  const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                  const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr,
                  int activation, const void* residual, int residual_dtype, int64_t ldr,
                  void* out, int out_dtype, int64_t ldo, int splits,
                  float* workspace, int64_t workspace_elems, void* stream);

/* INT8-out GEMM for chained layers (int8_gemm_int8out,
 * kernels/triton_int8_gemm.py:402-536), with a row-global scale instead of
 * the reference's per-tile one: y = act(dequant GEMM + bias) in fp32,
 * s_c[m] = max(max_n |y[m, n]|, 1e-8) / 127, c = rint(y / s_c) (ties to even,
 * clamped), so that (c, s_c) is exactly what dynamic quantisation of the fp32
 * output would give.  workspace: M*N + M floats (the fp32 values and the row
 * maxima).  c [M, ldc] int8, s_c [M] fp32. */
int ic_gemm_a8_int8out(const int8_t* xq, int64_t M, int64_t K, int64_t ldq,
                       const void* w, int w_kind, int64_t N, int64_t ldw,
                       const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                       const void* bias, int bias_dtype, int activation,
                       int8_t* c, int64_t ldc, float* s_c,
                       float* workspace, int64_t workspace_elems, void* stream);

/* Requantise a float weight on the device, as the layout classes' quantize
 * (quant_layout.py:100-129 INT4, :179-200 INT8) that set_weight calls
 * (_ops.py:770-807): per row amax = max|w|; bits 4: scale fp16
 * fp16(max(amax/7, 1e-8)), q = clamp(rint(w / scale), -8, 7) packed two per
 * byte (low nibble = even column, odd K padded with 0), q [N, ldq >=
 * ceil(K/2)] uint8; bits 8: scale fp32 max(amax/127, 1e-8),
 * q = clamp(rint(w / scale), -128, 127), q [N, ldq >= K] int8.  IEEE
 * division, ties to even; a 0/0 quotient stores 0.  w [N, ldw] fp32. */
int ic_quantize_weight(const float* w, int64_t N, int64_t K, int64_t ldw, int bits,
                       void* q, int64_t ldq, void* scale, void* stream);

/* LoKr residual in place (_apply_lokr, _ops.py:88-138):
 * out[t] viewed [out_l, out_k] += scale * (w1 @ X_t) @ w2^T, X_t = x[t]
 * viewed [in_m, in_n]; w1 [out_l, in_m], w2 [out_k, in_n] (the combined
 * factors; the reference's w2_t is w2 transposed).  temp = T(w1 @ X_t) is
 * rounded to the activation dtype as the reference's matmul does, then
 * out = T(out + scale * temp @ w2^T) with fp32 sums.  out contiguous
 * [M, N = out_l*out_k]; x [M, ldx], K = in_m*in_n; in_n <= 256,
 * out_l*in_m <= 12288; temp holds M*out_l*in_n elements of dtype. */
int ic_lokr_add(void* out, int dtype, int64_t M, int64_t N, const void* x, int64_t ldx, int64_t K,
                const void* w1, int64_t out_l, int64_t in_m, const void* w2, int64_t out_k, int64_t in_n,
                float scale, void* temp, int64_t temp_elems, void* stream);

/* ic_gemm_a8_splitk with no allocation and no caller workspace.  No
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they run the GEMM -- a C or FFI host without a device
 * allocator of its own, a process whose device memory is fully reserved by
 * another framework's pool, or a path where cudaMalloc is not allowed because
 * it can synchronise the device.  The partials go to a scratch array built
 * into the library (IC_NOALLOC_SCRATCH_FLOATS floats = 8 MiB, held on every
 * GPU that loads the library until the process exits); calls that would need
 * more (splits * M * N floats) are rejected with IC_ERR_ARG before any work is
 * queued.  The first call in a CUDA context (normally the device's primary
 * context) looks up the scratch address for that context
 * (cudaGetSymbolAddress, with the device current); make that first call
 * before any stream capture.  Every call shares the one array and the GEMM
 * overwrites every element the reduce reads, so nothing needs clearing, but
 * calls whose GPU work overlaps (different streams, or different host threads
 * on one device) race on it: serialise them.  Arguments as ic_gemm_a8_splitk
 * without the workspace. */
#define IC_NOALLOC_SCRATCH_FLOATS 2097152
int ic_gemm_a8_splitk_noalloc(const int8_t* xq, int64_t M, int64_t K, int64_t ldq,
                              const void* w, int w_kind, int64_t N, int64_t ldw,
                              const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                              const void* bias, int bias_dtype, const float* rowsum,
                              const float* zp_corr, void* out, int out_dtype, int64_t ldo,
                              int splits, void* stream);

/*
 * (a4) W4A16: out = x @ dequant(w)^T with fp32 accumulation, fused bias and
 * low-rank term
 *   out = T(T(x @ W^T + bias) + lr_scale * lr_mid @ lr_up^T)
 * (the second rounding reproduces the reference's separate addmm_), T the
 * activation dtype.  fp16: dequant(w)[n,k] = fp16(q[n,k] * fp16(s[n, g])),
 * the Triton unpack's product (kernels/triton_int4_unpack.py:48-56); bf16:
 * bf16(q[n,k] * s[n, g]) from the fp32 product, the PyTorch path's
 * dequantisation cast to the activation dtype (quant_layout.py:81-87,
 * _ops.py:483-491).
 *
 * Replaces unpack_int4_to_float16 (kernels/triton_int4_unpack.py:62-88) +
 * F.linear (_ops.py:473-474), the PyTorch INT4 path (_ops.py:483-491) and the
 * LoRA residual (_ops.py:236-244) for standard LoRA.
 *
 *   x      [M, K] fp16 or bf16 (x_dtype), row stride ldx
 *   w      uint8 [N, ceil(K/2)], row stride ldw bytes; w_layout 0 = the
 *          reference packing, 1 = ic_repack_int4 layout 1 (faster)
 *   scale  [N, G] in scale_dtype (f16 or f32), group_size % 128 == 0 when G > 1
 *   bias   [N] or NULL
 *   lr_mid [M, R], lr_up [N, R] in x_dtype (R <= 256) or NULL
 *   out    [M, N] in x_dtype, row stride ldo
 */
int ic_gemm_w4a16(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                  const uint8_t* w, int64_t N, int64_t ldw, int w_layout,
                  const void* scale, int scale_dtype, int64_t G, int64_t group_size,
                  const void* bias, int bias_dtype,
                  const void* lr_mid, const void* lr_up, int64_t R, float lr_scale,
                  void* out, int64_t ldo, void* stream);

/* ic_gemm_w4a16 with split-K for the M > 128 (tcgen05) path: the 64-wide K
 * blocks are cut into `splits` equal parts (1..8, dividing ceil(K / 64)),
 * each run as its own work unit writing fp32 partials to workspace
 * [splits, M, N]; a reduce kernel forms out = T(sum + bias).  splits = 0
 * picks the count that fills the SMs with one unit each (token tiles of
 * 128), falling back to 1 when workspace is NULL or smaller than
 * splits * M * N floats.  Replaces the same callables as ic_gemm_w4a16
 * (_ops.py:466-481 with kernels/triton_int4_unpack.py:62-88 + F.linear);
 * the reference has no split form.  M <= 128 ignores splits (weight-stream
 * kernel). */
int ic_gemm_w4a16_splitk(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                         const uint8_t* w, int64_t N, int64_t ldw, int w_layout,
                         const void* scale, int scale_dtype, int64_t G, int64_t group_size,
                         const void* bias, int bias_dtype,
                         const void* lr_mid, const void* lr_up, int64_t R, float lr_scale,
                         void* out, int64_t ldo, int splits, float* workspace,
                         int64_t workspace_elems, void* stream);

/* Low-rank "down" projection mid = T(x @ down^T) with fp32 accumulation
 * (_ops.py:242, F.linear in the activation dtype T): x [M, K] (ldx),
 * down [R, K], mid [M, R], all in dtype (IC_DTYPE_F16 or IC_DTYPE_BF16). */
int ic_lowrank_down_ex(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, const void* down,
                       int64_t R, void* mid, void* stream);
/* ic_lowrank_down_ex with dtype IC_DTYPE_F16. */
int ic_lowrank_down(const void* x, int64_t M, int64_t K, int64_t ldx, const void* down,
                    int64_t R, void* mid, void* stream);

/* In-place low-rank residual out = T(out + scale * mid @ up^T), fp32 sums
 * (out.addmm_ of _ops.py:243 / :384): out [M, N] (ldo), mid [M, R],
 * up [N, R], all in dtype (f16 or bf16); R <= 256. */
int ic_lowrank_add_ex(void* out, int dtype, int64_t M, int64_t N, int64_t ldo, const void* mid,
                      const void* up, int64_t R, float scale, void* stream);
/* ic_lowrank_add_ex with dtype IC_DTYPE_F16. */
int ic_lowrank_add(void* out, int64_t M, int64_t N, int64_t ldo, const void* mid,
                   const void* up, int64_t R, float scale, void* stream);

/* Self-test of the kernels' bounded waits (no counterpart in the
 * reference; failure detection): launches one thread that waits on an
 * mbarrier nothing arrives on, gives up after limit_ns (<= 0.1 s), records
 * IC_DEV_ERR_TIMEOUT in the device error word (ic_read_device_error) and
 * returns.  The context stays usable. */
int ic_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* Load-time weight repack.  The reference's packing (_quant_utils.py:
 * 170-182) stays the input format; this permutes the nibbles of each 4-byte
 * word (8 consecutive k) so the GEMMs expand INT4 with shifts and masks only.
 * layout 0 (for ic_gemm_a8, IC_W_INT4R): byte b of a word = q[b] | q[b+4] << 4;
 * layout 1 (for ic_gemm_w4a16, w_layout 1): nibble t = q[2t] + 8, nibble t+4 =
 * q[2t+1] + 8.  src/dst [N, ceil(K/2)] uint8 with row strides lds/ldd; src and
 * dst must not overlap. */
int ic_repack_int4(const uint8_t* src, int64_t N, int64_t K, int64_t lds, uint8_t* dst, int64_t ldd,
                   int layout, void* stream);

/* unpack_int4_to_int8 (kernels/triton_int4_to_int8_unpack.py:55-81):
 * packed [N, ldp bytes] -> out int8 [N, K] (row stride K). */
int ic_unpack_int4_to_int8(const uint8_t* packed, int64_t N, int64_t K, int64_t ldp,
                           int8_t* out, void* stream);

/* unpack_int4_to_float16 (kernels/triton_int4_unpack.py:62-88), extended to
 * group scales: out[n,k] = fp16(q * fp16(scale[n, k // group_size])). */
int ic_unpack_int4_to_f16(const uint8_t* packed, int64_t N, int64_t K, int64_t ldp,
                          const void* scale, int scale_dtype, int64_t G, int64_t group_size,
                          void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* INTCRUSH_B200_H_ */

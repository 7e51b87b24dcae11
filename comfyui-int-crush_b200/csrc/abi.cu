// extern "C" entry points of libintcrush_b200.so (declared in
// include/intcrush_b200.h).  Each validates its arguments, launches on the
// caller's stream and returns a status code; no exception crosses the ABI.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <math.h>

#include <mutex>

#include "ic_common.cuh"

namespace {

thread_local char g_err[512] = "";

__device__ __forceinline__ void mbar_init_for_selftest(uint64_t* bar) {
  ic::mbar_init(bar, 1);
  ic::fence_barrier_init();
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return IC_OK;
  return fail(IC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool is_pow2(long long v) { return v > 0 && (v & (v - 1)) == 0; }
bool is_pow4(long long v) { return v >= 4 && is_pow2(v) && (v & 0x55555555LL) == v; }
int ilog2(long long v) { int r = 0; while ((1LL << r) < v) ++r; return r; }

// fp16(fp32(1/sqrt(n))): the Sylvester entry as the reference materialises it
// (fp16 tensor times a Python float, _quant_utils.py:112).
double sylvester_entry(int n) {
  const float f = (float)(1.0 / sqrt((double)n));
  return (double)__half2float(__float2half_rn(f));
}

}  // namespace

extern "C" {

int ic_version(void) { return (1 << 16) | 0; }

#if defined(IC_TRACE)
int ic_trace_read(unsigned long long* out, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, ic::g_ic_trace, sizeof(unsigned long long) * 16);
  if (clear) { unsigned long long z[16] = {0}; cudaMemcpyToSymbol(ic::g_ic_trace, z, sizeof(z)); }
  return e == cudaSuccess ? 0 : 3;
}
#endif

const char* ic_last_error(void) { return g_err; }

// Self-test of the bounded waits: one thread waits on an mbarrier that
// nothing arrives on, with a limit of limit_ns, so the wait runs out the way
// a stuck pipeline's would and records IC_DEV_ERR_TIMEOUT in the device
// error word; the kernel then returns normally.  No fault, no trap.
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init_for_selftest(&bar);
  const uint64_t t0 = ic::globaltimer();
  while (!ic::mbar_try_wait(&bar, 0)) {
    if (ic::globaltimer() - t0 > limit_ns) {
      ic::set_dev_error(IC_DEV_ERR_TIMEOUT);
      break;
    }
  }
}

int ic_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  g_err[0] = 0;
  if (limit_ns <= 0 || limit_ns > 100000000LL)
    return fail(IC_ERR_ARG, "ic_selftest_wait_timeout: limit must be in (0, 0.1 s]");
  selftest_wait_kernel<<<1, 1, 0, (cudaStream_t)stream>>>((uint64_t)limit_ns);
  return cuda_status(cudaGetLastError(), "ic_selftest_wait_timeout launch");
}

int ic_read_device_error(int clear, int* code_out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_ic_dev_error, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "reading the device error word");
  if (clear && v) {
    const int z = 0;
    e = cudaMemcpyToSymbol(g_ic_dev_error, &z, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clearing the device error word");
  }
  if (code_out) *code_out = v;
  return IC_OK;
}

static int prep_impl(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int norm, const float* gamma,
                     const float* beta, float eps, const float* smoothrot, int rot_size, int64_t w_in,
                     const int32_t* perm, const float* smooth, int8_t* x_int8, int64_t ldq, float* s_a,
                     void* x_prep, float* rowsum, void* stream) {
  g_err[0] = 0;
  if (x_dtype != IC_DTYPE_F16 && x_dtype != IC_DTYPE_BF16)
    return fail(IC_ERR_ARG, "ic_prep_quant: x dtype must be f16 or bf16");
  if (M < 0 || K <= 0 || ldx < K) return fail(IC_ERR_ARG, "ic_prep_quant: bad M/K/ldx (%lld, %lld, %lld)",
                                              (long long)M, (long long)K, (long long)ldx);
  if (M == 0) return IC_OK;
  if (!x) return fail(IC_ERR_ARG, "ic_prep_quant: x is NULL");
  if (rot_size != 0 && (!is_pow2(rot_size) || rot_size < 2 || rot_size > 4096))
    return fail(IC_ERR_ARG, "ic_prep_quant: rot_size must be 0 or a power of two in [2, 4096], got %d", rot_size);
  const int64_t Kr = rot_size ? ((K + rot_size - 1) / rot_size) * rot_size : K;
  if (w_in < Kr) return fail(IC_ERR_ARG, "ic_prep_quant: w_in (%lld) < rotated width (%lld)",
                             (long long)w_in, (long long)Kr);
  if (x_int8) {
    if (!s_a) return fail(IC_ERR_ARG, "ic_prep_quant: s_a is required with x_int8");
    if (ldq < w_in || (ldq % 16) != 0 || !aligned16(x_int8))
      return fail(IC_ERR_ARG, "ic_prep_quant: ldq must be >= w_in, a multiple of 16, and x_int8 16-byte aligned");
  }
  if (!x_int8 && !x_prep && !rowsum) return fail(IC_ERR_ARG, "ic_prep_quant: no output requested");
  if (w_in > 65536 || M > 0x7fffffffLL) return fail(IC_ERR_UNSUPPORTED, "ic_prep_quant: w_in > 65536 or M >= 2^31");
  if (norm < 0 || norm > 2) return fail(IC_ERR_ARG, "ic_prep_quant_norm: norm must be 0, 1 (layer) or 2 (rms)");
  if (norm && !gamma) return fail(IC_ERR_ARG, "ic_prep_quant_norm: gamma is required with a norm");
  if (norm == 2 && beta) return fail(IC_ERR_ARG, "ic_prep_quant_norm: RMSNorm takes no beta");
  if (norm && smooth) return fail(IC_ERR_UNSUPPORTED, "ic_prep_quant_norm: a norm with SmoothQuant factors is not built");
  if (norm && rot_size && (rot_size < 16 || rot_size > 256))
    return fail(IC_ERR_UNSUPPORTED, "ic_prep_quant_norm: with a norm, rot_size must be 0 or in [16, 256]");
  ic::PrepArgs a;
  memset(&a, 0, sizeof(a));
  a.norm = norm; a.gamma = gamma; a.beta = beta; a.eps = eps;
  a.x = x; a.M = M; a.K = K; a.ldx = ldx; a.smoothrot = smoothrot; a.w_in = w_in; a.perm = perm;
  a.smooth = smooth; a.xq = x_int8; a.ldq = ldq; a.s_a = s_a; a.x_prep = x_prep; a.rowsum = rowsum;
  a.Kr = Kr; a.Wp = Kr > w_in ? Kr : w_in;
  a.syl_h = (rot_size && !is_pow4(rot_size)) ? sylvester_entry(rot_size) : 0.0;
  a.vec_ok = aligned16(x) && (ldx % 8 == 0);
  const int log2r = rot_size ? ilog2(rot_size) : 0;
  const bool syl = rot_size && !is_pow4(rot_size);
  return cuda_status(ic::launch_prep(a, x_dtype, log2r, syl, (cudaStream_t)stream), "ic_prep_quant launch");
}

int ic_prep_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const float* smoothrot,
                  int rot_size, int64_t w_in, const int32_t* perm, const float* smooth, int8_t* x_int8,
                  int64_t ldq, float* s_a, void* x_prep, float* rowsum, void* stream) {
  return prep_impl(x, x_dtype, M, K, ldx, 0, nullptr, nullptr, 0.f, smoothrot, rot_size, w_in, perm, smooth,
                   x_int8, ldq, s_a, x_prep, rowsum, stream);
}

int ic_prep_quant_norm(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int norm,
                       const float* gamma, const float* beta, float eps, const float* smoothrot, int rot_size,
                       int64_t w_in, const int32_t* perm, int8_t* x_int8, int64_t ldq, float* s_a, void* x_prep,
                       float* rowsum, void* stream) {
  return prep_impl(x, x_dtype, M, K, ldx, norm, gamma, beta, eps, smoothrot, rot_size, w_in, perm, nullptr,
                   x_int8, ldq, s_a, x_prep, rowsum, stream);
}

int ic_dynamic_quantize(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int8_t* x_int8,
                        int64_t ldq, float* s_a, void* stream) {
  return ic_prep_quant(x, x_dtype, M, K, ldx, nullptr, 0, K, nullptr, nullptr, x_int8, ldq, s_a, nullptr,
                       nullptr, stream);
}

struct EpiArgs {
  int act = 0;
  const void* residual = nullptr;
  int residual_dtype = 0;
  int64_t ldr = 0;
  float* rowmax = nullptr;
};

static int gemm_a8_impl(const char* fn, const int8_t* xq, int64_t M, int64_t K, int64_t ldq, const void* w, int w_kind, int64_t N,
               int64_t ldw, const float* s_w, int64_t G, int64_t group_size, const float* s_a,
               const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr, void* out,
               int out_dtype, int64_t ldo, int splits, float* ws, int64_t ws_elems,
                        void* stream, const EpiArgs& epi = EpiArgs()) {
  g_err[0] = 0;
  if (epi.act < 0 || epi.act > 3) return fail(IC_ERR_ARG, "%s: activation must be 0 (none), 1 (SiLU), 2 (GELU) or 3 (GELU tanh)", fn);
  if (epi.residual && (epi.residual_dtype < IC_DTYPE_F16 || epi.residual_dtype > IC_DTYPE_F32 || epi.ldr < N))
    return fail(IC_ERR_ARG, "%s: residual needs a dtype code and ldr >= N", fn);
  if (M < 0 || N < 0 || K <= 0) return fail(IC_ERR_ARG, "%s: bad M/N/K", fn);
  if (M == 0 || N == 0) return IC_OK;
  if (!xq || !w || !s_w || !s_a || !out) return fail(IC_ERR_ARG, "%s: NULL operand", fn);
  if (w_kind != IC_W_INT8 && w_kind != IC_W_INT4 && w_kind != IC_W_INT4R) return fail(IC_ERR_ARG, "%s: bad w_kind", fn);
  if (out_dtype < IC_DTYPE_F16 || out_dtype > IC_DTYPE_F32) return fail(IC_ERR_ARG, "%s: bad out dtype", fn);
  if (bias && (bias_dtype < IC_DTYPE_F16 || bias_dtype > IC_DTYPE_F32)) return fail(IC_ERR_ARG, "%s: bad bias dtype", fn);
  if ((rowsum == nullptr) != (zp_corr == nullptr)) return fail(IC_ERR_ARG, "%s: rowsum and zp_corr go together", fn);
  if (ldq < K || ldq % 16 || !aligned16(xq)) return fail(IC_ERR_ARG, "%s: xq needs ldq >= K, ldq %% 16 == 0, 16-byte alignment", fn);
  if (!aligned16(w) || ldw % 16) return fail(IC_ERR_ARG, "%s: weights need 16-byte aligned base and row stride", fn);
  if (w_kind == IC_W_INT8 && (K % 16 || ldw < K)) return fail(IC_ERR_ARG, "%s: int8 weights need K %% 16 == 0 and ldw >= K", fn);
  if (w_kind != IC_W_INT8 && (K % 32 || ldw < K / 2)) return fail(IC_ERR_ARG, "%s: int4 weights need K %% 32 == 0 and ldw >= K/2", fn);
  if (ldo < N) return fail(IC_ERR_ARG, "%s: ldo < N", fn);
  if (G < 1) return fail(IC_ERR_ARG, "%s: G must be >= 1", fn);
  if (G > 1) {
    if (group_size <= 0 || group_size % 128) return fail(IC_ERR_UNSUPPORTED, "%s: group_size must be a multiple of 128", fn);
    if ((K + group_size - 1) / group_size != G) return fail(IC_ERR_ARG, "%s: G != ceil(K / group_size)", fn);
    if (w_kind == IC_W_INT8 && group_size > 128)
      return fail(IC_ERR_UNSUPPORTED, "%s: int8 weights with group scales need group_size == 128", fn);
    // INT4 is held as 16*q inside the kernel; a group's int32 partial is then
    // at most 2^22 in magnitude for 256-wide groups, the limit of the exact
    // int -> float hand-off (1.5*2^23 + P must keep its exponent).
    if (w_kind != IC_W_INT8 && group_size > 256)
      return fail(IC_ERR_UNSUPPORTED, "%s: int4 weights with group scales need group_size 128 or 256", fn);
    // every group must span whole 128-wide K blocks, the last one included
    if (((K + 127) / 128) % (group_size / 128) != 0)
      return fail(IC_ERR_UNSUPPORTED, "%s: ceil(K / 128) must be a multiple of group_size / 128", fn);
  }
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return fail(IC_ERR_UNSUPPORTED, "%s: dims >= 2^31", fn);
  ic::GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.G = (int)G; a.kb_per_group = G > 1 ? (int)(group_size / 128) : 0; a.group_size = (int)group_size;
  a.s_w = s_w; a.s_a = s_a; a.bias = bias; a.bias_dtype = bias_dtype; a.rowsum = rowsum; a.zp_corr = zp_corr;
  a.out = out; a.out_dtype = out_dtype; a.ldo = ldo;
  a.w_repacked = (w_kind == IC_W_INT4R);
  if (splits < 1 || splits > 16) return fail(IC_ERR_ARG, "%s: splits must be in [1, 16]", fn);
  if (splits > 1) {
    const int64_t nkb = (K + 127) / 128;
    if (nkb % splits) return fail(IC_ERR_ARG, "%s: ceil(K / 128) must be a multiple of splits", fn);
    if (G > 1 && (K % group_size || G % splits))
      return fail(IC_ERR_ARG, "%s: with group scales, K %% group_size == 0 and G %% splits == 0", fn);
    // M, N < 2^31 and splits <= 16 here: the product fits in 128 bits
    if (!ws || (__int128)ws_elems < (__int128)splits * M * N)
      return fail(IC_ERR_ARG, "%s: workspace needs splits*M*N floats", fn);
  }
  a.splits = splits;
  a.ws = ws;
  a.act = epi.act; a.residual = epi.residual; a.residual_dtype = epi.residual_dtype; a.ldr = epi.ldr;
  a.rowmax = epi.rowmax;
  const char* why = "kernel launch";
  const int force_bn = 0;
  cudaError_t e = ic::launch_gemm_a8(xq, (int)M, (int)K, ldq, w, w_kind == IC_W_INT8 ? IC_W_INT8 : IC_W_INT4, (int)N, ldw, a, force_bn,
                                     (cudaStream_t)stream, &why);
  return cuda_status(e, why);
}

int ic_gemm_a8(const int8_t* xq, int64_t M, int64_t K, int64_t ldq, const void* w, int w_kind, int64_t N,
               int64_t ldw, const float* s_w, int64_t G, int64_t group_size, const float* s_a,
               const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr, void* out,
               int out_dtype, int64_t ldo, void* stream) {
  return gemm_a8_impl("ic_gemm_a8", xq, M, K, ldq, w, w_kind, N, ldw, s_w, G, group_size, s_a, bias, bias_dtype,
                      rowsum, zp_corr, out, out_dtype, ldo, 1, nullptr, 0, stream);
}

int ic_gemm_a8_splitk(const int8_t* xq, int64_t M, int64_t K, int64_t ldq, const void* w, int w_kind, int64_t N,
                      int64_t ldw, const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                      const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr, void* out,
                      int out_dtype, int64_t ldo, int splits, float* workspace, int64_t workspace_elems,
                      void* stream) {
  return gemm_a8_impl("ic_gemm_a8_splitk", xq, M, K, ldq, w, w_kind, N, ldw, s_w, G, group_size, s_a, bias,
                      bias_dtype, rowsum, zp_corr, out, out_dtype, ldo, splits, workspace, workspace_elems, stream);
}

int ic_gemm_a8_ex(const int8_t* xq, int64_t M, int64_t K, int64_t ldq, const void* w, int w_kind, int64_t N,
                  int64_t ldw, const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                  const void* bias, int bias_dtype, const float* rowsum, const float* zp_corr, int activation,
                  const void* residual, int residual_dtype, int64_t ldr, void* out, int out_dtype, int64_t ldo,
                  int splits, float* workspace, int64_t workspace_elems, void* stream) {
  EpiArgs e;
  e.act = activation; e.residual = residual; e.residual_dtype = residual_dtype; e.ldr = ldr;
  return gemm_a8_impl("ic_gemm_a8_ex", xq, M, K, ldq, w, w_kind, N, ldw, s_w, G, group_size, s_a, bias,
                      bias_dtype, rowsum, zp_corr, out, out_dtype, ldo, splits, workspace, workspace_elems, stream, e);
}

int ic_gemm_a8_int8out(const int8_t* xq, int64_t M, int64_t K, int64_t ldq, const void* w, int w_kind, int64_t N,
                       int64_t ldw, const float* s_w, int64_t G, int64_t group_size, const float* s_a,
                       const void* bias, int bias_dtype, int activation, int8_t* c, int64_t ldc, float* s_c,
                       float* workspace, int64_t workspace_elems, void* stream) {
  const char* fn = "ic_gemm_a8_int8out";
  g_err[0] = 0;
  if (M < 0 || N < 0) return fail(IC_ERR_ARG, "%s: bad M/N", fn);
  if (M == 0 || N == 0) return IC_OK;
  if (!c || !s_c || !workspace) return fail(IC_ERR_ARG, "%s: NULL output or workspace", fn);
  if (ldc < N) return fail(IC_ERR_ARG, "%s: ldc < N", fn);
  if (M > 0x7fffffffLL || N > 0x7fffffffLL) return fail(IC_ERR_UNSUPPORTED, "%s: dims >= 2^31", fn);
  // workspace: the fp32 epilogue values [M, N], then the row maxima [M]
  if ((__int128)workspace_elems < (__int128)M * N + M) return fail(IC_ERR_ARG, "%s: workspace needs M*N + M floats", fn);
  float* y = workspace;
  float* rowmax = workspace + M * N;
  cudaError_t er = cudaMemsetAsync(rowmax, 0, (size_t)M * sizeof(float), (cudaStream_t)stream);
  if (er != cudaSuccess) return cuda_status(er, "clearing the row maxima");
  EpiArgs e;
  e.act = activation; e.rowmax = rowmax;
  const int st = gemm_a8_impl(fn, xq, M, K, ldq, w, w_kind, N, ldw, s_w, G, group_size, s_a, bias, bias_dtype,
                              nullptr, nullptr, y, IC_DTYPE_F32, N, 1, nullptr, 0, stream, e);
  if (st != IC_OK) return st;
  return cuda_status(ic::launch_requant_rows(y, (int)M, (int)N, N, rowmax, c, ldc, s_c, (cudaStream_t)stream),
                     "ic_gemm_a8_int8out requantisation launch");
}

// ---------------------------------------------------------------------------
// Split-K A8 GEMM without any allocation.
//
// Some callers cannot allocate device memory at the moment they run this
// GEMM: a plain C or FFI host that has no device allocator of its own to hand
// out a workspace, a process whose device memory is already fully reserved by
// another framework's pool, or a latency-critical path where cudaMalloc is not
// allowed because it can synchronise the whole device.  For them the split-K
// partials live in this file-scope array instead of a caller workspace.  Every
// GPU that loads the library holds it until the process exits.
static __device__ __align__(256) float g_splitk_scratch[IC_NOALLOC_SCRATCH_FLOATS];

namespace {
std::mutex g_scratch_mu;
// Device address of g_splitk_scratch per CUDA context.  An address is valid
// only in the context that produced it, so the cache is keyed on the current
// context (cuCtxGetCurrent, fetched through the runtime so that the library
// does not link libcuda), not on the device index: a host that drives the
// device through its own driver-API context, or that reset the device, gets
// the address of its own context.
struct ScratchEntry { void* ctx; float* ptr; };
ScratchEntry g_scratch[64];
int g_scratch_used = 0;
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
}  // namespace

static void* current_context() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (CtxGetCurrentFn) nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return (void*)c;
}

// Host code sees g_splitk_scratch only as a host-side stand-in: its device
// address is asked for once per context, with the caller's device current.
static int scratch_for_current_device(const char* fn, float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  (void)dev;
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  for (int i = 0; ctx && i < g_scratch_used; ++i)
    if (g_scratch[i].ctx == ctx) { *out = g_scratch[i].ptr; return IC_OK; }
  // first call in this context (the runtime makes the device's primary
  // context current here if nothing was current yet)
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_splitk_scratch);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress of the split-K scratch");
  if (!ctx) ctx = current_context();
  if (ctx && g_scratch_used < 64) g_scratch[g_scratch_used++] = ScratchEntry{ctx, static_cast<float*>(p)};
  *out = static_cast<float*>(p);
  return IC_OK;
}

int ic_gemm_a8_splitk_noalloc(const int8_t* xq, int64_t M, int64_t K, int64_t ldq, const void* w, int w_kind,
                              int64_t N, int64_t ldw, const float* s_w, int64_t G, int64_t group_size,
                              const float* s_a, const void* bias, int bias_dtype, const float* rowsum,
                              const float* zp_corr, void* out, int out_dtype, int64_t ldo, int splits,
                              void* stream) {
  const char* fn = "ic_gemm_a8_splitk_noalloc";
  g_err[0] = 0;
  if (M < 0 || N < 0 || splits < 1 || splits > 16) return fail(IC_ERR_ARG, "%s: bad M/N/splits", fn);
  // compared without forming splits * M * N first (it could overflow int64)
  if (splits > 1 && N > 0 && M > (int64_t)IC_NOALLOC_SCRATCH_FLOATS / splits / N)
    return fail(IC_ERR_ARG, "%s: splits*M*N (%d * %lld * %lld) exceeds the built-in scratch of %lld floats", fn,
                splits, (long long)M, (long long)N, (long long)IC_NOALLOC_SCRATCH_FLOATS);
  float* ws = nullptr;
  if (splits > 1 && M > 0 && N > 0) {
    const int st = scratch_for_current_device(fn, &ws);
    if (st != IC_OK) return st;
  }
  return gemm_a8_impl(fn, xq, M, K, ldq, w, w_kind, N, ldw, s_w, G, group_size, s_a, bias, bias_dtype, rowsum,
                      zp_corr, out, out_dtype, ldo, splits, ws, (int64_t)IC_NOALLOC_SCRATCH_FLOATS, stream);
}

static int gemm_w4a16_impl(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const uint8_t* w,
                           int64_t N, int64_t ldw, int w_layout, const void* scale, int scale_dtype, int64_t G,
                           int64_t group_size, const void* bias, int bias_dtype, const void* lr_mid,
                           const void* lr_up, int64_t R, float lr_scale, void* out, int64_t ldo, int splits,
                           float* ws, int64_t ws_elems, void* stream) {
  g_err[0] = 0;
  if (x_dtype != IC_DTYPE_F16 && x_dtype != IC_DTYPE_BF16)
    return fail(IC_ERR_UNSUPPORTED, "ic_gemm_w4a16: x must be fp16 or bf16");
  if (M < 0 || N < 0 || K <= 0 || ldx < K || ldo < N) return fail(IC_ERR_ARG, "ic_gemm_w4a16: bad sizes");
  if (M == 0 || N == 0) return IC_OK;
  if (!x || !w || !scale || !out) return fail(IC_ERR_ARG, "ic_gemm_w4a16: NULL operand");
  if (scale_dtype != IC_DTYPE_F16 && scale_dtype != IC_DTYPE_F32) return fail(IC_ERR_ARG, "ic_gemm_w4a16: scale dtype");
  if (G < 1) return fail(IC_ERR_ARG, "ic_gemm_w4a16: G must be >= 1");
  if (G > 1 && (group_size <= 0 || group_size % 128 || (K + group_size - 1) / group_size != G))
    return fail(IC_ERR_UNSUPPORTED, "ic_gemm_w4a16: group_size must be a multiple of 128 with G == ceil(K/group_size)");
  if (ldw < (K + 1) / 2) return fail(IC_ERR_ARG, "ic_gemm_w4a16: ldw < ceil(K/2)");
  if (w_layout != 0 && w_layout != 1) return fail(IC_ERR_ARG, "ic_gemm_w4a16: w_layout must be 0 or 1");
  if ((lr_mid == nullptr) != (lr_up == nullptr)) return fail(IC_ERR_ARG, "ic_gemm_w4a16: lr_mid and lr_up go together");
  if (lr_mid && (R <= 0 || R > 256)) return fail(IC_ERR_UNSUPPORTED, "ic_gemm_w4a16: low-rank R must be in [1, 256]");
  const cudaStream_t st = (cudaStream_t)stream;
  static const int skinny_max = [] {
    const char* e = getenv("INTCRUSH_W4A16_SKINNY_MAX");   // tuning only
    return e ? atoi(e) : 128;   // measured crossover with the tcgen05 path (3072 x 3072)
  }();
  if (M <= skinny_max) {
    ic::SkinnyArgs s;
    s.x = x; s.M = (int)M; s.K = (int)K; s.ldx = ldx; s.w = w; s.N = (int)N; s.ldw = ldw;
    s.scale = scale; s.scale_dtype = scale_dtype; s.G = (int)G; s.group_size = (int)group_size;
    s.bias = bias; s.bias_dtype = bias_dtype; s.lr_mid = lr_mid; s.lr_up = lr_up;
    s.R = (int)R; s.lr_scale = lr_scale; s.out = out; s.ldo = ldo; s.repacked = w_layout;
    return cuda_status(ic::launch_w4a16_skinny(s, x_dtype, st), "ic_gemm_w4a16 (small M) launch");
  }
  if (K % 64 || ldx % 8 || !aligned16(x) || ldw % 16 || !aligned16(w))
    return fail(IC_ERR_UNSUPPORTED, "ic_gemm_w4a16: M > 128 needs K %% 64 == 0 and 16-byte aligned rows");
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
    return fail(IC_ERR_UNSUPPORTED, "ic_gemm_w4a16: dims >= 2^31");
  ic::GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.G = (int)G; a.group_size = (int)group_size; a.w_scale = scale; a.w_scale_dtype = scale_dtype;
  a.bias = bias; a.bias_dtype = bias_dtype; a.out = out; a.out_dtype = x_dtype; a.ldo = ldo;
  a.w_repacked = w_layout;
  int force_bn = 0;
  if (splits < 0 || splits > 8) return fail(IC_ERR_ARG, "ic_gemm_w4a16_splitk: splits must be in [0, 8]");
  if (splits == 0) {
    ic::plan_w4a16_splits((int)M, (int)N, (int)K, &force_bn, &splits);
    // the plan needs a workspace; without one (or too small a one) the GEMM runs unsplit
    if (splits > 1 && (!ws || (__int128)ws_elems < (__int128)splits * M * N)) { splits = 1; force_bn = 0; }
    if (splits == 1) force_bn = 0;
  } else if (splits > 1) {
    if (((K + 63) / 64) % splits) return fail(IC_ERR_ARG, "ic_gemm_w4a16_splitk: ceil(K / 64) must be a multiple of splits");
    if (!ws || (__int128)ws_elems < (__int128)splits * M * N)
      return fail(IC_ERR_ARG, "ic_gemm_w4a16_splitk: workspace needs splits*M*N floats");
    force_bn = M <= 64 ? 64 : 128;   // the plan's token tile
  }
  a.splits = splits;
  a.ws = ws;
  const char* why = "kernel launch";
  cudaError_t e = ic::launch_gemm_w4a16_tc(x, x_dtype, (int)M, (int)K, ldx, w, (int)N, ldw, a, force_bn, st, &why);
  if (e != cudaSuccess) return cuda_status(e, why);
  if (lr_mid)
    return cuda_status(ic::launch_lowrank_add(out, x_dtype, (int)M, (int)N, ldo, lr_mid, lr_up, (int)R, lr_scale, st),
                       "ic_gemm_w4a16 low-rank launch");
  return IC_OK;
}

int ic_gemm_w4a16(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const uint8_t* w, int64_t N,
                  int64_t ldw, int w_layout, const void* scale, int scale_dtype, int64_t G, int64_t group_size,
                  const void* bias, int bias_dtype, const void* lr_mid, const void* lr_up, int64_t R,
                  float lr_scale, void* out, int64_t ldo, void* stream) {
  return gemm_w4a16_impl(x, x_dtype, M, K, ldx, w, N, ldw, w_layout, scale, scale_dtype, G, group_size, bias,
                         bias_dtype, lr_mid, lr_up, R, lr_scale, out, ldo, 1, nullptr, 0, stream);
}

int ic_gemm_w4a16_splitk(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const uint8_t* w,
                         int64_t N, int64_t ldw, int w_layout, const void* scale, int scale_dtype, int64_t G,
                         int64_t group_size, const void* bias, int bias_dtype, const void* lr_mid,
                         const void* lr_up, int64_t R, float lr_scale, void* out, int64_t ldo, int splits,
                         float* workspace, int64_t workspace_elems, void* stream) {
  return gemm_w4a16_impl(x, x_dtype, M, K, ldx, w, N, ldw, w_layout, scale, scale_dtype, G, group_size, bias,
                         bias_dtype, lr_mid, lr_up, R, lr_scale, out, ldo, splits, workspace, workspace_elems,
                         stream);
}

int ic_lowrank_down_ex(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, const void* down, int64_t R,
                       void* mid, void* stream) {
  g_err[0] = 0;
  if (dtype != IC_DTYPE_F16 && dtype != IC_DTYPE_BF16) return fail(IC_ERR_ARG, "ic_lowrank_down: dtype must be f16 or bf16");
  if (M < 0 || K <= 0 || ldx < K || R <= 0) return fail(IC_ERR_ARG, "ic_lowrank_down: bad sizes");
  if (R > 65535) return fail(IC_ERR_UNSUPPORTED, "ic_lowrank_down: R must be < 65536");
  if (M == 0) return IC_OK;
  if (!x || !down || !mid) return fail(IC_ERR_ARG, "ic_lowrank_down: NULL operand");
  return cuda_status(ic::launch_lowrank_down(x, dtype, (int)M, (int)K, ldx, down, (int)R, mid, (cudaStream_t)stream),
                     "ic_lowrank_down launch");
}

int ic_lowrank_down(const void* x, int64_t M, int64_t K, int64_t ldx, const void* down, int64_t R, void* mid,
                    void* stream) {
  return ic_lowrank_down_ex(x, IC_DTYPE_F16, M, K, ldx, down, R, mid, stream);
}

int ic_lowrank_add_ex(void* out, int dtype, int64_t M, int64_t N, int64_t ldo, const void* mid, const void* up,
                      int64_t R, float scale, void* stream) {
  g_err[0] = 0;
  if (dtype != IC_DTYPE_F16 && dtype != IC_DTYPE_BF16) return fail(IC_ERR_ARG, "ic_lowrank_add: dtype must be f16 or bf16");
  if (M < 0 || N < 0 || ldo < N || R <= 0) return fail(IC_ERR_ARG, "ic_lowrank_add: bad sizes");
  if (R > 256) return fail(IC_ERR_UNSUPPORTED, "ic_lowrank_add: R must be <= 256");
  if (M == 0 || N == 0) return IC_OK;
  if (!out || !mid || !up) return fail(IC_ERR_ARG, "ic_lowrank_add: NULL operand");
  return cuda_status(ic::launch_lowrank_add(out, dtype, (int)M, (int)N, ldo, mid, up, (int)R, scale,
                                            (cudaStream_t)stream),
                     "ic_lowrank_add launch");
}

int ic_lowrank_add(void* out, int64_t M, int64_t N, int64_t ldo, const void* mid, const void* up, int64_t R,
                   float scale, void* stream) {
  return ic_lowrank_add_ex(out, IC_DTYPE_F16, M, N, ldo, mid, up, R, scale, stream);
}

int ic_quantize_weight(const float* w, int64_t N, int64_t K, int64_t ldw, int bits, void* q, int64_t ldq,
                       void* scale, void* stream) {
  g_err[0] = 0;
  if (bits != 4 && bits != 8) return fail(IC_ERR_ARG, "ic_quantize_weight: bits must be 4 or 8");
  if (N < 0 || K < 0 || ldw < K || ldq < (bits == 4 ? (K + 1) / 2 : K))
    return fail(IC_ERR_ARG, "ic_quantize_weight: bad sizes");
  if (N > 0x7fffffffLL || K > 0x7fffffffLL) return fail(IC_ERR_UNSUPPORTED, "ic_quantize_weight: dims >= 2^31");
  if (N == 0) return IC_OK;
  if (!w || !q || !scale) return fail(IC_ERR_ARG, "ic_quantize_weight: NULL operand");
  return cuda_status(ic::launch_quantize_weight(w, (int)N, (int)K, ldw, bits, (uint8_t*)q, ldq, scale,
                                                (cudaStream_t)stream),
                     "ic_quantize_weight launch");
}

int ic_lokr_add(void* out, int dtype, int64_t M, int64_t N, const void* x, int64_t ldx, int64_t K,
                const void* w1, int64_t out_l, int64_t in_m, const void* w2, int64_t out_k, int64_t in_n,
                float scale, void* temp, int64_t temp_elems, void* stream) {
  g_err[0] = 0;
  if (dtype != IC_DTYPE_F16 && dtype != IC_DTYPE_BF16) return fail(IC_ERR_ARG, "ic_lokr_add: dtype must be f16 or bf16");
  if (M < 0 || out_l <= 0 || in_m <= 0 || out_k <= 0 || in_n <= 0 || ldx < K)
    return fail(IC_ERR_ARG, "ic_lokr_add: bad sizes");
  if (out_l * out_k != N || in_m * in_n != K)
    return fail(IC_ERR_ARG, "ic_lokr_add: factor shapes must satisfy out_l*out_k == N and in_m*in_n == K");
  if (in_n > 256) return fail(IC_ERR_UNSUPPORTED, "ic_lokr_add: in_n (the w2 input width) must be <= 256");
  if (out_l * in_m > 12288) return fail(IC_ERR_UNSUPPORTED, "ic_lokr_add: w1 larger than 12288 elements");
  if (M > 0x7fffffffLL / out_l) return fail(IC_ERR_UNSUPPORTED, "ic_lokr_add: M * out_l >= 2^31");
  if (M == 0) return IC_OK;
  if (!out || !x || !w1 || !w2 || !temp) return fail(IC_ERR_ARG, "ic_lokr_add: NULL operand");
  if ((__int128)temp_elems < (__int128)M * out_l * in_n) return fail(IC_ERR_ARG, "ic_lokr_add: temp needs M*out_l*in_n elements");
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = ic::launch_lokr_w1(x, dtype, (int)M, ldx, w1, (int)out_l, (int)in_m, (int)in_n, temp, st);
  if (e != cudaSuccess) return cuda_status(e, "ic_lokr_add w1 launch");
  // rows (t, l) of out viewed [M * out_l, out_k] (out is contiguous [M, N])
  return cuda_status(ic::launch_lowrank_add(out, dtype, (int)(M * out_l), (int)out_k, out_k, temp, w2, (int)in_n,
                                            scale, st),
                     "ic_lokr_add w2 launch");
}

int ic_repack_int4(const uint8_t* src, int64_t N, int64_t K, int64_t lds, uint8_t* dst, int64_t ldd, int layout,
                   void* stream) {
  g_err[0] = 0;
  if (N < 0 || K < 0 || lds < (K + 1) / 2 || ldd < (K + 1) / 2) return fail(IC_ERR_ARG, "ic_repack_int4: bad sizes");
  if (layout != 0 && layout != 1) return fail(IC_ERR_ARG, "ic_repack_int4: layout must be 0 or 1");
  if (N == 0 || K == 0) return IC_OK;
  if (!src || !dst) return fail(IC_ERR_ARG, "ic_repack_int4: NULL operand");
  const uintptr_t s0 = (uintptr_t)src, s1 = s0 + (uintptr_t)(N * lds), d0 = (uintptr_t)dst, d1 = d0 + (uintptr_t)(N * ldd);
  if (s0 < d1 && d0 < s1) return fail(IC_ERR_ARG, "ic_repack_int4: src and dst overlap");
  return cuda_status(ic::launch_repack(src, (int)N, (int)K, lds, dst, ldd, layout, (cudaStream_t)stream),
                     "ic_repack_int4 launch");
}

int ic_unpack_int4_to_int8(const uint8_t* packed, int64_t N, int64_t K, int64_t ldp, int8_t* out, void* stream) {
  g_err[0] = 0;
  if (N < 0 || K < 0 || ldp < (K + 1) / 2) return fail(IC_ERR_ARG, "ic_unpack_int4_to_int8: bad sizes");
  if (N == 0 || K == 0) return IC_OK;
  if (!packed || !out) return fail(IC_ERR_ARG, "ic_unpack_int4_to_int8: NULL operand");
  return cuda_status(ic::launch_unpack_i8(packed, (int)N, (int)K, ldp, out, (cudaStream_t)stream),
                     "ic_unpack_int4_to_int8 launch");
}

int ic_unpack_int4_to_f16(const uint8_t* packed, int64_t N, int64_t K, int64_t ldp, const void* scale,
                          int scale_dtype, int64_t G, int64_t group_size, void* out, void* stream) {
  g_err[0] = 0;
  if (N < 0 || K < 0 || ldp < (K + 1) / 2 || G < 1) return fail(IC_ERR_ARG, "ic_unpack_int4_to_f16: bad sizes");
  if (G > 1 && group_size <= 0) return fail(IC_ERR_ARG, "ic_unpack_int4_to_f16: bad group_size");
  if (N == 0 || K == 0) return IC_OK;
  if (!packed || !scale || !out) return fail(IC_ERR_ARG, "ic_unpack_int4_to_f16: NULL operand");
  return cuda_status(ic::launch_unpack_f16(packed, (int)N, (int)K, ldp, scale, scale_dtype, (int)G,
                                           (int)group_size, (__half*)out, (cudaStream_t)stream),
                     "ic_unpack_int4_to_f16 launch");
}

}  // extern "C"

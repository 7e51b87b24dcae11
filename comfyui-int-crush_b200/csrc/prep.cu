// (a1) Fused activation prep + dynamic per-token INT8 quantisation.
//
// One CTA owns one token row.  The row is read from HBM once (16-byte
// vectors), divided by the SmoothRot factors, rotated group-wise by the block
// Hadamard transform, zero padded, gathered through the PermuQuant
// permutation, divided by the SmoothQuant factors and quantised, and the int8
// row (plus optionally the prepped fp16 row and its sum) is written back with
// 16-byte stores.  All intermediate state lives in shared memory.
//
// Rotation arithmetic.  The reference rotates in the activation dtype with a
// matmul against H^T (ComfyUI-INT-Crush _quant_utils.py:117-147), whose fp32
// accumulation order is unspecified.  Here the butterflies run in fp64: every
// partial sum of at most 4096 fp16 values times +-1 is exact in 53 bits, the
// normalisation is a power of two (regular Hadamard) or one multiply by the
// fp16 Sylvester entry, and the result is rounded to fp16 once.  The output is
// therefore the correctly rounded exact rotation.
//
// Transform structure.  H_regular(4^D) = kron(H4/2, ..., H4/2) with
// H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]] (_quant_utils.py:67-93),
// so it factors into one radix-4 butterfly per base-4 digit of the index:
// y_j = (v0+v1+v2+v3) - 2 v_{3-j}.  The Sylvester matrix (_quant_utils.py:
// 96-114) is kron([[1,1],[1,-1]], ...) and factors into radix-2 butterflies.
// A thread applies up to 4 index bits (16 values) of butterflies in registers
// per pass; passes exchange through a padded fp64 shared buffer.
#include "ic_common.cuh"
#include "prep_common.cuh"


namespace ic {



// Elements of a row rotated per block-wide step (a multiple of the rotation
// size); small enough that several rows fit in one SM's shared memory.
#ifndef IC_PREP_CHUNK
#define IC_PREP_CHUNK 1024
#endif
template <int LOG2R>
constexpr int kPrepChunk = (LOG2R == 0) ? 0 : ((1 << LOG2R) > IC_PREP_CHUNK ? (1 << LOG2R) : IC_PREP_CHUNK);

// Padded fp64 index: one pad slot every 16 values keeps the 16-value
// register blocks of neighbouring threads in different banks.
__device__ __forceinline__ int pidx(int e) { return e + (e >> 4); }

// Rotation arithmetic type: fp64 (exact for sums of fp16 values, see above).
template <typename T> struct RotT { using V = double; };

template <int L, bool SYL, typename V>
__device__ __forceinline__ void butterflies(V (&v)[1 << L]) {
  constexpr int N = 1 << L;
  if constexpr (SYL) {
#pragma unroll
    for (int s = 0; s < L; ++s) {
      const int h = 1 << s;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if ((i & h) == 0) {
          const V a = v[i], b = v[i + h];
          v[i] = a + b;
          v[i + h] = a - b;
        }
      }
    }
  } else {
#pragma unroll
    for (int d = 0; d < L / 2; ++d) {
      const int st = 1 << (2 * d);
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (((i >> (2 * d)) & 3) == 0) {
          const V a0 = v[i], a1 = v[i + st], a2 = v[i + 2 * st], a3 = v[i + 3 * st];
          const V s = (a0 + a1) + (a2 + a3);
          v[i] = s - (a3 + a3);
          v[i + st] = s - (a2 + a2);
          v[i + 2 * st] = s - (a1 + a1);
          v[i + 3 * st] = s - (a0 + a0);
        }
      }
    }
  }
}

// Load x[row, k] (k may be past K: zero), divided by fp16(smoothrot[k]).
template <typename T>
__device__ __forceinline__ float load_x(const PrepArgs& a, const T* xrow, int64_t k) {
  if (k >= a.K) return 0.f;
  float v = DT<T>::to_f(xrow[k]);
  if (a.smoothrot) {
    const float f = DT<T>::to_f(DT<T>::from_f(a.smoothrot[k]));
    v = DT<T>::to_f(DT<T>::from_f(__fdiv_rn(v, f)));
  }
  return v;
}

template <typename V, typename T> __device__ __forceinline__ V to_rot(float f) { return (V)f; }

// Load 16 consecutive inputs starting at k0 (vectorised when legal).
template <typename T, typename V>
__device__ __forceinline__ void load16(const PrepArgs& a, const T* xrow, int64_t k0, V (&v)[16]) {
  if (a.vec_ok && k0 + 16 <= a.K) {
    const uint4* p = reinterpret_cast<const uint4*>(xrow + k0);
    uint4 q0 = __ldg(p), q1 = __ldg(p + 1);
    const T* e0 = reinterpret_cast<const T*>(&q0);
    const T* e1 = reinterpret_cast<const T*>(&q1);
    // the 16 SmoothRot factors as four 16-byte loads (k0 is a multiple of 16)
    float srf[16];
    if (a.smoothrot) {
      if ((reinterpret_cast<uintptr_t>(a.smoothrot) & 15) == 0) {
        const float4* sp = reinterpret_cast<const float4*>(a.smoothrot + k0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 f4 = __ldg(sp + i);
          srf[4 * i] = f4.x; srf[4 * i + 1] = f4.y; srf[4 * i + 2] = f4.z; srf[4 * i + 3] = f4.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) srf[i] = a.smoothrot[k0 + i];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f0 = DT<T>::to_f(e0[j]), f1 = DT<T>::to_f(e1[j]);
      if (a.smoothrot) {
        const float s0 = DT<T>::to_f(DT<T>::from_f(srf[j]));
        const float s1 = DT<T>::to_f(DT<T>::from_f(srf[8 + j]));
        f0 = DT<T>::to_f(DT<T>::from_f(__fdiv_rn(f0, s0)));
        f1 = DT<T>::to_f(DT<T>::from_f(__fdiv_rn(f1, s1)));
      }
      v[j] = to_rot<V, T>(f0);
      v[8 + j] = to_rot<V, T>(f1);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = to_rot<V, T>(load_x<T>(a, xrow, k0 + j));
  }
}

// Block-wide reductions over NT threads.
template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += red[i];
  return r;
}

// One rotation pass over a chunk [c0, c0 + CH) of the row.  The pass covers
// index bits [S, S + L) of each rotation group of size 2^LOG2R.
template <typename T, int LOG2R, bool SYL, int S, int L, bool FIRST, bool LAST, int NT>
__device__ __forceinline__ void rot_pass(const PrepArgs& a, const T* xrow, int c0, int CH,
                                         typename RotT<T>::V* buf, T* xr) {
  using V = typename RotT<T>::V;
  constexpr int R = 1 << LOG2R;
  constexpr int E = 1 << L;
  constexpr int HIGH = R >> (S + L);
  const int items = CH >> L;
  for (int it = threadIdx.x; it < items; it += NT) {
    const int low = it & ((1 << S) - 1);
    const int rest = it >> S;
    const int high = rest % HIGH;
    const int g = rest / HIGH;
    const int base = g * R + low + (high << (S + L));
    V v[E];
    if constexpr (FIRST) {
      static_assert(S == 0, "first pass starts at bit 0");
      if constexpr (E == 16) {
        load16<T, V>(a, xrow, (int64_t)c0 + base, v);
      } else {
#pragma unroll
        for (int j = 0; j < E; ++j) v[j] = to_rot<V, T>(load_x<T>(a, xrow, (int64_t)c0 + base + j));
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = buf[pidx(base + (j << S))];
    }
    butterflies<L, SYL, V>(v);
    if constexpr (LAST) {
#pragma unroll
      for (int j = 0; j < E; ++j) {
        T out;
        if constexpr (SYL) out = DT<T>::from_d(v[j] * a.syl_h);
        else out = DT<T>::from_d(v[j] * (1.0 / (double)(1 << (LOG2R / 2))));   // 2^-D, exact
        xr[c0 + base + (j << S)] = out;
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) buf[pidx(base + (j << S))] = v[j];
    }
  }
}

template <typename T, int LOG2R, bool SYL, int S, int NT>
__device__ __forceinline__ void rot_passes(const PrepArgs& a, const T* xrow, int c0, int CH,
                                           typename RotT<T>::V* buf, T* xr) {
  // bits per pass: 4 (two radix-4 digits / four radix-2 stages); the last
  // pass takes what is left (2 for an odd digit count of a regular size).
  constexpr int REM = LOG2R - S;
  constexpr int L = REM >= 4 ? 4 : REM;
  constexpr bool FIRST = (S == 0);
  constexpr bool LAST = (S + L == LOG2R);
  rot_pass<T, LOG2R, SYL, S, L, FIRST, LAST, NT>(a, xrow, c0, CH, buf, xr);
  if constexpr (!LAST) {
    __syncthreads();
    rot_passes<T, LOG2R, SYL, S + L, NT>(a, xrow, c0, CH, buf, xr);
  }
}

template <typename T, int LOG2R, bool SYL, int NT>
__global__ void __launch_bounds__(NT) prep_quant_kernel(const PrepArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float red[NT / 32];
  const int64_t row = blockIdx.x;
  const T* xrow = reinterpret_cast<const T*>(a.x) + row * a.ldx;

  // layout: [64-bit rotation buffer][xr: Wp values of T][xp: w_in values of T]
  constexpr int CH = kPrepChunk<LOG2R>;
  typename RotT<T>::V* buf = reinterpret_cast<typename RotT<T>::V*>(smem);
  const int buf_bytes = (LOG2R > 4) ? ((CH + CH / 16) * 8) : 0;
  T* xr = reinterpret_cast<T*>(smem + buf_bytes);
  const int Wp = (int)a.Wp, w_in = (int)a.w_in;
  const bool need_xp = (a.perm != nullptr) || (a.smooth != nullptr);
  T* xp = need_xp ? xr + ((Wp + 7) & ~7) : xr;

  // 1. load (+SmoothRot) and rotate into xr[0, Kr)
  if constexpr (LOG2R == 0) {
    for (int k0 = threadIdx.x * 8; k0 < (int)a.K; k0 += NT * 8) {
      if (a.vec_ok && k0 + 8 <= a.K && !a.smoothrot) {
        *reinterpret_cast<uint4*>(xr + k0) = __ldg(reinterpret_cast<const uint4*>(xrow + k0));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < a.K) xr[k0 + j] = DT<T>::from_f(load_x<T>(a, xrow, k0 + j));
      }
    }
  } else {
    const int Kr = (int)a.Kr;
    for (int c0 = 0; c0 < Kr; c0 += CH) {
      const int ch = (Kr - c0) < CH ? (Kr - c0) : CH;   // multiple of the rotation size
      rot_passes<T, LOG2R, SYL, 0, NT>(a, xrow, c0, ch, buf, xr);
      __syncthreads();
    }
  }
  // zero padding [Kr, Wp)
  for (int k = (int)a.Kr + threadIdx.x; k < Wp; k += NT) xr[k] = DT<T>::from_f(0.f);
  __syncthreads();

  // 2. gather + SmoothQuant divide into xp, row absmax (and sum).  Four
  // consecutive outputs per thread per step with 16-byte index / factor loads,
  // unrolled so that the global (L2) loads of all steps are in flight at once.
  float amax = 0.f, rsum = 0.f;
  const bool vec4 = ((w_in & 3) == 0) &&
                    ((reinterpret_cast<uintptr_t>(a.perm) | reinterpret_cast<uintptr_t>(a.smooth)) & 15) == 0;
  auto one = [&](int j, int src, float f_s) {
    T v = xr[src];
    if (a.smooth) v = DT<T>::from_f(__fdiv_rn(DT<T>::to_f(v), f_s));
    if (need_xp) xp[j] = v;
    const float fv = DT<T>::to_f(v);
    amax = fmaxf(amax, fabsf(fv));
    rsum += fv;
  };
  if (vec4) {
#pragma unroll 4
    for (int j0 = threadIdx.x * 4; j0 < w_in; j0 += NT * 4) {
      int4 src = make_int4(j0, j0 + 1, j0 + 2, j0 + 3);
      if (a.perm) src = __ldg(reinterpret_cast<const int4*>(a.perm + j0));
      float4 sm = make_float4(1.f, 1.f, 1.f, 1.f);
      if (a.smooth) sm = __ldg(reinterpret_cast<const float4*>(a.smooth + j0));
      const float f0 = DT<T>::to_f(DT<T>::from_f(sm.x)), f1 = DT<T>::to_f(DT<T>::from_f(sm.y));
      const float f2 = DT<T>::to_f(DT<T>::from_f(sm.z)), f3 = DT<T>::to_f(DT<T>::from_f(sm.w));
      one(j0, src.x, f0);
      one(j0 + 1, src.y, f1);
      one(j0 + 2, src.z, f2);
      one(j0 + 3, src.w, f3);
    }
  } else {
    for (int j = threadIdx.x; j < w_in; j += NT)
      one(j, a.perm ? a.perm[j] : j, a.smooth ? DT<T>::to_f(DT<T>::from_f(a.smooth[j])) : 1.f);
  }
  amax = block_max<NT>(amax, red);
  if (a.rowsum) {
    const float s = block_sum<NT>(rsum, red);
    if (threadIdx.x == 0) a.rowsum[row] = s;
  }
  __syncthreads();   // xp complete

  // 3. prepped row out (optional)
  if (a.x_prep) {
    T* dst = reinterpret_cast<T*>(a.x_prep) + row * (int64_t)w_in;
    const bool vec = ((w_in & 7) == 0) && ((reinterpret_cast<uintptr_t>(a.x_prep) & 15) == 0);
    if (vec) {
      for (int j = threadIdx.x * 8; j < w_in; j += NT * 8)
        *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(xp + j);
    } else {
      for (int j = threadIdx.x; j < w_in; j += NT) dst[j] = xp[j];
    }
  }

  // 4. quantise: s = max(amax, 1e-8) / 127, q = clamp(rint(x / s))
  if (a.xq) {
    const float s = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
    const float rs = __frcp_rn(s);
    if (threadIdx.x == 0) a.s_a[row] = s;
    int8_t* qrow = a.xq + row * a.ldq;
    const int ldq = (int)a.ldq;
    for (int j0 = threadIdx.x * 16; j0 < ldq; j0 += NT * 16) {
      uint32_t wv[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int j = j0 + w * 4 + b;
          int q = 0;
          if (j < w_in) {
            // q = rint(x / s) with the quotient correctly rounded to fp32.
            // x * (1/s) is within 2 fp32 ulps of that quotient, so it rounds
            // to the same integer unless it lies within 2^-21 (relative) of
            // a half-integer; only then is the exact division evaluated.
            // Adding 1.5 * 2^23 rounds to the nearest integer, ties to even
            // (|x / s| <= 127.x), leaving it in the low mantissa bits.
            const float xv = DT<T>::to_f(xp[j]);
            float y = xv * rs;
            const float fy = fabsf(y);
            if (fabsf(fy - (floorf(fy) + 0.5f)) <= fy * 4.8e-7f) y = __fdiv_rn(xv, s);
            q = max(-128, min(127, __float_as_int(y + 12582912.0f) - 0x4B400000));
          }
          word |= ((uint32_t)(q & 0xFF)) << (8 * b);
        }
        wv[w] = word;
      }
      *reinterpret_cast<uint4*>(qrow + j0) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }
}

template <typename T, int LOG2R, bool SYL>
static cudaError_t launch_prep_t(const PrepArgs& a, cudaStream_t st) {
  constexpr int CH = kPrepChunk<LOG2R>;
  const int buf_bytes = (LOG2R > 4) ? ((CH + CH / 16) * 8) : 0;
  const bool need_xp = (a.perm != nullptr) || (a.smooth != nullptr);
  const size_t xr_elems = (size_t)((a.Wp + 7) & ~7LL);
  const size_t smem = buf_bytes + (xr_elems + (need_xp ? (size_t)a.w_in : 0)) * sizeof(T) + 16;
  // one CTA per token row: 64 threads when there are rows enough to fill the
  // GPU several times over, 256 (more parallelism per row) for few rows
  const bool few = a.M < 4 * num_sms();
  auto kern = few ? prep_quant_kernel<T, LOG2R, SYL, 256> : prep_quant_kernel<T, LOG2R, SYL, 64>;
  if (smem > 220 * 1024) return cudaErrorInvalidValue;   // dynamic + static shared memory must fit 227 KB
  if (smem > 48 * 1024) {
    cudaError_t e = set_smem_once(kern, 220 * 1024);
    if (e != cudaSuccess) return e;
  }
  kern<<<(unsigned)a.M, few ? 256 : 64, smem, st>>>(a);
  return cudaGetLastError();
}

constexpr int kPwBufDoubles = 512 + 32;   // per-warp fp64 exchange buffer (pidx(511) = 542)


// INTCRUSH_PREP_V1=1 routes every request to prep_quant_kernel (tests use it
// to check the two kernels against each other).
static bool prep_v1_forced() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("INTCRUSH_PREP_V1");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// ---------------------------------------------------------------------------
// prep_row_kernel: rotation sizes 16..256 without SmoothQuant divide (the
// W4A8 / SmoothRot layout).  Persistent 256-thread CTAs loop over rows; the
// arithmetic and the results are those of prep_quant_kernel (bit-identical),
// with less work per value and one CTA barrier per row in the hot path:
//  * each warp rotates whole 512-value chunks of the row on its own: lane l
//    loads 16 consecutive inputs, applies the butterflies of index bits 0-3 in
//    fp64 registers, exchanges through a warp-private fp64 buffer, finishes
//    the remaining bits and writes the once-rounded values to the row buffer;
//  * the SmoothRot quotient fp16(x / fp16(f)) is x * (1 / fp16(f)) from a
//    per-CTA reciprocal table, except within 4 fp32 ulps of a rounding
//    midpoint of the activation dtype, where the IEEE division is evaluated
//    (the product is within 2 ulps of the correctly rounded quotient, so
//    elsewhere both round to the same value);
//  * the PermuQuant gather runs once: the gathered values stay in registers
//    for the absmax, the optional prepped row / row sum and the quantisation.
constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;

template <typename T, int LOG2R, bool SYL, int MAXIT>
__global__ void __launch_bounds__(kRowThreads) prep_row_kernel(const PrepArgs a, int xr_stride) {
  static_assert(LOG2R == 0 || (LOG2R >= 4 && LOG2R <= 8), "prep_row_kernel covers no rotation and sizes 16..256");
  constexpr bool ROT = LOG2R > 0;
  constexpr int R = 1 << LOG2R;
  constexpr int HB = ROT ? LOG2R - 4 : 0;  // index bits of the second pass
  constexpr int NE = 1 << HB;              // values per second-pass group
  constexpr int GPL = 16 / NE;             // second-pass groups per lane
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float red[2][kRowWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = (int)a.K, Kr = (int)a.Kr, Wp = (int)a.Wp, w_in = (int)a.w_in, ldq = (int)a.ldq;
  double* buf = reinterpret_cast<double*>(smem) + warp * kPwBufDoubles;
  T* xr = reinterpret_cast<T*>(smem + kRowWarps * kPwBufDoubles * 8);
  float* sr = reinterpret_cast<float*>(smem + kRowWarps * kPwBufDoubles * 8 + (size_t)xr_stride * sizeof(T));
  const double scale = SYL ? a.syl_h : 1.0 / (double)(1 << (LOG2R / 2));
  const bool vperm = a.perm && ((w_in & 3) == 0) && ((reinterpret_cast<uintptr_t>(a.perm) & 15) == 0);
  __shared__ float nred[kRowWarps];

  // reciprocals of the SmoothRot factors rounded to the activation dtype
  if (a.smoothrot) {
    for (int k = threadIdx.x; k < K; k += kRowThreads) sr[k] = __frcp_rn(DT<T>::to_f(DT<T>::from_f(a.smoothrot[k])));
  }
  __syncthreads();

  // fp32 sum of v over the CTA (every thread gets it)
  auto block_sum_f = [&](float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) nred[warp] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int w = 0; w < kRowWarps; ++w) r += nred[w];
    __syncthreads();
    return r;
  };

  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x) {
    const T* xrow = reinterpret_cast<const T*>(a.x) + row * a.ldx;
    // ---- optional normalisation statistics (fp32, two passes for LayerNorm)
    float mean = 0.f, rstd = 1.f, rms = 1.f;
    if (a.norm) {
      float s1 = 0.f;
      for (int k = threadIdx.x; k < K; k += kRowThreads) {
        const float f = DT<T>::to_f(xrow[k]);
        s1 += (a.norm == 1) ? f : f * f;
      }
      s1 = block_sum_f(s1);
      if (a.norm == 1) {
        mean = s1 / (float)K;
        float s2 = 0.f;
        for (int k = threadIdx.x; k < K; k += kRowThreads) {
          const float d = DT<T>::to_f(xrow[k]) - mean;
          s2 += d * d;
        }
        s2 = block_sum_f(s2);
        rstd = 1.f / sqrtf(s2 / (float)K + a.eps);
      } else {
        rms = sqrtf(s1 / (float)K + a.eps);
      }
    }
    // ---- rotation into xr[0, Kr): warp w takes chunks w, w + 8, ...
    for (int c0 = warp * 512; c0 < Kr; c0 += kRowWarps * 512) {
      const int e0 = c0 + 16 * lane;
      if (e0 < Kr) {
        uint4 r0, r1;
        if (a.vec_ok && e0 + 16 <= K) {
          const uint4* p = reinterpret_cast<const uint4*>(xrow + e0);
          r0 = __ldg(p);
          r1 = __ldg(p + 1);
        } else {
          T t[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) t[j] = (e0 + j < K) ? xrow[e0 + j] : DT<T>::from_f(0.f);
          r0 = *reinterpret_cast<const uint4*>(&t[0]);
          r1 = *reinterpret_cast<const uint4*>(&t[8]);
        }
        const T* t0 = reinterpret_cast<const T*>(&r0);
        const T* t1 = reinterpret_cast<const T*>(&r1);
        double v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float f = DT<T>::to_f(j < 8 ? t0[j] : t1[j - 8]);
          if (a.norm && e0 + j < K) {
            const int k = e0 + j;
            if (a.norm == 1) f = (f - mean) * rstd * __ldg(a.gamma + k) + (a.beta ? __ldg(a.beta + k) : 0.f);
            else f = f / rms * __ldg(a.gamma + k);
            f = DT<T>::to_f(DT<T>::from_f(f));
          }
          if (a.smoothrot && e0 + j < K) f = smoothrot_div<T>(f, a.smoothrot, e0 + j, sr[e0 + j]);
          v[j] = (double)f;
        }
        if constexpr (ROT) butterflies<4, SYL, double>(v);
        if constexpr (!ROT) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (e0 + j < Kr) xr[e0 + j] = DT<T>::from_d(v[j]);
        } else if constexpr (HB == 0) {
#pragma unroll
          for (int j = 0; j < 16; ++j) xr[e0 + j] = DT<T>::from_d(v[j] * scale);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) buf[pidx(16 * lane + j)] = v[j];
        }
      }
      if constexpr (ROT && HB > 0) {
        __syncwarp();
#pragma unroll
        for (int gi = 0; gi < GPL; ++gi) {
          const int q = lane * GPL + gi;         // group: block q / 16, low bits q % 16
          const int base = (q >> 4) * R + (q & 15);
          if (c0 + base < Kr) {
            double v[NE];
#pragma unroll
            for (int h = 0; h < NE; ++h) v[h] = buf[pidx(base + 16 * h)];
            butterflies<HB, SYL, double>(v);
#pragma unroll
            for (int h = 0; h < NE; ++h) xr[c0 + base + 16 * h] = DT<T>::from_d(v[h] * scale);
          }
        }
        __syncwarp();
      }
    }
    for (int k = Kr + threadIdx.x; k < Wp; k += kRowThreads) xr[k] = DT<T>::from_f(0.f);
    __syncthreads();

    // ---- gather (once): thread t holds outputs 4t + 1024 i .. + 3
    float g[MAXIT][4];
    float amax = 0.f, rsum = 0.f;
#pragma unroll
    for (int i = 0; i < MAXIT; ++i) {
      const int j0 = 4 * threadIdx.x + 1024 * i;
      int src[4] = {j0, j0 + 1, j0 + 2, j0 + 3};
      if (a.perm) {
        if (vperm && j0 + 4 <= w_in) {
          const int4 p = __ldg(reinterpret_cast<const int4*>(a.perm + j0));
          src[0] = p.x; src[1] = p.y; src[2] = p.z; src[3] = p.w;
        } else {
#pragma unroll
          for (int t = 0; t < 4; ++t) src[t] = (j0 + t < w_in) ? a.perm[j0 + t] : 0;
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        g[i][t] = (j0 + t < w_in) ? DT<T>::to_f(xr[src[t]]) : 0.f;
        amax = fmaxf(amax, fabsf(g[i][t]));
        rsum += g[i][t];
      }
      if (a.x_prep && j0 < w_in) {
        T* dst = reinterpret_cast<T*>(a.x_prep) + row * (int64_t)w_in + j0;
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (j0 + t < w_in) dst[t] = DT<T>::from_f(g[i][t]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      rsum += __shfl_xor_sync(0xffffffffu, rsum, o);
    }
    if (lane == 0) {
      red[0][warp] = amax;
      red[1][warp] = rsum;
    }
    __syncthreads();
    amax = red[0][0];
    rsum = red[1][0];
#pragma unroll
    for (int w = 1; w < kRowWarps; ++w) {
      amax = fmaxf(amax, red[0][w]);
      rsum += red[1][w];
    }
    if (a.rowsum && threadIdx.x == 0) a.rowsum[row] = rsum;

    // ---- quantise from registers: 4 bytes per thread per step
    if (a.xq) {
      const float s = __fdiv_rn(fmaxf(amax, 1e-8f), 127.0f);
      const float rs = __frcp_rn(s);
      if (threadIdx.x == 0) a.s_a[row] = s;
      int8_t* qrow = a.xq + row * a.ldq;
#pragma unroll
      for (int i = 0; i < MAXIT; ++i) {
        const int j0 = 4 * threadIdx.x + 1024 * i;
        if (j0 < ldq) {
          uint32_t word = 0;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int8_t qv = (j0 + t < w_in) ? quant1(g[i][t], s, rs) : (int8_t)0;
            word |= ((uint32_t)(uint8_t)qv) << (8 * t);
          }
          *reinterpret_cast<uint32_t*>(qrow + j0) = word;
        }
      }
    }
    __syncthreads();   // red and xr are rewritten by the next row
  }
}

template <typename T, int LOG2R, bool SYL>
static cudaError_t launch_prep_row(const PrepArgs& a, cudaStream_t st) {
  const int xr_stride = (int)((a.Wp + 15) & ~15LL);
  const size_t kpad = (size_t)((a.K + 3) & ~3LL);
  const size_t smem = (size_t)kRowWarps * kPwBufDoubles * 8 + (size_t)xr_stride * sizeof(T) +
                      (a.smoothrot ? kpad * sizeof(float) : 0);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  const int its = (int)((a.ldq + 1023) / 1024);
  cudaError_t e;
  int per_sm = 0;
  auto go = [&](auto kern) -> cudaError_t {
    if (smem > 48 * 1024) {
      cudaError_t e2 = set_smem_once(kern, 220 * 1024);
      if (e2 != cudaSuccess) return e2;
    }
    cudaError_t e2 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRowThreads, smem);
    if (e2 != cudaSuccess) return e2;
    if (per_sm < 1) per_sm = 1;
    const int64_t cap = (int64_t)per_sm * num_sms();
    const unsigned grid = (unsigned)(a.M < cap ? a.M : cap);
    kern<<<grid, kRowThreads, smem, st>>>(a, xr_stride);
    return cudaGetLastError();
  };
  if (its <= 4) e = go(prep_row_kernel<T, LOG2R, SYL, 4>);
  else if (its <= 16) e = go(prep_row_kernel<T, LOG2R, SYL, 16>);
  else e = cudaErrorInvalidValue;
  return e;
}

// Whether prep_row_kernel takes this request.
static bool prep_row_fits(const PrepArgs& a, int log2r, size_t tsize) {
  // measured: faster for few rows (4.5 vs 5.7 us for one row); for thousands
  // of rows prep_quant_kernel is faster (68 vs 78 us for 4096 x 3072)
  static const int force_row = [] { const char* e = getenv("INTCRUSH_PREP_ROW"); return (e && e[0] == '1') ? 1 : 0; }();
  if (a.smooth || a.M == 0) return false;
  if (log2r == 0 ? !a.norm : (log2r < 4 || log2r > 8)) return false;
  // many short rows: prep_quant_kernel (68 vs 78 us at 4096 x 3072); few rows
  // or wide rows: this kernel
  if (a.M >= 4 * num_sms() && a.Wp <= 4096 && !force_row && !a.norm) return false;
  if ((a.ldq + 1023) / 1024 > 16) return false;
  const size_t smem = (size_t)kRowWarps * kPwBufDoubles * 8 + (size_t)((a.Wp + 15) & ~15LL) * tsize +
                      (a.smoothrot ? (size_t)((a.K + 3) & ~3LL) * sizeof(float) : 0);
  return smem <= 200 * 1024 && !prep_v1_forced();
}

}  // namespace ic
#include "prep_tile.cu"
namespace ic {

template <typename T>
static cudaError_t launch_prep_dt(const PrepArgs& a, int log2r, bool syl, cudaStream_t st) {
  if (prep_tile_fits(a, log2r, sizeof(T)) && !prep_v1_forced()) return launch_prep_tile_dt<T>(a, log2r, st);
  if (a.norm) {
    // row normalisation exists only in prep_row_kernel
    if (!prep_row_fits(a, log2r, sizeof(T))) return cudaErrorNotSupported;
    if (log2r == 0) return launch_prep_row<T, 0, false>(a, st);
  }
  if (log2r == 0) return launch_prep_t<T, 0, false>(a, st);
  if (prep_row_fits(a, log2r, sizeof(T))) {
    if (syl) {
      if (log2r == 5) return launch_prep_row<T, 5, true>(a, st);
      if (log2r == 7) return launch_prep_row<T, 7, true>(a, st);
    } else {
      if (log2r == 4) return launch_prep_row<T, 4, false>(a, st);
      if (log2r == 6) return launch_prep_row<T, 6, false>(a, st);
      if (log2r == 8) return launch_prep_row<T, 8, false>(a, st);
    }
  }
  if (!syl) {
    switch (log2r) {
      case 2: return launch_prep_t<T, 2, false>(a, st);
      case 4: return launch_prep_t<T, 4, false>(a, st);
      case 6: return launch_prep_t<T, 6, false>(a, st);
      case 8: return launch_prep_t<T, 8, false>(a, st);
      case 10: return launch_prep_t<T, 10, false>(a, st);
      case 12: return launch_prep_t<T, 12, false>(a, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (log2r) {
    case 1: return launch_prep_t<T, 1, true>(a, st);
    case 3: return launch_prep_t<T, 3, true>(a, st);
    case 5: return launch_prep_t<T, 5, true>(a, st);
    case 7: return launch_prep_t<T, 7, true>(a, st);
    case 9: return launch_prep_t<T, 9, true>(a, st);
    case 11: return launch_prep_t<T, 11, true>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_prep(const PrepArgs& a, int x_dtype, int log2r, bool syl, cudaStream_t st) {
  if (x_dtype == IC_DTYPE_F16) return launch_prep_dt<__half>(a, log2r, syl, st);
  return launch_prep_dt<__nv_bfloat16>(a, log2r, syl, st);
}

}  // namespace ic

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


namespace ic {

struct PrepArgs {
  const void* x;
  int64_t M, K, ldx;
  const float* smoothrot;
  int64_t w_in;
  const int32_t* perm;
  const float* smooth;
  int8_t* xq;
  int64_t ldq;
  float* s_a;
  void* x_prep;
  float* rowsum;
  int64_t Kr;       // rotated width (K rounded up to the rotation size), or K
  int64_t Wp;       // max(Kr, w_in): width of the padded row in shared memory
  double syl_h;     // Sylvester entry (only used for Sylvester sizes)
  int vec_ok;       // 16-byte vector loads of x are legal
};

int num_sms();   // gemm_tc.cu

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
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float f0 = DT<T>::to_f(e0[j]), f1 = DT<T>::to_f(e1[j]);
      if (a.smoothrot) {
        const float s0 = DT<T>::to_f(DT<T>::from_f(a.smoothrot[k0 + j]));
        const float s1 = DT<T>::to_f(DT<T>::from_f(a.smoothrot[k0 + 8 + j]));
#if defined(IC_DIAG_NODIV)   // tuning-only timing variants (wrong results)
        f0 = DT<T>::to_f(DT<T>::from_f(f0 * s0));
        f1 = DT<T>::to_f(DT<T>::from_f(f1 * s1));
#else
        f0 = DT<T>::to_f(DT<T>::from_f(__fdiv_rn(f0, s0)));
        f1 = DT<T>::to_f(DT<T>::from_f(__fdiv_rn(f1, s1)));
#endif
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
#if defined(IC_DIAG_NOD2H)
        out = DT<T>::from_f((float)(v[j] * (1.0 / (double)(1 << (LOG2R / 2)))));
#else
        if constexpr (SYL) out = DT<T>::from_d(v[j] * a.syl_h);
        else out = DT<T>::from_d(v[j] * (1.0 / (double)(1 << (LOG2R / 2))));   // 2^-D, exact
#endif
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
#if !defined(IC_DIAG_NOQCHK)
            if (fabsf(fy - (floorf(fy) + 0.5f)) <= fy * 4.8e-7f) y = __fdiv_rn(xv, s);
#endif
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

template <typename T>
static cudaError_t launch_prep_dt(const PrepArgs& a, int log2r, bool syl, cudaStream_t st) {
  if (log2r == 0) return launch_prep_t<T, 0, false>(a, st);
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

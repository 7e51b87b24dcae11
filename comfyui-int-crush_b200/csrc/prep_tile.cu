// (a1) Activation prep + per-token INT8 quantisation, tiled over 4 rows.
//
// Same arithmetic and results as prep_quant_kernel / prep_row_kernel
// (bit-identical: SmoothRot quotient correctly rounded to the activation
// dtype, exact fp64 block-Hadamard sums rounded once, quantisation
// q = rint(RN32(x / s)) with s = RN32(max(amax, 1e-8) / 127)), organised so
// that a row costs few instructions and little shared-memory traffic:
//
//  * thread t owns the 16 consecutive input columns [16t, 16t + 16) of four
//    rows at a time (the CTA covers a whole padded row, <= 4096 columns), so
//    the SmoothRot reciprocals of its columns and the output positions of its
//    values stay in registers for the whole kernel;
//  * the rotation is two in-register fp64 butterfly stages (index bits 0-3,
//    then the bits above, rotation sizes 16..256) with one exchange through a
//    warp-private, XOR-swizzled buffer between them (conflict-free 8-byte
//    accesses for every group width);
//  * the PermuQuant permutation is applied on the way out as a scatter through
//    the inverse permutation (built once per CTA): the four rows' int8 values
//    of one position travel as one 32-bit word, so the random-position shared
//    memory stores are a quarter of the values; the tile is then read back in
//    row order and written with 16-byte stores;
//  * quantisation scales need the row maximum, the only cross-warp step: two
//    CTA barriers per 4 rows (tiles and partial maxima are double-buffered).
//
// The reference's path (ComfyUI-INT-Crush): _ops.py:337-365 (prep order),
// _quant_utils.py:67-147 (Hadamard, rotation), _ops.py:529-533 (SmoothQuant
// divide), kernels/triton_quantize.py:43-54 (quantisation, CPU form).
#include "ic_common.cuh"
#include "prep_common.cuh"

namespace ic {

constexpr int kTileRowsPT = 4;          // rows per tile
constexpr int kMaxSlotsPT = 256;        // 16-column slots per CTA (4096 columns)

// fp16 / bf16 value -> fp64 (exact; one conversion for fp16).
template <typename T> __device__ __forceinline__ double act_to_d(T v) { return (double)DT<T>::to_f(v); }
// fp16 bits placed in the high word of a double (sign to bit 63, exponent
// and mantissa 10 bits up) encode the value times 2^-1008, subnormal inputs
// included; one exact multiply by 2^1008 restores it.  Integer ops and one
// DMUL instead of a conversion on the (narrow) XU pipe.
template <> __device__ __forceinline__ double act_to_d<__half>(__half v) {
  const uint32_t h = __half_as_ushort(v);
  const uint32_t hi = ((h & 0x8000u) << 16) | ((h & 0x7FFFu) << 10);
  return __hiloint2double((int)hi, 0) * 0x1p1008;
}
template <> __device__ __forceinline__ double act_to_d<__nv_bfloat16>(__nv_bfloat16 v) {
  const uint32_t b = (uint32_t)__bfloat16_as_ushort(v) << 16;   // the fp32 bits
  const uint32_t hi = (b & 0x80000000u) | ((b & 0x7FFFFFFFu) >> 3);
  return __hiloint2double((int)hi, 0) * 0x1p896;
}

// Round a pair to T on the ALU (the packed conversion; the scalar one runs on
// the XU pipe).
template <typename T> __device__ __forceinline__ void round_pair(float y0, float y1, T& h0, T& h1);
template <> __device__ __forceinline__ void round_pair<__half>(float y0, float y1, __half& h0, __half& h1) {
  const __half2 p = __floats2half2_rn(y0, y1);
  h0 = __low2half(p);
  h1 = __high2half(p);
}
template <> __device__ __forceinline__ void round_pair<__nv_bfloat16>(float y0, float y1, __nv_bfloat16& h0,
                                                                      __nv_bfloat16& h1) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(y0, y1);
  h0 = __low2bfloat16(p);
  h1 = __high2bfloat16(p);
}

// XOR swizzle of the exchange buffer: lane L stores its stage-1 value j at
// slot L * 16 + (j ^ sw(L)).  With NL lanes per rotation group, sw maps the
// lane's index inside the group to the high bits and the group index to the
// low bits, which makes both the row-wise stores (fixed j, 16 lanes) and the
// column-wise loads (fixed h, cc) hit 16 distinct 8-byte bank pairs per
// half-warp.
template <int HB>
__device__ __forceinline__ int xsw(int L) {
  if constexpr (HB == 0) return 0;
  else return ((L & ((1 << HB) - 1)) << (4 - HB)) | ((L >> HB) & ((1 << (4 - HB)) - 1));
}

// Radix-4 butterfly of the regular Hadamard factor H4 = [[1,1,1,-1],
// [1,1,-1,1],[1,-1,1,1],[-1,1,1,1]] (unnormalised); 8 exact fp64 adds.
__device__ __forceinline__ void h4(double& a0, double& a1, double& a2, double& a3) {
  const double p = a0 + a1, q = a2 + a3, r = a0 - a1, t = a2 - a3;
  a0 = p + t;
  a1 = p - t;
  a2 = r + q;
  a3 = q - r;
}

// In-register butterflies over the L index bits of v (stride 1 << (S*...)).
// Regular sizes: one radix-4 step per base-4 digit; Sylvester: radix-2 steps.
template <int L, bool SYL, int N>
__device__ __forceinline__ void bfly(double (&v)[N]) {
  static_assert((1 << L) == N, "one butterfly network per array");
  if constexpr (SYL) {
#pragma unroll
    for (int s = 0; s < L; ++s) {
#pragma unroll
      for (int i = 0; i < N; ++i)
        if ((i & (1 << s)) == 0) {
          const double a = v[i], b = v[i + (1 << s)];
          v[i] = a + b;
          v[i + (1 << s)] = a - b;
        }
    }
  } else {
    static_assert(L % 2 == 0, "regular Hadamard sizes are powers of four");
#pragma unroll
    for (int d = 0; d < L / 2; ++d) {
      const int st = 1 << (2 * d);
#pragma unroll
      for (int i = 0; i < N; ++i)
        if (((i >> (2 * d)) & 3) == 0) h4(v[i], v[i + st], v[i + 2 * st], v[i + 3 * st]);
    }
  }
}

// Pack 4 int8 (low bytes of q0..q3) into one word, byte r = q_r.
__device__ __forceinline__ uint32_t pack4(int q0, int q1, int q2, int q3) {
  const uint32_t lo = __byte_perm((uint32_t)q0, (uint32_t)q1, 0x0040);   // q0.b0, q1.b0
  const uint32_t hi = __byte_perm((uint32_t)q2, (uint32_t)q3, 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

// 4 x 4 byte transpose: in[i] byte r -> out[r] byte i.
__device__ __forceinline__ void transpose4x4(uint32_t i0, uint32_t i1, uint32_t i2, uint32_t i3, uint32_t& o0,
                                             uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  const uint32_t a = __byte_perm(i0, i1, 0x5140);   // i0.b0 i1.b0 i0.b1 i1.b1
  const uint32_t b = __byte_perm(i0, i1, 0x7362);   // i0.b2 i1.b2 i0.b3 i1.b3
  const uint32_t c = __byte_perm(i2, i3, 0x5140);
  const uint32_t d = __byte_perm(i2, i3, 0x7362);
  o0 = __byte_perm(a, c, 0x5410);   // i0.b0 i1.b0 i2.b0 i3.b0
  o1 = __byte_perm(a, c, 0x7632);
  o2 = __byte_perm(b, d, 0x5410);
  o3 = __byte_perm(b, d, 0x7632);
}

// Shared-memory plan (bytes), given the number of 16-column slots NS (a
// multiple of 32) and the quantised row stride ldq:
//   xbuf : NS * 16 doubles      stage-1 -> stage-2 exchange (warp-private parts)
//   ft   : NS * 16 floats       reciprocal factors, [j / 2][slot] float pairs
//   qt   : ldq words            int8 tile [position][4 rows]
//   inv  : NS * 16 uint16       inverse permutation
//   red  : 2 * 32 floats        per-warp row maxima, double-buffered
struct TilePlan {
  int xbuf, ft, qt, inv, red, total;
};

__host__ __device__ inline TilePlan tile_plan(int ns, int ldq, bool factors) {
  TilePlan p;
  p.xbuf = 0;
  p.ft = p.xbuf + ns * 16 * 8;
  p.qt = p.ft + (factors ? ns * 16 * 4 : 0);
  p.inv = p.qt + ldq * 4;
  p.red = p.inv + ((ns * 16 * 2 + 15) & ~15);
  p.total = p.red + 2 * 32 * 4;
  return p;
}

// SmoothRot / SmoothQuant quotient x / f rounded to the activation dtype T,
// from y = x * r with r = RN32(1 / f): y is within 2 fp32 ulps of the
// correctly rounded fp32 quotient, and rounding fp32 to T (p = 24 >= 2 q + 2)
// is an innocuous double rounding, so RN_T(y) is the correctly rounded
// quotient unless y lies within 4 fp32 ulps of a rounding midpoint of T or
// outside T's normal range.  Those cases (rare) are flagged for the IEEE
// division.  Integer tests on the bits of y; zero is exact.
template <typename T> struct QuotBits;
template <> struct QuotBits<__half> {
  static constexpr uint32_t MASK = 0x1FFFu, MID = 0x1000u, MINN = 0x38800000u, MAXN = 0x477FE000u;
};
template <> struct QuotBits<__nv_bfloat16> {
  static constexpr uint32_t MASK = 0xFFFFu, MID = 0x8000u, MINN = 0x00800000u, MAXN = 0x7F7F0000u;
};
template <typename T> __device__ __forceinline__ bool quot_ambiguous(float y) {
  const uint32_t b = __float_as_uint(y), a = b & 0x7FFFFFFFu;
  const bool mid = ((b + 4u - QuotBits<T>::MID) & QuotBits<T>::MASK) <= 8u;
  const bool range = (a - 1u < QuotBits<T>::MINN - 1u) | (a > QuotBits<T>::MAXN);
  return mid | range;
}

// Quantise a pair with one check: q = rint(x * rs) unless a product lies
// within 2^-15 of a half-integer, where the IEEE quotient x / s could round
// to the other side (x * rs is within 2 fp32 ulps of it and |x / s| <= 127.x,
// so 2^-15 > 2 ulps); then *bad is set and the caller redoes the row's values
// with the division.  Returns the integers (the 1.5 * 2^23 add rounds ties to
// even) and needs no clamp: |x| <= amax gives |x / s| < 127.5.
__device__ __forceinline__ void quant_pair(float x0, float x1, float rs, int& q0, int& q1, bool& bad) {
  // y = x * rs, t = y + M (ties to even), d = y - (t - M), two values per op
  float t0, t1, d0, d1;
  asm("{\n\t.reg .b64 x, r, m, nm, y, t, u, d;\n\t"
      "mov.b64 x, {%4, %5};\n\tmov.b64 r, {%6, %6};\n\t"
      "mov.b64 m, {%7, %7};\n\tmov.b64 nm, {%8, %8};\n\t"
      "mul.rn.f32x2 y, x, r;\n\tadd.rn.f32x2 t, y, m;\n\t"
      "add.rn.f32x2 u, t, nm;\n\tsub.rn.f32x2 d, y, u;\n\t"
      "mov.b64 {%0, %1}, t;\n\tmov.b64 {%2, %3}, d;\n\t}"
      : "=f"(t0), "=f"(t1), "=f"(d0), "=f"(d1)
      : "f"(x0), "f"(x1), "f"(rs), "f"(12582912.0f), "f"(-12582912.0f));
  bad |= (fabsf(d0) > 0.5f - 3.0517578125e-05f) | (fabsf(d1) > 0.5f - 3.0517578125e-05f);
  q0 = __float_as_int(t0) - 0x4B400000;
  q1 = __float_as_int(t1) - 0x4B400000;
}

// FT: 0 no factors, 1 SmoothRot factors (input columns), 2 SmoothQuant
// factors (output positions).
template <typename T, int LOG2R, bool SYL, int FT>
// 96 registers: three 192-thread CTAs (3072-column rows) per SM.  Register
// files are split between the four schedulers and a CTA's six warps land
// 2/2/1/1 on them, so three CTAs need <= 5 warps' worth (16384 / (5 * 32))
// per scheduler; at 112 registers only two CTAs fit.
__global__ void __maxnreg__(96) prep_tile_kernel(const PrepArgs a) {
  static_assert(LOG2R == 0 || (LOG2R >= 4 && LOG2R <= 8), "rotation sizes 16..256 (or none)");
  constexpr bool ROT = LOG2R > 0;
  constexpr int R = 1 << LOG2R;
  constexpr int HB = ROT ? LOG2R - 4 : 0;   // stage-2 index bits
  constexpr int NL = 1 << HB;               // lanes per rotation group
  constexpr int CPL = 16 / NL;              // stage-2 columns per lane
  constexpr int TR = kTileRowsPT;
  extern __shared__ __align__(16) unsigned char smem[];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nwarps = blockDim.x >> 5;
  const int NS = blockDim.x;
  const int K = (int)a.K, w_in = (int)a.w_in, ldq = (int)a.ldq;
  const TilePlan P = tile_plan(NS, ldq, FT != 0);
  double* xb = reinterpret_cast<double*>(smem + P.xbuf) + warp * 32 * 16;
  const float2* ft2 = reinterpret_cast<const float2*>(smem + P.ft);
  uint32_t* qt = reinterpret_cast<uint32_t*>(smem + P.qt);
  uint16_t* inv = reinterpret_cast<uint16_t*>(smem + P.inv);
  float* red = reinterpret_cast<float*>(smem + P.red);

  // ---- once per CTA: inverse permutation, zeroed tile tails, factors -------
  const int Wq = NS * 16;   // positions covered by the slots (>= w_in)
  if (a.perm) {
    for (int j = t; j < w_in; j += NS) {
      const int p = __ldg(a.perm + j);
      if ((unsigned)p < (unsigned)Wq) inv[p] = (uint16_t)j;   // a value out of range is dropped, not written
    }
  } else {
    for (int j = t; j < Wq; j += NS) inv[j] = (uint16_t)j;
  }
  for (int j = w_in + t; j < ldq; j += NS) qt[j] = 0u;
  const int c0 = 16 * t;                // first input column of this slot
  const int gbase = (lane / NL) * NL;   // first lane of this lane's rotation group
  const int li = lane - gbase;          // index inside the group
  const int gpos = (t / NL) * R;        // first position of the group
  __syncthreads();   // inv complete
  // output position of value e (stage-2 column cc = e / NL, high index h = e % NL)
  uint32_t opos[8];  // inverse-permuted positions, two 16-bit entries per word (0xFFFF: padding)
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int p = ROT ? gpos + 16 * (e % NL) + li * CPL + e / NL : c0 + e;
    const uint32_t j = (p < w_in) ? inv[p] : 0xFFFFu;
    if (e & 1) opos[e >> 1] |= j << 16;
    else opos[e >> 1] = j;
  }
  if constexpr (FT != 0) {
    float* ftw = reinterpret_cast<float*>(smem + P.ft);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float f = 1.f;
      if (FT == 1 && c0 + e < K) f = DT<T>::to_f(DT<T>::from_f(__ldg(a.smoothrot + c0 + e)));
      if (FT == 2) {
        const uint32_t j = (e & 1) ? (opos[e >> 1] >> 16) : (opos[e >> 1] & 0xFFFFu);
        if (j != 0xFFFFu) f = DT<T>::to_f(DT<T>::from_f(__ldg(a.smooth + j)));
      }
      ftw[((e >> 1) * NS + t) * 2 + (e & 1)] = __frcp_rn(f);
    }
    __syncthreads();
  }
  const double rscale = SYL ? a.syl_h : 1.0 / (double)(1 << (LOG2R / 2));
  const bool vec = a.vec_ok && (c0 + 16 <= K);
  const int64_t ntiles = (a.M + TR - 1) / TR;

  auto load_row = [&](int64_t row, uint4 (&raw)[2]) {
    const T* xr = reinterpret_cast<const T*>(a.x) + row * a.ldx + c0;
    if (row < a.M && vec) {
      raw[0] = __ldg(reinterpret_cast<const uint4*>(xr));
      raw[1] = __ldg(reinterpret_cast<const uint4*>(xr) + 1);
    } else {
      T v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (row < a.M && c0 + j < K) ? xr[j] : DT<T>::from_f(0.f);
      raw[0] = *reinterpret_cast<const uint4*>(&v[0]);
      raw[1] = *reinterpret_cast<const uint4*>(&v[8]);
    }
  };
  // the k-th row this CTA handles (rows run tile by tile, 4 per tile)
  auto row_of = [&](int64_t k) -> int64_t {
    const int64_t tl = blockIdx.x + (k >> 2) * (int64_t)gridDim.x;
    return tl < ntiles ? tl * TR + (k & 3) : a.M;   // past the end: a masked (zero) load
  };

  // two rows of loads in flight ahead of the row being processed
  uint4 pa[2], pb[2];
  load_row(row_of(0), pa);
  load_row(row_of(1), pb);
  int64_t k = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t r0 = tile * TR;
    uint32_t qw[16];   // int8 of the 16 output positions, byte r = row r of the tile
#pragma unroll
    for (int e = 0; e < 16; ++e) qw[e] = 0u;
#pragma unroll 1
    for (int r = 0; r < TR; ++r, ++k) {
      uint4 raw[2] = {pa[0], pa[1]};
      pa[0] = pb[0];
      pa[1] = pb[1];
      load_row(row_of(k + 2), pb);
      const T* in = reinterpret_cast<const T*>(&raw[0]);
      // -- SmoothRot quotient, rounded to T (exact, see quot_ambiguous)
      double v[16];
      if constexpr (FT == 1) {
        bool amb = false;
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const float2 r2 = ft2[(j >> 1) * NS + t];
          const float y0 = DT<T>::to_f(in[j]) * r2.x, y1 = DT<T>::to_f(in[j + 1]) * r2.y;
          amb |= quot_ambiguous<T>(y0) | quot_ambiguous<T>(y1);
          T h0, h1;
          round_pair<T>(y0, y1, h0, h1);
          v[j] = act_to_d(h0);
          v[j + 1] = act_to_d(h1);
        }
        // rare (about 1 value in 900): the IEEE division for exactly those
        // values (the test is redone), so that a warp pays for one division,
        // not sixteen
        if (amb) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (quot_ambiguous<T>(DT<T>::to_f(in[j]) * (j & 1 ? ft2[(j >> 1) * NS + t].y : ft2[(j >> 1) * NS + t].x))
                && c0 + j < K) {
              const float f = DT<T>::to_f(DT<T>::from_f(__ldg(a.smoothrot + c0 + j)));
              v[j] = act_to_d(DT<T>::from_f(__fdiv_rn(DT<T>::to_f(in[j]), f)));
            }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = act_to_d(in[j]);
      }
      // -- rotation: bits 0-3 in registers, exchange, the bits above
      double w[16];
      if constexpr (ROT) {
        bfly<4, SYL>(v);
        if constexpr (HB > 0) {
          const int s = xsw<HB>(lane);
#pragma unroll
          for (int j = 0; j < 16; ++j) xb[lane * 16 + (j ^ s)] = v[j];
          __syncwarp();
#pragma unroll
          for (int cc = 0; cc < CPL; ++cc) {
            double u[NL];
#pragma unroll
            for (int h = 0; h < NL; ++h) {
              const int src = gbase + h;
              u[h] = xb[src * 16 + ((li * CPL + cc) ^ xsw<HB>(src))];
            }
            bfly<HB, SYL>(u);
#pragma unroll
            for (int h = 0; h < NL; ++h) w[cc * NL + h] = u[h];
          }
          __syncwarp();   // the buffer is rewritten by the next row
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = v[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = v[j];
      }
      // -- round once to T (and the SmoothQuant quotient), row maximum
      float fv[16];
      float mx = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e)
        fv[e] = DT<T>::to_f(ROT ? DT<T>::from_d(w[e] * rscale) : DT<T>::from_d(w[e]));
      if constexpr (FT == 2) {   // SmoothQuant divide at the output positions
        bool amb = false;
        float o[16];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 r2 = ft2[(e >> 1) * NS + t];
          const float y0 = fv[e] * r2.x, y1 = fv[e + 1] * r2.y;
          amb |= quot_ambiguous<T>(y0) | quot_ambiguous<T>(y1);
          T h0, h1;
          round_pair<T>(y0, y1, h0, h1);
          o[e] = DT<T>::to_f(h0);
          o[e + 1] = DT<T>::to_f(h1);
        }
        if (amb) {   // rare: the IEEE division for those values only
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint32_t j = (e & 1) ? (opos[e >> 1] >> 16) : (opos[e >> 1] & 0xFFFFu);
            if (quot_ambiguous<T>(fv[e] * (e & 1 ? ft2[(e >> 1) * NS + t].y : ft2[(e >> 1) * NS + t].x))
                && j != 0xFFFFu)
              o[e] = DT<T>::to_f(DT<T>::from_f(__fdiv_rn(fv[e], DT<T>::to_f(DT<T>::from_f(__ldg(a.smooth + j))))));
          }
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) fv[e] = o[e];
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) mx = fmaxf(mx, fabsf(fv[e]));
      // -- row maximum over the CTA (the only cross-warp step of a row)
      asm("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(mx));   // mx >= 0
      float* rb = red + (k & 1) * 32;
      if (lane == 0) rb[warp] = mx;
      __syncthreads();
      mx = rb[0];
      for (int w2 = 1; w2 < nwarps; ++w2) mx = fmaxf(mx, rb[w2]);
      const float s = __fdiv_rn(fmaxf(mx, 1e-8f), 127.0f);
      const float rs = __frcp_rn(s);
      if (t == 0 && r0 + r < a.M) a.s_a[r0 + r] = s;
      // -- quantise into byte r of the position words
      const uint32_t sel = (0x3210u & ~(0xFu << (4 * r))) | (4u << (4 * r));
      bool bad = false;
      int q[16];
#pragma unroll
      for (int e = 0; e < 16; e += 2) quant_pair(fv[e], fv[e + 1], rs, q[e], q[e + 1], bad);
      if (bad) {   // rare: a product near a half-integer, take the IEEE quotient
#pragma unroll
        for (int e = 0; e < 16; ++e) q[e] = quant1(fv[e], s, rs);
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) qw[e] = __byte_perm(qw[e], (uint32_t)q[e], sel);
    }
    // ---- scatter the four rows' bytes through the inverse permutation
    // (one tile buffer: the next tile's scatter comes four row barriers after
    // this tile's read-out)
    uint32_t* qb = qt;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const uint32_t j = (e & 1) ? (opos[e >> 1] >> 16) : (opos[e >> 1] & 0xFFFFu);
      if (j != 0xFFFFu) qb[j] = qw[e];
    }
    __syncthreads();
    // ---- tile out in row order: 16 positions x 4 rows per thread per step
    for (int c = t; c < ldq / 16; c += NS) {
      const uint4 w0 = *reinterpret_cast<const uint4*>(qb + 16 * c);
      const uint4 w1 = *reinterpret_cast<const uint4*>(qb + 16 * c + 4);
      const uint4 w2 = *reinterpret_cast<const uint4*>(qb + 16 * c + 8);
      const uint4 w3 = *reinterpret_cast<const uint4*>(qb + 16 * c + 12);
      uint4 o[TR];
      transpose4x4(w0.x, w0.y, w0.z, w0.w, o[0].x, o[1].x, o[2].x, o[3].x);
      transpose4x4(w1.x, w1.y, w1.z, w1.w, o[0].y, o[1].y, o[2].y, o[3].y);
      transpose4x4(w2.x, w2.y, w2.z, w2.w, o[0].z, o[1].z, o[2].z, o[3].z);
      transpose4x4(w3.x, w3.y, w3.z, w3.w, o[0].w, o[1].w, o[2].w, o[3].w);
#pragma unroll
      for (int rr = 0; rr < TR; ++rr)
        if (r0 + rr < a.M) *reinterpret_cast<uint4*>(a.xq + (r0 + rr) * a.ldq + 16 * c) = o[rr];
    }
  }
}

// Whether prep_tile_kernel takes the request: quantised output only (no
// prepped row, no row sums), rotation 0 or 16..256, no row normalisation, the
// padded row in at most 4096 columns, shared memory fits.
static bool prep_tile_fits(const PrepArgs& a, int log2r, size_t tsize) {
  static const int off = [] { const char* e = getenv("INTCRUSH_PREP_TILE"); return (e && e[0] == '0') ? 1 : 0; }();
  (void)tsize;
  if (off || a.norm || a.M == 0 || (a.smooth && a.smoothrot)) return false;
  if (!a.xq || a.x_prep || a.rowsum) return false;
  if (log2r != 0 && (log2r < 4 || log2r > 8)) return false;
  const int64_t W = a.Wp > a.w_in ? a.Wp : a.w_in;
  const int64_t ns = ((W + 15) / 16 + 31) / 32 * 32;
  if (ns > kMaxSlotsPT || a.ldq > ns * 16) return false;   // the tile covers ldq positions
  const TilePlan p = tile_plan((int)ns, (int)a.ldq, a.smooth || a.smoothrot);
  return p.total <= 110 * 1024;
}

template <typename T, int LOG2R, bool SYL, int FT>
static cudaError_t launch_prep_tile(const PrepArgs& a, cudaStream_t st) {
  const int64_t W = a.Wp > a.w_in ? a.Wp : a.w_in;
  const int ns = (int)(((W + 15) / 16 + 31) / 32 * 32);
  const TilePlan p = tile_plan(ns, (int)a.ldq, FT != 0);
  auto kern = prep_tile_kernel<T, LOG2R, SYL, FT>;
  cudaError_t e = cudaSuccess;
  // all of the unified L1 as shared memory: rows are streamed (no reuse
  // through L1), and three CTAs of ~56 KB must fit
  e = set_smem_once(kern, 110 * 1024, 100);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, ns, p.total);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  const int64_t ntiles = (a.M + kTileRowsPT - 1) / kTileRowsPT;
  const int64_t cap = (int64_t)per_sm * num_sms();
  const unsigned grid = (unsigned)(ntiles < cap ? ntiles : cap);
  kern<<<grid, ns, p.total, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int FT>
static cudaError_t launch_prep_tile_r(const PrepArgs& a, int log2r, cudaStream_t st) {
  switch (log2r) {
    case 0: return launch_prep_tile<T, 0, false, FT>(a, st);
    case 4: return launch_prep_tile<T, 4, false, FT>(a, st);
    case 5: return launch_prep_tile<T, 5, true, FT>(a, st);
    case 6: return launch_prep_tile<T, 6, false, FT>(a, st);
    case 7: return launch_prep_tile<T, 7, true, FT>(a, st);
    case 8: return launch_prep_tile<T, 8, false, FT>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

// SmoothQuant factors come only without SmoothRot factors (the INT8 path,
// _ops.py:529-533); both at once route to the other kernels.
template <typename T>
static cudaError_t launch_prep_tile_dt(const PrepArgs& a, int log2r, cudaStream_t st) {
  if (a.smooth) return launch_prep_tile_r<T, 2>(a, log2r, st);
  if (a.smoothrot) return launch_prep_tile_r<T, 1>(a, log2r, st);
  return launch_prep_tile_r<T, 0>(a, log2r, st);
}

}  // namespace ic

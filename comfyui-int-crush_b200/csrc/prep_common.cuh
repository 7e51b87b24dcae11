// Declarations shared by the activation-prep kernels (prep.cu, prep_tile.cu).
#pragma once

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
  // optional row normalisation before everything else (prep_row_kernel only):
  // 0 none, 1 LayerNorm (x - mean) * rstd * gamma + beta, 2 RMSNorm
  // x / sqrt(mean(x^2) + eps) * gamma; rounded once to the activation dtype
  int norm;
  const float* gamma;
  const float* beta;
  float eps;
};

int num_sms();   // gemm_tc.cu

template <typename T> struct MidBits;
template <> struct MidBits<__half> {          // 10-bit mantissa: 13 fp32 bits below it
  static constexpr uint32_t MASK = 0x1FFFu, MID = 0x1000u;
  static constexpr float MIN_NORMAL = 6.103515625e-05f, MAX = 65504.0f;
};
template <> struct MidBits<__nv_bfloat16> {   // 7-bit mantissa: 16 fp32 bits below it
  static constexpr uint32_t MASK = 0xFFFFu, MID = 0x8000u;
  static constexpr float MIN_NORMAL = 1.1754943508e-38f, MAX = 3.38e38f;
};

// fp16-rounded (or bf16-rounded) quotient x / f given r = RN(1 / f).
// (fp32 factor f[k] read from global memory only on the exact path)
template <typename T>
__device__ __forceinline__ float smoothrot_div(float x, const float* fg, int k, float r) {
  const float y = x * r;
  const float ay = fabsf(y);
  const uint32_t low = __float_as_uint(y) & MidBits<T>::MASK;
  const uint32_t d = low > MidBits<T>::MID ? low - MidBits<T>::MID : MidBits<T>::MID - low;
  float q = y;
  if (d <= 4u || ay < MidBits<T>::MIN_NORMAL || ay > MidBits<T>::MAX)
    q = __fdiv_rn(x, DT<T>::to_f(DT<T>::from_f(__ldg(fg + k))));
  return DT<T>::to_f(DT<T>::from_f(q));
}

__device__ __forceinline__ int8_t quant1(float xv, float s, float rs) {
  // q = rint(x / s) with the quotient correctly rounded to fp32: x * (1/s) is
  // within 2 fp32 ulps of it, so both round to the same integer unless the
  // product lies within 2^-21 (relative) of a half-integer; then the exact
  // division is evaluated.  1.5 * 2^23 rounds to nearest, ties to even.
  float y = xv * rs;
  const float fy = fabsf(y);
  if (fabsf(fy - (floorf(fy) + 0.5f)) <= fy * 4.8e-7f) y = __fdiv_rn(xv, s);
  return (int8_t)max(-128, min(127, __float_as_int(y + 12582912.0f) - 0x4B400000));
}

}  // namespace ic

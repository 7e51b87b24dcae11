// Weight-side kernels: on-device requantisation of a patched float weight
// (set_weight) and the first factor of the LoKr residual.
//
// * quantize_weight_kernel follows the layout classes' quantize
//   (quant_layout.py:100-129 INT4, :179-200 INT8): per output row
//   amax = max|w|, INT4 s = fp16(max(amax / 7, 1e-8)), INT8
//   s = max(amax / 127, 1e-8) (fp32), q = clamp(rint(w / s)) (IEEE
//   division, ties to even), INT4 packed two per byte, low nibble = even
//   column, an odd K padded with a zero nibble.  A NaN quotient (a zero row
//   whose fp16 scale underflows to 0) stores 0.
// * lokr_w1_kernel is step 1 of _apply_lokr (_ops.py:88-138):
//   temp[t, l, j] = T(sum_i w1[l, i] * x[t, i * in_n + j]) with fp32 sums,
//   i.e. ``w1 @ X`` for X = x_t viewed [in_m, in_n].  Step 2
//   (out += scale * temp @ w2^T) is lowrank_add_kernel over the rows (t, l)
//   of out viewed [M * out_l, out_k].

namespace ic {

template <int BITS>
__global__ void __launch_bounds__(256) quantize_weight_kernel(const float* w, int N, int K, long long ldw,
                                                              uint8_t* q, long long ldq, void* scale) {
  const int n = blockIdx.x;
  const float* row = w + (long long)n * ldw;
  __shared__ float red[8];
  float m = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) m = fmaxf(m, fabsf(row[k]));
  // fmaxf drops NaN like torch's amax does not; a NaN row is propagated below
  bool has_nan = false;
  for (int k = threadIdx.x; k < K; k += 256) has_nan |= (row[k] != row[k]);
  has_nan = __syncthreads_or(has_nan);
  asm("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(m));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  if (has_nan) amax = __int_as_float(0x7fc00000);
  float s;
  if (BITS == 4) {
    const __half sh = __float2half_rn(fmaxf(__fdiv_rn(amax, 7.0f), 1e-8f));
    if (has_nan) s = amax;
    else s = __half2float(sh);
    if (threadIdx.x == 0) reinterpret_cast<__half*>(scale)[n] = has_nan ? __float2half_rn(amax) : sh;
  } else {
    s = has_nan ? amax : fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
    if (threadIdx.x == 0) reinterpret_cast<float*>(scale)[n] = s;
  }
  constexpr int QMIN = BITS == 4 ? -8 : -128, QMAX = BITS == 4 ? 7 : 127;
  auto quant = [&](float v) -> int {
    const float t = __fdiv_rn(v, s);
    if (t != t) return 0;
    const float c = fminf(fmaxf(t, (float)QMIN), (float)QMAX);
    return (int)rintf(c);
  };
  uint8_t* qrow = q + (long long)n * ldq;
  if (BITS == 8) {
    for (int k = threadIdx.x; k < K; k += 256) qrow[k] = (uint8_t)(int8_t)quant(row[k]);
  } else {
    const int nb = (K + 1) / 2;
    for (int b = threadIdx.x; b < nb; b += 256) {
      const int lo = quant(row[2 * b]);
      const int hi = (2 * b + 1 < K) ? quant(row[2 * b + 1]) : 0;
      qrow[b] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
    }
  }
}

cudaError_t launch_quantize_weight(const float* w, int N, int K, long long ldw, int bits, uint8_t* q,
                                   long long ldq, void* scale, cudaStream_t st) {
  if (bits == 4) quantize_weight_kernel<4><<<N, 256, 0, st>>>(w, N, K, ldw, q, ldq, scale);
  else quantize_weight_kernel<8><<<N, 256, 0, st>>>(w, N, K, ldw, q, ldq, scale);
  return cudaGetLastError();
}

// One CTA per (token, 256-wide slice of j); w1 [out_l, in_m] in shared
// memory as fp32, the out_l sums of each thread's column j in registers in
// groups of 16 rows.
template <typename T>
__global__ void __launch_bounds__(256) lokr_w1_kernel(const T* x, int M, long long ldx, const T* w1, int out_l,
                                                      int in_m, int in_n, T* temp) {
  extern __shared__ float w1s[];   // [out_l * in_m]
  for (int i = threadIdx.x; i < out_l * in_m; i += 256) w1s[i] = DT<T>::to_f(w1[i]);
  __syncthreads();
  const int t = blockIdx.y;
  const int j = blockIdx.x * 256 + threadIdx.x;
  if (t >= M || j >= in_n) return;
  const T* xt = x + (long long)t * ldx + j;
  T* tt = temp + (long long)t * out_l * in_n + j;
  for (int l0 = 0; l0 < out_l; l0 += 16) {
    float acc[16];
#pragma unroll
    for (int l = 0; l < 16; ++l) acc[l] = 0.f;
    for (int i = 0; i < in_m; ++i) {
      const float xv = DT<T>::to_f(xt[(long long)i * in_n]);
#pragma unroll
      for (int l = 0; l < 16; ++l)
        if (l0 + l < out_l) acc[l] = fmaf(w1s[(l0 + l) * in_m + i], xv, acc[l]);
    }
#pragma unroll
    for (int l = 0; l < 16; ++l)
      if (l0 + l < out_l) tt[(long long)(l0 + l) * in_n] = DT<T>::from_f(acc[l]);
  }
}

cudaError_t launch_lokr_w1(const void* x, int dtype, int M, long long ldx, const void* w1, int out_l, int in_m,
                           int in_n, void* temp, cudaStream_t st) {
  const dim3 grid((in_n + 255) / 256, M);
  const size_t smem = (size_t)out_l * in_m * sizeof(float);
  if (dtype == IC_DTYPE_BF16)
    lokr_w1_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>((const __nv_bfloat16*)x, M, ldx,
                                                           (const __nv_bfloat16*)w1, out_l, in_m, in_n,
                                                           (__nv_bfloat16*)temp);
  else
    lokr_w1_kernel<__half><<<grid, 256, smem, st>>>((const __half*)x, M, ldx, (const __half*)w1, out_l, in_m,
                                                    in_n, (__half*)temp);
  return cudaGetLastError();
}

}  // namespace ic

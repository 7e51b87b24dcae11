// (a4, a5) Weight-streaming W4A16 for small token counts, the low-rank
// (LoRA / SVD) down projection and residual, and the INT4 unpack utilities.
//
// W4A16 small-M kernel.  For M <= 128 tokens (32 per CTA row of the grid) the GEMM is a weight stream:
// 0.5 byte of HBM per weight against 2*M flops, so the kernel is built to
// keep the HBM pipe busy, not the tensor pipe.  Weights never touch shared
// memory: each lane loads 16 packed bytes of two weight rows per 128-k block
// (coalesced 64-byte row segments), expands them in registers to
// fp16(q * s[n, g]) -- bit-identical to the reference's dequantised weight
// (kernels/triton_int4_unpack.py:48-56, quant_layout.py:81-87) -- and feeds
// them as the A operand of a register-sourced m16n8k16 MMA whose B operand is
// the activation (weights as rows, tokens as columns).  Inside a 128-k block
// the k order is permuted consistently for A and B so that every lane's
// 16-byte load covers exactly the k values its fragments need; the dot
// product is unchanged.  Eight warps split K, and their fp32 partials are
// reduced in a fixed order in shared memory (deterministic).
#include "ic_common.cuh"

#include <type_traits>

namespace ic {

constexpr int kSkinnyWarps = 8;

__device__ __forceinline__ uint32_t i4pair_f16(uint32_t xo, uint32_t yo, int i, __half2 s2) {
  const uint32_t sel = (uint32_t)i | ((uint32_t)(i + 4) << 8);
  uint32_t t = (__byte_perm(xo, yo, sel) & 0x00FF00FFu) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&t);
  h = __hsub2(h, __half2half2(__ushort_as_half((unsigned short)0x6408u)));
  h = __hmul2(h, s2);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Layout 1 of ic_repack_int4: nibbles (t, t+4) of a word hold (k_2t, k_2t+1) + 8.
__device__ __forceinline__ uint32_t r16pair_f16(uint32_t v, int t, __half2 s2) {
  uint32_t bits = ((v >> (4 * t)) & 0x000F000Fu) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&bits);
  h = __hsub2(h, __half2half2(__ushort_as_half((unsigned short)0x6408u)));
  h = __hmul2(h, s2);
  return *reinterpret_cast<uint32_t*>(&h);
}

// bf16 weights: bf16(q * s) from the fp32 product (exact for a 4-bit q and
// an fp16-valued s), the reference's PyTorch dequantisation followed by its
// cast to the activation dtype (quant_layout.py:81-87, _ops.py:483-491).
// n0, n1: offset-binary nibbles (q + 8) of k and k + 1.
__device__ __forceinline__ uint32_t pair_bf16(uint32_t n0, uint32_t n1, float s) {
  const float q0 = __uint_as_float(0x4B000000u | n0) - 8388616.0f;   // (2^23 + n) - (2^23 + 8)
  const float q1 = __uint_as_float(0x4B000000u | n1) - 8388616.0f;
  const __nv_bfloat162 h = __floats2bfloat162_rn(q0 * s, q1 * s);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t i4pair_bf16(uint32_t xo, uint32_t yo, int i, float s) {
  return pair_bf16((xo >> (8 * i)) & 0xFu, (yo >> (8 * i)) & 0xFu, s);
}
__device__ __forceinline__ uint32_t r16pair_bf16(uint32_t v, int t, float s) {
  return pair_bf16((v >> (4 * t)) & 0xFu, (v >> (4 * t + 16)) & 0xFu, s);
}

template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct SkinnyArgs {
  const void* x; int M, K; long long ldx;     // activations in the activation dtype (fp16 / bf16)
  const uint8_t* w; int N; long long ldw;
  const void* scale; int scale_dtype; int G, group_size;
  const void* bias; int bias_dtype;
  const void* lr_mid; const void* lr_up; int R; float lr_scale;   // activation dtype
  void* out; long long ldo;                   // activation dtype
  int repacked;     // weights in ic_repack_int4 layout 1
};

__device__ __forceinline__ uint4 load_packed16(const SkinnyArgs& a, int n, int kb, int t) {
  // 16 packed bytes of row n covering k in [kb*128 + 32t, +32)
  uint4 v = make_uint4(0, 0, 0, 0);
  if (n >= a.N) return v;
  const long long b0 = (long long)kb * 64 + 16 * t;
  const long long nbytes = (a.K + 1) / 2;
  const uint8_t* p = a.w + (long long)n * a.ldw + b0;
  if (b0 + 16 <= nbytes) return __ldg(reinterpret_cast<const uint4*>(p));
  uint8_t tmp[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) tmp[i] = (b0 + i < nbytes) ? p[i] : 0;
  return *reinterpret_cast<uint4*>(tmp);
}

__device__ __forceinline__ __half load_scale(const SkinnyArgs& a, int n, int g) {
  if (n >= a.N) return __float2half_rn(0.f);
  const size_t i = (size_t)n * a.G + g;
  return a.scale_dtype == IC_DTYPE_F16 ? reinterpret_cast<const __half*>(a.scale)[i]
                                       : __float2half_rn(reinterpret_cast<const float*>(a.scale)[i]);
}
__device__ __forceinline__ float load_scale_f(const SkinnyArgs& a, int n, int g) {
  if (n >= a.N) return 0.f;
  const size_t i = (size_t)n * a.G + g;
  return a.scale_dtype == IC_DTYPE_F16 ? __half2float(reinterpret_cast<const __half*>(a.scale)[i])
                                       : reinterpret_cast<const float*>(a.scale)[i];
}

// 32 activations of token m at k in [k0, k0 + 32), zero past K or M.
template <typename T>
__device__ __forceinline__ void load_x32(const SkinnyArgs& a, int m, long long k0, uint32_t (&w)[16]) {
  if (m >= a.M) {   // token slot past M: zeros, no loads
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0u;
    return;
  }
  const T* x = reinterpret_cast<const T*>(a.x);
  if (k0 + 32 <= a.K && ((a.ldx & 7) == 0)) {
    const uint4* p = reinterpret_cast<const uint4*>(x + (long long)m * a.ldx + k0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 v = __ldg(p + i);
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
    return;
  }
  T h[32];
#pragma unroll
  for (int i = 0; i < 32; ++i)
    h[i] = (m < a.M && k0 + i < a.K) ? x[(long long)m * a.ldx + k0 + i] : DT<T>::from_f(0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = *reinterpret_cast<uint32_t*>(&h[2 * i]);
}

template <int TT, typename T>
__global__ void __launch_bounds__(32 * kSkinnyWarps, 2) w4a16_skinny_kernel(const SkinnyArgs a) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  __shared__ float red[kSkinnyWarps][16][8 * TT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * 16;
  const int m0 = blockIdx.y * 8 * TT;   // token tile (M > 32: one CTA row per 32 tokens)
  const int nkb = (a.K + 127) / 128;
  float d[TT][4];
#pragma unroll
  for (int i = 0; i < TT; ++i) d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;

  // The packed weights and scales of PF K blocks per warp are requested
  // before any of them is used, so each warp has PF HBM loads in flight.
  constexpr int PF = (TT >= 4) ? 2 : 4;
  for (int kb0 = warp; kb0 < nkb; kb0 += kSkinnyWarps * PF) {
    uint4 pa[PF], pb[PF];
    __half2 sa[PF], sb[PF];   // fp16 path: the scale as half2
    float fa[PF], fb[PF];     // bf16 path: the scale in fp32
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int kb = kb0 + kSkinnyWarps * j;
      if (kb < nkb) {
        pa[j] = load_packed16(a, n0 + g, kb, t);
        pb[j] = load_packed16(a, n0 + g + 8, kb, t);
        const int grp = (a.G > 1) ? (kb * 128) / a.group_size : 0;
        if constexpr (BF) {
          fa[j] = load_scale_f(a, n0 + g, grp);
          fb[j] = load_scale_f(a, n0 + g + 8, grp);
        } else {
          sa[j] = __half2half2(load_scale(a, n0 + g, grp));
          sb[j] = __half2half2(load_scale(a, n0 + g + 8, grp));
        }
      } else {
        pa[j] = pb[j] = make_uint4(0u, 0u, 0u, 0u);
        sa[j] = sb[j] = __half2half2(__float2half_rn(0.f));
        fa[j] = fb[j] = 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int kb = kb0 + kSkinnyWarps * j;
      if (kb >= nkb) break;
      uint32_t xw[TT][16];
#pragma unroll
      for (int i = 0; i < TT; ++i) load_x32<T>(a, m0 + i * 8 + g, (long long)kb * 128 + 32 * t, xw[i]);
      const uint32_t wa[4] = {pa[j].x, pa[j].y, pa[j].z, pa[j].w};
      const uint32_t wb[4] = {pb[j].x, pb[j].y, pb[j].z, pb[j].w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t oa = wa[w] ^ 0x88888888u, ob = wb[w] ^ 0x88888888u;
        const uint32_t xa = oa & 0x0F0F0F0Fu, ya = (oa >> 4) & 0x0F0F0F0Fu;
        const uint32_t xb = ob & 0x0F0F0F0Fu, yb = (ob >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int h = 0; h < 2; ++h) {   // MMA step s = 2w + h uses k pairs 2h, 2h+1 of word w
          const int s = 2 * w + h;
          uint32_t a0, a1, a2, a3;
          if constexpr (BF) {
            if (a.repacked) {
              a0 = r16pair_bf16(wa[w], 2 * h, fa[j]);
              a2 = r16pair_bf16(wa[w], 2 * h + 1, fa[j]);
              a1 = r16pair_bf16(wb[w], 2 * h, fb[j]);
              a3 = r16pair_bf16(wb[w], 2 * h + 1, fb[j]);
            } else {
              a0 = i4pair_bf16(xa, ya, 2 * h, fa[j]);
              a2 = i4pair_bf16(xa, ya, 2 * h + 1, fa[j]);
              a1 = i4pair_bf16(xb, yb, 2 * h, fb[j]);
              a3 = i4pair_bf16(xb, yb, 2 * h + 1, fb[j]);
            }
          } else if (a.repacked) {
            a0 = r16pair_f16(wa[w], 2 * h, sa[j]);
            a2 = r16pair_f16(wa[w], 2 * h + 1, sa[j]);
            a1 = r16pair_f16(wb[w], 2 * h, sb[j]);
            a3 = r16pair_f16(wb[w], 2 * h + 1, sb[j]);
          } else {
            a0 = i4pair_f16(xa, ya, 2 * h, sa[j]);
            a2 = i4pair_f16(xa, ya, 2 * h + 1, sa[j]);
            a1 = i4pair_f16(xb, yb, 2 * h, sb[j]);
            a3 = i4pair_f16(xb, yb, 2 * h + 1, sb[j]);
          }
#pragma unroll
          for (int i = 0; i < TT; ++i) mma_16816<T>(d[i], a0, a1, a2, a3, xw[i][2 * s], xw[i][2 * s + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < TT; ++i) {
    red[warp][g][i * 8 + 2 * t] = d[i][0];
    red[warp][g][i * 8 + 2 * t + 1] = d[i][1];
    red[warp][g + 8][i * 8 + 2 * t] = d[i][2];
    red[warp][g + 8][i * 8 + 2 * t + 1] = d[i][3];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < 16 * 8 * TT; o += blockDim.x) {
    const int r = o % 16, ml = o / 16;   // consecutive threads -> consecutive n
    const int n = n0 + r, m = m0 + ml;
    if (n >= a.N || m >= a.M) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kSkinnyWarps; ++w) v += red[w][r][ml];
    if (a.bias) v += load_any(a.bias, a.bias_dtype, n);
    T ov = DT<T>::from_f(v);
    if (a.lr_mid) {
      const T* mid = reinterpret_cast<const T*>(a.lr_mid);
      const T* up = reinterpret_cast<const T*>(a.lr_up);
      float l = 0.f;
      const T* mr = mid + (long long)m * a.R;
      const T* ur = up + (long long)n * a.R;
      if ((a.R & 7) == 0 && ((reinterpret_cast<uintptr_t>(mr) | reinterpret_cast<uintptr_t>(ur)) & 15) == 0) {
        // 16-byte loads, eight of each in flight per round (one memory
        // latency per 64 rank instead of one per 8)
        for (int j0 = 0; j0 < a.R; j0 += 64) {
          uint4 mv[8], uv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (j0 + 8 * i < a.R) {
              mv[i] = __ldg(reinterpret_cast<const uint4*>(mr + j0) + i);
              uv[i] = __ldg(reinterpret_cast<const uint4*>(ur + j0) + i);
            }
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (j0 + 8 * i < a.R) {
              const T* mh = reinterpret_cast<const T*>(&mv[i]);
              const T* uh = reinterpret_cast<const T*>(&uv[i]);
#pragma unroll
              for (int q = 0; q < 8; ++q) l = fmaf(DT<T>::to_f(mh[q]), DT<T>::to_f(uh[q]), l);
            }
        }
      } else {
#pragma unroll 8
        for (int j = 0; j < a.R; ++j) l = fmaf(DT<T>::to_f(mr[j]), DT<T>::to_f(ur[j]), l);
      }
      ov = DT<T>::from_f(DT<T>::to_f(ov) + a.lr_scale * l);
    }
    reinterpret_cast<T*>(a.out)[(long long)m * a.ldo + n] = ov;
  }
}

template <typename T>
static cudaError_t launch_w4a16_skinny_t(const SkinnyArgs& a, cudaStream_t st) {
  // up to 32 tokens per CTA row of the grid; more tokens add CTA rows, each
  // streaming the (L2-resident) weights again
  const dim3 grid((a.N + 15) / 16, (a.M + 31) / 32);
  if (a.M <= 8) w4a16_skinny_kernel<1, T><<<grid, 32 * kSkinnyWarps, 0, st>>>(a);
  else if (a.M <= 16) w4a16_skinny_kernel<2, T><<<grid, 32 * kSkinnyWarps, 0, st>>>(a);
  else w4a16_skinny_kernel<4, T><<<grid, 32 * kSkinnyWarps, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_w4a16_skinny(const SkinnyArgs& a, int x_dtype, cudaStream_t st) {
  return x_dtype == IC_DTYPE_BF16 ? launch_w4a16_skinny_t<__nv_bfloat16>(a, st) : launch_w4a16_skinny_t<__half>(a, st);
}

// ------------------------------------------------------------ low rank
// mid[m, r] = T(sum_k x[m, k] * down[r, k]) with fp32 accumulation, T the
// activation dtype (F.linear(x_raw, down), _ops.py:242).  One CTA per (rank
// r, tile of 8 tokens): each thread takes 8-value slices of K (16-byte loads
// of the down row and of the tile's token rows) and the CTA reduces its
// partial sums in a fixed order (deterministic).
constexpr int kLrTok = 8;
template <typename T>
__global__ void __launch_bounds__(128) lowrank_down_kernel(const T* x, int M, int K, long long ldx,
                                                           const T* down, int R, T* mid) {
  __shared__ float red[4][kLrTok];
  const int r = blockIdx.x, m0 = blockIdx.y * kLrTok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* dr = down + (long long)r * K;
  float acc[kLrTok];
#pragma unroll
  for (int i = 0; i < kLrTok; ++i) acc[i] = 0.f;
  const bool vec = ((K & 7) == 0) && ((ldx & 7) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(down) & 15) == 0);
  if (vec) {
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
      const uint4 dv = __ldg(reinterpret_cast<const uint4*>(dr) + c);
      const T* d8 = reinterpret_cast<const T*>(&dv);
#pragma unroll
      for (int i = 0; i < kLrTok; ++i) {
        if (m0 + i >= M) break;
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (long long)(m0 + i) * ldx) + c);
        const T* x8 = reinterpret_cast<const T*>(&xv);
#pragma unroll
        for (int j = 0; j < 8; j += 2)
          acc[i] = fmaf(DT<T>::to_f(x8[j]), DT<T>::to_f(d8[j]),
                        fmaf(DT<T>::to_f(x8[j + 1]), DT<T>::to_f(d8[j + 1]), acc[i]));
      }
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float dv = DT<T>::to_f(dr[k]);
#pragma unroll
      for (int i = 0; i < kLrTok; ++i)
        if (m0 + i < M) acc[i] = fmaf(DT<T>::to_f(x[(long long)(m0 + i) * ldx + k]), dv, acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < kLrTok; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < kLrTok; ++i) red[warp][i] = acc[i];
  }
  __syncthreads();
  if (threadIdx.x < kLrTok && m0 + (int)threadIdx.x < M) {
    const int i = threadIdx.x;
    const float v = (red[0][i] + red[1][i]) + (red[2][i] + red[3][i]);
    mid[(long long)(m0 + i) * R + r] = DT<T>::from_f(v);
  }
}

cudaError_t launch_lowrank_down(const void* x, int dtype, int M, int K, long long ldx, const void* down, int R,
                                void* mid, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  const dim3 grid(R, (M + kLrTok - 1) / kLrTok);
  if (dtype == IC_DTYPE_BF16)
    lowrank_down_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>((const __nv_bfloat16*)x, M, K, ldx,
                                                             (const __nv_bfloat16*)down, R, (__nv_bfloat16*)mid);
  else
    lowrank_down_kernel<__half><<<grid, 128, 0, st>>>((const __half*)x, M, K, ldx, (const __half*)down, R,
                                                      (__half*)mid);
  return cudaGetLastError();
}

// out[m, n] = T(out[m, n] + scale * sum_r mid[m, r] * up[n, r]) (out.addmm_,
// _ops.py:243): fp32 sums over the rank in chunks of 64 (R <= 256).
template <typename T>
__global__ void __launch_bounds__(256) lowrank_add_kernel(T* out, int M, int N, long long ldo, const T* mid,
                                                          const T* up, int R, float scale) {
  __shared__ float ms[16][64];
  const int m0 = blockIdx.y * 16;
  const int n = blockIdx.x * 256 + threadIdx.x;
  float l[16];
#pragma unroll
  for (int mm = 0; mm < 16; ++mm) l[mm] = 0.f;
  for (int r0 = 0; r0 < R; r0 += 64) {
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int mm = i / 64, r = r0 + i % 64;
      ms[mm][i % 64] = (m0 + mm < M && r < R) ? DT<T>::to_f(mid[(long long)(m0 + mm) * R + r]) : 0.f;
    }
    __syncthreads();
    if (n < N) {
      float u[64];
#pragma unroll
      for (int r = 0; r < 64; ++r) u[r] = (r0 + r < R) ? DT<T>::to_f(up[(long long)n * R + r0 + r]) : 0.f;
#pragma unroll
      for (int mm = 0; mm < 16; ++mm) {
#pragma unroll
        for (int r = 0; r < 64; ++r) l[mm] = fmaf(ms[mm][r], u[r], l[mm]);
      }
    }
  }
  if (n >= N) return;
#pragma unroll
  for (int mm = 0; mm < 16; ++mm) {
    if (m0 + mm >= M) break;
    T* o = out + (long long)(m0 + mm) * ldo + n;
    *o = DT<T>::from_f(DT<T>::to_f(*o) + scale * l[mm]);
  }
}

cudaError_t launch_lowrank_add(void* out, int dtype, int M, int N, long long ldo, const void* mid, const void* up,
                               int R, float scale, cudaStream_t st) {
  const dim3 grid((N + 255) / 256, (M + 15) / 16);
  if (dtype == IC_DTYPE_BF16)
    lowrank_add_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((__nv_bfloat16*)out, M, N, ldo,
                                                            (const __nv_bfloat16*)mid, (const __nv_bfloat16*)up, R,
                                                            scale);
  else
    lowrank_add_kernel<__half><<<grid, 256, 0, st>>>((__half*)out, M, N, ldo, (const __half*)mid,
                                                     (const __half*)up, R, scale);
  return cudaGetLastError();
}

// ------------------------------------------------------------ unpack
__global__ void unpack_i4_i8_kernel(const uint8_t* p, int N, int K, long long ldp, int8_t* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)N * K;
  if (i >= total) return;
  const long long n = i / K, k = i % K;
  const uint8_t b = p[n * ldp + k / 2];
  int v = (k & 1) ? (b >> 4) : (b & 15);
  out[i] = (int8_t)(v >= 8 ? v - 16 : v);
}

__global__ void unpack_i4_f16_kernel(const uint8_t* p, int N, int K, long long ldp, const void* scale,
                                     int scale_dtype, int G, int gs, __half* out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)N * K;
  if (i >= total) return;
  const long long n = i / K, k = i % K;
  const uint8_t b = p[n * ldp + k / 2];
  int v = (k & 1) ? (b >> 4) : (b & 15);
  v = v >= 8 ? v - 16 : v;
  const size_t si = (size_t)n * G + (G > 1 ? k / gs : 0);
  const __half s = scale_dtype == IC_DTYPE_F16 ? reinterpret_cast<const __half*>(scale)[si]
                                               : __float2half_rn(reinterpret_cast<const float*>(scale)[si]);
  out[i] = __hmul(__int2half_rn(v), s);
}

// ------------------------------------------------------------ repack
// Reference packing: byte j of a row = q[2j] | q[2j+1] << 4 (low nibble = even
// k, _quant_utils.py:170-182).  Repacked layouts keep the row size and permute
// nibbles inside each 4-byte word (8 consecutive k) so that the GEMM's INT4
// expansion needs only shifts and masks:
//   layout 0 (W4A8):  byte b = q[b] | q[b+4] << 4                (two's complement)
//   layout 1 (W4A16): nibble t = q[2t] + 8, nibble t+4 = q[2t+1] + 8 (offset binary)
__global__ void repack_i4_kernel(const uint8_t* src, int N, int K, long long lds, uint8_t* dst, long long ldd,
                                 int layout) {
  const long long words = (K + 7) / 8;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)N * words) return;
  const long long n = i / words, w = i % words;
  const int nbytes = (K + 1) / 2;
  uint32_t q[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const long long k = w * 8 + t;
    uint32_t v = 0;
    if (k < K) {
      const uint8_t b = src[n * lds + k / 2];
      v = (k & 1) ? (b >> 4) : (b & 15);
    }
    q[t] = v;
  }
  uint32_t out = 0;
  if (layout == 0) {
#pragma unroll
    for (int b = 0; b < 4; ++b) out |= (q[b] | (q[b + 4] << 4)) << (8 * b);
  } else {
#pragma unroll
    for (int t = 0; t < 4; ++t) out |= ((q[2 * t] ^ 8u) << (4 * t)) | ((q[2 * t + 1] ^ 8u) << (4 * (t + 4)));
  }
#pragma unroll
  for (int b = 0; b < 4; ++b)
    if (w * 4 + b < nbytes) dst[n * ldd + w * 4 + b] = (uint8_t)(out >> (8 * b));
}

cudaError_t launch_repack(const uint8_t* src, int N, int K, long long lds, uint8_t* dst, long long ldd, int layout,
                          cudaStream_t st) {
  const long long total = (long long)N * ((K + 7) / 8);
  if (total == 0) return cudaSuccess;
  repack_i4_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, N, K, lds, dst, ldd, layout);
  return cudaGetLastError();
}

cudaError_t launch_unpack_i8(const uint8_t* p, int N, int K, long long ldp, int8_t* out, cudaStream_t st) {
  const long long total = (long long)N * K;
  if (total == 0) return cudaSuccess;
  unpack_i4_i8_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(p, N, K, ldp, out);
  return cudaGetLastError();
}

cudaError_t launch_unpack_f16(const uint8_t* p, int N, int K, long long ldp, const void* scale, int sdt, int G,
                              int gs, __half* out, cudaStream_t st) {
  const long long total = (long long)N * K;
  if (total == 0) return cudaSuccess;
  unpack_i4_f16_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(p, N, K, ldp, scale, sdt, G, gs, out);
  return cudaGetLastError();
}

}  // namespace ic

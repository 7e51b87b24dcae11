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

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct SkinnyArgs {
  const __half* x; int M, K; long long ldx;
  const uint8_t* w; int N; long long ldw;
  const void* scale; int scale_dtype; int G, group_size;
  const void* bias; int bias_dtype;
  const __half* lr_mid; const __half* lr_up; int R; float lr_scale;
  __half* out; long long ldo;
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

// 32 activations of token m at k in [k0, k0 + 32), zero past K or M.
__device__ __forceinline__ void load_x32(const SkinnyArgs& a, int m, long long k0, uint32_t (&w)[16]) {
  if (m >= a.M) {   // token slot past M: zeros, no loads
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = 0u;
    return;
  }
  if (k0 + 32 <= a.K && ((a.ldx & 7) == 0)) {
    const uint4* p = reinterpret_cast<const uint4*>(a.x + (long long)m * a.ldx + k0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 v = __ldg(p + i);
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
    return;
  }
  __half h[32];
#pragma unroll
  for (int i = 0; i < 32; ++i)
    h[i] = (m < a.M && k0 + i < a.K) ? a.x[(long long)m * a.ldx + k0 + i] : __float2half_rn(0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = *reinterpret_cast<uint32_t*>(&h[2 * i]);
}

template <int TT>
__global__ void __launch_bounds__(32 * kSkinnyWarps, 2) w4a16_skinny_kernel(const SkinnyArgs a) {
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
    __half2 sa[PF], sb[PF];
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int kb = kb0 + kSkinnyWarps * j;
      if (kb < nkb) {
        pa[j] = load_packed16(a, n0 + g, kb, t);
        pb[j] = load_packed16(a, n0 + g + 8, kb, t);
        const int grp = (a.G > 1) ? (kb * 128) / a.group_size : 0;
        sa[j] = __half2half2(load_scale(a, n0 + g, grp));
        sb[j] = __half2half2(load_scale(a, n0 + g + 8, grp));
      } else {
        pa[j] = pb[j] = make_uint4(0u, 0u, 0u, 0u);
        sa[j] = sb[j] = __half2half2(__float2half_rn(0.f));
      }
    }
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      const int kb = kb0 + kSkinnyWarps * j;
      if (kb >= nkb) break;
      uint32_t xw[TT][16];
#pragma unroll
      for (int i = 0; i < TT; ++i) load_x32(a, m0 + i * 8 + g, (long long)kb * 128 + 32 * t, xw[i]);
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
          if (a.repacked) {
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
          for (int i = 0; i < TT; ++i) mma_16816(d[i], a0, a1, a2, a3, xw[i][2 * s], xw[i][2 * s + 1]);
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
    __half o16 = __float2half_rn(v);
    if (a.lr_mid) {
      float l = 0.f;
#pragma unroll 8
      for (int j = 0; j < a.R; ++j)
        l = fmaf(__half2float(a.lr_mid[(long long)m * a.R + j]), __half2float(a.lr_up[(long long)n * a.R + j]), l);
      o16 = __float2half_rn(__half2float(o16) + a.lr_scale * l);
    }
    a.out[(long long)m * a.ldo + n] = o16;
  }
}

cudaError_t launch_w4a16_skinny(const SkinnyArgs& a, cudaStream_t st) {
  // up to 32 tokens per CTA row of the grid; more tokens add CTA rows, each
  // streaming the (L2-resident) weights again
  const dim3 grid((a.N + 15) / 16, (a.M + 31) / 32);
  if (a.M <= 8) w4a16_skinny_kernel<1><<<grid, 32 * kSkinnyWarps, 0, st>>>(a);
  else if (a.M <= 16) w4a16_skinny_kernel<2><<<grid, 32 * kSkinnyWarps, 0, st>>>(a);
  else w4a16_skinny_kernel<4><<<grid, 32 * kSkinnyWarps, 0, st>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------ low rank
// mid[m, r] = fp16(sum_k x[m, k] * down[r, k]) with fp32 accumulation.
// One CTA per (rank r, tile of 8 tokens): each thread takes 8-value slices
// of K (16-byte loads of the down row and of the tile's token rows) and the
// CTA reduces its partial sums in a fixed order (deterministic).
constexpr int kLrTok = 8;
__global__ void __launch_bounds__(128) lowrank_down_kernel(const __half* x, int M, int K, long long ldx,
                                                           const __half* down, int R, __half* mid) {
  __shared__ float red[4][kLrTok];
  const int r = blockIdx.x, m0 = blockIdx.y * kLrTok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __half* dr = down + (long long)r * K;
  float acc[kLrTok];
#pragma unroll
  for (int i = 0; i < kLrTok; ++i) acc[i] = 0.f;
  const bool vec = ((K & 7) == 0) && ((ldx & 7) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(down) & 15) == 0);
  if (vec) {
    for (int c = threadIdx.x; c < K / 8; c += blockDim.x) {
      const uint4 dv = __ldg(reinterpret_cast<const uint4*>(dr) + c);
      const __half2* d2 = reinterpret_cast<const __half2*>(&dv);
#pragma unroll
      for (int i = 0; i < kLrTok; ++i) {
        if (m0 + i >= M) break;
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + (long long)(m0 + i) * ldx) + c);
        const __half2* x2 = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = __half22float2(x2[j]), b = __half22float2(d2[j]);
          acc[i] = fmaf(a.x, b.x, fmaf(a.y, b.y, acc[i]));
        }
      }
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float dv = __half2float(dr[k]);
#pragma unroll
      for (int i = 0; i < kLrTok; ++i)
        if (m0 + i < M) acc[i] = fmaf(__half2float(x[(long long)(m0 + i) * ldx + k]), dv, acc[i]);
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
    mid[(long long)(m0 + i) * R + r] = __float2half_rn(v);
  }
}

cudaError_t launch_lowrank_down(const __half* x, int M, int K, long long ldx, const __half* down, int R,
                                __half* mid, cudaStream_t st) {
  if (M == 0) return cudaSuccess;
  const dim3 grid(R, (M + kLrTok - 1) / kLrTok);
  lowrank_down_kernel<<<grid, 128, 0, st>>>(x, M, K, ldx, down, R, mid);
  return cudaGetLastError();
}

// out[m, n] = fp16(out[m, n] + scale * sum_r mid[m, r] * up[n, r]); R <= 64.
__global__ void __launch_bounds__(256) lowrank_add_kernel(__half* out, int M, int N, long long ldo,
                                                          const __half* mid, const __half* up, int R,
                                                          float scale) {
  __shared__ float ms[16][64];
  const int m0 = blockIdx.y * 16;
  for (int i = threadIdx.x; i < 16 * 64; i += 256) {
    const int mm = i / 64, r = i % 64;
    ms[mm][r] = (m0 + mm < M && r < R) ? __half2float(mid[(long long)(m0 + mm) * R + r]) : 0.f;
  }
  __syncthreads();
  const int n = blockIdx.x * 256 + threadIdx.x;
  if (n >= N) return;
  float u[64];
#pragma unroll
  for (int r = 0; r < 64; ++r) u[r] = (r < R) ? __half2float(up[(long long)n * R + r]) : 0.f;
  for (int mm = 0; mm < 16 && m0 + mm < M; ++mm) {
    float l = 0.f;
#pragma unroll
    for (int r = 0; r < 64; ++r) l = fmaf(ms[mm][r], u[r], l);
    __half* o = out + (long long)(m0 + mm) * ldo + n;
    *o = __float2half_rn(__half2float(*o) + scale * l);
  }
}

cudaError_t launch_lowrank_add(__half* out, int M, int N, long long ldo, const __half* mid, const __half* up,
                               int R, float scale, cudaStream_t st) {
  const dim3 grid((N + 255) / 256, (M + 15) / 16);
  lowrank_add_kernel<<<grid, 256, 0, st>>>(out, M, N, ldo, mid, up, R, scale);
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

// (a2, a3, a4) Quantized-linear GEMMs on the 5th-generation tensor cores.
//
// One persistent, warp-specialised kernel template covers the three weight
// formats of the reference's forward path:
//
//   W_I8   int8 weights [N, K]          kind::i8   (W8A8, _ops.py:559-576)
//   W_I4   packed int4 weights [N, K/2] kind::i8   (W4A8, _ops.py:443-464)
//   W_I4F  packed int4 weights [N, K/2] kind::f16  (W4A16, _ops.py:466-481)
//
// Orientation ("swap AB").  The weight tile is the MMA's A operand (UMMA
// M = 128 weight rows) and the activation tile is the B operand (UMMA N = BN
// tokens), so the accumulator in tensor memory holds D[n, m]: TMEM lane = output
// feature n, TMEM column = token m.  Every per-feature quantity of the
// epilogue (weight scale s_w[n, g], bias[n], zero-point term) is then a scalar
// per thread, which is what makes the per-K-group rescale of group-quantised
// INT4 weights cheap: one FADD2 + one FFMA2 per two accumulator values.
//
// Per-K-group rescale (GROUPED).  For group scales s_w[n, g] (group size a
// multiple of 128, _quant_utils.py:255-270) the K loop is split into
// accumulation units of one group.  The MMA warp accumulates each group's int32
// partial P_g into one of two TMEM buffers; the epilogue warps read it back,
// add it to fp32 registers as acc += s_w[n, g] * P_g and hand the buffer back.
// Integer -> float conversion is done by the tensor core itself: the epilogue
// refills the buffer with the integer bit pattern of 1.5 * 2^23 (0x4B400000)
// and the MMA accumulates on top of it, so the buffer holds the IEEE bits of
// 1.5 * 2^23 + P_g (exact while |P_g| < 2^22; here |P_g| <= 2^21).  One FADD
// recovers P_g exactly.
//
// INT4 weights are expanded inside the kernel by two producer warps: the
// packed tile arrives by TMA, the warps turn nibbles into int8 (W_I4, stored
// as 16 * q in the high nibble: exact, the 1/16 is folded into the scale) or
// into fp16(q * s) (W_I4F, exactly the reference's dequantised weight) and
// write it in the 128-byte-swizzled K-major layout the MMA reads.
//
// Warp roles: 0 = TMA producer, 1 = MMA issuer (+ TMEM owner), 2-3 = INT4
// expansion, 4.. = epilogue (4 or 8 warps).  Every wait is bounded.
#include "ic_common.cuh"

namespace ic {

enum WMode : int { W_I8 = 0, W_I4 = 1, W_I4F = 2 };

struct GemmArgs {
  int M;            // tokens
  int N;            // output features (weight rows)
  int K;            // reduction length (elements)
  int num_kb;       // K blocks of 128 bytes of activation row
  int G;            // number of scale groups (1 = per channel)
  int kb_per_group; // K blocks per scale group (GROUPED)
  int m_tiles, n_tiles;
  const float* s_w;         // [N, G]
  const void* w_scale;      // W_I4F: [N, G] f16/f32
  int w_scale_dtype;
  int group_size;
  const float* s_a;         // [M]
  const void* bias;
  int bias_dtype;
  const float* rowsum;      // [M]
  const float* zp_corr;     // [N]
  void* out;
  int out_dtype;
  long long ldo;
};

constexpr int kTileN = 128;            // weight rows per tile (UMMA M)
constexpr uint32_t kMagic = 0x4B400000u;
constexpr float kMagicF = 12582912.0f; // 1.5 * 2^23

template <int MODE, int BN, bool GROUPED>
struct Cfg {
  static constexpr int EPI = (BN > 128) ? 8 : 4;                 // epilogue warps
  static constexpr int CPT = BN / (EPI / 4);                      // columns per epilogue thread
  static constexpr int THREADS = 32 * (4 + EPI);
  static constexpr int W_BYTES = kTileN * 128;                    // 16 KB
  static constexpr int X_BYTES = BN * 128;
  static constexpr int P_BYTES = (MODE == W_I4) ? kTileN * 64 : (MODE == W_I4F ? kTileN * 32 : 0);
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES + P_BYTES;
  static constexpr int STAGES_RAW = (220 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 6 ? 6 : STAGES_RAW;
  static constexpr int TMEM_COLS_RAW = 2 * BN;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 32 ? 32 : TMEM_COLS_RAW <= 64 ? 64
                                 : TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;   // + alignment slack
  static constexpr int KB_ELEMS = (MODE == W_I4F) ? 64 : 128;           // K elements per block
  static_assert(CPT % 32 == 0, "epilogue columns per thread must be a multiple of 32");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
  static_assert(STAGES >= 2, "pipeline depth");
  static_assert(!(GROUPED && MODE == W_I4F), "W4A16 folds scales into the weights");
};

// Nibble pairs -> int8 bytes holding 16*q (two's complement nibble in the
// high half of each byte).  Input word: 8 nibbles, k = 0..7 from the low end.
__device__ __forceinline__ void expand_i4_i8(uint32_t v, uint32_t& o0, uint32_t& o1) {
  const uint32_t lo = (v << 4) & 0xF0F0F0F0u;   // even k
  const uint32_t hi = v & 0xF0F0F0F0u;          // odd k
  o0 = __byte_perm(lo, hi, 0x5140);
  o1 = __byte_perm(lo, hi, 0x7362);
}

// Nibble pair i (byte i of v) -> half2 {q_even, q_odd} * s (fp16 products).
__device__ __forceinline__ uint32_t expand_i4_f16_pair(uint32_t xo, uint32_t yo, int i, __half2 s2) {
  // xo / yo: offset-binary low / high nibbles of each byte (n ^ 8), one per byte.
  const uint32_t sel = (uint32_t)i | ((uint32_t)(i + 4) << 8);
  uint32_t t = (__byte_perm(xo, yo, sel) & 0x00FF00FFu) | 0x64006400u;   // 1024 + (q + 8)
  __half2 h = *reinterpret_cast<__half2*>(&t);
  h = __hsub2(h, __half2half2(__ushort_as_half((unsigned short)0x6408u)));  // - 1032 -> q
  h = __hmul2(h, s2);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace ic

namespace ic {

template <int MODE, int BN, bool GROUPED>
__global__ void __launch_bounds__(Cfg<MODE, BN, GROUPED>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
               const GemmArgs a) {
  using C = Cfg<MODE, BN, GROUPED>;
  constexpr int S = C::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * C::STAGE_BYTES);
  uint64_t* full = bars;            // TMA -> consumers         (count 1 + tx)
  uint64_t* wready = bars + S;      // expansion warps -> MMA   (count 2)
  uint64_t* empty = bars + 2 * S;   // MMA commit -> TMA        (count 1)
  uint64_t* acc_full = bars + 3 * S;        // [2] MMA commit -> epilogue
  uint64_t* acc_empty = bars + 3 * S + 2;   // [2] epilogue -> MMA (count EPI)
  uint64_t* drain = bars + 3 * S + 4;       // abort path: MMA completion
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * S + 6);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&wready[s], 2);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], C::EPI);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = a.m_tiles * a.n_tiles;
  const int units = GROUPED ? a.G : 1;

  auto stage_w = [&](int s) { return smem + s * C::STAGE_BYTES; };
  auto stage_x = [&](int s) { return smem + s * C::STAGE_BYTES + C::W_BYTES; };
  auto stage_p = [&](int s) { return smem + s * C::STAGE_BYTES + C::W_BYTES + C::X_BYTES; };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        const int n_blk = tile / a.m_tiles, m_blk = tile % a.m_tiles;
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
          constexpr uint32_t wbytes = (MODE == W_I8) ? C::W_BYTES : C::P_BYTES;
          mbar_arrive_expect_tx(&full[s], (uint32_t)C::X_BYTES + wbytes);
          tma_load_2d(stage_x(s), &tm_x, &full[s], kb * C::KB_ELEMS, m_blk * BN);
          if constexpr (MODE == W_I8) tma_load_2d(stage_w(s), &tm_w, &full[s], kb * 128, n_blk * kTileN);
          else if constexpr (MODE == W_I4) tma_load_2d(stage_p(s), &tm_w, &full[s], kb * 64, n_blk * kTileN);
          else tma_load_2d(stage_p(s), &tm_w, &full[s], kb * 32, n_blk * kTileN);
        }
      }
      if (!ok) {
        // let the copies already issued land before the CTA exits
        volatile int never = 0;
        const int first = it > S ? it - S : 0;
        for (int j = first; j < it; ++j) mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = (MODE == W_I4F) ? idesc_f16(kTileN, BN, false) : idesc_i8(kTileN, BN);
      int it = 0, uc = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        for (int u = 0; ok && u < units; ++u, ++uc) {
          const int kb0 = GROUPED ? u * a.kb_per_group : 0;
          const int kb1 = GROUPED ? min(kb0 + a.kb_per_group, a.num_kb) : a.num_kb;
          const int b = uc & 1;
          if (!mbar_wait(&acc_empty[b], (uint32_t)(uc >> 1) & 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(b * BN);
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
            if constexpr (MODE != W_I8) {
              if (!mbar_wait(&wready[s], ph, abort_flag)) { ok = false; break; }
            }
            tc_fence_after();
            const uint64_t adesc = smem_desc_sw128(smem_u32(stage_w(s)));
            const uint64_t bdesc = smem_desc_sw128(smem_u32(stage_x(s)));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t acc = GROUPED ? 1u : ((kb > kb0 || k > 0) ? 1u : 0u);
              if constexpr (MODE == W_I4F) mma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, acc);
              else mma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, acc);
            }
            mma_commit(&empty[s]);
          }
          if (!ok) break;
          mma_commit(&acc_full[b]);
        }
      }
      if (!ok) {
        volatile int never = 0;
        mma_commit(drain);
        mbar_wait(drain, 0, &never);
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ INT4 expansion
    if constexpr (MODE != W_I8) {
      const int u = threadIdx.x - 64;   // 0..63
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        const int n_blk = tile / a.m_tiles;
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          uint8_t* W = stage_w(s);
          const uint8_t* P = stage_p(s);
          if constexpr (MODE == W_I4) {
#pragma unroll 2
            for (int i = 0; i < 8; ++i) {
              const int r = i * 16 + (u >> 2), c = u & 3;
              const uint4 p = *reinterpret_cast<const uint4*>(P + r * 64 + c * 16);
              uint4 o0, o1;
              expand_i4_i8(p.x, o0.x, o0.y);
              expand_i4_i8(p.y, o0.z, o0.w);
              expand_i4_i8(p.z, o1.x, o1.y);
              expand_i4_i8(p.w, o1.z, o1.w);
              *reinterpret_cast<uint4*>(W + sw128_offset(r, 2 * c)) = o0;
              *reinterpret_cast<uint4*>(W + sw128_offset(r, 2 * c + 1)) = o1;
            }
          } else {
            const int g = (a.G > 1) ? (kb * 64) / a.group_size : 0;
#pragma unroll 2
            for (int i = 0; i < 4; ++i) {
              const int r = i * 32 + (u >> 1), c = u & 1;
              const int n = n_blk * kTileN + r;
              __half sh = __float2half_rn(0.f);
              if (n < a.N) {
                const size_t si = (size_t)n * a.G + g;
                sh = (a.w_scale_dtype == IC_DTYPE_F16)
                         ? reinterpret_cast<const __half*>(a.w_scale)[si]
                         : __float2half_rn(reinterpret_cast<const float*>(a.w_scale)[si]);
              }
              const __half2 s2 = __half2half2(sh);
              const uint4 p = *reinterpret_cast<const uint4*>(P + r * 32 + c * 16);
              const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const uint32_t ob = pw[w] ^ 0x88888888u;
                const uint32_t xo = ob & 0x0F0F0F0Fu, yo = (ob >> 4) & 0x0F0F0F0Fu;
                uint4 o;
                o.x = expand_i4_f16_pair(xo, yo, 0, s2);
                o.y = expand_i4_f16_pair(xo, yo, 1, s2);
                o.z = expand_i4_f16_pair(xo, yo, 2, s2);
                o.w = expand_i4_f16_pair(xo, yo, 3, s2);
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 4 * c + w)) = o;
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&wready[s]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 4;
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int col0 = (e >> 2) * C::CPT;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    constexpr float wmul = (MODE == W_I4) ? 0.0625f : 1.0f;   // int4 held as 16*q
    if constexpr (GROUPED) {
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < C::CPT / 32; ++c)
          tmem_st32_const(tmem_base + lane_base + (uint32_t)(b * BN + col0 + 32 * c), kMagic);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&acc_empty[0]);
      mbar_arrive(&acc_empty[1]);
    }
    int uc = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
      const int n_blk = tile / a.m_tiles, m_blk = tile % a.m_tiles;
      const int n = n_blk * kTileN + 32 * q + lane;
      const bool nvalid = n < a.N;
      const float bias_n = (nvalid && a.bias) ? load_any(a.bias, a.bias_dtype, n) : 0.f;
      const float zpc_n = (nvalid && a.zp_corr) ? a.zp_corr[n] : 0.f;
      const int mbase = m_blk * BN + col0;
      if constexpr (GROUPED) {
        float acc[C::CPT];
#pragma unroll
        for (int j = 0; j < C::CPT; ++j) acc[j] = 0.f;
        for (int u = 0; u < units; ++u, ++uc) {
          const int b = uc & 1;
          const float sw = nvalid ? __ldg(&a.s_w[(size_t)n * a.G + u]) * wmul : 0.f;
          if (!mbar_wait(&acc_full[b], (uint32_t)(uc >> 1) & 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < C::CPT / 32; ++c) {
            const uint32_t ta = tmem_base + lane_base + (uint32_t)(b * BN + col0 + 32 * c);
            uint32_t r[32];
            tmem_ld32(ta, r);
            tmem_wait_ld();
            tmem_st32_const(ta, kMagic);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              acc[32 * c + j] = fmaf(__uint_as_float(r[j]) - kMagicF, sw, acc[32 * c + j]);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (!ok) break;
        if (nvalid) {
#pragma unroll
          for (int j = 0; j < C::CPT; ++j) {
            const int m = mbase + j;
            if (m < a.M) {
              float v = fmaf(acc[j], __ldg(&a.s_a[m]), bias_n);
              if (a.rowsum) v = fmaf(-__ldg(&a.rowsum[m]), zpc_n, v);
              store_out(a.out, a.out_dtype, (size_t)m * a.ldo + n, v);
            }
          }
        }
      } else {
        const int b = uc & 1;
        const float sw = (MODE == W_I4F) ? 1.f : (nvalid ? __ldg(&a.s_w[n]) * wmul : 0.f);
        if (!mbar_wait(&acc_full[b], (uint32_t)(uc >> 1) & 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < C::CPT / 32; ++c) {
          const uint32_t ta = tmem_base + lane_base + (uint32_t)(b * BN + col0 + 32 * c);
          uint32_t r[32];
          tmem_ld32(ta, r);
          tmem_wait_ld();
          if (nvalid) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = mbase + 32 * c + j;
              if (m < a.M) {
                float v;
                if constexpr (MODE == W_I4F) {
                  v = __uint_as_float(r[j]) + bias_n;
                } else {
                  v = fmaf((float)(int)r[j] * sw, __ldg(&a.s_a[m]), bias_n);
                  if (a.rowsum) v = fmaf(-__ldg(&a.rowsum[m]), zpc_n, v);
                }
                store_out(a.out, a.out_dtype, (size_t)m * a.ldo + n, v);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
        ++uc;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace ic

// ============================================================== host side
namespace ic {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled is fetched through the runtime so that the library
// does not link libcuda (it must load on hosts without a driver).
static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor [outer, inner] with row stride `ld_bytes`.
static bool make_tmap(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t inner,
                      uint64_t outer, uint64_t ld_bytes, uint32_t box_inner, uint32_t box_outer,
                      CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  static int cache[64] = {0};
  if (dev < 64 && cache[dev]) return cache[dev];
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) cache[dev] = n;
  return n;
}

template <int MODE, int BN, bool GROUPED>
static cudaError_t launch_gemm_t(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a,
                                 cudaStream_t st) {
  using C = Cfg<MODE, BN, GROUPED>;
  auto kern = gemm_tc_kernel<MODE, BN, GROUPED>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int tiles = a.m_tiles * a.n_tiles;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, C::THREADS, C::SMEM, st>>>(tw, tx, a);
  return cudaGetLastError();
}

// Token-tile width for M tokens.
static int pick_bn(int M, bool grouped) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return grouped ? 192 : 256;
}

template <int MODE, bool GROUPED>
static cudaError_t dispatch_bn(int bn, const CUtensorMap& tw, const CUtensorMap& tx, GemmArgs a,
                               cudaStream_t st) {
  a.m_tiles = (a.M + bn - 1) / bn;
  switch (bn) {
    case 32: return launch_gemm_t<MODE, 32, GROUPED>(tw, tx, a, st);
    case 64: return launch_gemm_t<MODE, 64, GROUPED>(tw, tx, a, st);
    case 128: return launch_gemm_t<MODE, 128, GROUPED>(tw, tx, a, st);
    case 192:
      if constexpr (GROUPED) return launch_gemm_t<MODE, 192, GROUPED>(tw, tx, a, st);
      else return cudaErrorInvalidValue;
    case 256:
      if constexpr (!GROUPED) return launch_gemm_t<MODE, 256, GROUPED>(tw, tx, a, st);
      else return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

// Entry used by ic_gemm_a8: xq [M, ldq] int8, w int8/int4.
cudaError_t launch_gemm_a8(const int8_t* xq, int M, int K, long long ldq, const void* w, int w_kind,
                           int N, long long ldw, GemmArgs a, int force_bn, cudaStream_t st,
                           const char** why) {
  CUtensorMap tx, tw;
  const bool grouped = a.G > 1;
  const int bn = force_bn ? force_bn : pick_bn(M, grouped);
  if (!make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)K, (uint64_t)M, (uint64_t)ldq, 128,
                 (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B)) {
    *why = "cuTensorMapEncodeTiled failed for the activation operand";
    return cudaErrorInvalidValue;
  }
  bool okw;
  if (w_kind == IC_W_INT8)
    okw = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, 128,
                    kTileN, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    okw = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)((K + 1) / 2), (uint64_t)N,
                    (uint64_t)ldw, 64, kTileN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!okw) {
    *why = "cuTensorMapEncodeTiled failed for the weight operand";
    return cudaErrorInvalidValue;
  }
  a.M = M; a.N = N; a.K = K;
  a.num_kb = (K + 127) / 128;
  a.n_tiles = (N + kTileN - 1) / kTileN;
  if (w_kind == IC_W_INT8) {
    return grouped ? dispatch_bn<W_I8, true>(bn, tw, tx, a, st) : dispatch_bn<W_I8, false>(bn, tw, tx, a, st);
  }
  return grouped ? dispatch_bn<W_I4, true>(bn, tw, tx, a, st) : dispatch_bn<W_I4, false>(bn, tw, tx, a, st);
}

// Entry used by ic_gemm_w4a16 for M above the skinny-kernel range.
cudaError_t launch_gemm_w4a16_tc(const void* x, int M, int K, long long ldx, const uint8_t* w, int N,
                                 long long ldw, GemmArgs a, int force_bn, cudaStream_t st, const char** why) {
  CUtensorMap tx, tw;
  const int bn = force_bn ? force_bn : pick_bn(M, false);
  if (!make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, 64,
                 (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B)) {
    *why = "cuTensorMapEncodeTiled failed for the activation operand";
    return cudaErrorInvalidValue;
  }
  if (!make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)((K + 1) / 2), (uint64_t)N, (uint64_t)ldw,
                 32, kTileN, CU_TENSOR_MAP_SWIZZLE_NONE)) {
    *why = "cuTensorMapEncodeTiled failed for the weight operand";
    return cudaErrorInvalidValue;
  }
  a.M = M; a.N = N; a.K = K;
  a.num_kb = (K + 63) / 64;
  a.n_tiles = (N + kTileN - 1) / kTileN;
  return dispatch_bn<W_I4F, false>(bn, tw, tx, a, st);
}

}  // namespace ic

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

#include <type_traits>

namespace ic {

// W_I4B: W4A16 with bf16 activations (bf16(q * s) weights, kind::f16 in bf16)
enum WMode : int { W_I8 = 0, W_I4 = 1, W_I4F = 2, W_I4B = 3 };
template <int MODE> constexpr bool kF16Kind = (MODE == W_I4F || MODE == W_I4B);

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
  int w_repacked;           // INT4 weights in the expansion-friendly layout (ic_repack_int4)
  const float* s_a;         // [M]
  const void* bias;
  int bias_dtype;
  const float* rowsum;      // [M]
  const float* zp_corr;     // [N]
  void* out;
  int out_dtype;
  long long ldo;
  // split-K: each (tile, split) work unit covers kb_per_unit consecutive K
  // blocks; with splits > 1 the epilogue stores fp32 partials (scaled by s_a
  // and s_w, without bias or zero-point term) to ws [splits, M, N] and
  // splitk_reduce_kernel finishes the output
  int splits;
  int kb_per_unit;
  float* ws;
  int group_m;      // tile order: all weight tiles of group_m consecutive token tiles, then the next group
  // optional epilogue after dequantisation + bias: act (0 none, 1 SiLU,
  // 2 GELU (erf), 3 GELU (tanh)), then + residual[m, n] (row stride ldr),
  // then (INT8-out) the row's running |max| into rowmax[m]
  int act;
  const void* residual;
  int residual_dtype;
  long long ldr;
  float* rowmax;
  // group-scaled tiles with a 16-bit output: the epilogue stages each slice
  // in shared memory and writes it with a TMA bulk-tensor store (tm_o)
  int tma_store;
};

// The activation epilogue of fused_int8_gemm_dequant
// (kernels/triton_int8_gemm.py:119-123): SiLU x * sigmoid(x), GELU
// 0.5 x (1 + erf(x / sqrt 2)); 3 adds the tanh form of GELU that Flux-class
// MLPs use (0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3)))).
__device__ __forceinline__ float apply_act(int act, float y) {
  if (act == 1) return y / (1.f + expf(-y));
  if (act == 2) return 0.5f * y * (1.f + erff(y * 0.70710678118654752f));
  if (act == 3) return 0.5f * y * (1.f + tanhf(0.79788456080286536f * fmaf(0.044715f * y, y * y, y)));
  return y;
}
__device__ __forceinline__ bool epi_extra(const GemmArgs& a) { return a.act || a.residual || a.rowmax; }
// apply_act as one out-of-line copy: the unrolled store calls it per value
// with the value in a register, instead of inlining the transcendental code
// 32 times per chunk.
__device__ __noinline__ float apply_act_call(int act, float y) { return apply_act(act, y); }

// Tile index -> (weight tile, token tile).  Tiles run in groups of group_m
// token tiles; within a group the token tile varies fastest.  A wave of CTAs
// then covers a few token tiles x many weight tiles, so both operands of the
// wave stay in L2 when the activations do not fit in it (large M).
__device__ __forceinline__ void tile_nm(const GemmArgs& a, int tile, int& n_blk, int& m_blk) {
  const int per_group = a.group_m * a.n_tiles;
  const int grp = tile / per_group;
  const int first_m = grp * a.group_m;
  const int gsz = min(a.group_m, a.m_tiles - first_m);
  const int r = tile - grp * per_group;
  m_blk = first_m + r % gsz;
  n_blk = r / gsz;
}

constexpr int kTileN = 128;            // weight rows per tile (UMMA M)
constexpr uint32_t kMagic = 0x4B400000u;
constexpr float kMagicF = 12582912.0f; // 1.5 * 2^23

// Shared-memory plan.  W_I8: one ring whose stages hold the weight tile and
// the activation tile (both by TMA).  W_I4 / W_I4F: three rings -- the packed
// weight tiles (P, by TMA, deep), the expanded weight tiles (W, written by the
// expansion warps) and the activation tiles (X, by TMA) -- so that the TMA
// latency of the packed stream is hidden independently of the MMA ring.
template <int MODE, int BN, bool GROUPED, bool PAIR = false>
struct Cfg {
  static constexpr bool I4 = (MODE != W_I8);
  // CTA pairs: the pair's tile is 256 weight rows x BN tokens; each CTA
  // holds 128 of the weight rows and BN / 2 of the token rows
  static constexpr int XROWS = PAIR ? BN / 2 : BN;
  static constexpr int TILE_N = PAIR ? 2 * kTileN : kTileN;
  // epilogue warps: group-scaled tiles keep 64 fp32 accumulators per thread
  // (one warp per 32 TMEM lanes x 64 columns); per-channel tiles stream.
  // (BN = 160, group-scaled: 8 warps of 80 columns, so that three accumulator
  // buffers fit in tensor memory)
  static constexpr int EPI = GROUPED ? (BN == 160 ? 8 : (BN >= 64 ? BN / 16 : 4)) : ((BN > 128) ? 8 : 4);
  static constexpr int CPT = BN / (EPI / 4);                      // columns per epilogue thread
  static constexpr int THREADS = 32 * (4 + EPI);
  static constexpr int W_BYTES = kTileN * 128;                    // 16 KB
  static constexpr int X_BYTES = XROWS * 128;
  static constexpr int P_BYTES = (MODE == W_I4) ? kTileN * 64 : (kF16Kind<MODE> ? kTileN * 32 : 0);
  // group-scaled tiles: four accumulator buffers when they fit in TMEM, and
  // two 1 KB constant atoms (the operands of the re-arming MMA) at offset 0
  static constexpr int NBUF = (GROUPED && BN <= 128) ? 4 : ((GROUPED && BN == 160) ? 3 : 2);
  static constexpr int MAGIC_BYTES = GROUPED ? 2048 : 0;
  static constexpr int BUDGET = 224 * 1024 - MAGIC_BYTES;
  // group-scaled tiles: each epilogue warp stages its 16-bit output, one
  // 32-token x 32-feature chunk (64-byte rows) at a time, for asynchronous
  // TMA stores (BN <= 192 with whole chunks: wider tiles leave no room)
  static constexpr int STG_WARP = (GROUPED && BN <= 192 && CPT % 32 == 0) ? 32 * 64 : 0;
  static constexpr int STG_BYTES = EPI * STG_WARP;
  // even: the two expansion warps own alternate stages
  static constexpr int S_P = I4 ? (STG_WARP ? 6 : 8) : 0;
  static constexpr int S_W = I4 ? 4 : 0;
  static constexpr int XSTAGE = I4 ? X_BYTES : (X_BYTES + W_BYTES);
  static constexpr int S_X_RAW = (BUDGET - S_P * P_BYTES - S_W * W_BYTES - STG_BYTES - (STG_WARP ? EPI * CPT * 4 : 0)) / XSTAGE;
  static constexpr int S_X = S_X_RAW > 6 ? 6 : S_X_RAW;
  static constexpr int OFF_X = MAGIC_BYTES;                       // X ring
  static constexpr int OFF_W = OFF_X + S_X * XSTAGE;              // W ring (I4)
  static constexpr int OFF_P = OFF_W + S_W * W_BYTES;             // P ring (I4)
  static constexpr int OFF_STG = OFF_P + S_P * P_BYTES;           // output staging (GROUPED)
  static constexpr int OFF_SA = OFF_STG + STG_BYTES;              // per-token scales of the tile (staged stores)
  static constexpr int SA_BYTES = STG_WARP ? EPI * CPT * 4 : 0;
  static constexpr int OFF_BAR = OFF_SA + SA_BYTES;
  static constexpr int TMEM_COLS_RAW = NBUF * BN;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 32 ? 32 : TMEM_COLS_RAW <= 64 ? 64
                                 : TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;               // barriers + alignment slack
  static constexpr int KB_ELEMS = kF16Kind<MODE> ? 64 : 128;      // K elements per block
  static_assert(EPI % 4 == 0, "epilogue warps cover the four TMEM lane quarters evenly");
  static_assert(CPT % 32 == 0 || (GROUPED && CPT % 16 == 0), "epilogue column slices of 32 (16 at the end)");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
  static_assert(S_X >= 2, "pipeline depth");
  static_assert(!(GROUPED && kF16Kind<MODE>), "W4A16 folds scales into the weights");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(!PAIR || (!kF16Kind<MODE> && BN % 32 == 0), "pair tiles: A8 kinds, BN / 2 a multiple of 16");
  static_assert(TMEM_COLS_RAW <= 512, "tensor memory");
};

// Nibble pairs -> int8 bytes holding 16*q (two's complement nibble in the
// high half of each byte).  Reference packing: 8 nibbles, k = 0..7 from the
// low end.
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

// Repacked layout 1: nibbles (t, t+4) of a word hold (k_2t, k_2t+1) + 8.
__device__ __forceinline__ uint32_t expand_r16_pair(uint32_t v, int t, __half2 s2) {
  uint32_t bits = ((v >> (4 * t)) & 0x000F000Fu) | 0x64006400u;
  __half2 h = *reinterpret_cast<__half2*>(&bits);
  h = __hsub2(h, __half2half2(__ushort_as_half((unsigned short)0x6408u)));
  h = __hmul2(h, s2);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Packed accumulator pair (two fp32 in one 64-bit register):
// acc += s2 * (bits_as_float(r pair) + mg2), with mg2 = (-1.5 * 2^23) x 2.
__device__ __forceinline__ void acc2p(unsigned long long& acc, uint32_t r0, uint32_t r1,
                                      unsigned long long s2, unsigned long long mg2) {
  asm("{\n\t.reg .b64 rv;\n\t"
      "mov.b64 rv, {%1, %2};\n\t"
      "add.rn.f32x2 rv, rv, %4;\n\t"
      "fma.rn.f32x2 %0, rv, %3, %0;\n\t}"
      : "+l"(acc)
      : "r"(r0), "r"(r1), "l"(s2), "l"(mg2));
}

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}

// acc(pair) += s * (bits_as_float(r pair) - 1.5 * 2^23), two lanes per op.
__device__ __forceinline__ void acc2_magic(float& a0, float& a1, uint32_t r0, uint32_t r1, float s) {
  asm("{\n\t.reg .b64 ac, rv, mg, sc;\n\t"
      "mov.b64 ac, {%0, %1};\n\t"
      "mov.b64 rv, {%2, %3};\n\t"
      "mov.b64 mg, {%4, %4};\n\t"
      "mov.b64 sc, {%5, %5};\n\t"
      "add.rn.f32x2 rv, rv, mg;\n\t"
      "fma.rn.f32x2 ac, rv, sc, ac;\n\t"
      "mov.b64 {%0, %1}, ac;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(r0), "r"(r1), "f"(-kMagicF), "f"(s));
}

// Rare epilogue forms of store_chunk_t (activation, residual add, INT8-out
// row maxima, zero-point row sums): one non-inlined, rolled loop, so that the
// common store below stays a short unrolled sequence.  The common path runs
// once per tile from cold instruction-cache lines; with these forms inlined
// 32 times per chunk and per output type it was several times longer.
template <typename T, bool STG>
__device__ __noinline__ void store_chunk_rare(const GemmArgs& a, T* out, const float* v, int m0, int n,
                                              bool nvalid, float bias_n, float zpc_n, int lane, int width,
                                              T* stg) {
  const int ml = m0 + lane;
  const bool has_rs = a.rowsum != nullptr;
  const float sa_l = (ml < a.M) ? __ldg(&a.s_a[ml]) : 0.f;
  const float rs_l = (has_rs && ml < a.M) ? __ldg(&a.rowsum[ml]) : 0.f;
  const int jmax = nvalid ? min(width, a.M - m0) : 0;   // valid tokens in this chunk
  T* p = STG ? stg + lane : out + (size_t)m0 * a.ldo + n;
#pragma unroll 1
  for (int j = 0; j < 32; ++j) {
    const float sa = __shfl_sync(0xffffffffu, sa_l, j);
    const float rs = __shfl_sync(0xffffffffu, rs_l, j);
    float y = fmaf(v[j], sa, bias_n);
    if (has_rs) y = fmaf(-rs, zpc_n, y);
    y = apply_act(a.act, y);
    if (a.residual && j < jmax) y += load_any(a.residual, a.residual_dtype, (size_t)(m0 + j) * a.ldr + n);
    if (a.rowmax) {   // one atomic per token per warp: the max over the warp's 32 features first
      float am = (j < jmax) ? fabsf(y) : 0.f;
      asm("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(am));
      if (lane == 0 && m0 + j < a.M) atomicMax(reinterpret_cast<int*>(a.rowmax) + m0 + j, __float_as_int(am));
    }
    if (STG || j < jmax) {
      if constexpr (sizeof(T) == 4) *p = y;
      else if constexpr (std::is_same<T, __half>::value) *p = __float2half_rn(y);
      else *p = __float2bfloat16_rn(y);
    }
    p += STG ? 32 : a.ldo;
  }
}

// Store 32 consecutive tokens [m0, m0 + 32) of output feature n:
// out[m, n] = act(v[j] * s_a[m] + bias_n), the activation (ACT) out of line
// per value.  Lane j loads the per-token scale of token m0 + j (coalesced)
// and shuffles it to all.
// STG: write the values into a staging slice in shared memory instead (row
// j of 64 bytes = the 32 features of token m0 + j), every row, valid or not;
// the TMA store that follows clips the rows and features outside [M, N).
template <typename T, bool STG, bool SAS, bool ACT>
__device__ __forceinline__ void store_chunk_loop(const GemmArgs& a, T* out, const float* v, int m0, int n,
                                                 bool nvalid, float bias_n, int lane, int width, T* stg,
                                                 const float* sa_s) {
  const int ml = m0 + lane;
  float sa_b = (!SAS && ml < a.M) ? __ldg(&a.s_a[ml]) : 0.f;
  const int jmax = nvalid ? min(width, a.M - m0) : 0;   // valid tokens in this chunk
  T* p = STG ? stg + lane : out + (size_t)m0 * a.ldo + n;
  float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    float sa;
    if constexpr (SAS) {
      if ((j & 3) == 0) s4 = *reinterpret_cast<const float4*>(sa_s + j);
      sa = (j & 3) == 0 ? s4.x : (j & 3) == 1 ? s4.y : (j & 3) == 2 ? s4.z : s4.w;
    } else {
      sa = __shfl_sync(0xffffffffu, sa_b, j);
    }
    float y = fmaf(v[j], sa, bias_n);
    if constexpr (ACT) y = apply_act_call(a.act, y);
    if (STG || j < jmax) {
      if constexpr (sizeof(T) == 4) *p = y;
      else if constexpr (std::is_same<T, __half>::value) *p = __float2half_rn(y);
      else *p = __float2bfloat16_rn(y);
    }
    p += STG ? 32 : a.ldo;
    // keep the compiler from hoisting all 32 shuffles (register pressure):
    // the next 8 shuffles depend on this empty asm, issued after these stores
    if ((j & 7) == 7) asm volatile("" : "+f"(sa_b)::"memory");
  }
}

// The output form of store_chunk_loop for the GEMM's epilogue.  SAS: the
// chunk's 32 per-token scales are already in shared memory at sa_s (16-byte
// aligned; the same address in every lane, so broadcast loads) instead of
// being loaded and shuffled.  Activation-only epilogues use
// their own copy of the unrolled loop; residual, row maxima and zero point
// take store_chunk_rare.
template <typename T, bool STG = false, bool SAS = false>
__device__ __forceinline__ void store_chunk_t(const GemmArgs& a, T* out, const float* v, int m0, int n,
                                              bool nvalid, float bias_n, float zpc_n, int lane, int width,
                                              T* stg = nullptr, const float* sa_s = nullptr) {
  if (a.residual || a.rowmax || a.rowsum) {
    store_chunk_rare<T, STG>(a, out, v, m0, n, nvalid, bias_n, zpc_n, lane, width, stg);
  } else if (a.act) {
    store_chunk_loop<T, STG, SAS, true>(a, out, v, m0, n, nvalid, bias_n, lane, width, stg, sa_s);
  } else {
    store_chunk_loop<T, STG, SAS, false>(a, out, v, m0, n, nvalid, bias_n, lane, width, stg, sa_s);
  }
}

__device__ __forceinline__ void store_chunk(const GemmArgs& a, const float* v, int m0, int n, bool nvalid,
                                            float bias_n, float zpc_n, int lane, int width = 32) {
  if (a.out_dtype == IC_DTYPE_F16)
    store_chunk_t(a, reinterpret_cast<__half*>(a.out), v, m0, n, nvalid, bias_n, zpc_n, lane, width);
  else if (a.out_dtype == IC_DTYPE_BF16)
    store_chunk_t(a, reinterpret_cast<__nv_bfloat16*>(a.out), v, m0, n, nvalid, bias_n, zpc_n, lane, width);
  else
    store_chunk_t(a, reinterpret_cast<float*>(a.out), v, m0, n, nvalid, bias_n, zpc_n, lane, width);
}

// Split-K partial of 32 consecutive tokens of feature n:
// ws[split, m, n] = v[j] * s_a[m] (fp32; bias and zero point come in the
// reduce; W4A16 has no activation scale: s_a == nullptr).
__device__ __forceinline__ void store_partial(const GemmArgs& a, const float* v, int split, int m0, int n,
                                              bool nvalid, int lane, int width = 32) {
  const int ml = m0 + lane;
  const float sa_b = (ml < a.M) ? (a.s_a ? __ldg(&a.s_a[ml]) : 1.f) : 0.f;
  const int jmax = nvalid ? min(width, a.M - m0) : 0;
  float* p = a.ws + ((size_t)split * a.M + m0) * a.N + n;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float sa = __shfl_sync(0xffffffffu, sa_b, j);
    if (j < jmax) *p = v[j] * sa;
    p += a.N;
  }
}

// out[m, n] = epilogue(sum_s ws[s, m, n] + bias[n] - rowsum[m] * zp_corr[n])
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmArgs a) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long MN = (long long)a.M * a.N;
  if (i >= MN) return;
  const int m = (int)(i / a.N), n = (int)(i % a.N);
  float v = 0.f;
  for (int s = 0; s < a.splits; ++s) v += a.ws[(long long)s * MN + i];
  const float bias_n = a.bias ? load_any(a.bias, a.bias_dtype, n) : 0.f;
  const float rs = a.rowsum ? a.rowsum[m] : 0.f;
  const float zc = a.zp_corr ? a.zp_corr[n] : 0.f;
  float y = fmaf(-rs, zc, v + bias_n);
  if (epi_extra(a)) {
    y = apply_act(a.act, y);
    if (a.residual) y += load_any(a.residual, a.residual_dtype, (size_t)m * a.ldr + n);
    if (a.rowmax) atomicMax(reinterpret_cast<int*>(a.rowmax) + m, __float_as_int(fabsf(y)));
  }
  store_out(a.out, a.out_dtype, (size_t)m * a.ldo + n, y);
}

// INT8 output with a row-global scale: s_c[m] = max(rowmax[m], 1e-8) / 127,
// q = rint(y / s_c) ties to even (the quantiser of
// kernels/triton_quantize.py:43-54), from the fp32 epilogue values y.
__global__ void __launch_bounds__(256) requant_rows_kernel(const float* y, int M, int N, long long ldy,
                                                           const float* rowmax, int8_t* q, long long ldq,
                                                           float* s_c) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)M * N) return;
  const int m = (int)(i / N), n = (int)(i % N);
  const float s = __fdiv_rn(fmaxf(rowmax[m], 1e-8f), 127.0f);
  if (n == 0) s_c[m] = s;
  const float t = __fdiv_rn(y[(long long)m * ldy + n], s);
  q[(long long)m * ldq + n] = (int8_t)max(-128, min(127, __float_as_int(t + 12582912.0f) - 0x4B400000));
}

cudaError_t launch_requant_rows(const float* y, int M, int N, long long ldy, const float* rowmax, int8_t* q,
                                long long ldq, float* s_c, cudaStream_t st) {
  const long long mn = (long long)M * N;
  if (mn == 0) return cudaSuccess;
  requant_rows_kernel<<<(unsigned)((mn + 255) / 256), 256, 0, st>>>(y, M, N, ldy, rowmax, q, ldq, s_c);
  return cudaGetLastError();
}

// W4A16: out[m, n] = fp16(v[j] + bias_n) (no activation scale).
template <typename T>
__device__ __forceinline__ void store_chunk_raw(const GemmArgs& a, const float* v, int m0, int n, bool nvalid,
                                                float bias_n) {
  T* out = reinterpret_cast<T*>(a.out);
  const int jmax = nvalid ? min(32, a.M - m0) : 0;
  T* p = out + (size_t)m0 * a.ldo + n;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < jmax) *p = DT<T>::from_f(v[j] + bias_n);
    p += a.ldo;
  }
}

// bf16(q * s) pairs from fp32 products (exact for 4-bit q and fp16-valued s);
// nibbles in offset binary (q + 8).
__device__ __forceinline__ uint32_t bf16_pair_q(uint32_t n0, uint32_t n1, float s) {
  const float q0 = __uint_as_float(0x4B000000u | n0) - 8388616.0f;
  const float q1 = __uint_as_float(0x4B000000u | n1) - 8388616.0f;
  const __nv_bfloat162 h = __floats2bfloat162_rn(q0 * s, q1 * s);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace ic

namespace ic {

#if defined(IC_TRACE)
// Tuning-only instrumentation (never in the shipped build): cycles spent per
// pipeline role, summed over CTAs.
__device__ unsigned long long g_ic_trace[16];
#define IC_T0() long long _t0 = clock64()
#define IC_TADD(i) atomicAdd(&g_ic_trace[i], (unsigned long long)(clock64() - _t0))
#else
#define IC_T0()
#define IC_TADD(i)
#endif

template <int MODE, int BN, bool GROUPED, bool PAIR>
__global__ void __launch_bounds__(Cfg<MODE, BN, GROUPED, PAIR>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
               const __grid_constant__ CUtensorMap tm_o, const GemmArgs a) {
  using C = Cfg<MODE, BN, GROUPED, PAIR>;
  constexpr int SX = C::S_X, SW = C::S_W, SP = C::S_P;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* x_full = bars;                    // [SX] TMA -> MMA (count 1 + tx)
  uint64_t* x_empty = bars + SX;              // [SX] MMA commit -> TMA
  uint64_t* w_full = bars + 2 * SX;           // [SW] expansion -> MMA (I4)
  uint64_t* w_empty = w_full + SW;            // [SW] MMA commit -> expansion (I4)
  uint64_t* p_full = w_empty + SW;            // [SP] TMA -> expansion (I4)
  constexpr int NB = C::NBUF;
  uint64_t* acc_full = p_full + SP;           // [NB] MMA commit -> epilogue
  uint64_t* acc_empty = acc_full + NB;        // [NB] epilogue -> MMA (count EPI)
  uint64_t* drain = acc_empty + NB;           // abort path: MMA completion
  uint64_t* fin = drain + 1;                  // pairs: end-of-kernel handshake
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pairs: rank 0 (the leader) issues the pair MMAs and owns the
  // barriers they wait on (operands full, accumulator free); both CTAs own
  // the barriers the MMA commits release (operands free, accumulator full)
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = (rank == 0);
  auto lead = [&](uint64_t* bar) -> uint32_t { return mapa_u32(smem_u32(bar), 0u); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SX; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(&w_full[s], PAIR ? 2 : 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int s = 0; s < SP; ++s) mbar_init(&p_full[s], 1);
    for (int b = 0; b < NB; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], PAIR ? 2 * C::EPI : C::EPI);
    }
    mbar_init(drain, 1);
    mbar_init(fin, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc2(tmem_slot, C::TMEM_COLS);
      tmem_relinquish2();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  if constexpr (GROUPED) {
    // Constant operands of the re-arming MMA: every fp16 of atom A is 1536,
    // every fp16 of atom B is 512, so a K = 16 product is 16 * 1536 * 512 =
    // 1.5 * 2^23 exactly, whose fp32 bits are the magic 0x4B400000.
    uint32_t* m = reinterpret_cast<uint32_t*>(smem);
    for (int i = threadIdx.x; i < 512; i += blockDim.x) m[i] = (i < 256) ? 0x66006600u : 0x60006000u;
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();   // the peer's barriers are initialised
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_units = a.m_tiles * a.n_tiles * a.splits;
  const int wu0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int wu_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int row0 = (int)rank * kTileN;   // this CTA's first weight row inside the tile
  // accumulation units (one K group each when GROUPED) per work unit
  const int units = GROUPED ? a.kb_per_unit / a.kb_per_group : 1;

  auto x_stage = [&](int s) { return smem + C::OFF_X + s * C::XSTAGE + (C::I4 ? 0 : C::W_BYTES); };
  auto w_stage = [&](int s) {
    return C::I4 ? smem + C::OFF_W + s * C::W_BYTES : smem + C::OFF_X + s * C::XSTAGE;
  };
  auto p_stage = [&](int s) { return smem + C::OFF_P + s * C::P_BYTES; };

  if (warp == 0) {
    // ------------------------------------------- TMA producer (X, and W for W_I8)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int wu = wu0; ok && wu < total_units; wu += wu_step) {
        const int tile = wu / a.splits, kb_lo = (wu % a.splits) * a.kb_per_unit;
        int n_blk, m_blk;
        tile_nm(a, tile, n_blk, m_blk);
        for (int kb = kb_lo; kb < kb_lo + a.kb_per_unit; ++kb, ++it) {
          const int s = it % SX;
          const uint32_t ph = (uint32_t)(it / SX) & 1u;
          { IC_T0();
          const bool got = PAIR ? mbar_wait_cl(&x_empty[s], ph ^ 1u, abort_flag)
                                : mbar_wait(&x_empty[s], ph ^ 1u, abort_flag);
          if (!got) { ok = false; break; }
          IC_TADD(8); }
          if constexpr (PAIR) {
            // both halves land on the leader's barrier; the leader expects them
            if (leader) mbar_arrive_expect_tx(&x_full[s], (uint32_t)(2 * C::XSTAGE));
            tma_load_2d_pair(x_stage(s), &tm_x, lead(&x_full[s]), kb * C::KB_ELEMS, m_blk * BN + (int)rank * C::XROWS);
            if constexpr (MODE == W_I8)
              tma_load_2d_pair(w_stage(s), &tm_w, lead(&x_full[s]), kb * 128, n_blk * C::TILE_N + row0);
          } else {
            mbar_arrive_expect_tx(&x_full[s], (uint32_t)C::XSTAGE);
            tma_load_2d(x_stage(s), &tm_x, &x_full[s], kb * C::KB_ELEMS, m_blk * BN);
            if constexpr (MODE == W_I8) tma_load_2d(w_stage(s), &tm_w, &x_full[s], kb * 128, n_blk * kTileN);
          }
        }
      }
      // (the peer's loads complete on the leader's barriers: only the leader
      // can wait for them; it does so below)
      if (!ok && (!PAIR || leader)) {
        volatile int never = 0;
        const int first = it > SX ? it - SX : 0;
        for (int j = first; j < it; ++j) mbar_wait(&x_full[j % SX], (uint32_t)(j / SX) & 1u, &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && (!PAIR || leader)) {
      constexpr int MM = PAIR ? 2 * kTileN : kTileN;
      const uint32_t idesc = kF16Kind<MODE> ? idesc_f16(MM, BN, MODE == W_I4B) : idesc_i8(MM, BN);
      // GROUPED: the re-arming MMA (kind::f16, K = 16, accumulate off) writes
      // 1.5 * 2^23 as fp32 into every element of the buffer; the group's
      // kind::i8 MMAs then add the int32 partial onto those bits.  SBO = 0 makes
      // all 8-row groups of an operand read the same 1 KB atom.
      const uint32_t idesc_m = idesc_f16(MM, BN, false);
      const uint64_t magic_a = smem_desc_sw128(smem_u32(smem)) & ~(0x3FFFull << 32);
      const uint64_t magic_b = smem_desc_sw128(smem_u32(smem + 1024)) & ~(0x3FFFull << 32);
      int it = 0, uc = 0;
      bool ok = true;
      // the peer's operands and free accumulators are counted on these
      // barriers too: cluster-scope acquires for the pair form
      auto wait_any = [&](uint64_t* bar, uint32_t par) {
        return PAIR ? mbar_wait_cl(bar, par, abort_flag) : mbar_wait(bar, par, abort_flag);
      };
      for (int wu = wu0; ok && wu < total_units; wu += wu_step) {
        const int kb_lo = (wu % a.splits) * a.kb_per_unit;
        for (int u = 0; ok && u < units; ++u, ++uc) {
          const int kb0 = GROUPED ? kb_lo + u * a.kb_per_group : kb_lo;
          const int kb1 = GROUPED ? min(kb0 + a.kb_per_group, kb_lo + a.kb_per_unit) : kb_lo + a.kb_per_unit;
          const int b = uc % NB;
          { IC_T0();
          if (!wait_any(&acc_empty[b], (uint32_t)(uc / NB) & 1u)) { ok = false; break; }
          IC_TADD(0); }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(b * BN);
          if constexpr (GROUPED) {
            if constexpr (PAIR) mma_f16_2(d, magic_a, magic_b, idesc_m, 0u);
            else mma_f16(d, magic_a, magic_b, idesc_m, 0u);
          }
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int sx = it % SX;
            { IC_T0();
            if (!wait_any(&x_full[sx], (uint32_t)(it / SX) & 1u)) { ok = false; break; }
            IC_TADD(1); }
            const int sw = C::I4 ? it % SW : sx;
            if constexpr (C::I4) {
              IC_T0();
              if (!wait_any(&w_full[sw], (uint32_t)(it / SW) & 1u)) { ok = false; break; }
              IC_TADD(2);
            }
            tc_fence_after();
#if defined(IC_TRACE)
            const long long _ti = clock64();
#endif
            const uint64_t adesc = smem_desc_sw128(smem_u32(w_stage(sw)));
            const uint64_t bdesc = smem_desc_sw128(smem_u32(x_stage(sx)));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t acc = GROUPED ? 1u : ((kb > kb0 || k > 0) ? 1u : 0u);
              if constexpr (kF16Kind<MODE>) mma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, acc);
              else if constexpr (PAIR) mma_i8_2(d, adesc + 2 * k, bdesc + 2 * k, idesc, acc);
              else mma_i8(d, adesc + 2 * k, bdesc + 2 * k, idesc, acc);
            }
            if constexpr (PAIR) {
              mma_commit2_both(&x_empty[sx]);
              if constexpr (C::I4) mma_commit2_both(&w_empty[sw]);
            } else {
              mma_commit(&x_empty[sx]);
              if constexpr (C::I4) mma_commit(&w_empty[sw]);
            }
#if defined(IC_TRACE)
            atomicAdd(&g_ic_trace[13], (unsigned long long)(clock64() - _ti));
#endif
          }
          if (!ok) break;
          if constexpr (PAIR) mma_commit2_both(&acc_full[b]);
          else mma_commit(&acc_full[b]);
        }
      }
      if (!ok) {
        volatile int never = 0;
        if constexpr (PAIR) mma_commit2_local(drain);
        else mma_commit(drain);
        mbar_wait(drain, 0, &never);
      }
    }
  } else if (warp < 4) {
    // ------------------------------------- INT4 expansion (+ packed-tile TMA)
    // Warp 2 handles the even K blocks of the CTA's sequence, warp 3 the odd
    // ones; each waits for its own packed stage, expands it into a weight
    // stage, and re-arms the packed stage with the block SP steps ahead.
    if constexpr (C::I4) {
      const int xw = warp - 2;
      int issued = 0;
      auto issue_p = [&](int j) {
        const int wu_j = wu0 + (j / a.kb_per_unit) * wu_step;
        if (wu_j >= total_units) return;
        const int kb = (wu_j % a.splits) * a.kb_per_unit + j % a.kb_per_unit;
        int n_blk, m_unused;
        tile_nm(a, wu_j / a.splits, n_blk, m_unused);
        const int sp = j % SP;
        mbar_arrive_expect_tx(&p_full[sp], (uint32_t)C::P_BYTES);
        tma_load_2d(p_stage(sp), &tm_w, &p_full[sp], kb * (MODE == W_I4 ? 64 : 32), n_blk * C::TILE_N + row0);
        issued = j + 1;
      };
      if (lane == 0)
        for (int j = xw; j < SP; j += 2) issue_p(j);
      int it = 0;
      bool ok = true;
      const bool rp = a.w_repacked != 0;
      for (int wu = wu0; ok && wu < total_units; wu += wu_step) {
        int n_blk, m_unused;
        tile_nm(a, wu / a.splits, n_blk, m_unused);
        const int kb_lo = (wu % a.splits) * a.kb_per_unit;
        for (int kb = kb_lo; kb < kb_lo + a.kb_per_unit; ++kb, ++it) {
          if ((it & 1) != xw) continue;
          const int sp = it % SP, sw = it % SW;
          IC_T0();
          bool w_ok = mbar_wait(&p_full[sp], (uint32_t)(it / SP) & 1u, abort_flag);
          if (lane == 0) IC_TADD(5);
#if defined(IC_TRACE)
          _t0 = clock64();
#endif
          if (w_ok)
            w_ok = PAIR ? mbar_wait_cl(&w_empty[sw], ((uint32_t)(it / SW) & 1u) ^ 1u, abort_flag)
                        : mbar_wait(&w_empty[sw], ((uint32_t)(it / SW) & 1u) ^ 1u, abort_flag);
          if (lane == 0) IC_TADD(6);
#if defined(IC_TRACE)
          _t0 = clock64();
#endif
          if (!__all_sync(0xffffffffu, w_ok)) { ok = false; break; }
          uint8_t* W = w_stage(sw);
          const uint8_t* P = p_stage(sp);
          if constexpr (MODE == W_I4) {
            // all sixteen 16-byte loads first: one shared-memory latency per
            // stage instead of one per few rows
            const int c = lane & 3;
            uint4 pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = *reinterpret_cast<const uint4*>(P + (i * 8 + (lane >> 2)) * 64 + c * 16);
            if (rp) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                // layout 0: byte b of a word = q[k_b] | q[k_{b+4}] << 4
                const uint4 p = pk[i];
                const int r = i * 8 + (lane >> 2);
                uint4 o0, o1;
                o0.x = (p.x << 4) & 0xF0F0F0F0u; o0.y = p.x & 0xF0F0F0F0u;
                o0.z = (p.y << 4) & 0xF0F0F0F0u; o0.w = p.y & 0xF0F0F0F0u;
                o1.x = (p.z << 4) & 0xF0F0F0F0u; o1.y = p.z & 0xF0F0F0F0u;
                o1.z = (p.w << 4) & 0xF0F0F0F0u; o1.w = p.w & 0xF0F0F0F0u;
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 2 * c)) = o0;
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 2 * c + 1)) = o1;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const uint4 p = pk[i];
                const int r = i * 8 + (lane >> 2);
                uint4 o0, o1;
                expand_i4_i8(p.x, o0.x, o0.y);
                expand_i4_i8(p.y, o0.z, o0.w);
                expand_i4_i8(p.z, o1.x, o1.y);
                expand_i4_i8(p.w, o1.z, o1.w);
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 2 * c)) = o0;
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 2 * c + 1)) = o1;
              }
            }
          } else if constexpr (MODE == W_I4B) {
            const int g = (a.G > 1) ? (kb * 64) / a.group_size : 0;
            const int c = lane & 1;
            float sf[8];
            uint4 pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = i * 16 + (lane >> 1);
              const int n = n_blk * kTileN + r;
              sf[i] = 0.f;
              if (n < a.N) {
                const size_t si = (size_t)n * a.G + g;
                sf[i] = (a.w_scale_dtype == IC_DTYPE_F16) ? __half2float(reinterpret_cast<const __half*>(a.w_scale)[si])
                                                          : reinterpret_cast<const float*>(a.w_scale)[si];
              }
              pk[i] = *reinterpret_cast<const uint4*>(P + r * 32 + c * 16);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = i * 16 + (lane >> 1);
              const uint32_t pw[4] = {pk[i].x, pk[i].y, pk[i].z, pk[i].w};
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                uint4 o;
                uint32_t* op = &o.x;
#pragma unroll
                for (int t2 = 0; t2 < 4; ++t2) {
                  if (rp) {   // layout 1: nibbles (t, t + 4) = (k_2t, k_2t+1) + 8
                    op[t2] = bf16_pair_q((pw[w] >> (4 * t2)) & 0xFu, (pw[w] >> (4 * t2 + 16)) & 0xFu, sf[i]);
                  } else {    // reference packing: byte t = q[2t] | q[2t+1] << 4
                    const uint32_t ob = pw[w] ^ 0x88888888u;
                    op[t2] = bf16_pair_q((ob >> (8 * t2)) & 0xFu, (ob >> (8 * t2 + 4)) & 0xFu, sf[i]);
                  }
                }
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 4 * c + w)) = o;
              }
            }
          } else {
            const int g = (a.G > 1) ? (kb * 64) / a.group_size : 0;
            const int c = lane & 1;
            // scales and packed words of the lane's eight rows, all loads first
            __half sh[8];
            uint4 pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = i * 16 + (lane >> 1);
              const int n = n_blk * kTileN + r;
              sh[i] = __float2half_rn(0.f);
              if (n < a.N) {
                const size_t si = (size_t)n * a.G + g;
                sh[i] = (a.w_scale_dtype == IC_DTYPE_F16)
                            ? reinterpret_cast<const __half*>(a.w_scale)[si]
                            : __float2half_rn(reinterpret_cast<const float*>(a.w_scale)[si]);
              }
              pk[i] = *reinterpret_cast<const uint4*>(P + r * 32 + c * 16);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = i * 16 + (lane >> 1);
              const __half2 s2 = __half2half2(sh[i]);
              const uint32_t pw[4] = {pk[i].x, pk[i].y, pk[i].z, pk[i].w};
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                uint4 o;
                if (rp) {
                  o.x = expand_r16_pair(pw[w], 0, s2);
                  o.y = expand_r16_pair(pw[w], 1, s2);
                  o.z = expand_r16_pair(pw[w], 2, s2);
                  o.w = expand_r16_pair(pw[w], 3, s2);
                } else {
                  const uint32_t ob = pw[w] ^ 0x88888888u;
                  const uint32_t xo = ob & 0x0F0F0F0Fu, yo = (ob >> 4) & 0x0F0F0F0Fu;
                  o.x = expand_i4_f16_pair(xo, yo, 0, s2);
                  o.y = expand_i4_f16_pair(xo, yo, 1, s2);
                  o.z = expand_i4_f16_pair(xo, yo, 2, s2);
                  o.w = expand_i4_f16_pair(xo, yo, 3, s2);
                }
                *reinterpret_cast<uint4*>(W + sw128_offset(r, 4 * c + w)) = o;
              }
            }
          }
#if defined(IC_TRACE)
          __syncwarp();
          if (lane == 0) IC_TADD(7);
          _t0 = clock64();
#endif
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) IC_TADD(9);
          if (lane == 0) {
            if constexpr (PAIR) mbar_arrive_cluster(lead(&w_full[sw]));   // the leader's MMA reads it
            else mbar_arrive(&w_full[sw]);
            issue_p(it + SP);   // same parity as it: this warp's next use of the stage
          }
        }
      }
      if (!ok && lane == 0) {
        volatile int never = 0;
        for (int j = it; j < issued; ++j)
          if ((j & 1) == xw) mbar_wait(&p_full[j % SP], (uint32_t)(j / SP) & 1u, &never);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 4;
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int col0 = (e >> 2) * C::CPT;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    constexpr float wmul = (MODE == W_I4) ? 0.0625f : 1.0f;   // int4 held as 16*q
    tc_fence_before();
    __syncwarp();
    // the accumulator buffers are free: counted on the leader for pairs
    auto acc_free = [&](int b) {
      if constexpr (PAIR) mbar_arrive_cluster(lead(&acc_empty[b]));
      else mbar_arrive(&acc_empty[b]);
    };
    auto acc_wait = [&](int b, uint32_t par) {
      return PAIR ? mbar_wait_cl(&acc_full[b], par, abort_flag) : mbar_wait(&acc_full[b], par, abort_flag);
    };
    if (lane == 0)
      for (int b = 0; b < NB; ++b) acc_free(b);
    int uc = 0;
    bool ok = true;
    for (int wu = wu0; ok && wu < total_units; wu += wu_step) {
      const int tile = wu / a.splits, split = wu % a.splits;
#if defined(IC_TRACE)
      const long long _ts = clock64();
      if (warp == 4 && lane == 0) atomicAdd(&g_ic_trace[14], 1ull);
#endif
      int n_blk, m_blk;
      tile_nm(a, tile, n_blk, m_blk);
      const int n = n_blk * C::TILE_N + row0 + 32 * q + lane;
      const bool nvalid = n < a.N;
      const float bias_n = (nvalid && a.bias) ? load_any(a.bias, a.bias_dtype, n) : 0.f;
      const float zpc_n = (nvalid && a.zp_corr) ? a.zp_corr[n] : 0.f;
      const int mbase = m_blk * BN + col0;
      if constexpr (GROUPED) {
        // staged stores: this warp's per-token scales of the tile go to shared
        // memory now (coalesced, long before the store needs them)
        float* sa_s = reinterpret_cast<float*>(smem + C::OFF_SA) + e * C::CPT;
        if (C::STG_WARP > 0 && a.tma_store) {
          __syncwarp();   // the previous tile's reads of sa_s are done
#pragma unroll
          for (int i = 0; i < C::CPT / 32; ++i) {
            const int m = mbase + 32 * i + lane;
            sa_s[32 * i + lane] = m < a.M ? __ldg(&a.s_a[m]) : 0.f;
          }
          __syncwarp();
        }
        unsigned long long accp[C::CPT / 2];   // fp32 pairs
#pragma unroll
        for (int j = 0; j < C::CPT / 2; ++j) accp[j] = 0ull;
        const unsigned long long mg2 = pack2(-kMagicF, -kMagicF);
        const float* swrow = a.s_w + (size_t)(nvalid ? n : 0) * a.G + (size_t)split * units;
        float sw = nvalid ? __ldg(swrow) * wmul : 0.f;
        for (int u = 0; u < units; ++u, ++uc) {
          const int b = uc % NB;
          // next group's scale is fetched while this group is consumed
          const float sw_next = (nvalid && u + 1 < units) ? __ldg(swrow + u + 1) * wmul : 0.f;
#if defined(IC_TRACE)
          if (u == 0 && warp == 4 && lane == 0) atomicAdd(&g_ic_trace[12], (unsigned long long)(clock64() - _ts));
#endif
          IC_T0();
          if (!acc_wait(b, (uint32_t)(uc / NB) & 1u)) { ok = false; break; }
          if (warp == 4 && lane == 0) IC_TADD(3);
#if defined(IC_TRACE)
          _t0 = clock64();
          if (warp == 4 && lane == 0) atomicAdd(&g_ic_trace[10], 1ull);
#endif
          tc_fence_after();
          // read the whole buffer, then hand it back at once: the MMA warp
          // re-arms it itself, so nothing is written to tensor memory here
          constexpr int C32 = C::CPT / 32, C16 = (C::CPT % 32) / 16;
          uint32_t r[C32][32];
          uint32_t r16[C16 ? 16 : 1];
#pragma unroll
          for (int c = 0; c < C32; ++c)
            tmem_ld32(tmem_base + lane_base + (uint32_t)(b * BN + col0 + 32 * c), r[c]);
          if constexpr (C16 > 0) tmem_ld16(tmem_base + lane_base + (uint32_t)(b * BN + col0 + 32 * C32), r16);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) acc_free(b);
          const unsigned long long sw2 = pack2(sw, sw);
#pragma unroll
          for (int c = 0; c < C32; ++c)
#pragma unroll
            for (int j = 0; j < 16; ++j) acc2p(accp[16 * c + j], r[c][2 * j], r[c][2 * j + 1], sw2, mg2);
          if constexpr (C16 > 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) acc2p(accp[16 * C32 + j], r16[2 * j], r16[2 * j + 1], sw2, mg2);
          }
          if (warp == 4 && lane == 0) IC_TADD(4);
          sw = sw_next;
        }
        if (!ok) break;
#if defined(IC_TRACE)
        const long long _tst = clock64();
#endif
        // 16-bit output: each 32-token chunk is staged, then written by one
        // TMA store per warp
        uint8_t* stg = smem + C::OFF_STG + e * C::STG_WARP;
        const bool tstore = C::STG_WARP > 0 && a.tma_store != 0;
        const int n_w = n_blk * C::TILE_N + row0 + 32 * q;   // first feature of this warp's slice
#pragma unroll
        for (int c = 0; c < (C::CPT + 31) / 32; ++c) {
          const int width = (32 * c + 32 <= C::CPT) ? 32 : 16;   // a last slice of 16 when CPT % 32 == 16
          float v[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const bool in = 16 * c + j < C::CPT / 2;
            v[2 * j] = in ? __uint_as_float((uint32_t)accp[in ? 16 * c + j : 0]) : 0.f;
            v[2 * j + 1] = in ? __uint_as_float((uint32_t)(accp[in ? 16 * c + j : 0] >> 32)) : 0.f;
          }
          if (tstore) {
            // the previous chunk's store has finished reading the staging slice
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            if (a.out_dtype == IC_DTYPE_F16)
              store_chunk_t<__half, true, true>(a, nullptr, v, mbase + 32 * c, n, nvalid, bias_n, zpc_n, lane,
                                                width, reinterpret_cast<__half*>(stg), sa_s + 32 * c);
            else
              store_chunk_t<__nv_bfloat16, true, true>(a, nullptr, v, mbase + 32 * c, n, nvalid, bias_n, zpc_n,
                                                       lane, width, reinterpret_cast<__nv_bfloat16*>(stg),
                                                       sa_s + 32 * c);
            fence_proxy_async_smem();   // generic-proxy writes -> the TMA engine's reads
            __syncwarp();
            if (lane == 0 && n_w < a.N && mbase + 32 * c < a.M) {
              tma_store_2d(&tm_o, stg, n_w, mbase + 32 * c);
              bulk_commit();
            }
          } else if (a.splits > 1) {
            store_partial(a, v, split, mbase + 32 * c, n, nvalid, lane, width);
          } else {
            store_chunk(a, v, mbase + 32 * c, n, nvalid, bias_n, zpc_n, lane, width);
          }
        }
#if defined(IC_TRACE)
        if (warp == 4 && lane == 0) atomicAdd(&g_ic_trace[11], (unsigned long long)(clock64() - _tst));
#endif
      } else {
        const int b = uc % NB;
        const float sw = kF16Kind<MODE> ? 1.f : (nvalid ? __ldg(&a.s_w[n]) * wmul : 0.f);
        if (!acc_wait(b, (uint32_t)(uc / NB) & 1u)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < C::CPT / 32; ++c) {
          const uint32_t ta = tmem_base + lane_base + (uint32_t)(b * BN + col0 + 32 * c);
          uint32_t r[32];
          tmem_ld32(ta, r);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = kF16Kind<MODE> ? __uint_as_float(r[j]) : (float)(int)r[j] * sw;
          if (a.splits > 1) store_partial(a, v, split, mbase + 32 * c, n, nvalid, lane);
          else if constexpr (MODE == W_I4F) store_chunk_raw<__half>(a, v, mbase + 32 * c, n, nvalid, bias_n);
          else if constexpr (MODE == W_I4B) store_chunk_raw<__nv_bfloat16>(a, v, mbase + 32 * c, n, nvalid, bias_n);
          else store_chunk(a, v, mbase + 32 * c, n, nvalid, bias_n, zpc_n, lane);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) acc_free(b);
        ++uc;
      }
    }
  }

#if defined(IC_TRACE)
  if (threadIdx.x == 0) { IC_T0(); (void)_t0; }
#endif
  // the epilogue's bulk stores have completed before the CTA leaves
  if (C::STG_WARP > 0 && a.tma_store && warp >= 4 && lane == 0) bulk_wait0();
  __syncthreads();
  if constexpr (PAIR) {
    // Neither CTA may leave while the other can still reach its shared
    // memory (remote arrivals, TMA bytes counted on the leader, the leader's
    // MMAs reading the peer's operands): each tells the other it is done and
    // waits (bounded) for the same word back.
    if (threadIdx.x == 0) {
      volatile int never = 0;
      mbar_arrive_cluster(mapa_u32(smem_u32(fin), rank ^ 1u));
      mbar_wait_cl(fin, 0, &never);
    }
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc2(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
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

// INTCRUSH_TMA_STORE=0 keeps the group-scaled epilogue on plain stores (A/B
// comparisons).
static bool tma_store_enabled() {
  static const int v = [] { const char* e = getenv("INTCRUSH_TMA_STORE"); return (e && e[0] == '0') ? 0 : 1; }();
  return v == 1;
}

template <int MODE, int BN, bool GROUPED, bool PAIR = false>
static cudaError_t launch_gemm_t(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a_in,
                                 cudaStream_t st) {
  using C = Cfg<MODE, BN, GROUPED, PAIR>;
  auto kern = gemm_tc_kernel<MODE, BN, GROUPED, PAIR>;
  cudaError_t e = set_smem_once(kern, C::SMEM);
  if (e != cudaSuccess) return e;
  GemmArgs a = a_in;
  // group-scaled tiles with a 16-bit output (no split-K): the output tensor
  // [M, N] as a TMA map whose box is one epilogue warp's chunk (32 features
  // x 32 tokens); otherwise the map stays unused
  CUtensorMap to{};
  a.tma_store = 0;
  if constexpr (GROUPED) {
    const bool out16 = a.out_dtype == IC_DTYPE_F16 || a.out_dtype == IC_DTYPE_BF16;
    const uint64_t ld_bytes = (uint64_t)a.ldo * 2;
    if (C::STG_WARP > 0 && tma_store_enabled() && out16 && a.splits == 1 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
        ld_bytes % 16 == 0 &&
        make_tmap(&to, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.out, (uint64_t)a.N, (uint64_t)a.M, ld_bytes, 32, 32,
                  CU_TENSOR_MAP_SWIZZLE_NONE))
      a.tma_store = 1;
  }
  const int tiles = a.m_tiles * a.n_tiles * a.splits;   // work units
  if constexpr (!PAIR) {
    const int grid = tiles < num_sms() ? tiles : num_sms();
    kern<<<grid, C::THREADS, C::SMEM, st>>>(tw, tx, to, a);
    return cudaGetLastError();
  } else {
    // one CTA pair (cluster of 2) per pair of SMs, persistent over the tiles
    const int pairs = num_sms() / 2;
    const int grid = 2 * (tiles < pairs ? tiles : pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tw, tx, to, a);
  }
}

// CTA pairs (tcgen05 cta_group::2) for large problems: the pair shares one
// 256-row x BN-token tile, each CTA stages half of the token rows, which
// halves the activation traffic through each SM's shared memory per MAC.
// INTCRUSH_PAIR=0 keeps one CTA per tile (A/B comparisons).
static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("INTCRUSH_PAIR");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Token-tile width for M tokens.  INTCRUSH_FORCE_BN (32/64/128/192/256)
// overrides the choice; it exists for tuning runs.
static int forced_bn() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("INTCRUSH_FORCE_BN");
    v = e ? atoi(e) : 0;
  }
  return v;
}

// Widest tile for M, narrowed (down to 64 tokens) while the output tiles
// would cover less than half of the SMs: for small problems parallelism
// matters more than the per-instruction efficiency of wide MMAs.
static int pick_bn(int M, int N, bool grouped) {
  const int f = forced_bn();
  if (f) return f;
  int bn = M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : (grouped ? 192 : 256);
  const int n_tiles = (N + kTileN - 1) / kTileN;
  while (bn > 64 && ((M + bn - 1) / bn) * n_tiles * 2 < num_sms()) bn = (bn > 128) ? 128 : 64;
  return bn;
}

template <int MODE, bool GROUPED>
static cudaError_t dispatch_bn(int bn, const CUtensorMap& tw, const CUtensorMap& tx, GemmArgs a,
                               cudaStream_t st) {
  a.m_tiles = (a.M + bn - 1) / bn;
  {
    static const int gm_env = [] { const char* e = getenv("INTCRUSH_GROUP_M"); return e ? atoi(e) : 0; }();
    const int gm = gm_env > 0 ? gm_env : 16;
    a.group_m = gm < a.m_tiles ? gm : a.m_tiles;
  }
  switch (bn) {
    case 32: return launch_gemm_t<MODE, 32, GROUPED>(tw, tx, a, st);
    case 64: return launch_gemm_t<MODE, 64, GROUPED>(tw, tx, a, st);
    case 128: return launch_gemm_t<MODE, 128, GROUPED>(tw, tx, a, st);
    case 160:
      if constexpr (GROUPED) return launch_gemm_t<MODE, 160, GROUPED>(tw, tx, a, st);
      else return cudaErrorInvalidValue;
    case 192:
      if constexpr (GROUPED) return launch_gemm_t<MODE, 192, GROUPED>(tw, tx, a, st);
      else return cudaErrorInvalidValue;
    case 256: return launch_gemm_t<MODE, 256, GROUPED>(tw, tx, a, st);
    default: return cudaErrorInvalidValue;
  }
}

// Entry used by ic_gemm_a8: xq [M, ldq] int8, w int8/int4.
// Pair tile width for M x N, or 0 when pairs do not apply: one CTA pair per
// tile, enough tiles to give every pair of SMs several.
static int pick_pair_bn(int M, int N, bool grouped, int splits) {
  if (!pair_enabled() || splits != 1 || forced_bn()) return 0;
  static const int env_bn = [] { const char* e = getenv("INTCRUSH_PAIR_BN"); return e ? atoi(e) : 0; }();   // tuning
  const int bn = (grouped && (env_bn == 128 || env_bn == 160 || env_bn == 192)) ? env_bn : (grouped ? 192 : 256);
  const long long tiles = (long long)((M + bn - 1) / bn) * ((N + 2 * kTileN - 1) / (2 * kTileN));
  return tiles >= (long long)num_sms() ? bn : 0;   // >= 2 tiles per pair
}

template <int MODE>
static cudaError_t launch_pair(int bn, const CUtensorMap& tw, const CUtensorMap& tx, GemmArgs a, cudaStream_t st) {
  a.m_tiles = (a.M + bn - 1) / bn;
  a.n_tiles = (a.N + 2 * kTileN - 1) / (2 * kTileN);
  a.group_m = 16 < a.m_tiles ? 16 : a.m_tiles;
  if (a.G > 1) {
    switch (bn) {
      case 128: return launch_gemm_t<MODE, 128, true, true>(tw, tx, a, st);
      case 160: return launch_gemm_t<MODE, 160, true, true>(tw, tx, a, st);
      case 192: return launch_gemm_t<MODE, 192, true, true>(tw, tx, a, st);
      default: return cudaErrorInvalidValue;
    }
  }
  if (bn != 256) return cudaErrorInvalidValue;
  return launch_gemm_t<MODE, 256, false, true>(tw, tx, a, st);
}

cudaError_t launch_gemm_a8(const int8_t* xq, int M, int K, long long ldq, const void* w, int w_kind,
                           int N, long long ldw, GemmArgs a, int force_bn, cudaStream_t st,
                           const char** why) {
  CUtensorMap tx, tw;
  const bool grouped = a.G > 1;
  const int pbn = force_bn ? 0 : pick_pair_bn(M, N, grouped, a.splits < 1 ? 1 : a.splits);
  if (pbn) {
    if (!make_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)K, (uint64_t)M, (uint64_t)ldq, 128,
                   (uint32_t)(pbn / 2), CU_TENSOR_MAP_SWIZZLE_128B)) {
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
    a.splits = 1;
    a.kb_per_unit = a.num_kb;
    return w_kind == IC_W_INT8 ? launch_pair<W_I8>(pbn, tw, tx, a, st) : launch_pair<W_I4>(pbn, tw, tx, a, st);
  }
  const int bn = force_bn ? force_bn : pick_bn(M, N, grouped);
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
  if (a.splits < 1) a.splits = 1;
  a.kb_per_unit = a.num_kb / a.splits;
  cudaError_t e;
  if (w_kind == IC_W_INT8)
    e = grouped ? dispatch_bn<W_I8, true>(bn, tw, tx, a, st) : dispatch_bn<W_I8, false>(bn, tw, tx, a, st);
  else
    e = grouped ? dispatch_bn<W_I4, true>(bn, tw, tx, a, st) : dispatch_bn<W_I4, false>(bn, tw, tx, a, st);
  if (e != cudaSuccess || a.splits == 1) return e;
  const long long mn = (long long)M * N;
  splitk_reduce_kernel<<<(unsigned)((mn + 255) / 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

// Entry used by ic_gemm_w4a16 for M above the skinny-kernel range.
cudaError_t launch_gemm_w4a16_tc(const void* x, int x_dtype, int M, int K, long long ldx, const uint8_t* w, int N,
                                 long long ldw, GemmArgs a, int force_bn, cudaStream_t st, const char** why) {
  CUtensorMap tx, tw;
  const int bn = force_bn ? force_bn : pick_bn(M, N, false);
  const bool bf = x_dtype == IC_DTYPE_BF16;
  if (!make_tmap(&tx, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)K,
                 (uint64_t)M, (uint64_t)ldx * 2, 64, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B)) {
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
  if (a.splits < 1) a.splits = 1;
  a.kb_per_unit = a.num_kb / a.splits;
  cudaError_t e = bf ? dispatch_bn<W_I4B, false>(bn, tw, tx, a, st) : dispatch_bn<W_I4F, false>(bn, tw, tx, a, st);
  if (e != cudaSuccess || a.splits == 1) return e;
  // fp32 partials [splits, M, N] -> out = RN(sum + bias), no activation scale
  const long long mn = (long long)M * N;
  splitk_reduce_kernel<<<(unsigned)((mn + 255) / 256), 256, 0, st>>>(a);
  return cudaGetLastError();
}

// Split-K plan for the tcgen05 W4A16 path: token tiles of 128 (64 for
// M <= 64) and as many K parts as fill the SMs with one work unit each (at
// most 8, dividing the 64-wide K blocks).  Few output tiles leave most SMs
// idle on a K loop of K / 64 blocks; split, each unit runs one part.
void plan_w4a16_splits(int M, int N, int K, int* bn, int* splits) {
  const int b = M <= 64 ? 64 : 128;
  const long long tiles = (long long)((M + b - 1) / b) * ((N + kTileN - 1) / kTileN);
  const int nkb = (K + 63) / 64;
  int s = (int)(num_sms() / (tiles > 0 ? tiles : 1));
  if (s > 8) s = 8;
  if (s < 1) s = 1;
  while (s > 1 && nkb % s) --s;
  *bn = b;
  *splits = s;
}

}  // namespace ic

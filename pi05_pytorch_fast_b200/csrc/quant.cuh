// Fused Walsh-Hadamard rotation + per-token symmetric INT4 activation quant.
//
// Replaces the reference's quant_rot_rb<K,R> and quant_rows
// (pi05_fast/w4a4/csrc/int4_gemm.cu:396-477) with a register/warp-shuffle
// design for sm_100a:
//
//  * each row is held in registers: lane l of a warp loads 16-byte vectors
//    (8 fp16) at element offsets 256*c + 8*l, so element index bits 0-2 live
//    inside a thread, bits 3-7 across the 32 lanes and bits 8 and up across
//    the thread's chunks c and the row's warps;
//  * butterflies run in ascending stride order (h = 1, 2, 4, ...), exactly the
//    order of the reference, so every value is bit-identical: stride bits 0-2
//    and 8-10 are in-register, bits 3-7 use __shfl_xor_sync, and for
//    K = 16384 bits 11-13 go through one shared-memory transpose between the
//    8 warps of the CTA;
//  * staging FP16 = the HIP kernel's arithmetic: stages with stride < R
//    (R = K/256) in fp32, then the values are rounded to fp16 and every later
//    stage adds/subtracts in fp32 and rounds back to fp16 (int4_gemm.cu:404-426).
//    Here those later stages run as packed half2 adds (__hadd2/__hsub2, and
//    __hfma2 with a +-1 factor across lanes): for
//    fp16 a, b the single rounding fl16(a + b) equals fl16(fl32(a + b)),
//    because binary32 carries at least 2 x 11 + 2 significand bits (double
//    rounding through it is innocuous), so the result is bit-identical while
//    two values move per instruction and no conversions are needed;
//    staging FP32 = the reference's CPU emulation (pack.py:113-131);
//  * amax, sdiv = amax/7 + 1e-12 and codes = clamp(rint(v/sdiv), -7, 7) with
//    the IEEE quotient and round-half-even (int4_gemm.cu:427-449), computed
//    through a reciprocal with an exact fallback next to ties (quant_code);
//  * codes are written either as int8 (one code per byte, the layout the
//    tensor-core GEMM consumes) or as the reference's packed int32 words
//    (8 nibbles per word, element j at bits 4j).
#pragma once

#include "common.cuh"

namespace w4a4 {

constexpr int kQuantThreads = 256;

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void load8_half_as_float(const __half* p, float (&v)[8]) {
  const uint4 raw = ld_nc_v4(p);
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// GeGLU of the Gemma MLP as PyTorch's eager CUDA ops round it
// (F.gelu(gate, approximate="tanh") * up on fp16 tensors): the tanh-form
// GELU 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) in fp32 with the
// constants rounded to fp32, x^3 as (x x) x, the inner sum as one fused
// multiply-add, rounded to fp16; then the fp16 product with up (the exact
// fp32 product of two fp16 values, rounded once).  tanhf is CUDA's.
// Two values at a time: the fp32 arithmetic through the two-lane fp32
// instructions (each lane rounded as the scalar instruction) and both
// results rounded to fp16 by one packed conversion.
__device__ __forceinline__ __half2 gelu_tanh_h2(__half2 g) {
  const float2 x = __half22float2(g);
  const float2 x3 = __fmul2_rn(__fmul2_rn(x, x), x);
  const float2 inner = __fmul2_rn(make_float2(0.7978845608028654f, 0.7978845608028654f),
                                  __ffma2_rn(make_float2(0.044715f, 0.044715f), x3, x));
  const float2 t = make_float2(tanhf(inner.x), tanhf(inner.y));
  const float2 r = __fmul2_rn(__fmul2_rn(make_float2(0.5f, 0.5f), x), __fadd2_rn(make_float2(1.f, 1.f), t));
  return __floats2half2_rn(r.x, r.y);
}

// Eight fp16 GeGLU values from 16-byte vectors of gate and up.  The product
// is the fp16 multiply: the fp32 product of two fp16 values is exact, so
// rounding it to fp16 once is the correctly rounded fp16 product.
__device__ __forceinline__ uint4 geglu8(const uint4 g, const uint4 u) {
  uint4 r;
  const __half2* gh = reinterpret_cast<const __half2*>(&g);
  const __half2* uh = reinterpret_cast<const __half2*>(&u);
  __half2* rh = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) rh[i] = __hmul2_rn(gelu_tanh_h2(gh[i]), uh[i]);
  return r;
}

__device__ __forceinline__ void half8_to_float(const uint4 raw, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Packed fp32 pairs: elements (2i, 2i + 1) of a vector go through the
// sm_100 two-lane fp32 instructions (add / fma .rn.f32x2), each lane rounded
// exactly like the scalar instruction.  a - b is fma(b, -1, a): the product is
// exact, so its one rounding is that of the subtraction.
__device__ __forceinline__ void bfly2(float& a0, float& a1, float& b0, float& b1) {
  const float2 a = make_float2(a0, a1), b = make_float2(b0, b1);
  const float2 s = __fadd2_rn(a, b);
  const float2 d = __ffma2_rn(b, make_float2(-1.f, -1.f), a);
  a0 = s.x;
  a1 = s.y;
  b0 = d.x;
  b1 = d.y;
}

// Butterfly stage inside each 8-vector: pairs (j, j + h), lower keeps a + b,
// upper a - b (fp32, round to nearest).
template <int C>
__device__ __forceinline__ void stage_in_vector(float (&v)[C][8], int h) {
#pragma unroll
  for (int c = 0; c < C; ++c) {
    if (h == 1) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float a = v[c][j], b = v[c][j + 1];
        v[c][j] = __fadd_rn(a, b);
        v[c][j + 1] = __fsub_rn(a, b);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; j += 2)
        if (!(j & h)) bfly2(v[c][j], v[c][j + 1], v[c][j + h], v[c][j + h + 1]);
    }
  }
}

// Butterfly across lanes: partner lane = lane ^ m.  The lane with the bit
// clear holds the lower element a and keeps a + b; its partner keeps a - b:
// both are fma(mine, +-1, other), one rounding of the exact sum.
template <int C>
__device__ __forceinline__ void stage_across_lanes(float (&v)[C][8], int lane, int m) {
  const float sg = (lane & m) ? -1.f : 1.f;
  const float2 sg2 = make_float2(sg, sg);
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float2 mine = make_float2(v[c][j], v[c][j + 1]);
      const float2 other = make_float2(__shfl_xor_sync(0xffffffffu, mine.x, m),
                                       __shfl_xor_sync(0xffffffffu, mine.y, m));
      const float2 r = __ffma2_rn(mine, sg2, other);
      v[c][j] = r.x;
      v[c][j + 1] = r.y;
    }
}

// Butterfly between chunks c and c + h (element index bit log2(h) + 8).
template <int C>
__device__ __forceinline__ void stage_across_chunks(float (&v)[C][8], int h) {
#pragma unroll
  for (int c = 0; c < C; ++c)
    if (!(c & h))
#pragma unroll
      for (int j = 0; j < 8; j += 2) bfly2(v[c][j], v[c][j + 1], v[c + h][j], v[c + h][j + 1]);
}

// ---- packed-half2 stages: h[c][i] holds elements (8c' + 2i, 8c' + 2i + 1) of
// the float layout v[c][2i], v[c][2i + 1]; index bit b >= 1 of the 8-vector is
// bit b - 1 of i.
template <int C>
__device__ __forceinline__ void pack_half2(const float (&v)[C][8], __half2 (&h)[C][4]) {
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) h[c][i] = __floats2half2_rn(v[c][2 * i], v[c][2 * i + 1]);
}

template <int C>
__device__ __forceinline__ void h2_stage_in_vector(__half2 (&h)[C][4], int hi) {
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (!(i & hi)) {
        const __half2 a = h[c][i], b = h[c][i + hi];
        h[c][i] = __hadd2(a, b);
        h[c][i + hi] = __hsub2(a, b);
      }
}

// Lower lane: mine + other; upper lane: other - mine; both fma(mine, +-1,
// other) with one fp16 rounding of the exact result.
template <int C>
__device__ __forceinline__ void h2_stage_across_lanes(__half2 (&h)[C][4], int lane, int m) {
  const __half2 sg = __float2half2_rn((lane & m) ? -1.f : 1.f);
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 mine = h[c][i];
      const __half2 other = __shfl_xor_sync(0xffffffffu, mine, m);
      h[c][i] = __hfma2(mine, sg, other);
    }
}

template <int C>
__device__ __forceinline__ void h2_stage_across_chunks(__half2 (&h)[C][4], int hc) {
#pragma unroll
  for (int c = 0; c < C; ++c)
    if (!(c & hc))
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __half2 a = h[c][i], b = h[c + hc][i];
        h[c][i] = __hadd2(a, b);
        h[c + hc][i] = __hsub2(a, b);
      }
}

// Stages for index bits [BEGIN, END) on packed half2 values (BEGIN >= 1).
template <int C, int BEGIN, int END>
__device__ __forceinline__ void fwht_h2_bits(__half2 (&h)[C][4], int lane) {
#pragma unroll
  for (int b = BEGIN; b < END; ++b) {
    if (b < 3)
      h2_stage_in_vector<C>(h, 1 << (b - 1));
    else if (b < 8)
      h2_stage_across_lanes<C>(h, lane, 1 << (b - 3));
    else
      h2_stage_across_chunks<C>(h, 1 << (b - 8));
  }
}

// Stages for index bits [BEGIN, END) on fp32 values (no rounding).
template <int C, int BEGIN, int END>
__device__ __forceinline__ void fwht_f32_bits(float (&v)[C][8], int lane) {
#pragma unroll
  for (int b = BEGIN; b < END; ++b) {
    if (b < 3)
      stage_in_vector<C>(v, 1 << b);
    else if (b < 8)
      stage_across_lanes<C>(v, lane, 1 << (b - 3));
    else
      stage_across_chunks<C>(v, 1 << (b - 8));
  }
}

template <int C>
__device__ __forceinline__ float amax_h2(const __half2 (&h)[C][4]) {
  __half2 m = __float2half2_rn(0.f);
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) m = __hmax2(m, __habs2(h[c][i]));
  return fmaxf(__low2float(m), __high2float(m));
}

template <int C>
__device__ __forceinline__ void unpack_half2(const __half2 (&h)[4], float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// clamp(rint(v / sdiv), -7, 7) with the IEEE quotient, bit for bit, but
// without a division per element.  rs = fl(1 / sdiv); t = fl(v * rs) then
// differs from the exact quotient Q by at most |Q| (2^-23 + 2^-48), and the
// correctly rounded quotient fl(Q) by at most 1.8e-7 |Q| <= 1.5e-6 for
// |Q| <= 8.  rint only changes at half-integers, so whenever t is farther
// than 4e-6 from one, rint(t) == rint(fl(Q)); the rare values that close to a
// tie (and NaN) take the IEEE division.  For |Q| > 8 both results clamp to
// +-7 (t >= 8 implies fl(Q) > 7.5).
__device__ __forceinline__ int quant_code(float v, float sdiv, float rs) {
  const float t = __fmul_rn(v, rs);
  const float frac = __fsub_rn(t, floorf(t));  // exact for |t| < 2^23
  const int q = fabsf(__fsub_rn(frac, 0.5f)) > 4e-6f ? __float2int_rn(t)
                                                      : __float2int_rn(__fdiv_rn(v, sdiv));
  return max(-7, min(7, q));
}

__device__ __forceinline__ float warp_max(float m) {
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

// Output formats of the activation codes.
enum CodesMode : int {
  kCodesInt8 = 0,    // one code per byte, natural element order
  kCodesPacked = 1,  // the reference's int32 words: 8 nibbles, element j at bits 4j
  kCodesGemm = 2,    // one code per byte, each group of 8 stored as elements 0,2,4,6,1,3,5,7
                     // (the K order the GEMM's nibble expansion produces)
};

// Eight codes (elements elem .. elem+7) in the chosen format.
template <int MODE>
__device__ __forceinline__ void store_codes8(void* out, long long elem, const float (&v)[8],
                                             float sdiv, float rs) {
  if constexpr (MODE != kCodesPacked) {
    // Fast path, the same decision as quant_code: r = fl(t + 1.5 * 2^23) is
    // 1.5 * 2^23 + rint(t) exactly (|t| < 2^22; the offset is even, so the
    // sum's round-half-even is rint's), e = t - rint(t) is exact, and
    // |e| < 0.5 - 4e-6 is quant_code's "farther than 4e-6 from a tie".  The
    // low byte of r's bit pattern is then rint(t) as a two's-complement
    // int8.  No clamp: |v| <= amax and sdiv >= fl(amax / 7) keep
    // |t| <= 7 (1 + 2^-22) < 7.5.  A group with a value near a tie (or NaN)
    // takes the exact path below.
    constexpr float kRound = 12582912.0f;
    uint32_t b[8];
    bool fast = true;
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const float2 t = __fmul2_rn(make_float2(v[j], v[j + 1]), make_float2(rs, rs));
      const float2 r = __fadd2_rn(t, make_float2(kRound, kRound));
      const float2 d = __fadd2_rn(r, make_float2(-kRound, -kRound));  // rint(t), exact
      const float2 e = __ffma2_rn(d, make_float2(-1.f, -1.f), t);     // t - rint(t), exact
      fast &= fabsf(e.x) < 0.499996f;
      fast &= fabsf(e.y) < 0.499996f;
      b[j] = __float_as_uint(r.x);
      b[j + 1] = __float_as_uint(r.y);
    }
    if (fast) {
      // bytes of the first word: elements 0,2,4,6 (GEMM order) or 0-3
      constexpr int a0 = 0, a1 = MODE == kCodesGemm ? 2 : 1, a2 = MODE == kCodesGemm ? 4 : 2,
                    a3 = MODE == kCodesGemm ? 6 : 3;
      constexpr int c0 = MODE == kCodesGemm ? 1 : 4, c1 = MODE == kCodesGemm ? 3 : 5,
                    c2 = MODE == kCodesGemm ? 5 : 6, c3 = 7;
      const uint32_t w0 = __byte_perm(__byte_perm(b[a0], b[a1], 0x0040),
                                      __byte_perm(b[a2], b[a3], 0x0040), 0x5410);
      const uint32_t w1 = __byte_perm(__byte_perm(b[c0], b[c1], 0x0040),
                                      __byte_perm(b[c2], b[c3], 0x0040), 0x5410);
      *reinterpret_cast<uint2*>(reinterpret_cast<int8_t*>(out) + elem) = make_uint2(w0, w1);
      return;
    }
  }
  int q[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) q[j] = quant_code(v[j], sdiv, rs);
  if constexpr (MODE == kCodesPacked) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) w |= (static_cast<uint32_t>(q[j]) & 0xFu) << (4 * j);
    reinterpret_cast<uint32_t*>(out)[elem >> 3] = w;
  } else {
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int a = MODE == kCodesGemm ? 2 * j : j;
      const int b = MODE == kCodesGemm ? 2 * j + 1 : j + 4;
      w0 |= (static_cast<uint32_t>(q[a]) & 0xFFu) << (8 * j);
      w1 |= (static_cast<uint32_t>(q[b]) & 0xFFu) << (8 * j);
    }
    *reinterpret_cast<uint2*>(reinterpret_cast<int8_t*>(out) + elem) = make_uint2(w0, w1);
  }
}

// The last index bits of a row, held across NW warps (index bits 9 .. 9 +
// log2(NW) - 1): every thread reads the NW warps' values at its own positions
// and applies those butterfly stages in ascending order, keeping its warp's
// outputs.  Stage bit 9 pairs warps w and w^1, bit 10 pairs w and w^2; the
// lower partner keeps a + b, the upper a - b, each rounded (T = __half2 for
// fp16 staging, float for fp32).
template <int NW, typename T>
__device__ __forceinline__ T cross_warp_stages(const T (&x)[NW], int w);
template <>
__device__ __forceinline__ __half2 cross_warp_stages<2, __half2>(const __half2 (&x)[2], int w) {
  return w ? __hsub2(x[0], x[1]) : __hadd2(x[0], x[1]);
}
template <>
__device__ __forceinline__ __half2 cross_warp_stages<4, __half2>(const __half2 (&x)[4], int w) {
  // after the bit-9 stage: s[0] = x0 + x1, s[1] = x0 - x1, s[2] = x2 + x3,
  // s[3] = x2 - x3; the bit-10 stage pairs s[w & 1] with s[(w & 1) + 2]
  const __half2 a = (w & 1) ? __hsub2(x[0], x[1]) : __hadd2(x[0], x[1]);
  const __half2 b = (w & 1) ? __hsub2(x[2], x[3]) : __hadd2(x[2], x[3]);
  return (w & 2) ? __hsub2(a, b) : __hadd2(a, b);
}
template <>
__device__ __forceinline__ float cross_warp_stages<2, float>(const float (&x)[2], int w) {
  return w ? __fsub_rn(x[0], x[1]) : __fadd_rn(x[0], x[1]);
}
template <>
__device__ __forceinline__ float cross_warp_stages<4, float>(const float (&x)[4], int w) {
  const float a = (w & 1) ? __fsub_rn(x[0], x[1]) : __fadd_rn(x[0], x[1]);
  const float b = (w & 1) ? __fsub_rn(x[2], x[3]) : __fadd_rn(x[2], x[3]);
  return (w & 2) ? __fsub_rn(a, b) : __fadd_rn(a, b);
}

// Shared memory of the row-split K <= 2048 quant: the cross-warp exchange
// and the per-warp amax.
template <int LOGK, bool FP16>
struct RowSplitSmem {
  static constexpr int NW = (1 << LOGK) / 512;
  uint4 xchg[NW][2][32][FP16 ? 1 : 2];
  float warp_amax[NW];
};

// The FWHT + codes of one K = 1024 / 2048 row held by a CTA of K / 16
// threads: thread (warp, lane) holds elements 512 warp + 256 c + 8 lane + j
// (c = 0, 1; j = 0..7) of the row in v, as fp32 copies of fp16 values.
// Index bits 0-2 are in a vector, 3-7 across lanes, bit 8 across the
// thread's two vectors and bits 9 and up across the row's warps, whose
// stages (the last, as in the reference's ascending order) go through one
// shared-memory exchange.  Writes the row's codes and row scale.
template <int LOGK, bool FP16, int MODE>
__device__ __forceinline__ void fwht_quant_row_split(float (&v)[2][8], RowSplitSmem<LOGK, FP16>& sm,
                                                     int warp, int lane, long long row,
                                                     void* __restrict__ codes,
                                                     float* __restrict__ row_scale,
                                                     float inv_sqrt_k) {
  constexpr int K = 1 << LOGK;
  constexpr int NW = K / 512;      // warps per row (2 or 4)
  constexpr int RBITS = LOGK - 8;  // log2(K / 256): stages kept in fp32
  static_assert(RBITS <= 3, "fp32 stages must stay inside a vector");
  fwht_f32_bits<2, 0, RBITS>(v, lane);
  float mx = 0.f;
  if constexpr (FP16) {
    __half2 h[2][4];
    pack_half2<2>(v, h);
    fwht_h2_bits<2, RBITS, 9>(h, lane);
#pragma unroll
    for (int c = 0; c < 2; ++c) sm.xchg[warp][c][lane][0] = *reinterpret_cast<const uint4*>(h[c]);
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      __half2 all[4][NW];
#pragma unroll
      for (int u = 0; u < NW; ++u) {
        const uint4 q = sm.xchg[u][c][lane][0];
        const __half2* qh = reinterpret_cast<const __half2*>(&q);
#pragma unroll
        for (int i = 0; i < 4; ++i) all[i][u] = qh[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) h[c][i] = cross_warp_stages<NW, __half2>(all[i], warp);
    }
    mx = amax_h2<2>(h);
#pragma unroll
    for (int c = 0; c < 2; ++c) unpack_half2<2>(h[c], v[c]);
  } else {
    fwht_f32_bits<2, RBITS, 9>(v, lane);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      sm.xchg[warp][c][lane][0] = make_uint4(__float_as_uint(v[c][0]), __float_as_uint(v[c][1]),
                                             __float_as_uint(v[c][2]), __float_as_uint(v[c][3]));
      sm.xchg[warp][c][lane][1] = make_uint4(__float_as_uint(v[c][4]), __float_as_uint(v[c][5]),
                                             __float_as_uint(v[c][6]), __float_as_uint(v[c][7]));
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float all[8][NW];
#pragma unroll
      for (int u = 0; u < NW; ++u) {
        const uint4 q0 = sm.xchg[u][c][lane][0], q1 = sm.xchg[u][c][lane][1];
        all[0][u] = __uint_as_float(q0.x); all[1][u] = __uint_as_float(q0.y);
        all[2][u] = __uint_as_float(q0.z); all[3][u] = __uint_as_float(q0.w);
        all[4][u] = __uint_as_float(q1.x); all[5][u] = __uint_as_float(q1.y);
        all[6][u] = __uint_as_float(q1.z); all[7][u] = __uint_as_float(q1.w);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[c][j] = cross_warp_stages<NW, float>(all[j], warp);
        mx = fmaxf(mx, fabsf(v[c][j]));
      }
    }
  }
  mx = warp_max(mx);
  if (lane == 0) sm.warp_amax[warp] = mx;
  __syncthreads();
  mx = sm.warp_amax[0];
#pragma unroll
  for (int u = 1; u < NW; ++u) mx = fmaxf(mx, sm.warp_amax[u]);
  const float sdiv = __fadd_rn(__fdiv_rn(mx, 7.0f), 1e-12f);
  const float rs = __frcp_rn(sdiv);
  if (warp == 0 && lane == 0) row_scale[row] = __fmul_rn(sdiv, inv_sqrt_k);
#pragma unroll
  for (int c = 0; c < 2; ++c)
    store_codes8<MODE>(codes, row * K + 512 * warp + 256 * c + 8 * lane, v[c], sdiv, rs);
}

// K = 1024 / 2048: one CTA of K / 16 threads (2 or 4 warps) per row, so a
// 776-row activation is resident in one wave at ~21 warps per SM with short
// per-thread dependency chains (layout: fwht_quant_row_split).
template <int LOGK, bool FP16, int MODE>
__global__ void __launch_bounds__((1 << LOGK) / 16) quant_rot_warp_kernel(
    const __half* __restrict__ x, long long ldx, long long m, void* __restrict__ codes,
    float* __restrict__ row_scale, float inv_sqrt_k) {
  __shared__ RowSplitSmem<LOGK, FP16> sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait();  // x is the previous kernel's output
  if (row >= m) return;
  float v[2][8];
  const __half* xr = x + row * ldx + 512 * warp + 8 * lane;
#pragma unroll
  for (int c = 0; c < 2; ++c) load8_half_as_float(xr + 256 * c, v[c]);
  fwht_quant_row_split<LOGK, FP16, MODE>(v, sm, warp, lane, row, codes, row_scale, inv_sqrt_k);
}

// K = 16384: one 256-thread CTA per row.  Phase 1: warp w transforms its
// 2048-element slice (index bits 0-10) in registers.  Phase 2: after a
// shared-memory transpose, thread (c, l) = (warp, lane) holds the 8 slices'
// values at offsets 256c + 8l + j and finishes bits 11-13 in registers.
// GEGLU: the row is gelu_tanh(x) * up (x = the gate), formed as it is
// loaded (geglu8) and, when h_out is not null, also written there.
// SEGMENTED: the row is stored as segments of `seg` elements (a multiple of
// 8), segment s of row r at x + s * seg_stride + r * ldx.
template <bool FP16, int MODE, bool GEGLU = false, bool SEGMENTED = false>
__global__ void __launch_bounds__(kQuantThreads) quant_rot_16k_kernel(
    const __half* __restrict__ x, long long ldx, long long m, void* __restrict__ codes,
    float* __restrict__ row_scale, float inv_sqrt_k, const __half* __restrict__ up = nullptr,
    long long ldu = 0, __half* __restrict__ h_out = nullptr, long long ldh = 0, int seg = 0,
    long long seg_stride = 0) {
  constexpr int K = 16384;
  constexpr int RBITS = 6;  // log2(16384 / 256)
  extern __shared__ __align__(16) unsigned char quant_smem[];
  __shared__ float warp_amax[kQuantThreads / 32];

  const long long row = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait();  // x is the previous kernel's output
  if (row >= m) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float v[8][8];
  {
    const __half* xr = x + row * ldx + 2048 * warp + 8 * lane;
    if constexpr (GEGLU) {
      const __half* ur = up + row * ldu + 2048 * warp + 8 * lane;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 h8 = geglu8(ld_nc_v4(xr + 256 * c), ld_nc_v4(ur + 256 * c));
        if (h_out) *reinterpret_cast<uint4*>(h_out + row * ldh + 2048 * warp + 8 * lane + 256 * c) = h8;
        half8_to_float(h8, v[c]);
      }
    } else if constexpr (SEGMENTED) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int e = 2048 * warp + 256 * c + 8 * lane;
        const int sgi = e / seg;
        load8_half_as_float(x + sgi * seg_stride + row * ldx + (e - sgi * seg), v[c]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) load8_half_as_float(xr + 256 * c, v[c]);
    }
    fwht_f32_bits<8, 0, RBITS>(v, lane);
    if constexpr (FP16) {
      __half2 h[8][4];
      pack_half2<8>(v, h);
      fwht_h2_bits<8, RBITS, 11>(h, lane);
      __half* buf = reinterpret_cast<__half*>(quant_smem);
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(buf + 2048 * warp + 256 * c + 8 * lane) =
            *reinterpret_cast<const uint4*>(h[c]);
    } else {
      fwht_f32_bits<8, RBITS, 11>(v, lane);
      float* buf = reinterpret_cast<float*>(quant_smem);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float* dst = buf + 2048 * warp + 256 * c + 8 * lane;
        *reinterpret_cast<float4*>(dst) = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(v[c][4], v[c][5], v[c][6], v[c][7]);
      }
    }
  }
  __syncthreads();
  // Phase 2: slot w holds element 2048w + 256*warp + 8*lane + j.
  float mx;
  if constexpr (FP16) {
    const __half* buf = reinterpret_cast<const __half*>(quant_smem);
    __half2 h[8][4];
#pragma unroll
    for (int w = 0; w < 8; ++w)
      *reinterpret_cast<uint4*>(h[w]) =
          *reinterpret_cast<const uint4*>(buf + 2048 * w + 256 * warp + 8 * lane);
#pragma unroll
    for (int b = 11; b < 14; ++b) h2_stage_across_chunks<8>(h, 1 << (b - 11));
    mx = amax_h2<8>(h);
#pragma unroll
    for (int w = 0; w < 8; ++w) unpack_half2<8>(h[w], v[w]);
  } else {
    const float* buf = reinterpret_cast<const float*>(quant_smem);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float* src = buf + 2048 * w + 256 * warp + 8 * lane;
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      v[w][0] = a.x; v[w][1] = a.y; v[w][2] = a.z; v[w][3] = a.w;
      v[w][4] = b.x; v[w][5] = b.y; v[w][6] = b.z; v[w][7] = b.w;
    }
#pragma unroll
    for (int b = 11; b < 14; ++b) stage_across_chunks<8>(v, 1 << (b - 11));
    mx = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w)
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[w][j]));
  }
  mx = warp_max(mx);
  if (lane == 0) warp_amax[warp] = mx;
  __syncthreads();
  mx = warp_amax[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, warp_amax[w]);
  const float sdiv = __fadd_rn(__fdiv_rn(mx, 7.0f), 1e-12f);
  const float rs = __frcp_rn(sdiv);
  if (threadIdx.x == 0) row_scale[row] = __fmul_rn(sdiv, inv_sqrt_k);
#pragma unroll
  for (int w = 0; w < 8; ++w)
    store_codes8<MODE>(codes, row * K + 2048 * w + 256 * warp + 8 * lane, v[w], sdiv, rs);
}

// ---- K = 16384, fp16 staging: every butterfly stage in registers.
// A row is 2048 16-byte vectors (8 fp16 elements, index bits 0-2 inside a
// vector); each of the 256 threads working on a row holds 8 of them.  Between
// phases the vectors move through a shared-memory buffer so that the next
// three index bits become the thread's vector index c:
//   A: vec = 8u + c                      -> element bits 3-5 across c (fp32, with 0-2)
//   B: vec = (u>>3)<<6 | c<<3 | (u&7)    -> bits 6-8
//   C: vec = (u>>6)<<9 | c<<6 | (u&63)   -> bits 9-11
//   D: vec = (c&3)<<9 | (c>>2)<<8 | u    -> bits 12-13 (c bits 0-1)
// Phase A reads the row from the TMA buffer (line u = vec 8u .. 8u + 7);
// every later phase reads and writes the transposed buffer in place.  Each
// thread writes back the vectors it read, so one barrier per transpose
// suffices.  Slot swizzle vec ^ ((vec >> 3) & 7): in every phase the 8 lanes
// of a quarter-warp hit 8 distinct 16-byte bank groups.
__device__ __forceinline__ int q16k_slot(int vec) { return vec ^ ((vec >> 3) & 7); }

// Shared memory of the K = 16384 fp16-staging kernel: one 32 KB row buffer
// (TMA destination, then the transposes' workspace), 1024-byte aligned for
// the 128-byte swizzle.
constexpr int kQ16RowBytes = 16384 * 2;
constexpr int kQ16Smem = kQ16RowBytes + 1024;
constexpr int kQ16CtasPerSm = 3;

// One row through phases A-D, the amax and the codes, by the 256 threads
// u = 0..255 of a row group.  base: the group's 1024-byte aligned buffer
// (the row's 128-byte lines, line u's 16-byte chunk c at chunk c ^ (u & 7)).
// load(c) gives the fp16 vector c of line u (phase A's input); sync() is the
// group's barrier; buffer_free() runs once every thread of the group has
// read the buffer for the last time (phase D's loads).
template <int MODE, class Load, class Sync, class Free>
__device__ __forceinline__ void q16k_row(unsigned char* base, int u, long long row, void* __restrict__ codes,
                                         float* __restrict__ row_scale, float inv_sqrt_k, float* warp_amax,
                                         Load load, Sync sync, Free buffer_free) {
  constexpr int K = 16384;
  const int warp = u >> 5, lane = u & 31;
  uint4* buf = reinterpret_cast<uint4*>(base);
  __half2 h[8][4];
  {
    // phase A: index bits 0-5 in fp32
    float v[8][8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 raw = load(c);
      const __half2* hp = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(hp[i]);
        v[c][2 * i] = f.x;
        v[c][2 * i + 1] = f.y;
      }
    }
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) stage_in_vector<8>(v, 1 << bb);
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) stage_across_chunks<8>(v, 1 << bb);
    pack_half2<8>(v, h);
  }
  sync();  // every thread has read its line before the buffer is rewritten
#pragma unroll
  for (int c = 0; c < 8; ++c) buf[q16k_slot(8 * u + c)] = *reinterpret_cast<const uint4*>(h[c]);
  sync();
  // phase B: bits 6-8
  {
    const int bq = ((u >> 3) << 6) | (u & 7);
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(h[c]) = buf[q16k_slot(bq | (c << 3))];
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) h2_stage_across_chunks<8>(h, 1 << bb);
#pragma unroll
    for (int c = 0; c < 8; ++c) buf[q16k_slot(bq | (c << 3))] = *reinterpret_cast<const uint4*>(h[c]);
  }
  sync();
  // phase C: bits 9-11
  {
    const int bq = ((u >> 6) << 9) | (u & 63);
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(h[c]) = buf[q16k_slot(bq | (c << 6))];
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) h2_stage_across_chunks<8>(h, 1 << bb);
#pragma unroll
    for (int c = 0; c < 8; ++c) buf[q16k_slot(bq | (c << 6))] = *reinterpret_cast<const uint4*>(h[c]);
  }
  sync();
  // phase D: bits 12-13
  const auto vec_d = [&](int c) { return ((c & 3) << 9) | ((c >> 2) << 8) | u; };
#pragma unroll
  for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(h[c]) = buf[q16k_slot(vec_d(c))];
  h2_stage_across_chunks<8>(h, 1);
  h2_stage_across_chunks<8>(h, 2);
  float mx = amax_h2<8>(h);
  mx = warp_max(mx);
  if (lane == 0) warp_amax[warp] = mx;
  sync();
  buffer_free();
  mx = warp_amax[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) mx = fmaxf(mx, warp_amax[w]);
  const float sdiv = __fadd_rn(__fdiv_rn(mx, 7.0f), 1e-12f);
  const float rs = __frcp_rn(sdiv);
  if (u == 0) row_scale[row] = __fmul_rn(sdiv, inv_sqrt_k);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float v[8];
    unpack_half2<8>(h[c], v);
    store_codes8<MODE>(codes, row * K + 8 * vec_d(c), v, sdiv, rs);
  }
}

// One CTA per row (the block scheduler hands rows to SMs as CTAs finish,
// which balanced the 776-row prefix better than persistent CTAs with a
// prefetched second row: 17.1 vs 18.6 us).  One thread loads the row with
// TMA (a 3-D map {64, 256, M} of 128-byte lines, 128-byte swizzle).  The
// swizzle puts 16-byte chunk c of line u at chunk c ^ (u & 7): thread u
// reads its line (elements 64u .. 64u + 63) without bank conflicts.
// SEGMENTED: xmap is 4-D {64, lines per segment, M, segments} (a row stored
// as several segments, each a [M, seg] matrix: the layout an all-to-all of
// column shards delivers), read with one box per row; same smem layout.
// GEGLU: xmap is the gate and umap the up projection (same shape), loaded
// into two row buffers; the row quantised is gelu_tanh(gate) * up, formed in
// a pass over each thread's line before phase A (geglu8, written back into
// the gate row and, when h_out is not null, to h_out), so the row body keeps
// the plain quant's registers and three CTAs fit per SM.  A table of the
// GELU's 65,536 fp16 results in shared memory instead of tanhf was measured
// slower (one persistent CTA of two rows per SM: 32.4 us at M = 776): the
// kernel is bound by the latency of its row pipeline, not by the GELU's
// arithmetic.
constexpr int kQ16SmemGeglu = 2 * kQ16RowBytes + 1024;

template <int MODE, bool SEGMENTED = false, bool GEGLU = false>
__global__ void __launch_bounds__(kQuantThreads, kQ16CtasPerSm) quant_rot_16k_fp16_kernel(
    const __grid_constant__ CUtensorMap xmap, long long m, void* __restrict__ codes,
    float* __restrict__ row_scale, float inv_sqrt_k, unsigned long long limit_ns,
    const __grid_constant__ CUtensorMap umap, __half* __restrict__ h_out, long long ldh) {
  extern __shared__ unsigned char quant_smem[];
  __shared__ float warp_amax[kQuantThreads / 32];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(quant_smem) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t bar_a = smem_addr(&bar);
  const int u = threadIdx.x;
  const long long row = blockIdx.x;
  if (u == 0) {
    mbar_init(bar_a, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // x is the previous kernel's output
  if (row >= m) return;
  if (u == 0) {
    mbar_arrive_expect_tx(bar_a, GEGLU ? 2 * kQ16RowBytes : kQ16RowBytes);
    if constexpr (SEGMENTED)
      tma_load_4d(smem_addr(base), &xmap, 0, 0, static_cast<int>(row), 0, bar_a);
    else
      tma_load_3d(smem_addr(base), &xmap, 0, 0, static_cast<int>(row), bar_a);
    if constexpr (GEGLU) tma_load_3d(smem_addr(base + kQ16RowBytes), &umap, 0, 0, static_cast<int>(row), bar_a);
  }
  mbar_wait_bounded(bar_a, 0, &abort_flag, &g_w4a4_device_error, kErrWaitTma, limit_ns);
  __syncthreads();  // a timed-out wait sets abort_flag first: every thread leaves together
  if (abort_flag) return;
  uint4* buf = reinterpret_cast<uint4*>(base);
  if constexpr (GEGLU) {
    // h = gelu(gate) * up over this thread's line, in place in the gate row
    // (no other thread reads the line before phase A's barrier)
#pragma unroll 2
    for (int c = 0; c < 8; ++c) {
      const int slot = 8 * u + (c ^ (u & 7));
      const uint4 r = geglu8(buf[slot], buf[2048 + slot]);
      buf[slot] = r;
      if (h_out) *reinterpret_cast<uint4*>(h_out + row * ldh + 64 * u + 8 * c) = r;
    }
  }
  q16k_row<MODE>(
      base, u, row, codes, row_scale, inv_sqrt_k, warp_amax,
      [&](int c) { return buf[8 * u + (c ^ (u & 7))]; }, [] { __syncthreads(); }, [] {});
}

// Any K (multiple of 64) without rotation: one warp per row, two passes
// (amax, then codes).  Replaces quant_rows (int4_gemm.cu:451-477).
template <int MODE>
__global__ void __launch_bounds__(kQuantThreads) quant_rows_kernel(
    const __half* __restrict__ x, long long ldx, long long m, int k, void* __restrict__ codes,
    float* __restrict__ row_scale) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (kQuantThreads / 32) + (threadIdx.x >> 5);
  pdl_launch_dependents();
  pdl_wait();  // x is the previous kernel's output
  if (row >= m) return;
  const __half* xr = x + row * ldx;
  float mx = 0.f;
  for (int e = 8 * lane; e < k; e += 256) {
    float v[8];
    load8_half_as_float(xr + e, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(v[j]));
  }
  mx = warp_max(mx);
  const float sdiv = __fadd_rn(__fdiv_rn(mx, 7.0f), 1e-12f);
  const float rs = __frcp_rn(sdiv);
  if (lane == 0) row_scale[row] = sdiv;
  for (int e = 8 * lane; e < k; e += 256) {
    float v[8];
    load8_half_as_float(xr + e, v);
    store_codes8<MODE>(codes, row * k + e, v, sdiv, rs);
  }
}

}  // namespace w4a4

// Load-time weight pack on the GPU: Linear.weight [N, K] -> the reference's
// packed INT4 weight, bit for bit (pi05_fast/w4a4/pack.py:85-101, the
// preshuffle :45-68): per row, in fp32, the unnormalised Walsh-Hadamard
// transform in ascending stride order (K in {1024, 2048, 16384}, or when
// asked), times fl(1/sqrt K); amax clamped to 1e-12; scale = amax / 7 (IEEE
// division); codes = clamp(rint(w / scale), -7, 7) (IEEE quotient,
// round-half-even: quant_code); 8 nibbles per int32 word, then the scale's
// bits.  Not on the inference path: one CTA per row, the row in shared
// memory, one barrier per butterfly stage.
#pragma once

#include "quant.cuh"

namespace w4a4 {

constexpr int kPackThreads = 256;
constexpr int kPackMaxK = 16384;

enum PackDtype : int { kPackF32 = 0, kPackF16 = 1, kPackBF16 = 2 };

__device__ __forceinline__ float pack_load(const void* w, int dtype, long long i) {
  if (dtype == kPackF16) return __half2float(static_cast<const __half*>(w)[i]);
  if (dtype == kPackBF16) {
    const uint32_t b = static_cast<uint32_t>(static_cast<const uint16_t*>(w)[i]) << 16;
    return __uint_as_float(b);
  }
  return static_cast<const float*>(w)[i];
}

// layout 0: row-major rows of out_row_words words (K/8 payload words, the
// scale word, zero padding); layout 1: fragment-major (payload [K/16][N][2
// words], then the N scales, then zeros up to N * (K/8 + 9) words).
__global__ void __launch_bounds__(kPackThreads) pack_weight_kernel(const void* __restrict__ w, int dtype,
                                                                    long long ldw, int n, int k, int rotate,
                                                                    float inv_sqrt_k, int layout,
                                                                    int32_t* __restrict__ out,
                                                                    int out_row_words) {
  extern __shared__ float pack_row[];
  __shared__ float red[kPackThreads / 32];
  const int r = blockIdx.x, t = threadIdx.x;
  if (r >= n) return;
  for (int i = t; i < k; i += kPackThreads) pack_row[i] = pack_load(w, dtype, static_cast<long long>(r) * ldw + i);
  __syncthreads();
  if (rotate) {
    for (int h = 1; h < k; h <<= 1) {
      for (int bfly = t; bfly < k / 2; bfly += kPackThreads) {
        const int i = (bfly / h) * 2 * h + (bfly % h);
        const float a = pack_row[i], c = pack_row[i + h];
        pack_row[i] = __fadd_rn(a, c);
        pack_row[i + h] = __fsub_rn(a, c);
      }
      __syncthreads();
    }
  }
  float m = 0.f;
  for (int i = t; i < k; i += kPackThreads) {
    float v = pack_row[i];
    if (rotate) {
      v = __fmul_rn(v, inv_sqrt_k);
      pack_row[i] = v;
    }
    m = fmaxf(m, fabsf(v));
  }
  m = warp_max(m);
  if ((t & 31) == 0) red[t >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int i = 1; i < kPackThreads / 32; ++i) m = fmaxf(m, red[i]);
  m = fmaxf(m, 1e-12f);
  const float scale = __fdiv_rn(m, 7.0f);
  const float rs = __frcp_rn(scale);
  const int words = k / 8;
  for (int p = t; p < words; p += kPackThreads) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      word |= (static_cast<uint32_t>(quant_code(pack_row[8 * p + j], scale, rs)) & 0xFu) << (4 * j);
    const long long at = layout == 0 ? static_cast<long long>(r) * out_row_words + p
                                     : static_cast<long long>(p >> 1) * 2 * n + 2 * r + (p & 1);
    out[at] = static_cast<int32_t>(word);
  }
  if (layout == 0) {
    for (int p = words + t; p < out_row_words; p += kPackThreads)
      out[static_cast<long long>(r) * out_row_words + p] = p == words ? __float_as_int(scale) : 0;
  } else {
    if (t == 0) out[static_cast<long long>(n) * words + r] = __float_as_int(scale);
    if (r == 0) {
      const long long tail0 = static_cast<long long>(n) * words + n;
      const long long total = static_cast<long long>(n) * out_row_words;
      for (long long i = tail0 + t; i < total; i += kPackThreads) out[i] = 0;
    }
  }
}

}  // namespace w4a4

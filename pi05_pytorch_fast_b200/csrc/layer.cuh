// Kernels of the Gemma-2B prefix-LM layer around the W4A4 GEMMs: the glue
// the reference runs as PyTorch ops between its pi05_w4a4 calls
// (pi05_fast/w4a4/apply.py:126-191 over transformers' Gemma layer), fused
// into the activation quant that follows it where there is one.
//
//  * rmsnorm_quant_kernel: residual add (hidden = residual + delta, one fp16
//    rounding, as `residual + hidden_states`), Gemma RMSNorm
//    (fp32: x * rsqrt(mean(x^2) + eps) * (1 + w), rounded to fp16), then the
//    K = 2048 Hadamard + INT4 quant of the normalised row (the q/k/v and
//    gate/up inputs) -- one launch instead of a norm, an add and a quant.
//    The same kernel without the quant is the final norm.
//  * rope_kernel: rotary position embedding of q and k exactly as
//    transformers' apply_rotary_pos_emb rounds it in fp16:
//    out = fl16(fl16(x * cos) + fl16(rotate_half(x) * sin)).
#pragma once

#include "quant.cuh"

namespace w4a4 {

constexpr int kNormK = 2048;  // Gemma-2B hidden size
constexpr int kNormThreads = kNormK / 16;

// One row of K = 2048 per CTA of 128 threads, thread (warp, lane) holding
// elements 512 warp + 256 c + 8 lane + j (the layout fwht_quant_row_split
// expects).  x_out may alias x (each element is read, then written, by the
// same thread).  The mean of squares is a sum in this kernel's own order
// (per thread, then lanes, then warps) times 1/2048; the result can differ
// from PyTorch's reduction in the last bit of the fp32 mean, hence by one
// fp16 ulp of the normalised value, rarely.
template <bool DELTA, bool QUANT, bool FP16, int MODE>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_quant_kernel(
    const __half* x, long long ldx, const __half* __restrict__ delta, long long ldd,
    const float* __restrict__ gain, float eps, __half* x_out, long long ldo,
    __half* __restrict__ h_out, long long ldh, long long m, void* __restrict__ codes,
    float* __restrict__ row_scale, float inv_sqrt_k) {
  __shared__ RowSplitSmem<11, FP16> sm;
  __shared__ float warp_ss[kNormK / 512];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait();  // x and delta are earlier kernels' outputs
  if (row >= m) return;
  const int e0 = 512 * warp + 8 * lane;
  uint4 s[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    s[c] = *reinterpret_cast<const uint4*>(x + row * ldx + e0 + 256 * c);
    if constexpr (DELTA) {
      const uint4 d = ld_nc_v4(delta + row * ldd + e0 + 256 * c);
      __half2* sh = reinterpret_cast<__half2*>(&s[c]);
      const __half2* dh = reinterpret_cast<const __half2*>(&d);
      // fl16(a + b): binary32 carries 24 >= 2 x 11 + 2 bits, so rounding
      // the fp32 sum to fp16 equals the single fp16 rounding of __hadd2
#pragma unroll
      for (int i = 0; i < 4; ++i) sh[i] = __hadd2(sh[i], dh[i]);
    }
    if (x_out) *reinterpret_cast<uint4*>(x_out + row * ldo + e0 + 256 * c) = s[c];
  }
  float v[2][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    half8_to_float(s[c], v[c]);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __fmaf_rn(v[c][j], v[c][j], ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  if (lane == 0) warp_ss[warp] = ss;
  __syncthreads();
  ss = __fadd_rn(__fadd_rn(warp_ss[0], warp_ss[1]), __fadd_rn(warp_ss[2], warp_ss[3]));
  const float rstd = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / kNormK), eps));
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gain + e0 + 256 * c));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gain + e0 + 256 * c + 4));
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    uint4 hv;
    __half* hh = reinterpret_cast<__half*>(&hv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      hh[j] = __float2half_rn(__fmul_rn(__fmul_rn(v[c][j], rstd), g[j]));
      v[c][j] = __half2float(hh[j]);
    }
    if (h_out) *reinterpret_cast<uint4*>(h_out + row * ldh + e0 + 256 * c) = hv;
  }
  if constexpr (QUANT)
    fwht_quant_row_split<11, FP16, MODE>(v, sm, warp, lane, row, codes, row_scale, inv_sqrt_k);
}

// GeGLU alone, h = fl16(fl16(gelu_tanh(gate)) * up) over [m, n] (n a
// multiple of 8): the MLP of a rank that holds a column shard of gate/up,
// whose rows are completed by an exchange before they are quantised.
__global__ void __launch_bounds__(256) geglu_kernel(const __half* __restrict__ gate,
                                                    const __half* __restrict__ up, long long ld,
                                                    __half* __restrict__ h, long long ldh, long long m,
                                                    int n) {
  pdl_launch_dependents();
  pdl_wait();
  const int vpr = n / 8;
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (idx >= m * vpr) return;
  const long long row = idx / vpr;
  const int c = static_cast<int>(idx - row * vpr) * 8;
  *reinterpret_cast<uint4*>(h + row * ldh + c) =
      geglu8(ld_nc_v4(gate + row * ld + c), ld_nc_v4(up + row * ld + c));
}

// The per-forward tables of a batch of prefixes.  CTA (x, b) covers rows
// [16 x, 16 x + 16) of observation b: it counts the real tokens before its
// rows (every CTA reads the mask up to its rows: at most 4 KB), scans its 16
// rows, and writes position ids cumsum(pad) - 1 as the rotary tables cos /
// sin [L, 2 half] in fp16 -- cos(fl32(pos * inv_freq[i])) rounded to fp16,
// duplicated over both halves: transformers' rotary embedding for these
// positions (its product of an fp32 position and an fp32 frequency is one
// rounding, as here; CUDA's cosf / sinf).  It also copies the key mask as
// bytes; CTA 0 of each observation writes the real-key span (last real
// token + 1).
constexpr int kTableThreads = 256;
constexpr int kTableRows = 16;
__global__ void __launch_bounds__(kTableThreads) prefix_tables_kernel(
    const uint8_t* __restrict__ pad, int seq, const float* __restrict__ inv_freq, int half,
    uint8_t* __restrict__ key_valid, int* __restrict__ kv_len, __half* __restrict__ cos_t,
    __half* __restrict__ sin_t) {
  __shared__ int warp_cnt[kTableThreads / 32];
  __shared__ int warp_span[kTableThreads / 32];
  __shared__ int row_pos[kTableRows];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y, r0 = blockIdx.x * kTableRows;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const uint8_t* pr = pad + static_cast<long long>(b) * seq;
  // real tokens before r0 (and, for CTA 0, the last real token of the row)
  const int scan_end = blockIdx.x == 0 ? seq : r0;
  int cnt = 0, last = 0;
  for (int i = t; i < scan_end; i += kTableThreads) {
    const bool v = pr[i] != 0;
    cnt += (v && i < r0) ? 1 : 0;
    if (v) last = max(last, i + 1);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  }
  if (lane == 0) {
    warp_cnt[warp] = cnt;
    warp_span[warp] = last;
  }
  __syncthreads();
  if (t < kTableRows) {
    int base = 0;
#pragma unroll
    for (int w = 0; w < kTableThreads / 32; ++w) base += warp_cnt[w];
    // scan of this CTA's rows (16 lanes of warp 0)
    const int i = r0 + t;
    const int v = (i < seq && pr[i]) ? 1 : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < kTableRows; o <<= 1) {
      const int y = __shfl_up_sync(0x0000ffffu, x, o);
      if (t >= o) x += y;
    }
    row_pos[t] = base + x - 1;
    if (i < seq) key_valid[static_cast<long long>(b) * seq + i] = static_cast<uint8_t>(v);
  }
  if (blockIdx.x == 0 && t == 0) {
    int span = 0;
#pragma unroll
    for (int w = 0; w < kTableThreads / 32; ++w) span = max(span, warp_span[w]);
    kv_len[b] = span;
  }
  __syncthreads();
  // rotary tables: 16 rows x half / 8 vectors of 8 frequencies
  const int nvec = kTableRows * (half / 8);
  for (int idx = t; idx < nvec; idx += kTableThreads) {
    const int j = idx / (half / 8), f = 8 * (idx - j * (half / 8));
    const int i = r0 + j;
    if (i >= seq) continue;
    const long long row = static_cast<long long>(b) * seq + i;
    const float pf = static_cast<float>(row_pos[j]);
    uint4 cv, sv;
    __half* ch = reinterpret_cast<__half*>(&cv);
    __half* sh = reinterpret_cast<__half*>(&sv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = __fmul_rn(pf, __ldg(inv_freq + f + e));
      ch[e] = __float2half_rn(cosf(a));
      sh[e] = __float2half_rn(sinf(a));
    }
    __half* cr = cos_t + row * (2 * half);
    __half* sr = sin_t + row * (2 * half);
    *reinterpret_cast<uint4*>(cr + f) = cv;
    *reinterpret_cast<uint4*>(cr + half + f) = cv;
    *reinterpret_cast<uint4*>(sr + f) = sv;
    *reinterpret_cast<uint4*>(sr + half + f) = sv;
  }
}

// Rotary embedding of 8 pairs (d, d + 128), d = d0 .. d0 + 7, of one head:
// a = x[d0 ..], b = x[d0 + 128 ..], ca / sa = cos / sin at d0, cb / sb at
// d0 + 128.  out_a = fl16(fl16(a cos) + fl16(-b sin)), out_b = fl16(fl16(b
// cos) + fl16(a sin)): transformers' apply_rotary_pos_emb in fp16 (products
// of two fp16 values are exact in fp32, so each rounds once).
__device__ __forceinline__ void rope_pairs8(uint4& a, uint4& b, const uint4 ca, const uint4 cb, const uint4 sa,
                                            const uint4 sb) {
  const __half* ah = reinterpret_cast<const __half*>(&a);
  const __half* bh = reinterpret_cast<const __half*>(&b);
  const __half* cah = reinterpret_cast<const __half*>(&ca);
  const __half* cbh = reinterpret_cast<const __half*>(&cb);
  const __half* sah = reinterpret_cast<const __half*>(&sa);
  const __half* sbh = reinterpret_cast<const __half*>(&sb);
  uint4 oa, ob;
  __half* oah = reinterpret_cast<__half*>(&oa);
  __half* obh = reinterpret_cast<__half*>(&ob);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x1 = __half2float(ah[j]), x2 = __half2float(bh[j]);
    const float p1 = __half2float(__float2half_rn(__fmul_rn(x1, __half2float(cah[j]))));
    const float r1 = __half2float(__float2half_rn(__fmul_rn(-x2, __half2float(sah[j]))));
    const float p2 = __half2float(__float2half_rn(__fmul_rn(x2, __half2float(cbh[j]))));
    const float r2 = __half2float(__float2half_rn(__fmul_rn(x1, __half2float(sbh[j]))));
    oah[j] = __float2half_rn(__fadd_rn(p1, r1));
    obh[j] = __float2half_rn(__fadd_rn(p2, r2));
  }
  a = oa;
  b = ob;
}

// Rotary embedding of `heads` heads of width 256 per row: element d < 128
// pairs with d + 128.  cos / sin are fp16 [m, 256] tables (row stride 256),
// the per-position values transformers' rotary embedding produces.  One
// thread per 8 pairs; out may alias x.
constexpr int kRopeHeadDim = 256;
__global__ void __launch_bounds__(256) rope_kernel(const __half* x, long long ldx, __half* out,
                                                   long long ldo, const __half* __restrict__ cos_t,
                                                   const __half* __restrict__ sin_t, long long m,
                                                   int heads) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int kVecPerHead = kRopeHeadDim / 2 / 8;  // 16 vectors of 8 pairs
  const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = m * heads * kVecPerHead;
  if (idx >= total) return;
  const int vec = static_cast<int>(idx % kVecPerHead);
  const long long rh = idx / kVecPerHead;
  const int head = static_cast<int>(rh % heads);
  const long long row = rh / heads;
  const int d = 8 * vec;
  const __half* xr = x + row * ldx + head * kRopeHeadDim;
  uint4 a = *reinterpret_cast<const uint4*>(xr + d);
  uint4 b = *reinterpret_cast<const uint4*>(xr + d + 128);
  const __half* cr = cos_t + row * kRopeHeadDim;
  const __half* sr = sin_t + row * kRopeHeadDim;
  rope_pairs8(a, b, __ldg(reinterpret_cast<const uint4*>(cr + d)), __ldg(reinterpret_cast<const uint4*>(cr + d + 128)),
              __ldg(reinterpret_cast<const uint4*>(sr + d)), __ldg(reinterpret_cast<const uint4*>(sr + d + 128)));
  __half* orow = out + row * ldo + head * kRopeHeadDim;
  *reinterpret_cast<uint4*>(orow + d) = a;
  *reinterpret_cast<uint4*>(orow + d + 128) = b;
}

}  // namespace w4a4

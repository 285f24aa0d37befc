// bf16 kernels of the config-4 neighbours of the W4A4 path: the SnapFlow
// step's SigLIP tower and action expert (pi05_fast/snapflow_pi05.py:127-195,
// lerobot's PI05 policy in PyTorch bf16).  Each replaces a chain of small
// PyTorch launches with one memory-bound pass; all arithmetic is fp32, each
// result rounded once to bf16.
//
//  * ada_rms_norm_bf16_kernel: pi0.5's adaptive RMSNorm,
//    y = x rsqrt(mean(x^2) + eps) (1 + scale) + shift, (1 + scale) and shift
//    given per observation in fp32 (one warp per row);
//  * rope_bf16_kernel: rotary position embedding of q and k in place,
//    x' = x cos + rotate_half(x) sin, one thread per 8 rotation pairs;
//  * layer_norm_bf16_kernel: LayerNorm with bf16 weight and bias (SigLIP),
//    mean and variance in two passes over the row held in registers.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace w4a4 {

constexpr int kNbThreads = 256;  // 8 warps, one row each for the norms

__device__ __forceinline__ void bf16x8_to_float(const uint4 raw, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 float8_to_bf16x8(const float (&v)[8]) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return raw;
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Row r of x [rows, h] (contiguous, h = 256 VPL): observation b = r /
// rows_per_batch; scale1 / shift rows at b * mod_stride (fp32, h each).
template <int VPL>
__global__ void __launch_bounds__(kNbThreads) ada_rms_norm_bf16_kernel(
    const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, long long rows, int rows_per_batch,
    const float* __restrict__ scale1, const float* __restrict__ shift, long long mod_stride, float eps) {
  constexpr int h = 256 * VPL;
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (kNbThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * h);
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    bf16x8_to_float(xr[lane + 32 * j], v[j]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[j][e], v[j][e], ss);
  }
  const float rstd = rsqrtf(warp_sum(ss) / static_cast<float>(h) + eps);
  const long long b = row / rows_per_batch;
  const float4* s1 = reinterpret_cast<const float4*>(scale1 + b * mod_stride);
  const float4* sh = reinterpret_cast<const float4*>(shift + b * mod_stride);
  uint4* yr = reinterpret_cast<uint4*>(y + row * h);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c = 2 * (lane + 32 * j);  // float4 index of element 8 (lane + 32 j)
    const float4 a0 = __ldg(s1 + c), a1 = __ldg(s1 + c + 1), b0 = __ldg(sh + c), b1 = __ldg(sh + c + 1);
    const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = fmaf(v[j][e] * rstd, a[e], bb[e]);
    yr[lane + 32 * j] = float8_to_bf16x8(o);
  }
}

// q [rows, heads_q, hd] and k [rows, heads_k, hd] (row strides ldq / ldk
// elements) rotated in place with cos / sin [rows, hd] (each half the same
// angles): for i < hd / 2, (x_i, x_{i+hd/2}) -> (x_i c_i - x_{i+hd/2} s_i,
// x_{i+hd/2} c_i + x_i s_i).  Thread t of a row takes 8 consecutive i of
// one head.
__global__ void __launch_bounds__(kNbThreads) rope_bf16_kernel(
    __nv_bfloat16* __restrict__ q, long long ldq, int heads_q, __nv_bfloat16* __restrict__ k, long long ldk,
    int heads_k, const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
    long long rows, int hd) {
  pdl_launch_dependents();
  pdl_wait();
  const int groups = hd / 16;  // 8-wide groups in a half
  const long long per_row = static_cast<long long>(heads_q + heads_k) * groups;
  const long long t = static_cast<long long>(blockIdx.x) * kNbThreads + threadIdx.x;
  if (t >= rows * per_row) return;
  const long long row = t / per_row;
  const int rem = static_cast<int>(t - row * per_row);
  const int head = rem / groups, g = rem - head * groups;
  __nv_bfloat16* xh = head < heads_q ? q + row * ldq + static_cast<long long>(head) * hd
                                     : k + row * ldk + static_cast<long long>(head - heads_q) * hd;
  const int i0 = 8 * g, half = hd / 2;
  float x1[8], x2[8], c[8], s[8];
  bf16x8_to_float(*reinterpret_cast<const uint4*>(xh + i0), x1);
  bf16x8_to_float(*reinterpret_cast<const uint4*>(xh + i0 + half), x2);
  bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(cos_t + row * hd + i0)), c);
  bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(sin_t + row * hd + i0)), s);
  float o1[8], o2[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    o1[e] = fmaf(x1[e], c[e], -x2[e] * s[e]);
    o2[e] = fmaf(x2[e], c[e], x1[e] * s[e]);
  }
  *reinterpret_cast<uint4*>(xh + i0) = float8_to_bf16x8(o1);
  *reinterpret_cast<uint4*>(xh + i0 + half) = float8_to_bf16x8(o2);
}

// LayerNorm of x [rows, h] (contiguous, h a multiple of 8, at most 256 VPL):
// y = (x - mean) rsqrt(var + eps) w + b, var the mean of (x - mean)^2.  One
// warp per row; lane l holds the 8-element vectors l, l + 32, ...
template <int VPL>
__global__ void __launch_bounds__(kNbThreads) layer_norm_bf16_kernel(
    const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, long long rows, int h,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias, float eps) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (kNbThreads / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = h / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * h);
  float v[VPL][8];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      bf16x8_to_float(xr[vi], v[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[j][e];
    }
  }
  const float mean = warp_sum(sum) / static_cast<float>(h);
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j)
    if (lane + 32 * j < nvec)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[j][e] - mean;
        var = fmaf(d, d, var);
      }
  const float rstd = rsqrtf(warp_sum(var) / static_cast<float>(h) + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + row * h);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      float wf[8], bf[8], o[8];
      bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(w) + vi), wf);
      bf16x8_to_float(__ldg(reinterpret_cast<const uint4*>(bias) + vi), bf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf((v[j][e] - mean) * rstd, wf[e], bf[e]);
      yr[vi] = float8_to_bf16x8(o);
    }
  }
}

}  // namespace w4a4

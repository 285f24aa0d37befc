// CPU stand-ins for the GPU built-ins the reference's quant_rot_rb kernel
// uses, so that its source (pi05_fast/w4a4/csrc/int4_gemm.cu:396-449) runs on
// host threads: one std::thread per GPU thread of a block, __shared__ arrays
// as statics of the (template) function (one block runs at a time), and
// __syncthreads as a std::barrier of the block's threads.  TEST
// INFRASTRUCTURE ONLY: the checker for the fp16-staging quant, never shipped.
#pragma once

#include <algorithm>
#include <barrier>
#include <cmath>
#include <cstdint>

struct GpuDim3 {
  int x = 0, y = 0, z = 0;
};
inline thread_local GpuDim3 threadIdx;
inline GpuDim3 blockIdx;
inline std::barrier<>* g_block_barrier = nullptr;

#define __global__
#define __shared__ static
inline void __syncthreads() { g_block_barrier->arrive_and_wait(); }
// the kernel scales with rsqrtf(K); on the host: the IEEE reciprocal of the
// IEEE square root
inline float rsqrtf(float x) { return 1.0f / std::sqrt(x); }
using std::max;
using std::min;

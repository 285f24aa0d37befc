// Packed-INT4 W4A4 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Computes, for each weight matrix W (N x K, 4-bit codes + fp32 row scale)
// sharing one quantised activation (M x K int8 codes + fp32 row scale):
//     acc[m, n] = sum_k qa[m, k] * qw[n, k]                  (exact int32)
//     y[m, n]   = fp16( (fp32(acc) * sa[m]) * sw[n] )         (RN, left to right)
// which is the reference's gemm_iu4 / gemm_iu4_shape contract
// (pi05_fast/w4a4/csrc/int4_gemm.cu:66-204, :207-394; epilogue :199-200).
//
// Tile mapping (weights on the MMA's M side, tokens on its N side):
//  * one CTA owns 128 weight rows (UMMA M = 128) and a tile of `tok_tile`
//    tokens (UMMA N, a multiple of 16 up to 256), so a ragged token count such
//    as 776 splits into near-equal tiles (e.g. 4 x 208) instead of wasting a
//    mostly-empty 128-row tile;
//  * warp 0 is the TMA producer: per 128-wide K step it loads the packed
//    weight tile (128 rows x 64 bytes, either reference layout) into a
//    staging buffer and the int8 token tile into a 128-byte-swizzled buffer;
//  * warps 2-5 unpack the staged nibbles to int8 (sign-extended) straight
//    into the 128-byte-swizzled K-major layout the tensor core reads;
//  * one thread of warp 1 issues 4 x tcgen05.mma (K = 32 each) per step with
//    the int32 accumulator in TMEM (<= 256 columns) and frees the stage with
//    tcgen05.commit;
//  * warps 2-5 then read the accumulator with tcgen05.ld, apply the token and
//    weight scales in fp32 and store fp16.
// Several weight matrices (gate/up, q/k/v) run in ONE launch: their 128-row
// tiles are numbered consecutively across "segments".
#pragma once

#include "common.cuh"

namespace w4a4 {

constexpr int kBlockW = 128;        // weight rows per CTA (UMMA M)
constexpr int kBlockK = 128;        // K elements per stage (one 128-byte swizzle row)
constexpr int kMaxTokTile = 256;    // max tokens per CTA (UMMA N)
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;   // 6 warps
constexpr int kTmemCols = 256;
constexpr int kMaxSegments = 3;

constexpr int kW8Bytes = kBlockW * kBlockK;          // 16 KB unpacked int8 weights
constexpr int kTokBytes = kMaxTokTile * kBlockK;     // 32 KB int8 tokens
constexpr int kWpkBytes = kBlockW * kBlockK / 2;     // 8 KB packed weights
constexpr int kStageBytes = kW8Bytes + kTokBytes + kWpkBytes;
constexpr int kGemmSmemBytes = kGemmStages * kStageBytes + 256 /*barriers*/ + 1024 /*align*/;

enum WeightLayout : int { kRowMajor = 0, kFragmentMajor = 1 };

struct alignas(64) GemmSegment {
  CUtensorMap tmap_w;          // packed payload, see make_weight_map()
  const float* scale;          // weight scales: scale[n * scale_stride]
  long long scale_stride;
  __half* y;                   // output [M, n] row-major
  int n;                       // weight rows of this matrix
  int tile_begin;              // first global weight-tile index of this matrix
};

struct alignas(64) GemmParams {
  CUtensorMap tmap_tok;        // int8 codes [M, K]: box {128, tok_tile}, 128-byte swizzle
  GemmSegment seg[kMaxSegments];
  const float* row_scale;      // [M] token scales
  unsigned long long wait_limit_ns;
  long long m;
  int k;
  int tok_tile;
  int n_seg;
  int k_tiles;
};

__device__ unsigned g_w4a4_device_error;

struct GemmSmem {
  uint8_t* base;
  __device__ uint8_t* w8(int s) const { return base + s * kStageBytes; }
  __device__ uint8_t* tok(int s) const { return base + s * kStageBytes + kW8Bytes; }
  __device__ uint8_t* wpk(int s) const { return base + s * kStageBytes + kW8Bytes + kTokBytes; }
  __device__ uint64_t* bars() const {
    return reinterpret_cast<uint64_t*>(base + kGemmStages * kStageBytes);
  }
  __device__ uint32_t full(int s) const { return smem_addr(bars() + s); }
  __device__ uint32_t unpacked(int s) const { return smem_addr(bars() + kGemmStages + s); }
  __device__ uint32_t empty(int s) const { return smem_addr(bars() + 2 * kGemmStages + s); }
  __device__ uint32_t accum() const { return smem_addr(bars() + 3 * kGemmStages); }
  __device__ uint32_t* tmem_slot() const {
    return reinterpret_cast<uint32_t*>(bars() + 3 * kGemmStages + 1);
  }
  __device__ volatile int* abort_flag() const {
    return reinterpret_cast<volatile int*>(bars() + 3 * kGemmStages + 2);
  }
};

template <int LAYOUT>
__device__ __forceinline__ void unpack_stage(const uint8_t* __restrict__ src,
                                             uint8_t* __restrict__ dst, int ut) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int n, g, src_off;
    if constexpr (LAYOUT == kRowMajor) {
      // staging = [128 rows][16 words]; 8 consecutive threads read one row
      const int u = i * 128 + ut;
      n = u >> 3;
      g = u & 7;
      src_off = n * 64 + g * 8;
    } else {
      // staging = [8 k16-groups][128 rows][2 words]
      n = ut;
      g = i;
      src_off = (g * 128 + n) * 8;
    }
    const uint2 w = *reinterpret_cast<const uint2*>(src + src_off);
    const uint4 o = unpack16_nibbles(w.x, w.y);
    *reinterpret_cast<uint4*>(dst + n * 128 + ((g ^ (n & 7)) << 4)) = o;
  }
}

// ACC_OUT = true writes the raw int32 accumulators (to seg.y reinterpreted
// as int32 [M, n]) instead of the dequantised fp16 values: a test hook that
// proves the integer products bit-exact.
template <int LAYOUT, bool ACC_OUT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a4_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t gemm_smem_raw[];
  GemmSmem sm;
  sm.base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned* err = &g_w4a4_device_error;

  // ---- which tile
  int si = 0;
#pragma unroll
  for (int s = 1; s < kMaxSegments; ++s)
    if (s < p.n_seg && static_cast<int>(blockIdx.y) >= p.seg[s].tile_begin) si = s;
  const GemmSegment& seg = p.seg[si];
  const int n0 = (static_cast<int>(blockIdx.y) - seg.tile_begin) * kBlockW;
  const long long t0 = static_cast<long long>(blockIdx.x) * p.tok_tile;
  const long long t_end = min(p.m, t0 + p.tok_tile);
  const int mma_n = ((static_cast<int>(t_end - t0) + 15) / 16) * 16;
  const uint32_t idesc = idesc_i8(kBlockW, mma_n);
  const uint32_t tx_bytes = kWpkBytes + static_cast<uint32_t>(p.tok_tile) * kBlockK;

  // ---- setup
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(sm.full(s), 1);
      mbar_init(sm.unpacked(s), 128);
      mbar_init(sm.empty(s), 1);
    }
    mbar_init(sm.accum(), 1);
    *sm.abort_flag() = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tmap_tok);
    tma_prefetch_desc(&seg.tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(sm.tmem_slot()), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *sm.tmem_slot();
  volatile int* abort_flag = sm.abort_flag();
  const uint64_t limit = p.wait_limit_ns;

  if (warp == 0) {
    // ---------------- TMA producer (lane 0 issues; the warp stays converged)
    int kt = 0;
    for (; kt < p.k_tiles; ++kt) {
      const int s = kt % kGemmStages;
      bool ok = true;
      if (lane == 0 && kt >= kGemmStages)
        ok = mbar_wait_bounded(sm.empty(s), ((kt / kGemmStages) - 1) & 1, abort_flag, err,
                               kErrWaitEmpty, limit);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(sm.full(s), tx_bytes);
        if constexpr (LAYOUT == kRowMajor)
          tma_load_2d(smem_addr(sm.wpk(s)), &seg.tmap_w, kt * (kBlockK / 8), n0, sm.full(s));
        else
          tma_load_2d(smem_addr(sm.wpk(s)), &seg.tmap_w, n0 * 2, kt * (kBlockK / 16),
                      sm.full(s));
        tma_load_2d(smem_addr(sm.tok(s)), &p.tmap_tok, kt * kBlockK, static_cast<int>(t0),
                    sm.full(s));
      }
      __syncwarp();
    }
    // Drain: no copy issued by this CTA may still be in flight at exit.
    if (lane == 0) {
      const int issued = kt;
      for (int s = 0; s < kGemmStages && s < issued; ++s) {
        const int last = s + ((issued - 1 - s) / kGemmStages) * kGemmStages;  // last kt on s
        volatile int no_abort = 0;
        mbar_wait_bounded(sm.full(s), (last / kGemmStages) & 1, &no_abort, err, kErrWaitDrain,
                          limit);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (lane 0 issues)
    for (int kt = 0; kt < p.k_tiles; ++kt) {
      const int s = kt % kGemmStages;
      const uint32_t parity = (kt / kGemmStages) & 1;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait_bounded(sm.full(s), parity, abort_flag, err, kErrWaitTma, limit) &&
             mbar_wait_bounded(sm.unpacked(s), parity, abort_flag, err, kErrWaitUnpack, limit);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (lane == 0) {
        tc_fence_after();
        const uint64_t adesc = smem_desc_sw128(smem_addr(sm.w8(s)));
        const uint64_t bdesc = smem_desc_sw128(smem_addr(sm.tok(s)));
#pragma unroll
        for (int kk = 0; kk < kBlockK / 32; ++kk)
          umma_i8_ss(tmem_base, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kt | kk) != 0);
        if (kt + kGemmStages < p.k_tiles) umma_commit(sm.empty(s));
      }
      __syncwarp();
    }
    if (lane == 0) {
      // Always commit, so the epilogue and the teardown can wait for every
      // MMA of this CTA to finish before TMEM is read or freed.
      umma_commit(sm.accum());
      volatile int no_abort = 0;
      mbar_wait_bounded(sm.accum(), 0, &no_abort, err, kErrWaitDrain, limit);
    }
    __syncwarp();
  } else {
    // ---------------- unpack (warps 2-5), then epilogue
    const int ut = threadIdx.x - 64;
    for (int kt = 0; kt < p.k_tiles; ++kt) {
      const int s = kt % kGemmStages;
      if (!mbar_wait_bounded(sm.full(s), (kt / kGemmStages) & 1, abort_flag, err, kErrWaitTma,
                             limit))
        break;
      unpack_stage<LAYOUT>(sm.wpk(s), sm.w8(s), ut);
      fence_proxy_async_smem();
      mbar_arrive(sm.unpacked(s));
    }
    const bool ok = mbar_wait_bounded(sm.accum(), 0, abort_flag, err, kErrWaitAccum, limit) &&
                    !*abort_flag;
    tc_fence_after();
    const int quarter = warp & 3;
    const int n = n0 + quarter * 32 + lane;
    const bool n_ok = ok && n < seg.n;
    const float sw =
        (n_ok && !ACC_OUT) ? __ldg(seg.scale + static_cast<long long>(n) * seg.scale_stride) : 0.f;
    __half* yc = seg.y + n;
    const long long ldy = seg.n;
    if (ok) {
      for (int c0 = 0; c0 < mma_n; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const long long t = t0 + c0 + i;
          if (n_ok && t < t_end) {
            if constexpr (ACC_OUT) {
              reinterpret_cast<int32_t*>(seg.y)[t * ldy + n] = static_cast<int32_t>(r[i]);
            } else {
              const float sa = __ldg(p.row_scale + t);
              const float v =
                  __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(r[i])), sa), sw);
              yc[t * ldy] = __float2half_rn(v);
            }
          }
        }
      }
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// A wait on a barrier nobody arrives at: exercises the bounded-wait path so
// tests can check that a timed-out kernel reports an error and returns.
__global__ void w4a4_selftest_wait_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    mbar_wait_bounded(smem_addr(&bar), 0, &abort_flag, &g_w4a4_device_error, kErrWaitSelfTest,
                      limit_ns);
  __syncthreads();
}

}  // namespace w4a4

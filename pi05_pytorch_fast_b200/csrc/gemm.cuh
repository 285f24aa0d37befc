// Packed-INT4 W4A4 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Computes, for each weight matrix W (N x K, 4-bit codes + fp32 row scale)
// sharing one quantised activation (M x K int8 codes + fp32 row scale):
//     acc[m, n] = sum_k qa[m, k] * qw[n, k]                  (exact int32)
//     y[m, n]   = fp16( (fp32(acc) * sa[m]) * sw[n] )         (RN, left to right)
// which is the reference's gemm_iu4 / gemm_iu4_shape contract
// (pi05_fast/w4a4/csrc/int4_gemm.cu:66-204, :207-394; epilogue :199-200).
//
// Design (one persistent CTA per SM, 14 warps):
//  * Tiles put weights on the MMA's M side (128 rows = UMMA M) and tokens on
//    its N side (a multiple of 16, <= 208), so a ragged token count such as
//    776 splits into near-equal tiles (4 x 208) instead of a mostly empty
//    128-row tile.  Several weight matrices (gate/up, q/k/v) form one tile
//    space, so each op is one launch.
//  * warp 0 (TMA producer) streams, per 128-wide K step, the packed weight
//    tile (8 KB, either reference layout, straight from the reference's
//    tensors) and the int8 token tile (128-byte swizzle) into a ring whose
//    depth is set by the token-tile size (6..12 stages).
//  * warps 2-9 (unpack, two groups of 4 taking alternate K steps) each own
//    32 weight rows: they read the staged nibbles, expand them to int8 (x16,
//    see expand_nibbles_x16) in registers and write them with tcgen05.st
//    straight into TMEM, where the MMA reads its A operand.  The unpacked
//    weights never touch shared memory, which leaves the shared-memory
//    bandwidth to the TMA writes and the MMA's reads of the token operand.
//  * one thread of warp 1 issues tcgen05.mma (A from TMEM, B = tokens from
//    shared memory) into one of two TMEM accumulators (double buffered, so
//    the epilogue of a tile overlaps the mainloop of the next) and frees each
//    step with ONE tcgen05.commit: the issuing thread has ~400 cycles of MMA
//    time per step to spend, so its loop carries no warp syncs or divisions.
//  * warps 10-13 (epilogue) read the accumulator with tcgen05.ld, divide by
//    16 (exact), apply the token and weight scales in fp32, round to fp16 and
//    transpose 16x32 blocks through shared memory into 16-byte row stores.
// TMEM map (512 columns): accumulators at [0, T) and [T, 2T) for a token tile
// of T columns, then A stages of 32 columns (128 K-bytes per row) up to 512.
#pragma once

#include "common.cuh"

namespace w4a4 {

constexpr int kBlockW = 128;      // weight rows per tile (UMMA M)
constexpr int kBlockK = 128;      // K elements per pipeline step
constexpr int kTokTileMax = 208;  // max tokens per tile (UMMA N)
constexpr int kMaxStages = 12;    // shared-memory ring (tokens + packed weights)
constexpr int kMaxAStages = 8;    // TMEM ring of unpacked weights
constexpr int kTmemCols = 512;
constexpr int kUnpackGroups = 2;
constexpr int kGemmThreads = 32 * (2 + 4 * kUnpackGroups + 4);  // 14 warps
constexpr int kEpiWarp0 = 2 + 4 * kUnpackGroups;
constexpr int kMaxSegments = 3;

constexpr int kWpkBytes = kBlockW * kBlockK / 2;  // 8 KB packed weights per step
constexpr int kEpiBytesPerWarp = 16 * 32 * 2;     // 16 tokens x 32 rows fp16
constexpr int kEpiScaleBytes = kTokTileMax * 4;   // a tile's token scales, per epilogue warp
// mbarrier slots reserved in shared memory; sized for the larger of the two
// layouts (1-CTA: 2 rings + A ring + 5; CTA pair: 3 rings + 5).
constexpr int kNumBars1 = 2 * kMaxStages + kMaxAStages + 4 + 1;
constexpr int kNumBarsPair = 3 * kMaxStages + 4 + 1;
constexpr int kNumBars = kNumBars1 > kNumBarsPair ? kNumBars1 : kNumBarsPair;
constexpr int kFixedSmem =
    4 * kEpiBytesPerWarp + 4 * kEpiScaleBytes + kNumBars * 8 + 16 + 1024 /*alignment slack*/;
constexpr int kSmemLimit = 232448;
static_assert(2 * kTokTileMax + 3 * 32 <= kTmemCols, "TMEM budget");

// Ring depth for a token tile of `tok_tile` rows.
__host__ __device__ constexpr int gemm_stages(int tok_tile) {
  return (kSmemLimit - kFixedSmem) / (tok_tile * kBlockK + kWpkBytes) < kMaxStages
             ? (kSmemLimit - kFixedSmem) / (tok_tile * kBlockK + kWpkBytes)
             : kMaxStages;
}
__host__ __device__ constexpr int gemm_smem_bytes(int tok_tile) {
  return gemm_stages(tok_tile) * (tok_tile * kBlockK + kWpkBytes) + kFixedSmem;
}
__host__ __device__ constexpr int gemm_a_stages(int tok_tile) {
  return (kTmemCols - 2 * tok_tile) / 32 < kMaxAStages ? (kTmemCols - 2 * tok_tile) / 32
                                                       : kMaxAStages;
}

enum WeightLayout : int { kRowMajor = 0, kFragmentMajor = 1 };

struct alignas(64) GemmSegment {
  CUtensorMap tmap_w;       // packed payload, see launch_gemm()
  const float* scale;       // weight scales: scale[n * scale_stride]
  long long scale_stride;
  void* y;                  // output [M, n] row-major (fp16, or int32 accumulators)
  int n;                    // weight rows of this matrix
  int tile_begin;           // first global weight-tile index of this matrix
  int vec_store;            // 1: y is 16-byte aligned and n % 8 == 0
};

struct alignas(64) GemmParams {
  CUtensorMap tmap_tok;     // int8 codes [M, K] in GEMM byte order: box {128, tok_tile}, SW128
  GemmSegment seg[kMaxSegments];
  const float* row_scale;   // [M] token scales
  unsigned long long wait_limit_ns;
  long long m;
  int k;
  int tok_tile;
  int stages;               // shared-memory ring depth (gemm_stages)
  int a_stages;             // TMEM A ring depth (gemm_a_stages)
  int n_tok_tiles;
  int w_tiles;
  int n_seg;
  int k_tiles;
};

__device__ unsigned g_w4a4_device_error;

struct TileCoord {
  int seg;
  int n0;
  long long t0;
  int rows;
};

__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, int tile) {
  const int wt = tile / p.n_tok_tiles;
  const int tt = tile - wt * p.n_tok_tiles;
  TileCoord c;
  c.seg = 0;
#pragma unroll
  for (int s = 1; s < kMaxSegments; ++s)
    if (s < p.n_seg && wt >= p.seg[s].tile_begin) c.seg = s;
  c.n0 = (wt - p.seg[c.seg].tile_begin) * kBlockW;
  c.t0 = static_cast<long long>(tt) * p.tok_tile;
  c.rows = static_cast<int>(min(static_cast<long long>(p.tok_tile), p.m - c.t0));
  return c;
}

__device__ __forceinline__ bool warp_all(bool v) { return __all_sync(0xffffffffu, v); }

// ACC_OUT = true writes the raw int32 accumulators (seg.y as int32 [M, n])
// instead of fp16: a test hook that proves the integer products bit-exact.
template <int LAYOUT, bool ACC_OUT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a4_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.stages, SA = p.a_stages;
  const int tok_bytes = p.tok_tile * kBlockK;
  uint8_t* tok_ring = base;                              // [S][tok_tile * 128], 1 KB aligned
  uint8_t* wpk_ring = base + S * tok_bytes;              // [S][8 KB]
  uint8_t* epi = wpk_ring + S * kWpkBytes;               // 4 warps x 1 KB
  float* tile_scale = reinterpret_cast<float*>(epi + 4 * kEpiBytesPerWarp);  // [4 warps][208]
  uint64_t* bars = reinterpret_cast<uint64_t*>(tile_scale + 4 * kTokTileMax);
  // full[s]: TMA bytes of step i landed.  empty[s]: MMA(i) completed, which
  // also means the unpack of step i finished (the MMA waited for it), so the
  // token buffer, the packed-weight buffer and -- once the A ring has wrapped
  // -- the TMEM A slot of step i are free.  One commit per step.
  const auto bar_full = [&](int s) { return smem_addr(bars + s); };
  const auto bar_empty = [&](int s) { return smem_addr(bars + kMaxStages + s); };
  const auto bar_afull = [&](int a) { return smem_addr(bars + 2 * kMaxStages + a); };
  const auto bar_accfull = [&](int b) { return smem_addr(bars + 2 * kMaxStages + kMaxAStages + b); };
  const auto bar_accempty = [&](int b) {
    return smem_addr(bars + 2 * kMaxStages + kMaxAStages + 2 + b);
  };
  const uint32_t bar_drain = smem_addr(bars + 2 * kMaxStages + kMaxAStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned* err = &g_w4a4_device_error;
  const uint64_t limit = p.wait_limit_ns;
  const int total_tiles = p.n_tok_tiles * p.w_tiles;
  const int acc_cols = p.tok_tile;
  const int a_col0 = 2 * acc_cols;

  // ---- setup
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int a = 0; a < SA; ++a) mbar_init(bar_afull(a), 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accfull(b), 1);
      mbar_init(bar_accempty(b), 4);
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tmap_tok);
    for (int s = 0; s < p.n_seg; ++s) tma_prefetch_desc(&p.seg[s].tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (lane 0)
    if (lane == 0) {
      const uint32_t tx_bytes = kWpkBytes + static_cast<uint32_t>(tok_bytes);
      RingPos st;
      int issued = 0;
      bool alive = true;
      for (int tile = blockIdx.x; alive && tile < total_tiles; tile += gridDim.x) {
        const TileCoord c = decode_tile(p, tile);
        const CUtensorMap* wmap = &p.seg[c.seg].tmap_w;
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (issued >= S &&
              !mbar_wait_bounded(bar_empty(st.idx), st.phase ^ 1u, abort_flag, err, kErrWaitEmpty,
                                 limit)) {
            alive = false;
            break;
          }
          const uint32_t full = bar_full(st.idx);
          mbar_arrive_expect_tx(full, tx_bytes);
          const uint32_t wdst = smem_addr(wpk_ring + st.idx * kWpkBytes);
          if constexpr (LAYOUT == kRowMajor)
            tma_load_2d(wdst, wmap, kt * (kBlockK / 8), c.n0, full);
          else
            tma_load_2d(wdst, wmap, c.n0 * 2, kt * (kBlockK / 16), full);
          tma_load_2d(smem_addr(tok_ring + st.idx * tok_bytes), &p.tmap_tok, kt * kBlockK,
                      static_cast<int>(c.t0), full);
          st.advance(S);
          ++issued;
        }
      }
      // Drain: no copy issued by this CTA may still be in flight at exit.  The
      // last load into ring slot i completed phase ((last use of i) / S) & 1.
      for (int i = 0; i < S && i < issued; ++i) {
        const int last = i + ((issued - 1 - i) / S) * S;
        volatile int no_abort = 0;
        mbar_wait_bounded(bar_full(i), (last / S) & 1, &no_abort, err, kErrWaitDrain, limit);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (lane 0)
    if (lane == 0) {
      RingPos st, at;
      int tcount = 0;
      bool alive = true;
      const uint64_t bdesc0 = smem_desc_sw128(smem_addr(tok_ring));
      const uint32_t a_base = tmem_base + a_col0;
      for (int tile = blockIdx.x; alive && tile < total_tiles; tile += gridDim.x, ++tcount) {
        const TileCoord c = decode_tile(p, tile);
        const uint32_t idesc = idesc_i8(kBlockW, (c.rows + 15) & ~15);
        const int buf = tcount & 1;
        if (tcount >= 2 &&
            !mbar_wait_bounded(bar_accempty(buf), ((tcount >> 1) - 1) & 1, abort_flag, err,
                               kErrWaitAccum, limit))
          break;
        const uint32_t d_tmem = tmem_base + buf * acc_cols;
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (!mbar_wait_bounded(bar_full(st.idx), st.phase, abort_flag, err, kErrWaitTma, limit) ||
              !mbar_wait_bounded(bar_afull(at.idx), at.phase, abort_flag, err, kErrWaitUnpack,
                                 limit)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = bdesc0 + static_cast<uint64_t>((st.idx * tok_bytes) >> 4);
          const uint32_t a_tmem = a_base + at.idx * 32;
#pragma unroll
          for (int kk = 0; kk < kBlockK / 32; ++kk)
            umma_i8_ts(d_tmem, a_tmem + 8 * kk, bdesc + 2 * kk, idesc, (kt | kk) != 0);
          umma_commit(bar_empty(st.idx));
          if (kt == p.k_tiles - 1) umma_commit(bar_accfull(buf));
          st.advance(S);
          at.advance(SA);
        }
      }
      // Every MMA of this CTA has completed once this commit arrives.
      umma_commit(bar_drain);
      volatile int no_abort = 0;
      mbar_wait_bounded(bar_drain, 0, &no_abort, err, kErrWaitDrain, limit);
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------ unpack -> TMEM (A operand)
    const int group = (warp - 2) >> 2;  // takes the K steps with step % 2 == group
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // weight row within the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // st: ring slot of this step; at: A slot; lag: ring slot of step - SA,
    // whose MMA must have completed before A slot `at` is overwritten.
    RingPos st, at, lag;
    int step = 0;
    bool alive = true;
    for (int tile = blockIdx.x; alive && tile < total_tiles; tile += gridDim.x) {
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        if ((step & 1) == group) {
          bool ok = mbar_wait_bounded(bar_full(st.idx), st.phase, abort_flag, err, kErrWaitTma,
                                      limit);
          if (ok && step >= SA)
            ok = mbar_wait_bounded(bar_empty(lag.idx), lag.phase, abort_flag, err,
                                   kErrWaitUnpack, limit);
          if (!warp_all(ok)) {
            alive = false;
            break;
          }
          const uint8_t* src = wpk_ring + st.idx * kWpkBytes;
          uint32_t w[16];
          if constexpr (LAYOUT == kRowMajor) {
            // [128 rows][64 B], 16-byte chunks swizzled by the TMA (64-byte mode)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 v =
                  *reinterpret_cast<const uint4*>(src + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
              w[4 * c] = v.x;
              w[4 * c + 1] = v.y;
              w[4 * c + 2] = v.z;
              w[4 * c + 3] = v.w;
            }
          } else {
            // [8 k16 groups][128 rows][2 words]
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const uint2 v = *reinterpret_cast<const uint2*>(src + (g * 128 + r) * 8);
              w[2 * g] = v.x;
              w[2 * g + 1] = v.y;
            }
          }
          uint32_t o[32];
#pragma unroll
          for (int i = 0; i < 16; ++i) expand_nibbles_x16(w[i], o[2 * i], o[2 * i + 1]);
          tmem_st_32x32b_x32(tmem_base + lane_addr + a_col0 + at.idx * 32, o);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_afull(at.idx));
        }
        ++step;
        st.advance(S);
        at.advance(SA);
        if (step > SA) lag.advance(S);
      }
    }
  } else {
    // ------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int ew = warp - kEpiWarp0;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    __half* stage = reinterpret_cast<__half*>(epi + ew * kEpiBytesPerWarp);
    int tcount = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tcount) {
      const TileCoord c = decode_tile(p, tile);
      const int buf = tcount & 1;
      // This warp's copy of the tile's token scales (warp-private: only the
      // warp's own lanes write and read it).
      float* ts = tile_scale + ew * kTokTileMax;
      __syncwarp();
      if (!ACC_OUT)
        for (int i = lane; i < c.rows; i += 32) ts[i] = __ldg(p.row_scale + c.t0 + i);
      __syncwarp();
      const bool ok = mbar_wait_bounded(bar_accfull(buf), (tcount >> 1) & 1, abort_flag, err,
                                        kErrWaitAccum, limit);
      if (!warp_all(ok)) break;
      tc_fence_after();
      const GemmSegment& seg = p.seg[c.seg];
      const int n = c.n0 + quarter * 32 + lane;
      const bool n_ok = n < seg.n;
      const float sw =
          (n_ok && !ACC_OUT) ? __ldg(seg.scale + static_cast<long long>(n) * seg.scale_stride) : 0.f;
      const int mma_n = (c.rows + 15) & ~15;
      const long long ldy = seg.n;
      for (int c0 = 0; c0 < mma_n; c0 += 16) {
        uint32_t acc[16];
        tmem_ld_32x32b_x16(tmem_base + lane_addr + buf * acc_cols + c0, acc);
        tmem_ld_wait();
        if (c0 + 16 >= mma_n) {
          // whole accumulator read: hand the buffer back to the MMA issuer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_accempty(buf));
        }
        if constexpr (ACC_OUT) {
          int32_t* y = static_cast<int32_t*>(seg.y);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (n_ok && c0 + i < c.rows)
              y[(c.t0 + c0 + i) * ldy + n] = static_cast<int32_t>(acc[i]) >> 4;
        } else {
          __half* y = static_cast<__half*>(seg.y);
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            // acc / 16 as fp32, exactly: |acc / 16| < 2^22, so adding it to the
            // integer bits of 1.5 * 2^23 and subtracting that value is exact.
            const float a0 = __fsub_rn(__int_as_float((static_cast<int32_t>(acc[i]) >> 4) + 0x4B400000), 12582912.0f);
            const float a1 = __fsub_rn(__int_as_float((static_cast<int32_t>(acc[i + 1]) >> 4) + 0x4B400000), 12582912.0f);
            const bool ok0 = c0 + i < c.rows, ok1 = c0 + i + 1 < c.rows;
            const float v0 = __fmul_rn(__fmul_rn(a0, ok0 ? ts[c0 + i] : 0.f), sw);
            const float v1 = __fmul_rn(__fmul_rn(a1, ok1 ? ts[c0 + i + 1] : 0.f), sw);
            const __half2 h = __floats2half2_rn(v0, v1);
            stage[i * 32 + lane] = __low2half(h);
            stage[(i + 1) * 32 + lane] = __high2half(h);
          }
          __syncwarp();
          if (seg.vec_store) {
            // 16 tokens x 32 rows -> per token a 64-byte row segment, 16 B per thread
#pragma unroll
            for (int pass = 0; pass < 2; ++pass) {
              const int i = pass * 8 + (lane >> 2);
              const int ch = lane & 3;
              const int nn = c.n0 + quarter * 32 + ch * 8;
              if (c0 + i < c.rows && nn < seg.n)
                *reinterpret_cast<uint4*>(y + (c.t0 + c0 + i) * ldy + nn) =
                    *reinterpret_cast<const uint4*>(stage + i * 32 + ch * 8);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (n_ok && c0 + i < c.rows) y[(c.t0 + c0 + i) * ldy + n] = stage[i * 32 + lane];
          }
          __syncwarp();
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

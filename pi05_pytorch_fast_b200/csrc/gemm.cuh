// Packed-INT4 W4A4 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8).
//
// Computes, for each weight matrix W (N x K, 4-bit codes + fp32 row scale)
// sharing one quantised activation (M x K int8 codes + fp32 row scale):
//     acc[m, n] = sum_k qa[m, k] * qw[n, k]                  (exact int32)
//     y[m, n]   = fp16( (fp32(acc) * sa[m]) * sw[n] )         (RN, left to right)
// which is the reference's gemm_iu4 / gemm_iu4_shape contract
// (pi05_fast/w4a4/csrc/int4_gemm.cu:66-204, :207-394; epilogue :199-200).
//
// Design (one persistent CTA per SM, 18 warps):
//  * Tiles put weights on the MMA's M side (128 rows = UMMA M) and tokens on
//    its N side (a multiple of 16, <= 208), so a ragged token count such as
//    776 splits into near-equal tiles (4 x 208) instead of a mostly empty
//    128-row tile.  Several weight matrices (gate/up, q/k/v) form one tile
//    space, so each op is one launch.
//  * warp 0 (TMA producer) streams, per 128-wide K step, the packed weight
//    tile (8 KB, either reference layout, straight from the reference's
//    tensors) and the int8 token tile (128-byte swizzle) into a ring of
//    kGemmRing (6) stages.  The ring depth is a compile-time constant, so
//    every ring index below is a constant after unrolling.
//  * warps 2-9 (unpack, two groups of 4 taking alternate K steps) each own
//    32 weight rows: they read the staged nibbles, expand them to int8 (x16,
//    see expand_nibbles_x16) in registers and write them with tcgen05.st
//    straight into TMEM, where the MMA reads its A operand.  The unpacked
//    weights never touch shared memory, which leaves the shared-memory
//    bandwidth to the TMA writes and the MMA's reads of the token operand.
//  * warp 1 runs the MMA loop (warp-uniform control flow and operands) and
//    one elected lane issues tcgen05.mma (A from TMEM, B = tokens from
//    shared memory) into one of two TMEM accumulators (double buffered, so
//    the epilogue of a tile overlaps the mainloop of the next) and frees each
//    step with ONE tcgen05.commit.
//  * warps 10-17 (epilogue, two per TMEM lane quarter taking alternate
//    16-column chunks) read the accumulator with tcgen05.ld, divide by 16
//    (exact), apply the token and weight scales in fp32, round to fp16 and
//    transpose 16x32 blocks through shared memory into 16-byte row stores.
//  * SPLIT = true (split-K): the two CTAs of a cluster run the two K halves
//    of one tile; each pushes the int32 partial sums of the half of the tile
//    its partner writes out into the partner's idle ring (distributed shared
//    memory, st.async with transaction bytes on the partner's barrier), then
//    adds the partner's sums to its own half and writes that half.
// TMEM map (512 columns): accumulators at [0, T) and [T, 2T) for a token tile
// of T columns, then A stages of 32 columns (128 K-bytes per row) up to 512.
#pragma once

#include "common.cuh"

namespace w4a4 {

constexpr int kBlockW = 128;      // weight rows per tile (UMMA M)
constexpr int kBlockK = 128;      // K elements per pipeline step
constexpr int kTokTileMax = 208;  // max tokens per tile (UMMA N)
constexpr int kMaxStages = 12;    // shared-memory ring (tokens + packed weights)
constexpr int kGemmRing = 6;      // single-CTA kernel: shared-memory ring depth (compile time)
constexpr int kTmemCols = 512;
constexpr int kUnpackGroups = 2;
constexpr int kEpiWarps = 8;       // two per TMEM lane quarter, alternate 16-column chunks
constexpr int kGemmThreads = 32 * (2 + 4 * kUnpackGroups + kEpiWarps);  // 18 warps
constexpr int kEpiWarp0 = 2 + 4 * kUnpackGroups;
constexpr int kMaxSegments = 3;

constexpr int kWpkBytes = kBlockW * kBlockK / 2;  // 8 KB packed weights per step
constexpr int kEpiBytesPerWarp = 16 * 32 * 2;     // 16 tokens x 32 rows fp16
constexpr int kEpiScaleBytes = kTokTileMax * 4;   // a tile's token scales, per epilogue warp
constexpr int kXchgChunkBytes = 16 * 32 * 4;      // split-K: one 16-column int32 chunk of one warp
// mbarrier slots reserved in shared memory: up to four rings of kMaxStages
// (single CTA: full / ready / empty; CTA pair: wfull / tfull / ready / empty),
// accfull[2], accempty[2] and drain.
constexpr int kNumBars = 4 * kMaxStages + 4 + 1 + kEpiWarps + 1;  // + split-K xfull per epilogue warp, xready
constexpr int kFixedSmem =
    kEpiWarps * kEpiBytesPerWarp + kEpiWarps * kEpiScaleBytes + kNumBars * 8 + 16 +
    1024 /*alignment slack*/;
constexpr int kSmemLimit = 232448;
static_assert(2 * kTokTileMax + 3 * 32 <= kTmemCols, "TMEM budget");

__host__ __device__ constexpr int gemm_smem_bytes(int tok_tile) {
  return kGemmRing * (tok_tile * kBlockK + kWpkBytes) + kFixedSmem;
}
// TMEM A slots of the single-CTA kernel: a divisor of kGemmRing that fits
// beside the two accumulators (6 up to 160-token tiles, else 3).
__host__ __device__ constexpr int gemm_ring_a_stages(int tok_tile) {
  return 2 * tok_tile + 6 * 32 <= kTmemCols ? 6 : 3;
}

static_assert(kGemmRing * (kTokTileMax * kBlockK + kWpkBytes) + kFixedSmem <= kSmemLimit,
              "the single-CTA ring must fit the widest tile");
static_assert(2 * kTokTileMax + 3 * 32 <= kTmemCols, "three A slots must fit beside the widest tile");
// Split-K: each rank pushes partial sums into the partner's idle ring (token
// and weight rings are contiguous), at most each epilogue warp's ceil(T / 32)
// chunks of 2 KB, 8 T / 32 * 2 KB <= 512 T bytes in all, which always fits in
// the ring's kGemmRing * (128 T + 8 KB) bytes.
static_assert(kEpiWarps * 2 * kXchgChunkBytes <= kGemmRing * (16 * kBlockK + kWpkBytes),
              "the split-K exchange must fit the ring of the narrowest tile");

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

// Up to this K, |acc / 16| <= 7 * 8 * K < 2^22 and the epilogue converts it
// to fp32 with the magic-number trick; beyond it the host runs the WIDE
// instantiation, which converts with cvt.rn.f32.s32 (the reference's
// (float)acc, correct for any int32).  A compile-time variant keeps the hot
// kernels' code unchanged: extra code in this epilogue slows the whole GEMM
// (its issue loops share the SM's instruction cache with it).
constexpr int kMagicMaxK = 65536;

struct alignas(64) GemmParams {
  CUtensorMap tmap_tok;     // int8 codes [M, K] in GEMM byte order: box {128, tok_tile}, SW128
  GemmSegment seg[kMaxSegments];
  const float* row_scale;   // [M] token scales
  unsigned long long wait_limit_ns;
  long long m;
  int k;
  int tok_tile;
  int stages;               // shared-memory ring depth (kGemmRing)
  int a_stages;             // TMEM A ring depth (gemm_ring_a_stages)
  int n_tok_tiles;
  int w_tiles;
  int tok_group;            // token tiles per rasterisation group (decode_tile)
  int n_seg;
  int k_tiles;
};

struct TileCoord {
  int seg;
  int n0;
  long long t0;
  int rows;
};

// Tile order: token tiles in groups of p.tok_group; within a group the weight
// tile changes every g tiles (g = the group's size), so the CTAs running at
// one time share a few weight tiles and the group's token tiles.  With one
// group (the activation codes fit in L2) each weight tile streams from HBM
// once; with several (large M) each group's codes stay in L2 while the
// weights stream once per group.
__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, int tile) {
  const int per_group = p.tok_group * p.w_tiles;
  const int group = tile / per_group;
  const int r = tile - group * per_group;
  const int g = min(p.tok_group, p.n_tok_tiles - group * p.tok_group);
  const int wt = r / g;
  const int tt = group * p.tok_group + (r - wt * g);
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

// Token scales of a tile into this warp's private copy, zero past the last
// valid token (up to the MMA width), so the epilogue needs no per-value test.
__device__ __forceinline__ void stage_tile_scales(float* ts, const float* row_scale,
                                                  const TileCoord& c, int lane) {
  const int mma_n = (c.rows + 15) & ~15;
  __syncwarp();
  for (int i = lane; i < mma_n; i += 32) ts[i] = i < c.rows ? __ldg(row_scale + c.t0 + i) : 0.f;
  __syncwarp();
}

// One 16-token chunk of the epilogue for one warp: thread `lane` owns weight
// row n (its TMEM lane) and acc[i] = 16 * sum_k qa[token c0+i] * qw[n].
template <bool ACC_OUT, bool WIDE = false>
__device__ __forceinline__ void epilogue_chunk(const GemmSegment& seg, const TileCoord& c, int n_warp,
                                               int lane, int c0, float sw, const uint32_t (&acc)[16],
                                               __half* stage, const float* ts) {
  const long long ldy = seg.n;
  const int n = n_warp + lane;
  const bool n_ok = n < seg.n;
  if constexpr (ACC_OUT) {
    int32_t* y = static_cast<int32_t*>(seg.y);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n_ok && c0 + i < c.rows) y[(c.t0 + c0 + i) * ldy + n] = static_cast<int32_t>(acc[i]) >> 4;
  } else {
    __half* y = static_cast<__half*>(seg.y);
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 v = *reinterpret_cast<const float4*>(ts + c0 + i);
      t[i] = v.x;
      t[i + 1] = v.y;
      t[i + 2] = v.z;
      t[i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      // acc / 16 as fp32: for K <= kMagicMaxK |acc / 16| < 2^22, so adding it
      // to the integer bits of 1.5 * 2^23 and subtracting that value is
      // exact; the WIDE kernel (K > kMagicMaxK) rounds it like (float)acc.
      float a0, a1;
      if constexpr (!WIDE) {
        a0 = __fsub_rn(__int_as_float((static_cast<int32_t>(acc[i]) >> 4) + 0x4B400000), 12582912.0f);
        a1 = __fsub_rn(__int_as_float((static_cast<int32_t>(acc[i + 1]) >> 4) + 0x4B400000), 12582912.0f);
      } else {
        a0 = __int2float_rn(static_cast<int32_t>(acc[i]) >> 4);
        a1 = __int2float_rn(static_cast<int32_t>(acc[i + 1]) >> 4);
      }
      const __half2 h = __floats2half2_rn(__fmul_rn(__fmul_rn(a0, t[i]), sw),
                                          __fmul_rn(__fmul_rn(a1, t[i + 1]), sw));
      stage[i * 32 + lane] = __low2half(h);
      stage[(i + 1) * 32 + lane] = __high2half(h);
    }
    __syncwarp();
    if (seg.vec_store) {
      // 16 tokens x 32 rows -> per token a 64-byte row segment, 16 B per thread
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int i = pass * 8 + (lane >> 2);
        const int nn = n_warp + (lane & 3) * 8;
        if (c0 + i < c.rows && nn < seg.n)
          *reinterpret_cast<uint4*>(y + (c.t0 + c0 + i) * ldy + nn) =
              *reinterpret_cast<const uint4*>(stage + i * 32 + (lane & 3) * 8);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n_ok && c0 + i < c.rows) y[(c.t0 + c0 + i) * ldy + n] = stage[i * 32 + lane];
    }
    __syncwarp();
  }
}

// The epilogue of one tile for one warp: its TMEM lane quarter (weight rows
// n_warp .. n_warp+31), 16-column chunks half + 2j for j = first, first +
// step, ... (all of them by default).  The next chunk's TMEM load is issued
// before the current chunk is processed, and release() is called once, as
// soon as this warp's last TMEM load completed (the accumulator buffer may
// then be overwritten).  combine(acc, j) sees each chunk first (split-K
// exchange) and returns whether to write it out.
struct NoCombine {
  __device__ __forceinline__ bool operator()(uint32_t (&)[16], int) const { return true; }
};

template <bool ACC_OUT, typename Release, typename Combine = NoCombine, bool WIDE = false>
__device__ __forceinline__ void epilogue_tile(const GemmSegment& seg, const TileCoord& c, int n_warp,
                                              uint32_t tacc, int half, int lane, __half* stage,
                                              const float* ts, Release release,
                                              Combine combine = Combine(), int first = 0,
                                              int step = 1) {
  const int nq = ((c.rows + 15) & ~15) >> 4;
  const int all = (nq - half + 1) >> 1;                              // chunks half + 2j, j < all
  const int my = all > first ? (all - first + step - 1) / step : 0;  // the ones taken here
  if (my <= 0) {
    release();
    return;
  }
  const auto col = [&](int i) { return (half + 2 * (first + step * i)) * 16; };
  const int n = n_warp + lane;
  const float sw =
      (n < seg.n && !ACC_OUT) ? __ldg(seg.scale + static_cast<long long>(n) * seg.scale_stride) : 0.f;
  uint32_t a0[16], a1[16];
  tmem_ld_32x32b_x16(tacc + col(0), a0);
  tmem_ld_wait();
  if (my == 1) release();
  for (int j = 0; j < my; j += 2) {
    if (j + 1 < my) tmem_ld_32x32b_x16(tacc + col(j + 1), a1);
    if (combine(a0, first + step * j))
      epilogue_chunk<ACC_OUT, WIDE>(seg, c, n_warp, lane, col(j), sw, a0, stage, ts);
    if (j + 1 >= my) break;
    tmem_ld_wait();
    if (j + 2 == my) release();
    if (j + 2 < my) tmem_ld_32x32b_x16(tacc + col(j + 2), a0);
    if (combine(a1, first + step * (j + 1)))
      epilogue_chunk<ACC_OUT, WIDE>(seg, c, n_warp, lane, col(j + 1), sw, a1, stage, ts);
    if (j + 2 >= my) break;
    tmem_ld_wait();
    if (j + 3 == my) release();
  }
}

// ACC_OUT = true writes the raw int32 accumulators (seg.y as int32 [M, n])
// instead of fp16: a test hook that proves the integer products bit-exact.
//
// SPLIT = true: split-K over clusters of two CTAs, each cluster one output
// tile (the host launches it only when the tiles do not outnumber the
// clusters).  Rank r runs K steps [r k_tiles, (r+1) k_tiles) through the same
// pipeline into its own TMEM.  Once a rank's MMAs are done its token ring is
// idle: each rank pushes the partial sums of the half of the tile's columns
// the partner writes out into the partner's ring (distributed shared memory),
// then adds the partner's partial sums of its own half (int32, exact) and
// writes that half.
// WIDE = true: the K > kMagicMaxK conversion (single-CTA, no split-K only).
template <int LAYOUT, bool ACC_OUT, bool SPLIT, bool WIDE = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a4_gemm_kernel(const __grid_constant__ GemmParams p) {
  constexpr int RING = kGemmRing;
  constexpr int SA_SMALL = 3;  // A slots when the full ring does not fit in TMEM
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.stages, SA = p.a_stages;
  const int tok_bytes = p.tok_tile * kBlockK;
  uint8_t* tok_ring = base;                              // [S][tok_tile * 128], 1 KB aligned
  uint8_t* wpk_ring = base + S * tok_bytes;              // [S][8 KB]
  uint8_t* epi = wpk_ring + S * kWpkBytes;               // kEpiWarps x 1 KB
  float* tile_scale = reinterpret_cast<float*>(epi + kEpiWarps * kEpiBytesPerWarp);  // [warps][208]
  uint64_t* bars = reinterpret_cast<uint64_t*>(tile_scale + kEpiWarps * kTokTileMax);
  // full[s]   TMA bytes (packed weights + tokens) of step i landed.
  // ready[s]  the unpack group wrote step i's A operand into TMEM (4 warps,
  //           each after observing full[s]): the MMA issuer's only wait.
  // empty[s]  MMA(i) completed (one commit per step): ring slot s is free,
  //           and so is the TMEM A slot of step i once the A ring wraps.
  const auto bar_full = [&](int s) { return smem_addr(bars + s); };
  const auto bar_ready = [&](int s) { return smem_addr(bars + kMaxStages + s); };
  const auto bar_empty = [&](int s) { return smem_addr(bars + 2 * kMaxStages + s); };
  const auto bar_accfull = [&](int b) { return smem_addr(bars + 3 * kMaxStages + b); };
  const auto bar_accempty = [&](int b) { return smem_addr(bars + 3 * kMaxStages + 2 + b); };
  const uint32_t bar_drain = smem_addr(bars + 3 * kMaxStages + 4);
  // split-K: xready the partner's MMAs are done, its token ring is free (one
  // arrival per partner epilogue warp); xfull[w] the partner warp's partial
  // sums landed (this warp's arrival with the expected bytes, then the
  // transaction bytes of the partner's st.async pushes).
  const auto bar_xfull = [&](int w) { return smem_addr(bars + 3 * kMaxStages + 5 + w); };
  const uint32_t bar_xready = smem_addr(bars + 3 * kMaxStages + 5 + kEpiWarps);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned* err = &g_w4a4_device_error;
  const uint64_t limit = p.wait_limit_ns;
  const int total_tiles = p.n_tok_tiles * p.w_tiles;
  const int acc_cols = p.tok_tile;
  const int a_col0 = 2 * acc_cols;
  // Tiles are dealt to CTAs (or, for split-K, to clusters) round robin.
  const uint32_t rank = SPLIT ? cluster_ctarank() : 0u;
  const int unit0 = SPLIT ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ustride = SPLIT ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int k_begin = static_cast<int>(rank) * p.k_tiles;  // first K step of this CTA

  // The issue loop is unrolled over the compile-time ring (RING slots, SA a
  // divisor of it).  A launch that breaks this touches nothing and reports it.
  if (S != RING || (SA != SA_SMALL && SA != RING) || 2 * p.tok_tile + 32 * SA > kTmemCols ||
      p.k_tiles < 1 || (SPLIT && total_tiles > ustride)) {
    if (threadIdx.x == 0) atomicOr(&g_w4a4_device_error, kErrBadParams);
    return;
  }

  // The next kernel may be scheduled as soon as every CTA got here; it waits
  // for this grid's completion itself before reading the outputs.
  pdl_launch_dependents();

  // ---- setup
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_ready(s), 4);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accfull(b), 1);
      mbar_init(bar_accempty(b), kEpiWarps);
    }
    mbar_init(bar_drain, 1);
    if (SPLIT) {
      for (int w = 0; w < kEpiWarps; ++w) mbar_init(bar_xfull(w), 1);
      mbar_init(bar_xready, kEpiWarps);
    }
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
  if (SPLIT) cluster_sync();  // the partner's barriers exist before any remote traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (lane 0)
    if (lane == 0) {
      const uint32_t tx_bytes = kWpkBytes + static_cast<uint32_t>(tok_bytes);
      const auto load_weights = [&](const TileCoord& c, int kt, int slot) {
        kt += k_begin;
        const uint32_t wdst = smem_addr(wpk_ring + slot * kWpkBytes);
        const CUtensorMap* wmap = &p.seg[c.seg].tmap_w;
        if constexpr (LAYOUT == kRowMajor)
          tma_load_2d(wdst, wmap, kt * (kBlockK / 8), c.n0, bar_full(slot));
        else
          tma_load_2d(wdst, wmap, c.n0 * 2, kt * (kBlockK / 16), bar_full(slot));
      };
      // Weights do not depend on the previous kernel: fill the first ring
      // pass with them before waiting for that kernel's tokens.
      int pre = 0;
      if (unit0 < total_tiles) {
        const TileCoord c0 = decode_tile(p, unit0);
        pre = min(S, p.k_tiles);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(bar_full(i), tx_bytes);
          load_weights(c0, i, i);
        }
      }
      pdl_wait();
      RingPos st;
      int issued = 0;
      bool alive = true;
      for (int tile = unit0; alive && tile < total_tiles; tile += ustride) {
        const TileCoord c = decode_tile(p, tile);
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (issued >= pre) {
            if (issued >= S &&
                !mbar_wait_bounded(bar_empty(st.idx), st.phase ^ 1u, abort_flag, err,
                                   kErrWaitEmpty, limit)) {
              alive = false;
              break;
            }
            mbar_arrive_expect_tx(bar_full(st.idx), tx_bytes);
            load_weights(c, kt, st.idx);
          }
          tma_load_2d(smem_addr(tok_ring + st.idx * tok_bytes), &p.tmap_tok, (kt + k_begin) * kBlockK,
                      static_cast<int>(c.t0), bar_full(st.idx));
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
    // ------------------------------------------------ MMA issuer (one elected lane)
    // The issue loop is the kernel's critical path: a 128 x T x 128 step is
    // 2T tensor cycles (416 at T = 208), and each tcgen05.mma takes ~85
    // cycles to issue.  The whole warp runs the loop (warp-uniform control
    // flow and operands) and one elected lane issues; the loop is unrolled
    // over the shared-memory ring, so every barrier address, B descriptor and
    // A slot is a compile-time offset or a register, and the next step's
    // ready barrier is tested while this step's MMAs issue.
    {
      const bool issuer = elect_one();  // the one lane that issues every MMA and commit
      const uint64_t bdesc0 = smem_desc_sw128(smem_addr(tok_ring));
      const uint64_t bstep = static_cast<uint64_t>(tok_bytes >> 4);
      uint64_t bd[RING];
#pragma unroll
      for (int r = 0; r < RING; ++r) bd[r] = bdesc0 + r * bstep;
      const uint32_t a_base = tmem_base + a_col0;
      const bool sa_full = SA == RING;
      const uint32_t ready0 = bar_ready(0), empty0 = bar_empty(0);
      uint32_t phase = 0;
      int tile = unit0, tcount = 0, kt = 0, buf = 0;
      uint32_t d_tmem = tmem_base, idesc = 0;
      // Starts tile `tile` (the tcount-th of this CTA): its accumulator buffer
      // must have been drained by the epilogue two tiles ago.
      const auto begin_tile = [&]() -> bool {
        const TileCoord c = decode_tile(p, tile);
        idesc = idesc_i8(kBlockW, (c.rows + 15) & ~15);
        buf = tcount & 1;
        d_tmem = tmem_base + buf * acc_cols;
        return tcount < 2 || warp_all(mbar_wait_bounded(bar_accempty(buf), ((tcount >> 1) - 1) & 1,
                                                        abort_flag, err, kErrWaitAccum, limit));
      };
      bool alive = tile < total_tiles && begin_tile();
      bool pre = false;  // the current step's ready, tested during the previous step's issue
      while (alive) {
#pragma unroll
        for (int r = 0; r < RING; ++r) {
          if (!pre && !warp_all(mbar_wait_fast(ready0 + 8u * r, phase, abort_flag, err,
                                               kErrWaitUnpack, limit))) {
            alive = false;
            break;
          }
          tc_fence_after();
          const bool pre_l =
              mbar_test_wait(ready0 + 8u * ((r + 1) % RING), r + 1 == RING ? phase ^ 1u : phase);
          const uint32_t a_slot = a_base + 32u * (sa_full ? r : r % SA_SMALL);
          if (issuer) {
            umma_i8_ts(d_tmem, a_slot, bd[r], idesc, kt != 0);
            umma_i8_ts(d_tmem, a_slot + 8, bd[r] + 2, idesc, 1u);
            umma_i8_ts(d_tmem, a_slot + 16, bd[r] + 4, idesc, 1u);
            umma_i8_ts(d_tmem, a_slot + 24, bd[r] + 6, idesc, 1u);
            umma_commit(empty0 + 8u * r);
          }
          pre = __all_sync(0xffffffffu, pre_l);
          if (++kt == p.k_tiles) {
            if (issuer) umma_commit(bar_accfull(buf));
            kt = 0;
            tile += ustride;
            ++tcount;
            if (tile >= total_tiles || !begin_tile()) {
              alive = false;
              break;
            }
          }
        }
        phase ^= 1u;
      }
      // Every MMA of this CTA has completed once this commit arrives.
      if (issuer) umma_commit(bar_drain);
      __syncwarp();
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
    for (int tile = unit0; alive && tile < total_tiles; tile += ustride) {
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
          if (lane == 0) mbar_arrive(bar_ready(st.idx));
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
    const int half = ew >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    __half* stage = reinterpret_cast<__half*>(epi + ew * kEpiBytesPerWarp);
    float* ts = tile_scale + ew * kTokTileMax;  // warp-private
    pdl_wait();  // token scales come from the previous kernel; y may be read by it
    int tcount = 0;
    for (int tile = unit0; tile < total_tiles; tile += ustride, ++tcount) {
      const TileCoord c = decode_tile(p, tile);
      const int buf = tcount & 1;
      if (!ACC_OUT) stage_tile_scales(ts, p.row_scale, c, lane);
      const bool ok = mbar_wait_bounded(bar_accfull(buf), (tcount >> 1) & 1, abort_flag, err,
                                        kErrWaitAccum, limit);
      if (!warp_all(ok)) break;
      tc_fence_after();
      const uint32_t accempty = bar_accempty(buf);
      const auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accempty);
      };
      const uint32_t tacc = tmem_base + lane_addr + buf * acc_cols;
      if constexpr (!SPLIT) {
        epilogue_tile<ACC_OUT, decltype(release), NoCombine, WIDE>(p.seg[c.seg], c, c.n0 + quarter * 32, tacc,
                                                                   half, lane, stage, ts, release);
      } else {
        // Both ranks finish half of the tile: rank r writes the chunks with
        // j % 2 == r (j indexes this warp's chunks half + 2j) and pushes its
        // partial sums of the others into the partner's token ring, which is
        // idle once the partner's MMAs are done.  Exchange area of a warp:
        // chunk j at [j][4 quads][32 lanes][4 int32] (a warp's 16-byte stores and
        // loads cover 512 contiguous bytes: no bank conflicts); ceil(T / 32)
        // chunks per warp.
        const int xstride = ((p.tok_tile / 16 + 1) / 2) * kXchgChunkBytes;
        const uint32_t xarea = smem_addr(tok_ring) + ew * xstride;
        const uint32_t peer = rank ^ 1u;
        // The partner's pushes into our ring complete bytes on xfull[ew]: arm it
        // with the bytes of the chunks this warp writes (j = rank, rank + 2, ...).
        if (lane == 0) {
          const int all = ((((c.rows + 15) & ~15) >> 4) - half + 1) >> 1;
          const int mine = all > static_cast<int>(rank) ? (all - static_cast<int>(rank) + 1) / 2 : 0;
          mbar_arrive_expect_tx(bar_xfull(ew), static_cast<uint32_t>(mine * kXchgChunkBytes));
        }
        // our MMAs are done: our ring is free for the partner's sums
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar_xready, peer));
        const bool free = warp_all(mbar_wait_bounded_cl(bar_xready, 0, abort_flag, err,
                                                        kErrWaitAccum, limit));
        const uint32_t dst0 = mapa_shared(xarea, peer) + lane * 16;
        const uint32_t peer_xfull = mapa_shared(bar_xfull(ew), peer);
        bool released = false;
        const auto release_once = [&] {
          if (!released) release();
          released = true;
        };
        epilogue_tile<ACC_OUT>(p.seg[c.seg], c, c.n0 + quarter * 32, tacc, half, lane, stage, ts,
                               [] {}, [&](uint32_t (&acc)[16], int j) -> bool {
          if (free) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st_async_v4(dst0 + j * kXchgChunkBytes + 512 * q, acc[4 * q], acc[4 * q + 1],
                          acc[4 * q + 2], acc[4 * q + 3], peer_xfull);
          }
          return false;
        }, static_cast<int>(peer), 2);
        const bool got = warp_all(mbar_wait_bounded_cl(bar_xfull(ew), 0, abort_flag, err,
                                                       kErrWaitAccum, limit));
        epilogue_tile<ACC_OUT>(p.seg[c.seg], c, c.n0 + quarter * 32, tacc, half, lane, stage, ts,
                               release_once, [&](uint32_t (&acc)[16], int j) -> bool {
          if (!got) return true;
          const uint4* src = reinterpret_cast<const uint4*>(tok_ring + ew * xstride +
                                                            j * kXchgChunkBytes + lane * 16);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = src[32 * q];
            acc[4 * q] += v.x;
            acc[4 * q + 1] += v.y;
            acc[4 * q + 2] += v.z;
            acc[4 * q + 3] += v.w;
          }
          return true;
        }, static_cast<int>(rank), 2);
        release_once();
      }
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (SPLIT) cluster_sync();  // no remote store or arrival may target an exited CTA
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

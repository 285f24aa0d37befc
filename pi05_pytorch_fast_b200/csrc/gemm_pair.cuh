// The W4A4 GEMM on CTA pairs (tcgen05 cta_group::2): same contract, tiles
// and roles as gemm.cuh's single-CTA kernel, but each MMA instruction spans
// the two SMs of a cluster.
//
// Why: a 1-CTA step feeds each token byte to only 128 weight rows, so the
// token copy alone needs ~64 B/clk of the ~123 B/clk an SM's TMA engine
// moves (plus ~136 cycles per box); the kernel is copy-bound.  With a pair,
// one MMA is M = 256 weight rows (128 per CTA, A in each CTA's own TMEM) x
// N tokens, and each CTA loads only HALF of the token tile (B is split by N
// across the pair's shared memory), halving the token traffic per SM.
//
// Per pair:
//  * both CTAs' producers load their own 128 weight rows (1-CTA TMA, local
//    barrier) and their half of the token tile (cta_group::2 TMA whose bytes
//    are counted on the LEADER's ready barrier; the leader announces the
//    whole tile's bytes);
//  * both CTAs' unpack warps write their rows' A operand into their own TMEM
//    and arrive remotely on the leader's ready barrier;
//  * the leader's MMA thread issues the pair MMAs and multicasts its commits
//    (step done / accumulator full / drain) to both CTAs;
//  * both CTAs' epilogues read their own TMEM (their 128 weight rows x all N
//    tokens) and arrive remotely on the leader's accumulator-empty barrier.
#pragma once

#include "gemm.cuh"

namespace w4a4 {

constexpr int kPairTmemCols = 512;

// Shared memory of the pair kernel for a token tile of `tok_tile` rows: a
// kGemmRing-stage ring, each CTA holding tok_tile / 2 token rows per stage.
__host__ __device__ constexpr int gemm_pair_smem_bytes(int tok_tile) {
  return kGemmRing * (tok_tile / 2 * kBlockK + kWpkBytes) + kFixedSmem;
}

__device__ __forceinline__ TileCoord decode_pair_tile(const GemmParams& p, int tile, int rank) {
  const int wt = tile / p.n_tok_tiles;  // 256-row weight tile (pair units)
  const int tt = tile - wt * p.n_tok_tiles;
  TileCoord c;
  c.seg = 0;
#pragma unroll
  for (int s = 1; s < kMaxSegments; ++s)
    if (s < p.n_seg && wt >= p.seg[s].tile_begin) c.seg = s;
  c.n0 = (wt - p.seg[c.seg].tile_begin) * (2 * kBlockW) + rank * kBlockW;
  c.t0 = static_cast<long long>(tt) * p.tok_tile;
  c.rows = static_cast<int>(min(static_cast<long long>(p.tok_tile), p.m - c.t0));
  return c;
}

template <int LAYOUT, bool ACC_OUT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w4a4_gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
  const int S = p.stages, SA = p.a_stages;
  const int half = p.tok_tile / 2;              // token rows held by each CTA
  const int tok_bytes = half * kBlockK;         // per CTA per stage
  uint8_t* tok_ring = base;                     // [S][half * 128], 1 KB aligned
  uint8_t* wpk_ring = base + S * tok_bytes;     // [S][8 KB]
  uint8_t* epi = wpk_ring + S * kWpkBytes;      // kEpiWarps x 1 KB
  float* tile_scale = reinterpret_cast<float*>(epi + kEpiWarps * kEpiBytesPerWarp);  // [warps][208]
  uint64_t* bars = reinterpret_cast<uint64_t*>(tile_scale + kEpiWarps * kTokTileMax);
  // wfull[s]  local: this CTA's packed weights of step i landed.
  // tfull[s]  leader: both CTAs' token halves of step i landed (the peer's
  //           .cta_group::2 copy completes on the leader's barrier).
  // ready[s]  leader: the 8 unpack warps of step i (4 per CTA) wrote their A
  //           rows; the leader's warps wait tfull first, so ready implies the
  //           whole B operand landed: the MMA issuer's only wait.
  // empty[s]  both (multicast commit): MMA(i) completed.
  // accfull/accempty[2]: accumulator handshake (accempty lives in the leader).
  const auto bar_wfull = [&](int s) { return smem_addr(bars + s); };
  const auto bar_tfull = [&](int s) { return smem_addr(bars + kMaxStages + s); };
  const auto bar_ready = [&](int s) { return smem_addr(bars + 2 * kMaxStages + s); };
  const auto bar_empty = [&](int s) { return smem_addr(bars + 3 * kMaxStages + s); };
  const auto bar_accfull = [&](int b) { return smem_addr(bars + 4 * kMaxStages + b); };
  const auto bar_accempty = [&](int b) { return smem_addr(bars + 4 * kMaxStages + 2 + b); };
  const uint32_t bar_drain = smem_addr(bars + 4 * kMaxStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned* err = &g_w4a4_device_error;
  const uint64_t limit = p.wait_limit_ns;
  const int total_tiles = p.n_tok_tiles * p.w_tiles;
  const int acc_cols = p.tok_tile;
  const int a_col0 = 2 * acc_cols;

  // The issue loop is unrolled over the compile-time ring (kGemmRing slots, SA
  // a divisor of it), as in the single-CTA kernel: a launch that breaks this
  // touches nothing and reports it.
  constexpr int RING = kGemmRing;
  constexpr int SA_SMALL = 3;
  if (S != RING || (SA != SA_SMALL && SA != RING) || 2 * p.tok_tile + 32 * SA > kPairTmemCols ||
      p.k_tiles < 1 || (p.tok_tile & 15)) {
    if (threadIdx.x == 0) atomicOr(&g_w4a4_device_error, kErrBadParams);
    return;
  }

  pdl_launch_dependents();
  pdl_wait();

  // ---- setup (both CTAs), then a cluster barrier before any remote traffic
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_wfull(s), 1);
      mbar_init(bar_tfull(s), 1);   // leader: its producer's expect_tx of both halves
      mbar_init(bar_ready(s), 8);   // leader: 4 unpack warps per CTA
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accfull(b), 1);
      mbar_init(bar_accempty(b), 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tmap_tok);
    for (int s = 0; s < p.n_seg; ++s) tma_prefetch_desc(&p.seg[s].tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), kPairTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (lane 0, both CTAs)
    if (lane == 0) {
      RingPos st;
      int issued = 0;
      bool alive = true;
      for (int tile = cluster; alive && tile < total_tiles; tile += n_clusters) {
        const TileCoord c = decode_pair_tile(p, tile, rank);
        const CUtensorMap* wmap = &p.seg[c.seg].tmap_w;
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (issued >= S &&
              !mbar_wait_bounded_cl(bar_empty(st.idx), st.phase ^ 1u, abort_flag, err,
                                    kErrWaitEmpty, limit)) {
            alive = false;
            break;
          }
          const uint32_t wfull = bar_wfull(st.idx), tfull = bar_tfull(st.idx);
          mbar_arrive_expect_tx(wfull, kWpkBytes);
          const uint32_t wdst = smem_addr(wpk_ring + st.idx * kWpkBytes);
          if constexpr (LAYOUT == kRowMajor)
            tma_load_2d(wdst, wmap, kt * (kBlockK / 8), c.n0, wfull);
          else
            tma_load_2d(wdst, wmap, c.n0 * 2, kt * (kBlockK / 16), wfull);
          if (leader) mbar_arrive_expect_tx(tfull, static_cast<uint32_t>(2 * tok_bytes));
          tma_load_2d_pair(smem_addr(tok_ring + st.idx * tok_bytes), &p.tmap_tok, kt * kBlockK,
                           static_cast<int>(c.t0) + static_cast<int>(rank) * half, tfull);
          st.advance(S);
          ++issued;
        }
      }
      // Drain: this CTA's weight copies, and on the leader every token copy
      // of both CTAs (they complete on the leader's tfull); the exit cluster
      // barrier keeps the peer resident until then.
      for (int i = 0; i < S && i < issued; ++i) {
        const int last = i + ((issued - 1 - i) / S) * S;
        volatile int no_abort = 0;
        mbar_wait_bounded(bar_wfull(i), (last / S) & 1, &no_abort, err, kErrWaitDrain, limit);
        if (leader)
          mbar_wait_bounded_cl(bar_tfull(i), (last / S) & 1, &no_abort, err, kErrWaitDrain, limit);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader lane 0)
    // Unrolled over the compile-time ring like the single-CTA issuer; each
    // instruction spans both SMs (M = 256), so one thread issues a step for
    // two SMs, and every commit is multicast to both CTAs.  With T = 208 the
    // TMEM holds 3 A slots: the unpack of step i waits for MMA(i - 3), which
    // leaves two steps of MMA time to hide the unpack -> ready -> issue loop.
    if (lane == 0 && leader) {
      const uint64_t bdesc0 = smem_desc_sw128(smem_addr(tok_ring));
      const uint64_t bstep = static_cast<uint64_t>(tok_bytes >> 4);
      uint64_t bd[RING];
#pragma unroll
      for (int r = 0; r < RING; ++r) bd[r] = bdesc0 + r * bstep;
      const uint32_t a_base = tmem_base + a_col0;
      const bool sa_full = SA == RING;
      const uint32_t ready0 = bar_ready(0), empty0 = bar_empty(0);
      // The pair splits B by N across the two CTAs' shared memory, so the
      // MMA's N is the width the token halves were loaded for: the full tile.
      const uint32_t idesc = idesc_i8(2 * kBlockW, p.tok_tile);
      uint32_t phase = 0;
      int tile = cluster, tcount = 0, kt = 0, buf = 0;
      uint32_t d_tmem = tmem_base;
      // Starts tile `tile` (the tcount-th of this pair): its accumulator
      // buffer must have been drained by both epilogues two tiles ago.
      const auto begin_tile = [&]() -> bool {
        buf = tcount & 1;
        d_tmem = tmem_base + buf * acc_cols;
        return tcount < 2 || mbar_wait_bounded_cl(bar_accempty(buf), ((tcount >> 1) - 1) & 1,
                                                  abort_flag, err, kErrWaitAccum, limit);
      };
      bool alive = tile < total_tiles && begin_tile();
      while (alive) {
#pragma unroll
        for (int r = 0; r < RING; ++r) {
          const uint32_t rbar = ready0 + 8u * r;
          if (!mbar_try_wait_cl(rbar, phase) &&
              !mbar_wait_bounded_cl(rbar, phase, abort_flag, err, kErrWaitUnpack, limit)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_slot = a_base + 32u * (sa_full ? r : r % SA_SMALL);
          umma_i8_ts_pair(d_tmem, a_slot, bd[r], idesc, kt != 0);
          umma_i8_ts_pair(d_tmem, a_slot + 8, bd[r] + 2, idesc, 1u);
          umma_i8_ts_pair(d_tmem, a_slot + 16, bd[r] + 4, idesc, 1u);
          umma_i8_ts_pair(d_tmem, a_slot + 24, bd[r] + 6, idesc, 1u);
          umma_commit_pair_mc(empty0 + 8u * r, 0x3);
          if (++kt == p.k_tiles) {
            umma_commit_pair_mc(bar_accfull(buf), 0x3);
            kt = 0;
            tile += n_clusters;
            ++tcount;
            if (tile >= total_tiles || !begin_tile()) {
              alive = false;
              break;
            }
          }
        }
        phase ^= 1u;
      }
      umma_commit_pair_mc(bar_drain, 0x3);
    }
    // Both CTAs: every MMA writing this CTA's TMEM has completed.
    if (lane == 0) {
      volatile int no_abort = 0;
      mbar_wait_bounded_cl(bar_drain, 0, &no_abort, err, kErrWaitDrain, limit);
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------ unpack -> own TMEM (A operand)
    const int group = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    RingPos st, at, lag;
    int step = 0;
    bool alive = true;
    for (int tile = cluster; alive && tile < total_tiles; tile += n_clusters) {
      for (int kt = 0; kt < p.k_tiles; ++kt) {
        if ((step & 1) == group) {
          bool ok = mbar_wait_bounded(bar_wfull(st.idx), st.phase, abort_flag, err, kErrWaitTma,
                                      limit);
          if (ok && leader)
            ok = mbar_wait_bounded_cl(bar_tfull(st.idx), st.phase, abort_flag, err, kErrWaitTma,
                                      limit);
          if (ok && step >= SA)
            ok = mbar_wait_bounded_cl(bar_empty(lag.idx), lag.phase, abort_flag, err,
                                      kErrWaitUnpack, limit);
          if (!warp_all(ok)) {
            alive = false;
            break;
          }
          const uint8_t* src = wpk_ring + st.idx * kWpkBytes;
          uint32_t w[16];
          if constexpr (LAYOUT == kRowMajor) {
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
          if (lane == 0) {
            if (leader) mbar_arrive(bar_ready(st.idx));
            else mbar_arrive_remote(mapa_shared(bar_ready(st.idx), 0));
          }
        }
        ++step;
        st.advance(S);
        at.advance(SA);
        if (step > SA) lag.advance(S);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int ew = warp - kEpiWarp0;
    const int half = ew >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    __half* stage = reinterpret_cast<__half*>(epi + ew * kEpiBytesPerWarp);
    float* ts = tile_scale + ew * kTokTileMax;
    int tcount = 0;
    for (int tile = cluster; tile < total_tiles; tile += n_clusters, ++tcount) {
      const TileCoord c = decode_pair_tile(p, tile, rank);
      const int buf = tcount & 1;
      if (!ACC_OUT) stage_tile_scales(ts, p.row_scale, c, lane);
      const bool ok = mbar_wait_bounded_cl(bar_accfull(buf), (tcount >> 1) & 1, abort_flag, err,
                                           kErrWaitAccum, limit);
      if (!warp_all(ok)) break;
      tc_fence_after();
      const uint32_t accempty = mapa_shared(bar_accempty(buf), 0);
      epilogue_tile<ACC_OUT>(p.seg[c.seg], c, c.n0 + quarter * 32,
                             tmem_base + lane_addr + buf * acc_cols, half, lane, stage, ts, [&] {
                               tc_fence_before();
                               __syncwarp();
                               if (lane == 0) mbar_arrive_remote(accempty);
                             });
    }
  }

  // ---- teardown: both CTAs done (incl. every remote arrival and MMA) before
  // the pair frees its TMEM.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

// ---- int8 weights: the CTA pair with both MMA operands in shared memory.
// The weights are repacked once at load (repack_int8_kernel) into int8 rows
// of 16 x code in the GEMM's K byte order (the bytes the unpack warps above
// write into TMEM), followed by the fp32 scale: int32 [N, K/4 + 4].  Then a
// step is two TMA copies per CTA (its 128 weight rows, 16 KB, and its half of
// the token tile) counted on the leader's barrier, and four SS MMAs: no
// unpack warps, no TMEM A slots (both TMEM halves hold accumulators).
constexpr int kA8Bytes = kBlockW * kBlockK;  // 16 KB of int8 weights per CTA per step
constexpr int kPairI8Warps = 2 + kEpiWarps;
constexpr int kPairI8Threads = 32 * kPairI8Warps;

__host__ __device__ constexpr int gemm_pair_i8_smem_bytes(int tok_tile) {
  return kGemmRing * (kA8Bytes + tok_tile / 2 * kBlockK) + kFixedSmem;
}
static_assert(gemm_pair_i8_smem_bytes(kTokTileMax) <= kSmemLimit, "int8 pair ring must fit");

// Packed word j (0 <= j < K/8) of weight row n -> int8 bytes 8j .. 8j + 7 of
// the repacked row (expand_nibbles_x16: even elements, then odd), and the
// row's scale word after the K bytes.  One thread per (row, word).
__global__ void repack_int8_kernel(const int32_t* __restrict__ src, int32_t n, int32_t k, int32_t row_words,
                                   int32_t layout, int32_t* __restrict__ dst) {
  const int32_t words = k / 8, dw = k / 4 + 4;
  const int64_t total = static_cast<int64_t>(n) * (words + 1);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / (words + 1);
    const int32_t j = static_cast<int32_t>(i - r * (words + 1));
    int32_t* row = dst + r * dw;
    if (j == words) {
      const int32_t sc = layout == kRowMajor ? src[r * row_words + words]
                                             : src[static_cast<int64_t>(n) * words + r];
      row[words * 2] = sc;
      row[words * 2 + 1] = 0;
      row[words * 2 + 2] = 0;
      row[words * 2 + 3] = 0;
    } else {
      const uint32_t w = static_cast<uint32_t>(
          layout == kRowMajor ? src[r * row_words + j]
                              : src[static_cast<int64_t>(j >> 1) * 2 * n + 2 * r + (j & 1)]);
      uint32_t lo, hi;
      expand_nibbles_x16(w, lo, hi);
      row[2 * j] = static_cast<int32_t>(lo);
      row[2 * j + 1] = static_cast<int32_t>(hi);
    }
  }
}

template <bool ACC_OUT>
__global__ void __launch_bounds__(kPairI8Threads, 1)
    w4a4_gemm_pair_i8_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
  const int S = p.stages;
  const int half = p.tok_tile / 2;              // token rows held by each CTA
  const int tok_bytes = half * kBlockK;         // per CTA per stage (a multiple of 1 KB)
  uint8_t* a_ring = base;                       // [S][16 KB]
  uint8_t* tok_ring = base + S * kA8Bytes;      // [S][tok_bytes]
  uint8_t* epi = tok_ring + S * tok_bytes;      // kEpiWarps x 1 KB
  float* tile_scale = reinterpret_cast<float*>(epi + kEpiWarps * kEpiBytesPerWarp);
  uint64_t* bars = reinterpret_cast<uint64_t*>(tile_scale + kEpiWarps * kTokTileMax);
  // full[s]   leader: both CTAs' weight rows and token halves of step i landed
  //           (every copy completes on the leader's barrier).
  // empty[s]  both (multicast commit): MMA(i) completed.
  // accfull/accempty[2]: accumulator handshake (accempty lives in the leader).
  const auto bar_full = [&](int s) { return smem_addr(bars + s); };
  const auto bar_empty = [&](int s) { return smem_addr(bars + kMaxStages + s); };
  const auto bar_accfull = [&](int b) { return smem_addr(bars + 2 * kMaxStages + b); };
  const auto bar_accempty = [&](int b) { return smem_addr(bars + 2 * kMaxStages + 2 + b); };
  const uint32_t bar_drain = smem_addr(bars + 2 * kMaxStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned* err = &g_w4a4_device_error;
  const uint64_t limit = p.wait_limit_ns;
  const int total_tiles = p.n_tok_tiles * p.w_tiles;
  const int acc_cols = p.tok_tile;

  constexpr int RING = kGemmRing;
  if (S != RING || 2 * p.tok_tile > kPairTmemCols || p.tok_tile > kTokTileMax || p.k_tiles < 1 ||
      (p.tok_tile & 15)) {
    if (threadIdx.x == 0) atomicOr(&g_w4a4_device_error, kErrBadParams);
    return;
  }

  pdl_launch_dependents();
  pdl_wait();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_full(s), 1);   // leader: its producer's expect_tx of both CTAs' bytes
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_accfull(b), 1);
      mbar_init(bar_accempty(b), 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tmap_tok);
    for (int s = 0; s < p.n_seg; ++s) tma_prefetch_desc(&p.seg[s].tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), kPairTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (lane 0, both CTAs)
    if (lane == 0) {
      RingPos st;
      int issued = 0;
      bool alive = true;
      for (int tile = cluster; alive && tile < total_tiles; tile += n_clusters) {
        const TileCoord c = decode_pair_tile(p, tile, rank);
        const CUtensorMap* wmap = &p.seg[c.seg].tmap_w;
        for (int kt = 0; kt < p.k_tiles; ++kt) {
          if (issued >= S &&
              !mbar_wait_bounded_cl(bar_empty(st.idx), st.phase ^ 1u, abort_flag, err,
                                    kErrWaitEmpty, limit)) {
            alive = false;
            break;
          }
          const uint32_t full = bar_full(st.idx);
          if (leader) mbar_arrive_expect_tx(full, static_cast<uint32_t>(2 * (kA8Bytes + tok_bytes)));
          tma_load_2d_pair(smem_addr(a_ring + st.idx * kA8Bytes), wmap, kt * kBlockK, c.n0, full);
          tma_load_2d_pair(smem_addr(tok_ring + st.idx * tok_bytes), &p.tmap_tok, kt * kBlockK,
                           static_cast<int>(c.t0) + static_cast<int>(rank) * half, full);
          st.advance(S);
          ++issued;
        }
      }
      // Drain (leader): every copy of both CTAs completes on the leader's
      // full barriers; the exit cluster barrier keeps the peer resident.
      if (leader)
        for (int i = 0; i < S && i < issued; ++i) {
          const int last = i + ((issued - 1 - i) / S) * S;
          volatile int no_abort = 0;
          mbar_wait_bounded_cl(bar_full(i), (last / S) & 1, &no_abort, err, kErrWaitDrain, limit);
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader, whole warp)
    // Warp-uniform waits; one elected lane issues the four pair MMAs of a
    // step and multicasts each commit to both CTAs.
    if (leader) {
      const bool issuer = elect_one();
      const uint64_t adesc0 = smem_desc_sw128(smem_addr(a_ring));
      const uint64_t bdesc0 = smem_desc_sw128(smem_addr(tok_ring));
      const uint64_t astep = static_cast<uint64_t>(kA8Bytes >> 4);
      const uint64_t bstep = static_cast<uint64_t>(tok_bytes >> 4);
      const uint32_t full0 = bar_full(0), empty0 = bar_empty(0);
      const uint32_t idesc = idesc_i8(2 * kBlockW, p.tok_tile);
      uint32_t phase = 0;
      int tile = cluster, tcount = 0, kt = 0, buf = 0;
      uint32_t d_tmem = tmem_base;
      const auto begin_tile = [&]() -> bool {
        buf = tcount & 1;
        d_tmem = tmem_base + buf * acc_cols;
        return tcount < 2 || warp_all(mbar_wait_bounded_cl(bar_accempty(buf), ((tcount >> 1) - 1) & 1,
                                                           abort_flag, err, kErrWaitAccum, limit));
      };
      bool alive = tile < total_tiles && begin_tile();
      while (alive) {
#pragma unroll
        for (int r = 0; r < RING; ++r) {
          const uint32_t fbar = full0 + 8u * r;
          const bool ok = mbar_try_wait_cl(fbar, phase) ||
                          mbar_wait_bounded_cl(fbar, phase, abort_flag, err, kErrWaitTma, limit);
          if (!warp_all(ok)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = adesc0 + r * astep, bd = bdesc0 + r * bstep;
          if (issuer) {
            umma_i8_ss_pair(d_tmem, ad, bd, idesc, kt != 0);
            umma_i8_ss_pair(d_tmem, ad + 2, bd + 2, idesc, 1u);
            umma_i8_ss_pair(d_tmem, ad + 4, bd + 4, idesc, 1u);
            umma_i8_ss_pair(d_tmem, ad + 6, bd + 6, idesc, 1u);
            umma_commit_pair_mc(empty0 + 8u * r, 0x3);
          }
          __syncwarp();
          if (++kt == p.k_tiles) {
            if (issuer) umma_commit_pair_mc(bar_accfull(buf), 0x3);
            __syncwarp();
            kt = 0;
            tile += n_clusters;
            ++tcount;
            if (tile >= total_tiles || !begin_tile()) {
              alive = false;
              break;
            }
          }
        }
        phase ^= 1u;
      }
      if (issuer) umma_commit_pair_mc(bar_drain, 0x3);
      __syncwarp();
    }
    // Both CTAs: every MMA writing this CTA's TMEM has completed.
    if (lane == 0) {
      volatile int no_abort = 0;
      mbar_wait_bounded_cl(bar_drain, 0, &no_abort, err, kErrWaitDrain, limit);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 2-9, both CTAs)
    const int quarter = warp & 3;
    const int ew = warp - 2;
    const int half_sel = ew >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    __half* stage = reinterpret_cast<__half*>(epi + ew * kEpiBytesPerWarp);
    float* ts = tile_scale + ew * kTokTileMax;
    int tcount = 0;
    for (int tile = cluster; tile < total_tiles; tile += n_clusters, ++tcount) {
      const TileCoord c = decode_pair_tile(p, tile, rank);
      const int buf = tcount & 1;
      if (!ACC_OUT) stage_tile_scales(ts, p.row_scale, c, lane);
      const bool ok = mbar_wait_bounded_cl(bar_accfull(buf), (tcount >> 1) & 1, abort_flag, err,
                                           kErrWaitAccum, limit);
      if (!warp_all(ok)) break;
      tc_fence_after();
      const uint32_t accempty = mapa_shared(bar_accempty(buf), 0);
      epilogue_tile<ACC_OUT>(p.seg[c.seg], c, c.n0 + quarter * 32,
                             tmem_base + lane_addr + buf * acc_cols, half_sel, lane, stage, ts, [&] {
                               tc_fence_before();
                               __syncwarp();
                               if (lane == 0) mbar_arrive_remote(accempty);
                             });
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

}  // namespace w4a4

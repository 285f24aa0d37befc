// Prefix attention of the Gemma-2B prefix LM on the sm_100a tensor cores
// (tcgen05.mma kind::f16, fp32 accumulators in TMEM).
//
// Replaces the reference's eager attention over the prefix
// (pi05_fast/w4a4/apply.py:170-188: transformers' eager_attention_forward,
// 8 query heads sharing 1 key/value head, head_dim 256) with the padding mask
// of a bidirectional prefix: query i sees key j iff both are real tokens; a
// padded query sees no key, so its softmax is uniform over all L keys (the
// result of the all-masked row in the reference's fp32 softmax).
//
// Design (a cluster of two CTAs per 128 (token, head) rows of one
// observation, each taking about half of the key blocks):
//  * the CTA's rows are `128 / heads` consecutive tokens x all heads, so every
//    row shares the one key/value head: Q is one 64 KB TMA load (4-D map
//    {d, head, token, batch}, 128-byte swizzle), K and V^T stream in blocks
//    of 64 keys through a two-stage ring (32 KB each);
//  * warp 1 issues S = Q K^T (M = 128, N = 64, 16 MMAs of K = 16 over d) into
//    one of two TMEM score buffers, and O += P V^T (M = 128, N = 256, 4 MMAs of
//    K = 16 keys) with P read from TMEM (the A operand of the TS form);
//  * warps 2-5 (one per TMEM lane quarter, thread = row) run an online
//    softmax in one pass: p = exp2(s - m) as fp16 into TMEM for the PV MMA,
//    with the running max m moved (and O rescaled in TMEM) only when a block
//    exceeds it by more than 2^8; then they scale O by 1 / sum and store fp16
//    rows;
//  * key blocks past the last real key are skipped for tiles of real queries;
//    for a padded query they are "tail" blocks, P V only with a constant P;
//  * the pair exchanges halves of O (with each row's m and l) through
//    distributed shared memory and each CTA finishes 128 output columns;
//  * every wait is bounded (the device error word, an abort flag, teardown
//    that drains its copies and MMAs and frees TMEM).
// Softmax is base 2: s2 = acc * (scale * log2 e), p = exp2(s2 - m).
#pragma once

#include "common.cuh"
#include "layer.cuh"
#include "quant.cuh"

namespace w4a4 {

constexpr int kAttnRows = 128;            // UMMA M: (token, head) rows of a CTA
constexpr int kAttnHeadDim = 256;
constexpr int kAttnKeyBlock = 64;         // keys per pipeline step (UMMA N of S)
constexpr int kAttnMaxKeys = 4096;        // longest prefix (key-mask words in shared memory)
constexpr int kAttnSlices = kAttnHeadDim / 64;                     // 128-byte rows of 64 fp16
constexpr int kAttnQBytes = kAttnRows * kAttnHeadDim * 2;          // 64 KB
constexpr int kAttnKBytes = kAttnKeyBlock * kAttnHeadDim * 2;      // 32 KB
constexpr int kAttnVBytes = kAttnHeadDim * kAttnKeyBlock * 2;      // 32 KB
constexpr int kAttnStages = 2;
constexpr int kAttnThreads = 192;                                  // 6 warps
constexpr int kAttnNumBars = 1 + 4 * kAttnStages + 4 * 2 + 4;      // q, k/v full/empty, s/p full/free, o, p tail, pair
// The pair's exchange (in the idle K/V ring once both CTAs' MMAs are done):
// per row 128 fp32 of O (the columns the partner finishes, 16-byte chunk c
// of row r at chunk c ^ (r & 31)) and a 16-byte (m, l) record.
constexpr int kAttnXchgO = kAttnRows * (kAttnHeadDim / 2) * 4;        // 64 KB
constexpr int kAttnXchgBytes = kAttnXchgO + kAttnRows * 16;
// The output staging (two 64-column slices of 128 rows, 128-byte swizzle, the
// TMA store's layout) in the ring after the exchange's receive region and
// send record.
constexpr int kAttnOutStage = 68 * 1024;
static_assert(kAttnOutStage >= kAttnXchgBytes + kAttnRows * 16 && kAttnOutStage % 1024 == 0 &&
                  kAttnOutStage + 2 * kAttnRows * 128 <= kAttnStages * (kAttnKBytes + kAttnVBytes),
              "attention smem map");
constexpr int kAttnSmem = kAttnQBytes + kAttnStages * (kAttnKBytes + kAttnVBytes) +
                          kAttnNumBars * 8 + 16 + (kAttnMaxKeys / 64) * 8 + 1024;
// TMEM columns: O [0, 256), S buffers at 256 and 320 (64 each), P buffers at
// 384 and 416 (32 columns: 64 fp16 per row), the tail blocks' constant P at
// 448.
constexpr uint32_t kAttnTmemCols = 512;
constexpr uint32_t kAttnOCol = 0, kAttnSCol = 256, kAttnPCol = 384, kAttnPTailCol = 448;

struct alignas(64) AttnParams {
  CUtensorMap tmap_q;   // fp16 {256 d, heads, L, B}, box {64, heads, 128 / heads, 1}, SW128
  CUtensorMap tmap_k;   // fp16 {256 d, L, B}, box {64, 64, 1}, SW128
  CUtensorMap tmap_vt;  // fp16 {L, 256 d, B} (V transposed per observation), box {64, 256, 1}, SW128
  CUtensorMap tmap_o;   // fp16 output, the same 4-D shape and box as tmap_q
  const uint8_t* key_valid;  // [B, L]: 1 = real token
  const int* kv_len;         // [B]: keys past this index are all padding
  __half* out;               // [B * L, ldo], row (b, t) columns head * 256 + d
  long long ldo;
  int seq;
  int heads;
  float scale_log2;          // head_dim^-0.5 * log2(e)
  unsigned long long wait_limit_ns;
};

// Instruction descriptor of tcgen05.mma.kind::f16: D = f32, A and B fp16,
// both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4)                                  // D format: F32
         | (static_cast<uint32_t>(n >> 3) << 17)    // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);   // M >> 4
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16 x fp16 -> fp32, K = 16.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, fp16 x fp16 -> fp32, K = 16: A is
// M rows in TMEM lanes, 16 fp16 in 8 consecutive 32-bit columns.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2^x with the MUFU instruction (ex2.approx.ftz.f32: relative error about
// 2^-22, flushes subnormal results; exp2(-inf) = +0).  The probabilities it
// produces are rounded to fp16 for the P V product, far coarser.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 16 consecutive 32-bit columns from registers.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ uint32_t pack_half2_bits(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    prefix_attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t attn_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(attn_smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_smem = base;                                   // [4 slices][128 rows][128 B]
  uint8_t* k_ring = base + kAttnQBytes;                     // [2][4 slices][64 rows][128 B]
  uint8_t* v_ring = k_ring + kAttnStages * kAttnKBytes;     // [2][256 rows][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(v_ring + kAttnStages * kAttnVBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kAttnNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* nkb_slot = reinterpret_cast<int*>(tmem_slot + 2);  // [0]: real-key blocks, [1]: all blocks
  unsigned long long* kmask = reinterpret_cast<unsigned long long*>(tmem_slot + 4);  // 8-byte aligned

  const auto bar_q = [&] { return smem_addr(bars); };
  const auto bar_kfull = [&](int s) { return smem_addr(bars + 1 + s); };
  const auto bar_kempty = [&](int s) { return smem_addr(bars + 3 + s); };
  const auto bar_vfull = [&](int s) { return smem_addr(bars + 5 + s); };
  const auto bar_vempty = [&](int s) { return smem_addr(bars + 7 + s); };
  const auto bar_sfull = [&](int s) { return smem_addr(bars + 9 + s); };
  const auto bar_sfree = [&](int s) { return smem_addr(bars + 11 + s); };
  const auto bar_pfull = [&](int s) { return smem_addr(bars + 13 + s); };
  const auto bar_pfree = [&](int s) { return smem_addr(bars + 15 + s); };
  const uint32_t bar_o = smem_addr(bars + 17);
  const uint32_t bar_ptail = smem_addr(bars + 18);
  const uint32_t bar_recv = smem_addr(bars + 19);   // the partner's O half and (m, l) landed
  const uint32_t bar_rdy = smem_addr(bars + 20);    // the partner's ring is free to receive

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int L = p.seq;
  const int tpt = kAttnRows / p.heads;  // tokens per tile
  // a cluster of two CTAs per tile: rank r takes about half of the tile's
  // key blocks, then the two exchange halves of O and each finishes 128 of
  // the 256 output columns
  const uint32_t rank = cluster_ctarank(), peer = rank ^ 1u;
  const int t0 = (blockIdx.x >> 1) * tpt;
  unsigned* err = &g_w4a4_device_error;
  const uint64_t limit = p.wait_limit_ns;

  if (L < 1 || L > kAttnMaxKeys || p.heads < 1 || kAttnRows % p.heads != 0) {
    if (threadIdx.x == 0) atomicOr(&g_w4a4_device_error, kErrBadParams);
    return;
  }
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    mbar_init(bar_q(), 1);
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(bar_kfull(s), 1);
      mbar_init(bar_kempty(s), 1);
      mbar_init(bar_vfull(s), 1);
      mbar_init(bar_vempty(s), 1);
      mbar_init(bar_sfull(s), 1);
      mbar_init(bar_sfree(s), 4);
      mbar_init(bar_pfull(s), 4);
      mbar_init(bar_pfree(s), 1);
    }
    mbar_init(bar_o, 1);
    mbar_init(bar_ptail, 4);
    mbar_init(bar_recv, 1);
    mbar_init(bar_rdy, 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tmap_q);
    tma_prefetch_desc(&p.tmap_k);
    tma_prefetch_desc(&p.tmap_vt);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), kAttnTmemCols);
    tmem_relinquish();
  }
  pdl_wait();  // q, k, v and the masks are earlier kernels' outputs
  const uint8_t* kv_row = p.key_valid + static_cast<long long>(b) * L;
  // Key blocks to visit.  Real query rows see the keys up to the last real
  // one: blocks [0, nkr) run Q K^T and the softmax.  A padded (or
  // past-the-end) query row's softmax is uniform over all L keys (p = 1 for
  // every key < L): when the tile has one, blocks [nkr, nka) up to L are
  // "tail" blocks, P V only, with a constant P (1 for padded rows, 0 for real
  // ones, whose keys there are all padding).  One load per lane (tpt <= 128
  // tokens: up to 4 per lane), then two votes.
  if (warp == 0) {
    bool pad_row = false, real_row = false;
#pragma unroll
    for (int i = 0; i < kAttnRows / 32; ++i) {
      const int t = t0 + lane + 32 * i;
      if (lane + 32 * i < tpt) {
        const bool real = t < L && kv_row[t];
        pad_row |= !real;
        real_row |= real;
      }
    }
    const int kv_len = p.kv_len[b];
    pad_row = __any_sync(0xffffffffu, pad_row);
    real_row = __any_sync(0xffffffffu, real_row);
    const int nkr = real_row ? (max(0, min(L, kv_len)) + kAttnKeyBlock - 1) / kAttnKeyBlock : 0;
    if (lane == 0) {
      nkb_slot[0] = nkr;
      nkb_slot[1] = pad_row ? (L + kAttnKeyBlock - 1) / kAttnKeyBlock : nkr;
    }
  }
  // 64-bit masks of the real keys of every block (warps 2-5; the loads of a
  // warp's blocks are independent and issued together)
  if (warp >= 2) {
    const int nblk = (L + kAttnKeyBlock - 1) / kAttnKeyBlock;
#pragma unroll 4
    for (int kb = warp - 2; kb < nblk; kb += 4) {
      const int j0 = kb * kAttnKeyBlock + lane, j1 = j0 + 32;
      const bool v0 = j0 < L && kv_row[j0];
      const bool v1 = j1 < L && kv_row[j1];
      const unsigned lo = __ballot_sync(0xffffffffu, v0), hi = __ballot_sync(0xffffffffu, v1);
      if (lane == 0) kmask[kb] = static_cast<unsigned long long>(hi) << 32 | lo;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nkb = nkb_slot[0];   // the tile's blocks with Q K^T and the softmax
  const int nka = nkb_slot[1];   // all of the tile's blocks (nka >= nkb)
  // This CTA's blocks: nn normal ones from n0, then nt tail ones from tb;
  // local step i < n is block kb_of(i).
  const int h0 = (nkb + 1) / 2, th = nkb + (nka - nkb + 1) / 2;
  const int n0 = rank ? h0 : 0, nn = rank ? nkb - h0 : h0;
  const int tb = rank ? th : nkb, nt = rank ? nka - th : th - nkb;
  const int n = nn + nt;
  const auto kb_of = [&](int i) { return i < nn ? n0 + i : tb + (i - nn); };

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (lane 0)
    if (lane == 0 && n > 0) {
      if (nn > 0) {
        mbar_arrive_expect_tx(bar_q(), kAttnQBytes);
        for (int s = 0; s < kAttnSlices; ++s)
          tma_load_4d(smem_addr(q_smem + s * (kAttnQBytes / kAttnSlices)), &p.tmap_q, 64 * s, 0, t0, b,
                      bar_q());
      }
      int nk = 0, nv = 0;
      // step i (block kb): K (normal blocks) into k slot i % 2, V^T into v slot i % 2
      for (int i = 0; i < n; ++i) {
        const int kb = kb_of(i), slot = i & 1;
        if (i < nn) {
          if (i >= kAttnStages &&
              !mbar_wait_spin(bar_kempty(slot), ((i >> 1) - 1) & 1, abort_flag, err, kErrWaitEmpty, limit))
            break;
          mbar_arrive_expect_tx(bar_kfull(slot), kAttnKBytes);
          for (int s = 0; s < kAttnSlices; ++s)
            tma_load_3d(smem_addr(k_ring + slot * kAttnKBytes + s * (kAttnKBytes / kAttnSlices)), &p.tmap_k,
                        64 * s, kb * kAttnKeyBlock, b, bar_kfull(slot));
          ++nk;
        }
        if (i >= kAttnStages &&
            !mbar_wait_spin(bar_vempty(slot), ((i >> 1) - 1) & 1, abort_flag, err, kErrWaitEmpty, limit))
          break;
        mbar_arrive_expect_tx(bar_vfull(slot), kAttnVBytes);
        tma_load_3d(smem_addr(v_ring + slot * kAttnVBytes), &p.tmap_vt, kb * kAttnKeyBlock, 0, b,
                    bar_vfull(slot));
        ++nv;
      }
      // Drain: no copy may still be in flight at exit.
      volatile int no_abort = 0;
      if (nn > 0) mbar_wait_bounded(bar_q(), 0, &no_abort, err, kErrWaitDrain, limit);
      for (int i = 0; i < kAttnStages && i < nk; ++i) {
        const int last = i + ((nk - 1 - i) / kAttnStages) * kAttnStages;
        mbar_wait_bounded(bar_kfull(i), (last / kAttnStages) & 1, &no_abort, err, kErrWaitDrain, limit);
      }
      for (int i = 0; i < kAttnStages && i < nv; ++i) {
        const int last = i + ((nv - 1 - i) / kAttnStages) * kAttnStages;
        mbar_wait_bounded(bar_vfull(i), (last / kAttnStages) & 1, &no_abort, err, kErrWaitDrain, limit);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (one elected lane)
    const bool issuer = elect_one();
    const uint32_t idesc_s = idesc_f16(kAttnRows, kAttnKeyBlock);
    const uint32_t idesc_o = idesc_f16(kAttnRows, kAttnHeadDim);
    const uint64_t qdesc = smem_desc_sw128(smem_addr(q_smem));
    bool alive = n > 0 &&
                 (nn == 0 || warp_all(mbar_wait_bounded(bar_q(), 0, abort_flag, err, kErrWaitTma, limit)));
    // S(i) = Q K(kb_of(i))^T into score buffer i % 2
    const auto issue_s = [&](int i) -> bool {
      const int slot = i & 1;
      bool ok = mbar_wait_spin(bar_kfull(slot), (i >> 1) & 1, abort_flag, err, kErrWaitTma, limit);
      if (ok && i >= 2)
        ok = mbar_wait_spin(bar_sfree(slot), ((i >> 1) - 1) & 1, abort_flag, err, kErrWaitAccum, limit);
      if (!warp_all(ok)) return false;
      tc_fence_after();
      const uint64_t kdesc = smem_desc_sw128(smem_addr(k_ring + slot * kAttnKBytes));
      // warp-uniform loop, one lane issues (a loop inside a one-lane branch
      // issues several times slower)
#pragma unroll
      for (int kk = 0; kk < kAttnHeadDim / 16; ++kk) {
        const uint64_t off = static_cast<uint64_t>((kk & 3) * 2);
        if (issuer)
          umma_f16_ss(tmem_base + kAttnSCol + slot * kAttnKeyBlock,
                      qdesc + static_cast<uint64_t>((kk >> 2) * (kAttnQBytes / kAttnSlices) >> 4) + off,
                      kdesc + static_cast<uint64_t>((kk >> 2) * (kAttnKBytes / kAttnSlices) >> 4) + off,
                      idesc_s, kk > 0);
      }
      if (issuer) {
        umma_commit(bar_kempty(slot));
        umma_commit(bar_sfull(slot));
      }
      __syncwarp();
      return true;
    };
    if (alive && nn > 0) alive = issue_s(0);
    for (int i = 0; alive && i < n; ++i) {
      if (i + 1 < nn && !(alive = issue_s(i + 1))) break;
      const int slot = i & 1;
      const bool tail = i >= nn;
      bool ok = mbar_wait_spin(bar_vfull(slot), (i >> 1) & 1, abort_flag, err, kErrWaitTma, limit);
      if (ok)
        ok = tail ? mbar_wait_spin(bar_ptail, 0, abort_flag, err, kErrWaitUnpack, limit)
                  : mbar_wait_spin(bar_pfull(slot), (i >> 1) & 1, abort_flag, err, kErrWaitUnpack, limit);
      if (!warp_all(ok)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint64_t vdesc = smem_desc_sw128(smem_addr(v_ring + slot * kAttnVBytes));
      const uint32_t pcol = tail ? kAttnPTailCol : kAttnPCol + slot * 32;
#pragma unroll
      for (int kk = 0; kk < kAttnKeyBlock / 16; ++kk)
        if (issuer)
          umma_f16_ts(tmem_base + kAttnOCol, tmem_base + pcol + 8 * kk,
                      vdesc + static_cast<uint64_t>(kk * 2), idesc_o, (i | kk) != 0);
      if (issuer) {
        umma_commit(bar_vempty(slot));
        if (!tail) umma_commit(bar_pfree(slot));
      }
      __syncwarp();
    }
    // Every MMA of this CTA has completed once this commit arrives (also
    // after an abort: the epilogue's bounded wait then gives up or passes).
    if (issuer && n > 0) umma_commit(bar_o);
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax + epilogue (warps 2-5)
    // Online softmax in one pass, base 2 (s2 = acc * scale * log2 e): the
    // row's running max m only moves up when a block's max exceeds it by
    // more than kRescaleLog2, and then O (TMEM) and l are rescaled by
    // exp2(m_old - m_new) once the previous P V MMA has completed; otherwise
    // p = exp2(s2 - m) <= 2^kRescaleLog2 is kept unnormalised (fp16 holds it).
    constexpr float kRescaleLog2 = 8.f;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;                // this thread's row (TMEM lane)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int tok = t0 + r / p.heads, head = r % p.heads;
    const bool q_real = tok < L && p.key_valid[static_cast<long long>(b) * L + tok];
    const float scale = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool alive = n > 0;
    if (alive && nt > 0) {
      // the tail blocks' P: 1 (fp16) for a padded row, 0 for a real one
      uint32_t pw[32];
      const uint32_t one = q_real ? 0u : 0x3C003C00u;
#pragma unroll
      for (int c = 0; c < 32; ++c) pw[c] = one;
      tmem_st_32x32b_x32(tmem_base + lane_addr + kAttnPTailCol, pw);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_ptail);
    }
    for (int i = 0; alive && i < nn; ++i) {
      const int kb = n0 + i, slot = i & 1;
      if (!warp_all(mbar_wait_spin(bar_sfull(slot), (i >> 1) & 1, abort_flag, err, kErrWaitAccum, limit))) {
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t raw[64];
      {
        const uint32_t t = tmem_base + lane_addr + kAttnSCol + slot * kAttnKeyBlock;
        tmem_ld_32x32b_x16(t, *reinterpret_cast<uint32_t(*)[16]>(&raw[0]));
        tmem_ld_32x32b_x16(t + 16, *reinterpret_cast<uint32_t(*)[16]>(&raw[16]));
        tmem_ld_32x32b_x16(t + 32, *reinterpret_cast<uint32_t(*)[16]>(&raw[32]));
        tmem_ld_32x32b_x16(t + 48, *reinterpret_cast<uint32_t(*)[16]>(&raw[48]));
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree(slot));
      // real query: its real keys; padded query: every key < L, score 0
      const int j0 = kb * kAttnKeyBlock;
      const unsigned long long vm =
          q_real ? kmask[kb]
                 : (L - j0 >= 64 ? ~0ull : ((1ull << (L - j0)) - 1ull));
      const unsigned vlo = static_cast<unsigned>(vm), vhi = static_cast<unsigned>(vm >> 32);
      float bm4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // 4 chains: ILP
      if (q_real && vm == ~0ull) {  // a real row, every key of the block real
#pragma unroll
        for (int c = 0; c < 64; ++c) bm4[c & 3] = fmaxf(bm4[c & 3], __uint_as_float(raw[c]));
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float v = q_real ? __uint_as_float(raw[c]) : 0.f;
          const bool ok = ((c < 32 ? vlo >> c : vhi >> (c - 32)) & 1u) != 0;
          const float mv = ok ? v : -INFINITY;
          raw[c] = __float_as_uint(mv);
          bm4[c & 3] = fmaxf(bm4[c & 3], mv);
        }
      }
      // scale > 0: the max of the scaled scores
      const float bmax = fmaxf(fmaxf(bm4[0], bm4[1]), fmaxf(bm4[2], bm4[3])) * scale;
      float f = 1.f;  // rescale of the previous O and l
      const bool grow = bmax > m + kRescaleLog2;  // false while the block is all masked
      if (grow) {
        f = m == -INFINITY ? 0.f : ex2_approx(m - bmax);
        m = bmax;
        l *= f;
      }
      if (__any_sync(0xffffffffu, grow && f != 0.f) && i >= 1) {
        // O holds P V of earlier blocks: wait for the last of them, rescale
        // this warp's rows (whole-warp TMEM access; others multiply by 1)
        if (!warp_all(mbar_wait_spin(bar_pfree((i - 1) & 1), ((i - 1) >> 1) & 1, abort_flag, err,
                                        kErrWaitAccum, limit))) {
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < kAttnHeadDim; c0 += 16) {
          uint32_t o[16];
          const uint32_t t = tmem_base + lane_addr + kAttnOCol + c0;
          tmem_ld_32x32b_x16(t, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st_32x32b_x16(t, o);
        }
        tmem_st_wait();
      }
      // p = exp2(s2 - m) as fp16 pairs, l += sum p (masked: exp2(-inf) = 0)
      const float nm = m == -INFINITY ? 0.f : -m;
      uint32_t pw[32];
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = ex2_approx(__fmaf_rn(__uint_as_float(raw[2 * c]), scale, nm));
        const float p1 = ex2_approx(__fmaf_rn(__uint_as_float(raw[2 * c + 1]), scale, nm));
        s4[c & 3] += p0 + p1;
        pw[c] = pack_half2_bits(p0, p1);
      }
      l += (s4[0] + s4[1]) + (s4[2] + s4[3]);
      if (i >= 2 && !warp_all(mbar_wait_spin(bar_pfree(slot), ((i >> 1) - 1) & 1, abort_flag, err,
                                                 kErrWaitAccum, limit))) {
        alive = false;
        break;
      }
      tc_fence_after();
      tmem_st_32x32b_x32(tmem_base + lane_addr + kAttnPCol + slot * 32, pw);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pfull(slot));
    }
    // ---- epilogue: the pair combines its two halves of the key range.  Once
    // this CTA's MMAs are done its K/V ring is idle: it tells the partner,
    // stages the partner's 128 columns of O with its (m, l) in its idle Q
    // buffer, and once the partner's ring is idle sends them there with bulk
    // copies (completion counted on the partner's bar_recv); then it finishes
    // its own 128 columns from its O and the partner's:  O = O_0 2^(m_0 - m) + O_1 2^(m_1 - m), m = max(m_0, m_1),
    // likewise l.  A padded row (p = 1 everywhere, in both halves) adds the
    // halves and divides by L.  A CTA without blocks contributes O = 0.
    const bool have = n > 0;
    bool ok = !have || (alive && warp_all(mbar_wait_bounded(bar_o, 0, abort_flag, err, kErrWaitAccum, limit)));
    tc_fence_after();
    if (warp == 2 && lane == 0) mbar_arrive_expect_tx(bar_recv, kAttnXchgBytes);
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(mapa_shared(bar_rdy, peer));
    const uint32_t ocol = tmem_base + lane_addr + kAttnOCol;
    // this CTA's send staging: the partner's 128 columns of O in the idle Q
    // buffer (same swizzled layout as the receive buffer), (m, l) after the
    // receive region of the ring
    float4* send = reinterpret_cast<float4*>(q_smem) + r * 32;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      uint32_t o[16];
      if (have && ok) {
        tmem_ld_32x32b_x16(ocol + peer * 128 + 16 * cc, o);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        send[(4 * cc + j) ^ (r & 31)] = make_float4(__uint_as_float(o[4 * j]), __uint_as_float(o[4 * j + 1]),
                                                    __uint_as_float(o[4 * j + 2]), __uint_as_float(o[4 * j + 3]));
    }
    reinterpret_cast<float4*>(k_ring + kAttnXchgBytes)[r] = make_float4(m, l, 0.f, 0.f);
    fence_proxy_async_smem();  // the bulk copy reads these through the async proxy
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 softmax warps
    if (warp == 2) {
      // one thread sends both blocks once the partner's ring is free
      bool sent = ok && mbar_wait_spin(bar_rdy, 0, abort_flag, err, kErrWaitAccum, limit);
      if (sent && lane == 0) {
        const uint32_t dst = mapa_shared(smem_addr(k_ring), peer), dst_bar = mapa_shared(bar_recv, peer);
        bulk_copy_s2cluster(dst, smem_addr(q_smem), kAttnXchgO, dst_bar);
        bulk_copy_s2cluster(dst + kAttnXchgO, smem_addr(k_ring + kAttnXchgBytes), kAttnRows * 16, dst_bar);
      }
      __syncwarp();
    }
    ok = warp_all(ok && mbar_wait_spin(bar_recv, 0, abort_flag, err, kErrWaitAccum, limit));
    if (ok) {
      const float4 ml = *reinterpret_cast<const float4*>(k_ring + kAttnXchgO + r * 16);
      const float mp = ml.x, lp = ml.y;
      float fo = 1.f, fp = 1.f, lt = static_cast<float>(L);
      if (q_real) {
        const float mm = fmaxf(m, mp);
        fo = m == -INFINITY ? 0.f : ex2_approx(m - mm);
        fp = mp == -INFINITY ? 0.f : ex2_approx(mp - mm);
        lt = l * fo + lp * fp;
      }
      const float inv = lt > 0.f ? 1.0f / lt : 0.f;
      const float so = fo * inv, sp = fp * inv;
      const float* recv = reinterpret_cast<const float*>(k_ring) + r * 128;
      uint8_t* stage = k_ring + kAttnOutStage + r * 128;  // + slice * 16 KB, chunk c at c ^ (r & 7)
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint32_t o[16];
        if (have) {
          tmem_ld_32x32b_x16(ocol + rank * 128 + 16 * cc, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = 0u;
        }
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = 4 * cc + j;
          const float4 q = *reinterpret_cast<const float4*>(recv + ((c ^ (r & 31)) << 2));
          w[2 * j] = pack_half2_bits(__uint_as_float(o[4 * j]) * so + q.x * sp,
                                     __uint_as_float(o[4 * j + 1]) * so + q.y * sp);
          w[2 * j + 1] = pack_half2_bits(__uint_as_float(o[4 * j + 2]) * so + q.z * sp,
                                         __uint_as_float(o[4 * j + 3]) * so + q.w * sp);
        }
        // 16 columns = 2 chunks of 8 fp16 in slice cc / 4
        const int slice = cc >> 2, c0 = 2 * (cc & 3);
        uint8_t* srow = stage + slice * (kAttnRows * 128);
        *reinterpret_cast<uint4*>(srow + ((c0 ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(srow + (((c0 + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
    // one thread stores the two slices (rows past L are clipped by the TMA)
    fence_proxy_async_smem();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (ok && warp == 2 && lane == 0) {
      for (int sl = 0; sl < 2; ++sl)
        tma_store_4d(&p.tmap_o, smem_addr(k_ring + kAttnOutStage + sl * (kAttnRows * 128)),
                     static_cast<int>(rank) * 128 + 64 * sl, 0, t0, b);
      bulk_commit_group();
      bulk_wait_group0();
    }
  }

  // ---- teardown: every MMA has completed (bar_o, or the issuer's last
  // commits when it gave up) before TMEM is freed
  if (warp == 1 && n > 0) {
    volatile int no_abort = 0;
    mbar_wait_bounded(bar_o, 0, &no_abort, err, kErrWaitDrain, limit);
  }
  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may still write into its ring
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttnTmemCols);
  }
}

// The attention's inputs in one launch.  CTA (x, b, z) covers tokens
// [16 x, 16 x + 16) of observation b; z = 0: V [B * L, ldv] (rows of 256)
// -> V^T per observation [B][256][ldt] (the PV MMA's B operand must be
// K-major: keys contiguous; keys in [seq, ldt) written as zeros) and, when
// cos_t is not null, RoPE of k into k_out (which may equal k); z >= 1 (only
// with cos_t): RoPE of q in place for heads [2 (z - 1), 2 z) -- a grid wide
// enough that the 3.2 MB of q at a 776-token prefix is not latency bound.
constexpr int kPrepTokens = 16;
constexpr int kPrepHeadsPerSlice = 2;
__global__ void __launch_bounds__(256) attn_prep_kernel(__half* q, long long ldq, const __half* k, long long ldk,
                                                        __half* k_out, long long ldko,
                                                        const __half* __restrict__ v, long long ldv,
                                                        __half* __restrict__ vt, long long ldt,
                                                        const __half* __restrict__ cos_t,
                                                        const __half* __restrict__ sin_t, int seq, int heads) {
  __shared__ __align__(16) __half tile[kPrepTokens][kAttnHeadDim + 8];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y, j0 = blockIdx.x * kPrepTokens;
  const int t = threadIdx.x;
  const long long row0 = static_cast<long long>(b) * seq + j0;
  if (blockIdx.z > 0) {
    // q: 16 rows x 2 heads x 16 vectors of 8 pairs, two per thread, loads first
    const int h0 = kPrepHeadsPerSlice * (blockIdx.z - 1);
    uint4 a[2], bb[2], ca[2], cb[2], sa[2], sb[2];
    bool ok[2];
    __half* qr[2];
    int dd[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = t + 256 * u;
      const int j = i >> 5, head = h0 + ((i >> 4) & 1), d = 8 * (i & 15);
      ok[u] = j0 + j < seq && head < heads;
      dd[u] = d;
      if (!ok[u]) continue;
      const long long row = row0 + j;
      qr[u] = q + row * ldq + head * kAttnHeadDim;
      a[u] = *reinterpret_cast<const uint4*>(qr[u] + d);
      bb[u] = *reinterpret_cast<const uint4*>(qr[u] + d + 128);
      const __half* cr = cos_t + row * kAttnHeadDim;
      const __half* sr = sin_t + row * kAttnHeadDim;
      ca[u] = __ldg(reinterpret_cast<const uint4*>(cr + d));
      cb[u] = __ldg(reinterpret_cast<const uint4*>(cr + d + 128));
      sa[u] = __ldg(reinterpret_cast<const uint4*>(sr + d));
      sb[u] = __ldg(reinterpret_cast<const uint4*>(sr + d + 128));
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!ok[u]) continue;
      rope_pairs8(a[u], bb[u], ca[u], cb[u], sa[u], sb[u]);
      *reinterpret_cast<uint4*>(qr[u] + dd[u]) = a[u];
      *reinterpret_cast<uint4*>(qr[u] + dd[u] + 128) = bb[u];
    }
    return;
  }
  // V rows -> shared memory: 16 keys x 32 vectors
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = t + 256 * h, j = i >> 5, c = i & 31;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (j0 + j < seq) val = ld_nc_v4(v + (row0 + j) * ldv + 8 * c);
    *reinterpret_cast<uint4*>(&tile[j][8 * c]) = val;
  }
  if (cos_t) {
    // k: 16 rows x 16 vectors of 8 pairs, one per thread
    const int j = t >> 4, d = 8 * (t & 15);
    if (j0 + j < seq) {
      const long long row = row0 + j;
      uint4 a = *reinterpret_cast<const uint4*>(k + row * ldk + d);
      uint4 bb = *reinterpret_cast<const uint4*>(k + row * ldk + d + 128);
      const __half* cr = cos_t + row * kAttnHeadDim;
      const __half* sr = sin_t + row * kAttnHeadDim;
      rope_pairs8(a, bb, __ldg(reinterpret_cast<const uint4*>(cr + d)),
                  __ldg(reinterpret_cast<const uint4*>(cr + d + 128)),
                  __ldg(reinterpret_cast<const uint4*>(sr + d)), __ldg(reinterpret_cast<const uint4*>(sr + d + 128)));
      *reinterpret_cast<uint4*>(k_out + row * ldko + d) = a;
      *reinterpret_cast<uint4*>(k_out + row * ldko + d + 128) = bb;
    }
  }
  __syncthreads();
  // V^T: 256 d-rows x 2 vectors of 8 keys
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = t + 256 * h, d = i >> 1, c = i & 1;
    const int key = j0 + 8 * c;
    if (key >= ldt) continue;
    uint4 out;
    __half* oh = reinterpret_cast<__half*>(&out);
#pragma unroll
    for (int e = 0; e < 8; ++e) oh[e] = tile[8 * c + e][d];
    *reinterpret_cast<uint4*>(vt + (static_cast<long long>(b) * kAttnHeadDim + d) * ldt + key) = out;
  }
}

}  // namespace w4a4

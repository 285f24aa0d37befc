// PTX helpers for sm_100a: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads) and descriptors.
//
// Every wait in this library is bounded: a wait that does not complete within
// its time limit records an error bit in the device error word, raises the
// CTA's abort flag and returns false, so a kernel never spins forever on a
// shared GPU.  The host reads the error word with w4a4_device_error().
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace w4a4 {

// Bits of the device error word.
enum DeviceError : unsigned {
  kErrWaitTma = 1u << 0,       // a stage's TMA bytes never arrived
  kErrWaitUnpack = 1u << 1,    // the MMA issuer waited too long for unpacked weights
  kErrWaitEmpty = 1u << 2,     // the producer waited too long for a free stage
  kErrWaitAccum = 1u << 3,     // the epilogue waited too long for the accumulator
  kErrWaitSelfTest = 1u << 4,  // the self-test wait ran out (expected in that test)
  kErrWaitDrain = 1u << 5,     // teardown gave up draining in-flight copies
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Gives up when the
// CTA's abort flag is raised by another role, or after `limit_ns`; in the
// latter case it raises the abort flag and ORs `err_bit` into `*err`.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, unsigned* err,
                                                  unsigned err_bit, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        *abort_flag = 1;
        atomicOr(err, err_bit);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completion counted in bytes
// on `bar`.  `x` is the innermost coordinate (elements), `y` the row.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32, K = 32.
__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp receives
// lane (warp quarter base + i), columns [col, col + 16).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (sm_100 format) for a K-major operand in
// the 128-byte swizzle layout: rows of 128 bytes, 8-row groups 1024 bytes
// apart (stride byte offset), leading byte offset unused (encoded 1),
// descriptor version 1, layout type 2 = SWIZZLE_128B.  The operand buffer
// must be 1024-byte aligned; stepping K inside the 128-byte swizzle row is
// done by adding the byte offset (>> 4) to the start address field.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address  [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                 // leading byte offset [16,30)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // stride byte offset  [32,46)
  d |= static_cast<uint64_t>(1u) << 46;                 // version [46,48)
  d |= static_cast<uint64_t>(2u) << 61;                 // SWIZZLE_128B [61,64)
  return d;
}

// Instruction descriptor for tcgen05.mma.kind::i8: D = s32, A and B signed
// 8-bit, both K-major, shape M x N (M in {64,128}, N a multiple of 16).
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4)                                  // D format: S32
         | (1u << 7)                                // A: signed 8-bit
         | (1u << 10)                               // B: signed 8-bit
         | (static_cast<uint32_t>(n >> 3) << 17)    // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);   // M >> 4
}

// ---------------------------------------------------------------- misc
// Byte-wise sign extension of the 4-bit two's-complement value held in the
// low nibble of each byte (the byte's high nibble must be zero).
__device__ __forceinline__ uint32_t sext_nibbles_in_bytes(uint32_t b) {
  return ((b ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Two packed words (16 nibbles: element j of word w at bits 4j) -> 16 int8
// values in element order.
__device__ __forceinline__ uint4 unpack16_nibbles(uint32_t w0, uint32_t w1) {
  const uint32_t e0 = sext_nibbles_in_bytes(w0 & 0x0F0F0F0Fu);         // k 0,2,4,6
  const uint32_t o0 = sext_nibbles_in_bytes((w0 >> 4) & 0x0F0F0F0Fu);  // k 1,3,5,7
  const uint32_t e1 = sext_nibbles_in_bytes(w1 & 0x0F0F0F0Fu);
  const uint32_t o1 = sext_nibbles_in_bytes((w1 >> 4) & 0x0F0F0F0Fu);
  uint4 r;
  r.x = prmt(e0, o0, 0x5140u);
  r.y = prmt(e0, o0, 0x7362u);
  r.z = prmt(e1, o1, 0x5140u);
  r.w = prmt(e1, o1, 0x7362u);
  return r;
}

}  // namespace w4a4

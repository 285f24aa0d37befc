// Host driver of the reference's quant_rot_rb: build_ref.py compiles one
// translation unit of gpu_shim.h, QUANT_TPB and the kernel template as the
// reference source defines them (read from the reference checkout, never
// stored here), then this file.  One block of QUANT_TPB host threads per row.
// TEST INFRASTRUCTURE ONLY.
#include <thread>
#include <vector>

template <int K, int R>
static void run_rows(const _Float16* x, int m, int32_t* q, float* sc) {
  static_assert(K / R == QUANT_TPB, "the reference launches K / R = QUANT_TPB threads per row");
  for (int row = 0; row < m; ++row) {
    std::barrier<> bar(QUANT_TPB);
    g_block_barrier = &bar;
    blockIdx.x = row;
    std::vector<std::thread> threads;
    threads.reserve(QUANT_TPB);
    for (int t = 0; t < QUANT_TPB; ++t)
      threads.emplace_back([=] {
        threadIdx.x = t;
        quant_rot_rb<K, R>(x, q, sc, m, static_cast<long>(K));
      });
    for (auto& th : threads) th.join();
  }
}

// x: fp16 bits [m, k]; q: packed int32 [m, k / 8] (nibble j of word p =
// element 8p + j); sc: [m] row scales.  Returns 0, or -1 for an unsupported k.
extern "C" int quant_rot_rb_ref(const uint16_t* x, int m, int k, int32_t* q, float* sc) {
  const _Float16* xh = reinterpret_cast<const _Float16*>(x);
  switch (k) {
    case 1024: run_rows<1024, 4>(xh, m, q, sc); return 0;
    case 2048: run_rows<2048, 8>(xh, m, q, sc); return 0;
    case 16384: run_rows<16384, 64>(xh, m, q, sc); return 0;
    default: return -1;
  }
}

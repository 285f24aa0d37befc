// libw4a4_sm100.so: the C ABI declared in include/w4a4_sm100.h.
//
// One translation unit holds every kernel (so the single device error word
// g_w4a4_device_error is shared), the launchers, a cache of TMA descriptors
// and the extern "C" entry points.  Argument checks mirror the reference's
// TORCH_CHECKs (pi05_fast/w4a4/csrc/int4_gemm.cu:487-501, :570-577) and keep
// their message text where the reference's tests match on it.
#include "w4a4_sm100.h"

#include <atomic>
#include <cstdlib>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"
#include "gemm.cuh"
#include "gemm_pair.cuh"
#include "attention.cuh"
#include "layer.cuh"
#include "pack.cuh"
#include "quant.cuh"
#include "neighbours.cuh"

// Scratch of w4a4_int4_gemm_noalloc: the intermediate activation codes and
// row scales, as file-scope device arrays (one copy per device, shared by
// every call on it; no allocation of any kind).  Calls on one stream are
// ordered only because every kernel that writes this scratch (the quants)
// executes griddepcontrol.wait (pdl_wait) before its first store: under
// programmatic dependent launch the previous call's GEMM may still be
// reading the codes when the next quant starts.
__device__ __align__(256) int8_t g_w4a4_noalloc_codes[W4A4_NOALLOC_MAX_CODES];
__device__ __align__(256) float g_w4a4_noalloc_scales[W4A4_NOALLOC_MAX_ROWS];

namespace w4a4 {
namespace {

thread_local std::string t_last_error;
thread_local int t_last_status = W4A4_OK;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  t_last_status = code;
  return code;
}

int ok() {
  t_last_status = W4A4_OK;
  return W4A4_OK;
}

#define W4A4_CUDA_TRY(expr)                                                                 \
  do {                                                                                     \
    const cudaError_t e_ = (expr);                                                         \
    if (e_ != cudaSuccess) return fail(W4A4_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// Status of a kernel launch, for callers that cannot return from the macro.
int cuda_status(cudaError_t e) {
  return e == cudaSuccess ? W4A4_OK
                          : fail(W4A4_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
}

std::atomic<unsigned long long> g_wait_limit_ns{1000000000ull};

// Programmatic dependent launch (on by default; W4A4_PDL=0 turns it off):
// the kernels call griddepcontrol.launch_dependents early and
// griddepcontrol.wait before they read the previous kernel's outputs or write
// anything, so a kernel's launch and prologue (barrier set-up, TMEM
// allocation, descriptor prefetch, the first weight tiles, which no kernel
// writes) overlap its predecessor's tail.  A dependent grid starts only once
// every CTA of its predecessor has started, so the early CTAs cannot hold
// resources a pending predecessor CTA needs.  On the 776-token prefix:
// 2.28 vs 2.34 ms per prefix.  Without the attribute the waits are no-ops.
const bool g_pdl = [] {
  const char* e = std::getenv("W4A4_PDL");
  return !(e && e[0] == '0');
}();

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (g_pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------- device info
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
uint64_t g_attr_done[kMaxDevices];  // bit per kernel whose smem attribute is set
std::mutex g_dev_mu;

int current_device(int* dev) {
  W4A4_CUDA_TRY(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(W4A4_ERR_UNSUPPORTED, "device %d out of range", *dev);
  return W4A4_OK;
}

int sm_count(int dev, int* out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_sm_count[dev] == 0) {
    int v = 0;
    W4A4_CUDA_TRY(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    g_sm_count[dev] = v;
  }
  *out = g_sm_count[dev];
  return W4A4_OK;
}

template <class Kernel>
int ensure_smem_attr(int dev, uint64_t bit, Kernel kernel, int bytes) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!(g_attr_done[dev] & bit)) {
    W4A4_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    g_attr_done[dev] |= bit;
  }
  return W4A4_OK;
}

// ------------------------------------------------------------- TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  uintptr_t ptr;
  uint64_t d[4], stride[3];
  uint32_t box[4];
  int rank, dtype, swizzle;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rank == o.rank && dtype == o.dtype && swizzle == o.swizzle &&
           std::memcmp(d, o.d, sizeof(d)) == 0 && std::memcmp(stride, o.stride, sizeof(stride)) == 0 &&
           std::memcmp(box, o.box, sizeof(box)) == 0;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = k.ptr * 0x9E3779B97F4A7C15ull;
    for (uint64_t v : {k.d[0], k.d[1], k.d[2], k.d[3], k.stride[0], k.stride[1], k.stride[2],
                       static_cast<uint64_t>(k.box[0]) << 32 | k.box[1],
                       static_cast<uint64_t>(k.box[2]) << 32 | k.box[3],
                       static_cast<uint64_t>(k.rank),
                       static_cast<uint64_t>(k.dtype) << 8 | static_cast<uint64_t>(k.swizzle)})
      h = (h ^ v) * 0x100000001B3ull;
    return static_cast<size_t>(h);
  }
};
std::mutex g_map_mu;
// Two caches: long-lived maps (packed weights, read by every call of a layer)
// and per-call maps (activations and codes, whose pointers and row counts
// change from call to call).  Each is bounded; when a cache is full its
// oldest entry is evicted (insertion order), so a stream of new activation
// shapes never pushes the weight maps out.
struct MapCache {
  std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
  std::deque<MapKey> order;
  size_t capacity;
};
MapCache g_weight_maps{{}, {}, 8192};
MapCache g_call_maps{{}, {}, 1024};

// Tiled tensor map of rank 2 to 4, cached by its parameters: dims[0]
// innermost (elements), strides_bytes[i] the byte stride of dims[i + 1].
int make_map(CUtensorMap* out, const void* ptr, CUtensorMapDataType dtype, int rank,
             const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
             CUtensorMapSwizzle swizzle, bool weight = false) {
  MapCache& cache = weight ? g_weight_maps : g_call_maps;
  MapKey key{};
  key.ptr = reinterpret_cast<uintptr_t>(ptr);
  key.rank = rank;
  key.dtype = static_cast<int>(dtype);
  key.swizzle = static_cast<int>(swizzle);
  for (int i = 0; i < rank; ++i) {
    key.d[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.stride[i] = strides_bytes[i];
  }
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = cache.maps.find(key);
    if (it != cache.maps.end()) {
      *out = it->second;
      return W4A4_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(W4A4_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (rank < 1 || rank > 4) return fail(W4A4_ERR_INVALID, "tensor map rank %d", rank);
  cuuint64_t cdims[4], cstrides[3];
  cuuint32_t cbox[4], estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    cdims[i] = dims[i];
    cbox[i] = box[i];
    if (i + 1 < rank) cstrides[i] = strides_bytes[i];
  }
  CUtensorMap map;
  const CUresult r = fn(&map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(ptr), cdims,
                        cstrides, cbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(W4A4_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d): rank %d, dims {%llu, %llu, %llu, %llu}, box {%u, %u, %u, %u}",
                static_cast<int>(r), rank, (unsigned long long)key.d[0], (unsigned long long)key.d[1],
                (unsigned long long)key.d[2], (unsigned long long)key.d[3], key.box[0], key.box[1],
                key.box[2], key.box[3]);
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (cache.maps.emplace(key, map).second) {
    cache.order.push_back(key);
    while (cache.maps.size() > cache.capacity) {
      cache.maps.erase(cache.order.front());
      cache.order.pop_front();
    }
  }
  *out = map;
  return W4A4_OK;
}

// 2-D tiled tensor map: dim0 innermost (elements), dim1 rows, row stride in bytes.
int make_map_2d(CUtensorMap* out, const void* ptr, CUtensorMapDataType dtype, uint64_t d0,
                uint64_t d1, uint64_t stride_bytes, uint32_t b0, uint32_t b1,
                CUtensorMapSwizzle swizzle, bool weight = false) {
  const uint64_t dims[2] = {d0, d1};
  const uint32_t box[2] = {b0, b1};
  return make_map(out, ptr, dtype, 2, dims, &stride_bytes, box, swizzle, weight);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------- quant
int launch_quant(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate,
                 int32_t staging, int32_t codes_format, void* codes, float* row_scale,
                 cudaStream_t stream) {
  if (k <= 0) return fail(W4A4_ERR_INVALID, "K must be positive, got %d", k);
  if (k % 64 != 0) return fail(W4A4_ERR_INVALID, "K must be a multiple of 64, got %d", k);
  if (m < 0) return fail(W4A4_ERR_INVALID, "M must be non-negative, got %lld", (long long)m);
  if (staging != W4A4_STAGING_FP16 && staging != W4A4_STAGING_FP32)
    return fail(W4A4_ERR_INVALID, "unknown staging mode %d", staging);
  if (codes_format != W4A4_CODES_INT8 && codes_format != W4A4_CODES_PACKED &&
      codes_format != W4A4_CODES_GEMM)
    return fail(W4A4_ERR_INVALID, "unknown codes format %d", codes_format);
  bool rot;
  if (rotate == W4A4_ROTATE_BY_K)
    rot = (k == 1024 || k == 2048 || k == 16384);
  else if (rotate == 0 || rotate == 1)
    rot = rotate == 1;
  else
    return fail(W4A4_ERR_INVALID, "rotate must be -1, 0 or 1, got %d", rotate);
  if (rot && !(k == 1024 || k == 2048 || k == 16384))
    return fail(W4A4_ERR_UNSUPPORTED, "Hadamard rotation is implemented for K in {1024, 2048, 16384}, got %d", k);
  if (m == 0) return ok();
  if (!x || !codes || !row_scale) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (ldx < k || ldx % 8 != 0)
    return fail(W4A4_ERR_INVALID, "activation row stride %lld must be >= K and a multiple of 8", (long long)ldx);
  if (!aligned(x, 16)) return fail(W4A4_ERR_INVALID, "activation pointer must be 16-byte aligned");
  if (!aligned(codes, 8)) return fail(W4A4_ERR_INVALID, "codes pointer must be 8-byte aligned");
  int dev;
  if (int e = current_device(&dev)) return e;

  const __half* xh = static_cast<const __half*>(x);
  const bool fp16 = staging == W4A4_STAGING_FP16;
  const float isk = static_cast<float>(1.0 / std::sqrt(static_cast<double>(k)));
  const unsigned rows_grid = static_cast<unsigned>((m + 7) / 8);
  if (m > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "M too large: %lld", (long long)m);

  // Instantiate a kernel for every (staging, format) pair.
  auto dispatch = [&](auto launch) {
    const auto by_mode = [&](auto fp16_tag) {
      constexpr bool F = decltype(fp16_tag)::value;
      switch (codes_format) {
        case W4A4_CODES_PACKED: launch(std::integral_constant<bool, F>{}, std::integral_constant<int, kCodesPacked>{}); break;
        case W4A4_CODES_GEMM: launch(std::integral_constant<bool, F>{}, std::integral_constant<int, kCodesGemm>{}); break;
        default: launch(std::integral_constant<bool, F>{}, std::integral_constant<int, kCodesInt8>{}); break;
      }
    };
    if (fp16) by_mode(std::true_type{});
    else by_mode(std::false_type{});
  };
  int err_code = W4A4_OK;
  if (rot && (k == 1024 || k == 2048)) {
    dispatch([&](auto f, auto mode) {
      constexpr bool F = decltype(f)::value;
      constexpr int MODE = decltype(mode)::value;
      const unsigned grid = static_cast<unsigned>(m);  // one CTA of K / 16 threads per row
      if (k == 1024)
        err_code = cuda_status(launch_kernel(quant_rot_warp_kernel<10, F, MODE>, dim3(grid), dim3(64), 0,
                                             stream, 1, xh, ldx, m, codes, row_scale, isk));
      else
        err_code = cuda_status(launch_kernel(quant_rot_warp_kernel<11, F, MODE>, dim3(grid), dim3(128), 0,
                                             stream, 1, xh, ldx, m, codes, row_scale, isk));
    });
  } else if (rot) {
    const unsigned grid = static_cast<unsigned>(m);
    dispatch([&](auto f, auto mode) {
      constexpr bool F = decltype(f)::value;
      constexpr int MODE = decltype(mode)::value;
      const int smem = F ? 16384 * 2 : 16384 * 4;
      if (!F) {
        if (int e = ensure_smem_attr(dev, 1u << (8 + MODE), quant_rot_16k_kernel<false, MODE>, smem)) {
          err_code = e;
          return;
        }
      }
      if (F) {
        // rows as {64 elements, 256 lines, m rows}: one 32 KB box per row
        CUtensorMap xmap;
        const uint64_t dims[3] = {64, 256, static_cast<uint64_t>(m)};
        const uint64_t strides[2] = {128, static_cast<uint64_t>(ldx) * 2};
        const uint32_t box[3] = {64, 256, 1};
        if (int e = make_map(&xmap, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box,
                             CU_TENSOR_MAP_SWIZZLE_128B)) {
          err_code = e;
          return;
        }
        if (int e = ensure_smem_attr(dev, 1u << (12 + MODE), quant_rot_16k_fp16_kernel<MODE>, kQ16Smem)) {
          err_code = e;
          return;
        }
        err_code = cuda_status(launch_kernel(quant_rot_16k_fp16_kernel<MODE>, dim3(grid),
                                             dim3(kQuantThreads), kQ16Smem, stream, 1, xmap, m, codes,
                                             row_scale, isk, g_wait_limit_ns.load(), xmap,
                                             static_cast<__half*>(nullptr), 0ll));
      } else
        err_code = cuda_status(launch_kernel(quant_rot_16k_kernel<F, MODE>, dim3(grid), dim3(kQuantThreads),
                                             smem, stream, 1, xh, ldx, m, codes, row_scale, isk,
                                             static_cast<const __half*>(nullptr), 0ll,
                                             static_cast<__half*>(nullptr), 0ll, 0, 0ll));
    });
  } else {
    dispatch([&](auto, auto mode) {
      constexpr int MODE = decltype(mode)::value;
      err_code = cuda_status(launch_kernel(quant_rows_kernel<MODE>, dim3(rows_grid), dim3(kQuantThreads), 0,
                                           stream, 1, xh, ldx, m, k, codes, row_scale));
    });
  }
  if (err_code) return err_code;
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

// ------------------------------------------------------------- layer glue
int check_codes_format(int32_t codes_format) {
  if (codes_format != W4A4_CODES_INT8 && codes_format != W4A4_CODES_PACKED &&
      codes_format != W4A4_CODES_GEMM)
    return fail(W4A4_ERR_INVALID, "unknown codes format %d", codes_format);
  return W4A4_OK;
}

// Calls launch(std::integral_constant<bool, FP16>, std::integral_constant<int, MODE>)
// for the runtime staging and codes format.
template <typename Launch>
void dispatch_staging_format(bool fp16, int32_t codes_format, Launch&& launch) {
  const auto by_mode = [&](auto fp16_tag) {
    constexpr bool F = decltype(fp16_tag)::value;
    switch (codes_format) {
      case W4A4_CODES_PACKED: launch(std::integral_constant<bool, F>{}, std::integral_constant<int, kCodesPacked>{}); break;
      case W4A4_CODES_GEMM: launch(std::integral_constant<bool, F>{}, std::integral_constant<int, kCodesGemm>{}); break;
      default: launch(std::integral_constant<bool, F>{}, std::integral_constant<int, kCodesInt8>{}); break;
    }
  };
  if (fp16) by_mode(std::true_type{});
  else by_mode(std::false_type{});
}

int launch_rmsnorm_quant(const void* x, int64_t ldx, const void* delta, int64_t ldd, const float* gain,
                         float eps, void* x_out, int64_t ldo, void* h_out, int64_t ldh, int64_t m,
                         int32_t k, int32_t staging, int32_t codes_format, void* codes,
                         float* row_scale, cudaStream_t stream) {
  if (k != kNormK) return fail(W4A4_ERR_UNSUPPORTED, "rmsnorm_quant supports K = %d only, got %d", kNormK, k);
  if (m < 0) return fail(W4A4_ERR_INVALID, "M must be non-negative, got %lld", (long long)m);
  if (staging != W4A4_STAGING_FP16 && staging != W4A4_STAGING_FP32)
    return fail(W4A4_ERR_INVALID, "unknown staging mode %d", staging);
  if (int e = check_codes_format(codes_format)) return e;
  if (!codes && !h_out) return fail(W4A4_ERR_INVALID, "rmsnorm_quant needs codes or h_out");
  if (codes && !row_scale) return fail(W4A4_ERR_INVALID, "codes need a row_scale output");
  if (m == 0) return ok();
  if (m > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "M too large: %lld", (long long)m);
  if (!x || !gain) return fail(W4A4_ERR_INVALID, "null pointer argument");
  const auto row_ok = [&](const void* p, int64_t ld) {
    return !p || (aligned(p, 16) && ld >= k && ld % 8 == 0);
  };
  if (!row_ok(x, ldx) || !row_ok(delta, ldd) || !row_ok(x_out, ldo) || !row_ok(h_out, ldh))
    return fail(W4A4_ERR_INVALID,
                "rows must be 16-byte aligned with a stride >= K and a multiple of 8 elements");
  if (!aligned(gain, 16)) return fail(W4A4_ERR_INVALID, "gain pointer must be 16-byte aligned");
  if (codes && !aligned(codes, 8)) return fail(W4A4_ERR_INVALID, "codes pointer must be 8-byte aligned");
  const float isk = static_cast<float>(1.0 / std::sqrt(static_cast<double>(k)));
  const __half* xh = static_cast<const __half*>(x);
  const __half* dh = static_cast<const __half*>(delta);
  __half* xo = static_cast<__half*>(x_out);
  __half* ho = static_cast<__half*>(h_out);
  int err_code = W4A4_OK;
  const dim3 grid(static_cast<unsigned>(m)), block(kNormThreads);
  const auto go = [&](auto kernel) {
    err_code = cuda_status(launch_kernel(kernel, grid, block, 0, stream, 1, xh, ldx, dh, ldd, gain, eps,
                                         xo, ldo, ho, ldh, m, codes, row_scale, isk));
  };
  if (!codes) {  // the norm alone (staging and codes format unused)
    if (delta) go(rmsnorm_quant_kernel<true, false, true, kCodesInt8>);
    else go(rmsnorm_quant_kernel<false, false, true, kCodesInt8>);
  } else {
    dispatch_staging_format(staging == W4A4_STAGING_FP16, codes_format, [&](auto f, auto mode) {
      constexpr bool F = decltype(f)::value;
      constexpr int MODE = decltype(mode)::value;
      if (delta) go(rmsnorm_quant_kernel<true, true, F, MODE>);
      else go(rmsnorm_quant_kernel<false, true, F, MODE>);
    });
  }
  if (err_code) return err_code;
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_geglu_quant(const void* gate, const void* up, int64_t m, int32_t k, int64_t ld,
                       int32_t staging, int32_t codes_format, void* codes, float* row_scale,
                       void* h_out, int64_t ldh, cudaStream_t stream) {
  if (k != 16384)
    return fail(W4A4_ERR_UNSUPPORTED, "geglu_quant supports K = 16384 only, got %d", k);
  if (m < 0) return fail(W4A4_ERR_INVALID, "M must be non-negative, got %lld", (long long)m);
  if (staging != W4A4_STAGING_FP16 && staging != W4A4_STAGING_FP32)
    return fail(W4A4_ERR_INVALID, "unknown staging mode %d", staging);
  if (int e = check_codes_format(codes_format)) return e;
  if (m == 0) return ok();
  if (m > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "M too large: %lld", (long long)m);
  if (!gate || !up || !codes || !row_scale) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (!aligned(gate, 16) || !aligned(up, 16) || ld < k || ld % 8 != 0)
    return fail(W4A4_ERR_INVALID,
                "gate/up rows must be 16-byte aligned with a stride >= K and a multiple of 8 elements");
  if (h_out && (!aligned(h_out, 16) || ldh < k || ldh % 8 != 0))
    return fail(W4A4_ERR_INVALID, "h_out rows must be 16-byte aligned with a stride >= K, multiple of 8");
  if (!aligned(codes, 8)) return fail(W4A4_ERR_INVALID, "codes pointer must be 8-byte aligned");
  int dev;
  if (int e = current_device(&dev)) return e;
  const float isk = static_cast<float>(1.0 / std::sqrt(static_cast<double>(k)));
  const unsigned grid = static_cast<unsigned>(m);
  __half* ho = static_cast<__half*>(h_out);
  int err_code = W4A4_OK;
  dispatch_staging_format(staging == W4A4_STAGING_FP16, codes_format, [&](auto f, auto mode) {
    constexpr bool F = decltype(f)::value;
    constexpr int MODE = decltype(mode)::value;
    if constexpr (F) {
      CUtensorMap gmap, umap;
      const uint64_t dims[3] = {64, 256, static_cast<uint64_t>(m)};
      const uint64_t strides[2] = {128, static_cast<uint64_t>(ld) * 2};
      const uint32_t box[3] = {64, 256, 1};
      if (int e = make_map(&gmap, gate, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B)) {
        err_code = e;
        return;
      }
      if (int e = make_map(&umap, up, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B)) {
        err_code = e;
        return;
      }
      if (int e = ensure_smem_attr(dev, 1ull << (32 + MODE), quant_rot_16k_fp16_kernel<MODE, false, true>,
                                   kQ16SmemGeglu)) {
        err_code = e;
        return;
      }
      err_code = cuda_status(launch_kernel(quant_rot_16k_fp16_kernel<MODE, false, true>, dim3(grid),
                                           dim3(kQuantThreads), kQ16SmemGeglu, stream, 1, gmap, m, codes,
                                           row_scale, isk, g_wait_limit_ns.load(), umap, ho, ldh));
    } else {
      const int smem = 16384 * 4;
      if (int e = ensure_smem_attr(dev, 1ull << (36 + MODE), quant_rot_16k_kernel<false, MODE, true>, smem)) {
        err_code = e;
        return;
      }
      err_code = cuda_status(launch_kernel(quant_rot_16k_kernel<false, MODE, true>, dim3(grid),
                                           dim3(kQuantThreads), smem, stream, 1,
                                           static_cast<const __half*>(gate), ld, m, codes, row_scale, isk,
                                           static_cast<const __half*>(up), ld, ho, ldh, 0, 0ll));
    }
  });
  if (err_code) return err_code;
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_geglu(const void* gate, const void* up, int64_t m, int32_t n, int64_t ld, void* h,
                 int64_t ldh, cudaStream_t stream) {
  if (m < 0 || n <= 0 || n % 8 != 0)
    return fail(W4A4_ERR_INVALID, "geglu: invalid shape m=%lld n=%d (n a positive multiple of 8)", (long long)m, n);
  if (m == 0) return ok();
  if (!gate || !up || !h) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(h, 16) || ld < n || ldh < n || ld % 8 || ldh % 8)
    return fail(W4A4_ERR_INVALID, "geglu rows must be 16-byte aligned with strides >= n, multiples of 8");
  const int64_t blocks = (m * (n / 8) + 255) / 256;
  if (blocks > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "geglu: too many rows");
  W4A4_CUDA_TRY(launch_kernel(geglu_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, 1,
                              static_cast<const __half*>(gate), static_cast<const __half*>(up), ld,
                              static_cast<__half*>(h), ldh, m, n));
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

// ------------------------------------------------------------- config-4 neighbours (bf16)
int launch_ada_rms_norm_bf16(const void* x, void* y, int64_t rows, int32_t h, int32_t rows_per_batch,
                             const float* scale1, const float* shift, int64_t mod_stride, float eps,
                             cudaStream_t stream) {
  if (rows < 0 || h <= 0 || h % 256 != 0 || h > 2048 || rows_per_batch <= 0 || mod_stride < h)
    return fail(W4A4_ERR_INVALID, "ada_rms_norm: invalid shape rows=%lld h=%d rows_per_batch=%d "
                "(h a multiple of 256 up to 2048, mod_stride >= h)", (long long)rows, h, rows_per_batch);
  if (rows == 0) return ok();
  if (!x || !y || !scale1 || !shift) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(scale1, 16) || !aligned(shift, 16) || mod_stride % 4)
    return fail(W4A4_ERR_INVALID, "ada_rms_norm: pointers must be 16-byte aligned, mod_stride a multiple of 4");
  const int64_t blocks = (rows + kNbThreads / 32 - 1) / (kNbThreads / 32);
  if (blocks > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "ada_rms_norm: too many rows");
  const auto go = [&](auto kernel) {
    return launch_kernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kNbThreads), 0, stream, 1,
                         static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y),
                         static_cast<long long>(rows), static_cast<int>(rows_per_batch), scale1, shift,
                         static_cast<long long>(mod_stride), eps);
  };
  cudaError_t e = cudaSuccess;
  switch (h / 256) {
    case 1: e = go(ada_rms_norm_bf16_kernel<1>); break;
    case 2: e = go(ada_rms_norm_bf16_kernel<2>); break;
    case 3: e = go(ada_rms_norm_bf16_kernel<3>); break;
    case 4: e = go(ada_rms_norm_bf16_kernel<4>); break;
    case 5: e = go(ada_rms_norm_bf16_kernel<5>); break;
    case 6: e = go(ada_rms_norm_bf16_kernel<6>); break;
    case 7: e = go(ada_rms_norm_bf16_kernel<7>); break;
    default: e = go(ada_rms_norm_bf16_kernel<8>); break;
  }
  W4A4_CUDA_TRY(e);
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_rope_qk_bf16(void* q, int64_t ldq, int32_t heads_q, void* k, int64_t ldk, int32_t heads_k,
                        const void* cos_t, const void* sin_t, int64_t rows, int32_t hd, cudaStream_t stream) {
  if (rows < 0 || hd <= 0 || hd % 16 != 0 || heads_q < 0 || heads_k < 0 || heads_q + heads_k == 0 ||
      ldq < static_cast<int64_t>(heads_q) * hd || ldk < static_cast<int64_t>(heads_k) * hd)
    return fail(W4A4_ERR_INVALID, "rope_qk: invalid shape rows=%lld hd=%d heads %d + %d (hd a multiple of 16, "
                "row strides >= heads * hd)", (long long)rows, hd, heads_q, heads_k);
  if (rows == 0) return ok();
  if ((heads_q && !q) || (heads_k && !k) || !cos_t || !sin_t)
    return fail(W4A4_ERR_INVALID, "null pointer argument");
  if ((heads_q && (!aligned(q, 16) || ldq % 8)) || (heads_k && (!aligned(k, 16) || ldk % 8)) ||
      !aligned(cos_t, 16) || !aligned(sin_t, 16))
    return fail(W4A4_ERR_INVALID, "rope_qk: rows must be 16-byte aligned with strides multiples of 8");
  const int64_t threads = rows * (heads_q + heads_k) * (hd / 16);
  const int64_t blocks = (threads + kNbThreads - 1) / kNbThreads;
  if (blocks > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "rope_qk: too many rows");
  W4A4_CUDA_TRY(launch_kernel(rope_bf16_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kNbThreads), 0,
                              stream, 1, static_cast<__nv_bfloat16*>(q), static_cast<long long>(ldq),
                              static_cast<int>(heads_q), static_cast<__nv_bfloat16*>(k),
                              static_cast<long long>(ldk), static_cast<int>(heads_k),
                              static_cast<const __nv_bfloat16*>(cos_t), static_cast<const __nv_bfloat16*>(sin_t),
                              static_cast<long long>(rows), static_cast<int>(hd)));
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_layer_norm_bf16(const void* x, void* y, int64_t rows, int32_t h, const void* w, const void* b,
                           float eps, cudaStream_t stream) {
  if (rows < 0 || h <= 0 || h % 8 != 0 || h > 2048)
    return fail(W4A4_ERR_INVALID, "layer_norm: invalid shape rows=%lld h=%d (h a multiple of 8 up to 2048)",
                (long long)rows, h);
  if (rows == 0) return ok();
  if (!x || !y || !w || !b) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(w, 16) || !aligned(b, 16))
    return fail(W4A4_ERR_INVALID, "layer_norm: pointers must be 16-byte aligned");
  const int64_t blocks = (rows + kNbThreads / 32 - 1) / (kNbThreads / 32);
  if (blocks > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "layer_norm: too many rows");
  const auto go = [&](auto kernel) {
    return launch_kernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kNbThreads), 0, stream, 1,
                         static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y),
                         static_cast<long long>(rows), static_cast<int>(h),
                         static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(b), eps);
  };
  cudaError_t e = cudaSuccess;
  switch ((h + 255) / 256) {
    case 1: e = go(layer_norm_bf16_kernel<1>); break;
    case 2: e = go(layer_norm_bf16_kernel<2>); break;
    case 3: e = go(layer_norm_bf16_kernel<3>); break;
    case 4: e = go(layer_norm_bf16_kernel<4>); break;
    case 5: e = go(layer_norm_bf16_kernel<5>); break;
    case 6: e = go(layer_norm_bf16_kernel<6>); break;
    case 7: e = go(layer_norm_bf16_kernel<7>); break;
    default: e = go(layer_norm_bf16_kernel<8>); break;
  }
  W4A4_CUDA_TRY(e);
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_quant_segments(const void* x, int64_t m, int32_t k, int32_t seg, int64_t ld,
                          int64_t seg_stride, int32_t staging, int32_t codes_format, void* codes,
                          float* row_scale, cudaStream_t stream) {
  if (k != 16384)
    return fail(W4A4_ERR_UNSUPPORTED, "quant_segments supports K = 16384 only, got %d", k);
  if (seg < 64 || seg % 64 != 0 || k % seg != 0 || k / seg > 256)
    return fail(W4A4_ERR_INVALID, "segment width %d must be a multiple of 64 dividing K = %d", seg, k);
  if (m < 0) return fail(W4A4_ERR_INVALID, "M must be non-negative, got %lld", (long long)m);
  if (staging != W4A4_STAGING_FP16 && staging != W4A4_STAGING_FP32)
    return fail(W4A4_ERR_INVALID, "unknown staging mode %d", staging);
  if (int e = check_codes_format(codes_format)) return e;
  if (m == 0) return ok();
  if (m > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "M too large: %lld", (long long)m);
  if (!x || !codes || !row_scale) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (!aligned(x, 16) || ld < seg || ld % 8 != 0 || seg_stride % 8 != 0 || seg_stride < ld * m)
    return fail(W4A4_ERR_INVALID,
                "segments must be 16-byte aligned [M, seg] blocks: stride >= seg and a multiple of 8, "
                "segment stride >= M x stride and a multiple of 8");
  if (!aligned(codes, 8)) return fail(W4A4_ERR_INVALID, "codes pointer must be 8-byte aligned");
  int dev;
  if (int e = current_device(&dev)) return e;
  const float isk = static_cast<float>(1.0 / std::sqrt(static_cast<double>(k)));
  const unsigned grid = static_cast<unsigned>(m);
  int err_code = W4A4_OK;
  dispatch_staging_format(staging == W4A4_STAGING_FP16, codes_format, [&](auto f, auto mode) {
    constexpr bool F = decltype(f)::value;
    constexpr int MODE = decltype(mode)::value;
    if constexpr (F) {
      CUtensorMap xmap;
      const uint64_t dims[4] = {64, static_cast<uint64_t>(seg / 64), static_cast<uint64_t>(m),
                                static_cast<uint64_t>(k / seg)};
      const uint64_t strides[3] = {128, static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(seg_stride) * 2};
      const uint32_t box[4] = {64, static_cast<uint32_t>(seg / 64), 1, static_cast<uint32_t>(k / seg)};
      if (int e = make_map(&xmap, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B)) {
        err_code = e;
        return;
      }
      if (int e = ensure_smem_attr(dev, 1ull << (44 + MODE), quant_rot_16k_fp16_kernel<MODE, true>,
                                   kQ16Smem)) {
        err_code = e;
        return;
      }
      err_code = cuda_status(launch_kernel(quant_rot_16k_fp16_kernel<MODE, true>, dim3(grid),
                                           dim3(kQuantThreads), kQ16Smem, stream, 1, xmap, m, codes,
                                           row_scale, isk, g_wait_limit_ns.load(), xmap,
                                           static_cast<__half*>(nullptr), 0ll));
    } else {
      const int smem = 16384 * 4;
      if (int e = ensure_smem_attr(dev, 1ull << (48 + MODE), quant_rot_16k_kernel<false, MODE, false, true>,
                                   smem)) {
        err_code = e;
        return;
      }
      err_code = cuda_status(launch_kernel(quant_rot_16k_kernel<false, MODE, false, true>, dim3(grid),
                                           dim3(kQuantThreads), smem, stream, 1, static_cast<const __half*>(x),
                                           ld, m, codes, row_scale, isk, static_cast<const __half*>(nullptr),
                                           0ll, static_cast<__half*>(nullptr), 0ll, seg, seg_stride));
    }
  });
  if (err_code) return err_code;
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_prefix_tables(const uint8_t* pad, int32_t batch, int32_t seq, const float* inv_freq, int32_t half,
                         uint8_t* key_valid, int32_t* kv_len, void* cos_t, void* sin_t, cudaStream_t stream) {
  if (batch < 0 || seq < 0 || half <= 0 || half % 8 != 0)
    return fail(W4A4_ERR_INVALID, "prefix tables: invalid shape batch %d seq %d half %d", batch, seq, half);
  if (batch == 0 || seq == 0) return ok();
  if (!pad || !inv_freq || !key_valid || !kv_len || !cos_t || !sin_t)
    return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (!aligned(cos_t, 16) || !aligned(sin_t, 16))
    return fail(W4A4_ERR_INVALID, "cos / sin tables must be 16-byte aligned");
  W4A4_CUDA_TRY(launch_kernel(prefix_tables_kernel,
                              dim3(static_cast<unsigned>((seq + kTableRows - 1) / kTableRows),
                                   static_cast<unsigned>(batch)),
                              dim3(kTableThreads), 0,
                              stream, 1, pad, static_cast<int>(seq), inv_freq, static_cast<int>(half), key_valid,
                              static_cast<int*>(kv_len), static_cast<__half*>(cos_t), static_cast<__half*>(sin_t)));
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int launch_rope(const void* x, int64_t ldx, void* out, int64_t ldo, const void* cos_t,
                const void* sin_t, int64_t m, int32_t heads, cudaStream_t stream) {
  if (m < 0 || heads <= 0) return fail(W4A4_ERR_INVALID, "invalid rope shape: m=%lld heads=%d", (long long)m, heads);
  if (m == 0) return ok();
  if (!x || !out || !cos_t || !sin_t) return fail(W4A4_ERR_INVALID, "null pointer argument");
  const int64_t width = static_cast<int64_t>(heads) * kRopeHeadDim;
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(cos_t, 16) || !aligned(sin_t, 16) ||
      ldx < width || ldo < width || ldx % 8 || ldo % 8)
    return fail(W4A4_ERR_INVALID,
                "rope rows must be 16-byte aligned with strides >= heads * 256, multiples of 8");
  const int64_t threads = m * heads * (kRopeHeadDim / 16);
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "rope: too many rows");
  W4A4_CUDA_TRY(launch_kernel(rope_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, 1,
                              static_cast<const __half*>(x), ldx, static_cast<__half*>(out), ldo,
                              static_cast<const __half*>(cos_t), static_cast<const __half*>(sin_t), m,
                              heads));
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

// ------------------------------------------------------------- attention
int64_t attn_vt_stride(int32_t seq) { return (static_cast<int64_t>(seq) + 7) / 8 * 8; }

int launch_attention(void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                     int64_t ldv, const uint8_t* key_valid, const int32_t* kv_len, int32_t batch,
                     int32_t seq, int32_t heads, void* vt, void* out, int64_t ldo, const void* cos_t,
                     const void* sin_t, void* k_out, int64_t ldko, cudaStream_t stream) {
  if (batch < 0 || seq < 0) return fail(W4A4_ERR_INVALID, "invalid attention shape: batch %d, seq %d", batch, seq);
  if (heads < 1 || heads > kAttnRows || kAttnRows % heads != 0)
    return fail(W4A4_ERR_UNSUPPORTED, "attention: heads must divide %d, got %d", kAttnRows, heads);
  if (seq > kAttnMaxKeys)
    return fail(W4A4_ERR_UNSUPPORTED, "attention: prefix of %d tokens exceeds %d", seq, kAttnMaxKeys);
  if (batch == 0 || seq == 0) return ok();
  if (!q || !k || !v || !key_valid || !kv_len || !vt || !out)
    return fail(W4A4_ERR_INVALID, "null pointer argument");
  const int64_t width = static_cast<int64_t>(heads) * kAttnHeadDim;
  const auto rows_ok = [](const void* ptr, int64_t ld, int64_t w) {
    return aligned(ptr, 16) && ld >= w && ld % 8 == 0;
  };
  if (!rows_ok(q, ldq, width) || !rows_ok(out, ldo, width) || !rows_ok(k, ldk, kAttnHeadDim) ||
      !rows_ok(v, ldv, kAttnHeadDim) || !aligned(vt, 16))
    return fail(W4A4_ERR_INVALID,
                "attention rows must be 16-byte aligned with strides >= their width and multiples of 8");
  const bool rope = cos_t != nullptr;
  if (rope && (!sin_t || !k_out || !aligned(cos_t, 16) || !aligned(sin_t, 16) ||
               !rows_ok(k_out, ldko, kAttnHeadDim)))
    return fail(W4A4_ERR_INVALID,
                "attention RoPE needs 16-byte aligned cos/sin tables and a k_out of rows >= 256, stride a "
                "multiple of 8");
  int dev;
  if (int e = current_device(&dev)) return e;
  const int64_t ldt = attn_vt_stride(seq);
  W4A4_CUDA_TRY(launch_kernel(attn_prep_kernel,
                              dim3(static_cast<unsigned>((ldt + kPrepTokens - 1) / kPrepTokens),
                                   static_cast<unsigned>(batch),
                                   rope ? 1u + static_cast<unsigned>((heads + kPrepHeadsPerSlice - 1) /
                                                                     kPrepHeadsPerSlice)
                                        : 1u),
                              dim3(256), 0, stream, 1, static_cast<__half*>(const_cast<void*>(q)), ldq,
                              static_cast<const __half*>(k), ldk, static_cast<__half*>(rope ? k_out : nullptr),
                              rope ? ldko : 0ll, static_cast<const __half*>(v), ldv, static_cast<__half*>(vt), ldt,
                              static_cast<const __half*>(cos_t), static_cast<const __half*>(sin_t), seq, heads));
  // the keys the attention reads: rotated into k_out, or k as given
  const void* kr = rope ? k_out : k;
  const int64_t ldkr = rope ? ldko : ldk;
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  {
    const uint64_t dims[4] = {kAttnHeadDim, static_cast<uint64_t>(heads), static_cast<uint64_t>(seq),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[3] = {kAttnHeadDim * 2, static_cast<uint64_t>(ldq) * 2,
                                 static_cast<uint64_t>(ldq) * 2 * static_cast<uint64_t>(seq)};
    const uint32_t box[4] = {64, static_cast<uint32_t>(heads), static_cast<uint32_t>(kAttnRows / heads), 1};
    if (int e = make_map(&p.tmap_q, q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
    const uint64_t ostrides[3] = {kAttnHeadDim * 2, static_cast<uint64_t>(ldo) * 2,
                                  static_cast<uint64_t>(ldo) * 2 * static_cast<uint64_t>(seq)};
    if (int e = make_map(&p.tmap_o, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, dims, ostrides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
  }
  {
    const uint64_t dims[3] = {kAttnHeadDim, static_cast<uint64_t>(seq), static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldkr) * 2,
                                 static_cast<uint64_t>(ldkr) * 2 * static_cast<uint64_t>(seq)};
    const uint32_t box[3] = {64, kAttnKeyBlock, 1};
    if (int e = make_map(&p.tmap_k, kr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(seq), kAttnHeadDim, static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldt) * 2,
                                 static_cast<uint64_t>(ldt) * 2 * kAttnHeadDim};
    const uint32_t box[3] = {kAttnKeyBlock, kAttnHeadDim, 1};
    if (int e = make_map(&p.tmap_vt, vt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
  }
  p.key_valid = key_valid;
  p.kv_len = kv_len;
  p.out = static_cast<__half*>(out);
  p.ldo = ldo;
  p.seq = seq;
  p.heads = heads;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kAttnHeadDim)));
  p.wait_limit_ns = g_wait_limit_ns.load();
  if (int e = ensure_smem_attr(dev, 1ull << 40, prefix_attention_kernel, kAttnSmem)) return e;
  const int tpt = kAttnRows / heads;
  // two CTAs (a cluster) per tile of tpt tokens, each half of its key range
  W4A4_CUDA_TRY(launch_kernel(prefix_attention_kernel,
                              dim3(2u * static_cast<unsigned>((seq + tpt - 1) / tpt), static_cast<unsigned>(batch)),
                              dim3(kAttnThreads), kAttnSmem, stream, 2, p));
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

// ------------------------------------------------------------- GEMM
// Tile width and split-K for the single-CTA kernel.  A K step of a tile of
// t tokens costs about 330 + 1.5 t SM cycles (per-step traces on B200: the
// MMA issue loop, ~480 at t = 96 and ~640 at t = 208), a tile about 2000
// more (pipeline fill, epilogue tail), and a split tile 12 t more for the
// partial-sum exchange.  Split-K runs a tile's two K halves on the two CTAs
// of a cluster, so it pays when the tiles do not fill the SMs.
struct GemmPlan {
  int tok_tile;
  bool split;
};
GemmPlan choose_plan(int64_t m, int w_tiles, int k_steps, int sms, int variant) {
  GemmPlan best{16, false};
  double best_cost = 1e300;
  const int64_t t_min = (m + kTokTileMax - 1) / kTokTileMax;
  for (int64_t t = t_min; t <= t_min + 64; ++t) {
    const int64_t per = (m + t - 1) / t;
    const int tile = static_cast<int>(((per + 15) / 16) * 16);
    const int64_t tiles = ((m + tile - 1) / tile) * w_tiles;
    for (int split = 0; split < 2; ++split) {
      // split-K needs an even K-step count and one tile per cluster
      const bool can_split = k_steps % 2 == 0 && k_steps >= 2 && tiles <= sms / 2;
      if (split && (!can_split || variant == W4A4_GEMM_NO_SPLIT)) continue;
      if (!split && can_split && variant == W4A4_GEMM_SPLIT_K) continue;
      const int64_t workers = split ? sms / 2 : sms;
      const int64_t waves = (tiles + workers - 1) / workers;
      const double steps = split ? k_steps / 2 : k_steps;
      // split-K adds the partial-sum exchange (~12 per token column) and a
      // per-cluster cost measured on B200 (~45 per cluster: 16-step GEMMs
      // at 64 clusters ran 1.5 us slower than at 32 with the same per-CTA
      // work, and lost to no split from ~60 clusters on).
      const double cost = static_cast<double>(waves) *
                          (steps * (330.0 + 1.5 * tile) + 2000.0 +
                           (split ? 12.0 * tile + 45.0 * static_cast<double>(tiles) : 0.0));
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = {tile, split != 0};
      }
    }
    if (tile <= 32) break;
  }
  return best;
}

// Token-tile width for the CTA-pair kernel (no split-K).  The tile count T
// is chosen to minimise ceil(tiles / workers) * (tile + kTileOverhead): the
// busiest pair's tile count times a per-tile cost in which the overhead term
// models the work that does not scale with the tile (streaming and unpacking
// the weight operand).  Tiles are multiples of 16 (the UMMA N granularity).
int choose_tok_tile(int64_t m, int w_tiles, int sms) {
  constexpr int kTileOverhead = 64;
  int best_tile = 16;
  double best_cost = 1e300;
  const int64_t t_min = (m + kTokTileMax - 1) / kTokTileMax;
  for (int64_t t = t_min; t <= t_min + 64; ++t) {
    const int64_t per = (m + t - 1) / t;
    const int tile = static_cast<int>(((per + 15) / 16) * 16);
    const int64_t tiles = ((m + tile - 1) / tile) * w_tiles;
    const int64_t waves = (tiles + sms - 1) / sms;
    const double cost = static_cast<double>(waves) * (tile + kTileOverhead);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best_tile = tile;
    }
    if (tile <= 32) break;
  }
  return best_tile;
}

// Everything about a GEMM launch's shape that follows from (M, weight tiles,
// K, SM count, variant): the token tile, split-K, rasterisation group and
// grid.  Shared by launch_gemm and the w4a4_gemm_plan test hook.
struct LaunchShape {
  int tok_tile;
  bool split;
  int n_tok_tiles;
  int tok_group;
  int64_t total_tiles;
  unsigned grid;
};

LaunchShape launch_shape(int64_t m, int w_tiles, int32_t k, int sms, bool pair, int variant) {
  LaunchShape ls{};
  const int workers = pair ? sms / 2 : sms;
  const int k_steps = (k + kBlockK - 1) / kBlockK;
  const GemmPlan plan = pair ? GemmPlan{choose_tok_tile(m, w_tiles, workers), false}
                             : choose_plan(m, w_tiles, k_steps, sms, variant);
  ls.tok_tile = plan.tok_tile;
  ls.split = plan.split;
  ls.n_tok_tiles = static_cast<int>((m + ls.tok_tile - 1) / ls.tok_tile);
  // Rasterisation: keep each group's activation codes (tok_group token tiles
  // x K bytes) within ~48 MB of the 126 MB L2, so the codes are read from HBM
  // once and the weights once per group.  Prefix-sized M is one group.
  const int64_t tile_code_bytes = static_cast<int64_t>(ls.tok_tile) * k;
  const int64_t g = std::max<int64_t>(1, (48ll << 20) / std::max<int64_t>(1, tile_code_bytes));
  ls.tok_group = static_cast<int>(std::min<int64_t>(g, ls.n_tok_tiles));
  ls.total_tiles = static_cast<int64_t>(ls.n_tok_tiles) * w_tiles;
  ls.grid = pair || ls.split ? 2u * static_cast<unsigned>(std::min<int64_t>(ls.total_tiles, sms / 2))
                             : static_cast<unsigned>(std::min<int64_t>(ls.total_tiles, sms));
  return ls;
}

constexpr int32_t kMaxGemmK = 1 << 21;

int check_weight(const w4a4_weight& w, int32_t k, int idx) {
  if (!w.data) return fail(W4A4_ERR_INVALID, "packed W %d: null data pointer", idx);
  if (w.n <= 0) return fail(W4A4_ERR_INVALID, "packed W %d: N must be positive, got %d", idx, w.n);
  if (w.row_words < k / 8 + 1)
    return fail(W4A4_ERR_INVALID, "packed W second dim must contain K/8 packed words plus a scale");
  if (!aligned(w.data, 16)) return fail(W4A4_ERR_INVALID, "packed W %d must be 16-byte aligned", idx);
  if (w.layout == W4A4_LAYOUT_ROW_MAJOR) {
    if ((static_cast<int64_t>(w.row_words) * 4) % 16 != 0)
      return fail(W4A4_ERR_UNSUPPORTED,
                  "row-major packed W row stride (%d words) must be a multiple of 4 words; pad the rows "
                  "(w4a4_pad_rows / the K/8+8 load-time pad)",
                  w.row_words);
  } else if (w.layout == W4A4_LAYOUT_INT8) {
    if (w.row_words != k / 4 + 4)
      return fail(W4A4_ERR_INVALID, "int8 weights must use the K/4+4 row stride (w4a4_repack_int8)");
    return W4A4_OK;
  } else if (w.layout == W4A4_LAYOUT_FRAGMENT_MAJOR) {
    if (w.row_words != k / 8 + 9)
      return fail(W4A4_ERR_INVALID, "WMMA-fragment-major weights must use the K/8+9 marker stride");
    if (k % 16 != 0 || (w.n % 2) != 0)
      return fail(W4A4_ERR_UNSUPPORTED, "fragment-major weights need K %% 16 == 0 and an even N");
  } else {
    return fail(W4A4_ERR_INVALID, "unknown weight layout %d", w.layout);
  }
  return W4A4_OK;
}

// The GEMM variant of later launches: W4A4_GEMM_SINGLE_CTA (the default,
// see use_pair_kernel for the shapes it still sends to CTA pairs), or a
// forced variant from w4a4_set_gemm_variant / W4A4_GEMM_PAIR=1 (CTA pairs
// for every shape).  All variants are bit-identical.
std::atomic<int> g_gemm_variant{[] {
  const char* e = std::getenv("W4A4_GEMM_PAIR");
  return (e && e[0] == '1') ? W4A4_GEMM_CTA_PAIR : W4A4_GEMM_SINGLE_CTA;
}()};

// The default variant runs fragment-major GEMMs (gate/up) of at least
// kPairMinRows tokens on the CTA pair: its token tile is split over two SMs,
// which halves each SM's token traffic.  Measured on the prefix pass: 2.144 vs
// 2.157 ms per 776-token prefix and 13.3 vs 13.7 ms per 8-prefix step,
// bit-identical; below ~200 tokens the single-CTA kernel is faster.
constexpr int64_t kPairMinRows = 768;
bool use_pair_kernel(int variant, int layout, int64_t m) {
  return variant == W4A4_GEMM_CTA_PAIR || layout == W4A4_LAYOUT_INT8 ||
         (variant == W4A4_GEMM_SINGLE_CTA && layout == W4A4_LAYOUT_FRAGMENT_MAJOR &&
          m >= kPairMinRows);
}


int launch_gemm(const void* codes, const float* row_scale, int64_t m, int32_t k, int32_t n_weights,
                const w4a4_weight* weights, void* const* y, cudaStream_t stream,
                bool acc_out = false) {
  if (k <= 0 || k % 64 != 0) return fail(W4A4_ERR_INVALID, "K must be a multiple of 64, got %d", k);
  // the tensor cores accumulate 16 x sum(qa * qw), |.| <= 16 * 7 * 8 * K, in int32
  if (k > kMaxGemmK)
    return fail(W4A4_ERR_UNSUPPORTED, "K = %d exceeds %d (int32 accumulator range)", k, kMaxGemmK);
  if (m < 0) return fail(W4A4_ERR_INVALID, "M must be non-negative");
  if (n_weights < 1 || n_weights > kMaxSegments)
    return fail(W4A4_ERR_INVALID, "n_weights must be 1..%d, got %d", kMaxSegments, n_weights);
  if (!weights || !y) return fail(W4A4_ERR_INVALID, "null weights/outputs array");
  const int layout = weights[0].layout;
  for (int i = 0; i < n_weights; ++i) {
    if (weights[i].layout != layout)
      return fail(W4A4_ERR_INVALID, "all weights of one call must share a layout");
    if (int e = check_weight(weights[i], k, i)) return e;
    if (m > 0 && !y[i]) return fail(W4A4_ERR_INVALID, "output %d is null", i);
  }
  if (m == 0) return ok();
  if (!codes || (!row_scale && !acc_out)) return fail(W4A4_ERR_INVALID, "null codes/scale pointer");
  if (!aligned(codes, 16)) return fail(W4A4_ERR_INVALID, "codes pointer must be 16-byte aligned");
  if (m > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "M too large");
  int dev, sms;
  if (int e = current_device(&dev)) return e;
  if (int e = sm_count(dev, &sms)) return e;

  // K > kMagicMaxK: the WIDE single-CTA kernel (exact int -> float of acc / 16)
  const bool wide = k > kMagicMaxK && !acc_out;
  if (wide && layout == W4A4_LAYOUT_INT8)
    return fail(W4A4_ERR_UNSUPPORTED, "int8 weights support K <= %d", kMagicMaxK);
  const int variant = wide ? W4A4_GEMM_NO_SPLIT : g_gemm_variant.load();
  const bool pair = !wide && use_pair_kernel(variant, layout, m);
  const int rows_per_wtile = pair ? 2 * kBlockW : kBlockW;
  GemmParams p;
  std::memset(&p, 0, sizeof(p));
  int w_tiles = 0;
  for (int i = 0; i < n_weights; ++i) {
    const w4a4_weight& w = weights[i];
    GemmSegment& s = p.seg[i];
    if (layout == W4A4_LAYOUT_INT8) {
      if (int e = make_map_2d(&s.tmap_w, w.data, CU_TENSOR_MAP_DATA_TYPE_UINT8, k, w.n,
                              static_cast<uint64_t>(w.row_words) * 4, kBlockK, kBlockW,
                              CU_TENSOR_MAP_SWIZZLE_128B, true))
        return e;
      s.scale = reinterpret_cast<const float*>(w.data + k / 4);
      s.scale_stride = w.row_words;
    } else if (layout == W4A4_LAYOUT_ROW_MAJOR) {
      if (int e = make_map_2d(&s.tmap_w, w.data, CU_TENSOR_MAP_DATA_TYPE_UINT32, k / 8, w.n,
                              static_cast<uint64_t>(w.row_words) * 4, kBlockK / 8, kBlockW,
                              CU_TENSOR_MAP_SWIZZLE_64B, true))
        return e;
      s.scale = reinterpret_cast<const float*>(w.data + k / 8);
      s.scale_stride = w.row_words;
    } else {
      if (int e = make_map_2d(&s.tmap_w, w.data, CU_TENSOR_MAP_DATA_TYPE_UINT32,
                              static_cast<uint64_t>(w.n) * 2, k / 16,
                              static_cast<uint64_t>(w.n) * 8, 2 * kBlockW, kBlockK / 16,
                              CU_TENSOR_MAP_SWIZZLE_NONE, true))
        return e;
      s.scale = reinterpret_cast<const float*>(w.data + static_cast<int64_t>(w.n) * (k / 8));
      s.scale_stride = 1;
    }
    s.y = y[i];
    s.n = w.n;
    s.tile_begin = w_tiles;
    s.vec_store = (!acc_out && w.n % 8 == 0 && aligned(y[i], 16)) ? 1 : 0;
    w_tiles += (w.n + rows_per_wtile - 1) / rows_per_wtile;
  }
  const int k_steps = (k + kBlockK - 1) / kBlockK;
  const LaunchShape ls = launch_shape(m, w_tiles, k, sms, pair, variant);
  const int tok_tile = ls.tok_tile;
  const bool split = ls.split;
  if (int e = make_map_2d(&p.tmap_tok, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, k, m, k, kBlockK,
                          pair ? tok_tile / 2 : tok_tile, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  p.row_scale = row_scale;
  p.wait_limit_ns = g_wait_limit_ns.load();
  p.m = m;
  p.k = k;
  p.tok_tile = tok_tile;
  p.n_seg = n_weights;
  // Every kernel's issue loop is unrolled over a compile-time ring (kGemmRing
  // stages, 3 or 6 TMEM A slots); split-K: the same, each CTA of a cluster
  // half the K steps.
  if (pair) {
    p.k_tiles = k_steps;
    p.stages = kGemmRing;
    p.a_stages = gemm_ring_a_stages(tok_tile);
  } else if (split) {
    p.k_tiles = k_steps / 2;
    p.stages = kGemmRing;
    p.a_stages = gemm_ring_a_stages(tok_tile);
  } else {
    p.k_tiles = k_steps;
    p.stages = kGemmRing;
    p.a_stages = gemm_ring_a_stages(tok_tile);
  }
  p.n_tok_tiles = ls.n_tok_tiles;
  p.w_tiles = w_tiles;
  p.tok_group = ls.tok_group;
  if (ls.total_tiles > 0x7fffffffLL) return fail(W4A4_ERR_UNSUPPORTED, "too many tiles");
  const dim3 grid(ls.grid);
#define W4A4_LAUNCH_GEMM(L, ACC, BIT)                                                          \
  do {                                                                                        \
    if (pair) {                                                                               \
      if (int e = ensure_smem_attr(dev, 1u << (16 + (BIT)), w4a4_gemm_pair_kernel<L, ACC>,     \
                                   kSmemLimit))                                               \
        return e;                                                                             \
      W4A4_CUDA_TRY(launch_kernel(w4a4_gemm_pair_kernel<L, ACC>, grid, dim3(kGemmThreads),    \
                                  gemm_pair_smem_bytes(tok_tile), stream, 2, p));             \
    } else if (split) {                                                                       \
      if (int e = ensure_smem_attr(dev, 1u << (20 + (BIT)), w4a4_gemm_kernel<L, ACC, true>,    \
                                   kSmemLimit))                                               \
        return e;                                                                             \
      W4A4_CUDA_TRY(launch_kernel(w4a4_gemm_kernel<L, ACC, true>, grid, dim3(kGemmThreads),   \
                                  gemm_smem_bytes(tok_tile), stream, 2, p));                  \
    } else {                                                                                  \
      if (int e = ensure_smem_attr(dev, 1u << (BIT), w4a4_gemm_kernel<L, ACC, false>,          \
                                   kSmemLimit))                                               \
        return e;                                                                             \
      W4A4_CUDA_TRY(launch_kernel(w4a4_gemm_kernel<L, ACC, false>, grid, dim3(kGemmThreads),  \
                                  gemm_smem_bytes(tok_tile), stream, 1, p));                  \
    }                                                                                         \
  } while (0)
  if (layout == W4A4_LAYOUT_INT8) {
    const auto go = [&](auto kernel, uint64_t bit) -> int {
      if (int e = ensure_smem_attr(dev, bit, kernel, kSmemLimit)) return e;
      W4A4_CUDA_TRY(launch_kernel(kernel, grid, dim3(kPairI8Threads), gemm_pair_i8_smem_bytes(tok_tile),
                                  stream, 2, p));
      return W4A4_OK;
    };
    if (int e = acc_out ? go(w4a4_gemm_pair_i8_kernel<true>, 1ull << 29)
                        : go(w4a4_gemm_pair_i8_kernel<false>, 1ull << 28))
      return e;
  } else if (wide) {
    const auto go = [&](auto kernel, uint64_t bit) -> int {
      if (int e = ensure_smem_attr(dev, bit, kernel, kSmemLimit)) return e;
      W4A4_CUDA_TRY(launch_kernel(kernel, grid, dim3(kGemmThreads), gemm_smem_bytes(tok_tile), stream, 1, p));
      return W4A4_OK;
    };
    if (int e = layout == W4A4_LAYOUT_ROW_MAJOR ? go(w4a4_gemm_kernel<kRowMajor, false, false, true>, 1ull << 26)
                                                : go(w4a4_gemm_kernel<kFragmentMajor, false, false, true>, 1ull << 27))
      return e;
  } else if (layout == W4A4_LAYOUT_ROW_MAJOR) {
    if (acc_out) W4A4_LAUNCH_GEMM(kRowMajor, true, 4);
    else W4A4_LAUNCH_GEMM(kRowMajor, false, 2);
  } else {
    if (acc_out) W4A4_LAUNCH_GEMM(kFragmentMajor, true, 5);
    else W4A4_LAUNCH_GEMM(kFragmentMajor, false, 3);
  }
#undef W4A4_LAUNCH_GEMM
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

__global__ void pad_rows_kernel(const int32_t* __restrict__ src, int32_t n, int32_t sw,
                                int32_t dw, int32_t* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(n) * dw;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / dw;
    const int32_t c = static_cast<int32_t>(i - r * dw);
    dst[i] = c < sw ? src[r * sw + c] : 0;
  }
}

// Device addresses of the no-allocation scratch arrays on the current
// device: looked up once per device, with that device current, and cached.
void* g_noalloc_codes[kMaxDevices];
float* g_noalloc_scales[kMaxDevices];

int noalloc_buffers(void** codes, float** scales) {
  int dev = 0;
  if (int e = current_device(&dev)) return e;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_noalloc_codes[dev]) {
    void* c = nullptr;
    void* sc = nullptr;
    W4A4_CUDA_TRY(cudaGetSymbolAddress(&c, g_w4a4_noalloc_codes));
    W4A4_CUDA_TRY(cudaGetSymbolAddress(&sc, g_w4a4_noalloc_scales));
    g_noalloc_scales[dev] = static_cast<float*>(sc);
    g_noalloc_codes[dev] = c;
  }
  *codes = g_noalloc_codes[dev];
  *scales = g_noalloc_scales[dev];
  return W4A4_OK;
}

}  // namespace
}  // namespace w4a4

using namespace w4a4;

extern "C" {

int w4a4_quant(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate, int32_t staging,
               int32_t codes_format, void* codes, float* row_scale, void* stream) {
  return launch_quant(x, m, k, ldx, rotate, staging, codes_format, codes, row_scale,
                      static_cast<cudaStream_t>(stream));
}

int w4a4_gemm(const void* codes, const float* row_scale, int64_t m, int32_t k, int32_t n_weights,
              const w4a4_weight* weights, void* const* y, void* stream) {
  return launch_gemm(codes, row_scale, m, k, n_weights, weights, y,
                     static_cast<cudaStream_t>(stream));
}

int w4a4_gemm_accumulators(const void* codes, int64_t m, int32_t k, int32_t n_weights,
                           const w4a4_weight* weights, int32_t* const* acc, void* stream) {
  return launch_gemm(codes, nullptr, m, k, n_weights, weights,
                     reinterpret_cast<void* const*>(acc), static_cast<cudaStream_t>(stream), true);
}

int w4a4_int4_gemm(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate,
                   int32_t staging, int32_t n_weights, const w4a4_weight* weights, void* const* y,
                   void* codes_scratch, float* scale_scratch, void* stream) {
  // Validate the weights before launching anything.
  if (n_weights < 1 || n_weights > kMaxSegments)
    return fail(W4A4_ERR_INVALID, "n_weights must be 1..%d, got %d", kMaxSegments, n_weights);
  if (!weights) return fail(W4A4_ERR_INVALID, "null weights array");
  if (k > 0 && k % 64 == 0)
    for (int i = 0; i < n_weights; ++i)
      if (int e = check_weight(weights[i], k, i)) return e;
  if (int e = launch_quant(x, m, k, ldx, rotate, staging, W4A4_CODES_GEMM, codes_scratch,
                           scale_scratch, static_cast<cudaStream_t>(stream)))
    return e;
  return launch_gemm(codes_scratch, scale_scratch, m, k, n_weights, weights, y,
                     static_cast<cudaStream_t>(stream));
}

int w4a4_int4_gemm_noalloc(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate,
                           int32_t staging, int32_t n_weights, const w4a4_weight* weights,
                           void* const* y, void* stream) {
  if (m < 0 || k <= 0) return fail(W4A4_ERR_INVALID, "invalid shape M=%lld K=%d", (long long)m, k);
  if (m > W4A4_NOALLOC_MAX_ROWS || m * static_cast<int64_t>(k) > W4A4_NOALLOC_MAX_CODES)
    return fail(W4A4_ERR_UNSUPPORTED,
                "w4a4_int4_gemm_noalloc: M=%lld x K=%d exceeds its static scratch (at most %d rows "
                "and %d codes); use w4a4_int4_gemm with caller-provided scratch",
                (long long)m, k, W4A4_NOALLOC_MAX_ROWS, W4A4_NOALLOC_MAX_CODES);
  void* codes = nullptr;
  float* scales = nullptr;
  if (int e = noalloc_buffers(&codes, &scales)) return e;
  return w4a4_int4_gemm(x, m, k, ldx, rotate, staging, n_weights, weights, y, codes, scales, stream);
}

int w4a4_rmsnorm_quant(const void* x, int64_t ldx, const void* delta, int64_t ldd,
                       const float* gain, float eps, void* x_out, int64_t ldo, void* h_out,
                       int64_t ldh, int64_t m, int32_t k, int32_t staging, int32_t codes_format,
                       void* codes, float* row_scale, void* stream) {
  return launch_rmsnorm_quant(x, ldx, delta, ldd, gain, eps, x_out, ldo, h_out, ldh, m, k, staging,
                              codes_format, codes, row_scale, static_cast<cudaStream_t>(stream));
}

int w4a4_geglu_quant(const void* gate, const void* up, int64_t m, int32_t k, int64_t ld,
                     int32_t staging, int32_t codes_format, void* codes, float* row_scale,
                     void* h_out, int64_t ldh, void* stream) {
  return launch_geglu_quant(gate, up, m, k, ld, staging, codes_format, codes, row_scale, h_out, ldh,
                            static_cast<cudaStream_t>(stream));
}

int w4a4_rope(const void* x, int64_t ldx, void* out, int64_t ldo, const void* cos_t,
              const void* sin_t, int64_t m, int32_t heads, void* stream) {
  return launch_rope(x, ldx, out, ldo, cos_t, sin_t, m, heads, static_cast<cudaStream_t>(stream));
}

int w4a4_prefix_attention(void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                          int64_t ldv, const uint8_t* key_valid, const int32_t* kv_len, int32_t batch,
                          int32_t seq, int32_t heads, void* vt_scratch, void* out, int64_t ldo,
                          const void* cos_t, const void* sin_t, void* k_out, int64_t ldko, void* stream) {
  return launch_attention(q, ldq, k, ldk, v, ldv, key_valid, kv_len, batch, seq, heads, vt_scratch, out,
                          ldo, cos_t, sin_t, k_out, ldko, static_cast<cudaStream_t>(stream));
}

int w4a4_geglu(const void* gate, const void* up, int64_t m, int32_t n, int64_t ld, void* h,
               int64_t ldh, void* stream) {
  return launch_geglu(gate, up, m, n, ld, h, ldh, static_cast<cudaStream_t>(stream));
}

int w4a4_ada_rms_norm_bf16(const void* x, void* y, int64_t rows, int32_t h, int32_t rows_per_batch,
                           const float* scale1, const float* shift, int64_t mod_stride, float eps,
                           void* stream) {
  return launch_ada_rms_norm_bf16(x, y, rows, h, rows_per_batch, scale1, shift, mod_stride, eps,
                                  static_cast<cudaStream_t>(stream));
}

int w4a4_rope_qk_bf16(void* q, int64_t ldq, int32_t heads_q, void* k, int64_t ldk, int32_t heads_k,
                      const void* cos_t, const void* sin_t, int64_t rows, int32_t hd, void* stream) {
  return launch_rope_qk_bf16(q, ldq, heads_q, k, ldk, heads_k, cos_t, sin_t, rows, hd,
                             static_cast<cudaStream_t>(stream));
}

int w4a4_layer_norm_bf16(const void* x, void* y, int64_t rows, int32_t h, const void* w, const void* b,
                         float eps, void* stream) {
  return launch_layer_norm_bf16(x, y, rows, h, w, b, eps, static_cast<cudaStream_t>(stream));
}

int w4a4_quant_segments(const void* x, int64_t m, int32_t k, int32_t seg, int64_t ld,
                        int64_t seg_stride, int32_t staging, int32_t codes_format, void* codes,
                        float* row_scale, void* stream) {
  return launch_quant_segments(x, m, k, seg, ld, seg_stride, staging, codes_format, codes, row_scale,
                               static_cast<cudaStream_t>(stream));
}

int w4a4_prefix_tables(const uint8_t* pad, int32_t batch, int32_t seq, const float* inv_freq,
                       int32_t half, uint8_t* key_valid, int32_t* kv_len, void* cos_t, void* sin_t,
                       void* stream) {
  return launch_prefix_tables(pad, batch, seq, inv_freq, half, key_valid, kv_len, cos_t, sin_t,
                              static_cast<cudaStream_t>(stream));
}

int w4a4_pack_weight(const void* w, int32_t dtype, int64_t ldw, int32_t n, int32_t k, int32_t rotate,
                     int32_t layout, int32_t* out, int32_t out_row_words, void* stream) {
  if (k <= 0 || k % 64 != 0) return fail(W4A4_ERR_INVALID, "K must be a multiple of 64, got %d", k);
  if (k > kPackMaxK) return fail(W4A4_ERR_UNSUPPORTED, "pack_weight supports K <= %d, got %d", kPackMaxK, k);
  if (n < 0) return fail(W4A4_ERR_INVALID, "N must be non-negative, got %d", n);
  if (dtype != kPackF32 && dtype != kPackF16 && dtype != kPackBF16)
    return fail(W4A4_ERR_INVALID, "unknown weight dtype %d", dtype);
  if (rotate != W4A4_ROTATE_BY_K && rotate != 0 && rotate != 1)
    return fail(W4A4_ERR_INVALID, "rotate must be -1 (by K), 0 or 1, got %d", rotate);
  const bool rot = rotate == W4A4_ROTATE_BY_K ? (k == 1024 || k == 2048 || k == 16384) : rotate == 1;
  if (rot && (k & (k - 1))) return fail(W4A4_ERR_INVALID, "rotation needs a power-of-two K, got %d", k);
  if (ldw < k) return fail(W4A4_ERR_INVALID, "weight row stride %lld < K", (long long)ldw);
  if (layout == W4A4_LAYOUT_ROW_MAJOR) {
    if (out_row_words < k / 8 + 1)
      return fail(W4A4_ERR_INVALID, "row-major packed rows need >= K/8+1 words, got %d", out_row_words);
  } else if (layout == W4A4_LAYOUT_FRAGMENT_MAJOR) {
    if (out_row_words != k / 8 + 9 || k % 16 != 0 || n % 2 != 0)
      return fail(W4A4_ERR_INVALID, "fragment-major packing needs the K/8+9 stride, K %% 16 == 0 and an even N");
  } else {
    return fail(W4A4_ERR_INVALID, "unknown weight layout %d", layout);
  }
  if (n == 0) return ok();
  if (!w || !out) return fail(W4A4_ERR_INVALID, "null pointer argument");
  int dev;
  if (int e = current_device(&dev)) return e;
  const int smem = k * 4;
  if (int e = ensure_smem_attr(dev, 1ull << 53, pack_weight_kernel, kPackMaxK * 4)) return e;
  const float isk = static_cast<float>(1.0 / std::sqrt(static_cast<double>(k)));
  pack_weight_kernel<<<static_cast<unsigned>(n), kPackThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      w, dtype, ldw, n, k, rot ? 1 : 0, isk, layout == W4A4_LAYOUT_ROW_MAJOR ? 0 : 1, out, out_row_words);
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int w4a4_repack_int8(const w4a4_weight* src, int32_t k, int32_t* dst, void* stream) {
  if (!src || !dst) return fail(W4A4_ERR_INVALID, "null pointer argument");
  if (k <= 0 || k % 64 != 0) return fail(W4A4_ERR_INVALID, "K must be a multiple of 64, got %d", k);
  if (k > kMagicMaxK) return fail(W4A4_ERR_UNSUPPORTED, "int8 weights support K <= %d", kMagicMaxK);
  if (src->layout == W4A4_LAYOUT_INT8) return fail(W4A4_ERR_INVALID, "the source is already int8");
  if (int e = check_weight(*src, k, 0)) return e;
  if (!aligned(dst, 16)) return fail(W4A4_ERR_INVALID, "dst must be 16-byte aligned");
  const int64_t total = static_cast<int64_t>(src->n) * (k / 8 + 1);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 4096));
  repack_int8_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src->data, src->n, k, src->row_words, src->layout == W4A4_LAYOUT_ROW_MAJOR ? kRowMajor : kFragmentMajor,
      dst);
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int w4a4_pad_rows(const int32_t* src, int32_t n, int32_t src_row_words, int32_t dst_row_words,
                  int32_t* dst, void* stream) {
  if (n < 0 || src_row_words <= 0 || dst_row_words < src_row_words)
    return fail(W4A4_ERR_INVALID, "invalid pad: n=%d, %d -> %d words", n, src_row_words, dst_row_words);
  if (n == 0) return ok();
  if (!src || !dst) return fail(W4A4_ERR_INVALID, "null pointer argument");
  const int64_t total = static_cast<int64_t>(n) * dst_row_words;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  pad_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(src, n, src_row_words,
                                                                         dst_row_words, dst);
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int w4a4_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::strncpy(buf, t_last_error.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return t_last_status;
}

int w4a4_device_error(uint32_t* bits, int32_t clear) {
  if (!bits) return fail(W4A4_ERR_INVALID, "null output pointer");
  W4A4_CUDA_TRY(cudaDeviceSynchronize());
  unsigned v = 0;
  W4A4_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_w4a4_device_error, sizeof(v)));
  *bits = v;
  if (clear) {
    const unsigned zero = 0;
    W4A4_CUDA_TRY(cudaMemcpyToSymbol(g_w4a4_device_error, &zero, sizeof(zero)));
  }
  return ok();
}

int w4a4_gemm_plan(int64_t m, int32_t k, int32_t n_weights, const int32_t* n, int32_t sms,
                   int32_t variant, int32_t layout, int32_t* out) {
  if (m <= 0 || k <= 0 || k % 64 != 0 || sms < 2 || !n || !out)
    return fail(W4A4_ERR_INVALID, "invalid plan query");
  if (n_weights < 1 || n_weights > kMaxSegments)
    return fail(W4A4_ERR_INVALID, "n_weights must be 1..%d, got %d", kMaxSegments, n_weights);
  if (variant < W4A4_GEMM_SINGLE_CTA || variant > W4A4_GEMM_SPLIT_K)
    return fail(W4A4_ERR_INVALID, "unknown GEMM variant %d", variant);
  if (layout != W4A4_LAYOUT_ROW_MAJOR && layout != W4A4_LAYOUT_FRAGMENT_MAJOR)
    return fail(W4A4_ERR_INVALID, "unknown weight layout %d", layout);
  const bool pair = use_pair_kernel(variant, layout, m);
  const int rows_per_wtile = pair ? 2 * kBlockW : kBlockW;
  int w_tiles = 0;
  for (int i = 0; i < n_weights; ++i) {
    if (n[i] <= 0) return fail(W4A4_ERR_INVALID, "N must be positive");
    w_tiles += (n[i] + rows_per_wtile - 1) / rows_per_wtile;
  }
  const LaunchShape ls = launch_shape(m, w_tiles, k, sms, pair, variant);
  out[0] = ls.tok_tile;
  out[1] = ls.split ? 1 : 0;
  out[2] = static_cast<int32_t>(ls.grid);
  out[3] = ls.n_tok_tiles;
  out[4] = ls.tok_group;
  out[5] = w_tiles;
  return ok();
}

int w4a4_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) return fail(W4A4_ERR_INVALID, "wait limit must be positive");
  g_wait_limit_ns.store(limit_ns);
  return ok();
}

int w4a4_set_gemm_variant(int32_t variant) {
  if (variant != W4A4_GEMM_SINGLE_CTA && variant != W4A4_GEMM_CTA_PAIR &&
      variant != W4A4_GEMM_NO_SPLIT && variant != W4A4_GEMM_SPLIT_K)
    return fail(W4A4_ERR_INVALID, "unknown GEMM variant %d", variant);
  g_gemm_variant.store(variant);
  return ok();
}

int w4a4_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(W4A4_ERR_INVALID, "self-test limit must be in (0, 10 s]");
  w4a4_selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns);
  W4A4_CUDA_TRY(cudaGetLastError());
  return ok();
}

int w4a4_version(void) { return 100; }

}  // extern "C"

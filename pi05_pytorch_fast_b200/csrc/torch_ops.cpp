// torch_ops.cpp -- the five pi05_w4a4 PyTorch ops, implemented in C++ on
// top of the C ABI of libw4a4_sm100.so (include/w4a4_sm100.h).
//
// Reference interface replaced (paths relative to harrysocool/pi05-pytorch-fast):
//   pi05_fast/w4a4/extension.py:78-143   torch.library.custom_op registration of
//                                         int4_gemm, int4_gemm_tiled, int4_gemm2,
//                                         int4_gemm2_tiled, int4_gemm3
//   pi05_fast/w4a4/csrc/int4_gemm.cu:487-501, :570-577, :618-642
//                                         argument checks (same TORCH_CHECK text)
//                                         and the op bodies
//
// The schemas (the reference's, as custom_op(..., mutates_args=()) derives
// them from its Python signatures) and the fake (shape) implementations are
// defined from Python, in w4a4/extension.py; this library only registers the
// bodies, under CompositeExplicitAutograd, so CPU tensors reach the checks
// below and fail with the reference's message instead of a dispatcher error.
//
// Why C++: a Python op body (checks, allocations, a ctypes call) costs about
// 10 us of host time per call, which shows whenever the host issues the 72
// ops of a prefix pass more slowly than the GPU runs them.

#include <torch/library.h>

#include <ATen/core/Tensor.h>
#include <ATen/ops/empty.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/util/Exception.h>

#include <array>
#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <string>
#include <tuple>
#include <vector>

#include "w4a4_sm100.h"

namespace {

using at::Tensor;

// PI05_W4A4_STAGING: fp16 (default; the HIP kernel's FWHT rounding) or fp32
// (the CPU emulation's).  Read on every call, like the reference reads it.
int32_t staging_mode() {
  const char* raw = std::getenv("PI05_W4A4_STAGING");
  if (raw == nullptr) return W4A4_STAGING_FP16;
  std::string v(raw);
  size_t b = 0, e = v.size();
  while (b < e && std::isspace(static_cast<unsigned char>(v[b]))) ++b;
  while (e > b && std::isspace(static_cast<unsigned char>(v[e - 1]))) --e;
  v = v.substr(b, e - b);
  for (char& c : v) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
  if (v.empty() || v == "fp16") return W4A4_STAGING_FP16;
  if (v == "fp32") return W4A4_STAGING_FP32;
  TORCH_CHECK(false, "PI05_W4A4_STAGING must be 'fp16' or 'fp32', got '", v, "'");
}

int64_t check_activation(const Tensor& x) {
  TORCH_CHECK(x.is_cuda(), "int4_gemm expects CUDA/HIP tensors");
  TORCH_CHECK(x.scalar_type() == at::kHalf, "int4_gemm activations must be float16");
  TORCH_CHECK(x.dim() > 0 && x.size(-1) > 0,
              "int4_gemm activations need a non-empty last dimension");
  const int64_t k = x.size(-1);
  TORCH_CHECK(k % 64 == 0, "K must be a multiple of 64, got ", k);
  return k;
}

void check_packed(const Tensor& w, int64_t k, const Tensor& x, bool fragment_major) {
  TORCH_CHECK(w.is_cuda(), "packed W must be on CUDA/HIP");
  TORCH_CHECK(w.scalar_type() == at::kInt && w.dim() == 2, "packed W must be int32 [N, K/8+1]");
  TORCH_CHECK(w.size(1) >= k / 8 + 1,
              "packed W second dim must contain K/8 packed words plus a scale");
  TORCH_CHECK(w.device() == x.device(), "packed W is on ", w.device(),
              " but the activations are on ", x.device());
  if (fragment_major) {
    TORCH_CHECK(k == 2048 && w.size(0) == 16384,
                "WMMA-fragment-major weights currently support only K=2048, N=16384");
    TORCH_CHECK(w.size(1) == k / 8 + 9,
                "WMMA-fragment-major weights must use the K/8+9 marker stride");
  }
}

[[noreturn]] void raise_status(int status) {
  char buf[1024];
  w4a4_last_error(buf, sizeof(buf));
  TORCH_CHECK(false, buf, " (status ", status, ")");
}

// The GEMM streams row-major weights with TMA, whose row stride must be a
// multiple of 16 bytes.  The reference's loader pads rows to K/8+8 words
// (apply.py:51, :68-69); any other stride is padded here on every call.
Tensor prepare_row_major(const Tensor& w_in, cudaStream_t stream) {
  Tensor w = w_in.contiguous();
  if ((w.size(1) * 4) % 16 == 0) return w;
  TORCH_WARN_ONCE(
      "pi05_w4a4: packed weight row stride is not a multiple of 4 words; padding it on every "
      "call. Pad once at load (PI05_W4A4_ROW_PAD_WORDS=8, the default) to avoid the copy.");
  const int64_t row_words = (w.size(1) + 3) / 4 * 4;
  Tensor out = at::empty({w.size(0), row_words}, w.options());
  const int st = w4a4_pad_rows(static_cast<const int32_t*>(w.const_data_ptr()),
                               static_cast<int32_t>(w.size(0)), static_cast<int32_t>(w.size(1)),
                               static_cast<int32_t>(row_words),
                               static_cast<int32_t*>(out.data_ptr()), stream);
  if (st != W4A4_OK) raise_status(st);
  return out;
}

// One activation quant shared by N (1..3) GEMMs, one GEMM launch.
template <size_t N>
std::array<Tensor, N> run(const Tensor& x, const std::array<const Tensor*, N>& weights,
                          bool fragment_major) {
  const int64_t k = check_activation(x);
  for (const Tensor* w : weights) check_packed(*w, k, x, fragment_major);

  Tensor x2 = x.contiguous();
  if (reinterpret_cast<uintptr_t>(x2.const_data_ptr()) % 16 != 0)
    x2 = x2.clone(at::MemoryFormat::Contiguous);
  const int64_t m = x2.numel() / k;

  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();

  std::array<Tensor, N> ws;
  std::array<Tensor, N> ys;
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  w4a4_weight desc[N];
  void* outs[N];
  for (size_t i = 0; i < N; ++i) {
    ws[i] = fragment_major ? weights[i]->contiguous() : prepare_row_major(*weights[i], stream);
    shape.back() = ws[i].size(0);
    ys[i] = at::empty(shape, x.options());
    desc[i].data = static_cast<const int32_t*>(ws[i].const_data_ptr());
    desc[i].n = static_cast<int32_t>(ws[i].size(0));
    desc[i].row_words = static_cast<int32_t>(ws[i].size(1));
    desc[i].layout = fragment_major ? W4A4_LAYOUT_FRAGMENT_MAJOR : W4A4_LAYOUT_ROW_MAJOR;
    outs[i] = ys[i].data_ptr();
  }
  if (m == 0) return ys;

  // one scratch allocation: int8 codes [m, k], then fp32 row scales [m]
  const int64_t codes_bytes = (m * k + 255) / 256 * 256;
  Tensor scratch = at::empty({codes_bytes + 4 * m}, x.options().dtype(at::kByte));
  uint8_t* base = static_cast<uint8_t*>(scratch.data_ptr());
  const int st = w4a4_int4_gemm(x2.const_data_ptr(), m, static_cast<int32_t>(k), k,
                                W4A4_ROTATE_BY_K, staging_mode(), static_cast<int32_t>(N), desc,
                                outs, base, reinterpret_cast<float*>(base + codes_bytes), stream);
  if (st != W4A4_OK) raise_status(st);
  return ys;
}

Tensor int4_gemm(const Tensor& x, const Tensor& packed) {
  return run<1>(x, {&packed}, false)[0];
}

Tensor int4_gemm_tiled(const Tensor& x, const Tensor& packed) {
  return run<1>(x, {&packed}, true)[0];
}

std::tuple<Tensor, Tensor> int4_gemm2(const Tensor& x, const Tensor& w0, const Tensor& w1) {
  auto y = run<2>(x, {&w0, &w1}, false);
  return {y[0], y[1]};
}

std::tuple<Tensor, Tensor> int4_gemm2_tiled(const Tensor& x, const Tensor& w0,
                                            const Tensor& w1) {
  auto y = run<2>(x, {&w0, &w1}, true);
  return {y[0], y[1]};
}

std::tuple<Tensor, Tensor, Tensor> int4_gemm3(const Tensor& x, const Tensor& w0,
                                              const Tensor& w1, const Tensor& w2) {
  auto y = run<3>(x, {&w0, &w1, &w2}, false);
  return {y[0], y[1], y[2]};
}

}  // namespace

TORCH_LIBRARY_IMPL(pi05_w4a4, CompositeExplicitAutograd, m) {
  m.impl("int4_gemm", &int4_gemm);
  m.impl("int4_gemm_tiled", &int4_gemm_tiled);
  m.impl("int4_gemm2", &int4_gemm2);
  m.impl("int4_gemm2_tiled", &int4_gemm2_tiled);
  m.impl("int4_gemm3", &int4_gemm3);
}

/*
 * w4a4_sm100.h -- C ABI of libw4a4_sm100.so, the B200 (sm_100a) W4A4
 * prefix-LM GEMM path.
 *
 * Plain C: device pointers, sizes and an opaque CUDA stream handle
 * (cudaStream_t passed as void*; NULL = the legacy default stream).  No torch
 * types.  Every entry point is asynchronous on `stream` (nothing
 * synchronises except w4a4_device_error), returns W4A4_OK or an error code,
 * and on error leaves a message retrievable with w4a4_last_error() (thread
 * local).  All device pointers must belong to the CURRENT CUDA device.
 *
 * Reference interfaces replaced (paths relative to the reference project,
 * harrysocool/pi05-pytorch-fast):
 *   pi05_fast/w4a4/csrc/int4_gemm.cu:496-531  quantize_x      -> w4a4_quant
 *   pi05_fast/w4a4/csrc/int4_gemm.cu:566-616  gemm_from_q     -> w4a4_gemm
 *   pi05_fast/w4a4/csrc/int4_gemm.cu:618-642  int4_gemm{,_tiled,2,2_tiled,3}
 *                                                             -> w4a4_int4_gemm
 *   pi05_fast/w4a4/apply.py:68-69             row padding     -> w4a4_pad_rows
 *   pi05_fast/w4a4/csrc/int4_gemm.cu:487-501  TORCH_CHECK text-> w4a4_last_error
 *   pi05_fast/w4a4/apply.py:126-191           layer glue      -> w4a4_rmsnorm_quant,
 *                                                                w4a4_geglu_quant, w4a4_rope,
 *                                                                w4a4_prefix_attention
 */
#ifndef W4A4_SM100_H_
#define W4A4_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define W4A4_OK 0
#define W4A4_ERR_INVALID 1     /* bad argument (shape, stride, pointer, layout) */
#define W4A4_ERR_UNSUPPORTED 2 /* valid in the reference, not supported here    */
#define W4A4_ERR_CUDA 3        /* a CUDA runtime / driver call failed            */

/* ---- FWHT staging of the activation quant ----
 * FP16: the reference HIP kernel's arithmetic (int4_gemm.cu:404-426).
 * FP32: the reference CPU emulation's arithmetic (pack.py:113-131). */
#define W4A4_STAGING_FP16 0
#define W4A4_STAGING_FP32 1

/* ---- activation code formats written by w4a4_quant ----
 * INT8:   one signed code per byte, row-major [M, K], natural order.
 * PACKED: the reference's int32 words [M, K/8], element j at bits 4j.
 * GEMM:   one signed code per byte, row-major [M, K], each group of 8
 *         elements stored in the order 0,2,4,6,1,3,5,7 (what w4a4_gemm reads;
 *         it matches the K order of the GEMM's in-register nibble expansion). */
#define W4A4_CODES_INT8 0
#define W4A4_CODES_PACKED 1
#define W4A4_CODES_GEMM 2

/* ---- weight layouts (the reference's in-memory formats) ----
 * ROW_MAJOR: int32 [N, row_words], word p of row n holds k = 8p..8p+7
 *   (element j at bits 4j), word K/8 holds the fp32 scale bits
 *   (pack.py:85-101); row_words >= K/8+1.  w4a4_gemm needs row_words*4 to be
 *   a multiple of 16 (the default load-time pad K/8+8 is); pad others with
 *   w4a4_pad_rows.
 * FRAGMENT_MAJOR: payload flat as [K/16][N][2 words], then N fp32 scales,
 *   inside a tensor declared [N, K/8+9] (pack.py:45-68). */
#define W4A4_LAYOUT_ROW_MAJOR 0
#define W4A4_LAYOUT_FRAGMENT_MAJOR 1
/* INT8: either layout repacked once by w4a4_repack_int8 (no reference
 *   counterpart; the load-time "Blackwell tile order"): int32 [N, K/4+4], a
 *   row = K int8 values (16 x code, in the GEMM's K byte order), then the
 *   fp32 scale and three zero words.  Runs on the CTA-pair kernel with both
 *   MMA operands in shared memory. */
#define W4A4_LAYOUT_INT8 2

/* variant argument of w4a4_set_gemm_variant */
#define W4A4_GEMM_SINGLE_CTA 0 /* single-CTA kernel; split-K where the planner finds it faster */
#define W4A4_GEMM_CTA_PAIR 1   /* tcgen05 cta_group::2 kernel                                 */
#define W4A4_GEMM_NO_SPLIT 2   /* single-CTA kernel, never split-K                            */
#define W4A4_GEMM_SPLIT_K 3    /* split-K whenever possible: even K-step count, <= 1 tile per cluster */

/* rotate argument of w4a4_quant */
#define W4A4_ROTATE_BY_K (-1) /* rotate iff K in {1024, 2048, 16384}: the op's dispatch */

typedef struct w4a4_weight {
  const int32_t* data; /* device pointer to the packed tensor's storage      */
  int32_t n;           /* output features (tensor size(0))                   */
  int32_t row_words;   /* tensor size(1)                                     */
  int32_t layout;      /* W4A4_LAYOUT_*                                      */
} w4a4_weight;

/* Fused Hadamard rotation + per-token symmetric INT4 quantisation.
 * Replaces quantize_x / quant_rot_rb / quant_rows (int4_gemm.cu:396-531).
 *   x          fp16 [m, k], row stride ldx elements (ldx >= k, ldx % 8 == 0,
 *              16-byte aligned base)
 *   k          > 0, multiple of 64
 *   rotate     W4A4_ROTATE_BY_K, 0 (never) or 1 (k must be 1024/2048/16384)
 *   staging    W4A4_STAGING_*
 *   codes      int8 [m, k] or int32 [m, k/8] (codes_format), 8-byte aligned
 *   row_scale  fp32 [m]: sdiv/sqrt(k) when rotated, sdiv otherwise          */
int w4a4_quant(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate,
               int32_t staging, int32_t codes_format, void* codes, float* row_scale,
               void* stream);

/* W4A4 GEMM of int8 activation codes against 1..3 packed weights that share
 * them (one launch).  Replaces gemm_from_q / gemm_iu4 / gemm_iu4_shape
 * (int4_gemm.cu:66-394, :566-616).
 *   codes      int8 [m, k] from w4a4_quant (W4A4_CODES_GEMM), 16-byte aligned
 *   row_scale  fp32 [m]
 *   weights    n_weights descriptors, all the same layout, all K = k
 *   y          n_weights fp16 outputs, y[i] is [m, weights[i].n] row-major  */
int w4a4_gemm(const void* codes, const float* row_scale, int64_t m, int32_t k,
              int32_t n_weights, const w4a4_weight* weights, void* const* y, void* stream);

/* Test hook: the same GEMM, but writes the raw int32 accumulators
 * acc[i] = int32 [m, weights[i].n] (sum_k qa*qw, before any scaling) so
 * tests can check them bit-exactly; row scales are not used. */
int w4a4_gemm_accumulators(const void* codes, int64_t m, int32_t k, int32_t n_weights,
                           const w4a4_weight* weights, int32_t* const* acc, void* stream);

/* The reference's op contract in one call: quantise x once, then run the
 * GEMM against every weight (int4_gemm: 1, int4_gemm2: 2, int4_gemm3: 3
 * weights; int4_gemm.cu:618-642).  The caller provides the intermediate
 * buffers: codes_scratch int8 [m, k] (16-byte aligned) and
 * scale_scratch fp32 [m].  rotate = W4A4_ROTATE_BY_K gives the op's behaviour. */
int w4a4_int4_gemm(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate,
                   int32_t staging, int32_t n_weights, const w4a4_weight* weights,
                   void* const* y, void* codes_scratch, float* scale_scratch, void* stream);

/* No counterpart in the reference: w4a4_int4_gemm without caller-provided
 * scratch.  The intermediate codes and row scales live in file-scope static
 * device arrays of the library (at most W4A4_NOALLOC_MAX_ROWS rows and
 * W4A4_NOALLOC_MAX_CODES = m * k codes; larger calls fail with
 * W4A4_ERR_UNSUPPORTED), so the call allocates nothing.  Every call on a
 * device shares that one scratch: calls that may overlap in time (other
 * streams, other threads, or another launch before this one's GEMM has read
 * the codes) race.  The arrays' addresses are looked up on the first call on
 * each device; make that first call before any CUDA graph capture. */
#define W4A4_NOALLOC_MAX_ROWS 65536
#define W4A4_NOALLOC_MAX_CODES (16 * 1024 * 1024)
int w4a4_int4_gemm_noalloc(const void* x, int64_t m, int32_t k, int64_t ldx, int32_t rotate,
                           int32_t staging, int32_t n_weights, const w4a4_weight* weights,
                           void* const* y, void* stream);

/* ---- prefix-LM layer glue fused with the quant that follows it ----
 * The reference runs this glue as PyTorch ops between its pi05_w4a4 calls
 * (pi05_fast/w4a4/apply.py:126-191 over transformers' GemmaDecoderLayer:
 * input_layernorm / post_attention_layernorm, the residual adds,
 * apply_rotary_pos_emb, act_fn(gate) * up). */

/* Residual add + Gemma RMSNorm + activation quant of K = 2048 rows.
 * Replaces `residual + hidden_states`, GemmaRMSNorm.forward and the
 * following quantize_x (int4_gemm.cu:496-531) of the q/k/v and gate/up
 * inputs.  Per row: s = fl16(x + delta) (delta may be NULL: s = x), written
 * to x_out when not NULL (x_out may equal x); h = fl16(s * rsqrt(mean(s^2)
 * + eps) * gain) in fp32 (gain = 1 + weight, fp32 [k], 16-byte aligned),
 * written to h_out when not NULL; when codes is not NULL, the codes and row
 * scale of h exactly as w4a4_quant(h, rotate = 1, staging, codes_format)
 * computes them.  codes == NULL is the norm alone (then h_out is required).
 * Rows: 16-byte aligned, strides >= k and multiples of 8 elements. */
int w4a4_rmsnorm_quant(const void* x, int64_t ldx, const void* delta, int64_t ldd,
                       const float* gain, float eps, void* x_out, int64_t ldo, void* h_out,
                       int64_t ldh, int64_t m, int32_t k, int32_t staging, int32_t codes_format,
                       void* codes, float* row_scale, void* stream);

/* GeGLU + activation quant of the down_proj input (K = 16384).  Replaces
 * `act_fn(gate) * up` (apply.py:138, F.gelu(approximate="tanh") on fp16)
 * and the following quantize_x.  h = fl16(fl16(gelu_tanh(gate)) * up), the
 * rounding of PyTorch's eager CUDA ops; its codes and row scale exactly as
 * w4a4_quant(h, rotate = 1, staging, codes_format) computes them; h itself
 * is written to h_out when not NULL.  gate and up share the row stride ld. */
int w4a4_geglu_quant(const void* gate, const void* up, int64_t m, int32_t k, int64_t ld,
                     int32_t staging, int32_t codes_format, void* codes, float* row_scale,
                     void* h_out, int64_t ldh, void* stream);

/* The per-forward tables of a batch of prefixes from its pad mask (uint8
 * [batch, seq], 1 = real token): key_valid (a byte copy of the mask),
 * kv_len[b] = last real token + 1, and the rotary tables cos_t / sin_t fp16
 * [batch * seq, 2 * half] at position cumsum(pad) - 1: cos / sin of
 * fl32(pos * inv_freq[i]), i < half, repeated over both halves.  Replaces
 * the position ids and rotary embedding of the reference's prefix pass
 * (lerobot's cumsum position ids; transformers' GemmaRotaryEmbedding). */
int w4a4_prefix_tables(const uint8_t* pad, int32_t batch, int32_t seq, const float* inv_freq,
                       int32_t half, uint8_t* key_valid, int32_t* kv_len, void* cos_t, void* sin_t,
                       void* stream);

/* Rotary position embedding of `heads` heads of width 256 in each of m rows
 * (apply_rotary_pos_emb: q * cos + rotate_half(q) * sin, each product and
 * the sum rounded to fp16).  cos_t / sin_t: fp16 [m, 256], row stride 256.
 * out may equal x. */
int w4a4_rope(const void* x, int64_t ldx, void* out, int64_t ldo, const void* cos_t,
              const void* sin_t, int64_t m, int32_t heads, void* stream);

/* ---- N-sharded gate/up (tensor-parallel MLP over P GPUs) ----
 * No counterpart in the reference, which runs on one GPU: a rank holding a
 * column shard [M, N/P] of gate and up forms its part of h with w4a4_geglu,
 * the ranks exchange row blocks (an all-to-all, NCCL), and each rank
 * quantises its complete rows straight from the P received segments with
 * w4a4_quant_segments. */

/* h = fl16(fl16(gelu_tanh(gate)) * up) elementwise over [m, n] (n a multiple
 * of 8; the rounding of w4a4_geglu_quant and of PyTorch's eager ops). */
int w4a4_geglu(const void* gate, const void* up, int64_t m, int32_t n, int64_t ld, void* h,
               int64_t ldh, void* stream);

/* w4a4_quant of K = 16384 rows (rotated) whose elements are stored as
 * K / seg segments: element e of row r at x + (e / seg) * seg_stride +
 * r * ld + e % seg (seg a multiple of 64 dividing K; ld >= seg; seg_stride >=
 * m * ld).  Codes and scales are those w4a4_quant gives the contiguous rows. */
int w4a4_quant_segments(const void* x, int64_t m, int32_t k, int32_t seg, int64_t ld,
                        int64_t seg_stride, int32_t staging, int32_t codes_format, void* codes,
                        float* row_scale, void* stream);

/* Bidirectional prefix attention with one shared key/value head (Gemma-2B:
 * 8 query heads, 1 kv head, head_dim 256) on the tensor cores.  Replaces
 * the reference's eager attention (apply.py:170-188, transformers'
 * eager_attention_forward) under lerobot's prefix mask: query i of
 * observation b sees key j iff key_valid[b, i] and key_valid[b, j]; a query
 * with key_valid 0 averages all seq values (its all-masked fp32 softmax is
 * uniform).  Scores in fp32 (scale 1/16 = 256^-0.5), softmax in fp32,
 * probabilities rounded to fp16 for the P V product, fp32 accumulation.
 *   q          fp16 [batch * seq, ldq], heads x 256 per row (after RoPE)
 *   k, v       fp16 [batch * seq, ldk / ldv], 256 per row (k after RoPE)
 *   key_valid  uint8 [batch, seq] (1 = real token)
 *   kv_len     int32 [batch]: every key at or past kv_len[b] is padding
 *   vt_scratch fp16 [batch, 256, W4A4_ATTN_VT_STRIDE(seq)]: V transposed
 *   out        fp16 [batch * seq, ldo], heads x 256 per row
 *   cos_t, sin_t  NULL: q and k are used as given; else fp16 [batch * seq,
 *              256] rotary tables: q is rotated in place and k into k_out
 *              [batch * seq, ldko] (k_out may equal k; it is the KV cache's
 *              key rows) in the first launch, with w4a4_rope's arithmetic,
 *              and the attention reads them
 * heads must divide 128; seq <= 4096.  Two launches (RoPE + V transpose,
 * attention). */
#define W4A4_ATTN_VT_STRIDE(seq) ((((int64_t)(seq)) + 7) / 8 * 8)
int w4a4_prefix_attention(void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                          int64_t ldv, const uint8_t* key_valid, const int32_t* kv_len, int32_t batch,
                          int32_t seq, int32_t heads, void* vt_scratch, void* out, int64_t ldo,
                          const void* cos_t, const void* sin_t, void* k_out, int64_t ldko,
                          void* stream);

/* Load-time weight pack on the GPU: Linear.weight [n, k] (row stride ldw
 * elements; dtype 0 = fp32, 1 = fp16, 2 = bf16) -> the reference's packed INT4
 * weight, bit for bit (pi05_fast/w4a4/pack.py:85-101 pack_linear_weight; the
 * fragment-major order of :45-68 preshuffle_wmma_weight): fp32 FWHT when
 * rotating (rotate = W4A4_ROTATE_BY_K: K in {1024, 2048, 16384}), times
 * fl(1/sqrt K), per-row scale amax/7, codes rint(w/scale) clamped to +-7.
 *   layout W4A4_LAYOUT_ROW_MAJOR: out int32 [n, out_row_words], out_row_words
 *          >= k/8 + 1 (payload, scale word, zero padding: the K/8+8 load-time
 *          pad of apply.py:68-69 included);
 *   layout W4A4_LAYOUT_FRAGMENT_MAJOR: out [n, k/8 + 9] as the preshuffle
 *          writes it (n even).
 * k a multiple of 64, at most 16384. */
int w4a4_pack_weight(const void* w, int32_t dtype, int64_t ldw, int32_t n, int32_t k, int32_t rotate,
                     int32_t layout, int32_t* out, int32_t out_row_words, void* stream);

/* Repack a packed weight (row-major or fragment-major, as w4a4_gemm takes
 * it) into W4A4_LAYOUT_INT8: dst int32 [src->n, k/4 + 4], 16-byte aligned.
 * The GEMM of the repacked weight is bit-identical to that of the packed
 * one.  No reference counterpart (the reference's pack.py:45-68 repack is
 * its WMMA fragment order). */
int w4a4_repack_int8(const w4a4_weight* src, int32_t k, int32_t* dst, void* stream);

/* Copy a row-major packed weight [n, src_row_words] into [n, dst_row_words]
 * (dst_row_words >= src_row_words), zero-filling the new words: the
 * load-time row pad of apply.py:68-69, done on the device. */
int w4a4_pad_rows(const int32_t* src, int32_t n, int32_t src_row_words,
                  int32_t dst_row_words, int32_t* dst, void* stream);

/* Copies the last error message of this thread into buf (NUL-terminated,
 * truncated to len) and returns the last status code. */
int w4a4_last_error(char* buf, size_t len);

/* Reads (and with clear != 0, resets) the current device's error word: a
 * bit mask set by kernels whose bounded waits ran out (0 = no error).
 * Synchronises the device. */
int w4a4_device_error(uint32_t* bits, int32_t clear);

/* Limit, in nanoseconds, of every bounded wait inside kernels launched
 * after this call (default 1e9).  Process-wide. */
int w4a4_set_wait_limit_ns(uint64_t limit_ns);

/* GEMM kernel variant for launches after this call (W4A4_GEMM_*; default
 * W4A4_GEMM_SINGLE_CTA, which also runs fragment-major GEMMs of 768 or more
 * tokens on the CTA pair).  Split-K runs a tile's two K halves on the two CTAs
 * of a cluster and adds the partial sums through distributed shared memory.
 * All variants give bit-identical results.  Process-wide; the environment
 * variable W4A4_GEMM_PAIR=1 sets the initial value to W4A4_GEMM_CTA_PAIR.  No
 * counterpart in the reference, which has one kernel per op. */
int w4a4_set_gemm_variant(int32_t variant);

/* Test hook (host only, no GPU needed): the launch shape w4a4_gemm would use
 * for m tokens, K = k and n_weights weights of n[i] rows in weight layout
 * `layout` (W4A4_LAYOUT_*) on `sms` SMs with GEMM variant `variant`.  out[6]
 * receives the token tile, split-K (0/1), the grid size, the number of token
 * tiles, the token tiles per rasterisation group and the number of weight
 * tiles (of 256 rows when the CTA pair runs).  No counterpart in the
 * reference. */
int w4a4_gemm_plan(int64_t m, int32_t k, int32_t n_weights, const int32_t* n, int32_t sms,
                   int32_t variant, int32_t layout, int32_t* out);

/* Test hook: launches one CTA that waits on a barrier nobody arrives at, with
 * the given limit; the kernel must give up, set its error bit and return. */
int w4a4_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/* ---- bf16 kernels of the config-4 neighbours (SigLIP, the action expert) ----
 * No counterpart in the reference, whose SnapFlow step (pi05_fast/
 * snapflow_pi05.py:127-195) runs lerobot's PI05 policy as PyTorch bf16 ops;
 * each entry point below does in one pass what a chain of those ops does.
 * All arithmetic fp32, each result rounded once to bf16; row-major,
 * 16-byte aligned rows. */

/* pi0.5's adaptive RMSNorm: y[r] = x[r] rsqrt(mean(x[r]^2) + eps) *
 * scale1[b] + shift[b], b = r / rows_per_batch, scale1 = 1 + scale and shift
 * fp32 rows of h at b * mod_stride floats; x, y bf16 [rows, h] contiguous, h a
 * multiple of 256 up to 2048. */
int w4a4_ada_rms_norm_bf16(const void* x, void* y, int64_t rows, int32_t h, int32_t rows_per_batch,
                           const float* scale1, const float* shift, int64_t mod_stride, float eps,
                           void* stream);

/* Rotary position embedding in place (transformers' rotate_half form): q
 * [rows, heads_q, hd] and k [rows, heads_k, hd] (bf16, row strides ldq / ldk
 * elements), cos / sin bf16 [rows, hd] with each half the same angles; for
 * i < hd / 2: (x_i, x_{i+hd/2}) -> (x_i c_i - x_{i+hd/2} s_i,
 * x_{i+hd/2} c_i + x_i s_i).  hd a multiple of 16. */
int w4a4_rope_qk_bf16(void* q, int64_t ldq, int32_t heads_q, void* k, int64_t ldk, int32_t heads_k,
                      const void* cos_t, const void* sin_t, int64_t rows, int32_t hd, void* stream);

/* LayerNorm: y = (x - mean) rsqrt(var + eps) w + b per row of x bf16 [rows, h]
 * (contiguous; h a multiple of 8 up to 2048), w and b bf16 [h]. */
int w4a4_layer_norm_bf16(const void* x, void* y, int64_t rows, int32_t h, const void* w, const void* b,
                         float eps, void* stream);

/* Library ABI version (major * 100 + minor). */
int w4a4_version(void);

#ifdef __cplusplus
}
#endif

#endif /* W4A4_SM100_H_ */

/*
 * gguf_b200.h - C ABI of the B200 GGUF weight-preparation library (libgguf_b200.so).
 *
 * The library turns GGUF block-quantized tensor bytes into the integer weight layout
 * LLiMa's model compiler hands to the Modalix compile step, on NVIDIA B200 (sm_100a):
 *
 *   Q8_0 -> f32 block scales (per 32) + int8 codes            (unpack_q8_0)
 *   Q4_0 -> f32 block scales (per 32) + int4 codes, 1 byte each (unpack_q4, SYMMETRIC)
 *   Q4_K, Q5_K -> f32 scales (per 32) + int8 codes, through the asymmetric -> symmetric
 *                 requantization (unpack_k_quant + convert_to_simple_block_quant)
 *   Q6_K -> f32 scales (per 16) + int8 codes                   (same path, no requant)
 *   Q5_0 -> f32 scales (per 32) + int8 codes q - 16           (unpack_q5, SYMMETRIC)
 *   Q4_1, Q5_1 -> f32 scales (per 32) + int8 codes via requantize_symmetric
 *   Q2_K -> f32 scales (per 16) + int8 codes via the K-quant requantization
 *   Q3_K -> f32 scales (per 16) + int8 codes q - 4
 *   F32 / F16 / BF16 -> copied unchanged
 *
 * and, on request, into f32 values exactly as gguf-py's dequantize computes them (the
 * reference's force_float path).  Results are bit-identical to the reference's numpy
 * path.  Reference interfaces replaced, in sima-neat/llima 0.6.2:
 *
 *   gq_convert / gq_convert_batch   sima_lmm/gguf/gguf_conversion.py:102-176
 *                                   (unpack_gguf_tensor), with the q/k head permutation of
 *                                   GgufModel._permute_qk_proj (gguf_conversion.py:314-332)
 *                                   fused into the output indexing
 *   gq_requantize_symmetric         sima_lmm/gguf/ggml_quant.py:785-886 (requantize_symmetric)
 *   gq_query                        sizes implied by ggml_quant.py:104-131 (format table)
 *   gq_convert_host                 the same as gq_convert_batch, on host buffers
 *   gq_convert_modalix(_batch)      unpack_gguf_tensor followed by ModelGraph._build_conv's
 *                                   layout (sima_lmm/model/model_graph.py:1012-1079), fused
 *   gq_unpack_fields                sima_lmm/gguf/ggml_quant.py:567-694 (unpack_k_quant) and
 *                                   :174-271 (unpack_q4 / unpack_q5, ASYMMETRIC)
 *   gq_remove_superblocks           sima_lmm/gguf/ggml_quant.py:739-782 (remove_superblocks)
 *
 * Conventions: every function returns GQ_OK (0) or a negative GQ_ERR_* code and never
 * aborts; gq_strerror() describes a code.  Device pointers are plain CUDA device
 * addresses of the current device; `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Work is enqueued on `stream` and the call returns without waiting, except
 * gq_convert_host which returns when its results are in host memory.
 */
#ifndef GGUF_B200_H
#define GGUF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GQ_ABI_VERSION 2

#if defined(__GNUC__)
#define GQ_API __attribute__((visibility("default")))
#else
#define GQ_API
#endif

/* status codes */
#define GQ_OK 0
#define GQ_ERR_TYPE (-1)      /* GGML type not handled by this path */
#define GQ_ERR_SIZE (-2)      /* sizes inconsistent with the type's block geometry */
#define GQ_ERR_ALIGN (-3)     /* a pointer is not aligned as required */
#define GQ_ERR_NULL (-4)      /* a pointer the requested outputs need is NULL */
#define GQ_ERR_ARG (-5)       /* other invalid argument (mode, count, head count) */
#define GQ_ERR_CUDA (-6)      /* CUDA runtime error; see gq_last_cuda_error() */
#define GQ_ERR_NOMEM (-7)     /* device or pinned host allocation failed */

/* GGML type ids: the numbers of QuantizationMode, sima_lmm/gguf/ggml_quant.py:9-26 */
#define GQ_TYPE_F32 0
#define GQ_TYPE_F16 1
#define GQ_TYPE_Q4_0 2
#define GQ_TYPE_Q4_1 3
#define GQ_TYPE_Q5_0 6
#define GQ_TYPE_Q5_1 7
#define GQ_TYPE_Q8_0 8
#define GQ_TYPE_Q2_K 10
#define GQ_TYPE_Q3_K 11
#define GQ_TYPE_Q4_K 12
#define GQ_TYPE_Q5_K 13
#define GQ_TYPE_Q6_K 14
#define GQ_TYPE_BF16 30

/* outputs (bit mask) */
#define GQ_OUT_CODES 1        /* f32 block scales + integer codes (force_float=False) */
#define GQ_OUT_F32 2          /* f32 values as gguf-py dequantize computes them (force_float=True) */

/* Requantization diagnostics of one tensor, accumulated as maxima over its blocks.
 * ggml_quant.py:866-880 computes the same two numbers and logs a warning when
 * clip_err > 0 or round_err > 0.5. */
typedef struct gq_diag {
    uint32_t round_err_bits;  /* bit pattern of the f32 max |int16(rint(r*sf)) - r*sf| (NaN wins) */
    int32_t clip_err;         /* max |clip(q') - q'| */
} gq_diag_t;

/* One tensor to convert.  Shape is (rows, cols) as unpack_gguf_tensor returns it (the
 * reversed GGUF dims); cols must be a multiple of the type's block (32, or 256 for K). */
typedef struct gq_tensor {
    int32_t type;             /* GQ_TYPE_* */
    int32_t perm_heads;       /* >0: apply the llama q/k row permutation for this many heads */
    int64_t rows;
    int64_t cols;
    const void* src;          /* GGUF bytes of the tensor, 16-byte aligned */
    size_t src_bytes;         /* must be >= the tensor's GGUF size */
    void* codes;              /* GQ_OUT_CODES: rows*cols bytes, 16-byte aligned */
    float* scales;            /* GQ_OUT_CODES: rows*cols/block floats (block 32, Q6_K 16) */
    float* values;            /* GQ_OUT_F32: rows*cols floats, 16-byte aligned; float types:
                                 the unchanged copy (rows*cols elements of the type) */
    gq_diag_t* diag;          /* optional; Q4_K/Q5_K with GQ_OUT_CODES accumulate into it */
} gq_tensor_t;

/* Sizes of one tensor's input and outputs. */
typedef struct gq_layout {
    int64_t n_values;
    int64_t n_units;          /* stored blocks / super-blocks */
    int64_t src_bytes;
    int64_t codes_bytes;
    int64_t scales_count;     /* f32 block scales */
    int64_t values_bytes;     /* f32 output (or the float copy) */
    int32_t block_values;     /* values per output scale: 32, 16, or 0 for float types */
    int32_t unit_values;      /* values per stored unit: 1, 32 or 256 */
} gq_layout_t;

GQ_API int gq_version(void);
GQ_API const char* gq_strerror(int status);
/* CUDA error code (cudaError_t) behind the last GQ_ERR_CUDA of the calling thread. */
GQ_API int gq_last_cuda_error(void);

/* Sticky error flags of the conversion kernels on `device`, or-ed over every launch since
 * the last clear.  GQ_KERNEL_WAIT_TIMEOUT: a kernel waited about a second for a tile copy
 * that did not complete and stopped early, so that launch's outputs are incomplete.  The
 * flags live in device memory: read them once the work they should cover has finished.
 * clear != 0 resets them.  No counterpart in the reference (whose numpy path cannot stall).
 * gq_convert_host and gq_convert_host_noalloc read and clear them themselves and fail with
 * GQ_ERR_CUDA (gq_last_cuda_error() = cudaErrorTimeout) when a flag was set. */
#define GQ_KERNEL_WAIT_TIMEOUT 1u
GQ_API int gq_kernel_errors(int32_t device, int32_t clear, uint32_t* flags);

GQ_API int gq_query(int32_t type, int64_t rows, int64_t cols, gq_layout_t* out);

/* Zero `count` diagnostics records (device memory) on `stream`. */
GQ_API int gq_diag_reset(gq_diag_t* diag, int32_t count, void* stream);

/* Convert one tensor (device buffers).  Replaces unpack_gguf_tensor
 * (gguf_conversion.py:102-176) plus, when perm_heads > 0, _permute_qk_proj (:314-332).
 * The tensor's diag, if any, is zeroed first. */
GQ_API int gq_convert(const gq_tensor_t* tensor, int32_t out_mask, void* stream);

/* Convert `count` tensors (device buffers) with one kernel launch per GGML type present.
 * Diagnostics accumulate (max) into each tensor's diag: zero them beforehand. */
GQ_API int gq_convert_batch(const gq_tensor_t* tensors, int32_t count, int32_t out_mask, void* stream);

/* requantize_symmetric (ggml_quant.py:785-886) as a standalone scheme:
 * block_consts (n_blocks, 2) f32 [scale, min]; codes (n_blocks, block) int8 unsigned values;
 * out: scales (n_blocks) f32 and codes (n_blocks, block) in [-2^(bits-1), 2^(bits-1)-1].
 * block must be 1..256 and output_bits 2..8.  All device pointers. */
GQ_API int gq_requantize_symmetric(const float* block_consts, const int8_t* codes, int64_t n_blocks,
                            int32_t block, int32_t output_bits, float* out_scales,
                            int8_t* out_codes, gq_diag_t* diag, void* stream);

/* Modalix weight layout of converted weights (ModelGraph._build_conv,
 * sima_lmm/model/model_graph.py:1012-1079): codes (rows = output channels, cols = input
 * channels, one byte each: int8 or int4-in-byte) -> out_codes (cols, rows_padded), the
 * memory order of the HWIGO weight (1, 1, cols, 1, rows_padded); scales (rows, cols/block)
 * f32 -> out_scales (cols/block, rows_padded).  Output channels rows..rows_padded-1 are
 * filled with zero codes and unit scales (the int4 32-way output padding of :1059-1079).
 * Either codes or scales may be NULL (with its output).  Device pointers. */
GQ_API int gq_modalix_layout(const void* codes, const float* scales, int64_t rows, int64_t cols,
                             int32_t block_values, int64_t rows_padded, void* out_codes, float* out_scales,
                             void* stream);

/* The conversion and the Modalix layout in one pass: unpack_gguf_tensor (+ the llama q/k
 * head permutation when perm_heads > 0; gguf_conversion.py:102-176, 314-332) followed by
 * ModelGraph._build_conv's reshape / transposes (model_graph.py:1012-1079), without the
 * row-major codes ever reaching memory.  tensor->codes receives (cols, rows_padded) bytes
 * (the memory order of the HWIGO weight (1, 1, cols, 1, rows_padded)), tensor->scales
 * (cols / block, rows_padded) f32; output channels rows..rows_padded-1 are the int4
 * 32-way padding: zero codes, unit scales.  tensor->values is not used; tensor->diag, if
 * any, is zeroed and receives the requantization maxima.  Takes cols a multiple of 256
 * and row lengths of a whole number of 16-byte chunks (cols / 256 * 210 for Q6_K, etc.);
 * other shapes return GQ_ERR_SIZE (convert, then gq_modalix_layout).  Device pointers:
 * src 16-byte aligned, scales 4. */
GQ_API int gq_convert_modalix(const gq_tensor_t* tensor, int64_t rows_padded, void* stream);

/* gq_convert_modalix for `count` tensors with one launch per GGML type present (at most 128
 * tensors per launch); rows_padded[i] per tensor, or NULL for no padding.  Each tensor's
 * diag, if any, is zeroed first. */
GQ_API int gq_convert_modalix_batch(const gq_tensor_t* tensors, const int64_t* rows_padded, int32_t count,
                                    void* stream);

/* The field-level steps of the reference's ggml_quant module, for callers that use them
 * one by one (the conversion entry points above fuse them).
 *
 * gq_unpack_fields: unpack_k_quant (sima_lmm/gguf/ggml_quant.py:567-694) for Q2_K, Q3_K,
 * Q4_K, Q5_K and Q6_K, and the ASYMMETRIC branches of unpack_q4 / unpack_q5
 * (ggml_quant.py:174-271) for Q4_1 / Q5_1.  Splits n_units stored units into their fields
 * with no arithmetic beyond widening the f16 constants to f32:
 *   K-quants: super_consts (n_units, k) f32 (k = 2: d, dmin for Q2_K / Q4_K / Q5_K;
 *             k = 1: d), block_consts (n_units, B, k) int8 (B = 8 for Q4_K / Q5_K, else
 *             16), values (n_units, B, 256 / B) int8 (Q3_K and Q6_K already offset by
 *             -4 / -32, the others unsigned).
 *   Q4_1 / Q5_1: super_consts receives the block constants (n_units, 2) f32 [d, m];
 *             block_consts must be NULL; values (n_units, 32): 0..15 / 0..31.
 * Device pointers: src and values 16-byte aligned, super_consts and block_consts 8. */
GQ_API int gq_unpack_fields(int32_t type, const void* src, size_t src_bytes, int64_t n_units,
                            float* super_consts, int8_t* block_consts, int8_t* values, void* stream);

/* remove_superblocks (ggml_quant.py:739-782): out[i*B + b, c] = f16(f32(block_consts[i, b, c]) *
 * super_consts[i, c]) (one f32 product, then round-to-nearest-even to f16), negated for
 * c = 1 when n_consts = 2 (the min).  block_consts are int8 (block_elem_bytes 1) or int16
 * (2); outputs (n_super * B, n_consts) as f16 bit patterns and / or their f32 widening
 * (either output may be NULL, not both).  Device pointers. */
GQ_API int gq_remove_superblocks(const float* super_consts, const void* block_consts, int32_t block_elem_bytes,
                                 int64_t n_super, int32_t blocks_per_super, int32_t n_consts,
                                 uint16_t* out_f16, float* out_f32, void* stream);

/* Token embeddings for the on-device runtime: LanguageModel.get_embeddings_tensor
 * (sima_lmm/model/language_model.py:578-611) fused with quantize_embedding_rows (:38-54).
 * Each row of a GGUF tensor (type F32, F16, BF16, Q8_0, Q4_0, Q4_K, Q5_K or Q6_K; src in
 * device memory, 16-byte aligned) is dequantized as gguf-py does, multiplied by
 * embed_scale (f32) and rounded to bf16.  quantize != 0: int8 codes (rows x cols) and one
 * bf16 scale per row (the row's absmax; 0 for an all-zero row); quantize == 0: the
 * bf16-rounded values as f32 (rows x cols).  cols must be a multiple of 4 and of the
 * type's block, and one row at most 51168 GGUF bytes. */
GQ_API int gq_embedding_rows(int32_t type, const void* src, size_t src_bytes, int64_t rows, int64_t cols,
                             float embed_scale, int32_t quantize, int8_t* codes, uint16_t* scales_bf16,
                             float* values, void* stream);

/* quantize_embedding_rows (language_model.py:38-54) on f32 rows in device memory:
 * int8 codes (rows x cols) and bf16 absmax scales (rows). */
GQ_API int gq_quantize_rows(const float* x, int64_t rows, int64_t cols, int8_t* codes, uint16_t* scales_bf16,
                            void* stream);

/* Host-buffer path: an opaque per-device session owning device staging memory, streams
 * and (on first use with pageable buffers) pinned bounce slots and host copy threads.
 * gq_convert_host copies each tensor's bytes host->device, converts and copies the results
 * device->host, pipelining pieces (of about 64 MB; permuted tensors in whole heads, one
 * head must fit `staging_bytes`) across three staging slots; host buffers may be pinned
 * (copied directly) or pageable (bounced through the pinned slots).  The pointers in
 * `tensors` are HOST pointers; diags (optional, host, one per tensor) receive the maxima.
 * Calls on one session are serialized.  A session belongs to the process that created it
 * (a forked child creates its own).  The caller's current device is the same after each
 * of these calls as before it. */
typedef struct gq_session gq_session_t;
GQ_API int gq_session_create(int32_t device, size_t staging_bytes, gq_session_t** out);
GQ_API int gq_session_destroy(gq_session_t* session);
GQ_API int gq_convert_host(gq_session_t* session, const gq_tensor_t* tensors, int32_t count,
                    int32_t out_mask, gq_diag_t* host_diags);

/* Page-locked host buffers for conversion results, recycled.  No counterpart in the
 * reference, whose calls return fresh numpy arrays (gguf_conversion.py:279-300).  A result
 * buffer in page-locked memory is written by the copy engines directly, where a fresh
 * pageable one costs page zeroing on first touch and a host copy out of a bounce slot;
 * gq_host_free keeps the buffer for the next request of its size class (classes of 2^k
 * and 1.5 * 2^k bytes, at least 64 KiB), so a caller converting one tensor at a time pins
 * memory once per class.  In use plus kept buffers stay under a limit (environment
 * LLIMA_B200_PINNED_RESULTS_MB; default a quarter of host memory, at most 16 GiB): past it
 * gq_host_alloc fails with GQ_ERR_NOMEM and the caller uses ordinary memory.  Kept buffers
 * of other classes are released first to make room; gq_host_trim releases all kept ones.
 * Thread-safe; a forked child starts with an empty arena. */
GQ_API int gq_host_alloc(size_t bytes, void** out);
GQ_API int gq_host_free(void* ptr);
GQ_API int gq_host_trim(void);

/* Allocation-free host-buffer conversion.  No counterpart in the reference: it exists for
 * callers that must not allocate device memory while they prepare weights, e.g. a process
 * whose device memory already belongs to another allocator (a framework's caching pool or
 * a fixed budget shared with an inference runtime), where cudaMalloc can fail or stall the
 * whole device.  Same inputs, outputs and results as gq_convert_host, but every byte of
 * device staging lives in one fixed array inside the library, GQ_NOALLOC_SCRATCH_BYTES per
 * GPU, held by every GPU that loads the library until the process exits; the call creates
 * no streams or events and allocates no host or device memory.  Work runs on `stream`
 * (NULL = legacy default stream), one piece at a time, and the call returns when the
 * results are in host memory.
 *   - The first call on a device looks up the array's device address (with `device`
 *     made current); make that first call before any stream capture.  The array's
 *     device memory is committed when the library's device code is loaded on that
 *     device, which under CUDA's lazy module loading (the default since CUDA 12.2) is
 *     this first call: a caller that hands all of a device's memory to another
 *     allocator should first make one call with count = 0 on that device (it loads the
 *     code, reserves the array and converts nothing).  A failed load is GQ_ERR_CUDA.
 *   - The caller's current device is the same after the call as before it.
 *   - An error after work was queued returns only once that work has finished, so no
 *     copy lands in the caller's buffers afterwards; the outputs are then incomplete.
 *   - Limits: the first 64 KiB of the array hold the diagnostics, so at most 8192 tensors
 *     per call when host_diags is given; the rest stages one piece at a time, so a piece
 *     of one unit (a head of rows for a permuted tensor) must fit.  Larger requests fail
 *     with GQ_ERR_SIZE before any device work.
 *   - All calls share the array.  Calls of this process on one device are serialized;
 *     anything else that runs on the GPU at the same time as a call and touches the array
 *     races with it. */
#define GQ_NOALLOC_SCRATCH_BYTES (16u << 20)
GQ_API int gq_convert_host_noalloc(int32_t device, const gq_tensor_t* tensors, int32_t count,
                                   int32_t out_mask, gq_diag_t* host_diags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GGUF_B200_H */

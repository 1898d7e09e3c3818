// Embedding rows: GGUF dequantize (force_float) -> x embed_scale -> bf16 round -> per-row
// int8 quantization, fused (sima_lmm/model/language_model.py:578-611 and 38-54).
//
// One warp per vocabulary row.  The row's GGUF bytes are staged in shared memory with
// 16-byte cp.async copies of the aligned window around the row; pass 1 decodes each value
// (gguf-py dequantize order), scales it, rounds it to bf16 and takes the row's absmax with
// a warp reduction; pass 2 decodes again and writes the int8 codes (4 per lane and step,
// 128 contiguous bytes per warp store).  The f32 embedding never touches HBM.
//
// Row quantization (the reference calls afe block_quantize_weight_tensor, which is not
// available, so this follows the restated rule of the CPU oracle): step = absmax / 127,
// q = clip(rint(x / step), -127, 127) (q = 0 when the row is all zeros), scale stored as
// bf16(step * 127) (language_model.py:51-54).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gq_device.cuh"
#include "gq_internal.h"

namespace gq {
namespace {

constexpr int kEmbWarps = 4;

// Shared bytes per warp: the 16-byte-aligned window around a row of row_bytes bytes that
// starts at any offset (at most row_bytes + 15 bytes, rounded up to 16).
__host__ __device__ __forceinline__ int64_t embed_stage_bytes(int64_t row_bytes) {
    return ((row_bytes + 15 + 15) / 16) * 16;
}

// Four consecutive f32 values starting at value v (a multiple of 4) of a row whose GGUF
// bytes start at `row` in shared memory, exactly as gguf-py's dequantize computes them.
template <int TYPE>
__device__ __forceinline__ void decode4(const uint8_t* row, int v, float out[4]) {
    if (TYPE == GQ_TYPE_F32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = __uint_as_float(lds16(row + 4 * (v + i)) | (lds16(row + 4 * (v + i) + 2) << 16));
    } else if (TYPE == GQ_TYPE_F16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = h2f(lds16(row + 2 * (v + i)));
    } else if (TYPE == GQ_TYPE_BF16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = __uint_as_float(lds16(row + 2 * (v + i)) << 16);
    } else if (TYPE == GQ_TYPE_Q8_0) {
        const uint8_t* bp = row + 34 * (v >> 5);
        const float d = h2f(lds16(bp));
        const int j = v & 31;
#pragma unroll
        for (int i = 0; i < 4; ++i) out[i] = __fmul_rn(static_cast<float>(static_cast<int8_t>(bp[2 + j + i])), d);
    } else if (TYPE == GQ_TYPE_Q4_0) {
        const uint8_t* bp = row + 18 * (v >> 5);
        const float d = h2f(lds16(bp));
        const int j = v & 31;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int jj = j + i;
            const int n = jj < 16 ? (bp[2 + jj] & 0xF) : (bp[2 + jj - 16] >> 4);
            out[i] = __fmul_rn(d, static_cast<float>(n - 8));
        }
    } else if (TYPE == GQ_TYPE_Q6_K) {
        const uint8_t* sp = row + 210 * (v >> 8);
        const int idx = v & 255;
        const float d = h2f(lds16(sp + 208));
        const float dd = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(sp[192 + (idx >> 4)])));
        const int h = idx >> 7, g = (idx >> 5) & 3, j = idx & 31;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int ql = sp[64 * h + 32 * (g & 1) + j + i];
            const int qh = sp[128 + 32 * h + j + i];
            const int q = (((ql >> (4 * (g >> 1))) & 0xF) | (((qh >> (2 * g)) & 3) << 4)) - 32;
            out[i] = __fmul_rn(dd, static_cast<float>(q));
        }
    } else {   // Q4_K / Q5_K
        constexpr bool Q5 = TYPE == GQ_TYPE_Q5_K;
        const uint8_t* sp = row + (Q5 ? 176 : 144) * (v >> 8);
        const int idx = v & 255;
        const int k = idx >> 5, j = idx & 31, g = k >> 1;
        int sc, mn;
        if (k < 4) {
            sc = sp[4 + k] & 63;
            mn = sp[8 + k] & 63;
        } else {
            sc = (sp[12 + k - 4] & 0xF) | ((sp[4 + k - 4] >> 6) << 4);
            mn = (sp[12 + k - 4] >> 4) | ((sp[8 + k - 4] >> 6) << 4);
        }
        const float ds = __fmul_rn(h2f(lds16(sp)), static_cast<float>(sc));
        const float dm = __fmul_rn(h2f(lds16(sp + 2)), static_cast<float>(mn));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int q = (sp[(Q5 ? 48 : 16) + 32 * g + j + i] >> (4 * (k & 1))) & 0xF;
            if (Q5) q |= ((sp[16 + j + i] >> k) & 1) << 4;
            out[i] = __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
        }
    }
}

__device__ __forceinline__ float to_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// `src_row_bytes`: GGUF bytes per row; FROM_F32: the source is already the f32 embedding
// (quantize_embedding_rows on its own: no scaling, no bf16 rounding).
template <int TYPE, bool FROM_F32>
__global__ void __launch_bounds__(32 * kEmbWarps) gq_embed_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                                                  int64_t cols, int64_t row_bytes, float embed_scale,
                                                                  int quantize, int8_t* __restrict__ codes,
                                                                  uint16_t* __restrict__ scales_bf16,
                                                                  float* __restrict__ values, int64_t src_bytes) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t stage_bytes = embed_stage_bytes(row_bytes);
    uint8_t* stage = smem + warp * stage_bytes;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kEmbWarps;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * kEmbWarps + warp; r < rows; r += nwarps) {
        const int64_t start = r * row_bytes;
        const int64_t a0 = start & ~int64_t(15);
        const int64_t end = start + row_bytes;
        const int skew = static_cast<int>(start - a0);
        for (int64_t c = a0 + 16 * lane; c < end; c += 32 * 16) {
            const int64_t left = src_bytes - c;
            cp_async16(stage + (c - a0), src + c, left < 16 ? static_cast<int>(left) : 16);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncwarp();
        const uint8_t* row = stage + skew;
        // pass 1: absmax of the bf16-rounded scaled values, as the max of the |x| bit
        // patterns (NaN wins, as in np.max)
        uint32_t amax_bits = 0;
        bool nonzero = false;
        for (int64_t v = 4 * lane; v < cols; v += 128) {
            float x[4];
            decode4<TYPE>(row, static_cast<int>(v), x);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float y = FROM_F32 ? x[i] : to_bf16(__fmul_rn(x[i], embed_scale));
                amax_bits = max(amax_bits, __float_as_uint(fabsf(y)));
                nonzero |= (y != 0.0f);
            }
        }
        const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, amax_bits));
        nonzero = __any_sync(0xffffffffu, nonzero);
        const float step = __fdiv_rn(amax, 127.0f);
        if (quantize) {
            // pass 2: codes
            for (int64_t v = 4 * lane; v < cols; v += 128) {
                float x[4];
                decode4<TYPE>(row, static_cast<int>(v), x);
                uint32_t packed = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float y = FROM_F32 ? x[i] : to_bf16(__fmul_rn(x[i], embed_scale));
                    int q = 0;
                    if (step > 0.0f) q = min(max(__float2int_rn(__fdiv_rn(y, step)), -127), 127);
                    packed |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * i);
                }
                *reinterpret_cast<uint32_t*>(codes + r * cols + v) = packed;
            }
            if (lane == 0) {
                const float s = nonzero ? __fmul_rn(step, 127.0f) : 0.0f;
                scales_bf16[r] = __bfloat16_as_ushort(__float2bfloat16_rn(s));
            }
        } else {
            for (int64_t v = 4 * lane; v < cols; v += 128) {
                float x[4];
                decode4<TYPE>(row, static_cast<int>(v), x);
                float y[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) y[i] = to_bf16(__fmul_rn(x[i], embed_scale));
                *reinterpret_cast<float4*>(values + r * cols + v) = make_float4(y[0], y[1], y[2], y[3]);
            }
        }
        __syncwarp();
    }
}

template <int TYPE, bool FROM_F32>
int launch_embed_t(const uint8_t* src, int64_t rows, int64_t cols, int64_t row_bytes, float embed_scale, int quantize,
                   int8_t* codes, uint16_t* scales, float* values, int64_t src_bytes, cudaStream_t s) {
    const int64_t smem = embed_stage_bytes(row_bytes) * kEmbWarps;
    if (smem > 200 * 1024) return static_cast<int>(cudaErrorInvalidValue);
    auto kern = gq_embed_kernel<TYPE, FROM_F32>;
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (rows + kEmbWarps - 1) / kEmbWarps;
    const int64_t cap = static_cast<int64_t>(sms) * 16;
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    kern<<<blocks, 32 * kEmbWarps, static_cast<size_t>(smem), s>>>(src, rows, cols, row_bytes, embed_scale, quantize,
                                                                   codes, scales, values, src_bytes);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

int64_t embed_max_row_bytes() { return (200 * 1024) / kEmbWarps - 32; }   // 51168 bytes

int launch_embed(int type, bool from_f32, const uint8_t* src, int64_t rows, int64_t cols, int64_t row_bytes,
                 float embed_scale, int quantize, int8_t* codes, uint16_t* scales, float* values, int64_t src_bytes,
                 void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (from_f32)
        return launch_embed_t<GQ_TYPE_F32, true>(src, rows, cols, row_bytes, 1.0f, 1, codes, scales, values,
                                                 src_bytes, s);
    switch (type) {
        case GQ_TYPE_F32: return launch_embed_t<GQ_TYPE_F32, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_F16: return launch_embed_t<GQ_TYPE_F16, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_BF16: return launch_embed_t<GQ_TYPE_BF16, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_Q8_0: return launch_embed_t<GQ_TYPE_Q8_0, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_Q4_0: return launch_embed_t<GQ_TYPE_Q4_0, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_Q4_K: return launch_embed_t<GQ_TYPE_Q4_K, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_Q5_K: return launch_embed_t<GQ_TYPE_Q5_K, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        case GQ_TYPE_Q6_K: return launch_embed_t<GQ_TYPE_Q6_K, false>(src, rows, cols, row_bytes, embed_scale, quantize, codes, scales, values, src_bytes, s);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

}  // namespace gq

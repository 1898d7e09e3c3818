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

// ---- block view of a row, for the quantized formats ------------------------------------
//
// Block b of a row (16 values for Q6_K, 32 otherwise) as unsigned byte codes v (packed in
// words, value j in byte j % 4 of word j / 4), an offset (the code is q = v - OFF) and the
// constants of gguf-py's dequantize: x = RN(A * q), or RN(RN(A * q) - B) for Q4_K / Q5_K.
template <int TYPE>
struct EmbBlock {
    static constexpr bool kOn = TYPE == GQ_TYPE_Q8_0 || TYPE == GQ_TYPE_Q4_0 || TYPE == GQ_TYPE_Q4_K ||
                                TYPE == GQ_TYPE_Q5_K || TYPE == GQ_TYPE_Q6_K;
    static constexpr int BV = TYPE == GQ_TYPE_Q6_K ? 16 : 32;
    static constexpr int NW = BV / 4;
    static constexpr int OFF = TYPE == GQ_TYPE_Q6_K ? 32 : (TYPE == GQ_TYPE_Q8_0 ? 128 : (TYPE == GQ_TYPE_Q4_0 ? 8 : 0));
    static constexpr bool kSub = TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K;
};

template <int TYPE>
__device__ __forceinline__ void decode_block(const uint8_t* row, int b, uint32_t (&w)[8], float& A, float& B) {
    B = 0.0f;
    if constexpr (TYPE == GQ_TYPE_Q6_K) {
        // ql[128] | qh[64] | scales int8[16] | d; value 128h + 32g + j (ggml_quant.py:274-308)
        const uint8_t* sp = row + 210 * (b >> 4);
        const int kb = b & 15, h = kb >> 3, g = (kb >> 1) & 3, j0 = 16 * (kb & 1);
        A = __fmul_rn(h2f(lds16(sp + 208)), static_cast<float>(static_cast<int8_t>(sp[192 + kb])));
        const uint4 l = lds128_align2(sp + 64 * h + 32 * (g & 1) + j0);
        const uint4 q = lds128_align2(sp + 128 + 32 * h + j0);
        const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
            w[i] = ((lw[i] >> (4 * (g >> 1))) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * g)) & 0x03030303u) << 4);
    } else if constexpr (TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K) {
        // d, dmin | scales[12] | (qh[32]) | qs[128]; block k: nibble k & 1 of qs[32(k/2) + j]
        constexpr bool Q5 = TYPE == GQ_TYPE_Q5_K;
        const uint8_t* sp = row + (Q5 ? 176 : 144) * (b >> 3);
        const int k = b & 7, g = k >> 1;
        int sc, mn;
        if (k < 4) {
            sc = sp[4 + k] & 63;
            mn = sp[8 + k] & 63;
        } else {
            sc = (sp[12 + k - 4] & 0xF) | ((sp[4 + k - 4] >> 6) << 4);
            mn = (sp[12 + k - 4] >> 4) | ((sp[8 + k - 4] >> 6) << 4);
        }
        A = __fmul_rn(h2f(lds16(sp)), static_cast<float>(sc));
        B = __fmul_rn(h2f(lds16(sp + 2)), static_cast<float>(mn));
        const uint8_t* qp = sp + (Q5 ? 48 : 16) + 32 * g;
        const uint4 a0 = lds128_align2(qp), a1 = lds128_align2(qp + 16);
        const uint32_t x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = (x[i] >> (4 * (k & 1))) & 0x0F0F0F0Fu;
        if constexpr (Q5) {
            const uint4 c0 = lds128_align2(sp + 16), c1 = lds128_align2(sp + 32);
            const uint32_t hb[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] |= ((hb[i] >> k) & 0x01010101u) << 4;
        }
    } else if constexpr (TYPE == GQ_TYPE_Q8_0) {
        // d | int8[32]: the codes biased by 128 to unsigned bytes
        const uint8_t* bp = row + 34 * b;
        A = h2f(lds16(bp));
        const uint4 a0 = lds128_align2(bp + 2), a1 = lds128_align2(bp + 18);
        const uint32_t x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = x[i] ^ 0x80808080u;
    } else {   // Q4_0: d | nibbles[16]; value j < 16 low nibble of byte j, else high of j - 16
        const uint8_t* bp = row + 18 * b;
        A = h2f(lds16(bp));
        const uint4 a0 = lds128_align2(bp + 2);
        const uint32_t x[4] = {a0.x, a0.y, a0.z, a0.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[i] = x[i] & 0x0F0F0F0Fu;
            w[4 + i] = (x[i] >> 4) & 0x0F0F0F0Fu;
        }
    }
}

// x of code q, as gguf-py computes it (Q8_0: x * d, the same product)
template <int TYPE>
__device__ __forceinline__ float block_value(float A, float B, int q) {
    const float p = __fmul_rn(A, static_cast<float>(q));
    return EmbBlock<TYPE>::kSub ? __fsub_rn(p, B) : p;
}

// code of y = bf16(x * embed_scale) for the row step: clip(rint(y / step), -127, 127).
// fast (step a normal number): y * (1/step) is within 2^-15 of y / step for every |y| <=
// absmax, so its rint is that of the correctly rounded quotient unless it lies within
// 2^-12 of a half-integer, where the quotient is divided exactly.
__device__ __forceinline__ int row_code(float y, float step, float rs, bool fast) {
    float k;
    if (fast) {
        const float t = __fmul_rn(y, rs);
        k = rintf(t);
        if (fabsf(fabsf(__fsub_rn(t, k)) - 0.5f) < 2.44140625e-4f) k = rintf(__fdiv_rn(y, step));
    } else {
        if (!(step > 0.0f)) return 0;
        k = __fdiv_rn(y, step);
    }
    return min(max(__float2int_rn(k), -127), 127);
}

// One row of a quantized format to int8 codes and its bf16 scale, by the warp.
//   pass 1, the row's absmax: every value is a monotone function of its code (x above,
//   then x * embed_scale and the bf16 rounding, all rounded the same way either side of
//   zero), so a block's largest |y| is reached at its smallest or largest code; blocks
//   whose constants (or the scale) are not finite, where inf * 0 can make a middle value
//   NaN, take every value;
//   pass 2, the codes, 16 or 32 per lane and block, stored as whole words.
template <int TYPE>
__device__ __forceinline__ void quantize_row_blocks(const uint8_t* row, int64_t r, int64_t cols, float embed_scale,
                                                    int8_t* __restrict__ codes, uint16_t* __restrict__ scales_bf16,
                                                    int lane) {
    using E = EmbBlock<TYPE>;
    const int nblocks = static_cast<int>(cols / E::BV);
    const bool s_finite = fabsf(embed_scale) < __int_as_float(0x7f800000);
    uint32_t amax_bits = 0;
    for (int b = lane; b < nblocks; b += 32) {
        uint32_t w[8];
        float A, B;
        decode_block<TYPE>(row, b, w, A, B);
        if (s_finite && fabsf(A) < __int_as_float(0x7f800000) && fabsf(B) < __int_as_float(0x7f800000)) {
            uint32_t mn = 0xFFFFFFFFu, mx = 0u;
#pragma unroll
            for (int i = 0; i < E::NW; ++i) {
                const uint32_t e = w[i] & 0x00FF00FFu, o = (w[i] >> 8) & 0x00FF00FFu;
                mn = __vminu2(mn, __vminu2(e, o));
                mx = __vmaxu2(mx, __vmaxu2(e, o));
            }
            const int qlo = static_cast<int>(min(mn & 0xFFFFu, mn >> 16)) - E::OFF;
            const int qhi = static_cast<int>(max(mx & 0xFFFFu, mx >> 16)) - E::OFF;
            const float ylo = to_bf16(__fmul_rn(block_value<TYPE>(A, B, qlo), embed_scale));
            const float yhi = to_bf16(__fmul_rn(block_value<TYPE>(A, B, qhi), embed_scale));
            amax_bits = max(amax_bits, max(__float_as_uint(fabsf(ylo)), __float_as_uint(fabsf(yhi))));
        } else {
#pragma unroll
            for (int j = 0; j < E::BV; ++j) {
                const int q = static_cast<int>((w[j >> 2] >> (8 * (j & 3))) & 0xFFu) - E::OFF;
                const float y = to_bf16(__fmul_rn(block_value<TYPE>(A, B, q), embed_scale));
                amax_bits = max(amax_bits, __float_as_uint(fabsf(y)));
            }
        }
    }
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, amax_bits));
    const float step = __fdiv_rn(amax, 127.0f);
    const bool fast = step >= 1.17549435e-38f && step < __int_as_float(0x7f800000);
    float rs = 0.0f;
    if (fast) asm("rcp.approx.f32 %0, %1;" : "=f"(rs) : "f"(step));
    int8_t* out = codes + r * cols;
    const bool vec = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    for (int b = lane; b < nblocks; b += 32) {
        uint32_t w[8];
        float A, B;
        decode_block<TYPE>(row, b, w, A, B);
        uint32_t c[8];
        if (fast) {
            // two values per instruction (f32x2: each half an IEEE round-to-nearest op, the
            // same results as the scalar chain), the bf16 rounding of a pair in one cvt
            const float2 A2 = make_float2(A, A), nB2 = make_float2(-B, -B);
            const float2 s2 = make_float2(embed_scale, embed_scale), rs2 = make_float2(rs, rs);
#pragma unroll
            for (int i = 0; i < E::NW; ++i) {
                uint32_t packed = 0;
#pragma unroll
                for (int e = 0; e < 4; e += 2) {
                    const float2 q2 = make_float2(static_cast<float>(static_cast<int>((w[i] >> (8 * e)) & 0xFFu) - E::OFF),
                                                  static_cast<float>(static_cast<int>((w[i] >> (8 * e + 8)) & 0xFFu) - E::OFF));
                    float2 x2 = __fmul2_rn(A2, q2);
                    if constexpr (E::kSub) x2 = __fadd2_rn(x2, nB2);
                    const float2 y2 = __bfloat1622float2(__float22bfloat162_rn(__fmul2_rn(x2, s2)));
                    const float2 t2 = __fmul2_rn(y2, rs2);
                    float kx = rintf(t2.x), ky = rintf(t2.y);
                    const float2 d2 = __fadd2_rn(t2, make_float2(-kx, -ky));
                    // within 2^-12 of a half-integer: the exactly divided quotient decides
                    if (fabsf(fabsf(d2.x) - 0.5f) < 2.44140625e-4f) kx = rintf(__fdiv_rn(y2.x, step));
                    if (fabsf(fabsf(d2.y) - 0.5f) < 2.44140625e-4f) ky = rintf(__fdiv_rn(y2.y, step));
                    const int cx = min(max(__float2int_rn(kx), -127), 127);
                    const int cy = min(max(__float2int_rn(ky), -127), 127);
                    packed |= ((static_cast<uint32_t>(cx) & 0xFFu) | ((static_cast<uint32_t>(cy) & 0xFFu) << 8)) << (8 * e);
                }
                c[i] = packed;
            }
        } else {
#pragma unroll
            for (int i = 0; i < E::NW; ++i) {
                uint32_t packed = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int q = static_cast<int>((w[i] >> (8 * e)) & 0xFFu) - E::OFF;
                    const float y = to_bf16(__fmul_rn(block_value<TYPE>(A, B, q), embed_scale));
                    packed |= (static_cast<uint32_t>(row_code(y, step, rs, fast)) & 0xFFu) << (8 * e);
                }
                c[i] = packed;
            }
        }
        int8_t* dst = out + b * E::BV;
        if (vec) {
#pragma unroll
            for (int i = 0; i < E::NW; i += 4) stg128(dst + 4 * i, make_uint4(c[i], c[i + 1], c[i + 2], c[i + 3]));
        } else {
#pragma unroll
            for (int i = 0; i < E::NW; ++i) st_global(reinterpret_cast<uint32_t*>(dst + 4 * i), c[i]);
        }
    }
    if (lane == 0) {
        // zero rows get scale 0 (language_model.py:53): absmax 0 means every value is 0
        const float sc = (amax == 0.0f) ? 0.0f : __fmul_rn(step, 127.0f);
        scales_bf16[r] = __bfloat16_as_ushort(__float2bfloat16_rn(sc));
    }
}

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
        if constexpr (EmbBlock<TYPE>::kOn && !FROM_F32) {
            if (quantize) {
                quantize_row_blocks<TYPE>(row, r, cols, embed_scale, codes, scales_bf16, lane);
                __syncwarp();
                continue;
            }
        }
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

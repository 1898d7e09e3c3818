// Modalix weight layout of converted weights (sima_lmm/model/model_graph.py:1012-1079).
//
// `_build_conv` takes the (out, in) codes of a projection to the SiMa IR HWIGO layout
// (oi -> oihw -> hwigo), which in memory is the (in, out) transpose, and the (out, in/B)
// block scales to (in/B, out).  For int4 weights it may pad the output channels to a
// uniform 32-way split with zero weights and unit scales.  These kernels do that on the
// device: a 64x64-byte tile transpose through shared memory with 4x4 byte blocks swapped
// in registers (PRMT), and a 32x32 f32 tile transpose for the scales.
#include <cuda_runtime.h>

#include "gq_device.cuh"
#include "gq_internal.h"

namespace gq {
namespace {

constexpr int kTile = 64;                 // bytes per tile side
constexpr int kRowWords = kTile / 4 + 1;  // padded shared row (words)

// codes (rows, cols) -> out (cols, rows_padded); columns r >= rows are zero.
__global__ void __launch_bounds__(256) gq_transpose_bytes(const uint8_t* __restrict__ in, int64_t rows, int64_t cols,
                                                          int64_t rows_padded, uint8_t* __restrict__ out) {
    __shared__ uint32_t tile[kTile * kRowWords];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kTile;
    const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kTile;
    const int t = threadIdx.x;
    // load: thread t -> input row t/4, 16 bytes at column 16*(t%4)
    {
        const int lr = t >> 2, lc = 16 * (t & 3);
        const int64_t r = r0 + lr, c = c0 + lc;
        uint32_t w[4] = {0, 0, 0, 0};
        if (r < rows) {
            if (c + 16 <= cols && ((reinterpret_cast<uintptr_t>(in + r * cols + c) & 15) == 0)) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(in + r * cols + c));
                w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
            } else {
#pragma unroll
                for (int b = 0; b < 16; ++b)
                    if (c + b < cols) w[b >> 2] |= static_cast<uint32_t>(in[r * cols + c + b]) << (8 * (b & 3));
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) tile[lr * kRowWords + (lc >> 2) + i] = w[i];
    }
    __syncthreads();
    // transpose: thread t -> 4x4 block (input rows 4a.., columns 4b..), a = t%16, b = t/16
    const int a = t & 15, b = t >> 4;
    const uint32_t x0 = tile[(4 * a + 0) * kRowWords + b];
    const uint32_t x1 = tile[(4 * a + 1) * kRowWords + b];
    const uint32_t x2 = tile[(4 * a + 2) * kRowWords + b];
    const uint32_t x3 = tile[(4 * a + 3) * kRowWords + b];
    const uint32_t t0 = __byte_perm(x0, x1, 0x5140), t1 = __byte_perm(x0, x1, 0x7362);
    const uint32_t t2 = __byte_perm(x2, x3, 0x5140), t3 = __byte_perm(x2, x3, 0x7362);
    const uint32_t y[4] = {__byte_perm(t0, t2, 0x5410), __byte_perm(t0, t2, 0x7632), __byte_perm(t1, t3, 0x5410),
                           __byte_perm(t1, t3, 0x7632)};
    // store: output row c0 + 4b + k holds input column 4b + k; 4 bytes at column r0 + 4a
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int64_t orow = c0 + 4 * b + k;
        const int64_t ocol = r0 + 4 * a;
        if (orow >= cols || ocol >= rows_padded) continue;
        uint8_t* dst = out + orow * rows_padded + ocol;
        if (ocol + 4 <= rows_padded && (reinterpret_cast<uintptr_t>(dst) & 3) == 0) {
            *reinterpret_cast<uint32_t*>(dst) = y[k];
        } else {
            for (int e = 0; e < 4 && ocol + e < rows_padded; ++e) dst[e] = static_cast<uint8_t>(y[k] >> (8 * e));
        }
    }
}

// scales (rows, nb) f32 -> out (nb, rows_padded); columns r >= rows are 1.0f.
__global__ void __launch_bounds__(256) gq_transpose_f32(const float* __restrict__ in, int64_t rows, int64_t nb,
                                                        int64_t rows_padded, float* __restrict__ out) {
    __shared__ float tile[32][33];
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 8 rows of 32 lanes
    for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i, c = c0 + tx;
        tile[i][tx] = (c < nb) ? (r < rows ? in[r * nb + c] : 1.0f) : 0.0f;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int64_t orow = c0 + i, ocol = r0 + tx;
        if (orow < nb && ocol < rows_padded) out[orow * rows_padded + ocol] = tile[tx][i];
    }
}

}  // namespace

int launch_layout(const uint8_t* codes, const float* scales, int64_t rows, int64_t cols, int64_t nb,
                  int64_t rows_padded, uint8_t* out_codes, float* out_scales, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (codes != nullptr && cols > 0 && rows_padded > 0) {
        const dim3 grid(static_cast<unsigned>((rows_padded + kTile - 1) / kTile),
                        static_cast<unsigned>((cols + kTile - 1) / kTile));
        gq_transpose_bytes<<<grid, 256, 0, s>>>(codes, rows, cols, rows_padded, out_codes);
        const int e = static_cast<int>(cudaGetLastError());
        if (e != 0) return e;
    }
    if (scales != nullptr && nb > 0 && rows_padded > 0) {
        const dim3 grid(static_cast<unsigned>((rows_padded + 31) / 32), static_cast<unsigned>((nb + 31) / 32));
        gq_transpose_f32<<<grid, 256, 0, s>>>(scales, rows, nb, rows_padded, out_scales);
        return static_cast<int>(cudaGetLastError());
    }
    return 0;
}

}  // namespace gq

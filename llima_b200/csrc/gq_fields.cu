// Field-level GGUF unpack and the super-block fold, on B200 (sm_100a).
//
// The conversion kernels (gq_kernels.cu) fuse the whole decode of a tensor.  These two
// kernels expose the steps the reference's ggml_quant module offers as functions of
// their own, for callers that use them one by one:
//
//   gq_fields_kernel       unpack_k_quant (sima_lmm/gguf/ggml_quant.py:567-694) for
//                          Q2_K..Q6_K, and the ASYMMETRIC branches of unpack_q4 /
//                          unpack_q5 (ggml_quant.py:174-271) for Q4_1 / Q5_1: stored
//                          units -> (super constants f32, block constants int8, values
//                          int8), with no arithmetic beyond the f16 -> f32 widening;
//   gq_superblocks_kernel  remove_superblocks (ggml_quant.py:739-782): block constant
//                          f16(f32(int) * f32 super constant), the min negated.
//
// gq_fields_kernel is a persistent grid of independent warps.  A warp streams tiles of
// stored units (8 super-blocks, or 32 blocks for Q4_1 / Q5_1; whole 16-byte chunks) into
// a two-stage shared ring with cp.async and writes each lane's 64 (K-quants) or 32
// contiguous value bytes with 16-byte stores.  HBM-bound: it reads the GGUF bytes once
// and writes 1 byte per value plus the constants.
#include <cuda_runtime.h>

#include "gq_device.cuh"
#include "gq_internal.h"

namespace gq {
namespace {

template <int TYPE>
struct FieldFmt;

// UB: stored unit bytes; UPT: units per tile; KQ: K-quant layout (256-value super-blocks)
#define GQ_FIELD_FMT(TYPE, UB_, UPT_, KQ_)                                          \
    template <>                                                                     \
    struct FieldFmt<TYPE> {                                                         \
        static constexpr int UB = UB_;                                              \
        static constexpr int UPT = UPT_;                                            \
        static constexpr bool KQ = KQ_;                                             \
        static constexpr int kTileBytes = UB_ * UPT_;                               \
        static constexpr int kStageBytes = kTileBytes + 16; /* lds128_align2 slack */ \
        static_assert(kTileBytes % 16 == 0, "tiles must be whole 16-byte chunks");  \
    };

GQ_FIELD_FMT(GQ_TYPE_Q4_K, 144, 8, true)
GQ_FIELD_FMT(GQ_TYPE_Q5_K, 176, 8, true)
GQ_FIELD_FMT(GQ_TYPE_Q6_K, 210, 8, true)
GQ_FIELD_FMT(GQ_TYPE_Q2_K, 84, 8, true)
GQ_FIELD_FMT(GQ_TYPE_Q3_K, 110, 8, true)
GQ_FIELD_FMT(GQ_TYPE_Q4_1, 20, 32, false)
GQ_FIELD_FMT(GQ_TYPE_Q5_1, 24, 32, false)
#undef GQ_FIELD_FMT

constexpr int kFieldWarps = 8;

// 4 bits b0..b3 -> bit 4 of bytes 0..3
__device__ __forceinline__ uint32_t bit4_to_bytes(uint32_t b) { return ((b * 0x00204081u) & 0x01010101u) << 4; }

// One lane of a K-quant tile: super-block sb = lane / 4 of the tile, quarter qq = lane % 4
// (values 64qq .. 64qq + 63 of the super-block, and the constants of the blocks they
// fall in).  Field offsets and bit positions as ggml_quant.py:274-498, 624-679.
template <int TYPE>
__device__ __forceinline__ void fields_kq(const uint8_t* p, int64_t u, int qq, float* sup, int8_t* blk,
                                          int8_t* vals) {
    using F = FieldFmt<TYPE>;
    uint32_t v[16];   // the lane's 64 value bytes
    const int h = qq >> 1, odd = qq & 1;
    if (TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K) {
        // d, dmin | scales[12] | (Q5_K: qh[32]) | qs[128]; group qq = 32 nibble bytes:
        // block 2qq = low nibbles, block 2qq+1 = high nibbles; Q5_K's fifth bit of block
        // k is bit k of qh[j]
        constexpr int QS = TYPE == GQ_TYPE_Q5_K ? 48 : 16;
        const uint4 a = lds128(p + QS + 32 * qq), b = lds128(p + QS + 32 * qq + 16);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[i] = w[i] & 0x0F0F0F0Fu;
            v[8 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
        if (TYPE == GQ_TYPE_Q5_K) {
            const uint4 c = lds128(p + 16), d = lds128(p + 32);
            const uint32_t hw[8] = {c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[i] |= ((hw[i] >> (2 * qq)) & 0x01010101u) << 4;
                v[8 + i] |= ((hw[i] >> (2 * qq + 1)) & 0x01010101u) << 4;
            }
        }
        // 6-bit (scale, min) of blocks 2qq, 2qq+1 (ggml_quant.py:352-375), interleaved
        const uint8_t* s = p + 4;
        uint32_t word = 0;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int bi = 2 * qq + t;
            int sc, mn;
            if (bi < 4) {
                sc = s[bi] & 0x3F;
                mn = s[bi + 4] & 0x3F;
            } else {
                sc = (s[bi + 4] & 0x0F) | ((s[bi - 4] >> 6) << 4);
                mn = (s[bi + 4] >> 4) | ((s[bi] >> 6) << 4);
            }
            word |= (static_cast<uint32_t>(sc) | (static_cast<uint32_t>(mn) << 8)) << (16 * t);
        }
        st_global(reinterpret_cast<uint32_t*>(blk + u * 16 + 4 * qq), word);
        if (qq < 2) st_global(sup + u * 2 + qq, h2f(lds16(p + 2 * qq)));
    } else if (TYPE == GQ_TYPE_Q6_K) {
        // ql[128] | qh[64] | scales int8[16] | d: value 128h + 32g + j = nibble of
        // ql[64h + 32(g&1) + j] (low for g < 2) | bits 2g..2g+1 of qh[32h + j] << 4, - 32
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int g = 2 * odd + t;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint4 l = lds128_align2(p + 64 * h + 32 * t + 16 * half);
                const uint4 q = lds128_align2(p + 128 + 32 * h + 16 * half);
                const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t x = ((lw[i] >> (4 * odd)) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * g)) & 0x03030303u) << 4);
                    v[8 * t + 4 * half + i] = (x + 0x60606060u) ^ 0x80808080u;   // x - 32 per byte
                }
            }
        }
        const uint32_t sw = lds16(p + 192 + 4 * qq) | (lds16(p + 194 + 4 * qq) << 16);
        st_global(reinterpret_cast<uint32_t*>(blk + u * 16 + 4 * qq), sw);
        if (qq == 0) st_global(sup + u, h2f(lds16(p + 208)));
    } else if (TYPE == GQ_TYPE_Q2_K) {
        // scales[16] | qs[64] | d | dmin: value 128h + 32j + b = bits 2j..2j+1 of qs[32h + b]
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int j = 2 * odd + t;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint4 x = lds128_align2(p + 16 + 32 * h + 16 * half);
                const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) v[8 * t + 4 * half + i] = (xw[i] >> (2 * j)) & 0x03030303u;
            }
        }
        // blocks 4qq..4qq+3: (scale, min) = (low nibble, high nibble) of scales[k]
        const uint32_t sb4 = lds32(p + 4 * qq);
        const uint32_t lo = sb4 & 0x0F0F0F0Fu, hi = (sb4 >> 4) & 0x0F0F0F0Fu;
        uint2 pair;
        pair.x = __byte_perm(lo, hi, 0x5140);
        pair.y = __byte_perm(lo, hi, 0x7362);
        st_global(reinterpret_cast<uint2*>(blk + u * 32 + 8 * qq), pair);
        if (qq < 2) st_global(sup + u * 2 + qq, h2f(lds16(p + 80 + 2 * qq)));
    } else {   // Q3_K
        // hmask[32] | qs[64] | scales[12] | d: low bits as Q2_K, third bit = bit 4h + j of
        // hmask[b], minus 4
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int j = 2 * odd + t;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint4 x = lds128_align2(p + 32 + 32 * h + 16 * half);
                const uint4 m = lds128_align2(p + 16 * half);
                const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, mw[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t q = ((xw[i] >> (2 * j)) & 0x03030303u) | (((mw[i] >> (4 * h + j)) & 0x01010101u) << 2);
                    v[8 * t + 4 * half + i] = (q + 0x7C7C7C7Cu) ^ 0x80808080u;   // q - 4 per byte
                }
            }
        }
        // scales 4qq..4qq+3: six bits minus 32 (ggml_quant.py:398-425)
        const uint8_t* s = p + 96;
        uint32_t word = 0;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int i = 4 * qq + t;
            const int low = i < 8 ? (s[i] & 0x0F) : (s[i - 8] >> 4);
            const int top = (s[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
            word |= (static_cast<uint32_t>((low | (top << 4)) - 32) & 0xFFu) << (8 * t);
        }
        st_global(reinterpret_cast<uint32_t*>(blk + u * 16 + 4 * qq), word);
        if (qq == 0) st_global(sup + u, h2f(lds16(p + 108)));
    }
    static_assert(F::KQ, "K-quant layout");
    int8_t* dst = vals + u * 256 + 64 * qq;
#pragma unroll
    for (int i = 0; i < 4; ++i) stg128(dst + 16 * i, make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
}

// One lane of a Q4_1 / Q5_1 tile: block u.  d, m | (Q5_1: qh u32) | qs[16]; value j < 16
// is the low nibble of qs[j], value 16 + j its high nibble; Q5_1 adds bit j of qh << 4
// (ggml_quant.py:174-271, ASYMMETRIC).
template <int TYPE>
__device__ __forceinline__ void fields_base(const uint8_t* p, int64_t u, float* consts, int8_t* vals) {
    constexpr bool Q5 = TYPE == GQ_TYPE_Q5_1;
    const uint4 x = lds128_align2(p + (Q5 ? 8 : 4));
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
    const uint32_t qh = Q5 ? lds32(p + 4) : 0u;
    uint32_t v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] = xw[i] & 0x0F0F0F0Fu;
        v[4 + i] = (xw[i] >> 4) & 0x0F0F0F0Fu;
        if (Q5) {
            v[i] |= bit4_to_bytes((qh >> (4 * i)) & 0xFu);
            v[4 + i] |= bit4_to_bytes((qh >> (16 + 4 * i)) & 0xFu);
        }
    }
    const uint32_t dm = lds32(p);
    st_global(reinterpret_cast<float2*>(consts + u * 2), make_float2(h2f(dm), h2f(dm >> 16)));
    stg128(vals + u * 32, make_uint4(v[0], v[1], v[2], v[3]));
    stg128(vals + u * 32 + 16, make_uint4(v[4], v[5], v[6], v[7]));
}

template <int TYPE>
__global__ void __launch_bounds__(32 * kFieldWarps) gq_fields_kernel(const uint8_t* __restrict__ src,
                                                                     int64_t n_units, float* sup, int8_t* blk,
                                                                     int8_t* vals) {
    using F = FieldFmt<TYPE>;
    __shared__ __align__(16) uint8_t ring[kFieldWarps][2][F::kStageBytes];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int64_t n_tiles = (n_units + F::UPT - 1) / F::UPT;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kFieldWarps;

    auto issue = [&](int64_t t, uint8_t* stage) {
        if (t >= n_tiles) return;
        const int64_t left = n_units - t * F::UPT;
        const int nbytes = static_cast<int>(left < F::UPT ? left : F::UPT) * F::UB;
        const uint8_t* s = src + t * F::kTileBytes;
        for (int c = lane * 16; c < nbytes; c += 32 * 16) cp_async16(stage + c, s + c, nbytes - c < 16 ? nbytes - c : 16);
    };

    int64_t t = static_cast<int64_t>(blockIdx.x) * kFieldWarps + warp;
    issue(t, ring[warp][0]);
    cp_async_commit();
    for (int stage = 0; t < n_tiles; t += nwarps, stage ^= 1) {
        issue(t + nwarps, ring[warp][stage ^ 1]);
        cp_async_commit();
        cp_async_wait<1>();
        __syncwarp();
        const uint8_t* tile = ring[warp][stage];
        const int64_t unit0 = t * F::UPT;
        const int64_t left = n_units - unit0;
        const int nunits = left < F::UPT ? static_cast<int>(left) : F::UPT;
        if constexpr (F::KQ) {
            const int sb = lane >> 2;
            if (sb < nunits) fields_kq<TYPE>(tile + sb * F::UB, unit0 + sb, lane & 3, sup, blk, vals);
        } else {
            if (lane < nunits) fields_base<TYPE>(tile + lane * F::UB, unit0 + lane, sup, vals);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
}

// remove_superblocks: element e of the (N, B, k) block constants, s = e / (B k), c = e % k
template <typename BT>
__global__ void __launch_bounds__(256) gq_superblocks_kernel(const float* __restrict__ sup,
                                                             const BT* __restrict__ blk, int64_t n, int bk, int k,
                                                             uint16_t* out_f16, float* out_f32) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += stride) {
        const int64_t s = e / bk;
        const int c = static_cast<int>((e - s * bk) % k);
        // f32 product of the integer constant and the super constant, then f16 RNE
        // (ggml_quant.py:771-772); the min column is negated in f16 (:775-776)
        uint16_t hbits = __half_as_ushort(__float2half_rn(__fmul_rn(static_cast<float>(blk[e]), sup[s * k + c])));
        if (k == 2 && c == 1) hbits ^= 0x8000u;
        if (out_f16) st_global(out_f16 + e, hbits);
        if (out_f32) st_global(out_f32 + e, h2f(hbits));
    }
}

int sm_count() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int& n = sms[dev & 63];
    if (n == 0) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

template <int TYPE>
int launch_fields_t(const uint8_t* src, int64_t n_units, float* sup, int8_t* blk, int8_t* vals, cudaStream_t s) {
    using F = FieldFmt<TYPE>;
    const int64_t tiles = (n_units + F::UPT - 1) / F::UPT;
    const int64_t want = (tiles + kFieldWarps - 1) / kFieldWarps;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    gq_fields_kernel<TYPE><<<blocks, 32 * kFieldWarps, 0, s>>>(src, n_units, sup, blk, vals);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

int launch_fields(int type, const uint8_t* src, int64_t n_units, float* sup, int8_t* blk, int8_t* vals,
                  void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (type) {
        case GQ_TYPE_Q4_K: return launch_fields_t<GQ_TYPE_Q4_K>(src, n_units, sup, blk, vals, s);
        case GQ_TYPE_Q5_K: return launch_fields_t<GQ_TYPE_Q5_K>(src, n_units, sup, blk, vals, s);
        case GQ_TYPE_Q6_K: return launch_fields_t<GQ_TYPE_Q6_K>(src, n_units, sup, blk, vals, s);
        case GQ_TYPE_Q2_K: return launch_fields_t<GQ_TYPE_Q2_K>(src, n_units, sup, blk, vals, s);
        case GQ_TYPE_Q3_K: return launch_fields_t<GQ_TYPE_Q3_K>(src, n_units, sup, blk, vals, s);
        case GQ_TYPE_Q4_1: return launch_fields_t<GQ_TYPE_Q4_1>(src, n_units, sup, blk, vals, s);
        case GQ_TYPE_Q5_1: return launch_fields_t<GQ_TYPE_Q5_1>(src, n_units, sup, blk, vals, s);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

int launch_superblocks(const float* sup, const void* blk, int blk_bytes, int64_t n_super, int nb, int k,
                       uint16_t* out_f16, float* out_f32, void* stream) {
    const int64_t n = n_super * nb * k;
    const int64_t want = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (blk_bytes == 1)
        gq_superblocks_kernel<int8_t><<<blocks, 256, 0, s>>>(sup, static_cast<const int8_t*>(blk), n, nb * k, k,
                                                             out_f16, out_f32);
    else
        gq_superblocks_kernel<int16_t><<<blocks, 256, 0, s>>>(sup, static_cast<const int16_t*>(blk), n, nb * k, k,
                                                              out_f16, out_f32);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace gq

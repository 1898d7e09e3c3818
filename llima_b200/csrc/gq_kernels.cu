// GGUF block decode + requantization kernels for B200 (sm_100a).
//
// One kernel per GGML format (Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K),
// a float pass-through copy, the standalone requantization scheme and the conversion fused
// with the Modalix layout.  Each format kernel is a persistent grid of independent warps.
// A warp owns a ring of shared-memory stages and brings whole tiles of stored blocks into
// it (tile sizes are multiples of 16 bytes): one bulk copy per tile by the TMA engine,
// completed on the stage's mbarrier with a bounded wait, or for Q6_K 16-byte cp.async
// copies of every lane; then it decodes the tile from shared memory.  For the asymmetric
// formats (Q4_K / Q5_K shown; the others alike):
//
//   * parameters: each lane takes one 32-byte code group (two blocks), scans its codes for
//     min / max in 16-bit SIMD lanes, unpacks the blocks' 6-bit scale / min and the f16
//     super constants, and derives the requantization parameters (requant_fast);
//   * codes: packed 16-bit integer arithmetic (q * sf + rm, one multiply-add per two codes)
//     for the blocks with an integer scale factor (99.5% on the benchmark data), written as
//     one 32-byte store per block; the other blocks are finished by a warp pass each, one
//     value per lane, with the per-value f32 formula.
//
// The fp32 intermediate of dequant -> requant never touches global memory.
#include <cuda_runtime.h>

#include <memory>
#include <new>
#include <type_traits>

#include "gq_device.cuh"
#include "gq_internal.h"

namespace gq {

// ---------------------------------------------------------------------------------------
// Format geometry: stored unit size, units per tile, pipeline depth
// ---------------------------------------------------------------------------------------

// Sub-tiles of 8 super-blocks per Q4_K / Q5_K loop iteration, processed one after the
// other (the per-tile bookkeeping is shared, the registers are not multiplied), the
// pipeline depth and the warps per CTA.  With one bulk copy per tile, fewer and larger
// tiles win at 8-warp CTAs (8-layer cuts, fraction of the measured copy peak, Q4_K / Q5_K):
// 6 (Q5_K 5) sub-tiles x 2 stages 0.795 / 0.749, 4 x 3 (Q5_K 4 x 2) 0.786 / 0.743, 3 x 4
// 0.768 / 0.725, 2 x 6 0.737 / 0.697, 4 x 4 at 6-warp CTAs 0.698 / 0.667.  Q4_K at 96
// registers fits two 10-warp CTAs per SM when their tiles are 4 sub-tiles x 2 stages (92 KB
// of stages per CTA): 20 warps per SM instead of 16 measured 0.4007 against 0.4042 ms on the
// 8-layer cut and 1.548 against 1.559 ms in the whole 8B step; 3 x 2 tiles at 10 warps 0.412.
#ifndef GQ_K45_SUB
#define GQ_K45_SUB 4
#endif
#ifndef GQ_K45_STAGES
#define GQ_K45_STAGES 2
#endif
#ifndef GQ_K45_WARPS
#define GQ_K45_WARPS 10
#endif
#ifndef GQ_Q6K_SUB
#define GQ_Q6K_SUB 2
#endif
#ifndef GQ_Q6K_STAGES
#define GQ_Q6K_STAGES 3
#endif
// Q5_K with per-lane copies (8-layer Qwen2.5-7B Q5_K set, GB/s): 1 sub-tile x 4 stages
// 3930, 2 x 3 4240, 3 x 3 4387, 4 x 2 4484-4493, 5 x 2 4487, 4 x 3 at 6 warps 4052.
// Re-checked with bulk copies and the byte-form 5-bit codes (96 registers; whole Qwen2.5-7B
// Q5_K set, ms): 5 x 2 at 8 warps 2.17-2.18, 4 x 2 2.20-2.21, 6-warp CTAs three per SM
// 4 x 2 2.35-2.37, 3 x 2 2.38-2.39; 10-warp CTAs (two per SM only with 3 x 2 tiles) 0.652
// against 0.640 ms on the 8-layer cut.
#ifndef GQ_Q5K_SUB
#define GQ_Q5K_SUB 5
#endif
#ifndef GQ_Q5K_STAGES
#define GQ_Q5K_STAGES 2
#endif
#ifndef GQ_Q5K_WARPS
#define GQ_Q5K_WARPS 8
#endif

template <int TYPE>
struct Fmt;

#ifndef GQ_Q6K_BULK
#define GQ_Q6K_BULK 0
#endif
#ifndef GQ_Q0_BULK
#define GQ_Q0_BULK 1
#endif
#ifndef GQ_Q0_SUB
#define GQ_Q0_SUB 8
#endif
#ifndef GQ_Q0_STAGES
#define GQ_Q0_STAGES 2
#endif

#define GQ_FMT(TYPE, UNIT_BYTES, UNITS_PER_TILE, STAGES, WARPS, BULK)                     \
    template <>                                                                           \
    struct Fmt<TYPE> {                                                                    \
        static constexpr int kWarps = WARPS;  /* warps per CTA */                         \
        static constexpr int kThreads = 32 * WARPS;                                       \
        static constexpr int kUnitBytes = UNIT_BYTES;                                     \
        static constexpr int kUnitsPerTile = UNITS_PER_TILE;                              \
        static constexpr int kTileBytes = UNIT_BYTES * UNITS_PER_TILE;                    \
        static constexpr int kStageBytes = kTileBytes + 16; /* slack for 20-byte reads */ \
        static constexpr int kStages = STAGES;                                            \
        /* tiles arrive by one bulk copy each, or by 16-byte copies of every lane */      \
        static constexpr bool kBulk = BULK;                                               \
        static_assert(kTileBytes % 16 == 0, "tiles must be whole 16-byte chunks");        \
    };

GQ_FMT(GQ_TYPE_Q4_K, 144, 8 * GQ_K45_SUB, GQ_K45_STAGES, GQ_K45_WARPS, true)   // sub-tiles of 8 super-blocks
GQ_FMT(GQ_TYPE_Q5_K, 176, 8 * GQ_Q5K_SUB, GQ_Q5K_STAGES, GQ_Q5K_WARPS, true)
GQ_FMT(GQ_TYPE_Q6_K, 210, 8 * GQ_Q6K_SUB, GQ_Q6K_STAGES, 8, GQ_Q6K_BULK)   // sub-tiles of 128 blocks of 16
GQ_FMT(GQ_TYPE_Q8_0, 34, 32 * GQ_Q0_SUB, GQ_Q0_STAGES, 8, GQ_Q0_BULK)   // sub-tiles of 32 blocks of 32
GQ_FMT(GQ_TYPE_Q4_0, 18, 32 * GQ_Q0_SUB, GQ_Q0_STAGES, 8, GQ_Q0_BULK)
GQ_FMT(GQ_TYPE_Q4_1, 20, 32, 4, 8, GQ_Q0_BULK)   // 32 blocks of 32 per tile, one per lane
GQ_FMT(GQ_TYPE_Q5_0, 22, 32, 4, 8, GQ_Q0_BULK)
GQ_FMT(GQ_TYPE_Q5_1, 24, 32, 4, 8, GQ_Q0_BULK)
GQ_FMT(GQ_TYPE_Q2_K, 84, 8, 4, 8, GQ_Q0_BULK)    // 128 blocks of 16 per tile, one per lane and round
GQ_FMT(GQ_TYPE_Q3_K, 110, 8, 4, 8, GQ_Q0_BULK)
#undef GQ_FMT

// Q4_K / Q5_K launches with few tiles per warp (one tensor of a BASELINE single-tensor
// config, a host call's piece) use 4 sub-tiles per tile instead (Q4_K with 3 stages): the
// C2 Q4_K 11008x4096 tensor alone measured 0.585 of the copy peak so against 0.485 in the
// big tiles, and 0.559 with 1 sub-tile x 6 stages.
// Q8_0 / Q4_0 likewise: big launches in tiles of 8 x 32 blocks with 2 stages (Qwen2.5-7B
// Q8_0 embedding and output 0.98 of the copy peak against 0.82 in 32-block tiles), small
// ones in 32-block tiles with 4 stages (C1 0.72 against 0.52 in the big tiles).
template <int TYPE>
struct FmtSmall : Fmt<TYPE> {
    static constexpr bool kQ0 = TYPE == GQ_TYPE_Q8_0 || TYPE == GQ_TYPE_Q4_0;
    static constexpr int kUnitsPerTile = 32;
    static constexpr int kTileBytes = Fmt<TYPE>::kUnitBytes * 32;
    static constexpr int kStageBytes = kTileBytes + 16;
    static constexpr int kStages = kQ0 ? 4 : (TYPE == GQ_TYPE_Q4_K ? 3 : 2);
    // 8-warp CTAs whatever the large tiles use (the measured small-launch configuration)
    static constexpr int kWarps = 8;
    static constexpr int kThreads = 32 * kWarps;
};

// Minimum resident CTAs per SM the Q4_K kernel is compiled for (caps its registers; the
// other formats leave the register count to the compiler).
#ifndef GQ_MIN_BLOCKS
#define GQ_MIN_BLOCKS 2
#endif

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
[[maybe_unused]] constexpr unsigned kFull = 0xffffffffu;

// Tensor owning global tile `t` (binary search over tile_begin).
__device__ __forceinline__ int find_desc(const GqBatch& b, int64_t t) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (b.d[mid].tile_begin <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// A warp visits its tiles in increasing order, so the owning tensor only moves forward:
// a cursor that steps ahead replaces a search per tile.
struct DescCursor {
    int idx = 0;
    __device__ __forceinline__ int seek(const GqBatch& b, int64_t t) {
        while (idx + 1 < b.n && b.d[idx + 1].tile_begin <= t) ++idx;
        return idx;
    }
};

// Enqueue the cp.async copies of tile `t` into `stage` (nothing when t is past the end).
template <class F>
__device__ __forceinline__ void issue_tile(const GqBatch& b, DescCursor& cur, int64_t t, uint8_t* stage,
                                           int lane) {
    if (t >= b.total_tiles) return;
    const GqDesc& d = b.d[cur.seek(b, t)];
    const int64_t unit0 = (t - d.tile_begin) * F::kUnitsPerTile;
    const int64_t left = d.n_units - unit0;
    const int nunits = left < F::kUnitsPerTile ? static_cast<int>(left) : F::kUnitsPerTile;
    const int nbytes = nunits * F::kUnitBytes;
    const uint8_t* src = d.src + unit0 * F::kUnitBytes;
    for (int c = lane * 16; c < nbytes; c += 32 * 16) {
        const int n = nbytes - c;
        cp_async16(stage + c, src + c, n < 16 ? n : 16);
    }
}

// Tile `t` as one bulk copy into `stage`, completed on `bar` (lane 0 only; nothing when t is
// past the end).  A whole tile is a multiple of 16 bytes, so every tile starts 16-byte
// aligned (the tensor's bytes do); the last tile of a tensor may end with fewer than 16
// bytes past its last whole chunk, which lane 0 copies itself before it arrives on the
// barrier (the arrival releases those stores to the lanes that wait on it).
template <class F>
__device__ __forceinline__ void issue_tile_bulk(const GqBatch& b, DescCursor& cur, int64_t t, uint8_t* stage,
                                                uint64_t* bar) {
    if (t >= b.total_tiles) return;
    const GqDesc& d = b.d[cur.seek(b, t)];
    const int64_t unit0 = (t - d.tile_begin) * F::kUnitsPerTile;
    const int64_t left = d.n_units - unit0;
    const int nunits = left < F::kUnitsPerTile ? static_cast<int>(left) : F::kUnitsPerTile;
    const uint32_t nbytes = static_cast<uint32_t>(nunits * F::kUnitBytes);
    const uint32_t whole = nbytes & ~15u;
    const uint8_t* src = d.src + unit0 * F::kUnitBytes;
    if (F::kUnitBytes % 16 != 0) {
        for (uint32_t i = whole; i < nbytes; ++i) stage[i] = src[i];
    }
    mbar_arrive_expect_tx(bar, whole);
    if (whole != 0) bulk_load(stage, src, whole, bar);
}

// Sticky error flags of this device's conversion kernels (kErrWaitTimeout: a tile copy did
// not complete within the wait limit, so the launch stopped early).
__device__ unsigned int gq_kernel_errors;

// ---------------------------------------------------------------------------------------
// Q4_K / Q5_K: 256-value super-blocks -> 8 blocks of 32, asymmetric -> symmetric int8
//   Q4_K: d, dmin | scales[12] | qs[128]          (ggml_quant.py:624-642)
//   Q5_K: d, dmin | scales[12] | qh[32] | qs[128]  (ggml_quant.py:643-661)
//
// A tile is 8 super-blocks = 32 groups of 32 nibble bytes; lane l owns group l
// (super-block l/4, group g = l%4), i.e. block 2g (low nibbles) and block 2g+1 (high
// nibbles).  Codes are kept in 16-bit lanes without shifting them down: for a word of
// four bytes b0..b3,
//   EL = w & 0x000F000F   low nibbles of b0, b2  (value << 0)
//   OL = w & 0x0F000F00   low nibbles of b1, b3  (value << 8)
//   EH = w & 0x00F000F0   high nibbles of b0, b2 (value << 4)
//   OH = w & 0xF000F000   high nibbles of b1, b3 (value << 12)
// so the same masked words feed the min/max scan and the requantization: q*sf + rm is
// one IMAD per two codes (mad.hi undoes the << 8 / << 12 for free).  Q5_K first builds,
// once per word, the 5-bit codes of both blocks as bytes (L: low nibbles with the block-2g
// fifth bits, H: high nibbles with the block-2g+1 fifth bits, each merge one IMAD); its
// layouts are then L and H masked to bytes 0, 2 (<< 0) and 1, 3 (<< 8), and both blocks
// take the low block's arithmetic.
// ---------------------------------------------------------------------------------------

// Codes of one block side from its two 16-bit-lane words (E holds bytes 0 and 2, O bytes
// 1 and 3, both already at bits 0..4 of their lanes) as a word of four code bytes.
__device__ __forceinline__ uint32_t codes_word(uint32_t e, uint32_t o) { return __byte_perm(e, o, 0x6240); }

// Requantized bytes of one word, slow path (non-integer scale factor) or with clipping.
__device__ __forceinline__ uint32_t requant_word_general(uint32_t q4, const Requant& p) {
    if (p.fast) {
        uint32_t out = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int v = min(max(static_cast<int>((q4 >> (8 * b)) & 0xFF) * p.sfi + p.rm, -128), 127);
            out |= (static_cast<uint32_t>(v) & 0xFFu) << (8 * b);
        }
        return out;
    }
    return requant_word_slow(q4, p.sf, p.rm, -128, 127);
}

// The 32 code bytes of one group: Q4_K the raw nibble words; Q5_K the 5-bit codes, w[i] of
// block 2g and h[i] of block 2g+1, one code per byte.
template <bool Q5>
struct GroupWords {
    uint32_t w[8];
    uint32_t h[Q5 ? 8 : 1];
};

// The four 16-bit lane layouts of word i (see above).
template <bool Q5>
__device__ __forceinline__ void group_layouts(const GroupWords<Q5>& q, int i, uint32_t& el, uint32_t& ol,
                                              uint32_t& eh, uint32_t& oh) {
    const uint32_t w = q.w[i];
    if (!Q5) {
        el = w & 0x000F000Fu;
        ol = w & 0x0F000F00u;
        eh = w & 0x00F000F0u;
        oh = w & 0xF000F000u;
    } else {
        const uint32_t h = q.h[Q5 ? i : 0];
        el = w & 0x00FF00FFu;
        ol = w & 0xFF00FF00u;
        eh = h & 0x00FF00FFu;
        oh = h & 0xFF00FF00u;
    }
}

// The constants of a lane's two blocks, S = f16(sc * d) and P = f16(m * dmin), from the
// 6-bit pairs sc2 = scL | scH << 8, mn2 = mnL | mnH << 8 and the header word (d | dmin << 16).
// The f32 product of a 6-bit integer and an f16 value is exact, so rounding it to f16 (what
// remove_superblocks does, ggml_quant.py:771-777) equals one correctly rounded f16 multiply:
// both blocks' products are one mul.rn.f16x2 each for S and P, with the integers made f16 by
// the bias trick (f16 bits 0x6400 | k = 1024 + k for k < 1024, minus 1024, exactly).
__device__ __forceinline__ void block_constants_h2(uint32_t sc2, uint32_t mn2, uint32_t hdr, float& SL, float& SH,
                                                   float& PL, float& PH) {
    const __half2 k1024 = __halves2half2(__ushort_as_half(0x6400u), __ushort_as_half(0x6400u));
    const __half2 scf = __hsub2(u32_as_h2(__byte_perm(sc2, 0x6464u, 0x4140u)), k1024);
    const __half2 mnf = __hsub2(u32_as_h2(__byte_perm(mn2, 0x6464u, 0x4140u)), k1024);
    const __half2 s2 = __hmul2_rn(scf, u32_as_h2(__byte_perm(hdr, 0u, 0x1010u)));
    const __half2 p2 = __hmul2_rn(mnf, u32_as_h2(__byte_perm(hdr, 0u, 0x3232u)));
    SL = __low2float(s2);
    SH = __high2float(s2);
    PL = __low2float(p2);
    PH = __high2float(p2);
}

// Block constants of block b (0..7) of a Q4_K / Q5_K super-block, read by every lane of
// the warp: S = f16(sc * d) and M = -f16(m * dmin) (ggml_quant.py:352-375, 771-777).
__device__ __forceinline__ void k45_block_constants(const uint8_t* sbp, int b, float& S, float& M) {
    const uint8_t* sc12 = sbp + 4;
    int sc, mn;
    if (b < 4) {
        sc = sc12[b] & 0x3F;
        mn = sc12[b + 4] & 0x3F;
    } else {
        sc = (sc12[b + 4] & 0x0F) | ((sc12[b - 4] >> 6) << 4);
        mn = (sc12[b + 4] >> 4) | ((sc12[b] >> 6) << 4);
    }
    const uint32_t hdr = lds32(sbp);
    S = round_to_f16(__fmul_rn(static_cast<float>(sc), h2f(hdr)));
    M = -round_to_f16(__fmul_rn(static_cast<float>(mn), h2f(hdr >> 16)));
}

// Exact requantization of one block of the sub-tile by the whole warp (the blocks that
// requant_fast leaves: non-integer scale factor, clipping, non-finite constants).  Lane k
// takes value k: the low (H = false) or high nibble of byte k of the block's group,
// with Q5_K's fifth bit; min / max come from warp reductions, then requant_block and the
// per-value formula (ggml_quant.py:785-886).  Returns the block's diagnostics.
template <bool Q5, int MODE>
__device__ __noinline__ gq_diag_t k45_block_exact(const uint8_t* sbp, int g, bool H, int lane, uint8_t* codes,
                                                  float* scale, const float* recip) {
    constexpr int QS = Q5 ? 48 : 16;
    const int byte = sbp[QS + 32 * g + lane];
    int q = H ? (byte >> 4) : (byte & 15);
    if (Q5) q |= ((sbp[16 + lane] >> (2 * g + (H ? 1 : 0))) & 1) << 4;
    const int qmin = static_cast<int>(__reduce_min_sync(kFull, static_cast<unsigned>(q)));
    const int qmax = static_cast<int>(__reduce_max_sync(kFull, static_cast<unsigned>(q)));
    float S, M;
    k45_block_constants(sbp, 2 * g + (H ? 1 : 0), S, M);
    const Requant p = requant_block(S, M, qmin, qmax, -128, 127, recip);
    st_out<MODE>(codes + lane, static_cast<uint8_t>(requant_value(q, p.sf, p.rm, -128, 127)));
    if (lane == 0) st_out<MODE>(scale, p.scale);
    gq_diag_t diag;
    diag.round_err_bits = __float_as_uint(p.round_err);
    diag.clip_err = p.clip_err;
    return diag;
}

// Lane l owns group l of an 8-super-block sub-tile: super-block l/4, group g = l%4, i.e.
// block 2g (low nibbles) and block 2g+1 (high nibbles).  The min / max scan comes first,
// then the two requantization chains, then the codes from the raw words.
template <bool Q5, int MODE>
__device__ __forceinline__ void process_k45(const GqDesc& D, int64_t unit0, int nunits,
                                            const uint8_t* tile, int lane, DiagAcc& acc,
                                            const float* recip) {
    constexpr int UB = Q5 ? 176 : 144;
    constexpr int QS = Q5 ? 48 : 16;   // offset of the nibble bytes
    constexpr int kEHShift = Q5 ? 0 : 4;    // high block: layout shift of bytes 0, 2
    constexpr int kOHShift = Q5 ? 8 : 12;   // and of bytes 1, 3
    const int g = lane & 3;
    const uint32_t sel = (g & 1) ? 0x4432u : 0x4410u;

    const int sb = lane >> 2;
    const bool valid = sb < nunits;
    const uint8_t* sbp = tile + sb * UB;
    // 6-bit scale / min of blocks 2g and 2g+1 (ggml_quant.py:352-375): byte j' of the
    // first / second / third word of the 12 scale bytes, j' = (2g)&3 and (2g)&3 + 1
    const uint32_t hdr = lds32(sbp);
    const uint32_t b0 = __byte_perm(lds32(sbp + 4), 0, sel);
    const uint32_t b1 = __byte_perm(lds32(sbp + 8), 0, sel);
    const uint32_t b2 = __byte_perm(lds32(sbp + 12), 0, sel);
    const uint32_t sc2 = (g < 2) ? (b0 & 0x3F3Fu) : ((b2 & 0x0F0Fu) | ((b0 >> 2) & 0x3030u));
    const uint32_t mn2 = (g < 2) ? (b1 & 0x3F3Fu) : (((b2 >> 4) & 0x0F0Fu) | ((b1 >> 2) & 0x3030u));
    const float d = h2f(hdr);
    const float dmin = h2f(hdr >> 16);
    const int scL = sc2 & 0xFF, scH = sc2 >> 8, mnL = mn2 & 0xFF, mnH = mn2 >> 8;
    GroupWords<Q5> q;
    {
        const uint8_t* qp = sbp + QS + 32 * g;
        const uint4 qa = lds128(qp), qb = lds128(qp + 16);
        q.w[0] = qa.x; q.w[1] = qa.y; q.w[2] = qa.z; q.w[3] = qa.w;
        q.w[4] = qb.x; q.w[5] = qb.y; q.w[6] = qb.z; q.w[7] = qb.w;
        if (Q5) {
            // fifth bit of block k is bit k of qh[j] (ggml_quant.py:311-349): bit 2g for the
            // low nibbles, 2g+1 for the high nibbles; the bits are disjoint from the
            // nibbles, so each merge is a multiply-add
            const uint4 ha = lds128(sbp + 16), hb = lds128(sbp + 32);
            const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t t = hw[i] >> (2 * g), w = q.w[i];
                q.w[i] = (t & 0x01010101u) * 16u + (w & 0x0F0F0F0Fu);
                q.h[Q5 ? i : 0] = (t & 0x02020202u) * 8u + ((w >> 4) & 0x0F0F0F0Fu);
            }
        }
    }

    // codes / values of block 2g, then 2g+1: unit ou, byte 64g of it (unpermuted, the
    // warp's 8 units are consecutive and lane l writes bytes 64l.. of them); the block
    // scales of the pair sit at off / 32
    const int64_t off = D.perm_heads == 0 ? unit0 * 256 + 64 * lane : permute_unit(D, unit0 + sb) * 256 + 64 * g;
    if (MODE & kOutCodes) {
        // block min / max of the codes (16-bit-lane SIMD), two words per step
        uint32_t mnEL, mxEL, mnOL, mxOL, mnEH, mxEH, mnOH, mxOH;
        {
            uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
            group_layouts(q, 0, a0, a1, a2, a3);
            group_layouts(q, 1, c0, c1, c2, c3);
            mnEL = vmin16(a0, c0); mxEL = vmax16(a0, c0);
            mnOL = vmin16(a1, c1); mxOL = vmax16(a1, c1);
            mnEH = vmin16(a2, c2); mxEH = vmax16(a2, c2);
            mnOH = vmin16(a3, c3); mxOH = vmax16(a3, c3);
        }
#pragma unroll
        for (int i = 2; i < 8; i += 2) {
            uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
            group_layouts(q, i, a0, a1, a2, a3);
            group_layouts(q, i + 1, c0, c1, c2, c3);
            mnEL = vmin16(mnEL, a0, c0); mxEL = vmax16(mxEL, a0, c0);
            mnOL = vmin16(mnOL, a1, c1); mxOL = vmax16(mxOL, a1, c1);
            mnEH = vmin16(mnEH, a2, c2); mxEH = vmax16(mxEH, a2, c2);
            mnOH = vmin16(mnOH, a3, c3); mxOH = vmax16(mxOH, a3, c3);
        }
        const uint32_t aminL = vmin16(mnEL, mnOL >> 8), amaxL = vmax16(mxEL, mxOL >> 8);
        const uint32_t aminH = vmin16(mnEH >> kEHShift, mnOH >> kOHShift);
        const uint32_t amaxH = vmax16(mxEH >> kEHShift, mxOH >> kOHShift);
        const int qminL = min(aminL & 0xFFFF, aminL >> 16), qmaxL = max(amaxL & 0xFFFF, amaxL >> 16);
        const int qminH = min(aminH & 0xFFFF, aminH >> 16), qmaxH = max(amaxH & 0xFFFF, amaxH >> 16);

        // block constants f16(f32 product), min negated (ggml_quant.py:771-777), then
        // requantize_symmetric (ggml_quant.py:785-886) for the common case (P = -M)
        float SL, SH, PL, PH;
        block_constants_h2(sc2, mn2, hdr, SL, SH, PL, PH);
        const FastRequant pL = requant_fast(SL, PL, qminL, qmaxL, recip);
        const FastRequant pH = requant_fast(SH, PH, qminH, qmaxH, recip);
        if (valid) {
            st_out<MODE>(reinterpret_cast<float2*>(D.scales + (off >> 5)), make_float2(pL.scale, pH.scale));
            acc.add(fmaxf(pL.round_err, pH.round_err), 0);
        }
        constexpr uint32_t kBias = 0x400u;   // lane value q*sf + rm + bias stays in [0, 4096)
        const uint32_t sfiL = static_cast<uint32_t>(pL.sfi), sfiH = static_cast<uint32_t>(pH.sfi);
        const uint32_t KL = static_cast<uint32_t>(pL.rm + static_cast<int>(kBias)) * 0x00010001u;
        const uint32_t KH = static_cast<uint32_t>(pH.rm + static_cast<int>(kBias)) * 0x00010001u;
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // low nibbles: EL*sf + K and high32(OL * (sf << 24)) + K; high nibbles:
            // (EH*sf + 16K) >> 4 and high32(OH * (sf << 20)) + K (Q5_K: as the low ones);
            // the low bytes of the 16-bit lanes are the codes (the bias has a zero low byte)
            uint32_t el, ol, eh, oh;
            group_layouts(q, i, el, ol, eh, oh);
            lo[i] = codes_word(el * sfiL + KL, mad_hi(ol, sfiL << 24, KL));
            hi[i] = Q5 ? codes_word(eh * sfiH + KH, mad_hi(oh, sfiH << 24, KH))
                       : codes_word((eh * sfiH + (KH << 4)) >> 4, mad_hi(oh, sfiH << 20, KH));
        }
        uint8_t* base = D.codes + off;
        if ((MODE & kOutSmem) == 0 && (reinterpret_cast<uintptr_t>(D.codes) & 31u) == 0) {
            // a block's 32 codes as one 32-byte store: whole sectors, half the instructions
            if (valid && pL.good) stg256(base, lo);
            if (valid && pH.good) stg256(base + 32, hi);
        } else {
            if (valid && pL.good) {
                st_out128<MODE>(base, make_uint4(lo[0], lo[1], lo[2], lo[3]));
                st_out128<MODE>(base + 16, make_uint4(lo[4], lo[5], lo[6], lo[7]));
            }
            if (valid && pH.good) {
                st_out128<MODE>(base + 32, make_uint4(hi[0], hi[1], hi[2], hi[3]));
                st_out128<MODE>(base + 48, make_uint4(hi[4], hi[5], hi[6], hi[7]));
            }
        }
        // the other blocks (about 0.5%): one warp pass each, after the scale stores above;
        // a block with finite constants is finished from its lane's r and sf0, one with a
        // non-finite S or M is recomputed from the tile
        unsigned pending = __ballot_sync(kFull, valid && !(pL.good && pH.good));
        if (pending) __syncwarp();
        while (pending) {
            const int src = __ffs(pending) - 1;
            pending &= pending - 1;
            const int which = __shfl_sync(kFull, (pL.good ? 0 : 1) | (pH.good ? 0 : 2) | (pL.finite ? 0 : 4) |
                                                     (pH.finite ? 0 : 8), src);
            const int64_t soff = __shfl_sync(kFull, off, src);
            const int sg = src & 3;
            const uint8_t* ssbp = tile + (src >> 2) * UB;
            const int byte = ssbp[QS + 32 * sg + lane];
            int qlo = byte & 15, qhi = byte >> 4;
            if (Q5) {
                const int hb = ssbp[16 + lane] >> (2 * sg);
                qlo |= (hb & 1) << 4;
                qhi |= (hb & 2) << 3;
            }
#pragma unroll
            for (int side = 0; side < 2; ++side) {
                if (!(which & (1 << side))) continue;
                gq_diag_t e;
                if (which & (4 << side)) {
                    e = k45_block_exact<Q5, MODE>(ssbp, sg, side == 1, lane, D.codes + soff + 32 * side,
                                            D.scales + (soff >> 5) + side, recip);
                } else {
                    const float bS = __shfl_sync(kFull, side ? SH : SL, src);
                    const float br = __shfl_sync(kFull, side ? pH.r : pL.r, src);
                    float bsf0 = __shfl_sync(kFull, side ? pH.sf0 : pL.sf0, src);
                    const float bden = __shfl_sync(kFull, side ? pH.den : pL.den, src);
                    if (!(bsf0 > 0.98f)) bsf0 = exact_sf0(bden);
                    e = finish_block<MODE>(side ? qhi : qlo, bS, br, bsf0, -128, 127, D.codes + soff + 32 * side + lane,
                                     D.scales + (soff >> 5) + side, lane);
                }
                acc.add(__uint_as_float(e.round_err_bits), e.clip_err);
            }
        }
    }
    if ((MODE & kOutF32) && valid) {
        // gguf-py dequantize: (d*sc)*q - dmin*m, each product rounded
        // (Q4_K/Q5_K.dequantize_blocks)
        const float dsL = __fmul_rn(d, static_cast<float>(scL));
        const float dmL = __fmul_rn(dmin, static_cast<float>(mnL));
        const float dsH = __fmul_rn(d, static_cast<float>(scH));
        const float dmH = __fmul_rn(dmin, static_cast<float>(mnH));
        float* vdst = D.values + off;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t el, ol, eh, oh;
            group_layouts(q, i, el, ol, eh, oh);
            const uint32_t ql = codes_word(el, ol >> 8);
            const uint32_t qh = codes_word(eh >> kEHShift, oh >> kOHShift);
            stg128f(vdst + 4 * i, __fsub_rn(__fmul_rn(dsL, static_cast<float>(byte_of(ql, 0))), dmL),
                    __fsub_rn(__fmul_rn(dsL, static_cast<float>(byte_of(ql, 1))), dmL),
                    __fsub_rn(__fmul_rn(dsL, static_cast<float>(byte_of(ql, 2))), dmL),
                    __fsub_rn(__fmul_rn(dsL, static_cast<float>(byte_of(ql, 3))), dmL));
            stg128f(vdst + 32 + 4 * i, __fsub_rn(__fmul_rn(dsH, static_cast<float>(byte_of(qh, 0))), dmH),
                    __fsub_rn(__fmul_rn(dsH, static_cast<float>(byte_of(qh, 1))), dmH),
                    __fsub_rn(__fmul_rn(dsH, static_cast<float>(byte_of(qh, 2))), dmH),
                    __fsub_rn(__fmul_rn(dsH, static_cast<float>(byte_of(qh, 3))), dmH));
        }
    }
}

// ---------------------------------------------------------------------------------------
// Q6_K: ql[128] | qh[64] | scales int8[16] | d  (ggml_quant.py:662-679) -> 16 blocks of 16
// ---------------------------------------------------------------------------------------

// STRIDE: bytes from one super-block of the tile to the next (210 when packed)
template <int MODE, int STRIDE = 210>
__device__ __forceinline__ void process_q6k(const GqDesc& D, int64_t unit0, int nunits,
                                            const uint8_t* tile, int lane) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int c = 32 * r + lane;      // block of 16 values within the tile
        const int sb = c >> 4;
        if (sb >= nunits) continue;
        const int kb = c & 15;
        const uint8_t* sbp = tile + sb * STRIDE;
        const float d = h2f(lds16(sbp + 208));
        const int sc = static_cast<int>(static_cast<int8_t>(sbp[192 + kb]));
        // value 128*hh + 32*g + j: nibble of ql[64hh + 32(g&1) + j] (low for g<2),
        // high bits 2g..2g+1 of qh[32hh + j] (ggml_quant.py:274-308)
        const int hh = kb >> 3, g = (kb >> 1) & 3, j0 = 16 * (kb & 1);
        const uint4 ql = lds128_align2<(MODE & kOutSmem) != 0>(sbp + 64 * hh + 32 * (g & 1) + j0);
        const uint4 qh = lds128_align2<(MODE & kOutSmem) != 0>(sbp + 128 + 32 * hh + j0);
        const int qls = 4 * (g >> 1), qhs = 2 * g;
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
        const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
        uint32_t code[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = ((lw[i] >> qls) & 0x0F0F0F0Fu) | (((hw[i] >> qhs) & 0x03030303u) << 4);
            code[i] = (v + 0x60606060u) ^ 0x80808080u;   // 6-bit v - 32 as int8, per byte
        }
        const int64_t ou = permute_unit(D, unit0 + sb);
        const int64_t off = ou * 256 + 16 * kb;
        if (MODE & kOutCodes) {
            st_out128<MODE>(D.codes + off, make_uint4(code[0], code[1], code[2], code[3]));
            // block scale f16(f32(sc) * f32(d)) (ggml_quant.py:771-773), no requant (:700)
            st_out<MODE>(D.scales + ou * 16 + kb, round_to_f16(__fmul_rn(static_cast<float>(sc), d)));
        }
        if (MODE & kOutF32) {
            // gguf-py Q6_K.dequantize_blocks: (d * sc) * q
            const float dd = __fmul_rn(d, static_cast<float>(sc));
            float* dst = D.values + off;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    v[b] = __fmul_rn(dd, static_cast<float>(static_cast<int8_t>(byte_of(code[i], b))));
                stg128f(dst + 4 * i, v[0], v[1], v[2], v[3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// Q8_0: d | int8[32]   and   Q4_0: d | nibbles[16]   (ggml_quant.py:136-210)
// ---------------------------------------------------------------------------------------

template <bool Q4, int MODE>
__device__ __forceinline__ void process_q0(const GqDesc& D, int64_t unit0, int nunits,
                                           const uint8_t* tile, int lane) {
    constexpr int UB = Q4 ? 18 : 34;
    if ((MODE & kOutCodes) && lane < nunits) {
        st_out<MODE>(D.scales + permute_unit(D, unit0 + lane), h2f(lds16(tile + UB * lane)));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int c = 32 * r + lane;
        const int b = c >> 1;
        const int h = c & 1;
        if (b >= nunits) continue;
        const uint8_t* bp = tile + UB * b;
        const uint4 xv = lds128_align2<(MODE & kOutSmem) != 0>(bp + 2 + (Q4 ? 0 : 16 * h));
        uint32_t x[4] = {xv.x, xv.y, xv.z, xv.w};
        if (Q4) {
            // value j: low nibble of byte j, value 16+j: high nibble; int4 byte = (n-8)&15 = n^8
#pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = ((x[i] >> (4 * h)) & 0x0F0F0F0Fu) ^ 0x08080808u;
        }
        const int64_t off = permute_unit(D, unit0 + b) * 32 + 16 * h;
        if (MODE & kOutCodes) st_out128<MODE>(D.codes + off, make_uint4(x[0], x[1], x[2], x[3]));
        if (MODE & kOutF32) {
            const float d = h2f(lds16(bp));
            float* dst = D.values + off;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    // Q4_0: d * (n - 8); Q8_0: x * d (gguf-py dequantize_blocks)
                    const int q = Q4 ? (static_cast<int>(((x[i] >> (8 * j)) & 0xF) ^ 8) - 8)
                                     : static_cast<int>(static_cast<int8_t>(byte_of(x[i], j)));
                    v[j] = Q4 ? __fmul_rn(d, static_cast<float>(q)) : __fmul_rn(static_cast<float>(q), d);
                }
                stg128f(dst + 4 * i, v[0], v[1], v[2], v[3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// Q4_1 / Q5_0 / Q5_1 (ggml_quant.py:174-271; gguf_conversion.py:149-161) and the 16-value
// K-quants Q2_K / Q3_K (ggml_quant.py:398-498, 587-623): one lane per output block, which
// decodes, requantizes where the format is asymmetric, and stores its codes.
// ---------------------------------------------------------------------------------------

// 32 bits from a 2-byte-aligned shared address
__device__ __forceinline__ uint32_t lds32_align2(const uint8_t* p) { return lds16(p) | (lds16(p + 2) << 16); }

// 4 bits b0..b3 -> bit 4 of bytes 0..3 (the fifth bit of four 5-bit codes)
__device__ __forceinline__ uint32_t spread_bits4(uint32_t b) { return ((b * 0x00204081u) & 0x01010101u) << 4; }

// Codes of one block with requantization parameters p (any scale factor, with clipping).
__device__ __forceinline__ uint32_t requant_word(uint32_t q4, const Requant& p) {
    if (p.fast && !p.clip) {
        const uint32_t k2 = static_cast<uint32_t>(p.rm + static_cast<int>(kLaneBias)) * 0x00010001u;
        return requant_word_fast(q4, static_cast<uint32_t>(p.sfi), k2, false, 0u, 0u);
    }
    return requant_word_general(q4, p);
}

__device__ __forceinline__ void minmax_words(const uint32_t* q, int n, int& qmin, int& qmax) {
    uint32_t mn = 0xFFFFFFFFu, mx = 0u;
    for (int i = 0; i < n; ++i) {
        mn = vmin16(vmin16(mn, q[i] & 0x00FF00FFu), (q[i] >> 8) & 0x00FF00FFu);
        mx = vmax16(vmax16(mx, q[i] & 0x00FF00FFu), (q[i] >> 8) & 0x00FF00FFu);
    }
    qmin = min(mn & 0xFFFF, mn >> 16);
    qmax = max(mx & 0xFFFF, mx >> 16);
}

template <int TYPE, int MODE>
__device__ __forceinline__ void process_q32(const GqDesc& D, int64_t unit0, int nunits, const uint8_t* tile,
                                            int lane, DiagAcc& acc, const float* recip) {
    constexpr bool kQ5 = TYPE != GQ_TYPE_Q4_1;
    constexpr bool kAsym = TYPE != GQ_TYPE_Q5_0;
    constexpr int UB = Fmt<TYPE>::kUnitBytes;
    constexpr int QH = TYPE == GQ_TYPE_Q5_0 ? 2 : 4;               // offset of qh (Q5_x)
    constexpr int QS = TYPE == GQ_TYPE_Q4_1 ? 4 : (TYPE == GQ_TYPE_Q5_0 ? 6 : 8);
    const bool valid = lane < nunits;
    const uint8_t* bp = tile + UB * lane;
    const float d = h2f(lds16(bp));
    const float m = kAsym ? h2f(lds16(bp + 2)) : 0.0f;
    const uint32_t qh = kQ5 ? lds32_align2(bp + QH) : 0u;
    const uint4 nb = lds128_align2<(MODE & kOutSmem) != 0>(bp + QS);
    const uint32_t nw[4] = {nb.x, nb.y, nb.z, nb.w};
    uint32_t q[8];   // values 0..15: low nibbles of bytes 0..15; 16..31: high nibbles
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        q[i] = nw[i] & 0x0F0F0F0Fu;
        q[4 + i] = (nw[i] >> 4) & 0x0F0F0F0Fu;
        if (kQ5) {
            q[i] |= spread_bits4((qh >> (4 * i)) & 0xFu);
            q[4 + i] |= spread_bits4((qh >> (16 + 4 * i)) & 0xFu);
        }
    }
    const int64_t ou = permute_unit(D, unit0 + lane);
    if (MODE & kOutCodes) {
        uint32_t c[8];
        float scale;
        if (kAsym) {
            // requantize_symmetric on the raw constants [d, m] (gguf_conversion.py:155-161)
            int qmin, qmax;
            minmax_words(q, 8, qmin, qmax);
            const Requant p = requant_block(d, m, qmin, qmax, -128, 127, recip);
            scale = p.scale;
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = requant_word(q[i], p);
            if (valid) acc.add(p.round_err, p.clip_err);
        } else {
            // Q5_0: codes v - 16 as int8, per byte (v <= 31): (v + 0x70) ^ 0x80
            scale = d;
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = (q[i] + 0x70707070u) ^ 0x80808080u;
        }
        if (valid) {
            st_out<MODE>(D.scales + ou, scale);
            st_out128<MODE>(D.codes + ou * 32, make_uint4(c[0], c[1], c[2], c[3]));
            st_out128<MODE>(D.codes + ou * 32 + 16, make_uint4(c[4], c[5], c[6], c[7]));
        }
    }
    if ((MODE & kOutF32) && valid) {
        // gguf-py: Q4_1 / Q5_1 (d * q) + m, Q5_0 d * (q - 16)
        float* dst = D.values + ou * 32;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int qv = static_cast<int>(byte_of(q[i], b));
                v[b] = kAsym ? __fadd_rn(__fmul_rn(d, static_cast<float>(qv)), m)
                             : __fmul_rn(d, static_cast<float>(qv - 16));
            }
            stg128f(dst + 4 * i, v[0], v[1], v[2], v[3]);
        }
    }
}

// STRIDE: bytes from one super-block of the tile to the next (the unit size when packed)
template <int TYPE, int MODE, int STRIDE = Fmt<TYPE>::kUnitBytes>
__device__ __forceinline__ void process_k16(const GqDesc& D, int64_t unit0, int nunits, const uint8_t* tile,
                                            int lane, DiagAcc& acc, const float* recip) {
    constexpr bool kQ2 = TYPE == GQ_TYPE_Q2_K;
    constexpr int UB = Fmt<TYPE>::kUnitBytes;
#pragma unroll 1
    for (int r = 0; r < 4; ++r) {
        const int c = 32 * r + lane;      // block of 16 values within the tile
        const int sb = c >> 4;
        const bool valid = sb < nunits;
        const int kb = c & 15;
        const uint8_t* sbp = tile + sb * STRIDE;
        const int h = kb >> 3, j = (kb >> 1) & 3, b0 = 16 * (kb & 1);
        uint32_t q[4];
        float d, dmin = 0.0f;
        int sc, mn = 0;
        if (kQ2) {
            // scales[16] | qs[64] | d | dmin; value 128h + 32j + b = bits 2j..2j+1 of qs[32h + b]
            const uint32_t sbyte = sbp[kb];
            sc = sbyte & 0xF;
            mn = sbyte >> 4;
            d = h2f(lds16(sbp + 80));
            dmin = h2f(lds16(sbp + 82));
            const uint4 x = lds128_align2<(MODE & kOutSmem) != 0>(sbp + 16 + 32 * h + b0);
            const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) q[i] = (xw[i] >> (2 * j)) & 0x03030303u;
        } else {
            // hmask[32] | qs[64] | scales[12] | d; third bit = bit 4h + j of hmask[b]; scale
            // kb: low 4 bits from byte kb (low nibble) or kb - 8 (high nibble), top 2 bits
            // from bits 2(kb/4).. of byte 8 + kb % 4, minus 32
            const uint8_t* sp = sbp + 96;
            const int low = kb < 8 ? (sp[kb] & 0xF) : (sp[kb - 8] >> 4);
            const int top = (sp[8 + (kb & 3)] >> (2 * (kb >> 2))) & 3;
            sc = (low | (top << 4)) - 32;
            d = h2f(lds16(sbp + 108));
            const uint4 x = lds128_align2<(MODE & kOutSmem) != 0>(sbp + 32 + 32 * h + b0);
            const uint4 hm = lds128_align2<(MODE & kOutSmem) != 0>(sbp + b0);
            const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
            const uint32_t hw[4] = {hm.x, hm.y, hm.z, hm.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
                q[i] = ((xw[i] >> (2 * j)) & 0x03030303u) | (((hw[i] >> (4 * h + j)) & 0x01010101u) << 2);
        }
        const int64_t ou = permute_unit(D, unit0 + sb);
        if (MODE & kOutCodes) {
            // block constants f16(f32 product), min negated (ggml_quant.py:771-777)
            const float S = round_to_f16(__fmul_rn(static_cast<float>(sc), d));
            uint32_t cw[4];
            if (kQ2) {
                const float M = -round_to_f16(__fmul_rn(static_cast<float>(mn), dmin));
                int qmin, qmax;
                minmax_words(q, 4, qmin, qmax);
                const Requant p = requant_block(S, M, qmin, qmax, -128, 127, recip);
#pragma unroll
                for (int i = 0; i < 4; ++i) cw[i] = requant_word(q[i], p);
                if (valid) {
                    acc.add(p.round_err, p.clip_err);
                    st_out<MODE>(D.scales + ou * 16 + kb, p.scale);
                }
            } else {
                // Q3_K: codes q - 4 (per byte, q <= 7: (q + 0x7C) ^ 0x80), scale f16(sc * d)
#pragma unroll
                for (int i = 0; i < 4; ++i) cw[i] = (q[i] + 0x7C7C7C7Cu) ^ 0x80808080u;
                if (valid) st_out<MODE>(D.scales + ou * 16 + kb, S);
            }
            if (valid) st_out128<MODE>(D.codes + ou * 256 + 16 * kb, make_uint4(cw[0], cw[1], cw[2], cw[3]));
        }
        if ((MODE & kOutF32) && valid) {
            // gguf-py: Q2_K (d*sc)*q - dmin*m; Q3_K (d*sc)*(q - 4)
            const float dl = __fmul_rn(d, static_cast<float>(sc));
            const float ml = __fmul_rn(dmin, static_cast<float>(mn));
            float* dst = D.values + ou * 256 + 16 * kb;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float v[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int qv = static_cast<int>(byte_of(q[i], b));
                    v[b] = kQ2 ? __fsub_rn(__fmul_rn(dl, static_cast<float>(qv)), ml)
                               : __fmul_rn(dl, static_cast<float>(qv - 4));
                }
                stg128f(dst + 4 * i, v[0], v[1], v[2], v[3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// The persistent per-warp pipeline shared by all block formats
// ---------------------------------------------------------------------------------------

template <int TYPE, int MODE, bool SMALL = false>
__global__ void __launch_bounds__(std::conditional<SMALL, FmtSmall<TYPE>, Fmt<TYPE>>::type::kThreads,
                                  TYPE == GQ_TYPE_Q4_K ? GQ_MIN_BLOCKS : (TYPE == GQ_TYPE_Q5_K ? 2 : 1))
    gq_convert_kernel(const __grid_constant__ GqBatch batch) {
    using F = typename std::conditional<SMALL, FmtSmall<TYPE>, Fmt<TYPE>>::type;
    constexpr bool kBulk = F::kBulk;
    extern __shared__ __align__(16) uint8_t smem[];
    // exact reciprocals 1/k, k = 1..16, for the block-scale division of requant_block
    __shared__ float recip[17];
    // one mbarrier per stage of each warp's ring (bulk-copy formats)
    __shared__ uint64_t bars[kBulk ? F::kWarps * F::kStages : 1];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    uint64_t* wbar = bars + (kBulk ? warp * F::kStages : 0);
    if (threadIdx.x < 17) recip[threadIdx.x] = threadIdx.x ? __fdiv_rn(1.0f, static_cast<float>(threadIdx.x)) : 0.0f;
    if (kBulk && lane == 0) {
        for (int s = 0; s < F::kStages; ++s) mbar_init(&wbar[s], 1);
        mbar_init_fence();
    }
    __syncthreads();
    uint8_t* ring = smem + warp * (F::kStages * F::kStageBytes);
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * F::kWarps;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * F::kWarps + warp;
    const int64_t total = batch.total_tiles;

    DescCursor issue_cur, proc_cur;
    int64_t t_issue = first;
#pragma unroll
    for (int s = 0; s < F::kStages - 1; ++s) {
        if constexpr (kBulk) {
            if (lane == 0) issue_tile_bulk<F>(batch, issue_cur, t_issue, ring + s * F::kStageBytes, &wbar[s]);
        } else {
            issue_tile<F>(batch, issue_cur, t_issue, ring + s * F::kStageBytes, lane);
            cp_async_commit();
        }
        t_issue += nwarps;
    }

    DiagAcc acc;
    int stage = 0;
    uint32_t phase = 0;   // bit s: parity of stage s's next completion
    for (int64_t t = first; t < total; t += nwarps) {
        if constexpr (kBulk) {
            const bool ok = mbar_wait(&wbar[stage], (phase >> stage) & 1u);
            if (__any_sync(kFull, !ok)) {
                // give up: record it, let the copies still owed to this warp's ring land
                // (each wait again bounded), and stop
                if (lane == 0) atomicOr(&gq_kernel_errors, kErrWaitTimeout);
                for (int k = 0; k < F::kStages - 1; ++k) {
                    const int s = (stage + k) % F::kStages;
                    if (t + k * nwarps < total) mbar_wait(&wbar[s], (phase >> s) & 1u);
                }
                break;
            }
            phase ^= 1u << stage;
        } else {
            cp_async_wait<F::kStages - 2>();
            __syncwarp();
        }
        // refill the stage consumed in the previous iteration
        const int refill = (stage == 0) ? F::kStages - 1 : stage - 1;
        if constexpr (kBulk) {
            if (lane == 0) issue_tile_bulk<F>(batch, issue_cur, t_issue, ring + refill * F::kStageBytes, &wbar[refill]);
        } else {
            issue_tile<F>(batch, issue_cur, t_issue, ring + refill * F::kStageBytes, lane);
            cp_async_commit();
        }
        t_issue += nwarps;

        const GqDesc& D = batch.d[proc_cur.seek(batch, t)];
        const int64_t unit0 = (t - D.tile_begin) * F::kUnitsPerTile;
        const int64_t left = D.n_units - unit0;
        const int nunits = left < F::kUnitsPerTile ? static_cast<int>(left) : F::kUnitsPerTile;
        const uint8_t* tile = ring + stage * F::kStageBytes;
        if (TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K) {
            if (MODE & kOutCodes) acc.retarget(D.diag, lane);
#pragma unroll 1
            for (int j = 0; j < F::kUnitsPerTile / 8; ++j) {
                const int rest = nunits - 8 * j;
                if (rest <= 0) break;
                process_k45<TYPE == GQ_TYPE_Q5_K, MODE>(D, unit0 + 8 * j, rest < 8 ? rest : 8,
                                                           tile + 8 * j * F::kUnitBytes, lane, acc, recip);
            }
        } else if (TYPE == GQ_TYPE_Q6_K) {
#pragma unroll 1
            for (int j = 0; j < F::kUnitsPerTile / 8; ++j) {
                const int rest = nunits - 8 * j;
                if (rest <= 0) break;
                process_q6k<MODE>(D, unit0 + 8 * j, rest < 8 ? rest : 8, tile + 8 * j * F::kUnitBytes, lane);
            }
        } else if (TYPE == GQ_TYPE_Q4_1 || TYPE == GQ_TYPE_Q5_0 || TYPE == GQ_TYPE_Q5_1) {
            if (MODE & kOutCodes) acc.retarget(D.diag, lane);
            process_q32<TYPE, MODE>(D, unit0, nunits, tile, lane, acc, recip);
        } else if (TYPE == GQ_TYPE_Q2_K || TYPE == GQ_TYPE_Q3_K) {
            if (MODE & kOutCodes) acc.retarget(D.diag, lane);
            process_k16<TYPE, MODE>(D, unit0, nunits, tile, lane, acc, recip);
        } else {
            // Q8_0 / Q4_0: sub-tiles of 32 blocks
#pragma unroll 1
            for (int j = 0; j < F::kUnitsPerTile / 32; ++j) {
                const int rest = nunits - 32 * j;
                if (rest <= 0) break;
                process_q0<TYPE == GQ_TYPE_Q4_0, MODE>(D, unit0 + 32 * j, rest < 32 ? rest : 32,
                                                       tile + 32 * j * F::kUnitBytes, lane);
            }
        }
        __syncwarp();
        stage = (stage + 1 == F::kStages) ? 0 : stage + 1;
    }
    if constexpr (!kBulk) cp_async_wait<0>();
    if ((MODE & kOutCodes) && (TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K || TYPE == GQ_TYPE_Q4_1 ||
                               TYPE == GQ_TYPE_Q5_0 || TYPE == GQ_TYPE_Q5_1 || TYPE == GQ_TYPE_Q2_K ||
                               TYPE == GQ_TYPE_Q3_K))
        acc.flush(lane);
}

// ---------------------------------------------------------------------------------------
// F32 / F16 / BF16 pass-through (tile = 4096 bytes), with the head permutation for
// 1-D bias vectors and 2-D float weights
// ---------------------------------------------------------------------------------------

constexpr int kCopyTileBytes = 4096;

template <int ES>
__global__ void __launch_bounds__(kThreads) gq_copy_kernel(const __grid_constant__ GqBatch batch) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarps;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); t < batch.total_tiles;
         t += nwarps) {
        const GqDesc& D = batch.d[find_desc(batch, t)];
        const int64_t b0 = (t - D.tile_begin) * kCopyTileBytes;
        const int64_t nbytes_total = D.n_units * ES;
        const int64_t left = nbytes_total - b0;
        const int nbytes = left < kCopyTileBytes ? static_cast<int>(left) : kCopyTileBytes;
        const uint8_t* src = D.src + b0;
        uint8_t* dst = reinterpret_cast<uint8_t*>(D.values) + b0;
        if (D.perm_heads == 0) {
            // all of the lane's loads go out before its stores (one memory latency per
            // tile instead of one per 512 bytes)
            constexpr int kRounds = kCopyTileBytes / (32 * 16);
            uint4 v[kRounds];
#pragma unroll
            for (int k = 0; k < kRounds; ++k) {
                const int c = lane * 16 + k * 32 * 16;
                if (c + 16 <= nbytes) v[k] = __ldg(reinterpret_cast<const uint4*>(src + c));
            }
#pragma unroll
            for (int k = 0; k < kRounds; ++k) {
                const int c = lane * 16 + k * 32 * 16;
                if (c + 16 <= nbytes) stg128(dst + c, v[k]);
            }
            for (int c = (nbytes & ~15) + lane * ES; c < nbytes; c += 32 * ES) {
                if (ES == 4) *reinterpret_cast<uint32_t*>(dst + c) = *reinterpret_cast<const uint32_t*>(src + c);
                else *reinterpret_cast<uint16_t*>(dst + c) = *reinterpret_cast<const uint16_t*>(src + c);
            }
        } else {
            uint8_t* base = reinterpret_cast<uint8_t*>(D.values);
            const int64_t e0 = b0 / ES;
            for (int e = lane; e < nbytes / ES; e += 32) {
                const int64_t oe = permute_unit(D, e0 + e);
                if (ES == 4) reinterpret_cast<uint32_t*>(base)[oe] = reinterpret_cast<const uint32_t*>(src)[e];
                else reinterpret_cast<uint16_t*>(base)[oe] = reinterpret_cast<const uint16_t*>(src)[e];
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// requantize_symmetric as a standalone scheme (ggml_quant.py:785-886): one thread per block
// ---------------------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreads) gq_requant_kernel(const float* __restrict__ bc,
                                                              const int8_t* __restrict__ codes,
                                                              int64_t n_blocks, int block, int bits,
                                                              float* __restrict__ out_scales,
                                                              int8_t* __restrict__ out_codes,
                                                              gq_diag_t* diag) {
    const int lane = threadIdx.x & 31;
    const int lo_out = -(1 << (bits - 1));
    const int hi_out = (1 << (bits - 1)) - 1;
    DiagAcc acc;
    acc.target = diag;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t start = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    // every lane walks the same number of iterations so the warp-collective flush stays uniform
    const int64_t iters = (n_blocks + stride - 1) / stride;
    for (int64_t it = 0; it < iters; ++it) {
        const int64_t i = start + it * stride;
        if (i >= n_blocks) continue;
        const int8_t* q = codes + i * block;
        int qmin = 127, qmax = -128;
        for (int j = 0; j < block; ++j) {
            qmin = min(qmin, static_cast<int>(q[j]));
            qmax = max(qmax, static_cast<int>(q[j]));
        }
        const Requant p = requant_block(bc[2 * i], bc[2 * i + 1], qmin, qmax, lo_out, hi_out);
        out_scales[i] = p.scale;
        for (int j = 0; j < block; ++j)
            out_codes[i * block + j] = static_cast<int8_t>(requant_value(q[j], p.sf, p.rm, lo_out, hi_out));
        acc.add(p.round_err, p.clip_err);
    }
    acc.flush(lane);
}

// ---------------------------------------------------------------------------------------
// Conversion fused with the Modalix weight layout (ModelGraph._build_conv,
// sima_lmm/model/model_graph.py:1012-1079): codes (rows, cols) -> (cols, rows_padded) and
// block scales (rows, cols / B) -> (cols / B, rows_padded), written in one pass.
//
// A CTA runs two workers of 4 warps; a worker owns a tile of 64 output channels (rows of
// the converted tensor in output order; the llama q/k head permutation becomes a gather of
// source rows) x 256 input channels.  Each warp copies the stored bytes of its 16 rows
// with cp.async: the 16-byte-aligned span around each row's segment, so a unit sits
// `shift` bytes into its slot (0 unless the unit size is not a multiple of 16).  The
// format's decode runs unchanged with its code / scale stores directed to a shared row
// tile (kOutSmem).  The row tile is transposed by ldmatrix (.m16n16 .trans .b8: a thread
// receives 4 consecutive rows of one column) with the rows of each 16x16 matrix chosen so
// that a lane ends up holding 16 consecutive output channels of 2 input channels, written
// out as 16-byte stores: a quarter warp covers 64 contiguous bytes of 2 input channels.
// Output channels rows..rows_padded-1 are the layout's padding: zero codes and unit scales.
// ---------------------------------------------------------------------------------------

template <int TYPE>
struct MxFmt {
    static constexpr int UB = Fmt<TYPE>::kUnitBytes;
    static constexpr bool K = TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K || TYPE == GQ_TYPE_Q6_K ||
                              TYPE == GQ_TYPE_Q2_K || TYPE == GQ_TYPE_Q3_K;
    static constexpr int UNITS = K ? 1 : 8;                 // stored units per row of a tile
    static constexpr int SEG = UNITS * UB;                  // bytes of one row's segment
    // slot stride: the segment plus room for the alignment shift
    static constexpr int STR = (SEG % 16 == 0) ? SEG : ((SEG + 15 + 15) / 16) * 16;
    static constexpr int CH = STR / 16;                     // 16-byte chunks per slot
    static constexpr int NBS = 256 / (TYPE == GQ_TYPE_Q6_K || TYPE == GQ_TYPE_Q2_K || TYPE == GQ_TYPE_Q3_K ? 16 : 32);
    static constexpr int kWarpStaging = 16 * STR + 16;      // + slack for lds128_align2
    static constexpr int kRBytes = 2 * kModalixRows * kModalixCols;   // row tile, both workers
    static constexpr int kSBytes = 2 * kModalixRows * NBS * 4;        // scale tile, both workers
    // two staging buffers per warp: the next tile's copies land during this tile's work
    static constexpr int kSmem = kRBytes + kSBytes + 16 * kWarpStaging + 8192;   // + alignment
};

// Source row of output channel o (inverse of the q/k permutation of
// gguf_conversion.py:314-332: row 2a + t of a head moves to t * D/2 + a).
__device__ __forceinline__ uint32_t modalix_src_row(const GqModalix& m, uint32_t o) {
    if (m.head_dim == 0) return o;
    const uint32_t d = static_cast<uint32_t>(m.head_dim), half = d >> 1;
    const uint32_t h = o / d, rem = o - h * d;
    const uint32_t t = rem >= half ? 1u : 0u, a = rem - t * half;
    return h * d + 2 * a + t;
}

template <int TYPE>
__global__ void __launch_bounds__(256, 2) gq_modalix_kernel(const __grid_constant__ GqModalixBatch b) {
    using X = MxFmt<TYPE>;
    constexpr int MODE = kOutCodes | kOutSmem;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ float recip[17];
    if (threadIdx.x < 17) recip[threadIdx.x] = threadIdx.x ? __fdiv_rn(1.0f, static_cast<float>(threadIdx.x)) : 0.0f;
    // the row tile starts on an 8 KiB boundary: its swizzle key (shared-address bits 8, 9
    // and 12) is then made of bits 0, 1 and 4 of the row index (the offset is added to the
    // shared pointer, not formed through an integer, so that loads through the staging
    // pointers stay shared loads)
    uint8_t* smem = smem_raw + ((8192u - (smem_u32addr(smem_raw) & 8191u)) & 8191u);
    uint8_t* rtile = smem;                                         // 128 rows x 256 bytes
    float* stile = reinterpret_cast<float*>(smem + X::kRBytes);    // 128 rows x NBS
    const uint32_t r_s = smem_u32addr(rtile);
    const uint32_t s_s = smem_u32addr(stile);
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    // Two independent workers per CTA: warps 0-3 and 4-7, each with its own tiles (64 output
    // channels x 256 input channels), its half of the row and scale tiles and its own block
    // barrier, so that one worker's decode overlaps the other's transpose and stores.
    const int half = warp >> 2;           // worker
    const int wq = warp & 3;              // warp within the worker
    const int hid = threadIdx.x & 127;    // thread within the worker
    auto worker_sync = [&]() {
        if (half == 0) {
            asm volatile("bar.sync 1, 128;" ::: "memory");
        } else {
            asm volatile("bar.sync 2, 128;" ::: "memory");
        }
    };
    uint8_t* const staging0 = smem + X::kRBytes + X::kSBytes + warp * 2 * X::kWarpStaging;
    __syncthreads();

    // a worker visits its tiles in increasing order, so each tensor cursor only moves forward
    int c_issue = 0, c_tile = 0;
    auto seek = [&](int& c, uint32_t t) -> const GqModalix& {
        while (c + 1 < b.n && b.d[c + 1].tile_begin <= t) ++c;
        return b.d[c];
    };

    // tile t of the batch: tensor m, row block rb (output channels d0..d0+63), column
    // block cb (256 input channels)
    // (every call commits one cp.async group, empty past the last tile)
    auto issue = [&](uint32_t t, uint8_t* staging) {
        if (t >= b.total_tiles) {
            cp_async_commit();
            return;
        }
        const GqModalix& m = seek(c_issue, t);
        const uint32_t lt = t - m.tile_begin;
        const uint32_t rb = fast_div(lt, m.ncol_mul, m.ncol_shift), cb = lt - rb * m.n_col_tiles;
        const uint32_t rows = static_cast<uint32_t>(m.rows);
        const uint32_t o_lane = rb * kModalixRows + 16 * wq + (lane & 15);
        // lanes l and l + 16 copy row l & 15's segment (the 16-byte-aligned span around it),
        // alternate 16-byte chunks each
        if (o_lane < rows) {
            const int64_t off = (static_cast<int64_t>(modalix_src_row(m, o_lane)) * m.units_per_row + cb * X::UNITS) * X::UB;
            const int64_t end = off + X::SEG;
            uint8_t* dst = staging + (lane & 15) * X::STR;
#pragma unroll
            for (int c = lane >> 4; c < X::CH; c += 2) {
                const int64_t start = (off & ~int64_t(15)) + 16 * c;
                if (start < end) cp_async16(dst + 16 * c, m.src + start, end - start < 16 ? static_cast<int>(end - start) : 16);
            }
        }
        cp_async_commit();
    };

    DiagAcc acc;
    GqDesc dt{};
    dt.codes = rtile;
    dt.scales = stile;

    const uint32_t workers = 2 * gridDim.x;
    uint32_t t = 2 * blockIdx.x + half;
    int buf = 0;
    issue(t, staging0);
    for (; t < b.total_tiles; t += workers, buf ^= 1) {
        // the next tile's copies go to the other buffer (its last reader, this warp's
        // decode two tiles back, is done), then this tile's group is waited for
        __syncwarp();
        issue(t + workers, staging0 + (buf ^ 1) * X::kWarpStaging);
        uint8_t* const staging = staging0 + buf * X::kWarpStaging;
        const GqModalix& m = seek(c_tile, t);
        acc.retarget(m.diag, lane);
        const uint32_t lt = t - m.tile_begin;
        const uint32_t rb = fast_div(lt, m.ncol_mul, m.ncol_shift), cb = lt - rb * m.n_col_tiles;
        const uint32_t rows = static_cast<uint32_t>(m.rows);
        const uint32_t d0 = rb * kModalixRows;
        // rows of this tile below `rows` (0..64)
        const int valid_rows = d0 >= rows ? 0 : (rows - d0 < kModalixRows ? static_cast<int>(rows - d0) : kModalixRows);
        const int shift = static_cast<int>((cb * X::SEG) & 15);   // row starts are 16-byte aligned
        cp_async_wait<1>();
        __syncwarp();
        // phase A: decode this warp's 16 rows into the row tile / scale tile
        if constexpr (X::K) {
#pragma unroll 1
            for (int sub = 0; sub < 2; ++sub) {
                const int left = valid_rows - (16 * wq + 8 * sub);
                const int n = left <= 0 ? 0 : (left < 8 ? left : 8);
                if (n == 0) continue;
                const uint8_t* tile = staging + 8 * sub * X::STR + shift;
                const int u0 = 16 * warp + 8 * sub;
                if constexpr (TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K) {
                    process_k45<TYPE == GQ_TYPE_Q5_K, MODE>(dt, u0, n, tile, lane, acc, recip);
                } else if constexpr (TYPE == GQ_TYPE_Q6_K) {
                    process_q6k<MODE, X::STR>(dt, u0, n, tile, lane);
                } else {
                    process_k16<TYPE, MODE, X::STR>(dt, u0, n, tile, lane, acc, recip);
                }
            }
        } else {
#pragma unroll 1
            for (int j = 0; j < 4; ++j) {
                const int left = valid_rows - (16 * wq + 4 * j);
                const int n = left <= 0 ? 0 : (left < 4 ? left * 8 : 32);
                if (n == 0) continue;
                const uint8_t* tile = staging + 4 * j * X::STR;
                const int u0 = (16 * warp + 4 * j) * 8;
                if constexpr (TYPE == GQ_TYPE_Q8_0 || TYPE == GQ_TYPE_Q4_0) {
                    process_q0<TYPE == GQ_TYPE_Q4_0, MODE>(dt, u0, n, tile, lane);
                } else {
                    process_q32<TYPE, MODE>(dt, u0, n, tile, lane, acc, recip);
                }
            }
        }
        // rows of the worker's half at or past valid_rows are layout padding: zero codes and
        // unit scales in the row and scale tiles, so that the transpose reads every row
        {
            const int first = valid_rows > 16 * wq ? valid_rows - 16 * wq : 0;
            if (first < 16) {
                __syncwarp();
                const uint32_t r0 = r_s + (16 * warp + first) * 256;
                for (int q = lane; q < (16 - first) * 16; q += 32) sts(r0 + 16 * q, make_uint4(0u, 0u, 0u, 0u));
                const uint32_t s0 = s_s + 4 * (16 * warp + first) * X::NBS;
                for (int q = lane; q < (16 - first) * X::NBS; q += 32) sts(s0 + 4 * q, 1.0f);
            }
        }
        worker_sync();
        // phase B: codes leave through ldmatrix transposes.  A
        // warp takes the worker's 16-channel chunks 4 wq..4 wq + 3.  Per chunk, two x2 loads
        // read four 16x16 matrices; lane t addresses row i = t & 15 of matrix mm = t >> 4 (and
        // mm + 2 in the second load): tile row 16 (i >> 2) + 4 mm + (i & 3).  Lane t then holds
        // rows 16 (t & 3)..+15 of channels t / 4 and t / 4 + 8 of the chunk.
        const int64_t rp = m.rows_padded;
        {
            const int i = lane & 15;
            const uint32_t ra = 64 * half + 16 * (i >> 2) + 4 * (lane >> 4) + (i & 3);
            const uint32_t ga = (ra & 3u) | ((ra >> 2) & 4u);   // swizzle key of rows ra and ra + 8
            const int64_t o0 = d0 + 16 * (lane & 3);
            // (every lane runs the ldmatrix loads: they are warp-wide; only the stores of lanes
            // past rows_padded are skipped)
            const bool any = o0 < rp;
            const bool vec = o0 + 16 <= rp && ((reinterpret_cast<uintptr_t>(m.out_codes) | static_cast<uintptr_t>(rp)) & 15) == 0;
            const int ne = !any ? 0 : (rp - o0 < 16 ? static_cast<int>(rp - o0) : 16);
            uint8_t* const dst0 = m.out_codes + static_cast<int64_t>(cb * kModalixCols + (lane >> 2)) * rp + (any ? o0 : 0);
            // all shared reads of the tile first (codes through ldmatrix, this thread's scale
            // quads), then the block barrier that frees the row and scale tiles for the next
            // decode, then the global stores, which so overlap the other warps' work
            constexpr int kNT = X::NBS * 16 / 128;   // scale quads per thread
            uint32_t v[4][8];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                const uint32_t c = 4 * wq + cc;
                const uint32_t a = r_s + ra * 256 + ((c ^ ga ^ (3u * (c >> 3))) << 4);
                ldsm_x2_trans_b8(a, v[cc][0], v[cc][1], v[cc][2], v[cc][3]);            // rows 16q + 0..7
                ldsm_x2_trans_b8(a + 8 * 256, v[cc][4], v[cc][5], v[cc][6], v[cc][7]);  // rows 16q + 8..15
            }
            float sv[kNT][4];
#pragma unroll
            for (int j = 0; j < kNT; ++j) {
                const int task = hid + 128 * j;
                const int bb = task % X::NBS, quad = task / X::NBS;   // scale column, 4 output channels
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    sv[j][e] = __uint_as_float(lds_u32(s_s + 4 * ((64 * half + 4 * quad + e) * X::NBS + bb)));
            }
            // the row and scale tiles are read: the next decode may overwrite them
            worker_sync();
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint8_t* dst = dst0 + static_cast<int64_t>(16 * (4 * wq + cc)) * rp;
                if (vec) {
                    stg128(dst, make_uint4(v[cc][0], v[cc][2], v[cc][4], v[cc][6]));
                    stg128(dst + 8 * rp, make_uint4(v[cc][1], v[cc][3], v[cc][5], v[cc][7]));
                } else if (any) {
                    // (indices fixed at compile time, so that v stays in registers)
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        if (e < ne) {
                            st_global(dst + e, static_cast<uint8_t>(v[cc][2 * (e >> 2)] >> (8 * (e & 3))));
                            st_global(dst + 8 * rp + e, static_cast<uint8_t>(v[cc][2 * (e >> 2) + 1] >> (8 * (e & 3))));
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kNT; ++j) {
                const int task = hid + 128 * j;
                const int bb = task % X::NBS, quad = task / X::NBS;
                const int64_t s0 = d0 + 4 * quad;
                if (s0 >= rp) continue;
                float* dst = m.out_scales + static_cast<int64_t>(cb * X::NBS + bb) * rp + s0;
                if (s0 + 4 <= rp && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                    st_global(reinterpret_cast<float4*>(dst), make_float4(sv[j][0], sv[j][1], sv[j][2], sv[j][3]));
                } else {
                    for (int e = 0; e < 4 && s0 + e < rp; ++e) st_global(dst + e, sv[j][e]);
                }
            }
        }
    }
    cp_async_wait<0>();
    acc.flush(lane);
}

// ---------------------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------------------

namespace {

struct DeviceInfo {
    int sms = 0;
};

DeviceInfo& device_info() {
    static DeviceInfo info[64];
    int dev = 0;
    cudaGetDevice(&dev);
    DeviceInfo& di = info[dev & 63];
    if (di.sms == 0) cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev);
    return di;
}

// Resident CTAs per SM of one kernel instance on the current device (queried once).
template <int TYPE, int MODE, bool SMALL>
int occupancy(int smem) {
    static int per_sm[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int& occ = per_sm[dev & 63];
    if (occ == 0) {
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(gq_convert_kernel<TYPE, MODE, SMALL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &occ, gq_convert_kernel<TYPE, MODE, SMALL>,
                std::conditional<SMALL, FmtSmall<TYPE>, Fmt<TYPE>>::type::kThreads, smem) != cudaSuccess ||
            occ < 1)
            occ = 1;
    }
    return occ;
}

template <int TYPE, int MODE, bool SMALL = false>
int launch_fmt(const GqBatch& b, cudaStream_t s) {
    using F = typename std::conditional<SMALL, FmtSmall<TYPE>, Fmt<TYPE>>::type;
    constexpr int smem = F::kWarps * F::kStages * F::kStageBytes;
    static_assert(smem <= 200 * 1024, "dynamic shared memory per CTA");
    const int occ = occupancy<TYPE, MODE, SMALL>(smem);
    const int64_t want = (b.total_tiles + F::kWarps - 1) / F::kWarps;
    const int64_t cap = static_cast<int64_t>(device_info().sms) * occ;
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    gq_convert_kernel<TYPE, MODE, SMALL><<<blocks, F::kThreads, smem, s>>>(b);
    return static_cast<int>(cudaGetLastError());
}

// Q4_K / Q5_K / Q8_0 / Q4_0: a launch with fewer than 8 tiles per resident warp goes out
// in the small tiles, its batch renumbered for them (the host copy of the parameter block
// is the cost).
template <int TYPE, int MODE>
int launch_k45(const GqBatch& b, cudaStream_t s) {
    using F = Fmt<TYPE>;
    constexpr int smem = F::kWarps * F::kStages * F::kStageBytes;
    const int64_t warps = static_cast<int64_t>(device_info().sms) * occupancy<TYPE, MODE, false>(smem) * F::kWarps;
    if (b.total_tiles >= 8 * warps) return launch_fmt<TYPE, MODE, false>(b, s);
    std::unique_ptr<GqBatch> sb(new (std::nothrow) GqBatch(b));
    if (!sb) return static_cast<int>(cudaErrorMemoryAllocation);
    sb->total_tiles = 0;
    for (int i = 0; i < sb->n; ++i) {
        sb->d[i].tile_begin = sb->total_tiles;
        sb->total_tiles += (sb->d[i].n_units + FmtSmall<TYPE>::kUnitsPerTile - 1) / FmtSmall<TYPE>::kUnitsPerTile;
    }
    return launch_fmt<TYPE, MODE, true>(*sb, s);
}

template <int TYPE>
int launch_modes(int out_mask, const GqBatch& b, cudaStream_t s) {
    if constexpr (TYPE == GQ_TYPE_Q4_K || TYPE == GQ_TYPE_Q5_K || TYPE == GQ_TYPE_Q8_0 || TYPE == GQ_TYPE_Q4_0) {
        switch (out_mask) {
            case kOutCodes: return launch_k45<TYPE, kOutCodes>(b, s);
            case kOutF32: return launch_k45<TYPE, kOutF32>(b, s);
            default: return launch_k45<TYPE, kOutCodes | kOutF32>(b, s);
        }
    }
    switch (out_mask) {
        case kOutCodes: return launch_fmt<TYPE, kOutCodes>(b, s);
        case kOutF32: return launch_fmt<TYPE, kOutF32>(b, s);
        default: return launch_fmt<TYPE, kOutCodes | kOutF32>(b, s);
    }
}

template <int ES>
int launch_copy(const GqBatch& b, cudaStream_t s) {
    const int64_t want = (b.total_tiles + kWarps - 1) / kWarps;
    const int64_t cap = static_cast<int64_t>(device_info().sms) * 8;
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    gq_copy_kernel<ES><<<blocks, kThreads, 0, s>>>(b);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

int64_t tiles_for(int type, int64_t n_units) {
    int upt;
    switch (type) {
        case GQ_TYPE_Q4_K: upt = Fmt<GQ_TYPE_Q4_K>::kUnitsPerTile; break;
        case GQ_TYPE_Q5_K: upt = Fmt<GQ_TYPE_Q5_K>::kUnitsPerTile; break;
        case GQ_TYPE_Q6_K: upt = Fmt<GQ_TYPE_Q6_K>::kUnitsPerTile; break;
        case GQ_TYPE_Q8_0: upt = Fmt<GQ_TYPE_Q8_0>::kUnitsPerTile; break;
        case GQ_TYPE_Q4_0: upt = Fmt<GQ_TYPE_Q4_0>::kUnitsPerTile; break;
        case GQ_TYPE_Q4_1: upt = Fmt<GQ_TYPE_Q4_1>::kUnitsPerTile; break;
        case GQ_TYPE_Q5_0: upt = Fmt<GQ_TYPE_Q5_0>::kUnitsPerTile; break;
        case GQ_TYPE_Q5_1: upt = Fmt<GQ_TYPE_Q5_1>::kUnitsPerTile; break;
        case GQ_TYPE_Q2_K: upt = Fmt<GQ_TYPE_Q2_K>::kUnitsPerTile; break;
        case GQ_TYPE_Q3_K: upt = Fmt<GQ_TYPE_Q3_K>::kUnitsPerTile; break;
        case GQ_TYPE_F32: upt = kCopyTileBytes / 4; break;
        default: upt = kCopyTileBytes / 2; break;   // F16, BF16
    }
    return (n_units + upt - 1) / upt;
}

namespace {

template <int TYPE>
int launch_modalix_t(const GqModalixBatch& m, cudaStream_t s) {
    using X = MxFmt<TYPE>;
    static_assert(X::kSmem <= 113 * 1024, "two CTAs per SM");
    static int per_sm[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int& occ = per_sm[dev & 63];
    if (occ == 0) {
        cudaFuncSetAttribute(gq_modalix_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, X::kSmem);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gq_modalix_kernel<TYPE>, 256, X::kSmem) != cudaSuccess ||
            occ < 1)
            occ = 1;
    }
    const int64_t cap = static_cast<int64_t>(device_info().sms) * occ;
    const int64_t want = (static_cast<int64_t>(m.total_tiles) + 1) / 2;   // two workers per CTA
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    gq_modalix_kernel<TYPE><<<blocks, 256, X::kSmem, s>>>(m);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace

int kernel_errors(bool clear, uint32_t* flags) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, gq_kernel_errors, sizeof(v));
    if (e == cudaSuccess && clear && v != 0) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(gq_kernel_errors, &zero, sizeof(zero));
    }
    *flags = v;
    return static_cast<int>(e);
}

int launch_modalix(int type, const GqModalixBatch& m, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (type) {
        case GQ_TYPE_Q4_K: return launch_modalix_t<GQ_TYPE_Q4_K>(m, s);
        case GQ_TYPE_Q5_K: return launch_modalix_t<GQ_TYPE_Q5_K>(m, s);
        case GQ_TYPE_Q6_K: return launch_modalix_t<GQ_TYPE_Q6_K>(m, s);
        case GQ_TYPE_Q8_0: return launch_modalix_t<GQ_TYPE_Q8_0>(m, s);
        case GQ_TYPE_Q4_0: return launch_modalix_t<GQ_TYPE_Q4_0>(m, s);
        case GQ_TYPE_Q4_1: return launch_modalix_t<GQ_TYPE_Q4_1>(m, s);
        case GQ_TYPE_Q5_0: return launch_modalix_t<GQ_TYPE_Q5_0>(m, s);
        case GQ_TYPE_Q5_1: return launch_modalix_t<GQ_TYPE_Q5_1>(m, s);
        case GQ_TYPE_Q2_K: return launch_modalix_t<GQ_TYPE_Q2_K>(m, s);
        case GQ_TYPE_Q3_K: return launch_modalix_t<GQ_TYPE_Q3_K>(m, s);
        default: return static_cast<int>(cudaErrorInvalidValue);
    }
}

int launch_batch(int type, int out_mask, const GqBatch& b, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (type) {
        case GQ_TYPE_Q4_K: return launch_modes<GQ_TYPE_Q4_K>(out_mask, b, s);
        case GQ_TYPE_Q5_K: return launch_modes<GQ_TYPE_Q5_K>(out_mask, b, s);
        case GQ_TYPE_Q6_K: return launch_modes<GQ_TYPE_Q6_K>(out_mask, b, s);
        case GQ_TYPE_Q8_0: return launch_modes<GQ_TYPE_Q8_0>(out_mask, b, s);
        case GQ_TYPE_Q4_0: return launch_modes<GQ_TYPE_Q4_0>(out_mask, b, s);
        case GQ_TYPE_Q4_1: return launch_modes<GQ_TYPE_Q4_1>(out_mask, b, s);
        case GQ_TYPE_Q5_0: return launch_modes<GQ_TYPE_Q5_0>(out_mask, b, s);
        case GQ_TYPE_Q5_1: return launch_modes<GQ_TYPE_Q5_1>(out_mask, b, s);
        case GQ_TYPE_Q2_K: return launch_modes<GQ_TYPE_Q2_K>(out_mask, b, s);
        case GQ_TYPE_Q3_K: return launch_modes<GQ_TYPE_Q3_K>(out_mask, b, s);
        case GQ_TYPE_F32: return launch_copy<4>(b, s);
        default: return launch_copy<2>(b, s);
    }
}

int launch_requant(const float* bc, const int8_t* codes, int64_t n_blocks, int block, int bits,
                   float* out_scales, int8_t* out_codes, gq_diag_t* diag, void* stream) {
    const int64_t want = (n_blocks + kThreads - 1) / kThreads;
    const int64_t cap = static_cast<int64_t>(device_info().sms) * 8;
    const int blocks = static_cast<int>(want < cap ? want : cap);
    if (blocks <= 0) return 0;
    gq_requant_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        bc, codes, n_blocks, block, bits, out_scales, out_codes, diag);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace gq

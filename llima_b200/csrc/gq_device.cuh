// Device helpers for the GGUF conversion kernels (sm_100a).
//
// Exactness: every floating-point step that the reference performs in numpy f32 is
// written with an explicitly rounded intrinsic (__fmul_rn, __fadd_rn, __fsub_rn,
// __fdiv_rn) so that no FMA contraction or fast-math substitution can change a bit.
// The library is also compiled with -fmad=false and without --use_fast_math (no FTZ).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "gq_internal.h"

namespace gq {

// ---- f16 <-> f32 ------------------------------------------------------------------

__device__ __forceinline__ float h2f(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xFFFFu)));
}

__device__ __forceinline__ __half2 u32_as_h2(uint32_t w) {
    __half2 h;
    static_assert(sizeof(h) == sizeof(w), "half2 is 32 bits");
    memcpy(&h, &w, sizeof(w));
    return h;
}

// numpy's f32 -> f16 astype: round to nearest even, overflow to inf, subnormals kept.
__device__ __forceinline__ float round_to_f16(float x) { return __half2float(__float2half_rn(x)); }

// numpy float32 -> int16 on x86-64: converted through int32 (cvttss2si), which turns NaN
// and values outside int32 into INT32_MIN; the low 16 bits are kept.
__device__ __forceinline__ int f32_to_i16_x86(float x) {
    if (!(fabsf(x) < 2147483648.0f)) return 0;
    return static_cast<int>(static_cast<short>(__float2int_rz(x)));
}

// ---- global memory --------------------------------------------------------------------

// Output stores name the global state space (st.global.wb) rather than going through a
// generic pointer, so that the compiler knows they cannot alias the shared-memory tiles.
template <class T>
__device__ __forceinline__ void st_global(T* p, T v) {
    __stwb(p, v);
}
__device__ __forceinline__ void stg128(void* p, uint4 v) { st_global(reinterpret_cast<uint4*>(p), v); }
__device__ __forceinline__ void stg128f(float* p, float a, float b, float c, float d) {
    st_global(reinterpret_cast<float4*>(p), make_float4(a, b, c, d));
}

// 32 bytes to a 32-byte-aligned global address in one store (sm_100's 256-bit st.global):
// a warp of such stores writes whole 32-byte sectors.
__device__ __forceinline__ void stg256(void* p, const uint32_t (&w)[8]) {
    asm volatile("st.global.wb.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}

// Code / scale store of a conversion (defined with the shared-memory helpers below).
template <int MODE, class T>
__device__ __forceinline__ void st_out(T* p, T v);

// ---- per-block requantization parameters (requantize_symmetric) --------------------

// f32(f16(1e-4)): SCALE_EPSILON of ggml_quant.py:836 widened exactly (f16 bits 0x068E).
constexpr float kScaleEpsilon = 1.0001659393310547e-4f;

struct Requant {
    float sf;        // scale factor (integer-valued on the fast path)
    int rm;          // int16(rint(r * sf))
    float scale;     // S / sf, the output block scale
    float round_err; // |rm - r * sf|
    int clip_err;    // max |clip(q') - q'| over the block
    int sfi;         // integer scale factor, valid when fast
    bool fast;       // sf is an integer: q' = q * sfi + rm exactly
    bool clip;       // some code of the block needs clipping
};

// ggml_quant.py:826-882 for one block with scale S, min M (already the negated f16
// min), and the block's smallest / largest unsigned code.  Output range [lo_out, hi_out].
//
// Bound used below: for finite r, |r * sf| < 2200 (if r >= 0, sf <= 127/(qmax + r) or
// r <= 7.94; if r < 0, sf <= 128/(|r| - qmin) or |r| <= qmin + 8, with int8 codes), and
// for infinite or NaN r the product is NaN.  So numpy's int16(int32(rint(r*sf))) equals
// cvt.rni (round half even, NaN -> 0) here, and no int16 sum can wrap.
__device__ __forceinline__ Requant requant_block(float S, float M, int qmin, int qmax,
                                                 int lo_out, int hi_out, const float* recip = nullptr) {
    Requant p;
    const float s_eff = (S == 0.0f) ? ((fabsf(M) > kScaleEpsilon) ? M : kScaleEpsilon) : S;
    const float r = __fdiv_rn(M, s_eff);
    const float qminf = static_cast<float>(qmin);
    const float qmaxf = static_cast<float>(qmax);
    const float lo = __fadd_rn(qminf, r);
    const float hi = __fadd_rn(qmaxf, r);
    // sf = min(16, lo_out/lo if lo < 0, hi_out/hi if hi > 0).  A quotient of 16 or more
    // cannot lower sf, so only lo < lo_out/16 and hi > hi_out/16 matter; neither quotient
    // can be NaN, so fminf matches np.minimum.  When both matter, the smaller one is found
    // without dividing: lo_out/lo < hi_out/hi  <=>  lo_out*hi - hi_out*lo > 0 (lo < 0 < hi),
    // whose sign one fma gives exactly (lo_out*hi is exact, |lo|, |hi| < 400 here), and
    // since rounding is monotone the rounded quotient of the smaller one is the minimum.
    const bool need_lo = lo < static_cast<float>(lo_out) / 16.0f;
    const bool need_hi = hi > static_cast<float>(hi_out) / 16.0f;
    // the candidate quotient is computed unconditionally and selected, which keeps the
    // dependent chain free of divergent branches (the quotient is discarded when neither
    // bound applies; its operands are then finite or the result is unused)
    const float e = __fmaf_rn(-static_cast<float>(hi_out), lo, __fmul_rn(static_cast<float>(lo_out), hi));
    const bool use_lo = need_lo && (!need_hi || e > 0.0f);
    const float t = __fdiv_rn(static_cast<float>(use_lo ? lo_out : hi_out), use_lo ? lo : hi);
    float sf = (need_lo || need_hi) ? fminf(16.0f, t) : 16.0f;
    const bool big = sf > 0.98f;
    sf = big ? fmaxf(floorf(sf), 1.0f) : sf;
    const float rmv = __fmul_rn(r, sf);
    const int rm = __float2int_rn(rmv);
    p.sf = sf;
    p.rm = rm;
    p.round_err = fabsf(__fsub_rn(rintf(rmv), rmv));
    p.fast = big || (sf == 0.0f);
    p.sfi = p.fast ? static_cast<int>(sf) : 0;
    const int vmin = (p.fast ? qmin * p.sfi : __float2int_rn(__fmul_rn(qminf, sf))) + rm;
    const int vmax = (p.fast ? qmax * p.sfi : __float2int_rn(__fmul_rn(qmaxf, sf))) + rm;
    // scale = S / sf (the original S, ggml_quant.py:882).  For an integer sf in 1..16 and a
    // finite S: q0 = S*(1/sf) and one fma correction, which equals IEEE division for every
    // f16-derived S (checked exhaustively, tests/numerics/div_by_small_int.c).
    if (recip != nullptr && big && fabsf(S) < __int_as_float(0x7f800000)) {
        const float y = recip[p.sfi];
        const float q0 = __fmul_rn(S, y);
        const float res = __fmaf_rn(-sf, q0, S);
        p.scale = (res == 0.0f) ? q0 : __fmaf_rn(res, y, q0);
    } else {
        p.scale = __fdiv_rn(S, sf);
    }
    // q' is monotone in q (sf >= 0), so the block's extreme codes bound every code's clipping.
    p.clip = (vmax > hi_out) || (vmin < lo_out);
    p.clip_err = max(0, max(vmax - hi_out, lo_out - vmin));
    return p;
}

// The common case of requant_block on its own: finite S and M, an integer scale factor
// (sf > 0.98) and no code that clips.  Such a block is `good` and its fields equal
// requant_block's; for any other block `good` is false, round_err is 0 and the other
// fields are unspecified (the caller recomputes the block with requant_block).  sfi stays
// in 1..16 for every input, so recip[sfi] is always in bounds.
struct FastRequant {
    int sfi;          // integer scale factor
    int rm;           // int16(rint(r * sf))
    float scale;      // S / sf
    float round_err;  // |rm - r * sf| (good blocks), else 0
    float r;          // M / S' (exact when `finite`)
    float sf0;        // min(16, lo_out/lo, hi_out/hi) before the integer rounding: exact
                      // when > 0.98 and S, M are finite; a smaller one is exact_sf0(den)
    float den;        // the denominator of that quotient (lo or hi), 0 when neither bound applies
    bool good;
    bool finite;      // S and M are finite
};

// rcp.approx of -b: the negation goes into the approximation's operand.
__device__ __forceinline__ float rcp_approx_neg(float b) {
    float y;
    asm("{ .reg .f32 t; neg.f32 t, %1; rcp.approx.f32 %0, t; }" : "=f"(y) : "f"(b));
    return y;
}

// The requantization parameters of one block (lo_out = -128, hi_out = 127): S is the
// block scale, P = -M the block min before its negation.  This is requant_block's fast
// case with two divisions replaced: r = RN(M / S') from a reciprocal approximation (S' = M
// when S = 0 and |M| > eps gives r = 1 exactly), and the bound quotient
// sf0 = min(16, -128/lo, 127/hi) by Markstein's division with a refined reciprocal
// (P. Markstein, IBM J. Res. Dev. 34(1), 1990), whose floor and comparison with 0.98
// equal those of the IEEE quotient for every reachable denominator (exhaustive check:
// tests/numerics/scale_factor_quotient.c), so sfi, rm, good and scale are requant_block's.
// A block whose sf0 is at most 0.98 takes the rare path, which recomputes the quotient
// from `den` with an IEEE division (exact_sf0).
__device__ __forceinline__ FastRequant requant_fast(float S, float P, int qmin, int qmax, const float* recip) {
    FastRequant p;
    const bool zero = S == 0.0f;
    const float s = zero ? kScaleEpsilon : S;
    // r = RN(M / s) = RN(P / -s), both operands widened finite f16 values, without a
    // branch: with b = -s and y = rcp.approx(b) (within 1 ulp of 1/b), e = 1 - b*y is exact
    // in one fma (b has at most 11 significant bits); y + e*y approximates 1/b to about
    // 2^-45 relative, and P*(y + e*y) rounded once is RN(P/b), since a quotient of two
    // 11-bit significands lies at least 2^-36 (relative) from every f32 rounding midpoint.
    // Checked exhaustively, with any y within 2 ulp, by tests/numerics/f16_quotient.c.  A
    // zero quotient may come out with either sign (nothing below distinguishes them).
    const float ny = rcp_approx_neg(s);
    const float e = __fmaf_rn(s, ny, 1.0f);
    const float rq = __fmaf_rn(P, ny, __fmul_rn(P, __fmul_rn(e, ny)));
    const float r = (zero && fabsf(P) > kScaleEpsilon) ? 1.0f : rq;
    const float lo = __fadd_rn(static_cast<float>(qmin), r);
    const float hi = __fadd_rn(static_cast<float>(qmax), r);
    const bool need_lo = lo < -8.0f;
    const bool need_hi = hi > 127.0f / 16.0f;
    // which bound sets sf (see requant_block): -128*hi - 127*lo > 0 <=> -128/lo < 127/hi
    const float w = __fmaf_rn(-127.0f, lo, __fmul_rn(-128.0f, hi));
    const bool use_lo = need_lo && (!need_hi || w > 0.0f);
    const float num = use_lo ? -128.0f : 127.0f;
    const float den = use_lo ? lo : hi;
    // t = num / den with nz = -z, z ~ 1/den: e2 = 1 + den*nz, nz1 = -(z refined once),
    // nq0 = -RN(num * z1), rem = num - den*q0 (exact), t = -nq1 = q0 + rem*z1
    const float nz = rcp_approx_neg(den);
    const float ez = __fmaf_rn(den, nz, 1.0f);
    const float nz1 = __fmaf_rn(ez, nz, nz);
    const float nq0 = __fmul_rn(num, nz1);
    const float rem = __fmaf_rn(den, nq0, num);
    const float nt = __fmaf_rn(rem, nz1, nq0);
    const float sf0 = (need_lo || need_hi) ? fminf(16.0f, -nt) : 16.0f;
    const float sf = fmaxf(floorf(sf0), 1.0f);
    p.sfi = static_cast<int>(sf);
    const float rmv = __fmul_rn(r, sf);
    p.rm = __float2int_rn(rmv);
    // for big blocks |r * sf| < 2200 (see requant_block), so these sums do not wrap
    const int vmin = qmin * p.sfi + p.rm, vmax = qmax * p.sfi + p.rm;
    const float inf = __int_as_float(0x7f800000);
    p.finite = fabsf(S) < inf && fabsf(P) < inf;
    p.good = p.finite && sf0 > 0.98f && vmin >= -128 && vmax <= 127;
    p.r = r;
    p.sf0 = sf0;
    p.den = (need_lo || need_hi) ? den : 0.0f;
    p.round_err = p.good ? fabsf(__fsub_rn(rintf(rmv), rmv)) : 0.0f;
    // S / sf for an integer sf and finite S: q0 = S*(1/sf) and one fma correction, exact
    // for every f16-derived S (tests/numerics/div_by_small_int.c)
    const float y = recip[p.sfi];
    const float q0 = __fmul_rn(S, y);
    const float res = __fmaf_rn(-sf, q0, S);
    p.scale = (res == 0.0f) ? q0 : __fmaf_rn(res, y, q0);
    return p;
}

// The exact sf0 of a block whose bound quotient came out at most 0.98 in requant_fast
// (num / den by IEEE division), 16 when no bound applies (den == 0).
__device__ __forceinline__ float exact_sf0(float den) {
    return den == 0.0f ? 16.0f : fminf(16.0f, __fdiv_rn(den < 0.0f ? -128.0f : 127.0f, den));
}

// Finish one block whose S and M are finite but that is not `good` (non-integer scale
// factor or clipping), one value per lane of the warp, from requant_fast's exact r and
// exact sf0 (ggml_quant.py:859-882): sf, rm and the block scale as requant_block derives them,
// the per-value codes and the clipping error as the largest |clip(v) - v| of the block.
// Returns the block's rounding and clipping errors (the same in every lane).
template <int MODE = kOutCodes>
__device__ __forceinline__ gq_diag_t finish_block(int q, float S, float r, float sf0, int lo_out, int hi_out,
                                                  uint8_t* code, float* scale, int lane) {
    const bool big = sf0 > 0.98f;
    const float sf = big ? fmaxf(floorf(sf0), 1.0f) : sf0;
    const float rmv = __fmul_rn(r, sf);
    const int rm = __float2int_rn(rmv);   // |r * sf| < 2200 for finite r (see requant_block)
    const int c = f32_to_i16_x86(rintf(__fmul_rn(static_cast<float>(q), sf)));
    const int u = static_cast<int>(static_cast<short>(c + rm));
    const int v = min(max(u, lo_out), hi_out);
    st_out<MODE>(code, static_cast<uint8_t>(v));
    if (lane == 0) st_out<MODE>(scale, __fdiv_rn(S, sf));
    gq_diag_t e;
    e.round_err_bits = __float_as_uint(fabsf(__fsub_rn(rintf(rmv), rmv)));
    e.clip_err = static_cast<int>(__reduce_max_sync(0xffffffffu, static_cast<unsigned>(abs(v - u))));
    return e;
}

// General per-value requant (non-integer scale factor).
__device__ __forceinline__ int requant_value(int q, float sf, int rm, int lo_out, int hi_out) {
    const int c = f32_to_i16_x86(rintf(__fmul_rn(static_cast<float>(q), sf)));
    const int v = static_cast<int>(static_cast<short>(c + rm));
    return min(max(v, lo_out), hi_out);
}

// Fast path on a word holding 4 unsigned codes (one per byte, each <= 31):
// q' = q * sfi + rm computed in 16-bit lanes with a 0x4000 bias (no cross-lane carry),
// optionally clamped, and the low bytes packed back in order.
constexpr uint32_t kLaneBias = 0x4000u;

__device__ __forceinline__ uint32_t requant_word_fast(uint32_t x, uint32_t sfi, uint32_t k2,
                                                      bool clip, uint32_t lo2, uint32_t hi2) {
    uint32_t e = x & 0x00FF00FFu;
    uint32_t o = (x >> 8) & 0x00FF00FFu;
    e = e * sfi + k2;
    o = o * sfi + k2;
    if (clip) {
        e = __vminu2(__vmaxu2(e, lo2), hi2);
        o = __vminu2(__vmaxu2(o, lo2), hi2);
    }
    return __byte_perm(e, o, 0x6240);
}

__device__ __forceinline__ uint32_t requant_word_slow(uint32_t x, float sf, int rm, int lo_out,
                                                      int hi_out) {
    uint32_t out = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const int q = (x >> (8 * b)) & 0xFF;
        out |= (static_cast<uint32_t>(requant_value(q, sf, rm, lo_out, hi_out)) & 0xFFu) << (8 * b);
    }
    return out;
}

// 16-bit-lane SIMD min / max (native on sm_90+) and multiply-high-add
__device__ __forceinline__ uint32_t vmin16(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("min.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t vmax16(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t vmin16(uint32_t a, uint32_t b, uint32_t c) { return vmin16(vmin16(a, b), c); }
__device__ __forceinline__ uint32_t vmax16(uint32_t a, uint32_t b, uint32_t c) { return vmax16(vmax16(a, b), c); }
// high 32 bits of a*b, plus c
__device__ __forceinline__ uint32_t mad_hi(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("mad.hi.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// min / max of the 4 bytes of a word
__device__ __forceinline__ int byte_min4(uint32_t w) {
    w = __vminu4(w, w >> 16);
    w = __vminu4(w, w >> 8);
    return w & 0xFF;
}
__device__ __forceinline__ int byte_max4(uint32_t w) {
    w = __vmaxu4(w, w >> 16);
    w = __vmaxu4(w, w >> 8);
    return w & 0xFF;
}

// ---- shared memory access ------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
    return *reinterpret_cast<const uint32_t*>(p);
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) {
    return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) {
    return *reinterpret_cast<const uint16_t*>(p);
}

// 16 bytes from a 2-byte-aligned shared address: five aligned words and funnel shifts.
// SMEM_LD selects how the words are read: explicit shared loads at the word-aligned shared
// address (the fused layout writer's decode, whose staging reads measured faster so:
// Q6_K 1.644 -> 1.580 ms per Llama-3-8B set), or plain loads through the word pointer (the
// conversion kernels, where the explicit form measured slower: Q8_0 0.368 -> 0.420 ms on
// the Qwen2.5-7B set).
template <bool SMEM_LD = false>
__device__ __forceinline__ uint4 lds128_align2(const uint8_t* p) {
    uint32_t w0, w1, w2, w3, w4, sh;
    if constexpr (SMEM_LD) {
        const uint32_t a = smem_u32addr(p);
        const uint32_t b = a & ~3u;
        sh = (a & 3u) * 8u;
        asm volatile("ld.shared.u32 %0, [%5];\n\tld.shared.u32 %1, [%5+4];\n\tld.shared.u32 %2, [%5+8];\n\t"
                     "ld.shared.u32 %3, [%5+12];\n\tld.shared.u32 %4, [%5+16];"
                     : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3), "=r"(w4)
                     : "r"(b)
                     : "memory");
    } else {
        const uintptr_t a = reinterpret_cast<uintptr_t>(p);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
        sh = static_cast<uint32_t>(a & 3u) * 8u;
        w0 = w[0];
        w1 = w[1];
        w2 = w[2];
        w3 = w[3];
        w4 = w[4];
    }
    uint4 r;
    r.x = __funnelshift_r(w0, w1, sh);
    r.y = __funnelshift_r(w1, w2, sh);
    r.z = __funnelshift_r(w2, w3, sh);
    r.w = __funnelshift_r(w3, w4, sh);
    return r;
}

// cp.async of one 16-byte chunk, reading only `src_bytes` (1..16) bytes; the rest of the
// shared chunk is zero-filled.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                 :: "r"(smem_u32addr(smem_dst)), "l"(gmem_src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" :: "n"(N) : "memory"); }

// ---- bulk copies (the TMA engine) into shared memory, completed on an mbarrier --------
//
// One lane issues a whole tile as a single 1-D bulk copy from this GPU's global memory
// (no cluster multicast); the warp waits on the stage's mbarrier phase.  The copy engine
// keeps far more bytes in flight per SM than per-lane 16-byte copies can.

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32addr(bar)), "r"(count) : "memory");
}
// makes barrier initialisation visible to the copy engine (before the CTA-wide barrier)
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32addr(bar)), "r"(bytes)
                 : "memory");
}

// `bytes` (a multiple of 16) from 16-byte-aligned global `src` to 16-byte-aligned shared `dst`
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32addr(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every wait on a copy ends: after kWaitLimitNs of global time without the phase completing,
// the wait gives up and returns false (the kernel then records kErrWaitTimeout and stops).
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr unsigned kErrWaitTimeout = GQ_KERNEL_WAIT_TIMEOUT;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// ---- code / scale stores of a conversion ---------------------------------------------

// Shared row tiles of 256-byte rows (the fused Modalix writer, 8 KiB aligned) keep their
// 16-byte chunks swizzled: chunk c of row r sits at chunk c ^ g(r) ^ 3 (c >> 3), with
// g(r) = (r & 3) | 4 ((r >> 4) & 1).  A quarter warp's 16-byte stores then fill all eight
// bank groups in every decode pattern (Q4_K / Q5_K: lanes 64 bytes apart over a row pair;
// Q6_K and the 16-value K formats: 8 consecutive chunks of a row; Q8_0 / Q4_0: 32-byte
// units), and so do the 8 rows {4m + e, 16 + 4m + e} (e < 4) that one ldmatrix phase of the
// transpose reads at one chunk.  A bijection on every 256-byte row.
__device__ __forceinline__ uint32_t row_swizzle(uint32_t a) {
    const uint32_t g = ((a >> 8) & 3u) | (((a >> 12) & 1u) << 2);
    return a ^ ((g ^ (3u * ((a >> 7) & 1u))) << 4);
}

// Two 16x16 byte matrices transposed out of shared memory: lanes 0-15 give the row addresses
// of matrix 0, lanes 16-31 those of matrix 1.  Lane t receives, of matrix m, column t / 4
// (register 2m) and column t / 4 + 8 (register 2m + 1), rows 4 (t % 4)..4 (t % 4) + 3 in
// its bytes 0..3.
__device__ __forceinline__ void ldsm_x2_trans_b8(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a)
                 : "memory");
}

__device__ __forceinline__ void sts(uint32_t a, uint8_t v) {
    asm volatile("st.shared.u8 [%0], %1;" ::"r"(a), "r"(static_cast<uint32_t>(v)) : "memory");
}
__device__ __forceinline__ void sts(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void sts(uint32_t a, float2 v) {
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(v.x), "f"(v.y) : "memory");
}
__device__ __forceinline__ void sts(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void sts(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a)
                 : "memory");
    return v;
}

// Code / scale stores: to global memory, or (kOutSmem) to a shared tile (codes swizzled
// as above, scales as they are).
template <int MODE, class T>
__device__ __forceinline__ void st_out(T* p, T v) {
    if constexpr ((MODE & kOutSmem) != 0) {
        const uint32_t a = smem_u32addr(p);
        if constexpr (sizeof(T) == 1 || sizeof(T) == 16) {
            sts(row_swizzle(a), v);
        } else {
            sts(a, v);
        }
    } else {
        st_global(p, v);
    }
}
template <int MODE>
__device__ __forceinline__ void st_out128(void* p, uint4 v) { st_out<MODE>(reinterpret_cast<uint4*>(p), v); }

// ---- misc ------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// Output unit index after the llama q/k head permutation (gguf_conversion.py:314-332):
// row h*D + 2a + t moves to h*D + t*D/2 + a.
__device__ __forceinline__ uint32_t fast_div(uint32_t n, uint32_t mul, uint32_t shift) {
    const uint32_t t1 = __umulhi(mul, n);
    return (t1 + ((n - t1) >> (shift & 0xFF))) >> (shift >> 8);
}

__device__ __forceinline__ int64_t permute_unit(const GqDesc& d, int64_t unit) {
    if (d.perm_heads == 0) return unit;
    if (d.upr_mul != 0) {
        const uint32_t upr = static_cast<uint32_t>(d.units_per_row), rph = static_cast<uint32_t>(d.rows_per_head);
        const uint32_t u = static_cast<uint32_t>(unit);
        const uint32_t row = fast_div(u, d.upr_mul, d.upr_shift);
        const uint32_t col = u - row * upr;
        const uint32_t head = fast_div(row, d.rph_mul, d.rph_shift);
        const uint32_t i = row - head * rph;
        const uint32_t out_row = head * rph + (i & 1) * (rph >> 1) + (i >> 1);
        return static_cast<int64_t>(out_row * upr + col);
    }
    const int64_t row = unit / d.units_per_row;
    const int64_t col = unit - row * d.units_per_row;
    const int64_t head = row / d.rows_per_head;
    const int64_t i = row - head * d.rows_per_head;
    const int64_t out_row = head * d.rows_per_head + (i & 1) * (d.rows_per_head >> 1) + (i >> 1);
    return out_row * d.units_per_row + col;
}

// Diagnostics accumulated per warp while its tiles stay in one tensor.
struct DiagAcc {
    gq_diag_t* target = nullptr;
    uint32_t round_bits = 0;
    int clip = 0;

    __device__ __forceinline__ void add(float round_err, int clip_err) {
        round_bits = max(round_bits, __float_as_uint(fabsf(round_err)));
        clip = max(clip, clip_err);
    }
    // Warp-collective: reduce over lanes and publish with atomics (skipped when it cannot
    // raise the stored maxima).
    __device__ __forceinline__ void flush(int lane) {
        const uint32_t rb = __reduce_max_sync(0xffffffffu, round_bits);
        const int ce = __reduce_max_sync(0xffffffffu, clip);
        if (lane == 0 && target != nullptr) {
            volatile gq_diag_t* t = target;
            if (rb > t->round_err_bits) atomicMax(&target->round_err_bits, rb);
            if (ce > t->clip_err) atomicMax(&target->clip_err, ce);
        }
        round_bits = 0;
        clip = 0;
    }
    __device__ __forceinline__ void retarget(gq_diag_t* t, int lane) {
        if (t != target) {
            flush(lane);
            target = t;
        }
    }
};

}  // namespace gq

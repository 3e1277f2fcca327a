// slx_device.cuh -- device-side integer helpers shared by the slx kernels.
//
// The arithmetic follows C# semantics of SparseLattice's integer path:
//   * long / Int128 arithmetic wraps (unchecked), so sums are carried in unsigned __int128;
//   * `/` truncates toward zero, `>>` on signed values floors;
//   * (long)double truncates, NaN / out of range gives long.MinValue (x64 .NET 8 conversion);
//   * (Half)float rounds to nearest even (__float2half_rn).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

typedef __int128 i128;
typedef unsigned __int128 u128;

#define SLX_DEV __device__ __forceinline__

SLX_DEV int64_t lo64(i128 v) { return (int64_t)(uint64_t)(u128)v; }
SLX_DEV i128 sar128(i128 v, int n) { return v >> (n & 127); }
SLX_DEV int64_t wadd(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }
SLX_DEV int64_t wsub(int64_t a, int64_t b) { return (int64_t)((uint64_t)a - (uint64_t)b); }
SLX_DEV int64_t wmul(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }
SLX_DEV int64_t cs_div64(int64_t a, int64_t b) { return b == -1 ? wsub(0, a) : a / b; }

SLX_DEV int64_t cs_d2l(double v) {
    if (v >= -9223372036854775808.0 && v < 9223372036854775808.0) return __double2ll_rz(v);
    return INT64_MIN;
}

SLX_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
SLX_DEV uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
SLX_DEV uint16_t ld_u16(const uint8_t* p) { return *(const uint16_t*)p; }

// GGUF dtype ids (GgufTypes.cs:21-38).
enum : int { DT_F32 = 0, DT_F16 = 1, DT_Q4_0 = 2, DT_Q8_0 = 8, DT_BF16 = 30 };

// One element of a flat GGUF tensor, decoded the way GgufDequantizer decodes it
// (Q8_0: GgufDequantizer.cs:31-49, Q4_0: :51-76 with element 2j in the low nibble, F16: :19-29,
// BF16: :78-89, F32: :7-17). `nblocks` bounds the 32-element blocks (ComputeByteCount truncates).
SLX_DEV float dequant_elem(int dtype, const uint8_t* base, int64_t e, int64_t nblocks) {
    switch (dtype) {
        case DT_Q8_0: {
            int64_t b = e >> 5;
            if (b >= nblocks) return 0.0f;
            const uint8_t* blk = base + b * 34;
            return __fmul_rn(h2f(ld_u16(blk)), (float)(int8_t)blk[2 + (e & 31)]);
        }
        case DT_Q4_0: {
            int64_t b = e >> 5;
            if (b >= nblocks) return 0.0f;
            const uint8_t* blk = base + b * 18;
            int j = (int)(e & 31);
            uint8_t raw = blk[2 + (j >> 1)];
            int q = ((j & 1) ? (raw >> 4) : (raw & 0x0F)) - 8;
            return __fmul_rn(h2f(ld_u16(blk)), (float)q);
        }
        case DT_F16: return h2f(((const uint16_t*)base)[e]);
        case DT_BF16: return __uint_as_float((uint32_t)((const uint16_t*)base)[e] << 16);
        default: return ((const float*)base)[e];
    }
}

// Composite Q30 weight as the reference forms it from a dequantized float:
//   mode 0 (IntegerTransformerSource.Q, IntegerMatMul.QuantizeFromFloat :297-304): (long)(f * 2^s)
//   mode 1 (IntegerCausalSource.ReadAsHalf + DotInt128Mixed(Half) :255-275): (long)((float)(Half)f * 2^s)
SLX_DEV int64_t composite(float f, int mode, double scale) {
    if (mode == 1) f = h2f(f2h(f));
    return cs_d2l((double)f * scale);
}

// Exact floor square root of a non-negative 128-bit value (ISqrt64 / ISqrt128,
// IntegerLayerNorm.cs:99-149). Returned as the low 64 bits, like the reference's (long)x.
// Out of line: one call per row, and its Newton steps divide in 128 bits.
static __device__ __noinline__ int64_t isqrt_u128(u128 v) {
    if (v == 0) return 0;
    u128 x = (u128)sqrt((double)v);
    if (x == 0) x = 1;
    if ((v >> 104) != 0) {  // double seed is short of bits: Newton steps
        for (int it = 0; it < 4; it++) {
            u128 nx = (x + v / x) >> 1;
            if (nx == x) break;
            x = nx;
        }
    }
    while (x * x > v) x--;
    while ((x + 1) * (x + 1) <= v) x++;
    return (int64_t)(uint64_t)x;
}

// FixedExp (IntegerTranscendentals.cs:13-47), fracBits = 30. The Taylor term update
// (long)((Int128)term * r / (n << 30)) equals ((term * r) >> 30) / n whenever term, r >= 0 and
// term * r < 2^64 (floor of floor); that fast path covers every input after range reduction,
// the general Int128 form stays for anything else. The loop is unrolled, so each division by n
// is a multiply by a constant; it stops, as the reference does, once a term is 0 past n = 4.
SLX_DEV int64_t fixed_exp30(int64_t x) {
    const int64_t ln2 = 744261117;  // (long)(0.6931471805599453 * 2^30)
    int64_t k = x >= 0 ? x / ln2 : wsub(0, cs_div64(wsub(wadd(wsub(0, x), ln2), 1), ln2));
    int64_t r = wsub(x, wmul(k, ln2));
    if (k > 62) return INT64_MAX;
    if (k < -40) return 0;
    const int64_t one = 1LL << 30;
    int64_t sum = one;
    if (r >= 0 && r < ln2) {
        // After range reduction 0 <= r < ln2 < 2^30 and every term stays <= 2^30, so term * r fits
        // 60 bits and ((term * r) >> 30) / n is the exact quotient in 32-bit arithmetic.
        uint32_t term = (uint32_t)one;
        const uint32_t rr = (uint32_t)r;
        uint32_t s32 = (uint32_t)one;  // e^r * 2^30 < 2^31
#pragma unroll
        for (int n = 1; n <= 14; n++) {
            term = (uint32_t)(((uint64_t)term * rr) >> 30) / (uint32_t)n;
            s32 += term;
            if (term == 0 && n > 4) break;
        }
        sum = (int64_t)s32;
    } else {
        int64_t term = one;
#pragma unroll
        for (int n = 1; n <= 14; n++) {
            if (term >= 0 && r >= 0 && __umul64hi((uint64_t)term, (uint64_t)r) == 0) {
                uint64_t p = (uint64_t)term * (uint64_t)r;
                term = (int64_t)((p >> 30) / (uint64_t)n);
            } else {
                term = lo64(((i128)term * r) / ((i128)n << 30));
            }
            sum = wadd(sum, term);
            if (term == 0 && n > 4) break;
        }
    }
    if (k >= 0) {
        if (k >= 63 || sum > (INT64_MAX >> k)) return INT64_MAX;
        return (int64_t)((uint64_t)sum << k);
    }
    int sh = (int)(-k);
    if (sh >= 63) return 0;
    return sum >> sh;
}

// (long)(x / d), truncating toward zero, for d >= 1 and rd ~ 1 / d: a double estimate of |x| / d
// (off by at most one below 2^52) corrected by the remainder; wider values take the 64-bit division.
SLX_DEV int64_t div_small(int64_t x, int64_t d, double rd) {
    const uint64_t ax = x < 0 ? (uint64_t)0 - (uint64_t)x : (uint64_t)x;
    if (ax < (1ULL << 52)) {
        int64_t q = (int64_t)((double)ax * rd);
        int64_t r = (int64_t)ax - q * d;
        while (r < 0) { q--; r += d; }
        while (r >= d) { q++; r -= d; }
        return x < 0 ? -q : q;
    }
    return cs_div64(x, d);
}

// ---- exact fixed-point steps on the fp64 pipe
// The doubles in [2^52, 2^53) are exactly the integers there. For doubles a, b holding exact values
// and |floor(a b)| < 2^51, fma_rd(a, b, 1.5 * 2^52) rounds the exact a b + 1.5 * 2^52 toward minus
// infinity, which is 1.5 * 2^52 + floor(a b): one instruction for a floored fixed-point product.
// The integer is the bit pattern minus that of 1.5 * 2^52 (its low word when it fits in 32 bits),
// and an integer below 2^51 in magnitude becomes an exact double the same way backwards.
constexpr double RD_BASE = 6755399441055744.0;  // 1.5 * 2^52
constexpr int64_t RD_BASE_BITS = 0x4338000000000000LL;
SLX_DEV double rd_floor(double a, double b) { return __fma_rd(a, b, RD_BASE); }
SLX_DEV int32_t rd_i32(double y) { return __double2loint(y); }
SLX_DEV int64_t rd_i64(double y) { return __double_as_longlong(y) - RD_BASE_BITS; }
SLX_DEV double d_u32(uint32_t x) { return __hiloint2double(0x43380000, (int)x) - RD_BASE; }
SLX_DEV double d_i64(int64_t x) { return __longlong_as_double(RD_BASE_BITS + x) - RD_BASE; }  // |x| < 2^51
SLX_DEV double pow2d(int k) { return __hiloint2double((1023 + k) << 20, 0); }                  // |k| < 1023

// trunc(a w / d) for d >= 1 (the reference's Int128 division, truncating toward zero) with wd = w as
// a double and rd = 1 / (double)d rounded to nearest. When |a|, |w| < 2^51, d < 2^60 and the quotient
// is below 2^49 in magnitude, P rd, with P = |a w| rounded to a double, is within Q 2^-51 of the exact
// quotient Q = |a w| / d (three roundings of relative size 2^-53 at most: the product, d as a double
// and its reciprocal). One rounded-down FMA gives q = floor(P rd); a second FMA gives P rd - q. Where
// that fraction lies at least (q + 1) 2^-50 away from both integers, no integer lies between P rd and
// Q, so q = floor(Q); only nearer to an integer does the remainder |a w| - q d, exact in wrapping
// 64-bit arithmetic because |r| < 2 d, decide. Anything else takes the Int128 division.
// The Int128 division (rare: outside the fast path's ranges), kept out of line so the callers' code
// stays small.
static __device__ __noinline__ int64_t muldiv_trunc_slow(int64_t a, int64_t w, int64_t d) { return lo64(((i128)a * w) / (i128)d); }

SLX_DEV int64_t muldiv_trunc(int64_t a, int64_t w, double wd, int64_t d, double rd) {
    constexpr int64_t lim = 1LL << 51;
    if (a > -lim && a < lim && w > -lim && w < lim && d < (1LL << 60)) {
        const double P = fabs(d_i64(a) * wd);
        const double y = rd_floor(P, rd);  // 1.5 * 2^52 + floor(P rd)
        int64_t q = rd_i64(y);
        if (q < (1LL << 49)) {
            const double fl = y - RD_BASE;
            const double frac = __fma_rn(P, rd, -fl);  // P rd - q
            const double tol = (fl + 1.0) * 0x1p-50;
            if (frac < tol || frac > 1.0 - tol) {
                const uint64_t ua = a < 0 ? (uint64_t)0 - (uint64_t)a : (uint64_t)a;
                const uint64_t uw = w < 0 ? (uint64_t)0 - (uint64_t)w : (uint64_t)w;
                int64_t r = (int64_t)(ua * uw - (uint64_t)q * (uint64_t)d);
                while (r < 0) { q--; r += d; }
                while (r >= d) { q++; r -= d; }
            }
            return (a < 0) != (w < 0) ? -q : q;
        }
    }
    return muldiv_trunc_slow(a, w, d);
}

// FixedExp's Taylor branch (IntegerTranscendentals.cs:13-47), fracBits = 30: e^r * 2^30 for r in
// [0, ln2) by the truncating recurrence term_n = (term * r >> 30) / n. Every term past the tenth is
// zero on this range, and each floor(x / n) equals umulhi(x, ceil(2^32 / n)) for the x that step can
// see, so the sum agrees with the recurrence for every r in [0, ln2). The work is split between the
// fp64 and integer pipes: floor(t r / 2^30) is one fp64 FMA rounded down (so are the whole terms
// n = 2, 4, 8, whose divisions are powers of two folded into r), the other divisions by n are those
// multiply-high constants, and the terms n = 3 and 7 are umulhi(umulhi(t, 4r), c) on the integer
// pipe. rd = r.
SLX_DEV uint32_t exp_taylor30_fp(uint32_t r, double rd) {
    const uint32_t r4 = r << 2;
    const double r30 = rd * 0x1p-30;
    uint32_t sum = (1u << 30) + r, t;                                                          // n = 1
    double y = rd_floor(rd, rd * 0x1p-31);
    t = (uint32_t)rd_i32(y); sum += t;                                                         // n = 2
    t = __umulhi(__umulhi(t, r4), 1431655766u); sum += t;                                      // n = 3
    y = rd_floor(d_u32(t), rd * 0x1p-32);
    t = (uint32_t)rd_i32(y); sum += t;                                                         // n = 4
    y = rd_floor(y - RD_BASE, r30);
    t = __umulhi((uint32_t)rd_i32(y), 858993460u); sum += t;                                   // n = 5
    y = rd_floor(d_u32(t), r30);
    t = __umulhi((uint32_t)rd_i32(y), 715827883u); sum += t;                                   // n = 6
    t = __umulhi(__umulhi(t, r4), 613566757u); sum += t;                                       // n = 7
    y = rd_floor(d_u32(t), rd * 0x1p-33);
    t = (uint32_t)rd_i32(y); sum += t;                                                         // n = 8
    y = rd_floor(y - RD_BASE, r30);
    t = __umulhi((uint32_t)rd_i32(y), 477218589u); sum += t;                                   // n = 9
    y = rd_floor(d_u32(t), r30);
    t = __umulhi((uint32_t)rd_i32(y), 429496730u); sum += t;                                   // n = 10
    return sum;
}

// floor(y / ln2) and y - floor(y / ln2) ln2 in [0, ln2) for |y| < 2^50, ln2 = 744261117 (2^30 ln 2
// truncated): the fp64 estimate is within one, the exact remainder (an integer below 2^51) picks it.
SLX_DEV int ln2_reduce(double yd, double& rem) {
    constexpr double LN2D = 744261117.0;
    const double ky = rd_floor(yd, 1.0 / LN2D);
    int k = rd_i32(ky);
    double r = __fma_rn(-(ky - RD_BASE), LN2D, yd);
    if (r < 0.0) { k--; r += LN2D; }
    else if (r >= LN2D) { k++; r -= LN2D; }
    rem = r;
    return k;
}

// FixedSigmoid / FixedSiLU (IntegerTranscendentals.cs:49-69), fracBits = 30, and the gated product
// (long)((Int128)FixedSiLU(g) * u >> 30) of IntegerFFN (Math/IntegerFFN.cs:70-100).
// FixedExp(-g) for |g| <= 20 * 2^30: the reference's k = floor(y / ln2) (truncation for y >= 0,
// -ceil(-y / ln2) below), r = y - k ln2, so its 32-bit Taylor branch always runs; k <= 28, so
// e = sum << k never overflows, and k >= -29. den = 2^30 + e < 2^60 is an exact double (at most 32
// significant bits). 2^60 / den: the fp64 estimate floor(2^60 rcp(den)), corrected by the exact
// remainder where it lies near an integer. FixedSiLU = floor(g sig / 2^30) is one rounded-down FMA (|result| <= 20 * 2^30). The
// gated product takes the same FMA when |s|, |u| < 2^51 and |s u| < 2^80, else Int128.
SLX_DEV int64_t silu_gate30(int64_t g, int64_t u) {
    constexpr int64_t one = 1LL << 30, thr = 20LL << 30;
    int64_t s;
    if (g > thr) s = g;
    else if (g < -thr) s = 0;
    else {
        double rem;
        const int k = ln2_reduce(d_i64(-g), rem);
        const uint32_t sum = exp_taylor30_fp((uint32_t)rd_i32(rem + RD_BASE), rem);
        const int64_t den = one + (k >= 0 ? (int64_t)sum << k : (int64_t)(sum >> -k));
        const double den_d = k >= 0 ? __fma_rn(d_u32(sum), pow2d(k), 1073741824.0) : d_i64(den);
        // 2^60 * rcp(den) is within 2^-23 of 2^60 / den (at most 2^30): its floor is exact unless it
        // lies within 2^-22 of an integer, where the exact remainder decides
        const double rcp = __drcp_rn(den_d);
        const double y = rd_floor(1152921504606846976.0, rcp);
        int64_t q = rd_i32(y);
        const double frac = __fma_rn(1152921504606846976.0, rcp, -(y - RD_BASE));
        if (frac < 0x1p-22 || frac > 1.0 - 0x1p-22) {
            int64_t r = (int64_t)((1ULL << 60) - (uint64_t)q * (uint64_t)den);
            while (r < 0) { q--; r += den; }
            while (r >= den) { q++; r -= den; }
        }
        s = rd_i64(rd_floor(d_i64(g), d_u32((uint32_t)q) * 0x1p-30));
    }
    const int64_t lim = 1LL << 51;
    if (s > -lim && s < lim && u > -lim && u < lim) {
        const double sd = d_i64(s), ud = d_i64(u);
        if (fabs(sd * ud) < 0x1p80) return rd_i64(rd_floor(sd, ud * 0x1p-30));
    }
    return lo64(sar128((i128)s * u, 30));
}

// Five balanced base-256 digits (each in [-128, 127]) of four values x0..x3: w[i] holds digit i of
// x_j in byte j. For x in [-0x8080808080, 0x7F7F7F7F7F] the digits are the low five bytes of
// (x + 0x8080808080) ^ 0x8080808080 (adding 128 at every byte position leaves bytes d_i + 128 with no
// carries); bad is set when a value lies outside that range (it would need a sixth digit).
SLX_DEV void digit_words4(int64_t x0, int64_t x1, int64_t x2, int64_t x3, uint32_t (&w)[5], bool& bad) {
    constexpr uint64_t OFF = 0x8080808080ull;
    const uint64_t y0 = (uint64_t)x0 + OFF, y1 = (uint64_t)x1 + OFF, y2 = (uint64_t)x2 + OFF, y3 = (uint64_t)x3 + OFF;
    bad |= ((y0 | y1 | y2 | y3) >> 40) != 0;
    const uint64_t z0 = y0 ^ OFF, z1 = y1 ^ OFF, z2 = y2 ^ OFF, z3 = y3 ^ OFF;
    const uint32_t l0 = (uint32_t)z0, l1 = (uint32_t)z1, l2 = (uint32_t)z2, l3 = (uint32_t)z3;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t sel = (uint32_t)i | ((uint32_t)(4 + i) << 4);
        w[i] = __byte_perm(__byte_perm(l0, l1, sel), __byte_perm(l2, l3, sel), 0x5410);
    }
    w[4] = __byte_perm(__byte_perm((uint32_t)(z0 >> 32), (uint32_t)(z1 >> 32), 0x40),
                       __byte_perm((uint32_t)(z2 >> 32), (uint32_t)(z3 >> 32), 0x40), 0x5410);
}

// 128-bit warp reductions (wrap-around sums).
SLX_DEV u128 warp_sum_u128(u128 v) {
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t lo = __shfl_xor_sync(0xffffffffu, (unsigned long long)(uint64_t)v, o);
        uint64_t hi = __shfl_xor_sync(0xffffffffu, (unsigned long long)(uint64_t)(v >> 64), o);
        v += ((u128)hi << 64) | lo;
    }
    return v;
}
SLX_DEV int64_t warp_max_i64(int64_t v) {
    for (int o = 16; o > 0; o >>= 1) {
        int64_t w = (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v, o);
        v = w > v ? w : v;
    }
    return v;
}

// hb_arith.cuh -- 64-bit RNS modular arithmetic for sm_100a.
//
// Every residue is a uint64 in [0, q) with q < 2^61.  Multiplication by a
// precomputed constant uses Shoup's method (Shoup, NTL; Harvey 2014);
// products of two variable residues are formed exactly as 128-bit values
// and reduced with the fold x = hi*2^64 + lo -> hi*(2^64 mod q) + lo, each
// half reduced by a Shoup multiplication.  Sums of up to 32 products of
// residues below 2^61 stay below 2^127, so multiply-accumulate loops add
// 128-bit products lazily and reduce once.
#pragma once
#include <cstdint>

namespace hb {

typedef unsigned long long u64;

#define HB_MAX_PRIMES 64

// Per-prime constants, one entry per prime index (main primes first, then
// the special primes).  Kept in __constant__ memory: every thread of a
// warp reads the same entry, which the constant cache broadcasts.
struct PrimeConst {
    u64 q;
    u64 r64;      // 2^64 mod q
    u64 r64p;     // Shoup companion of r64
    u64 onep;     // floor(2^64 / q) (Shoup companion of 1)
    u64 ninv;     // N^-1 mod q
    u64 ninvp;
    u64 c60, c60p;  // 2^60 mod q
    u64 c58, c58p;  // 2^58 mod q (Karatsuba split-29 recombination)
    double qinv;    // fl(1/q), quotient estimates on the FP64 pipe
    double c58d;    // 2^58 mod q as a double (exact for q < 2^53)
    u64 c90;        // 2^90 mod q
    double c60d, c90d;  // 2^60 and 2^90 mod q as doubles (rounded above 2^53)
};

#define HB_SPLIT_MASK 0x3FFFFFFFull
// split-30 packed form (v >> 30) << 32 | (v mod 2^30), for v < 2^62
__device__ __forceinline__ u64 split_pack(u64 v) { return ((v >> 30) << 32) | (v & HB_SPLIT_MASK); }

__device__ __forceinline__ u64 add_mod(u64 a, u64 b, u64 q) {
    u64 s = a + b;
    return s >= q ? s - q : s;
}
__device__ __forceinline__ u64 sub_mod(u64 a, u64 b, u64 q) {
    return a >= b ? a - b : a + (q - b);
}
__device__ __forceinline__ u64 neg_mod(u64 a, u64 q) { return a ? q - a : 0; }

// a * w mod q for any a < 2^64, w < q, wp = floor(w 2^64 / q).
__device__ __forceinline__ u64 mul_shoup(u64 a, u64 w, u64 wp, u64 q) {
    u64 hi = __umul64hi(a, wp);
    u64 r = a * w - hi * q;
    return r >= q ? r - q : r;
}
// same, result left in [0, 2q)
__device__ __forceinline__ u64 mul_shoup_lazy(u64 a, u64 w, u64 wp, u64 q) {
    u64 hi = __umul64hi(a, wp);
    return a * w - hi * q;
}

struct u128 {
    u64 lo, hi;
};

__device__ __forceinline__ void mac128(u128 &acc, u64 a, u64 b) {
    u64 lo = a * b;
    u64 hi = __umul64hi(a, b);
    acc.lo += lo;
    acc.hi += hi + (acc.lo < lo ? 1ull : 0ull);
}

// (hi*2^64 + lo) mod q
__device__ __forceinline__ u64 reduce128(u64 hi, u64 lo, const PrimeConst &pc) {
    u64 h = mul_shoup(hi, pc.r64, pc.r64p, pc.q);
    u64 l = mul_shoup(lo, 1ull, pc.onep, pc.q);
    return add_mod(h, l, pc.q);
}
__device__ __forceinline__ u64 reduce128(const u128 &x, const PrimeConst &pc) {
    return reduce128(x.hi, x.lo, pc);
}
__device__ __forceinline__ u64 mul_mod(u64 a, u64 b, const PrimeConst &pc) {
    return reduce128(__umul64hi(a, b), a * b, pc);
}
// ---- exact modular arithmetic on the FP64 pipe (moduli below 2^40) -----------
// Integers below 2^53 are exact doubles.  u64_to_d converts v < 2^52 by
// placing it in the mantissa of 2^52.  mulmod_d(y, {w, fl(w/q)}, q) returns
// y w - Q q with Q = round(y fl(w/q)) (magic-number rounding), computed
// exactly: ph + pl = Q q (TwoProduct: ph = fl(Q q), pl = fma(Q, q, -ph)) and
// fma(y, w, -ph) is the exact integer y w - ph, below 2^41 in magnitude; the
// result is centred, |t| <= 0.502 q, for |y| < 2^44 and w < q < 2^40.
// center_d(v) = v - round(v / q) q, |result| <= 0.5 q (+ rounding slack).
__device__ __forceinline__ double u64_to_d(u64 v) {
    return __dsub_rn(__longlong_as_double((long long)(v | 0x4330000000000000ull)), 4503599627370496.0);
}
__device__ __forceinline__ double mulmod_d(double y, const double2 tw, double q) {
    const double magic = 6755399441055744.0;  // 1.5 * 2^52
    const double Qd = __dsub_rn(__fma_rn(y, tw.y, magic), magic);
    const double ph = __dmul_rn(Qd, q);
    const double pl = __fma_rn(Qd, q, -ph);
    return __dsub_rn(__fma_rn(y, tw.x, -ph), pl);
}
// centred double v (|v| < 2^51) -> v mod q in [0, q) as u64
__device__ __forceinline__ u64 d_mod_to_u64(double v, double q, double qinv) {
    const double magic = 6755399441055744.0;
    const double Qd = __dsub_rn(__fma_rn(v, qinv, magic), magic);
    double r = __fma_rn(-Qd, q, v);  // exact: |r| <= 0.5 q + tiny
    if (r < 0.0) r = __dadd_rn(r, q);
    return (u64)__double_as_longlong(__dadd_rn(r, 4503599627370496.0)) & 0x000FFFFFFFFFFFFFull;
}
__device__ __forceinline__ double center_d(double v, double q, double qinv) {
    const double magic = 6755399441055744.0;
    const double Qd = __dsub_rn(__fma_rn(v, qinv, magic), magic);
    return __fma_rn(-Qd, q, v);  // exact
}

// Karatsuba split-29 sums of products, both factors below 2^40: a = ah 2^29
// + al (al < 2^29, ah < 2^11), same for b.  A sum of up to 33 products is
// kept as S0 = sum al*bl (< 2^58 per term), M = sum (al+ah)(bl+bh) (< 2^58.01
// per term) and S2 = sum ah*bh (< 2^22 per term), none of which can
// overflow its word; the middle sum S1 = M - S0 - S2 (< 2^47) is exact in
// 64-bit arithmetic.  Two 32x32->64 multiply-adds and one 32-bit
// multiply-add per product.  The caller passes the sum bl + bh, which it
// usually shares between products.
#define HB_K29_MASK 0x1FFFFFFFull
struct Kara29 {
    u64 s0, m;
    unsigned s2;
};
__device__ __forceinline__ u64 k29_pack(u64 v) { return ((v >> 29) << 32) | (v & HB_K29_MASK); }
__device__ __forceinline__ unsigned k29_sum(u64 packed) { return (unsigned)packed + (unsigned)(packed >> 32); }
__device__ __forceinline__ void k29_mac(Kara29 &acc, u64 a_packed, u64 b_packed, unsigned b_sum) {
    const unsigned al = (unsigned)a_packed, ah = (unsigned)(a_packed >> 32);
    const unsigned bl = (unsigned)b_packed, bh = (unsigned)(b_packed >> 32);
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s0) : "r"(al), "r"(bl));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.m) : "r"(al + ah), "r"(b_sum));
    acc.s2 += ah * bh;
}
// the same product from unpacked halves and both digit sums
__device__ __forceinline__ void k29_mac_s(Kara29 &acc, unsigned al, unsigned ah, unsigned a_sum, unsigned bl,
                                          unsigned bh, unsigned b_sum) {
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s0) : "r"(al), "r"(bl));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.m) : "r"(a_sum), "r"(b_sum));
    acc.s2 += ah * bh;
}
// a 32-bit unsigned integer as an exact double: the bit pattern 0x43300000:x
// is 2^52 + x
__device__ __forceinline__ double u32_to_double(unsigned x) {
    return __hiloint2double(0x43300000, (int)x) - 4503599627370496.0;
}
// (S0 + S1 2^29 + S2 2^58) mod q for q < 2^40.  Carries give
// a0 + a1 2^29 + hi 2^58 with a0, a1 < 2^29 and hi < 2^28; with c = 2^58 mod q
// the value is congruent to W = a0 + a1 2^29 + hi c < 2^68.  W is formed
// modulo 2^64 on the integer pipe and, approximately, as a double on the
// FP64 pipe (error <= 2^16); Q = round(W / q) from fl(1/q) is then within
// 0.5 + 2^-19 of W/q, so W - Q q (modulo 2^64) lies in (-0.51q, 0.51q) and one
// conditional addition of q finishes.  Five integer multiply instructions
// instead of two 64-bit Shoup reductions.
__device__ __forceinline__ u64 k29_reduce(const Kara29 &a, const PrimeConst &pc) {
    const u64 s1 = a.m - a.s0 - a.s2;
    const u64 t = s1 + (a.s0 >> 29);
    const unsigned a0 = (unsigned)(a.s0 & HB_K29_MASK), a1 = (unsigned)(t & HB_K29_MASK);
    const unsigned hi = a.s2 + (unsigned)(t >> 29);
    const u64 W = (u64)a0 + ((u64)a1 << 29) + (u64)hi * pc.c58;
    const double wd = __fma_rn(u32_to_double(hi), pc.c58d, __fma_rn(u32_to_double(a1), 536870912.0, u32_to_double(a0)));
    const u64 Q = (u64)__double_as_longlong(__fma_rn(wd, pc.qinv, 4503599627370496.0)) & 0x000FFFFFFFFFFFFFull;
    const u64 r = W - Q * pc.q;
    return (long long)r < 0 ? r + pc.q : r;
}

// Split-30 sums of products a*b with one factor below 2^40 and the other
// below 2^61 (basis conversion: a main-prime residue times a constant modulo
// any prime, or a special-prime residue times a constant modulo a main
// prime).  Per term al*bl < 2^60 goes to S0, al*bh + ah*bl < 2^61 + 2^40 to
// S1 and ah*bh < 2^41 to S2.  After at most 4 terms the sums are normalised
// (carries of S0 into S1 and of S1 into S2; the value is unchanged), which
// keeps S0 and S1 below 2^64.
struct SplitW {
    u64 s0, s1, s2;
};
__device__ __forceinline__ void splitw_mac(SplitW &acc, u64 a_packed, u64 b_packed) {
    const unsigned al = (unsigned)a_packed, ah = (unsigned)(a_packed >> 32);
    const unsigned bl = (unsigned)b_packed, bh = (unsigned)(b_packed >> 32);
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s0) : "r"(al), "r"(bl));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s1) : "r"(al), "r"(bh));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s1) : "r"(ah), "r"(bl));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s2) : "r"(ah), "r"(bh));
}
// a * b for a small count a < 2^32 (no high half)
__device__ __forceinline__ void splitw_mac_small(SplitW &acc, unsigned a, u64 b_packed) {
    const unsigned bl = (unsigned)b_packed, bh = (unsigned)(b_packed >> 32);
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s0) : "r"(a), "r"(bl));
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc.s1) : "r"(a), "r"(bh));
}
__device__ __forceinline__ void splitw_normalize(SplitW &acc) {
    acc.s1 += acc.s0 >> 30;
    acc.s0 &= HB_SPLIT_MASK;
    acc.s2 += acc.s1 >> 30;
    acc.s1 &= HB_SPLIT_MASK;
}
// (S0 + S1 2^30 + S2 2^60) mod q for S0 < 2^64, S1 < 2^64 - 2^34,
// S2 < 2^61 - 2^34 (so that hh below fits 31 bits) and 2^26 <= q < 2^62.  Carries give lo + hi 2^60 with lo = a0 + a1 2^30
// (a0, a1 < 2^30); hi = hl + hh 2^30, so the value is congruent to
// W = lo + hl (2^60 mod q) + hh (2^90 mod q) < 2^60 + 2^31 q.  W is formed
// modulo 2^64 on the integer pipe and, approximately (error below
// 2^8 + q 2^-22), as a double; Q = round(W / q) from fl(1/q) is within
// 0.5 + 2^-16 of W/q, so W - Q q (modulo 2^64) is centred below 0.51 q and one
// conditional addition of q finishes.
__device__ __forceinline__ u64 splitw_reduce(const SplitW &s, const PrimeConst &pc) {
    const u64 s1 = s.s1 + (s.s0 >> 30);
    const unsigned a0 = (unsigned)(s.s0 & HB_SPLIT_MASK), a1 = (unsigned)(s1 & HB_SPLIT_MASK);
    const u64 hi = s.s2 + (s1 >> 30);
    const unsigned hl = (unsigned)(hi & HB_SPLIT_MASK), hh = (unsigned)(hi >> 30);
    const u64 W = (u64)a0 + ((u64)a1 << 30) + (u64)hl * pc.c60 + (u64)hh * pc.c90;
    const double lod = __fma_rn(u32_to_double(a1), 1073741824.0, u32_to_double(a0));
    const double wd = __fma_rn(u32_to_double(hh), pc.c90d, __fma_rn(u32_to_double(hl), pc.c60d, lod));
    const u64 Q = (u64)__double_as_longlong(__fma_rn(wd, pc.qinv, 4503599627370496.0)) & 0x000FFFFFFFFFFFFFull;
    const u64 r = W - Q * pc.q;
    return (long long)r < 0 ? r + pc.q : r;
}

// The same reduction for sums of products of two factors below 2^60 (basis
// conversion over primes of up to 60 bits): S0 < 2^64, S1 < 2^64 - 2^34,
// S2 < 2^64 - 2^35, 2^26 <= q < 2^62.  With hi = S2 + (S1 >> 30) < 2^64 split
// as hl + hh 2^30 (hh < 2^34), W = lo + hl (2^60 mod q) + hh (2^90 mod q) is
// congruent to the sum and below 2^60 + 2^35 q; its double image is within
// q 2^-17 of it, so Q = round(W / q) is within 0.5 + 2^-16 of W / q and
// W - Q q (modulo 2^64) lies in (-0.51 q, 0.51 q).
__device__ __forceinline__ u64 splitw_reduce_wide(const SplitW &s, const PrimeConst &pc) {
    const u64 s1 = s.s1 + (s.s0 >> 30);
    const unsigned a0 = (unsigned)(s.s0 & HB_SPLIT_MASK), a1 = (unsigned)(s1 & HB_SPLIT_MASK);
    const u64 hi = s.s2 + (s1 >> 30);
    const unsigned hl = (unsigned)(hi & HB_SPLIT_MASK);
    const u64 hh = hi >> 30;
    const u64 W = (u64)a0 + ((u64)a1 << 30) + (u64)hl * pc.c60 + hh * pc.c90;
    const double lod = __fma_rn(u32_to_double(a1), 1073741824.0, u32_to_double(a0));
    const double wd = __fma_rn(__ull2double_rn(hh), pc.c90d, __fma_rn(u32_to_double(hl), pc.c60d, lod));
    const u64 Q = (u64)__double_as_longlong(__fma_rn(wd, pc.qinv, 4503599627370496.0)) & 0x000FFFFFFFFFFFFFull;
    const u64 r = W - Q * pc.q;
    return (long long)r < 0 ? r + pc.q : r;
}

// bit reversal of the low `bits` bits
__device__ __forceinline__ unsigned brev_bits(unsigned x, int bits) {
    return __brev(x) >> (32 - bits);
}

// Automorphism X -> X^g in the bit-reversed NTT domain: the value at
// position t after the automorphism is the input value at tau_g(t).
__device__ __forceinline__ unsigned aut_index(unsigned t, u64 g, int logN) {
    const u64 mask = (2ull << logN) - 1;  // 2N - 1
    u64 e = 2ull * brev_bits(t, logN) + 1ull;
    u64 e2 = (e * g) & mask;
    return brev_bits((unsigned)((e2 - 1) >> 1), logN);
}

}  // namespace hb

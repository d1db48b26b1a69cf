// Device arithmetic for the sumcheck round and fold passes, shaped for the
// integer pipes of sm_100a.
//
// The generic qmul in qm31.cuh reduces every CM31 product with 64-bit
// shift/and/compare sequences, all of which issue on the ALU pipe; a fused
// fold + round pass then becomes ALU-bound at about a third of HBM bandwidth.
// Here the work is moved onto 32x32->64 multiply-adds (IMAD.WIDE, FMA pipe):
//
//  * sums of products are formed as chains of mad.wide.u32 with the 64-bit
//    running value as the addend; with factors <= P = 2^31 - 1 a chain of four
//    products stays below 4 P^2 < 2^64;
//  * a 64-bit value v = H 2^32 + L is congruent to 2H + L mod P (2^32 = 2 mod P),
//    so a chain result is added to a lazy accumulator with two more
//    multiply-adds and no reduction (acc_fold);
//  * a full reduction (canon64) is one multiply-add plus five ALU operations;
//  * differences of canonical values use the unsigned-min trick (csub).
//
// A QM31 product x * y is written as 4 x 4 base-field coefficients applied to
// y: with x = A + B u, y = C + D u (A, B, C, D in CM31, u^2 = 2 + i),
//   x y = A C + (2 + i) B D + (A D + B C) u,
// so, for a fixed x (a fold challenge), every output coordinate is a four-term
// chain over y's coordinates (alpha_rows).  For sums of products the three CM31
// parts A C, B D and A D + B C are accumulated separately and (2 + i) is
// applied once per thread (QAcc).
#pragma once
#include "qm31.cuh"

namespace zk {

__device__ __forceinline__ uint64_t mad_wide(uint32_t a, uint32_t b, uint64_t c) {
    uint64_t r;
    asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(r) : "r"(a), "r"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t mul_wide(uint32_t a, uint32_t b) {
    uint64_t r;
    asm("mul.wide.u32 %0, %1, %2;" : "=l"(r) : "r"(a), "r"(b));
    return r;
}

// acc + v, congruent mod P: adds 2 * hi(v) + lo(v) (< 3 * 2^32) to acc.
__device__ __forceinline__ uint64_t acc_fold(uint64_t acc, uint64_t v) {
    return mad_wide((uint32_t)v, 1u, mad_wide((uint32_t)(v >> 32), 2u, acc));
}

// Any u64 -> [0, P).
__device__ __forceinline__ uint32_t canon64(uint64_t v) {
    const uint64_t t = mad_wide((uint32_t)(v >> 32), 2u, (uint64_t)(uint32_t)v);  // < 3 * 2^32
    const uint32_t tl = (uint32_t)t, th = (uint32_t)(t >> 32);                      // th <= 2
    const uint32_t u = (tl & P) + (tl >> 31) + 2u * th;                            // <= 2^31 + 4 < 2P
    return min(u, u - P);
}

// a - b mod P for a, b <= P; result <= P.
__device__ __forceinline__ uint32_t csub(uint32_t a, uint32_t b) {
    const uint32_t d = a - b;
    return min(d, d + P);
}

// 2x mod P for x <= P (a 31-bit rotation, since 2^31 = 1 mod P); result <= P.
__device__ __forceinline__ uint32_t cdbl(uint32_t x) { return ((x << 1) | (x >> 30)) & P; }

// 2 hi - lo, coordinate-wise, for canonical inputs (the evaluation at X = 2).
__device__ __forceinline__ qm31 at_two(const qm31& lo, const qm31& hi) {
    return qm(csub(cdbl(hi.a), lo.a), csub(cdbl(hi.b), lo.b), csub(cdbl(hi.c), lo.c), csub(cdbl(hi.d), lo.d));
}

// Lazy accumulator of a sum of QM31 products.
struct QAcc {
    uint64_t ac_re, ac_im, bd_re, bd_im, x_re, x_im;
};

__device__ __forceinline__ void qacc_zero(QAcc& s) { s.ac_re = s.ac_im = s.bd_re = s.bd_im = s.x_re = s.x_im = 0; }

// s += x * y for coordinates <= P.
__device__ __forceinline__ void qacc_mul(QAcc& s, const qm31& x, const qm31& y) {
    const uint32_t nb = P - x.b, nd = P - x.d;
    s.ac_re = acc_fold(s.ac_re, mad_wide(x.a, y.a, mul_wide(nb, y.b)));
    s.ac_im = acc_fold(s.ac_im, mad_wide(x.a, y.b, mul_wide(x.b, y.a)));
    s.bd_re = acc_fold(s.bd_re, mad_wide(x.c, y.c, mul_wide(nd, y.d)));
    s.bd_im = acc_fold(s.bd_im, mad_wide(x.c, y.d, mul_wide(x.d, y.c)));
    s.x_re = acc_fold(s.x_re, mad_wide(x.a, y.c, mad_wide(nb, y.d, mad_wide(x.c, y.a, mul_wide(nd, y.b)))));
    s.x_im = acc_fold(s.x_im, mad_wide(x.a, y.d, mad_wide(x.b, y.c, mad_wide(x.c, y.b, mul_wide(x.d, y.a)))));
}

// The canonical QM31 value of an accumulator: A C + (2 + i) B D + (A D + B C) u.
__device__ __forceinline__ qm31 qacc_value(const QAcc& s) {
    const uint32_t acr = canon64(s.ac_re), aci = canon64(s.ac_im);
    const uint32_t bdr = canon64(s.bd_re), bdi = canon64(s.bd_im);
    const uint32_t r0 = madd(acr, msub(madd(bdr, bdr), bdi));
    const uint32_t r1 = madd(aci, madd(bdr, madd(bdi, bdi)));
    return qm(r0, r1, canon64(s.x_re), canon64(s.x_im));
}

// Multiplication by a fixed x as a 4 x 4 matrix over y's coordinates.
struct AlphaRows {
    uint32_t r[4][4];
};

ZK_HD AlphaRows alpha_rows(const qm31& x) {
    const uint32_t s = msub(madd(x.c, x.c), x.d);  // 2c - d
    const uint32_t t = madd(x.c, madd(x.d, x.d));  // c + 2d
    AlphaRows m;
    m.r[0][0] = x.a; m.r[0][1] = mneg(x.b); m.r[0][2] = s;   m.r[0][3] = mneg(t);
    m.r[1][0] = x.b; m.r[1][1] = x.a;       m.r[1][2] = t;   m.r[1][3] = s;
    m.r[2][0] = x.c; m.r[2][1] = mneg(x.d); m.r[2][2] = x.a; m.r[2][3] = mneg(x.b);
    m.r[3][0] = x.d; m.r[3][1] = x.c;       m.r[3][2] = x.b; m.r[3][3] = x.a;
    return m;
}

// lo + alpha (hi - lo) for canonical QM31 lo, hi; canonical result.
__device__ __forceinline__ qm31 fold_qq(const qm31& lo, const qm31& hi, const AlphaRows& m) {
    const uint32_t d0 = csub(hi.a, lo.a), d1 = csub(hi.b, lo.b), d2 = csub(hi.c, lo.c), d3 = csub(hi.d, lo.d);
    qm31 r;
    r.a = canon64(mad_wide(d0, m.r[0][0], mad_wide(d1, m.r[0][1], mad_wide(d2, m.r[0][2], mad_wide(d3, m.r[0][3], lo.a)))));
    r.b = canon64(mad_wide(d0, m.r[1][0], mad_wide(d1, m.r[1][1], mad_wide(d2, m.r[1][2], mad_wide(d3, m.r[1][3], lo.b)))));
    r.c = canon64(mad_wide(d0, m.r[2][0], mad_wide(d1, m.r[2][1], mad_wide(d2, m.r[2][2], mad_wide(d3, m.r[2][3], lo.c)))));
    r.d = canon64(mad_wide(d0, m.r[3][0], mad_wide(d1, m.r[3][1], mad_wide(d2, m.r[3][2], mad_wide(d3, m.r[3][3], lo.d)))));
    return r;
}

// lo + alpha (hi - lo) for M31 lo, hi <= P; canonical QM31 result.
__device__ __forceinline__ qm31 fold_mq(uint32_t lo, uint32_t hi, const qm31& alpha) {
    const uint32_t d = csub(hi, lo);
    return qm(canon64(mad_wide(d, alpha.a, lo)), canon64(mul_wide(d, alpha.b)), canon64(mul_wide(d, alpha.c)),
              canon64(mul_wide(d, alpha.d)));
}

// lo + alpha d for canonical M31 lo and difference d; canonical QM31 result.
__device__ __forceinline__ qm31 fold_md(uint32_t lo, uint32_t d, const qm31& alpha) {
    return qm(canon64(mad_wide(d, alpha.a, lo)), canon64(mul_wide(d, alpha.b)), canon64(mul_wide(d, alpha.c)),
              canon64(mul_wide(d, alpha.d)));
}

// Per-thread accumulators of one degree-2 product round over QM31 vectors:
// s0 = sum a_lo b_lo, s1 = sum a_hi b_hi, s2 = sum (2 a_hi - a_lo)(2 b_hi - b_lo).
struct RoundAcc {
    QAcc p0, p1, p2;
};

__device__ __forceinline__ void racc_zero(RoundAcc& s) {
    qacc_zero(s.p0);
    qacc_zero(s.p1);
    qacc_zero(s.p2);
}

__device__ __forceinline__ void racc_add(RoundAcc& s, const qm31& alo, const qm31& ahi, const qm31& blo,
                                         const qm31& bhi) {
    qacc_mul(s.p0, alo, blo);
    qacc_mul(s.p1, ahi, bhi);
    qacc_mul(s.p2, at_two(alo, ahi), at_two(blo, bhi));
}

}  // namespace zk

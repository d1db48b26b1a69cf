// Device felt252 arithmetic in radix 2^26 for the Poseidon Merkle kernels.
//
// The 8 x 32-bit form of felt252.cuh needs PTX carry chains (mad.lo.cc /
// madc.hi.cc), which the compiler expands into several integer instructions
// each: a Montgomery product costs ~400 instructions there (measured).  Here an
// element is 10 limbs of 26 bits held in u32 registers, so a 26 x 26-bit
// product is one mad.wide.u32 into a 64-bit column accumulator and no carry
// flag is ever needed: the 100 partial products of a multiplication are 100
// multiply-adds, a squaring 55.
//
// Montgomery form with R = 2^260: x is held as x * 2^260 mod p, any
// representative below 2^258 (limbs may exceed 26 bits between operations, up
// to 2^30).  p = 2^251 + 17 * 2^192 + 1 has radix-2^26 limbs l0 = 1,
// l7 = 17 * 2^10 (192 = 7 * 26 + 10), l9 = 2^17 (251 = 9 * 26 + 17), so
// p = 1 mod 2^26, the Montgomery digit is m = -t mod 2^26, and adding m * p
// touches three columns.  mul26(a, b) returns a * b / 2^260 + M * p / 2^260 <
// a * b / 2^260 + p: for inputs below 2^256 the output is below 2^252 + p <
// 3p, and a cube of an input below 2^256 is below 1.2 p.
#pragma once
#include <stdint.h>

namespace zk {

constexpr uint32_t F26_MASK = (1u << 26) - 1;
constexpr uint32_t F26_P7 = 17u << 10;
constexpr uint32_t F26_P9 = 1u << 17;

struct f26 {
    uint32_t l[10];
};

__device__ __forceinline__ uint64_t f26_mad(uint32_t a, uint32_t b, uint64_t c) {
    uint64_t r;
    asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(r) : "r"(a), "r"(b), "l"(c));
    return r;
}

// Montgomery reduction of the 20 column sums t (t = a * b) into r = t / 2^260 mod p,
// limbs normalised to 26 bits (the top limb keeps the rest).
__device__ __forceinline__ f26 f26_redc(uint64_t (&t)[20]) {
#pragma unroll
    for (int i = 0; i < 10; i++) {
        const uint32_t m = (0u - (uint32_t)t[i]) & F26_MASK;
        t[i] += m;  // low 26 bits become zero
        t[i + 7] = f26_mad(m, F26_P7, t[i + 7]);
        t[i + 9] = f26_mad(m, F26_P9, t[i + 9]);
        t[i + 1] += t[i] >> 26;
    }
    f26 r;
    uint64_t c = 0;
#pragma unroll
    for (int k = 0; k < 9; k++) {
        const uint64_t v = t[10 + k] + c;
        r.l[k] = (uint32_t)v & F26_MASK;
        c = v >> 26;
    }
    r.l[9] = (uint32_t)(t[19] + c);
    return r;
}

__device__ __forceinline__ f26 mul26(const f26& a, const f26& b) {
    uint64_t t[20];
#pragma unroll
    for (int k = 0; k < 20; k++) t[k] = 0;
#pragma unroll
    for (int i = 0; i < 10; i++)
#pragma unroll
        for (int j = 0; j < 10; j++) t[i + j] = f26_mad(a.l[i], b.l[j], t[i + j]);
    return f26_redc(t);
}

// a^2 with the cross products formed once from doubled limbs (limbs < 2^29).
__device__ __forceinline__ f26 sqr26(const f26& a) {
    uint64_t t[20];
#pragma unroll
    for (int k = 0; k < 20; k++) t[k] = 0;
#pragma unroll
    for (int i = 0; i < 10; i++) {
        t[2 * i] = f26_mad(a.l[i], a.l[i], t[2 * i]);
        const uint32_t d = a.l[i] << 1;
#pragma unroll
        for (int j = i + 1; j < 10; j++) t[i + j] = f26_mad(d, a.l[j], t[i + j]);
    }
    return f26_redc(t);
}

// Kept out of line: a Hades permutation calls it 107 times.
__device__ __noinline__ f26 cube26(const f26 x) { return mul26(sqr26(x), x); }

__device__ __forceinline__ f26 add26(const f26& a, const f26& b) {
    f26 r;
#pragma unroll
    for (int i = 0; i < 10; i++) r.l[i] = a.l[i] + b.l[i];
    return r;
}

// Carry-propagate signed limbs to [0, 2^26) (top limb keeps the rest); the
// value must be non-negative.
__device__ __forceinline__ f26 norm26(const f26& a) {
    f26 r;
    int32_t c = 0;
#pragma unroll
    for (int i = 0; i < 9; i++) {
        const int32_t v = (int32_t)a.l[i] + c;
        r.l[i] = (uint32_t)v & F26_MASK;
        c = v >> 26;  // arithmetic shift: floor division
    }
    r.l[9] = (uint32_t)((int32_t)a.l[9] + c);
    return r;
}

// Value below 2^256 (limbs up to 2^30, as left by a few additions) -> a
// representative below 3p with 26-bit limbs, with one carry pass.  The carry the
// lower limbs would bring into limb 9 is below 2^4, so q = l9 >> 17 of the
// unnormalised top limb is floor(v / 2^251) or one less, floor(v / 2^251) is
// floor(v / p) or one more, and subtracting max(q - 1, 0) p limb-wise (limbs may
// go negative; the value does not) leaves v - q' p in [0, 3p).  Every lane the
// permutation keeps below 3p keeps its sums below 2^256 (bounds at each use).
__device__ __forceinline__ f26 red26(const f26& a) {
    f26 n = a;
    uint32_t q = n.l[9] >> 17;
    q -= (q != 0);
    n.l[0] -= q;
    n.l[7] -= q * F26_P7;
    n.l[9] -= q * F26_P9;
    return norm26(n);
}

// Constants, built on the host from the Montgomery (2^256) values of felt252.cpp.
struct F26Consts {
    f26 rc[107];  // compressed round keys, Montgomery (2^260) form
    f26 two;      // Montgomery form of 2 (hash capacity)
    f26 r2;       // 2^520 mod p: canonical integer -> Montgomery form
    f26 one256;   // 2^256 mod p: Montgomery (2^260) -> Montgomery (2^256)
    f26 kp4;      // 4 p with limbs 0-8 >= 2^28 - 4 (so kp4 + a - 2 b keeps limbs >= 0 for 26-bit b)
};
static __constant__ F26Consts c26;

// Full rounds: every lane through the S-box, then the MDS matrix
// [[3,1,1],[1,-1,1],[1,1,-2]].  Inputs below 3p keep every intermediate below
// 2^256 (S-box inputs below 4p, outputs below 1.2p, sums below 7.6p); outputs are
// reduced below 3p.
__device__ __forceinline__ void full_round26(f26 s[3], const f26* rc) {
    const f26 y0 = cube26(add26(s[0], rc[0]));
    const f26 y1 = cube26(add26(s[1], rc[1]));
    const f26 y2 = cube26(add26(s[2], rc[2]));
    const f26 t = add26(add26(y0, y1), y2);  // < 3.6p
    f26 n0 = add26(add26(t, y0), y0);          // < 6p
    f26 n1, n2;
#pragma unroll
    for (int i = 0; i < 10; i++) {
        n1.l[i] = t.l[i] + c26.kp4.l[i] - 2 * y1.l[i];               // < 7.6p
        n2.l[i] = t.l[i] + c26.kp4.l[i] - 3 * y2.l[i];               // < 7.6p
    }
    s[0] = red26(n0);
    s[1] = red26(n1);
    s[2] = red26(n2);
}

// Hades on Montgomery (2^260) lanes below 3p; the result lanes are below 3p.
// The 83 partial rounds keep lane 2 as x = s2 + key (compressed schedule: one
// key per partial round).
__device__ __forceinline__ void hades26(f26 s[3]) {
#pragma unroll 1
    for (int r = 0; r < 4; r++) full_round26(s, c26.rc + 3 * r);
    f26 s0 = s[0], s1 = s[1];
    f26 x = add26(s[2], c26.rc[12]);  // < 4p (lane 2 stays below 11p)
#pragma unroll 1
    for (int r = 0; r < 83; r++) {
        const f26 y = cube26(x);                    // < 1.2p
        const f26 u = add26(s0, s1);                // < 6p
        const f26 t = add26(u, y);                  // < 7.2p
        f26 n0 = add26(add26(t, s0), s0);           // < 13.2p
        f26 n1, xn;
        // w = s0 + s1 (+ the next round's key), left unreduced: the next lane-2
        // value is w - 2y, below 11p with limbs below 2^29, which the S-box takes
        const f26 w = r + 1 < 83 ? add26(u, c26.rc[13 + r]) : u;  // < 7p, limbs < 3 * 2^26
#pragma unroll
        for (int i = 0; i < 10; i++) {
            n1.l[i] = t.l[i] + c26.kp4.l[i] - 2 * s1.l[i];               // t >= s1: in (0, 11.2p)
            xn.l[i] = w.l[i] + c26.kp4.l[i] - 2 * y.l[i];                // 2y < 2.4p: in (0, 11p), limbs >= 0
        }
        s0 = red26(n0);
        s1 = red26(n1);
        x = xn;
    }
    s[0] = s0;
    s[1] = s1;
    s[2] = red26(x);
#pragma unroll 1
    for (int r = 0; r < 4; r++) full_round26(s, c26.rc + 95 + 3 * r);
}

}  // namespace zk

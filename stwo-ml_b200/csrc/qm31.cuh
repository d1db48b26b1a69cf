// M31 / CM31 / QM31 arithmetic shared by the host prover and the CUDA kernels.
//
// Field definitions follow stwo (stwo-gpu/crates/stwo/src/core/fields/):
//   M31  = Z / (2^31 - 1)                                   (m31.rs:14)
//   CM31 = M31[i] / (i^2 + 1)                                (cm31.rs)
//   QM31 = CM31[u] / (u^2 - (2 + i))                         (qm31.rs:14,78-86)
// A QM31 is stored as four u32 words [a, b, c, d] = (a + b i) + (c + d i) u,
// the AoS layout the reference moves between host and GPU
// (engine/src/gpu_sumcheck.rs:3614-3630), so one element is one 16-byte uint4.
//
// Multiplication is written "lazy": CM31 products are formed as sums of
// 32x32->64-bit products (each < 2^62) and reduced once, instead of reducing
// after every M31 multiply.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define ZK_HD __host__ __device__ __forceinline__
#else
#define ZK_HD inline
#endif

namespace zk {

constexpr uint32_t P = 0x7fffffffu;
constexpr uint64_t P2 = (uint64_t)P * P;  // (2^31-1)^2: added before subtracting a product

struct qm31 {
    uint32_t a, b, c, d;
};

// Reduce any u64 to [0, P).
ZK_HD uint32_t red64(uint64_t x) {
    x = (x & P) + (x >> 31);  // < 2^34
    x = (x & P) + (x >> 31);  // < 2^31 + 8
    uint32_t r = (uint32_t)x;
    return r >= P ? r - P : r;
}
// Reduce x < 2^32 to [0, P).
ZK_HD uint32_t red32(uint32_t x) {
    uint32_t r = (x & P) + (x >> 31);
    return r >= P ? r - P : r;
}
ZK_HD uint32_t madd(uint32_t x, uint32_t y) { return red32(x + y); }
ZK_HD uint32_t msub(uint32_t x, uint32_t y) { return red32(x + (P - y)); }
ZK_HD uint32_t mneg(uint32_t x) { return x == 0 ? 0 : P - x; }
ZK_HD uint32_t mmul(uint32_t x, uint32_t y) { return red64((uint64_t)x * y); }

ZK_HD qm31 qm(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    qm31 r;
    r.a = a;
    r.b = b;
    r.c = c;
    r.d = d;
    return r;
}
ZK_HD qm31 qzero() { return qm(0, 0, 0, 0); }
ZK_HD qm31 qone() { return qm(1, 0, 0, 0); }
ZK_HD qm31 qadd(qm31 x, qm31 y) { return qm(madd(x.a, y.a), madd(x.b, y.b), madd(x.c, y.c), madd(x.d, y.d)); }
ZK_HD qm31 qsub(qm31 x, qm31 y) { return qm(msub(x.a, y.a), msub(x.b, y.b), msub(x.c, y.c), msub(x.d, y.d)); }
ZK_HD qm31 qdbl(qm31 x) { return qadd(x, x); }
ZK_HD bool qeq(qm31 x, qm31 y) { return x.a == y.a && x.b == y.b && x.c == y.c && x.d == y.d; }

// (x0 + x1 i)(y0 + y1 i) -> real/imag parts, each reduced once.
ZK_HD void cmul(uint32_t x0, uint32_t x1, uint32_t y0, uint32_t y1, uint32_t& r0, uint32_t& r1) {
    uint64_t re = (uint64_t)x0 * y0 + (P2 - (uint64_t)x1 * y1);  // < 2^63
    uint64_t im = (uint64_t)x0 * y1 + (uint64_t)x1 * y0;         // < 2^63
    r0 = red64(re);
    r1 = red64(im);
}

// (a + b u)(c + d u) = (ac + (2 + i) bd) + (ad + bc) u
ZK_HD qm31 qmul(qm31 x, qm31 y) {
    uint32_t ac0, ac1, bd0, bd1, ad0, ad1, bc0, bc1;
    cmul(x.a, x.b, y.a, y.b, ac0, ac1);
    cmul(x.c, x.d, y.c, y.d, bd0, bd1);
    cmul(x.a, x.b, y.c, y.d, ad0, ad1);
    cmul(x.c, x.d, y.a, y.b, bc0, bc1);
    // (2 + i)(bd0 + bd1 i) = (2 bd0 - bd1) + (bd0 + 2 bd1) i
    uint32_t r0 = red64((uint64_t)ac0 + 2ull * bd0 + (P - bd1));
    uint32_t r1 = red64((uint64_t)ac1 + bd0 + 2ull * bd1);
    return qm(r0, r1, madd(ad0, bc0), madd(ad1, bc1));
}

// QM31 times an M31 scalar.
ZK_HD qm31 qmul_m(qm31 x, uint32_t s) { return qm(mmul(x.a, s), mmul(x.b, s), mmul(x.c, s), mmul(x.d, s)); }

ZK_HD uint32_t mpow(uint32_t x, uint64_t e) {
    uint32_t r = 1;
    while (e) {
        if (e & 1) r = mmul(r, x);
        x = mmul(x, x);
        e >>= 1;
    }
    return r;
}
ZK_HD uint32_t minv(uint32_t x) { return mpow(x, P - 2); }

// (a + b u)^-1 = (a - b u) / (a^2 - (2 + i) b^2); CM31 inverse by the norm.
ZK_HD qm31 qinv(qm31 x) {
    uint32_t a2r, a2i, b2r, b2i;
    cmul(x.a, x.b, x.a, x.b, a2r, a2i);
    cmul(x.c, x.d, x.c, x.d, b2r, b2i);
    uint32_t rb0 = red64(2ull * b2r + (P - b2i));
    uint32_t rb1 = red64((uint64_t)b2r + 2ull * b2i);
    uint32_t d0 = msub(a2r, rb0), d1 = msub(a2i, rb1);
    uint32_t n = minv(red64((uint64_t)d0 * d0 + (uint64_t)d1 * d1));
    uint32_t i0 = mmul(d0, n), i1 = mmul(mneg(d1), n);
    uint32_t r0, r1, r2, r3;
    cmul(x.a, x.b, i0, i1, r0, r1);
    cmul(mneg(x.c), mneg(x.d), i0, i1, r2, r3);
    return qm(r0, r1, r2, r3);
}

}  // namespace zk

// Device felt252 Montgomery multiplication (Stark prime) in 8 x 32-bit limbs,
// used to bring securefield_to_felt leaves into the host's Montgomery form.
// The Merkle kernels' Hades permutation itself runs in radix 2^26 (felt26.cuh).
//
// Representation: 8 x u32 little-endian limbs, Montgomery form with R = 2^256
// (bit-identical to the host's 4 x u64 Montgomery limbs, so host and device
// exchange Montgomery values without conversion).
// p = 2^251 + 17 * 2^192 + 1 has 32-bit limbs [1, 0, 0, 0, 0, 0, 0x11, 0x08000000]:
// p = 1 mod 2^32, so the CIOS quotient digit is m = -t0 and adding m * p
// only touches limbs 0, 6 and 7.  The multiply is written with PTX carry chains.
#pragma once
#include <stdint.h>

namespace zk {

struct dfelt {
    uint32_t w[8];
};

__device__ __forceinline__ bool dgeq_p(const uint32_t t[8]) {
    // compare with p from the top limb down
    if (t[7] != 0x08000000u) return t[7] > 0x08000000u;
    if (t[6] != 0x11u) return t[6] > 0x11u;
    if (t[5] | t[4] | t[3] | t[2] | t[1]) return true;
    return t[0] >= 1u;
}

__device__ __forceinline__ void dsub_p(uint32_t t[8]) {
    asm("sub.cc.u32  %0, %0, 1;\n\t"
        "subc.cc.u32 %1, %1, 0;\n\t"
        "subc.cc.u32 %2, %2, 0;\n\t"
        "subc.cc.u32 %3, %3, 0;\n\t"
        "subc.cc.u32 %4, %4, 0;\n\t"
        "subc.cc.u32 %5, %5, 0;\n\t"
        "subc.cc.u32 %6, %6, 0x11;\n\t"
        "subc.u32    %7, %7, 0x08000000;"
        : "+r"(t[0]), "+r"(t[1]), "+r"(t[2]), "+r"(t[3]), "+r"(t[4]), "+r"(t[5]), "+r"(t[6]), "+r"(t[7]));
}

// One CIOS step: t += a * bi, then t = (t + m p) / 2^32 with m = -t0.
// t has 10 limbs on entry/exit (t[8], t[9] carry words).
__device__ __forceinline__ void cios_step(uint32_t t[10], const uint32_t a[8], uint32_t bi) {
    // low halves of a_j * bi into t[j]
    asm("mad.lo.cc.u32  %0, %10, %18, %0;\n\t"
        "madc.lo.cc.u32 %1, %11, %18, %1;\n\t"
        "madc.lo.cc.u32 %2, %12, %18, %2;\n\t"
        "madc.lo.cc.u32 %3, %13, %18, %3;\n\t"
        "madc.lo.cc.u32 %4, %14, %18, %4;\n\t"
        "madc.lo.cc.u32 %5, %15, %18, %5;\n\t"
        "madc.lo.cc.u32 %6, %16, %18, %6;\n\t"
        "madc.lo.cc.u32 %7, %17, %18, %7;\n\t"
        "addc.cc.u32    %8, %8, 0;\n\t"
        "addc.u32       %9, 0, 0;"
        : "+r"(t[0]), "+r"(t[1]), "+r"(t[2]), "+r"(t[3]), "+r"(t[4]), "+r"(t[5]), "+r"(t[6]), "+r"(t[7]), "+r"(t[8]),
          "=r"(t[9])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(bi));
    // high halves into t[j + 1]
    asm("mad.hi.cc.u32  %0, %9, %17, %0;\n\t"
        "madc.hi.cc.u32 %1, %10, %17, %1;\n\t"
        "madc.hi.cc.u32 %2, %11, %17, %2;\n\t"
        "madc.hi.cc.u32 %3, %12, %17, %3;\n\t"
        "madc.hi.cc.u32 %4, %13, %17, %4;\n\t"
        "madc.hi.cc.u32 %5, %14, %17, %5;\n\t"
        "madc.hi.cc.u32 %6, %15, %17, %6;\n\t"
        "madc.hi.cc.u32 %7, %16, %17, %7;\n\t"
        "addc.u32       %8, %8, 0;"
        : "+r"(t[1]), "+r"(t[2]), "+r"(t[3]), "+r"(t[4]), "+r"(t[5]), "+r"(t[6]), "+r"(t[7]), "+r"(t[8]), "+r"(t[9])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(bi));
    // reduction: m = -t0; add m * (1 + 17 * 2^192 + 2^251) and drop limb 0
    const uint32_t m = 0u - t[0];
    const uint32_t m_lo27 = m << 27, m_hi27 = m >> 5;
    uint32_t dummy;  // receives t0 + m, which is zero mod 2^32; only its carry is used
    asm volatile("add.cc.u32     %10, %0, %11;\n\t"  // t0 + m: zero with carry (t0 != 0)
        "addc.cc.u32    %0, %1, 0;\n\t"
        "addc.cc.u32    %1, %2, 0;\n\t"
        "addc.cc.u32    %2, %3, 0;\n\t"
        "addc.cc.u32    %3, %4, 0;\n\t"
        "addc.cc.u32    %4, %5, 0;\n\t"
        "madc.lo.cc.u32 %5, %11, 17, %6;\n\t"
        "madc.hi.cc.u32 %6, %11, 17, %7;\n\t"
        "addc.cc.u32    %7, %8, %13;\n\t"
        "addc.u32       %8, %9, 0;\n\t"
        "add.cc.u32     %6, %6, %12;\n\t"
        "addc.cc.u32    %7, %7, 0;\n\t"
        "addc.u32       %8, %8, 0;"
        : "+r"(t[0]), "+r"(t[1]), "+r"(t[2]), "+r"(t[3]), "+r"(t[4]), "+r"(t[5]), "+r"(t[6]), "+r"(t[7]), "+r"(t[8]),
          "+r"(t[9]), "=r"(dummy)
        : "r"(m), "r"(m_lo27), "r"(m_hi27));
    t[9] = 0;
}

// Montgomery product a * b / 2^256 mod p (inputs < p, output < p).
__device__ __forceinline__ dfelt dmul(const dfelt& a, const dfelt& b) {
    uint32_t t[10] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; i++) cios_step(t, a.w, b.w[i]);
    dfelt r;
#pragma unroll
    for (int i = 0; i < 8; i++) r.w[i] = t[i];
    if (dgeq_p(r.w)) dsub_p(r.w);
    return r;
}

}  // namespace zk

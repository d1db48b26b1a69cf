// Exact M31 products on the integer tensor pipe: byte planes and u8 MMAs.
//
// An M31 value (or a QM31 coordinate) is split into four bytes, x = sum_b 256^b x_b,
// so a sum of products sum_t x_t y_t becomes sum_{b,c} 256^(b+c) sum_t x_{t,b} y_{t,c}:
// every inner sum is an exact u8 x u8 -> s32 matrix product (mma.m16n8k32), and
// the byte weights 256^s mod P = 2^(8s mod 31) are applied once at the end.
#pragma once
#include <stdint.h>

namespace zk {

// D += A (16 x 32, u8, row) * B (32 x 8, u8, col), s32 accumulators.
__device__ __forceinline__ void mma_u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A (16 x 32, s8, row) * B (32 x 8, s8, col), s32 accumulators.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D += A (16 x 32, u8, row) * B (32 x 8, s8, col), s32 accumulators.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Signed value of an M31 element v < 2^31 read as v (v <= (P-1)/2) or v - P.
__device__ __forceinline__ int m31_signed(uint32_t v) {
    const uint32_t r = (v & 0x7fffffffu) + (v >> 31);
    const uint32_t c = r >= 0x7fffffffu ? r - 0x7fffffffu : r;
    return c <= 0x3fffffffu ? (int)c : (int)c - 0x7fffffff;
}

// Balanced signed byte digit: the low byte of s sign-extended; s - digit is a multiple of 256.
__device__ __forceinline__ int sdigit(int s) { return (int)(int8_t)(s & 0xff); }

// Byte planes of four consecutive u32 elements: plane b = [e0.b, e1.b, e2.b, e3.b].
__device__ __forceinline__ void byte_planes(const uint4& e, uint32_t& p0, uint32_t& p1, uint32_t& p2,
                                            uint32_t& p3) {
    const uint32_t t01 = __byte_perm(e.x, e.y, 0x5140), t23 = __byte_perm(e.z, e.w, 0x5140);
    const uint32_t u01 = __byte_perm(e.x, e.y, 0x7362), u23 = __byte_perm(e.z, e.w, 0x7362);
    p0 = __byte_perm(t01, t23, 0x5410);
    p1 = __byte_perm(t01, t23, 0x7632);
    p2 = __byte_perm(u01, u23, 0x5410);
    p3 = __byte_perm(u01, u23, 0x7632);
}

// 256^s mod P for s = 0..6 (256^s = 2^(8s), 2^31 = 1 mod P).
__device__ __forceinline__ uint32_t pow256(int s) { return 1u << ((8 * s) % 31); }

}  // namespace zk

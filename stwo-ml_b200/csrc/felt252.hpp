// Host felt252 arithmetic and the Starknet Poseidon (Hades) permutation.
//
// Replaces, on the host side of the prover, the starknet-crypto 0.6.2 /
// starknet-ff 0.3.7 calls the reference makes (engine/src/crypto/hades.rs:21-23,
// poseidon_channel.rs:224,251,290, poseidon_merkle.rs:100-110).
//
// Representation: 4 x u64 little-endian limbs in Montgomery form, R = 2^256.
// The Stark prime p = 2^251 + 17 * 2^192 + 1 has limbs [1, 0, 0, 0x0800000000000011],
// so p = 1 mod 2^64: the Montgomery factor -p^-1 mod 2^64 is all-ones, the
// per-limb quotient is simply m = -t0, and adding m*p touches only limb 0
// (which it clears) and limb 3.  The multiply below is specialised to that.
//
// Hades uses the "compressed" round-key schedule: in the 83 partial rounds only
// lane 2 goes through the S-box, so the keys of lanes 0 and 1 are pushed
// through the MDS into the following round; each partial round then adds a
// single key.  The schedule (12 + 83 + 12 = 107 keys) is derived at start-up
// from the 91 x 3 raw keys by compress_round_keys() below.
#pragma once
#include <stdint.h>
#include <string.h>
#include <x86intrin.h>

namespace zk {

typedef unsigned __int128 u128;

struct felt {
    uint64_t l[4];
};

constexpr uint64_t FP0 = 1ull, FP3 = 0x0800000000000011ull;

inline bool f_geq_p(const felt& a) {
    if (a.l[3] != FP3) return a.l[3] > FP3;
    if (a.l[2] != 0 || a.l[1] != 0) return true;
    return a.l[0] >= FP0;
}

inline void f_sub_p(felt& a) {
    // a -= p
    u128 d = (u128)a.l[0] - FP0;
    a.l[0] = (uint64_t)d;
    uint64_t br = (uint64_t)(d >> 64) & 1;
    d = (u128)a.l[1] - br;
    a.l[1] = (uint64_t)d;
    br = (uint64_t)(d >> 64) & 1;
    d = (u128)a.l[2] - br;
    a.l[2] = (uint64_t)d;
    br = (uint64_t)(d >> 64) & 1;
    a.l[3] = a.l[3] - FP3 - br;
}

// r = x < p ? x : x - p, for x < 2p, without data-dependent branches
// (the selects compile to cmov: the Hades adds are unpredictable).
inline felt f_reduce_once(const felt& x) {
    uint64_t d0, d1, d2, d3;
    unsigned char br = _subborrow_u64(0, x.l[0], FP0, (unsigned long long*)&d0);
    br = _subborrow_u64(br, x.l[1], 0, (unsigned long long*)&d1);
    br = _subborrow_u64(br, x.l[2], 0, (unsigned long long*)&d2);
    br = _subborrow_u64(br, x.l[3], FP3, (unsigned long long*)&d3);
    const uint64_t keep = (uint64_t)0 - (uint64_t)br;  // all-ones when x < p
    felt r;
    r.l[0] = (x.l[0] & keep) | (d0 & ~keep);
    r.l[1] = (x.l[1] & keep) | (d1 & ~keep);
    r.l[2] = (x.l[2] & keep) | (d2 & ~keep);
    r.l[3] = (x.l[3] & keep) | (d3 & ~keep);
    return r;
}

inline felt f_add(const felt& a, const felt& b) {
    felt r;
    unsigned char c = _addcarry_u64(0, a.l[0], b.l[0], (unsigned long long*)&r.l[0]);
    c = _addcarry_u64(c, a.l[1], b.l[1], (unsigned long long*)&r.l[1]);
    c = _addcarry_u64(c, a.l[2], b.l[2], (unsigned long long*)&r.l[2]);
    _addcarry_u64(c, a.l[3], b.l[3], (unsigned long long*)&r.l[3]);  // < 2^253: no carry out
    return f_reduce_once(r);
}

inline felt f_sub(const felt& a, const felt& b) {
    felt r;
    unsigned char br = _subborrow_u64(0, a.l[0], b.l[0], (unsigned long long*)&r.l[0]);
    br = _subborrow_u64(br, a.l[1], b.l[1], (unsigned long long*)&r.l[1]);
    br = _subborrow_u64(br, a.l[2], b.l[2], (unsigned long long*)&r.l[2]);
    br = _subborrow_u64(br, a.l[3], b.l[3], (unsigned long long*)&r.l[3]);
    const uint64_t mask = (uint64_t)0 - (uint64_t)br;  // add p back on borrow
    unsigned char c = _addcarry_u64(0, r.l[0], FP0 & mask, (unsigned long long*)&r.l[0]);
    c = _addcarry_u64(c, r.l[1], 0, (unsigned long long*)&r.l[1]);
    c = _addcarry_u64(c, r.l[2], 0, (unsigned long long*)&r.l[2]);
    _addcarry_u64(c, r.l[3], FP3 & mask, (unsigned long long*)&r.l[3]);
    return r;
}

// Montgomery reduction of a 512-bit t[0..8) (t < p * 2^256) to t / 2^256 mod p.
// Each step adds m * p with m = -t[i]: m * 1 clears limb i (carry iff t[i] != 0)
// and m * FP3 lands on limbs i+3, i+4.
inline felt f_redc(uint64_t t[8]) {
    uint64_t extra = 0;  // carry out of limb 7
    for (int i = 0; i < 4; i++) {
        const uint64_t m = (uint64_t)0 - t[i];
        unsigned char c = t[i] != 0;
        c = _addcarry_u64(c, t[i + 1], 0, (unsigned long long*)&t[i + 1]);
        c = _addcarry_u64(c, t[i + 2], 0, (unsigned long long*)&t[i + 2]);
        const u128 mp = (u128)m * FP3;
        c = _addcarry_u64(c, t[i + 3], (uint64_t)mp, (unsigned long long*)&t[i + 3]);
        c = _addcarry_u64(c, t[i + 4], (uint64_t)(mp >> 64), (unsigned long long*)&t[i + 4]);
        for (int j = i + 5; j < 8; j++) c = _addcarry_u64(c, t[j], 0, (unsigned long long*)&t[j]);
        extra += c;
    }
    felt r = {{t[4], t[5], t[6], t[7]}};
    (void)extra;  // t < p * 2^256 keeps the result below 2p < 2^253
    return f_reduce_once(r);
}

// BMI2 + ADX assembly multiply (felt252_x86.S) and whether this CPU can run it.
extern "C" void zk_felt_mont_mul_adx(uint64_t r[4], const uint64_t a[4], const uint64_t b[4]);
extern "C" void zk_felt_mont_cube_adx(uint64_t r[4], const uint64_t a[4]);
extern bool g_felt_use_adx;

// Montgomery product a * b / 2^256 mod p for a, b < p (CIOS, one limb of b per step).
inline felt f_mul_portable(const felt& a, const felt& b) {
    uint64_t t0 = 0, t1 = 0, t2 = 0, t3 = 0, t4 = 0;
    for (int i = 0; i < 4; i++) {
        const uint64_t bi = b.l[i];
        u128 s = (u128)a.l[0] * bi + t0;
        t0 = (uint64_t)s;
        s = (u128)a.l[1] * bi + t1 + (uint64_t)(s >> 64);
        t1 = (uint64_t)s;
        s = (u128)a.l[2] * bi + t2 + (uint64_t)(s >> 64);
        t2 = (uint64_t)s;
        s = (u128)a.l[3] * bi + t3 + (uint64_t)(s >> 64);
        t3 = (uint64_t)s;
        s = (u128)t4 + (uint64_t)(s >> 64);
        t4 = (uint64_t)s;
        const uint64_t t5 = (uint64_t)(s >> 64);
        // m = -t0 mod 2^64; t0 + m * 1 = 0 with a carry iff t0 != 0.
        const uint64_t m = (uint64_t)0 - t0;
        s = (u128)t1 + (t0 != 0);
        t0 = (uint64_t)s;
        s = (u128)t2 + (uint64_t)(s >> 64);
        t1 = (uint64_t)s;
        s = (u128)m * FP3 + t3 + (uint64_t)(s >> 64);
        t2 = (uint64_t)s;
        s = (u128)t4 + (uint64_t)(s >> 64);
        t3 = (uint64_t)s;
        t4 = t5 + (uint64_t)(s >> 64);
    }
    felt r = {{t0, t1, t2, t3}};
    return f_reduce_once(r);
}

inline felt f_mul(const felt& a, const felt& b) {
    if (__builtin_expect(g_felt_use_adx, 1)) {
        felt r;
        zk_felt_mont_mul_adx(r.l, a.l, b.l);
        return r;
    }
    return f_mul_portable(a, b);
}

// Montgomery square: the 6 cross products once, doubled, plus the 4 squares.
inline felt f_sqr(const felt& a) {
    uint64_t t[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    // cross products a_i a_j, i < j
    for (int i = 0; i < 3; i++) {
        uint64_t carry = 0;
        for (int j = i + 1; j < 4; j++) {
            const u128 p = (u128)a.l[i] * a.l[j] + t[i + j] + carry;
            t[i + j] = (uint64_t)p;
            carry = (uint64_t)(p >> 64);
        }
        t[i + 4] = carry;
    }
    // double
    t[7] = t[6] >> 63;
    t[6] = (t[6] << 1) | (t[5] >> 63);
    t[5] = (t[5] << 1) | (t[4] >> 63);
    t[4] = (t[4] << 1) | (t[3] >> 63);
    t[3] = (t[3] << 1) | (t[2] >> 63);
    t[2] = (t[2] << 1) | (t[1] >> 63);
    t[1] = t[1] << 1;
    // squares on the diagonal
    unsigned char c = 0;
    for (int i = 0; i < 4; i++) {
        const u128 sq = (u128)a.l[i] * a.l[i];
        c = _addcarry_u64(c, t[2 * i], (uint64_t)sq, (unsigned long long*)&t[2 * i]);
        c = _addcarry_u64(c, t[2 * i + 1], (uint64_t)(sq >> 64), (unsigned long long*)&t[2 * i + 1]);
    }
    return f_redc(t);
}

// Constants (Montgomery form) set up by felt_init().
extern felt F_R2;     // 2^512 mod p
extern felt F_ONE;    // Montgomery 1
extern felt HADES_RC[107];

void felt_init();  // idempotent, thread-safe

inline felt f_from_u64(uint64_t x) {
    felt r = {{x, 0, 0, 0}};
    return f_mul(r, F_R2);
}
inline felt f_from_canon(const uint64_t v[4]) {
    felt r;
    memcpy(r.l, v, 32);
    return f_mul(r, F_R2);
}
inline void f_to_canon(const felt& a, uint64_t out[4]) {
    felt one = {{1, 0, 0, 0}};
    felt r = f_mul(a, one);
    memcpy(out, r.l, 32);
}
inline felt f_cube(const felt& x) {
    if (__builtin_expect(g_felt_use_adx, 1)) return f_mul(f_mul(x, x), x);
    return f_mul(f_sqr(x), x);
}

// Hades permutation on Montgomery-form state.
void hades(felt s[3]);

// Canonical-integer convenience wrappers.
void poseidon_hash_canon(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]);
void poseidon_hash_many_canon(const uint64_t* in, size_t n, uint64_t out[4]);
felt poseidon_hash_many_m(const felt* in, size_t n);

}  // namespace zk

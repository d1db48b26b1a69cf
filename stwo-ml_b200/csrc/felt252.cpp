// Host felt252 constants, compressed Hades schedule and Poseidon hashes.
// See felt252.hpp for the representation.
#include "felt252.hpp"

#include <mutex>
#include <vector>

namespace zk {

bool g_felt_use_adx = __builtin_cpu_supports("adx") && __builtin_cpu_supports("bmi2");
felt F_R2;
felt F_ONE;
felt HADES_RC[107];

static const uint64_t RAW_ROUND_KEYS[273][4] = {
#include "poseidon3_round_keys.inc"
};

// MDS [[3,1,1],[1,-1,1],[1,1,-2]] as t = s0+s1+s2; (t + 2 s0, t - 2 s1, t - 3 s2).
static inline void mds(felt s[3]) {
    felt t = f_add(f_add(s[0], s[1]), s[2]);
    felt n0 = f_add(t, f_add(s[0], s[0]));
    felt n1 = f_sub(t, f_add(s[1], s[1]));
    felt n2 = f_sub(t, f_add(f_add(s[2], s[2]), s[2]));
    s[0] = n0;
    s[1] = n1;
    s[2] = n2;
}

// Push the lane-0/1 keys of every partial round forward through the MDS.
// Round r of the 91 adds key k_r to the state, so with a carried vector c the
// partial round r effectively adds k_r + c: lane 2's part must stay in round r
// (it feeds the S-box); lanes 0 and 1 are linear, so MDS(k0 + c0, k1 + c1, 0)
// becomes the carry into round r + 1.  The final carry lands on the first
// full round after the partial rounds.
static void compress_round_keys(const felt raw[91][3], felt out[107]) {
    int o = 0;
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 3; i++) out[o++] = raw[r][i];
    felt zero = {{0, 0, 0, 0}};
    felt c[3] = {zero, zero, zero};
    for (int r = 4; r < 87; r++) {
        felt k[3] = {f_add(raw[r][0], c[0]), f_add(raw[r][1], c[1]), f_add(raw[r][2], c[2])};
        out[o++] = k[2];
        felt v[3] = {k[0], k[1], zero};
        mds(v);
        c[0] = v[0];
        c[1] = v[1];
        c[2] = v[2];
    }
    for (int i = 0; i < 3; i++) out[o++] = f_add(raw[87][i], c[i]);
    for (int r = 88; r < 91; r++)
        for (int i = 0; i < 3; i++) out[o++] = raw[r][i];
}

static void init_impl() {
    // R mod p, then R^2 mod p, by doubling from 1 (canonical domain).
    felt x = {{1, 0, 0, 0}};
    for (int i = 0; i < 512; i++) {
        if (i == 256) F_ONE = x;
        felt y;
        u128 s = (u128)x.l[0] + x.l[0];
        y.l[0] = (uint64_t)s;
        s = (u128)x.l[1] + x.l[1] + (uint64_t)(s >> 64);
        y.l[1] = (uint64_t)s;
        s = (u128)x.l[2] + x.l[2] + (uint64_t)(s >> 64);
        y.l[2] = (uint64_t)s;
        y.l[3] = x.l[3] + x.l[3] + (uint64_t)(s >> 64);
        if (f_geq_p(y)) f_sub_p(y);
        x = y;
    }
    F_R2 = x;
    felt raw[91][3];
    for (int r = 0; r < 91; r++)
        for (int i = 0; i < 3; i++) raw[r][i] = f_from_canon(RAW_ROUND_KEYS[3 * r + i]);
    compress_round_keys(raw, HADES_RC);
}

void felt_init() {
    static std::once_flag once;
    std::call_once(once, init_impl);
}

// ---------------------------------------------------------------------------
// Fast path (BMI2 + ADX): lazy reduction.  The cube accepts inputs < 5p and
// returns values < 1.3p, so additions in front of it need no reduction; in the
// 83 partial rounds the S-box lane carries x = s2 + key (< 5p) and its critical
// path is x -> x^2 -> x^3 -> (w + 3p - 2 x^3), where w = (s0 + s1 + next key)
// mod p is computed off that path.
// ---------------------------------------------------------------------------
namespace {

inline felt mul_adx(const felt& a, const felt& b) {
    felt r;
    zk_felt_mont_mul_adx(r.l, a.l, b.l);
    return r;
}
// x^3 (in Montgomery form: x^3 / R^2) for x < 5p, both multiplications in one call; the
// result is below 1.3 p (not reduced).
inline felt cube_adx(const felt& a) {
    felt r;
    zk_felt_mont_cube_adx(r.l, a.l);
    return r;
}
// 256-bit add / subtract without reduction (callers keep results in range).
// Early-clobber outputs: the carry chains write limbs before reading later inputs.
inline felt add4(const felt& a, const felt& b) {
    felt r = a;
    asm("addq %4, %0\n\tadcq %5, %1\n\tadcq %6, %2\n\tadcq %7, %3"
        : "+&r"(r.l[0]), "+&r"(r.l[1]), "+&r"(r.l[2]), "+&r"(r.l[3])
        : "rm"(b.l[0]), "rm"(b.l[1]), "rm"(b.l[2]), "rm"(b.l[3])
        : "cc");
    return r;
}
inline felt sub4(const felt& a, const felt& b) {
    felt r = a;
    asm("subq %4, %0\n\tsbbq %5, %1\n\tsbbq %6, %2\n\tsbbq %7, %3"
        : "+&r"(r.l[0]), "+&r"(r.l[1]), "+&r"(r.l[2]), "+&r"(r.l[3])
        : "rm"(b.l[0]), "rm"(b.l[1]), "rm"(b.l[2]), "rm"(b.l[3])
        : "cc");
    return r;
}
inline felt dbl4(const felt& a) { return add4(a, a); }
// x < 2p -> x mod p (cmov, no branch)
inline felt red_once(const felt& x) {
    felt r = x;
    uint64_t t0, t1, t2, t3;
    asm("movq %0, %4\n\tsubq $1, %4\n\t"
        "movq %1, %5\n\tsbbq $0, %5\n\t"
        "movq %2, %6\n\tsbbq $0, %6\n\t"
        "movq %3, %7\n\tsbbq %8, %7\n\t"
        "cmovncq %4, %0\n\tcmovncq %5, %1\n\tcmovncq %6, %2\n\tcmovncq %7, %3"
        : "+&r"(r.l[0]), "+&r"(r.l[1]), "+&r"(r.l[2]), "+&r"(r.l[3]), "=&r"(t0), "=&r"(t1), "=&r"(t2), "=&r"(t3)
        : "r"(FP3)
        : "cc");
    return r;
}
// x < 16p -> x mod p: q = floor(x / 2^251) is floor(x / p) or one more, so
// x - max(q - 1, 0) p is in [0, 2p).
inline felt red_full(const felt& x) {
    uint64_t q = x.l[3] >> 59;
    q -= (q != 0);
    const felt qp = {{q, 0, 0, q * FP3}};
    return red_once(sub4(x, qp));
}

const felt kP = {{1, 0, 0, FP3}};

inline void full_round_fast(felt s[3], const felt* rc, const felt& p2, const felt& p3) {
    felt y0 = add4(s[0], rc[0]), y1 = add4(s[1], rc[1]), y2 = add4(s[2], rc[2]);
    y0 = cube_adx(y0);
    y1 = cube_adx(y1);
    y2 = cube_adx(y2);
    const felt t = add4(add4(y0, y1), y2);                             // < 3.9p
    s[0] = red_full(add4(t, dbl4(y0)));                                // < 6.5p
    s[1] = red_full(sub4(add4(t, p2), dbl4(y1)));                      // t >= y1: >= 0, < 5.9p
    s[2] = red_full(sub4(add4(t, p3), add4(dbl4(y2), y2)));            // t >= y2: >= 0, < 6.9p
}

void hades_fast(felt s[3]) {
    const felt p2 = add4(kP, kP), p3 = add4(p2, kP);
    const felt* rc = HADES_RC;
    for (int r = 0; r < 4; r++, rc += 3) full_round_fast(s, rc, p2, p3);
    felt s0 = s[0], s1 = s[1];
    felt x = add4(s[2], rc[0]);
    for (int r = 0; r < 83; r++) {
        const felt y = cube_adx(x);                                    // < 1.3p
        const felt u = add4(s0, s1);                                   // < 2p
        const felt t = add4(u, y);                                     // < 3.3p
        const felt n0 = red_full(add4(t, dbl4(s0)));
        const felt n1 = red_full(sub4(add4(t, p2), dbl4(s1)));
        if (r + 1 < 83) {
            const felt w = red_full(add4(u, rc[r + 1]));               // s0 + s1 + next key
            x = sub4(add4(w, p3), dbl4(y));                            // next s2 + key, in (0.4p, 4p)
        } else {
            x = red_full(sub4(add4(u, p3), dbl4(y)));                  // s2 after the last partial round
        }
        s0 = n0;
        s1 = n1;
    }
    rc += 83;
    s[0] = s0;
    s[1] = s1;
    s[2] = x;
    for (int r = 0; r < 4; r++, rc += 3) full_round_fast(s, rc, p2, p3);
}

}  // namespace

void hades(felt s[3]) {
    if (__builtin_expect(g_felt_use_adx, 1)) {
        hades_fast(s);
        return;
    }
    const felt* rc = HADES_RC;
    for (int r = 0; r < 4; r++, rc += 3) {
        s[0] = f_cube(f_add(s[0], rc[0]));
        s[1] = f_cube(f_add(s[1], rc[1]));
        s[2] = f_cube(f_add(s[2], rc[2]));
        mds(s);
    }
    for (int r = 0; r < 83; r++, rc += 1) {
        s[2] = f_cube(f_add(s[2], rc[0]));
        mds(s);
    }
    for (int r = 0; r < 4; r++, rc += 3) {
        s[0] = f_cube(f_add(s[0], rc[0]));
        s[1] = f_cube(f_add(s[1], rc[1]));
        s[2] = f_cube(f_add(s[2], rc[2]));
        mds(s);
    }
}

void poseidon_hash_canon(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]) {
    felt_init();
    felt s[3] = {f_from_canon(a), f_from_canon(b), f_from_u64(2)};
    hades(s);
    f_to_canon(s[0], out);
}

felt poseidon_hash_many_m(const felt* in, size_t n) {
    felt zero = {{0, 0, 0, 0}};
    felt s[3] = {zero, zero, zero};
    size_t i = 0;
    for (; n - i >= 2; i += 2) {
        s[0] = f_add(s[0], in[i]);
        s[1] = f_add(s[1], in[i + 1]);
        hades(s);
    }
    if (n - i == 1) {
        s[0] = f_add(s[0], in[i]);
        s[1] = f_add(s[1], F_ONE);
    } else {
        s[0] = f_add(s[0], F_ONE);
    }
    hades(s);
    return s[0];
}

void poseidon_hash_many_canon(const uint64_t* in, size_t n, uint64_t out[4]) {
    felt_init();
    std::vector<felt> v(n);
    for (size_t i = 0; i < n; i++) v[i] = f_from_canon(in + 4 * i);
    f_to_canon(poseidon_hash_many_m(v.data(), n), out);
}

}  // namespace zk

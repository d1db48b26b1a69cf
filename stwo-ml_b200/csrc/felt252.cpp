// Host felt252 constants, compressed Hades schedule and Poseidon hashes.
// See felt252.hpp for the representation.
#include "felt252.hpp"

#include <mutex>
#include <vector>

namespace zk {

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

void hades(felt s[3]) {
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

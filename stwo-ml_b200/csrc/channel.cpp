// Host Poseidon channel and the C-ABI wrappers for it (see channel.hpp).
#include "channel.hpp"

#include <vector>

namespace zk {

felt felt_of_qm31(const qm31& v) {
    // 2^124 sentinel | a << 93 | b << 62 | c << 31 | d  (< 2^125, already canonical)
    u128 lo = ((u128)1 << 124) | ((u128)v.a << 93) | ((u128)v.b << 62) | ((u128)v.c << 31) | v.d;
    felt r = {{(uint64_t)lo, (uint64_t)(lo >> 64), 0, 0}};
    return f_mul(r, F_R2);
}

felt pack_m31s(const uint32_t* m, size_t cnt) {
    uint64_t a[4] = {1, 0, 0, 0};
    for (size_t i = 0; i < cnt; i++) {
        a[3] = (a[3] << 31) | (a[2] >> 33);
        a[2] = (a[2] << 31) | (a[1] >> 33);
        a[1] = (a[1] << 31) | (a[0] >> 33);
        a[0] = (a[0] << 31) | m[i];
    }
    return f_from_canon(a);
}

void Channel::hash_many_into_digest(const felt* tail, size_t n) {
    felt buf[8];
    std::vector<felt> big;
    felt* in = buf;
    if (n + 1 > 8) {
        big.resize(n + 1);
        in = big.data();
    }
    in[0] = f_from_canon(st->digest);
    for (size_t i = 0; i < n; i++) in[i + 1] = tail[i];
    f_to_canon(poseidon_hash_many_m(in, n + 1), st->digest);
    st->n_draws = 0;
    st->hash_count++;
}

void Channel::mix_poly_coeffs(const qm31& c0, const qm31& c1, const qm31& c2) {
    const uint32_t w[12] = {c0.a, c0.b, c0.c, c0.d, c1.a, c1.b, c1.c, c1.d, c2.a, c2.b, c2.c, c2.d};
    felt t[2] = {pack_m31s(w, 8), pack_m31s(w + 8, 4)};
    hash_many_into_digest(t, 2);
}

void Channel::mix_poly_coeffs_deg3(const qm31& c0, const qm31& c1, const qm31& c2, const qm31& c3) {
    const uint32_t w[16] = {c0.a, c0.b, c0.c, c0.d, c1.a, c1.b, c1.c, c1.d,
                            c2.a, c2.b, c2.c, c2.d, c3.a, c3.b, c3.c, c3.d};
    felt t[2] = {pack_m31s(w, 8), pack_m31s(w + 8, 8)};
    hash_many_into_digest(t, 2);
}

void Channel::mix_felts(const qm31* v, size_t n) {
    if (n == 0) return;
    std::vector<felt> t;
    t.reserve(n / 2 + 1);
    for (size_t i = 0; i < n; i += 2) {
        uint32_t w[8] = {v[i].a, v[i].b, v[i].c, v[i].d, 0, 0, 0, 0};
        if (i + 1 < n) {
            w[4] = v[i + 1].a;
            w[5] = v[i + 1].b;
            w[6] = v[i + 1].c;
            w[7] = v[i + 1].d;
            t.push_back(pack_m31s(w, 8));
        } else {
            t.push_back(pack_m31s(w, 4));
        }
    }
    hash_many_into_digest(t.data(), t.size());
}

}  // namespace zk

using namespace zk;

static inline qm31 ld(const uint32_t* p) { return qm(p[0], p[1], p[2], p[3]); }

extern "C" {

void zkml_channel_init(zkml_channel* ch) {
    felt_init();
    memset(ch, 0, sizeof(*ch));
}
void zkml_channel_mix_u64(zkml_channel* ch, uint64_t v) { Channel(ch).mix_u64(v); }
void zkml_channel_mix_felt(zkml_channel* ch, const uint64_t v[4]) {
    Channel c(ch);
    c.mix_m(f_from_canon(v));
}
void zkml_channel_mix_qm31(zkml_channel* ch, const uint32_t v[4]) { Channel(ch).mix_qm31(ld(v)); }
void zkml_channel_draw_felt252(zkml_channel* ch, uint64_t out[4]) { Channel(ch).draw_canon(out); }
void zkml_channel_draw_qm31(zkml_channel* ch, uint32_t out[4]) {
    qm31 q = Channel(ch).draw_qm31();
    out[0] = q.a;
    out[1] = q.b;
    out[2] = q.c;
    out[3] = q.d;
}
void zkml_channel_mix_poly_coeffs(zkml_channel* ch, const uint32_t c[12]) {
    Channel(ch).mix_poly_coeffs(ld(c), ld(c + 4), ld(c + 8));
}
void zkml_channel_mix_poly_coeffs_deg3(zkml_channel* ch, const uint32_t c[16]) {
    Channel(ch).mix_poly_coeffs_deg3(ld(c), ld(c + 4), ld(c + 8), ld(c + 12));
}
void zkml_channel_mix_felts(zkml_channel* ch, const uint32_t* qm31s, size_t n) {
    Channel(ch).mix_felts(reinterpret_cast<const qm31*>(qm31s), n);
}
void zkml_hades_permutation(uint64_t state[12]) {
    felt_init();
    felt s[3] = {f_from_canon(state), f_from_canon(state + 4), f_from_canon(state + 8)};
    hades(s);
    for (int i = 0; i < 3; i++) f_to_canon(s[i], state + 4 * i);
}
void zkml_poseidon_hash(const uint64_t a[4], const uint64_t b[4], uint64_t out[4]) {
    poseidon_hash_canon(a, b, out);
}
void zkml_poseidon_hash_many(const uint64_t* in, size_t n, uint64_t out[4]) {
    poseidon_hash_many_canon(in, n, out);
}
void zkml_securefield_to_felt(const uint32_t v[4], uint64_t out[4]) {
    felt_init();
    f_to_canon(felt_of_qm31(ld(v)), out);
}

}  // extern "C"

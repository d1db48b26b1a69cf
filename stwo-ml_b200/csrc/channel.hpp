// Host Poseidon Fiat-Shamir channel, transcript-compatible with the engine's
// PoseidonChannel (engine/src/crypto/poseidon_channel.rs:83-306).
//
//   mix_felt(v)        digest = hades([digest, v, 2])[0]; n_draws = 0
//   mix_u64(v)         mix_felt(v)
//   draw_felt252()     hades([digest, n_draws, 3])[0]; n_draws += 1
//   draw_qm31()        one draw; four times: remainder mod 2^31 reduced mod P,
//                      then floor-divide by 2^31 (least significant limb first)
//   mix_poly_coeffs    digest = poseidon_hash_many([digest, pack(c0,c1), pack(c2)])
//   mix_poly_coeffs_deg3  ... [digest, pack(c0,c1), pack(c2,c3)]
//   mix_felts(qs)      digest = poseidon_hash_many([digest, pack pairs of QM31 ...])
// where pack() is acc = 1; acc = acc * 2^31 + m over the M31 words (a sentinel
// "1" keeps leading zeros), which never exceeds 2^249 < p for 8 words.
//
// The state is kept in the C-ABI struct zkml_channel (canonical digest limbs,
// n_draws, hash_count) so callers can carry it across calls losslessly.
#pragma once
#include "../../include/zkml_b200.h"
#include "felt252.hpp"
#include "qm31.cuh"

namespace zk {

felt felt_of_qm31(const qm31& v);  // securefield_to_felt, Montgomery form

struct Channel {
    zkml_channel* st;
    explicit Channel(zkml_channel* s) : st(s) { felt_init(); }

    void mix_m(const felt& v) {
        felt s[3] = {f_from_canon(st->digest), v, f_from_u64(2)};
        hades(s);
        f_to_canon(s[0], st->digest);
        st->n_draws = 0;
        st->hash_count++;
    }
    void mix_u64(uint64_t v) { mix_m(f_from_u64(v)); }
    void mix_qm31(const qm31& v) { mix_m(felt_of_qm31(v)); }  // mix_secure_field
    // Returns the draw in canonical limbs.
    void draw_canon(uint64_t out[4]) {
        felt s[3] = {f_from_canon(st->digest), f_from_u64(st->n_draws), f_from_u64(3)};
        hades(s);
        st->n_draws++;
        st->hash_count++;
        f_to_canon(s[0], out);
    }
    qm31 draw_qm31() {
        uint64_t v[4];
        draw_canon(v);
        uint32_t m[4];
        for (int i = 0; i < 4; i++) {
            uint32_t rem = (uint32_t)(v[0] & 0x7fffffffu);
            m[i] = rem == P ? 0 : rem;
            v[0] = (v[0] >> 31) | (v[1] << 33);
            v[1] = (v[1] >> 31) | (v[2] << 33);
            v[2] = (v[2] >> 31) | (v[3] << 33);
            v[3] >>= 31;
        }
        return qm(m[0], m[1], m[2], m[3]);
    }
    void hash_many_into_digest(const felt* tail, size_t n);
    void mix_poly_coeffs(const qm31& c0, const qm31& c1, const qm31& c2);
    void mix_poly_coeffs_deg3(const qm31& c0, const qm31& c1, const qm31& c2, const qm31& c3);
    void mix_felts(const qm31* v, size_t n);
};

// pack_m31s (poseidon_channel.rs:22-29) for up to 8 words; Montgomery result.
felt pack_m31s(const uint32_t* m, size_t cnt);

}  // namespace zk

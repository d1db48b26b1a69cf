// Host writer of serialize_gkr_model_proof records (cairo_serde.rs): felts as
// 4 canonical u64 limbs, u32/u64 fields as one felt, QM31 as four felts.
#pragma once
#include <cstdint>
#include <cstring>

#include "qm31.cuh"

namespace zk {

struct Out {
    uint64_t* buf;
    size_t cap, len = 0;
    bool overflow = false;
    void push(const uint64_t f[4]) {
        if (len < cap) memcpy(buf + 4 * len, f, 32);
        else overflow = true;
        len++;
    }
    void u64(uint64_t x) {
        const uint64_t f[4] = {x, 0, 0, 0};
        push(f);
    }
    void qm(const uint32_t v[4]) {
        for (int i = 0; i < 4; i++) u64(v[i]);
    }
    void q(const qm31& v) {
        u64(v.a);
        u64(v.b);
        u64(v.c);
        u64(v.d);
    }
};

typedef Out FeltOut;

}  // namespace zk

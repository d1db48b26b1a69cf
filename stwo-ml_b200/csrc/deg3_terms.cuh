// Quadratic constraint terms of the algebraic activation sumchecks (piecewise, ReLU).
// Over one pair every folded vector is x0 + t xd, so a term x (u - g in - e x) of the
// combined constraint h is a quadratic in t; its coefficients are accumulated lazily.
#pragma once
#include "round_arith.cuh"

namespace zk {

__device__ __forceinline__ qm31 qmul_fr(const qm31& x, const qm31& y) {
    QAcc s;
    qacc_zero(s);
    qacc_mul(s, x, y);
    return qacc_value(s);
}

// h(t) = h0 + h1 t + h2 t^2 accumulated lazily over one pair.
struct PwAcc {
    QAcc H0, H1, H2;
};

// One indicator (or segment bit) with value x0 + t xd: adds x (u - g in - e x), where
// in = in0 + t ind and g is null for a segment bit.
__device__ __forceinline__ void pw_term(PwAcc& a, const qm31& x0, const qm31& xd, const qm31& u, const qm31* g,
                                        const qm31& e, const qm31& in0, const qm31& ind) {
    qm31 y0 = qsub(u, qmul_fr(e, x0)), yd = qsub(qzero(), qmul_fr(e, xd));
    if (g) {
        y0 = qsub(y0, qmul_fr(*g, in0));
        yd = qsub(yd, qmul_fr(*g, ind));
    }
    qacc_mul(a.H0, x0, y0);
    qacc_mul(a.H1, x0, yd);
    qacc_mul(a.H1, xd, y0);
    qacc_mul(a.H2, xd, yd);
}

}  // namespace zk

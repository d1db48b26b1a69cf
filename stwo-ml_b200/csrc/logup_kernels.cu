// sm_100a kernels for the LogUp activation layer (gkr/prover.rs:6390-6600):
// range masking + table lookup + multiplicity histogram, the denominators
// d = gamma - in - beta * out and their inverses w = 1/d, the trace / table
// LogUp sums, eq-weighted dot products, and the degree-3 eq-sumcheck rounds
// (s(t) = sum eq_t w_t d_t at t = 0..3) with the fold of eq, w and d fused in.
#include "logup.cuh"
#include "logup_device.cuh"

namespace zk {

// ---------------------------------------------------------------------------
__global__ void logup_prepare_kernel(const uint32_t* __restrict__ input, uint32_t rows, uint32_t cols, size_t pc,
                                     size_t n, uint32_t mask, const uint32_t* __restrict__ table,
                                     uint32_t* __restrict__ x_out, uint32_t* __restrict__ m_in,
                                     uint32_t* __restrict__ m_out, uint32_t* __restrict__ mult,
                                     uint32_t* __restrict__ err) {
    uint32_t bad = 0;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t i = idx / pc, j = idx % pc;
        uint32_t x = 0;
        if (i < rows && j < cols) {
            x = input[i * cols + j];
            bad |= x;
            x = red32(x);
        }
        const uint32_t mi = x & mask;
        x_out[idx] = x;
        m_in[idx] = mi;
        m_out[idx] = __ldg(table + mi);
        // lanes of a warp that hit the same table entry add once (inputs cluster on few entries)
        const unsigned active = __activemask();
        const unsigned peers = __match_any_sync(active, mi);
        if ((__ffs(peers) - 1) == (int)(threadIdx.x & 31)) atomicAdd(mult + mi, (uint32_t)__popc(peers));
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

void launch_logup_prepare(const uint32_t* input, uint32_t rows, uint32_t cols, size_t pc, size_t n, uint32_t mask,
                          const uint32_t* table, uint32_t* x_out, uint32_t* m_in, uint32_t* m_out, uint32_t* mult,
                          uint32_t* err, int max_blocks, cudaStream_t s) {
    logup_prepare_kernel<<<grid_for(n, max_blocks * 4), 256, 0, s>>>(input, rows, cols, pc, n, mask, table, x_out,
                                                                      m_in, m_out, mult, err);
}

// d = gamma - in - beta * out, w = 1 / d, and trace_sum = sum w  (4 words).
// Each thread inverts its DW_BATCH elements (grid-strided, so loads stay
// coalesced) with one QM31 inversion: prefix products, one inverse, and a
// backward pass (three products per element).  A batch containing d = 0 is
// inverted element by element, so the result is the same as qinv of each d.
constexpr int DW_BATCH = 8;

__global__ void __launch_bounds__(256) logup_dw_kernel(const uint32_t* __restrict__ m_in,
                                                       const uint32_t* __restrict__ m_out, size_t n, qm31 gamma,
                                                       qm31 beta, uint4* __restrict__ d, uint4* __restrict__ w,
                                                       ReduceScratch rs) {
    unsigned long long acc[4] = {0, 0, 0, 0};
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i0 < n; i0 += stride * DW_BATCH) {
        qm31 dv[DW_BATCH], pre[DW_BATCH];
        bool zero = false;
        qm31 run = qone();
#pragma unroll
        for (int e = 0; e < DW_BATCH; e++) {
            const size_t i = i0 + e * stride;
            dv[e] = qone();
            if (i < n) {
                dv[e] = qsub(qsub(gamma, qm(m_in[i], 0, 0, 0)), qmul_m(beta, m_out[i]));
                stq4(d + i, dv[e]);
                zero |= (dv[e].a | dv[e].b | dv[e].c | dv[e].d) == 0;
            }
            pre[e] = run;  // product of dv[0..e)
            run = qmul_f(run, dv[e]);
        }
        if (!zero) {
            qm31 inv = qinv(run);  // 1 / prod dv
#pragma unroll
            for (int e = DW_BATCH - 1; e >= 0; e--) {
                const size_t i = i0 + e * stride;
                const qm31 we = qmul_f(inv, pre[e]);
                inv = qmul_f(inv, dv[e]);
                if (i < n) {
                    stq4(w + i, we);
                    acc_q<4>(acc, 0, we);
                }
            }
        } else {
#pragma unroll
            for (int e = 0; e < DW_BATCH; e++) {
                const size_t i = i0 + e * stride;
                if (i < n) {
                    const qm31 we = qinv(dv[e]);
                    stq4(w + i, we);
                    acc_q<4>(acc, 0, we);
                }
            }
        }
    }
    grid_reduce<4>(acc, rs);
}

void launch_logup_dw(const uint32_t* m_in, const uint32_t* m_out, size_t n, qm31 gamma, qm31 beta, uint4* d,
                     uint4* w, const ReduceScratch& rs, cudaStream_t s) {
    logup_dw_kernel<<<grid_for((n + DW_BATCH - 1) / DW_BATCH, rs.max_blocks), 256, 0, s>>>(m_in, m_out, n, gamma,
                                                                                           beta, d, w, rs);
}

// table_sum = sum_{j : mult_j > 0} mult_j / (gamma - j - beta * table_j)  (4 words)
__global__ void __launch_bounds__(256) logup_table_sum_kernel(const uint32_t* __restrict__ mult,
                                                              const uint32_t* __restrict__ table, size_t tsize,
                                                              qm31 gamma, qm31 beta, ReduceScratch rs) {
    unsigned long long acc[4] = {0, 0, 0, 0};
    for (size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x; j < tsize; j += (size_t)gridDim.x * blockDim.x) {
        const uint32_t m = mult[j];
        if (!m) continue;
        const qm31 dj = qsub(qsub(gamma, qm((uint32_t)j, 0, 0, 0)), qmul_m(beta, table[j]));
        acc_q<4>(acc, 0, qmul_m(qinv(dj), red32(m)));
    }
    grid_reduce<4>(acc, rs);
}

void launch_logup_table_sum(const uint32_t* mult, const uint32_t* table, size_t tsize, qm31 gamma, qm31 beta,
                            const ReduceScratch& rs, cudaStream_t s) {
    logup_table_sum_kernel<<<grid_for(tsize, rs.max_blocks), 256, 0, s>>>(mult, table, tsize, gamma, beta, rs);
}

// sum_i eq[i] * x_v[i] for NV (1..4) M31 vectors: 4 * NV words.
struct EqDotSrc {
    const uint32_t* x[4];
};

template <int NV>
__global__ void __launch_bounds__(256) eq_dot_kernel(const uint4* __restrict__ eq, const EqDotSrc src, size_t n,
                                                     ReduceScratch rs) {
    unsigned long long acc[4 * NV];
#pragma unroll
    for (int i = 0; i < 4 * NV; i++) acc[i] = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const qm31 e = ldq4(eq + i);
#pragma unroll
        for (int v = 0; v < NV; v++) acc_q<4 * NV>(acc, 4 * v, qmul_m(e, __ldg(src.x[v] + i)));
    }
    grid_reduce<4 * NV>(acc, rs);
}

void launch_eq_dot(const uint4* eq, const uint32_t* const* xs, int nv, size_t n, const ReduceScratch& rs,
                   cudaStream_t s) {
    EqDotSrc src{};
    for (int v = 0; v < nv && v < 4; v++) src.x[v] = xs[v];
    const unsigned g = grid_for(n, rs.max_blocks);
    switch (nv) {
        case 1: eq_dot_kernel<1><<<g, 256, 0, s>>>(eq, src, n, rs); break;
        case 2: eq_dot_kernel<2><<<g, 256, 0, s>>>(eq, src, n, rs); break;
        case 3: eq_dot_kernel<3><<<g, 256, 0, s>>>(eq, src, n, rs); break;
        default: eq_dot_kernel<4><<<g, 256, 0, s>>>(eq, src, n, rs); break;
    }
}

void launch_eq_dot(const uint4* eq, const uint32_t* x0, const uint32_t* x1, size_t n, const ReduceScratch& rs,
                   cudaStream_t s) {
    const uint32_t* xs[2] = {x0, x1};
    launch_eq_dot(eq, xs, x1 ? 2 : 1, n, rs, s);
}

// Degree-3 eq-sumcheck round.  With FOLD, first folds (eq, w, d) in place with
// alpha (length 2h -> h); then emits s(t) = sum_{i < q} eq_t w_t d_t for
// t = 0, 1, 2, 3 over pairs (i, i + q), q = h / 2 (16 words).
template <bool FOLD>
__global__ void __launch_bounds__(256) logup_round_kernel(uint4* __restrict__ E, uint4* __restrict__ W,
                                                          uint4* __restrict__ D, size_t h, const AlphaRows m,
                                                          ReduceScratch rs) {
    const size_t q = h / 2;
    QAcc acc[4];
#pragma unroll
    for (int t = 0; t < 4; t++) qacc_zero(acc[t]);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        qm31 v[3][2];  // [vector][lo/hi]
        uint4* vec[3] = {E, W, D};
#pragma unroll
        for (int k = 0; k < 3; k++) {
            if (FOLD) {
                const qm31 a0 = ldq4(vec[k] + i), a1 = ldq4(vec[k] + i + q);
                const qm31 a2 = ldq4(vec[k] + i + h), a3 = ldq4(vec[k] + i + q + h);
                v[k][0] = fold_qq(a0, a2, m);
                v[k][1] = fold_qq(a1, a3, m);
                stq4(vec[k] + i, v[k][0]);
                stq4(vec[k] + i + q, v[k][1]);
            } else {
                v[k][0] = ldq4(vec[k] + i);
                v[k][1] = ldq4(vec[k] + i + q);
            }
        }
        qm31 x[3], dlt[3];
#pragma unroll
        for (int k = 0; k < 3; k++) {
            x[k] = v[k][0];
            dlt[k] = qsub(v[k][1], v[k][0]);
        }
#pragma unroll
        for (int t = 0; t < 4; t++) {
            qacc_mul(acc[t], qmul_f(x[0], x[1]), x[2]);
#pragma unroll
            for (int k = 0; k < 3; k++) x[k] = qadd(x[k], dlt[k]);
        }
    }
    unsigned long long words[16];
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const qm31 r = qacc_value(acc[t]);
        words[4 * t] = r.a;
        words[4 * t + 1] = r.b;
        words[4 * t + 2] = r.c;
        words[4 * t + 3] = r.d;
    }
    grid_reduce<16>(words, rs);
}

void launch_logup_round(uint4* E, uint4* W, uint4* D, size_t len, bool fold, qm31 alpha, const ReduceScratch& rs,
                        cudaStream_t s) {
    if (fold) {
        const size_t h = len / 2;
        logup_round_kernel<true><<<grid_for(h / 2, rs.max_blocks), 256, 0, s>>>(E, W, D, h, alpha_rows(alpha), rs);
    } else {
        logup_round_kernel<false><<<grid_for(len / 2, rs.max_blocks), 256, 0, s>>>(E, W, D, len, alpha_rows(alpha),
                                                                                   rs);
    }
}

// Final fold of length-2 (eq, w, d) vectors: publishes w and d (8 words).
__global__ void logup_final_kernel(const uint4* E, const uint4* W, const uint4* D, qm31 alpha, ReduceScratch rs) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const qm31 w0 = ldq4(W), w1 = ldq4(W + 1), d0 = ldq4(D), d1 = ldq4(D + 1);
    const qm31 w = qadd(w0, qmul(alpha, qsub(w1, w0)));
    const qm31 d = qadd(d0, qmul(alpha, qsub(d1, d0)));
    const uint32_t words[8] = {w.a, w.b, w.c, w.d, d.a, d.b, d.c, d.d};
    for (int i = 0; i < 8; i++) rs.out[i] = words[i];
    if (rs.sig) publish_words(rs.sig, rs.seq, words, 8);
    (void)E;
}

void launch_logup_final(const uint4* E, const uint4* W, const uint4* D, qm31 alpha, const ReduceScratch& rs,
                        cudaStream_t s) {
    logup_final_kernel<<<1, 32, 0, s>>>(E, W, D, alpha, rs);
}

// Degree-1 sumcheck over the multiplicity MLE: (sum lo-half, sum hi-half).
// M31 mode reads the raw counts (first round); QM31 mode folds first when FOLD.
template <bool M31IN, bool FOLD>
__global__ void __launch_bounds__(256) mult_round_kernel(const uint32_t* __restrict__ src32, uint4* __restrict__ V,
                                                         size_t h, qm31 alpha, ReduceScratch rs) {
    // with FOLD: fold length 2h -> h (from src32 when M31IN, else V in place), then
    // sum the halves of the folded vector (q = h / 2); without FOLD: halves of length h.
    unsigned long long acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const size_t q = FOLD ? h / 2 : h / 2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        qm31 lo, hi;
        if (FOLD) {
            qm31 a0, a1, a2, a3;
            if (M31IN) {
                a0 = qm(red32(src32[i]), 0, 0, 0);
                a1 = qm(red32(src32[i + q]), 0, 0, 0);
                a2 = qm(red32(src32[i + h]), 0, 0, 0);
                a3 = qm(red32(src32[i + q + h]), 0, 0, 0);
            } else {
                a0 = ldq4(V + i);
                a1 = ldq4(V + i + q);
                a2 = ldq4(V + i + h);
                a3 = ldq4(V + i + q + h);
            }
            const AlphaRows m = alpha_rows(alpha);
            lo = fold_qq(a0, a2, m);
            hi = fold_qq(a1, a3, m);
            stq4(V + i, lo);
            stq4(V + i + q, hi);
        } else {
            if (M31IN) {
                lo = qm(red32(src32[i]), 0, 0, 0);
                hi = qm(red32(src32[i + q]), 0, 0, 0);
            } else {
                lo = ldq4(V + i);
                hi = ldq4(V + i + q);
            }
        }
        acc_q<8>(acc, 0, lo);
        acc_q<8>(acc, 4, hi);
    }
    grid_reduce<8>(acc, rs);
}

void launch_mult_round(const uint32_t* src32, uint4* V, size_t len, bool first, bool fold, qm31 alpha,
                       const ReduceScratch& rs, cudaStream_t s) {
    if (!fold) {
        if (first)
            mult_round_kernel<true, false><<<grid_for(len / 2, rs.max_blocks), 256, 0, s>>>(src32, V, len, alpha, rs);
        else
            mult_round_kernel<false, false><<<grid_for(len / 2, rs.max_blocks), 256, 0, s>>>(src32, V, len, alpha, rs);
        return;
    }
    const size_t h = len / 2;
    if (first)
        mult_round_kernel<true, true><<<grid_for(h / 2, rs.max_blocks), 256, 0, s>>>(src32, V, h, alpha, rs);
    else
        mult_round_kernel<false, true><<<grid_for(h / 2, rs.max_blocks), 256, 0, s>>>(src32, V, h, alpha, rs);
}

// Last fold of a length-2 multiplicity vector (from counts if M31IN): 4 words.
__global__ void mult_final_kernel(const uint32_t* src32, const uint4* V, qm31 alpha, ReduceScratch rs) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    qm31 a0, a1;
    if (src32) {
        a0 = qm(red32(src32[0]), 0, 0, 0);
        a1 = qm(red32(src32[1]), 0, 0, 0);
    } else {
        a0 = ldq4(V);
        a1 = ldq4(V + 1);
    }
    const qm31 r = qadd(a0, qmul(alpha, qsub(a1, a0)));
    const uint32_t words[4] = {r.a, r.b, r.c, r.d};
    for (int i = 0; i < 4; i++) rs.out[i] = words[i];
    if (rs.sig) publish_words(rs.sig, rs.seq, words, 4);
}

void launch_mult_final(const uint32_t* src32, const uint4* V, qm31 alpha, const ReduceScratch& rs, cudaStream_t s) {
    mult_final_kernel<<<1, 32, 0, s>>>(src32, V, alpha, rs);
}

}  // namespace zk

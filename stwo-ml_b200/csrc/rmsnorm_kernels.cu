// sm_100a kernels of the RMSNorm layer reduction (gkr/prover.rs:8424-8790):
// the per-row rms^2 / rsqrt lookup that builds every vector the three
// sumchecks read, and the rounds of the plain sumcheck sum_x input(x)^2.
// The degree-3 eq-sumchecks and the LogUp passes are the LogUp kernels.
#include "logup_device.cuh"

namespace zk {

// One block per padded row (grid-strided).  Pass 1 sums the squares of the
// row's first n_active columns (values canonicalised, so a 64-bit sum of
// < 2^31 terms per thread cannot overflow); thread 0 forms rms^2 and looks up
// rsqrt; pass 2 writes the row's vectors.  Padding rows and columns hold 0.
__global__ void __launch_bounds__(256) rmsnorm_prepare_kernel(
    const uint32_t* __restrict__ input, uint32_t rows, uint32_t cols, uint32_t pr, uint32_t pc, uint32_t n_active,
    uint32_t inv_n, const uint32_t* __restrict__ gamma, uint32_t gamma_len, const uint32_t* __restrict__ table,
    uint32_t mask, uint32_t* __restrict__ x_out, uint32_t* __restrict__ m_in, uint32_t* __restrict__ m_out,
    uint32_t* __restrict__ outv, uint4* __restrict__ W, uint4* __restrict__ D, uint32_t* __restrict__ row_rms,
    uint32_t* __restrict__ mult, uint32_t* __restrict__ err) {
    __shared__ unsigned long long part[8];
    __shared__ uint32_t s_rms, s_rs;
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t bad = 0;
    for (uint32_t i = blockIdx.x; i < pr; i += gridDim.x) {
        const uint32_t* row = input + (size_t)i * cols;
        const bool real = i < rows;
        unsigned long long sq = 0;
        if (real) {
            const uint32_t lim = min(n_active, cols);
            for (uint32_t j = threadIdx.x; j < lim; j += blockDim.x) {
                const uint32_t x = red32(__ldg(row + j));
                sq += canon64(mul_wide(x, x));
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        if (lane == 0) part[warp] = sq;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long t = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += part[w];
            const uint32_t rms = mmul(red64(t), inv_n) & mask;
            s_rms = rms;
            s_rs = __ldg(table + rms);
            row_rms[i] = rms;
            atomicAdd(mult + rms, pc);
        }
        __syncthreads();
        const uint32_t rms = s_rms, rs = s_rs;
        const size_t base = (size_t)i * pc;
        for (uint32_t j = threadIdx.x; j < pc; j += blockDim.x) {
            uint32_t x = 0;
            if (real && j < cols) {
                x = __ldg(row + j);
                bad |= x;
                x = red32(x);
            }
            uint32_t sc = rs, o = x;
            if (j < n_active) {
                if (gamma) {
                    const uint32_t g = __ldg(gamma + min(j, gamma_len - 1));
                    bad |= g;
                    sc = mmul(rs, red32(g));
                }
                o = mmul(x, sc);
            }
            const size_t idx = base + j;
            x_out[idx] = x;
            m_in[idx] = rms;
            m_out[idx] = rs;
            outv[idx] = o;
            W[idx] = make_uint4(x, 0, 0, 0);
            D[idx] = make_uint4(sc, 0, 0, 0);
        }
        __syncthreads();  // s_rms / part are rewritten by the next row
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

void launch_rmsnorm_prepare(const uint32_t* input, uint32_t rows, uint32_t cols, uint32_t pr, uint32_t pc,
                            uint32_t n_active, uint32_t inv_n, const uint32_t* gamma, uint32_t gamma_len,
                            const uint32_t* table, uint32_t mask, uint32_t* x_out, uint32_t* m_in, uint32_t* m_out,
                            uint32_t* outv, uint4* W, uint4* D, uint32_t* row_rms, uint32_t* mult, uint32_t* err,
                            int max_blocks, cudaStream_t s) {
    const size_t cap = (size_t)max_blocks * 8;
    const unsigned g = (unsigned)(pr < cap ? pr : cap);
    rmsnorm_prepare_kernel<<<g, 256, 0, s>>>(input, rows, cols, pr, pc, n_active, inv_n, gamma, gamma_len, table,
                                             mask, x_out, m_in, m_out, outv, W, D, row_rms, mult, err);
}

// Plain sumcheck round: s(0) = sum lo^2, s(1) = sum hi^2, s(2) = sum (2 hi - lo)^2
// over pairs (i, i + q) of the current vector (12 words).  With FOLD the
// vector is first folded 2h -> h with alpha (from src32 when M31IN, else V in place).
template <bool M31IN, bool FOLD>
__global__ void __launch_bounds__(256) sq_round_kernel(const uint32_t* __restrict__ src32, uint4* __restrict__ V,
                                                       size_t h, const AlphaRows m, ReduceScratch rs) {
    const size_t q = h / 2;
    QAcc acc[3];
#pragma unroll
    for (int t = 0; t < 3; t++) qacc_zero(acc[t]);
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
            lo = fold_qq(a0, a2, m);
            hi = fold_qq(a1, a3, m);
            stq4(V + i, lo);
            stq4(V + i + q, hi);
        } else if (M31IN) {
            lo = qm(red32(src32[i]), 0, 0, 0);
            hi = qm(red32(src32[i + q]), 0, 0, 0);
        } else {
            lo = ldq4(V + i);
            hi = ldq4(V + i + q);
        }
        const qm31 two = at_two(lo, hi);
        qacc_mul(acc[0], lo, lo);
        qacc_mul(acc[1], hi, hi);
        qacc_mul(acc[2], two, two);
    }
    unsigned long long words[12];
#pragma unroll
    for (int t = 0; t < 3; t++) {
        const qm31 r = qacc_value(acc[t]);
        words[4 * t] = r.a;
        words[4 * t + 1] = r.b;
        words[4 * t + 2] = r.c;
        words[4 * t + 3] = r.d;
    }
    grid_reduce<12>(words, rs);
}

void launch_sq_round(const uint32_t* src32, uint4* V, size_t len, bool first, bool fold, qm31 alpha,
                     const ReduceScratch& rs, cudaStream_t s) {
    const AlphaRows m = alpha_rows(alpha);
    if (!fold) {
        const unsigned g = grid_for(len / 2, rs.max_blocks);
        if (first)
            sq_round_kernel<true, false><<<g, 256, 0, s>>>(src32, V, len, m, rs);
        else
            sq_round_kernel<false, false><<<g, 256, 0, s>>>(src32, V, len, m, rs);
        return;
    }
    const size_t h = len / 2;
    const unsigned g = grid_for(h / 2, rs.max_blocks);
    if (first)
        sq_round_kernel<true, true><<<g, 256, 0, s>>>(src32, V, h, m, rs);
    else
        sq_round_kernel<false, true><<<g, 256, 0, s>>>(src32, V, h, m, rs);
}

}  // namespace zk

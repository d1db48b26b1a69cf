// sm_100a kernels of the LayerNorm layer reduction (reduce_layernorm_layer,
// gkr/prover.rs:7944-8354): the per-row mean / variance / rsqrt pass that builds
// every vector the three sumchecks read, and the rounds of the batched mean /
// variance plain sumcheck.  The degree-3 eq-sumchecks and the LogUp passes are
// the LogUp kernels.
#include "logup.cuh"
#include "logup_device.cuh"
#include "round_arith.cuh"

namespace zk {

// Sum over a block of 64-bit lazily accumulated values < 2^63 (canonical terms).
__device__ __forceinline__ unsigned long long block_sum64(unsigned long long v, unsigned long long* part) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0) part[warp] = v;
    __syncthreads();
    unsigned long long t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += part[w];
    __syncthreads();
    return t;
}

// One block per padded row (grid-strided): mean over the first n_active columns
// (zero past cols), variance = sum (x - mean)^2 / n_active masked to the table,
// rsqrt from the table; then per element x, centered = x - mean, mean, variance,
// rsqrt and the output centered * rsqrt (apply_layernorm_detailed,
// compiler/prove.rs:977-1060).  Padding rows are all zero (mean 0, variance 0).
__global__ void __launch_bounds__(256) layernorm_prepare_kernel(
    const uint32_t* __restrict__ input, uint32_t rows, uint32_t cols, uint32_t pr, uint32_t pc, uint32_t n_active,
    uint32_t inv_n, const uint32_t* __restrict__ table, uint32_t mask, uint32_t* __restrict__ x_out,
    uint32_t* __restrict__ cen, uint32_t* __restrict__ mean_v, uint32_t* __restrict__ var_v,
    uint32_t* __restrict__ rs_v, uint32_t* __restrict__ outv, uint32_t* __restrict__ row_mean,
    uint32_t* __restrict__ row_var, uint32_t* __restrict__ mult, uint32_t* __restrict__ err) {
    __shared__ unsigned long long part[8];
    uint32_t bad = 0;
    for (uint32_t i = blockIdx.x; i < pr; i += gridDim.x) {
        const uint32_t* row = input + (size_t)i * cols;
        const bool real = i < rows;
        unsigned long long sum = 0;
        if (real)
            for (uint32_t j = threadIdx.x; j < min(n_active, cols); j += blockDim.x) sum += red32(__ldg(row + j));
        const uint32_t mean = mmul(red64(block_sum64(sum, part)), inv_n);
        unsigned long long sq = 0;
        for (uint32_t j = threadIdx.x; j < n_active; j += blockDim.x) {
            const uint32_t x = (real && j < cols) ? red32(__ldg(row + j)) : 0u;
            const uint32_t d = msub(x, mean);
            sq += canon64(mul_wide(d, d));
        }
        const uint32_t var = mmul(red64(block_sum64(sq, part)), inv_n) & mask;
        const uint32_t rs = __ldg(table + var);
        if (threadIdx.x == 0) {
            row_mean[i] = mean;
            row_var[i] = var;
            atomicAdd(mult + var, pc);
        }
        const size_t base = (size_t)i * pc;
        for (uint32_t j = threadIdx.x; j < pc; j += blockDim.x) {
            uint32_t x = 0;
            if (real && j < cols) {
                x = __ldg(row + j);
                bad |= x;
                x = red32(x);
            }
            const uint32_t c = msub(x, mean);
            const size_t idx = base + j;
            x_out[idx] = x;
            cen[idx] = c;
            mean_v[idx] = mean;
            var_v[idx] = var;
            rs_v[idx] = rs;
            outv[idx] = mmul(c, rs);
        }
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

void launch_layernorm_prepare(const uint32_t* input, uint32_t rows, uint32_t cols, uint32_t pr, uint32_t pc,
                              uint32_t n_active, uint32_t inv_n, const uint32_t* table, uint32_t mask,
                              uint32_t* x_out, uint32_t* cen, uint32_t* mean_v, uint32_t* var_v, uint32_t* rs_v,
                              uint32_t* outv, uint32_t* row_mean, uint32_t* row_var, uint32_t* mult, uint32_t* err,
                              int max_blocks, cudaStream_t s) {
    const size_t cap = (size_t)max_blocks * 8;
    const unsigned g = (unsigned)(pr < cap ? pr : cap);
    layernorm_prepare_kernel<<<g, 256, 0, s>>>(input, rows, cols, pr, pc, n_active, inv_n, table, mask, x_out, cen,
                                               mean_v, var_v, rs_v, outv, row_mean, row_var, mult, err);
}

// Batched mean / variance round (prover.rs:8062-8085): s(t) = sum eta0 in_t + eta1 c_t^2 at
// t = 0, 1, 2 over pairs (i, i + q) (12 words).  With FOLD the input, centered and mean
// vectors are first folded 2h -> h with alpha (from the M31 vectors when M31IN).
template <bool M31IN, bool FOLD>
__global__ void __launch_bounds__(256) mv_round_kernel(const uint32_t* __restrict__ x32,
                                                       const uint32_t* __restrict__ c32,
                                                       const uint32_t* __restrict__ m32, uint4* __restrict__ IN,
                                                       uint4* __restrict__ C, uint4* __restrict__ M, size_t h,
                                                       const AlphaRows am, qm31 eta0, qm31 eta1, ReduceScratch rs) {
    const size_t q = h / 2;
    QAcc acc[3];
#pragma unroll
    for (int t = 0; t < 3; t++) qacc_zero(acc[t]);
    auto ld = [&](const uint32_t* s32, const uint4* V, size_t i) {
        return M31IN ? qm(red32(s32[i]), 0, 0, 0) : ldq4(V + i);
    };
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        qm31 il, ih, cl, ch;
        if (FOLD) {
            il = fold_qq(ld(x32, IN, i), ld(x32, IN, i + h), am);
            ih = fold_qq(ld(x32, IN, i + q), ld(x32, IN, i + q + h), am);
            cl = fold_qq(ld(c32, C, i), ld(c32, C, i + h), am);
            ch = fold_qq(ld(c32, C, i + q), ld(c32, C, i + q + h), am);
            const qm31 ml = fold_qq(ld(m32, M, i), ld(m32, M, i + h), am);
            const qm31 mh = fold_qq(ld(m32, M, i + q), ld(m32, M, i + q + h), am);
            stq4(IN + i, il);
            stq4(IN + i + q, ih);
            stq4(C + i, cl);
            stq4(C + i + q, ch);
            stq4(M + i, ml);
            stq4(M + i + q, mh);
        } else {
            il = ld(x32, IN, i);
            ih = ld(x32, IN, i + q);
            cl = ld(c32, C, i);
            ch = ld(c32, C, i + q);
        }
        const qm31 ins[3] = {il, ih, at_two(il, ih)};
        const qm31 cs[3] = {cl, ch, at_two(cl, ch)};
#pragma unroll
        for (int t = 0; t < 3; t++) {
            qacc_mul(acc[t], eta0, ins[t]);
            qacc_mul(acc[t], eta1, qmul_f(cs[t], cs[t]));
        }
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

void launch_mv_round(const uint32_t* x32, const uint32_t* c32, const uint32_t* m32, uint4* IN, uint4* C, uint4* M,
                     size_t len, bool first, bool fold, qm31 alpha, qm31 eta0, qm31 eta1, const ReduceScratch& rs,
                     cudaStream_t s) {
    const AlphaRows am = alpha_rows(alpha);
    if (!fold) {
        const unsigned g = grid_for(len / 2, rs.max_blocks);
        if (first)
            mv_round_kernel<true, false><<<g, 256, 0, s>>>(x32, c32, m32, IN, C, M, len, am, eta0, eta1, rs);
        else
            mv_round_kernel<false, false><<<g, 256, 0, s>>>(x32, c32, m32, IN, C, M, len, am, eta0, eta1, rs);
        return;
    }
    const size_t h = len / 2;
    const unsigned g = grid_for(h / 2, rs.max_blocks);
    if (first)
        mv_round_kernel<true, true><<<g, 256, 0, s>>>(x32, c32, m32, IN, C, M, h, am, eta0, eta1, rs);
    else
        mv_round_kernel<false, true><<<g, 256, 0, s>>>(x32, c32, m32, IN, C, M, h, am, eta0, eta1, rs);
}

// Last fold of the length-2 input and mean vectors: input then mean (8 words).
__global__ void mv_final_kernel(const uint32_t* x32, const uint32_t* m32, const uint4* IN, const uint4* M,
                                qm31 alpha, ReduceScratch rs) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    qm31 v[2][2];
    for (int u = 0; u < 2; u++) {
        v[0][u] = x32 ? qm(red32(x32[u]), 0, 0, 0) : ldq4(IN + u);
        v[1][u] = m32 ? qm(red32(m32[u]), 0, 0, 0) : ldq4(M + u);
    }
    uint32_t words[8];
    for (int k = 0; k < 2; k++) {
        const qm31 r = qadd(v[k][0], qmul(alpha, qsub(v[k][1], v[k][0])));
        words[4 * k] = r.a;
        words[4 * k + 1] = r.b;
        words[4 * k + 2] = r.c;
        words[4 * k + 3] = r.d;
    }
    for (int i = 0; i < 8; i++) rs.out[i] = words[i];
    if (rs.sig) publish_words(rs.sig, rs.seq, words, 8);
}

void launch_mv_final(const uint32_t* x32, const uint32_t* m32, const uint4* IN, const uint4* M, qm31 alpha,
                     const ReduceScratch& rs, cudaStream_t s) {
    mv_final_kernel<<<1, 32, 0, s>>>(x32, m32, IN, M, alpha, rs);
}

// W = centered, D = rsqrt as QM31 (the linear eq-sumcheck's operands).
__global__ void lift2_kernel(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, size_t n,
                             uint4* __restrict__ W, uint4* __restrict__ D) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        W[i] = make_uint4(a[i], 0, 0, 0);
        D[i] = make_uint4(b[i], 0, 0, 0);
    }
}

void launch_lift2(const uint32_t* a, const uint32_t* b, size_t n, uint4* W, uint4* D, cudaStream_t s) {
    size_t g = (n + 255) / 256;
    if (g > 8192) g = 8192;
    lift2_kernel<<<(unsigned)g, 256, 0, s>>>(a, b, n, W, D);
}

// apply_layernorm_detailed (compiler/prove.rs:977-1060) with dim = cols: one block per row.
__global__ void __launch_bounds__(256) layernorm_forward_kernel(const uint32_t* __restrict__ x, uint32_t rows,
                                                                uint32_t cols, uint32_t inv_n,
                                                                const uint32_t* __restrict__ table,
                                                                uint32_t* __restrict__ y) {
    __shared__ unsigned long long part[8];
    for (uint32_t i = blockIdx.x; i < rows; i += gridDim.x) {
        const uint32_t* row = x + (size_t)i * cols;
        unsigned long long sum = 0;
        for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) sum += red32(row[j]);
        const uint32_t mean = mmul(red64(block_sum64(sum, part)), inv_n);
        unsigned long long sq = 0;
        for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) {
            const uint32_t d = msub(red32(row[j]), mean);
            sq += canon64(mul_wide(d, d));
        }
        const uint32_t rs = table[mmul(red64(block_sum64(sq, part)), inv_n) & 0xFFFFu];
        for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x)
            y[(size_t)i * cols + j] = mmul(msub(red32(row[j]), mean), rs);
    }
}

void launch_layernorm_forward(const uint32_t* x, uint32_t rows, uint32_t cols, uint32_t inv_n, const uint32_t* table,
                              uint32_t* y, cudaStream_t s) {
    layernorm_forward_kernel<<<rows < 8192 ? rows : 8192, 256, 0, s>>>(x, rows, cols, inv_n, table, y);
}

}  // namespace zk

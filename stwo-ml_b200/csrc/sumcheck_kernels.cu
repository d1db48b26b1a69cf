// sm_100a kernels for the GKR matmul sumcheck: eq tables, the W.eq(r)
// restrictions, and the degree-2 round reductions with fused in-place folds.
//
// All arithmetic is M31/QM31 integer work (no tensor cores).  The restriction
// is HBM-bound: it streams the weight matrix once with 16-byte loads and keeps
// 4 x 4 64-bit accumulators per thread, reducing modulo 2^31 - 1 only every
// four products (each product < 2^62, so four of them plus a reduced residue
// still fit in 64 bits).
#include "kernels.cuh"
#include "round_arith.cuh"

namespace zk {

__device__ __forceinline__ qm31 ld_q(const uint4* p) {
    uint4 v = *p;
    return qm(v.x, v.y, v.z, v.w);
}
__device__ __forceinline__ void st_q(uint4* p, qm31 x) { *p = make_uint4(x.a, x.b, x.c, x.d); }

// Reduce a u64 accumulator to < 2^34 (keeps it congruent mod P).
__device__ __forceinline__ unsigned long long lazy(unsigned long long x) { return (x & P) + (x >> 31); }

// acc += a * b as one 32x32 -> 64-bit multiply-add with a 64-bit addend.
__device__ __forceinline__ void mac(unsigned long long& acc, uint32_t a, uint32_t b) {
    asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc) : "r"(a), "r"(b));
}

// Cheap partial reduction: x = H 2^32 + L = 2H + L (mod P) since 2^32 = 2 mod P;
// the result is < 2^34, so four more products (< 2^62 each) fit in 64 bits.
__device__ __forceinline__ unsigned long long lazy2(unsigned long long x) {
    unsigned long long r;
    asm("{\n\t.reg .u32 lo, hi;\n\t.reg .u64 l64;\n\t"
        "mov.b64 {lo, hi}, %1;\n\t"
        "cvt.u64.u32 l64, lo;\n\t"
        "mad.wide.u32 %0, hi, 2, l64;\n\t}"
        : "=l"(r)
        : "l"(x));
    return r;
}

// ---------------------------------------------------------------------------
// eq table
// ---------------------------------------------------------------------------
__global__ void eq_table_kernel(EqChallenges ch, uint4* __restrict__ table, size_t len) {
    const size_t n = (size_t)1 << ch.v;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < len;
         idx += (size_t)gridDim.x * blockDim.x) {
        qm31 w = qzero();
        if (idx < n) {
            w = qone();
            for (int l = 0; l < ch.v; l++) {
                const int bit = (idx >> (ch.v - 1 - l)) & 1;
                w = qmul(w, bit ? ch.c[l] : qsub(qone(), ch.c[l]));
            }
        }
        st_q(table + idx, w);
    }
}

void launch_eq_table(const qm31* c, int v, uint4* table, size_t table_len, cudaStream_t s) {
    EqChallenges ch;
    ch.v = v;
    for (int i = 0; i < v; i++) ch.c[i] = c[i];
    const int threads = 256;
    size_t blocks = (table_len + threads - 1) / threads;
    if (blocks > 4096) blocks = 4096;
    if (blocks == 0) blocks = 1;
    eq_table_kernel<<<(unsigned)blocks, threads, 0, s>>>(ch, table, table_len);
}

// ---------------------------------------------------------------------------
// Column restriction f_b[i] = sum_j B[i][j] L_j  (the HBM-bound hot spot)
//
// The row-major matrix is viewed as a flat sequence of "stripes" of 64
// columns of one row.  Each warp owns a contiguous range of stripes (so the
// work is balanced to within one stripe whatever k and n are); lane t loads
// columns 2t, 2t+1 of every stripe with one 8-byte streaming load (a warp
// reads 256 contiguous bytes per stripe).  The eq table is split as
// L_j = lhi[j >> 6] * llo[j & 63]: lane t accumulates
// sum_stripes lhi[stripe] * B[., 2t + e] for its two columns e in 2 x 4 64-bit
// accumulators, and only when the warp leaves a row it multiplies by its two
// llo entries, reduces across the warp and adds the row's partial with one
// 64-bit atomic per component.  UNROLL stripes are loaded before any is used
// to keep enough bytes in flight per SM.
// ---------------------------------------------------------------------------
constexpr int RC_UNROLL = 8;

constexpr uint32_t RC_SMEM_LHI = 1024;  // lhi entries staged in shared memory (n <= 65536)

template <bool VEC, bool SMEM_LHI>
__global__ void __launch_bounds__(256, 4)
    restrict_cols_kernel(const uint32_t* __restrict__ B, uint32_t k, uint32_t n, uint32_t s_row,
                         unsigned long long total, const uint4* __restrict__ lhi_g,
                         const uint4* __restrict__ llo, unsigned long long* __restrict__ acc_out,
                         uint32_t* __restrict__ err) {
    // The per-stripe lhi factor is read from shared memory when the table fits:
    // a global (L1) read there sits on the multiply's dependency chain.
    __shared__ uint4 sh_lhi[SMEM_LHI ? RC_SMEM_LHI : 1];
    if (SMEM_LHI) {
        for (uint32_t i = threadIdx.x; i < s_row; i += blockDim.x) sh_lhi[i] = lhi_g[i];
        __syncthreads();
    }
    const uint4* lhi = SMEM_LHI ? sh_lhi : lhi_g;
    const uint32_t lane = threadIdx.x & 31;
    const unsigned long long warp = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    unsigned long long s = warp * total / nwarps;
    const unsigned long long s_end = (warp + 1) * total / nwarps;
    if (s >= s_end) return;
    uint32_t row = (uint32_t)(s / s_row);
    uint32_t jh = (uint32_t)(s - (unsigned long long)row * s_row);
    unsigned long long acc[2][4];
#pragma unroll
    for (int e = 0; e < 2; e++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[e][c] = 0;
    uint32_t bad = 0;
    while (s < s_end) {
        unsigned long long left = s_end - s;
        uint32_t cnt = s_row - jh;
        if (left < cnt) cnt = (uint32_t)left;
        if (cnt > RC_UNROLL) cnt = RC_UNROLL;
        const size_t rbase = (size_t)row * n;
        if (VEC && cnt == RC_UNROLL && (jh + RC_UNROLL) * 64u <= n) {
            // Fast path: RC_UNROLL full stripes of this row, no per-stripe predicates.
            const uint2* base = reinterpret_cast<const uint2*>(B + rbase + jh * 64u + 2u * lane);
            uint2 v[RC_UNROLL];
#pragma unroll
            for (int u = 0; u < RC_UNROLL; u++) v[u] = __ldcs(base + 32 * u);
#pragma unroll
            for (int u = 0; u < RC_UNROLL; u++) {
                const uint4 lh = lhi[jh + u];
                bad |= v[u].x | v[u].y;
                acc[0][0] += (unsigned long long)v[u].x * lh.x;
                acc[0][1] += (unsigned long long)v[u].x * lh.y;
                acc[0][2] += (unsigned long long)v[u].x * lh.z;
                acc[0][3] += (unsigned long long)v[u].x * lh.w;
                acc[1][0] += (unsigned long long)v[u].y * lh.x;
                acc[1][1] += (unsigned long long)v[u].y * lh.y;
                acc[1][2] += (unsigned long long)v[u].y * lh.z;
                acc[1][3] += (unsigned long long)v[u].y * lh.w;
                if ((u & 3) == 3) {
#pragma unroll
                    for (int e = 0; e < 2; e++)
#pragma unroll
                        for (int c = 0; c < 4; c++) acc[e][c] = lazy(acc[e][c]);
                }
            }
        } else {
            uint2 v[RC_UNROLL];
#pragma unroll
            for (int u = 0; u < RC_UNROLL; u++) {
                v[u] = make_uint2(0, 0);
                const uint32_t col = (jh + u) * 64u + 2u * lane;
                if (u < (int)cnt) {
                    if (VEC) {
                        if (col < n) v[u] = __ldcs(reinterpret_cast<const uint2*>(B + rbase + col));
                    } else {
                        if (col < n) v[u].x = __ldcs(B + rbase + col);
                        if (col + 1 < n) v[u].y = __ldcs(B + rbase + col + 1);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < RC_UNROLL; u++) {
                if (u < (int)cnt) {
                    const uint4 lh = lhi[jh + u];
                    bad |= v[u].x | v[u].y;
                    acc[0][0] += (unsigned long long)v[u].x * lh.x;
                    acc[0][1] += (unsigned long long)v[u].x * lh.y;
                    acc[0][2] += (unsigned long long)v[u].x * lh.z;
                    acc[0][3] += (unsigned long long)v[u].x * lh.w;
                    acc[1][0] += (unsigned long long)v[u].y * lh.x;
                    acc[1][1] += (unsigned long long)v[u].y * lh.y;
                    acc[1][2] += (unsigned long long)v[u].y * lh.z;
                    acc[1][3] += (unsigned long long)v[u].y * lh.w;
                }
                if ((u & 3) == 3) {
#pragma unroll
                    for (int e = 0; e < 2; e++)
#pragma unroll
                        for (int c = 0; c < 4; c++) acc[e][c] = lazy(acc[e][c]);
                }
            }
        }
        s += cnt;
        jh += cnt;
        if (jh == s_row || s == s_end) {
            // Flush this warp's contribution to `row`.
            qm31 t = qzero();
#pragma unroll
            for (int e = 0; e < 2; e++) {
                qm31 q = qm(red64(acc[e][0]), red64(acc[e][1]), red64(acc[e][2]), red64(acc[e][3]));
                t = qadd(t, qmul(q, ld_q(llo + 2 * lane + e)));
#pragma unroll
                for (int c = 0; c < 4; c++) acc[e][c] = 0;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                qm31 o;
                o.a = __shfl_xor_sync(0xffffffffu, t.a, off);
                o.b = __shfl_xor_sync(0xffffffffu, t.b, off);
                o.c = __shfl_xor_sync(0xffffffffu, t.c, off);
                o.d = __shfl_xor_sync(0xffffffffu, t.d, off);
                t = qadd(t, o);
            }
            if (lane == 0) {
                atomicAdd(acc_out + 4 * (size_t)row + 0, (unsigned long long)t.a);
                atomicAdd(acc_out + 4 * (size_t)row + 1, (unsigned long long)t.b);
                atomicAdd(acc_out + 4 * (size_t)row + 2, (unsigned long long)t.c);
                atomicAdd(acc_out + 4 * (size_t)row + 3, (unsigned long long)t.d);
            }
            if (jh == s_row) {
                row++;
                jh = 0;
            }
        }
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

void launch_restrict_cols(const uint32_t* B, uint32_t k, uint32_t n, const uint4* lhi, const uint4* llo,
                          unsigned long long* acc, uint32_t* err, int num_sms, cudaStream_t s) {
    const uint32_t s_row = (n + 63) / 64;
    const unsigned long long total = (unsigned long long)k * s_row;
    const int threads = 256;
    // Persistent grid: 4 CTAs of 8 warps per SM, never more warps than stripes.
    unsigned long long blocks = (unsigned long long)num_sms * 4;
    const unsigned long long need = (total + 7) / 8;
    if (blocks > need) blocks = need;
    if (blocks == 0) blocks = 1;
    const bool vec = (n % 2 == 0) && ((reinterpret_cast<uintptr_t>(B) & 7) == 0);
    const bool sm = s_row <= RC_SMEM_LHI;
    if (vec && sm)
        restrict_cols_kernel<true, true><<<(unsigned)blocks, threads, 0, s>>>(B, k, n, s_row, total, lhi, llo, acc, err);
    else if (vec)
        restrict_cols_kernel<true, false><<<(unsigned)blocks, threads, 0, s>>>(B, k, n, s_row, total, lhi, llo, acc, err);
    else if (sm)
        restrict_cols_kernel<false, true><<<(unsigned)blocks, threads, 0, s>>>(B, k, n, s_row, total, lhi, llo, acc, err);
    else
        restrict_cols_kernel<false, false><<<(unsigned)blocks, threads, 0, s>>>(B, k, n, s_row, total, lhi, llo, acc, err);
}

// ---------------------------------------------------------------------------
// Row restriction f_a[j] = sum_i A[i][j] L_i.  A is small (m x k activations);
// each thread owns one column and a chunk of 16 rows, partials meet in
// 64-bit atomics.
// ---------------------------------------------------------------------------
__global__ void restrict_rows_kernel(const uint32_t* __restrict__ A, uint32_t m, uint32_t k,
                                     const uint4* __restrict__ L, unsigned long long* __restrict__ acc_out,
                                     uint32_t* __restrict__ err) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t i0 = blockIdx.y * 16;
    if (j >= k) return;
    unsigned long long acc[4] = {0, 0, 0, 0};
    uint32_t bad = 0;
    const uint32_t i1 = min(m, i0 + 16);
    for (uint32_t i = i0; i < i1; i++) {
        const uint32_t v = __ldg(A + (size_t)i * k + j);
        bad |= v;
        const uint4 l = __ldg(L + i);
        acc[0] += (unsigned long long)v * l.x;
        acc[1] += (unsigned long long)v * l.y;
        acc[2] += (unsigned long long)v * l.z;
        acc[3] += (unsigned long long)v * l.w;
        if (((i - i0) & 3) == 3)
            for (int c = 0; c < 4; c++) acc[c] = lazy(acc[c]);
    }
    for (int c = 0; c < 4; c++) atomicAdd(acc_out + 4 * (size_t)j + c, (unsigned long long)red64(acc[c]));
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

void launch_restrict_rows(const uint32_t* A, uint32_t m, uint32_t k, const uint4* L, unsigned long long* acc,
                          uint32_t* err, cudaStream_t s) {
    dim3 grid((k + 255) / 256, (m + 15) / 16);
    restrict_rows_kernel<<<grid, 256, 0, s>>>(A, m, k, L, acc, err);
}

__global__ void acc_finalize_kernel(const unsigned long long* __restrict__ acc, size_t n_rows,
                                    uint4* __restrict__ out, size_t out_len) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < out_len;
         i += (size_t)gridDim.x * blockDim.x) {
        uint4 r = make_uint4(0, 0, 0, 0);
        if (i < n_rows) {
            r.x = red64(acc[4 * i + 0]);
            r.y = red64(acc[4 * i + 1]);
            r.z = red64(acc[4 * i + 2]);
            r.w = red64(acc[4 * i + 3]);
        }
        out[i] = r;
    }
}

void launch_acc_finalize(const unsigned long long* acc, size_t n_rows, uint4* out, size_t out_len, cudaStream_t s) {
    size_t blocks = (out_len + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    if (blocks == 0) blocks = 1;
    acc_finalize_kernel<<<(unsigned)blocks, 256, 0, s>>>(acc, n_rows, out, out_len);
}

__global__ void canon_words_kernel(uint32_t* __restrict__ w, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        w[i] = red32(w[i]);
}

void launch_canon_words(uint32_t* w, size_t n, cudaStream_t s) {
    size_t blocks = (n + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    if (blocks == 0) blocks = 1;
    canon_words_kernel<<<(unsigned)blocks, 256, 0, s>>>(w, n);
}

__global__ void m31_to_qm31_kernel(const uint32_t* __restrict__ in, size_t n, uint4* __restrict__ out,
                                   size_t out_len, uint32_t* __restrict__ err) {
    uint32_t bad = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < out_len;
         i += (size_t)gridDim.x * blockDim.x) {
        uint32_t v = i < n ? in[i] : 0;
        bad |= v;
        out[i] = make_uint4(red32(v), 0, 0, 0);
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

void launch_m31_to_qm31(const uint32_t* in, size_t n, uint4* out, size_t out_len, uint32_t* err, cudaStream_t s) {
    size_t blocks = (out_len + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    if (blocks == 0) blocks = 1;
    m31_to_qm31_kernel<<<(unsigned)blocks, 256, 0, s>>>(in, n, out, out_len, err);
}

// ---------------------------------------------------------------------------
// Sumcheck rounds.  Each launch reduces (s0, s1, s2) over the grid: per-block
// partials go to global memory and the last block to finish (atomic ticket)
// sums them, so the host reads the round's 12 words after one launch.
// ---------------------------------------------------------------------------
struct Sums {
    unsigned long long v[12];
};

__device__ __forceinline__ void sums_add(Sums& s, const qm31& x0, const qm31& x1, const qm31& x2) {
    s.v[0] += x0.a; s.v[1] += x0.b; s.v[2] += x0.c; s.v[3] += x0.d;
    s.v[4] += x1.a; s.v[5] += x1.b; s.v[6] += x1.c; s.v[7] += x1.d;
    s.v[8] += x2.a; s.v[9] += x2.b; s.v[10] += x2.c; s.v[11] += x2.d;
}

// Publish `n` result words to mapped host memory: words first, then the
// sequence number with a system-scope release (called by one thread).
__device__ __forceinline__ void publish(uint32_t* sig, uint32_t seq, const uint32_t* words, int n) {
    volatile uint32_t* v = sig;
    for (int i = 0; i < n; i++) v[1 + i] = words[i];
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(sig), "r"(seq) : "memory");
}

// Block-reduce the 12 lazily accumulated words and finish the grid reduction.
__device__ void finish_sums(Sums& s, uint32_t* __restrict__ partials, unsigned int* __restrict__ ticket,
                            uint32_t* __restrict__ out, uint32_t* sig, uint32_t seq) {
    __shared__ uint32_t sh[32][12];
    __shared__ uint32_t res[12];
    __shared__ bool is_last;
    uint32_t r[12];
#pragma unroll
    for (int i = 0; i < 12; i++) {
        r[i] = red64(s.v[i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) r[i] = madd(r[i], __shfl_xor_sync(0xffffffffu, r[i], off));
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0)
        for (int i = 0; i < 12; i++) sh[warp][i] = r[i];
    __syncthreads();
    if (threadIdx.x < 12) {
        uint32_t acc = 0;
        for (int w = 0; w < nw; w++) acc = madd(acc, sh[w][threadIdx.x]);
        partials[blockIdx.x * 12 + threadIdx.x] = acc;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // Last block: 12 components x blocks partials.
    for (int i = warp; i < 12; i += nw) {
        unsigned long long acc = 0;
        for (unsigned b = lane; b < gridDim.x; b += 32) acc += __ldcg(partials + b * 12 + i);
        uint32_t v = red64(acc);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = madd(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) {
            out[i] = v;
            res[i] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *ticket = 0;
        if (sig) publish(sig, seq, res, 12);
    }
}

__device__ __forceinline__ void sums_zero(Sums& s) {
#pragma unroll
    for (int i = 0; i < 12; i++) s.v[i] = 0;
}

// The per-thread round accumulators as the 12 canonical words of finish_sums.
__device__ __forceinline__ void racc_to_sums(const RoundAcc& r, Sums& s) {
    const qm31 x0 = qacc_value(r.p0), x1 = qacc_value(r.p1), x2 = qacc_value(r.p2);
    sums_zero(s);
    sums_add(s, x0, x1, x2);
}

__global__ void __launch_bounds__(256) round_qm31_kernel(const uint4* __restrict__ A, const uint4* __restrict__ B,
                                                         size_t q, uint32_t* partials, unsigned int* ticket,
                                                         uint32_t* out, uint32_t* sig, uint32_t seq) {
    RoundAcc acc;
    racc_zero(acc);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x)
        racc_add(acc, ld_q(A + i), ld_q(A + i + q), ld_q(B + i), ld_q(B + i + q));
    Sums s;
    racc_to_sums(acc, s);
    finish_sums(s, partials, ticket, out, sig, seq);
}

// In-place fold with alpha fused with the next round's sums.  Thread i reads
// elements i, i+q, i+h, i+q+h (h = len/2, q = h/2) and writes i and i+q: every
// element is read by exactly one thread, so the in-place update is race-free.
// Inputs must be canonical (< P); outputs are canonical.
__global__ void __launch_bounds__(256) fold_round_qm31_kernel(uint4* __restrict__ A, uint4* __restrict__ B, size_t h,
                                                              qm31 alpha, uint32_t* partials, unsigned int* ticket,
                                                              uint32_t* out, uint32_t* sig, uint32_t seq) {
    const size_t q = h / 2;
    const AlphaRows m = alpha_rows(alpha);
    RoundAcc acc;
    racc_zero(acc);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        const qm31 a0 = ld_q(A + i), a1 = ld_q(A + i + q), a2 = ld_q(A + i + h), a3 = ld_q(A + i + q + h);
        const qm31 b0 = ld_q(B + i), b1 = ld_q(B + i + q), b2 = ld_q(B + i + h), b3 = ld_q(B + i + q + h);
        const qm31 alo = fold_qq(a0, a2, m), ahi = fold_qq(a1, a3, m);
        const qm31 blo = fold_qq(b0, b2, m), bhi = fold_qq(b1, b3, m);
        st_q(A + i, alo);
        st_q(A + i + q, ahi);
        st_q(B + i, blo);
        st_q(B + i + q, bhi);
        racc_add(acc, alo, ahi, blo, bhi);
    }
    Sums s;
    racc_to_sums(acc, s);
    finish_sums(s, partials, ticket, out, sig, seq);
}

// Base-field round: products of M31 values accumulate lazily (acc_fold).  Any
// input word with bit 31 set is not an M31 element and raises the error flag.
__global__ void __launch_bounds__(256) round_m31_kernel(const uint32_t* __restrict__ A, const uint32_t* __restrict__ B,
                                                        size_t q, uint32_t* partials, unsigned int* ticket,
                                                        uint32_t* out, uint32_t* err, uint32_t* sig, uint32_t seq) {
    uint64_t s0 = 0, s1 = 0, s2 = 0;
    uint32_t bad = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t alo = __ldcs(A + i), ahi = __ldcs(A + i + q), blo = __ldcs(B + i), bhi = __ldcs(B + i + q);
        bad |= alo | ahi | blo | bhi;
        s0 = acc_fold(s0, mul_wide(alo, blo));
        s1 = acc_fold(s1, mul_wide(ahi, bhi));
        s2 = acc_fold(s2, mul_wide(csub(cdbl(ahi), alo), csub(cdbl(bhi), blo)));
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
    Sums s;
    sums_zero(s);
    s.v[0] = canon64(s0);
    s.v[4] = canon64(s1);
    s.v[8] = canon64(s2);
    finish_sums(s, partials, ticket, out, sig, seq);
}

// lo + alpha (hi - lo) with lo, hi in M31.
__device__ __forceinline__ qm31 fold_m31(uint32_t lo, uint32_t hi, const qm31& alpha) {
    return fold_mq(red32(lo), red32(hi), alpha);
}

__global__ void __launch_bounds__(256) fold_round_m31_kernel(const uint32_t* __restrict__ A,
                                                             const uint32_t* __restrict__ B, size_t h, qm31 alpha,
                                                             uint4* __restrict__ Ao, uint4* __restrict__ Bo,
                                                             uint32_t* partials, unsigned int* ticket, uint32_t* out,
                                                             uint32_t* sig, uint32_t seq) {
    const size_t q = h / 2;
    RoundAcc acc;
    racc_zero(acc);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x) {
        const qm31 alo = fold_mq(A[i], A[i + h], alpha), ahi = fold_mq(A[i + q], A[i + q + h], alpha);
        const qm31 blo = fold_mq(B[i], B[i + h], alpha), bhi = fold_mq(B[i + q], B[i + q + h], alpha);
        st_q(Ao + i, alo);
        st_q(Ao + i + q, ahi);
        st_q(Bo + i, blo);
        st_q(Bo + i + q, bhi);
        racc_add(acc, alo, ahi, blo, bhi);
    }
    Sums s;
    racc_to_sums(acc, s);
    finish_sums(s, partials, ticket, out, sig, seq);
}

static unsigned round_blocks(size_t work, int max_blocks) {
    size_t b = (work + 255) / 256;
    if (b > (size_t)max_blocks) b = max_blocks;
    if (b == 0) b = 1;
    return (unsigned)b;
}

void launch_round_qm31(uint4* A, uint4* B, size_t len, const RoundScratch& rs, cudaStream_t s) {
    const size_t q = len / 2;
    round_qm31_kernel<<<round_blocks(q, rs.max_blocks), 256, 0, s>>>(A, B, q, rs.partials, rs.ticket, rs.out, rs.sig,
                                                                                  rs.seq);
}

void launch_fold_round_qm31(uint4* A, uint4* B, size_t len, qm31 alpha, const RoundScratch& rs, cudaStream_t s) {
    const size_t h = len / 2;
    fold_round_qm31_kernel<<<round_blocks(h / 2, rs.max_blocks), 256, 0, s>>>(A, B, h, alpha, rs.partials,
                                                                                rs.ticket, rs.out, rs.sig, rs.seq);
}

void launch_round_m31(const uint32_t* A, const uint32_t* B, size_t len, const RoundScratch& rs, uint32_t* err,
                      cudaStream_t s) {
    const size_t q = len / 2;
    round_m31_kernel<<<round_blocks(q, rs.max_blocks), 256, 0, s>>>(A, B, q, rs.partials, rs.ticket, rs.out, err,
                                                                                 rs.sig, rs.seq);
}

void launch_fold_round_m31(const uint32_t* A, const uint32_t* B, size_t len, qm31 alpha, uint4* Ao, uint4* Bo,
                           const RoundScratch& rs, cudaStream_t s) {
    const size_t h = len / 2;
    fold_round_m31_kernel<<<round_blocks(h / 2, rs.max_blocks), 256, 0, s>>>(A, B, h, alpha, Ao, Bo, rs.partials,
                                                                               rs.ticket, rs.out, rs.sig, rs.seq);
}

__global__ void final_fold_kernel(const uint4* A, const uint4* B, const uint32_t* A32, const uint32_t* B32,
                                  qm31 alpha, uint32_t* out, uint32_t* sig, uint32_t seq) {
    if (threadIdx.x != 0) return;
    qm31 a, b;
    if (A32) {
        a = fold_m31(red32(A32[0]), red32(A32[1]), alpha);
        b = fold_m31(red32(B32[0]), red32(B32[1]), alpha);
    } else {
        qm31 a0 = ld_q(A), a1 = ld_q(A + 1), b0 = ld_q(B), b1 = ld_q(B + 1);
        a = qadd(a0, qmul(alpha, qsub(a1, a0)));
        b = qadd(b0, qmul(alpha, qsub(b1, b0)));
    }
    const uint32_t w[8] = {a.a, a.b, a.c, a.d, b.a, b.b, b.c, b.d};
    for (int i = 0; i < 8; i++) out[i] = w[i];
    if (sig) publish(sig, seq, w, 8);
}

void launch_final_fold(const uint4* A, const uint4* B, const uint32_t* A32, const uint32_t* B32, size_t len,
                       qm31 alpha, uint32_t* out, uint32_t* sig, uint32_t seq, cudaStream_t s) {
    (void)len;
    final_fold_kernel<<<1, 32, 0, s>>>(A, B, A32, B32, alpha, out, sig, seq);
}

// ---------------------------------------------------------------------------
// Persistent cooperative round loop (see kernels.cuh).
// ---------------------------------------------------------------------------
constexpr unsigned long long kSpinLimit = 1ull << 25;  // ~ seconds with the back-off below

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded grid barrier among the co-resident blocks of one cooperative launch.
__device__ bool grid_barrier(unsigned int* bar, uint32_t* status) {
    __shared__ bool ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        ok = true;
        volatile unsigned int* gen = bar + 1;
        const unsigned int my_gen = *gen;
        __threadfence();
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            unsigned long long it = 0;
            while (*gen == my_gen) {
                if (++it > kSpinLimit) {
                    atomicOr(status, 1u);
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
    }
    __syncthreads();
    return ok;
}

__global__ void __launch_bounds__(256) sumcheck_persistent_kernel(PersistArgs p) {
    __shared__ uint32_t sh[32][12];
    __shared__ uint32_t res[12];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, nthreads = (size_t)gridDim.x * blockDim.x;
    uint4* A = p.A;
    uint4* B = p.B;
    size_t len = p.len;
    qm31 alpha = qzero();
    for (int r = 0; r <= p.log_k; r++) {
        if (r == p.log_k) {
            // final fold of the length-2 vectors by block 0
            if (blockIdx.x == 0 && threadIdx.x == 0) {
                qm31 a, b;
                if (p.A32 && r == 1) {
                    a = fold_m31(red32(p.A32[0]), red32(p.A32[1]), alpha);
                    b = fold_m31(red32(p.B32[0]), red32(p.B32[1]), alpha);
                } else {
                    const qm31 a0 = ld_q(A), a1 = ld_q(A + 1), b0 = ld_q(B), b1 = ld_q(B + 1);
                    a = qadd(a0, qmul(alpha, qsub(a1, a0)));
                    b = qadd(b0, qmul(alpha, qsub(b1, b0)));
                }
                const uint32_t w[8] = {a.a, a.b, a.c, a.d, b.a, b.b, b.c, b.d};
                publish(p.sig, p.seq_base + r, w, 8);
            }
            return;
        }
        Sums s;
        sums_zero(s);
        RoundAcc racc;
        racc_zero(racc);
        if (r == 0) {
            const size_t q = len / 2;
            if (p.A32) {
                uint64_t s0 = 0, s1 = 0, s2 = 0;
                for (size_t i = tid; i < q; i += nthreads) {
                    const uint32_t alo = red32(p.A32[i]), ahi = red32(p.A32[i + q]);
                    const uint32_t blo = red32(p.B32[i]), bhi = red32(p.B32[i + q]);
                    s0 = acc_fold(s0, mul_wide(alo, blo));
                    s1 = acc_fold(s1, mul_wide(ahi, bhi));
                    s2 = acc_fold(s2, mul_wide(csub(cdbl(ahi), alo), csub(cdbl(bhi), blo)));
                }
                s.v[0] = canon64(s0);
                s.v[4] = canon64(s1);
                s.v[8] = canon64(s2);
            } else {
                for (size_t i = tid; i < q; i += nthreads)
                    racc_add(racc, ld_q(A + i), ld_q(A + i + q), ld_q(B + i), ld_q(B + i + q));
                racc_to_sums(racc, s);
            }
        } else {
            // fold (len -> len / 2) fused with this round's sums
            const size_t h = len / 2, q = h / 2;
            const bool from_m31 = p.A32 && r == 1;
            const AlphaRows m = alpha_rows(alpha);
            for (size_t i = tid; i < q; i += nthreads) {
                qm31 alo, ahi, blo, bhi;
                if (from_m31) {
                    alo = fold_m31(red32(p.A32[i]), red32(p.A32[i + h]), alpha);
                    ahi = fold_m31(red32(p.A32[i + q]), red32(p.A32[i + q + h]), alpha);
                    blo = fold_m31(red32(p.B32[i]), red32(p.B32[i + h]), alpha);
                    bhi = fold_m31(red32(p.B32[i + q]), red32(p.B32[i + q + h]), alpha);
                } else {
                    const qm31 a0 = ld_q(A + i), a1 = ld_q(A + i + q), a2 = ld_q(A + i + h), a3 = ld_q(A + i + q + h);
                    const qm31 b0 = ld_q(B + i), b1 = ld_q(B + i + q), b2 = ld_q(B + i + h), b3 = ld_q(B + i + q + h);
                    alo = fold_qq(a0, a2, m);
                    ahi = fold_qq(a1, a3, m);
                    blo = fold_qq(b0, b2, m);
                    bhi = fold_qq(b1, b3, m);
                }
                st_q(A + i, alo);
                st_q(A + i + q, ahi);
                st_q(B + i, blo);
                st_q(B + i + q, bhi);
                racc_add(racc, alo, ahi, blo, bhi);
            }
            racc_to_sums(racc, s);
            len = h;
        }
        // block partials
#pragma unroll
        for (int i = 0; i < 12; i++) {
            uint32_t v = red64(s.v[i]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v = madd(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0) sh[warp][i] = v;
        }
        __syncthreads();
        if (threadIdx.x < 12) {
            uint32_t acc = 0;
            for (int w = 0; w < nw; w++) acc = madd(acc, sh[w][threadIdx.x]);
            p.partials[blockIdx.x * 12 + threadIdx.x] = acc;
        }
        if (!grid_barrier(p.bar, p.status)) return;
        if (blockIdx.x == 0) {
            for (int i = warp; i < 12; i += nw) {
                unsigned long long acc = 0;
                for (unsigned b = lane; b < gridDim.x; b += 32) acc += __ldcg(p.partials + b * 12 + i);
                uint32_t v = red64(acc);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v = madd(v, __shfl_xor_sync(0xffffffffu, v, off));
                if (lane == 0) res[i] = v;
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                publish(p.sig, p.seq_base + r, res, 12);
                // wait for the host's challenge for this round
                const uint32_t want = p.seq_base + r;
                unsigned long long it = 0;
                bool got = false;
                volatile const uint32_t* hm = p.hostmsg;
                while (!got) {
                    if (ld_acquire_sys(p.hostmsg) == want || hm[5] != 0) {
                        got = true;
                        break;
                    }
                    if (++it > kSpinLimit) break;
                    __nanosleep(128);
                }
                const bool abort = !got || hm[5] != 0;
                if (abort) atomicOr(p.status, 2u);
                *p.alpha_dev = make_uint4(hm[1], hm[2], hm[3], hm[4]);
                __threadfence();
            }
        }
        if (!grid_barrier(p.bar, p.status)) return;
        if (*((volatile uint32_t*)p.status) & 2u) return;
        const uint4 av = __ldcg(p.alpha_dev);
        alpha = qm(av.x, av.y, av.z, av.w);
    }
}

int launch_sumcheck_persistent(const PersistArgs& a, int num_sms, cudaStream_t s, cudaError_t* err) {
    int per_sm = 0;
    *err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sumcheck_persistent_kernel, 256, 0);
    if (*err != cudaSuccess || per_sm <= 0) return 0;
    size_t want = (a.len / 2 + 255) / 256;
    size_t cap = (size_t)per_sm * num_sms;
    if (cap > (size_t)num_sms * 4) cap = (size_t)num_sms * 4;
    if (want > cap) want = cap;
    if (want == 0) want = 1;
    PersistArgs args = a;
    void* params[] = {&args};
    *err = cudaLaunchCooperativeKernel((const void*)sumcheck_persistent_kernel, dim3((unsigned)want), dim3(256),
                                       params, 0, s);
    return *err == cudaSuccess ? (int)want : 0;
}

__global__ void mle_fold_kernel(const uint4* src, uint4* dst, size_t h, qm31 r) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < h; i += (size_t)gridDim.x * blockDim.x) {
        qm31 lo = ld_q(src + i), hi = ld_q(src + i + h);
        st_q(dst + i, qadd(lo, qmul(r, qsub(hi, lo))));
    }
}

void launch_mle_fold(const uint4* src, uint4* dst, size_t h, qm31 r, cudaStream_t s) {
    size_t blocks = (h + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    if (blocks == 0) blocks = 1;
    mle_fold_kernel<<<(unsigned)blocks, 256, 0, s>>>(src, dst, h, r);
}

}  // namespace zk

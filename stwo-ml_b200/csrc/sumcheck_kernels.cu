// sm_100a kernels for the GKR matmul sumcheck: eq tables, the W.eq(r)
// restrictions, and the degree-2 round reductions with fused in-place folds.
//
// All arithmetic is M31/QM31 integer work (no tensor cores).  The restriction
// is HBM-bound: it streams the weight matrix once with 16-byte loads and keeps
// 4 x 4 64-bit accumulators per thread, reducing modulo 2^31 - 1 only every
// four products (each product < 2^62, so four of them plus a reduced residue
// still fit in 64 bits).
#include <cstdio>
#include "kernels.cuh"
#include "round_arith.cuh"
#include "imma.cuh"

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
// eq(idx, c) = prod_l (bit_l ? c_l : 1 - c_l), variable l on bit v - 1 - l (MSB first).
// The product is split at k = min(v, 10) low bits: a block builds the 2^k-entry
// table of the low variables in shared memory once (by doubling, one product per
// entry; the product order only regroups field multiplications), then for each high prefix
// h (one QM31 product chain of v - k factors, by one thread) writes the 2^k
// entries h * 2^k + t as one product each.  Entries in [2^v, len) are zero.
constexpr int EQ_LO_MAX = 10;
constexpr int EQ_HI_BATCH = 8;

__global__ void __launch_bounds__(256) eq_table_kernel(EqChallenges ch, uint4* __restrict__ table, size_t len) {
    __shared__ uint4 buf[2][1 << EQ_LO_MAX];
    const int v = ch.v, k = v < EQ_LO_MAX ? v : EQ_LO_MAX;
    const size_t n = (size_t)1 << v, nlo = (size_t)1 << k, nh = n >> k;
    // low table by doubling, most significant low variable first: one product per entry
    if (threadIdx.x == 0) st_q(&buf[0][0], qone());
    int cur = 0;
    for (int j = 0; j < k; j++) {
        __syncthreads();
        const qm31 c = ch.c[v - k + j], c1 = qsub(qone(), c);
        const size_t sz = (size_t)1 << j;
        for (size_t e = threadIdx.x; e < sz; e += blockDim.x) {
            const qm31 w = ld_q(&buf[cur][e]);
            st_q(&buf[cur ^ 1][2 * e], qmul(w, c1));
            st_q(&buf[cur ^ 1][2 * e + 1], qmul(w, c));
        }
        cur ^= 1;
    }
    const uint4* lo = buf[cur];
    // high prefixes in batches of EQ_HI_BATCH, one thread per prefix
    __shared__ uint4 hs[EQ_HI_BATCH];
    for (size_t hb = blockIdx.x * (size_t)EQ_HI_BATCH; hb < nh; hb += (size_t)gridDim.x * EQ_HI_BATCH) {
        __syncthreads();
        if (threadIdx.x < EQ_HI_BATCH && hb + threadIdx.x < nh) {
            const size_t h = hb + threadIdx.x;
            qm31 w = qone();
            for (int l = 0; l < v - k; l++) {
                const int bit = (int)((h >> (v - k - 1 - l)) & 1);
                w = qmul(w, bit ? ch.c[l] : qsub(qone(), ch.c[l]));
            }
            st_q(&hs[threadIdx.x], w);
        }
        __syncthreads();
        const size_t nb = nh - hb < (size_t)EQ_HI_BATCH ? nh - hb : (size_t)EQ_HI_BATCH;
        for (size_t u = threadIdx.x; u < nb * nlo; u += blockDim.x) {
            const size_t hh = u / nlo, t = u % nlo, idx = (hb + hh) * nlo + t;
            if (idx < len) st_q(table + idx, qmul(ld_q(&hs[hh]), ld_q(lo + t)));
        }
    }
    for (size_t idx = n + blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < len;
         idx += (size_t)gridDim.x * blockDim.x)
        st_q(table + idx, qzero());
}

void launch_eq_table(const qm31* c, int v, uint4* table, size_t table_len, cudaStream_t s) {
    EqChallenges ch;
    ch.v = v;
    for (int i = 0; i < v; i++) ch.c[i] = c[i];
    const int k = v < EQ_LO_MAX ? v : EQ_LO_MAX;
    size_t blocks = ((((size_t)1 << v) >> k) + EQ_HI_BATCH - 1) / EQ_HI_BATCH;  // batches of high prefixes
    if (table_len > ((size_t)1 << v)) {
        const size_t tail = (table_len - ((size_t)1 << v) + 255) / 256;
        if (tail > blocks) blocks = tail;
    }
    if (blocks > 2048) blocks = 2048;
    if (blocks == 0) blocks = 1;
    eq_table_kernel<<<(unsigned)blocks, 256, 0, s>>>(ch, table, table_len);
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
// Column restriction on the tensor pipe (n % 4 == 0, 16-byte aligned B).
//
// f_b[i] = sum_j B[i][j] L_j is an exact integer GEMM of the k x n matrix B
// with the n x 4 matrix of eq components, reduced mod P.  Both sides are split
// into bytes: B[i][j] = sum_b 256^b B_b[i][j] and L_j^c = sum_l 256^l L_l^c[j],
// so f_b[i]^c = sum_{b,l} 256^(b+l) (B_b L_l^c)[i] with every partial product
// an exact u8 x u8 -> s32 MMA (a block chunk has 1024 columns, so a partial is
// at most 1024 * 255^2 < 2^31).  A warp takes 16 rows at a time; each 16 x 32
// tile of B arrives as four 16-byte loads per thread whose byte planes (three
// PRMTs per plane register) are exactly the A fragments of mma.m16n8k32, with
// K running over consecutive columns.  The eq side is a 16 x chunk byte-plane
// table (row c * 4 + l) that each block computes for its chunk straight into
// shared memory.  Each warp's loads for the next 64 columns are in flight while
// it runs the MMAs of the current 64 (register double buffering).  Per 16 x 32 tile: 8 MMAs (4 byte planes x 2
// N-tiles of 8 (c, l) columns), ~1.5 PRMT per element, no 64-bit integer work:
// the kernel is left with the HBM stream.
// ---------------------------------------------------------------------------
// One eq-table entry: prod_l (bit_{v-1-l}(idx) ? c_l : 1 - c_l), first challenge on the MSB.
__device__ __forceinline__ qm31 eq_entry(const EqChallenges& ch, uint32_t idx) {
    qm31 r = qm(1, 0, 0, 0);
    for (int l = 0; l < ch.v; l++) {
        const qm31 c = ch.c[l];
        r = qmul(r, ((idx >> (ch.v - 1 - l)) & 1u) ? c : qsub(qm(1, 0, 0, 0), c));
    }
    return r;
}

constexpr int TC_CH = 1024;                 // columns per block chunk
constexpr int TC_TROW = TC_CH + 16;         // padded table row (bytes): conflict-free fragment loads
constexpr int TC_WARPS = 8;
constexpr int TC_MINB = 2;   // launch-bounds minimum blocks per SM
constexpr int TC_STEPS = 2;  // 32-column steps loaded per iteration (one iteration ahead of the MMAs)

template <int MINB, int STEPS>
__global__ void __launch_bounds__(TC_WARPS * 32, MINB) restrict_cols_tc_kernel(const uint32_t* __restrict__ B, uint32_t k,
                                                                         uint32_t n, const EqChallenges hi,
                                                                         const EqChallenges lo, uint32_t hi_base,
                                                                         uint32_t npad,
                                                                         unsigned long long* __restrict__ acc_out,
                                                                         uint32_t* __restrict__ err) {
    __shared__ __align__(16) uint8_t tb[16 * TC_TROW];
    __shared__ qm31 s_hi[TC_CH / 64], s_lo[64];
    const uint32_t c0 = blockIdx.x * TC_CH;
    const uint32_t cw = min((uint32_t)TC_CH, npad - c0);  // chunk width (multiple of 32)
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tg = lane & 3;
    const uint32_t row_tiles = (k + 15) / 16;
    const uint32_t c_end = min(n, c0 + cw);
    const uint32_t rt0 = blockIdx.y * TC_WARPS + warp;
    // the first row tile's first loads go out before the eq weights are formed
    uint4 xn[STEPS][4];
    {
        const uint32_t r0 = rt0 * 16 + g, r1 = r0 + 8;
        const bool v0 = rt0 < row_tiles && r0 < k, v1 = rt0 < row_tiles && r1 < k;
        const uint4* p0 = reinterpret_cast<const uint4*>(B + (size_t)(v0 ? r0 : 0) * n);
        const uint4* p1 = reinterpret_cast<const uint4*>(B + (size_t)(v1 ? r1 : 0) * n);
#pragma unroll
        for (int h = 0; h < STEPS; h++) {
            const uint32_t ja = c0 + 32 * h + 4 * tg, jb = ja + 16;
            const uint4 z = make_uint4(0, 0, 0, 0);
            xn[h][0] = (v0 && ja < c_end) ? __ldcs(p0 + ja / 4) : z;
            xn[h][1] = (v1 && ja < c_end) ? __ldcs(p1 + ja / 4) : z;
            xn[h][2] = (v0 && jb < c_end) ? __ldcs(p0 + jb / 4) : z;
            xn[h][3] = (v1 && jb < c_end) ? __ldcs(p1 + jb / 4) : z;
        }
    }
    // eq(r_j, j) = lhi[j / 64] * llo[j % 64]: the chunk's 16 high factors (stripe hi_base + j / 64 of
    // the high challenges) and the 64 low ones (zero past 2^lo.v), straight from the challenges
    if (threadIdx.x < 64) {
        const uint32_t u = threadIdx.x;
        s_lo[u] = u < (1u << lo.v) ? eq_entry(lo, u) : qzero();
    } else if (threadIdx.x < 64 + TC_CH / 64) {
        s_hi[threadIdx.x - 64] = eq_entry(hi, hi_base + (c0 >> 6) + (threadIdx.x - 64));
    }
    __syncthreads();
    // the chunk's eq byte planes: row c * 4 + l holds byte l of component c of L_j (zero past
    // n), four columns per thread and row word
    for (uint32_t j4 = threadIdx.x; j4 < cw / 4; j4 += blockDim.x) {
        uint32_t w[4][4];  // [column][component]
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t col = c0 + 4 * j4 + u;
            qm31 L = qzero();
            if (col < n) L = qmul(s_hi[(col - c0) >> 6], s_lo[col & 63]);
            w[u][0] = L.a;
            w[u][1] = L.b;
            w[u][2] = L.c;
            w[u][3] = L.d;
        }
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
            for (int l = 0; l < 4; l++) {
                uint32_t v = 0;
#pragma unroll
                for (int u = 0; u < 4; u++) v |= ((w[u][c] >> (8 * l)) & 0xFFu) << (8 * u);
                *reinterpret_cast<uint32_t*>(tb + (c * 4 + l) * TC_TROW + 4 * j4) = v;
            }
    }
    __syncthreads();
    uint32_t bad = 0;
    for (uint32_t rt = rt0; rt < row_tiles; rt += gridDim.y * TC_WARPS) {
        const uint32_t r0 = rt * 16 + g, r1 = r0 + 8;
        const bool v0 = r0 < k, v1 = r1 < k;
        const uint4* p0 = reinterpret_cast<const uint4*>(B + (size_t)(v0 ? r0 : 0) * n);
        const uint4* p1 = reinterpret_cast<const uint4*>(B + (size_t)(v1 ? r1 : 0) * n);
        int acc[4][2][4];
#pragma unroll
        for (int b = 0; b < 4; b++)
#pragma unroll
            for (int t = 0; t < 2; t++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[b][t][e] = 0;
        // STEPS 32-column steps per iteration: all their 16-byte loads issue before any MMA,
        // and the next iteration's loads are issued before this iteration's MMAs
        auto load = [&](uint4 (&x)[STEPS][4], uint32_t j0) {
#pragma unroll
            for (int h = 0; h < STEPS; h++) {
                const uint32_t ja = j0 + 32 * h + 4 * tg, jb = ja + 16;
                const uint4 z = make_uint4(0, 0, 0, 0);
                x[h][0] = (v0 && ja < c_end) ? __ldcs(p0 + ja / 4) : z;
                x[h][1] = (v1 && ja < c_end) ? __ldcs(p1 + ja / 4) : z;
                x[h][2] = (v0 && jb < c_end) ? __ldcs(p0 + jb / 4) : z;
                x[h][3] = (v1 && jb < c_end) ? __ldcs(p1 + jb / 4) : z;
            }
        };
        if (rt != rt0) load(xn, c0);
        for (uint32_t j0 = c0; j0 < c_end; j0 += 32 * STEPS) {
            uint4 x[STEPS][4];
#pragma unroll
            for (int h = 0; h < STEPS; h++)
#pragma unroll
                for (int f = 0; f < 4; f++) x[h][f] = xn[h][f];
            load(xn, j0 + 32 * STEPS);  // past c_end: zeros, no loads
#pragma unroll
            for (int h = 0; h < STEPS; h++) {
                const uint32_t jj = j0 + 32 * h - c0;
                if (jj >= cw) break;
                uint32_t a[4][4];  // [plane][fragment register]
#pragma unroll
                for (int f = 0; f < 4; f++) {
                    bad |= x[h][f].x | x[h][f].y | x[h][f].z | x[h][f].w;
                    byte_planes(x[h][f], a[0][f], a[1][f], a[2][f], a[3][f]);
                }
#pragma unroll
                for (int t = 0; t < 2; t++) {
                    const uint8_t* trow = tb + (8 * t + g) * TC_TROW + jj + 4 * tg;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(trow);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(trow + 16);
#pragma unroll
                    for (int b = 0; b < 4; b++) mma_u8(acc[b][t], a[b], b0, b1);
                }
            }
        }
        // acc[b][t][e]: rows (g, g, g+8, g+8), columns 8t + 2tg + (e & 1) = (c, l) with
        // c = 2t + (tg >> 1), l = 2 (tg & 1) + (e & 1).  Combine the byte weights, then add the
        // partner lane's (other two l) and let the even lane post one atomic per (row, c).
#pragma unroll
        for (int t = 0; t < 2; t++) {
#pragma unroll
            for (int hr = 0; hr < 2; hr++) {
                uint64_t sum = 0;
#pragma unroll
                for (int b = 0; b < 4; b++)
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int l = 2 * (tg & 1) + e;
                        sum = acc_fold(sum, mul_wide((uint32_t)acc[b][t][2 * hr + e], pow256(b + l)));
                    }
                uint32_t v = canon64(sum);
                v = madd(v, __shfl_xor_sync(0xffffffffu, v, 1));
                const uint32_t row = hr ? r1 : r0;
                if ((tg & 1) == 0 && row < k) atomicAdd(acc_out + 4 * (size_t)row + 2 * t + (tg >> 1), (unsigned long long)v);
            }
        }
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
}

bool restrict_cols_tc_ok(const uint32_t* B, uint32_t n) {
    return n % 4 == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0;
}

void launch_restrict_cols_tc(const uint32_t* B, uint32_t k, uint32_t n, const qm31* r_j, unsigned hi_vars,
                             unsigned lo_vars, uint32_t hi_base, unsigned long long* acc, uint32_t* err, int num_sms,
                             cudaStream_t s) {
    EqChallenges hi, lo;
    hi.v = (int)hi_vars;
    lo.v = (int)lo_vars;
    for (unsigned i = 0; i < hi_vars; i++) hi.c[i] = r_j[i];
    for (unsigned i = 0; i < lo_vars; i++) lo.c[i] = r_j[hi_vars + i];
    const uint32_t npad = (n + 31) / 32 * 32;
    const uint32_t chunks = (npad + TC_CH - 1) / TC_CH;
    const uint32_t row_tiles = (k + 15) / 16;
    // one wave of TC_MINB resident 8-warp blocks per SM
    uint32_t gy = (uint32_t)((num_sms * TC_MINB + chunks - 1) / chunks);
    const uint32_t gy_max = (row_tiles + TC_WARPS - 1) / TC_WARPS;
    if (gy > gy_max) gy = gy_max;
    if (gy == 0) gy = 1;
    restrict_cols_tc_kernel<TC_MINB, TC_STEPS><<<dim3(chunks, gy), TC_WARPS * 32, 0, s>>>(B, k, n, hi, lo,
                                                                                          hi_base, npad, acc, err);
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

// Row restriction and both finalisations in one launch, for m <= 2^RF_MAX_VARS rows:
// f_a[j] = sum_i A[i][j] eq(i, r_i) written directly as QM31 (each block builds the
// eq table of the row variables in shared memory, its 8 warps take 1/8 of the rows
// of its 32 columns each and add their partials), zeros for k <= j < pk; and,
// when acc_b is set, f_b[i] = acc_b[i] mod P for i < k_b, zeros up to pk.  Replaces
// eq_table + memset + restrict_rows + two acc_finalize launches between the column
// restriction and the first round kernel.
constexpr int RF_MAX_VARS = 8;
constexpr int RF_COLS = 32;

__global__ void __launch_bounds__(256) restrict_rows_fused_kernel(const uint32_t* __restrict__ A, uint32_t m,
                                                                  uint32_t k, EqChallenges ch,
                                                                  const unsigned long long* __restrict__ acc_b,
                                                                  size_t k_b, uint4* __restrict__ fa,
                                                                  uint4* __restrict__ fb, size_t pk,
                                                                  uint32_t* __restrict__ err) {
    __shared__ uint4 eq[2][1 << RF_MAX_VARS];
    __shared__ uint32_t part[8][4][RF_COLS];
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    // f_b first (independent of the table)
    if (acc_b)
        for (size_t i = blockIdx.x * (size_t)blockDim.x + t; i < pk; i += (size_t)gridDim.x * blockDim.x) {
            uint4 r = make_uint4(0, 0, 0, 0);
            if (i < k_b) {
                r.x = red64(acc_b[4 * i + 0]);
                r.y = red64(acc_b[4 * i + 1]);
                r.z = red64(acc_b[4 * i + 2]);
                r.w = red64(acc_b[4 * i + 3]);
            }
            fb[i] = r;
        }
    // eq table of the v row variables, most significant first, by doubling
    const int v = ch.v;
    if (t == 0) st_q(&eq[0][0], qone());
    int cur = 0;
    for (int l = 0; l < v; l++) {
        __syncthreads();
        const qm31 c = ch.c[l], c1 = qsub(qone(), c);
        for (int e = t; e < (1 << l); e += blockDim.x) {
            const qm31 w = ld_q(&eq[cur][e]);
            st_q(&eq[cur ^ 1][2 * e], qmul(w, c1));
            st_q(&eq[cur ^ 1][2 * e + 1], qmul(w, c));
        }
        cur ^= 1;
    }
    __syncthreads();
    const uint32_t j = blockIdx.x * RF_COLS + lane;
    const uint32_t per = (m + 7) / 8, i0 = warp * per, i1 = min(m, i0 + per);
    unsigned long long acc[4] = {0, 0, 0, 0};
    uint32_t bad = 0;
    if (j < k) {
#pragma unroll 4
        for (uint32_t i = i0; i < i1; i++) {
            const uint32_t a = __ldg(A + (size_t)i * k + j);
            bad |= a;
            const uint4 l = eq[cur][i];
            acc[0] += (unsigned long long)a * l.x;
            acc[1] += (unsigned long long)a * l.y;
            acc[2] += (unsigned long long)a * l.z;
            acc[3] += (unsigned long long)a * l.w;
            if (((i - i0) & 3) == 3)
                for (int c = 0; c < 4; c++) acc[c] = lazy(acc[c]);
        }
    }
    for (int c = 0; c < 4; c++) part[warp][c][lane] = red64(acc[c]);
    if (bad & 0x80000000u) atomicOr(err, 1u);
    __syncthreads();
    if (warp == 0 && j < pk) {
        uint32_t r[4];
        for (int c = 0; c < 4; c++) {
            uint32_t x = 0;
            for (int w = 0; w < 8; w++) x = madd(x, part[w][c][lane]);
            r[c] = x;
        }
        fa[j] = make_uint4(r[0], r[1], r[2], r[3]);
    }
}

int launch_restrict_rows_fused(const uint32_t* A, uint32_t m, uint32_t k, const qm31* r_i, int n_ri,
                               const unsigned long long* acc_b, size_t k_b, uint4* fa, uint4* fb, size_t pk,
                               uint32_t* err, cudaStream_t s) {
    if (n_ri < 1 || n_ri > RF_MAX_VARS || pk < k) return -1;
    EqChallenges ch;
    ch.v = n_ri;
    for (int i = 0; i < n_ri; i++) ch.c[i] = r_i[i];
    const size_t blocks = (pk + RF_COLS - 1) / RF_COLS;
    restrict_rows_fused_kernel<<<(unsigned)blocks, 256, 0, s>>>(A, m, k, ch, acc_b, k_b, fa, fb, pk, err);
    return 0;
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

__global__ void canon_u64_kernel(unsigned long long* __restrict__ w, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        w[i] = red64(w[i]);
}

void launch_canon_u64(unsigned long long* w, size_t n, cudaStream_t s) {
    size_t blocks = (n + 255) / 256;
    if (blocks > 8192) blocks = 8192;
    if (blocks == 0) blocks = 1;
    canon_u64_kernel<<<(unsigned)blocks, 256, 0, s>>>(w, n);
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
    // the release store orders the word stores before the sequence number
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(sig), "r"(seq) : "memory");
}

// Block-reduce the 12 lazily accumulated words and finish the grid reduction.
// With a peer mesh, the grid's result is summed over the ranks before it is stored.
__device__ void finish_sums(Sums& s, uint32_t* __restrict__ partials, unsigned int* __restrict__ ticket,
                            uint32_t* __restrict__ out, uint32_t* sig, uint32_t seq, MeshArg mesh = {nullptr, 0}) {
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
        if (lane == 0) res[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *ticket = 0;
        if (mesh.desc) mesh_allreduce12(res, mesh);
        for (int i = 0; i < 12; i++) out[i] = res[i];
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
                                                         uint32_t* out, uint32_t* sig, uint32_t seq, MeshArg mesh) {
    RoundAcc acc;
    racc_zero(acc);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < q; i += (size_t)gridDim.x * blockDim.x)
        racc_add(acc, ld_q(A + i), ld_q(A + i + q), ld_q(B + i), ld_q(B + i + q));
    Sums s;
    racc_to_sums(acc, s);
    finish_sums(s, partials, ticket, out, sig, seq, mesh);
}

// In-place fold with alpha fused with the next round's sums.  Thread i reads
// elements i, i+q, i+h, i+q+h (h = len/2, q = h/2) and writes i and i+q: every
// element is read by exactly one thread, so the in-place update is race-free.
// Inputs must be canonical (< P); outputs are canonical.  The next iteration's
// eight loads are issued before this iteration's arithmetic, so each warp keeps
// two iterations of HBM reads in flight; the challenge's 4 x 4 coefficient
// matrix is a kernel parameter (constant bank, no registers).
struct FoldLoads {
    uint4 a0, a1, a2, a3, b0, b1, b2, b3;
};

__device__ __forceinline__ void fold_loads(FoldLoads& v, const uint4* A, const uint4* B, size_t i, size_t q,
                                           size_t h) {
    v.a0 = A[i];
    v.a1 = A[i + q];
    v.a2 = A[i + h];
    v.a3 = A[i + q + h];
    v.b0 = B[i];
    v.b1 = B[i + q];
    v.b2 = B[i + h];
    v.b3 = B[i + q + h];
}

__device__ __forceinline__ qm31 u2q(const uint4& v) { return qm(v.x, v.y, v.z, v.w); }

__global__ void __launch_bounds__(256, 2) fold_round_qm31_kernel(uint4* __restrict__ A, uint4* __restrict__ B,
                                                                 size_t h, const AlphaRows m, uint32_t* partials,
                                                                 unsigned int* ticket, uint32_t* out, uint32_t* sig,
                                                                 uint32_t seq, MeshArg mesh) {
    const size_t q = h / 2, stride = (size_t)gridDim.x * blockDim.x;
    RoundAcc acc;
    racc_zero(acc);
    size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    FoldLoads cur;
    if (i < q) fold_loads(cur, A, B, i, q, h);
    while (i < q) {
        const size_t nx = i + stride;
        FoldLoads nxt;
        if (nx < q) fold_loads(nxt, A, B, nx, q, h);
        const qm31 alo = fold_qq(u2q(cur.a0), u2q(cur.a2), m), ahi = fold_qq(u2q(cur.a1), u2q(cur.a3), m);
        const qm31 blo = fold_qq(u2q(cur.b0), u2q(cur.b2), m), bhi = fold_qq(u2q(cur.b1), u2q(cur.b3), m);
        st_q(A + i, alo);
        st_q(A + i + q, ahi);
        st_q(B + i, blo);
        st_q(B + i + q, bhi);
        racc_add(acc, alo, ahi, blo, bhi);
        cur = nxt;
        i = nx;
    }
    Sums s;
    racc_to_sums(acc, s);
    finish_sums(s, partials, ticket, out, sig, seq, mesh);
}

// Base-field round: products of M31 values accumulate lazily (acc_fold).  Any
// input word with bit 31 set is not an M31 element and raises the error flag.
// VEC = 4 reads four consecutive indices per 16-byte load (q % 4 == 0, 16-byte
// aligned inputs); VEC = 1 is the general path.
template <int VEC>
__global__ void __launch_bounds__(256) round_m31_kernel(const uint32_t* __restrict__ A, const uint32_t* __restrict__ B,
                                                        size_t q, uint32_t* partials, unsigned int* ticket,
                                                        uint32_t* out, uint32_t* err, uint32_t* sig, uint32_t seq,
                                                        MeshArg mesh) {
    uint64_t s0 = 0, s1 = 0, s2 = 0;
    uint32_t bad = 0;
    const size_t nq = q / VEC;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nq; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t alo[VEC], ahi[VEC], blo[VEC], bhi[VEC];
        if constexpr (VEC == 4) {
            const uint4 x0 = __ldcs(reinterpret_cast<const uint4*>(A) + i);
            const uint4 x1 = __ldcs(reinterpret_cast<const uint4*>(A) + i + nq);
            const uint4 y0 = __ldcs(reinterpret_cast<const uint4*>(B) + i);
            const uint4 y1 = __ldcs(reinterpret_cast<const uint4*>(B) + i + nq);
            alo[0] = x0.x; alo[1] = x0.y; alo[2] = x0.z; alo[3] = x0.w;
            ahi[0] = x1.x; ahi[1] = x1.y; ahi[2] = x1.z; ahi[3] = x1.w;
            blo[0] = y0.x; blo[1] = y0.y; blo[2] = y0.z; blo[3] = y0.w;
            bhi[0] = y1.x; bhi[1] = y1.y; bhi[2] = y1.z; bhi[3] = y1.w;
        } else {
            alo[0] = __ldcs(A + i); ahi[0] = __ldcs(A + i + q); blo[0] = __ldcs(B + i); bhi[0] = __ldcs(B + i + q);
        }
#pragma unroll
        for (int e = 0; e < VEC; e++) {
            bad |= alo[e] | ahi[e] | blo[e] | bhi[e];
            s0 = acc_fold(s0, mul_wide(alo[e], blo[e]));
            s1 = acc_fold(s1, mul_wide(ahi[e], bhi[e]));
            s2 = acc_fold(s2, mul_wide(csub(cdbl(ahi[e]), alo[e]), csub(cdbl(bhi[e]), blo[e])));
        }
    }
    if (bad & 0x80000000u) atomicOr(err, 1u);
    Sums s;
    sums_zero(s);
    s.v[0] = canon64(s0);
    s.v[4] = canon64(s1);
    s.v[8] = canon64(s2);
    finish_sums(s, partials, ticket, out, sig, seq, mesh);
}

// lo + alpha (hi - lo) with lo, hi in M31.
__device__ __forceinline__ qm31 fold_m31(uint32_t lo, uint32_t hi, const qm31& alpha) {
    return fold_mq(red32(lo), red32(hi), alpha);
}


// First fold (M31 -> QM31) fused with the next round's sums.  A block works on
// tiles of FR_UNROLL x 256 consecutive indices: its thread t takes indices
// tile + t + 256 e (e < FR_UNROLL), so every load (4 bytes a thread) and every
// 16-byte store of a warp is one contiguous run, and all FR_UNROLL x 8 loads of
// a tile are issued before its arithmetic.
//
// The round sums need no QM31 product: every folded value is x0 + alpha x1 with
// base-field x0 (the low input) and x1 (high - low), so a product of two folded
// values is x0 y0 + alpha (x0 y1 + x1 y0) + alpha^2 x1 y1.  Each of the three sums
// (s0, s1 and s2, whose factors 2 hi - lo are again of that form) is kept as three
// lazily reduced base-field sums, and alpha, alpha^2 are applied once per thread.
constexpr int FR_UNROLL = 4;

struct BaseSums {  // [sum][x0 y0, x0 y1 + x1 y0, x1 y1]
    uint64_t v[3][3];
};

__device__ __forceinline__ void base_sums_add(BaseSums& s, int k, uint32_t x0, uint32_t x1, uint32_t y0,
                                              uint32_t y1) {
    s.v[k][0] = acc_fold(s.v[k][0], mul_wide(x0, y0));
    s.v[k][1] = acc_fold(s.v[k][1], mad_wide(x0, y1, mul_wide(x1, y0)));
    s.v[k][2] = acc_fold(s.v[k][2], mul_wide(x1, y1));
}

__global__ void __launch_bounds__(256) fold_round_m31_kernel(const uint32_t* __restrict__ A,
                                                             const uint32_t* __restrict__ B, size_t h, qm31 alpha,
                                                             uint4* __restrict__ Ao, uint4* __restrict__ Bo,
                                                             uint32_t* partials, unsigned int* ticket, uint32_t* out,
                                                             uint32_t* sig, uint32_t seq, MeshArg mesh) {
    const size_t q = h / 2;
    const size_t tile = (size_t)FR_UNROLL * blockDim.x;
    BaseSums bs;
#pragma unroll
    for (int k = 0; k < 3; k++)
#pragma unroll
        for (int j = 0; j < 3; j++) bs.v[k][j] = 0;
    for (size_t base = blockIdx.x * tile; base < q; base += (size_t)gridDim.x * tile) {
        uint32_t a0[FR_UNROLL], a1[FR_UNROLL], a2[FR_UNROLL], a3[FR_UNROLL];
        uint32_t b0[FR_UNROLL], b1[FR_UNROLL], b2[FR_UNROLL], b3[FR_UNROLL];
#pragma unroll
        for (int e = 0; e < FR_UNROLL; e++) {
            const size_t j = base + threadIdx.x + (size_t)e * blockDim.x;
            if (j < q) {
                a0[e] = __ldcs(A + j); a1[e] = __ldcs(A + j + q); a2[e] = __ldcs(A + j + h); a3[e] = __ldcs(A + j + q + h);
                b0[e] = __ldcs(B + j); b1[e] = __ldcs(B + j + q); b2[e] = __ldcs(B + j + h); b3[e] = __ldcs(B + j + q + h);
            }
        }
#pragma unroll
        for (int e = 0; e < FR_UNROLL; e++) {
            const size_t j = base + threadIdx.x + (size_t)e * blockDim.x;
            if (j < q) {
                // canonical base-field lows and differences (inputs <= P)
                const uint32_t la = red32(a0[e]), ha = red32(a1[e]), lb = red32(b0[e]), hb = red32(b1[e]);
                const uint32_t da = csub(red32(a2[e]), la), ea = csub(red32(a3[e]), ha);
                const uint32_t db = csub(red32(b2[e]), lb), eb = csub(red32(b3[e]), hb);
                st_q(Ao + j, fold_md(la, da, alpha));
                st_q(Ao + j + q, fold_md(ha, ea, alpha));
                st_q(Bo + j, fold_md(lb, db, alpha));
                st_q(Bo + j + q, fold_md(hb, eb, alpha));
                base_sums_add(bs, 0, la, da, lb, db);
                base_sums_add(bs, 1, ha, ea, hb, eb);
                base_sums_add(bs, 2, csub(cdbl(ha), la), csub(cdbl(ea), da), csub(cdbl(hb), lb), csub(cdbl(eb), db));
            }
        }
    }
    // s_k = S_k0 + alpha S_k1 + alpha^2 S_k2, once per thread
    const qm31 alpha2 = qmul(alpha, alpha);
    Sums s;
    sums_zero(s);
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const uint32_t c0 = canon64(bs.v[k][0]), c1 = canon64(bs.v[k][1]), c2 = canon64(bs.v[k][2]);
        const qm31 v = qadd(qadd(qm(c0, 0, 0, 0), qmul_m(alpha, c1)), qmul_m(alpha2, c2));
        s.v[4 * k] = v.a;
        s.v[4 * k + 1] = v.b;
        s.v[4 * k + 2] = v.c;
        s.v[4 * k + 3] = v.d;
    }
    finish_sums(s, partials, ticket, out, sig, seq, mesh);
}

// ---------------------------------------------------------------------------
// Look-ahead round (small vectors).  One launch folds V_{r-1} with the previous
// challenge into V_r (in place; skipped for the first round) and returns, besides
// round r's own sums, the round r+1 sums as quadratics in the challenge not yet
// drawn, so the host can evaluate them the moment it draws that challenge and
// the GPU work of a round runs while the host hashes the previous one.
//
// With L = |V_r|, h = L/2, q = L/4, d[j] = V[j+h] - V[j] and P[j] = A[j] B[j]:
//   round r:    s0 = sum_{j<h} P,  s1 = sum_{j>=h} P,  s2 = sum_{j<h} T[j]
//               (T[j] = (2A[j+h] - A[j])(2B[j+h] - B[j]));
//   round r+1:  s0(x) = Q0 + x (Q2 - Q0 - D0) + x^2 D0,
//               s1(x) = Q1 + x (Q3 - Q1 - D1) + x^2 D1,
//               s2(x) = U + x (UW - U - W) + x^2 W,
// where Qk = sum of P over the k-th quarter of V_r, D0/D1 = sum d_A d_B over the
// first/second quarter, and with u = 2V[j+q] - V[j], w = 2d[j+q] - d[j] (j < q):
// U = sum u_A u_B, W = sum w_A w_B, UW = sum (u_A + w_A)(u_B + w_B) (note
// u + w = 2V[j+q+h] - V[j+h]).  The kernel publishes the ten sums
// [Q0 Q1 Q2 Q3 T D0 D1 U W UW] (40 words).  For L = 2 (the last round) it
// publishes [P0 P1 T A0 A1 B0 B1] (28 words): the final values are then
// A0 + x (A1 - A0) and B0 + x (B1 - B0).
// ---------------------------------------------------------------------------
// The look-ahead kernel runs on small vectors, one launch per round, so its
// time is dominated by fetching its own instructions into a cold instruction
// cache, not by arithmetic.  It is therefore written for small code: the fold
// and the product are out-of-line device functions called in loops, and the
// 40 result words are reduced through shared memory by a rolled loop.
constexpr int LA_WORDS = 40;
// Words 40-41 of a last round's publication: the M31 input-error word and the
// look-ahead wait status, read after every earlier kernel of the stream ended.
constexpr int LA_FLAG_WORDS = 2;
constexpr int LA_THREADS = 256;
constexpr unsigned long long kLaSpinLimit = 1ull << 21;  // a few seconds with the back-off below

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Optional device timeline of the look-ahead kernels (ZKML_LAYER_TRACE=1): per
// signal sequence number (mod 64) the %globaltimer at kernel entry (0), when the
// challenge was seen (1), two intermediate points (3, 4: block 0 done and the
// last block's start; the tail's fold and products done), when the data were
// ready (5: the predecessor grid waited for, the tail's vectors loaded) and when
// the words were published (2).  Off by default: the
// kernels then read one flag word.
__device__ unsigned long long g_la_stamp[64][6];
__device__ int g_la_stamp_on;

__device__ __forceinline__ void la_stamp(uint32_t seq, int what) {
    if (*(volatile int*)&g_la_stamp_on) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        g_la_stamp[seq & 63][what] = t;
    }
}

void la_stamps_enable(bool on) {
    const int v = on ? 1 : 0;
    cudaMemcpyToSymbol(g_la_stamp_on, &v, sizeof(v));
    if (on) {
        static const unsigned long long zero[64][6] = {};
        cudaMemcpyToSymbol(g_la_stamp, zero, sizeof(zero));
    }
}

// Prints the stamps of sequence numbers [lo, hi] in microseconds from the first one.
void la_stamps_print(uint32_t lo, uint32_t hi) {
    unsigned long long st[64][6];
    if (cudaMemcpyFromSymbol(st, g_la_stamp, sizeof(st)) != cudaSuccess) return;
    unsigned long long t0 = ~0ull;
    for (uint32_t q = lo; q <= hi && q - lo < 64; q++)
        for (int w = 0; w < 6; w++)
            if (st[q & 63][w] && st[q & 63][w] < t0) t0 = st[q & 63][w];
    fprintf(stderr, "[zkml device]");
    for (uint32_t q = lo; q <= hi && q - lo < 64; q++) {
        const unsigned long long* e = st[q & 63];
        auto us = [&](unsigned long long v) { return v ? (double)(v - t0) / 1e3 : -1.0; };
        fprintf(stderr, " %u:%.1f/%.1f/%.1f/%.1f/%.1f/%.1f", q - lo, us(e[0]), us(e[5]), us(e[1]), us(e[3]), us(e[4]),
                us(e[2]));
    }
    fprintf(stderr, "\n");
}

// The 8-word challenge slot [tag, 4 challenge words, abort, check, -] in mapped
// host memory, read as two 16-byte loads issued together (one PCIe round trip).
// The host writes words 1-6 before the tag; check = tag ^ words 1-5 ^ LA_SLOT_MIX,
// so a read whose two halves straddle a post fails the check and is retried.

// Both halves in one round trip: the second half relaxed, the first (with the tag)
// an acquire, issued back to back (the acquire orders only what follows it).
__device__ __forceinline__ void load_slot(const uint32_t* slot, uint4& lo, uint4& hi) {
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w) : "l"(slot + 4) : "memory");
    asm volatile("ld.acquire.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w) : "l"(slot) : "memory");
}

// Polls the slot until it holds tag `want` with a valid check (bounded; false on
// timeout).  Later loads of this thread are ordered after the acquire that saw it.
__device__ __forceinline__ bool poll_slot(const uint32_t* slot, uint32_t want, uint4& lo, uint4& hi) {
    unsigned long long it = 0;
    while (true) {
        load_slot(slot, lo, hi);
        if (lo.x == want && hi.z == (lo.x ^ lo.y ^ lo.z ^ lo.w ^ hi.x ^ hi.y ^ LA_SLOT_MIX)) return true;
        if (++it > kLaSpinLimit) return false;
        __nanosleep(it < 4096 ? 32 : 256);
    }
}

__device__ __noinline__ qm31 la_fold(const uint4* V, size_t p, size_t L, int fold, const AlphaRows* m) {
    const qm31 lo = u2q(__ldcg(V + p));  // through L2: V may have been folded by the kernel before
    return fold ? fold_qq(lo, u2q(__ldcg(V + p + L)), *m) : lo;
}

__device__ __noinline__ qm31 la_mul(qm31 x, qm31 y) {
    QAcc s;
    qacc_zero(s);
    qacc_mul(s, x, y);
    return qacc_value(s);
}

// Lanes [16 g, 16 g + 16) of a warp work on one quad together: lanes 0-7 of the
// half fold one element each (A at the four positions, then B), the eight
// folded values are broadcast within the half by shuffles, and lane k < 11
// forms the k-th product (k = 10 is the second half of T).  So a quad costs
// one fold and one product of latency instead of eight and eleven.
__device__ __forceinline__ qm31 shfl_q(const qm31& v, int src) {
    return qm(__shfl_sync(0xffffffffu, v.a, src), __shfl_sync(0xffffffffu, v.b, src),
              __shfl_sync(0xffffffffu, v.c, src), __shfl_sync(0xffffffffu, v.d, src));
}

__global__ void __launch_bounds__(LA_THREADS) round_lookahead_kernel(uint4* __restrict__ A, uint4* __restrict__ B,
                                                                     size_t L, int fold, const AlphaRows m,
                                                                     unsigned long long* gacc, unsigned int* ticket,
                                                                     uint32_t* sig, uint32_t seq,
                                                                     const uint32_t* wait_msg, uint32_t wait_seq,
                                                                     uint32_t* status, uint32_t* mailbox,
                                                                     const uint32_t* err_word) {
    constexpr int COLS = 2 * LA_THREADS / 32;  // two half-warps per warp
    __shared__ uint32_t sh[11][4][COLS];
    __shared__ AlphaRows ms;
    __shared__ int skip;
    // A queued successor may become resident now (it waits for its own challenge).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        skip = 0;
        if (blockIdx.x == 0) la_stamp(seq, 0);
        if (wait_msg) {
            // Block 0 polls the host slot and forwards the challenge through a
            // device mailbox [tag, 4 challenge words, abort] that the other
            // blocks poll, so only one thread reads host memory.
            volatile uint32_t* box = mailbox;
            uint32_t w[5] = {0, 0, 0, 0, 1};
            bool ok = false;
            unsigned long long it = 0;
            if (blockIdx.x == 0) {
                uint4 lo, hi;
                ok = poll_slot(wait_msg, wait_seq, lo, hi);
                if (ok) {
                    la_stamp(seq, 1);
                    w[0] = lo.y; w[1] = lo.z; w[2] = lo.w; w[3] = hi.x; w[4] = hi.y;
                }
                for (int k = 0; k < 5; k++) box[1 + k] = w[k];
                __threadfence();
                asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(mailbox), "r"(wait_seq) : "memory");
            } else {
                while (true) {
                    uint32_t tag;
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(tag) : "l"(mailbox) : "memory");
                    if (tag == wait_seq) {
                        ok = true;
                        break;
                    }
                    if (++it > kLaSpinLimit) break;
                    __nanosleep(it < 4096 ? 32 : 256);
                }
                if (ok)
                    for (int k = 0; k < 5; k++) w[k] = box[1 + k];
            }
            if (!ok) {
                skip = 1;
                if (status) atomicOr(status, 1u);
            } else if (w[4] != 0) {
                skip = 1;
            } else {
                ms = alpha_rows(qm(w[0], w[1], w[2], w[3]));
            }
        } else {
            ms = m;
        }
    }
    __syncthreads();
    // A kernel launched early behind its predecessor reads the vectors only after
    // the acquires that saw its challenge (host slot, then the mailbox): the
    // predecessor's folds were complete when it published the words the host's
    // challenge follows.
    if (skip) L = 0;  // no work: publish zeros so the queue drains
    const unsigned lane = threadIdx.x & 31, sub = lane & 15, half = lane >> 4, warp = threadIdx.x >> 5;
    const int col = 2 * warp + half;
    qm31 acc = qzero();
    if (L == 2) {  // last round: lanes 0-3 of warp 0 fold, lanes 0-2 multiply
        if (blockIdx.x == 0 && warp == 0) {
            qm31 x = qzero();
            if (lane < 4) {
                const uint4* V = lane < 2 ? A : B;
                x = la_fold(V, lane & 1, 2, fold, &ms);
                if (fold) st_q((lane < 2 ? A : B) + (lane & 1), x);
            }
            const qm31 a0 = shfl_q(x, 0), a1 = shfl_q(x, 1), b0 = shfl_q(x, 2), b1 = shfl_q(x, 3);
            qm31 px = a0, py = b0;
            if (lane == 1) { px = a1; py = b1; }
            if (lane == 2) { px = at_two(a0, a1); py = at_two(b0, b1); }
            const qm31 pr = la_mul(px, py);
            if (half == 0 && sub < 3) acc = pr;
            if (half == 0 && sub >= 3 && sub < 7) acc = sub == 3 ? a0 : sub == 4 ? a1 : sub == 5 ? b0 : b1;
        }
    } else {
        const size_t h = L / 2, q = L / 4;
        const size_t warps = (size_t)gridDim.x * (LA_THREADS / 32);
#pragma unroll 1
        for (size_t base = 2 * (blockIdx.x * (size_t)(LA_THREADS / 32) + warp); base < q; base += 2 * warps) {
            const size_t i = base + half;
            const bool valid = i < q;
            qm31 x = qzero();
            if (valid && sub < 8) {
                const size_t e = sub & 3;
                const size_t pos = i + (e & 1 ? q : 0) + (e & 2 ? h : 0);
                uint4* V = sub < 4 ? A : B;
                x = la_fold(V, pos, L, fold, &ms);
                if (fold) st_q(V + pos, x);
            }
            const int s0 = 16 * half;
            const qm31 a0 = shfl_q(x, s0), a1 = shfl_q(x, s0 + 1), a2 = shfl_q(x, s0 + 2), a3 = shfl_q(x, s0 + 3);
            const qm31 b0 = shfl_q(x, s0 + 4), b1 = shfl_q(x, s0 + 5), b2 = shfl_q(x, s0 + 6), b3 = shfl_q(x, s0 + 7);
            // factor pair of product `sub` among [Q0 Q1 Q2 Q3 T D0 D1 U W UW T']
            qm31 px, py;
            switch (sub) {
                case 0: px = a0; py = b0; break;
                case 1: px = a1; py = b1; break;
                case 2: px = a2; py = b2; break;
                case 3: px = a3; py = b3; break;
                case 4: px = at_two(a0, a2); py = at_two(b0, b2); break;
                case 5: px = qsub(a2, a0); py = qsub(b2, b0); break;
                case 6: px = qsub(a3, a1); py = qsub(b3, b1); break;
                case 7: px = at_two(a0, a1); py = at_two(b0, b1); break;
                case 8: px = at_two(qsub(a2, a0), qsub(a3, a1)); py = at_two(qsub(b2, b0), qsub(b3, b1)); break;
                case 9: px = at_two(a2, a3); py = at_two(b2, b3); break;
                case 10: px = at_two(a1, a3); py = at_two(b1, b3); break;
                default: px = qzero(); py = qzero(); break;
            }
            const qm31 pr = la_mul(px, py);
            if (valid && sub < 11) acc = qadd(acc, pr);
        }
    }
    // block reduction: lane `sub` of each half-warp holds word group `sub`
    if (sub < 11) {
        sh[sub][0][col] = acc.a;
        sh[sub][1][col] = acc.b;
        sh[sub][2][col] = acc.c;
        sh[sub][3][col] = acc.d;
    }
    __syncthreads();
    if (threadIdx.x < LA_WORDS) {  // the block's word, added into the grid's 64-bit accumulator
        const int g = threadIdx.x >> 2, c = threadIdx.x & 3;
        uint32_t v = 0;
#pragma unroll 1
        for (int k = 0; k < COLS; k++) {
            v = madd(v, sh[g][c][k]);
            if (g == 4 && L > 2) v = madd(v, sh[10][c][k]);
        }
        if (v) atomicAdd(gacc + threadIdx.x, (unsigned long long)v);
    }
    __shared__ bool is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        if (blockIdx.x == 0) la_stamp(seq, 3);
        is_last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    if (threadIdx.x == 0) la_stamp(seq, 4);
    __threadfence();
    // Last block: every block's words are in the accumulators (each block's
    // atomics precede its fence and ticket); take them and leave zeros for the
    // next look-ahead kernel.
    __shared__ uint32_t res[LA_WORDS + LA_FLAG_WORDS];
    if (threadIdx.x < LA_WORDS) res[threadIdx.x] = red64(atomicExch(gacc + threadIdx.x, 0ull));
    __syncthreads();
    if (threadIdx.x == 0) {
        *ticket = 0;
        la_stamp(seq, 2);
        int n = LA_WORDS;
        if (L == 2 && err_word) {  // last round: the error words ride with the final values
            res[LA_WORDS] = *(volatile const uint32_t*)err_word;
            res[LA_WORDS + 1] = status ? *(volatile const uint32_t*)status : 0u;
            n += LA_FLAG_WORDS;
        }
        if (sig) publish(sig, seq, res, n);
    }
}

void launch_round_lookahead(uint4* A, uint4* B, size_t L, bool fold, qm31 alpha, const RoundScratch& rs,
                            cudaStream_t s, const uint32_t* wait_msg, uint32_t wait_seq, uint32_t* status,
                            uint32_t* mailbox, const uint32_t* err_word, bool pdl) {
    size_t blocks = L >= 4 ? (L / 4 + 15) / 16 : 1;  // 16 quads per block per pass
    const size_t cap = (size_t)rs.max_blocks * 16 / LA_WORDS;
    if (blocks > cap) blocks = cap;
    if (blocks == 0) blocks = 1;
    // the 40 result words go to the host signal area only (rs.out holds 32 words)
    static_assert(LA_WORDS + LA_FLAG_WORDS <= 48, "signal area");
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(LA_THREADS);
    cfg.stream = s;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaLaunchKernelEx(&cfg, round_lookahead_kernel, A, B, L, fold ? 1 : 0, alpha_rows(alpha), rs.la_acc, rs.ticket,
                       rs.sig, rs.seq, wait_msg, wait_seq, status, mailbox, err_word);
}

// ---------------------------------------------------------------------------
// Look-ahead tail: every remaining round of a sumcheck whose vectors have at
// most LA_TAIL_MAX elements, in ONE block with both vectors resident in shared
// memory.  The L0 input elements are folded first when fold0 is set (round 0
// then has L0 / 2 elements).  Round j waits for its challenge in host slot
// (tag_base + j) % slots (round 0 only when wait0 is set; otherwise it folds
// with alpha0), folds in shared memory and publishes the same words as
// round_lookahead_kernel with sequence seq_base + j.  Thread t < 11 * TAIL_COLS
// forms product k = t / TAIL_COLS of the quads t % TAIL_COLS, t % TAIL_COLS +
// TAIL_COLS, ..., so a thread's product kind is fixed for the whole kernel.
// ---------------------------------------------------------------------------
constexpr int TAIL_THREADS = 1024;
constexpr int TAIL_COLS = 93;  // 11 * 93 = 1023 product threads

// Product kind K over the quads c, c + TAIL_COLS, ... of the resident vectors, with
// a0..a3 = A[i], A[i + q], A[i + h], A[i + q + h] (the same for B): kinds 0-3 are
// a_K b_K, then (a0, a2) at two, a2 - a0, a3 - a1, (a0, a1) at two, (a2 - a0,
// a3 - a1) at two, (a2, a3) at two and (a1, a3) at two -- the products of
// round_lookahead_kernel.  Accumulated lazily; only the elements kind K needs are
// read from shared memory.
template <int K>
__device__ __forceinline__ void tail_kind(const uint4* SA, const uint4* SB, int c, int q, int h, QAcc& s) {
    for (int i = c; i < q; i += TAIL_COLS) {
        qm31 px, py;
        if (K < 4) {
            const int o = i + ((K & 1) ? q : 0) + ((K & 2) ? h : 0);
            px = u2q(SA[o]);
            py = u2q(SB[o]);
        } else if (K == 4) {  // at two, first variable: (a0, a2)
            px = at_two(u2q(SA[i]), u2q(SA[i + h]));
            py = at_two(u2q(SB[i]), u2q(SB[i + h]));
        } else if (K == 5) {
            px = qsub(u2q(SA[i + h]), u2q(SA[i]));
            py = qsub(u2q(SB[i + h]), u2q(SB[i]));
        } else if (K == 6) {
            px = qsub(u2q(SA[i + q + h]), u2q(SA[i + q]));
            py = qsub(u2q(SB[i + q + h]), u2q(SB[i + q]));
        } else if (K == 7) {  // at two, second variable: (a0, a1)
            px = at_two(u2q(SA[i]), u2q(SA[i + q]));
            py = at_two(u2q(SB[i]), u2q(SB[i + q]));
        } else if (K == 8) {
            px = at_two(qsub(u2q(SA[i + h]), u2q(SA[i])), qsub(u2q(SA[i + q + h]), u2q(SA[i + q])));
            py = at_two(qsub(u2q(SB[i + h]), u2q(SB[i])), qsub(u2q(SB[i + q + h]), u2q(SB[i + q])));
        } else if (K == 9) {
            px = at_two(u2q(SA[i + h]), u2q(SA[i + q + h]));
            py = at_two(u2q(SB[i + h]), u2q(SB[i + q + h]));
        } else {  // 10: (a1, a3), the second half of T
            px = at_two(u2q(SA[i + q]), u2q(SA[i + q + h]));
            py = at_two(u2q(SB[i + q]), u2q(SB[i + q + h]));
        }
        qacc_mul(s, px, py);
    }
}

__global__ void __launch_bounds__(TAIL_THREADS, 1) lookahead_tail_kernel(const uint4* __restrict__ A,
                                                                         const uint4* __restrict__ B, int L0,
                                                                         int fold0, int wait0, qm31 alpha0,
                                                                         uint32_t* sig,
                                                                         uint32_t seq_base, const uint32_t* msg,
                                                                         uint32_t tag_base, int slots,
                                                                         uint32_t* status,
                                                                         const uint32_t* err_word) {
    extern __shared__ uint4 tail_sh[];
    uint4* SA = tail_sh;
    uint4* SB = tail_sh + L0;
    __shared__ uint32_t red[11][4][32];
    __shared__ uint32_t res[LA_WORDS + LA_FLAG_WORDS];
    __shared__ AlphaRows ms;
    __shared__ int state;  // 0 run, 1 stop
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int k = t / TAIL_COLS, c = t % TAIL_COLS;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (t == 0) la_stamp(seq_base, 0);
    // Thread 0 takes round j's challenge (sets ms, or state = 1 to stop).
    auto take = [&](int j) {
        state = 0;
        if (j == 0 && !wait0) {
            if (fold0) ms = alpha_rows(alpha0);
            return;
        }
        const uint32_t* slot = msg + 8 * ((tag_base + j) % slots);
        uint4 lo, hi;
        if (!poll_slot(slot, tag_base + j, lo, hi)) {
            atomicOr(status, 1u);
            state = 1;
            return;
        }
        if (hi.y != 0) {  // abort
            state = 1;
        } else {
            la_stamp(seq_base + j, 1);
            ms = alpha_rows(qm(lo.y, lo.z, lo.w, hi.x));
        }
    };
    // Round 0's challenge first: a kernel launched early behind the previous round's
    // kernel reads the vectors only after the acquire that saw the challenge (the
    // previous kernel published before the host posted it), through L2.
    if (t == 0) take(0);
    __syncthreads();
    if (state) return;
    int L = L0;
    if (fold0) {  // fold on load: V_0 = fold(input), both halves read from global memory
        L = L0 / 2;
#pragma unroll
        for (int r = 0; r < 2 * (int)LA_TAIL_MAX * 2 / TAIL_THREADS; r++) {
            const int p = t + r * TAIL_THREADS;
            if (p < 2 * L) {
                const int e = p < L ? p : p - L;
                const uint4* V = p < L ? A : B;
                const qm31 x = fold_qq(u2q(__ldcg(V + e)), u2q(__ldcg(V + e + L)), ms);
                st_q((p < L ? SA : SB) + e, x);
            }
        }
    } else {
#pragma unroll
        for (int r = 0; r < 2 * (int)LA_TAIL_MAX / TAIL_THREADS; r++) {
            const int i = t + r * TAIL_THREADS;
            if (i < L0) {
                SA[i] = __ldcg(A + i);
                SB[i] = __ldcg(B + i);
            }
        }
    }
    __syncthreads();
    if (t == 0) la_stamp(seq_base, 5);
    for (int j = 0;; j++) {
        if (j > 0) {  // challenge of the previous round, then V_j = fold(V_{j-1}) in place
            if (t == 0) take(j);
            __syncthreads();
            if (state) return;
            L /= 2;
            for (int p = t; p < 2 * L; p += TAIL_THREADS) {  // thread writes p < L, reads p and p + L
                const int e = p < L ? p : p - L;
                uint4* V = p < L ? SA : SB;
                const qm31 x = fold_qq(u2q(V[e]), u2q(V[e + L]), ms);
                st_q(V + e, x);
            }
            __syncthreads();
        }
        if (t == 0) la_stamp(seq_base + j, 3);
        qm31 acc = qzero();
        if (L == 2) {
            if (t < 7) {
                const qm31 a0 = u2q(SA[0]), a1 = u2q(SA[1]), b0 = u2q(SB[0]), b1 = u2q(SB[1]);
                if (t == 0) acc = la_mul(a0, b0);
                if (t == 1) acc = la_mul(a1, b1);
                if (t == 2) acc = la_mul(at_two(a0, a1), at_two(b0, b1));
                if (t == 3) acc = a0;
                if (t == 4) acc = a1;
                if (t == 5) acc = b0;
                if (t == 6) acc = b1;
                res[4 * t] = acc.a; res[4 * t + 1] = acc.b; res[4 * t + 2] = acc.c; res[4 * t + 3] = acc.d;
            } else if (t < 10) {
                res[4 * t] = res[4 * t + 1] = res[4 * t + 2] = res[4 * t + 3] = 0;
            }
            __syncthreads();
            if (t == 0) {
                la_stamp(seq_base + j, 2);
                int n = LA_WORDS;
                if (err_word) {  // the error words ride with the final values
                    res[LA_WORDS] = *(volatile const uint32_t*)err_word;
                    res[LA_WORDS + 1] = *(volatile const uint32_t*)status;
                    n += LA_FLAG_WORDS;
                }
                publish(sig, seq_base + j, res, n);
            }
            return;
        }
        const int h = L / 2, q = L / 4;
        if (k < 11) {
            QAcc sacc;
            qacc_zero(sacc);
            switch (k) {
                case 0: tail_kind<0>(SA, SB, c, q, h, sacc); break;
                case 1: tail_kind<1>(SA, SB, c, q, h, sacc); break;
                case 2: tail_kind<2>(SA, SB, c, q, h, sacc); break;
                case 3: tail_kind<3>(SA, SB, c, q, h, sacc); break;
                case 4: tail_kind<4>(SA, SB, c, q, h, sacc); break;
                case 5: tail_kind<5>(SA, SB, c, q, h, sacc); break;
                case 6: tail_kind<6>(SA, SB, c, q, h, sacc); break;
                case 7: tail_kind<7>(SA, SB, c, q, h, sacc); break;
                case 8: tail_kind<8>(SA, SB, c, q, h, sacc); break;
                case 9: tail_kind<9>(SA, SB, c, q, h, sacc); break;
                default: tail_kind<10>(SA, SB, c, q, h, sacc); break;
            }
            acc = qacc_value(sacc);
        }
        // per product kind: warp w < 11 sums the TAIL_COLS partials of kind w
        __shared__ qm31 part[TAIL_THREADS];
        part[t] = acc;
        __syncthreads();
        if (t == 0) la_stamp(seq_base + j, 4);
        if (warp < 11) {
            qm31 v = qzero();
            for (int i = lane; i < TAIL_COLS; i += 32) v = qadd(v, part[warp * TAIL_COLS + i]);
            for (int off = 16; off > 0; off >>= 1) {
                v.a = madd(v.a, __shfl_xor_sync(0xffffffffu, v.a, off));
                v.b = madd(v.b, __shfl_xor_sync(0xffffffffu, v.b, off));
                v.c = madd(v.c, __shfl_xor_sync(0xffffffffu, v.c, off));
                v.d = madd(v.d, __shfl_xor_sync(0xffffffffu, v.d, off));
            }
            if (lane == 0) {
                red[warp][0][0] = v.a; red[warp][1][0] = v.b; red[warp][2][0] = v.c; red[warp][3][0] = v.d;
            }
        }
        __syncthreads();
        if (t < LA_WORDS) {
            const int g = t >> 2, w = t & 3;
            uint32_t v = red[g][w][0];
            if (g == 4) v = madd(v, red[10][w][0]);
            res[t] = v;
        }
        __syncthreads();
        if (t == 0) {
            la_stamp(seq_base + j, 2);
            publish(sig, seq_base + j, res, LA_WORDS);
        }
        __syncthreads();
    }
}

int launch_lookahead_tail(const uint4* A, const uint4* B, size_t L0, bool fold0, bool wait0, qm31 alpha0,
                          uint32_t* sig, uint32_t seq_base, const uint32_t* msg, uint32_t tag_base, int slots,
                          uint32_t* status, cudaStream_t s, const uint32_t* err_word, bool pdl) {
    const size_t smem = 2 * L0 * sizeof(uint4);
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(lookahead_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(4 * LA_TAIL_MAX * sizeof(uint4))) != cudaSuccess)
            return -1;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(TAIL_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaLaunchKernelEx(&cfg, lookahead_tail_kernel, A, B, (int)L0, fold0 ? 1 : 0, wait0 ? 1 : 0, alpha0, sig, seq_base,
                       msg, tag_base, slots, status, err_word);
    return 0;
}

// Gathered shards (rank-major: rank g's A part then B part, `len` elements each)
// -> global order, global[j * G + g] = local_g[j].
__global__ void interleave_gather_kernel(const uint4* __restrict__ in, size_t len, size_t G, uint4* __restrict__ fa,
                                        uint4* __restrict__ fb) {
    const size_t glen = len * G;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < glen; i += (size_t)gridDim.x * blockDim.x) {
        const size_t j = i / G, g = i % G;
        fa[i] = in[g * 2 * len + j];
        fb[i] = in[g * 2 * len + len + j];
    }
}

void launch_interleave_gather(const uint4* in, size_t len, size_t G, uint4* fa, uint4* fb, cudaStream_t s) {
    size_t blocks = (len * G + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks == 0) blocks = 1;
    interleave_gather_kernel<<<(unsigned)blocks, 256, 0, s>>>(in, len, G, fa, fb);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static unsigned round_blocks(size_t work, int max_blocks) {
    size_t b = (work + 255) / 256;
    if (b > (size_t)max_blocks) b = max_blocks;
    if (b == 0) b = 1;
    return (unsigned)b;
}

void launch_round_qm31(uint4* A, uint4* B, size_t len, const RoundScratch& rs, cudaStream_t s) {
    const size_t q = len / 2;
    round_qm31_kernel<<<round_blocks(q, rs.max_blocks), 256, 0, s>>>(A, B, q, rs.partials, rs.ticket, rs.out, rs.sig,
                                                                      rs.seq, rs.mesh);
}

void launch_fold_round_qm31(uint4* A, uint4* B, size_t len, qm31 alpha, const RoundScratch& rs, cudaStream_t s) {
    const size_t h = len / 2;
    fold_round_qm31_kernel<<<round_blocks(h / 2, rs.max_blocks), 256, 0, s>>>(A, B, h, alpha_rows(alpha),
                                                                                rs.partials, rs.ticket, rs.out,
                                                                                rs.sig, rs.seq, rs.mesh);
}

void launch_round_m31(const uint32_t* A, const uint32_t* B, size_t len, const RoundScratch& rs, uint32_t* err,
                      cudaStream_t s) {
    const size_t q = len / 2;
    if (q % 4 == 0 && aligned16(A) && aligned16(B))
        round_m31_kernel<4><<<round_blocks(q / 4, rs.max_blocks), 256, 0, s>>>(A, B, q, rs.partials, rs.ticket,
                                                                               rs.out, err, rs.sig, rs.seq, rs.mesh);
    else
        round_m31_kernel<1><<<round_blocks(q, rs.max_blocks), 256, 0, s>>>(A, B, q, rs.partials, rs.ticket, rs.out,
                                                                           err, rs.sig, rs.seq, rs.mesh);
}

void launch_fold_round_m31(const uint32_t* A, const uint32_t* B, size_t len, qm31 alpha, uint4* Ao, uint4* Bo,
                           const RoundScratch& rs, cudaStream_t s) {
    const size_t h = len / 2;
    fold_round_m31_kernel<<<round_blocks((h / 2 + FR_UNROLL - 1) / FR_UNROLL, rs.max_blocks), 256, 0, s>>>(
        A, B, h, alpha, Ao, Bo, rs.partials, rs.ticket, rs.out, rs.sig, rs.seq, rs.mesh);
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

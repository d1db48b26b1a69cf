// Forward M31 matrix product C = A * B mod P on the integer tensor pipe
// (replaces gpu_matmul_m31_full, engine/src/gpu_sumcheck.rs:3104-3196, the
// forward pass that produces the GraphExecution the GKR prover walks).
//
// Both operands are split into byte planes (imma.cuh): C = sum_{a,b} 256^(a+b)
// A_a B_b, each A_a B_b an exact u8 GEMM on mma.m16n8k32.  A (m x k, row major)
// is read as is: four consecutive k of a row are one 16-byte load whose byte
// planes are A fragments; B (k x n, row major) is read in place, four rows at a
// time, and split into planes in registers.  The sixteen plane pairs share seven accumulators
// by weight w = a + b (at most four pairs per weight, each below
// 255^2 * 8192 per K chunk, so a chunk of 8192 stays below 2^31); every K
// chunk ends with sum_w 256^w acc_w mod P added to 64-bit lazy sums.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "context.hpp"
#include "gkr.cuh"
#include "imma.cuh"
#include "round_arith.cuh"

namespace zk {

constexpr uint32_t GEMM_KCHUNK = 8192;

// One block = 4 x NT x KS warps over a 64-row group and 8 NT output columns:
// warp w takes row tile w % 4 (16 rows), N-tile (w / 4) % NT and K part
// w / (4 NT); K parts meet in shared memory at the end.  B is read in place (row major): the four
// values B[t .. t+3][j] a B-fragment word needs are four 4-byte loads whose
// byte planes are the four planes' words; the lanes of a warp cover 8
// consecutive columns x 4 rows per load, so every 32-byte sector is used.
// The next K step's loads are issued before this step's MMAs.
constexpr int GEMM_NT = 1;  // 8-column N-tiles per block
constexpr int GEMM_KS = 2;  // K splits per block

struct GemmLoads {
    uint4 a[4];      // A: rows r0 / r1, k = t + 4 tg (+16)
    uint32_t b[8];   // B: rows t + 4 tg + e (e < 4) and t + 16 + 4 tg + e, column j
};

__device__ __forceinline__ void gemm_load(GemmLoads& L, const uint4* a0p, const uint4* a1p, bool v0, bool v1,
                                          const uint32_t* __restrict__ B, uint32_t k, uint32_t n, uint32_t j,
                                          bool wj, uint32_t t, uint32_t tg) {
    const uint32_t ta = t + 4 * tg, tb = ta + 16;
    const uint4 z = make_uint4(0, 0, 0, 0);
    L.a[0] = (v0 && ta < k) ? __ldg(a0p + ta / 4) : z;
    L.a[1] = (v1 && ta < k) ? __ldg(a1p + ta / 4) : z;
    L.a[2] = (v0 && tb < k) ? __ldg(a0p + tb / 4) : z;
    L.a[3] = (v1 && tb < k) ? __ldg(a1p + tb / 4) : z;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        L.b[e] = (wj && ta + e < k) ? __ldg(B + (size_t)(ta + e) * n + j) : 0u;
        L.b[4 + e] = (wj && tb + e < k) ? __ldg(B + (size_t)(tb + e) * n + j) : 0u;
    }
}

template <int NT, int KS>
__global__ void __launch_bounds__(4 * NT * KS * 32) m31_gemm_tc_kernel(const uint32_t* __restrict__ A,
                                                                     const uint32_t* __restrict__ B,
                                                                     uint32_t* __restrict__ Cm, uint32_t m, uint32_t k,
                                                                     uint32_t n, uint32_t* __restrict__ err) {
    __shared__ uint64_t part[KS > 1 ? 4 * NT : 1][32][4];
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, tg = lane & 3;
    const uint32_t rt = warp & 3, nt = (warp >> 2) % NT, half = warp / (4 * NT);
    const uint32_t r0 = blockIdx.y * 64 + rt * 16 + g, r1 = r0 + 8;
    const uint32_t j0 = blockIdx.x * 8 * NT + 8 * nt, j = j0 + g;
    const bool v0 = r0 < m, v1 = r1 < m, wj = j < n;
    const uint4* a0p = reinterpret_cast<const uint4*>(A + (size_t)(v0 ? r0 : 0) * k);
    const uint4* a1p = reinterpret_cast<const uint4*>(A + (size_t)(v1 ? r1 : 0) * k);
    // this warp's half of the K steps
    const uint32_t steps = (k + 31) / 32, per = (steps + KS - 1) / KS;
    const uint32_t s_begin = min(steps, half * per), s_end = min(steps, s_begin + per);
    uint64_t tot[4] = {0, 0, 0, 0};
    uint32_t bad = 0;
    GemmLoads cur, nxt;
    if (s_begin < s_end) gemm_load(cur, a0p, a1p, v0, v1, B, k, n, j, wj, 32 * s_begin, tg);
    for (uint32_t c0 = s_begin; c0 < s_end; c0 += GEMM_KCHUNK / 32) {
        const uint32_t c_end = min(s_end, c0 + GEMM_KCHUNK / 32);
        int acc[7][4];
#pragma unroll
        for (int w = 0; w < 7; w++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[w][e] = 0;
        for (uint32_t st = c0; st < c_end; st++) {
            if (st + 1 < s_end) gemm_load(nxt, a0p, a1p, v0, v1, B, k, n, j, wj, 32 * (st + 1), tg);
            uint32_t pa[4][4], pb[4][2];
#pragma unroll
            for (int f = 0; f < 4; f++) {
                bad |= cur.a[f].x | cur.a[f].y | cur.a[f].z | cur.a[f].w;
                byte_planes(cur.a[f], pa[0][f], pa[1][f], pa[2][f], pa[3][f]);
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint4 bw = make_uint4(cur.b[4 * h], cur.b[4 * h + 1], cur.b[4 * h + 2], cur.b[4 * h + 3]);
                bad |= bw.x | bw.y | bw.z | bw.w;
                byte_planes(bw, pb[0][h], pb[1][h], pb[2][h], pb[3][h]);
            }
#pragma unroll
            for (int a = 0; a < 4; a++)
#pragma unroll
                for (int b = 0; b < 4; b++) mma_u8(acc[a + b], pa[a], pb[b][0], pb[b][1]);
            cur = nxt;
        }
#pragma unroll
        for (int e = 0; e < 4; e++) {
            uint64_t sum = 0;
#pragma unroll
            for (int w = 0; w < 7; w++) sum = acc_fold(sum, mul_wide((uint32_t)acc[w][e], pow256(w)));
            tot[e] = acc_fold(tot[e], (uint64_t)canon64(sum));
        }
    }
    static_assert(KS == 1 || KS == 2, "K split");
    if (bad & 0x80000000u) atomicOr(err, 1u);
    if (KS > 1) {  // K halves meet in shared memory
        if (half) {
#pragma unroll
            for (int e = 0; e < 4; e++) part[warp % (4 * NT)][lane][e] = tot[e];
        }
        __syncthreads();
        if (half) return;
#pragma unroll
        for (int e = 0; e < 4; e++) tot[e] = acc_fold(tot[e], part[warp][lane][e]);
    }
    {
        // C fragment: e = 0, 1 -> row r0, columns 2 tg, 2 tg + 1; e = 2, 3 -> row r1
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t row = e < 2 ? r0 : r1, col = j0 + 2 * tg + (e & 1);
            if (row < m && col < n) Cm[(size_t)row * n + col] = canon64(tot[e]);
        }
    }
}

// ---------------------------------------------------------------------------
// Narrow-value path.  Quantised layers carry small signed values (int8 weights, int16
// activations embedded in M31 as v or p - |v|).  Read as signed integers, an A value is
// a = 256 a_1 + a_0 with a_0 in [0, 256) and a_1 in [-128, 128) (every int16), a B value
// is one signed byte, so C = A_0 B + 256 A_1 B takes one u8 x s8 and one s8 x s8 MMA per
// element pair instead of the 16 u8 byte-plane pairs.  A value that does not fit sets a
// flag and the caller recomputes with the full kernel, so the result is the same exact
// product for every input.
constexpr int GEMM_GA = 2;        // byte digits of A

// A (m x k, row major) -> GA digit planes, each m x kp int8 (kp = k rounded up to 32,
// zero padded); sets *narrow_bad if a value needs more digits.
__global__ void gemm_a_digits_kernel(const uint32_t* __restrict__ A, uint32_t m, uint32_t k, uint32_t kp,
                                     int8_t* __restrict__ D, uint32_t* __restrict__ narrow_bad) {
    uint32_t bad = 0;
    const size_t total = (size_t)m * kp;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(idx / kp), c = (uint32_t)(idx % kp);
        const int q = c < k ? m31_signed(A[(size_t)r * k + c]) : 0;
        const int d0 = q & 0xff, d1 = (q - d0) >> 8;  // q = 256 d1 + d0, d0 unsigned
        D[idx] = (int8_t)(uint8_t)d0;
        D[total + idx] = (int8_t)d1;
        bad |= (uint32_t)(d1 < -128 || d1 > 127);
    }
    if (bad) atomicOr(narrow_bad, 1u);
}

// One block: 64 rows (4 row tiles) x GN_COLS columns, 8 warps = 4 row tiles x 2 column
// halves (4 N-tiles each).  Per stage of GN_BK rows of K, the block loads the B tile
// (GN_BK rows x GN_COLS columns, 16-byte coalesced loads along the rows), converts it once
// to signed bytes and stores it transposed ([column][k], pitch GN_BK + 4 bytes) in shared
// memory, where each B fragment is one 4-byte read; the block's A digit tile (64 rows x
// GN_BK, both digits) is staged beside it.  The next stage's tiles are loaded into registers
// while this stage's MMAs run.
// gridDim.z splits K: each split writes its partial products (mod p) to its own plane of
// `part`, added by gemm_combine_kernel.
constexpr int GN_COLS = 64;
constexpr int GN_BK = 64;
constexpr int GN_PITCH = GN_BK + 4;
static_assert(GN_BK * GN_COLS == 256 * 16, "one 4 x 4 block of the B tile per thread and stage");
constexpr int GN_APITCH = GN_BK + 16;                  // A tile row pitch (bytes)
constexpr int GN_APIECES = GEMM_GA * 64 * GN_BK / 16 / 256;  // 16-byte A pieces per thread and stage

__global__ void __launch_bounds__(256, 3) m31_gemm_narrow_kernel(const int8_t* __restrict__ D,
                                                              const uint32_t* __restrict__ B,
                                                              uint32_t* __restrict__ part, uint32_t m, uint32_t k,
                                                              uint32_t kp, uint32_t n,
                                                              uint32_t* __restrict__ narrow_bad) {
    __shared__ __align__(16) uint8_t bs[2][GN_COLS * GN_PITCH];
    __shared__ __align__(16) uint8_t as[2][GEMM_GA * 64 * GN_APITCH];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tg = lane & 3;
    const uint32_t rt = warp & 3, ch = warp >> 2;  // row tile, column half
    const uint32_t r0 = blockIdx.y * 64 + rt * 16 + g, r1 = r0 + 8;
    const uint32_t col0 = blockIdx.x * GN_COLS;
    const size_t plane = (size_t)m * kp;
    const bool vec_ok = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(B) & 15) == 0);
    // this block's stages (of GN_BK rows) of the K range
    const uint32_t stages = (kp + GN_BK - 1) / GN_BK, per = (stages + gridDim.z - 1) / gridDim.z;
    const uint32_t s_begin = min(stages, blockIdx.z * per), s_end = min(stages, s_begin + per);
    // this thread's 4 x 4 block of the B tile: rows 4 br .. 4 br + 3, columns 4 bc .. 4 bc + 3
    const uint32_t br = tid >> 4, bc = tid & 15;
    uint32_t raw[4][4];  // [row][column]
    uint4 araw[GN_APIECES];
    auto load_tile = [&](uint32_t sg) {
#pragma unroll
        for (int h = 0; h < GN_APIECES; h++) {
            const uint32_t idx = tid + 256 * h, per_row = GN_BK / 16, dg = idx / (64 * per_row);
            const uint32_t row = (idx / per_row) % 64, c16 = idx % per_row;
            const uint32_t grow = blockIdx.y * 64 + row, kk = GN_BK * sg + 16 * c16;
            araw[h] = (grow < m && kk < kp)
                          ? __ldg(reinterpret_cast<const uint4*>(D + dg * plane + (size_t)grow * kp + kk))
                          : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int rr = 0; rr < 4; rr++) {
            const uint32_t row = GN_BK * sg + 4 * br + rr, col = col0 + 4 * bc;
            if (row < k && vec_ok && col + 3 < n) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(B + (size_t)row * n + col));
                raw[rr][0] = v.x;
                raw[rr][1] = v.y;
                raw[rr][2] = v.z;
                raw[rr][3] = v.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; e++)
                    raw[rr][e] = (row < k && col + e < n) ? __ldg(B + (size_t)row * n + col + e) : 0u;
            }
        }
    };
    uint32_t bad = 0;
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int h = 0; h < GN_APIECES; h++) {
            const uint32_t idx = tid + 256 * h, per_row = GN_BK / 16, dg = idx / (64 * per_row);
            const uint32_t row = (idx / per_row) % 64, c16 = idx % per_row;
            *reinterpret_cast<uint4*>(as[buf] + (dg * 64 + row) * GN_APITCH + 16 * c16) = araw[h];
        }
        // signed bytes, transposed: column 4 bc + e gets the 4 bytes of rows 4 br .. 4 br + 3.
        // For v < 2^31, t = v + (v >> 30) has the signed value's byte as its low byte when v
        // is in [0, 127] or in [P - 128, P] (t = 2^31 + s there); every other v leaves a bit of
        // 8..30 set in t + 128.  Inputs with bit 31 set are caught by vor.
        uint32_t tb[4][4], vor = 0;
#pragma unroll
        for (int rr = 0; rr < 4; rr++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const uint32_t v = raw[rr][e];
                const uint32_t t = v + (v >> 30);
                bad |= (t + 128u) & 0x7fffff00u;
                vor |= v;
                tb[rr][e] = t;
            }
        bad |= vor >> 31;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t lo = __byte_perm(tb[0][e], tb[1][e], 0x0040);
            const uint32_t hi = __byte_perm(tb[2][e], tb[3][e], 0x0040);
            *reinterpret_cast<uint32_t*>(bs[buf] + (4 * bc + e) * GN_PITCH + 4 * br) = __byte_perm(lo, hi, 0x5410);
        }
    };
    uint32_t tot[4][4];  // canonical partial sums
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int e = 0; e < 4; e++) tot[t][e] = 0;
    if (s_begin < s_end) {
        load_tile(s_begin);
        store_tile(0);
    }
    __syncthreads();
    int buf = 0;
    constexpr uint32_t CHUNK = GEMM_KCHUNK / GN_BK;  // stages per s32 accumulation chunk
    for (uint32_t c0 = s_begin; c0 < s_end; c0 += CHUNK) {
        const uint32_t c_end = min(s_end, c0 + CHUNK);
        int acc[4][GEMM_GA][4];
#pragma unroll
        for (int t = 0; t < 4; t++)
#pragma unroll
            for (int a = 0; a < GEMM_GA; a++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[t][a][e] = 0;
        for (uint32_t sg = c0; sg < c_end; sg++) {
            if (sg + 1 < s_end) load_tile(sg + 1);
#pragma unroll
            for (int ks = 0; ks < GN_BK / 32; ks++) {
                const uint32_t ta = 32 * ks + 4 * tg, tb = ta + 16;
                uint32_t af[GEMM_GA][4];
#pragma unroll
                for (int a = 0; a < GEMM_GA; a++) {
                    // the four 8 x 16-byte pieces of the 16 x 32 A fragment in one ldmatrix: lane l
                    // gives row (l & 7) of piece l >> 3 (rows +8 for odd pieces, bytes +16 for the
                    // upper two); the 80-byte row pitch keeps the eight rows of a piece on distinct banks
                    const uint32_t mi = lane >> 3;
                    const uint8_t* rowp = as[buf] + (a * 64 + rt * 16 + (mi & 1) * 8 + (lane & 7)) * GN_APITCH +
                                          32 * ks + (mi >> 1) * 16;
                    const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(rowp));
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(af[a][0]), "=r"(af[a][1]), "=r"(af[a][2]), "=r"(af[a][3])
                                 : "r"(addr));
                }
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const uint8_t* col = bs[buf] + (ch * 32 + t * 8 + g) * GN_PITCH + 32 * ks;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(col + 4 * tg);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(col + 16 + 4 * tg);
                    mma_u8s8(acc[t][0], af[0], b0, b1);
                    mma_s8(acc[t][1], af[1], b0, b1);
                }
            }
            if (sg + 1 < s_end) {
                store_tile(buf ^ 1);
                __syncthreads();
                buf ^= 1;
            }
        }
#pragma unroll
        for (int t = 0; t < 4; t++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                uint64_t sum = 0;
#pragma unroll
                for (int a = 0; a < GEMM_GA; a++) {
                    const int v = acc[t][a][e];
                    const uint32_t u = v < 0 ? (uint32_t)(v + 0x7fffffff) : (uint32_t)v;  // v mod P, <= P
                    sum = acc_fold(sum, mul_wide(u, pow256(a)));
                }
                tot[t][e] = canon64((uint64_t)tot[t][e] + canon64(sum));
            }
    }
    if (bad) atomicOr(narrow_bad, 1u);
    uint32_t* out = part + (size_t)blockIdx.z * m * n;
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t row = e < 2 ? r0 : r1, col = col0 + ch * 32 + t * 8 + 2 * tg + (e & 1);
            if (row < m && col < n) out[(size_t)row * n + col] = tot[t][e];
        }
}

// C = sum of the K splits' partial products mod p.
__global__ void gemm_combine_kernel(const uint32_t* __restrict__ part, uint32_t splits, size_t mn,
                                    uint32_t* __restrict__ C) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < mn; i += (size_t)gridDim.x * blockDim.x) {
        uint64_t s = 0;
        for (uint32_t z = 0; z < splits; z++) s += part[z * mn + i];
        C[i] = red64(s);
    }
}

}  // namespace zk

using namespace zk;

extern "C" int zkml_matmul_m31(zkml_ctx* ctx, const uint32_t* a, size_t m, size_t k, const uint32_t* b, size_t n,
                               uint32_t* c) {
    if (!ctx || !a || !b || !c) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (m == 0 || k == 0 || n == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty matrix");
    if (m > (1u << 30) || k > (1u << 30) || n > (1u << 30) || m * k > ((size_t)1 << 34) || k * n > ((size_t)1 << 34))
        return set_error(ZKML_ERR_INVALID_ARG, "matrix too large");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const void *A = nullptr, *B = nullptr;
    int rc = device_view(ctx, a, m * k * 4, ctx->a_in, &A);
    if (!rc) rc = device_view(ctx, b, k * n * 4, ctx->b_in, &B);
    if (rc) return rc;
    // output: in place when c is device memory of this GPU, else staged and copied back
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, c) != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    const bool dev_out = attr.type == cudaMemoryTypeDevice && attr.device == ctx->device;
    uint32_t* C = c;
    if (!dev_out) {
        if ((rc = ctx->op.cbuf.ensure(m * n * 4))) return rc;
        C = ctx->op.cbuf.as<uint32_t>();
    }
    const uint32_t* Ad = static_cast<const uint32_t*>(A);
    static const bool tc_on = !(getenv("ZKML_GEMM_TC") && getenv("ZKML_GEMM_TC")[0] == '0');  // 0: CUDA cores
    static const bool narrow_on = !(getenv("ZKML_GEMM_NARROW") && getenv("ZKML_GEMM_NARROW")[0] == '0');
    bool done = false;
    if (tc_on && narrow_on) {
        // narrow-value path; falls through to the full kernel if a value does not fit
        const uint32_t kp = (uint32_t)((k + 31) / 32 * 32);
        if ((rc = ctx->op.adig.ensure((size_t)GEMM_GA * m * kp + 16))) return rc;
        uint32_t* flag = ctx->err_flag() + 2;  // spare word of the error-flag block
        ZK_CUDA(cudaMemsetAsync(flag, 0, 4, s));
        {
            const size_t total = (size_t)m * kp;
            const unsigned g = (unsigned)std::min<size_t>((total + 255) / 256, (size_t)ctx->num_sms * 8);
            gemm_a_digits_kernel<<<g, 256, 0, s>>>(Ad, (uint32_t)m, (uint32_t)k, kp, ctx->op.adig.as<int8_t>(), flag);
        }
        // K splits so that the whole grid is resident at once (one wave): as many splits as
        // fit in the resident block slots, rounded down
        const unsigned bx = (unsigned)((n + GN_COLS - 1) / GN_COLS), by = (unsigned)((m + 63) / 64);
        const unsigned stages = (kp + GN_BK - 1) / GN_BK;
        static int per_sm = 0;
        if (!per_sm && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, m31_gemm_narrow_kernel, 256, 0) !=
                           cudaSuccess) {
            cudaGetLastError();
            per_sm = 3;
        }
        const size_t want = (size_t)std::max(per_sm, 1) * ctx->num_sms, have = (size_t)bx * by;
        unsigned splits = (unsigned)std::max<size_t>(1, want / have);
        splits = std::min(splits, std::min(stages, 8u));
        uint32_t* target = C;
        if (splits > 1) {
            if ((rc = ctx->op.gpart.ensure((size_t)splits * m * n * 4))) return rc;
            target = ctx->op.gpart.as<uint32_t>();
        }
        m31_gemm_narrow_kernel<<<dim3(bx, by, splits), 256, 0, s>>>(ctx->op.adig.as<int8_t>(),
                                                                    static_cast<const uint32_t*>(B), target,
                                                                    (uint32_t)m, (uint32_t)k, kp, (uint32_t)n, flag);
        if (splits > 1) {
            const unsigned g = (unsigned)std::min<size_t>((m * n + 255) / 256, (size_t)ctx->num_sms * 8);
            gemm_combine_kernel<<<g, 256, 0, s>>>(target, splits, m * n, C);
            ctx->launches++;
        }
        ctx->launches += 2;
        ZK_CUDA(cudaGetLastError());
        uint32_t hflag = 0;
        ZK_CUDA(cudaMemcpyAsync(&hflag, flag, 4, cudaMemcpyDeviceToHost, s));
        ZK_CUDA(cudaStreamSynchronize(s));
        done = hflag == 0;
    }
    if (done) {
    } else if (tc_on && k % 4 == 0 && (reinterpret_cast<uintptr_t>(Ad) & 15) == 0) {
        dim3 gg((unsigned)((n + 8 * GEMM_NT - 1) / (8 * GEMM_NT)), (unsigned)((m + 63) / 64));
        m31_gemm_tc_kernel<GEMM_NT, GEMM_KS><<<gg, 4 * GEMM_NT * GEMM_KS * 32, 0, s>>>(Ad, static_cast<const uint32_t*>(B), C, (uint32_t)m,
                                                           (uint32_t)k, (uint32_t)n, ctx->err_flag());
        ctx->launches++;
    } else {
        launch_m31_gemm(Ad, static_cast<const uint32_t*>(B), C, (uint32_t)m, (uint32_t)k, (uint32_t)n, s);
        ctx->launches++;
    }
    ZK_CUDA(cudaGetLastError());
    if (!dev_out) ZK_CUDA(cudaMemcpyAsync(c, C, m * n * 4, cudaMemcpyDeviceToHost, s));
    if ((rc = read_err_flag(ctx)) || (rc = check_err_flag(ctx, "matmul_m31"))) return rc;
    return ZKML_OK;
}

// Device helpers shared by the LogUp-family kernels (logup_kernels.cu,
// rmsnorm_kernels.cu): QM31 vector loads/stores, the publish of result words
// to mapped host memory, and the grid-wide reduction of lazily accumulated words.
#pragma once
#include "logup.cuh"
#include "round_arith.cuh"

namespace zk {

__device__ __forceinline__ qm31 ldq4(const uint4* p) {
    uint4 v = *p;
    return qm(v.x, v.y, v.z, v.w);
}
__device__ __forceinline__ void stq4(uint4* p, qm31 x) { *p = make_uint4(x.a, x.b, x.c, x.d); }

__device__ __forceinline__ void publish_words(uint32_t* sig, uint32_t seq, const uint32_t* words, int n) {
    volatile uint32_t* v = sig;
    for (int i = 0; i < n; i++) v[1 + i] = words[i];
    // the release store orders the word stores before the sequence number
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(sig), "r"(seq) : "memory");
}

// Grid reduction of NW lazily accumulated words (each accumulator is a sum of
// values < P): per-block partials, then the last block (atomic ticket) reduces
// them, stores the NW reduced words to out and optionally publishes them.
template <int NW>
__device__ void grid_reduce(unsigned long long (&acc)[NW], const ReduceScratch& rs) {
    __shared__ uint32_t sh[32][NW];
    __shared__ uint32_t res[NW];
    __shared__ bool is_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
#pragma unroll
    for (int i = 0; i < NW; i++) {
        uint32_t r = red64(acc[i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) r = madd(r, __shfl_xor_sync(0xffffffffu, r, off));
        if (lane == 0) sh[warp][i] = r;
    }
    __syncthreads();
    if (threadIdx.x < NW) {
        uint32_t a = 0;
        for (int w = 0; w < nw; w++) a = madd(a, sh[w][threadIdx.x]);
        rs.partials[blockIdx.x * NW + threadIdx.x] = a;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = (atomicAdd(rs.ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int i = warp; i < NW; i += nw) {
        unsigned long long a = 0;
        for (unsigned b = lane; b < gridDim.x; b += 32) a += __ldcg(rs.partials + b * NW + i);
        uint32_t v = red64(a);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = madd(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) {
            rs.out[i] = v;
            res[i] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *rs.ticket = 0;
        if (rs.sig) publish_words(rs.sig, rs.seq, res, NW);
    }
}

template <int NW>
__device__ __forceinline__ void acc_q(unsigned long long (&acc)[NW], int at, const qm31& x) {
    acc[at] += x.a;
    acc[at + 1] += x.b;
    acc[at + 2] += x.c;
    acc[at + 3] += x.d;
}

inline unsigned grid_for(size_t work, int max_blocks) {
    size_t b = (work + 255) / 256;
    if (b > (size_t)max_blocks) b = max_blocks;
    if (b == 0) b = 1;
    return (unsigned)b;
}

__device__ __forceinline__ qm31 qmul_f(const qm31& x, const qm31& y) {
    QAcc s;
    qacc_zero(s);
    qacc_mul(s, x, y);
    return qacc_value(s);
}

}  // namespace zk

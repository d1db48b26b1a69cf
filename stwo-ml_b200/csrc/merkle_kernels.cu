// Poseidon-252 Merkle kernels (engine/src/crypto/poseidon_merkle.rs:91-280).
//
// Leaves are securefield_to_felt(v) of QM31 MLE evaluations (no leaf hash),
// internal nodes poseidon_hash(left, right) = hades([left, right, 2])[0], and
// the leaf layer is zero-padded to a power of two (at least 2).  One thread
// computes one node; every level is one launch.  Nodes are stored in
// Montgomery form (identical bytes on host and device).
#include <cuda_runtime.h>

#include "felt252.cuh"
#include "merkle.cuh"
#include "qm31.cuh"

namespace zk {

__constant__ dfelt c_mont_r2;  // 2^512 mod p: Montgomery conversion factor
__constant__ dfelt c_mont_two; // Montgomery form of 2 (poseidon_hash capacity)

// securefield_to_felt(v) in Montgomery form.
__device__ __forceinline__ dfelt leaf_felt(uint4 v) {
    // canonical integer 2^124 | a << 93 | b << 62 | c << 31 | d, as 8 x u32
    dfelt x;
    x.w[0] = v.w | (v.z << 31);
    x.w[1] = (v.z >> 1) | (v.y << 30);
    x.w[2] = (v.y >> 2) | (v.x << 29);
    x.w[3] = (v.x >> 3) | (1u << 28);
    x.w[4] = x.w[5] = x.w[6] = x.w[7] = 0;
    return dmul(x, c_mont_r2);
}

__device__ __forceinline__ dfelt hash2(const dfelt& l, const dfelt& r) {
    dfelt s[3] = {l, r, c_mont_two};
    dhades(s);
    return s[0];
}

__device__ __forceinline__ dfelt ld_f(const dfelt* p) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    uint4 a = q[0], b = q[1];
    dfelt f;
    f.w[0] = a.x; f.w[1] = a.y; f.w[2] = a.z; f.w[3] = a.w;
    f.w[4] = b.x; f.w[5] = b.y; f.w[6] = b.z; f.w[7] = b.w;
    return f;
}

__device__ __forceinline__ void st_f(dfelt* p, const dfelt& f) {
    uint4* q = reinterpret_cast<uint4*>(p);
    q[0] = make_uint4(f.w[0], f.w[1], f.w[2], f.w[3]);
    q[1] = make_uint4(f.w[4], f.w[5], f.w[6], f.w[7]);
}

__global__ void __launch_bounds__(128) merkle_leaf_level_kernel(const uint4* __restrict__ leaves, size_t n_leaves,
                                                                size_t n_pairs, dfelt* __restrict__ out) {
    const dfelt zero = {{0, 0, 0, 0, 0, 0, 0, 0}};
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_pairs; i += (size_t)gridDim.x * blockDim.x) {
        const size_t l = 2 * i, r = 2 * i + 1;
        dfelt fl = l < n_leaves ? leaf_felt(leaves[l]) : zero;
        dfelt fr = r < n_leaves ? leaf_felt(leaves[r]) : zero;
        st_f(out + i, hash2(fl, fr));
    }
}

__global__ void __launch_bounds__(128) merkle_node_level_kernel(const dfelt* __restrict__ in, size_t n_pairs,
                                                                dfelt* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_pairs; i += (size_t)gridDim.x * blockDim.x)
        st_f(out + i, hash2(ld_f(in + 2 * i), ld_f(in + 2 * i + 1)));
}

__global__ void leaf_felts_kernel(const uint4* __restrict__ leaves, size_t n, dfelt* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        st_f(out + i, leaf_felt(leaves[i]));
}

__global__ void hash_pairs_kernel(const dfelt* __restrict__ a, const dfelt* __restrict__ b, size_t n,
                                  dfelt* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        st_f(out + i, hash2(ld_f(a + i), ld_f(b + i)));
}

__global__ void gather_felts_kernel(const dfelt* __restrict__ base, const unsigned long long* __restrict__ idx,
                                    size_t n, dfelt* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        st_f(out + i, ld_f(base + idx[i]));
}

__global__ void gather_qm31_kernel(const uint4* __restrict__ base, const unsigned long long* __restrict__ idx,
                                   size_t n, uint4* __restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = base[idx[i]];
}

static unsigned blocks_for(size_t n, int threads, int num_sms) {
    size_t b = (n + threads - 1) / threads;
    const size_t cap = (size_t)num_sms * 64;
    if (b > cap) b = cap;
    if (b == 0) b = 1;
    return (unsigned)b;
}

cudaError_t upload_hades_constants(const void* rc107_mont, const void* r2_mont, const void* two_mont) {
    cudaError_t e = cudaMemcpyToSymbol(c_hades_rc, rc107_mont, sizeof(dfelt) * 107);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_mont_r2, r2_mont, sizeof(dfelt));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_mont_two, two_mont, sizeof(dfelt));
    return e;
}

size_t merkle_padded_leaves(size_t n) {
    size_t p = 2;
    while (p < n) p <<= 1;
    return p;
}

size_t merkle_node_count(size_t n) { return merkle_padded_leaves(n) - 1; }

void launch_merkle_tree(const uint4* leaves, size_t n, void* nodes_v, int num_sms, cudaStream_t s) {
    dfelt* nodes = static_cast<dfelt*>(nodes_v);
    const size_t pn = merkle_padded_leaves(n);
    size_t pairs = pn / 2;
    merkle_leaf_level_kernel<<<blocks_for(pairs, 128, num_sms), 128, 0, s>>>(leaves, n, pairs, nodes);
    dfelt* in = nodes;
    while (pairs > 1) {
        dfelt* out = in + pairs;
        const size_t np = pairs / 2;
        merkle_node_level_kernel<<<blocks_for(np, 128, num_sms), 128, 0, s>>>(in, np, out);
        in = out;
        pairs = np;
    }
}

int merkle_tree_launches(size_t n) {
    const size_t pn = merkle_padded_leaves(n);
    int c = 0;
    for (size_t p = pn / 2; p >= 1; p /= 2) c++;
    return c;
}

void launch_leaf_felts(const uint4* leaves, size_t n, void* out, int num_sms, cudaStream_t s) {
    leaf_felts_kernel<<<blocks_for(n, 256, num_sms), 256, 0, s>>>(leaves, n, static_cast<dfelt*>(out));
}

void launch_hash_pairs(const void* a, const void* b, size_t n, void* out, int num_sms, cudaStream_t s) {
    hash_pairs_kernel<<<blocks_for(n, 128, num_sms), 128, 0, s>>>(static_cast<const dfelt*>(a),
                                                                   static_cast<const dfelt*>(b), n,
                                                                   static_cast<dfelt*>(out));
}

void launch_gather_felts(const void* base, const unsigned long long* idx, size_t n, void* out, cudaStream_t s) {
    gather_felts_kernel<<<blocks_for(n, 128, 148), 128, 0, s>>>(static_cast<const dfelt*>(base), idx, n,
                                                                 static_cast<dfelt*>(out));
}

void launch_gather_qm31(const uint4* base, const unsigned long long* idx, size_t n, uint4* out, cudaStream_t s) {
    gather_qm31_kernel<<<blocks_for(n, 128, 148), 128, 0, s>>>(base, idx, n, out);
}

}  // namespace zk

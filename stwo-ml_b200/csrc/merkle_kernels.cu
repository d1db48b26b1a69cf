// Poseidon-252 Merkle kernels (engine/src/crypto/poseidon_merkle.rs:91-280).
//
// Leaves are securefield_to_felt(v) of QM31 MLE evaluations (no leaf hash),
// internal nodes poseidon_hash(left, right) = hades([left, right, 2])[0], and
// the leaf layer is zero-padded to a power of two (at least 2).  One thread
// computes one node; every level is one launch.  Nodes are stored in
// Montgomery form (identical bytes on host and device).
#include <cuda_runtime.h>

#include <cstring>

#include "felt252.cuh"
#include "felt26.cuh"
#include "merkle.cuh"
#include "qm31.cuh"

namespace zk {

__constant__ dfelt c_mont_r2;  // 2^512 mod p: Montgomery conversion factor

// securefield_to_felt(v) in Montgomery form.
__device__ __forceinline__ dfelt leaf_int(uint4 v) {
    // canonical integer 2^124 | a << 93 | b << 62 | c << 31 | d, as 8 x u32
    dfelt x;
    x.w[0] = v.w | (v.z << 31);
    x.w[1] = (v.z >> 1) | (v.y << 30);
    x.w[2] = (v.y >> 2) | (v.x << 29);
    x.w[3] = (v.x >> 3) | (1u << 28);
    x.w[4] = x.w[5] = x.w[6] = x.w[7] = 0;
    return x;
}

__device__ __forceinline__ dfelt leaf_felt(uint4 v) { return dmul(leaf_int(v), c_mont_r2); }


// 256-bit value in 8 x 32-bit words <-> 10 limbs of 26 bits.
__device__ __forceinline__ f26 f26_from_words(const dfelt& x) {
    f26 a;
#pragma unroll
    for (int i = 0; i < 10; i++) {
        const int b = 26 * i, w = b >> 5, sh = b & 31;
        uint64_t win = x.w[w];
        if (w + 1 < 8) win |= (uint64_t)x.w[w + 1] << 32;
        a.l[i] = (uint32_t)(win >> sh) & F26_MASK;
    }
    return a;
}

__device__ __forceinline__ dfelt f26_to_words(const f26& a) {  // 26-bit limbs, value < 2^256
    dfelt x;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const int b = 32 * w, i = b / 26, sh = b % 26;
        uint64_t win = (uint64_t)a.l[i] >> sh;
        if (i + 1 < 10) win |= (uint64_t)a.l[i + 1] << (26 - sh);
        if (i + 2 < 10) win |= (uint64_t)a.l[i + 2] << (52 - sh);
        x.w[w] = (uint32_t)win;
    }
    return x;
}

// Montgomery (2^256) node value -> Montgomery (2^260) lane: times 16.
__device__ __forceinline__ f26 m256_to_m260(const dfelt& m) {
    f26 a = f26_from_words(m);
#pragma unroll
    for (int i = 0; i < 10; i++) a.l[i] <<= 4;
    return norm26(a);
}

// Montgomery (2^260) lane below 3p -> canonical Montgomery (2^256) node value.
__device__ __forceinline__ dfelt m260_to_m256(const f26& x) {
    const f26 r = mul26(x, c26.one256);  // < 1.01 p, 26-bit limbs
    f26 d = r;
    d.l[0] -= 1;
    d.l[7] -= F26_P7;
    d.l[9] -= F26_P9;
    d = norm26(d);
    return f26_to_words((int32_t)d.l[9] < 0 ? r : d);
}

__device__ __forceinline__ dfelt hash2(const dfelt& l, const dfelt& r) {
    f26 s[3] = {m256_to_m260(l), m256_to_m260(r), c26.two};
    hades26(s);
    return m260_to_m256(s[0]);
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

// securefield_to_felt(v) as a Montgomery (2^260) lane.
__device__ __forceinline__ f26 leaf26(uint4 v) { return mul26(f26_from_words(leaf_int(v)), c26.r2); }

__global__ void __launch_bounds__(128) merkle_leaf_level_kernel(const uint4* __restrict__ leaves, size_t n_leaves,
                                                                size_t n_pairs, dfelt* __restrict__ out) {
    f26 zero;
#pragma unroll
    for (int i = 0; i < 10; i++) zero.l[i] = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n_pairs; i += (size_t)gridDim.x * blockDim.x) {
        const size_t l = 2 * i, r = 2 * i + 1;
        f26 s[3] = {l < n_leaves ? leaf26(leaves[l]) : zero, r < n_leaves ? leaf26(leaves[r]) : zero, c26.two};
        hades26(s);
        st_f(out + i, m260_to_m256(s[0]));
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

// One level of many trees in one launch: job j hashes n_j nodes of its tree from its level
// below (QM31 leaves for level 1, node felts above).  Thread-per-node over the concatenated
// node ranges, so the small levels of small trees share the GPU instead of each paying a
// launch and a full permutation latency of its own.
template <bool LEAF>
__global__ void __launch_bounds__(128) merkle_level_batch_kernel(const MerkleLevelJobs jobs) {
    const unsigned long long total = jobs.start[jobs.count];
    for (unsigned long long idx = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; idx < total;
         idx += (unsigned long long)gridDim.x * blockDim.x) {
        int lo = 0, hi = jobs.count - 1;  // the job with start[j] <= idx < start[j + 1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (jobs.start[mid] <= idx) lo = mid;
            else hi = mid - 1;
        }
        const MerkleLevelJob& jb = jobs.job[lo];
        const unsigned long long i = idx - jobs.start[lo];
        dfelt* out = static_cast<dfelt*>(jb.out);
        if (LEAF) {
            const uint4* leaves = static_cast<const uint4*>(jb.in);
            f26 st[3] = {leaf26(leaves[2 * i]), leaf26(leaves[2 * i + 1]), c26.two};
            hades26(st);
            st_f(out + i, m260_to_m256(st[0]));
        } else {
            const dfelt* in = static_cast<const dfelt*>(jb.in);
            st_f(out + i, hash2(ld_f(in + 2 * i), ld_f(in + 2 * i + 1)));
        }
    }
}

__global__ void scatter_felts_kernel(const dfelt* __restrict__ src, const unsigned long long* __restrict__ idx,
                                     size_t n, dfelt* __restrict__ base) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        st_f(base + idx[i], ld_f(src + i));
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

// ---- host: the radix-2^26 constants -------------------------------------------
namespace {
const uint64_t kP64[4] = {1, 0, 0, 0x0800000000000011ull};

bool geq_p(const uint64_t v[4]) {
    for (int i = 3; i >= 0; i--)
        if (v[i] != kP64[i]) return v[i] > kP64[i];
    return true;
}
void sub_p(uint64_t v[4]) {
    unsigned __int128 br = 0;
    for (int i = 0; i < 4; i++) {
        const unsigned __int128 d = (unsigned __int128)v[i] - kP64[i] - br;
        v[i] = (uint64_t)d;
        br = (d >> 64) & 1;
    }
}
void dbl_modp(uint64_t v[4]) {  // v < p -> 2v mod p
    uint64_t c = 0;
    for (int i = 0; i < 4; i++) {
        const uint64_t n = (v[i] << 1) | c;
        c = v[i] >> 63;
        v[i] = n;
    }
    if (geq_p(v)) sub_p(v);
}
f26 limbs26(const uint64_t v[4]) {
    f26 a;
    for (int i = 0; i < 10; i++) {
        const int b = 26 * i, w = b / 64, sh = b % 64;
        unsigned __int128 win = v[w];
        if (w + 1 < 4) win |= (unsigned __int128)v[w + 1] << 64;
        a.l[i] = (uint32_t)(win >> sh) & F26_MASK;
    }
    return a;
}
f26 times_2k(const void* mont256, int k) {  // value * 2^k mod p, as limbs
    uint64_t v[4];
    memcpy(v, mont256, 32);
    for (int i = 0; i < k; i++) dbl_modp(v);
    return limbs26(v);
}
}  // namespace

cudaError_t upload_hades_constants(const void* rc107_mont, const void* r2_mont, const void* two_mont,
                                   const void* one_mont) {
    cudaError_t e = cudaMemcpyToSymbol(c_mont_r2, r2_mont, sizeof(dfelt));
    if (e != cudaSuccess) return e;
    static F26Consts h;  // Montgomery (2^256) x -> x * 2^260 = value * 16
    const uint64_t* rc = static_cast<const uint64_t*>(rc107_mont);
    for (int i = 0; i < 107; i++) h.rc[i] = times_2k(rc + 4 * i, 4);
    h.two = times_2k(two_mont, 4);
    h.r2 = times_2k(r2_mont, 8);          // 2^512 * 2^8 = 2^520 mod p
    h.one256 = times_2k(one_mont, 0);     // 2^256 mod p
    const uint64_t p4[4] = {4, 0, 0, 4 * 0x0800000000000011ull};
    f26 k = limbs26(p4);                  // 4p < 2^256, then lend 2^28 to every lower limb
    k.l[0] += 1u << 28;
    for (int i = 1; i < 9; i++) k.l[i] += (1u << 28) - 4;
    k.l[9] -= 4;
    h.kp4 = k;
    return cudaMemcpyToSymbol(c26, &h, sizeof(h));
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

// Level-major offset (in felts) of level l >= 1 of a tree over S = 2^k >= 2 leaves.
static inline size_t level_base(size_t S, unsigned l) { return S - (S >> (l - 1)); }

void launch_merkle_subtree(const uint4* leaves, size_t S, size_t lo, size_t cnt, void* nodes_v, int num_sms,
                           cudaStream_t s) {
    dfelt* nodes = static_cast<dfelt*>(nodes_v);
    size_t pairs = cnt / 2;
    dfelt* out = nodes + level_base(S, 1) + lo / 2;
    merkle_leaf_level_kernel<<<blocks_for(pairs, 128, num_sms), 128, 0, s>>>(leaves + lo, cnt, pairs, out);
    unsigned l = 1;
    while (pairs > 1) {
        const dfelt* in = out;
        l++;
        out = nodes + level_base(S, l) + (lo >> l);
        const size_t np = pairs / 2;
        merkle_node_level_kernel<<<blocks_for(np, 128, num_sms), 128, 0, s>>>(in, np, out);
        pairs = np;
    }
}

int merkle_subtree_launches(size_t cnt) {
    int c = 0;
    for (size_t p = cnt / 2; p >= 1; p /= 2) c++;
    return c;
}

void launch_merkle_upper_levels(void* nodes_v, size_t S, unsigned from_level, int num_sms, cudaStream_t s) {
    dfelt* nodes = static_cast<dfelt*>(nodes_v);
    for (unsigned l = from_level + 1; (S >> l) >= 1; l++) {
        const size_t np = S >> l;
        merkle_node_level_kernel<<<blocks_for(np, 128, num_sms), 128, 0, s>>>(nodes + level_base(S, l - 1), np,
                                                                               nodes + level_base(S, l));
        if (np == 1) break;
    }
}

void launch_merkle_level_batch(const MerkleLevelJobs& jobs, bool leaf_level, int num_sms, cudaStream_t s) {
    const unsigned long long total = jobs.start[jobs.count];
    if (total == 0) return;
    if (leaf_level)
        merkle_level_batch_kernel<true><<<blocks_for(total, 128, num_sms), 128, 0, s>>>(jobs);
    else
        merkle_level_batch_kernel<false><<<blocks_for(total, 128, num_sms), 128, 0, s>>>(jobs);
}

void launch_scatter_felts(const void* src, const unsigned long long* idx, size_t n, void* base, cudaStream_t s) {
    scatter_felts_kernel<<<blocks_for(n, 128, 148), 128, 0, s>>>(static_cast<const dfelt*>(src), idx, n,
                                                                  static_cast<dfelt*>(base));
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

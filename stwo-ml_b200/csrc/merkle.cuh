// Host launchers for the Poseidon-252 Merkle kernels (merkle_kernels.cu).
// Node buffers hold 32-byte felts in Montgomery form; a tree over n leaves
// (padded to pn = max(2, next_pow2(n))) stores its pn - 1 internal nodes level
// by level: level 1 (pn/2 nodes), level 2 (pn/4), ..., the root last.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace zk {

cudaError_t upload_hades_constants(const void* rc107_mont, const void* r2_mont, const void* two_mont,
                                   const void* one_mont);
size_t merkle_padded_leaves(size_t n);
size_t merkle_node_count(size_t n);
int merkle_tree_launches(size_t n);
// Full tree over QM31 leaves; nodes must hold merkle_node_count(n) felts.
void launch_merkle_tree(const uint4* leaves, size_t n, void* nodes, int num_sms, cudaStream_t s);
// The subtree over leaves [lo, lo + cnt) of a tree over S leaves (S, cnt powers of two >= 2,
// lo a multiple of cnt): levels 1 .. log2(cnt), written to their places in the full tree's
// level-major node array.
void launch_merkle_subtree(const uint4* leaves, size_t S, size_t lo, size_t cnt, void* nodes, int num_sms,
                           cudaStream_t s);
int merkle_subtree_launches(size_t cnt);
// Levels from_level + 1 .. root of a tree over S leaves (S a power of two), from level from_level.
void launch_merkle_upper_levels(void* nodes, size_t S, unsigned from_level, int num_sms, cudaStream_t s);
// One level of up to MERKLE_MAX_JOBS trees in one launch: job j hashes start[j + 1] - start[j]
// nodes into out from in (QM31 leaves when leaf_level, else node felts of the level below);
// every leaf count is even (no padding).
constexpr int MERKLE_MAX_JOBS = 48;
struct MerkleLevelJob {
    const void* in;
    void* out;
};
struct MerkleLevelJobs {  // a kernel parameter
    MerkleLevelJob job[MERKLE_MAX_JOBS];
    unsigned long long start[MERKLE_MAX_JOBS + 1];
    int count;
};
void launch_merkle_level_batch(const MerkleLevelJobs& jobs, bool leaf_level, int num_sms, cudaStream_t s);
// base[idx[i]] = src[i] (felts).
void launch_scatter_felts(const void* src, const unsigned long long* idx, size_t n, void* base, cudaStream_t s);
// securefield_to_felt of each leaf (Montgomery form).
void launch_leaf_felts(const uint4* leaves, size_t n, void* out, int num_sms, cudaStream_t s);
// out[i] = poseidon_hash(a[i], b[i]).
void launch_hash_pairs(const void* a, const void* b, size_t n, void* out, int num_sms, cudaStream_t s);
void launch_gather_felts(const void* base, const unsigned long long* idx, size_t n, void* out, cudaStream_t s);
void launch_gather_qm31(const uint4* base, const unsigned long long* idx, size_t n, uint4* out, cudaStream_t s);

}  // namespace zk

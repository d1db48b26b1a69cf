// C-ABI: Poseidon Merkle commitment, MLE opening proof and the single-MatMul
// GKR proof with its calldata serialization.
//
// MLE opening (crypto/mle_opening.rs:1654-1916).  The reference commits each
// folded layer root-only and later rebuilds every layer's tree to extract the
// query paths (about 4N Poseidon hashes for N leaves).  Here every layer's full
// tree is kept in HBM from the first pass (about 64 N bytes, 8 GB at N = 2^27),
// so each node is hashed once (about 2N hashes) and the auth paths are gathered
// with one kernel; the proof bytes are identical.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "calldata.hpp"
#include "channel.hpp"
#include "context.hpp"
#include "gkr.cuh"
#include "merkle.cuh"
#include "mesh.hpp"
#include "opening.hpp"

namespace zk {

namespace {

struct dfelt_t {  // a 32-byte node felt, for pointer arithmetic on the tree buffer
    uint32_t w[8];
};

inline size_t next_pow2(size_t x) {
    size_t p = 1;
    while (p < x) p <<= 1;
    return p;
}
inline unsigned ilog2(size_t x) {
    unsigned l = 0;
    while (((size_t)1 << (l + 1)) <= x) l++;
    return l;
}

int dev_view(zkml_ctx* ctx, const void* p, size_t bytes, DevBuf& stage, const void** out) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        if (attr.type == cudaMemoryTypeDevice && attr.device != ctx->device)
            return set_error(ZKML_ERR_INVALID_ARG, "input pointer is device memory of another GPU");
        *out = p;
        return ZKML_OK;
    }
    int rc = stage.ensure(bytes);
    if (rc) return rc;
    ZK_CUDA(cudaMemcpyAsync(stage.ptr, p, bytes, cudaMemcpyHostToDevice, ctx->stream));
    *out = stage.ptr;
    return ZKML_OK;
}

inline void mont_to_canon(const uint32_t w[8], uint64_t out[4]) {
    felt f;
    memcpy(f.l, w, 32);
    f_to_canon(f, out);
}

inline void canon_qm31_felt(const uint32_t v[4], uint64_t out[4]) {
    f_to_canon(felt_of_qm31(qm(v[0], v[1], v[2], v[3])), out);
}

}  // namespace

// Proves the opening of the MLE `evals` (device, 2^n_vars QM31) at `point`,
// appending the serialized MleOpeningProof to `out`.  Advances `chs`.
//
// With a peer mesh of G ranks (G a power of two), every rank folds all layers, but the hashing
// of each layer with at least G x 1024 leaves is split: rank g hashes the subtree over the g-th
// 1/G of the leaves, the G subtree roots of every such layer are all-gathered over the mesh,
// and every rank hashes the top log2(G) levels itself; the auth-path nodes below the subtree
// roots are gathered from their owners the same way.  Every rank ends with the same proof.
int prove_opening_dev(zkml_ctx* ctx, const uint4* evals, unsigned n_vars, const qm31* point, zkml_channel* chs,
                      size_t n_queries_cfg, uint64_t commitment[4], FeltOut& out, uint32_t final_out[4],
                      MeshState* mesh) {
    Channel ch(chs);
    const size_t G = (mesh && mesh->world > 1 && !(mesh->world & (mesh->world - 1))) ? (size_t)mesh->world : 1;
    const size_t grank = G > 1 ? (size_t)mesh->rank : 0;
    constexpr size_t kSplitMinLeaves = 1024;
    if (n_vars + 1 > (unsigned)MERKLE_MAX_JOBS) return set_error(ZKML_ERR_INVALID_ARG, "MLE opening: too many variables");
    cudaStream_t s = ctx->stream;
    const size_t N = (size_t)1 << n_vars;
    OpeningScratch& ob = ctx->op;
    int rc;
    // layer r (r >= 1) of size N >> r lives at offset N - (N >> (r - 1)) in `layers`.
    if ((rc = ob.layers.ensure(N * 16))) return rc;
    std::vector<size_t> tree_off(n_vars + 1, 0), layer_size(n_vars + 1);
    size_t total_nodes = 0;
    for (unsigned r = 0; r <= n_vars; r++) {
        layer_size[r] = N >> r;
        tree_off[r] = total_nodes;
        if (r == 0 || layer_size[r] > 1) total_nodes += merkle_node_count(layer_size[r]);
    }
    if ((rc = ob.trees.ensure(total_nodes * 32))) return rc;
    auto layer_ptr = [&](unsigned r) -> const uint4* {
        return r == 0 ? evals : ob.layers.as<uint4>() + (N - (N >> (r - 1)));
    };
    auto root_index = [&](unsigned r) { return tree_off[r] + merkle_node_count(layer_size[r]) - 1; };
    // All folds and trees are independent of the transcript.  The folds run first (each layer
    // from the previous one); then the trees are hashed level by level, one launch per level
    // for all layers together, so the many small levels do not each pay a launch and a full
    // permutation latency.
    auto is_split = [&](unsigned r) { return G > 1 && layer_size[r] >= G * kSplitMinLeaves; };
    auto sub_level = [&](unsigned r) { return ilog2(layer_size[r] / G); };  // level of the subtree roots
    auto level_base = [&](unsigned r, unsigned l) -> size_t {  // felt offset of level l >= 1 of tree r
        return tree_off[r] + (layer_size[r] - (layer_size[r] >> (l - 1)));
    };
    for (unsigned r = 0; r < n_vars; r++) {
        launch_mle_fold(layer_ptr(r), const_cast<uint4*>(layer_ptr(r + 1)), layer_size[r] / 2, point[r], s);
        ctx->launches++;
    }
    dfelt_t* trees = ob.trees.as<dfelt_t>();
    if (N == 1) {  // a single value: its tree is the leaf and a zero pad
        launch_merkle_tree(layer_ptr(0), 1, ob.trees.as<char>() + 32 * tree_off[0], ctx->num_sms, s);
        ctx->launches += merkle_tree_launches(1);
    }
    unsigned max_levels = 0;
    for (unsigned r = 0; r <= n_vars; r++)
        if (layer_size[r] > 1) max_levels = std::max(max_levels, is_split(r) ? sub_level(r) : ilog2(layer_size[r]));
    for (unsigned l = 1; l <= max_levels; l++) {
        MerkleLevelJobs jobs;
        jobs.count = 0;
        jobs.start[0] = 0;
        for (unsigned r = 0; r <= n_vars; r++) {
            const size_t S = layer_size[r];
            if (S < 2) continue;
            const unsigned top = is_split(r) ? sub_level(r) : ilog2(S);
            if (l > top) continue;
            // this rank's range of the layer: all of it, or its 1/G share when split
            const size_t lo = is_split(r) ? grank * (S / G) : 0;
            const size_t cnt = is_split(r) ? S / G : S;
            MerkleLevelJob& jb = jobs.job[jobs.count];
            jb.in = l == 1 ? static_cast<const void*>(layer_ptr(r) + lo)
                           : static_cast<const void*>(trees + level_base(r, l - 1) + (lo >> (l - 1)));
            jb.out = trees + level_base(r, l) + (lo >> l);
            jobs.start[jobs.count + 1] = jobs.start[jobs.count] + (cnt >> l);
            jobs.count++;
        }
        launch_merkle_level_batch(jobs, l == 1, ctx->num_sms, s);
        ctx->launches++;
    }
    if (G > 1 && is_split(0)) {
        // the subtree roots of every split layer, all-gathered, then the top levels on every rank
        std::vector<unsigned> split_layers;
        for (unsigned r = 0; r <= n_vars; r++)
            if (layer_size[r] > 1 && is_split(r)) split_layers.push_back(r);
        const size_t ne = split_layers.size();
        std::vector<unsigned long long> own_idx(ne), dst_idx(G * ne);
        for (size_t e = 0; e < ne; e++) {
            const unsigned r = split_layers[e];
            const size_t base = level_base(r, sub_level(r));
            own_idx[e] = base + grank;
            for (size_t q = 0; q < G; q++) dst_idx[q * ne + e] = base + q;
        }
        const size_t stage_felts = (ne + 1) & ~(size_t)1;  // a multiple of 16 bytes
        if ((rc = ob.idx.ensure((ne + G * ne) * 8)) || (rc = ob.gathered.ensure((stage_felts + G * stage_felts) * 32)))
            return rc;
        ZK_CUDA(cudaMemcpyAsync(ob.idx.ptr, own_idx.data(), ne * 8, cudaMemcpyHostToDevice, s));
        ZK_CUDA(cudaMemcpyAsync(ob.idx.as<unsigned long long>() + ne, dst_idx.data(), G * ne * 8,
                                cudaMemcpyHostToDevice, s));
        char* stage = ob.gathered.as<char>();
        char* all = stage + 32 * stage_felts;
        launch_gather_felts(ob.trees.ptr, ob.idx.as<unsigned long long>(), ne, stage, s);
        if ((rc = mesh_allgather(ctx, mesh, stage, stage_felts * 32, all))) return rc;
        // rank q's roots sit at all[q * stage_felts + e]: scatter them layer by layer
        for (size_t q = 0; q < G; q++)
            launch_scatter_felts(all + 32 * q * stage_felts, ob.idx.as<unsigned long long>() + ne + q * ne, ne,
                                 ob.trees.ptr, s);
        ctx->launches += 1 + G;
        // the top log2(G) levels of every split tree, one launch per level
        for (unsigned u = 1; (size_t(1) << u) <= G; u++) {
            MerkleLevelJobs jobs;
            jobs.count = 0;
            jobs.start[0] = 0;
            for (unsigned r : split_layers) {
                const unsigned l = sub_level(r) + u;
                MerkleLevelJob& jb = jobs.job[jobs.count];
                jb.in = trees + level_base(r, l - 1);
                jb.out = trees + level_base(r, l);
                jobs.start[jobs.count + 1] = jobs.start[jobs.count] + (layer_size[r] >> l);
                jobs.count++;
            }
            launch_merkle_level_batch(jobs, false, ctx->num_sms, s);
            ctx->launches++;
        }
    }
    // roots (and the final value) to the host
    std::vector<unsigned long long> ridx;
    for (unsigned r = 0; r <= n_vars; r++)
        if (r == 0 || layer_size[r] > 1) ridx.push_back(root_index(r));
    const size_t n_roots = ridx.size();
    if ((rc = ob.idx.ensure(n_roots * 8)) || (rc = ob.gathered.ensure(n_roots * 32))) return rc;
    ZK_CUDA(cudaMemcpyAsync(ob.idx.ptr, ridx.data(), n_roots * 8, cudaMemcpyHostToDevice, s));
    launch_gather_felts(ob.trees.ptr, ob.idx.as<unsigned long long>(), n_roots, ob.gathered.ptr, s);
    ctx->launches++;
    std::vector<uint32_t> roots_m(n_roots * 8);
    uint32_t fin[4];
    ZK_CUDA(cudaMemcpyAsync(roots_m.data(), ob.gathered.ptr, n_roots * 32, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaMemcpyAsync(fin, layer_ptr(n_vars), 16, cudaMemcpyDeviceToHost, s));
    ZK_CUDA(cudaStreamSynchronize(s));
    std::vector<uint64_t> roots(n_roots * 4);
    for (size_t i = 0; i < n_roots; i++) mont_to_canon(&roots_m[8 * i], &roots[4 * i]);
    memcpy(commitment, &roots[0], 32);
    for (size_t i = 0; i < n_roots; i++) ch.mix_m(f_from_canon(&roots[4 * i]));
    // queries
    const size_t half_n = N / 2;
    const size_t nq = n_queries_cfg < half_n ? n_queries_cfg : half_n;
    std::vector<size_t> qidx(nq);
    for (size_t q = 0; q < nq; q++) {
        uint64_t f[4];
        ch.draw_canon(f);
        qidx[q] = (size_t)(f[0] % half_n);
    }
    // gather values and siblings: per (q, r): left/right values and their sibling leaves,
    // then the internal-node siblings of both paths.
    std::vector<unsigned long long> node_idx;
    std::vector<int> node_owner;  // the rank whose subtree holds the node, -1: every rank has it
    std::vector<std::vector<unsigned long long>> val_idx(n_vars);
    std::vector<size_t> cur(qidx);
    for (unsigned r = 0; r < n_vars; r++) {
        const size_t S = layer_size[r], mid = S / 2, depth = ilog2(merkle_padded_leaves(S));
        for (size_t q = 0; q < nq; q++) {
            const size_t li = cur[q], ri = mid + cur[q];
            val_idx[r].push_back(li);
            val_idx[r].push_back(ri);
            val_idx[r].push_back(li ^ 1);
            val_idx[r].push_back(ri ^ 1);
            for (size_t x : {li, ri})
                for (size_t l = 1; l < depth; l++) {
                    const size_t xi = (x >> l) ^ 1;
                    node_idx.push_back(tree_off[r] + (S - (S >> (l - 1))) + xi);
                    node_owner.push_back(is_split(r) && l < sub_level(r) ? (int)(xi / ((S / G) >> l)) : -1);
                }
            const size_t next_half = mid / 2 > 0 ? mid / 2 : 1;
            cur[q] %= next_half;
        }
    }
    size_t n_vals = 0;
    for (auto& v : val_idx) n_vals += v.size();
    const size_t n_nodes = node_idx.size();
    if ((rc = ob.idx.ensure((n_nodes + n_vals + 1) * 8)) || (rc = ob.gathered.ensure((n_nodes + 1) * 32)) ||
        (rc = ob.qvals.ensure((n_vals + 1) * 16)))
        return rc;
    std::vector<unsigned long long> all_idx(node_idx);
    for (auto& v : val_idx) all_idx.insert(all_idx.end(), v.begin(), v.end());
    if (!all_idx.empty())
        ZK_CUDA(cudaMemcpyAsync(ob.idx.ptr, all_idx.data(), all_idx.size() * 8, cudaMemcpyHostToDevice, s));
    if (n_nodes) {
        launch_gather_felts(ob.trees.ptr, ob.idx.as<unsigned long long>(), n_nodes, ob.gathered.ptr, s);
        ctx->launches++;
    }
    size_t off = n_nodes;
    for (unsigned r = 0; r < n_vars; r++) {
        if (val_idx[r].empty()) continue;
        launch_gather_qm31(layer_ptr(r), ob.idx.as<unsigned long long>() + off, val_idx[r].size(),
                           ob.qvals.as<uint4>() + (off - n_nodes), s);
        ctx->launches++;
        off += val_idx[r].size();
    }
    std::vector<uint32_t> nodes_m(n_nodes * 8 + 8), vals(n_vals * 4 + 4);
    bool foreign = false;
    for (int o : node_owner) foreign |= o >= 0 && (size_t)o != grank;
    if (foreign) {
        // every rank's gathered nodes over the mesh; each node is taken from its owner
        const size_t padded = (n_nodes + 1) & ~(size_t)1;
        DevBuf& allb = ob.nodes;
        if ((rc = allb.ensure(G * padded * 32))) return rc;
        if ((rc = mesh_allgather(ctx, mesh, ob.gathered.ptr, padded * 32, allb.ptr))) return rc;
        std::vector<uint32_t> all(G * padded * 8);
        ZK_CUDA(cudaMemcpyAsync(all.data(), allb.ptr, G * padded * 32, cudaMemcpyDeviceToHost, s));
        if (n_vals) ZK_CUDA(cudaMemcpyAsync(vals.data(), ob.qvals.ptr, n_vals * 16, cudaMemcpyDeviceToHost, s));
        ZK_CUDA(cudaStreamSynchronize(s));
        for (size_t i = 0; i < n_nodes; i++) {
            const size_t from = node_owner[i] >= 0 ? (size_t)node_owner[i] : grank;
            memcpy(&nodes_m[8 * i], &all[8 * (from * padded + i)], 32);
        }
    } else {
        if (n_nodes) ZK_CUDA(cudaMemcpyAsync(nodes_m.data(), ob.gathered.ptr, n_nodes * 32, cudaMemcpyDeviceToHost, s));
        if (n_vals) ZK_CUDA(cudaMemcpyAsync(vals.data(), ob.qvals.ptr, n_vals * 16, cudaMemcpyDeviceToHost, s));
        ZK_CUDA(cudaStreamSynchronize(s));
    }
    if (G > 1 && (rc = mesh_check(ctx))) return rc;
    // serialize (cairo_serde::serialize_mle_opening_proof): query-major
    out.u64(n_roots - 1);
    for (size_t i = 1; i < n_roots; i++) out.push(&roots[4 * i]);
    out.u64(nq);
    // per-round offsets into the gathered arrays
    std::vector<size_t> node_base(n_vars + 1, 0), val_base(n_vars + 1, 0);
    for (unsigned r = 0; r < n_vars; r++) {
        const size_t depth = ilog2(merkle_padded_leaves(layer_size[r]));
        node_base[r + 1] = node_base[r] + nq * 2 * (depth - 1);
        val_base[r + 1] = val_base[r] + val_idx[r].size();
    }
    for (size_t q = 0; q < nq; q++) {
        out.u64(qidx[q]);
        out.u64(n_vars);
        for (unsigned r = 0; r < n_vars; r++) {
            const size_t depth = ilog2(merkle_padded_leaves(layer_size[r]));
            const uint32_t* v = &vals[4 * (val_base[r] + 4 * q)];
            out.qm(v);      // left value
            out.qm(v + 4);  // right value
            for (int side = 0; side < 2; side++) {
                out.u64(depth);
                uint64_t f[4];
                canon_qm31_felt(v + 8 + 4 * side, f);  // sibling leaf
                out.push(f);
                const size_t nb = node_base[r] + (q * 2 + side) * (depth - 1);
                for (size_t l = 1; l < depth; l++) {
                    mont_to_canon(&nodes_m[8 * (nb + l - 1)], f);
                    out.push(f);
                }
            }
        }
    }
    out.qm(fin);
    if (final_out) memcpy(final_out, fin, 16);
    return ZKML_OK;
}

}  // namespace zk

using namespace zk;

extern "C" {

int zkml_commit_mle_root(zkml_ctx* ctx, const uint32_t* evals, size_t n, uint64_t out_root[4]) {
    if (!ctx || !evals || !out_root || n == 0) return set_error(ZKML_ERR_INVALID_ARG, "NULL or empty argument");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const void* E = nullptr;
    int rc = dev_view(ctx, evals, n * 16, ctx->a_in, &E);
    if (rc) return rc;
    DevBuf& nodes = ctx->op.nodes;
    if ((rc = nodes.ensure(merkle_node_count(n) * 32))) return rc;
    {
        KTimer t(ctx, KC_MERKLE);
        launch_merkle_tree(static_cast<const uint4*>(E), n, nodes.ptr, ctx->num_sms, ctx->stream);
    }
    ctx->launches += merkle_tree_launches(n);
    uint32_t root[8];
    cudaError_t e = cudaMemcpyAsync(root, nodes.as<char>() + 32 * (merkle_node_count(n) - 1), 32,
                                    cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_error(e, "commit_mle_root");
    mont_to_canon(root, out_root);
    return ZKML_OK;
}

int zkml_prove_mle_opening(zkml_ctx* ctx, const uint32_t* evals, size_t n_vars, const uint32_t* point,
                           zkml_channel* ch, size_t n_queries, uint64_t out_commitment[4], uint64_t* out_calldata,
                           size_t cap, size_t* out_len) {
    if (!ctx || !evals || !ch || !out_commitment || !out_len || (n_vars && !point))
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (n_vars > 34) return set_error(ZKML_ERR_INVALID_ARG, "too many variables");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const void* E = nullptr;
    int rc = dev_view(ctx, evals, ((size_t)16) << n_vars, ctx->a_in, &E);
    if (rc) return rc;
    FeltOut out{out_calldata, out_calldata ? cap : 0};
    {
        KTimer t(ctx, KC_MERKLE);
        rc = prove_opening_dev(ctx, static_cast<const uint4*>(E), (unsigned)n_vars,
                               reinterpret_cast<const qm31*>(point), ch, n_queries, out_commitment, out, nullptr);
    }
    if (rc) return rc;
    *out_len = out.len;
    if (out.overflow) return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " +
                                                                 std::to_string(out.len) + " felts");
    return ZKML_OK;
}

int zkml_io_commitment(const uint32_t* input, size_t in_rows, size_t in_cols, const uint32_t* output,
                       size_t out_rows, size_t out_cols, uint64_t out[4]) {
    if (!input || !output || !out) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    felt_init();
    std::vector<felt> v;
    v.reserve(6 + in_rows * in_cols + out_rows * out_cols);
    v.push_back(f_from_u64(in_rows));
    v.push_back(f_from_u64(in_cols));
    v.push_back(f_from_u64(in_rows * in_cols));
    for (size_t i = 0; i < in_rows * in_cols; i++) v.push_back(f_from_u64(input[i]));
    v.push_back(f_from_u64(out_rows));
    v.push_back(f_from_u64(out_cols));
    v.push_back(f_from_u64(out_rows * out_cols));
    for (size_t i = 0; i < out_rows * out_cols; i++) v.push_back(f_from_u64(output[i]));
    f_to_canon(poseidon_hash_many_m(v.data(), v.size()), out);
    return ZKML_OK;
}

int zkml_prove_gkr_matmul(zkml_ctx* ctx, const uint32_t* input, size_t m, size_t k, const uint32_t* weight, size_t n,
                          const uint64_t* policy, size_t n_queries, uint64_t* out_calldata, size_t cap,
                          size_t* out_len, uint64_t out_digest[4], uint64_t out_io[4]) {
    if (!ctx || !input || !weight || !out_len || !out_digest || !out_io)
        return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (m == 0 || k == 0 || n == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty matrix");
    if (m > (1u << 30) || k > (1u << 30) || n > (1u << 30))
        return set_error(ZKML_ERR_INVALID_ARG, "matrix dimension exceeds 2^30");
    ZK_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    const size_t pm = next_pow2(m), pk = next_pow2(k), pn = next_pow2(n);
    const unsigned log_m = ilog2(pm), log_k = ilog2(pk), log_n = ilog2(pn);
    const void* Av = nullptr;
    const void* Bv = nullptr;
    int rc = dev_view(ctx, input, m * k * 4, ctx->a_in, &Av);
    if (!rc) rc = dev_view(ctx, weight, k * n * 4, ctx->b_in, &Bv);
    if (rc) return rc;
    const uint32_t* A = static_cast<const uint32_t*>(Av);
    const uint32_t* B = static_cast<const uint32_t*>(Bv);

    zkml_channel chs;
    zkml_channel_init(&chs);
    Channel ch(&chs);
    // prove_gkr_with_cache prefix (gkr/prover.rs:1516-1537): depth, input shape, policy
    ch.mix_u64(1);
    ch.mix_u64(m);
    ch.mix_u64(k);
    if (policy && (policy[0] | policy[1] | policy[2] | policy[3])) ch.mix_m(f_from_canon(policy));
    // output claim at r_out (prover.rs:1543-1561).  The output MLE at (r_i, r_j) equals
    // sum_k f_a[k] f_b[k] of the restricted operands, so the restriction runs first and
    // the value is read from the first round's p(0) + p(1).
    std::vector<qm31> r_out(log_m + log_n + 1);
    for (unsigned i = 0; i < log_m + log_n; i++) r_out[i] = ch.draw_qm31();
    // output matrix for the IO commitment (forward pass on the GPU)
    DevBuf& cbuf = ctx->op.cbuf;
    DevBuf& bmle = ctx->op.bmle;
    if ((rc = cbuf.ensure(m * n * 4))) return rc;
    launch_m31_gemm(A, B, cbuf.as<uint32_t>(), (uint32_t)m, (uint32_t)k, (uint32_t)n, s);
    ctx->launches++;
    std::vector<uint32_t> out_host(m * n);
    ZK_CUDA(cudaMemcpyAsync(out_host.data(), cbuf.ptr, m * n * 4, cudaMemcpyDeviceToHost, s));
    // The value is known once the restriction and round 0 ran; the hook then
    // performs the output-claim mix and the matmul layer's seeding mixes
    // (reduce_matmul_layer_with_backend, gkr/prover.rs:5996-5999) before round 0's
    // polynomial enters the transcript.
    struct HookState {
        Channel* ch;
        size_t m, k, n;
        qm31 value;
    } hs{&ch, m, k, n, qzero()};
    ClaimHook hook;
    hook.arg = &hs;
    hook.fn = [](void* arg, const qm31& v) {
        HookState* h = static_cast<HookState*>(arg);
        h->value = v;
        h->ch->mix_qm31(v);  // output claim (prover.rs:1560)
        h->ch->mix_u64(h->m);
        h->ch->mix_u64(h->k);
        h->ch->mix_u64(h->n);
        h->ch->mix_qm31(v);  // the matmul layer's claimed value
    };
    std::vector<uint32_t> rps(12 * (log_k + 1)), chal(4 * (log_k + 1)), next_pt(4 * (log_m + log_k + 1));
    uint32_t fa[4], fb[4];
    rc = reduce_matmul_internal(ctx, A, m, k, B, k, n, reinterpret_cast<const uint32_t*>(r_out.data()), log_m,
                                reinterpret_cast<const uint32_t*>(r_out.data() + log_m), log_n, pk, &chs, rps.data(),
                                chal.data(), fa, fb, &hook);
    if (rc) return rc;
    ch.mix_qm31(qm(fa[0], fa[1], fa[2], fa[3]));
    ch.mix_qm31(qm(fb[0], fb[1], fb[2], fb[3]));
    memcpy(next_pt.data(), r_out.data(), 16 * log_m);
    memcpy(next_pt.data() + 4 * log_m, chal.data(), 16 * log_k);

    FeltOut out{out_calldata, out_calldata ? cap : 0};
    out.u64(1);  // layer proofs
    out.u64(0);  // tag MatMul
    out.u64(log_k);
    for (unsigned r = 0; r < log_k; r++) {
        out.qm(&rps[12 * r]);      // c0
        out.qm(&rps[12 * r + 8]);  // c2 (c1 is implied by the claim)
    }
    out.qm(fa);
    out.qm(fb);
    out.u64(log_m + log_k);  // input claim
    for (unsigned i = 0; i < log_m + log_k; i++) out.qm(&next_pt[4 * i]);
    out.qm(fa);
    // weight opening (Sequential mode): col-major padded B MLE at r_j || challenges
    if ((rc = bmle.ensure(pk * pn * 16))) return rc;
    launch_colmajor_mle(B, (uint32_t)k, (uint32_t)n, pk, pn, bmle.as<uint4>(), s);
    ctx->launches++;
    std::vector<qm31> wpt(log_n + log_k + 1);
    for (unsigned i = 0; i < log_n; i++) wpt[i] = r_out[log_m + i];
    for (unsigned i = 0; i < log_k; i++)
        wpt[log_n + i] = qm(next_pt[4 * (log_m + i)], next_pt[4 * (log_m + i) + 1], next_pt[4 * (log_m + i) + 2],
                            next_pt[4 * (log_m + i) + 3]);
    uint64_t commitment[4];
    FeltOut opening{nullptr, 0};
    std::vector<uint64_t> obuf;
    // size the opening buffer: generous upper bound
    const unsigned nv = log_n + log_k;
    const size_t qcap = 16 + (n_queries + 1) * (2 + (size_t)nv * (10 + 2 * (nv + 1))) + 64;
    obuf.resize(qcap * 4);
    opening.buf = obuf.data();
    opening.cap = qcap;
    {
        KTimer t(ctx, KC_MERKLE);
        rc = prove_opening_dev(ctx, bmle.as<uint4>(), nv, wpt.data(), &chs, n_queries, commitment, opening, nullptr);
    }
    if (rc) return rc;
    out.u64(1);  // weight commitments
    out.push(commitment);
    out.u64(1);  // weight openings
    out.u64(nv);
    for (unsigned i = 0; i < nv; i++) {
        const uint32_t w[4] = {wpt[i].a, wpt[i].b, wpt[i].c, wpt[i].d};
        out.qm(w);
    }
    out.qm(fb);
    for (size_t i = 0; i < opening.len; i++) out.push(&obuf[4 * i]);
    // IO commitment (aggregation.rs:235-254)
    ZK_CUDA(cudaStreamSynchronize(s));
    std::vector<uint32_t> in_host(m * k);
    ZK_CUDA(cudaMemcpy(in_host.data(), A, m * k * 4, cudaMemcpyDeviceToHost));
    zkml_io_commitment(in_host.data(), m, k, out_host.data(), m, n, out_io);
    out.push(out_io);
    memcpy(out_digest, chs.digest, 32);
    *out_len = out.len;
    if (out.overflow)
        return set_error(ZKML_ERR_INVALID_ARG, "calldata buffer too small: need " + std::to_string(out.len) + " felts");
    return ZKML_OK;
}

}  // extern "C"

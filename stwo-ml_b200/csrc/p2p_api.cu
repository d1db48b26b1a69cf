// Column-block sharded matmul layer with the partial-f_b exchange over peer memory
// (NVLink / NVSwitch) instead of a collective library.
//
// Each rank owns an inbox in its HBM: world slots of 4k u64 words plus world flag words,
// exported with a CUDA IPC handle and mapped by every other rank.  After its block
// restriction, a rank's scatter kernel canonicalises its 4k partial words and stores them
// straight into slot [rank] of every rank's inbox (peer stores), then, once all of its
// blocks have fenced their stores, publishes the call's epoch in flag [rank] of every inbox
// with a system-scope release.  The consuming kernel on each rank waits (bounded) for all
// flags to reach the epoch and adds the slots into the f_b words the layer's sumcheck
// starts from.  No host step sits between the two kernels.
//
// Every wait is bounded: a rank that never publishes makes the others' gather kernels give
// up after about two seconds, record the timeout in the error flag and return, so the
// call fails with ZKML_ERR_TIMEOUT and the GPU stays usable.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "context.hpp"

namespace zk {
namespace {

struct P2PState {
    int world = 0, rank = -1;
    size_t words = 0;                // u64 words per slot (4 k)
    void* own = nullptr;             // this rank's inbox allocation
    std::vector<uint8_t*> peers;     // every rank's inbox (own included), as mapped here
    uint32_t scattered = 0;          // epoch of this rank's last scatter
    uint32_t gathered = 0;           // epoch of this rank's last gather
};

std::vector<P2PState>& states() {
    static std::vector<P2PState> s(64);
    return s;
}

// inbox layout, double-buffered by epoch parity: [2][world][words] u64 slots, then
// [2][world] u32 flags, then one u32 ticket.  A rank starts call e + 2 only after its call
// e + 1 saw every rank's scatter of e + 1, and each rank issues that scatter after its
// gather of call e on the same stream; so no rank writes a parity half that another rank
// is still reading.
inline size_t slots_bytes(size_t world, size_t words) { return 2 * world * words * 8; }
inline size_t inbox_bytes(size_t world, size_t words) { return slots_bytes(world, words) + 8 * world + 64; }

struct PeerPtrs {
    uint8_t* p[8];
};

// Canonical partial words of this rank, stored into slot [rank] of every inbox; the last
// block to finish publishes `epoch` in flag [rank] of every inbox.
__global__ void p2p_scatter_kernel(const unsigned long long* __restrict__ acc, size_t words, PeerPtrs peers,
                                   int world, int rank, uint32_t epoch, unsigned int* ticket, size_t flags_off) {
    const size_t slot = ((size_t)(epoch & 1) * world + rank) * words;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words; i += (size_t)gridDim.x * blockDim.x) {
        const unsigned long long w = red64(acc[i]);
        for (int r = 0; r < world; r++) reinterpret_cast<unsigned long long*>(peers.p[r])[slot + i] = w;
    }
    __threadfence_system();
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    *ticket = 0;
    __threadfence_system();
    for (int r = 0; r < world; r++) {
        uint32_t* f = reinterpret_cast<uint32_t*>(peers.p[r] + flags_off) + (epoch & 1) * world + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
    }
}

// Waits (bounded) until every flag of this rank's inbox equals `epoch`, then
// out[i] = sum over slots of the words.  err bit 4: a rank did not publish in time.
__global__ void p2p_gather_kernel(const uint8_t* inbox, size_t words, int world, uint32_t epoch, size_t flags_off,
                                  unsigned long long* __restrict__ out, uint32_t* err) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = 1;
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(inbox + flags_off) + (epoch & 1) * world;
        for (int r = 0; r < world && ok; r++) {
            uint32_t v = 0;
            long long it = 0;
            for (;; it++) {
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
                if (v == epoch) break;
                if (it > (1ll << 24)) {  // ~2 s with the back-off below
                    ok = 0;
                    atomicOr(err, 16u);
                    break;
                }
                __nanosleep(100);
            }
        }
    }
    __syncthreads();
    const unsigned long long* slots =
        reinterpret_cast<const unsigned long long*>(inbox) + (size_t)(epoch & 1) * world * words;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words; i += (size_t)gridDim.x * blockDim.x) {
        unsigned long long s = 0;
        if (ok)
            for (int r = 0; r < world; r++) s += __ldcv(slots + (size_t)r * words + i);
        out[i] = s;
    }
}

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" {

int zkml_p2p_inbox_create(zkml_ctx* ctx, size_t k, int world, int rank, uint8_t out_handle[64]) {
    if (!ctx || !out_handle || world < 1 || world > 8 || rank < 0 || rank >= world || k == 0)
        return set_error(ZKML_ERR_INVALID_ARG, "p2p inbox: bad arguments (1 to 8 ranks)");
    P2PState& st = states()[ctx->device % 64];
    if (st.own) return set_error(ZKML_ERR_INVALID_ARG, "p2p inbox already created on this device");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const size_t words = 4 * k;
    ZK_CUDA(cudaMalloc(&st.own, inbox_bytes(world, words)));
    ZK_CUDA(cudaMemset(st.own, 0, inbox_bytes(world, words)));
    cudaIpcMemHandle_t h;
    ZK_CUDA(cudaIpcGetMemHandle(&h, st.own));
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(out_handle, &h, 64);
    st.world = world;
    st.rank = rank;
    st.words = words;
    st.peers.assign(world, nullptr);
    st.peers[rank] = static_cast<uint8_t*>(st.own);
    return ZKML_OK;
}

int zkml_p2p_open(zkml_ctx* ctx, const uint8_t* handles, int world) {
    if (!ctx || !handles) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    P2PState& st = states()[ctx->device % 64];
    if (!st.own || st.world != world) return set_error(ZKML_ERR_INVALID_ARG, "p2p inbox not created for this world");
    ZK_CUDA(cudaSetDevice(ctx->device));
    for (int r = 0; r < world; r++) {
        if (r == st.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + 64 * r, 64);
        void* p = nullptr;
        ZK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        st.peers[r] = static_cast<uint8_t*>(p);
    }
    return ZKML_OK;
}

int zkml_p2p_close(zkml_ctx* ctx) {
    if (!ctx) return ZKML_OK;
    P2PState& st = states()[ctx->device % 64];
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < (int)st.peers.size(); r++)
        if (r != st.rank && st.peers[r]) cudaIpcCloseMemHandle(st.peers[r]);
    if (st.own) cudaFree(st.own);
    st = P2PState();
    return ZKML_OK;
}

int zkml_restrict_cols_block_p2p(zkml_ctx* ctx, const uint32_t* b_block, size_t k, size_t n_block, size_t col_offset,
                                 const uint32_t* r_j, size_t n_rj, uint32_t epoch) {
    if (!ctx) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    P2PState& st = states()[ctx->device % 64];
    if (!st.own || st.words != 4 * k) return set_error(ZKML_ERR_INVALID_ARG, "p2p inbox not created for this k");
    for (int r = 0; r < st.world; r++)
        if (!st.peers[r]) return set_error(ZKML_ERR_INVALID_ARG, "p2p peers not opened");
    // The flags start at 0, so epoch 0 would pass every wait at once; and the parity double
    // buffer is safe only if call e + 1's scatter follows call e's gather on this context.
    if (epoch == 0 || epoch != st.gathered + 1 || st.scattered != st.gathered)
        return set_error(ZKML_ERR_INVALID_ARG, "p2p scatter: epochs start at 1 and go up by one per call, each "
                                               "call's scatter after the previous call's gather (expected " +
                                                   std::to_string(st.gathered + 1) + ", got " +
                                                   std::to_string(epoch) + ")");
    int rc;
    if ((rc = ctx->acc_b.ensure(k * 32))) return rc;
    unsigned long long* acc = ctx->acc_b.as<unsigned long long>();
    if (n_block) {
        if ((rc = zkml_restrict_cols_block(ctx, b_block, k, n_block, col_offset, r_j, n_rj,
                                           reinterpret_cast<uint64_t*>(acc))))
            return rc;
    } else {
        ZK_CUDA(cudaMemsetAsync(acc, 0, k * 32, ctx->stream));
    }
    PeerPtrs pp{};
    for (int r = 0; r < st.world; r++) pp.p[r] = st.peers[r];
    const size_t words = st.words, flags_off = slots_bytes(st.world, words);
    unsigned int* ticket = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(st.own) + flags_off + 8 * st.world);
    const unsigned g = (unsigned)std::min<size_t>((words + 255) / 256, (size_t)ctx->num_sms * 4);
    p2p_scatter_kernel<<<g, 256, 0, ctx->stream>>>(acc, words, pp, st.world, st.rank, epoch, ticket, flags_off);
    ctx->launches++;
    ZK_CUDA(cudaGetLastError());
    st.scattered = epoch;
    return ZKML_OK;
}

int zkml_reduce_matmul_layer_gkr_p2p(zkml_ctx* ctx, const uint32_t* claim_point, size_t n_point,
                                     const uint32_t claim_value[4], const uint32_t* a, size_t m, size_t k, size_t n,
                                     uint32_t epoch, zkml_channel* chs, uint32_t* out_round_polys,
                                     uint32_t out_final_a[4], uint32_t out_final_b[4], uint32_t* out_next_point) {
    if (!ctx) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    P2PState& st = states()[ctx->device % 64];
    if (!st.own || st.words != 4 * k) return set_error(ZKML_ERR_INVALID_ARG, "p2p inbox not created for this k");
    if (epoch == 0 || epoch != st.scattered || st.gathered + 1 != epoch)
        return set_error(ZKML_ERR_INVALID_ARG, "p2p gather: epoch must be the one this rank scattered last (" +
                                                   std::to_string(st.scattered) + "), got " + std::to_string(epoch));
    st.gathered = epoch;
    int rc;
    if ((rc = ctx->acc_a.ensure(k * 32))) return rc;  // acc_a is free until the layer's row restriction
    DevBuf& words = ctx->op.gpart;
    if ((rc = words.ensure(k * 32))) return rc;
    const size_t flags_off = slots_bytes(st.world, st.words);
    const unsigned g = (unsigned)std::min<size_t>((st.words + 255) / 256, (size_t)ctx->num_sms * 4);
    p2p_gather_kernel<<<g, 256, 0, ctx->stream>>>(static_cast<const uint8_t*>(st.own), st.words, st.world, epoch,
                                                  flags_off, words.as<unsigned long long>(), ctx->err_flag());
    ctx->launches++;
    ZK_CUDA(cudaGetLastError());
    if ((rc = read_err_flag(ctx))) return rc;
    if (ctx->h_small[48] & 16u) {
        ctx->h_small[48] = 0;
        ZK_CUDA(cudaMemsetAsync(ctx->err_flag(), 0, 4, ctx->stream));
        return set_error(ZKML_ERR_TIMEOUT, "p2p gather: a rank did not publish its partial words in time");
    }
    return zkml_reduce_matmul_layer_gkr_fb(ctx, claim_point, n_point, claim_value, a, m, k,
                                           reinterpret_cast<const uint64_t*>(words.ptr), n, chs, out_round_polys,
                                           out_final_a, out_final_b, out_next_point);
}

}  // extern "C"

// C-ABI: the peer-memory mesh between the ranks of one node (one process per GPU).
//
// zkml_mesh_create allocates this rank's inbox and returns its CUDA IPC handle; after the
// ranks have exchanged the handles (through their process group), zkml_mesh_open maps every
// peer's inbox.  The sharded product sumcheck then exchanges its round words inside the round
// kernels (mesh_allreduce12: peer stores of 12 words, a release flag per rank, a bounded
// acquire wait) and gathers its folded vectors with one scatter kernel of plain peer stores
// plus one bounded wait: no host step and no collective library on the data path.
#include <algorithm>
#include <cstring>
#include <string>

#include "mesh.hpp"

namespace zk {
namespace {

MeshState g_mesh[64];

// Copies `words` u32 of `local` into slot [rank] of every inbox's gather region; the grid's
// last block publishes the epoch in gather flag [rank] of every inbox (system-scope release).
__global__ void mesh_scatter_kernel(const uint4* __restrict__ local, size_t n16, const MeshDesc* d, size_t slot_bytes,
                                    uint32_t epoch) {
    const uint32_t world = d->world, rank = d->rank;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 v = local[i];
        for (uint32_t r = 0; r < world; r++)
            reinterpret_cast<uint4*>(d->peers[r] + MESH_DATA_OFF + rank * slot_bytes)[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    __shared__ bool last;
    unsigned int* ticket = reinterpret_cast<unsigned int*>(d->peers[rank] + MESH_TICKET_OFF);
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    *ticket = 0;
    __threadfence_system();
    for (uint32_t r = 0; r < world; r++) {
        uint32_t* f = reinterpret_cast<uint32_t*>(d->peers[r] + MESH_GFLAGS_OFF) + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
    }
}

// Waits (bounded) for every rank's gather flag, then copies the rank-major slots to out.
__global__ void mesh_collect_kernel(const MeshDesc* d, size_t n16, size_t slot_bytes, uint32_t epoch,
                                    uint4* __restrict__ out) {
    __shared__ int ok;
    const uint32_t world = d->world;
    const uint8_t* own = d->peers[d->rank];
    if (threadIdx.x == 0) {
        ok = 1;
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(own + MESH_GFLAGS_OFF);
        for (uint32_t r = 0; r < world && ok; r++) {
            uint32_t v = 0;
            for (long long it = 0;; it++) {
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
                if (v == epoch) break;
                if (it > (1ll << 24)) {  // ~2 s with the back-off below
                    ok = 0;
                    atomicOr(d->err, MESH_ERR_TIMEOUT);
                    break;
                }
                __nanosleep(100);
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    const size_t total = n16 * world;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / n16, j = i % n16;
        out[i] = __ldcv(reinterpret_cast<const uint4*>(own + MESH_DATA_OFF + r * slot_bytes) + j);
    }
}

}  // namespace

MeshState* mesh_of(::zkml_ctx* ctx) {
    MeshState& m = g_mesh[ctx->device % 64];
    return m.open ? &m : nullptr;
}

MeshArg mesh_next(MeshState* m) { return MeshArg{m->d_desc, ++m->epoch}; }

int mesh_allgather(::zkml_ctx* ctx, MeshState* m, const void* local, size_t bytes, void* out) {
    if (bytes % 16 || bytes > m->gather_bytes)
        return set_error(ZKML_ERR_INVALID_ARG, "mesh gather: " + std::to_string(bytes) +
                                                   " bytes per rank (a multiple of 16, at most " +
                                                   std::to_string(m->gather_bytes) + ")");
    const uint32_t epoch = ++m->epoch;
    const size_t n16 = bytes / 16;
    const unsigned g = (unsigned)std::max<size_t>(1, std::min<size_t>((n16 + 255) / 256, (size_t)ctx->num_sms * 4));
    mesh_scatter_kernel<<<g, 256, 0, ctx->stream>>>(static_cast<const uint4*>(local), n16, m->d_desc, m->gather_bytes,
                                                   epoch);
    const unsigned g2 =
        (unsigned)std::max<size_t>(1, std::min<size_t>((n16 * m->world + 255) / 256, (size_t)ctx->num_sms * 4));
    mesh_collect_kernel<<<g2, 256, 0, ctx->stream>>>(m->d_desc, n16, m->gather_bytes, epoch, static_cast<uint4*>(out));
    ctx->launches += 2;
    ZK_CUDA(cudaGetLastError());
    return ZKML_OK;
}

int mesh_check(::zkml_ctx* ctx) {
    int rc = read_err_flag(ctx);
    if (rc) return rc;
    if (ctx->h_small[48] & MESH_ERR_TIMEOUT) {
        ctx->h_small[48] &= ~MESH_ERR_TIMEOUT;
        ZK_CUDA(cudaMemsetAsync(ctx->err_flag(), 0, 4, ctx->stream));
        return set_error(ZKML_ERR_TIMEOUT, "mesh: a rank did not arrive within about two seconds");
    }
    return ZKML_OK;
}

}  // namespace zk

using namespace zk;

extern "C" {

int zkml_mesh_create(zkml_ctx* ctx, int world, int rank, size_t max_gather_bytes, uint8_t out_handle[64]) {
    if (!ctx || !out_handle || world < 1 || world > MESH_MAX_RANKS || rank < 0 || rank >= world)
        return set_error(ZKML_ERR_INVALID_ARG, "mesh: bad arguments (1 to 8 ranks)");
    MeshState& m = g_mesh[ctx->device % 64];
    if (m.own) return set_error(ZKML_ERR_INVALID_ARG, "mesh already created on this device");
    ZK_CUDA(cudaSetDevice(ctx->device));
    const size_t gb = (max_gather_bytes + 255) / 256 * 256;
    const size_t bytes = MESH_DATA_OFF + (size_t)world * gb;
    ZK_CUDA(cudaMalloc(&m.own, bytes));
    ZK_CUDA(cudaMemset(m.own, 0, bytes));
    ZK_CUDA(cudaMalloc(&m.d_desc, sizeof(MeshDesc)));
    cudaIpcMemHandle_t h;
    ZK_CUDA(cudaIpcGetMemHandle(&h, m.own));
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(out_handle, &h, 64);
    m.world = world;
    m.rank = rank;
    m.gather_bytes = gb;
    m.epoch = 0;
    for (int r = 0; r < MESH_MAX_RANKS; r++) m.peers[r] = nullptr;
    m.peers[rank] = static_cast<uint8_t*>(m.own);
    return ZKML_OK;
}

int zkml_mesh_open(zkml_ctx* ctx, const uint8_t* handles, int world) {
    if (!ctx || !handles) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    MeshState& m = g_mesh[ctx->device % 64];
    if (!m.own || m.world != world) return set_error(ZKML_ERR_INVALID_ARG, "mesh not created for this world");
    ZK_CUDA(cudaSetDevice(ctx->device));
    for (int r = 0; r < world; r++) {
        if (r == m.rank || m.peers[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, handles + 64 * r, 64);
        void* p = nullptr;
        ZK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        m.peers[r] = static_cast<uint8_t*>(p);
    }
    MeshDesc d{};
    for (int r = 0; r < MESH_MAX_RANKS; r++) d.peers[r] = m.peers[r];
    d.world = (uint32_t)world;
    d.rank = (uint32_t)m.rank;
    d.err = ctx->err_flag();
    ZK_CUDA(cudaMemcpy(m.d_desc, &d, sizeof(d), cudaMemcpyHostToDevice));
    m.open = true;
    return ZKML_OK;
}

int zkml_mesh_close(zkml_ctx* ctx) {
    if (!ctx) return ZKML_OK;
    MeshState& m = g_mesh[ctx->device % 64];
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < MESH_MAX_RANKS; r++)
        if (r != m.rank && m.peers[r]) cudaIpcCloseMemHandle(m.peers[r]);
    if (m.own) cudaFree(m.own);
    if (m.d_desc) cudaFree(m.d_desc);
    m = MeshState();
    return ZKML_OK;
}

}  // extern "C"

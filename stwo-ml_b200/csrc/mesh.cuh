// Peer-memory mesh of the ranks of one node (one process per GPU): the device side.
//
// Each rank owns an inbox in its HBM, exported with a CUDA IPC handle and mapped by every
// other rank.  Layout (byte offsets):
//   MESH_WORDS_OFF   [2 parity][8 ranks][16] u32   round words, double-buffered by epoch parity
//   MESH_WFLAGS_OFF  [2 parity][8 ranks] u32       round-word epochs
//   MESH_GFLAGS_OFF  [8 ranks] u32                 gather epochs
//   MESH_TICKET_OFF  u32                           gather kernel's block ticket
//   MESH_DATA_OFF    [8 ranks][gather bytes]       gathered vectors, rank-major
// All stores into another rank's inbox are plain peer stores over NVLink (no TMA, no
// multicast); every wait is bounded and ends in an error bit instead of a hang.
#pragma once
#include <stdint.h>

namespace zk {

constexpr int MESH_MAX_RANKS = 8;
constexpr size_t MESH_WORDS_OFF = 0;
constexpr size_t MESH_WFLAGS_OFF = 1024;
constexpr size_t MESH_GFLAGS_OFF = 1152;
constexpr size_t MESH_TICKET_OFF = 1184;
constexpr size_t MESH_DATA_OFF = 4096;
constexpr uint32_t MESH_ERR_TIMEOUT = 32;  // error-flag bit: a peer did not arrive in time

struct MeshDesc {                      // in device memory, written once when the mesh opens
    uint8_t* peers[MESH_MAX_RANKS];    // every rank's inbox as mapped on this GPU (own included)
    uint32_t world, rank;
    uint32_t* err;                     // the context's error flag
};

struct MeshArg {                       // kernel parameter: no mesh when desc is null
    const MeshDesc* desc;
    uint32_t epoch;
};

#ifdef __CUDACC__
// The 12 round words of every rank, summed mod P, in place (one thread).  When a rank does not
// arrive in time the words become 0xFFFFFFFF (no M31 value is) and the error flag is set.  Stores this rank's
// words into slot [parity][rank] of every inbox, publishes the epoch with a system-scope
// release, then waits (about two seconds at most) for every rank's epoch in its own inbox.
__device__ __forceinline__ void mesh_allreduce12(uint32_t* res, const MeshArg& m) {
    const MeshDesc* d = m.desc;
    const uint32_t world = d->world, rank = d->rank, par = m.epoch & 1u;
    for (uint32_t r = 0; r < world; r++) {
        volatile uint32_t* dst =
            reinterpret_cast<uint32_t*>(d->peers[r] + MESH_WORDS_OFF) + (par * MESH_MAX_RANKS + rank) * 16;
        for (int i = 0; i < 12; i++) dst[i] = res[i];
    }
    __threadfence_system();
    for (uint32_t r = 0; r < world; r++) {
        uint32_t* f = reinterpret_cast<uint32_t*>(d->peers[r] + MESH_WFLAGS_OFF) + par * MESH_MAX_RANKS + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(m.epoch) : "memory");
    }
    const uint8_t* own = d->peers[rank];
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(own + MESH_WFLAGS_OFF) + par * MESH_MAX_RANKS;
    unsigned long long acc[12];
    for (int i = 0; i < 12; i++) acc[i] = 0;
    for (uint32_t r = 0; r < world; r++) {
        uint32_t v = 0;
        for (long long it = 0;; it++) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
            if (v == m.epoch) break;
            if (it > (1ll << 25)) {  // ~2 s with the back-off below
                atomicOr(d->err, MESH_ERR_TIMEOUT);
                for (int i = 0; i < 12; i++) res[i] = 0xFFFFFFFFu;  // not an M31 word: the host sees it
                return;
            }
            __nanosleep(64);
        }
        const volatile uint32_t* src =
            reinterpret_cast<const uint32_t*>(own + MESH_WORDS_OFF) + (par * MESH_MAX_RANKS + r) * 16;
        for (int i = 0; i < 12; i++) acc[i] += src[i];
    }
    for (int i = 0; i < 12; i++) res[i] = (uint32_t)(acc[i] % 2147483647ull);
}
#endif

}  // namespace zk

// Peer-memory mesh (host side): see mesh.cuh for the inbox layout.
#pragma once
#include <cuda_runtime.h>

#include "context.hpp"

namespace zk {

struct MeshState {
    int world = 0, rank = -1;
    size_t gather_bytes = 0;       // per-rank capacity of the gather region
    void* own = nullptr;           // this rank's inbox
    uint8_t* peers[MESH_MAX_RANKS] = {};
    MeshDesc* d_desc = nullptr;    // device copy of the descriptor
    uint32_t epoch = 0;            // last epoch handed out (every exchange takes the next one)
    bool open = false;
};

// The mesh of a context's device, or null when none is open.
MeshState* mesh_of(::zkml_ctx* ctx);
// A mesh argument for the next round kernel (takes the next epoch).
MeshArg mesh_next(MeshState* m);
// All-gather of `bytes_per_rank` bytes of device memory `local` from every rank into `out`
// (device, rank-major, world x bytes_per_rank) over the peers' inboxes, on the context's stream.
int mesh_allgather(::zkml_ctx* ctx, MeshState* m, const void* local, size_t bytes_per_rank, void* out);
// Reads and clears the mesh timeout bit of the error flag (ZKML_ERR_TIMEOUT when set).
int mesh_check(::zkml_ctx* ctx);

}  // namespace zk

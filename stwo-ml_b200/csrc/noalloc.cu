// Allocation-free column restriction: zkml_restrict_cols_noalloc.
//
// Some callers cannot allocate device memory at all: code that runs inside a
// memory pool it does not own, allocator hooks, or embedders whose GPU memory is
// budgeted up front.  This entry point computes the same W . eq(r) column
// restriction as the context-based path, but every scratch byte it needs (the
// split eq table, the per-row 64-bit accumulators and the error flag) lives in
// one file-scope __device__ array of fixed size.  The caller passes the device
// input matrix and the device output vector; nothing is allocated.
//
// Limits: at most ZKML_NOALLOC_MAX_ROWS rows and ZKML_NOALLOC_MAX_COLS columns.
// The array is created when the library's device code is loaded on a GPU and
// stays resident on every GPU that loads it until the process exits.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/zkml_b200.h"
#include "context.hpp"
#include "kernels.cuh"

namespace zk {
namespace {

constexpr size_t kAccBytes = (size_t)ZKML_NOALLOC_MAX_ROWS * 32;               // 4 x u64 per row
constexpr size_t kLhiEntries = (size_t)ZKML_NOALLOC_MAX_COLS / 64;             // eq over the high column bits
constexpr size_t kLhiBytes = kLhiEntries * 16;
constexpr size_t kLloBytes = 64 * 16;                                          // eq over the low 6 column bits
constexpr size_t kErrBytes = 256;
constexpr size_t kScratchBytes = kAccBytes + kLhiBytes + kLloBytes + kErrBytes;

// The shared scratch.  In host code this name is only a host-side stand-in for
// the device symbol: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceSetup {
    unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this GPU
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
DeviceSetup g_setup[kMaxDevices];

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

// Once per device, with that device current: resolve the scratch address.
int setup_device(int dev, DeviceSetup& out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceSetup& s = g_setup[dev];
    if (!s.base) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_error(e, "cudaDeviceGetAttribute");
        s.base = static_cast<unsigned char*>(ptr);
        s.num_sms = sms;
    }
    out = s;
    return ZKML_OK;
}

}  // namespace
}  // namespace zk

using namespace zk;

extern "C" int zkml_restrict_cols_noalloc(const uint32_t* b, size_t rows, size_t cols, const uint32_t* r_j,
                                          size_t n_rj, uint32_t* out, size_t out_len, void* stream) {
    if (!b || !out || (n_rj && !r_j)) return set_error(ZKML_ERR_INVALID_ARG, "NULL argument");
    if (rows == 0 || cols == 0) return set_error(ZKML_ERR_INVALID_ARG, "empty matrix");
    if (rows > ZKML_NOALLOC_MAX_ROWS || cols > ZKML_NOALLOC_MAX_COLS)
        return set_error(ZKML_ERR_INVALID_ARG,
                         "zkml_restrict_cols_noalloc handles at most " + std::to_string(ZKML_NOALLOC_MAX_ROWS) +
                             " rows and " + std::to_string(ZKML_NOALLOC_MAX_COLS) + " columns (got " +
                             std::to_string(rows) + " x " + std::to_string(cols) + ")");
    if (n_rj != ilog2(next_pow2(cols)))
        return set_error(ZKML_ERR_INVALID_ARG, "r_j must have log2(next_pow2(cols)) challenges");
    if (out_len < rows) return set_error(ZKML_ERR_INVALID_ARG, "out_len must be at least rows");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return set_error(ZKML_ERR_UNSUPPORTED, "device ordinal too large");
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, b) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
        attr.device != dev || cudaPointerGetAttributes(&attr, out) != cudaSuccess ||
        attr.type != cudaMemoryTypeDevice || attr.device != dev) {
        cudaGetLastError();
        return set_error(ZKML_ERR_INVALID_ARG, "b and out must be device memory of the current GPU");
    }
    DeviceSetup ds;
    int rc = setup_device(dev, ds);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(ds.base);
    uint4* lhi = reinterpret_cast<uint4*>(ds.base + kAccBytes);
    uint4* llo = reinterpret_cast<uint4*>(ds.base + kAccBytes + kLhiBytes);
    uint32_t* err = reinterpret_cast<uint32_t*>(ds.base + kAccBytes + kLhiBytes + kLloBytes);
    const qm31* r = reinterpret_cast<const qm31*>(r_j);
    const unsigned lo_vars = n_rj < 6 ? (unsigned)n_rj : 6u;
    const unsigned hi_vars = (unsigned)n_rj - lo_vars;
    // the array keeps the previous call's contents: clear what accumulates
    if ((e = cudaMemsetAsync(acc, 0, rows * 32, s)) != cudaSuccess) return cuda_error(e, "cudaMemsetAsync");
    if ((e = cudaMemsetAsync(err, 0, 4, s)) != cudaSuccess) return cuda_error(e, "cudaMemsetAsync");
    launch_eq_table(r, (int)hi_vars, lhi, (size_t)1 << hi_vars, s);
    launch_eq_table(r + hi_vars, (int)lo_vars, llo, 64, s);
    launch_restrict_cols(b, (uint32_t)rows, (uint32_t)cols, lhi, llo, acc, err, ds.num_sms, s);
    launch_acc_finalize(acc, rows, reinterpret_cast<uint4*>(out), out_len, s);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_error(e, "restrict_cols_noalloc launch");
    uint32_t flag = 0;
    if ((e = cudaMemcpyAsync(&flag, err, 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
        return cuda_error(e, "cudaMemcpyAsync");
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_error(e, "cudaStreamSynchronize");
    if (flag) return set_error(ZKML_ERR_INVALID_ARG, "input value >= 2^31 is not an M31 element");
    return ZKML_OK;
}

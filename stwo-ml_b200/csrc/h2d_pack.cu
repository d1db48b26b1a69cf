// Host -> device upload of a large M31 matrix that sits in host memory, with values that fit
// a signed byte crossing PCIe as one byte each.
//
// Quantised weights (int8 embedded in M31 as x >= 0 ? x : p + x, gadgets/quantize.rs:105-110)
// arrive through the ZkmlOps boundary as 4-byte words, and PCIe moves them at ~55 GB/s:
// 283 MB of a config-2 weight take 5.1 ms to upload against 0.25 ms for the whole layer
// reduction.  Here the matrix is cut into chunks of 2^18 words; host threads pack each chunk
// into bytes in a pinned staging buffer (80-100 GB/s of input with 15-16 threads on the GPU
// host), the calling thread copies each packed chunk as soon as it is ready, and once all are
// on the device one kernel widens the packed chunks back to canonical M31 words in HBM.  A chunk holding any value outside
// [0, 127] U [p - 128, p] (or with bit 31 set) goes over unchanged from the caller's buffer,
// so every input gives the device exactly the words the plain copy would give, up to the
// representative of zero (p is stored as 0, the same field element); words with bit 31 set
// reach the kernels as they are and fail the call as before.
#include <sched.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <exception>
#include <memory>
#include <thread>
#include <vector>

#include "context.hpp"

namespace zk {

constexpr size_t PACK_CHUNK = (size_t)1 << 18;  // words per chunk (a multiple of 16)

__device__ __forceinline__ uint32_t s8_to_m31(uint32_t byte) {
    const int32_t s = (int32_t)(int8_t)(uint8_t)byte;
    return (uint32_t)s + ((uint32_t)(s >> 31) & 0x7fffffffu);
}

// out[i] = the M31 word of the signed byte in[i] for every i in a chunk whose flag is 1 (packed);
// the words of the other chunks were copied as they are.  16 bytes in, 64 bytes out per step.
__global__ void unpack_s8_m31_kernel(const int8_t* __restrict__ in, size_t n, const uint8_t* __restrict__ packed,
                                     uint32_t* __restrict__ out) {
    const size_t n16 = n / 16, stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    for (size_t i = t0; i < n16; i += stride) {
        if (packed[i * 16 / PACK_CHUNK] != 1) continue;
        const uint4 v = __ldcs(reinterpret_cast<const uint4*>(in) + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint4* o = reinterpret_cast<uint4*>(out) + 4 * i;
#pragma unroll
        for (int q = 0; q < 4; q++)
            o[q] = make_uint4(s8_to_m31(w[q] & 0xff), s8_to_m31((w[q] >> 8) & 0xff), s8_to_m31((w[q] >> 16) & 0xff),
                              s8_to_m31(w[q] >> 24));
    }
    for (size_t i = n16 * 16 + t0; i < n; i += stride)
        if (packed[i / PACK_CHUNK] == 1) out[i] = s8_to_m31((uint8_t)in[i]);
}

namespace {

// Packs n words into bytes; false if a word is not a signed byte's M31 image.  For v < 2^31,
// t = v + (v >> 30) has the signed value's byte as its low byte exactly when v is in [0, 127]
// or [p - 128, p] (t = 2^31 + s there), and every other v leaves a bit of 8..30 set in t + 128.
bool pack_words(const uint32_t* in, int8_t* out, size_t n) {
    uint32_t bad = 0;
    for (size_t i = 0; i < n; i++) {
        const uint32_t v = in[i];
        const uint32_t t = v + (v >> 30);
        bad |= ((t + 128u) & 0x7fffff00u) | (v >> 31);
        out[i] = (int8_t)(uint8_t)t;
    }
    return bad == 0;
}

// Packing threads: the calling thread's CPUs (at most 16) less the one it polls on;
// ZKML_PACK_THREADS overrides.
int host_threads() {
    if (const char* e = getenv("ZKML_PACK_THREADS")) return std::max(1, atoi(e));
    cpu_set_t cs;
    int n = sched_getaffinity(0, sizeof(cs), &cs) == 0 ? CPU_COUNT(&cs) : (int)std::thread::hardware_concurrency();
    return std::max(1, std::min(n - 1, 16));
}

}  // namespace

int upload_m31_packed(::zkml_ctx* ctx, const uint32_t* host, size_t count, DevBuf& dst, const void** out) {
    // Packing reads every word once on the CPUs and then lets the DMA engine read a quarter of
    // the bytes: it beats the plain copy (one DMA read of everything) only with enough cores to
    // out-run PCIe.  With fewer than 8 packing threads (for example one rank of several bound to
    // a share of the host's CPUs, which also share its memory bandwidth) the plain copy is used.
    const int threads = host_threads();
    if (threads < 8) return device_view(ctx, host, count * 4, dst, out);
    cudaStream_t s = ctx->stream;
    int rc;
    const size_t chunks = (count + PACK_CHUNK - 1) / PACK_CHUNK;
    const size_t staging = count + chunks;  // packed bytes, then one flag per chunk
    if ((rc = dst.ensure(count * 4)) || (rc = ctx->pack_dev.ensure(staging + 16))) return rc;
    if (ctx->pack_host_bytes < staging) {
        if (ctx->pack_event) ZK_CUDA(cudaEventSynchronize(ctx->pack_event));
        if (ctx->pack_host) cudaFreeHost(ctx->pack_host);
        ctx->pack_host = nullptr;
        ctx->pack_host_bytes = 0;
        ZK_CUDA(cudaMallocHost(&ctx->pack_host, staging));
        ctx->pack_host_bytes = staging;
    }
    if (!ctx->pack_event) ZK_CUDA(cudaEventCreateWithFlags(&ctx->pack_event, cudaEventDisableTiming));
    // the staging buffer is reused: the previous upload's copies must be done reading it
    ZK_CUDA(cudaEventSynchronize(ctx->pack_event));
    std::unique_ptr<std::atomic<uint8_t>[]> state(new std::atomic<uint8_t>[chunks]);
    for (size_t c = 0; c < chunks; c++) state[c].store(0, std::memory_order_relaxed);
    std::atomic<size_t> next{0};
    std::atomic<bool> stop{false};
    int8_t* hp = reinterpret_cast<int8_t*>(ctx->pack_host);
    auto worker = [&]() {
        for (;;) {
            const size_t c = next.fetch_add(1, std::memory_order_relaxed);
            if (c >= chunks || stop.load(std::memory_order_relaxed)) return;
            const size_t off = c * PACK_CHUNK, len = std::min(PACK_CHUNK, count - off);
            const bool ok = pack_words(host + off, hp + off, len);
            state[c].store(ok ? 1 : 2, std::memory_order_release);
        }
    };
    // ZKML_PACK_TRACE=1 prints, per call, when the last copy was issued and when the threads ended
    static const bool trace = getenv("ZKML_PACK_TRACE") && getenv("ZKML_PACK_TRACE")[0] == '1';
    const auto t0 = std::chrono::steady_clock::now();
    const int nt = (int)std::min<size_t>((size_t)threads, chunks);
    std::vector<std::thread> pool;
    pool.reserve(nt);
    try {
        for (int t = 0; t < nt; t++) pool.emplace_back(worker);
    } catch (const std::exception&) {  // no more threads: go on with those that started
    }
    if (pool.empty()) return device_view(ctx, host, count * 4, dst, out);
    uint32_t* dev = static_cast<uint32_t*>(dst.ptr);
    int8_t* dp = ctx->pack_dev.as<int8_t>();
    size_t packed_bytes = 0;
    cudaError_t err = cudaSuccess;
    for (size_t c = 0; c < chunks && err == cudaSuccess; c++) {
        uint8_t st;
        while ((st = state[c].load(std::memory_order_acquire)) == 0) std::this_thread::yield();
        const size_t off = c * PACK_CHUNK, len = std::min(PACK_CHUNK, count - off);
        hp[count + c] = (int8_t)st;
        if (st == 1) {
            err = cudaMemcpyAsync(dp + off, hp + off, len, cudaMemcpyHostToDevice, s);
            packed_bytes += len;
        } else {
            err = cudaMemcpyAsync(dev + off, host + off, len * 4, cudaMemcpyHostToDevice, s);
            packed_bytes += len * 4;
        }
    }
    // one widening pass over the packed chunks once they are all on the device
    if (err == cudaSuccess) err = cudaMemcpyAsync(dp + count, hp + count, chunks, cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess) {
        const unsigned g = (unsigned)std::min<size_t>((count / 16 + 255) / 256 + 1, (size_t)ctx->num_sms * 8);
        unpack_s8_m31_kernel<<<g, 256, 0, s>>>(dp, count, reinterpret_cast<const uint8_t*>(dp + count), dev);
        err = cudaGetLastError();
        ctx->launches++;
    }
    packed_bytes += chunks;
    const auto t_issued = std::chrono::steady_clock::now();
    if (err != cudaSuccess) stop.store(true);
    for (auto& th : pool) th.join();
    if (trace)
        fprintf(stderr, "[zkml pack] %zu words, %d threads: copies issued after %.1f us, threads joined after %.1f us\n",
                count, nt, std::chrono::duration<double, std::micro>(t_issued - t0).count(),
                std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count());
    if (err == cudaSuccess) err = cudaEventRecord(ctx->pack_event, s);
    if (err != cudaSuccess) {
        cudaStreamSynchronize(s);
        return set_error(ZKML_ERR_CUDA, std::string("packed upload: ") + cudaGetErrorString(err));
    }
    ctx->h2d_bytes += packed_bytes;
    *out = dst.ptr;
    return ZKML_OK;
}

}  // namespace zk

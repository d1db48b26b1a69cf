// Shared-memory exchange between the ranks of one node (see zkml_shm_exchange_open).
//
// The sharded product sumcheck exchanges 12 words per round and, once, the
// folded vectors at the gather point.  Both are host-side data (the round words
// arrive in mapped host memory, the transcript runs on the host), so between
// processes of one node the cheapest collective is a POSIX shared-memory
// segment: each rank writes its contribution into its own slot, publishes a
// sequence number with a release store, and reads the other slots once their
// sequence numbers have arrived.  Slots are double-buffered by sequence parity,
// which is enough because no rank can start exchange s + 2 before every rank
// has finished exchange s + 1 (and so finished reading exchange s): while a
// rank waits for exchange s, a peer's slot holds either s - 2 or s, so the waits
// test for equality.  A segment left behind by an earlier job under the same
// name is told apart by the job nonce every rank passes in: rank 0 recreates the
// segment and writes the nonce before marking it ready, and the other ranks
// re-open the name until they see their own nonce.  Every wait is bounded.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

#include "../../include/zkml_b200.h"

namespace zk {
int set_error(int status, const std::string& msg);
}

namespace {

constexpr int kMaxRanks = 64;
constexpr int kWords = 64;  // u64 words per reduce slot
constexpr double kTimeoutS = 60.0;

struct alignas(64) ReduceSlot {
    std::atomic<uint64_t> seq;
    uint64_t pad[7];
    uint64_t w[kWords];
};

struct Header {
    std::atomic<uint32_t> ready;  // set by rank 0 once the segment is initialised
    uint32_t world;
    uint64_t nonce;               // the job's nonce, written by rank 0 before ready
    uint64_t gather_bytes;        // per rank per buffer
    std::atomic<uint64_t> gather_seq[2][kMaxRanks];
    std::atomic<uint32_t> closed[kMaxRanks];
};

struct Shm {
    std::string name;
    int world = 0, rank = 0;
    size_t bytes = 0;
    uint8_t* base = nullptr;
    uint64_t reduce_seq = 0, gather_seq = 0;
    Header* hdr() { return reinterpret_cast<Header*>(base); }
    ReduceSlot* slot(int parity, int r) {
        return reinterpret_cast<ReduceSlot*>(base + 4096) + parity * kMaxRanks + r;
    }
    uint8_t* gather_buf(int parity, int r) {
        const size_t off = 4096 + 2 * kMaxRanks * sizeof(ReduceSlot);
        return base + off + ((size_t)parity * world + r) * hdr()->gather_bytes;
    }
};

bool wait_until(const std::atomic<uint64_t>& v, uint64_t want) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint64_t it = 0; v.load(std::memory_order_acquire) != want; it++) {
        if ((it & 255) == 255) {
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > kTimeoutS)
                return false;
            std::this_thread::yield();
        }
    }
    return true;
}

int shm_allreduce(void* user, uint64_t* words, int n) {
    Shm* s = static_cast<Shm*>(user);
    if (n > kWords) return zk::set_error(ZKML_ERR_INVALID_ARG, "exchange: too many words");
    const uint64_t seq = ++s->reduce_seq;
    const int par = (int)(seq & 1);
    ReduceSlot* mine = s->slot(par, s->rank);
    memcpy(mine->w, words, n * sizeof(uint64_t));
    mine->seq.store(seq, std::memory_order_release);
    uint64_t acc[kWords] = {0};
    for (int r = 0; r < s->world; r++) {
        ReduceSlot* o = s->slot(par, r);
        if (!wait_until(o->seq, seq)) return zk::set_error(ZKML_ERR_TIMEOUT, "exchange: a rank did not arrive");
        for (int i = 0; i < n; i++) acc[i] += o->w[i];
    }
    memcpy(words, acc, n * sizeof(uint64_t));
    return ZKML_OK;
}

int shm_allgather(void* user, const void* local, void* out, size_t bytes) {
    Shm* s = static_cast<Shm*>(user);
    if (bytes > s->hdr()->gather_bytes) return zk::set_error(ZKML_ERR_INVALID_ARG, "exchange: gather too large");
    const uint64_t seq = ++s->gather_seq;
    const int par = (int)(seq & 1);
    memcpy(s->gather_buf(par, s->rank), local, bytes);
    s->hdr()->gather_seq[par][s->rank].store(seq, std::memory_order_release);
    for (int r = 0; r < s->world; r++) {
        if (!wait_until(s->hdr()->gather_seq[par][r], seq))
            return zk::set_error(ZKML_ERR_TIMEOUT, "exchange: a rank did not arrive at the gather");
        memcpy(static_cast<uint8_t*>(out) + (size_t)r * bytes, s->gather_buf(par, r), bytes);
    }
    return ZKML_OK;
}

}  // namespace

extern "C" {

int zkml_shm_exchange_open(const char* name, int world, int rank, size_t max_gather_bytes, uint64_t job_nonce,
                           zkml_exchange* out) {
    if (!name || !out || world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return zk::set_error(ZKML_ERR_INVALID_ARG, "exchange: bad name, world or rank");
    Shm* s = new Shm;
    s->name = std::string("/") + name;
    s->world = world;
    s->rank = rank;
    const size_t gb = (max_gather_bytes + 63) / 64 * 64;
    s->bytes = 4096 + 2 * kMaxRanks * sizeof(ReduceSlot) + 2 * (size_t)world * gb;
    auto elapsed = [](std::chrono::steady_clock::time_point t) {
        return std::chrono::duration<double>(std::chrono::steady_clock::now() - t).count();
    };
    const auto t0 = std::chrono::steady_clock::now();
    if (rank == 0) {
        shm_unlink(s->name.c_str());  // a stale segment of an earlier job
        int fd = shm_open(s->name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
        if (fd >= 0 && ftruncate(fd, (off_t)s->bytes) != 0) {
            close(fd);
            fd = -1;
        }
        void* p = fd >= 0 ? mmap(nullptr, s->bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0) : MAP_FAILED;
        if (fd >= 0) close(fd);
        if (p == MAP_FAILED) {
            delete s;
            return zk::set_error(ZKML_ERR_UNSUPPORTED, "exchange: cannot create the shared-memory segment");
        }
        s->base = static_cast<uint8_t*>(p);
        Header* h = s->hdr();
        h->world = (uint32_t)world;
        h->gather_bytes = gb;
        h->nonce = job_nonce;
        h->ready.store(1, std::memory_order_release);
    } else {
        // Open the name until it holds this job's initialised segment: a segment of an
        // earlier job (other nonce) is unmapped and the name opened again.
        for (;;) {
            if (elapsed(t0) > kTimeoutS) {
                delete s;
                return zk::set_error(ZKML_ERR_TIMEOUT, "exchange: rank 0 did not create this job's segment");
            }
            int fd = shm_open(s->name.c_str(), O_RDWR, 0600);
            if (fd < 0) {
                std::this_thread::sleep_for(std::chrono::milliseconds(1));
                continue;
            }
            struct stat st;
            if (fstat(fd, &st) != 0 || (size_t)st.st_size < s->bytes) {
                close(fd);
                std::this_thread::sleep_for(std::chrono::milliseconds(1));
                continue;
            }
            void* p = mmap(nullptr, s->bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
            close(fd);
            if (p == MAP_FAILED) {
                delete s;
                return zk::set_error(ZKML_ERR_UNSUPPORTED, "exchange: mmap failed");
            }
            Header* h = reinterpret_cast<Header*>(p);
            // give rank 0 a moment to finish initialising a fresh segment
            const auto t1 = std::chrono::steady_clock::now();
            while (h->ready.load(std::memory_order_acquire) != 1 && elapsed(t1) < 0.05)
                std::this_thread::sleep_for(std::chrono::microseconds(200));
            if (h->ready.load(std::memory_order_acquire) == 1 && h->nonce == job_nonce) {
                if (h->world != (uint32_t)world || h->gather_bytes != gb) {
                    munmap(p, s->bytes);
                    delete s;
                    return zk::set_error(ZKML_ERR_INVALID_ARG,
                                         "exchange: ranks disagree on world size or gather size");
                }
                s->base = static_cast<uint8_t*>(p);
                break;
            }
            munmap(p, s->bytes);  // not (yet) this job's segment
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
        }
    }
    out->user = s;
    out->allreduce_u64 = shm_allreduce;
    out->allgather = shm_allgather;
    out->world = world;
    out->rank = rank;
    return ZKML_OK;
}

int zkml_shm_exchange_close(zkml_exchange* ex) {
    if (!ex || !ex->user) return ZKML_OK;
    Shm* s = static_cast<Shm*>(ex->user);
    s->hdr()->closed[s->rank].store(1, std::memory_order_release);
    if (s->rank == 0) shm_unlink(s->name.c_str());  // mappings stay valid until every rank unmaps
    munmap(s->base, s->bytes);
    delete s;
    ex->user = nullptr;
    return ZKML_OK;
}

}  // extern "C"

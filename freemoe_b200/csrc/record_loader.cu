// record_loader.cu -- cold -> warm expert loads on the host side of the path:
// file extents are read straight into rings of pinned chunks by several reader
// threads and copied to the HBM slot with cudaMemcpyAsync (one copy stream per
// reader) while the next chunks are read; the checksum is FNV-1a 64 of the
// slot computed on the device (fnv.cu).
//
// What it replaces in the reference's demand load (ResidencyManager::load_slot,
// src/residency.cpp:624-724):
//   ReadScheduler::read_record (src/io.cpp:313-400)  reads the coalesced extent
//       groups into a pageable std::vector (DirectReader: through a second
//       aligned bounce buffer, src/io.cpp:180-206);
//   fnv1a64(payload) against the record checksum      (src/residency.cpp:656-667);
//   Backend::upload                                    copies the vector again
//       (the CUDA adapter's pinned staging ring) before the DMA;
//   the slot read-back + fnv1a64 of the copy           (src/residency.cpp:700-720).
// Here the bytes are read once into pinned memory, cross PCIe once, and are
// hashed once, on the device, from the slot itself: a checksum that matches
// shows both the source bytes and the transfer correct.
//
// Kept from the reference: extents are coalesced exactly like coalesce_extents
// (src/io.cpp:46-78), reads past the end of the file fail SHORT_READ before
// any byte moves (src/io.cpp:115-117), the Direct mode reads aligned spans
// with O_DIRECT and falls back to buffered reads when the file system refuses
// (src/io.cpp:161-218), and the source identity (size, device, inode, mtime,
// ctime, sparse content probe; src/common.cpp:79-119) is verified before every
// record (src/io.cpp:262-278).
#include <fcntl.h>
#include <sys/stat.h>
#include <sys/statvfs.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <limits>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

namespace fmb {
uint64_t fnv1a64_workspace_bytes(uint64_t n);
int fnv1a64_launch(const void *data, uint64_t n, uint64_t *out, void *workspace, uint64_t ws_bytes,
                   cudaStream_t stream);
} // namespace fmb

using fmb::set_error;

namespace {

constexpr uint64_t kBasis = 0xCBF29CE484222325ull, kPrime = 0x100000001B3ull;

int file_identity_of(const char *path, fmcuda_file_identity *id) {
    struct stat st {};
    if (::stat(path, &st) != 0)
        return set_error(FM_STATUS_IO_ERROR, std::string("stat failed for ") + path + ": " + std::strerror(errno));
    *id = fmcuda_file_identity{};
    id->size = static_cast<uint64_t>(st.st_size);
    id->dev = static_cast<uint64_t>(st.st_dev);
    id->ino = static_cast<uint64_t>(st.st_ino);
    id->mtime_ns = static_cast<int64_t>(st.st_mtim.tv_sec) * 1000000000ll + st.st_mtim.tv_nsec;
    id->ctime_ns = static_cast<int64_t>(st.st_ctim.tv_sec) * 1000000000ll + st.st_ctim.tv_nsec;
    // sparse content probe: FNV-1a over the first, middle and last 64 bytes
    const int fd = ::open(path, O_RDONLY);
    if (fd >= 0 && id->size > 0) {
        uint64_t h = kBasis;
        const uint64_t len = std::min<uint64_t>(64, id->size);
        const uint64_t mid = id->size > 64 ? id->size / 2 - std::min<uint64_t>(32, id->size / 2) : 0;
        const uint64_t last = id->size > len ? id->size - len : 0;
        uint8_t buf[64];
        for (uint64_t off : {uint64_t(0), mid, last}) {
            const ssize_t got = ::pread(fd, buf, static_cast<size_t>(len), static_cast<off_t>(off));
            for (ssize_t i = 0; i < got; ++i) h = (h ^ buf[i]) * kPrime;
        }
        id->content_probe = h;
    }
    if (fd >= 0) ::close(fd);
    return FM_STATUS_OK;
}

bool same_identity(const fmcuda_file_identity &a, const fmcuda_file_identity &b) {
    return a.size == b.size && a.dev == b.dev && a.ino == b.ino && a.mtime_ns == b.mtime_ns &&
           a.ctime_ns == b.ctime_ns && a.content_probe == b.content_probe;
}

struct Group {
    uint64_t offset = 0, end = 0;
    std::vector<uint32_t> members;
};

int coalesce(const fmcuda_extent *ext, uint32_t n, uint64_t max_gap, std::vector<Group> &groups) {
    std::vector<uint32_t> order(n);
    for (uint32_t i = 0; i < n; ++i) order[i] = i;
    std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        if (ext[a].offset != ext[b].offset) return ext[a].offset < ext[b].offset;
        if (ext[a].size != ext[b].size) return ext[a].size < ext[b].size;
        return a < b;
    });
    groups.clear();
    for (uint32_t i : order) {
        const fmcuda_extent &e = ext[i];
        if (e.size == 0 || e.offset > std::numeric_limits<uint64_t>::max() - e.size)
            return set_error(FM_STATUS_INVALID_ARGUMENT, "invalid extent");
        const uint64_t end = e.offset + e.size;
        if (!groups.empty()) {
            Group &g = groups.back();
            if (max_gap <= std::numeric_limits<uint64_t>::max() - g.end && e.offset <= g.end + max_gap) {
                g.end = std::max(g.end, end);
                g.members.push_back(i);
                continue;
            }
        }
        Group g;
        g.offset = e.offset;
        g.end = end;
        g.members.push_back(i);
        groups.push_back(std::move(g));
    }
    return FM_STATUS_OK;
}

// pread until `n` bytes or end of file; -1 with errno on failure
ssize_t pread_full(int fd, void *buf, uint64_t n, uint64_t off) {
    uint64_t done = 0;
    while (done < n) {
        const ssize_t r = ::pread(fd, static_cast<uint8_t *>(buf) + done, static_cast<size_t>(n - done),
                                  static_cast<off_t>(off + done));
        if (r < 0) {
            if (errno == EINTR) continue;
            return -1;
        }
        if (r == 0) break;
        done += static_cast<uint64_t>(r);
    }
    return static_cast<ssize_t>(done);
}

} // namespace

// One reader thread's share: a copy stream and a ring of pinned chunks.
struct Reader {
    cudaStream_t stream = nullptr;
    std::vector<void *> raw;         // pinned allocations, chunk + alignment bytes
    std::vector<uint8_t *> buf;      // the aligned chunk inside each
    std::vector<cudaEvent_t> ev;     // last copy out of each chunk
    std::vector<bool> busy;
    cudaEvent_t tail = nullptr;      // end of this reader's copies of a record
    size_t next = 0;
};

struct fmcuda_record_loader {
    std::string path;
    int fd = -1;
    int direct_fd = -1;
    int mode = FM_READER_BUFFERED;
    bool force_fallback = false;
    uint64_t gap = 4096;
    uint64_t alignment = 4096;
    uint64_t chunk = 0;
    fmcuda_file_identity expected{};
    std::vector<Reader> readers;
    cudaEvent_t entry = nullptr;      // the caller's stream at the start of a load
    uint64_t *host_word = nullptr;    // pinned: the checksum read back
    cudaEvent_t done = nullptr;

    ~fmcuda_record_loader() {
        for (Reader &r : readers) {
            for (size_t i = 0; i < r.ev.size(); ++i) {
                if (r.ev[i]) {
                    (void)cudaEventSynchronize(r.ev[i]);
                    (void)cudaEventDestroy(r.ev[i]);
                }
                if (r.raw[i]) (void)cudaFreeHost(r.raw[i]);
            }
            if (r.tail) (void)cudaEventDestroy(r.tail);
            if (r.stream) (void)cudaStreamDestroy(r.stream);
        }
        if (entry) (void)cudaEventDestroy(entry);
        if (done) {
            (void)cudaEventSynchronize(done);
            (void)cudaEventDestroy(done);
        }
        if (host_word) (void)cudaFreeHost(host_word);
        if (fd >= 0) ::close(fd);
        if (direct_fd >= 0) ::close(direct_fd);
    }
};

namespace {

// polled, bounded wait for one event (Backend::wait_fence semantics)
int wait_event(cudaEvent_t ev, uint32_t timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t spin = 0;; ++spin) {
        const cudaError_t err = cudaEventQuery(ev);
        if (err == cudaSuccess) return FM_STATUS_OK;
        if (err != cudaErrorNotReady) return fmb::cuda_status(err, "record load: copy");
        (void)cudaGetLastError();
        if (std::chrono::steady_clock::now() - t0 >= std::chrono::milliseconds(timeout_ms))
            return set_error(FM_STATUS_FENCE_TIMEOUT, "record load: copy did not complete within " +
                                                          std::to_string(timeout_ms) + " ms");
        if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(5));
    }
}

// One chunk-sized read: file bytes [lo, hi) of group g, read from `pos`
// (Direct: an aligned span of n bytes; buffered: pos = lo, n = hi - lo).
struct Job {
    uint32_t group;
    bool direct;
    uint64_t pos, n, lo, hi;
};

} // namespace

extern "C" int fmcuda_file_identity_get(const char *path, fmcuda_file_identity *id) {
    if (!path || !id) return set_error(FM_STATUS_INVALID_ARGUMENT, "file identity: null argument");
    return file_identity_of(path, id);
}

extern "C" int fmcuda_coalesce_extents(const fmcuda_extent *extents, uint32_t n, uint64_t max_gap,
                                       uint64_t *group_offset, uint64_t *group_end, uint32_t *group_of,
                                       uint32_t *n_groups) {
    if ((n && !extents) || !n_groups) return set_error(FM_STATUS_INVALID_ARGUMENT, "coalesce: null argument");
    std::vector<Group> groups;
    if (int rc = coalesce(extents, n, max_gap, groups)) return rc;
    *n_groups = static_cast<uint32_t>(groups.size());
    for (size_t g = 0; g < groups.size(); ++g) {
        if (group_offset) group_offset[g] = groups[g].offset;
        if (group_end) group_end[g] = groups[g].end;
        if (group_of)
            for (uint32_t i : groups[g].members) group_of[i] = static_cast<uint32_t>(g);
    }
    return FM_STATUS_OK;
}

extern "C" int fmcuda_record_loader_create(const char *path, int reader_mode, uint64_t coalesce_gap,
                                           uint64_t chunk_bytes, uint32_t ring_depth, uint32_t reader_threads,
                                           int force_direct_fallback, const fmcuda_file_identity *expected,
                                           fmcuda_record_loader **out) {
    if (!path || !out) return set_error(FM_STATUS_INVALID_ARGUMENT, "record loader: null argument");
    *out = nullptr;
    if (reader_mode != FM_READER_BUFFERED && reader_mode != FM_READER_DIRECT)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "record loader: reader mode must be buffered or direct");
    if (ring_depth < 2 || ring_depth > 64 || chunk_bytes < (1u << 16) || chunk_bytes > (1ull << 30) ||
        reader_threads < 1 || reader_threads > 32)
        return set_error(FM_STATUS_INVALID_ARGUMENT,
                         "record loader: 1..32 readers, each a ring of 2..64 chunks of 64 KiB..1 GiB");
    auto *L = new fmcuda_record_loader();
    L->path = path;
    L->mode = reader_mode;
    L->gap = coalesce_gap;
    L->force_fallback = force_direct_fallback != 0;
    int rc = FM_STATUS_OK;
    if (expected) {
        L->expected = *expected;
    } else if ((rc = file_identity_of(path, &L->expected))) {
        delete L;
        return rc;
    }
    L->fd = ::open(path, O_RDONLY);
    if (L->fd < 0) {
        rc = set_error(FM_STATUS_IO_ERROR, "open failed for " + L->path + ": " + std::strerror(errno));
        delete L;
        return rc;
    }
#ifdef O_DIRECT
    if (reader_mode == FM_READER_DIRECT) {
        L->direct_fd = ::open(path, O_RDONLY | O_DIRECT);
        if (L->direct_fd >= 0) {
            struct statvfs vfs {};
            uint64_t a = 4096;
            if (::fstatvfs(L->direct_fd, &vfs) == 0 && vfs.f_bsize >= 512) a = static_cast<uint64_t>(vfs.f_bsize);
            if (a && (a & (a - 1)) == 0 && a <= (1u << 20)) L->alignment = a;
        }
    }
#endif
    // chunks are whole multiples of the direct-I/O alignment, so every chunk
    // of an aligned span starts aligned in the file and in memory
    L->chunk = (chunk_bytes + L->alignment - 1) / L->alignment * L->alignment;
    L->readers.resize(reader_threads);
    cudaError_t err = cudaSuccess;
    for (Reader &r : L->readers) {
        r.raw.assign(ring_depth, nullptr);
        r.buf.assign(ring_depth, nullptr);
        r.ev.assign(ring_depth, nullptr);
        r.busy.assign(ring_depth, false);
        if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking);
        if (err == cudaSuccess) err = cudaEventCreateWithFlags(&r.tail, cudaEventDisableTiming);
        for (uint32_t i = 0; i < ring_depth && err == cudaSuccess; ++i) {
            err = cudaHostAlloc(&r.raw[i], L->chunk + L->alignment, cudaHostAllocDefault);
            if (err == cudaSuccess) {
                const uintptr_t a = reinterpret_cast<uintptr_t>(r.raw[i]);
                r.buf[i] = reinterpret_cast<uint8_t *>((a + L->alignment - 1) & ~uintptr_t(L->alignment - 1));
                err = cudaEventCreateWithFlags(&r.ev[i], cudaEventDisableTiming);
            }
        }
    }
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&L->entry, cudaEventDisableTiming);
    if (err == cudaSuccess) err = cudaHostAlloc(reinterpret_cast<void **>(&L->host_word), 64, cudaHostAllocDefault);
    if (err == cudaSuccess) err = cudaEventCreateWithFlags(&L->done, cudaEventDisableTiming);
    if (err != cudaSuccess) {
        rc = fmb::cuda_status(err, "record loader: pinned ring");
        (void)cudaGetLastError();
        delete L;
        return rc;
    }
    *out = L;
    return FM_STATUS_OK;
}

extern "C" int fmcuda_record_loader_destroy(fmcuda_record_loader *loader) {
    delete loader;
    return FM_STATUS_OK;
}

extern "C" uint64_t fmcuda_record_load_workspace_bytes(uint64_t payload_bytes) {
    return 256 + fmb::fnv1a64_workspace_bytes(payload_bytes);
}

extern "C" int fmcuda_record_load(fmcuda_record_loader *L, const fmcuda_extent *extents, uint32_t n_extents,
                                  void *slot, uint64_t slot_bytes, int checksum_known,
                                  uint64_t expected_checksum, void *workspace, uint64_t workspace_bytes,
                                  void *stream_, uint32_t timeout_ms, fmcuda_record_load_stats *stats) {
    if (!L || (n_extents && !extents) || !slot || !stats)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "record load: null argument");
    *stats = fmcuda_record_load_stats{};
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const auto t0 = std::chrono::steady_clock::now();
    // the source must still be the file the manifest indexed
    fmcuda_file_identity now{};
    if (int rc = file_identity_of(L->path.c_str(), &now)) return rc;
    if (!same_identity(now, L->expected))
        return set_error(FM_STATUS_SOURCE_CHANGED, "model source changed after index creation: " + L->path);
    std::vector<Group> groups;
    if (int rc = coalesce(extents, n_extents, L->gap, groups)) return rc;
    std::vector<uint64_t> out_off(n_extents);
    uint64_t payload = 0;
    for (uint32_t i = 0; i < n_extents; ++i) {
        out_off[i] = payload;
        if (extents[i].size > std::numeric_limits<uint64_t>::max() - payload)
            return set_error(FM_STATUS_INVALID_ARGUMENT, "extent total overflow");
        payload += extents[i].size;
    }
    if (payload > slot_bytes) return set_error(FM_STATUS_INVALID_ARGUMENT, "record load: payload larger than the slot");
    if (!workspace || workspace_bytes < fmcuda_record_load_workspace_bytes(payload) ||
        (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return set_error(FM_STATUS_INVALID_ARGUMENT, "record load: workspace too small or not 256-byte aligned");
    for (const Group &g : groups)
        if (g.end > now.size)
            return set_error(FM_STATUS_SHORT_READ, "read beyond EOF: " + L->path);
    stats->payload_bytes = payload;
    stats->read_requests = groups.size();
    for (const Group &g : groups) stats->coalesced_requests += g.members.size() - 1;

    // chunk-sized reads of every group, in file order
    const bool direct = L->mode == FM_READER_DIRECT && !L->force_fallback && L->direct_fd >= 0;
    if (L->mode == FM_READER_DIRECT && !direct) stats->direct_fallbacks = groups.size();
    std::vector<Job> jobs;
    for (uint32_t gi = 0; gi < groups.size(); ++gi) {
        const Group &g = groups[gi];
        const uint64_t A = L->alignment;
        const uint64_t s0 = direct ? g.offset & ~(A - 1) : g.offset;
        const uint64_t s1 = direct ? (g.end + A - 1) & ~(A - 1) : g.end;
        for (uint64_t pos = s0; pos < s1; pos += L->chunk) {
            const uint64_t n = std::min(L->chunk, s1 - pos);
            jobs.push_back({gi, direct, pos, n, std::max(pos, g.offset), std::min(pos + n, g.end)});
        }
    }

    int dev = 0;
    cudaError_t cerr = cudaGetDevice(&dev);
    if (cerr == cudaSuccess) cerr = cudaEventRecord(L->entry, stream);
    if (cerr != cudaSuccess) return fmb::cuda_status(cerr, "record load: entry event");
    uint8_t *dst = static_cast<uint8_t *>(slot);
    std::atomic<size_t> next_job{0};
    std::atomic<uint64_t> physical{0}, fallbacks{0};
    std::vector<std::atomic<bool>> fell_back(groups.size());
    for (auto &f : fell_back) f.store(false);
    std::atomic<bool> failed{false};
    std::mutex err_mutex;
    int err_code = FM_STATUS_OK;
    std::string err_msg;
    const size_t n_readers = std::max<size_t>(1, std::min(L->readers.size(), jobs.size()));

    auto reader = [&](size_t t) {
        auto fail = [&](int code) {
            std::lock_guard<std::mutex> lock(err_mutex);
            if (err_code == FM_STATUS_OK) {
                err_code = code;
                err_msg = fmcuda_last_error();
            }
            failed.store(true);
        };
        auto cuda_fail = [&](cudaError_t e, const char *what) {
            (void)cudaGetLastError();
            const int code = fmb::cuda_status(e, what);
            fail(code == FM_STATUS_DEVICE_LOSS || code == FM_STATUS_ALLOCATION_FAILED ? code
                 : set_error(FM_STATUS_TRANSFER_FAILED, fmcuda_last_error()));
        };
        Reader &R = L->readers[t];
        cudaError_t e = cudaSetDevice(dev);
        // copies into the slot start after the caller's earlier work on it
        if (e == cudaSuccess) e = cudaStreamWaitEvent(R.stream, L->entry, 0);
        if (e != cudaSuccess) return cuda_fail(e, "record load: reader stream");
        for (;;) {
            const size_t j = next_job.fetch_add(1);
            if (j >= jobs.size() || failed.load()) break;
            const Job &J = jobs[j];
            const size_t i = R.next;
            R.next = (R.next + 1) % R.buf.size();
            if (R.busy[i]) {
                if (int rc = wait_event(R.ev[i], timeout_ms)) return fail(rc);
                R.busy[i] = false;
            }
            uint8_t *buf = R.buf[i];
            uint64_t base = J.pos;
            bool have = false;
            if (J.direct && !fell_back[J.group].load()) {
                const ssize_t r = pread_full(L->direct_fd, buf, J.n, J.pos);
                if (r >= 0 && J.pos + static_cast<uint64_t>(r) >= J.hi) {
                    physical += static_cast<uint64_t>(r);
                    have = true;
                } else if (!fell_back[J.group].exchange(true)) {
                    ++fallbacks; // the file system refused: buffered reads for the rest of the group
                }
            }
            if (!have) {
                const uint64_t n = J.hi - J.lo;
                const ssize_t r = pread_full(L->fd, buf, n, J.lo);
                if (r < 0) return fail(set_error(FM_STATUS_IO_ERROR, "pread failed for " + L->path + ": " +
                                                                         std::strerror(errno)));
                if (static_cast<uint64_t>(r) < n) return fail(set_error(FM_STATUS_SHORT_READ, "short read from " + L->path));
                physical += n;
                base = J.lo;
            }
            for (uint32_t m : groups[J.group].members) {
                const uint64_t a = std::max(J.lo, extents[m].offset);
                const uint64_t b = std::min(J.hi, extents[m].offset + extents[m].size);
                if (a >= b) continue;
                e = cudaMemcpyAsync(dst + out_off[m] + (a - extents[m].offset), buf + (a - base), b - a,
                                    cudaMemcpyHostToDevice, R.stream);
                if (e != cudaSuccess) return cuda_fail(e, "record load: host-to-device copy");
            }
            if ((e = cudaEventRecord(R.ev[i], R.stream)) != cudaSuccess) return cuda_fail(e, "record load: chunk event");
            R.busy[i] = true;
        }
        if ((e = cudaEventRecord(R.tail, R.stream)) != cudaSuccess) return cuda_fail(e, "record load: reader tail");
    };
    if (n_readers == 1) {
        reader(0);
    } else {
        std::vector<std::thread> pool;
        for (size_t t = 0; t < n_readers; ++t) pool.emplace_back(reader, t);
        for (auto &th : pool) th.join();
    }
    stats->physical_bytes = physical.load();
    stats->direct_fallbacks += fallbacks.load();
    if (err_code != FM_STATUS_OK) {
        // Copies the other readers issued before the failure may still be
        // writing into the slot: order the caller's stream after every
        // reader's last copy, and give them the timeout to finish, so a caller
        // that reuses the slot after this error never sees late writes.
        for (size_t t = 0; t < n_readers; ++t) {
            Reader &R = L->readers[t];
            if (cudaEventRecord(R.tail, R.stream) != cudaSuccess ||
                cudaStreamWaitEvent(stream, R.tail, 0) != cudaSuccess) {
                (void)cudaGetLastError();
                continue;
            }
            if (wait_event(R.tail, timeout_ms) == FM_STATUS_OK) R.busy.assign(R.busy.size(), false);
        }
        return set_error(err_code, err_msg);
    }
    for (size_t t = 0; t < n_readers; ++t) {
        cerr = cudaStreamWaitEvent(stream, L->readers[t].tail, 0);
        if (cerr != cudaSuccess) return fmb::cuda_status(cerr, "record load: join");
    }

    // FNV-1a 64 of the slot bytes, on the device, then back to the host
    uint64_t *d_sum = static_cast<uint64_t *>(workspace);
    if (int rc = fmb::fnv1a64_launch(dst, payload, d_sum, static_cast<uint8_t *>(workspace) + 256,
                                     workspace_bytes - 256, stream))
        return rc;
    cerr = cudaMemcpyAsync(L->host_word, d_sum, 8, cudaMemcpyDeviceToHost, stream);
    if (cerr == cudaSuccess) cerr = cudaEventRecord(L->done, stream);
    if (cerr != cudaSuccess) return fmb::cuda_status(cerr, "record load: checksum read-back");
    if (int rc = wait_event(L->done, timeout_ms)) return rc;
    // every reader's copies are behind `done`
    for (size_t t = 0; t < n_readers; ++t) L->readers[t].busy.assign(L->readers[t].busy.size(), false);
    stats->checksum = *L->host_word;
    stats->elapsed_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (checksum_known && stats->checksum != expected_checksum)
        return set_error(FM_STATUS_EXPERT_CHECKSUM_MISMATCH, "expert checksum mismatch (source or transfer)");
    return FM_STATUS_OK;
}

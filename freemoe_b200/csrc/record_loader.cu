// record_loader.cu -- cold -> warm expert loads on the host side of the path:
// file extents are read straight into a ring of pinned chunks and copied to the
// HBM slot with cudaMemcpyAsync while the next chunk is read; the checksum is
// FNV-1a 64 of the slot computed on the device (fnv.cu).
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
#include <cerrno>
#include <chrono>
#include <cstring>
#include <limits>
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
    std::vector<void *> ring_raw;     // pinned allocations, `chunk` + `alignment` bytes
    std::vector<void *> ring;         // the aligned `chunk` bytes inside each
    std::vector<cudaEvent_t> ring_ev; // last copy out of each chunk
    std::vector<bool> ring_busy;
    uint64_t *host_word = nullptr;    // pinned: the checksum read back
    cudaEvent_t done = nullptr;
    size_t next = 0;

    ~fmcuda_record_loader() {
        for (size_t i = 0; i < ring.size(); ++i) {
            if (ring_ev[i]) {
                (void)cudaEventSynchronize(ring_ev[i]);
                (void)cudaEventDestroy(ring_ev[i]);
            }
            if (ring_raw[i]) (void)cudaFreeHost(ring_raw[i]);
        }
        if (done) {
            (void)cudaEventSynchronize(done);
            (void)cudaEventDestroy(done);
        }
        if (host_word) (void)cudaFreeHost(host_word);
        if (fd >= 0) ::close(fd);
        if (direct_fd >= 0) ::close(direct_fd);
    }

    // polled, bounded wait for one event (Backend::wait_fence semantics)
    int wait(cudaEvent_t ev, uint32_t timeout_ms) {
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
};

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
                                           uint64_t chunk_bytes, uint32_t ring_depth,
                                           int force_direct_fallback, const fmcuda_file_identity *expected,
                                           fmcuda_record_loader **out) {
    if (!path || !out) return set_error(FM_STATUS_INVALID_ARGUMENT, "record loader: null argument");
    *out = nullptr;
    if (reader_mode != FM_READER_BUFFERED && reader_mode != FM_READER_DIRECT)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "record loader: reader mode must be buffered or direct");
    if (ring_depth < 2 || ring_depth > 64 || chunk_bytes < (1u << 16) || chunk_bytes > (1ull << 30))
        return set_error(FM_STATUS_INVALID_ARGUMENT, "record loader: ring of 2..64 chunks of 64 KiB..1 GiB");
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
    L->ring_raw.assign(ring_depth, nullptr);
    L->ring.assign(ring_depth, nullptr);
    L->ring_ev.assign(ring_depth, nullptr);
    L->ring_busy.assign(ring_depth, false);
    for (uint32_t i = 0; i < ring_depth && !rc; ++i) {
        cudaError_t err = cudaHostAlloc(&L->ring_raw[i], L->chunk + L->alignment, cudaHostAllocDefault);
        if (err == cudaSuccess) {
            const uintptr_t a = reinterpret_cast<uintptr_t>(L->ring_raw[i]);
            L->ring[i] = reinterpret_cast<void *>((a + L->alignment - 1) & ~uintptr_t(L->alignment - 1));
        }
        if (err == cudaSuccess) err = cudaEventCreateWithFlags(&L->ring_ev[i], cudaEventDisableTiming);
        if (err != cudaSuccess) rc = fmb::cuda_status(err, "record loader: pinned ring");
    }
    if (!rc) {
        cudaError_t err = cudaHostAlloc(reinterpret_cast<void **>(&L->host_word), 64, cudaHostAllocDefault);
        if (err == cudaSuccess) err = cudaEventCreateWithFlags(&L->done, cudaEventDisableTiming);
        if (err != cudaSuccess) rc = fmb::cuda_status(err, "record loader: checksum word");
    }
    if (rc) {
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
    uint8_t *dst = static_cast<uint8_t *>(slot);

    // copies of the file bytes [lo, hi), held in `buf` from file offset `base`
    auto dispatch = [&](const Group &g, const uint8_t *buf, uint64_t base, uint64_t lo, uint64_t hi) -> int {
        for (uint32_t i : g.members) {
            const uint64_t a = std::max(lo, extents[i].offset);
            const uint64_t b = std::min(hi, extents[i].offset + extents[i].size);
            if (a >= b) continue;
            const cudaError_t err = cudaMemcpyAsync(dst + out_off[i] + (a - extents[i].offset), buf + (a - base),
                                                    b - a, cudaMemcpyHostToDevice, stream);
            if (err != cudaSuccess) {
                (void)cudaGetLastError();
                const int code = fmb::cuda_status(err, "record load: host-to-device copy");
                return code == FM_STATUS_DEVICE_LOSS ? code : set_error(FM_STATUS_TRANSFER_FAILED, fmcuda_last_error());
            }
        }
        return FM_STATUS_OK;
    };
    // next ring chunk, once the copies out of it have finished
    auto take = [&](uint8_t **buf, size_t *idx) -> int {
        const size_t i = L->next;
        L->next = (L->next + 1) % L->ring.size();
        if (L->ring_busy[i]) {
            if (int rc = L->wait(L->ring_ev[i], timeout_ms)) return rc;
            L->ring_busy[i] = false;
        }
        *buf = static_cast<uint8_t *>(L->ring[i]);
        *idx = i;
        return FM_STATUS_OK;
    };
    auto release = [&](size_t i) -> int {
        const cudaError_t err = cudaEventRecord(L->ring_ev[i], stream);
        if (err != cudaSuccess) return fmb::cuda_status(err, "record load: chunk event");
        L->ring_busy[i] = true;
        return FM_STATUS_OK;
    };
    // buffered reads of [from, g.end)
    auto read_buffered = [&](const Group &g, uint64_t from) -> int {
        for (uint64_t pos = from; pos < g.end;) {
            uint8_t *buf;
            size_t idx;
            if (int rc = take(&buf, &idx)) return rc;
            const uint64_t n = std::min(L->chunk, g.end - pos);
            const ssize_t r = pread_full(L->fd, buf, n, pos);
            if (r < 0) return set_error(FM_STATUS_IO_ERROR, "pread failed for " + L->path + ": " + std::strerror(errno));
            if (static_cast<uint64_t>(r) < n) return set_error(FM_STATUS_SHORT_READ, "short read from " + L->path);
            stats->physical_bytes += n;
            if (int rc = dispatch(g, buf, pos, pos, pos + n)) return rc;
            if (int rc = release(idx)) return rc;
            pos += n;
        }
        return FM_STATUS_OK;
    };

    for (const Group &g : groups) {
        ++stats->read_requests;
        stats->coalesced_requests += g.members.size() - 1;
        const bool direct = L->mode == FM_READER_DIRECT && !L->force_fallback && L->direct_fd >= 0;
        if (!direct) {
            if (L->mode == FM_READER_DIRECT) ++stats->direct_fallbacks;
            if (int rc = read_buffered(g, g.offset)) return rc;
            continue;
        }
        // aligned span [a0, a1) in chunk-sized direct reads
        const uint64_t A = L->alignment;
        const uint64_t a0 = g.offset & ~(A - 1);
        const uint64_t a1 = (g.end + A - 1) & ~(A - 1);
        uint64_t covered = g.offset; // file bytes of the group already dispatched
        for (uint64_t pos = a0; pos < a1 && covered < g.end;) {
            uint8_t *buf;
            size_t idx;
            if (int rc = take(&buf, &idx)) return rc;
            const uint64_t n = std::min(L->chunk, a1 - pos);
            const ssize_t r = pread_full(L->direct_fd, buf, n, pos);
            const uint64_t want = std::min(pos + n, g.end) - covered; // bytes this chunk must supply
            if (r < 0 || pos + static_cast<uint64_t>(r) < covered + want) {
                // the file system refused or came up short: buffered reads for the rest
                L->ring_busy[idx] = false;
                ++stats->direct_fallbacks;
                break;
            }
            stats->physical_bytes += static_cast<uint64_t>(r);
            if (int rc = dispatch(g, buf, pos, covered, covered + want)) return rc;
            if (int rc = release(idx)) return rc;
            covered += want;
            pos += n;
        }
        if (covered < g.end)
            if (int rc = read_buffered(g, covered)) return rc;
    }

    // FNV-1a 64 of the slot bytes, on the device, then back to the host
    uint64_t *d_sum = static_cast<uint64_t *>(workspace);
    if (int rc = fmb::fnv1a64_launch(dst, payload, d_sum, static_cast<uint8_t *>(workspace) + 256,
                                     workspace_bytes - 256, stream))
        return rc;
    cudaError_t err = cudaMemcpyAsync(L->host_word, d_sum, 8, cudaMemcpyDeviceToHost, stream);
    if (err == cudaSuccess) err = cudaEventRecord(L->done, stream);
    if (err != cudaSuccess) return fmb::cuda_status(err, "record load: checksum read-back");
    if (int rc = L->wait(L->done, timeout_ms)) return rc;
    for (size_t i = 0; i < L->ring.size(); ++i) L->ring_busy[i] = false; // all copies are behind `done`
    stats->checksum = *L->host_word;
    stats->elapsed_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (checksum_known && stats->checksum != expected_checksum)
        return set_error(FM_STATUS_EXPERT_CHECKSUM_MISMATCH, "expert checksum mismatch (source or transfer)");
    return FM_STATUS_OK;
}

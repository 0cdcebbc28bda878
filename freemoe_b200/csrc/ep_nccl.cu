// ep_nccl.cu -- expert parallelism over NCCL from the C ABI: a communicator
// per expert-parallel group and one call for a whole MoE layer, so that a C++
// host (FreeMoe's engine, a serving loop) drives the sharded layer without
// Python.  No counterpart in the reference (FreeMoe runs every expert in one
// process); the per-rank arithmetic is the reference's expert loop
// (src/engine.cpp:1711-1772) on this library's kernels.
//
// One fmcuda_ep_layer call, all on the caller's stream (the same steps as the
// Python layer's "rows" exchange, freemoe_b200/ep.py, and the same results bit
// for bit):
//   route     this rank's tokens -> ids, weights                (router.cu)
//   dispatch  one fp16 row per (token, destination rank) holding any of the
//             token's experts, with its local expert ids and routing weights
//             (fmcuda_ep_dispatch_rows)
//   counts    per-destination row counts, ncclSend/ncclRecv of one uint32 per
//             peer; the host reads both count vectors (one stream
//             synchronisation per call) to size the row exchange
//   rows out  grouped ncclSend/ncclRecv of the rows and their metadata
//   experts   every received row through this rank's experts, the outputs of
//             its slots summed in top-k order (fmcuda_moe_experts_partial)
//   rows back the f32 partial rows to the tokens' owners
//   combine   y[t] = sum over ranks of the partial rows (fmcuda_ep_combine_rows)
//
// NCCL is resolved at run time (dlopen of libnccl.so.2), so the library shares
// the NCCL a host process already holds (PyTorch's, for instance) and needs no
// link-time dependency; only the long-stable part of the API is used.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace fmb {

int launch_route_cfg(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
                     const fmcuda_router_config *cfg, int32_t normalise, double epsilon, double scale,
                     uint32_t *ids, float *weights, float *probs, cudaStream_t s);

namespace {

inline uint64_t a256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto get = [&](auto &fn, const char *name) { fn = reinterpret_cast<std::decay_t<decltype(fn)>>(dlsym(h, name)); };
        get(n.get_unique_id, "ncclGetUniqueId");
        get(n.comm_init_rank, "ncclCommInitRank");
        get(n.comm_destroy, "ncclCommDestroy");
        get(n.group_start, "ncclGroupStart");
        get(n.group_end, "ncclGroupEnd");
        get(n.send, "ncclSend");
        get(n.recv, "ncclRecv");
        get(n.error_string, "ncclGetErrorString");
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.group_start && n.group_end && n.send &&
               n.recv && n.error_string;
    });
    return n;
}

// An NCCL failure is a TRANSFER_FAILED status with NCCL's message.
int nccl_status(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return FM_STATUS_OK;
    return set_error(FM_STATUS_TRANSFER_FAILED, std::string(what) + ": " + nccl().error_string(r));
}

int need_nccl() {
    return nccl().ok ? FM_STATUS_OK
                     : set_error(FM_STATUS_INTERNAL_ERROR, "NCCL (libnccl.so.2) could not be loaded");
}

struct EpComm {
    ncclComm_t comm = nullptr;
    uint32_t rank = 0, world = 0;
    int device = 0;
    std::vector<uint32_t> send_counts, recv_counts; // host copies of the last call's counts
};

// Workspace of one layer call.
struct LayerLayout {
    uint64_t ids, w, send_counts, recv_counts, send_offsets, items, row_of, send_x, meta_e, meta_w, scratch;
    uint64_t recv_x, recv_e, recv_w, partial, back, experts, total;
};

LayerLayout layer_layout(uint32_t tokens_max, uint32_t world, uint32_t experts_local, uint32_t top_k, uint32_t d,
                         uint32_t ffn) {
    LayerLayout L{};
    const uint64_t T = tokens_max, n = T * world; // send rows and, at most, received rows
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = o;
        o += a256(bytes);
        return at;
    };
    L.ids = take(T * top_k * 4);
    L.w = take(T * top_k * 4);
    L.send_counts = take(world * 4ull);
    L.recv_counts = take(world * 4ull);
    L.send_offsets = take((world + 1ull) * 4);
    L.items = take(n * 4);
    L.row_of = take(n * 4);
    L.send_x = take(n * d * 2);
    L.meta_e = take(n * top_k * 4);
    L.meta_w = take(n * top_k * 4);
    L.scratch = take(fmcuda_ep_dispatch_rows_scratch_bytes(static_cast<uint32_t>(T), world));
    L.recv_x = take(n * d * 2);
    L.recv_e = take(n * top_k * 4);
    L.recv_w = take(n * top_k * 4);
    L.partial = take(n * d * 4);
    L.back = take(n * d * 4);
    L.experts = take(fmcuda_moe_experts_partial_workspace_bytes(static_cast<uint32_t>(n), top_k, experts_local, d, ffn));
    L.total = o;
    return L;
}

} // namespace
} // namespace fmb

using namespace fmb;

extern "C" int fmcuda_ep_nccl_unique_id(void *uid) {
    if (!uid) return set_error(FM_STATUS_INVALID_ARGUMENT, "null NCCL id buffer");
    int rc = need_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    if ((rc = nccl_status(nccl().get_unique_id(&id), "ncclGetUniqueId"))) return rc;
    memcpy(uid, &id, sizeof(id));
    return FM_STATUS_OK;
}

extern "C" int fmcuda_ep_init(const void *nccl_uid, uint32_t rank, uint32_t world, void **comm) {
    if (!nccl_uid || !comm) return set_error(FM_STATUS_INVALID_ARGUMENT, "null expert-parallel init pointer");
    if (world == 0 || rank >= world) return set_error(FM_STATUS_INVALID_ARGUMENT, "rank must be below world");
    int rc = need_nccl();
    if (rc) return rc;
    auto *c = new EpComm;
    c->rank = rank;
    c->world = world;
    cudaGetDevice(&c->device);
    ncclUniqueId id;
    memcpy(&id, nccl_uid, sizeof(id));
    if ((rc = nccl_status(nccl().comm_init_rank(&c->comm, static_cast<int>(world), id, static_cast<int>(rank)),
                          "ncclCommInitRank"))) {
        delete c;
        return rc;
    }
    c->send_counts.assign(world, 0);
    c->recv_counts.assign(world, 0);
    *comm = c;
    return FM_STATUS_OK;
}

extern "C" int fmcuda_ep_destroy(void *comm) {
    if (!comm) return FM_STATUS_OK;
    auto *c = static_cast<EpComm *>(comm);
    const int rc = nccl_status(nccl().comm_destroy(c->comm), "ncclCommDestroy");
    delete c;
    return rc;
}

extern "C" int fmcuda_ep_layer_workspace_bytes(uint32_t tokens_max, uint32_t world, uint32_t experts_local,
                                               uint32_t top_k, uint32_t d_model, uint32_t ffn, uint64_t *bytes) {
    if (!bytes) return set_error(FM_STATUS_INVALID_ARGUMENT, "null size pointer");
    if (world == 0) return set_error(FM_STATUS_INVALID_ARGUMENT, "world must be positive");
    *bytes = layer_layout(tokens_max, world, experts_local, top_k, d_model, ffn).total;
    return FM_STATUS_OK;
}

extern "C" int fmcuda_ep_layer(void *comm, const fmcuda_ep_layer_args *a, uint32_t tokens_max, void *workspace,
                               uint64_t workspace_bytes, void *stream) {
    if (!comm || !a) return set_error(FM_STATUS_INVALID_ARGUMENT, "null expert-parallel layer argument");
    auto *c = static_cast<EpComm *>(comm);
    const uint32_t world = c->world, T = a->tokens, k = a->top_k, d = a->d_model;
    if (a->experts == 0 || a->experts % world)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "experts must shard evenly over the ranks");
    if (T > tokens_max) return set_error(FM_STATUS_INVALID_ARGUMENT, "tokens above tokens_max");
    if (!a->x || !a->logits || !a->local_slots || !a->y || !workspace)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null expert-parallel layer pointer");
    const uint32_t per = a->experts / world;
    const LayerLayout L = layer_layout(tokens_max, world, per, k, d, a->ffn);
    if (workspace_bytes < L.total)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "expert-parallel workspace too small: need " +
                                                         std::to_string(L.total) + " bytes");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    auto *ids = reinterpret_cast<uint32_t *>(ws + L.ids);
    auto *w = reinterpret_cast<float *>(ws + L.w);
    auto *send_counts = reinterpret_cast<uint32_t *>(ws + L.send_counts);
    auto *recv_counts = reinterpret_cast<uint32_t *>(ws + L.recv_counts);
    auto *row_of = reinterpret_cast<uint32_t *>(ws + L.row_of);
    auto *send_x = reinterpret_cast<__half *>(ws + L.send_x);
    auto *meta_e = reinterpret_cast<int32_t *>(ws + L.meta_e);
    auto *meta_w = reinterpret_cast<float *>(ws + L.meta_w);
    auto *recv_x = reinterpret_cast<__half *>(ws + L.recv_x);
    auto *recv_e = reinterpret_cast<int32_t *>(ws + L.recv_e);
    auto *recv_w = reinterpret_cast<float *>(ws + L.recv_w);
    auto *partial = reinterpret_cast<float *>(ws + L.partial);
    auto *back = reinterpret_cast<float *>(ws + L.back);
    const Nccl &n = nccl();

    int rc = launch_route_cfg(a->logits, T, a->experts, k, nullptr, a->normalise, a->epsilon, a->scale, ids, w,
                              nullptr, s);
    if (rc) return rc;
    if ((rc = fmcuda_ep_dispatch_rows(ids, w, T, k, per, world, a->x, a->x_dtype, d, send_counts,
                                      reinterpret_cast<uint32_t *>(ws + L.send_offsets),
                                      reinterpret_cast<uint32_t *>(ws + L.items), row_of, send_x, meta_e, meta_w,
                                      ws + L.scratch, s)))
        return rc;
    // counts: one uint32 to and from every rank, then read on the host
    if ((rc = nccl_status(n.group_start(), "ncclGroupStart"))) return rc;
    for (uint32_t p = 0; p < world; ++p) {
        if ((rc = nccl_status(n.send(send_counts + p, 1, ncclUint32, static_cast<int>(p), c->comm, s), "ncclSend")) ||
            (rc = nccl_status(n.recv(recv_counts + p, 1, ncclUint32, static_cast<int>(p), c->comm, s), "ncclRecv"))) {
            (void)n.group_end();
            return rc;
        }
    }
    if ((rc = nccl_status(n.group_end(), "ncclGroupEnd"))) return rc;
    cudaError_t err = cudaMemcpyAsync(c->send_counts.data(), send_counts, world * 4ull, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess)
        err = cudaMemcpyAsync(c->recv_counts.data(), recv_counts, world * 4ull, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return cuda_status(err, "expert-parallel counts");
    std::vector<uint64_t> so(world + 1, 0), ro(world + 1, 0);
    for (uint32_t p = 0; p < world; ++p) {
        so[p + 1] = so[p] + c->send_counts[p];
        ro[p + 1] = ro[p] + c->recv_counts[p];
    }
    if (ro[world] > static_cast<uint64_t>(tokens_max) * world)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "a peer sent more rows than tokens_max allows");
    // rows out: fp16 rows and their slot metadata, grouped by peer
    if ((rc = nccl_status(n.group_start(), "ncclGroupStart"))) return rc;
    for (uint32_t p = 0; p < world && !rc; ++p) {
        const int peer = static_cast<int>(p);
        const uint64_t ns = c->send_counts[p], nr = c->recv_counts[p];
        if (ns)
            rc = nccl_status(n.send(send_x + so[p] * d, ns * d, ncclFloat16, peer, c->comm, s), "ncclSend");
        if (!rc && ns) rc = nccl_status(n.send(meta_e + so[p] * k, ns * k, ncclInt32, peer, c->comm, s), "ncclSend");
        if (!rc && ns) rc = nccl_status(n.send(meta_w + so[p] * k, ns * k, ncclFloat32, peer, c->comm, s), "ncclSend");
        if (!rc && nr) rc = nccl_status(n.recv(recv_x + ro[p] * d, nr * d, ncclFloat16, peer, c->comm, s), "ncclRecv");
        if (!rc && nr) rc = nccl_status(n.recv(recv_e + ro[p] * k, nr * k, ncclInt32, peer, c->comm, s), "ncclRecv");
        if (!rc && nr) rc = nccl_status(n.recv(recv_w + ro[p] * k, nr * k, ncclFloat32, peer, c->comm, s), "ncclRecv");
    }
    const int rc_end = nccl_status(n.group_end(), "ncclGroupEnd");
    if (rc || (rc = rc_end)) return rc;
    // this rank's experts
    const uint32_t R = static_cast<uint32_t>(ro[world]), S = static_cast<uint32_t>(so[world]);
    if (R && (rc = fmcuda_moe_experts_partial(recv_x, recv_e, recv_w, R, k, per, a->local_slots, a->up_offset,
                                              a->down_offset, a->gate_type, a->up_type, a->down_type, d, a->ffn,
                                              partial, ws + L.experts, L.total - L.experts, s)))
        return rc;
    // rows back: the partial sums to the tokens' owners
    if ((rc = nccl_status(n.group_start(), "ncclGroupStart"))) return rc;
    for (uint32_t p = 0; p < world && !rc; ++p) {
        const int peer = static_cast<int>(p);
        const uint64_t ns = c->send_counts[p], nr = c->recv_counts[p];
        if (nr) rc = nccl_status(n.send(partial + ro[p] * d, nr * d, ncclFloat32, peer, c->comm, s), "ncclSend");
        if (!rc && ns) rc = nccl_status(n.recv(back + so[p] * d, ns * d, ncclFloat32, peer, c->comm, s), "ncclRecv");
    }
    const int rc_end2 = nccl_status(n.group_end(), "ncclGroupEnd");
    if (rc || (rc = rc_end2)) return rc;
    (void)S;
    return fmcuda_ep_combine_rows(back, row_of, T, world, d, a->y, s);
}

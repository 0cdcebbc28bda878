// ep_p2p.cu -- the expert-parallel exchange over peer memory (NVLink P2P
// stores into the peers' mailboxes), fused into the kernels that produce the
// data: the pack kernel writes each token row straight into the destination
// rank's receive rows, and the kernel that sums a received row's expert
// outputs writes the partial sum straight back into the source rank's return
// rows.  No collective library call and no host read of the split sizes.
//
// Every rank owns one mailbox (cudaMalloc, shared with the other ranks of the
// node through CUDA IPC handles):
//   matrix[s][r]  rows rank s sends to rank r (each rank writes its own row s
//                 into every mailbox, then raises mflag[s])
//   mflag/dflag/bflag[s]  epochs: s's matrix row / s's token rows / s's
//                 returned partial rows have arrived in this mailbox
//   plan          derived locally: recv offsets per source, rows received,
//                 this rank's first row at every destination
//   recv_x, recv_e, recv_w   received token rows (fp16), local expert ids and
//                 routing weights per top-k slot (-1 / 0 for other ranks')
//   back          f32 partial sums returned for this rank's sent rows
// A call carries an epoch (1, 2, ...); flags are only ever raised to the
// current epoch, so nothing is reset between calls.  Epoch 0 in the three
// calls means "the device's epoch": one past a counter in this rank's own
// mailbox, which the combine call advances when it has finished, so a layer's
// calls can be captured once in a CUDA graph and replayed (a layer uses either
// explicit epochs or device epochs, not both).
// For decode-sized calls (tokens x ranks <= 512, <= 32 ranks) the dispatch is
// one kernel: every CTA derives the grouping by destination and the plan
// itself, CTA 0 publishes this rank's counts, and every CTA packs its rows once
// all ranks' counts are in.  The combine kernel waits for the returned rows
// itself.  Buffer reuse is ordered
// by the protocol itself: a rank sends epoch e+1 rows only after its epoch-e
// partials came back from every destination, which each destination writes
// only after it has read its epoch-e rows.
//
// Every wait is bounded (default 2 s of %globaltimer): on expiry the kernel
// raises FM_STATUS_FENCE_TIMEOUT in the device status word and carries on, so
// a missing peer turns into an error the host reads, never a hang.
// Flags use release stores / acquire loads at system scope; data stores are
// ordered before them by a system fence in every writing thread and a
// last-block count.
#include <string>

#include "common.cuh"
#include "p2p_flags.cuh"
#include "tgemv_host.h"
#include "router_core.cuh"

namespace fmb {

uint64_t group_scratch_bytes(uint32_t n_pairs, uint32_t experts);
int launch_group_large(const uint32_t *ids, uint32_t n_pairs, uint32_t experts, uint32_t *counts,
                       uint32_t *offsets, uint32_t *pairs, uint32_t *slot_of, uint32_t *scratch, cudaStream_t s);
int experts_partial_run(const void *x, const int32_t *meta_expert, const float *meta_weight, uint32_t rows,
                        const uint32_t *rows_dev, uint32_t top_k, uint32_t experts, const void *const *expert_slots,
                        uint64_t up_offset, uint64_t down_offset, uint32_t gate_type, uint32_t up_type,
                        uint32_t down_type, uint32_t d_model, uint32_t ffn, float *out_pairs, void *workspace,
                        uint64_t workspace_bytes, cudaStream_t s, const TgRecvWait *recv);
bool partial_fused_recv(uint32_t rows, uint32_t top_k, uint32_t experts, uint32_t d_model, uint32_t ffn,
                        uint32_t gate_type, uint32_t up_type, uint32_t down_type, uint64_t up_offset,
                        uint64_t down_offset);
uint64_t experts_pairs_workspace_bytes(uint32_t rows, uint32_t top_k, uint32_t experts, uint32_t d, uint32_t ffn);

namespace {

inline uint64_t a256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

struct Mailbox {
    uint64_t matrix, mflag, dflag, bflag, ctr, recv_off, n_recv, my_pos, src_pos, recv_x, recv_e, recv_w, back,
        total;
};

// cap: rows a mailbox can receive (and return rows it can take back).
Mailbox mailbox_layout(uint32_t world, uint32_t cap, uint32_t top_k, uint32_t d) {
    Mailbox L{};
    uint64_t o = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t at = o;
        o += a256(bytes);
        return at;
    };
    L.matrix = take(static_cast<uint64_t>(world) * world * 4);
    L.mflag = take(world * 4ull);
    L.dflag = take(world * 4ull);
    L.bflag = take(world * 4ull);
    L.ctr = take(16);
    L.recv_off = take((world + 1ull) * 4);
    L.n_recv = take(4);
    L.my_pos = take(world * 4ull);  // this rank's first row in destination r's receive rows
    L.src_pos = take(world * 4ull); // source s's first send row of the rows it sends here
    L.recv_x = take(static_cast<uint64_t>(cap) * d * 2);
    L.recv_e = take(static_cast<uint64_t>(cap) * top_k * 4);
    L.recv_w = take(static_cast<uint64_t>(cap) * top_k * 4);
    L.back = take(static_cast<uint64_t>(cap) * d * 4);
    L.total = o;
    return L;
}

template <typename T> __device__ __forceinline__ T *at(uint8_t *base, uint64_t off) {
    return reinterpret_cast<T *>(base + off);
}

// Thread p writes this rank's row of the count matrix into mailbox p, then
// raises mflag[rank] there.
__global__ void p2p_counts_kernel(uint8_t *const *peers, uint32_t world, uint32_t rank, const uint32_t *send_counts,
                                  uint64_t off_matrix, uint64_t off_mflag, uint32_t epoch, const uint32_t *ectr) {
    const uint32_t p = threadIdx.x;
    if (p >= world) return;
    epoch = call_epoch(epoch, ectr);
    uint32_t *m = at<uint32_t>(peers[p], off_matrix) + static_cast<uint64_t>(rank) * world;
    for (uint32_t r = 0; r < world; ++r) m[r] = send_counts[r];
    __threadfence_system();
    flag_release(at<uint32_t>(peers[p], off_mflag) + rank, epoch);
}

// One warp: wait for every source's matrix row, then derive this rank's plan.
__global__ void p2p_plan_kernel(uint8_t *mine, Mailbox L, uint32_t world, uint32_t rank, uint32_t cap,
                                uint32_t epoch, uint64_t timeout_ns, int *status) {
    const uint32_t lane = threadIdx.x;
    epoch = call_epoch(epoch, at<uint32_t>(mine, L.ctr) + 2);
    for (uint32_t s = lane; s < world; s += 32) wait_flag(at<uint32_t>(mine, L.mflag) + s, epoch, timeout_ns, status);
    __syncwarp();
    if (lane != 0) return;
    const uint32_t *m = at<uint32_t>(mine, L.matrix);
    uint32_t *recv_off = at<uint32_t>(mine, L.recv_off), *my_pos = at<uint32_t>(mine, L.my_pos),
             *src_pos = at<uint32_t>(mine, L.src_pos);
    uint32_t acc = 0;
    for (uint32_t s = 0; s < world; ++s) {
        recv_off[s] = acc;
        acc += m[static_cast<uint64_t>(s) * world + rank];
        uint32_t before = 0; // rows source s sends to ranks below this one
        for (uint32_t r = 0; r < rank; ++r) before += m[static_cast<uint64_t>(s) * world + r];
        src_pos[s] = before;
    }
    recv_off[world] = acc;
    // rows past the capacity were dropped by their senders: count only the kept ones
    if (acc > cap) raise_device_status(status, FM_STATUS_INVALID_ARGUMENT);
    *at<uint32_t>(mine, L.n_recv) = acc < cap ? acc : cap;
    for (uint32_t r = 0; r < world; ++r) {
        uint32_t before = 0; // rows of lower sources at destination r
        for (uint32_t s = 0; s < rank; ++s) before += m[static_cast<uint64_t>(s) * world + r];
        my_pos[r] = before;
    }
}

// Block j: send item j (token t = item / world to rank dest = item % world):
// the fp16 token row and the top-k metadata, into the destination's mailbox.
// The last block to finish raises dflag[rank] in every mailbox.
template <typename XT>
__global__ void p2p_pack_send_kernel(const XT *__restrict__ x, const uint32_t *__restrict__ ids,
                                     const float *__restrict__ w, const uint32_t *__restrict__ items,
                                     const uint32_t *__restrict__ send_offsets, uint32_t top_k, uint32_t per_rank,
                                     uint32_t world, uint32_t rank, uint32_t d, uint8_t *const *peers, uint8_t *mine,
                                     Mailbox L, uint32_t cap, uint32_t epoch, int *status) {
    const uint32_t j = blockIdx.x;
    epoch = call_epoch(epoch, at<uint32_t>(mine, L.ctr) + 2);
    if (j < send_offsets[world]) {
        const uint32_t item = items[j], t = item / world, dest = item % world;
        const uint32_t pos = at<uint32_t>(mine, L.my_pos)[dest] + (j - send_offsets[dest]);
        if (pos >= cap) { // a destination receiving more than its capacity: refuse, never write past it
            if (threadIdx.x == 0) raise_device_status(status, FM_STATUS_INVALID_ARGUMENT);
            goto done;
        }
        {
        uint8_t *peer = peers[dest];
        const XT *src = x + static_cast<uint64_t>(t) * d;
        uint4 *dst = reinterpret_cast<uint4 *>(at<__half>(peer, L.recv_x) + static_cast<uint64_t>(pos) * d);
        const bool vec = sizeof(XT) == 2 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
        // this block's share of the row's 16-byte pieces (grid.y splits the row)
        const uint32_t per = (d / 8 + gridDim.y - 1) / gridDim.y, c0 = blockIdx.y * per;
        const uint32_t c1 = min(d / 8, c0 + per);
        for (uint32_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
            __align__(16) __half h[8];
            if (vec) { // eight bf16 in one 16-byte load
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src) + c);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    h[2 * i] = __float2half_rn(__uint_as_float(u[i] << 16));
                    h[2 * i + 1] = __float2half_rn(__uint_as_float(u[i] & 0xFFFF0000u));
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(load_x(src + 8 * c + i));
            }
            dst[c] = *reinterpret_cast<const uint4 *>(h);
        }
        int32_t *me = at<int32_t>(peer, L.recv_e) + static_cast<uint64_t>(pos) * top_k;
        float *mw = at<float>(peer, L.recv_w) + static_cast<uint64_t>(pos) * top_k;
        for (uint32_t r = threadIdx.x; blockIdx.y == 0 && r < top_k; r += blockDim.x) {
            const uint32_t e = ids[static_cast<uint64_t>(t) * top_k + r];
            const bool local = e / per_rank == dest;
            me[r] = local ? static_cast<int32_t>(e % per_rank) : -1;
            mw[r] = local ? w[static_cast<uint64_t>(t) * top_k + r] : 0.0f;
        }
        }
    }
done:
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t *ctr = at<uint32_t>(mine, L.ctr);
        if (atomicAdd(ctr, 1u) == gridDim.x * gridDim.y - 1) {
            *ctr = 0;
            __threadfence_system();
            for (uint32_t r = 0; r < world; ++r) flag_release(at<uint32_t>(peers[r], L.dflag) + rank, epoch);
        }
    }
}

// The whole dispatch of a decode-sized call in one launch (grid = items x
// column pieces, 128 threads):
//   every CTA: keys (token t, destination r) -> r when t has an expert there,
//              the stable grouping by destination (router_core.cuh), then,
//              once every rank's counts have arrived, this rank's first row at
//              every destination;
//   CTA (0, 0): row_of, this rank's counts into every mailbox (+ mflag), and
//              the plan of the rows this rank receives (recv_off, n_recv,
//              src_pos) for the experts and return kernels;
//   block (j, c): item j's fp16 row piece c and metadata into the
//              destination's mailbox, as p2p_pack_send_kernel; the last block
//              raises dflag[rank] everywhere.
// Same rows, positions and flags as the counts / plan / pack kernels.
constexpr uint32_t kFusedMaxItems = 512, kFusedMaxWorld = 32;

template <typename XT>
__global__ void __launch_bounds__(128)
    p2p_send_kernel(const XT *__restrict__ x, const uint32_t *__restrict__ ids, const float *__restrict__ w,
                    uint32_t tokens, uint32_t top_k, uint32_t per_rank, uint32_t world, uint32_t rank, uint32_t d,
                    uint8_t *const *peers, uint8_t *mine, Mailbox L, uint32_t cap, uint32_t epoch, uint32_t *row_of,
                    uint64_t timeout_ns, int *status) {
    __shared__ uint32_t s_keys[kFusedMaxItems], s_items[kFusedMaxItems], s_slot[kFusedMaxItems];
    __shared__ uint32_t s_cnt[kFusedMaxWorld], s_offs[kFusedMaxWorld + 1], s_count[kFusedMaxWorld],
        s_off[kFusedMaxWorld], s_warp_tot[32], s_mypos[kFusedMaxWorld];
    epoch = call_epoch(epoch, at<uint32_t>(mine, L.ctr) + 2);
    const uint32_t n = tokens * world, tid = threadIdx.x;
    const bool first = blockIdx.x == 0 && blockIdx.y == 0;
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const uint32_t t = i / world, dest = i % world;
        bool any = false;
        for (uint32_t r = 0; r < top_k; ++r) any |= ids[static_cast<uint64_t>(t) * top_k + r] / per_rank == dest;
        s_keys[i] = any ? dest : 0xFFFFFFFFu;
    }
    if (tid < 32) s_warp_tot[tid] = 0;
    __syncthreads();
    group_block(s_keys, n, world, s_cnt, s_offs, s_items, s_slot, status, s_count, s_off, s_warp_tot);
    __syncthreads();
    if (first) {
        for (uint32_t i = tid; i < n; i += blockDim.x) row_of[i] = s_slot[i];
        for (uint32_t p = tid; p < world; p += blockDim.x) {
            uint32_t *m = at<uint32_t>(peers[p], L.matrix) + static_cast<uint64_t>(rank) * world;
            for (uint32_t r = 0; r < world; ++r) m[r] = s_cnt[r];
            __threadfence_system();
            flag_release(at<uint32_t>(peers[p], L.mflag) + rank, epoch);
        }
    }
    wait_flags_cta(at<uint32_t>(mine, L.mflag), world, epoch, timeout_ns, status);
    const uint32_t *m = at<uint32_t>(mine, L.matrix);
    for (uint32_t r = tid; r < world; r += blockDim.x) {
        uint32_t before = 0; // rows of lower sources at destination r
        for (uint32_t q = 0; q < rank; ++q) before += m[static_cast<uint64_t>(q) * world + r];
        s_mypos[r] = before;
    }
    if (first && tid == 0) {
        uint32_t *recv_off = at<uint32_t>(mine, L.recv_off), *src_pos = at<uint32_t>(mine, L.src_pos);
        uint32_t acc = 0;
        for (uint32_t q = 0; q < world; ++q) {
            recv_off[q] = acc;
            acc += m[static_cast<uint64_t>(q) * world + rank];
            uint32_t before = 0; // rows source q sends to ranks below this one
            for (uint32_t r = 0; r < rank; ++r) before += m[static_cast<uint64_t>(q) * world + r];
            src_pos[q] = before;
        }
        recv_off[world] = acc;
        // rows past the capacity were dropped by their senders: count only the kept ones
        if (acc > cap) raise_device_status(status, FM_STATUS_INVALID_ARGUMENT);
        *at<uint32_t>(mine, L.n_recv) = acc < cap ? acc : cap;
    }
    if (first)
        for (uint32_t r = tid; r < world; r += blockDim.x) at<uint32_t>(mine, L.my_pos)[r] = s_mypos[r];
    __syncthreads();
    const uint32_t j = blockIdx.x;
    if (j < s_offs[world]) {
        const uint32_t item = s_items[j], t = item / world, dest = item % world;
        const uint32_t pos = s_mypos[dest] + (j - s_offs[dest]);
        if (pos >= cap) { // a destination receiving more than its capacity: refuse, never write past it
            if (tid == 0) raise_device_status(status, FM_STATUS_INVALID_ARGUMENT);
        } else {
            uint8_t *peer = peers[dest];
            const XT *src = x + static_cast<uint64_t>(t) * d;
            uint4 *dst = reinterpret_cast<uint4 *>(at<__half>(peer, L.recv_x) + static_cast<uint64_t>(pos) * d);
            const bool vec = sizeof(XT) == 2 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
            const uint32_t per = (d / 8 + gridDim.y - 1) / gridDim.y, c0 = blockIdx.y * per;
            const uint32_t c1 = min(d / 8, c0 + per);
            for (uint32_t c = c0 + tid; c < c1; c += blockDim.x) {
                __align__(16) __half h[8];
                if (vec) { // eight bf16 in one 16-byte load
                    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src) + c);
                    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        h[2 * i] = __float2half_rn(__uint_as_float(u[i] << 16));
                        h[2 * i + 1] = __float2half_rn(__uint_as_float(u[i] & 0xFFFF0000u));
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(load_x(src + 8 * c + i));
                }
                dst[c] = *reinterpret_cast<const uint4 *>(h);
            }
            int32_t *me = at<int32_t>(peer, L.recv_e) + static_cast<uint64_t>(pos) * top_k;
            float *mw = at<float>(peer, L.recv_w) + static_cast<uint64_t>(pos) * top_k;
            for (uint32_t r = tid; blockIdx.y == 0 && r < top_k; r += blockDim.x) {
                const uint32_t e = ids[static_cast<uint64_t>(t) * top_k + r];
                const bool local = e / per_rank == dest;
                me[r] = local ? static_cast<int32_t>(e % per_rank) : -1;
                mw[r] = local ? w[static_cast<uint64_t>(t) * top_k + r] : 0.0f;
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        uint32_t *ctr = at<uint32_t>(mine, L.ctr);
        if (atomicAdd(ctr, 1u) == gridDim.x * gridDim.y - 1) {
            *ctr = 0;
            __threadfence_system();
            for (uint32_t r = 0; r < world; ++r) flag_release(at<uint32_t>(peers[r], L.dflag) + rank, epoch);
        }
    }
}

// One warp waits until every source's rows (flag `off_flag`) are in.
__global__ void p2p_wait_kernel(uint8_t *mine, uint64_t off_flag, uint32_t world, uint32_t epoch, uint64_t off_ctr,
                                uint64_t timeout_ns, int *status) {
    epoch = call_epoch(epoch, at<uint32_t>(mine, off_ctr) + 2);
    for (uint32_t s = threadIdx.x; s < world; s += 32)
        wait_flag(at<uint32_t>(mine, off_flag) + s, epoch, timeout_ns, status);
}

// Block (j, c) (j < rows received): columns piece c of partial[j] = sum over
// the row's top-k slots of w_r * out[j*k + r] (top-k order, multiply then add),
// written straight into the source rank's return rows.  The last block to
// finish raises bflag[rank] there.
__global__ void p2p_partial_return_kernel(const float *__restrict__ out, uint32_t top_k, uint32_t d, uint32_t world,
                                          uint32_t rank, uint8_t *const *peers, uint8_t *mine, Mailbox L, uint32_t cap,
                                          uint32_t epoch, int *status) {
    const uint32_t j = blockIdx.x;
    epoch = call_epoch(epoch, at<uint32_t>(mine, L.ctr) + 2);
    const uint32_t n = *at<uint32_t>(mine, L.n_recv);
    if (j < n) {
        const uint32_t *recv_off = at<uint32_t>(mine, L.recv_off);
        uint32_t s = 0;
        while (s + 1 < world && recv_off[s + 1] <= j) ++s;
        const uint32_t pos = at<uint32_t>(mine, L.src_pos)[s] + (j - recv_off[s]);
        if (pos >= cap) {
            if (threadIdx.x == 0) raise_device_status(status, FM_STATUS_INVALID_ARGUMENT);
            goto done;
        }
        {
        const int32_t *me = at<int32_t>(mine, L.recv_e) + static_cast<uint64_t>(j) * top_k;
        const float *mw = at<float>(mine, L.recv_w) + static_cast<uint64_t>(j) * top_k;
        float4 *dst = reinterpret_cast<float4 *>(at<float>(peers[s], L.back) + static_cast<uint64_t>(pos) * d);
        const uint32_t per = (d / 4 + gridDim.y - 1) / gridDim.y, c0 = blockIdx.y * per;
        const uint32_t c1 = min(d / 4, c0 + per);
        for (uint32_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (uint32_t r = 0; r < top_k; ++r) {
                if (me[r] < 0) continue;
                const float wr = mw[r];
                const float4 v = reinterpret_cast<const float4 *>(out + (static_cast<uint64_t>(j) * top_k + r) * d)[c];
                acc.x = __fadd_rn(acc.x, __fmul_rn(wr, v.x));
                acc.y = __fadd_rn(acc.y, __fmul_rn(wr, v.y));
                acc.z = __fadd_rn(acc.z, __fmul_rn(wr, v.z));
                acc.w = __fadd_rn(acc.w, __fmul_rn(wr, v.w));
            }
            dst[c] = acc;
        }
        }
    }
done:
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t *ctr = at<uint32_t>(mine, L.ctr) + 1;
        if (atomicAdd(ctr, 1u) == gridDim.x * gridDim.y - 1) {
            *ctr = 0;
            __threadfence_system();
            for (uint32_t r = 0; r < world; ++r) flag_release(at<uint32_t>(peers[r], L.bflag) + rank, epoch);
        }
    }
}

// y[t] = sum over destination ranks (ascending) of the returned rows, once
// every destination's rows are back (each CTA waits for the flags itself).
// With device epochs the last CTA to finish advances the epoch counter: the
// call is over.
__global__ void p2p_combine_kernel(uint8_t *mine, Mailbox L, const uint32_t *__restrict__ row_of, uint32_t tokens,
                                   uint32_t world, uint32_t d, float *__restrict__ y, uint32_t epoch,
                                   uint64_t timeout_ns, int *status) {
    uint32_t *ctr = at<uint32_t>(mine, L.ctr);
    const uint32_t ep = call_epoch(epoch, ctr + 2);
    wait_flags_cta(at<uint32_t>(mine, L.bflag), world, ep, timeout_ns, status);
    const uint64_t id = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (id < static_cast<uint64_t>(tokens) * d) {
        const float *back = at<float>(mine, L.back);
        const uint32_t t = static_cast<uint32_t>(id / d), c = static_cast<uint32_t>(id % d);
        float acc = 0.0f;
        for (uint32_t r = 0; r < world; ++r) {
            const uint32_t row = row_of[static_cast<uint64_t>(t) * world + r];
            if (row != 0xFFFFFFFFu) acc = __fadd_rn(acc, back[static_cast<uint64_t>(row) * d + c]);
        }
        y[id] = acc;
    }
    if (epoch) return;
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(ctr + 3, 1u) == gridDim.x - 1) {
        ctr[3] = 0;
        ctr[2] += 1; // every CTA has read the counter
    }
}

__global__ void ep_row_keys_p2p_kernel(const uint32_t *__restrict__ ids, uint32_t tokens, uint32_t top_k,
                                       uint32_t per_rank, uint32_t world, uint32_t *__restrict__ keys) {
    const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
    if (i >= static_cast<uint64_t>(tokens) * world) return;
    const uint32_t t = static_cast<uint32_t>(i / world), dest = static_cast<uint32_t>(i % world);
    bool any = false;
    for (uint32_t r = 0; r < top_k; ++r) any |= ids[static_cast<uint64_t>(t) * top_k + r] / per_rank == dest;
    keys[i] = any ? dest : 0xFFFFFFFFu;
}

uint64_t timeout_ns_of(uint32_t timeout_ms) { return (timeout_ms ? timeout_ms : 2000u) * 1000000ull; }

int check_p2p(uint32_t world, uint32_t rank, uint32_t capacity, uint32_t d_model, uint32_t top_k) {
    if (world == 0 || world > 64 || rank >= world)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "peer exchange needs 1..64 ranks and rank < world");
    if (capacity == 0 || d_model == 0 || d_model % 8 || top_k == 0 || top_k > 32)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "peer exchange: capacity >= 1, d_model a multiple of 8, "
                                                     "1 <= top_k <= 32");
    return FM_STATUS_OK;
}

} // namespace
} // namespace fmb

using namespace fmb;

extern "C" uint64_t fmcuda_ep_mailbox_bytes(uint32_t world, uint32_t capacity, uint32_t top_k, uint32_t d_model) {
    return mailbox_layout(world, capacity, top_k, d_model).total;
}

extern "C" int fmcuda_ep_mailbox_alloc(uint64_t bytes, void **mailbox, void *ipc_handle) {
    if (!mailbox || !ipc_handle || bytes == 0) return set_error(FM_STATUS_INVALID_ARGUMENT, "mailbox arguments");
    void *p = nullptr;
    cudaError_t err = cudaMalloc(&p, bytes);
    if (err != cudaSuccess) return cuda_status(err, "mailbox allocation");
    if ((err = cudaMemset(p, 0, bytes)) == cudaSuccess)
        err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), p);
    if (err != cudaSuccess) {
        cudaFree(p);
        return cuda_status(err, "mailbox IPC handle");
    }
    *mailbox = p;
    return FM_STATUS_OK;
}

extern "C" int fmcuda_ep_mailbox_open(const void *ipc_handle, void **mailbox) {
    if (!ipc_handle || !mailbox) return set_error(FM_STATUS_INVALID_ARGUMENT, "mailbox arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t err = cudaIpcOpenMemHandle(mailbox, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return cuda_status(err, "mailbox IPC open");
    return FM_STATUS_OK;
}

extern "C" int fmcuda_ep_mailbox_close(void *mailbox) {
    const cudaError_t err = cudaIpcCloseMemHandle(mailbox);
    return err == cudaSuccess ? FM_STATUS_OK : cuda_status(err, "mailbox IPC close");
}

extern "C" int fmcuda_ep_mailbox_free(void *mailbox) {
    const cudaError_t err = cudaFree(mailbox);
    return err == cudaSuccess ? FM_STATUS_OK : cuda_status(err, "mailbox free");
}

extern "C" uint64_t fmcuda_ep_p2p_dispatch_scratch_bytes(uint32_t tokens, uint32_t world) {
    const uint64_t n = static_cast<uint64_t>(tokens) * world;
    return a256(n * 4) + a256(world * 4ull) + a256((world + 1ull) * 4) + a256(n * 4) + a256(n * 4) +
           group_scratch_bytes(static_cast<uint32_t>(n), world);
}

extern "C" int fmcuda_ep_p2p_dispatch(const uint32_t *ids, const float *weights, uint32_t tokens, uint32_t top_k,
                                      uint32_t experts_per_rank, uint32_t world, uint32_t rank, const void *x,
                                      int32_t x_dtype, uint32_t d_model, void *mailbox, void *const *peers,
                                      uint32_t capacity,
                                      uint32_t epoch, uint32_t *row_of, void *scratch, uint32_t timeout_ms,
                                      void *stream) {
    int rc = check_p2p(world, rank, capacity, d_model, top_k);
    if (rc) return rc;
    if (!ids || !weights || !x || !mailbox || !peers || !row_of || !scratch)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "null peer-dispatch pointer");
    if (x_dtype != FM_X_F32 && x_dtype != FM_X_BF16)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "unknown activation dtype");
    if (experts_per_rank == 0) return set_error(FM_STATUS_INVALID_ARGUMENT, "no experts per rank");
    const uint64_t n64 = static_cast<uint64_t>(tokens) * world;
    if (n64 > capacity) return set_error(FM_STATUS_INVALID_ARGUMENT, "tokens x world exceeds the mailbox capacity");
    const uint32_t n = static_cast<uint32_t>(n64);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Mailbox L = mailbox_layout(world, capacity, top_k, d_model);
    uint8_t *sc = static_cast<uint8_t *>(scratch);
    uint32_t *keys = reinterpret_cast<uint32_t *>(sc);
    uint32_t *counts = reinterpret_cast<uint32_t *>(sc + a256(n64 * 4));
    uint32_t *offsets = reinterpret_cast<uint32_t *>(sc + a256(n64 * 4) + a256(world * 4ull));
    uint32_t *items = reinterpret_cast<uint32_t *>(sc + a256(n64 * 4) + a256(world * 4ull) + a256((world + 1ull) * 4));
    uint32_t *gscratch = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(items) + a256(n64 * 4) + a256(n64 * 4));
    uint8_t *const *pp = reinterpret_cast<uint8_t *const *>(peers);
    uint8_t *mine = static_cast<uint8_t *>(mailbox);
    const dim3 grid(n ? n : 1, (d_model / 8 + 127) / 128); // rows x column pieces of 128 x 16 bytes
    if (n <= kFusedMaxItems && world <= kFusedMaxWorld) {
        if (x_dtype == FM_X_F32)
            p2p_send_kernel<float><<<grid, 128, 0, s>>>(static_cast<const float *>(x), ids, weights, tokens, top_k,
                                                        experts_per_rank, world, rank, d_model, pp, mine, L, capacity,
                                                        epoch, row_of, timeout_ns_of(timeout_ms),
                                                        device_status_word());
        else
            p2p_send_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
                static_cast<const __nv_bfloat16 *>(x), ids, weights, tokens, top_k, experts_per_rank, world, rank,
                d_model, pp, mine, L, capacity, epoch, row_of, timeout_ns_of(timeout_ms), device_status_word());
        return check_launch("peer send launch");
    }
    if (n) {
        ep_row_keys_p2p_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, tokens, top_k, experts_per_rank, world, keys);
        if ((rc = check_launch("peer dispatch keys launch"))) return rc;
    }
    if ((rc = launch_group_large(keys, n, world, counts, offsets, items, row_of, gscratch, s))) return rc;
    p2p_counts_kernel<<<1, 64, 0, s>>>(pp, world, rank, counts, L.matrix, L.mflag, epoch,
                                       reinterpret_cast<const uint32_t *>(mine + L.ctr) + 2);
    if ((rc = check_launch("peer counts launch"))) return rc;
    p2p_plan_kernel<<<1, 32, 0, s>>>(mine, L, world, rank, capacity, epoch, timeout_ns_of(timeout_ms),
                                     device_status_word());
    if ((rc = check_launch("peer plan launch"))) return rc;
    if (x_dtype == FM_X_F32)
        p2p_pack_send_kernel<float><<<grid, 128, 0, s>>>(static_cast<const float *>(x), ids, weights, items, offsets,
                                                         top_k, experts_per_rank, world, rank, d_model, pp, mine, L,
                                                         capacity, epoch, device_status_word());
    else
        p2p_pack_send_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16 *>(x), ids, weights,
                                                                 items, offsets, top_k, experts_per_rank, world, rank,
                                                                 d_model, pp, mine, L, capacity, epoch,
                                                                 device_status_word());
    return check_launch("peer pack-send launch");
}

extern "C" uint64_t fmcuda_ep_p2p_experts_workspace_bytes(uint32_t capacity, uint32_t top_k, uint32_t experts,
                                                          uint32_t d_model, uint32_t ffn) {
    return a256(static_cast<uint64_t>(capacity) * top_k * d_model * 4) +
           experts_pairs_workspace_bytes(capacity, top_k, experts, d_model, ffn);
}

extern "C" int fmcuda_ep_p2p_experts(void *mailbox, void *const *peers, uint32_t world, uint32_t rank, uint32_t capacity,
                                     uint32_t epoch, uint32_t top_k, uint32_t experts, const void *const *expert_slots,
                                     uint64_t up_offset, uint64_t down_offset, uint32_t gate_type, uint32_t up_type,
                                     uint32_t down_type, uint32_t d_model, uint32_t ffn, void *workspace,
                                     uint64_t workspace_bytes, uint32_t timeout_ms, void *stream) {
    int rc = check_p2p(world, rank, capacity, d_model, top_k);
    if (rc) return rc;
    if (!mailbox || !peers || !expert_slots || !workspace) return set_error(FM_STATUS_INVALID_ARGUMENT, "null peer-experts pointer");
    const uint64_t need = fmcuda_ep_p2p_experts_workspace_bytes(capacity, top_k, experts, d_model, ffn);
    if (workspace_bytes < need)
        return set_error(FM_STATUS_INVALID_ARGUMENT, "peer-experts workspace too small: need " + std::to_string(need));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Mailbox L = mailbox_layout(world, capacity, top_k, d_model);
    uint8_t *const *pp = reinterpret_cast<uint8_t *const *>(peers);
    uint8_t *mine = static_cast<uint8_t *>(mailbox);
    // decode-sized Q4_K batches: the receive front of the tcgen05 stage waits for
    // the rows itself; otherwise one warp waits before the expert compute
    const bool fused = partial_fused_recv(capacity, top_k, experts, d_model, ffn, gate_type, up_type, down_type,
                                          up_offset, down_offset);
    TgRecvWait wt{};
    if (fused) {
        wt.flags = reinterpret_cast<const uint32_t *>(mine + L.dflag);
        wt.world = world;
        wt.epoch = epoch;
        wt.ectr = reinterpret_cast<const uint32_t *>(mine + L.ctr) + 2;
        wt.timeout_ns = timeout_ns_of(timeout_ms);
        wt.n_rows = reinterpret_cast<const uint32_t *>(mine + L.n_recv);
        wt.meta_e = reinterpret_cast<const int32_t *>(mine + L.recv_e);
        wt.rows = capacity;
    } else {
        p2p_wait_kernel<<<1, 32, 0, s>>>(mine, L.dflag, world, epoch, L.ctr, timeout_ns_of(timeout_ms),
                                         device_status_word());
        if ((rc = check_launch("peer wait launch"))) return rc;
    }
    float *out_pairs = static_cast<float *>(workspace);
    uint8_t *ws = static_cast<uint8_t *>(workspace) + a256(static_cast<uint64_t>(capacity) * top_k * d_model * 4);
    if ((rc = experts_partial_run(mine + L.recv_x, reinterpret_cast<const int32_t *>(mine + L.recv_e),
                                  reinterpret_cast<const float *>(mine + L.recv_w), capacity,
                                  reinterpret_cast<const uint32_t *>(mine + L.n_recv), top_k, experts, expert_slots,
                                  up_offset, down_offset, gate_type, up_type, down_type, d_model, ffn, out_pairs, ws,
                                  workspace_bytes - (ws - static_cast<uint8_t *>(workspace)), s,
                                  fused ? &wt : nullptr)))
        return rc;
    p2p_partial_return_kernel<<<dim3(capacity, (d_model / 4 + 127) / 128), 128, 0, s>>>(out_pairs, top_k, d_model, world, rank, pp, mine, L, capacity,
                                                       epoch, device_status_word());
    return check_launch("peer partial-return launch");
}

extern "C" int fmcuda_ep_p2p_combine(void *mailbox, uint32_t world, uint32_t rank, uint32_t capacity,
                                     uint32_t epoch, uint32_t top_k, const uint32_t *row_of, uint32_t tokens,
                                     uint32_t d_model, float *y, uint32_t timeout_ms, void *stream) {
    int rc = check_p2p(world, rank, capacity, d_model, top_k);
    if (rc) return rc;
    if (!mailbox || !row_of || !y) return set_error(FM_STATUS_INVALID_ARGUMENT, "null peer-combine pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Mailbox L = mailbox_layout(world, capacity, top_k, d_model);
    uint8_t *mine = static_cast<uint8_t *>(mailbox);
    const uint64_t n = static_cast<uint64_t>(tokens) * d_model;
    const unsigned blocks = n ? static_cast<unsigned>((n + 255) / 256) : 1u;
    p2p_combine_kernel<<<blocks, 256, 0, s>>>(mine, L, row_of, tokens, world, d_model, y, epoch,
                                              timeout_ns_of(timeout_ms), device_status_word());
    return check_launch("peer combine launch");
}

// ref_shim.cpp -- C entry points over the reference's OWN code, for tests.
//
// TEST INFRASTRUCTURE ONLY.  Linked with the reference's sources (compiled
// unmodified from the reference tree by oracle/Makefile) into
// oracle/_ref/libfmref.so.  Used to pin the C restatement in fm_oracle.c and
// as the timed CPU baseline; never part of the product path.
//
// Engine::softmax / Engine::topk are private members of fm::Engine
// (include/fm/engine.hpp:264-265); this translation unit alone re-declares the
// access so the test can call the reference's own router arithmetic.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <thread>
#include <vector>

#include "fm/activation.hpp"
#include "fm/common.hpp"
#include "fm/io.hpp"
#include "fm/kernels.hpp"
#include "fm/quant.hpp"
#define private public
#include "fm/engine.hpp"
#undef private

namespace {

thread_local std::string g_last_error;

int code_of(const fm::Error &e) {
    g_last_error = e.what();
    return static_cast<int>(e.code);
}

uint64_t row_bytes_of(uint32_t type_id, uint32_t in_dim) {
    const fm::QuantGeometry &geo = fm::quant_geometry(type_id);
    return static_cast<uint64_t>(in_dim / geo.block_size) * geo.block_bytes;
}

} // namespace

extern "C" {

const char *fmr_last_error(void) { return g_last_error.c_str(); }

// fm::dequantize_block (src/quant.cpp:163)
int fmr_dequant_block(uint32_t type_id, const uint8_t *src, float *dst) {
    try {
        fm::dequantize_block(type_id, src, dst);
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// fm::dequantize_tensor_region (src/quant.cpp:723)
int fmr_dequant_region(uint32_t type_id, const uint8_t *src, float *dst, uint64_t n) {
    try {
        fm::dequantize_tensor_region(type_id, src, dst, n);
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// Name of the ISA the reference's `auto` dispatch resolves to on this host.
const char *fmr_resolved_isa(void) {
    fm::KernelConfig cfg;
    return fm::kernel_isa_name(fm::resolved_isa(cfg));
}

// fm::gemv_quant (src/kernels.cpp:846) at threads=1 per call, over `threads`
// contiguous row slices run on one std::thread each.  Rows are independent, so
// the result is bit-identical to the serial call.  The reference's WorkerPool
// is not used: parallel_for (src/kernels.cpp:416-464) waits on worker 0's
// counter alone and hangs for more than two ranges.
int fmr_gemv_quant(uint32_t type_id, const uint8_t *w, const float *x, float *y,
                   uint32_t out_dim, uint32_t in_dim, uint32_t threads, int scalar) {
    try {
        fm::KernelConfig cfg;
        cfg.threads = 1;
        cfg.requested = scalar ? fm::KernelIsa::Scalar : fm::KernelIsa::Auto;
        const uint64_t rb = type_id == 0 ? static_cast<uint64_t>(in_dim) * 4
                                         : row_bytes_of(type_id, in_dim);
        if (threads <= 1 || out_dim < 2 * threads) {
            fm::gemv_quant(cfg, type_id, w, x, y, out_dim, in_dim);
            return 0;
        }
        std::vector<std::thread> pool;
        std::vector<int> rcs(threads, 0);
        std::vector<std::string> msgs(threads);
        const uint32_t chunk = (out_dim + threads - 1) / threads;
        for (uint32_t i = 0; i < threads; ++i) {
            const uint32_t begin = i * chunk;
            const uint32_t end = begin + chunk < out_dim ? begin + chunk : out_dim;
            if (begin >= end) break;
            pool.emplace_back([&, i, begin, end]() {
                try {
                    fm::gemv_quant(cfg, type_id, w + begin * rb, x, y + begin, end - begin, in_dim);
                } catch (const fm::Error &e) {
                    rcs[i] = static_cast<int>(e.code);
                    msgs[i] = e.what();
                }
            });
        }
        for (auto &t : pool) t.join();
        for (uint32_t i = 0; i < threads; ++i)
            if (rcs[i]) {
                g_last_error = msgs[i];
                return rcs[i];
            }
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// fm::gemv_scalar (src/kernels.cpp:132) or fm::gemv_isa (:262) with the
// `auto` ISA.
int fmr_gemv_f32(const float *w, const float *x, float *y, uint32_t out_dim, uint32_t in_dim,
                 int scalar) {
    if (scalar) fm::gemv_scalar(w, x, y, out_dim, in_dim);
    else fm::gemv_isa(fm::resolve_kernel_isa(fm::KernelIsa::Auto), w, x, y, out_dim, in_dim);
    return 0;
}

// Router of the native adapter, per token: Engine::softmax and Engine::topk
// (src/engine.cpp:378-411) called on the reference's own Engine, then the
// renormalisation of src/engine.cpp:1680-1702 with the adapter's settings
// (norm on, scale 1.0, clamped epsilon 6.103515625e-5; gguf.cpp:3027-3028).
int fmr_route(const float *logits, uint32_t tokens, uint32_t experts, uint32_t top_k,
              uint32_t *ids, float *weights, float *probs_out) {
    try {
        fm::RunConfig rc;
        fm::Engine engine(rc);
        const double eps = 6.103515625e-5;
        for (uint32_t t = 0; t < tokens; ++t) {
            std::vector<float> v(logits + static_cast<uint64_t>(t) * experts,
                                 logits + static_cast<uint64_t>(t + 1) * experts);
            std::vector<float> probs = engine.softmax(v);
            if (probs_out)
                std::memcpy(probs_out + static_cast<uint64_t>(t) * experts, probs.data(),
                            experts * sizeof(float));
            std::vector<uint32_t> sel = engine.topk(probs, top_k);
            float total = 0.0f;
            std::vector<float> w(top_k);
            for (uint32_t i = 0; i < top_k; ++i) {
                w[i] = probs[sel[i]];
                total += w[i];
            }
            const double denom = std::max(static_cast<double>(total), eps);
            for (float &x : w) x = static_cast<float>(x / denom);
            for (float &x : w) x = static_cast<float>(x * 1.0);
            for (uint32_t i = 0; i < top_k; ++i) {
                ids[static_cast<uint64_t>(t) * top_k + i] = sel[i];
                weights[static_cast<uint64_t>(t) * top_k + i] = w[i];
            }
        }
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// Plain SwiGLU of include/fm/activation.hpp:62-84 (silu at :33).
float fmr_swiglu(float gate, float up) {
    return static_cast<float>(fm::silu(static_cast<double>(gate))) * up;
}

uint64_t fmr_fnv1a64(const uint8_t *data, uint64_t size) { return fm::fnv1a64(data, size); }

// The routed-expert loop of src/engine.cpp:1711-1772 for `tokens` tokens over
// the reference's own kernels: per selected expert, fm::gemv_quant for gate
// and up, the plain gated activation (include/fm/activation.hpp:62-84), the
// down fm::gemv_quant, then ffn[j] += w * down[j] in top-k order.  The
// (token, expert) products are independent, so they are spread over
// `threads` std::threads (each gemv_quant at threads=1); the combine runs per
// token in top-k order afterwards, exactly as the engine accumulates.
int fmr_moe_block(uint32_t type_id, const uint8_t *const *slots, uint64_t up_offset,
                  uint64_t down_offset, const float *x, uint32_t tokens, uint32_t d,
                  uint32_t ffn, uint32_t top_k, const uint32_t *ids, const float *weights,
                  float *y, uint32_t threads) {
    try {
        fm::KernelConfig cfg;
        cfg.threads = 1;
        const uint64_t items = static_cast<uint64_t>(tokens) * top_k;
        std::vector<float> down(items * d);
        std::atomic<uint64_t> next{0};
        std::vector<std::string> errors(threads ? threads : 1);
        std::vector<int> codes(threads ? threads : 1, 0);
        auto worker = [&](uint32_t tid) {
            std::vector<float> gate(ffn), up(ffn), act(ffn);
            for (;;) {
                const uint64_t it = next.fetch_add(1);
                if (it >= items) return;
                const uint32_t t = static_cast<uint32_t>(it / top_k);
                const uint8_t *base = slots[ids[it]];
                const float *xt = x + static_cast<uint64_t>(t) * d;
                try {
                    fm::gemv_quant(cfg, type_id, base, xt, gate.data(), ffn, d);
                    fm::gemv_quant(cfg, type_id, base + up_offset, xt, up.data(), ffn, d);
                    for (uint32_t j = 0; j < ffn; ++j)
                        act[j] = static_cast<float>(fm::silu(static_cast<double>(gate[j]))) * up[j];
                    fm::gemv_quant(cfg, type_id, base + down_offset, act.data(),
                                   down.data() + it * d, d, ffn);
                } catch (const fm::Error &e) {
                    codes[tid] = static_cast<int>(e.code);
                    errors[tid] = e.what();
                    return;
                }
            }
        };
        const uint32_t n = threads ? threads : 1;
        std::vector<std::thread> pool;
        for (uint32_t i = 1; i < n; ++i) pool.emplace_back(worker, i);
        worker(0);
        for (auto &th : pool) th.join();
        for (uint32_t i = 0; i < n; ++i)
            if (codes[i]) {
                g_last_error = errors[i];
                return codes[i];
            }
        for (uint32_t t = 0; t < tokens; ++t) {
            float *ffn_out = y + static_cast<uint64_t>(t) * d;
            for (uint32_t j = 0; j < d; ++j) ffn_out[j] = 0.0f;
            for (uint32_t r = 0; r < top_k; ++r) {
                const float w = weights[static_cast<uint64_t>(t) * top_k + r];
                const float *dn = down.data() + (static_cast<uint64_t>(t) * top_k + r) * d;
                for (uint32_t j = 0; j < d; ++j) ffn_out[j] += w * dn[j];
            }
        }
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// coalesce_extents (src/io.cpp:46-78): group [offset, end) and the group of
// every extent (extents are pairs offset, size).
int fmr_coalesce_extents(const uint64_t *ext, uint32_t n, uint64_t max_gap, uint64_t *group_offset,
                         uint64_t *group_end, uint32_t *group_of, uint32_t *n_groups) {
    try {
        std::vector<fm::Extent> v(n);
        for (uint32_t i = 0; i < n; ++i) v[i] = {ext[2 * i], ext[2 * i + 1]};
        std::vector<fm::CoalescedGroup> g = fm::coalesce_extents(v, max_gap);
        *n_groups = static_cast<uint32_t>(g.size());
        for (size_t j = 0; j < g.size(); ++j) {
            group_offset[j] = g[j].offset;
            group_end[j] = g[j].end;
            for (size_t idx : g[j].request_indices) group_of[idx] = static_cast<uint32_t>(j);
        }
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// current_identity (src/common.cpp:79-119) as six words: size, dev, ino,
// mtime_ns, ctime_ns, content_probe.
int fmr_file_identity(const char *path, uint64_t *out) {
    try {
        fm::FileIdentity id = fm::current_identity(path);
        out[0] = id.size;
        out[1] = id.dev;
        out[2] = id.ino;
        out[3] = static_cast<uint64_t>(id.mtime_ns);
        out[4] = static_cast<uint64_t>(id.ctime_ns);
        out[5] = id.content_probe;
        return 0;
    } catch (const fm::Error &e) {
        return code_of(e);
    }
}

// The data path of ResidencyManager::load_slot (src/residency.cpp:637-720) on
// the reference's CPU backend: ReadScheduler::read_record through the
// reference's own reader, fnv1a64 of the payload against the record
// checksum, the upload (CpuBackend::upload is a memcpy into the slot,
// src/backend.cpp:262-283), then the slot read-back and its fnv1a64.  Records
// are `n_records` x `n_ext` extents (offset, size pairs); slot receives each
// record in turn.  Returns the number of records loaded, or -code.
int64_t fmr_load_records_cpu(const char *path, int reader_mode, uint64_t coalesce_gap, const uint64_t *ext,
                             uint32_t n_ext, uint32_t n_records, const uint64_t *checksums, uint8_t *slot) {
    try {
        fm::SchedulerConfig cfg;
        cfg.mode = static_cast<fm::ReaderMode>(reader_mode);
        cfg.path = path;
        cfg.expected_identity = fm::current_identity(path);
        cfg.coalesce_gap = coalesce_gap;
        fm::ReadScheduler sched(cfg, fm::make_reader(cfg.mode, path, nullptr, false));
        for (uint32_t r = 0; r < n_records; ++r) {
            std::vector<fm::Extent> v(n_ext);
            for (uint32_t i = 0; i < n_ext; ++i)
                v[i] = {ext[2 * (r * n_ext + i)], ext[2 * (r * n_ext + i) + 1]};
            std::vector<uint8_t> payload = sched.read_record(v, fm::ReadPriority::Demand);
            if (fm::fnv1a64(payload) != checksums[r])
                fm::fail(fm::ErrorCode::EXPERT_CHECKSUM_MISMATCH, "source expert checksum mismatch");
            std::memcpy(slot, payload.data(), payload.size());
            std::vector<uint8_t> slot_copy(payload.size());
            std::memcpy(slot_copy.data(), slot, payload.size());
            if (fm::fnv1a64(slot_copy) != checksums[r])
                fm::fail(fm::ErrorCode::EXPERT_CHECKSUM_MISMATCH, "slot payload checksum mismatch");
        }
        return n_records;
    } catch (const fm::Error &e) {
        return -code_of(e);
    }
}

} // extern "C"

// engine_main.cpp -- command-line driver over engine_harness.cpp.
//
// TEST INFRASTRUCTURE ONLY.  Runs the reference's unmodified fm::Engine in a
// process of its own (tests call it through subprocess), so the engine's
// iostream and locale state never share a process with the test runner.
//
//   fm_engine write-tiny PATH [SEED]
//   fm_engine run PATH cpu|gpu PROMPT_HEX N_GEN SLOTS SCALAR(0|1) OUT.bin
//   fm_engine compare PATH cpu|gpu REFERENCE_ROOT PROMPTS TOKENS SLOTS   (JSON on stdout)
//   fm_engine residency PATH cpu|gpu                                   (JSON on stdout)
//
// OUT.bin: u32 n_ids, i32 ids[n]; u32 n_logits, f32 logits[n];
//          u32 n_routing, u32 routing[n]; u32 n_json, char json[n].
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

extern "C" {
const char *fme_last_error(void);
int fme_write_tiny(const char *path, uint64_t seed, uint32_t layers, uint32_t hidden, uint32_t heads,
                   uint32_t experts, uint32_t ffn, uint32_t top_k, uint32_t vocab, uint32_t context,
                   float std_dev);
int fme_run(const char *path, int backend, int scalar_kernels, const uint8_t *prompt, uint32_t prompt_len,
            uint32_t n_gen, uint32_t cache_slots, int32_t *ids_out, uint32_t ids_cap, uint32_t *n_ids,
            float *logits_out, uint32_t logits_cap, uint32_t *n_logits, uint32_t *routing_out,
            uint32_t routing_cap, uint32_t *n_routing, char *metrics_out, uint32_t metrics_cap);
int fme_compare(const char *path, int backend, const char *reference_root, uint32_t prompts, uint32_t tokens,
                uint32_t cache_slots, char *json_out, uint32_t json_cap);
int fme_residency_faults(const char *path, int backend, char *json_out, uint32_t json_cap);
}

int main(int argc, char **argv) {
    if (argc >= 3 && std::strcmp(argv[1], "write-tiny") == 0) {
        const uint64_t seed = argc > 3 ? std::strtoull(argv[3], nullptr, 10) : 0;
        // freemoe-tiny-v1: d 64, 2 layers, 4 heads x 16, 4 experts ffn 128, top-2,
        // vocab 258 (256 bytes + BOS + EOS), context 256, N(0, 0.02)
        const int rc = fme_write_tiny(argv[2], seed, 2, 64, 4, 4, 128, 2, 258, 256, 0.02f);
        if (rc) std::fprintf(stderr, "write-tiny failed (%d): %s\n", rc, fme_last_error());
        return rc;
    }
    if (argc == 9 && std::strcmp(argv[1], "run") == 0) {
        const std::string hex = argv[4];
        std::vector<uint8_t> prompt(hex.size() / 2);
        for (size_t i = 0; i < prompt.size(); ++i)
            prompt[i] = static_cast<uint8_t>(std::strtoul(hex.substr(2 * i, 2).c_str(), nullptr, 16));
        const int backend = std::strcmp(argv[3], "gpu") == 0 ? 2 : 0;
        const uint32_t n_gen = static_cast<uint32_t>(std::atoi(argv[5]));
        const uint32_t slots = static_cast<uint32_t>(std::atoi(argv[6]));
        const int scalar = std::atoi(argv[7]);
        std::vector<int32_t> ids(4096);
        std::vector<float> logits(1 << 20);
        std::vector<uint32_t> routing(1 << 20);
        std::vector<char> json(1 << 22);
        uint32_t n_ids = 0, n_logits = 0, n_routing = 0;
        const int rc = fme_run(argv[2], backend, scalar, prompt.data(), static_cast<uint32_t>(prompt.size()),
                               n_gen, slots, ids.data(), static_cast<uint32_t>(ids.size()), &n_ids,
                               logits.data(), static_cast<uint32_t>(logits.size()), &n_logits,
                               routing.data(), static_cast<uint32_t>(routing.size()), &n_routing,
                               json.data(), static_cast<uint32_t>(json.size()));
        if (rc) {
            std::fprintf(stderr, "run failed (%d): %s\n", rc, fme_last_error());
            return rc;
        }
        FILE *f = std::fopen(argv[8], "wb");
        if (!f) return 11;
        const uint32_t n_json = static_cast<uint32_t>(std::strlen(json.data()));
        std::fwrite(&n_ids, 4, 1, f);
        std::fwrite(ids.data(), 4, n_ids, f);
        std::fwrite(&n_logits, 4, 1, f);
        std::fwrite(logits.data(), 4, n_logits, f);
        std::fwrite(&n_routing, 4, 1, f);
        std::fwrite(routing.data(), 4, n_routing, f);
        std::fwrite(&n_json, 4, 1, f);
        std::fwrite(json.data(), 1, n_json, f);
        std::fclose(f);
        return 0;
    }
    if (argc == 8 && std::strcmp(argv[1], "compare") == 0) {
        std::vector<char> json(1 << 22);
        const int rc = fme_compare(argv[2], std::strcmp(argv[3], "gpu") == 0 ? 2 : 0, argv[4],
                                   static_cast<uint32_t>(std::atoi(argv[5])), static_cast<uint32_t>(std::atoi(argv[6])),
                                   static_cast<uint32_t>(std::atoi(argv[7])), json.data(),
                                   static_cast<uint32_t>(json.size()));
        if (rc) {
            std::fprintf(stderr, "compare failed (%d): %s\n", rc, fme_last_error());
            return rc;
        }
        std::printf("%s\n", json.data());
        return 0;
    }
    if (argc == 4 && std::strcmp(argv[1], "residency") == 0) {
        std::vector<char> json(1 << 20);
        const int rc = fme_residency_faults(argv[2], std::strcmp(argv[3], "gpu") == 0 ? 2 : 0, json.data(),
                                            static_cast<uint32_t>(json.size()));
        if (rc) {
            std::fprintf(stderr, "residency failed (%d): %s\n", rc, fme_last_error());
            return rc;
        }
        std::printf("%s\n", json.data());
        return 0;
    }
    std::fprintf(stderr, "usage: fm_engine write-tiny PATH [SEED] | run PATH cpu|gpu HEX N SLOTS SCALAR OUT | "
                         "compare PATH cpu|gpu REFROOT PROMPTS TOKENS SLOTS | residency PATH cpu|gpu\n");
    return 2;
}

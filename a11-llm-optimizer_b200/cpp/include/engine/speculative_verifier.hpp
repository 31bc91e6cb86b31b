// speculative_verifier.hpp - the reference's C++ verifier interface
// (include/engine/speculative_verifier.hpp:15-125 of the reference: namespace
// A11::Engine, SPEC_K, TreeNode, SpecDiagnosticCounters, SpeculativeTreeVerifier
// with its Config) implemented over liba11spec's C ABI. Code written against
// the reference header compiles unchanged against this one; acceptance
// decisions run on the GPU (a11s_verify_chain).
#pragma once

#include <cstddef>
#include <cstdint>
#include <iostream>
#include <random>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

constexpr uint32_t SPEC_K = 8;  // drafts per speculation step

namespace A11 {
namespace Engine {

struct TreeNode {
    int32_t token_id = -1;
    float log_prob = 0.0f;
    uint32_t parent_idx = UINT32_MAX;
    uint32_t depth = 0;
    std::vector<uint32_t> children;
};

struct SpecDiagnosticCounters {
    uint64_t steps_accepted = 0;
    uint64_t steps_rejected = 0;
    uint64_t fallback_count = 0;
    uint64_t total_draft_tokens = 0;
    uint64_t total_steps = 0;

    void log_fallback(uint32_t draft_len, uint32_t accepted) {
        ++fallback_count;
        std::cerr << "[SpeculativeVerifier DIAGNOSTIC] Fallback to autoregressive: draft=" << draft_len
                  << ", accepted=" << accepted << ", step #" << total_steps << std::endl;
    }
    void reset() { *this = SpecDiagnosticCounters{}; }
};

class SpeculativeTreeVerifier {
public:
    struct Config {
        uint32_t max_draft_depth = SPEC_K;
        uint32_t vocab_size = 32000;
        float acceptance_threshold = 1.0f;  // interface field; the rule is min(1, ratio)
        bool log_diagnostics = true;
    };

    explicit SpeculativeTreeVerifier(const Config &cfg);
    ~SpeculativeTreeVerifier();
    SpeculativeTreeVerifier(const SpeculativeTreeVerifier &) = delete;
    SpeculativeTreeVerifier &operator=(const SpeculativeTreeVerifier &) = delete;

    TreeNode build_draft_tree(int32_t root_token);
    // One-hot [n x vocab] token mask of the reference API; the device path
    // derives ancestor bits from parents and never materialises this.
    std::vector<float> construct_tree_mask(const std::vector<TreeNode> &tree);
    // Rejection rule of the reference, decided on the GPU with uniforms from
    // this thread's std::mt19937(42) stream (one draw per judged token).
    std::pair<uint32_t, uint32_t> verify_draft_tokens(const std::vector<int32_t> &draft_tokens,
                                                      const std::vector<float> &draft_log_probs,
                                                      const std::vector<float> &target_log_probs);
    std::pair<std::vector<int32_t>, bool> speculate_step(const std::vector<int32_t> &context_tokens,
                                                         int32_t root_draft_token);
    const SpecDiagnosticCounters &diagnostics() const { return diags_; }
    void reset_diagnostics() { diags_.reset(); }

private:
    Config config_;
    SpecDiagnosticCounters diags_;
    struct Device;  // device buffers and stream, created on first use
    Device *dev_ = nullptr;
    static std::mt19937 &rng();
    static float rand_uniform();
};

}  // namespace Engine
}  // namespace A11

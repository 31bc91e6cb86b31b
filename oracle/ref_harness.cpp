// ref_harness.cpp - extern "C" shim over the reference's own C++ verifier.
//
// TEST INFRASTRUCTURE ONLY. Compiled (by oracle/Makefile, target `ref`) together
// with the reference source src/engine/speculative_verifier.cpp, read in place
// from the reference tree, into oracle/_ref/libref_verifier.so. Nothing of the
// reference is copied into this repository.
//
// The reference draws its rejection uniforms from a thread_local
// std::mt19937(42) (src/engine/speculative_verifier.cpp:65-69). ref_verify runs
// every call on a fresh std::thread, so draw i of the stream judges token i,
// and ref_uniform_stream reproduces that stream for callers that must hand the
// same uniforms to the GPU.
#include "engine/speculative_verifier.hpp"

#include <cstdint>
#include <random>
#include <stdexcept>
#include <thread>
#include <vector>

using A11::Engine::SpeculativeTreeVerifier;

extern "C" {

int ref_spec_k(void) { return static_cast<int>(SPEC_K); }

// Returns 0 and (accepted_len, last_idx), or 1 when the reference throws.
int ref_verify(int n, const int32_t* tokens, const float* draft, const float* target,
               uint32_t* accepted_len, uint32_t* last_idx) {
    int rc = 0;
    std::thread t([&] {
        SpeculativeTreeVerifier::Config cfg;
        cfg.log_diagnostics = false;
        SpeculativeTreeVerifier v(cfg);
        try {
            auto r = v.verify_draft_tokens(std::vector<int32_t>(tokens, tokens + n),
                                           std::vector<float>(draft, draft + n),
                                           std::vector<float>(target, target + n));
            *accepted_len = r.first;
            *last_idx = r.second;
        } catch (const std::runtime_error&) {
            rc = 1;
        }
    });
    t.join();
    return rc;
}

// Length-mismatch form: the reference must throw (tests/test_speculative_verifier.cpp:151-163).
int ref_verify_mismatch(int n_tok, int n_draft, int n_target) {
    SpeculativeTreeVerifier::Config cfg;
    cfg.log_diagnostics = false;
    SpeculativeTreeVerifier v(cfg);
    try {
        v.verify_draft_tokens(std::vector<int32_t>(n_tok, 1), std::vector<float>(n_draft, -0.5f),
                              std::vector<float>(n_target, 0.9f));
    } catch (const std::runtime_error&) {
        return 1;
    }
    return 0;
}

void ref_uniform_stream(int n, float* out) {
    std::mt19937 rng(42);
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    for (int i = 0; i < n; ++i) out[i] = dist(rng);
}

// Batch of independent chains on `threads` host threads, for the CPU baseline:
// chain s uses tokens/draft/target[s*k .. s*k+k). Each thread keeps its own
// reference RNG stream, as the reference does.
void ref_verify_batch(int nseq, int k, const int32_t* tokens, const float* draft,
                      const float* target, uint32_t* accepted_len, int threads) {
    if (threads < 1) threads = 1;
    std::vector<std::thread> pool;
    for (int w = 0; w < threads; ++w) {
        pool.emplace_back([=] {
            SpeculativeTreeVerifier::Config cfg;
            cfg.log_diagnostics = false;
            SpeculativeTreeVerifier v(cfg);
            std::vector<int32_t> tk(k);
            std::vector<float> d(k), t(k);
            for (int s = w; s < nseq; s += threads) {
                tk.assign(tokens + (size_t)s * k, tokens + (size_t)s * k + k);
                d.assign(draft + (size_t)s * k, draft + (size_t)s * k + k);
                t.assign(target + (size_t)s * k, target + (size_t)s * k + k);
                accepted_len[s] = v.verify_draft_tokens(tk, d, t).first;
            }
        });
    }
    for (auto& th : pool) th.join();
}

// One-hot token mask of construct_tree_mask for a chain of tokens.
int ref_tree_mask(int n, const int32_t* tokens, int vocab, float* out) {
    SpeculativeTreeVerifier::Config cfg;
    cfg.log_diagnostics = false;
    cfg.vocab_size = static_cast<uint32_t>(vocab);
    SpeculativeTreeVerifier v(cfg);
    std::vector<A11::Engine::TreeNode> tree(n);
    for (int i = 0; i < n; ++i) {
        tree[i].token_id = tokens[i];
        tree[i].parent_idx = i == 0 ? UINT32_MAX : static_cast<uint32_t>(i - 1);
        tree[i].depth = static_cast<uint32_t>(i);
    }
    auto m = v.construct_tree_mask(tree);
    for (size_t i = 0; i < m.size(); ++i) out[i] = m[i];
    return static_cast<int>(m.size());
}

}  // extern "C"

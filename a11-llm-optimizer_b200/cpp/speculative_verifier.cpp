// speculative_verifier.cpp - A11::Engine::SpeculativeTreeVerifier over liba11spec.
//
// verify_draft_tokens copies the chain (draft, target, uniforms) to the device,
// runs a11s_verify_chain and reads back (accepted_len, last_idx). Errors follow
// the reference (src/engine/speculative_verifier.cpp:89-97): std::runtime_error
// for mismatched lengths and for NaN/Inf target values; a missing or failing
// CUDA device also throws (there is no host fallback).
#include "engine/speculative_verifier.hpp"

#include <cuda_runtime.h>

#include <cmath>

#include "a11spec.h"

namespace A11 {
namespace Engine {

struct SpeculativeTreeVerifier::Device {
    cudaStream_t stream = nullptr;
    float *buf = nullptr;   // draft | target | uniforms, `cap` floats each
    int32_t *out = nullptr; // accepted_len, last_idx
    void *ws = nullptr;     // status word
    size_t cap = 0;

    void ensure(size_t n) {
        if (!stream && cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess)
            throw std::runtime_error("SpeculativeTreeVerifier: no usable CUDA device");
        if (n <= cap) return;
        release_buffers();
        size_t c = 64;
        while (c < n) c *= 2;
        if (cudaMalloc(&buf, 3 * c * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&out, 2 * sizeof(int32_t)) != cudaSuccess || cudaMalloc(&ws, 256) != cudaSuccess)
            throw std::runtime_error("SpeculativeTreeVerifier: device allocation failed");
        cap = c;
    }
    void release_buffers() {
        if (buf) cudaFree(buf);
        if (out) cudaFree(out);
        if (ws) cudaFree(ws);
        buf = nullptr;
        out = nullptr;
        ws = nullptr;
        cap = 0;
    }
    ~Device() {
        release_buffers();
        if (stream) cudaStreamDestroy(stream);
    }
};

SpeculativeTreeVerifier::SpeculativeTreeVerifier(const Config &cfg) : config_(cfg), diags_{} {}

SpeculativeTreeVerifier::~SpeculativeTreeVerifier() { delete dev_; }

std::mt19937 &SpeculativeTreeVerifier::rng() {
    thread_local std::mt19937 r(42);  // the reference's stream (speculative_verifier.cpp:65-69)
    return r;
}

float SpeculativeTreeVerifier::rand_uniform() {
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    return dist(rng());
}

TreeNode SpeculativeTreeVerifier::build_draft_tree(int32_t root_token) {
    TreeNode root;
    root.token_id = root_token;
    if (config_.log_diagnostics)
        std::cerr << "[SpeculativeTree] Built tree root: token=" << root_token
                  << ", max_depth=" << config_.max_draft_depth << std::endl;
    return root;
}

std::vector<float> SpeculativeTreeVerifier::construct_tree_mask(const std::vector<TreeNode> &tree) {
    if (tree.empty()) return {};
    std::vector<float> mask(tree.size() * config_.vocab_size, 0.0f);
    for (size_t i = 0; i < tree.size(); ++i) {
        const int32_t t = tree[i].token_id;
        if (t >= 0 && static_cast<uint32_t>(t) < config_.vocab_size) mask[i * config_.vocab_size + t] = 1.0f;
    }
    return mask;
}

std::pair<uint32_t, uint32_t> SpeculativeTreeVerifier::verify_draft_tokens(
    const std::vector<int32_t> &draft_tokens, const std::vector<float> &draft_log_probs,
    const std::vector<float> &target_log_probs) {
    const size_t n = draft_tokens.size();
    if (draft_log_probs.size() != n || target_log_probs.size() != n)
        throw std::runtime_error("SpeculativeTreeVerifier: draft_tokens, draft_log_probs, and "
                                 "target_log_probs must have same length");
    bool finite = n > 0;
    for (float p : target_log_probs) finite = finite && std::isfinite(p);
    if (!finite) throw std::runtime_error("SpeculativeTreeVerifier: invalid target probabilities");

    // Draw the chain's uniforms ahead, then leave the stream where the
    // reference leaves it: one draw per judged token, none after a rejection.
    const std::mt19937 saved = rng();
    std::vector<float> host(3 * n);
    for (size_t i = 0; i < n; ++i) {
        host[i] = draft_log_probs[i];
        host[n + i] = target_log_probs[i];
        host[2 * n + i] = rand_uniform();
    }
    if (!dev_) dev_ = new Device();
    dev_->ensure(n);
    float *d = dev_->buf;
    int32_t res[2] = {0, 0};
    cudaStream_t s = dev_->stream;
    bool ok = cudaMemcpyAsync(d, host.data(), n * sizeof(float), cudaMemcpyHostToDevice, s) == cudaSuccess &&
              cudaMemcpyAsync(d + dev_->cap, host.data() + n, n * sizeof(float), cudaMemcpyHostToDevice, s) ==
                  cudaSuccess &&
              cudaMemcpyAsync(d + 2 * dev_->cap, host.data() + 2 * n, n * sizeof(float), cudaMemcpyHostToDevice,
                              s) == cudaSuccess;
    if (!ok) throw std::runtime_error("SpeculativeTreeVerifier: host-to-device copy failed");
    const int rc = a11s_verify_chain(d, d + dev_->cap, d + 2 * dev_->cap, 1, static_cast<int32_t>(n), dev_->out,
                                     dev_->out + 1, dev_->ws, 256, s);
    if (rc != A11S_OK) throw std::runtime_error(std::string("SpeculativeTreeVerifier: ") + a11s_last_error());
    if (cudaMemcpyAsync(res, dev_->out, sizeof res, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        throw std::runtime_error("SpeculativeTreeVerifier: device-to-host copy failed");
    if (res[0] < 0) throw std::runtime_error("SpeculativeTreeVerifier: invalid target probabilities");
    const uint32_t accepted = static_cast<uint32_t>(res[0]);
    const size_t consumed = accepted < n ? accepted + 1 : n;
    rng() = saved;
    rng().discard(consumed);
    return {accepted, static_cast<uint32_t>(res[1])};
}

std::pair<std::vector<int32_t>, bool> SpeculativeTreeVerifier::speculate_step(
    const std::vector<int32_t> &context_tokens, int32_t root_draft_token) {
    ++diags_.total_steps;
    build_draft_tree(root_draft_token);
    if (config_.log_diagnostics)
        std::cerr << "[SpeculativeTree] Speculation step #" << diags_.total_steps
                  << ", context_tokens=" << context_tokens.size() << ", root_draft=" << root_draft_token
                  << std::endl;
    // the reference's synthetic chain (speculative_verifier.cpp:155-166)
    std::vector<int32_t> draft(SPEC_K);
    std::vector<float> dlp(SPEC_K), tlp(SPEC_K);
    for (uint32_t i = 0; i < SPEC_K; ++i) {
        draft[i] = root_draft_token + static_cast<int32_t>(i) + 1;
        dlp[i] = -std::log(static_cast<float>(SPEC_K)) * (1.0f - i * 0.05f);
        tlp[i] = dlp[i] + (rand_uniform() < 0.9f ? -0.1f : -2.0f);
    }
    diags_.total_draft_tokens += SPEC_K;
    const auto [accepted, last] = verify_draft_tokens(draft, dlp, tlp);
    if (config_.log_diagnostics)
        std::cerr << "[SpeculativeTree] Verification: accepted=" << accepted << ", last_accepted_idx=" << last
                  << " / " << SPEC_K << std::endl;
    if (accepted == 0) {
        ++diags_.steps_rejected;
        diags_.log_fallback(SPEC_K, 0);
    } else {
        ++diags_.steps_accepted;
    }
    std::vector<int32_t> out(draft.begin(), draft.begin() + accepted);
    out.push_back(root_draft_token + static_cast<int32_t>(SPEC_K));
    return {out, accepted == SPEC_K};
}

}  // namespace Engine
}  // namespace A11

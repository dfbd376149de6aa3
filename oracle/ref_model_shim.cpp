// TEST INFRASTRUCTURE ONLY — never linked into, loaded by, or called from the
// product library.
//
// C entry points over the reference's own model oracle: ReferenceModel and
// referenceGeneration, which live test-local in the reference's runner
// contract test (tests/cuda/cuda_model_runner_test.cpp:213-457), together
// with that test's deterministic weight builder TestArchive (:55-211). The
// test file is compiled here from where it lies in the reference tree
// (oracle/Makefile passes its directory as an include path); its main() and
// its CUDA test cases are renamed into an unused internal function and are
// never emitted, so nothing of the reference's CUDA runtime is linked.
//
// The model is either the contract archive exactly as the reference test
// builds it, or an archive of another configuration whose config and
// weights are replaced by the caller's FP16 tensors (ReferenceModel reads
// only TestArchive::config and TestArchive::weights). Rounding points are the
// reference's: its rounded() is the CUDA host FP16 conversion.
#include "kim-kv/cuda/cuda_engine_kv_backend.h"
#include "kim-kv/cuda/cuda_model_runner.h"
#include "kim-kv/engine/iteration_scheduler.h"
#include "kim-kv/model/weight_manifest.h"

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <limits>
#include <memory>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

#define main kref_model_test_main_unused
namespace {
#include "cuda/cuda_model_runner_test.cpp"
}
#undef main

extern "C" {

typedef struct kref_model_config {
    uint32_t hidden, intermediate, layers, q_heads, kv_heads, head_dim, vocab, max_positions;
    float eps, theta;
} kref_model_config;

#define KREF_API __attribute__((visibility("default")))

} // extern "C"

namespace {

struct RefModel {
    std::unique_ptr<TestArchive> archive;
    std::unique_ptr<ReferenceModel> model;
    std::vector<std::string> names;  // tensors in the oracle's order
};

std::atomic<unsigned> g_archive_seq{0};

// Tensor names in the oracle's order: embed, lm_head, final norm, then per
// layer input norm, post norm, q, k, v, o, gate, up, down.
std::vector<std::string> tensorNames(std::uint32_t layers)
{
    std::vector<std::string> n{"model.embed_tokens.weight", "lm_head.weight", "model.norm.weight"};
    for (std::uint32_t l = 0; l < layers; ++l) {
        std::string const p = "model.layers." + std::to_string(l) + ".";
        for (char const* t : {"input_layernorm.weight", "post_attention_layernorm.weight",
                 "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                 "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                 "mlp.down_proj.weight"}) {
            n.push_back(p + t);
        }
    }
    return n;
}

std::size_t tensorElements(TinyLlamaConfig const& c, std::string const& name)
{
    std::size_t const H = c.hidden_size, I = c.intermediate_size, V = c.vocabulary_size;
    std::size_t const KV = std::size_t(c.kv_head_count) * c.head_dimension;
    auto ends = [&](char const* s) {
        std::size_t const n = std::strlen(s);
        return name.size() >= n && name.compare(name.size() - n, n, s) == 0;
    };
    if (ends("embed_tokens.weight") || ends("lm_head.weight")) return V * H;
    if (ends("norm.weight")) return H;
    if (ends("k_proj.weight") || ends("v_proj.weight")) return KV * H;
    if (ends("q_proj.weight") || ends("o_proj.weight")) return H * H;
    return I * H;  // gate, up, down
}

} // namespace

extern "C" {

// config NULL: the reference test's contract archive with its own weights.
// Otherwise the weights (FP16 bits, oracle order) replace the archive's.
KREF_API void* kref_model_create(const kref_model_config* config, const uint16_t* const* weights,
    const char* scratch_dir)
{
    auto h = std::make_unique<RefModel>();
    std::filesystem::path const dir = std::filesystem::path(scratch_dir)
        / ("kref_model_" + std::to_string(g_archive_seq.fetch_add(1)));
    h->archive = std::make_unique<TestArchive>(dir);
    if (config != nullptr) {
        TinyLlamaConfig c = h->archive->config;
        c.hidden_size = config->hidden;
        c.intermediate_size = config->intermediate;
        c.layer_count = config->layers;
        c.attention_head_count = config->q_heads;
        c.kv_head_count = config->kv_heads;
        c.head_dimension = config->head_dim;
        c.vocabulary_size = config->vocab;
        c.max_position_embeddings = config->max_positions;
        c.rms_norm_epsilon = config->eps;
        c.rope_theta = config->theta;
        h->archive->config = c;
        h->archive->weights.clear();
        std::vector<std::string> const names = tensorNames(c.layer_count);
        for (std::size_t i = 0; i < names.size(); ++i) {
            std::size_t const n = tensorElements(c, names[i]);
            std::vector<float> values(n);
            for (std::size_t e = 0; e < n; ++e) {
                values[e] = fp32(weights[i][e]);
            }
            h->archive->weights.emplace(names[i], std::move(values));
        }
    }
    h->names = tensorNames(h->archive->config.layer_count);
    h->model = std::make_unique<ReferenceModel>(*h->archive);
    return h.release();
}

KREF_API void kref_model_destroy(void* p) { delete static_cast<RefModel*>(p); }

KREF_API void kref_model_config_of(void* p, kref_model_config* out)
{
    TinyLlamaConfig const& c = static_cast<RefModel*>(p)->archive->config;
    *out = kref_model_config{c.hidden_size, c.intermediate_size, c.layer_count, c.attention_head_count,
        c.kv_head_count, c.head_dimension, c.vocabulary_size, c.max_position_embeddings,
        c.rms_norm_epsilon, c.rope_theta};
}

KREF_API uint32_t kref_model_tensor_count(void* p)
{
    return static_cast<uint32_t>(static_cast<RefModel*>(p)->names.size());
}

// FP16 bits of tensor `index` (oracle order); returns its element count
// (out may be NULL to query it).
KREF_API uint64_t kref_model_tensor(void* p, uint32_t index, uint16_t* out)
{
    auto* h = static_cast<RefModel*>(p);
    if (index >= h->names.size()) return 0;
    std::vector<float> const& v = h->archive->weights.at(h->names[index]);
    if (out != nullptr) {
        for (std::size_t e = 0; e < v.size(); ++e) {
            out[e] = fp16(v[e]);
        }
    }
    return v.size();
}

// ReferenceModel::forward of the next position: logits [vocab] FP32 and the
// final normalised hidden state [hidden] FP16 (either may be NULL).
KREF_API int kref_model_forward(void* p, uint32_t token, uint32_t position, float* logits,
    uint16_t* final_hidden)
{
    auto* h = static_cast<RefModel*>(p);
    TinyLlamaConfig const& c = h->archive->config;
    if (token >= c.vocabulary_size || position != h->model->keys[0].size()) return 0;
    std::vector<float> const out = h->model->forward(token, position);
    if (logits != nullptr) std::memcpy(logits, out.data(), out.size() * sizeof(float));
    if (final_hidden != nullptr) {
        for (std::size_t i = 0; i < h->model->final_hidden.size(); ++i) {
            final_hidden[i] = fp16(h->model->final_hidden[i]);
        }
    }
    return 1;
}

// ---- lanes: further ReferenceModel instances over the same archive --------
// A lane is one ReferenceModel (its own keys / values) reading the shared,
// immutable archive; lanes may run forward concurrently.

KREF_API void* kref_model_lane_create(void* p)
{
    try {
        return new ReferenceModel(*static_cast<RefModel*>(p)->archive);
    } catch (...) {
        return nullptr;
    }
}

KREF_API void kref_model_lane_destroy(void* lane) { delete static_cast<ReferenceModel*>(lane); }

KREF_API uint32_t kref_model_lane_length(void* lane)
{
    return static_cast<uint32_t>(static_cast<ReferenceModel*>(lane)->keys[0].size());
}

// Appends n past tokens of given K / V (FP16 bits, [n][layers][kv_heads *
// head_dim] each) to the lane's cache, as forward would have stored them.
KREF_API int kref_model_lane_append_kv(void* p, void* lane, uint32_t n, const uint16_t* k,
    const uint16_t* v)
{
    TinyLlamaConfig const& c = static_cast<RefModel*>(p)->archive->config;
    auto* m = static_cast<ReferenceModel*>(lane);
    std::size_t const row = std::size_t(c.kv_head_count) * c.head_dimension;
    for (uint32_t t = 0; t < n; ++t) {
        for (uint32_t l = 0; l < c.layer_count; ++l) {
            std::size_t const base = (std::size_t(t) * c.layer_count + l) * row;
            std::vector<float> kr(row), vr(row);
            for (std::size_t e = 0; e < row; ++e) {
                kr[e] = fp32(k[base + e]);
                vr[e] = fp32(v[base + e]);
            }
            m->keys[l].push_back(std::move(kr));
            m->values[l].push_back(std::move(vr));
        }
    }
    return 1;
}

// One ReferenceModel::forward per lane, lanes spread over `threads` host
// threads; next[i] is the lane's greedy token (first maximum, as
// referenceGeneration takes it). Returns 1 when every lane ran.
KREF_API int kref_model_forward_lanes(void* p, uint32_t n, void* const* lanes, const uint32_t* tokens,
    const uint32_t* positions, uint32_t* next, uint32_t threads)
{
    TinyLlamaConfig const& c = static_cast<RefModel*>(p)->archive->config;
    for (uint32_t i = 0; i < n; ++i) {
        auto* m = static_cast<ReferenceModel*>(lanes[i]);
        if (tokens[i] >= c.vocabulary_size || positions[i] != m->keys[0].size()) return 0;
    }
    std::atomic<uint32_t> cursor{0};
    auto work = [&]() {
        for (uint32_t i = cursor.fetch_add(1); i < n; i = cursor.fetch_add(1)) {
            std::vector<float> const logits = static_cast<ReferenceModel*>(lanes[i])->forward(
                tokens[i], positions[i]);
            next[i] = static_cast<uint32_t>(std::max_element(logits.begin(), logits.end()) - logits.begin());
        }
    };
    std::vector<std::thread> pool;
    for (uint32_t t = 1; t < std::max<uint32_t>(1u, std::min(threads, n)); ++t) {
        pool.emplace_back(work);
    }
    work();
    for (std::thread& t : pool) {
        t.join();
    }
    return 1;
}

// referenceGeneration (a fresh ReferenceModel): greedy tokens after the prompt.
KREF_API int kref_model_generate(void* p, const uint32_t* prompt, uint32_t n, uint32_t max_new,
    uint32_t* out)
{
    auto* h = static_cast<RefModel*>(p);
    std::vector<std::uint32_t> const tokens = referenceGeneration(*h->archive,
        std::vector<std::uint32_t>(prompt, prompt + n), max_new);
    std::copy(tokens.begin(), tokens.end(), out);
    return static_cast<int>(tokens.size());
}

} // extern "C"

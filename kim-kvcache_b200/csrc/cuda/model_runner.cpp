// CUDA TinyLlama runner on the sm_100a kernels. Reference behaviour:
// src/cuda/model/runner.cpp:53-880 (forwardToken, generationForwardBatch),
// src/cuda/model/runner_factory.cpp:12-194 (load), runner_support.cpp (workspace).
#include "model_runner.h"

#include "kernels_internal.h"

#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstring>
#include <fstream>
#include <unordered_map>
#include <unordered_set>

namespace kimkvcache {
namespace {

CudaModelRunnerStatus failure(CudaModelRunnerError e, int code, std::string detail)
{
    return CudaModelRunnerStatus{e, code, std::move(detail)};
}

CudaModelRunnerStatus cudaFailure(int code, std::string const& what)
{
    return failure(code == KK_EINVAL ? CudaModelRunnerError::InvalidArgument
                                     : CudaModelRunnerError::SubmissionFailed,
        code, what + ": " + (code == KK_EINVAL ? "invalid kernel arguments"
                                                : cudaGetErrorString(static_cast<cudaError_t>(code))));
}

CudaModelRunnerStatus kvFailure(EngineKvStatus s, std::string const& what)
{
    return failure(CudaModelRunnerError::KvBackendFailed, static_cast<int>(s.error),
        what + " failed: " + std::string(toString(s.error)));
}


std::size_t align256(std::size_t x) { return (x + 255) & ~std::size_t(255); }

struct LayerWeights {
    std::uint16_t const* in_norm;
    std::uint16_t const* post_norm;
    // Projection matrices, packed by kk_gemm_pack_weight (16 KB swizzled tiles).
    std::uint16_t const* w_qkv;   // [(Hq + 2 Hkv) D][H]: q rows, k rows, v rows
    std::uint16_t const* w_o;     // [H][H]
    std::uint16_t const* w_gu;    // [2 I][H]: row 2i = gate_i, row 2i+1 = up_i
    std::uint16_t const* w_down;  // [H][I]
};

// Prepared projections of one batch size.
struct BatchPlans {
    std::vector<kk::GemmPlanPtr> qkv, o, gu, down;
    kk::GemmPlanPtr lm_head;
    kk::GemmPlanPtr lm_head_logits;  // same, also storing FP32 logits
};

} // namespace

struct CudaTinyLlamaModelRunner::Impl {
    TinyLlamaConfig cfg{};
    WeightManifest manifest{};
    EngineKvBackend* kv{nullptr};
    cudaStream_t stream{nullptr};
    CudaModelRunnerOptions options{};
    kk_kv_pools pools{};

    std::uint8_t* weights{nullptr};   // embedding table and norm weights (row-major)
    std::uint8_t* packed{nullptr};    // projection matrices and LM head, packed tiles
    std::uint64_t weight_bytes{0};
    std::uint16_t const* embed{nullptr};
    std::uint16_t const* lm_head{nullptr};
    std::uint16_t const* final_norm{nullptr};
    std::vector<LayerWeights> layers;

    // Workspace (device).
    std::uint8_t* ws{nullptr};
    std::uint64_t ws_bytes{0};
    std::uint32_t bpad{0};
    std::uint16_t* hidden{nullptr};
    std::uint16_t* normed{nullptr};
    std::uint16_t* q{nullptr};
    std::uint16_t* attn{nullptr};
    std::uint16_t* act{nullptr};
    float* logits{nullptr};
    std::uint32_t* out_tokens{nullptr};  // in the step's result block (below)
    void* attn_ws{nullptr};
    std::uint64_t attn_ws_bytes{0};
    void* argmax_ws{nullptr};
    // RMSNorm statistics handed from the kernel that writes the residual rows
    // to the projection that normalises them: per 128-row tile and batch row,
    // the sum of squares (rows of 64 floats). sq_embed: the embedding rows
    // (one tile), sq_attn_out: after the output projection, sq_mlp_out:
    // after the down projection.
    float* sq_embed{nullptr};
    float* sq_attn_out{nullptr};
    float* sq_mlp_out{nullptr};
    // RoPE factors (cos, sin) of every position and rotation pair, computed
    // once on the host with the math library the reference's model uses.
    float* rope_cs{nullptr};

    // Step inputs: one region on the device, a pinned mirror on the host.
    std::uint32_t max_items{0};
    std::uint32_t sm_count{148};
    std::uint32_t max_descs{0};
    std::size_t off_counts{0}, off_result{0}, off_tokens{0}, off_positions{0}, off_slots{0},
        off_copies{0}, off_lanes{0}, off_items{0}, off_descs{0}, step_bytes{0};
    std::uint8_t* step_dev{nullptr};
    std::uint8_t* step_host{nullptr};
    // Result block of a step: the step's error word (kResultHeader bytes, the
    // word first), then the greedy token ids. It sits inside the uploaded
    // part of the step record, so every upload clears the error word; the
    // kernels of the step report errors there (first error wins), and one
    // device-to-host copy brings back the word and the tokens together.
    static constexpr std::size_t kResultHeader = 16;
    unsigned int* status_dev{nullptr};
    std::uint8_t* host_result{nullptr};
    std::uint32_t const* host_tokens{nullptr};

    cudaEvent_t ev_begin{nullptr};
    cudaEvent_t ev_end{nullptr};
    // Graphs are captured on this private stream (capture is not allowed on
    // the legacy default stream a caller may pass) and replayed on `stream`.
    cudaStream_t capture_stream{nullptr};
    std::string last_error;
    bool auto_promote{false};
    float last_ms{0.f};
    std::uint32_t last_launches{0};
    std::uint64_t last_h2d{0};
    std::uint64_t last_d2h{0};
    // Host wall time of the last fused step's phases (microseconds): lane
    // reservations, step record, upload + launch, wait, commits.
    std::array<float, 5> last_host_us{};

    std::unordered_map<std::uint32_t, BatchPlans> plans;
    std::unordered_map<std::uint32_t, cudaGraphExec_t> graphs;

    ~Impl()
    {
        if (stream != nullptr) {
            cudaStreamSynchronize(stream);
        }
        for (auto& g : graphs) {
            cudaGraphExecDestroy(g.second);
        }
        plans.clear();
        cudaFree(weights);
        cudaFree(packed);
        cudaFree(ws);
        cudaFree(step_dev);
        cudaFreeHost(step_host);
        cudaFreeHost(host_result);
        if (capture_stream != nullptr) cudaStreamDestroy(capture_stream);
        if (ev_begin != nullptr) cudaEventDestroy(ev_begin);
        if (ev_end != nullptr) cudaEventDestroy(ev_end);
    }

    template <typename T>
    T* stepHost(std::size_t off) { return reinterpret_cast<T*>(step_host + off); }
    template <typename T>
    T* stepDev(std::size_t off) { return reinterpret_cast<T*>(step_dev + off); }

    CudaModelRunnerStatus buildPlans(std::uint32_t batch, BatchPlans& out);
    CudaModelRunnerStatus enqueueForward(cudaStream_t on, std::uint32_t batch, bool has_copies,
        BatchPlans const& p, bool want_logits, ModelRunnerDebugCapture* debug);
    CudaModelRunnerStatus runStep(std::uint32_t batch, bool has_copies, bool want_logits,
        ModelRunnerDebugCapture* debug);
    CudaModelRunnerStatus finishStep(std::uint32_t batch, std::vector<float>* logits_out, char const* what);
};

CudaTinyLlamaModelRunner::CudaTinyLlamaModelRunner(std::unique_ptr<Impl> impl) noexcept
    : impl_(std::move(impl))
{
}

CudaTinyLlamaModelRunner::~CudaTinyLlamaModelRunner() = default;

TinyLlamaConfig CudaTinyLlamaModelRunner::config() const noexcept { return impl_->cfg; }
TinyLlamaConfig CudaTinyLlamaModelRunner::generationConfig() const noexcept { return impl_->cfg; }
std::uint64_t CudaTinyLlamaModelRunner::deviceWeightBytes() const noexcept { return impl_->weight_bytes; }
std::uint64_t CudaTinyLlamaModelRunner::deviceWorkspaceBytes() const noexcept
{
    return impl_->ws_bytes + impl_->step_bytes;
}
std::uint32_t CudaTinyLlamaModelRunner::maxBatchSize() const noexcept { return impl_->options.max_batch_size; }
std::uint32_t CudaTinyLlamaModelRunner::generationMaxBatchSize() const noexcept
{
    return impl_->options.max_batch_size;
}
float CudaTinyLlamaModelRunner::lastStepDeviceMs() const noexcept { return impl_->last_ms; }
void CudaTinyLlamaModelRunner::setAutoPromote(bool enabled) noexcept { impl_->auto_promote = enabled; }
std::string CudaTinyLlamaModelRunner::lastError() const { return impl_->last_error; }
std::uint32_t CudaTinyLlamaModelRunner::lastStepLaunches() const noexcept { return impl_->last_launches; }
std::uint64_t CudaTinyLlamaModelRunner::lastStepH2dBytes() const noexcept { return impl_->last_h2d; }
std::uint64_t CudaTinyLlamaModelRunner::lastStepD2hBytes() const noexcept { return impl_->last_d2h; }
std::array<float, 5> CudaTinyLlamaModelRunner::lastStepHostUs() const noexcept { return impl_->last_host_us; }

CudaModelRunnerStatus CudaTinyLlamaModelRunner::Impl::buildPlans(std::uint32_t batch, BatchPlans& out)
{
    TinyLlamaConfig const& c = cfg;
    std::uint32_t const qkv_rows = (c.attention_head_count + 2 * c.kv_head_count) * c.head_dimension;
    auto make = [&](kk_gemm_desc const& d, kk::GemmPlanPtr& slot) -> bool {
        int rc = 0;
        slot = kk::gemmPlan(d, rc);
        return slot != nullptr;
    };
    auto base = [&](std::uint16_t const* w, std::uint32_t m, std::uint32_t k, std::uint16_t const* x,
                    std::uint32_t epi, void* o, std::uint32_t ostride) {
        kk_gemm_desc d{};
        d.weight = w;
        d.M = m;
        d.K = k;
        d.x = x;
        d.N = batch;
        d.x_stride = k;
        d.x_rows = bpad;
        d.epilogue = epi;
        d.out = o;
        d.out_stride = ostride;
        d.weight_layout = KK_W_PACKED;
        return d;
    };
    // RMSNorm fused into the projection: the GEMM normalises the residual
    // rows in shared memory, half(x * r * g), before the tensor cores read them.
    auto normedInput = [&](kk_gemm_desc d, std::uint16_t const* g) {
        d.norm_input = hidden;
        d.norm_stride = c.hidden_size;
        d.norm_eps = c.rms_norm_epsilon;
        d.norm_weight = g;
        return d;
    };
    for (std::uint32_t l = 0; l < c.layer_count; ++l) {
        LayerWeights const& w = layers[l];
        kk_gemm_desc d = normedInput(base(w.w_qkv, qkv_rows, c.hidden_size, hidden, KK_EPI_QKV_ROPE, q,
            c.hidden_size), w.in_norm);
        d.positions = stepDev<std::uint32_t>(off_positions);
        d.slots = stepDev<kk_kv_slot>(off_slots);
        d.pools = pools;
        d.layer = l;
        d.q_rows = c.attention_head_count * c.head_dimension;
        d.kv_rows = c.kv_head_count * c.head_dimension;
        d.head_dim = c.head_dimension;
        d.rope_theta = c.rope_theta;
        d.rope_cos_sin = rope_cs;
        d.rope_positions = c.max_position_embeddings;
        out.qkv.emplace_back();
        out.o.emplace_back();
        out.gu.emplace_back();
        out.down.emplace_back();
        auto atLayer = [l](kk_gemm_desc x) {
            x.layer = l;
            return x;
        };
        if (!make(d, out.qkv.back())
            || !make(atLayer(base(w.w_o, c.hidden_size, c.hidden_size, attn, KK_EPI_RESIDUAL, hidden,
                          c.hidden_size)), out.o.back())
            || !make(atLayer(normedInput(base(w.w_gu, 2 * c.intermediate_size, c.hidden_size, hidden,
                          KK_EPI_SILU_PAIRS, act, c.intermediate_size), w.post_norm)), out.gu.back())
            || !make(atLayer(base(w.w_down, c.hidden_size, c.intermediate_size, act, KK_EPI_RESIDUAL, hidden,
                          c.hidden_size)), out.down.back())) {
            return failure(CudaModelRunnerError::InvalidArgument, KK_EINVAL, "projection plan rejected");
        }
    }
    // RMSNorm statistics travel with the residual rows (see sq_* above).
    std::uint32_t const sq_tiles = (c.hidden_size + 127) / 128;
    for (std::uint32_t l = 0; l < c.layer_count; ++l) {
        if (!kk::gemmSetNormPartials(*out.qkv[l], l == 0 ? sq_embed : sq_mlp_out, l == 0 ? 1u : sq_tiles)
            || !kk::gemmSetSumSquaresOut(*out.o[l], sq_attn_out)
            || !kk::gemmSetNormPartials(*out.gu[l], sq_attn_out, sq_tiles)
            || !kk::gemmSetSumSquaresOut(*out.down[l], sq_mlp_out)) {
            return failure(CudaModelRunnerError::InvalidArgument, KK_EINVAL, "norm statistics rejected");
        }
    }
    // L2 prefetch: the output projection's weights are already on chip when
    // its dependency wait returns (its CTAs load them while attention runs),
    // and HBM then idles while it exchanges partials; its CTAs use that time
    // to fetch the down projection's weights into L2. (Measured on the c4
    // step: fetching the gate/up weights during attention, or attention's
    // first pages during the QKV projection, did not pay: attention streams
    // at the HBM rate already.)
    for (std::uint32_t l = 0; l < c.layer_count; ++l) {
        kk::gemmSetL2Prefetch(*out.o[l], layers[l].w_down,
            kk_gemm_packed_bytes(c.hidden_size, c.intermediate_size));
        for (kk::GemmPlan* g : {out.qkv[l].get(), out.o[l].get(), out.gu[l].get(), out.down[l].get()}) {
            kk::gemmSetStatus(*g, status_dev);
        }
    }
    kk_gemm_desc lm = normedInput(base(lm_head, c.vocabulary_size, c.hidden_size, hidden, KK_EPI_ARGMAX,
        nullptr, 0), final_norm);
    lm.tokens = out_tokens;
    lm.argmax_workspace = argmax_ws;
    kk_gemm_desc lm_logits = lm;
    lm_logits.out = logits;
    lm_logits.out_stride = c.vocabulary_size;
    if (!make(lm, out.lm_head) || !make(lm_logits, out.lm_head_logits)
        || !kk::gemmSetNormPartials(*out.lm_head, sq_mlp_out, sq_tiles)
        || !kk::gemmSetNormPartials(*out.lm_head_logits, sq_mlp_out, sq_tiles)) {
        return failure(CudaModelRunnerError::InvalidArgument, KK_EINVAL, "LM head plan rejected");
    }
    kk::gemmSetStatus(*out.lm_head, status_dev);
    kk::gemmSetStatus(*out.lm_head_logits, status_dev);
    return {};
}

CudaModelRunnerStatus CudaTinyLlamaModelRunner::Impl::enqueueForward(cudaStream_t stream,
    std::uint32_t batch, bool has_copies, BatchPlans const& p, bool want_logits,
    ModelRunnerDebugCapture* debug)
{
    TinyLlamaConfig const& c = cfg;
    std::uint32_t const H = c.hidden_size;
    std::uint32_t const qrow = c.attention_head_count * c.head_dimension;
    float const scale = 1.0f / std::sqrt(static_cast<float>(c.head_dimension));
    std::uint32_t launches = 0;
    auto check = [&](int rc, char const* what) {
        ++launches;
        return rc == 0 ? CudaModelRunnerStatus{} : cudaFailure(rc, what);
    };
    CudaModelRunnerStatus s;
    if (has_copies) {
        s = check(kk::kvCopyDevCount(&pools, 0, c.layer_count, stepDev<kk_kv_copy>(off_copies),
                      stepDev<std::uint32_t>(off_counts) + 1, batch, status_dev, stream), "copy-on-write");
        if (!s.ok()) return s;
    }
    // Embedding gather starts the residual stream; the first projection
    // normalises its rows with the sums of squares written here.
    s = check(kk::embedSumSquares(embed, stepDev<std::uint32_t>(off_tokens), hidden, sq_embed, batch, H,
                  stream), "embedding");
    if (!s.ok()) return s;
    std::unordered_map<std::uint32_t, std::size_t> capture;
    if (debug != nullptr) {
        cudaMemcpyAsync(debug->embedding.data(), hidden, H * 2, cudaMemcpyDeviceToHost, stream);
        for (std::size_t i = 0; i < debug->layer_indices.size(); ++i) {
            capture.emplace(debug->layer_indices[i], i);
        }
    }
    for (std::uint32_t l = 0; l < c.layer_count; ++l) {
        if (!(s = check(kk::gemmRun(*p.qkv[l], stream), "qkv projection")).ok()
            || !(s = check(kk::attentionDevCount(&pools, l, c.attention_head_count,
                     stepDev<kk_page_desc>(off_descs), stepDev<kk_attn_lane>(off_lanes), batch,
                     stepDev<kk_attn_item>(off_items), stepDev<std::uint32_t>(off_counts), max_items,
                     q, qrow, attn, qrow, scale, attn_ws, attn_ws_bytes, status_dev, stream),
                     "paged attention")).ok()
            || !(s = check(kk::gemmRun(*p.o[l], stream), "output projection")).ok()
            || !(s = check(kk::gemmRun(*p.gu[l], stream), "gate/up projection")).ok()
            || !(s = check(kk::gemmRun(*p.down[l], stream), "down projection")).ok()) {
            return s;
        }
        if (debug != nullptr) {
            auto const f = capture.find(l);
            if (f != capture.end()) {
                cudaMemcpyAsync(debug->layer_hidden_states[f->second].data(), hidden, H * 2,
                    cudaMemcpyDeviceToHost, stream);
            }
        }
    }
    s = check(kk::gemmRun(want_logits ? *p.lm_head_logits : *p.lm_head, stream), "lm head + argmax");
    if (!s.ok()) return s;
    if (debug != nullptr) {
        // The decode step never materialises the final normalised rows (the
        // LM head normalises internally); the debug capture computes them.
        s = check(kk_rmsnorm(hidden, final_norm, normed, batch, H, c.rms_norm_epsilon, stream), "final rmsnorm");
        if (!s.ok()) return s;
        cudaMemcpyAsync(debug->final_hidden_state.data(), normed, H * 2, cudaMemcpyDeviceToHost, stream);
    }
    last_launches = launches;
    return {};
}

CudaModelRunnerStatus CudaTinyLlamaModelRunner::Impl::runStep(std::uint32_t batch, bool has_copies,
    bool want_logits, ModelRunnerDebugCapture* debug)
{
    auto found = plans.find(batch);
    if (found == plans.end()) {
        BatchPlans fresh;
        CudaModelRunnerStatus const built = buildPlans(batch, fresh);
        if (!built.ok()) {
            return built;
        }
        found = plans.emplace(batch, std::move(fresh)).first;
    }
    kk_set_pdl(1);
    cudaEventRecord(ev_begin, stream);
    bool const graphable = options.use_cuda_graphs && debug == nullptr && !want_logits;
    CudaModelRunnerStatus s;
    if (graphable) {
        std::uint32_t const key = batch * 2 + (has_copies ? 1u : 0u);
        auto g = graphs.find(key);
        if (g == graphs.end()) {
            cudaGraph_t graph = nullptr;
            cudaError_t e = cudaStreamBeginCapture(capture_stream, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                s = enqueueForward(capture_stream, batch, has_copies, found->second, false, nullptr);
                cudaError_t const ended = cudaStreamEndCapture(capture_stream, &graph);
                e = s.ok() ? ended : cudaSuccess;
            }
            cudaGraphExec_t exec = nullptr;
            if (e == cudaSuccess && s.ok()) {
                e = cudaGraphInstantiate(&exec, graph, 0);
            }
            if (graph != nullptr) {
                cudaGraphDestroy(graph);
            }
            if (!s.ok()) {
                kk_set_pdl(0);
                return s;
            }
            if (e != cudaSuccess) {
                kk_set_pdl(0);
                return cudaFailure(static_cast<int>(e), "capture decode graph");
            }
            g = graphs.emplace(key, exec).first;
        }
        cudaError_t const e = cudaGraphLaunch(g->second, stream);
        if (e != cudaSuccess) {
            s = cudaFailure(static_cast<int>(e), "launch decode graph");
        }
    } else {
        s = enqueueForward(stream, batch, has_copies, found->second, want_logits, debug);
    }
    kk_set_pdl(0);
    cudaEventRecord(ev_end, stream);
    return s;
}

char const* deviceErrorName(unsigned int code)
{
    switch (code) {
    case 1: return "a bounded device wait ran out";
    case 2: return "a page descriptor or KV slot outside its pool";
    case 3: return "an inconsistent work list";
    default: return "an unknown device error";
    }
}

// Brings back the step's result block (error word + greedy ids) and the
// optional logits, waits for the step, and turns a device-reported error into
// ExecutionFailed. After such an error the split-attention completion
// counters and the LM head's counter may be left mid-count by the CTAs that
// gave up; both are cleared so that the next step starts clean.
CudaModelRunnerStatus CudaTinyLlamaModelRunner::Impl::finishStep(std::uint32_t batch,
    std::vector<float>* logits_out, char const* what)
{
    std::size_t const bytes = kResultHeader + std::size_t(batch) * 4u;
    cudaError_t e = cudaMemcpyAsync(host_result, status_dev, bytes, cudaMemcpyDeviceToHost, stream);
    last_d2h += bytes;
    if (e == cudaSuccess && logits_out != nullptr) {
        std::size_t const n = std::size_t(batch) * cfg.vocabulary_size;
        logits_out->resize(n);
        e = cudaMemcpyAsync(logits_out->data(), logits, n * 4u, cudaMemcpyDeviceToHost, stream);
        last_d2h += n * 4u;
    }
    if (e == cudaSuccess) {
        e = cudaStreamSynchronize(stream);
    }
    if (e != cudaSuccess) {
        return failure(CudaModelRunnerError::ExecutionFailed, static_cast<int>(e),
            std::string(what) + " failed: " + cudaGetErrorString(e));
    }
    unsigned int code = 0;
    std::memcpy(&code, host_result, sizeof(code));
    if (code == 0) {
        return {};
    }
    cudaError_t const reset = cudaMemsetAsync(attn_ws, 0, align256(std::size_t(options.max_batch_size) * 4u),
        stream);
    if (reset == cudaSuccess && cudaMemsetAsync(argmax_ws, 0, 256, stream) == cudaSuccess) {
        cudaStreamSynchronize(stream);
    }
    return failure(CudaModelRunnerError::ExecutionFailed, static_cast<int>(code),
        std::string(what) + " failed: the device reported " + deviceErrorName(code));
}

// One fused step over every valid lane of `items`.
GenerationBatchResult runBatch(CudaTinyLlamaModelRunner::Impl& im,
    std::vector<GenerationBatchItem> const& items, bool want_logits, ModelRunnerDebugCapture* debug,
    std::vector<float>* logits_out)
{
    GenerationBatchResult result;
    TinyLlamaConfig const& c = im.cfg;
    if (items.empty() || items.size() > im.options.max_batch_size) {
        result.detail = "generation batch is empty or exceeds max batch size";
        return result;
    }
    using Clock = std::chrono::steady_clock;
    Clock::time_point const t_begin = Clock::now();
    Clock::time_point t_mark = t_begin;
    auto phase = [&](std::size_t i) {
        Clock::time_point const now = Clock::now();
        im.last_host_us[i] = std::chrono::duration<float, std::micro>(now - t_mark).count();
        t_mark = now;
    };
    im.last_host_us = {};
    result.steps.resize(items.size());
    std::vector<std::size_t> lane_index;
    std::vector<TokenTransaction> txns;
    lane_index.reserve(items.size());
    txns.reserve(items.size());
    for (std::size_t i = 0; i < items.size(); ++i) {
        GenerationBatchItem const& it = items[i];
        if (it.request_id == kInvalidRequestId || it.token_id >= c.vocabulary_size
            || it.expected_position >= c.max_position_embeddings) {
            result.steps[i] = {false, 0, "request, token, or position is out of range"};
            continue;
        }
        TokenReserveResult reserved = im.kv->reserveToken(
            ReserveTokenRequest{it.request_id, it.expected_position, im.stream});
        if (!reserved.ok()) {
            result.steps[i] = {false, 0, kvFailure(reserved.status, "reserve token").detail};
            continue;
        }
        EngineKvStatus const submitted = reserved.transaction.submitFusedLayers();
        if (!submitted.ok()) {
            result.steps[i] = {false, 0, kvFailure(submitted, "submit fused layers").detail};
            continue;  // the transaction rolls back when it goes out of scope
        }
        lane_index.push_back(i);
        txns.push_back(std::move(reserved.transaction));
    }
    result.success = true;
    std::uint32_t const B = static_cast<std::uint32_t>(txns.size());
    if (B == 0) {
        return result;
    }

    phase(0);
    // Step inputs into the pinned mirror.
    auto* tokens = im.stepHost<std::uint32_t>(im.off_tokens);
    auto* positions = im.stepHost<std::uint32_t>(im.off_positions);
    auto* slots = im.stepHost<kk_kv_slot>(im.off_slots);
    auto* copies = im.stepHost<kk_kv_copy>(im.off_copies);
    auto* lanes = im.stepHost<kk_attn_lane>(im.off_lanes);
    auto* descs = im.stepHost<kk_page_desc>(im.off_descs);
    std::uint32_t n_copies = 0;
    std::uint32_t n_descs = 0;
    for (std::uint32_t b = 0; b < B; ++b) {
        FusedLane lane{};
        if (!fusedLane(txns[b], lane)) {
            result.success = false;
            result.detail = "KV backend does not support the fused decode step";
            return result;
        }
        GenerationBatchItem const& it = items[lane_index[b]];
        tokens[b] = it.token_id;
        positions[b] = it.expected_position;
        auto const& entries = lane.reserved->entries();
        MappingEntry const& target = entries.back();
        slots[b] = kk_kv_slot{target.handle.slot,
            static_cast<std::uint16_t>(lane.reserved->tokenCount() - 1 - target.logical_token_begin),
            static_cast<std::uint8_t>(target.kind), 1};
        if (!lane.before->entries().empty()) {
            MappingEntry const& old_tail = lane.before->entries().back();
            if (old_tail.logical_token_begin == target.logical_token_begin
                && old_tail.handle != target.handle) {
                copies[n_copies++] = kk_kv_copy{old_tail.handle.slot, target.handle.slot,
                    old_tail.valid_tokens, static_cast<std::uint8_t>(old_tail.kind),
                    static_cast<std::uint8_t>(target.kind)};
            }
        }
        if (n_descs + entries.size() > im.max_descs) {
            result.success = false;
            result.detail = "step descriptor capacity exceeded";
            return result;
        }
        lanes[b] = kk_attn_lane{n_descs, static_cast<std::uint32_t>(entries.size()),
            lane.reserved->tokenCount(), 0, 0, b, 0, 0};
        for (MappingEntry const& e : entries) {
            descs[n_descs++] = kk_page_desc{e.handle.slot, e.logical_token_begin, e.valid_tokens,
                static_cast<std::uint8_t>(e.kind), 0, 0};
        }
    }
    // One token-balanced run per SM, none shorter than the cost of a first
    // stage and a combine (the TMA attention kernel serves every shape this
    // runner accepts).
    std::uint32_t const n_items = kk_attention_plan_balanced(descs, lanes, B,
        kk::attentionPlanParts(lanes, B, im.sm_count), im.stepHost<kk_attn_item>(im.off_items), im.max_items);
    if (n_items > im.max_items) {
        result.success = false;
        result.detail = "attention work list capacity exceeded";
        return result;
    }
    auto* counts = im.stepHost<std::uint32_t>(im.off_counts);
    counts[0] = n_items;
    counts[1] = n_copies;
    std::size_t const bytes = im.off_descs + std::size_t(n_descs) * sizeof(kk_page_desc);
    phase(1);
    cudaError_t e = cudaMemcpyAsync(im.step_dev, im.step_host, bytes, cudaMemcpyHostToDevice, im.stream);
    im.last_h2d = bytes;
    im.last_d2h = 0;
    CudaModelRunnerStatus s = e == cudaSuccess
        ? im.runStep(B, n_copies != 0, want_logits, debug)
        : cudaFailure(static_cast<int>(e), "upload step inputs");
    phase(2);
    if (s.ok()) {
        s = im.finishStep(B, logits_out, "decode step");
    }
    if (s.ok() && logits_out != nullptr) {
        // Rows of the step are its lanes; hand them back in item order
        // (rows of items that did not enter the step are zero).
        std::size_t const V = c.vocabulary_size;
        std::vector<float> rows = std::move(*logits_out);
        logits_out->assign(items.size() * V, 0.0f);
        for (std::uint32_t b = 0; b < B; ++b) {
            std::copy(rows.begin() + b * V, rows.begin() + (b + 1) * V, logits_out->begin() + lane_index[b] * V);
        }
    }
    if (!s.ok()) {
        im.last_error = s.detail;
    }
    if (s.ok()) {
        noteStreamCompleted(*im.kv, im.stream);
        cudaEventElapsedTime(&im.last_ms, im.ev_begin, im.ev_end);
    }
    phase(3);
    std::vector<std::pair<RequestId, std::uint32_t>> promote;
    for (std::uint32_t b = 0; b < B; ++b) {
        std::size_t const i = lane_index[b];
        if (!s.ok()) {
            result.steps[i] = {false, 0, s.detail};
            continue;  // rolled back by the transaction destructor
        }
        EngineKvStatus const committed = txns[b].commit();
        result.steps[i] = committed.ok()
            ? GenerationStepResult{true, im.host_tokens[b], {}}
            : GenerationStepResult{false, 0, kvFailure(committed, "commit batched model token").detail};
        std::uint32_t const length = items[i].expected_position + 1;
        if (committed.ok() && im.auto_promote && length % 64 == 0) {
            promote.emplace_back(items[i].request_id, length - 64);
        }
    }
    if (!promote.empty()) {
        // The last 8 micro pages of each lane just filled a 64-token run:
        // fold them into one extent page (skipped when they are shared).
        static_cast<void>(cudaBackendPromoteMany(*im.kv, promote, im.stream));
    }
    phase(4);
    return result;
}

ModelTokenResult CudaTinyLlamaModelRunner::forwardToken(RequestId request_id,
    std::uint32_t token_id, std::uint32_t expected_position, ModelRunnerDebugCapture* debug,
    ModelRunnerOutputOptions output)
{
    ModelTokenResult result;
    TinyLlamaConfig const& c = impl_->cfg;
    if (request_id == kInvalidRequestId || token_id >= c.vocabulary_size
        || expected_position >= c.max_position_embeddings) {
        result.status = failure(CudaModelRunnerError::InvalidArgument, 0,
            "request, token, or position is out of range");
        return result;
    }
    if (debug != nullptr) {
        std::unordered_set<std::uint32_t> seen;
        for (std::uint32_t l : debug->layer_indices) {
            if (l >= c.layer_count || !seen.insert(l).second) {
                result.status = failure(CudaModelRunnerError::InvalidArgument, 0,
                    "debug layer is duplicated or out of range");
                return result;
            }
        }
        debug->embedding.assign(c.hidden_size, 0);
        debug->final_hidden_state.assign(c.hidden_size, 0);
        debug->layer_hidden_states.assign(debug->layer_indices.size(),
            std::vector<KvScalar>(c.hidden_size, 0));
    }
    GenerationBatchResult batch;
    std::vector<GenerationBatchItem> items{GenerationBatchItem{request_id, token_id, expected_position}};
    // The single-token path shares the batched implementation.
    std::vector<float> logits;
    batch = runBatch(*impl_, items, output.copy_logits, debug, output.copy_logits ? &logits : nullptr);
    if (!batch.success || batch.steps.size() != 1) {
        result.status = failure(CudaModelRunnerError::ExecutionFailed, 0, batch.detail);
        return result;
    }
    if (!batch.steps[0].success) {
        result.status = failure(CudaModelRunnerError::KvBackendFailed, 0, batch.steps[0].detail);
        return result;
    }
    result.greedy_token_id = batch.steps[0].greedy_token_id;
    result.logits = std::move(logits);
    return result;
}

// One fused step over `n` consecutive prompt tokens of one request whose
// metadata was just appended (table `before` -> `after`).
GenerationStepResult prefillStep(CudaTinyLlamaModelRunner::Impl& im, RequestId id,
    std::uint32_t const* tokens_in, std::uint32_t n, std::uint32_t first, BlockTable const& before,
    BlockTable const& after)
{
    auto* tokens = im.stepHost<std::uint32_t>(im.off_tokens);
    auto* positions = im.stepHost<std::uint32_t>(im.off_positions);
    auto* slots = im.stepHost<kk_kv_slot>(im.off_slots);
    auto* copies = im.stepHost<kk_kv_copy>(im.off_copies);
    auto* lanes = im.stepHost<kk_attn_lane>(im.off_lanes);
    auto* descs = im.stepHost<kk_page_desc>(im.off_descs);
    auto const& entries = after.entries();
    std::uint32_t n_copies = 0;
    // Partial-tail copy-on-write: the old tail's tokens move to the new page
    // at the same logical begin before the new tokens land there.
    if (!before.entries().empty()) {
        MappingEntry const& old_tail = before.entries().back();
        for (MappingEntry const& e : entries) {
            if (e.logical_token_begin == old_tail.logical_token_begin && e.handle != old_tail.handle) {
                copies[n_copies++] = kk_kv_copy{old_tail.handle.slot, e.handle.slot, old_tail.valid_tokens,
                    static_cast<std::uint8_t>(old_tail.kind), static_cast<std::uint8_t>(e.kind)};
            }
        }
    }
    std::uint32_t n_descs = 0;
    for (std::uint32_t i = 0; i < n; ++i) {
        std::uint32_t const p = first + i;
        tokens[i] = tokens_in[i];
        positions[i] = p;
        std::uint32_t const lane_first = n_descs;
        bool placed = false;
        for (MappingEntry const& e : entries) {
            if (e.logical_token_begin > p) {
                break;
            }
            std::uint32_t const end = e.logical_token_begin + e.valid_tokens;
            if (p < end) {
                slots[i] = kk_kv_slot{e.handle.slot, static_cast<std::uint16_t>(p - e.logical_token_begin),
                    static_cast<std::uint8_t>(e.kind), 1};
                placed = true;
            }
            if (n_descs >= im.max_descs) {
                return {false, 0, "step descriptor capacity exceeded"};
            }
            // Causal: position p attends to tokens [0, p].
            std::uint32_t const valid = p < end ? p + 1 - e.logical_token_begin : e.valid_tokens;
            descs[n_descs++] = kk_page_desc{e.handle.slot, e.logical_token_begin,
                static_cast<std::uint16_t>(valid), static_cast<std::uint8_t>(e.kind), 0, 0};
        }
        if (!placed) {
            return {false, 0, "appended table does not cover the prompt position"};
        }
        lanes[i] = kk_attn_lane{lane_first, n_descs - lane_first, p + 1, 0, 0, i, 0, 0};
    }
    std::uint32_t const n_items = kk_attention_plan_balanced(descs, lanes, n,
        kk::attentionPlanParts(lanes, n, im.sm_count), im.stepHost<kk_attn_item>(im.off_items), im.max_items);
    if (n_items > im.max_items) {
        return {false, 0, "attention work list capacity exceeded"};
    }
    auto* counts = im.stepHost<std::uint32_t>(im.off_counts);
    counts[0] = n_items;
    counts[1] = n_copies;
    std::size_t const bytes = im.off_descs + std::size_t(n_descs) * sizeof(kk_page_desc);
    cudaError_t e = cudaMemcpyAsync(im.step_dev, im.step_host, bytes, cudaMemcpyHostToDevice, im.stream);
    im.last_h2d = bytes;
    im.last_d2h = 0;
    CudaModelRunnerStatus s = e == cudaSuccess ? im.runStep(n, n_copies != 0, false, nullptr)
                                               : cudaFailure(static_cast<int>(e), "upload step inputs");
    if (s.ok()) {
        s = im.finishStep(n, nullptr, "prefill step");
    }
    if (!s.ok()) {
        im.last_error = s.detail;
        return {false, 0, s.detail};
    }
    noteStreamCompleted(*im.kv, im.stream);
    cudaEventElapsedTime(&im.last_ms, im.ev_begin, im.ev_end);
    static_cast<void>(id);
    return {true, im.host_tokens[n - 1], {}};
}

GenerationStepResult CudaTinyLlamaModelRunner::prefill(RequestId request_id,
    std::vector<std::uint32_t> const& prompt, std::uint32_t first_position)
{
    GenerationStepResult r = prefillChunks(request_id, prompt.data(), static_cast<std::uint32_t>(prompt.size()),
        first_position, true);
    if (!r.success) {
        impl_->last_error = r.detail;
    }
    return r;
}

GenerationStepResult CudaTinyLlamaModelRunner::generationPrefill(RequestId request_id, std::uint32_t const* tokens,
    std::uint32_t count, std::uint32_t first_position)
{
    GenerationStepResult r = prefillChunks(request_id, tokens, count, first_position, false);
    if (!r.success) {
        impl_->last_error = r.detail;
    }
    return r;
}

GenerationStepResult CudaTinyLlamaModelRunner::prefillChunks(RequestId request_id,
    std::uint32_t const* prompt, std::uint32_t count, std::uint32_t first_position, bool release_on_failure)
{
    Impl& im = *impl_;
    TinyLlamaConfig const& c = im.cfg;
    if (request_id == kInvalidRequestId || prompt == nullptr || count == 0
        || std::uint64_t(first_position) + count > c.max_position_embeddings) {
        return {false, 0, "request, prompt, or position is out of range"};
    }
    for (std::uint32_t i = 0; i < count; ++i) {
        if (prompt[i] >= c.vocabulary_size) {
            return {false, 0, "token id is out of range"};
        }
    }
    GenerationStepResult last{false, 0, "empty prompt"};
    std::uint32_t const chunk = im.options.max_batch_size;
    std::vector<std::pair<RequestId, std::uint32_t>> promote;
    for (std::uint32_t done = 0; done < count; done += chunk) {
        std::uint32_t const n = std::min<std::uint32_t>(chunk, count - done);
        std::uint32_t const first = first_position + done;
        BlockTable before;
        if (!cudaBackendTable(*im.kv, request_id, before) || before.tokenCount() != first) {
            return {false, 0, "request not found or its committed length differs from the prompt position"};
        }
        EngineKvStatus const appended = cudaBackendAppend(*im.kv, request_id, n);
        if (!appended.ok()) {
            return {false, 0, kvFailure(appended, "append prompt tokens").detail};
        }
        BlockTable after;
        if (!cudaBackendTable(*im.kv, request_id, after)) {
            return {false, 0, "request vanished during prefill"};
        }
        last = prefillStep(im, request_id, prompt + done, n, first, before, after);
        if (!last.success) {
            // As the reference's append data path does after a device failure:
            // the request's pages cannot be trusted any more, release it (or
            // leave that to the owner, the scheduler, which releases it when
            // it ends the request).
            if (release_on_failure) {
                static_cast<void>(im.kv->releaseRequest(request_id));
            }
            return last;
        }
        if (im.auto_promote) {
            for (std::uint32_t end = (first / 64 + 1) * 64; end <= first + n; end += 64) {
                promote.emplace_back(request_id, end - 64);
            }
        }
    }
    if (!promote.empty()) {
        static_cast<void>(cudaBackendPromoteMany(*im.kv, promote, im.stream));
    }
    return last;
}

GenerationBatchResult CudaTinyLlamaModelRunner::generationForwardBatch(
    std::vector<GenerationBatchItem> const& batch)
{
    return runBatch(*impl_, batch, false, nullptr, nullptr);
}

GenerationBatchResult CudaTinyLlamaModelRunner::generationForwardBatchLogits(
    std::vector<GenerationBatchItem> const& batch, std::vector<float>& logits)
{
    return runBatch(*impl_, batch, true, nullptr, &logits);
}

GenerationStepResult CudaTinyLlamaModelRunner::generationForwardToken(RequestId request_id,
    std::uint32_t token_id, std::uint32_t expected_position)
{
    GenerationBatchResult r = runBatch(*impl_, {GenerationBatchItem{request_id, token_id, expected_position}},
        false, nullptr, nullptr);
    if (!r.success || r.steps.size() != 1) {
        return {false, 0, r.detail.empty() ? "single-token batch returned an invalid result" : r.detail};
    }
    return std::move(r.steps[0]);
}

// ---- construction ---------------------------------------------------------------------

CudaModelRunnerCreateResult createCudaTinyLlamaModelRunner(std::string const& manifest_path,
    std::string const& data_path, EngineKvBackend& kv_backend, EngineStream stream,
    CudaModelRunnerOptions options)
{
    CudaModelRunnerCreateResult out;
    if (!options.valid()) {
        out.status = failure(CudaModelRunnerError::InvalidArgument, 0, "invalid runner options");
        return out;
    }
    WeightManifestLoadResult loaded = loadWeightManifest(manifest_path);
    if (!loaded.ok()) {
        out.status = failure(CudaModelRunnerError::ManifestError, static_cast<int>(loaded.status.error),
            loaded.status.detail);
        return out;
    }
    if (options.verify_checksums) {
        WeightManifestStatus const data = validateWeightDataFile(loaded.manifest, data_path);
        if (!data.ok()) {
            out.status = failure(CudaModelRunnerError::DataFileError, static_cast<int>(data.error), data.detail);
            return out;
        }
    }
    TinyLlamaConfig const c = loaded.manifest.config;
    EngineKvConfig const kvc = kv_backend.config();
    if (kvc.kv_layout.layer_count != c.layer_count || kvc.kv_layout.kv_head_count != c.kv_head_count
        || kvc.kv_layout.head_dimension != c.head_dimension
        || kvc.query_head_count != c.attention_head_count) {
        out.status = failure(CudaModelRunnerError::InvalidArgument, 0,
            "KV backend layout does not match the model");
        return out;
    }
    kk_kv_pools const* pools = cudaBackendPools(kv_backend);
    if (pools == nullptr) {
        out.status = failure(CudaModelRunnerError::InvalidArgument, 0,
            "the fused decode step needs a CUDA KV backend of this library");
        return out;
    }
    std::uint32_t const group = c.attention_head_count / c.kv_head_count;
    if (c.head_dimension != 64 || (c.kv_head_count != 1 && c.kv_head_count != 2 && c.kv_head_count != 4)
        || group > 16 || c.hidden_size % 64 != 0 || c.intermediate_size % 8 != 0) {
        out.status = failure(CudaModelRunnerError::InvalidArgument, 0,
            "model shape outside the sm_100a kernels (head_dim 64, kv_heads 1/2/4, group <= 16)");
        return out;
    }
    auto im = std::make_unique<CudaTinyLlamaModelRunner::Impl>();
    im->cfg = c;
    im->manifest = loaded.manifest;
    im->kv = &kv_backend;
    im->stream = static_cast<cudaStream_t>(stream);
    im->options = options;
    im->auto_promote = options.auto_promote;
    im->pools = *pools;

    // Weights: one device allocation in the fused layout.
    std::uint64_t const H = c.hidden_size, I = c.intermediate_size, V = c.vocabulary_size;
    std::uint64_t const kvr = std::uint64_t(c.kv_head_count) * c.head_dimension;
    std::uint64_t const qkv_rows = H + 2 * kvr;
    auto pad = [](std::uint64_t n) { return (n + 63) & ~std::uint64_t(63); };  // 128-byte aligned tensors
    std::uint64_t const padded = 2 * pad(V * H) + pad(H)
        + c.layer_count * (2 * pad(H) + pad(qkv_rows * H) + pad(H * H) + pad(2 * I * H) + pad(H * I));
    im->weight_bytes = padded * 2;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&im->weights), im->weight_bytes);
    if (e != cudaSuccess) {
        out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e), "weight allocation");
        return out;
    }
    std::uint16_t* w16 = reinterpret_cast<std::uint16_t*>(im->weights);
    std::uint64_t cursor = 0;
    auto take = [&](std::uint64_t elems) {
        std::uint16_t* p = w16 + cursor;
        cursor += pad(elems);
        return p;
    };
    std::uint16_t* embed = take(V * H);
    std::uint16_t* lm = take(V * H);
    std::uint16_t* fnorm = take(H);
    im->embed = embed;
    im->lm_head = lm;
    im->final_norm = fnorm;
    struct Dest {
        std::uint16_t* base;
        std::uint64_t row_pitch;  // destination row pitch (elements); 0 = contiguous
        std::uint64_t rows;
    };
    std::unordered_map<std::string, Dest> dest;
    dest["model.embed_tokens.weight"] = {embed, 0, 0};
    dest["lm_head.weight"] = {lm, 0, 0};
    dest["model.norm.weight"] = {fnorm, 0, 0};
    for (std::uint32_t l = 0; l < c.layer_count; ++l) {
        std::string const p = "model.layers." + std::to_string(l) + ".";
        LayerWeights lw{};
        std::uint16_t* in_norm = take(H);
        std::uint16_t* post_norm = take(H);
        std::uint16_t* qkv = take(qkv_rows * H);
        std::uint16_t* o = take(H * H);
        std::uint16_t* gu = take(2 * I * H);
        std::uint16_t* down = take(H * I);
        lw = LayerWeights{in_norm, post_norm, qkv, o, gu, down};
        im->layers.push_back(lw);
        dest[p + "input_layernorm.weight"] = {in_norm, 0, 0};
        dest[p + "post_attention_layernorm.weight"] = {post_norm, 0, 0};
        dest[p + "self_attn.q_proj.weight"] = {qkv, 0, 0};
        dest[p + "self_attn.k_proj.weight"] = {qkv + H * H, 0, 0};
        dest[p + "self_attn.v_proj.weight"] = {qkv + (H + kvr) * H, 0, 0};
        dest[p + "self_attn.o_proj.weight"] = {o, 0, 0};
        dest[p + "mlp.gate_proj.weight"] = {gu, 2 * H, I};      // rows 0, 2, 4, ...
        dest[p + "mlp.up_proj.weight"] = {gu + H, 2 * H, I};    // rows 1, 3, 5, ...
        dest[p + "mlp.down_proj.weight"] = {down, 0, 0};
    }
    {
        std::ifstream in(data_path, std::ios::binary);
        if (!in) {
            out.status = failure(CudaModelRunnerError::DataFileError, 0, "cannot open " + data_path);
            return out;
        }
        std::vector<char> staging;
        for (WeightTensorDescriptor const& t : im->manifest.tensors) {
            auto const d = dest.find(t.name);
            if (d == dest.end()) {
                continue;
            }
            staging.resize(t.byte_size);
            in.seekg(static_cast<std::streamoff>(t.offset));
            in.read(staging.data(), static_cast<std::streamsize>(t.byte_size));
            if (in.gcount() != static_cast<std::streamsize>(t.byte_size)) {
                out.status = failure(CudaModelRunnerError::DataFileError, 0, "short read: " + t.name);
                return out;
            }
            if (d->second.row_pitch == 0) {
                e = cudaMemcpy(d->second.base, staging.data(), t.byte_size, cudaMemcpyHostToDevice);
            } else {
                std::uint64_t const width = t.byte_size / d->second.rows;
                e = cudaMemcpy2D(d->second.base, d->second.row_pitch * 2, staging.data(), width, width,
                    d->second.rows, cudaMemcpyHostToDevice);
            }
            if (e != cudaSuccess) {
                out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e),
                    "weight upload: " + t.name);
                return out;
            }
        }
    }

    // Pack the projection matrices into 16 KB swizzled tiles (one allocation),
    // move the embedding table and norm weights into a compact row-major
    // allocation, and release the upload buffer.
    {
        // Projection matrices are packed as they are; the RMSNorm weight that
        // precedes a projection is applied by the GEMM when it normalises its
        // input rows (qkv: input norm, gate/up: post-attention norm, LM head:
        // final norm).
        struct PackJob {
            std::uint16_t const* src;
            std::uint32_t M, K;
            std::uint16_t const** dst;
            std::uint16_t const* col_scale;
        };
        std::vector<PackJob> jobs;
        jobs.push_back({im->lm_head, static_cast<std::uint32_t>(V), static_cast<std::uint32_t>(H), &im->lm_head,
            nullptr});
        for (LayerWeights& lw : im->layers) {
            jobs.push_back({lw.w_qkv, static_cast<std::uint32_t>(qkv_rows), static_cast<std::uint32_t>(H), &lw.w_qkv,
                nullptr});
            jobs.push_back({lw.w_o, static_cast<std::uint32_t>(H), static_cast<std::uint32_t>(H), &lw.w_o, nullptr});
            jobs.push_back({lw.w_gu, static_cast<std::uint32_t>(2 * I), static_cast<std::uint32_t>(H), &lw.w_gu,
                nullptr});
            jobs.push_back({lw.w_down, static_cast<std::uint32_t>(H), static_cast<std::uint32_t>(I), &lw.w_down,
                nullptr});
        }
        std::uint64_t packed_bytes = 0;
        for (PackJob const& j : jobs) {
            packed_bytes += kk_gemm_packed_bytes(j.M, j.K);
        }
        std::uint64_t const small_elems = pad(V * H) + pad(H) + 2 * c.layer_count * pad(H);
        std::uint8_t* small = nullptr;
        e = cudaMalloc(reinterpret_cast<void**>(&im->packed), packed_bytes);
        if (e == cudaSuccess) {
            e = cudaMalloc(reinterpret_cast<void**>(&small), small_elems * 2);
        }
        if (e != cudaSuccess) {
            cudaFree(small);
            out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e), "packed weight allocation");
            return out;
        }
        std::uint64_t at = 0;
        for (PackJob const& j : jobs) {
            std::uint16_t* dst = reinterpret_cast<std::uint16_t*>(im->packed + at);
            int const rc = kk_gemm_pack_weight_scaled(j.src, j.M, j.K, j.col_scale, dst, nullptr);
            if (rc != 0) {
                cudaFree(small);
                out.status = failure(CudaModelRunnerError::AllocationFailed, rc, "weight packing");
                return out;
            }
            *j.dst = dst;
            at += kk_gemm_packed_bytes(j.M, j.K);
        }
        std::uint16_t* s16 = reinterpret_cast<std::uint16_t*>(small);
        std::uint64_t scur = 0;
        auto move = [&](std::uint16_t const* src, std::uint64_t elems) {
            std::uint16_t* d = s16 + scur;
            scur += pad(elems);
            cudaMemcpy(d, src, elems * 2, cudaMemcpyDeviceToDevice);
            return d;
        };
        im->embed = move(im->embed, V * H);
        im->final_norm = move(im->final_norm, H);
        for (LayerWeights& lw : im->layers) {
            lw.in_norm = move(lw.in_norm, H);
            lw.post_norm = move(lw.post_norm, H);
        }
        e = cudaDeviceSynchronize();
        cudaFree(im->weights);
        im->weights = small;
        im->weight_bytes = packed_bytes + small_elems * 2;
        if (e != cudaSuccess) {
            out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e), "weight packing");
            return out;
        }
    }

    // Workspace.
    std::uint32_t const bmax = options.max_batch_size;
    im->bpad = std::max<std::uint32_t>(64, (bmax + 15) / 16 * 16);
    std::uint32_t const positions_cap = c.max_position_embeddings + 8;
    im->max_descs = bmax * (positions_cap / 8 + 2);
    {
        int dev = 0;
        int sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        im->sm_count = sms > 0 ? static_cast<std::uint32_t>(sms) : 148u;
    }
    im->max_items = im->sm_count + bmax + 8;
    std::size_t off = 0;
    auto region = [&](std::size_t bytes) {
        std::size_t const at = off;
        off = align256(off + bytes);
        return at;
    };
    std::size_t const o_hidden = region(std::size_t(im->bpad) * H * 2);
    std::size_t const o_normed = region(std::size_t(im->bpad) * H * 2);
    std::size_t const o_q = region(std::size_t(im->bpad) * H * 2);
    std::size_t const o_attn = region(std::size_t(im->bpad) * H * 2);
    std::size_t const o_act = region(std::size_t(im->bpad) * I * 2);
    std::size_t const o_logits = region(std::size_t(bmax) * V * 4);
    im->attn_ws_bytes = kk_attention_workspace_bytes(bmax, im->max_items, c.attention_head_count,
        c.head_dimension);
    std::size_t const o_attn_ws = region(im->attn_ws_bytes);
    std::size_t const o_argmax = region(kk_argmax_workspace_bytes(c.vocabulary_size, bmax));
    std::size_t const o_rope = region(std::size_t(c.max_position_embeddings) * (c.head_dimension / 2) * 8);
    std::size_t const sq_bytes = std::size_t((H + 127) / 128) * 64 * 4;
    std::size_t const o_sq_embed = region(sq_bytes);
    std::size_t const o_sq_attn = region(sq_bytes);
    std::size_t const o_sq_mlp = region(sq_bytes);
    im->ws_bytes = off;
    e = cudaMalloc(reinterpret_cast<void**>(&im->ws), im->ws_bytes);
    if (e == cudaSuccess) {
        e = cudaMemset(im->ws, 0, im->ws_bytes);
    }
    if (e != cudaSuccess) {
        out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e), "workspace");
        return out;
    }
    im->hidden = reinterpret_cast<std::uint16_t*>(im->ws + o_hidden);
    im->normed = reinterpret_cast<std::uint16_t*>(im->ws + o_normed);
    im->q = reinterpret_cast<std::uint16_t*>(im->ws + o_q);
    im->attn = reinterpret_cast<std::uint16_t*>(im->ws + o_attn);
    im->act = reinterpret_cast<std::uint16_t*>(im->ws + o_act);
    im->logits = reinterpret_cast<float*>(im->ws + o_logits);
    im->attn_ws = im->ws + o_attn_ws;
    im->argmax_ws = im->ws + o_argmax;
    im->sq_embed = reinterpret_cast<float*>(im->ws + o_sq_embed);
    im->sq_attn_out = reinterpret_cast<float*>(im->ws + o_sq_attn);
    im->sq_mlp_out = reinterpret_cast<float*>(im->ws + o_sq_mlp);
    im->rope_cs = reinterpret_cast<float*>(im->ws + o_rope);
    {
        // angle = position * theta^(-2d / head_dim), as the reference's model
        // computes it (float arithmetic, host libm), pairs (cos, sin).
        std::uint32_t const half = c.head_dimension / 2;
        std::vector<float> table(std::size_t(c.max_position_embeddings) * half * 2);
        for (std::uint32_t d = 0; d < half; ++d) {
            float const inv = ::powf(c.rope_theta, -2.0f * static_cast<float>(d) / static_cast<float>(c.head_dimension));
            for (std::uint32_t p = 0; p < c.max_position_embeddings; ++p) {
                float const angle = static_cast<float>(p) * inv;
                table[(std::size_t(p) * half + d) * 2] = ::cosf(angle);
                table[(std::size_t(p) * half + d) * 2 + 1] = ::sinf(angle);
            }
        }
        e = cudaMemcpy(im->rope_cs, table.data(), table.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e), "RoPE table");
            return out;
        }
    }

    off = 0;
    im->off_counts = region(16);
    im->off_result = region(CudaTinyLlamaModelRunner::Impl::kResultHeader + std::size_t(bmax) * 4);
    im->off_tokens = region(std::size_t(bmax) * 4);
    im->off_positions = region(std::size_t(bmax) * 4);
    im->off_slots = region(std::size_t(bmax) * sizeof(kk_kv_slot));
    im->off_copies = region(std::size_t(bmax) * sizeof(kk_kv_copy));
    im->off_lanes = region(std::size_t(bmax) * sizeof(kk_attn_lane));
    im->off_items = region(std::size_t(im->max_items) * sizeof(kk_attn_item));
    im->off_descs = region(std::size_t(im->max_descs) * sizeof(kk_page_desc));
    im->step_bytes = off;
    e = cudaMalloc(reinterpret_cast<void**>(&im->step_dev), im->step_bytes);
    if (e == cudaSuccess) {
        e = cudaMallocHost(reinterpret_cast<void**>(&im->step_host), im->step_bytes);
    }
    if (e == cudaSuccess) {
        e = cudaMallocHost(reinterpret_cast<void**>(&im->host_result),
            CudaTinyLlamaModelRunner::Impl::kResultHeader + std::size_t(bmax) * 4);
    }
    if (e == cudaSuccess) {
        im->status_dev = reinterpret_cast<unsigned int*>(im->step_dev + im->off_result);
        im->out_tokens = reinterpret_cast<std::uint32_t*>(im->step_dev + im->off_result + CudaTinyLlamaModelRunner::Impl::kResultHeader);
        im->host_tokens = reinterpret_cast<std::uint32_t const*>(im->host_result + CudaTinyLlamaModelRunner::Impl::kResultHeader);
    }
    if (e == cudaSuccess) {
        e = cudaStreamCreateWithFlags(&im->capture_stream, cudaStreamNonBlocking);
    }
    if (e == cudaSuccess) {
        e = cudaEventCreate(&im->ev_begin);
    }
    if (e == cudaSuccess) {
        e = cudaEventCreate(&im->ev_end);
    }
    if (e == cudaSuccess) {
        std::memset(im->step_host, 0, im->step_bytes);
        e = cudaDeviceSynchronize();
    }
    if (e != cudaSuccess) {
        out.status = failure(CudaModelRunnerError::AllocationFailed, static_cast<int>(e), "step buffers");
        return out;
    }
    out.runner.reset(new CudaTinyLlamaModelRunner(std::move(im)));
    return out;
}

} // namespace kimkvcache

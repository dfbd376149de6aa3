// Single-request greedy generation loop (reference semantics:
// src/engine/generation.cpp:27-343): validate, create the KV request, prefill
// one position per model call, then decode until EOS / max_new_tokens /
// cancellation / stop; the KV request is always released at the end.
#include "generation.h"

#include <chrono>
#include <limits>
#include <new>

namespace kimkvcache {
namespace {

using Clock = std::chrono::steady_clock;

std::uint64_t nanosBetween(Clock::time_point a, Clock::time_point b) noexcept
{
    auto const d = std::chrono::duration_cast<std::chrono::nanoseconds>(b - a).count();
    return d > 0 ? static_cast<std::uint64_t>(d) : 0;
}

} // namespace

std::string_view toString(GenerationError e) noexcept
{
    static constexpr std::string_view n[] = {"none", "invalid_argument", "runtime_stopped",
        "model_failed", "kv_backend_failed", "internal_error"};
    auto const i = static_cast<std::size_t>(e);
    return i < 6 ? n[i] : "unknown";
}

std::string_view toString(GenerationTerminalReason r) noexcept
{
    static constexpr std::string_view n[] = {"eos_token", "max_new_tokens", "cancelled",
        "runtime_stopped", "failed"};
    auto const i = static_cast<std::size_t>(r);
    return i < 5 ? n[i] : "unknown";
}

GenerationBatchResult GenerationModelRunner::generationForwardBatch(
    std::vector<GenerationBatchItem> const& batch)
{
    GenerationBatchResult result;
    if (batch.empty()) {
        result.detail = "generation batch must not be empty";
        return result;
    }
    try {
        result.steps.reserve(batch.size());
        for (GenerationBatchItem const& item : batch) {
            result.steps.push_back(
                generationForwardToken(item.request_id, item.token_id, item.expected_position));
        }
    } catch (std::bad_alloc const&) {
        result.steps.clear();
        result.detail = "generation batch result allocation failed";
        return result;
    }
    result.success = true;
    return result;
}

std::uint32_t GenerationModelRunner::generationMaxBatchSize() const noexcept
{
    return std::numeric_limits<std::uint32_t>::max();
}

GenerationTerminal SingleRequestGenerationRuntime::generate(GenerationRequest const& request)
{
    Clock::time_point const started = Clock::now();
    GenerationTerminal terminal;
    terminal.request_id = request.request_id;
    bool idle = false;
    if (!generating_.compare_exchange_strong(idle, true, std::memory_order_acq_rel)) {
        terminal.error = GenerationError::InvalidArgument;
        terminal.detail = "single-request runtime is already generating";
        terminal.metrics.e2e_ns = nanosBetween(started, Clock::now());
        return terminal;
    }
    struct Guard {
        std::atomic<bool>& flag;
        ~Guard() { flag.store(false, std::memory_order_release); }
    } guard{generating_};

    TinyLlamaConfig const config = runner_->generationConfig();
    bool created = false;
    bool emitted = false;
    Clock::time_point first_token{};
    Clock::time_point last_token{};
    auto cancelled = [&] { return request.cancellation && request.cancellation->cancelled(); };
    auto finish = [&](GenerationTerminalReason reason, GenerationError error, std::string detail) {
        terminal.reason = reason;
        terminal.error = error;
        terminal.detail = std::move(detail);
        terminal.usage.completion_tokens = static_cast<std::uint32_t>(terminal.output_token_ids.size());
        terminal.usage.total_tokens = terminal.usage.prompt_tokens + terminal.usage.completion_tokens;
        if (created) {
            EngineKvStatus const released = kv_->releaseRequest(request.request_id);
            created = false;
            if (!released.ok()) {
                terminal.reason = GenerationTerminalReason::Failed;
                terminal.error = GenerationError::KvBackendFailed;
                terminal.detail = "release request failed: ";
                terminal.detail += toString(released.error);
            }
        }
        Clock::time_point const done = Clock::now();
        terminal.metrics.e2e_ns = nanosBetween(started, done);
        if (emitted) {
            terminal.metrics.ttft_ns = nanosBetween(started, first_token);
            if (terminal.output_token_ids.size() > 1) {
                terminal.metrics.tpot_ns = nanosBetween(first_token, last_token)
                    / (terminal.output_token_ids.size() - 1);
            }
        }
        return terminal;
    };

    if (stopped()) {
        return finish(GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
            "runtime is stopped");
    }
    if (!config.valid() || request.request_id == kInvalidRequestId
        || request.prompt_token_ids.empty() || request.sampling.max_new_tokens == 0) {
        return finish(GenerationTerminalReason::Failed, GenerationError::InvalidArgument,
            "request id, prompt, model config, and max_new_tokens are required");
    }
    terminal.usage.prompt_tokens = static_cast<std::uint32_t>(request.prompt_token_ids.size());
    if (request.prompt_token_ids.size() > config.max_position_embeddings
        || request.sampling.max_new_tokens
            > config.max_position_embeddings - request.prompt_token_ids.size() + 1) {
        return finish(GenerationTerminalReason::Failed, GenerationError::InvalidArgument,
            "prompt and completion exceed the model position limit");
    }
    std::uint32_t const eos = request.sampling.eos_token_id.value_or(config.eos_token_id);
    if (eos >= config.vocabulary_size) {
        return finish(GenerationTerminalReason::Failed, GenerationError::InvalidArgument,
            "EOS token is outside the model vocabulary");
    }
    for (std::uint32_t t : request.prompt_token_ids) {
        if (t >= config.vocabulary_size) {
            return finish(GenerationTerminalReason::Failed, GenerationError::InvalidArgument,
                "prompt token is outside the model vocabulary");
        }
    }
    if (cancelled()) {
        return finish(GenerationTerminalReason::Cancelled, GenerationError::None,
            "request cancelled before prefill");
    }
    EngineKvStatus const made = kv_->createRequest(request.request_id);
    if (!made.ok()) {
        return finish(GenerationTerminalReason::Failed, GenerationError::KvBackendFailed,
            std::string("create request failed: ") + std::string(toString(made.error)));
    }
    created = true;

    auto step = [&](std::uint32_t token, std::uint32_t position, std::uint32_t& next) -> bool {
        GenerationStepResult s = runner_->generationForwardToken(request.request_id, token, position);
        if (!s.success) {
            finish(GenerationTerminalReason::Failed, GenerationError::ModelFailed, std::move(s.detail));
            return false;
        }
        if (s.greedy_token_id >= config.vocabulary_size) {
            finish(GenerationTerminalReason::Failed, GenerationError::ModelFailed,
                "model returned a token outside the vocabulary");
            return false;
        }
        next = s.greedy_token_id;
        return true;
    };

    std::uint32_t next = 0;
    for (std::size_t pos = 0; pos < request.prompt_token_ids.size(); ++pos) {
        if (stopped()) {
            return finish(GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
                "runtime stopped during prefill");
        }
        if (cancelled()) {
            return finish(GenerationTerminalReason::Cancelled, GenerationError::None,
                "request cancelled during prefill");
        }
        if (!step(request.prompt_token_ids[pos], static_cast<std::uint32_t>(pos), next)) {
            return terminal;
        }
    }
    for (std::uint32_t generated = 0; generated < request.sampling.max_new_tokens; ++generated) {
        if (stopped()) {
            return finish(GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
                "runtime stopped during decode");
        }
        if (cancelled()) {
            return finish(GenerationTerminalReason::Cancelled, GenerationError::None,
                "request cancelled during decode");
        }
        try {
            terminal.output_token_ids.push_back(next);
        } catch (std::bad_alloc const&) {
            return finish(GenerationTerminalReason::Failed, GenerationError::InternalError,
                "completion token allocation failed");
        }
        last_token = Clock::now();
        if (!emitted) {
            first_token = last_token;
            emitted = true;
        }
        if (next == eos) {
            return finish(GenerationTerminalReason::EosToken, GenerationError::None, "EOS token generated");
        }
        if (generated + 1 == request.sampling.max_new_tokens) {
            return finish(GenerationTerminalReason::MaxNewTokens, GenerationError::None,
                "max_new_tokens reached");
        }
        if (!step(next, terminal.usage.prompt_tokens + generated, next)) {
            return terminal;
        }
    }
    return finish(GenerationTerminalReason::Failed, GenerationError::InternalError,
        "generation loop exited without a terminal reason");
}

} // namespace kimkvcache

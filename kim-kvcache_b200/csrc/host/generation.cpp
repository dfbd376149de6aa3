// Single-request greedy generation and the default model SPI behaviour.
// Reference semantics: src/engine/generation.cpp (validation, terminal
// reasons and errors, release of the KV request on every exit, TTFT/TPOT).
//
// generate() walks the request's positions once: positions below the prompt
// length feed prompt tokens, the ones after feed back the previous greedy
// token, which is emitted first. Before every position the run may end
// (stop, cancellation, EOS, max_new_tokens); close() turns any ending into
// the terminal and releases the KV request.
#include "generation.h"

#include <chrono>
#include <limits>
#include <new>
#include <optional>

namespace kimkvcache {
namespace {

using Clock = std::chrono::steady_clock;

std::uint64_t elapsedNs(Clock::time_point from, Clock::time_point to) noexcept
{
    auto const ns = std::chrono::duration_cast<std::chrono::nanoseconds>(to - from).count();
    return ns > 0 ? static_cast<std::uint64_t>(ns) : 0;
}

struct Ending {
    GenerationTerminalReason reason;
    GenerationError error;
    std::string detail;
};

Ending failure(GenerationError e, std::string detail)
{
    return Ending{GenerationTerminalReason::Failed, e, std::move(detail)};
}

// Why a request cannot run on this model, if it cannot.
std::optional<std::string> rejectReason(GenerationRequest const& r, TinyLlamaConfig const& m)
{
    std::size_t const prompt = r.prompt_token_ids.size();
    std::uint32_t const max_new = r.sampling.max_new_tokens;
    if (!m.valid() || r.request_id == kInvalidRequestId || prompt == 0 || max_new == 0) {
        return std::string("a request needs an id, a prompt, max_new_tokens and a valid model");
    }
    if (prompt > m.max_position_embeddings || max_new > m.max_position_embeddings - prompt + 1) {
        return std::string("prompt plus completion is longer than the model's positions");
    }
    if (r.sampling.eos_token_id.value_or(m.eos_token_id) >= m.vocabulary_size) {
        return std::string("EOS token id is outside the vocabulary");
    }
    for (std::uint32_t t : r.prompt_token_ids) {
        if (t >= m.vocabulary_size) {
            return std::string("a prompt token id is outside the vocabulary");
        }
    }
    return std::nullopt;
}

} // namespace

std::string_view toString(GenerationError e) noexcept
{
    switch (e) {
    case GenerationError::None: return "none";
    case GenerationError::InvalidArgument: return "invalid_argument";
    case GenerationError::RuntimeStopped: return "runtime_stopped";
    case GenerationError::ModelFailed: return "model_failed";
    case GenerationError::KvBackendFailed: return "kv_backend_failed";
    case GenerationError::InternalError: return "internal_error";
    }
    return "unknown";
}

std::string_view toString(GenerationTerminalReason r) noexcept
{
    switch (r) {
    case GenerationTerminalReason::EosToken: return "eos_token";
    case GenerationTerminalReason::MaxNewTokens: return "max_new_tokens";
    case GenerationTerminalReason::Cancelled: return "cancelled";
    case GenerationTerminalReason::RuntimeStopped: return "runtime_stopped";
    case GenerationTerminalReason::Failed: return "failed";
    }
    return "unknown";
}

// ---- default model SPI -------------------------------------------------------------------------

GenerationBatchResult GenerationModelRunner::generationForwardBatch(std::vector<GenerationBatchItem> const& batch)
{
    GenerationBatchResult out;
    if (batch.empty()) {
        out.detail = "an empty generation batch";
        return out;
    }
    try {
        out.steps.resize(batch.size());
    } catch (std::bad_alloc const&) {
        out.detail = "no memory for the batch result";
        return out;
    }
    for (std::size_t i = 0; i < batch.size(); ++i) {
        out.steps[i] = generationForwardToken(batch[i].request_id, batch[i].token_id, batch[i].expected_position);
    }
    out.success = true;
    return out;
}

std::uint32_t GenerationModelRunner::generationMaxBatchSize() const noexcept
{
    return std::numeric_limits<std::uint32_t>::max();
}

GenerationStepResult GenerationModelRunner::generationPrefill(RequestId, std::uint32_t const*, std::uint32_t,
    std::uint32_t)
{
    return GenerationStepResult{false, 0, "this model runner has no fused prefill"};
}

// ---- single-request runtime ---------------------------------------------------------------------

GenerationTerminal SingleRequestGenerationRuntime::generate(GenerationRequest const& request)
{
    Clock::time_point const t0 = Clock::now();
    GenerationTerminal out;
    out.request_id = request.request_id;
    bool expected_idle = false;
    if (!generating_.compare_exchange_strong(expected_idle, true, std::memory_order_acq_rel)) {
        out.error = GenerationError::InvalidArgument;
        out.detail = "another generation is running on this runtime";
        out.metrics.e2e_ns = elapsedNs(t0, Clock::now());
        return out;
    }
    struct Idle {
        std::atomic<bool>& busy;
        ~Idle() { busy.store(false, std::memory_order_release); }
    } const idle_on_exit{generating_};

    TinyLlamaConfig const model = runner_->generationConfig();
    bool kv_open = false;
    std::optional<Clock::time_point> first_emit;
    Clock::time_point last_emit{};
    auto close = [&](Ending e) -> GenerationTerminal {
        out.reason = e.reason;
        out.error = e.error;
        out.detail = std::move(e.detail);
        out.usage.completion_tokens = static_cast<std::uint32_t>(out.output_token_ids.size());
        out.usage.total_tokens = out.usage.prompt_tokens + out.usage.completion_tokens;
        if (kv_open) {
            kv_open = false;
            EngineKvStatus const released = kv_->releaseRequest(request.request_id);
            if (!released.ok()) {
                out.reason = GenerationTerminalReason::Failed;
                out.error = GenerationError::KvBackendFailed;
                out.detail = std::string("the KV request could not be released: ") + std::string(toString(released.error));
            }
        }
        out.metrics.e2e_ns = elapsedNs(t0, Clock::now());
        if (first_emit) {
            out.metrics.ttft_ns = elapsedNs(t0, *first_emit);
            std::size_t const n = out.output_token_ids.size();
            out.metrics.tpot_ns = n > 1 ? elapsedNs(*first_emit, last_emit) / (n - 1) : 0;
        }
        return out;
    };
    auto cancelled = [&] { return request.cancellation != nullptr && request.cancellation->cancelled(); };
    // Stop wins over cancellation at every boundary.
    auto interruption = [&](char const* where) -> std::optional<Ending> {
        if (stopped()) {
            return Ending{GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
                std::string("runtime stopped ") + where};
        }
        if (cancelled()) {
            return Ending{GenerationTerminalReason::Cancelled, GenerationError::None,
                std::string("request cancelled ") + where};
        }
        return std::nullopt;
    };

    if (stopped()) {
        return close(Ending{GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
            "runtime is stopped"});
    }
    std::size_t const prompt = request.prompt_token_ids.size();
    bool const shaped = model.valid() && request.request_id != kInvalidRequestId && prompt != 0
        && request.sampling.max_new_tokens != 0;
    if (shaped) {
        out.usage.prompt_tokens = static_cast<std::uint32_t>(prompt);
    }
    if (std::optional<std::string> why = rejectReason(request, model)) {
        return close(failure(GenerationError::InvalidArgument, std::move(*why)));
    }
    if (cancelled()) {
        return close(Ending{GenerationTerminalReason::Cancelled, GenerationError::None,
            "request cancelled before its prompt"});
    }
    EngineKvStatus const created = kv_->createRequest(request.request_id);
    if (!created.ok()) {
        return close(failure(GenerationError::KvBackendFailed,
            std::string("the KV request could not be created: ") + std::string(toString(created.error))));
    }
    kv_open = true;

    std::uint32_t const eos = request.sampling.eos_token_id.value_or(model.eos_token_id);
    std::uint32_t next = 0;
    for (std::size_t pos = 0;; ++pos) {
        bool const decoding = pos >= prompt;
        if (std::optional<Ending> e = interruption(decoding ? "during decode" : "during the prompt")) {
            return close(std::move(*e));
        }
        if (decoding) {
            try {
                out.output_token_ids.push_back(next);
            } catch (std::bad_alloc const&) {
                return close(failure(GenerationError::InternalError, "no memory for the completion"));
            }
            last_emit = Clock::now();
            first_emit = first_emit.value_or(last_emit);
            if (next == eos) {
                return close(Ending{GenerationTerminalReason::EosToken, GenerationError::None, "EOS generated"});
            }
            if (out.output_token_ids.size() == request.sampling.max_new_tokens) {
                return close(Ending{GenerationTerminalReason::MaxNewTokens, GenerationError::None,
                    "max_new_tokens generated"});
            }
        }
        std::uint32_t const token = decoding ? next : request.prompt_token_ids[pos];
        GenerationStepResult step = runner_->generationForwardToken(request.request_id, token,
            static_cast<std::uint32_t>(pos));
        if (!step.success) {
            return close(failure(GenerationError::ModelFailed, std::move(step.detail)));
        }
        if (step.greedy_token_id >= model.vocabulary_size) {
            return close(failure(GenerationError::ModelFailed, "the model returned a token outside the vocabulary"));
        }
        next = step.greedy_token_id;
    }
}

} // namespace kimkvcache

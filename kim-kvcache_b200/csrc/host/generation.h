// Greedy generation SPI and the single-request generation loop.
// Types and semantics follow the reference (include/kim-kv/engine/generation.h
// :14-202, src/engine/generation.cpp:27-343).
#pragma once

#include "engine_kv.h"
#include "weight_manifest.h"

#include <atomic>
#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

namespace kimkvcache {

enum class GenerationError : std::uint8_t {
    None,
    InvalidArgument,
    RuntimeStopped,
    ModelFailed,
    KvBackendFailed,
    InternalError,
};

enum class GenerationTerminalReason : std::uint8_t {
    EosToken,
    MaxNewTokens,
    Cancelled,
    RuntimeStopped,
    Failed,
};

struct SamplingConfig final {
    std::uint32_t max_new_tokens{0};
    std::optional<std::uint32_t> eos_token_id{};  // nullopt: the model's EOS
};

class GenerationCancellationToken final {
public:
    void cancel() noexcept { cancelled_.store(true, std::memory_order_release); }
    [[nodiscard]] bool cancelled() const noexcept { return cancelled_.load(std::memory_order_acquire); }

private:
    std::atomic<bool> cancelled_{false};
};

struct GenerationRequest final {
    RequestId request_id{kInvalidRequestId};
    std::vector<std::uint32_t> prompt_token_ids{};
    SamplingConfig sampling{};
    std::shared_ptr<GenerationCancellationToken> cancellation{};
    // Extension (no counterpart in the reference): the first
    // kv_prefix_tokens prompt positions are already committed under
    // request_id in the KV backend, e.g. a prefix shared by forking another
    // request. The scheduler then neither creates the KV request nor feeds
    // those positions; it must be below the prompt length. 0: none.
    std::uint32_t kv_prefix_tokens{0};
};

struct GenerationUsage final {
    std::uint32_t prompt_tokens{0};
    std::uint32_t completion_tokens{0};
    std::uint32_t total_tokens{0};
};

struct GenerationMetrics final {
    std::uint64_t ttft_ns{0};
    std::uint64_t tpot_ns{0};
    std::uint64_t e2e_ns{0};
};

struct GenerationTerminal final {
    RequestId request_id{kInvalidRequestId};
    GenerationTerminalReason reason{GenerationTerminalReason::Failed};
    GenerationError error{GenerationError::InternalError};
    std::string detail{};
    std::vector<std::uint32_t> output_token_ids{};
    GenerationUsage usage{};
    GenerationMetrics metrics{};

    [[nodiscard]] bool ok() const noexcept
    {
        return error == GenerationError::None
            && (reason == GenerationTerminalReason::EosToken
                || reason == GenerationTerminalReason::MaxNewTokens);
    }
};

struct GenerationStepResult final {
    bool success{false};
    std::uint32_t greedy_token_id{0};
    std::string detail{};
};

struct GenerationBatchItem final {
    RequestId request_id{kInvalidRequestId};
    std::uint32_t token_id{0};
    std::uint32_t expected_position{0};
};

struct GenerationBatchResult final {
    bool success{false};
    std::vector<GenerationStepResult> steps{};
    std::string detail{};
};

// Model SPI of the generation loops: greedy next token only.
class GenerationModelRunner {
public:
    virtual ~GenerationModelRunner() = default;
    GenerationModelRunner(GenerationModelRunner const&) = delete;
    GenerationModelRunner& operator=(GenerationModelRunner const&) = delete;

    [[nodiscard]] virtual TinyLlamaConfig generationConfig() const noexcept = 0;
    [[nodiscard]] virtual GenerationStepResult generationForwardToken(
        RequestId request_id, std::uint32_t token_id, std::uint32_t expected_position) = 0;
    // Independent sequence positions as one model batch; default: one by one.
    [[nodiscard]] virtual GenerationBatchResult generationForwardBatch(
        std::vector<GenerationBatchItem> const& batch);
    [[nodiscard]] virtual std::uint32_t generationMaxBatchSize() const noexcept;
    // Extension (no counterpart in the reference, which feeds a prompt one
    // position per model batch): consecutive prompt positions
    // [first_position, first_position + count) of one request in one call,
    // each attending causally; returns the greedy token after the last one.
    // The committed KV length must equal first_position. Runners without a
    // fused prefill keep the default, which reports it unsupported.
    [[nodiscard]] virtual bool generationSupportsPrefill() const noexcept { return false; }
    [[nodiscard]] virtual GenerationStepResult generationPrefill(RequestId request_id,
        std::uint32_t const* tokens, std::uint32_t count, std::uint32_t first_position);

protected:
    GenerationModelRunner() = default;
};

// One synchronous request at a time; stop() is thread-safe.
class SingleRequestGenerationRuntime final {
public:
    SingleRequestGenerationRuntime(EngineKvBackend& kv, GenerationModelRunner& runner) noexcept
        : kv_(&kv), runner_(&runner)
    {
    }
    SingleRequestGenerationRuntime(SingleRequestGenerationRuntime const&) = delete;
    SingleRequestGenerationRuntime& operator=(SingleRequestGenerationRuntime const&) = delete;

    [[nodiscard]] GenerationTerminal generate(GenerationRequest const& request);
    void stop() noexcept { stopped_.store(true, std::memory_order_release); }
    [[nodiscard]] bool stopped() const noexcept { return stopped_.load(std::memory_order_acquire); }

private:
    EngineKvBackend* kv_;
    GenerationModelRunner* runner_;
    std::atomic<bool> stopped_{false};
    std::atomic<bool> generating_{false};
};

[[nodiscard]] std::string_view toString(GenerationError e) noexcept;
[[nodiscard]] std::string_view toString(GenerationTerminalReason r) noexcept;

} // namespace kimkvcache

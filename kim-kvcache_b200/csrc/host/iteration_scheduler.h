// Synchronous iteration-level FIFO scheduler with chunked prefill.
// API and semantics follow the reference (include/kim-kv/engine/
// iteration_scheduler.h:14-183, src/engine/iteration_scheduler.cpp:1-772):
// admission gates (max active requests, worst-case KV-token budget), per
// iteration quota min(prompt remaining, prefill_chunk_size) or 1 for decode,
// "waves" in which every selected request advances by one position, waves
// split into model batches of at most the runner's batch size. Two
// extensions are off by default: fused prefill chunks
// (IterationSchedulerConfig::fused_prefill) and requests whose prompt prefix
// is already in the KV backend (GenerationRequest::kv_prefix_tokens).
#pragma once

#include "generation.h"

#include <atomic>
#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <vector>

namespace kimkvcache {

enum class SchedulerRequestState : std::uint8_t {
    Created,
    Waiting,
    Running,
    Cancelling,
    Terminal,
    Rejected,
};

enum class SchedulerAdmissionError : std::uint8_t {
    None,
    InvalidArgument,
    RuntimeStopped,
    DuplicateRequest,
    MaxActiveRequests,
    KvTokenBudget,
    InternalError,
};

struct IterationSchedulerConfig final {
    std::uint32_t max_active_requests{0};
    std::uint32_t max_batched_tokens{0};
    std::uint64_t max_kv_tokens{0};
    std::uint32_t prefill_chunk_size{16};
    // Extension (no counterpart in the reference): when the runner has a
    // fused prefill (GenerationModelRunner::generationPrefill), a request's
    // prompt quota of an iteration goes to the model as one multi-position
    // call instead of one position per wave. Off: the reference's waves.
    bool fused_prefill{false};

    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return max_active_requests != 0 && max_batched_tokens != 0 && max_kv_tokens != 0
            && prefill_chunk_size != 0;
    }
};

struct SchedulerAdmissionResult final {
    bool accepted{false};
    SchedulerAdmissionError error{SchedulerAdmissionError::InternalError};
    std::string detail{};
    [[nodiscard]] bool ok() const noexcept
    {
        return accepted && error == SchedulerAdmissionError::None;
    }
};

struct SchedulerIterationResult final {
    std::uint64_t iteration{0};
    std::uint32_t model_forward_tokens{0};
    std::uint32_t model_forward_batches{0};
    std::uint32_t prefill_tokens{0};
    std::uint32_t decode_tokens{0};
    std::uint32_t terminals_produced{0};
};

struct IterationSchedulerSnapshot final {
    std::uint64_t iteration_count{0};
    std::uint64_t accepted_count{0};
    std::uint64_t rejected_count{0};
    std::uint64_t waiting_count{0};
    std::uint64_t running_count{0};
    std::uint64_t cancelling_count{0};
    std::uint64_t terminal_count{0};
    std::uint64_t reserved_kv_tokens{0};
    std::uint64_t model_forward_tokens{0};
    std::uint64_t model_forward_batches{0};
    std::uint64_t prefill_tokens{0};
    std::uint64_t decode_tokens{0};
    bool stopped{false};

    [[nodiscard]] constexpr std::uint64_t activeCount() const noexcept
    {
        return waiting_count + running_count + cancelling_count;
    }
};

class IterationSchedulerRuntime final {
public:
    IterationSchedulerRuntime(EngineKvBackend& kv, GenerationModelRunner& runner,
        IterationSchedulerConfig config);
    ~IterationSchedulerRuntime();
    IterationSchedulerRuntime(IterationSchedulerRuntime const&) = delete;
    IterationSchedulerRuntime& operator=(IterationSchedulerRuntime const&) = delete;

    [[nodiscard]] SchedulerAdmissionResult submit(GenerationRequest request);
    [[nodiscard]] bool cancel(RequestId request_id) noexcept;
    [[nodiscard]] SchedulerIterationResult runIteration();
    [[nodiscard]] std::vector<GenerationTerminal> drain();
    [[nodiscard]] std::vector<GenerationTerminal> takeTerminals();
    [[nodiscard]] std::optional<SchedulerRequestState> requestState(RequestId request_id) const;
    [[nodiscard]] IterationSchedulerSnapshot snapshot() const;
    [[nodiscard]] bool idle() const noexcept;
    void stop() noexcept;
    [[nodiscard]] bool stopped() const noexcept;

private:
    class Impl;
    std::unique_ptr<Impl> impl_;
};

} // namespace kimkvcache

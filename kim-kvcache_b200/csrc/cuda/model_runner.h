// TinyLlama-shaped FP16 decoder runner on the B200 kernels.
//
// Public API follows the reference CUDA runner
// (include/kim-kv/cuda/cuda_model_runner.h:14-186): factory from a weight
// manifest + archive, an EngineKvBackend and a stream; forwardToken with
// optional debug capture; the GenerationModelRunner SPI.
//
// Execution: one model batch (all lanes) runs as one fused device step:
// COW copies -> embedding -> per layer [QKV projection (input RMSNorm fused,
// RoPE and KV-page write in its epilogue), paged attention over all lanes, O
// projection + residual, gate/up projection (post-attention RMSNorm fused) +
// SiLU gate, down projection + residual] -> LM head (final RMSNorm fused) +
// greedy argmax -> token ids to host. The norm weights are folded into the
// packed projection weights; each projection computes its rows' rsqrt factor. Host work per step: reserve each lane, one upload of the step inputs
// (tokens, positions, write slots, page descriptors, attention work list),
// one stream synchronisation, commit each lane. With graphs enabled the
// device part is replayed from a CUDA graph captured per batch size.
#pragma once

#include "../host/generation.h"
#include "cuda_backend.h"

#include <array>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace kimkvcache {

enum class CudaModelRunnerError : std::uint8_t {
    None,
    InvalidArgument,
    InvalidState,
    ManifestError,
    DataFileError,
    AllocationFailed,
    CublasFailed,  // kept for API compatibility; never produced (no cuBLAS)
    SubmissionFailed,
    ExecutionFailed,
    KvBackendFailed,
};

struct CudaModelRunnerStatus final {
    CudaModelRunnerError error{CudaModelRunnerError::None};
    int native_code{0};
    std::string detail{};
    [[nodiscard]] bool ok() const noexcept { return error == CudaModelRunnerError::None; }
    [[nodiscard]] explicit operator bool() const noexcept { return ok(); }
};

struct ModelRunnerDebugCapture final {
    std::vector<std::uint32_t> layer_indices{};
    std::vector<KvScalar> embedding{};
    std::vector<std::vector<KvScalar>> layer_hidden_states{};
    std::vector<KvScalar> final_hidden_state{};
};

struct ModelTokenResult final {
    CudaModelRunnerStatus status{};
    std::uint32_t greedy_token_id{0};
    std::vector<float> logits{};
    [[nodiscard]] bool ok() const noexcept { return status.ok(); }
};

struct ModelRunnerOutputOptions final {
    bool copy_logits{true};
};

struct CudaModelRunnerOptions final {
    std::uint32_t max_batch_size{8};   // at most 64 lanes per model batch
    bool use_cuda_graphs{true};        // replay the device step from a CUDA graph
    bool verify_checksums{true};       // SHA-256 of every tensor at load
    // After a step commits the 64th token of a 64-aligned run, fold that
    // run's 8 sealed micro pages into one extent page (8 micro -> 1 extent
    // promotion), so decode tails stay under 64 tokens of micro pages. The
    // reference never promotes during generation; off by default.
    bool auto_promote{false};
    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return max_batch_size != 0 && max_batch_size <= 64;
    }
};

struct CudaModelRunnerCreateResult;

class CudaTinyLlamaModelRunner final : public GenerationModelRunner {
public:
    struct Impl;
    ~CudaTinyLlamaModelRunner() override;

    [[nodiscard]] TinyLlamaConfig config() const noexcept;
    [[nodiscard]] std::uint64_t deviceWeightBytes() const noexcept;
    [[nodiscard]] std::uint64_t deviceWorkspaceBytes() const noexcept;
    [[nodiscard]] std::uint32_t maxBatchSize() const noexcept;

    [[nodiscard]] ModelTokenResult forwardToken(RequestId request_id, std::uint32_t token_id,
        std::uint32_t expected_position, ModelRunnerDebugCapture* debug_capture = nullptr,
        ModelRunnerOutputOptions output_options = {});

    [[nodiscard]] TinyLlamaConfig generationConfig() const noexcept override;
    [[nodiscard]] GenerationStepResult generationForwardToken(RequestId request_id,
        std::uint32_t token_id, std::uint32_t expected_position) override;
    [[nodiscard]] GenerationBatchResult generationForwardBatch(
        std::vector<GenerationBatchItem> const& batch) override;
    [[nodiscard]] std::uint32_t generationMaxBatchSize() const noexcept override;

    // generationForwardBatch that also returns every lane's FP32 logits
    // (logits[i * vocab ...], row i = batch item i; rows of failed items are
    // zero). The step runs the same kernels outside the captured graph (the
    // LM head also stores its logits). No counterpart in the reference, whose
    // batched path returns tokens only; used to check the fused step lane by
    // lane against the reference arithmetic.
    [[nodiscard]] GenerationBatchResult generationForwardBatchLogits(
        std::vector<GenerationBatchItem> const& batch, std::vector<float>& logits);

    // Fused multi-token prefill (no counterpart in the reference, which feeds
    // prompts one position per wave): the prompt tokens at positions
    // first_position.. of one request run through the decode step as one
    // batch of up to max_batch_size consecutive positions per step. The
    // metadata is appended up front (KvCacheManager::append, with partial-tail
    // copy-on-write), every token's K/V is written by the QKV projection, and
    // position p attends causally to tokens [0, p] of the request. The
    // request's committed length must equal first_position; on success it
    // grows by prompt.size() and the result carries the greedy token after
    // the last prompt position. A device failure releases the request, as
    // the reference's append data path does.
    [[nodiscard]] GenerationStepResult prefill(RequestId request_id,
        std::vector<std::uint32_t> const& prompt, std::uint32_t first_position);

    // The scheduler's view of prefill() (GenerationModelRunner extension):
    // on a device failure the request stays for its owner to release.
    [[nodiscard]] bool generationSupportsPrefill() const noexcept override { return true; }
    [[nodiscard]] GenerationStepResult generationPrefill(RequestId request_id, std::uint32_t const* tokens,
        std::uint32_t count, std::uint32_t first_position) override;

    // Device time of the last fused step (ms, from CUDA events), 0 if unknown.
    [[nodiscard]] float lastStepDeviceMs() const noexcept;
    // Detail of the last failed fused step (empty if none).
    [[nodiscard]] std::string lastError() const;
    // Kernels launched by the last fused step.
    [[nodiscard]] std::uint32_t lastStepLaunches() const noexcept;
    // Bytes the last fused step copied host -> device (the step record) and
    // device -> host (greedy token ids, plus logits or captures when asked).
    [[nodiscard]] std::uint64_t lastStepH2dBytes() const noexcept;
    [[nodiscard]] std::uint64_t lastStepD2hBytes() const noexcept;
    // Host wall time of the last fused step, in microseconds, by phase:
    // [0] lane reservations, [1] step record (descriptors and work list),
    // [2] upload + graph launch + readback enqueue, [3] wait for the device,
    // [4] commits and auto-promotion.
    [[nodiscard]] std::array<float, 5> lastStepHostUs() const noexcept;
    // Turns auto-promotion (CudaModelRunnerOptions::auto_promote) on or off.
    void setAutoPromote(bool enabled) noexcept;

private:
    explicit CudaTinyLlamaModelRunner(std::unique_ptr<Impl> impl) noexcept;
    std::unique_ptr<Impl> impl_;
    [[nodiscard]] GenerationStepResult prefillChunks(RequestId request_id,
        std::uint32_t const* prompt, std::uint32_t count, std::uint32_t first_position,
        bool release_on_failure);
    friend GenerationStepResult prefillStep(Impl&, RequestId, std::uint32_t const*, std::uint32_t,
        std::uint32_t, BlockTable const&, BlockTable const&);
    friend CudaModelRunnerCreateResult createCudaTinyLlamaModelRunner(std::string const&,
        std::string const&, EngineKvBackend&, EngineStream, CudaModelRunnerOptions);
};

struct CudaModelRunnerCreateResult final {
    CudaModelRunnerStatus status{};
    std::unique_ptr<CudaTinyLlamaModelRunner> runner{};
    [[nodiscard]] bool ok() const noexcept { return status.ok() && runner != nullptr; }
};

// kv_backend and stream are borrowed and must outlive the runner.
[[nodiscard]] CudaModelRunnerCreateResult createCudaTinyLlamaModelRunner(
    std::string const& manifest_path, std::string const& data_path, EngineKvBackend& kv_backend,
    EngineStream stream, CudaModelRunnerOptions options = {});

} // namespace kimkvcache

// Engine <-> KV-backend SPI: per-token RAII transactions, device descriptor
// structs and ragged attention batches. Types, names, state machine and error
// mapping follow the reference (include/kim-kv/engine/engine_kv.h:14-427,
// src/engine/engine_kv.cpp:1-320) so model runners and schedulers written
// against it compile unchanged.
//
// One addition: TokenTransaction::submitFusedLayers() lets a backend that runs
// all layers of a token in one fused device step (this library's CUDA
// backend) advance the per-layer state machine in one call, with the same
// ordering checks as calling writeLayer/attendLayer for every layer.
#pragma once

#include "kv_cache_manager.h"

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string_view>
#include <type_traits>

namespace kimkvcache {

using EngineStream = void*;
using TokenTransactionId = std::uint64_t;
constexpr TokenTransactionId kInvalidTokenTransactionId = 0;

enum class EngineKvBackendKind : std::uint8_t { Heterogeneous, Fixed };

enum class EngineKvError : std::uint8_t {
    None,
    InvalidArgument,
    InvalidState,
    RequestNotFound,
    RequestAlreadyExists,
    RequestConflict,
    ResourceExhausted,
    LayerOutOfOrder,
    SubmissionFailed,
    ExecutionFailed,
    InternalError,
};

[[nodiscard]] std::string_view toString(EngineKvError error) noexcept;

struct EngineKvStatus final {
    EngineKvError error{EngineKvError::None};
    [[nodiscard]] constexpr bool ok() const noexcept { return error == EngineKvError::None; }
    [[nodiscard]] explicit constexpr operator bool() const noexcept { return ok(); }
};

struct EngineKvConfig final {
    KvLayout kv_layout{};
    std::uint32_t query_head_count{0};
    std::size_t attention_workspace_bytes{0};

    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return kv_layout.valid() && query_head_count >= kv_layout.kv_head_count
            && query_head_count % kv_layout.kv_head_count == 0
            && attention_workspace_bytes != 0;
    }
};

struct DeviceBlockDescriptor final {
    std::uint32_t slot{PageHandle::kInvalidSlot};
    std::uint32_t generation{PageHandle::kInvalidGeneration};
    std::uint32_t logical_token_begin{0};
    std::uint16_t valid_tokens{0};
    std::uint16_t page_token_capacity{0};
    PageKind kind{PageKind::Micro};

    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return slot != PageHandle::kInvalidSlot && generation != PageHandle::kInvalidGeneration
            && valid_tokens != 0 && page_token_capacity != 0
            && valid_tokens <= page_token_capacity && isKnownPageKind(kind);
    }
};
static_assert(std::is_trivially_copyable_v<DeviceBlockDescriptor>);

struct DeviceBlockTableView final {
    DeviceBlockDescriptor const* device_descriptors{nullptr};
    std::uint32_t descriptor_count{0};
    std::uint32_t committed_token_count{0};
    std::uint32_t current_token_position{0};

    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return device_descriptors != nullptr && descriptor_count != 0
            && current_token_position == committed_token_count;
    }
};

struct LayerKvWrite final {
    std::uint32_t layer{0};
    KvScalar const* device_key{nullptr};
    KvScalar const* device_value{nullptr};
};

struct PagedDecodeRequest final {
    std::uint32_t layer{0};
    KvScalar const* device_query{nullptr};
    KvScalar* device_output{nullptr};
    void* device_workspace{nullptr};
    std::size_t workspace_bytes{0};
    float attention_scale{0.0F};
};

class TokenTransaction;

struct PagedDecodeBatchItem final {
    TokenTransaction* transaction{nullptr};
    PagedDecodeRequest request{};
    EngineKvStatus status{EngineKvError::InvalidState};
    bool dispatched{false};
};

struct DevicePagedDecodeBatchItem final {
    DeviceBlockDescriptor const* device_descriptors{nullptr};
    std::uint32_t descriptor_count{0};
    std::uint32_t token_count{0};
    std::uint32_t layer{0};
    KvScalar const* device_query{nullptr};
    float* device_scores{nullptr};
    KvScalar* device_output{nullptr};
    float attention_scale{0.0F};
};
static_assert(std::is_trivially_copyable_v<DevicePagedDecodeBatchItem>);

struct PagedDecodeBatch final {
    PagedDecodeBatchItem* items{nullptr};
    std::size_t item_count{0};
    DevicePagedDecodeBatchItem* host_items{nullptr};
    DevicePagedDecodeBatchItem* device_items{nullptr};
    std::size_t item_capacity{0};
};

struct ReserveTokenRequest final {
    RequestId request_id{kInvalidRequestId};
    std::uint32_t expected_committed_tokens{0};
    EngineStream stream{nullptr};
};

enum class TokenTransactionPhase : std::uint8_t {
    Empty,
    AwaitingLayerWrite,
    AwaitingLayerAttention,
    ReadyToCommit,
    Failed,
    Committed,
    RolledBack,
};

struct TokenTransactionSnapshot final {
    TokenTransactionId transaction_id{kInvalidTokenTransactionId};
    RequestId request_id{kInvalidRequestId};
    std::uint32_t logical_token_position{0};
    std::uint32_t layer_count{0};
    std::uint32_t next_layer{0};
    TokenTransactionPhase phase{TokenTransactionPhase::Empty};
};

// write/attend only enqueue work on the bound stream; commit is the single
// completion point of a token; rollback waits for in-flight access to end
// before the staged page and the lease are released.
class TokenTransactionBackend {
public:
    virtual ~TokenTransactionBackend() = default;
    TokenTransactionBackend(TokenTransactionBackend const&) = delete;
    TokenTransactionBackend& operator=(TokenTransactionBackend const&) = delete;

    [[nodiscard]] virtual EngineKvStatus writeLayer(LayerKvWrite const& write, EngineStream s) = 0;
    [[nodiscard]] virtual EngineKvStatus attendLayer(PagedDecodeRequest const& r, EngineStream s) = 0;
    // Default: every valid lane is submitted on its own.
    virtual void attendLayerBatch(PagedDecodeBatch& batch);
    // Default: not supported (only fused-step backends implement it).
    [[nodiscard]] virtual EngineKvStatus submitFusedLayers(EngineStream s);
    [[nodiscard]] virtual EngineKvStatus commit(EngineStream s) = 0;
    virtual void rollback(EngineStream s) noexcept = 0;

protected:
    TokenTransactionBackend() = default;
    [[nodiscard]] static TokenTransactionBackend* batchBackend(PagedDecodeBatchItem const& item) noexcept;
    [[nodiscard]] static EngineStream batchStream(PagedDecodeBatchItem const& item) noexcept;
};

class TokenTransaction final {
public:
    TokenTransaction() noexcept = default;
    TokenTransaction(std::unique_ptr<TokenTransactionBackend> backend, TokenTransactionId id,
        RequestId request_id, std::uint32_t logical_token_position, std::uint32_t layer_count,
        EngineStream stream) noexcept;
    ~TokenTransaction();

    TokenTransaction(TokenTransaction const&) = delete;
    TokenTransaction& operator=(TokenTransaction const&) = delete;
    TokenTransaction(TokenTransaction&& other) noexcept;
    TokenTransaction& operator=(TokenTransaction&& other) noexcept;

    [[nodiscard]] bool valid() const noexcept { return active(); }
    [[nodiscard]] TokenTransactionSnapshot snapshot() const noexcept;
    [[nodiscard]] EngineKvStatus writeLayer(LayerKvWrite const& write);
    [[nodiscard]] EngineKvStatus attendLayer(PagedDecodeRequest const& request);
    // All layers at once (see the file comment); requires no layer submitted yet.
    [[nodiscard]] EngineKvStatus submitFusedLayers();
    [[nodiscard]] EngineKvStatus commit();
    [[nodiscard]] EngineKvStatus rollback() noexcept;
    [[nodiscard]] TokenTransactionBackend* backend() const noexcept { return backend_.get(); }

private:
    // The three ways of advancing through the layers.
    enum class Step : std::uint8_t { Write, Attend, AllLayers };
    // None when `step` on `layer` is the transaction's next move;
    // InvalidState when it is not live, LayerOutOfOrder otherwise.
    [[nodiscard]] EngineKvError admit(Step step, std::uint32_t layer) const noexcept;
    // The phase after an admitted step: the next one, or Failed.
    void settle(Step step, EngineKvStatus const& outcome) noexcept;
    // Ends a live transaction in `end` (Committed or RolledBack).
    void finish(TokenTransactionPhase end) noexcept;
    void adopt(TokenTransaction& other) noexcept;
    [[nodiscard]] bool active() const noexcept;
    void rollbackNoexcept() noexcept;
    void resetMovedFrom() noexcept;

    std::unique_ptr<TokenTransactionBackend> backend_{};
    TokenTransactionId transaction_id_{kInvalidTokenTransactionId};
    RequestId request_id_{kInvalidRequestId};
    std::uint32_t logical_token_position_{0};
    std::uint32_t layer_count_{0};
    std::uint32_t next_layer_{0};
    TokenTransactionPhase phase_{TokenTransactionPhase::Empty};
    EngineStream stream_{nullptr};

    friend class TokenTransactionBackend;
    friend void attendLayerBatch(PagedDecodeBatch& batch);
};

// Checks every lane against the scalar state machine, dispatches one backend
// batch operation, then advances or fails each lane on its own.
void attendLayerBatch(PagedDecodeBatch& batch);

struct TokenReserveResult final {
    EngineKvStatus status{};
    TokenTransaction transaction{};
    [[nodiscard]] bool ok() const noexcept { return status.ok() && transaction.valid(); }
    [[nodiscard]] explicit operator bool() const noexcept { return ok(); }
};

struct EngineKvBackendSnapshot final {
    std::uint64_t request_count{0};
    std::uint64_t active_transaction_count{0};
    std::uint64_t committed_token_count{0};
    std::uint64_t batched_attention_submissions{0};
    std::uint64_t batched_attention_lanes{0};
    std::uint16_t primary_page_tokens{0};
    std::uint16_t secondary_page_tokens{0};
    std::uint32_t primary_page_capacity{0};
    std::uint32_t secondary_page_capacity{0};
    std::uint32_t allocated_primary_pages{0};
    std::uint32_t allocated_secondary_pages{0};
    std::uint64_t successful_primary_allocations{0};
    std::uint64_t successful_secondary_allocations{0};
    std::uint64_t failed_primary_allocations{0};
    std::uint64_t failed_secondary_allocations{0};
    std::uint64_t storage_reserved_bytes{0};
};

class EngineKvBackend {
public:
    virtual ~EngineKvBackend() = default;
    EngineKvBackend(EngineKvBackend const&) = delete;
    EngineKvBackend& operator=(EngineKvBackend const&) = delete;

    [[nodiscard]] virtual EngineKvBackendKind kind() const noexcept = 0;
    [[nodiscard]] virtual EngineKvConfig config() const noexcept = 0;
    [[nodiscard]] virtual EngineKvStatus createRequest(RequestId request_id) = 0;
    [[nodiscard]] virtual EngineKvStatus forkRequest(RequestId source, RequestId child) = 0;
    [[nodiscard]] virtual EngineKvStatus releaseRequest(RequestId request_id) = 0;
    [[nodiscard]] virtual TokenReserveResult reserveToken(ReserveTokenRequest const& request) = 0;
    [[nodiscard]] virtual EngineKvBackendSnapshot snapshot() const = 0;
    [[nodiscard]] virtual bool checkInvariants() const = 0;

protected:
    EngineKvBackend() = default;
};

} // namespace kimkvcache

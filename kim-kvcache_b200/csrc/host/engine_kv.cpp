// TokenTransaction state machine and ragged attention batch dispatch
// (reference semantics: src/engine/engine_kv.cpp:1-320).
#include "engine_kv.h"

#include <utility>

namespace kimkvcache {
namespace {

constexpr EngineKvStatus status(EngineKvError e) noexcept { return EngineKvStatus{e}; }

bool attentionRequestValid(PagedDecodeRequest const& r) noexcept
{
    return r.device_query != nullptr && r.device_output != nullptr
        && r.device_workspace != nullptr && r.workspace_bytes != 0 && r.attention_scale > 0.0F;
}

} // namespace

std::string_view toString(EngineKvError error) noexcept
{
    static constexpr std::string_view names[] = {
        "none", "invalid_argument", "invalid_state", "request_not_found",
        "request_already_exists", "request_conflict", "resource_exhausted",
        "layer_out_of_order", "submission_failed", "execution_failed", "internal_error",
    };
    auto const i = static_cast<std::size_t>(error);
    return i < sizeof(names) / sizeof(names[0]) ? names[i] : "unknown";
}

TokenTransactionBackend* TokenTransactionBackend::batchBackend(PagedDecodeBatchItem const& item) noexcept
{
    return item.transaction != nullptr ? item.transaction->backend_.get() : nullptr;
}

EngineStream TokenTransactionBackend::batchStream(PagedDecodeBatchItem const& item) noexcept
{
    return item.transaction != nullptr ? item.transaction->stream_ : nullptr;
}

void TokenTransactionBackend::attendLayerBatch(PagedDecodeBatch& batch)
{
    for (std::size_t i = 0; i < batch.item_count; ++i) {
        PagedDecodeBatchItem& item = batch.items[i];
        if (!item.status.ok()) {
            continue;
        }
        TokenTransactionBackend* const backend = batchBackend(item);
        item.status = backend == nullptr ? status(EngineKvError::InvalidState)
                                         : backend->attendLayer(item.request, batchStream(item));
    }
}

EngineKvStatus TokenTransactionBackend::submitFusedLayers(EngineStream)
{
    return status(EngineKvError::InvalidState);
}

TokenTransaction::TokenTransaction(std::unique_ptr<TokenTransactionBackend> backend,
    TokenTransactionId id, RequestId request_id, std::uint32_t logical_token_position,
    std::uint32_t layer_count, EngineStream stream) noexcept
    : backend_(std::move(backend))
    , transaction_id_(id)
    , request_id_(request_id)
    , logical_token_position_(logical_token_position)
    , layer_count_(layer_count)
    , phase_(TokenTransactionPhase::AwaitingLayerWrite)
    , stream_(stream)
{
    if (backend_ == nullptr || id == kInvalidTokenTransactionId
        || request_id == kInvalidRequestId || layer_count == 0) {
        if (backend_ != nullptr) {
            backend_->rollback(stream_);
        }
        backend_.reset();
        resetMovedFrom();
    }
}

TokenTransaction::~TokenTransaction() { rollbackNoexcept(); }

TokenTransaction::TokenTransaction(TokenTransaction&& other) noexcept
    : backend_(std::move(other.backend_))
    , transaction_id_(other.transaction_id_)
    , request_id_(other.request_id_)
    , logical_token_position_(other.logical_token_position_)
    , layer_count_(other.layer_count_)
    , next_layer_(other.next_layer_)
    , phase_(other.phase_)
    , stream_(other.stream_)
{
    other.resetMovedFrom();
}

TokenTransaction& TokenTransaction::operator=(TokenTransaction&& other) noexcept
{
    if (this != &other) {
        rollbackNoexcept();
        backend_ = std::move(other.backend_);
        transaction_id_ = other.transaction_id_;
        request_id_ = other.request_id_;
        logical_token_position_ = other.logical_token_position_;
        layer_count_ = other.layer_count_;
        next_layer_ = other.next_layer_;
        phase_ = other.phase_;
        stream_ = other.stream_;
        other.resetMovedFrom();
    }
    return *this;
}

bool TokenTransaction::active() const noexcept
{
    switch (phase_) {
    case TokenTransactionPhase::AwaitingLayerWrite:
    case TokenTransactionPhase::AwaitingLayerAttention:
    case TokenTransactionPhase::ReadyToCommit:
    case TokenTransactionPhase::Failed:
        return backend_ != nullptr;
    default:
        return false;
    }
}

TokenTransactionSnapshot TokenTransaction::snapshot() const noexcept
{
    return TokenTransactionSnapshot{transaction_id_, request_id_, logical_token_position_,
        layer_count_, next_layer_, phase_};
}

EngineKvStatus TokenTransaction::writeLayer(LayerKvWrite const& write)
{
    if (!active()) {
        return status(EngineKvError::InvalidState);
    }
    if (phase_ != TokenTransactionPhase::AwaitingLayerWrite || write.layer != next_layer_) {
        return status(EngineKvError::LayerOutOfOrder);
    }
    if (write.device_key == nullptr || write.device_value == nullptr) {
        return status(EngineKvError::InvalidArgument);
    }
    EngineKvStatus const result = backend_->writeLayer(write, stream_);
    if (!result.ok()) {
        phase_ = TokenTransactionPhase::Failed;
        return result;
    }
    phase_ = TokenTransactionPhase::AwaitingLayerAttention;
    return {};
}

EngineKvStatus TokenTransaction::attendLayer(PagedDecodeRequest const& request)
{
    if (!active()) {
        return status(EngineKvError::InvalidState);
    }
    if (phase_ != TokenTransactionPhase::AwaitingLayerAttention || request.layer != next_layer_) {
        return status(EngineKvError::LayerOutOfOrder);
    }
    if (!attentionRequestValid(request)) {
        return status(EngineKvError::InvalidArgument);
    }
    EngineKvStatus const result = backend_->attendLayer(request, stream_);
    if (!result.ok()) {
        phase_ = TokenTransactionPhase::Failed;
        return result;
    }
    ++next_layer_;
    phase_ = next_layer_ == layer_count_ ? TokenTransactionPhase::ReadyToCommit
                                         : TokenTransactionPhase::AwaitingLayerWrite;
    return {};
}

EngineKvStatus TokenTransaction::submitFusedLayers()
{
    if (!active()) {
        return status(EngineKvError::InvalidState);
    }
    if (phase_ != TokenTransactionPhase::AwaitingLayerWrite || next_layer_ != 0) {
        return status(EngineKvError::LayerOutOfOrder);
    }
    EngineKvStatus const result = backend_->submitFusedLayers(stream_);
    if (!result.ok()) {
        phase_ = TokenTransactionPhase::Failed;
        return result;
    }
    next_layer_ = layer_count_;
    phase_ = TokenTransactionPhase::ReadyToCommit;
    return {};
}

EngineKvStatus TokenTransaction::commit()
{
    if (!active() || phase_ != TokenTransactionPhase::ReadyToCommit) {
        return status(EngineKvError::InvalidState);
    }
    EngineKvStatus const result = backend_->commit(stream_);
    if (!result.ok()) {
        backend_->rollback(stream_);
    }
    backend_.reset();
    phase_ = result.ok() ? TokenTransactionPhase::Committed : TokenTransactionPhase::RolledBack;
    return result;
}

EngineKvStatus TokenTransaction::rollback() noexcept
{
    if (!active()) {
        return status(EngineKvError::InvalidState);
    }
    rollbackNoexcept();
    return {};
}

void TokenTransaction::rollbackNoexcept() noexcept
{
    if (!active()) {
        return;
    }
    backend_->rollback(stream_);
    backend_.reset();
    phase_ = TokenTransactionPhase::RolledBack;
}

void TokenTransaction::resetMovedFrom() noexcept
{
    transaction_id_ = kInvalidTokenTransactionId;
    request_id_ = kInvalidRequestId;
    logical_token_position_ = 0;
    layer_count_ = 0;
    next_layer_ = 0;
    phase_ = TokenTransactionPhase::Empty;
    stream_ = nullptr;
}

void attendLayerBatch(PagedDecodeBatch& batch)
{
    if (batch.items == nullptr || batch.item_count == 0) {
        return;
    }
    bool const scratch_ok = batch.host_items != nullptr && batch.device_items != nullptr
        && batch.item_capacity >= batch.item_count;
    TokenTransactionBackend* dispatcher = nullptr;
    for (std::size_t i = 0; i < batch.item_count; ++i) {
        PagedDecodeBatchItem& item = batch.items[i];
        item.status = {};
        item.dispatched = false;
        TokenTransaction* const t = item.transaction;
        if (!scratch_ok) {
            item.status = status(EngineKvError::InvalidArgument);
        } else if (t == nullptr || !t->active()) {
            item.status = status(EngineKvError::InvalidState);
        } else if (t->phase_ != TokenTransactionPhase::AwaitingLayerAttention
            || item.request.layer != t->next_layer_) {
            item.status = status(EngineKvError::LayerOutOfOrder);
        } else if (!attentionRequestValid(item.request)) {
            item.status = status(EngineKvError::InvalidArgument);
        } else {
            item.dispatched = true;
            if (dispatcher == nullptr) {
                dispatcher = t->backend_.get();
            }
        }
    }
    if (dispatcher == nullptr) {
        return;
    }
    dispatcher->attendLayerBatch(batch);
    for (std::size_t i = 0; i < batch.item_count; ++i) {
        PagedDecodeBatchItem& item = batch.items[i];
        TokenTransaction* const t = item.transaction;
        if (!item.dispatched || t == nullptr
            || t->phase_ != TokenTransactionPhase::AwaitingLayerAttention
            || item.request.layer != t->next_layer_) {
            continue;
        }
        if (!item.status.ok()) {
            t->phase_ = TokenTransactionPhase::Failed;
            continue;
        }
        ++t->next_layer_;
        t->phase_ = t->next_layer_ == t->layer_count_ ? TokenTransactionPhase::ReadyToCommit
                                                      : TokenTransactionPhase::AwaitingLayerWrite;
    }
}

} // namespace kimkvcache

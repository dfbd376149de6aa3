// TokenTransaction: the per-token, per-layer state machine over a backend
// transaction, and the ragged attention batch across transactions.
// Reference semantics: src/engine/engine_kv.cpp (phases, error precedence,
// rollback on destruction, per-lane batch status).
//
// Every move is a Step checked by admit() against the phase and the next
// layer, run on the backend, and settled into the next phase (or Failed).
// Commit and rollback end the transaction through finish().
#include "engine_kv.h"

#include <utility>

namespace kimkvcache {
namespace {

constexpr EngineKvStatus fail(EngineKvError e) noexcept { return EngineKvStatus{e}; }

bool attentionRequestValid(PagedDecodeRequest const& r) noexcept
{
    return r.device_query != nullptr && r.device_output != nullptr && r.device_workspace != nullptr
        && r.workspace_bytes != 0 && r.attention_scale > 0.0F;
}

} // namespace

std::string_view toString(EngineKvError error) noexcept
{
    switch (error) {
    case EngineKvError::None: return "none";
    case EngineKvError::InvalidArgument: return "invalid_argument";
    case EngineKvError::InvalidState: return "invalid_state";
    case EngineKvError::RequestNotFound: return "request_not_found";
    case EngineKvError::RequestAlreadyExists: return "request_already_exists";
    case EngineKvError::RequestConflict: return "request_conflict";
    case EngineKvError::ResourceExhausted: return "resource_exhausted";
    case EngineKvError::LayerOutOfOrder: return "layer_out_of_order";
    case EngineKvError::SubmissionFailed: return "submission_failed";
    case EngineKvError::ExecutionFailed: return "execution_failed";
    case EngineKvError::InternalError: return "internal_error";
    }
    return "unknown";
}

// ---- backend defaults ------------------------------------------------------------------

TokenTransactionBackend* TokenTransactionBackend::batchBackend(PagedDecodeBatchItem const& item) noexcept
{
    return item.transaction == nullptr ? nullptr : item.transaction->backend_.get();
}

EngineStream TokenTransactionBackend::batchStream(PagedDecodeBatchItem const& item) noexcept
{
    return item.transaction == nullptr ? nullptr : item.transaction->stream_;
}

// A backend without a batched kernel serves the lanes one by one.
void TokenTransactionBackend::attendLayerBatch(PagedDecodeBatch& batch)
{
    for (PagedDecodeBatchItem* it = batch.items; it != batch.items + batch.item_count; ++it) {
        if (it->status.ok()) {
            TokenTransactionBackend* const b = batchBackend(*it);
            it->status = b != nullptr ? b->attendLayer(it->request, batchStream(*it))
                                      : fail(EngineKvError::InvalidState);
        }
    }
}

EngineKvStatus TokenTransactionBackend::submitFusedLayers(EngineStream)
{
    return fail(EngineKvError::InvalidState);
}

// ---- lifetime ------------------------------------------------------------------------------

TokenTransaction::TokenTransaction(std::unique_ptr<TokenTransactionBackend> backend,
    TokenTransactionId id, RequestId request_id, std::uint32_t logical_token_position,
    std::uint32_t layer_count, EngineStream stream) noexcept
    : backend_(std::move(backend)), transaction_id_(id), request_id_(request_id)
    , logical_token_position_(logical_token_position), layer_count_(layer_count)
    , phase_(TokenTransactionPhase::AwaitingLayerWrite), stream_(stream)
{
    bool const well_formed = backend_ != nullptr && id != kInvalidTokenTransactionId
        && request_id != kInvalidRequestId && layer_count != 0;
    if (!well_formed) {
        // Whatever the backend reserved is given back at once.
        if (backend_ != nullptr) {
            backend_->rollback(stream_);
            backend_.reset();
        }
        resetMovedFrom();
    }
}

TokenTransaction::~TokenTransaction() { rollbackNoexcept(); }

TokenTransaction::TokenTransaction(TokenTransaction&& other) noexcept { adopt(other); }

TokenTransaction& TokenTransaction::operator=(TokenTransaction&& other) noexcept
{
    if (this != &other) {
        rollbackNoexcept();
        adopt(other);
    }
    return *this;
}

void TokenTransaction::adopt(TokenTransaction& other) noexcept
{
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

bool TokenTransaction::active() const noexcept
{
    bool const open_phase = phase_ == TokenTransactionPhase::AwaitingLayerWrite
        || phase_ == TokenTransactionPhase::AwaitingLayerAttention
        || phase_ == TokenTransactionPhase::ReadyToCommit || phase_ == TokenTransactionPhase::Failed;
    return open_phase && backend_ != nullptr;
}

TokenTransactionSnapshot TokenTransaction::snapshot() const noexcept
{
    return TokenTransactionSnapshot{transaction_id_, request_id_, logical_token_position_, layer_count_,
        next_layer_, phase_};
}

// ---- the state machine ---------------------------------------------------------------------

EngineKvError TokenTransaction::admit(Step step, std::uint32_t layer) const noexcept
{
    if (!active()) {
        return EngineKvError::InvalidState;
    }
    bool in_order = false;
    switch (step) {
    case Step::Write:
        in_order = phase_ == TokenTransactionPhase::AwaitingLayerWrite && layer == next_layer_;
        break;
    case Step::Attend:
        in_order = phase_ == TokenTransactionPhase::AwaitingLayerAttention && layer == next_layer_;
        break;
    case Step::AllLayers:
        in_order = phase_ == TokenTransactionPhase::AwaitingLayerWrite && next_layer_ == 0;
        break;
    }
    return in_order ? EngineKvError::None : EngineKvError::LayerOutOfOrder;
}

void TokenTransaction::settle(Step step, EngineKvStatus const& outcome) noexcept
{
    if (!outcome.ok()) {
        phase_ = TokenTransactionPhase::Failed;
        return;
    }
    switch (step) {
    case Step::Write:
        phase_ = TokenTransactionPhase::AwaitingLayerAttention;
        return;
    case Step::Attend:
        next_layer_ += 1;
        break;
    case Step::AllLayers:
        next_layer_ = layer_count_;
        break;
    }
    phase_ = next_layer_ == layer_count_ ? TokenTransactionPhase::ReadyToCommit
                                         : TokenTransactionPhase::AwaitingLayerWrite;
}

void TokenTransaction::finish(TokenTransactionPhase end) noexcept
{
    backend_.reset();
    phase_ = end;
}

EngineKvStatus TokenTransaction::writeLayer(LayerKvWrite const& write)
{
    EngineKvError const gate = admit(Step::Write, write.layer);
    if (gate != EngineKvError::None) {
        return fail(gate);
    }
    if (write.device_key == nullptr || write.device_value == nullptr) {
        return fail(EngineKvError::InvalidArgument);
    }
    EngineKvStatus const outcome = backend_->writeLayer(write, stream_);
    settle(Step::Write, outcome);
    return outcome;
}

EngineKvStatus TokenTransaction::attendLayer(PagedDecodeRequest const& request)
{
    EngineKvError const gate = admit(Step::Attend, request.layer);
    if (gate != EngineKvError::None) {
        return fail(gate);
    }
    if (!attentionRequestValid(request)) {
        return fail(EngineKvError::InvalidArgument);
    }
    EngineKvStatus const outcome = backend_->attendLayer(request, stream_);
    settle(Step::Attend, outcome);
    return outcome;
}

EngineKvStatus TokenTransaction::submitFusedLayers()
{
    EngineKvError const gate = admit(Step::AllLayers, 0);
    if (gate != EngineKvError::None) {
        return fail(gate);
    }
    EngineKvStatus const outcome = backend_->submitFusedLayers(stream_);
    settle(Step::AllLayers, outcome);
    return outcome;
}

EngineKvStatus TokenTransaction::commit()
{
    if (!active() || phase_ != TokenTransactionPhase::ReadyToCommit) {
        return fail(EngineKvError::InvalidState);
    }
    EngineKvStatus const outcome = backend_->commit(stream_);
    if (outcome.ok()) {
        finish(TokenTransactionPhase::Committed);
    } else {
        backend_->rollback(stream_);  // a completion failure undoes the token
        finish(TokenTransactionPhase::RolledBack);
    }
    return outcome;
}

EngineKvStatus TokenTransaction::rollback() noexcept
{
    if (!active()) {
        return fail(EngineKvError::InvalidState);
    }
    rollbackNoexcept();
    return {};
}

void TokenTransaction::rollbackNoexcept() noexcept
{
    if (active()) {
        backend_->rollback(stream_);
        finish(TokenTransactionPhase::RolledBack);
    }
}

// ---- ragged batches --------------------------------------------------------------------------

void attendLayerBatch(PagedDecodeBatch& batch)
{
    if (batch.items == nullptr || batch.item_count == 0) {
        return;
    }
    using Step = TokenTransaction::Step;
    bool const scratch = batch.host_items != nullptr && batch.device_items != nullptr
        && batch.item_capacity >= batch.item_count;
    // Each lane is admitted as if attendLayer were called on it alone; the
    // first admitted lane's backend runs the whole batch.
    TokenTransactionBackend* runner = nullptr;
    for (PagedDecodeBatchItem* it = batch.items; it != batch.items + batch.item_count; ++it) {
        it->dispatched = false;
        TokenTransaction* const t = it->transaction;
        EngineKvError gate = EngineKvError::None;
        if (!scratch) {
            gate = EngineKvError::InvalidArgument;
        } else if (t == nullptr) {
            gate = EngineKvError::InvalidState;
        } else if ((gate = t->admit(Step::Attend, it->request.layer)) == EngineKvError::None
            && !attentionRequestValid(it->request)) {
            gate = EngineKvError::InvalidArgument;
        }
        it->status = fail(gate);
        if (gate == EngineKvError::None) {
            it->dispatched = true;
            runner = runner != nullptr ? runner : t->backend_.get();
        }
    }
    if (runner == nullptr) {
        return;
    }
    runner->attendLayerBatch(batch);
    // Every dispatched lane that is still where it was advances or fails on
    // its own status.
    for (PagedDecodeBatchItem* it = batch.items; it != batch.items + batch.item_count; ++it) {
        TokenTransaction* const t = it->transaction;
        if (it->dispatched && t != nullptr && t->admit(Step::Attend, it->request.layer) == EngineKvError::None) {
            t->settle(Step::Attend, it->status);
        }
    }
}

} // namespace kimkvcache

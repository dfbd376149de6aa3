// FIFO iteration scheduler (reference semantics:
// src/engine/iteration_scheduler.cpp:27-772). Batch composition, terminal
// order and metrics bookkeeping follow the reference step by step, so the
// same submissions produce the same sequence of model batches.
#include "iteration_scheduler.h"

#include <algorithm>
#include <chrono>
#include <deque>
#include <new>
#include <unordered_map>

namespace kimkvcache {
namespace {

using Clock = std::chrono::steady_clock;

std::uint64_t nanosBetween(Clock::time_point a, Clock::time_point b) noexcept
{
    auto const d = std::chrono::duration_cast<std::chrono::nanoseconds>(b - a).count();
    return d > 0 ? static_cast<std::uint64_t>(d) : 0;
}

// Worst-case committed KV tokens of a request: the last generated token is
// never fed back through the model.
std::uint64_t kvBudget(GenerationRequest const& r) noexcept
{
    return static_cast<std::uint64_t>(r.prompt_token_ids.size()) + r.sampling.max_new_tokens - 1;
}

} // namespace

class IterationSchedulerRuntime::Impl final {
public:
    struct Record final {
        GenerationRequest request{};
        SchedulerRequestState state{SchedulerRequestState::Created};
        GenerationTerminal terminal{};
        std::uint64_t kv_budget{0};
        std::uint32_t prompt_position{0};
        bool kv_created{false};
        bool cancel_requested{false};
        bool emitted{false};
        Clock::time_point started{};
        Clock::time_point first_token{};
        Clock::time_point last_token{};
    };

    Impl(EngineKvBackend& k, GenerationModelRunner& r, IterationSchedulerConfig c) noexcept
        : kv(&k), runner(&r), config(c)
    {
    }

    void setState(RequestId id, SchedulerRequestState s)
    {
        auto const f = states.find(id);
        if (f != states.end()) {
            f->second = s;
        }
    }

    SchedulerAdmissionResult reject(RequestId id, SchedulerAdmissionError e, std::string detail,
        bool remember)
    {
        if (remember && id != kInvalidRequestId) {
            try {
                states.emplace(id, SchedulerRequestState::Rejected);
            } catch (std::bad_alloc const&) {
                return {false, SchedulerAdmissionError::InternalError, "failed to record rejected request"};
            }
        }
        return {false, e, std::move(detail)};
    }

    std::optional<std::string> invalidReason(GenerationRequest const& r) const
    {
        TinyLlamaConfig const m = runner->generationConfig();
        if (!config.valid()) {
            return "scheduler configuration is invalid";
        }
        if (!m.valid() || r.request_id == kInvalidRequestId || r.prompt_token_ids.empty()
            || r.sampling.max_new_tokens == 0) {
            return "request id, prompt, model config, and max_new_tokens are required";
        }
        if (r.prompt_token_ids.size() > m.max_position_embeddings
            || r.sampling.max_new_tokens > m.max_position_embeddings - r.prompt_token_ids.size() + 1) {
            return "prompt and completion exceed the model position limit";
        }
        if (r.sampling.eos_token_id.value_or(m.eos_token_id) >= m.vocabulary_size) {
            return "EOS token is outside the model vocabulary";
        }
        for (std::uint32_t t : r.prompt_token_ids) {
            if (t >= m.vocabulary_size) {
                return "prompt token is outside the model vocabulary";
            }
        }
        return std::nullopt;
    }

    void finish(Record& rec, GenerationTerminalReason reason, GenerationError error, std::string detail)
    {
        if (rec.state == SchedulerRequestState::Terminal) {
            return;
        }
        GenerationTerminal& t = rec.terminal;
        t.reason = reason;
        t.error = error;
        t.detail = std::move(detail);
        t.usage.completion_tokens = static_cast<std::uint32_t>(t.output_token_ids.size());
        t.usage.total_tokens = t.usage.prompt_tokens + t.usage.completion_tokens;
        if (rec.kv_created) {
            EngineKvStatus const released = kv->releaseRequest(rec.request.request_id);
            rec.kv_created = false;
            if (!released.ok()) {
                t.reason = GenerationTerminalReason::Failed;
                t.error = GenerationError::KvBackendFailed;
                t.detail = "release request failed: ";
                t.detail += toString(released.error);
            }
        }
        Clock::time_point const now = Clock::now();
        t.metrics.e2e_ns = nanosBetween(rec.started, now);
        if (rec.emitted) {
            t.metrics.ttft_ns = nanosBetween(rec.started, rec.first_token);
            if (t.output_token_ids.size() > 1) {
                t.metrics.tpot_ns = nanosBetween(rec.first_token, rec.last_token)
                    / (t.output_token_ids.size() - 1);
            }
        }
        rec.state = SchedulerRequestState::Terminal;
        setState(rec.request.request_id, SchedulerRequestState::Terminal);
        reserved_kv_tokens -= rec.kv_budget;
        try {
            terminals.push_back(t);
        } catch (std::bad_alloc const&) {
        }
    }

    void stopRecord(Record& rec)
    {
        finish(rec, GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
            "runtime stopped at iteration boundary");
    }

    void stopAll()
    {
        while (!queue.empty()) {
            RequestId const id = queue.front();
            queue.pop_front();
            auto const f = records.find(id);
            if (f != records.end() && f->second.state != SchedulerRequestState::Terminal) {
                stopRecord(f->second);
            }
        }
    }

    bool cancelledOrStopped(Record& rec)
    {
        if (rec.cancel_requested || (rec.request.cancellation && rec.request.cancellation->cancelled())) {
            finish(rec, GenerationTerminalReason::Cancelled, GenerationError::None,
                "request cancelled at iteration boundary");
            return true;
        }
        if (stopped.load(std::memory_order_acquire)) {
            stopRecord(rec);
            return true;
        }
        return false;
    }

    // Next position of a request; creates its KV request on first touch.
    bool prepare(Record& rec, GenerationBatchItem& item, bool& prefill)
    {
        if (cancelledOrStopped(rec)) {
            return false;
        }
        if (!rec.kv_created) {
            EngineKvStatus const created = kv->createRequest(rec.request.request_id);
            if (!created.ok()) {
                finish(rec, GenerationTerminalReason::Failed, GenerationError::KvBackendFailed,
                    std::string("create request failed: ") + std::string(toString(created.error)));
                return false;
            }
            rec.kv_created = true;
            rec.state = SchedulerRequestState::Running;
            setState(rec.request.request_id, SchedulerRequestState::Running);
        }
        prefill = rec.prompt_position < rec.request.prompt_token_ids.size();
        if (prefill) {
            item = {rec.request.request_id, rec.request.prompt_token_ids[rec.prompt_position],
                rec.prompt_position};
        } else {
            std::uint32_t const pos = rec.terminal.usage.prompt_tokens
                + static_cast<std::uint32_t>(rec.terminal.output_token_ids.size()) - 1;
            item = {rec.request.request_id, rec.terminal.output_token_ids.back(), pos};
        }
        return true;
    }

    void apply(Record& rec, GenerationStepResult step, bool prefill)
    {
        if (!step.success) {
            finish(rec, GenerationTerminalReason::Failed, GenerationError::ModelFailed, std::move(step.detail));
            return;
        }
        TinyLlamaConfig const m = runner->generationConfig();
        if (step.greedy_token_id >= m.vocabulary_size) {
            finish(rec, GenerationTerminalReason::Failed, GenerationError::ModelFailed,
                "model returned a token outside the vocabulary");
            return;
        }
        if (prefill) {
            ++rec.prompt_position;
        }
        if (stopped.load(std::memory_order_acquire)) {
            stopRecord(rec);
            return;
        }
        if (rec.cancel_requested || (rec.request.cancellation && rec.request.cancellation->cancelled())) {
            finish(rec, GenerationTerminalReason::Cancelled, GenerationError::None,
                "request cancelled at iteration boundary");
            return;
        }
        if (rec.prompt_position != rec.request.prompt_token_ids.size()) {
            return;  // still prefilling: the step's token is not an output
        }
        try {
            rec.terminal.output_token_ids.push_back(step.greedy_token_id);
        } catch (std::bad_alloc const&) {
            finish(rec, GenerationTerminalReason::Failed, GenerationError::InternalError,
                "completion token allocation failed");
            return;
        }
        rec.last_token = Clock::now();
        if (!rec.emitted) {
            rec.first_token = rec.last_token;
            rec.emitted = true;
        }
        std::uint32_t const eos = rec.request.sampling.eos_token_id.value_or(m.eos_token_id);
        if (step.greedy_token_id == eos) {
            finish(rec, GenerationTerminalReason::EosToken, GenerationError::None, "EOS token generated");
        } else if (rec.terminal.output_token_ids.size() == rec.request.sampling.max_new_tokens) {
            finish(rec, GenerationTerminalReason::MaxNewTokens, GenerationError::None,
                "max_new_tokens reached");
        }
    }

    EngineKvBackend* kv;
    GenerationModelRunner* runner;
    IterationSchedulerConfig config;
    std::atomic<bool> stopped{false};
    std::unordered_map<RequestId, Record> records;
    std::unordered_map<RequestId, SchedulerRequestState> states;
    std::deque<RequestId> queue;
    std::vector<GenerationTerminal> terminals;
    std::uint64_t iterations{0};
    std::uint64_t reserved_kv_tokens{0};
    std::uint64_t forward_tokens{0};
    std::uint64_t forward_batches{0};
    std::uint64_t prefill_tokens{0};
    std::uint64_t decode_tokens{0};
};

IterationSchedulerRuntime::IterationSchedulerRuntime(EngineKvBackend& kv,
    GenerationModelRunner& runner, IterationSchedulerConfig config)
    : impl_(std::make_unique<Impl>(kv, runner, config))
{
}

IterationSchedulerRuntime::~IterationSchedulerRuntime()
{
    if (impl_) {
        impl_->stopped.store(true, std::memory_order_release);
        impl_->stopAll();
    }
}

SchedulerAdmissionResult IterationSchedulerRuntime::submit(GenerationRequest request)
{
    Impl& im = *impl_;
    if (stopped()) {
        return im.reject(request.request_id, SchedulerAdmissionError::RuntimeStopped,
            "runtime is stopped", true);
    }
    if (im.states.find(request.request_id) != im.states.end()) {
        return im.reject(request.request_id, SchedulerAdmissionError::DuplicateRequest,
            "request id has already been submitted", false);
    }
    if (std::optional<std::string> why = im.invalidReason(request)) {
        return im.reject(request.request_id, SchedulerAdmissionError::InvalidArgument,
            std::move(*why), true);
    }
    if (snapshot().activeCount() >= im.config.max_active_requests) {
        return im.reject(request.request_id, SchedulerAdmissionError::MaxActiveRequests,
            "max_active_requests admission gate rejected request", true);
    }
    std::uint64_t const budget = kvBudget(request);
    if (budget > im.config.max_kv_tokens
        || im.reserved_kv_tokens > im.config.max_kv_tokens - budget) {
        return im.reject(request.request_id, SchedulerAdmissionError::KvTokenBudget,
            "KV token budget admission gate rejected request", true);
    }
    try {
        Impl::Record rec;
        rec.request = std::move(request);
        rec.state = SchedulerRequestState::Waiting;
        rec.terminal.request_id = rec.request.request_id;
        rec.terminal.usage.prompt_tokens = static_cast<std::uint32_t>(rec.request.prompt_token_ids.size());
        rec.kv_budget = budget;
        rec.started = Clock::now();
        RequestId const id = rec.request.request_id;
        im.records.emplace(id, std::move(rec));
        try {
            im.states.emplace(id, SchedulerRequestState::Waiting);
            im.queue.push_back(id);
        } catch (...) {
            im.states.erase(id);
            im.records.erase(id);
            throw;
        }
        im.reserved_kv_tokens += budget;
    } catch (std::bad_alloc const&) {
        return {false, SchedulerAdmissionError::InternalError, "scheduler admission allocation failed"};
    }
    return {true, SchedulerAdmissionError::None, {}};
}

bool IterationSchedulerRuntime::cancel(RequestId id) noexcept
{
    auto const f = impl_->records.find(id);
    if (f == impl_->records.end() || f->second.state == SchedulerRequestState::Terminal) {
        return false;
    }
    f->second.cancel_requested = true;
    f->second.state = SchedulerRequestState::Cancelling;
    impl_->setState(id, SchedulerRequestState::Cancelling);
    return true;
}

SchedulerIterationResult IterationSchedulerRuntime::runIteration()
{
    Impl& im = *impl_;
    SchedulerIterationResult result;
    result.iteration = ++im.iterations;
    std::size_t const terminals_before = im.terminals.size();
    if (stopped()) {
        im.stopAll();
        result.terminals_produced = static_cast<std::uint32_t>(im.terminals.size() - terminals_before);
        return result;
    }

    struct Selected {
        Impl::Record* rec;
        std::uint32_t steps_left;
    };
    struct Planned {
        Impl::Record* rec;
        GenerationBatchItem item;
        bool prefill;
    };
    auto failAll = [&](std::vector<Selected> const& sel, GenerationError e, char const* why) {
        for (Selected const& s : sel) {
            if (s.rec->state != SchedulerRequestState::Terminal) {
                im.finish(*s.rec, GenerationTerminalReason::Failed, e, why);
            }
        }
    };

    // FIFO selection: at most max_batched_tokens requests, each with its quota.
    std::size_t const take = std::min<std::size_t>(im.queue.size(), im.config.max_batched_tokens);
    std::vector<Selected> selected;
    try {
        selected.reserve(take);
        for (std::size_t i = 0; i < take; ++i) {
            RequestId const id = im.queue.front();
            im.queue.pop_front();
            auto const f = im.records.find(id);
            if (f == im.records.end() || f->second.state == SchedulerRequestState::Terminal) {
                continue;
            }
            Impl::Record& rec = f->second;
            std::uint32_t const prompt_left =
                static_cast<std::uint32_t>(rec.request.prompt_token_ids.size()) - rec.prompt_position;
            std::uint32_t const quota = prompt_left == 0 ? 1 : std::min(prompt_left, im.config.prefill_chunk_size);
            selected.push_back(Selected{&rec, quota});
        }
    } catch (std::bad_alloc const&) {
        failAll(selected, GenerationError::InternalError, "scheduler batch planning allocation failed");
    }

    std::uint32_t budget = im.config.max_batched_tokens;
    std::uint32_t const batch_cap = im.runner->generationMaxBatchSize();
    if (batch_cap == 0) {
        failAll(selected, GenerationError::ModelFailed, "model runner reported a zero maximum batch size");
    }
    // Waves: every selected request with quota left contributes one position.
    while (budget != 0 && batch_cap != 0) {
        std::vector<Planned> plan;
        try {
            plan.reserve(std::min<std::size_t>(selected.size(), budget));
            for (Selected& s : selected) {
                if (s.steps_left == 0 || budget == 0 || s.rec->state == SchedulerRequestState::Terminal) {
                    continue;
                }
                GenerationBatchItem item;
                bool prefill = false;
                if (im.prepare(*s.rec, item, prefill)) {
                    plan.push_back(Planned{s.rec, item, prefill});
                    --s.steps_left;
                    --budget;
                } else {
                    s.steps_left = 0;
                }
            }
        } catch (std::bad_alloc const&) {
            failAll(selected, GenerationError::InternalError, "scheduler model batch allocation failed");
            break;
        }
        if (plan.empty()) {
            break;
        }
        for (std::size_t begin = 0; begin < plan.size(); begin += batch_cap) {
            std::size_t const end = std::min<std::size_t>(plan.size(), begin + batch_cap);
            std::vector<GenerationBatchItem> batch;
            try {
                batch.reserve(end - begin);
                for (std::size_t i = begin; i < end; ++i) {
                    batch.push_back(plan[i].item);
                }
            } catch (std::bad_alloc const&) {
                for (std::size_t i = begin; i < end; ++i) {
                    im.finish(*plan[i].rec, GenerationTerminalReason::Failed,
                        GenerationError::InternalError, "scheduler model batch allocation failed");
                }
                continue;
            }
            GenerationBatchResult out = im.runner->generationForwardBatch(batch);
            ++result.model_forward_batches;
            result.model_forward_tokens += static_cast<std::uint32_t>(batch.size());
            for (std::size_t i = begin; i < end; ++i) {
                ++(plan[i].prefill ? result.prefill_tokens : result.decode_tokens);
            }
            if (!out.success || out.steps.size() != batch.size()) {
                std::string const detail = out.detail.empty()
                    ? "model returned an invalid batch result" : std::move(out.detail);
                for (std::size_t i = begin; i < end; ++i) {
                    im.finish(*plan[i].rec, GenerationTerminalReason::Failed,
                        GenerationError::ModelFailed, detail);
                }
            } else {
                for (std::size_t i = begin; i < end; ++i) {
                    im.apply(*plan[i].rec, std::move(out.steps[i - begin]), plan[i].prefill);
                }
            }
            if (stopped()) {
                break;
            }
        }
        if (stopped()) {
            break;
        }
    }

    im.forward_tokens += result.model_forward_tokens;
    im.forward_batches += result.model_forward_batches;
    im.prefill_tokens += result.prefill_tokens;
    im.decode_tokens += result.decode_tokens;
    for (Selected const& s : selected) {
        if (s.rec->state != SchedulerRequestState::Terminal) {
            if (stopped()) {
                im.stopRecord(*s.rec);
            } else {
                im.queue.push_back(s.rec->request.request_id);
            }
        }
    }
    if (stopped()) {
        im.stopAll();
    }
    result.terminals_produced = static_cast<std::uint32_t>(im.terminals.size() - terminals_before);
    return result;
}

std::vector<GenerationTerminal> IterationSchedulerRuntime::drain()
{
    while (!idle()) {
        SchedulerIterationResult const it = runIteration();
        if (it.model_forward_tokens == 0 && it.terminals_produced == 0 && !stopped()) {
            break;
        }
    }
    return takeTerminals();
}

std::vector<GenerationTerminal> IterationSchedulerRuntime::takeTerminals()
{
    std::vector<GenerationTerminal> out;
    out.swap(impl_->terminals);
    return out;
}

std::optional<SchedulerRequestState> IterationSchedulerRuntime::requestState(RequestId id) const
{
    auto const f = impl_->states.find(id);
    if (f == impl_->states.end()) {
        return std::nullopt;
    }
    return f->second;
}

IterationSchedulerSnapshot IterationSchedulerRuntime::snapshot() const
{
    Impl const& im = *impl_;
    IterationSchedulerSnapshot s;
    s.iteration_count = im.iterations;
    s.accepted_count = im.records.size();
    s.reserved_kv_tokens = im.reserved_kv_tokens;
    s.model_forward_tokens = im.forward_tokens;
    s.model_forward_batches = im.forward_batches;
    s.prefill_tokens = im.prefill_tokens;
    s.decode_tokens = im.decode_tokens;
    s.stopped = stopped();
    for (auto const& e : im.states) {
        switch (e.second) {
        case SchedulerRequestState::Waiting: ++s.waiting_count; break;
        case SchedulerRequestState::Running: ++s.running_count; break;
        case SchedulerRequestState::Cancelling: ++s.cancelling_count; break;
        case SchedulerRequestState::Terminal: ++s.terminal_count; break;
        case SchedulerRequestState::Rejected: ++s.rejected_count; break;
        default: break;
        }
    }
    return s;
}

bool IterationSchedulerRuntime::idle() const noexcept { return impl_->queue.empty(); }
void IterationSchedulerRuntime::stop() noexcept { impl_->stopped.store(true, std::memory_order_release); }
bool IterationSchedulerRuntime::stopped() const noexcept
{
    return impl_->stopped.load(std::memory_order_acquire);
}

} // namespace kimkvcache

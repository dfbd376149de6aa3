// Iteration-level FIFO scheduler. Reference semantics:
// src/engine/iteration_scheduler.cpp (admission gates, quotas, waves, batch
// splitting, terminal handling); the parity tests replay the same
// submissions on both and compare every model batch, counter and terminal.
//
// An iteration takes up to max_batched_tokens requests off the FIFO as
// Lanes, each with its quota of positions. Lanes are then advanced in waves:
// a wave asks every lane with quota left for its next position (in FIFO
// order, while the token budget lasts), and runs the wave as model batches
// of at most the runner's batch size. A Slot is one admitted request: what
// it feeds next, how it takes a model step, how it ends.
#include "iteration_scheduler.h"

#include <algorithm>
#include <chrono>
#include <deque>
#include <new>
#include <unordered_map>

namespace kimkvcache {
namespace {

using Clock = std::chrono::steady_clock;

std::uint64_t elapsedNs(Clock::time_point from, Clock::time_point to) noexcept
{
    auto const ns = std::chrono::duration_cast<std::chrono::nanoseconds>(to - from).count();
    return ns > 0 ? static_cast<std::uint64_t>(ns) : 0;
}

// Committed KV tokens a request can reach: prompt + completion minus the
// last generated token, which never goes back through the model.
std::uint64_t kvTokensNeeded(GenerationRequest const& r) noexcept
{
    return r.prompt_token_ids.size() + std::uint64_t(r.sampling.max_new_tokens) - 1;
}

struct Slot {
    GenerationRequest req;
    GenerationTerminal out;
    SchedulerRequestState state{SchedulerRequestState::Waiting};
    std::uint64_t kv_tokens{0};
    std::uint32_t fed{0};          // prompt positions that went through the model (or came as a prefix)
    bool kv_open{false};
    bool cancel{false};
    Clock::time_point admitted{};
    bool emitted{false};
    Clock::time_point first_emit{};
    Clock::time_point last_emit{};

    [[nodiscard]] std::uint32_t promptLen() const noexcept
    {
        return static_cast<std::uint32_t>(req.prompt_token_ids.size());
    }
    [[nodiscard]] bool prefilling() const noexcept { return fed < promptLen(); }
    [[nodiscard]] bool closed() const noexcept { return state == SchedulerRequestState::Terminal; }
    [[nodiscard]] bool cancelSeen() const noexcept
    {
        return cancel || (req.cancellation != nullptr && req.cancellation->cancelled());
    }
    // The position this request feeds next: a prompt token, or its last
    // output fed back.
    [[nodiscard]] GenerationBatchItem nextItem() const
    {
        if (prefilling()) {
            return GenerationBatchItem{req.request_id, req.prompt_token_ids[fed], fed};
        }
        std::uint32_t const pos = out.usage.prompt_tokens + static_cast<std::uint32_t>(out.output_token_ids.size()) - 1;
        return GenerationBatchItem{req.request_id, out.output_token_ids.back(), pos};
    }
};

struct Lane {
    Slot* slot;
    std::uint32_t quota;
};

// A planned model position of a wave.
struct Cell {
    Slot* slot;
    GenerationBatchItem item;
    bool prompt;
};

} // namespace

class IterationSchedulerRuntime::Impl final {
public:
    Impl(EngineKvBackend& k, GenerationModelRunner& r, IterationSchedulerConfig c) noexcept
        : kv(&k), runner(&r), config(c)
    {
    }

    EngineKvBackend* kv;
    GenerationModelRunner* runner;
    IterationSchedulerConfig config;
    std::atomic<bool> halted{false};
    std::unordered_map<RequestId, Slot> slots;
    std::unordered_map<RequestId, SchedulerRequestState> status;  // every id ever submitted
    std::deque<RequestId> fifo;
    std::vector<GenerationTerminal> done;
    std::uint64_t iterations{0};
    std::uint64_t kv_reserved{0};
    SchedulerIterationResult totals{};

    [[nodiscard]] bool stopped() const noexcept { return halted.load(std::memory_order_acquire); }

    void mark(Slot& s, SchedulerRequestState st)
    {
        s.state = st;
        auto const f = status.find(s.req.request_id);
        if (f != status.end()) {
            f->second = st;
        }
    }

    // ---- admission ----

    SchedulerAdmissionResult refuse(RequestId id, SchedulerAdmissionError e, std::string why, bool record)
    {
        if (record && id != kInvalidRequestId) {
            try {
                status.emplace(id, SchedulerRequestState::Rejected);
            } catch (std::bad_alloc const&) {
                return {false, SchedulerAdmissionError::InternalError, "no memory to record the rejection"};
            }
        }
        return {false, e, std::move(why)};
    }

    std::optional<std::string> invalid(GenerationRequest const& r) const
    {
        if (!config.valid()) {
            return std::string("the scheduler configuration is invalid");
        }
        TinyLlamaConfig const m = runner->generationConfig();
        std::size_t const prompt = r.prompt_token_ids.size();
        if (!m.valid() || r.request_id == kInvalidRequestId || prompt == 0 || r.sampling.max_new_tokens == 0) {
            return std::string("a request needs an id, a prompt, max_new_tokens and a valid model");
        }
        if (prompt > m.max_position_embeddings || r.sampling.max_new_tokens > m.max_position_embeddings - prompt + 1) {
            return std::string("prompt plus completion is longer than the model's positions");
        }
        if (r.sampling.eos_token_id.value_or(m.eos_token_id) >= m.vocabulary_size) {
            return std::string("EOS token id is outside the vocabulary");
        }
        if (std::any_of(r.prompt_token_ids.begin(), r.prompt_token_ids.end(),
                [&](std::uint32_t t) { return t >= m.vocabulary_size; })) {
            return std::string("a prompt token id is outside the vocabulary");
        }
        if (r.kv_prefix_tokens >= prompt) {
            return std::string("the KV prefix must leave at least one prompt position to feed");
        }
        return std::nullopt;
    }

    // ---- endings ----

    void close(Slot& s, GenerationTerminalReason reason, GenerationError error, std::string detail)
    {
        if (s.closed()) {
            return;
        }
        GenerationTerminal& t = s.out;
        t.reason = reason;
        t.error = error;
        t.detail = std::move(detail);
        t.usage.completion_tokens = static_cast<std::uint32_t>(t.output_token_ids.size());
        t.usage.total_tokens = t.usage.prompt_tokens + t.usage.completion_tokens;
        if (s.kv_open) {
            s.kv_open = false;
            EngineKvStatus const released = kv->releaseRequest(s.req.request_id);
            if (!released.ok()) {
                t.reason = GenerationTerminalReason::Failed;
                t.error = GenerationError::KvBackendFailed;
                t.detail = std::string("the KV request could not be released: ") + std::string(toString(released.error));
            }
        }
        t.metrics.e2e_ns = elapsedNs(s.admitted, Clock::now());
        if (s.emitted) {
            t.metrics.ttft_ns = elapsedNs(s.admitted, s.first_emit);
            std::size_t const n = t.output_token_ids.size();
            t.metrics.tpot_ns = n > 1 ? elapsedNs(s.first_emit, s.last_emit) / (n - 1) : 0;
        }
        mark(s, SchedulerRequestState::Terminal);
        kv_reserved -= s.kv_tokens;
        try {
            done.push_back(t);
        } catch (std::bad_alloc const&) {
        }
    }

    void closeStopped(Slot& s)
    {
        close(s, GenerationTerminalReason::RuntimeStopped, GenerationError::RuntimeStopped,
            "runtime stopped between iterations");
    }

    void closeCancelled(Slot& s)
    {
        close(s, GenerationTerminalReason::Cancelled, GenerationError::None, "request cancelled between iterations");
    }

    void closeFailed(Slot& s, GenerationError e, std::string why)
    {
        close(s, GenerationTerminalReason::Failed, e, std::move(why));
    }

    void stopQueued()
    {
        while (!fifo.empty()) {
            auto const f = slots.find(fifo.front());
            fifo.pop_front();
            if (f != slots.end() && !f->second.closed()) {
                closeStopped(f->second);
            }
        }
    }

    // ---- one model position of a slot ----

    // True when the slot may feed a position now: not cancelled or stopped,
    // and its KV request open (created on first use unless it came with a
    // committed prefix).
    bool ready(Slot& s)
    {
        if (s.cancelSeen()) {
            closeCancelled(s);
            return false;
        }
        if (stopped()) {
            closeStopped(s);
            return false;
        }
        if (!s.kv_open) {
            if (s.req.kv_prefix_tokens == 0) {
                EngineKvStatus const made = kv->createRequest(s.req.request_id);
                if (!made.ok()) {
                    closeFailed(s, GenerationError::KvBackendFailed,
                        std::string("the KV request could not be created: ") + std::string(toString(made.error)));
                    return false;
                }
            }
            s.kv_open = true;
            mark(s, SchedulerRequestState::Running);
        }
        return true;
    }

    // Takes the model's answer for `positions` positions of the slot (one
    // unless a fused prompt chunk).
    void take(Slot& s, GenerationStepResult step, std::uint32_t prompt_positions)
    {
        TinyLlamaConfig const m = runner->generationConfig();
        if (!step.success) {
            closeFailed(s, GenerationError::ModelFailed, std::move(step.detail));
            return;
        }
        if (step.greedy_token_id >= m.vocabulary_size) {
            closeFailed(s, GenerationError::ModelFailed, "the model returned a token outside the vocabulary");
            return;
        }
        s.fed += prompt_positions;
        // After a model step, stop wins over cancellation.
        if (stopped()) {
            closeStopped(s);
            return;
        }
        if (s.cancelSeen()) {
            closeCancelled(s);
            return;
        }
        if (s.prefilling()) {
            return;  // a prompt position's prediction is not an output
        }
        try {
            s.out.output_token_ids.push_back(step.greedy_token_id);
        } catch (std::bad_alloc const&) {
            closeFailed(s, GenerationError::InternalError, "no memory for the completion");
            return;
        }
        s.last_emit = Clock::now();
        if (!s.emitted) {
            s.emitted = true;
            s.first_emit = s.last_emit;
        }
        if (step.greedy_token_id == s.req.sampling.eos_token_id.value_or(m.eos_token_id)) {
            close(s, GenerationTerminalReason::EosToken, GenerationError::None, "EOS generated");
        } else if (s.out.output_token_ids.size() == s.req.sampling.max_new_tokens) {
            close(s, GenerationTerminalReason::MaxNewTokens, GenerationError::None, "max_new_tokens generated");
        }
    }

    // ---- an iteration ----

    std::vector<Lane> pickLanes(SchedulerIterationResult&)
    {
        std::vector<Lane> lanes;
        std::size_t n = std::min<std::size_t>(fifo.size(), config.max_batched_tokens);
        try {
            lanes.reserve(n);
            for (; n != 0; --n) {
                auto const f = slots.find(fifo.front());
                fifo.pop_front();
                if (f == slots.end() || f->second.closed()) {
                    continue;
                }
                Slot& s = f->second;
                std::uint32_t const left = s.promptLen() - s.fed;
                lanes.push_back(Lane{&s, left == 0 ? 1u : std::min(left, config.prefill_chunk_size)});
            }
        } catch (std::bad_alloc const&) {
            failLanes(lanes, GenerationError::InternalError, "no memory to plan the iteration");
        }
        return lanes;
    }

    void failLanes(std::vector<Lane> const& lanes, GenerationError e, char const* why)
    {
        for (Lane const& l : lanes) {
            closeFailed(*l.slot, e, why);
        }
    }

    // Fused prompt chunks: one model call per prompt lane for its quota
    // (bounded by the token budget); decode lanes are left for the waves.
    void fusedPrompts(std::vector<Lane>& lanes, std::uint32_t& budget, SchedulerIterationResult& r)
    {
        for (Lane& l : lanes) {
            Slot& s = *l.slot;
            if (budget == 0 || l.quota == 0 || s.closed() || !s.prefilling()) {
                continue;
            }
            if (!ready(s)) {
                l.quota = 0;
                continue;
            }
            std::uint32_t const n = std::min(l.quota, budget);
            GenerationStepResult step = runner->generationPrefill(s.req.request_id, s.req.prompt_token_ids.data() + s.fed,
                n, s.fed);
            l.quota = 0;
            budget -= n;
            ++r.model_forward_batches;
            r.model_forward_tokens += n;
            r.prefill_tokens += n;
            take(s, std::move(step), n);
            if (stopped()) {
                return;
            }
        }
    }

    // The next wave: one position of every lane with quota left, in FIFO
    // order, while the budget lasts.
    std::vector<Cell> nextWave(std::vector<Lane>& lanes, std::uint32_t& budget)
    {
        std::vector<Cell> wave;
        wave.reserve(std::min<std::size_t>(lanes.size(), budget));
        for (Lane& l : lanes) {
            if (budget == 0) {
                break;
            }
            if (l.quota == 0 || l.slot->closed()) {
                continue;
            }
            if (!ready(*l.slot)) {
                l.quota = 0;
                continue;
            }
            wave.push_back(Cell{l.slot, l.slot->nextItem(), l.slot->prefilling()});
            --l.quota;
            --budget;
        }
        return wave;
    }

    // Runs a wave as model batches of at most `cap` positions.
    void runWave(std::vector<Cell> const& wave, std::uint32_t cap, SchedulerIterationResult& r)
    {
        for (std::size_t lo = 0; lo < wave.size(); lo += cap) {
            std::size_t const hi = std::min<std::size_t>(wave.size(), lo + cap);
            std::vector<GenerationBatchItem> batch;
            try {
                batch.reserve(hi - lo);
                for (std::size_t i = lo; i < hi; ++i) {
                    batch.push_back(wave[i].item);
                }
            } catch (std::bad_alloc const&) {
                for (std::size_t i = lo; i < hi; ++i) {
                    closeFailed(*wave[i].slot, GenerationError::InternalError, "no memory for the model batch");
                }
                continue;
            }
            GenerationBatchResult res = runner->generationForwardBatch(batch);
            ++r.model_forward_batches;
            r.model_forward_tokens += static_cast<std::uint32_t>(batch.size());
            for (std::size_t i = lo; i < hi; ++i) {
                ++(wave[i].prompt ? r.prefill_tokens : r.decode_tokens);
            }
            bool const well_formed = res.success && res.steps.size() == batch.size();
            std::string const why = well_formed ? std::string()
                : (res.detail.empty() ? std::string("the model returned a malformed batch result") : res.detail);
            for (std::size_t i = lo; i < hi; ++i) {
                if (well_formed) {
                    take(*wave[i].slot, std::move(res.steps[i - lo]), wave[i].prompt ? 1u : 0u);
                } else {
                    closeFailed(*wave[i].slot, GenerationError::ModelFailed, why);
                }
            }
            if (stopped()) {
                return;
            }
        }
    }

    SchedulerIterationResult iterate()
    {
        SchedulerIterationResult r;
        r.iteration = ++iterations;
        std::size_t const ended_before = done.size();
        if (stopped()) {
            stopQueued();
            r.terminals_produced = static_cast<std::uint32_t>(done.size() - ended_before);
            return r;
        }
        std::vector<Lane> lanes = pickLanes(r);
        std::uint32_t budget = config.max_batched_tokens;
        std::uint32_t const cap = runner->generationMaxBatchSize();
        if (cap == 0) {
            failLanes(lanes, GenerationError::ModelFailed, "the model runner reports a zero batch size");
        } else {
            if (config.fused_prefill && runner->generationSupportsPrefill()) {
                fusedPrompts(lanes, budget, r);
            }
            while (budget != 0) {
                std::vector<Cell> wave;
                try {
                    wave = nextWave(lanes, budget);
                } catch (std::bad_alloc const&) {
                    failLanes(lanes, GenerationError::InternalError, "no memory for the model batch");
                    break;
                }
                if (wave.empty()) {
                    break;
                }
                runWave(wave, cap, r);
                if (stopped()) {
                    break;
                }
            }
        }
        totals.model_forward_tokens += r.model_forward_tokens;
        totals.model_forward_batches += r.model_forward_batches;
        totals.prefill_tokens += r.prefill_tokens;
        totals.decode_tokens += r.decode_tokens;
        // Live lanes go back to the end of the FIFO (or end, on a stop).
        for (Lane const& l : lanes) {
            if (l.slot->closed()) {
                continue;
            }
            if (stopped()) {
                closeStopped(*l.slot);
            } else {
                fifo.push_back(l.slot->req.request_id);
            }
        }
        if (stopped()) {
            stopQueued();
        }
        r.terminals_produced = static_cast<std::uint32_t>(done.size() - ended_before);
        return r;
    }
};

IterationSchedulerRuntime::IterationSchedulerRuntime(EngineKvBackend& kv, GenerationModelRunner& runner,
    IterationSchedulerConfig config)
    : impl_(std::make_unique<Impl>(kv, runner, config))
{
}

IterationSchedulerRuntime::~IterationSchedulerRuntime()
{
    if (impl_ != nullptr) {
        impl_->halted.store(true, std::memory_order_release);
        impl_->stopQueued();
    }
}

SchedulerAdmissionResult IterationSchedulerRuntime::submit(GenerationRequest request)
{
    Impl& im = *impl_;
    RequestId const id = request.request_id;
    if (stopped()) {
        return im.refuse(id, SchedulerAdmissionError::RuntimeStopped, "runtime is stopped", true);
    }
    if (im.status.count(id) != 0) {
        return im.refuse(id, SchedulerAdmissionError::DuplicateRequest, "this request id was submitted before", false);
    }
    if (std::optional<std::string> why = im.invalid(request)) {
        return im.refuse(id, SchedulerAdmissionError::InvalidArgument, std::move(*why), true);
    }
    if (snapshot().activeCount() >= im.config.max_active_requests) {
        return im.refuse(id, SchedulerAdmissionError::MaxActiveRequests, "max_active_requests reached", true);
    }
    std::uint64_t const need = kvTokensNeeded(request);
    if (need > im.config.max_kv_tokens || im.kv_reserved > im.config.max_kv_tokens - need) {
        return im.refuse(id, SchedulerAdmissionError::KvTokenBudget, "max_kv_tokens would be exceeded", true);
    }
    try {
        Slot s;
        s.kv_tokens = need;
        s.fed = request.kv_prefix_tokens;
        s.out.request_id = id;
        s.out.usage.prompt_tokens = static_cast<std::uint32_t>(request.prompt_token_ids.size());
        s.req = std::move(request);
        s.admitted = Clock::now();
        im.slots.emplace(id, std::move(s));
        try {
            im.status.emplace(id, SchedulerRequestState::Waiting);
            im.fifo.push_back(id);
        } catch (...) {
            im.status.erase(id);
            im.slots.erase(id);
            throw;
        }
    } catch (std::bad_alloc const&) {
        return {false, SchedulerAdmissionError::InternalError, "no memory to admit the request"};
    }
    im.kv_reserved += need;
    return {true, SchedulerAdmissionError::None, {}};
}

bool IterationSchedulerRuntime::cancel(RequestId id) noexcept
{
    auto const f = impl_->slots.find(id);
    if (f == impl_->slots.end() || f->second.closed()) {
        return false;
    }
    f->second.cancel = true;
    impl_->mark(f->second, SchedulerRequestState::Cancelling);
    return true;
}

SchedulerIterationResult IterationSchedulerRuntime::runIteration() { return impl_->iterate(); }

std::vector<GenerationTerminal> IterationSchedulerRuntime::drain()
{
    while (!idle()) {
        SchedulerIterationResult const r = runIteration();
        bool const progressed = r.model_forward_tokens != 0 || r.terminals_produced != 0;
        if (!progressed && !stopped()) {
            break;
        }
    }
    return takeTerminals();
}

std::vector<GenerationTerminal> IterationSchedulerRuntime::takeTerminals()
{
    std::vector<GenerationTerminal> out;
    out.swap(impl_->done);
    return out;
}

std::optional<SchedulerRequestState> IterationSchedulerRuntime::requestState(RequestId id) const
{
    auto const f = impl_->status.find(id);
    return f == impl_->status.end() ? std::nullopt : std::optional<SchedulerRequestState>(f->second);
}

IterationSchedulerSnapshot IterationSchedulerRuntime::snapshot() const
{
    Impl const& im = *impl_;
    IterationSchedulerSnapshot s;
    s.iteration_count = im.iterations;
    s.accepted_count = im.slots.size();
    s.reserved_kv_tokens = im.kv_reserved;
    s.model_forward_tokens = im.totals.model_forward_tokens;
    s.model_forward_batches = im.totals.model_forward_batches;
    s.prefill_tokens = im.totals.prefill_tokens;
    s.decode_tokens = im.totals.decode_tokens;
    s.stopped = stopped();
    for (auto const& [id, st] : im.status) {
        static_cast<void>(id);
        switch (st) {
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

bool IterationSchedulerRuntime::idle() const noexcept { return impl_->fifo.empty(); }
void IterationSchedulerRuntime::stop() noexcept { impl_->halted.store(true, std::memory_order_release); }
bool IterationSchedulerRuntime::stopped() const noexcept { return impl_->stopped(); }

} // namespace kimkvcache

// TEST INFRASTRUCTURE ONLY — C shim over the reference's own generation loop
// and iteration scheduler (src/engine/generation.cpp, iteration_scheduler.cpp),
// driven by the same SPI test doubles as the product's kkrt_fake_* (a KV
// backend that tracks request lifecycles, a model runner whose greedy token
// is a fixed hash of (request, token, position) and which logs its batches).
// Exposes kref_sched_* / kref_generate / kref_fake_* with the signatures of
// the kkrt_* twins in include/kk_runtime.h.
#include "../include/kk_runtime.h"

#include "kim-kv/engine/iteration_scheduler.h"

#include <memory>
#include <new>
#include <unordered_set>
#include <vector>

using namespace kimkvcache;

namespace {

class FakeBackend final : public EngineKvBackend {
public:
    EngineKvBackendKind kind() const noexcept override { return EngineKvBackendKind::Heterogeneous; }
    EngineKvConfig config() const noexcept override { return {KvLayout{1, 1, 64}, 1, 1}; }
    EngineKvStatus createRequest(RequestId id) override
    {
        if (id == kInvalidRequestId) return {EngineKvError::InvalidArgument};
        return live_.insert(id).second ? EngineKvStatus{} : EngineKvStatus{EngineKvError::RequestAlreadyExists};
    }
    EngineKvStatus forkRequest(RequestId s, RequestId c) override
    {
        if (!live_.count(s)) return {EngineKvError::RequestNotFound};
        return live_.insert(c).second ? EngineKvStatus{} : EngineKvStatus{EngineKvError::RequestAlreadyExists};
    }
    EngineKvStatus releaseRequest(RequestId id) override
    {
        return live_.erase(id) ? EngineKvStatus{} : EngineKvStatus{EngineKvError::RequestNotFound};
    }
    TokenReserveResult reserveToken(ReserveTokenRequest const&) override
    {
        TokenReserveResult r;
        r.status = {EngineKvError::InvalidState};
        return r;
    }
    EngineKvBackendSnapshot snapshot() const override
    {
        EngineKvBackendSnapshot s;
        s.request_count = live_.size();
        return s;
    }
    bool checkInvariants() const override { return true; }

private:
    std::unordered_set<RequestId> live_;
};

class FakeRunner final : public GenerationModelRunner {
public:
    FakeRunner(uint32_t vocab, uint32_t max_batch, uint32_t eos, uint32_t positions, RequestId fail)
        : vocab_(vocab), max_batch_(max_batch), fail_(fail)
    {
        cfg_ = TinyLlamaConfig{64, 64, 1, 1, 1, 64, vocab, positions, 0, eos, 1e-5F, 10000.0F, false};
    }
    TinyLlamaConfig generationConfig() const noexcept override { return cfg_; }
    GenerationStepResult generationForwardToken(RequestId r, uint32_t t, uint32_t p) override
    {
        return generationForwardBatch({GenerationBatchItem{r, t, p}}).steps.at(0);
    }
    GenerationBatchResult generationForwardBatch(std::vector<GenerationBatchItem> const& batch) override
    {
        GenerationBatchResult out;
        sizes.push_back(static_cast<uint32_t>(batch.size()));
        for (GenerationBatchItem const& it : batch) {
            items.push_back(it.request_id);
            items.push_back(it.token_id);
            items.push_back(it.expected_position);
            if (it.request_id == fail_) {
                out.steps.push_back({false, 0, "injected model failure"});
                continue;
            }
            uint64_t h = it.request_id * 0x9e3779b97f4a7c15ull ^ (uint64_t(it.token_id) << 20)
                ^ it.expected_position;
            h ^= h >> 29;
            h *= 0xbf58476d1ce4e5b9ull;
            h ^= h >> 32;
            out.steps.push_back({true, static_cast<uint32_t>(h % vocab_), {}});
        }
        out.success = true;
        return out;
    }
    uint32_t generationMaxBatchSize() const noexcept override { return max_batch_; }

    std::vector<uint32_t> sizes;
    std::vector<uint64_t> items;

private:
    TinyLlamaConfig cfg_{};
    uint32_t vocab_;
    uint32_t max_batch_;
    RequestId fail_;
};

EngineKvBackend* KV(void* p) { return static_cast<EngineKvBackend*>(p); }
GenerationModelRunner* RUN(void* p) { return static_cast<GenerationModelRunner*>(p); }
struct Sched {
    std::unique_ptr<IterationSchedulerRuntime> rt;
};

uint32_t terminalsOut(std::vector<GenerationTerminal> const& ts, kk_terminal* out, uint32_t cap,
    uint32_t* tokens, uint32_t token_cap)
{
    uint32_t n = 0, used = 0;
    for (GenerationTerminal const& t : ts) {
        if (n >= cap) break;
        kk_terminal& o = out[n++];
        o.request_id = t.request_id;
        o.reason = static_cast<uint8_t>(t.reason);
        o.error = static_cast<uint8_t>(t.error);
        o.reserved = 0;
        o.token_count = static_cast<uint32_t>(t.output_token_ids.size());
        o.prompt_tokens = t.usage.prompt_tokens;
        o.completion_tokens = t.usage.completion_tokens;
        o.ttft_ns = t.metrics.ttft_ns;
        o.tpot_ns = t.metrics.tpot_ns;
        o.e2e_ns = t.metrics.e2e_ns;
        for (uint32_t tok : t.output_token_ids) {
            if (tokens != nullptr && used < token_cap) tokens[used] = tok;
            ++used;
        }
    }
    return n;
}

} // namespace

extern "C" {

KK_API void* kref_fake_backend_create(void) { return static_cast<EngineKvBackend*>(new FakeBackend); }
KK_API void kref_fake_backend_destroy(void* b) { delete KV(b); }
KK_API void* kref_fake_runner_create(uint32_t vocab, uint32_t max_batch, uint32_t eos, uint32_t positions,
    uint64_t fail)
{
    return static_cast<GenerationModelRunner*>(new FakeRunner(vocab, max_batch, eos, positions, fail));
}
KK_API void kref_fake_runner_destroy(void* r) { delete RUN(r); }
KK_API uint32_t kref_fake_runner_log(void* r, uint32_t* sizes, uint32_t cap_b, uint64_t* items, uint32_t cap_i)
{
    auto* f = dynamic_cast<FakeRunner*>(RUN(r));
    for (std::size_t i = 0; i < f->sizes.size() && i < cap_b; ++i) sizes[i] = f->sizes[i];
    for (std::size_t i = 0; i < f->items.size() && i < cap_i; ++i) items[i] = f->items[i];
    return static_cast<uint32_t>(f->sizes.size());
}

KK_API void* kref_sched_create(void* b, void* r, uint32_t max_active, uint32_t max_tokens,
    uint64_t max_kv, uint32_t chunk)
{
    auto* s = new Sched;
    s->rt = std::make_unique<IterationSchedulerRuntime>(*KV(b), *RUN(r),
        IterationSchedulerConfig{max_active, max_tokens, max_kv, chunk});
    return s;
}
KK_API void kref_sched_destroy(void* s) { delete static_cast<Sched*>(s); }
KK_API int kref_sched_submit(void* s, uint64_t id, const uint32_t* prompt, uint32_t len, uint32_t max_new,
    int64_t eos)
{
    GenerationRequest req;
    req.request_id = id;
    req.prompt_token_ids.assign(prompt, prompt + len);
    req.sampling.max_new_tokens = max_new;
    if (eos >= 0) req.sampling.eos_token_id = static_cast<uint32_t>(eos);
    return static_cast<int>(static_cast<Sched*>(s)->rt->submit(std::move(req)).error);
}
KK_API int kref_sched_cancel(void* s, uint64_t id) { return static_cast<Sched*>(s)->rt->cancel(id) ? 1 : 0; }
KK_API void kref_sched_run_iteration(void* s, kk_iteration* out)
{
    SchedulerIterationResult const r = static_cast<Sched*>(s)->rt->runIteration();
    *out = kk_iteration{r.iteration, r.model_forward_tokens, r.model_forward_batches, r.prefill_tokens,
        r.decode_tokens, r.terminals_produced, 0};
}
KK_API void kref_sched_stop(void* s) { static_cast<Sched*>(s)->rt->stop(); }
KK_API int kref_sched_idle(void* s) { return static_cast<Sched*>(s)->rt->idle() ? 1 : 0; }
KK_API uint32_t kref_sched_drain(void* s, kk_terminal* out, uint32_t cap, uint32_t* tokens, uint32_t tcap)
{
    return terminalsOut(static_cast<Sched*>(s)->rt->drain(), out, cap, tokens, tcap);
}
KK_API uint32_t kref_sched_take_terminals(void* s, kk_terminal* out, uint32_t cap, uint32_t* tokens,
    uint32_t tcap)
{
    return terminalsOut(static_cast<Sched*>(s)->rt->takeTerminals(), out, cap, tokens, tcap);
}
KK_API int kref_generate(void* b, void* r, uint64_t id, const uint32_t* prompt, uint32_t len,
    uint32_t max_new, int64_t eos, kk_terminal* out, uint32_t* tokens, uint32_t tcap)
{
    SingleRequestGenerationRuntime rt(*KV(b), *RUN(r));
    GenerationRequest req;
    req.request_id = id;
    req.prompt_token_ids.assign(prompt, prompt + len);
    req.sampling.max_new_tokens = max_new;
    if (eos >= 0) req.sampling.eos_token_id = static_cast<uint32_t>(eos);
    std::vector<GenerationTerminal> one{rt.generate(req)};
    return static_cast<int>(terminalsOut(one, out, 1, tokens, tcap));
}

} // extern "C"

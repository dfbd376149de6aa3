// C ABI over the CUDA KV backend, per-layer token transactions, the model
// runner, the generation loops, and the SPI test doubles (declarations and
// reference citations in include/kk_runtime.h).
#include "../../../include/kk_runtime.h"
#include "../cuda/cuda_backend.h"
#include "../cuda/model_runner.h"
#include "../host/iteration_scheduler.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>
#include <unordered_set>
#include <vector>

using namespace kimkvcache;

namespace {

// Test double: a KV backend that only tracks request lifecycles (the
// reference contract tests use the same kind of fake).
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

// Test double: greedy token = fixed hash of (request, token, position); logs batches.
class FakeRunner final : public GenerationModelRunner {
public:
    FakeRunner(std::uint32_t vocab, std::uint32_t max_batch, std::uint32_t eos, std::uint32_t positions,
        RequestId fail_request)
        : vocab_(vocab), max_batch_(max_batch), fail_(fail_request)
    {
        cfg_ = TinyLlamaConfig{64, 64, 1, 1, 1, 64, vocab, positions, 0, eos, 1e-5F, 10000.0F, false};
    }
    TinyLlamaConfig generationConfig() const noexcept override { return cfg_; }
    GenerationStepResult generationForwardToken(RequestId r, std::uint32_t t, std::uint32_t p) override
    {
        return generationForwardBatch({GenerationBatchItem{r, t, p}}).steps.at(0);
    }
    GenerationBatchResult generationForwardBatch(std::vector<GenerationBatchItem> const& batch) override
    {
        GenerationBatchResult out;
        sizes.push_back(static_cast<std::uint32_t>(batch.size()));
        for (GenerationBatchItem const& it : batch) {
            items.push_back(it.request_id);
            items.push_back(it.token_id);
            items.push_back(it.expected_position);
            if (it.request_id == fail_) {
                out.steps.push_back({false, 0, "injected model failure"});
                continue;
            }
            std::uint64_t h = it.request_id * 0x9e3779b97f4a7c15ull ^ (std::uint64_t(it.token_id) << 20)
                ^ it.expected_position;
            h ^= h >> 29;
            h *= 0xbf58476d1ce4e5b9ull;
            h ^= h >> 32;
            out.steps.push_back({true, static_cast<std::uint32_t>(h % vocab_), {}});
        }
        out.success = true;
        return out;
    }
    std::uint32_t generationMaxBatchSize() const noexcept override { return max_batch_; }

    std::vector<std::uint32_t> sizes;
    std::vector<std::uint64_t> items;

private:
    TinyLlamaConfig cfg_{};
    std::uint32_t vocab_;
    std::uint32_t max_batch_;
    RequestId fail_;
};

EngineKvBackend* KV(void* p) { return static_cast<EngineKvBackend*>(p); }
GenerationModelRunner* RUN(void* p) { return static_cast<GenerationModelRunner*>(p); }

struct Sched {
    std::unique_ptr<IterationSchedulerRuntime> rt;
};

void tableOut(BlockTable const& t, kk_table_out* out)
{
    out->count = static_cast<uint32_t>(t.entries().size());
    out->version = t.version();
    for (std::size_t i = 0; i < t.entries().size() && i < out->capacity; ++i) {
        MappingEntry const& m = t.entries()[i];
        out->entries[i] = kk_entry{m.logical_token_begin, m.valid_tokens,
            static_cast<uint8_t>(m.kind), 0, m.handle.slot, m.handle.generation};
    }
}

uint32_t terminalsOut(std::vector<GenerationTerminal> const& ts, kk_terminal* out, uint32_t cap,
    uint32_t* tokens, uint32_t token_cap)
{
    uint32_t n = 0;
    uint32_t used = 0;
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

void* kkrt_backend_create(uint32_t layers, uint32_t kv_heads, uint32_t head_dim, uint32_t q_heads,
    uint64_t ws_bytes, uint32_t micro, uint32_t extent)
{
    EngineKvConfig const c{KvLayout{layers, kv_heads, head_dim}, q_heads, static_cast<std::size_t>(ws_bytes)};
    return createHeterogeneousCudaEngineKvBackend(c, micro, extent).release();
}
void* kkrt_fixed_backend_create(uint32_t layers, uint32_t kv_heads, uint32_t head_dim, uint32_t q_heads,
    uint64_t ws_bytes, uint32_t tokens_per_page, uint32_t page_capacity)
{
    if (tokens_per_page > 0xffffu) {
        return nullptr;
    }
    EngineKvConfig const c{KvLayout{layers, kv_heads, head_dim}, q_heads, static_cast<std::size_t>(ws_bytes)};
    return createFixedCudaEngineKvBackend(c, static_cast<std::uint16_t>(tokens_per_page), page_capacity).release();
}
int kkrt_backend_kind(void* b) { return static_cast<int>(KV(b)->kind()); }
void kkrt_backend_destroy(void* b) { delete KV(b); }
int kkrt_backend_create_request(void* b, uint64_t id) { return int(KV(b)->createRequest(id).error); }
int kkrt_backend_fork(void* b, uint64_t s, uint64_t c) { return int(KV(b)->forkRequest(s, c).error); }
int kkrt_backend_release(void* b, uint64_t id) { return int(KV(b)->releaseRequest(id).error); }
int kkrt_backend_check_invariants(void* b) { return KV(b)->checkInvariants() ? 1 : 0; }

void kkrt_backend_snapshot(void* b, kk_backend_snapshot* o)
{
    EngineKvBackendSnapshot const s = KV(b)->snapshot();
    *o = kk_backend_snapshot{s.request_count, s.active_transaction_count, s.committed_token_count,
        s.batched_attention_submissions, s.batched_attention_lanes, s.allocated_primary_pages,
        s.allocated_secondary_pages, s.storage_reserved_bytes};
}

int kkrt_backend_inject_failure(void* b, int point)
{
    return injectCudaEngineFailureOnce(*KV(b), point == 0 ? CudaFailurePoint::Submission
                                                          : CudaFailurePoint::Completion) ? 1 : 0;
}

int kkrt_backend_pools(void* b, void* out)
{
    kk_kv_pools const* p = cudaBackendPools(*KV(b));
    if (p == nullptr) return 0;
    std::memcpy(out, p, sizeof(kk_kv_pools));
    return 1;
}

int kkrt_backend_block_table(void* b, uint64_t id, kk_table_out* out)
{
    BlockTable t;
    if (!cudaBackendTable(*KV(b), id, t)) return 0;
    tableOut(t, out);
    return 1;
}

int kkrt_backend_append(void* b, uint64_t id, uint32_t n) { return int(cudaBackendAppend(*KV(b), id, n).error); }
int kkrt_backend_seal(void* b, uint64_t id) { return int(cudaBackendSeal(*KV(b), id).error); }
int kkrt_backend_promote(void* b, uint64_t id, uint32_t begin, void* stream)
{
    return int(cudaBackendPromote(*KV(b), id, begin, stream).error);
}

int kkrt_backend_gather(void* b, uint64_t id, void* device_output, void* stream)
{
    return int(cudaBackendGather(*KV(b), id, device_output, stream).error);
}

void* kkrt_txn_reserve(void* b, uint64_t id, uint32_t expected, void* stream, int* status)
{
    TokenReserveResult r = KV(b)->reserveToken(ReserveTokenRequest{id, expected, stream});
    if (status != nullptr) *status = static_cast<int>(r.status.error);
    if (!r.ok()) return nullptr;
    return new (std::nothrow) TokenTransaction(std::move(r.transaction));
}

static TokenTransaction* T(void* p) { return static_cast<TokenTransaction*>(p); }

int kkrt_txn_write_layer(void* t, uint32_t layer, const void* k, const void* v)
{
    return int(T(t)->writeLayer(LayerKvWrite{layer, static_cast<KvScalar const*>(k),
        static_cast<KvScalar const*>(v)}).error);
}

int kkrt_txn_attend_layer(void* t, uint32_t layer, const void* q, void* o, void* ws, uint64_t ws_bytes,
    float scale)
{
    return int(T(t)->attendLayer(PagedDecodeRequest{layer, static_cast<KvScalar const*>(q),
        static_cast<KvScalar*>(o), ws, static_cast<std::size_t>(ws_bytes), scale}).error);
}

namespace {

// Device batch item buffer of kkrt_txn_attend_batch: grown on demand, never
// shrunk (a replaced buffer is kept: a launch queued earlier may still read it).
DevicePagedDecodeBatchItem* batchItemScratch(uint32_t n)
{
    static std::mutex mutex;
    static std::vector<DevicePagedDecodeBatchItem*> buffers;
    static uint32_t capacity = 0;
    std::lock_guard<std::mutex> lock(mutex);
    if (n > capacity || buffers.empty()) {
        uint32_t const want = std::max<uint32_t>(n, 64u);
        DevicePagedDecodeBatchItem* p = nullptr;
        if (cudaMalloc(reinterpret_cast<void**>(&p), sizeof(DevicePagedDecodeBatchItem) * want) != cudaSuccess) {
            return nullptr;
        }
        buffers.push_back(p);
        capacity = want;
    }
    return buffers.back();
}

} // namespace

void kkrt_txn_attend_batch(void* const* txns, uint32_t n, uint32_t layer, const void* q, void* o,
    uint64_t row_bytes, void* ws, uint64_t ws_bytes, float scale, int* statuses)
{
    // The batch item buffers the engine API asks for. This library's backend
    // keeps its work lists in per-stream device scratch of its own and reads
    // them only when that scratch could not be allocated; the device buffer
    // is therefore one process-wide allocation, grown on demand, instead of
    // a cudaMalloc / synchronize / cudaFree per call.
    std::vector<PagedDecodeBatchItem> items(n);
    std::vector<DevicePagedDecodeBatchItem> host(n);
    DevicePagedDecodeBatchItem* dev = batchItemScratch(n);
    for (uint32_t i = 0; i < n; ++i) {
        items[i].transaction = T(txns[i]);
        items[i].request = PagedDecodeRequest{layer,
            reinterpret_cast<KvScalar const*>(static_cast<std::uint8_t const*>(q) + i * row_bytes),
            reinterpret_cast<KvScalar*>(static_cast<std::uint8_t*>(o) + i * row_bytes), ws,
            static_cast<std::size_t>(ws_bytes), scale};
    }
    PagedDecodeBatch batch{items.data(), n, host.data(), dev, dev != nullptr ? n : 0u};
    attendLayerBatch(batch);
    for (uint32_t i = 0; i < n; ++i) {
        statuses[i] = static_cast<int>(items[i].status.error);
    }
}

int kkrt_txn_reserved_table(void* t, kk_table_out* out)
{
    FusedLane lane{};
    if (!fusedLane(*T(t), lane)) return 0;
    tableOut(*lane.reserved, out);
    return 1;
}

int kkrt_txn_commit(void* t) { return int(T(t)->commit().error); }
int kkrt_txn_rollback(void* t) { return int(T(t)->rollback().error); }
int kkrt_txn_phase(void* t) { return int(T(t)->snapshot().phase); }
void kkrt_txn_destroy(void* t) { delete T(t); }

void* kkrt_runner_create(const char* manifest, const char* data, void* backend, void* stream,
    uint32_t max_batch, int graphs, int verify, int* status, char* detail, uint32_t detail_cap)
{
    CudaModelRunnerOptions opt;
    opt.max_batch_size = max_batch;
    opt.use_cuda_graphs = graphs != 0;
    opt.verify_checksums = verify != 0;
    CudaModelRunnerCreateResult r = createCudaTinyLlamaModelRunner(manifest, data, *KV(backend), stream, opt);
    if (status != nullptr) *status = static_cast<int>(r.status.error);
    if (detail != nullptr && detail_cap != 0) {
        std::strncpy(detail, r.status.detail.c_str(), detail_cap - 1);
        detail[detail_cap - 1] = 0;
    }
    if (!r.ok()) return nullptr;
    return static_cast<GenerationModelRunner*>(r.runner.release());
}

void kkrt_runner_destroy(void* r) { delete RUN(r); }

int kkrt_runner_forward_batch(void* r, uint32_t n, const uint64_t* ids, const uint32_t* tokens,
    const uint32_t* positions, uint32_t* out_tokens, uint8_t* out_ok)
{
    std::vector<GenerationBatchItem> batch(n);
    for (uint32_t i = 0; i < n; ++i) {
        batch[i] = GenerationBatchItem{ids[i], tokens[i], positions[i]};
    }
    GenerationBatchResult const res = RUN(r)->generationForwardBatch(batch);
    if (!res.success || res.steps.size() != n) return 0;
    for (uint32_t i = 0; i < n; ++i) {
        out_tokens[i] = res.steps[i].greedy_token_id;
        out_ok[i] = res.steps[i].success ? 1 : 0;
    }
    return 1;
}

int kkrt_runner_forward_batch_logits(void* r, uint32_t n, const uint64_t* ids, const uint32_t* tokens,
    const uint32_t* positions, uint32_t* out_tokens, uint8_t* out_ok, float* logits)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    if (runner == nullptr || logits == nullptr) return 0;
    std::vector<GenerationBatchItem> batch(n);
    for (uint32_t i = 0; i < n; ++i) {
        batch[i] = GenerationBatchItem{ids[i], tokens[i], positions[i]};
    }
    std::vector<float> rows;
    GenerationBatchResult const res = runner->generationForwardBatchLogits(batch, rows);
    if (!res.success || res.steps.size() != n) return 0;
    std::size_t const V = runner->config().vocabulary_size;
    for (uint32_t i = 0; i < n; ++i) {
        out_tokens[i] = res.steps[i].greedy_token_id;
        out_ok[i] = res.steps[i].success ? 1 : 0;
        if (rows.size() >= (i + 1) * V) {
            std::memcpy(logits + i * V, rows.data() + i * V, V * sizeof(float));
        } else {
            std::memset(logits + i * V, 0, V * sizeof(float));
        }
    }
    return 1;
}

int kkrt_runner_forward_token(void* r, uint64_t id, uint32_t token, uint32_t position,
    uint32_t* out_token, float* logits, uint16_t* embedding, uint16_t* final_hidden,
    const uint32_t* layers, uint32_t n_layers, uint16_t* layer_hidden)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    if (runner == nullptr) return static_cast<int>(CudaModelRunnerError::InvalidArgument);
    ModelRunnerDebugCapture debug;
    bool const capture = embedding != nullptr || final_hidden != nullptr || n_layers != 0;
    if (capture) debug.layer_indices.assign(layers, layers + n_layers);
    ModelRunnerOutputOptions out;
    out.copy_logits = logits != nullptr;
    ModelTokenResult const res = runner->forwardToken(id, token, position, capture ? &debug : nullptr, out);
    if (!res.ok()) return static_cast<int>(res.status.error);
    if (out_token != nullptr) *out_token = res.greedy_token_id;
    if (logits != nullptr) std::memcpy(logits, res.logits.data(), res.logits.size() * sizeof(float));
    if (embedding != nullptr) std::memcpy(embedding, debug.embedding.data(), debug.embedding.size() * 2);
    if (final_hidden != nullptr) {
        std::memcpy(final_hidden, debug.final_hidden_state.data(), debug.final_hidden_state.size() * 2);
    }
    if (layer_hidden != nullptr) {
        std::size_t const h = runner->config().hidden_size;
        for (uint32_t i = 0; i < n_layers; ++i) {
            std::memcpy(layer_hidden + i * h, debug.layer_hidden_states[i].data(), h * 2);
        }
    }
    return 0;
}

float kkrt_runner_last_step_ms(void* r)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    return runner == nullptr ? 0.f : runner->lastStepDeviceMs();
}

int kkrt_runner_prefill(void* r, uint64_t id, const uint32_t* tokens, uint32_t n, uint32_t first_position,
    uint32_t* out_token)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    if (runner == nullptr || tokens == nullptr || n == 0) {
        return 0;
    }
    GenerationStepResult const res = runner->prefill(id, std::vector<uint32_t>(tokens, tokens + n), first_position);
    if (!res.success) {
        return 0;
    }
    if (out_token != nullptr) {
        *out_token = res.greedy_token_id;
    }
    return 1;
}

int kkrt_runner_set_auto_promote(void* r, int enabled)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    if (runner == nullptr) {
        return 0;
    }
    runner->setAutoPromote(enabled != 0);
    return 1;
}

uint32_t kkrt_runner_last_error(void* r, char* out, uint32_t cap)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    std::string const e = runner == nullptr ? std::string("not a CUDA runner") : runner->lastError();
    if (out != nullptr && cap != 0) {
        std::strncpy(out, e.c_str(), cap - 1);
        out[cap - 1] = 0;
    }
    return static_cast<uint32_t>(e.size());
}

uint32_t kkrt_runner_last_launches(void* r)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    return runner == nullptr ? 0 : runner->lastStepLaunches();
}

int kkrt_runner_last_host_us(void* r, float* out)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    if (runner == nullptr || out == nullptr) {
        return 0;
    }
    std::array<float, 5> const us = runner->lastStepHostUs();
    std::copy(us.begin(), us.end(), out);
    return 5;
}

int kkrt_runner_last_transfer_bytes(void* r, uint64_t* h2d, uint64_t* d2h)
{
    auto* runner = dynamic_cast<CudaTinyLlamaModelRunner*>(RUN(r));
    if (runner == nullptr) {
        return 0;
    }
    if (h2d != nullptr) {
        *h2d = runner->lastStepH2dBytes();
    }
    if (d2h != nullptr) {
        *d2h = runner->lastStepD2hBytes();
    }
    return 1;
}

void* kkrt_sched_create(void* b, void* r, uint32_t max_active, uint32_t max_tokens, uint64_t max_kv,
    uint32_t chunk)
{
    auto* s = new (std::nothrow) Sched;
    if (s == nullptr) return nullptr;
    s->rt = std::make_unique<IterationSchedulerRuntime>(*KV(b), *RUN(r),
        IterationSchedulerConfig{max_active, max_tokens, max_kv, chunk});
    return s;
}

void* kkrt_sched_create_ex(void* b, void* r, uint32_t max_active, uint32_t max_tokens, uint64_t max_kv,
    uint32_t chunk, uint32_t flags)
{
    auto* s = new (std::nothrow) Sched;
    if (s == nullptr) return nullptr;
    IterationSchedulerConfig cfg{max_active, max_tokens, max_kv, chunk};
    cfg.fused_prefill = (flags & KKRT_SCHED_FUSED_PREFILL) != 0;
    s->rt = std::make_unique<IterationSchedulerRuntime>(*KV(b), *RUN(r), cfg);
    return s;
}

void kkrt_sched_destroy(void* s) { delete static_cast<Sched*>(s); }

int kkrt_sched_submit_prefixed(void* s, uint64_t id, const uint32_t* prompt, uint32_t len, uint32_t max_new,
    int64_t eos, uint32_t kv_prefix_tokens)
{
    GenerationRequest req;
    req.request_id = id;
    if (len != 0) req.prompt_token_ids.assign(prompt, prompt + len);
    req.sampling.max_new_tokens = max_new;
    if (eos >= 0) req.sampling.eos_token_id = static_cast<std::uint32_t>(eos);
    req.kv_prefix_tokens = kv_prefix_tokens;
    return static_cast<int>(static_cast<Sched*>(s)->rt->submit(std::move(req)).error);
}

int kkrt_sched_submit(void* s, uint64_t id, const uint32_t* prompt, uint32_t len, uint32_t max_new,
    int64_t eos)
{
    return kkrt_sched_submit_prefixed(s, id, prompt, len, max_new, eos, 0);
}

int kkrt_sched_cancel(void* s, uint64_t id) { return static_cast<Sched*>(s)->rt->cancel(id) ? 1 : 0; }

void kkrt_sched_run_iteration(void* s, kk_iteration* out)
{
    SchedulerIterationResult const r = static_cast<Sched*>(s)->rt->runIteration();
    *out = kk_iteration{r.iteration, r.model_forward_tokens, r.model_forward_batches, r.prefill_tokens,
        r.decode_tokens, r.terminals_produced, 0};
}

void kkrt_sched_stop(void* s) { static_cast<Sched*>(s)->rt->stop(); }
int kkrt_sched_idle(void* s) { return static_cast<Sched*>(s)->rt->idle() ? 1 : 0; }

uint32_t kkrt_sched_drain(void* s, kk_terminal* out, uint32_t cap, uint32_t* tokens, uint32_t token_cap)
{
    return terminalsOut(static_cast<Sched*>(s)->rt->drain(), out, cap, tokens, token_cap);
}

uint32_t kkrt_sched_take_terminals(void* s, kk_terminal* out, uint32_t cap, uint32_t* tokens,
    uint32_t token_cap)
{
    return terminalsOut(static_cast<Sched*>(s)->rt->takeTerminals(), out, cap, tokens, token_cap);
}

int kkrt_generate(void* b, void* r, uint64_t id, const uint32_t* prompt, uint32_t len, uint32_t max_new,
    int64_t eos, kk_terminal* out, uint32_t* tokens, uint32_t token_cap)
{
    SingleRequestGenerationRuntime rt(*KV(b), *RUN(r));
    GenerationRequest req;
    req.request_id = id;
    req.prompt_token_ids.assign(prompt, prompt + len);
    req.sampling.max_new_tokens = max_new;
    if (eos >= 0) req.sampling.eos_token_id = static_cast<std::uint32_t>(eos);
    std::vector<GenerationTerminal> one{rt.generate(req)};
    return static_cast<int>(terminalsOut(one, out, 1, tokens, token_cap));
}

void* kkrt_fake_backend_create(void) { return static_cast<EngineKvBackend*>(new (std::nothrow) FakeBackend); }
void kkrt_fake_backend_destroy(void* b) { delete KV(b); }

void* kkrt_fake_runner_create(uint32_t vocab, uint32_t max_batch, uint32_t eos, uint32_t positions,
    uint64_t fail_request)
{
    return static_cast<GenerationModelRunner*>(
        new (std::nothrow) FakeRunner(vocab, max_batch, eos, positions, fail_request));
}

void kkrt_fake_runner_destroy(void* r) { delete RUN(r); }

uint32_t kkrt_fake_runner_log(void* r, uint32_t* sizes, uint32_t cap_batches, uint64_t* items,
    uint32_t cap_items)
{
    auto* f = dynamic_cast<FakeRunner*>(RUN(r));
    if (f == nullptr) return 0;
    for (std::size_t i = 0; i < f->sizes.size() && i < cap_batches; ++i) sizes[i] = f->sizes[i];
    for (std::size_t i = 0; i < f->items.size() && i < cap_items; ++i) items[i] = f->items[i];
    return static_cast<uint32_t>(f->sizes.size());
}

} // extern "C"

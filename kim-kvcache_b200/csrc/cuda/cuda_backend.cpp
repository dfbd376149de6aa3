// CUDA heterogeneous KV backend (reference semantics:
// src/cuda/engine/backend.cpp:19-610, src/cuda/engine/transaction.cpp:1-425,
// src/cuda/kv/storage.cpp:99-234). See cuda_backend.h for the design.
#include "cuda_backend.h"

#include "../host/fixed_page_manager.h"
#include "kernels_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <limits>
#include <mutex>
#include <optional>
#include <unordered_map>
#include <vector>

namespace kimkvcache {
namespace {

EngineKvStatus mapMetadata(KvCacheError e) noexcept
{
    switch (e) {
    case KvCacheError::None: return {};
    case KvCacheError::InvalidArgument: return {EngineKvError::InvalidArgument};
    case KvCacheError::RequestNotFound: return {EngineKvError::RequestNotFound};
    case KvCacheError::RequestAlreadyExists: return {EngineKvError::RequestAlreadyExists};
    case KvCacheError::RequestConflict:
    case KvCacheError::PromotionConflict: return {EngineKvError::RequestConflict};
    case KvCacheError::ResourceExhausted: return {EngineKvError::ResourceExhausted};
    case KvCacheError::InvalidState: return {EngineKvError::InvalidState};
    default: return {EngineKvError::InternalError};
    }
}

EngineKvStatus mapCuda(CudaStatus s) noexcept
{
    switch (s.error) {
    case CudaError::None: return {};
    case CudaError::InvalidArgument: return {EngineKvError::InvalidArgument};
    case CudaError::AllocationFailed: return {EngineKvError::ResourceExhausted};
    case CudaError::SubmissionFailed: return {EngineKvError::SubmissionFailed};
    case CudaError::ExecutionFailed: return {EngineKvError::ExecutionFailed};
    default: return {EngineKvError::InternalError};
    }
}

CudaStatus submitError(int code) noexcept
{
    return code == KK_EINVAL ? CudaStatus{CudaError::InvalidArgument, code}
                             : CudaStatus{CudaError::SubmissionFailed, code};
}

// Device page pools: [capacity][layers][K/V][tokens][kv_heads][dim] FP16, zeroed.
struct Storage {
    kk_kv_pools pools{};
    CudaStatus status{};
    std::size_t micro_bytes{0};
    std::size_t extent_bytes{0};

    Storage(KvLayout layout, std::uint32_t micro_cap, std::uint32_t extent_cap)
    {
        std::size_t micro_page = 0, extent_page = 0;
        if (!layout.pageElements(PageKind::Micro, micro_page)
            || !layout.pageElements(PageKind::Extent, extent_page)) {
            status = {CudaError::InvalidArgument, 0};
            return;
        }
        micro_bytes = micro_page * 2 * micro_cap;
        extent_bytes = extent_page * 2 * extent_cap;
        void* micro = nullptr;
        void* extent = nullptr;
        cudaError_t e = cudaMalloc(&micro, micro_bytes);
        if (e == cudaSuccess) {
            e = cudaMalloc(&extent, extent_bytes);
        }
        if (e == cudaSuccess) {
            e = cudaMemset(micro, 0, micro_bytes);
        }
        if (e == cudaSuccess) {
            e = cudaMemset(extent, 0, extent_bytes);
        }
        pools = kk_kv_pools{micro, extent, micro_cap, extent_cap, layout.layer_count,
            layout.kv_head_count, layout.head_dimension, 0};
        if (e != cudaSuccess) {
            status = {CudaError::AllocationFailed, static_cast<int>(e)};
        }
    }

    // Fixed-page storage: one pool of page_capacity pages of tokens_per_page
    // tokens (reference EngineBackendState(config, tokens_per_page,
    // page_capacity), src/cuda/engine/backend.cpp:91-106); no extent pool.
    Storage(KvLayout layout, std::uint16_t tokens_per_page, std::uint32_t page_capacity)
    {
        if (!layout.valid() || (tokens_per_page != 8 && tokens_per_page != 16 && tokens_per_page != 32
                                   && tokens_per_page != 64)) {
            status = {CudaError::InvalidArgument, 0};
            return;
        }
        std::size_t const page = std::size_t(layout.layer_count) * 2u * tokens_per_page
            * layout.kv_head_count * layout.head_dimension;
        micro_bytes = page * 2 * page_capacity;
        void* micro = nullptr;
        cudaError_t e = cudaMalloc(&micro, micro_bytes);
        if (e == cudaSuccess) {
            e = cudaMemset(micro, 0, micro_bytes);
        }
        pools = kk_kv_pools{micro, nullptr, page_capacity, 0, layout.layer_count, layout.kv_head_count,
            layout.head_dimension, tokens_per_page};
        if (e != cudaSuccess) {
            status = {CudaError::AllocationFailed, static_cast<int>(e)};
        }
    }

    ~Storage()
    {
        cudaDeviceSynchronize();
        cudaFree(pools.micro);
        cudaFree(pools.extent);
    }
};

// Preallocated per-transaction device metadata for the per-layer SPI path.
struct Arena {
    static constexpr std::uint32_t kSlots = 64;
    static constexpr std::size_t kHeader = 96;  // kv_slot | copy | lane | item
    // Device error words of the per-layer path, one per stream it launched on.
    static constexpr std::uint32_t kStatusWords = 64;
    std::uint32_t max_desc{0};
    std::size_t slot_bytes{0};
    std::uint8_t* dev{nullptr};
    std::uint8_t* host{nullptr};
    unsigned int* status{nullptr};
    // Pinned mirror of the error words: a commit that synchronizes a stream
    // queues the copy of the stream's word in front of the synchronize, so
    // the word is on the host when the synchronize returns.
    unsigned int* status_host{nullptr};
    // Other reads of the error words go through this stream, so that they
    // never wait for work that callers queued after the point being checked.
    cudaStream_t watch_stream{nullptr};
    std::vector<std::uint32_t> free_slots;

    bool init(std::uint32_t descriptors)
    {
        max_desc = descriptors;
        slot_bytes = (kHeader + std::size_t(descriptors) * sizeof(kk_page_desc) + 255) & ~std::size_t(255);
        if (cudaMalloc(reinterpret_cast<void**>(&dev), slot_bytes * kSlots) != cudaSuccess
            || cudaMallocHost(reinterpret_cast<void**>(&host), slot_bytes * kSlots) != cudaSuccess
            || cudaMalloc(reinterpret_cast<void**>(&status), kStatusWords * sizeof(unsigned int)) != cudaSuccess
            || cudaMemset(status, 0, kStatusWords * sizeof(unsigned int)) != cudaSuccess
            || cudaMallocHost(reinterpret_cast<void**>(&status_host), kStatusWords * sizeof(unsigned int))
                != cudaSuccess
            || cudaStreamCreateWithFlags(&watch_stream, cudaStreamNonBlocking) != cudaSuccess) {
            return false;
        }
        for (std::uint32_t i = kSlots; i > 0; --i) {
            free_slots.push_back(i - 1);
        }
        return true;
    }

    ~Arena()
    {
        cudaFree(dev);
        cudaFreeHost(host);
        cudaFree(status);
        cudaFreeHost(status_host);
        if (watch_stream != nullptr) {
            cudaStreamDestroy(watch_stream);
        }
    }

    // Offsets inside a slot.
    static constexpr std::size_t kSlotOff = 0, kCopyOff = 16, kLaneOff = 32, kItemOff = 64,
                                 kDescOff = kHeader;
};

struct State {
    EngineKvConfig config;
    EngineKvBackendKind kind;
    // Exactly one metadata runtime: the two-pool manager (heterogeneous
    // backend) or the fixed-page manager.
    std::unique_ptr<KvCacheManager> mgr;
    std::unique_ptr<FixedPageManager> fixed;
    Storage storage;
    Arena arena;
    std::unordered_map<RequestId, std::uint32_t> committed_lengths;
    std::uint64_t active{0};
    std::atomic<std::uint64_t> batched_submissions{0};
    std::atomic<std::uint64_t> batched_lanes{0};
    mutable std::mutex mutex;

    std::mutex fault_mutex;
    bool fail_submission{false};
    bool fail_completion{false};
    // Set while either injected failure is armed, so the per-lane checks of
    // every transaction skip the mutex when none is.
    std::atomic<bool> failure_armed{false};

    std::atomic<std::uint64_t> submit_seq{0};
    std::mutex sync_mutex;
    std::unordered_map<void*, std::uint64_t> completed_seq;

    // Device-detected errors of the per-layer path (a descriptor outside its
    // pool, a bounded wait that ran out). The kernels that transactions
    // launch on a stream report into that stream's error word; a commit reads
    // it once the stream is synchronized. An error fails every transaction
    // with work queued on the stream before the word is cleared again (the
    // conservative reading: a word cannot tell which launch set it).
    struct StreamWatch {
        std::uint32_t word;
        std::uint64_t checked;      // submissions up to here were checked
        std::uint64_t failed_upto;  // submissions up to here are covered by a device error
        std::uint64_t mirrored;     // the pinned mirror holds the word as of this submission
    };
    std::unordered_map<void*, StreamWatch> watch;  // under sync_mutex

    // Per-stream device scratch of the per-layer attention launches: the
    // lane records and balanced work list, and the split-lane workspace
    // (completion counters zeroed when created; the kernel leaves them
    // zero). Work on one stream is ordered, so one set per stream suffices.
    static constexpr std::uint32_t kMaxPlanItems = 1024;
    struct AttendScratch {
        std::uint8_t* plan{nullptr};
        void* workspace{nullptr};
        std::uint64_t workspace_bytes{0};
    };
    std::unordered_map<void*, AttendScratch> attend_scratch;  // under sync_mutex
    std::uint32_t sm_count{1};

    State(EngineKvConfig c, std::uint32_t micro_cap, std::uint32_t extent_cap)
        : config(c), kind(EngineKvBackendKind::Heterogeneous)
        , mgr(std::make_unique<KvCacheManager>(micro_cap, extent_cap))
        , storage(c.kv_layout, micro_cap, extent_cap)
    {
        if (storage.status.ok() && !arena.init(micro_cap + extent_cap)) {
            storage.status = {CudaError::AllocationFailed, 0};
        }
        initSmCount();
    }

    State(EngineKvConfig c, std::uint16_t tokens_per_page, std::uint32_t page_capacity, bool)
        : config(c), kind(EngineKvBackendKind::Fixed)
        , fixed(std::make_unique<FixedPageManager>(tokens_per_page, page_capacity))
        , storage(c.kv_layout, tokens_per_page, page_capacity)
    {
        if (storage.status.ok() && !arena.init(page_capacity)) {
            storage.status = {CudaError::AllocationFailed, 0};
        }
        initSmCount();
    }

    void initSmCount()
    {
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) == cudaSuccess
            && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0) {
            sm_count = static_cast<std::uint32_t>(sms);
        }
    }

    // Metadata operations of whichever runtime this backend holds.
    KvCacheError create(RequestId id) { return mgr ? mgr->createRequest(id) : fixed->createRequest(id); }
    KvCacheError fork(RequestId s, RequestId c) { return mgr ? mgr->forkRequest(s, c) : fixed->forkRequest(s, c); }
    KvCacheError release(RequestId id) { return mgr ? mgr->releaseRequest(id) : fixed->releaseRequest(id); }
    KvCacheError append(RequestId id, std::uint32_t n) { return mgr ? mgr->append(id, n) : fixed->append(id, n); }
    KvCacheError seal(RequestId id) { return mgr ? mgr->sealTail(id) : fixed->sealTail(id); }
    TokenReservationResult reserve(RequestId id, std::uint32_t expected)
    {
        return mgr ? mgr->reserveToken(id, expected) : fixed->reserveToken(id, expected);
    }
    KvCacheError commit(KvTokenReservationId id)
    {
        return mgr ? mgr->commitTokenReservation(id) : fixed->commitTokenReservation(id);
    }
    KvCacheError rollback(KvTokenReservationId id)
    {
        return mgr ? mgr->rollbackTokenReservation(id) : fixed->rollbackTokenReservation(id);
    }
    std::optional<BlockTable> table(RequestId id) const { return mgr ? mgr->blockTable(id) : fixed->blockTable(id); }
    bool metadataConsistent() const
    {
        return mgr ? mgr->checkInvariants() && active == mgr->snapshot().token_reservation_count
                   : fixed->checkInvariants() && active == fixed->snapshot().token_reservation_count;
    }
    // A block table's structure, checked against the page size of its pool.
    bool tableWellFormed(BlockTable const& t) const
    {
        return fixed ? t.checkInvariants(fixed->tokensPerPage()) : t.checkInvariants();
    }

    bool consumeFailure(CudaFailurePoint point)
    {
        if (!failure_armed.load(std::memory_order_acquire)) {
            return false;
        }
        std::lock_guard<std::mutex> lock(fault_mutex);
        bool& flag = point == CudaFailurePoint::Submission ? fail_submission : fail_completion;
        bool const was = flag;
        flag = false;
        failure_armed.store(fail_submission || fail_completion, std::memory_order_release);
        return was;
    }

    // True when a synchronize of `stream` already covered submission `seq`;
    // `covered` receives the submission it covered up to.
    bool completed(void* stream, std::uint64_t seq, std::uint64_t& covered)
    {
        std::lock_guard<std::mutex> lock(sync_mutex);
        auto const f = completed_seq.find(stream);
        if (f == completed_seq.end() || f->second < seq) {
            return false;
        }
        covered = f->second;
        return true;
    }

    void noteCompleted(void* stream, std::uint64_t covered)
    {
        std::lock_guard<std::mutex> lock(sync_mutex);
        std::uint64_t& c = completed_seq[stream];
        c = c > covered ? c : covered;
    }

    // The stream's attention scratch (created on first use; nullptr when the
    // allocation fails, and the caller then plans one item per lane).
    AttendScratch const* attendScratch(void* stream)
    {
        std::lock_guard<std::mutex> lock(sync_mutex);
        auto f = attend_scratch.find(stream);
        if (f != attend_scratch.end()) {
            return &f->second;
        }
        AttendScratch sc;
        std::uint32_t const hq = config.query_head_count;
        sc.workspace_bytes = kk_attention_workspace_bytes(Arena::kSlots, kMaxPlanItems, hq,
            config.kv_layout.head_dimension);
        std::size_t const plan_bytes = Arena::kSlots * sizeof(kk_attn_lane) + kMaxPlanItems * sizeof(kk_attn_item);
        if (cudaMalloc(reinterpret_cast<void**>(&sc.plan), plan_bytes) != cudaSuccess
            || cudaMalloc(&sc.workspace, sc.workspace_bytes) != cudaSuccess
            || kk_attention_workspace_init(sc.workspace, Arena::kSlots, stream) != 0) {
            cudaFree(sc.plan);
            cudaFree(sc.workspace);
            return nullptr;
        }
        return &attend_scratch.emplace(stream, sc).first->second;
    }

    ~State()
    {
        for (auto& [stream, sc] : attend_scratch) {
            cudaFree(sc.plan);
            cudaFree(sc.workspace);
        }
    }

    // One layer of attention over host lane records whose descriptors are in
    // the arena, with the work list in the stream's scratch. Where the TMA
    // kernel serves the shape: a token-balanced work list
    // (kk_attention_plan_balanced, no part shorter than
    // kk::kAttnMinPartCost) with the scratch's split-lane workspace, so a
    // long lane is spread over many SMs. Otherwise one item per lane for the
    // process-wide kernel choice, with the caller's workspace. Returns 0, a
    // CUDA error or KK_EINVAL; -1 when the scratch is unavailable.
    int attendPlanned(kk_attn_lane const* lanes, std::uint32_t n, std::uint32_t layer, void const* query,
        void* output, float scale, void* workspace, std::uint64_t workspace_bytes, void* stream)
    {
        std::uint32_t const hq = config.query_head_count;
        if (n == 0 || n > Arena::kSlots) {
            return -1;
        }
        AttendScratch const* sc = attendScratch(stream);
        if (sc == nullptr) {
            return -1;
        }
        bool const tma = kk::attentionTmaSupported(&storage.pools, hq);
        std::size_t const lane_bytes = n * sizeof(kk_attn_lane);
        std::vector<std::uint8_t> host(lane_bytes + kMaxPlanItems * sizeof(kk_attn_item));
        auto* planned = reinterpret_cast<kk_attn_lane*>(host.data());
        std::memcpy(planned, lanes, lane_bytes);
        auto* items = reinterpret_cast<kk_attn_item*>(host.data() + lane_bytes);
        std::uint32_t count = n;
        if (tma) {
            count = kk_attention_plan_balanced(reinterpret_cast<kk_page_desc const*>(arena.host), planned, n,
                kk::attentionPlanParts(planned, n, sm_count), items, kMaxPlanItems);
            if (count == 0 || count > kMaxPlanItems) {
                return KK_EINVAL;
            }
        } else {
            for (std::uint32_t j = 0; j < n; ++j) {
                planned[j].item_offset = j;
                planned[j].item_count = 1;
                planned[j].first_item_shared = 0;
                items[j] = kk_attn_item{j, planned[j].desc_offset, planned[j].desc_offset + planned[j].desc_count, 0};
            }
        }
        auto const s = static_cast<cudaStream_t>(stream);
        // From pageable memory: the bytes are staged when the call returns.
        cudaError_t const e = cudaMemcpyAsync(sc->plan, host.data(), lane_bytes + count * sizeof(kk_attn_item),
            cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) {
            return static_cast<int>(e);
        }
        std::uint32_t const row = hq * config.kv_layout.head_dimension;
        auto const* descs = reinterpret_cast<kk_page_desc const*>(arena.dev);
        auto const* dl = reinterpret_cast<kk_attn_lane const*>(sc->plan);
        auto const* di = reinterpret_cast<kk_attn_item const*>(sc->plan + lane_bytes);
        auto const* q = static_cast<std::uint16_t const*>(query);
        auto* o = static_cast<std::uint16_t*>(output);
        return tma ? kk::attentionLaunchTma(&storage.pools, layer, hq, descs, dl, n, di, count, q, row, o, row, scale,
                         sc->workspace, sc->workspace_bytes, statusWord(stream), s)
                   : kk::attentionLaunch(&storage.pools, layer, hq, descs, dl, n, di, count, q, row, o, row, scale,
                         workspace, workspace_bytes, statusWord(stream), s);
    }

    // Error word of the per-layer kernels launched on `stream`.
    unsigned int* statusWord(void* stream)
    {
        std::lock_guard<std::mutex> lock(sync_mutex);
        auto f = watch.find(stream);
        if (f == watch.end()) {
            // More streams than words: the last word is shared (errors then
            // fail the transactions of every stream that shares it).
            std::uint32_t const n = static_cast<std::uint32_t>(watch.size());
            std::uint32_t const w = n < Arena::kStatusWords ? n : Arena::kStatusWords - 1;
            f = watch.emplace(stream, StreamWatch{w, 0, 0, 0}).first;
        }
        return arena.status + f->second.word;
    }

    // Queues, on `stream`, the copy of its error word into the pinned mirror
    // (to be followed by a synchronize of the stream that covers `seq`).
    void queueStatusRead(void* stream, std::uint64_t seq)
    {
        std::lock_guard<std::mutex> lock(sync_mutex);
        auto const f = watch.find(stream);
        if (f == watch.end()) {
            return;
        }
        if (cudaMemcpyAsync(arena.status_host + f->second.word, arena.status + f->second.word, sizeof(unsigned int),
                cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)) == cudaSuccess) {
            f->second.mirrored = seq;
        }
    }

    // Called once `stream` is synchronized up to submission `covered`: reads
    // the stream's error word (once per such point; from the pinned mirror
    // when the synchronize brought it along) and, when it is set, clears it
    // on the stream behind everything queued so far. Returns the last
    // submission that a device error covers (0: none).
    std::uint64_t checkStream(void* stream, std::uint64_t covered)
    {
        std::lock_guard<std::mutex> lock(sync_mutex);
        auto const f = watch.find(stream);
        if (f == watch.end()) {
            return 0;  // no per-layer kernel ran on this stream
        }
        StreamWatch& w = f->second;
        if (w.checked < covered) {
            unsigned int code = 0;
            cudaError_t e = cudaSuccess;
            if (w.mirrored >= covered) {
                code = *static_cast<unsigned int volatile*>(arena.status_host + w.word);
            } else {
                e = cudaMemcpyAsync(&code, arena.status + w.word, sizeof(code), cudaMemcpyDeviceToHost,
                    arena.watch_stream);
                if (e == cudaSuccess) {
                    e = cudaStreamSynchronize(arena.watch_stream);
                }
            }
            if (e != cudaSuccess || code != 0) {
                // Everything queued on the stream until the clear below is
                // covered: the word may also hold an error of later work.
                w.failed_upto = submit_seq.load();
                cudaMemsetAsync(arena.status + w.word, 0, sizeof(unsigned int), static_cast<cudaStream_t>(stream));
                // An attention launch that gave up may have left split-lane
                // completion counts behind: the stream's next launch starts
                // from zero again.
                auto const sc = attend_scratch.find(stream);
                if (sc != attend_scratch.end()) {
                    static_cast<void>(kk_attention_workspace_init(sc->second.workspace, Arena::kSlots, stream));
                }
            }
            w.checked = covered;
        }
        return w.failed_upto;
    }
};

class CudaTxn final : public TokenTransactionBackend {
public:
    CudaTxn(std::shared_ptr<State> st, KvTokenReservationId reservation, RequestId request,
        PageLeaseId lease, BlockTable before, BlockTable reserved, void* stream)
        : st_(std::move(st)), reservation_(reservation), request_(request), lease_(lease)
        , before_(std::move(before)), reserved_(std::move(reserved)), stream_(stream)
    {
    }

    ~CudaTxn() override { freeArenaSlot(); }

    BlockTable const& before() const noexcept { return before_; }
    BlockTable const& reserved() const noexcept { return reserved_; }
    State* state() const noexcept { return st_.get(); }

    EngineKvStatus writeLayer(LayerKvWrite const& write, EngineStream) override
    {
        if (!submission_.ok()) {
            return mapCuda(submission_);
        }
        if (write.layer >= st_->config.kv_layout.layer_count || write.device_key == nullptr
            || write.device_value == nullptr) {
            return {EngineKvError::InvalidArgument};
        }
        if (st_->consumeFailure(CudaFailurePoint::Submission)) {
            return fail({CudaError::SubmissionFailed, 0});
        }
        if (!upload()) {
            return mapCuda(submission_);
        }
        std::uint8_t* const dev = slotDev();
        cudaStream_t const s = static_cast<cudaStream_t>(stream_);
        int rc = 0;
        unsigned int* const status = st_->statusWord(stream_);
        if (needs_copy_) {
            rc = kk::kvCopy(&st_->storage.pools, write.layer, 1,
                reinterpret_cast<kk_kv_copy const*>(dev + Arena::kCopyOff), 1, status, s);
        }
        if (rc == 0) {
            rc = kk::kvWrite(&st_->storage.pools, write.layer, 1,
                reinterpret_cast<kk_kv_slot const*>(dev + Arena::kSlotOff), 1,
                static_cast<std::uint16_t const*>(write.device_key),
                static_cast<std::uint16_t const*>(write.device_value), 0, 0, status, s);
        }
        if (rc != 0) {
            return fail(submitError(rc));
        }
        markSubmitted();
        return {};
    }

    EngineKvStatus attendLayer(PagedDecodeRequest const& r, EngineStream) override
    {
        CudaStatus const checked = prepareAttention(r);
        if (!checked.ok()) {
            return mapCuda(checked);
        }
        kk_attn_lane lane{descOffset() + static_cast<std::uint32_t>(Arena::kDescOff / sizeof(kk_page_desc)),
            static_cast<std::uint32_t>(reserved_.entries().size()), reserved_.tokenCount(), 0, 1, 0, 0, 0};
        int const planned = st_->attendPlanned(&lane, 1, r.layer, r.device_query, r.device_output,
            r.attention_scale, r.device_workspace, r.workspace_bytes, stream_);
        if (planned >= 0) {
            if (planned != 0) {
                return fail(submitError(planned));
            }
            markSubmitted();
            return {};
        }
        std::uint8_t* const dev = slotDev();
        std::uint32_t const hq = st_->config.query_head_count;
        std::uint32_t const row = hq * st_->config.kv_layout.head_dimension;
        int const rc = kk::attentionLaunch(&st_->storage.pools, r.layer, hq,
            reinterpret_cast<kk_page_desc const*>(st_->arena.dev),
            reinterpret_cast<kk_attn_lane const*>(dev + Arena::kLaneOff), 1,
            reinterpret_cast<kk_attn_item const*>(dev + Arena::kItemOff), 1,
            static_cast<std::uint16_t const*>(r.device_query), row,
            static_cast<std::uint16_t*>(r.device_output), row, r.attention_scale, r.device_workspace,
            r.workspace_bytes, st_->statusWord(stream_), static_cast<cudaStream_t>(stream_));
        if (rc != 0) {
            return fail(submitError(rc));
        }
        markSubmitted();
        return {};
    }

    void attendLayerBatch(PagedDecodeBatch& batch) override;

    EngineKvStatus submitFusedLayers(EngineStream) override
    {
        if (!submission_.ok()) {
            return mapCuda(submission_);
        }
        if (st_->consumeFailure(CudaFailurePoint::Submission)) {
            return fail({CudaError::SubmissionFailed, 0});
        }
        markSubmitted();
        return {};
    }

    EngineKvStatus commit(EngineStream) override
    {
        CudaStatus const done = complete();
        if (!done.ok()) {
            return mapCuda(done);
        }
        std::lock_guard<std::mutex> lock(st_->mutex);
        EngineKvStatus const lease = releaseLeaseLocked();
        if (!lease.ok()) {
            return lease;
        }
        KvCacheError const committed = st_->commit(reservation_);
        if (committed != KvCacheError::None) {
            return mapMetadata(committed);
        }
        auto length = st_->committed_lengths.find(request_);
        if (length == st_->committed_lengths.end()) {
            return {EngineKvError::InternalError};
        }
        ++length->second;
        --st_->active;
        resolved_ = true;
        return {};
    }

    void rollback(EngineStream) noexcept override
    {
        if (resolved_) {
            return;
        }
        static_cast<void>(complete());
        std::lock_guard<std::mutex> lock(st_->mutex);
        static_cast<void>(releaseLeaseLocked());
        static_cast<void>(st_->rollback(reservation_));
        if (st_->active != 0) {
            --st_->active;
        }
        resolved_ = true;
    }

    // Attention preconditions of the reference (transaction.cpp:43-82).
    CudaStatus prepareAttention(PagedDecodeRequest const& r)
    {
        if (!submission_.ok()) {
            return submission_;
        }
        std::uint32_t const tokens = reserved_.tokenCount();
        std::size_t const scores = std::size_t(st_->config.query_head_count) * tokens;
        if (r.layer >= st_->config.kv_layout.layer_count || r.device_query == nullptr
            || r.device_output == nullptr || r.device_workspace == nullptr
            || !(r.attention_scale > 0.0F) || tokens == 0
            || r.workspace_bytes < scores * sizeof(float)) {
            return {CudaError::InvalidArgument, 0};
        }
        if (st_->consumeFailure(CudaFailurePoint::Submission)) {
            submission_ = final_ = {CudaError::SubmissionFailed, 0};
            return submission_;
        }
        if (!upload()) {
            return submission_;
        }
        return {};
    }

    std::uint8_t* slotDev() const noexcept
    {
        return st_->arena.dev + std::size_t(slot_) * st_->arena.slot_bytes;
    }
    std::uint32_t descOffset() const noexcept
    {
        return static_cast<std::uint32_t>(
            (std::size_t(slot_) * st_->arena.slot_bytes) / sizeof(kk_page_desc));
    }
    EngineKvStatus fail(CudaStatus s) noexcept
    {
        submission_ = final_ = s;
        return mapCuda(s);
    }
    void markSubmitted() noexcept
    {
        last_submit_ = ++st_->submit_seq;
        if (first_submit_ == 0) {
            first_submit_ = last_submit_;
        }
    }

private:
    // Copies this transaction's write target, COW record, lane and descriptors
    // into its arena slot (first per-layer SPI use only).
    bool upload()
    {
        if (uploaded_) {
            return true;
        }
        {
            std::lock_guard<std::mutex> lock(st_->mutex);
            if (st_->arena.free_slots.empty()) {
                submission_ = final_ = {CudaError::SubmissionFailed, 0};
                return false;
            }
            slot_ = static_cast<int>(st_->arena.free_slots.back());
            st_->arena.free_slots.pop_back();
        }
        auto const& entries = reserved_.entries();
        if (entries.size() > st_->arena.max_desc) {
            submission_ = final_ = {CudaError::InvalidArgument, 0};
            return false;
        }
        std::uint8_t* const host = st_->arena.host + std::size_t(slot_) * st_->arena.slot_bytes;
        MappingEntry const& target = entries.back();
        kk_kv_slot ks{target.handle.slot,
            static_cast<std::uint16_t>(reserved_.tokenCount() - 1 - target.logical_token_begin),
            static_cast<std::uint8_t>(target.kind), 1};
        std::memcpy(host + Arena::kSlotOff, &ks, sizeof(ks));
        kk_kv_copy copy{};
        needs_copy_ = false;
        if (!before_.entries().empty()) {
            MappingEntry const& old_tail = before_.entries().back();
            if (old_tail.logical_token_begin == target.logical_token_begin
                && old_tail.handle != target.handle) {
                copy = kk_kv_copy{old_tail.handle.slot, target.handle.slot, old_tail.valid_tokens,
                    static_cast<std::uint8_t>(old_tail.kind), static_cast<std::uint8_t>(target.kind)};
                needs_copy_ = true;
            }
        }
        std::memcpy(host + Arena::kCopyOff, &copy, sizeof(copy));
        kk_attn_lane lane{descOffset() + static_cast<std::uint32_t>(Arena::kDescOff / sizeof(kk_page_desc)),
            static_cast<std::uint32_t>(entries.size()), reserved_.tokenCount(), 0, 1, 0, 0, 0};
        std::memcpy(host + Arena::kLaneOff, &lane, sizeof(lane));
        kk_attn_item item{0, lane.desc_offset, lane.desc_offset + lane.desc_count, 0};
        std::memcpy(host + Arena::kItemOff, &item, sizeof(item));
        auto* descs = reinterpret_cast<kk_page_desc*>(host + Arena::kDescOff);
        for (std::size_t i = 0; i < entries.size(); ++i) {
            descs[i] = kk_page_desc{entries[i].handle.slot, entries[i].logical_token_begin,
                entries[i].valid_tokens, static_cast<std::uint8_t>(entries[i].kind), 0, 0};
        }
        std::size_t const bytes = Arena::kDescOff + entries.size() * sizeof(kk_page_desc);
        cudaError_t const e = cudaMemcpyAsync(slotDev(), host, bytes, cudaMemcpyHostToDevice,
            static_cast<cudaStream_t>(stream_));
        if (e != cudaSuccess) {
            submission_ = final_ = {CudaError::SubmissionFailed, static_cast<int>(e)};
            return false;
        }
        uploaded_ = true;
        return true;
    }

    CudaStatus complete() noexcept
    {
        if (finished_) {
            return final_;
        }
        finished_ = true;
        if (!submission_.ok()) {
            cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
            final_ = submission_;
            return final_;
        }
        std::uint64_t covered = 0;
        if (!st_->completed(stream_, last_submit_, covered)) {
            covered = st_->submit_seq.load();
            st_->queueStatusRead(stream_, covered);
            cudaError_t const e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
            if (e != cudaSuccess) {
                final_ = {CudaError::ExecutionFailed, static_cast<int>(e)};
                return final_;
            }
            st_->noteCompleted(stream_, covered);
        }
        // A device-detected error of work queued on this stream fails the
        // transaction at commit (reference: a completion failure surfaces as
        // ExecutionFailed, src/cuda/engine/transaction.cpp:84-120).
        if (first_submit_ != 0 && st_->checkStream(stream_, covered) >= first_submit_) {
            final_ = {CudaError::ExecutionFailed, KK_EDEVICE};
            return final_;
        }
        if (st_->consumeFailure(CudaFailurePoint::Completion)) {
            final_ = {CudaError::ExecutionFailed, static_cast<int>(cudaErrorUnknown)};
            return final_;
        }
        final_ = {};
        return final_;
    }

    EngineKvStatus releaseLeaseLocked() noexcept
    {
        if (lease_ == kInvalidPageLeaseId) {
            return {};
        }
        KvCacheError const released = st_->mgr->releasePageLease(lease_);
        if (released == KvCacheError::None) {
            lease_ = kInvalidPageLeaseId;
        }
        return mapMetadata(released);
    }

    void freeArenaSlot() noexcept
    {
        if (slot_ >= 0) {
            std::lock_guard<std::mutex> lock(st_->mutex);
            st_->arena.free_slots.push_back(static_cast<std::uint32_t>(slot_));
            slot_ = -1;
        }
    }

    std::shared_ptr<State> st_;
    KvTokenReservationId reservation_;
    RequestId request_;
    PageLeaseId lease_;
    BlockTable before_;
    BlockTable reserved_;
    void* stream_;
    int slot_{-1};
    bool uploaded_{false};
    bool needs_copy_{false};
    CudaStatus submission_{};
    CudaStatus final_{};
    bool finished_{false};
    bool resolved_{false};
    std::uint64_t last_submit_{0};
    std::uint64_t first_submit_{0};

    friend void batchAttend(CudaTxn& self, PagedDecodeBatch& batch);
};

// One ragged launch for all lanes when their queries/outputs are rows of one
// buffer each (as the reference runner lays them out); otherwise per lane.
void CudaTxn::attendLayerBatch(PagedDecodeBatch& batch)
{
    std::vector<std::size_t> idx;
    std::vector<CudaTxn*> txns;
    for (std::size_t i = 0; i < batch.item_count; ++i) {
        PagedDecodeBatchItem const& item = batch.items[i];
        if (!item.status.ok()) {
            continue;
        }
        auto* t = dynamic_cast<CudaTxn*>(batchBackend(item));
        if (t == nullptr || t->st_ != st_ || (!txns.empty() && batchStream(item) != txns[0]->stream_)
            || item.request.layer != batch.items[idx.empty() ? i : idx[0]].request.layer) {
            TokenTransactionBackend::attendLayerBatch(batch);
            return;
        }
        idx.push_back(i);
        txns.push_back(t);
    }
    if (txns.size() < 2) {
        TokenTransactionBackend::attendLayerBatch(batch);
        return;
    }
    std::uint32_t const hq = st_->config.query_head_count;
    std::size_t const row_bytes = std::size_t(hq) * st_->config.kv_layout.head_dimension * 2;
    auto const* q0 = reinterpret_cast<std::uint8_t const*>(batch.items[idx[0]].request.device_query);
    auto const* o0 = reinterpret_cast<std::uint8_t const*>(batch.items[idx[0]].request.device_output);
    std::uint8_t const* qmin = q0;
    std::uint8_t const* omin = o0;
    for (std::size_t i : idx) {
        qmin = std::min(qmin, reinterpret_cast<std::uint8_t const*>(batch.items[i].request.device_query));
        omin = std::min(omin, reinterpret_cast<std::uint8_t const*>(batch.items[i].request.device_output));
    }
    bool strided = true;
    for (std::size_t i : idx) {
        PagedDecodeRequest const& r = batch.items[i].request;
        std::ptrdiff_t const dq = reinterpret_cast<std::uint8_t const*>(r.device_query) - qmin;
        std::ptrdiff_t const dout = reinterpret_cast<std::uint8_t const*>(r.device_output) - omin;
        strided = strided && dq % row_bytes == 0 && dout == dq && r.attention_scale
            == batch.items[idx[0]].request.attention_scale;
    }
    if (!strided) {
        TokenTransactionBackend::attendLayerBatch(batch);
        return;
    }
    // Validate and upload every lane first (per-lane status like the reference).
    std::vector<std::size_t> ready;
    for (std::size_t k = 0; k < idx.size(); ++k) {
        CudaStatus const s = txns[k]->prepareAttention(batch.items[idx[k]].request);
        batch.items[idx[k]].status = mapCuda(s);
        if (s.ok()) {
            ready.push_back(k);
        }
    }
    if (ready.empty()) {
        return;
    }
    std::vector<kk_attn_lane> lanes(ready.size());
    std::vector<kk_attn_item> items(ready.size());
    for (std::size_t j = 0; j < ready.size(); ++j) {
        CudaTxn* t = txns[ready[j]];
        PagedDecodeRequest const& r = batch.items[idx[ready[j]]].request;
        std::uint32_t const off = t->descOffset() + static_cast<std::uint32_t>(Arena::kDescOff / sizeof(kk_page_desc));
        std::uint32_t const count = static_cast<std::uint32_t>(t->reserved_.entries().size());
        std::uint32_t const row = static_cast<std::uint32_t>(
            (reinterpret_cast<std::uint8_t const*>(r.device_query) - qmin) / row_bytes);
        lanes[j] = kk_attn_lane{off, count, t->reserved_.tokenCount(), static_cast<std::uint32_t>(j), 1, row, 0, 0};
        items[j] = kk_attn_item{static_cast<std::uint32_t>(j), off, off + count, 0};
    }
    cudaStream_t const s = static_cast<cudaStream_t>(stream_);
    PagedDecodeRequest const& rq = batch.items[idx[ready[0]]].request;
    int rc = st_->attendPlanned(lanes.data(), static_cast<std::uint32_t>(lanes.size()), rq.layer, qmin,
        const_cast<std::uint8_t*>(omin), rq.attention_scale, rq.device_workspace, rq.workspace_bytes, stream_);
    if (rc < 0) {
        // Without the stream's scratch: one item per lane, through the
        // caller's batch buffers (as the reference's batched launch uses them).
        std::size_t const lane_bytes = ready.size() * sizeof(kk_attn_lane);
        std::size_t const bytes = lane_bytes + ready.size() * sizeof(kk_attn_item);
        if (batch.host_items == nullptr || batch.device_items == nullptr
            || batch.item_capacity * sizeof(DevicePagedDecodeBatchItem) < bytes) {
            rc = KK_EINVAL;
        } else {
            auto* host = reinterpret_cast<std::uint8_t*>(batch.host_items);
            std::memcpy(host, lanes.data(), lane_bytes);
            std::memcpy(host + lane_bytes, items.data(), bytes - lane_bytes);
            rc = static_cast<int>(cudaMemcpyAsync(batch.device_items, batch.host_items, bytes,
                cudaMemcpyHostToDevice, s));
        }
        if (rc == 0) {
            auto* dev = reinterpret_cast<std::uint8_t*>(batch.device_items);
            std::uint32_t const row = hq * st_->config.kv_layout.head_dimension;
            rc = kk::attentionLaunch(&st_->storage.pools, rq.layer, hq,
                reinterpret_cast<kk_page_desc const*>(st_->arena.dev),
                reinterpret_cast<kk_attn_lane const*>(dev), static_cast<std::uint32_t>(ready.size()),
                reinterpret_cast<kk_attn_item const*>(dev + lane_bytes), static_cast<std::uint32_t>(ready.size()),
                reinterpret_cast<std::uint16_t const*>(qmin), row,
                reinterpret_cast<std::uint16_t*>(const_cast<std::uint8_t*>(omin)), row, rq.attention_scale,
                rq.device_workspace, rq.workspace_bytes, st_->statusWord(stream_), s);
        }
    }
    std::uint64_t ok_lanes = 0;
    for (std::size_t k : ready) {
        if (rc != 0) {
            batch.items[idx[k]].status = txns[k]->fail(submitError(rc));
        } else {
            txns[k]->markSubmitted();
            ++ok_lanes;
        }
    }
    if (ok_lanes != 0) {
        st_->batched_submissions.fetch_add(1, std::memory_order_relaxed);
        st_->batched_lanes.fetch_add(ok_lanes, std::memory_order_relaxed);
    }
}

class CudaBackend final : public EngineKvBackend {
public:
    explicit CudaBackend(std::shared_ptr<State> st) : st_(std::move(st)) {}

    EngineKvBackendKind kind() const noexcept override { return st_->kind; }
    EngineKvConfig config() const noexcept override { return st_->config; }

    EngineKvStatus createRequest(RequestId id) override
    {
        std::lock_guard<std::mutex> lock(st_->mutex);
        if (!st_->config.valid() || !st_->storage.status.ok()) {
            return {EngineKvError::InvalidState};
        }
        KvCacheError const e = st_->create(id);
        if (e == KvCacheError::None) {
            st_->committed_lengths.emplace(id, 0);
        }
        return mapMetadata(e);
    }

    EngineKvStatus forkRequest(RequestId source, RequestId child) override
    {
        std::lock_guard<std::mutex> lock(st_->mutex);
        auto const src = st_->committed_lengths.find(source);
        if (src == st_->committed_lengths.end()) {
            return {EngineKvError::RequestNotFound};
        }
        std::uint32_t const length = src->second;
        KvCacheError const e = st_->fork(source, child);
        if (e == KvCacheError::None) {
            st_->committed_lengths.emplace(child, length);
        }
        return mapMetadata(e);
    }

    EngineKvStatus releaseRequest(RequestId id) override
    {
        std::lock_guard<std::mutex> lock(st_->mutex);
        KvCacheError const e = st_->release(id);
        if (e == KvCacheError::None) {
            st_->committed_lengths.erase(id);
        }
        return mapMetadata(e);
    }

    TokenReserveResult reserveToken(ReserveTokenRequest const& request) override
    {
        TokenReserveResult result;
        std::lock_guard<std::mutex> lock(st_->mutex);
        auto const length = st_->committed_lengths.find(request.request_id);
        if (request.request_id == kInvalidRequestId) {
            result.status = {EngineKvError::InvalidArgument};
            return result;
        }
        if (length == st_->committed_lengths.end()) {
            result.status = {EngineKvError::RequestNotFound};
            return result;
        }
        TokenReservationResult reservation = st_->reserve(request.request_id, request.expected_committed_tokens);
        if (!reservation.ok()) {
            result.status = mapMetadata(reservation.error);
            return result;
        }
        // The two-pool runtime pins the reservation's pages with a lease; the
        // fixed-page runtime has none (its pages cannot be promoted away, and
        // its device work is waited for under the backend lock, as in the
        // reference's FixedCudaKvCache).
        PageLeaseAcquireResult lease;
        if (st_->mgr) {
            lease = st_->mgr->acquireTokenReservationPin(reservation.reservation_id);
            if (!lease.ok()) {
                static_cast<void>(st_->rollback(reservation.reservation_id));
                result.status = mapMetadata(lease.error);
                return result;
            }
        }
        CudaStatus const begun = beginChecks(reservation);
        if (!begun.ok()) {
            if (st_->mgr) {
                static_cast<void>(st_->mgr->releasePageLease(lease.lease_id));
            }
            static_cast<void>(st_->rollback(reservation.reservation_id));
            result.status = mapCuda(begun);
            return result;
        }
        std::unique_ptr<CudaTxn> txn;
        try {
            txn = std::make_unique<CudaTxn>(st_, reservation.reservation_id, reservation.request_id,
                lease.lease_id, std::move(reservation.before), std::move(reservation.reserved),
                request.stream);
        } catch (...) {
            if (st_->mgr) {
                static_cast<void>(st_->mgr->releasePageLease(lease.lease_id));
            }
            static_cast<void>(st_->rollback(reservation.reservation_id));
            result.status = {EngineKvError::ResourceExhausted};
            return result;
        }
        result.transaction = TokenTransaction(std::move(txn), reservation.reservation_id,
            reservation.request_id, reservation.logical_token_position,
            st_->config.kv_layout.layer_count, request.stream);
        if (!result.transaction.valid()) {
            result.status = {EngineKvError::InternalError};
            return result;
        }
        ++st_->active;
        result.status = {};
        return result;
    }

    EngineKvBackendSnapshot snapshot() const override
    {
        std::lock_guard<std::mutex> lock(st_->mutex);
        EngineKvBackendSnapshot r;
        std::uint64_t committed = 0;
        for (auto const& e : st_->committed_lengths) {
            committed += e.second;
        }
        r.request_count = st_->committed_lengths.size();
        r.active_transaction_count = st_->active;
        r.committed_token_count = committed;
        r.batched_attention_submissions = st_->batched_submissions.load(std::memory_order_relaxed);
        r.batched_attention_lanes = st_->batched_lanes.load(std::memory_order_relaxed);
        r.storage_reserved_bytes = st_->storage.micro_bytes + st_->storage.extent_bytes;
        if (st_->fixed) {
            FixedPageManagerSnapshot const f = st_->fixed->snapshot();
            r.primary_page_tokens = st_->fixed->tokensPerPage();
            r.secondary_page_tokens = 0;
            r.primary_page_capacity = f.pool.total_slots;
            r.allocated_primary_pages = f.pool.allocated_slots;
            r.successful_primary_allocations = f.pool.successful_allocations;
            r.failed_primary_allocations = f.pool.failed_allocations;
            return r;
        }
        KvCacheManagerSnapshot const m = st_->mgr->snapshot();
        r.primary_page_tokens = kMicroPageTokenCapacity;
        r.secondary_page_tokens = kExtentPageTokenCapacity;
        r.primary_page_capacity = m.micro_pool.total_slots;
        r.secondary_page_capacity = m.extent_pool.total_slots;
        r.allocated_primary_pages = m.micro_pool.allocated_slots;
        r.allocated_secondary_pages = m.extent_pool.allocated_slots;
        r.successful_primary_allocations = m.micro_pool.successful_allocations;
        r.successful_secondary_allocations = m.extent_pool.successful_allocations;
        r.failed_primary_allocations = m.micro_pool.failed_allocations;
        r.failed_secondary_allocations = m.extent_pool.failed_allocations;
        return r;
    }

    bool checkInvariants() const override
    {
        std::lock_guard<std::mutex> lock(st_->mutex);
        return st_->config.valid() && st_->storage.status.ok() && st_->metadataConsistent();
    }

    State* state() const noexcept { return st_.get(); }

private:
    // Storage-side checks of a new transaction (reference
    // CudaKvStorage::beginEngineTransaction, transaction.cpp:336-370).
    CudaStatus beginChecks(TokenReservationResult const& r)
    {
        if (!st_->storage.status.ok()) {
            return st_->storage.status;
        }
        auto valid = [this](BlockTable const& t) {
            if (!st_->tableWellFormed(t)) {
                return false;
            }
            for (MappingEntry const& e : t.entries()) {
                std::uint32_t const cap = e.kind == PageKind::Micro ? st_->storage.pools.micro_capacity
                                                                    : st_->storage.pools.extent_capacity;
                if (e.handle.slot >= cap) {
                    return false;
                }
            }
            return true;
        };
        // `before` is `reserved` less the token just reserved: once `reserved`
        // passed, every entry the two share is valid, and only the entry
        // where they differ needs a look (the same verdict as checking
        // `before` in full, which any other shape falls back to).
        auto valid_before = [&](BlockTable const& b, BlockTable const& res) {
            auto const& be = b.entries();
            auto const& re = res.entries();
            std::size_t const nb = be.size();
            if (nb == 0 || (re.size() != nb && re.size() != nb + 1)
                || !std::equal(be.begin(), be.end() - 1, re.begin())) {
                return valid(b);
            }
            MappingEntry const& last = be.back();
            if (re.size() == nb + 1 && last == re[nb - 1]) {
                return true;  // a prefix of a valid table
            }
            std::uint16_t const cap = st_->fixed ? st_->fixed->tokensPerPage() : pageTokenCapacity(last.kind);
            std::uint32_t const slots = last.kind == PageKind::Micro ? st_->storage.pools.micro_capacity
                                                                     : st_->storage.pools.extent_capacity;
            if (!last.handle.isStructurallyValid() || last.kind != last.handle.kind || cap == 0
                || last.valid_tokens == 0 || last.valid_tokens > cap || last.handle.slot >= slots
                || last.logical_token_begin != (nb > 1 ? be[nb - 2].logicalTokenEnd() : 0u)) {
                return false;
            }
            return std::none_of(be.begin(), be.end() - 1,
                [&](MappingEntry const& e) { return e.handle == last.handle; });
        };
        std::uint32_t const kv = st_->config.kv_layout.kv_head_count;
        if (!valid(r.reserved) || !valid_before(r.before, r.reserved)
            || r.reserved.tokenCount() != r.before.tokenCount() + 1
            || st_->config.query_head_count < kv || st_->config.query_head_count % kv != 0
            || r.reserved.entries().empty()) {
            return {CudaError::InvalidArgument, 0};
        }
        if (st_->consumeFailure(CudaFailurePoint::Submission)) {
            return {CudaError::SubmissionFailed, 0};
        }
        return {};
    }

    std::shared_ptr<State> st_;
};

} // namespace

std::unique_ptr<EngineKvBackend> createHeterogeneousCudaEngineKvBackend(
    EngineKvConfig config, std::uint32_t micro_cap, std::uint32_t extent_cap)
{
    if (!config.valid() || micro_cap == 0 || extent_cap == 0) {
        return nullptr;
    }
    try {
        return std::make_unique<CudaBackend>(std::make_shared<State>(config, micro_cap, extent_cap));
    } catch (...) {
        return nullptr;
    }
}

std::unique_ptr<EngineKvBackend> createFixedCudaEngineKvBackend(
    EngineKvConfig config, std::uint16_t tokens_per_page, std::uint32_t page_capacity)
{
    if (!config.valid() || tokens_per_page == 0 || page_capacity == 0) {
        return nullptr;
    }
    try {
        return std::make_unique<CudaBackend>(
            std::make_shared<State>(config, tokens_per_page, page_capacity, true));
    } catch (...) {
        return nullptr;
    }
}

bool injectCudaEngineFailureOnce(EngineKvBackend& backend, CudaFailurePoint point) noexcept
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr) {
        return false;
    }
    std::lock_guard<std::mutex> lock(b->state()->fault_mutex);
    (point == CudaFailurePoint::Submission ? b->state()->fail_submission
                                           : b->state()->fail_completion) = true;
    b->state()->failure_armed.store(true, std::memory_order_release);
    return true;
}

kk_kv_pools const* cudaBackendPools(EngineKvBackend const& backend) noexcept
{
    auto const* b = dynamic_cast<CudaBackend const*>(&backend);
    return b == nullptr ? nullptr : &b->state()->storage.pools;
}

bool fusedLane(TokenTransaction const& transaction, FusedLane& out) noexcept
{
    auto const* t = dynamic_cast<CudaTxn const*>(transaction.backend());
    if (t == nullptr) {
        return false;
    }
    out.before = &t->before();
    out.reserved = &t->reserved();
    return true;
}

bool cudaBackendTable(EngineKvBackend const& backend, RequestId id, BlockTable& out)
{
    auto const* b = dynamic_cast<CudaBackend const*>(&backend);
    if (b == nullptr) {
        return false;
    }
    std::optional<BlockTable> t = b->state()->table(id);
    if (!t) {
        return false;
    }
    out = std::move(*t);
    return true;
}

EngineKvStatus cudaBackendAppend(EngineKvBackend& backend, RequestId id, std::uint32_t n)
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr) {
        return {EngineKvError::InvalidArgument};
    }
    State* st = b->state();
    std::lock_guard<std::mutex> lock(st->mutex);
    auto length = st->committed_lengths.find(id);
    if (length == st->committed_lengths.end()) {
        return {EngineKvError::RequestNotFound};
    }
    KvCacheError const e = st->append(id, n);
    if (e == KvCacheError::None) {
        length->second += n;
    }
    return mapMetadata(e);
}

EngineKvStatus cudaBackendSeal(EngineKvBackend& backend, RequestId id)
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr) {
        return {EngineKvError::InvalidArgument};
    }
    std::lock_guard<std::mutex> lock(b->state()->mutex);
    return mapMetadata(b->state()->seal(id));
}

EngineKvStatus cudaBackendPromote(EngineKvBackend& backend, RequestId id, std::uint32_t begin,
    CudaStream stream)
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr) {
        return {EngineKvError::InvalidArgument};
    }
    State* st = b->state();
    if (!st->mgr) {
        return {EngineKvError::InvalidArgument};  // fixed pages have no extent pool
    }
    PromotionPrepareResult prepared;
    PageLeaseAcquireResult lease;
    {
        std::lock_guard<std::mutex> lock(st->mutex);
        prepared = st->mgr->preparePromotion(id, begin);
        if (!prepared.ok()) {
            return mapMetadata(prepared.error);
        }
        lease = st->mgr->acquirePromotionIoLease(prepared.promotion_id);
        if (!lease.ok()) {
            static_cast<void>(st->mgr->rollbackPromotion(prepared.promotion_id));
            return mapMetadata(lease.error);
        }
    }
    std::uint32_t slots[8];
    for (int k = 0; k < 8; ++k) {
        slots[k] = prepared.source_handles[k].slot;
    }
    cudaStream_t const s = static_cast<cudaStream_t>(stream);
    int rc = kk_kv_promote(&st->storage.pools, slots, prepared.target_handle.slot, s);
    if (rc == 0) {
        rc = static_cast<int>(cudaStreamSynchronize(s));
    }
    std::lock_guard<std::mutex> lock(st->mutex);
    static_cast<void>(st->mgr->releasePageLease(lease.lease_id));
    if (rc != 0) {
        static_cast<void>(st->mgr->rollbackPromotion(prepared.promotion_id));
        return {EngineKvError::ExecutionFailed};
    }
    return mapMetadata(st->mgr->commitPromotion(prepared.promotion_id));
}

EngineKvStatus cudaBackendGather(EngineKvBackend& backend, RequestId id, void* device_output,
    CudaStream stream)
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr || device_output == nullptr) {
        return {EngineKvError::InvalidArgument};
    }
    State* st = b->state();
    std::vector<kk_page_desc> descs;
    std::uint32_t tokens = 0;
    PageLeaseAcquireResult lease;
    // The fixed-page runtime has no leases: its gather runs under the
    // backend lock, start to finish (the reference's FixedCudaKvCache waits
    // for its device work inside the lock).
    std::unique_lock<std::mutex> fixed_lock(st->mutex, std::defer_lock);
    if (!st->mgr) {
        fixed_lock.lock();
    }
    {
        std::unique_lock<std::mutex> lock(st->mutex, std::defer_lock);
        if (st->mgr) {
            lock.lock();
            lease = st->mgr->acquireRequestReadLease(id);
            if (!lease.ok()) {
                return mapMetadata(lease.error);
            }
        }
        std::optional<BlockTable> const table = st->table(id);
        if (!table && !st->mgr) {
            return {EngineKvError::RequestNotFound};
        }
        if (table) {
            tokens = table->tokenCount();
            for (MappingEntry const& e : table->entries()) {
                descs.push_back(kk_page_desc{e.handle.slot, e.logical_token_begin, e.valid_tokens,
                    static_cast<std::uint8_t>(e.kind), 0, 0});
            }
        }
    }
    cudaStream_t const s = static_cast<cudaStream_t>(stream);
    int rc = 0;
    if (!descs.empty()) {
        void* d_descs = nullptr;
        std::size_t const bytes = descs.size() * sizeof(kk_page_desc);
        rc = static_cast<int>(cudaMallocAsync(&d_descs, bytes, s));
        if (rc == 0) {
            rc = static_cast<int>(cudaMemcpyAsync(d_descs, descs.data(), bytes, cudaMemcpyHostToDevice, s));
            if (rc == 0) {
                rc = kk_kv_gather(&st->storage.pools, static_cast<kk_page_desc const*>(d_descs),
                    static_cast<std::uint32_t>(descs.size()), tokens, static_cast<std::uint16_t*>(device_output), s);
            }
            cudaFreeAsync(d_descs, s);
        }
        if (rc == 0) {
            rc = static_cast<int>(cudaStreamSynchronize(s));
        }
    }
    if (st->mgr) {
        std::lock_guard<std::mutex> lock(st->mutex);
        static_cast<void>(st->mgr->releasePageLease(lease.lease_id));
    }
    if (descs.empty()) {
        return {EngineKvError::InvalidArgument};  // nothing committed to gather
    }
    return rc == 0 ? EngineKvStatus{} : EngineKvStatus{EngineKvError::ExecutionFailed};
}

namespace {

std::uint32_t promoteWave(EngineKvBackend& backend,
    std::vector<std::pair<RequestId, std::uint32_t>> const& runs, CudaStream stream);

} // namespace

std::uint32_t cudaBackendPromoteMany(EngineKvBackend& backend,
    std::vector<std::pair<RequestId, std::uint32_t>> const& runs, CudaStream stream)
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr || !b->state()->mgr) {
        return 0;  // only the two-pool runtime promotes
    }
    // A request with a prepared promotion holds a reservation, so a second
    // run of the same request cannot be prepared until the first commits:
    // promote in waves holding at most one run per request, in run order.
    std::vector<std::pair<RequestId, std::uint32_t>> rest = runs;
    std::uint32_t committed = 0;
    while (!rest.empty()) {
        std::vector<std::pair<RequestId, std::uint32_t>> wave;
        std::vector<std::pair<RequestId, std::uint32_t>> later;
        for (auto const& run : rest) {
            bool const taken = std::any_of(wave.begin(), wave.end(),
                [&run](auto const& w) { return w.first == run.first; });
            (taken ? later : wave).push_back(run);
        }
        committed += promoteWave(backend, wave, stream);
        rest.swap(later);
    }
    return committed;
}

namespace {

std::uint32_t promoteWave(EngineKvBackend& backend,
    std::vector<std::pair<RequestId, std::uint32_t>> const& runs, CudaStream stream)
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr || runs.empty()) {
        return 0;
    }
    State* st = b->state();
    struct Pending {
        PromotionPrepareResult prepared;
        PageLeaseAcquireResult lease;
    };
    std::vector<Pending> pending;
    pending.reserve(runs.size());
    {
        std::lock_guard<std::mutex> lock(st->mutex);
        for (auto const& run : runs) {
            Pending p;
            p.prepared = st->mgr->preparePromotion(run.first, run.second);
            if (!p.prepared.ok()) {
                continue;
            }
            p.lease = st->mgr->acquirePromotionIoLease(p.prepared.promotion_id);
            if (!p.lease.ok()) {
                static_cast<void>(st->mgr->rollbackPromotion(p.prepared.promotion_id));
                continue;
            }
            pending.push_back(p);
        }
    }
    if (pending.empty()) {
        return 0;
    }
    cudaStream_t const s = static_cast<cudaStream_t>(stream);
    int rc = 0;
    for (Pending const& p : pending) {
        std::uint32_t slots[8];
        for (int k = 0; k < 8; ++k) {
            slots[k] = p.prepared.source_handles[k].slot;
        }
        if (rc == 0) {
            rc = kk_kv_promote(&st->storage.pools, slots, p.prepared.target_handle.slot, s);
        }
    }
    if (rc == 0) {
        rc = static_cast<int>(cudaStreamSynchronize(s));
    }
    std::uint32_t committed = 0;
    std::lock_guard<std::mutex> lock(st->mutex);
    for (Pending const& p : pending) {
        static_cast<void>(st->mgr->releasePageLease(p.lease.lease_id));
        if (rc != 0) {
            static_cast<void>(st->mgr->rollbackPromotion(p.prepared.promotion_id));
        } else if (st->mgr->commitPromotion(p.prepared.promotion_id) == KvCacheError::None) {
            ++committed;
        }
    }
    return committed;
}

} // namespace

void noteStreamCompleted(EngineKvBackend& backend, CudaStream stream) noexcept
{
    auto* b = dynamic_cast<CudaBackend*>(&backend);
    if (b == nullptr) {
        return;
    }
    State* st = b->state();
    st->noteCompleted(stream, st->submit_seq.load());
}

} // namespace kimkvcache

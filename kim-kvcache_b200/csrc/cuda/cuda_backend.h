// CUDA heterogeneous KV backend behind the EngineKvBackend SPI.
//
// Public factory and fault hook follow the reference
// (include/kim-kv/cuda/cuda_engine_kv_backend.h:11-29, cuda_status.h:9-82):
// createHeterogeneousCudaEngineKvBackend owns a KvCacheManager and two device
// page pools; reserveToken = metadata reservation + page lease + a
// transaction object; commit = completion check + lease release + metadata
// commit; rollback = wait + lease release + metadata rollback.
//
// B200 design differences (same observable semantics):
//  * no per-token cudaMalloc / event: per-transaction device metadata lives in
//    a preallocated arena and is uploaded only if the per-layer SPI is used;
//  * the fused decode step of this library's model runner reads the
//    transaction tables directly (fusedLane) and advances the state machine
//    with TokenTransaction::submitFusedLayers; the runner synchronises its
//    stream once per step and tells the backend (noteStreamCompleted), so
//    commits do not synchronise again.
#pragma once

#include "../host/engine_kv.h"
#include "../../../include/kk_kernels.h"

#include <cstdint>
#include <utility>
#include <vector>
#include <memory>
#include <string_view>

namespace kimkvcache {

using CudaStream = void*;

enum class CudaError : std::uint8_t {
    None,
    InvalidArgument,
    RuntimeUnavailable,
    AllocationFailed,
    SubmissionFailed,
    NotReady,
    ExecutionFailed,
    InternalError,
};

struct CudaStatus final {
    CudaError error{CudaError::None};
    int native_error{0};
    [[nodiscard]] constexpr bool ok() const noexcept { return error == CudaError::None; }
};

enum class CudaFailurePoint : std::uint8_t { Submission, Completion };

[[nodiscard]] std::unique_ptr<EngineKvBackend> createHeterogeneousCudaEngineKvBackend(
    EngineKvConfig config, std::uint32_t micro_page_capacity, std::uint32_t extent_page_capacity);

// Fixed-page backend behind the same SPI (reference createFixedCudaEngineKvBackend,
// include/kim-kv/cuda/cuda_engine_kv_backend.h:19-22, src/cuda/engine/backend.cpp:579-598):
// FixedPageManager metadata, one device pool of page_capacity pages of
// tokens_per_page tokens (8, 16, 32 or 64; the kernels read the page size from
// kk_kv_pools::micro_page_tokens). Fork, partial-tail copy-on-write, rollback
// and the fused decode step work as for the two-pool backend; there is no
// promotion and there are no page leases.
[[nodiscard]] std::unique_ptr<EngineKvBackend> createFixedCudaEngineKvBackend(
    EngineKvConfig config, std::uint16_t tokens_per_page, std::uint32_t page_capacity);
[[nodiscard]] bool injectCudaEngineFailureOnce(EngineKvBackend& backend, CudaFailurePoint point) noexcept;

// ---- library-internal hooks used by the CUDA model runner ---------------------

// What the fused step needs to know about one lane's reserved token.
struct FusedLane final {
    BlockTable const* before{nullptr};
    BlockTable const* reserved{nullptr};
};

// Device pools of a CUDA backend created by this library (nullptr otherwise).
[[nodiscard]] kk_kv_pools const* cudaBackendPools(EngineKvBackend const& backend) noexcept;

// Lane view of a transaction reserved from a CUDA backend of this library.
[[nodiscard]] bool fusedLane(TokenTransaction const& transaction, FusedLane& out) noexcept;

// The runner synchronised `stream`: every transaction submitted on it so far
// has completed (commits then skip their own synchronisation).
void noteStreamCompleted(EngineKvBackend& backend, CudaStream stream) noexcept;

// Library extensions for building long prefixes without running the model
// (used by the synthetic workloads and tests; the reference builds such
// tables with KvCacheManager::append and the promotion path of CudaKvCache):
[[nodiscard]] bool cudaBackendTable(EngineKvBackend const& backend, RequestId id, BlockTable& out);
// Metadata append of n tokens (KV contents are written separately).
[[nodiscard]] EngineKvStatus cudaBackendAppend(EngineKvBackend& backend, RequestId id, std::uint32_t n);
[[nodiscard]] EngineKvStatus cudaBackendSeal(EngineKvBackend& backend, RequestId id);
// prepare -> IO lease -> device copy (8 micro -> 1 extent) -> wait -> release
// -> commit, rolled back on any failure (reference CudaKvCache::promote,
// src/cuda/kv/cache.cpp:172-229).
[[nodiscard]] EngineKvStatus cudaBackendPromote(EngineKvBackend& backend, RequestId id,
    std::uint32_t logical_begin, CudaStream stream);
// K6 gather (reference CudaKvCache::gather / CudaKvStorage::gatherAsync,
// src/cuda/kv/gather.cpp:9-107): the request's committed KV as one
// contiguous [layer][K|V][token][head][dim] FP16 tensor at device_output
// (tokenCount() tokens). Pages are pinned by a read lease for the copy; the
// call waits for it.
[[nodiscard]] EngineKvStatus cudaBackendGather(EngineKvBackend& backend, RequestId id,
    void* device_output, CudaStream stream);
// The same for several (request, logical_begin) runs with one device wait:
// every promotion that prepares is copied, then all are committed (or rolled
// back if the copies failed). Runs that cannot be promoted (not 8 sealed,
// full, unshared micro pages) are skipped. Returns how many were committed.
[[nodiscard]] std::uint32_t cudaBackendPromoteMany(EngineKvBackend& backend,
    std::vector<std::pair<RequestId, std::uint32_t>> const& runs, CudaStream stream);

} // namespace kimkvcache

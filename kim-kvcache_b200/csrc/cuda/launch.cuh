// Kernel launch helper: cudaLaunchKernelEx with optional programmatic
// dependent launch (PDL) and thread-block cluster dimensions.
#pragma once

#include "common.cuh"

#include <cuda_runtime.h>

namespace kk {

// Set by kk_set_pdl(); read when a launch is issued on this host thread.
extern thread_local bool g_pdl_enabled;

// Asks, once per kernel, for the largest shared-memory carveout. CTAs of
// different kernels share an SM only when the SM's L1/shared split fits
// both; with every kernel of the decode step on the maximum split, a CTA of
// the next kernel (launched early under programmatic dependent launch) can
// sit beside one of the current kernel and prefetch its weights.
void preferMaxSharedCarveout(void const* kernel);

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, std::size_t smem,
    cudaStream_t stream, unsigned cluster_x, Args&&... args)
{
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attrs[2];
    unsigned n = 0;
    if (g_pdl_enabled) {
        attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_x > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = cluster_x;
        attrs[n].val.clusterDim.y = 1;
        attrs[n].val.clusterDim.z = 1;
        ++n;
    }
    config.attrs = attrs;
    config.numAttrs = n;
    preferMaxSharedCarveout(reinterpret_cast<void const*>(kernel));
    return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

// Reads and clears one module's device status word (synchronous).
inline int readStatus(void const* symbol, cudaStream_t stream)
{
    unsigned int value = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&value, symbol, sizeof(value), 0,
        cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) {
        e = cudaStreamSynchronize(stream);
    }
    if (e != cudaSuccess) {
        return static_cast<int>(e);
    }
    if (value != 0) {
        unsigned int const zero = 0;
        cudaMemcpyToSymbolAsync(symbol, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    return static_cast<int>(value);
}

} // namespace kk

// Device status words of the kernel modules, the PDL switch and the
// shared-memory carveout requests of the launch helper.
#include "../../../include/kk_kernels.h"
#include "launch.cuh"

#include <algorithm>
#include <mutex>
#include <vector>

namespace kk {

thread_local bool g_pdl_enabled = false;

void preferMaxSharedCarveout(void const* kernel)
{
    static std::mutex mutex;
    static std::vector<void const*> done;
    std::lock_guard<std::mutex> lock(mutex);
    if (std::find(done.begin(), done.end(), kernel) != done.end()) {
        return;
    }
    // A hint: a failure leaves the default split, which only costs overlap.
    static_cast<void>(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
        cudaSharedmemCarveoutMaxShared));
    done.push_back(kernel);
}

int attentionStatus(cudaStream_t stream);
int attentionTmaStatus(cudaStream_t stream);
int pagesStatus(cudaStream_t stream);
int gemmStatus(cudaStream_t stream);

} // namespace kk

extern "C" {

int kk_device_status(void* stream)
{
    cudaStream_t const s = static_cast<cudaStream_t>(stream);
    int const codes[4] = {kk::attentionStatus(s), kk::attentionTmaStatus(s), kk::pagesStatus(s),
        kk::gemmStatus(s)};
    for (int c : codes) {
        if (c != 0) {
            return c;
        }
    }
    return 0;
}

void kk_set_pdl(int enabled) { kk::g_pdl_enabled = enabled != 0; }

} // extern "C"

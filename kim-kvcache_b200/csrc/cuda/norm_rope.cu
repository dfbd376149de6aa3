// K3 — row-wise kernels of the decoder: RMSNorm (optionally fused with the
// embedding gather that starts the residual stream), rotate-half RoPE,
// SiLU-gate and the FP16 residual add. Rounding points follow the reference
// (src/cuda/model/kernels.cu:16-218): FP32 statistics, FP16 outputs.
// In the decode step RoPE and the SiLU gate run fused in the projection
// epilogues (gemm_tc.cu); the standalone kernels serve the per-layer SPI path.
#include "../../../include/kk_kernels.h"
#include "kernels_internal.h"
#include "launch.cuh"

namespace kk {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* scratch)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    int const warp = threadIdx.x / 32;
    if ((threadIdx.x & 31) == 0) {
        scratch[warp] = v;
    }
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) {
        total += scratch[w];
    }
    return total;
}

// One CTA per row; 8 FP16 per thread per step (cols % 8 == 0). y (the
// normalised row) and sq_out (the row's sum of squares) are optional.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(__half const* x,
    __half const* embed, std::uint32_t const* tokens, __half const* weight, __half* hidden,
    __half* y, std::uint32_t cols, float eps, float* sq_out)
{
    pdl_launch_dependents();  // dependents only prefetch weights before their own wait
    pdl_wait();
    __shared__ float scratch[kNormThreads / 32];
    std::uint32_t const row = blockIdx.x;
    __half const* src = embed != nullptr
        ? embed + std::uint64_t(tokens[row]) * cols
        : x + std::uint64_t(row) * cols;
    float sum = 0.f;
    for (std::uint32_t i = threadIdx.x * 8u; i < cols; i += kNormThreads * 8u) {
        uint4 const raw = *reinterpret_cast<uint4 const*>(src + i);
        __half const* h = reinterpret_cast<__half const*>(&raw);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float const f = __half2float(h[e]);
            sum += f * f;
        }
        if (hidden != nullptr) {
            *reinterpret_cast<uint4*>(hidden + std::uint64_t(row) * cols + i) = raw;
        }
    }
    float const total = block_sum(sum, scratch);
    if (sq_out != nullptr && threadIdx.x == 0) {
        sq_out[row] = total;
    }
    if (y == nullptr) {
        return;
    }
    float const scale = rsqrtf(total / static_cast<float>(cols) + eps);
    for (std::uint32_t i = threadIdx.x * 8u; i < cols; i += kNormThreads * 8u) {
        uint4 const raw = *reinterpret_cast<uint4 const*>(src + i);
        uint4 const wraw = *reinterpret_cast<uint4 const*>(weight + i);
        __half const* h = reinterpret_cast<__half const*>(&raw);
        __half const* w = reinterpret_cast<__half const*>(&wraw);
        __align__(16) __half out[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            out[e] = __float2half_rn(__half2float(h[e]) * scale * __half2float(w[e]));
        }
        *reinterpret_cast<uint4*>(y + std::uint64_t(row) * cols + i) =
            *reinterpret_cast<uint4 const*>(out);
    }
}

// grid (rows, heads); thread d < head_dim/2 rotates the pair (d, d + half).
__global__ void rope_kernel(__half* q, std::uint32_t q_stride, __half* k,
    std::uint32_t k_stride, std::uint32_t const* positions, std::uint32_t q_heads,
    std::uint32_t head_dim, float theta)
{
    pdl_wait();
    std::uint32_t const row = blockIdx.x;
    std::uint32_t const head = blockIdx.y;
    std::uint32_t const half_dim = head_dim / 2;
    std::uint32_t const d = threadIdx.x;
    if (d >= half_dim) {
        return;
    }
    __half* base = head < q_heads ? q + std::uint64_t(row) * q_stride + head * head_dim
                                  : k + std::uint64_t(row) * k_stride + (head - q_heads) * head_dim;
    float const inv_freq = powf(theta, -2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
    float const angle = static_cast<float>(positions[row]) * inv_freq;
    float const c = cosf(angle);
    float const s = sinf(angle);
    float const a = __half2float(base[d]);
    float const b = __half2float(base[d + half_dim]);
    base[d] = __float2half_rn(a * c - b * s);
    base[d + half_dim] = __float2half_rn(b * c + a * s);
}

__global__ void silu_mul_kernel(__half const* gate, __half const* up, __half* out,
    std::uint64_t count)
{
    pdl_wait();
    for (std::uint64_t i = blockIdx.x * std::uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += std::uint64_t(gridDim.x) * blockDim.x) {
        float const g = __half2float(gate[i]);
        out[i] = __float2half_rn(g / (1.0f + expf(-g)) * __half2float(up[i]));
    }
}

__global__ void residual_add_kernel(__half* hidden, __half const* update, std::uint64_t count)
{
    pdl_wait();
    for (std::uint64_t i = blockIdx.x * std::uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += std::uint64_t(gridDim.x) * blockDim.x) {
        hidden[i] = __hadd(hidden[i], update[i]);
    }
}

unsigned gridFor(std::uint64_t count)
{
    std::uint64_t const blocks = (count + 255u) / 256u;
    return static_cast<unsigned>(blocks < 4096u ? (blocks == 0 ? 1 : blocks) : 4096u);
}

} // namespace
} // namespace kk

extern "C" {

int kk_rmsnorm(const uint16_t* x, const uint16_t* weight, uint16_t* y, uint32_t rows,
    uint32_t cols, float eps, void* stream)
{
    if (x == nullptr || weight == nullptr || y == nullptr || cols == 0 || cols % 8 != 0
        || !(eps > 0.f)) {
        return KK_EINVAL;
    }
    if (rows == 0) {
        return 0;
    }
    return static_cast<int>(kk::launch(kk::rmsnorm_kernel, dim3(rows), dim3(kk::kNormThreads), 0,
        static_cast<cudaStream_t>(stream), 1, reinterpret_cast<__half const*>(x),
        static_cast<__half const*>(nullptr), static_cast<std::uint32_t const*>(nullptr),
        reinterpret_cast<__half const*>(weight), static_cast<__half*>(nullptr),
        reinterpret_cast<__half*>(y), cols, eps, static_cast<float*>(nullptr)));
}

int kk_embed_rmsnorm(const uint16_t* embed, const uint32_t* tokens, const uint16_t* weight,
    uint16_t* hidden, uint16_t* y, uint32_t rows, uint32_t cols, float eps, void* stream)
{
    if (embed == nullptr || tokens == nullptr || weight == nullptr || y == nullptr || cols == 0
        || cols % 8 != 0 || !(eps > 0.f)) {
        return KK_EINVAL;
    }
    if (rows == 0) {
        return 0;
    }
    return static_cast<int>(kk::launch(kk::rmsnorm_kernel, dim3(rows), dim3(kk::kNormThreads), 0,
        static_cast<cudaStream_t>(stream), 1, static_cast<__half const*>(nullptr),
        reinterpret_cast<__half const*>(embed), tokens, reinterpret_cast<__half const*>(weight),
        reinterpret_cast<__half*>(hidden), reinterpret_cast<__half*>(y), cols, eps,
        static_cast<float*>(nullptr)));
}

int kk_rope(uint16_t* q, uint32_t q_stride, uint16_t* k, uint32_t k_stride,
    const uint32_t* positions, uint32_t rows, uint32_t q_heads, uint32_t kv_heads,
    uint32_t head_dim, float theta, void* stream)
{
    if (q == nullptr || k == nullptr || positions == nullptr || head_dim == 0 || head_dim % 2 != 0
        || head_dim > 2048 || !(theta > 0.f) || q_heads + kv_heads > 65535u) {
        return KK_EINVAL;
    }
    if (rows == 0) {
        return 0;
    }
    unsigned const threads = ((head_dim / 2 + 31) / 32) * 32;
    return static_cast<int>(kk::launch(kk::rope_kernel, dim3(rows, q_heads + kv_heads),
        dim3(threads), 0, static_cast<cudaStream_t>(stream), 1, reinterpret_cast<__half*>(q),
        q_stride, reinterpret_cast<__half*>(k), k_stride, positions, q_heads, head_dim, theta));
}

int kk_silu_mul(const uint16_t* gate, const uint16_t* up, uint16_t* out, uint32_t rows,
    uint32_t cols, void* stream)
{
    if (gate == nullptr || up == nullptr || out == nullptr) {
        return KK_EINVAL;
    }
    std::uint64_t const count = std::uint64_t(rows) * cols;
    if (count == 0) {
        return 0;
    }
    return static_cast<int>(kk::launch(kk::silu_mul_kernel, dim3(kk::gridFor(count)), dim3(256), 0,
        static_cast<cudaStream_t>(stream), 1, reinterpret_cast<__half const*>(gate),
        reinterpret_cast<__half const*>(up), reinterpret_cast<__half*>(out), count));
}

int kk_residual_add(uint16_t* hidden, const uint16_t* update, uint64_t count, void* stream)
{
    if (hidden == nullptr || update == nullptr) {
        return KK_EINVAL;
    }
    if (count == 0) {
        return 0;
    }
    return static_cast<int>(kk::launch(kk::residual_add_kernel, dim3(kk::gridFor(count)),
        dim3(256), 0, static_cast<cudaStream_t>(stream), 1, reinterpret_cast<__half*>(hidden),
        reinterpret_cast<__half const*>(update), count));
}

} // extern "C"

namespace kk {
int embedSumSquares(std::uint16_t const* embed, std::uint32_t const* tokens, std::uint16_t* hidden,
    float* sq_out, std::uint32_t rows, std::uint32_t cols, cudaStream_t stream)
{
    if (embed == nullptr || tokens == nullptr || hidden == nullptr || sq_out == nullptr || cols == 0
        || cols % 8 != 0) {
        return KK_EINVAL;
    }
    if (rows == 0) {
        return 0;
    }
    return static_cast<int>(launch(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, stream, 1,
        static_cast<__half const*>(nullptr), reinterpret_cast<__half const*>(embed), tokens,
        static_cast<__half const*>(nullptr), reinterpret_cast<__half*>(hidden), static_cast<__half*>(nullptr),
        cols, 1.0f, sq_out));
}
} // namespace kk

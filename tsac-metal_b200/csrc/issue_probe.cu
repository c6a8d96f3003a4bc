// FP32 issue-rate probe: the denominator of the exact convolution's roofline.
//
// The exact-order analysis convolution issues, per multiply-accumulate, one
// separately rounded FP32 multiply and one FP32 add (the reference's unfused
// `sum += x * w`).  Its ceiling is therefore the rate at which the SMs issue
// FMUL and FADD, not a tensor or FMA peak.  This probe measures that rate on
// the device it runs on: every thread runs 16 independent two-term
// recurrences of exactly that instruction pair (a <- a + b * c, b <- b + a * d),
// enough independent work per warp to hide the arithmetic latency, over a grid
// of 8 CTAs of 256 threads per SM.  Timed with CUDA events on the caller's
// stream; the result is operations (multiplies + adds) per second.
#include "cuda_util.cuh"

namespace
{
constexpr int chains = 16;
constexpr int probe_threads = 256;

__global__ void __launch_bounds__(probe_threads) fp32_issue_kernel(float* out, int iterations)
{
    float a[chains], b[chains];
    const float seed = 1.0f + 1e-6f * static_cast<float>(threadIdx.x + blockIdx.x);
#pragma unroll
    for (int j = 0; j < chains; ++j)
    {
        a[j] = seed + 0.01f * static_cast<float>(j);
        b[j] = seed - 0.01f * static_cast<float>(j);
    }
    const float c = 1.0e-3f, d = -1.0e-3f;
#pragma unroll 1
    for (int i = 0; i < iterations; ++i)
    {
#pragma unroll
        for (int j = 0; j < chains; ++j)
        {
            a[j] = __fadd_rn(a[j], __fmul_rn(b[j], c));
            b[j] = __fadd_rn(b[j], __fmul_rn(a[j], d));
        }
    }
    float total = 0.0f;
#pragma unroll
    for (int j = 0; j < chains; ++j)
        total = __fadd_rn(total, __fadd_rn(a[j], b[j]));
    // The sum is always finite and positive; the store keeps the work live.
    if (total == 0.0f)
        out[blockIdx.x * blockDim.x + threadIdx.x] = total;
}
} // namespace

extern "C"
{
int tsac_cuda_fp32_issue_rate(int iterations, double* ops_per_second, double* milliseconds, void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(ops_per_second && iterations > 0 && iterations <= (1 << 24), "invalid probe arguments");
            int device = 0, sms = 0;
            cuda_check(cudaGetDevice(&device), "cudaGetDevice");
            cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "SM count");
            const auto s = static_cast<cudaStream_t>(stream);
            const dim3 grid(static_cast<unsigned>(sms) * 8);
            float* sink = nullptr;
            cudaEvent_t start = nullptr, stop = nullptr;
            cuda_check(cudaMalloc(&sink, sizeof(float) * grid.x * probe_threads), "probe sink");
            cuda_check(cudaEventCreate(&start), "event");
            cuda_check(cudaEventCreate(&stop), "event");
            fp32_issue_kernel<<<grid, probe_threads, 0, s>>>(sink, iterations); // warm
            cuda_check(cudaEventRecord(start, s), "event record");
            fp32_issue_kernel<<<grid, probe_threads, 0, s>>>(sink, iterations);
            cuda_check(cudaEventRecord(stop, s), "event record");
            const auto status = cudaEventSynchronize(stop);
            float ms = 0.0f;
            if (status == cudaSuccess)
                cudaEventElapsedTime(&ms, start, stop);
            cudaEventDestroy(start);
            cudaEventDestroy(stop);
            cudaFree(sink);
            cuda_check(status, "probe");
            require(ms > 0.0f, "probe timing failed");
            // Per iteration and chain: two multiplies and two adds.
            const double ops = 4.0 * chains * static_cast<double>(iterations) * grid.x * probe_threads;
            *ops_per_second = ops / (ms * 1e-3);
            if (milliseconds)
                *milliseconds = ms;
        });
}
}

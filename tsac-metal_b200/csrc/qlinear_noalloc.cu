// Quantized linear projection that allocates no device memory.
//
// tsac_cuda_qlinear needs a scratch buffer for the BF8L-quantized activations,
// which its caller allocates.  Some callers cannot: a host program that sizes
// and reserves all of its GPU memory once at start-up and then forbids further
// cudaMalloc (an embedded or real-time audio service that must not stall on the
// driver's allocator, or whose memory budget is owned by another framework), or
// a caller that has no allocator at hand where it makes the call.  This entry
// point serves them: its scratch is a fixed array in this library's own device
// image, so a call needs only the caller's inputs and outputs.
//
// The array lives in every GPU that loads the library until the process
// exits.  All calls share it and it keeps the last call's contents; a call
// writes every scratch byte it reads before reading it, so nothing has to be
// cleared first.  Calls whose execution overlaps on the GPU (concurrent
// streams, devices are separate) race on the array and must be serialised by
// the caller.
#include "cuda_util.cuh"
#include "kernels/qlinear.cuh"

#include <mutex>

namespace
{
// Quantized activations: int8 [m][k] in the first 1 MiB, f32 scales
// [m][k/256] in the following 16 KiB, so m * k may be at most 1 MiB
// (for example 256 columns of 4096 inputs).
constexpr size_t activation_bytes = size_t{1} << 20;
constexpr size_t scale_bytes = size_t{16} << 10;
constexpr size_t max_columns_times_inputs = activation_bytes;

static __device__ __align__(256) unsigned char noalloc_scratch[activation_bytes + scale_bytes];

constexpr int max_devices = 64;
std::mutex setup_mutex;
void* scratch_address[max_devices] = {};

// Device address of the array on the current device.  The host-side symbol is
// only a stand-in, so the first call on each device looks the address up with
// that device current and keeps it.  The kept address belongs to the device's
// primary context: a cudaDeviceReset destroys it, so this entry point must not
// be used on a device after cudaDeviceReset in the same process.
void* device_scratch()
{
    int device = 0;
    tsacb::cuda_check(cudaGetDevice(&device), "cudaGetDevice");
    tsacb::require(device >= 0 && device < max_devices, "CUDA device ordinal out of range");
    std::lock_guard lock(setup_mutex);
    if (!scratch_address[device])
    {
        void* ptr = nullptr;
        tsacb::cuda_check(cudaGetSymbolAddress(&ptr, noalloc_scratch),
                          "cudaGetSymbolAddress(no-allocation qlinear scratch)");
        scratch_address[device] = ptr;
    }
    // Kernel attributes are per device; qlinear_init keeps one bit per device
    // and returns at once when this device is already set up.
    tsacb::dev::qlinear_init();
    return scratch_address[device];
}
} // namespace

extern "C"
{
size_t tsac_cuda_qlinear_noalloc_max_elements(void)
{
    return max_columns_times_inputs;
}

int tsac_cuda_qlinear_noalloc(const int8_t* weights, const float* weight_scales,
                              const float* bias, size_t k, size_t n, const uint16_t* x, size_t m,
                              const uint16_t* residual, uint16_t* y, unsigned* error_word,
                              void* stream)
{
    return tsacb::guarded(
        [&]
        {
            using namespace tsacb;
            require_device();
            require(weights && weight_scales && bias && x && y, "null argument");
            require(k >= 256 && k % 256 == 0 && k <= 8192,
                    "qlinear input width must be 256..8192, a multiple of 256");
            require(n >= 64 && n % 64 == 0, "qlinear output width must be a positive multiple of 64");
            require(m > 0, "qlinear column count out of range");
            require(m <= max_columns_times_inputs / k,
                    "no-allocation qlinear: columns x inputs exceeds its fixed 1 MiB scratch "
                    "(use tsac_cuda_qlinear with a caller-allocated scratch buffer)");
            require(aligned16(weights) && aligned16(x) && aligned16(y),
                    "qlinear buffers must be 16-byte aligned");
            auto* base = static_cast<unsigned char*>(device_scratch());
            auto* xq = reinterpret_cast<std::int8_t*>(base);
            auto* xs = reinterpret_cast<float*>(base + activation_bytes);
            const auto s = static_cast<cudaStream_t>(stream);
            dev::qlinear_quantize(x, static_cast<int>(m), static_cast<int>(k), xq, xs, error_word, s);
            dev::QLinearArgs a;
            a.weights = weights;
            a.weight_scales = weight_scales;
            a.bias = bias;
            a.xq = xq;
            a.xscale = xs;
            a.residual = residual;
            a.y = y;
            a.m = static_cast<int>(m);
            a.n = static_cast<int>(n);
            a.k = static_cast<int>(k);
            a.error_word = error_word;
            dev::qlinear_matmul(a, s);
            cuda_check(cudaGetLastError(), "qlinear launch");
        });
}
}

// C ABI: error reporting and the host-only package tooling entry points.
#include "abi_util.hpp"
#include "models.hpp"

#include <cstdlib>

namespace tsacb
{
thread_local std::string last_error_message;
}

extern "C"
{
const char* tsac_cuda_last_error(void)
{
    return tsacb::last_error_message.c_str();
}

void tsac_cuda_free(void* pointer)
{
    std::free(pointer);
}

int tsac_cuda_write_seeded_sources(const char* directory, uint64_t seed)
{
    return tsacb::guarded([&] { tsacb::write_seeded_sources(directory, seed); });
}

int tsac_cuda_pack_models(const char* input_directory, const char* output_directory,
                          const char* pack_id, int include_transformer)
{
    return tsacb::guarded(
        [&]
        {
            tsacb::require(input_directory && output_directory && pack_id, "null argument");
            tsacb::pack_models(input_directory, output_directory, pack_id,
                               include_transformer != 0);
        });
}
}

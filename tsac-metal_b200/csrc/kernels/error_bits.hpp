// Bits of the device error word that kernels OR in and the host checks after
// completion (the reference's Metal kernels use the same pattern,
// src/metal/dac/snake.metal:49-52).  Shared by device and host code.
#pragma once

namespace tsacb::dev
{
enum ErrorBits : unsigned
{
    error_nonfinite = 1u,
    error_range = 2u,
    error_timeout = 4u, // a bounded pipeline wait gave up; the kernel returned early
};
} // namespace tsacb::dev

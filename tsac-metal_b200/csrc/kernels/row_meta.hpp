// Per-row metadata of the Transformer kernels (decode steps and prefills).
#pragma once

namespace tsacb::dev
{
struct RowMeta
{
    int slot;      // cache slot receiving this row's key/value
    int base;      // cache slot of position 0 of the row's sequence
    int time;      // number of keys visible to the row (position + 1)
    int rotary;    // rotary coefficient row (position), -1 = no rotary
    int round;     // 1: bf16-round block value sums (time > 64 or replay prefill)
};
} // namespace tsacb::dev

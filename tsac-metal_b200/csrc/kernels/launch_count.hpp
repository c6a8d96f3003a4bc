// Process-wide count of the kernels this library launches, for the benchmark's
// launch tally.  Every launch site calls note_launch() after its <<<...>>>.
// While a thread captures a CUDA graph its launch sites add to that thread's
// capture tally instead; the graph's owner then adds the tally each time it
// launches the graph, so replays count their kernel nodes.
#pragma once

namespace tsacb::dev
{
void note_launch(unsigned long long kernels = 1);
unsigned long long launch_count();

// Counts the launch sites that run while it lives (on this thread) as graph
// nodes instead of launches; kernels() is that tally.
class CaptureTally
{
public:
    CaptureTally();
    ~CaptureTally();
    unsigned long long kernels() const;

private:
    CaptureTally* outer_;
    unsigned long long kernels_ = 0;
    friend void note_launch(unsigned long long);
};
} // namespace tsacb::dev

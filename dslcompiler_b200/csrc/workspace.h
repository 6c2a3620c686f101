// workspace.h -- layout of a device workspace: the library's per-device
// buffer, or the scratch a caller passes in KernelContext.  Fixed offsets,
// the same for every shape and kernel, so one workspace serves every call:
// the counter regions are zero at rest (every launch leaves the counters it
// used at zero), the partial-sum region is always written before it is read.
#pragma once

#include <cstddef>

namespace llk_b200 {

// CTA-pair kernel: dynamic-schedule work counter at 0, K-split tail arrival
// counters from 256.
constexpr size_t kWsTc2Counters = 0;
constexpr size_t kWsTc2TailCounters = 256;
constexpr size_t kWsTc2CounterBytes = 8192;
// Decode kernel: per-tile arrival counters (65536 tiles of 128 columns).
constexpr size_t kWsDecodeCounters = kWsTc2CounterBytes;
constexpr size_t kWsDecodeCounterBytes = 256 * 1024;
// Partial sums: decode split-K slots, or the CTA-pair kernel's K-split tail.
constexpr size_t kWsPartials = kWsDecodeCounters + kWsDecodeCounterBytes;

}  // namespace llk_b200

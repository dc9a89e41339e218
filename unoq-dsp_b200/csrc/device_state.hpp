// device_state.hpp -- per-device, thread-safe one-time set-up of the kernels (host only).
//
// cudaFuncSetAttribute (the dynamic shared-memory limit of the 200+ KB tensor-core kernels) acts
// on the device that is current when it is called, so a flag per process would leave a second
// device without it: a process may load a graph on one device and a session on another
// (ug_set_device). The set-up below is keyed by (device, kernel family) and guarded by a lock.
#pragma once
#include <functional>

namespace uq {

// Runs `set` once per (current device, family) until it succeeds; returns its result (true when
// it succeeded now or before).
bool once_per_device(int family, const std::function<bool()> &set);
// Streaming multiprocessors of the current device (148 on B200 when the query fails).
int current_sm_count();

enum KernelFamily { kFamilyConvTc = 1, kFamilyConvRows = 2, kFamilyConvTaps = 3, kFamilyDecode = 4, kFamilyDwTc = 5 };

}  // namespace uq

// brotensor/runtime.h — process set-up of the reference's entry points
// (brotensor::init(), called first by the reference's tests). In this build it
// selects device 0 and creates its context, so the first entry point does not
// pay for it; it throws std::runtime_error when no CUDA device is usable.
#pragma once

namespace brotensor {

void init();
// waits for all work this process queued on the device
void synchronize();

}  // namespace brotensor

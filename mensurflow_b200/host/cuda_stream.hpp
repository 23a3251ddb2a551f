// The CUDA stream behind a Stream of this repository's CUDA backend (cuda_backend.cpp), for host
// code next to the backend that calls the C ABI of include/mfk.h itself (a pre-split weight
// owner, a multi-GPU split): the reference's Stream interface (src/backends/backend.hpp:32-44)
// hides the vendor handle.
#pragma once

#include "backends/backend.hpp"

namespace mensurflow::detail {

// The cudaStream_t of `stream`, which must come from the CUDA backend
// (Registry::instance().get({DeviceType::CUDA, i}).stream(i)); its device is made current.
void* cuda_stream_handle(Stream& stream);

} // namespace mensurflow::detail

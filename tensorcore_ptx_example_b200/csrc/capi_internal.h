// capi_internal.h -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "nvfp4.h"

namespace nvfp4 {

// Records a printf-style message as the calling thread's last error; returns `code`.
nvfp4_status_t fail(nvfp4_status_t code, const char* fmt, ...);
// Clears the calling thread's last error.
void clear_error();
// The calling thread's last error message ("" if none).
const char* last_error();
// Maps the last CUDA launch error (if any) to NVFP4_ERR_CUDA with a message.
nvfp4_status_t check_launch(const char* what);
// Number of SMs of the current device (cached per device).
int sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace nvfp4

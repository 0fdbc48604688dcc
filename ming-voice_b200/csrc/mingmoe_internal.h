// Internal constants and host-side helpers shared by the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/mingmoe.h"

namespace mv {

// Device-side error codes written to the workspace header (WsHeader::error).
constexpr unsigned int kErrTimeout = 1;     // an mbarrier wait gave up (bounded spin)
constexpr unsigned int kErrBadExpert = 2;   // an expert id outside [0, E1) was skipped
constexpr unsigned int kErrOverflow = 3;    // a token capacity was exceeded (skipped)

// Wall-clock limit of one bounded wait on the device.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

constexpr size_t kWsHeaderBytes = 256;

// Thread-local last-error message for mv_last_error().
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int elem_size(int dtype) {
  switch (dtype) {
    case MV_BF16:
    case MV_F16:
      return 2;
    case MV_F32:
    case MV_I32:
      return 4;
    case MV_I8:
      return 1;
    case MV_I64:
      return 8;
    default:
      return 0;
  }
}

int num_sms();

}  // namespace mv

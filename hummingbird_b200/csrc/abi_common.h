// Shared host-side checks for the C-ABI entry points.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "hb_status.h"

namespace hb {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The kernels are built for sm_100a only: refuse any other device (cached per device ordinal).
inline int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  static signed char ok[64] = {};
  if (dev >= 0 && dev < 64 && ok[dev]) return ok[dev] > 0 ? HB_OK : HB_ERR_ARCH;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return HB_ERR_LAUNCH;
  const bool good = (major == 10 && minor == 0);
  if (dev >= 0 && dev < 64) ok[dev] = good ? 1 : -1;
  return good ? HB_OK : HB_ERR_ARCH;
}

}  // namespace hb

// Status codes returned by every hummingbird-b200 C-ABI entry point (0 = success).
#pragma once

enum HbStatus {
  HB_OK = 0,
  HB_ERR_SHAPE = 1,        // unsupported or inconsistent shape / argument (the reference raises ValueError)
  HB_ERR_ALIGN = 2,        // a pointer or stride is not aligned as the kernel requires
  HB_ERR_ARCH = 3,         // the current device is not sm_100
  HB_ERR_LAUNCH = 4,       // a CUDA launch / runtime call failed
  HB_ERR_DEVICE = 5,       // a kernel recorded an error in the device status word
  HB_ERR_TIMEOUT = 6,      // a bounded device-side wait expired
  HB_ERR_WORKSPACE = 7,    // workspace missing or too small
  HB_ERR_NCCL = 8,         // a collective failed
  HB_ERR_NULL = 9,         // a required pointer is null
};

// SAME-L attention front-end GEMM (band_proj.cu): its translation unit's status word.
#pragma once

namespace hb {

// Read (and clear, when set) the status word of band_proj.cu's translation unit on the current device; an
// HbStatus.
int band_proj_take_status(unsigned int* status);

}  // namespace hb

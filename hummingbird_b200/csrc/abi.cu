// Library-wide C-ABI entry points: version and the device status word.
#include <cuda_runtime.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "band_fused.h"
#include "band_proj.h"
#include "hb_sm100.cuh"

extern "C" int hb_version(void) { return 100; }

extern "C" int hb_device_status(unsigned int* status_out, cudaStream_t stream) {
  if (!status_out) return HB_ERR_NULL;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return HB_ERR_LAUNCH;
  unsigned int v = 0, vb = 0, vp = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, hb::g_device_status, sizeof(v)) != cudaSuccess) return HB_ERR_LAUNCH;
  if (v && cudaMemcpyToSymbol(hb::g_device_status, &zero, sizeof(zero)) != cudaSuccess) return HB_ERR_LAUNCH;
  // the fused band kernel's and the band front end's units keep their own words (they are compiled as
  // whole-program device code)
  if (hb::band_fused_take_status(&vb) != HB_OK || hb::band_proj_take_status(&vp) != HB_OK) return HB_ERR_LAUNCH;
  *status_out = v ? v : (vb ? vb : vp);
  return HB_OK;
}

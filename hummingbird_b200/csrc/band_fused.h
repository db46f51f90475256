// Fused persistent band attention (window <= 128): parameters and launchers (band_fused.cu).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace hb {

struct BandFusedParams {
  const uint16_t* qkv;      // bf16 [B, rows, row_stride]
  int64_t row_stride;       // elements
  int B, rows, H_total, head0, heads;
  int q_begin, q_count, window, half;
  const float* q_norm;      // [129] alpha, gamma[64], beta[64]
  const float* k_norm;
  const float* inv_freq;    // [half]
  int64_t pos0;             // global position of buffer row 0
  const float* lam;
  int lam_pair0;
  uint16_t* out;
  int64_t out_row_stride;
  int qt_first, nqt, ntiles, units;
  int prepared;             // qkv already DyT'd and rotated (hb_band_qkv_project): no preparation stage
};

constexpr int kFusedMaxWindow = 128;

int band_fused_attend(const BandFusedParams& p, cudaStream_t stream);

// Read (and clear, when set) the status word of the fused band kernel's translation unit on the current
// device; an HbStatus.
int band_fused_take_status(unsigned int* status);

}  // namespace hb

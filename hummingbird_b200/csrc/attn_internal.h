// Internal interface between the dense / band front ends and the shared tcgen05 attention kernel.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace hb {

constexpr int kTileRows = 128;                      // query / key rows per tile
constexpr int kHeadDim = 64;                        // head_dim (the reference requires 64)
constexpr int kTileBytes = kTileRows * kHeadDim * 2;  // one bf16 128 x 64 tile in the SW128 image (16 KiB)
constexpr int kSections = 5;                        // q, k, v, q_diff, k_diff (the reference's qkv order)

// Prepared-operand workspace: for each (batch, local head, section, row tile) one 16 KiB tile holding
// 128 rows x 64 dims of bf16 in the 128-byte-swizzled UMMA image, rows past the end zero-filled.
__host__ __device__ inline size_t prep_tile_offset(int b, int h, int s, int t, int heads, int ntiles) {
  return ((((size_t)b * heads + h) * kSections + s) * (size_t)ntiles + t) * (size_t)kTileBytes;
}
inline size_t prep_workspace_bytes(int B, int rows, int heads) {
  const int ntiles = (rows + kTileRows - 1) / kTileRows;
  return (size_t)B * heads * kSections * ntiles * kTileBytes;
}

struct AttnParams {
  const uint8_t* ws;       // prepared tiles (prep_tile_offset layout)
  int B;
  int rows;                // rows held in the workspace (sequence length incl. any halo rows)
  int ntiles;              // ceil(rows / 128)
  int heads;               // local heads in the workspace
  int q_begin, q_count;    // query rows [q_begin, q_begin + q_count) are computed and stored
  int window;              // < 0: dense (every key); else band |k - q| <= window
  const float* lam;        // per pair lambda (index (lam_pair0 + h / 2)), or null for 1
  int lam_pair0;
  uint16_t* out;           // bf16; row i of query range -> out + (b * q_count + i) * out_row_stride + h * 64
  int64_t out_row_stride;  // elements
};

// Launch the shared differential-attention kernel on `stream`. Returns a cudaError_t as int.
int launch_diff_attention(const AttnParams& p, cudaStream_t stream);

// Dense mode only (window < 0, q_begin = 0): scores and probabilities in separate TMEM buffers (attn_dense.cu).
int launch_dense_attention(const AttnParams& p, cudaStream_t stream);

}  // namespace hb

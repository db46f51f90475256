// Dense differential self-attention (the DiT's `dense_attention`), C-ABI front end + its prologue.
//
// Prologue (`dense_prep_kernel`, HBM-bound): reads the `to_qkv` output once with 128-bit loads (a warp takes
// one row for four heads, all five sections' loads in flight together, the row's lane-table chunks loaded once)
// and writes per-(batch, head, section) 128-row tiles in the SW128 UMMA image:
//   q, k, q_diff, k_diff: RMSNorm in fp32 over the head's 64 dims -> bf16 -> RoPE in fp32 with the
//                         caller's cos / signed-sin lane tables -> bf16   (dense_attention.py:61-69)
//   v:                    bf16(v * mask)                                   (dense_attention.py:77)
// The 1/sqrt(64) score scale is applied in the softmax (exact: a power of two).
// Main kernel: attn_dense.cu (every key, no key mask, dense_attention.py:79-83).
#include <atomic>

#include <cuda_runtime.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "attn_internal.h"
#include "prep_common.cuh"

namespace hb {
namespace {

constexpr int kPrepThreads = 256;
constexpr int kHeadsPerWarp = 4;  // a warp: one row, four heads (an 8-lane group per head, 16 bytes per lane)

// n / d for 0 <= n < 2^31 by a multiply-high and a shift (the round-up reciprocal method: multiplier
// ceil(2^p / d) with p = 31 + ceil(log2 d)); replaces the integer divisions of the unit decode.
struct FastDiv {
  uint32_t d, mul, shift;
  void init(uint32_t div) {
    d = div;
    if (div == 1) {
      mul = 0;
      shift = 0;
      return;
    }
    uint32_t l = 0;
    while ((1ull << l) < div) ++l;
    const uint32_t pw = 31 + l;
    mul = static_cast<uint32_t>(((1ull << pw) + div - 1) / div);
    shift = pw - 32;
  }
  __device__ __forceinline__ uint32_t operator()(uint32_t n) const { return d == 1 ? n : (__umulhi(n, mul) >> shift); }
};

struct DensePrepParams {
  const uint16_t* qkv;
  int64_t qkv_row_stride;
  int B, L, H_total, head0, heads;
  const float* q_w;
  const float* k_w;
  const float* cos;
  const float* sin;
  int64_t table_stride;
  const uint16_t* vmask;
  int64_t mask_bstride, mask_lstride;
  float eps;
  int half;
  uint8_t* ws;
  int ntiles;
  int hgroups;  // ceil(heads / kHeadsPerWarp)
  int tasks;    // B * ntiles * 128 * hgroups (< 2^31, checked on the host)
  FastDiv by_hgroups, by_rows;
};

// 8 consecutive fp32 values; 16-byte vector loads when kVec (the caller checked the alignment)
template <bool kVec>
__device__ __forceinline__ void load8f(const float* src, float (&v)[8]) {
  if constexpr (kVec) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 c = __ldg(reinterpret_cast<const float4*>(src) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __ldg(src + i);
  }
}

// Task t = (b * rows_pad + row) * hgroups + hg, one warp each: lane = 8 * hsub + c takes the 16-byte chunk c of
// head 4 hg + hsub in all five sections of the row. The row's cos / sin chunks and the weight chunks are loaded
// once per task; the five data loads are issued before any computing. Padding rows (row >= L) are written as
// zeros, as the attention kernel expects.
template <bool kVec>
__global__ void __launch_bounds__(kPrepThreads, 3) dense_prep_kernel(const DensePrepParams p) {
  const int lane = threadIdx.x & 31;
  const int c = lane & 7, hsub = lane >> 3;
  const unsigned gmask = 0xFFu << (lane & 24);
  const int hc8 = p.half >> 3;
  const int task = blockIdx.x * (kPrepThreads / 32) + (threadIdx.x >> 5);
  if (task >= p.tasks) return;  // warp-uniform
  const uint32_t br = p.by_hgroups(static_cast<uint32_t>(task));
  const int hl = static_cast<int>(task - br * static_cast<uint32_t>(p.hgroups)) * kHeadsPerWarp + hsub;
  if (hl >= p.heads) return;  // the whole 8-lane group (its shuffles involve only its own lanes)
  const uint32_t bb = p.by_rows(br);
  const int row = static_cast<int>(br - bb * static_cast<uint32_t>(p.ntiles * kTileRows));
  const int b = static_cast<int>(bb);
  const bool valid = row < p.L;
  uint4 raw[kSections];
  if (valid) {
    const uint16_t* src = p.qkv + ((size_t)b * p.L + row) * p.qkv_row_stride + (size_t)(p.head0 + hl) * kHeadDim + c * 8;
#pragma unroll
    for (int s = 0; s < kSections; ++s) raw[s] = ld_nc_v4(src + (size_t)s * p.H_total * kHeadDim);
  } else {
#pragma unroll
    for (int s = 0; s < kSections; ++s) raw[s] = make_uint4(0, 0, 0, 0);
  }
  float cr[8], sr[8], qwv[8], kwv[8];
  if (valid) {
    load8f<kVec>(p.cos + (size_t)row * p.table_stride + c * 8, cr);
    load8f<kVec>(p.sin + (size_t)row * p.table_stride + c * 8, sr);
  }
  load8f<kVec>(p.q_w + c * 8, qwv);
  load8f<kVec>(p.k_w + c * 8, kwv);
  const float m = valid ? __uint_as_float((uint32_t)p.vmask[b * p.mask_bstride + row * p.mask_lstride] << 16) : 0.f;
  const int src_lane = (lane & 24) | rope_partner_chunk(c, hc8);
  uint8_t* dst = p.ws + prep_tile_offset(b, hl, 0, row / kTileRows, p.heads, p.ntiles) + sw128_offset(row % kTileRows, c);
  const size_t sec_bytes = (size_t)p.ntiles * kTileBytes;
#pragma unroll
  for (int s = 0; s < kSections; ++s) {
    float xv[8];
    unpack8(raw[s], xv);
    uint4 outv;
    if (s == 2) {  // v * mask
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] *= m;
      outv = pack8(xv);
    } else {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(xv[i], xv[i], ss);
      ss += __shfl_xor_sync(gmask, ss, 1);
      ss += __shfl_xor_sync(gmask, ss, 2);
      ss += __shfl_xor_sync(gmask, ss, 4);
      const float inv = rsqrtf(ss * (1.f / kHeadDim) + p.eps);
      const float* wv = (s == 0 || s == 3) ? qwv : kwv;
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {  // (x * inv) * w, each product rounded (packed pairs)
        fmul2(y[i], y[i + 1], xv[i], xv[i + 1], inv, inv);
        fmul2(y[i], y[i + 1], y[i], y[i + 1], wv[i], wv[i + 1]);
      }
      const uint4 yb = pack8(y);  // RMSNorm output rounded to bf16 (dense_attention.py:66)
      uint4 pb;
      pb.x = __shfl_sync(gmask, yb.x, src_lane);
      pb.y = __shfl_sync(gmask, yb.y, src_lane);
      pb.z = __shfl_sync(gmask, yb.z, src_lane);
      pb.w = __shfl_sync(gmask, yb.w, src_lane);
      float yv[8], pv[8];
      unpack8(yb, yv);
      unpack8(pb, pv);
      if (valid) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {  // y cos + partner * signed sin
          float t0, t1;
          fmul2(t0, t1, pv[i], pv[i + 1], sr[i], sr[i + 1]);
          ffma2(y[i], y[i + 1], yv[i], yv[i + 1], cr[i], cr[i + 1], t0, t1);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] = 0.f;
      }
      outv = pack8(y);
    }
    *reinterpret_cast<uint4*>(dst + s * sec_bytes) = outv;
  }
}

}  // namespace
}  // namespace hb

using namespace hb;

extern "C" int hb_dense_workspace_bytes(int batch, int length, int pair_count, size_t* bytes) {
  if (!bytes) return HB_ERR_NULL;
  if (batch < 1 || length < 1 || pair_count < 1) return HB_ERR_SHAPE;
  *bytes = prep_workspace_bytes(batch, length, 2 * pair_count);
  return HB_OK;
}

namespace {

// The host-side argument checks shared by both dense entry points (no device work, no workspace check).
int dense_check_args(const void* qkv, int64_t qkv_row_stride, const float* q_weight, const float* k_weight,
                     const float* cos, const float* sin, int64_t table_stride, const void* vmask, void* out,
                     int64_t out_row_stride, int batch, int length, int num_heads, int head_dim, int half,
                     int pair_begin, int pair_count) {
  if (!qkv || !q_weight || !k_weight || !cos || !sin || !vmask || !out) return HB_ERR_NULL;
  if (head_dim != kHeadDim || num_heads < 2 || num_heads % 2 || batch < 1 || length < 1) return HB_ERR_SHAPE;
  if (half < 8 || half > 32 || half % 8) return HB_ERR_SHAPE;
  if (pair_begin < 0 || pair_count < 1 || pair_begin + pair_count > num_heads / 2) return HB_ERR_SHAPE;
  if (qkv_row_stride < (int64_t)5 * num_heads * kHeadDim || table_stride < kHeadDim ||
      out_row_stride < (int64_t)2 * pair_count * kHeadDim)
    return HB_ERR_SHAPE;
  if (!aligned16(qkv) || qkv_row_stride % 8 || !aligned16(out) || out_row_stride % 8) return HB_ERR_ALIGN;
  return HB_OK;
}

}  // namespace

extern "C" int hb_dense_diff_attn(const void* qkv, int64_t qkv_row_stride, const float* q_weight,
                                  const float* k_weight, const float* cos, const float* sin, int64_t table_stride,
                                  const void* vmask, int64_t mask_batch_stride, int64_t mask_row_stride,
                                  const float* lam, void* out, int64_t out_row_stride, int batch, int length,
                                  int num_heads, int head_dim, int half, float eps, int pair_begin, int pair_count,
                                  void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const int chk = dense_check_args(qkv, qkv_row_stride, q_weight, k_weight, cos, sin, table_stride, vmask, out,
                                   out_row_stride, batch, length, num_heads, head_dim, half, pair_begin, pair_count);
  if (chk != HB_OK) return chk;
  if (!aligned16(workspace)) return HB_ERR_ALIGN;
  const int heads = 2 * pair_count;
  if (!workspace || workspace_bytes < prep_workspace_bytes(batch, length, heads)) return HB_ERR_WORKSPACE;
  int st = check_device();
  if (st != HB_OK) return st;

  const int ntiles = (length + kTileRows - 1) / kTileRows;
  const int hgroups = (heads + kHeadsPerWarp - 1) / kHeadsPerWarp;
  const int64_t tasks = (int64_t)batch * ntiles * kTileRows * hgroups;
  if (tasks >= (int64_t(1) << 31)) return HB_ERR_SHAPE;
  DensePrepParams pp{static_cast<const uint16_t*>(qkv), qkv_row_stride, batch, length, num_heads, 2 * pair_begin,
                     heads, q_weight, k_weight, cos, sin, table_stride, static_cast<const uint16_t*>(vmask),
                     mask_batch_stride, mask_row_stride, eps, half, static_cast<uint8_t*>(workspace), ntiles, hgroups,
                     (int)tasks, {}, {}};
  pp.by_hgroups.init(static_cast<uint32_t>(hgroups));
  pp.by_rows.init(static_cast<uint32_t>(ntiles * kTileRows));
  const int pblocks = (int)((tasks + kPrepThreads / 32 - 1) / (kPrepThreads / 32));
  // 16-byte loads of the weights and lane tables when their rows are 16-byte aligned
  const bool vec = aligned16(q_weight) && aligned16(k_weight) && aligned16(cos) && aligned16(sin) && table_stride % 4 == 0;
  if (vec)
    dense_prep_kernel<true><<<pblocks, kPrepThreads, 0, stream>>>(pp);
  else
    dense_prep_kernel<false><<<pblocks, kPrepThreads, 0, stream>>>(pp);
  if (cudaGetLastError() != cudaSuccess) return HB_ERR_LAUNCH;

  AttnParams ap{};
  ap.ws = static_cast<const uint8_t*>(workspace);
  ap.B = batch;
  ap.rows = length;
  ap.ntiles = ntiles;
  ap.heads = heads;
  ap.q_begin = 0;
  ap.q_count = length;
  ap.window = -1;
  ap.lam = lam;
  ap.lam_pair0 = pair_begin;
  ap.out = static_cast<uint16_t*>(out);
  ap.out_row_stride = out_row_stride;
  return launch_dense_attention(ap, stream) == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

// ------------------------------------------------------------------------------------------------------
// Allocation-free variant of hb_dense_diff_attn.
//
// Some callers cannot hand this library a workspace: an XLA FFI handler runs inside a runtime that has
// already reserved most of the GPU's memory for its own allocator (JAX pre-allocates about three quarters
// of it), so a cudaMalloc from the handler can fail, and cudaMalloc / cudaFree also synchronise the device
// in the middle of the caller's stream work. For them the prepared-tile scratch lives in one fixed array
// compiled into this library. Its size is a hard limit on the shapes this entry point accepts.
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;  // 64 MiB per device that loads the library, held until exit

// Device-side scratch shared by every call of hb_dense_diff_attn_noalloc on a device. Host code must not
// pass this symbol to a kernel: on the host it only names a stand-in, not the device address.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up once per device.
int noalloc_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HB_ERR_LAUNCH;
  static std::atomic<void*> cache[64];
  void* ptr = cache[dev].load(std::memory_order_acquire);
  if (!ptr) {
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) {
      cudaGetLastError();  // clear the failed lookup, so the next call does not report it as its own launch error
      return HB_ERR_LAUNCH;
    }
    cache[dev].store(ptr, std::memory_order_release);
  }
  *out = ptr;
  return HB_OK;
}

}  // namespace

extern "C" int hb_dense_noalloc_max_bytes(size_t* bytes) {
  if (!bytes) return HB_ERR_NULL;
  *bytes = kNoAllocScratchBytes;
  return HB_OK;
}

extern "C" int hb_dense_diff_attn_noalloc(const void* qkv, int64_t qkv_row_stride, const float* q_weight,
                                          const float* k_weight, const float* cos, const float* sin,
                                          int64_t table_stride, const void* vmask, int64_t mask_batch_stride,
                                          int64_t mask_row_stride, const float* lam, void* out,
                                          int64_t out_row_stride, int batch, int length, int num_heads,
                                          int head_dim, int half, float eps, int pair_begin, int pair_count,
                                          cudaStream_t stream) {
  if (batch < 1 || length < 1 || pair_count < 1) return HB_ERR_SHAPE;
  // refuse, before any device work, a problem whose prepared tiles would not fit the fixed scratch
  if (prep_workspace_bytes(batch, length, 2 * pair_count) > kNoAllocScratchBytes) return HB_ERR_WORKSPACE;
  // then the same host-side checks as the workspace entry point and the device check, so a bad argument or a
  // non-sm_100 device is reported as such before the scratch lookup touches the device
  int st = dense_check_args(qkv, qkv_row_stride, q_weight, k_weight, cos, sin, table_stride, vmask, out,
                            out_row_stride, batch, length, num_heads, head_dim, half, pair_begin, pair_count);
  if (st != HB_OK) return st;
  if ((st = check_device()) != HB_OK) return st;
  void* scratch = nullptr;
  if ((st = noalloc_scratch_address(&scratch)) != HB_OK) return st;
  return hb_dense_diff_attn(qkv, qkv_row_stride, q_weight, k_weight, cos, sin, table_stride, vmask, mask_batch_stride,
                            mask_row_stride, lam, out, out_row_stride, batch, length, num_heads, head_dim, half, eps,
                            pair_begin, pair_count, scratch, kNoAllocScratchBytes, stream);
}

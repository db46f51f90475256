// Elementwise glue of a DiT block (`dit._block`, dit.py:224-250; `_feed_forward`, dit.py:218-221; the
// cross-attention q norm, dit.py:150-176) as three HBM-bound row kernels, so each activation row is read and
// written once per step instead of once per torch op:
//
// hb_dit_residual_norm   h <- h + y * sigmoid(1 - gate[b])  (the gated residuals, dit.py:237, 250)
//                        h <- h + local on rows t >= local_row0  (`to_local_embed`, dit.py:244)
//                        x <- RMSNorm(h) * w, then x * (1 + scale[b]) + shift[b]  (dit.py:234-235, 247-248)
// hb_glu_rows            z = value * silu(gate) of a GLU projection row (value = first F columns), written as
//                        bf16 or quantised per row with the quantiser's rules for the W8A8 GEMM that follows
// hb_head_rms_norm       RMSNorm over every 64-dim head of each row (`_attend`'s q norm, dit.py:150-176)
//
// Rounding follows the torch ops they replace: every step computes in fp32 and rounds to bf16 where the
// unfused sequence stores a bf16 tensor (h after each residual, 1 + scale, 1 - gate and its sigmoid, silu).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "hb_sm100.cuh"
#include "prep_common.cuh"

namespace hb {
namespace {

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint4 ld_v4(const uint16_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// ------------------------------------------------------------------ residual + RMSNorm + modulation
struct ResNormParams {
  uint16_t* h;
  int64_t ldh;
  const uint16_t* y;
  int64_t ldy;
  const uint16_t* gate;   // [B, d] rows of stride ldc; y is multiplied by sigmoid(1 - gate)
  const uint16_t* scale;  // [B, d]; x is multiplied by (1 + scale)
  const uint16_t* shift;  // [B, d]
  int64_t ldc;
  const uint16_t* local;  // [d]
  int local_row0;
  const uint16_t* w;  // RMSNorm weight [d]
  uint16_t* x;
  int64_t ldx;
  int rows, rows_per_batch, d;
  float eps;
};

constexpr int kRowWarps = 8;

// One warp per row; lane l holds the 16-byte chunks l, l + 32, ... (NC chunks, d = 256 NC).
template <int NC>
__global__ void __launch_bounds__(32 * kRowWarps) residual_norm_kernel(const ResNormParams p) {
  const int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= p.rows) return;
  const int b = r / p.rows_per_batch, t = r - b * p.rows_per_batch;
  uint16_t* hr = p.h + (size_t)r * p.ldh;
  uint4 hv4[NC], yv4[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) hv4[i] = ld_v4(hr + (i * 32 + lane) * 8);
  if (p.y) {
    const uint16_t* yr = p.y + (size_t)r * p.ldy;
#pragma unroll
    for (int i = 0; i < NC; ++i) yv4[i] = ld_v4(yr + (i * 32 + lane) * 8);
  }
  const bool add_local = p.local && t >= p.local_row0;
  float v[NC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = (i * 32 + lane) * 8;
    unpack8(hv4[i], v[i]);
    if (p.y) {
      float yv[8];
      unpack8(yv4[i], yv);
      if (p.gate) {
        float g[8];
        unpack8(ld_v4(p.gate + (size_t)b * p.ldc + c), g);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = round_bf16(1.f - g[e]);
          const float gm = round_bf16(1.f / (1.f + __expf(-a)));
          v[i][e] = round_bf16(v[i][e] + yv[e] * gm);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = round_bf16(v[i][e] + yv[e]);
      }
    }
    if (add_local) {
      float lv[8];
      unpack8(ld_v4(p.local + c), lv);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = round_bf16(v[i][e] + lv[e]);
    }
    if (p.y || add_local) *reinterpret_cast<uint4*>(hr + c) = pack8(v[i]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
  }
  if (!p.x) return;
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(p.d) + p.eps);
  uint16_t* xr = p.x + (size_t)r * p.ldx;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = (i * 32 + lane) * 8;
    float w[8], o[8];
    unpack8(ld_v4(p.w + c), w);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = round_bf16(__fmul_rn(v[i][e], inv) * w[e]);
    if (p.scale) {
      float sc[8], sh[8];
      unpack8(ld_v4(p.scale + (size_t)b * p.ldc + c), sc);
      unpack8(ld_v4(p.shift + (size_t)b * p.ldc + c), sh);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = sh[e] + o[e] * round_bf16(1.f + sc[e]);
    }
    *reinterpret_cast<uint4*>(xr + c) = pack8(o);
  }
}

template <int NC>
void launch_residual_norm(const ResNormParams& p, cudaStream_t s) {
  residual_norm_kernel<NC><<<(p.rows + kRowWarps - 1) / kRowWarps, 32 * kRowWarps, 0, s>>>(p);
}

// ------------------------------------------------------------------ GLU (+ per-row int8 quantisation)
constexpr int kGluThreads = 256;
constexpr int kGluChunks = 4;  // F <= 256 * 8 * 4 = 8192

template <bool kQuant>
__global__ void __launch_bounds__(kGluThreads) glu_rows_kernel(const uint16_t* __restrict__ g, int64_t ldg, int F,
                                                              uint16_t* __restrict__ z, int64_t ldz,
                                                              int8_t* __restrict__ q, int64_t ldq,
                                                              float* __restrict__ scale) {
  __shared__ float warp_max[kGluThreads / 32];
  const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const uint16_t* value = g + (size_t)r * ldg;
  const uint16_t* gate = value + F;
  float zv[kGluChunks][8];
  float amax = 0.f;
  uint4 va[kGluChunks], ga[kGluChunks];
#pragma unroll
  for (int i = 0; i < kGluChunks; ++i) {
    const int k = (tid + kGluThreads * i) * 8;
    if (k < F) {
      va[i] = ld_nc_v4(value + k);
      ga[i] = ld_nc_v4(gate + k);
    }
  }
#pragma unroll
  for (int i = 0; i < kGluChunks; ++i) {
    const int k = (tid + kGluThreads * i) * 8;
    if (k >= F) continue;
    float a[8], b[8];
    unpack8(va[i], a);
    unpack8(ga[i], b);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float silu = round_bf16(b[e] / (1.f + __expf(-b[e])));
      zv[i][e] = round_bf16(a[e] * silu);
      amax = fmaxf(amax, fabsf(zv[i][e]));
    }
    if constexpr (!kQuant) *reinterpret_cast<uint4*>(z + (size_t)r * ldz + k) = pack8(zv[i]);
  }
  if constexpr (kQuant) {
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) warp_max[tid >> 5] = amax;
    __syncthreads();
    amax = warp_max[0];
#pragma unroll
    for (int w = 1; w < kGluThreads / 32; ++w) amax = fmaxf(amax, warp_max[w]);
    const float s = amax == 0.f ? 1.f : __fdiv_rn(amax, 127.f);
    if (tid == 0) scale[r] = s;
#pragma unroll
    for (int i = 0; i < kGluChunks; ++i) {
      const int k = (tid + kGluThreads * i) * 8;
      if (k >= F) continue;
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float qv = fminf(fmaxf(rintf(__fdiv_rn(zv[i][e], s)), -127.f), 127.f);
        packed[e >> 2] |= (static_cast<uint32_t>(static_cast<int>(qv)) & 0xFFu) << (8 * (e & 3));
      }
      *reinterpret_cast<uint2*>(q + (size_t)r * ldq + k) = make_uint2(packed[0], packed[1]);
    }
  }
}

// ------------------------------------------------------------------ per-head RMSNorm
// 8 threads per 64-dim head, one 16-byte chunk each; the sum of squares is reduced over the 8 lanes.
__global__ void __launch_bounds__(256) head_rms_kernel(const uint16_t* __restrict__ x, int64_t ldx, int rows,
                                                       int heads, const uint16_t* __restrict__ w, float eps,
                                                       uint16_t* __restrict__ out, int64_t ldo) {
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long unit = gid >> 3;
  const int sub = static_cast<int>(gid & 7);
  const bool live = unit < (long long)rows * heads;
  const int r = live ? static_cast<int>(unit / heads) : 0;
  const int hh = live ? static_cast<int>(unit - (long long)r * heads) : 0;
  float v[8], wv[8];
  if (live) unpack8(ld_v4(x + (size_t)r * ldx + hh * 64 + sub * 8), v);
  else
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  ss += __shfl_xor_sync(0xffffffffu, ss, 4);
  if (!live) return;
  const float inv = rsqrtf(ss / 64.f + eps);
  unpack8(ld_v4(w + sub * 8), wv);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], inv) * wv[e];
  *reinterpret_cast<uint4*>(out + (size_t)r * ldo + hh * 64 + sub * 8) = pack8(v);
}

}  // namespace
}  // namespace hb

using namespace hb;

extern "C" int hb_dit_residual_norm(void* h, int64_t ldh, const void* y, int64_t ldy, const void* gate,
                                    const void* scale, const void* shift, int64_t ldc, const void* local,
                                    int local_row0, const void* weight, void* x, int64_t ldx, int rows,
                                    int rows_per_batch, int d, float eps, cudaStream_t stream) {
  if (!h || (x && !weight) || (scale && !shift) || (!scale && shift)) return HB_ERR_NULL;
  if (rows < 1 || rows_per_batch < 1 || d < 256 || d > 2048 || d % 256 || ldh < d || (y && ldy < d) ||
      (x && ldx < d) || ((gate || scale) && ldc < d) || (gate && !y))
    return HB_ERR_SHAPE;
  const void* ptrs[] = {h, y, gate, scale, shift, local, weight, x};
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return HB_ERR_ALIGN;
  if (ldh % 8 || (y && ldy % 8) || (x && ldx % 8) || ldc % 8) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  ResNormParams p{static_cast<uint16_t*>(h), ldh, static_cast<const uint16_t*>(y), ldy,
                  static_cast<const uint16_t*>(gate), static_cast<const uint16_t*>(scale),
                  static_cast<const uint16_t*>(shift), ldc, static_cast<const uint16_t*>(local), local_row0,
                  static_cast<const uint16_t*>(weight), static_cast<uint16_t*>(x), ldx, rows, rows_per_batch, d,
                  eps};
  switch (d / 256) {
    case 1: launch_residual_norm<1>(p, stream); break;
    case 2: launch_residual_norm<2>(p, stream); break;
    case 3: launch_residual_norm<3>(p, stream); break;
    case 4: launch_residual_norm<4>(p, stream); break;
    case 5: launch_residual_norm<5>(p, stream); break;
    case 6: launch_residual_norm<6>(p, stream); break;
    case 7: launch_residual_norm<7>(p, stream); break;
    default: launch_residual_norm<8>(p, stream); break;
  }
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

extern "C" int hb_glu_rows(const void* glu, int64_t ldg, int rows, int F, void* z, int64_t ldz, void* q, int64_t ldq,
                           float* scale, cudaStream_t stream) {
  if (!glu || (!z && !q) || (z && q) || (q && !scale)) return HB_ERR_NULL;
  if (rows < 1 || F < 8 || F % 8 || F > kGluThreads * 8 * kGluChunks || ldg < 2 * F || (z && ldz < F) ||
      (q && ldq < F))
    return HB_ERR_SHAPE;
  if (!aligned16(glu) || ldg % 8 || (z && (!aligned16(z) || ldz % 8)) ||
      (q && ((reinterpret_cast<uintptr_t>(q) & 7u) || ldq % 8)))
    return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  if (q)
    glu_rows_kernel<true><<<rows, kGluThreads, 0, stream>>>(static_cast<const uint16_t*>(glu), ldg, F, nullptr, 0,
                                                             static_cast<int8_t*>(q), ldq, scale);
  else
    glu_rows_kernel<false><<<rows, kGluThreads, 0, stream>>>(static_cast<const uint16_t*>(glu), ldg, F,
                                                              static_cast<uint16_t*>(z), ldz, nullptr, 0, nullptr);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

extern "C" int hb_head_rms_norm(const void* x, int64_t ldx, int rows, int heads, const void* weight, float eps,
                                void* out, int64_t ldo, cudaStream_t stream) {
  if (!x || !weight || !out) return HB_ERR_NULL;
  if (rows < 1 || heads < 1 || ldx < heads * 64 || ldo < heads * 64) return HB_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || ldx % 8 || ldo % 8) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  const long long threads = (long long)rows * heads * 8;
  if ((threads + 255) / 256 > 0x7fffffffLL) return HB_ERR_SHAPE;
  head_rms_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      static_cast<const uint16_t*>(x), ldx, rows, heads, static_cast<const uint16_t*>(weight), eps,
      static_cast<uint16_t*>(out), ldo);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

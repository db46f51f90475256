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
#include <algorithm>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "hb_sm100.cuh"
#include "prep_common.cuh"
#include "quant_common.cuh"

namespace hb {
namespace {

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Two bf16 roundings with one packed conversion (the conversions share the transcendental pipe with exp and
// the reciprocal, which bounds the GLU); the same round-to-nearest-even as round_bf16 on each value.
__device__ __forceinline__ void round_bf16_pair(float& a, float& b) {
  const uint32_t w = pack_bf16x2(a, b);
  a = bf16_lo(w);
  b = bf16_hi(w);
}

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
  int8_t* xq;         // optional: x quantised per row (hb_quant_rows_int8's rules on the bf16 x) ...
  int64_t ldxq;
  float* xscale;      // ... and its per-row scales
};

constexpr int kRowWarps = 8;
constexpr size_t kResNormMaxSmem = 96 * 1024;  // per-column vectors of every batch element: nb * 5 * d fp32

// Persistent row stream: the per-column vectors of every batch element (sigmoid(1 - gate), the RMSNorm weight,
// 1 + scale, shift, local; fp32 with the torch sequence's roundings) are evaluated once per block into shared
// memory; then warp w of W walks rows w, w + W, ..., loading the next row's h and y while it finishes the
// current one. Lane l holds the 16-byte chunks l, l + 32, ... of a row (NC chunks, d = 256 NC).
constexpr int kStreamBlocksPerSm = 2;

__host__ __device__ constexpr int colv_floats(int nb, int d) { return nb * 5 * d; }

template <int NC>
__device__ __forceinline__ void residual_norm_row(const ResNormParams& p, const float* cv, int r, const uint4 (&hv4)[NC],
                                                  const uint4 (&yv4)[NC], int lane) {
  constexpr int d = 256 * NC;
  const float* gm = cv;           // sigmoid(1 - gate)
  const float* wv = cv + d;       // RMSNorm weight
  const float* sc1 = cv + 2 * d;  // 1 + scale
  const float* shv = cv + 3 * d;  // shift
  const float* lv = cv + 4 * d;   // local
  const int t = r % p.rows_per_batch;
  uint16_t* hr = p.h + (size_t)r * p.ldh;
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
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] + yv[e] * gm[c + e];
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] + yv[e];
      }
#pragma unroll
      for (int e = 0; e < 8; e += 2) round_bf16_pair(v[i][e], v[i][e + 1]);
    }
    if (add_local) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] + lv[c + e];
#pragma unroll
      for (int e = 0; e < 8; e += 2) round_bf16_pair(v[i][e], v[i][e + 1]);
    }
    if (p.y || add_local) *reinterpret_cast<uint4*>(hr + c) = pack8(v[i]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
  }
  if (!p.x && !p.xq) return;
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(d) + p.eps);
  // x = RMSNorm(h) * w (rounded to bf16), then (1 + scale) and shift; the bf16 rounding of the store is applied
  // here too, so the quantised form sees exactly the values of the bf16 x
  float (&o)[NC][8] = v;  // x overwrites the residual row in registers (h is stored already)
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = (i * 32 + lane) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[i][e] = __fmul_rn(v[i][e], inv) * wv[c + e];
#pragma unroll
    for (int e = 0; e < 8; e += 2) round_bf16_pair(o[i][e], o[i][e + 1]);
    if (p.scale) {
#pragma unroll
      for (int e = 0; e < 8; ++e) o[i][e] = __fadd_rn(shv[c + e], __fmul_rn(o[i][e], sc1[c + e]));
    }
#pragma unroll
    for (int e = 0; e < 8; e += 2) round_bf16_pair(o[i][e], o[i][e + 1]);
    if (p.x) *reinterpret_cast<uint4*>(p.x + (size_t)r * p.ldx + c) = pack8(o[i]);
  }
  if (!p.xq) return;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(o[i][e]));
#pragma unroll
  for (int s2 = 16; s2; s2 >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s2));
  const float s = amax == 0.f ? 1.f : __fdiv_rn(amax, 127.f);
  const float rs = __frcp_rn(s);
  if (lane == 0) p.xscale[r] = s;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = (i * 32 + lane) * 8;
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) packed[e >> 2] |= int8_bits(quantize_int8(o[i][e], s, rs)) << (8 * (e & 3));
    *reinterpret_cast<uint2*>(p.xq + (size_t)r * p.ldxq + c) = make_uint2(packed[0], packed[1]);
  }
}

template <int NC>
__device__ __forceinline__ void residual_norm_load(const ResNormParams& p, int r, int lane, uint4 (&hv4)[NC],
                                                   uint4 (&yv4)[NC]) {
  const uint16_t* hr = p.h + (size_t)r * p.ldh;
#pragma unroll
  for (int i = 0; i < NC; ++i) hv4[i] = ld_v4(hr + (i * 32 + lane) * 8);
  if (p.y) {
    const uint16_t* yr = p.y + (size_t)r * p.ldy;
#pragma unroll
    for (int i = 0; i < NC; ++i) yv4[i] = ld_v4(yr + (i * 32 + lane) * 8);
  }
}

template <int NC>
__global__ void __launch_bounds__(32 * kRowWarps, kStreamBlocksPerSm)
    residual_norm_kernel(const ResNormParams p, int nb) {
  constexpr int d = 256 * NC;
  extern __shared__ float colv[];
  const int lane = threadIdx.x & 31;
  const int total_warps = gridDim.x * kRowWarps;
  int r = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  uint4 hv4[NC], yv4[NC];
  if (r < p.rows) residual_norm_load<NC>(p, r, lane, hv4, yv4);  // in flight during the column setup
  for (int idx = threadIdx.x; idx < nb * (d / 8); idx += 32 * kRowWarps) {
    const int b = idx / (d / 8), c = (idx - b * (d / 8)) * 8;
    float* cv = colv + colv_floats(b, d);
    float u[8];
    if (p.y && p.gate) {
      unpack8(ld_v4(p.gate + (size_t)b * p.ldc + c), u);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float a = round_bf16(1.f - u[e]);
        cv[c + e] = round_bf16(1.f / (1.f + __expf(-a)));
      }
    }
    if (p.x || p.xq) {
      unpack8(ld_v4(p.w + c), u);
#pragma unroll
      for (int e = 0; e < 8; ++e) cv[d + c + e] = u[e];
    }
    if (p.scale) {
      unpack8(ld_v4(p.scale + (size_t)b * p.ldc + c), u);
#pragma unroll
      for (int e = 0; e < 8; ++e) cv[2 * d + c + e] = round_bf16(1.f + u[e]);
      unpack8(ld_v4(p.shift + (size_t)b * p.ldc + c), u);
#pragma unroll
      for (int e = 0; e < 8; ++e) cv[3 * d + c + e] = u[e];
    }
    if (p.local) {
      unpack8(ld_v4(p.local + c), u);
#pragma unroll
      for (int e = 0; e < 8; ++e) cv[4 * d + c + e] = u[e];
    }
  }
  __syncthreads();
  while (r < p.rows) {  // warp-uniform
    const int rn = r + total_warps;
    uint4 hn[NC], yn[NC];
    if (rn < p.rows) residual_norm_load<NC>(p, rn, lane, hn, yn);
    residual_norm_row<NC>(p, colv + colv_floats(r / p.rows_per_batch, d), r, hv4, yv4, lane);
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      hv4[i] = hn[i];
      yv4[i] = yn[i];
    }
    r = rn;
  }
}

// One launch per group of batch elements whose column vectors fit kResNormMaxSmem.
template <int NC>
int launch_residual_norm(const ResNormParams& p, cudaStream_t s) {
  const int nb_all = (p.rows + p.rows_per_batch - 1) / p.rows_per_batch;
  const int per_launch = static_cast<int>(kResNormMaxSmem / (colv_floats(1, 256 * NC) * sizeof(float)));
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(residual_norm_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kResNormMaxSmem) != cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  for (int b0 = 0; b0 < nb_all; b0 += per_launch) {
    const int nb = nb_all - b0 < per_launch ? nb_all - b0 : per_launch;
    const long long row0 = (long long)b0 * p.rows_per_batch;
    ResNormParams q = p;
    q.rows = static_cast<int>(std::min<long long>(p.rows - row0, (long long)nb * p.rows_per_batch));
    q.h = p.h + row0 * p.ldh;
    if (p.y) q.y = p.y + row0 * p.ldy;
    if (p.x) q.x = p.x + row0 * p.ldx;
    if (p.gate) q.gate = p.gate + (size_t)b0 * p.ldc;
    if (p.scale) q.scale = p.scale + (size_t)b0 * p.ldc;
    if (p.shift) q.shift = p.shift + (size_t)b0 * p.ldc;
    const size_t smem = colv_floats(nb, 256 * NC) * sizeof(float);
    const int need = (q.rows + kRowWarps - 1) / kRowWarps;
    const int grid = need < sms * kStreamBlocksPerSm ? need : sms * kStreamBlocksPerSm;
    residual_norm_kernel<NC><<<grid, 32 * kRowWarps, smem, s>>>(q, nb);
    if (cudaGetLastError() != cudaSuccess) return HB_ERR_LAUNCH;
  }
  return HB_OK;
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
    for (int e = 0; e < 8; e += 2) {
      float s0 = __fdividef(b[e], 1.f + __expf(-b[e])), s1 = __fdividef(b[e + 1], 1.f + __expf(-b[e + 1]));
      round_bf16_pair(s0, s1);  // silu, stored as bf16 by the unfused sequence
      zv[i][e] = a[e] * s0;
      zv[i][e + 1] = a[e + 1] * s1;
      round_bf16_pair(zv[i][e], zv[i][e + 1]);
      amax = fmaxf(amax, fmaxf(fabsf(zv[i][e]), fabsf(zv[i][e + 1])));
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
    const float rs = __frcp_rn(s);
    if (tid == 0) scale[r] = s;
#pragma unroll
    for (int i = 0; i < kGluChunks; ++i) {
      const int k = (tid + kGluThreads * i) * 8;
      if (k >= F) continue;
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        packed[e >> 2] |= int8_bits(quantize_int8(zv[i][e], s, rs)) << (8 * (e & 3));
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

namespace {

int residual_norm_entry(void* h, int64_t ldh, const void* y, int64_t ldy, const void* gate, const void* scale,
                        const void* shift, int64_t ldc, const void* local, int local_row0, const void* weight, void* x,
                        int64_t ldx, void* q, int64_t ldq, float* qscale, int rows, int rows_per_batch, int d,
                        float eps, cudaStream_t stream) {
  if (!h || ((x || q) && !weight) || (scale && !shift) || (!scale && shift) || (q && !qscale)) return HB_ERR_NULL;
  if (rows < 1 || rows_per_batch < 1 || d < 256 || d > 2048 || d % 256 || ldh < d || (y && ldy < d) ||
      (x && ldx < d) || (q && ldq < d) || ((gate || scale) && ldc < d) || (gate && !y))
    return HB_ERR_SHAPE;
  const void* ptrs[] = {h, y, gate, scale, shift, local, weight, x};
  for (const void* pp : ptrs)
    if (pp && !aligned16(pp)) return HB_ERR_ALIGN;
  if (ldh % 8 || (y && ldy % 8) || (x && ldx % 8) || ldc % 8) return HB_ERR_ALIGN;
  if (q && ((reinterpret_cast<uintptr_t>(q) & 7u) || ldq % 8)) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  ResNormParams p{static_cast<uint16_t*>(h), ldh, static_cast<const uint16_t*>(y), ldy,
                  static_cast<const uint16_t*>(gate), static_cast<const uint16_t*>(scale),
                  static_cast<const uint16_t*>(shift), ldc, static_cast<const uint16_t*>(local), local_row0,
                  static_cast<const uint16_t*>(weight), static_cast<uint16_t*>(x), ldx, rows, rows_per_batch, d,
                  eps, static_cast<int8_t*>(q), ldq, qscale};
  switch (d / 256) {
    case 1: return launch_residual_norm<1>(p, stream);
    case 2: return launch_residual_norm<2>(p, stream);
    case 3: return launch_residual_norm<3>(p, stream);
    case 4: return launch_residual_norm<4>(p, stream);
    case 5: return launch_residual_norm<5>(p, stream);
    case 6: return launch_residual_norm<6>(p, stream);
    case 7: return launch_residual_norm<7>(p, stream);
    default: return launch_residual_norm<8>(p, stream);
  }
}

}  // namespace

extern "C" int hb_dit_residual_norm(void* h, int64_t ldh, const void* y, int64_t ldy, const void* gate,
                                    const void* scale, const void* shift, int64_t ldc, const void* local,
                                    int local_row0, const void* weight, void* x, int64_t ldx, int rows,
                                    int rows_per_batch, int d, float eps, cudaStream_t stream) {
  return residual_norm_entry(h, ldh, y, ldy, gate, scale, shift, ldc, local, local_row0, weight, x, ldx, nullptr, 0,
                             nullptr, rows, rows_per_batch, d, eps, stream);
}

extern "C" int hb_dit_residual_norm_int8(void* h, int64_t ldh, const void* y, int64_t ldy, const void* gate,
                                         const void* scale, const void* shift, int64_t ldc, const void* local,
                                         int local_row0, const void* weight, void* q, int64_t ldq, float* qscale,
                                         int rows, int rows_per_batch, int d, float eps, cudaStream_t stream) {
  if (!q) return HB_ERR_NULL;
  return residual_norm_entry(h, ldh, y, ldy, gate, scale, shift, ldc, local, local_row0, weight, nullptr, 0, q, ldq,
                             qscale, rows, rows_per_batch, d, eps, stream);
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

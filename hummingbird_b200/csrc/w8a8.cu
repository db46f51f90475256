// W8A8 int8 GEMM for the DiT MLP (`dit._feed_forward` -> `dit._linear`, dit.py:33-36, 218-221, which the
// reference runs as a bf16 matmul; the quantised form is fixed by the benchmark configs).
//
// hb_quant_rows_int8: per row, absmax -> scale = absmax / 127 (correctly rounded fp32 division, 1 when the
//   row is all zero) -> q = clamp(rint(x / scale), -127, 127) with a correctly rounded division and
//   round-half-to-even. Activations are quantised per token, weights per output channel (rows of W[N, K]).
// hb_w8a8_gemm: acc[m, n] = sum_k qx[m, k] qw[n, k] on tcgen05 (kind::i8, s32 accumulators in TMEM, operands
//   staged by 2-D TMA with 128-byte swizzle), then y = bf16(((float)acc * sx[m]) * sw[n] + bias[n]) with each
//   fp32 step rounded separately (no contraction), so the output is reproducible bit for bit on the CPU.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

// ------------------------------------------------------------------ quantiser
constexpr int kQuantWarps = 8;

__global__ void __launch_bounds__(kQuantWarps * 32) quant_rows_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                                      int rows, int K, int8_t* __restrict__ q,
                                                                      int64_t ldq, float* __restrict__ scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kQuantWarps + warp;
  if (r >= rows) return;
  const uint16_t* xr = x + (size_t)r * ldx;
  float amax = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fmaxf(fabsf(bf16_lo(w[i])), fabsf(bf16_hi(w[i]))));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = amax == 0.f ? 1.f : __fdiv_rn(amax, 127.f);
  if (lane == 0) scale[r] = s;
  int8_t* qr = q + (size_t)r * ldq;
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t packed[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float xv = (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
      const float qv = fminf(fmaxf(rintf(__fdiv_rn(xv, s)), -127.f), 127.f);
      packed[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(qv)) & 0xFFu) << (8 * (i & 3));
    }
    *reinterpret_cast<uint2*>(qr + k) = make_uint2(packed[0], packed[1]);
  }
}

// ------------------------------------------------------------------ GEMM
constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int kGemmThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOffBars = kStages * kStageBytes;
  static constexpr int kSmem = kOffBars + (2 * kStages + 2) * 8 + 16 + 1024;
};

struct GemmEpi {
  const float* sx;
  const float* sw;
  const uint16_t* bias;
  uint16_t* out;
  int64_t ldo;
  int32_t* acc_out;
  int64_t ldacc;
  int M, N, K;
};

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const GemmEpi e) {
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  uint64_t* bar_empty = bar_full + C::kStages;
  uint64_t* bar_acc = bar_empty + C::kStages;
  uint64_t* bar_drain = bar_acc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
  const int nk = (e.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(bar_acc, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        if (i >= C::kStages && !mbar_wait(&bar_empty[st], ((i / C::kStages) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* sa = smem + st * C::kStageBytes;
        mbar_arrive_expect_tx(&bar_full[st], C::kStageBytes);
        tma_load_2d(sa, &tmap_a, i * kBK, m0, &bar_full[st]);
        tma_load_2d(sa + C::kABytes, &tmap_b, i * kBK, n0, &bar_full[st]);
        issued = i + 1;
      }
      for (int i = max(0, issued - C::kStages); i < issued; ++i)
        mbar_wait(&bar_full[i % C::kStages], (i / C::kStages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kBM, BN);
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int st = i % C::kStages;
        if (!mbar_wait(&bar_full[st], (i / C::kStages) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + st * C::kStageBytes);
        const uint32_t sb = sa + C::kABytes;
#pragma unroll
        for (int k = 0; k < kBK / 32; ++k)
          mma_i8_ss(tmem, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc, (i > 0 || k > 0));
        tc_commit(&bar_empty[st]);
      }
      if (ok) tc_commit(bar_acc);
      else *abort_flag = 1;
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0);
    }
  } else {
    // epilogue: warps 2..5 -> TMEM lane quadrants 2, 3, 0, 1
    const int quad = warp & 3;
    const int m = m0 + quad * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_acc, 0));
    tc_fence_after();
    if (ok) {
      const float sxm = m < e.M ? e.sx[m] : 0.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t acc[32];
        tmem_ld32(taddr + 32 * c, acc);
        tmem_wait_ld();
        const int n = n0 + 32 * c;
        if (m < e.M && n < e.N) {
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int nn = n + 2 * j + t;
              float v = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j + t])), sxm);
              v = __fmul_rn(v, __ldg(e.sw + nn));
              if (e.bias) v = __fadd_rn(v, __uint_as_float(static_cast<uint32_t>(__ldg(e.bias + nn)) << 16));
              y[t] = v;
            }
            w[j] = pack_bf16x2(y[0], y[1]);
          }
          uint4* d4 = reinterpret_cast<uint4*>(e.out + (size_t)m * e.ldo + n);
#pragma unroll
          for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          if (e.acc_out) {
            uint4* a4 = reinterpret_cast<uint4*>(e.acc_out + (size_t)m * e.ldacc + n);
#pragma unroll
            for (int j = 0; j < 8; ++j) a4[j] = make_uint4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D int8 tensor map over a row-major [rows, K] matrix with leading dimension `ld` bytes,
// box = 128 bytes of K x `box_rows` rows, 128-byte swizzle, out-of-range elements read as zero.
bool make_tmap_i8(CUtensorMap* map, const void* base, int rows, int K, int64_t ld, int box_rows) {
  auto encode = get_encode_fn();
  if (!encode) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmEpi& e, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(w8a8_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::kSmem) !=
        cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  dim3 grid((e.M + kBM - 1) / kBM, (e.N + BN - 1) / BN);
  w8a8_gemm_kernel<BN><<<grid, kGemmThreads, GemmCfg<BN>::kSmem, stream>>>(ta, tb, e);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

}  // namespace
}  // namespace hb

using namespace hb;

extern "C" int hb_quant_rows_int8(const void* x, int64_t ldx, int rows, int K, void* q, int64_t ldq, float* scale,
                                  cudaStream_t stream) {
  if (!x || !q || !scale) return HB_ERR_NULL;
  if (rows < 1 || K < 8 || K % 8 || ldx < K || ldq < K) return HB_ERR_SHAPE;
  if (!aligned16(x) || ldx % 8 || (reinterpret_cast<uintptr_t>(q) & 7u) || ldq % 8) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  quant_rows_kernel<<<(rows + kQuantWarps - 1) / kQuantWarps, kQuantWarps * 32, 0, stream>>>(
      static_cast<const uint16_t*>(x), ldx, rows, K, static_cast<int8_t*>(q), ldq, scale);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

extern "C" int hb_w8a8_gemm(const void* qx, int64_t ldqx, const float* sx, const void* qw, int64_t ldqw,
                            const float* sw, const void* bias, void* out, int64_t ldo, int32_t* acc_out,
                            int64_t ldacc, int M, int N, int K, cudaStream_t stream) {
  if (!qx || !sx || !qw || !sw || !out) return HB_ERR_NULL;
  if (M < 1 || N < 32 || N % 32 || K < 16 || K % 16 || ldqx < K || ldqw < K || ldo < N) return HB_ERR_SHAPE;
  if (acc_out && ldacc < N) return HB_ERR_SHAPE;
  if (!aligned16(qx) || ldqx % 16 || !aligned16(qw) || ldqw % 16 || !aligned16(out) || ldo % 8) return HB_ERR_ALIGN;
  if (acc_out && (!aligned16(acc_out) || ldacc % 4)) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  GemmEpi e{sx, sw, static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(out), ldo, acc_out, ldacc, M, N, K};
  const bool wide = (N % 256 == 0) && ((long)((M + kBM - 1) / kBM) * (N / 256) >= 148);
  CUtensorMap ta, tb;
  if (!make_tmap_i8(&ta, qx, M, K, ldqx, kBM)) return HB_ERR_LAUNCH;
  if (!make_tmap_i8(&tb, qw, N, K, ldqw, wide ? 256 : 128)) return HB_ERR_LAUNCH;
  return wide ? launch_gemm<256>(ta, tb, e, stream) : launch_gemm<128>(ta, tb, e, stream);
}

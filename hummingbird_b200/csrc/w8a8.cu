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
#include "quant_common.cuh"

namespace hb {

#ifdef HB_TRACE
extern __device__ unsigned int g_trace[8][2048];
extern __device__ unsigned int g_trace_n[8];
#define GTRACE(slot, id, t0)                                                          \
  do {                                                                                \
    if (blockIdx.x == 0) {                                                            \
      const unsigned n_ = g_trace_n[slot]++;                                          \
      if (n_ < 1024) {                                                                \
        g_trace[slot][2 * n_] = (id);                                                 \
        g_trace[slot][2 * n_ + 1] = static_cast<unsigned>(clock64() - (t0));          \
      }                                                                               \
    }                                                                                 \
  } while (0)
#else
#define GTRACE(slot, id, t0) \
  do {                       \
  } while (0)
#endif

namespace {

// ------------------------------------------------------------------ quantiser
// One 128-thread CTA per row: each thread holds up to kQuantChunks 16-byte chunks of the row in registers
// (all loads in flight together), a block reduction gives the row absmax, then the chunks are quantised and
// written. Rows longer than 128 * 8 * kQuantChunks elements take a second pass over global memory.
constexpr int kQuantThreads = 128;
constexpr int kQuantChunks = 4;  // rows up to 4096 elements held in registers

__device__ __forceinline__ uint2 quantize8(const uint4& v, float s, float rs) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t packed[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float xv = (i & 1) ? bf16_hi(w[i >> 1]) : bf16_lo(w[i >> 1]);
    packed[i >> 2] |= int8_bits(quantize_int8(xv, s, rs)) << (8 * (i & 3));
  }
  return make_uint2(packed[0], packed[1]);
}

__device__ __forceinline__ float absmax8(const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) a = fmaxf(a, fmaxf(fabsf(bf16_lo(w[i])), fabsf(bf16_hi(w[i]))));
  return a;
}

__global__ void __launch_bounds__(kQuantThreads) quant_rows_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                                                                   int rows, int K, int8_t* __restrict__ q,
                                                                   int64_t ldq, float* __restrict__ scale) {
  __shared__ float warp_max[kQuantThreads / 32];
  const int r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const uint16_t* xr = x + (size_t)r * ldx;
  int8_t* qr = q + (size_t)r * ldq;
  const bool resident = K <= kQuantThreads * 8 * kQuantChunks;
  uint4 v[kQuantChunks];
  float amax = 0.f;
  if (resident) {
#pragma unroll
    for (int i = 0; i < kQuantChunks; ++i) {
      const int k = (tid + kQuantThreads * i) * 8;
      v[i] = k < K ? __ldg(reinterpret_cast<const uint4*>(xr + k)) : make_uint4(0, 0, 0, 0);
      amax = fmaxf(amax, absmax8(v[i]));
    }
  } else {
    for (int k = tid * 8; k < K; k += kQuantThreads * 8)
      amax = fmaxf(amax, absmax8(__ldg(reinterpret_cast<const uint4*>(xr + k))));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) warp_max[tid >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(warp_max[0], warp_max[1]), fmaxf(warp_max[2], warp_max[3]));
  const float s = amax == 0.f ? 1.f : __fdiv_rn(amax, 127.f);
  const float rs = __frcp_rn(s);
  if (tid == 0) scale[r] = s;
  if (resident) {
#pragma unroll
    for (int i = 0; i < kQuantChunks; ++i) {
      const int k = (tid + kQuantThreads * i) * 8;
      if (k < K) *reinterpret_cast<uint2*>(qr + k) = quantize8(v[i], s, rs);
    }
  } else {
    for (int k = tid * 8; k < K; k += kQuantThreads * 8)
      *reinterpret_cast<uint2*>(qr + k) = quantize8(__ldg(reinterpret_cast<const uint4*>(xr + k)), s, rs);
  }
}

// ------------------------------------------------------------------ GEMM
// Persistent: grid = min(#SMs, tiles); CTA c takes tiles c, c + grid, ... ordered m-fastest so the CTAs
// working at the same time share B (weight) tiles in L2. Warp 0 issues TMA loads through a stage ring,
// warp 1 issues tcgen05.mma (kind::i8, M128 x BN x K32) into one of two TMEM accumulators, and warps 2-9
// run the epilogue of the previous tile from the other accumulator while the next tile's MMAs run (each
// TMEM lane quadrant is read by two warps, one per half of the tile's columns).
constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int kGemmThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (two per TMEM lane quadrant)
constexpr int kEpiThreads = 256;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 3 : 5;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOffOut = kStages * kStageBytes;             // bf16 output tile: BN / 64 boxes of 128 x 64
  static constexpr int kOutBytes = kBM * BN * 2;
  static constexpr int kOffParams = kOffOut + kOutBytes;            // sw, bias of the tile: [2][2][BN] fp32
  static constexpr int kOffBars = kOffParams + 2 * 2 * BN * 4;
  static constexpr int kNumBars = 2 * kStages + 2 + 2 + 2;           // full, empty, acc_full, acc_empty, drain
  static constexpr int kSmem = kOffBars + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;                      // two accumulators
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

// The GLU of `dit._feed_forward` (dit.py:218-221) in the epilogue (kGlu, BN = 256): the weight rows come
// interleaved in blocks of 128 (value rows [128 t, 128 t + 128), then the matching gate rows), so a tile's
// accumulator columns [0, 128) are value and [128, 256) gate columns of the same 128 outputs. Each pair is
// rounded to bf16 as the plain epilogue would store it, then z = value * silu(gate) with silu rounded to bf16
// and z rounded to bf16: the arithmetic of hb_glu_rows, so z is bit-identical to that kernel run on this GEMM's
// plain output. Only z (128 columns per tile) is written.
__device__ __forceinline__ float silu_glu(float g) { return __fdividef(g, 1.f + __expf(-g)); }

template <int BN, bool kGlu = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_out, const GemmEpi e) {
  static_assert(!kGlu || BN == 256, "the GLU epilogue pairs 128 value with 128 gate columns");
  using C = GemmCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* params = reinterpret_cast<float*>(smem + C::kOffParams);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  uint64_t* bar_empty = bar_full + C::kStages;
  uint64_t* acc_full = bar_empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;           // [2]
  uint64_t* drain = acc_empty + 2;              // [2] MMA thread, producer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long t0 = clock64();
  (void)t0;
  const int num_m = (e.M + kBM - 1) / kBM, num_n = (e.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int nk = (e.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiThreads / 32);
      mbar_init(&drain[a], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int it = 0;  // global k-step counter over this CTA's tiles
      for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
        const int m0 = (tile % num_m) * kBM, n0 = (tile / num_m) * BN;
        for (int i = 0; i < nk; ++i, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages && !mbar_wait(&bar_empty[st], ((it / C::kStages) & 1) ^ 1)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* sa = smem + st * C::kStageBytes;
          GTRACE(0, 100 + it, t0);
          mbar_arrive_expect_tx(&bar_full[st], C::kStageBytes);
          tma_load_2d(sa, &tmap_a, i * kBK, m0, &bar_full[st]);
          tma_load_2d(sa + C::kABytes, &tmap_b, i * kBK, n0, &bar_full[st]);
        }
      }
      for (int j = max(0, it - C::kStages); j < it; ++j) mbar_wait(&bar_full[j % C::kStages], (j / C::kStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kBM, BN);
      bool ok = true;
      int it = 0, local = 0;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++local) {
        const int a = local & 1;
        if (local >= 2 && !mbar_wait(&acc_empty[a], ((local >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        for (int i = 0; i < nk; ++i, ++it) {
          const int st = it % C::kStages;
          if (!mbar_wait(&bar_full[st], (it / C::kStages) & 1) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          GTRACE(1, 100 + it, t0);
          const uint32_t sa = smem_u32(smem + st * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_i8_ss(acc, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc, (i > 0 || k > 0));
          tc_commit(&bar_empty[st]);
        }
        if (ok) tc_commit(&acc_full[a]);
      }
      if (!ok) *abort_flag = 1;
      tc_commit(&drain[0]);
      mbar_wait(&drain[0], 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue: warps 2..9
    const int quad = warp & 3;                 // TMEM lanes 32 * quad .. + 31 (warp % 4 rule)
    const int half = (warp - 2) >> 2;          // columns [half * BN / 2, (half + 1) * BN / 2)
    const int et = threadIdx.x - 64;           // 0 .. kEpiThreads - 1
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int local = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
      const int a = local & 1;
      const int m0 = (tile % num_m) * kBM, n0 = (tile / num_m) * BN;
      // the previous tile's TMA store must have read the staging buffer before it is overwritten
      if (et == 0 && local > 0) bulk_wait_group_read0();
      // this tile's per-column scale and bias into shared memory (double-buffered by tile parity)
      float* psw = params + (local & 1) * 2 * BN;
      float* pbias = psw + BN;
      for (int c = et; c < BN; c += kEpiThreads) {
        const int n = n0 + c;
        psw[c] = n < e.N ? e.sw[n] : 0.f;
        pbias[c] = (e.bias && n < e.N) ? __uint_as_float(static_cast<uint32_t>(e.bias[n]) << 16) : 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      // same outcome in every epilogue warp (they meet at the named barriers of this and the next tile)
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[a], (local >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      const int r = quad * 32 + lane;  // row within the tile
      const int m = m0 + r;
      const float sxm = m < e.M ? e.sx[m] : 0.f;
      const uint32_t taddr = tmem + lane_base + a * BN;
      uint8_t* stage_out = smem + C::kOffOut;
      if constexpr (kGlu) {
        // z columns [32 c, 32 c + 32) of the tile from value chunk c and gate chunk c + 4 (two per warp)
#pragma unroll 1
        for (int c = 2 * half; c < 2 * half + 2; ++c) {
          uint32_t av[32], ag[32];
          tmem_ld32(taddr + 32 * c, av);
          tmem_ld32(taddr + 128 + 32 * c, ag);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float yv[2], yg[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int cv = 32 * c + 2 * j + t, cg = cv + 128;
              yv[t] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(av[2 * j + t])), sxm), psw[cv]),
                                pbias[cv]);
              yg[t] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(ag[2 * j + t])), sxm), psw[cg]),
                                pbias[cg]);
            }
            const uint32_t vw = pack_bf16x2(yv[0], yv[1]), gw = pack_bf16x2(yg[0], yg[1]);
            const float v0 = bf16_lo(vw), v1 = bf16_hi(vw), g0 = bf16_lo(gw), g1 = bf16_hi(gw);
            const uint32_t sw2 = pack_bf16x2(silu_glu(g0), silu_glu(g1));  // silu stored as bf16
            w[j] = pack_bf16x2(v0 * bf16_lo(sw2), v1 * bf16_hi(sw2));
          }
          uint8_t* box = stage_out + (c >> 1) * (kBM * 128);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(box + sw128_offset(r, (c & 1) * 4 + j)) =
                make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        }
      } else {
#pragma unroll 1
        for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
          uint32_t acc[32];
          tmem_ld32(taddr + 32 * c, acc);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int cc = 32 * c + 2 * j + t;
              float v = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j + t])), sxm);
              v = __fmul_rn(v, psw[cc]);
              y[t] = __fadd_rn(v, pbias[cc]);  // + 0 when there is no bias: exact
            }
            w[j] = pack_bf16x2(y[0], y[1]);
          }
          // 32 columns = half of a 64-column box: 4 16-byte chunks of this row in the swizzled staging
          uint8_t* box = stage_out + (c >> 1) * (kBM * 128);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(box + sw128_offset(r, (c & 1) * 4 + j)) =
                make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          if (e.acc_out && m < e.M && n0 + 32 * c < e.N) {
            uint4* a4 = reinterpret_cast<uint4*>(e.acc_out + (size_t)m * e.ldacc + n0 + 32 * c);
#pragma unroll
            for (int j = 0; j < 8; ++j) a4[j] = make_uint4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
          }
        }
      }
      // accumulator fully read: release it to the MMA thread
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      // staged tile -> global by TMA (rows past M and columns past N are clipped by the tensor map)
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (et == 0) {
        if constexpr (kGlu) {  // 128 z columns at z column n0 / 2
#pragma unroll 1
          for (int bx = 0; bx < 2; ++bx) tma_store_2d(&tmap_out, n0 / 2 + 64 * bx, m0, stage_out + bx * (kBM * 128));
        } else {
#pragma unroll 1
          for (int bx = 0; bx < BN / 64; ++bx)
            if (n0 + 64 * bx < e.N) tma_store_2d(&tmap_out, n0 + 64 * bx, m0, stage_out + bx * (kBM * 128));
        }
        bulk_commit_group();
      }
      if (et == 0) GTRACE(2, 200 + local, t0);
    }
    if (et == 0) bulk_wait_group0();  // stores complete before the CTA's shared memory goes away
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ GEMM on CTA pairs (cta_group::2)
// A cluster of two CTAs on neighbouring SMs computes a 256 x BN tile with one pair MMA stream: each CTA
// holds 128 rows of A and BN / 2 rows of W per stage, so every SM loads half the B bytes of the one-CTA
// kernel for the same MMA work. The even CTA's warp 1 issues `tcgen05.mma.cta_group::2`; each CTA's TMEM
// receives its own 128 rows of the accumulator and its epilogue warps convert and store them. Stage
// completion bytes of both CTAs count on the even CTA's `full` barrier; the pair MMA thread commits each
// stage and each accumulator to the barriers of both CTAs; both CTAs' epilogues release an accumulator on
// the even CTA's `acc_empty`. No TMA load uses multicast.
template <int BN>
struct PairCfg {
  static constexpr int kBHalf = BN / 2;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = kBHalf * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOffOut = kStages * kStageBytes;
  static constexpr int kOutBytes = kBM * BN * 2;
  static constexpr int kOffParams = kOffOut + kOutBytes;
  static constexpr int kOffBars = kOffParams + 2 * 2 * BN * 4;
  static constexpr int kNumBars = 2 * kStages + 2 + 2 + 1;  // full, empty, acc_full, acc_empty, drain
  static constexpr int kSmem = kOffBars + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;
};

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    w8a8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_out, const GemmEpi e) {
  using C = PairCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* params = reinterpret_cast<float*>(smem + C::kOffParams);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  uint64_t* bar_empty = bar_full + C::kStages;
  uint64_t* acc_full = bar_empty + C::kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;           // [2] used in the even CTA: 2 x 8 epilogue warps
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const int num_m = (e.M + 2 * kBM - 1) / (2 * kBM), num_n = (e.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int nk = (e.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * (kEpiThreads / 32));
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      for (int tile = cluster; tile < tiles && !*abort_flag; tile += clusters) {
        const int m0 = (tile % num_m) * 2 * kBM + static_cast<int>(rank) * kBM;
        const int nb = (tile / num_m) * BN + static_cast<int>(rank) * C::kBHalf;
        for (int i = 0; i < nk; ++i, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages && !mbar_wait(&bar_empty[st], ((it / C::kStages) & 1) ^ 1)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* sa = smem + st * C::kStageBytes;
          const uint32_t full0 = cluster_addr(smem_u32(&bar_full[st]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&bar_full[st], 2 * C::kStageBytes);
          tma_load_2d_pair(sa, &tmap_a, i * kBK, m0, full0);
          tma_load_2d_pair(sa + C::kABytes, &tmap_b, i * kBK, nb, full0);
        }
      }
      // every copy into this CTA's shared memory has landed before it exits: the even CTA's full barrier
      // completes only when both CTAs' bytes of a stage arrived, and the final cluster barrier below waits
      // for the even CTA, whose MMA thread consumed every stage
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- pair MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(2 * kBM, BN);
      bool ok = true;
      int it = 0, local = 0;
      for (int tile = cluster; ok && tile < tiles; tile += clusters, ++local) {
        const int a = local & 1;
        if (local >= 2 && !mbar_wait(&acc_empty[a], ((local >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        for (int i = 0; i < nk; ++i, ++it) {
          const int st = it % C::kStages;
          if (!mbar_wait(&bar_full[st], (it / C::kStages) & 1) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + st * C::kStageBytes);
          const uint32_t sb = sa + C::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k)
            mma_i8_ss_pair(acc, smem_desc_sw128(sa + 32 * k), smem_desc_sw128(sb + 32 * k), idesc, (i > 0 || k > 0));
          const uint32_t eb = smem_u32(&bar_empty[st]);
          tc_commit_pair(cluster_addr(eb, 0));
          tc_commit_pair(cluster_addr(eb, 1));
        }
        if (ok) {
          const uint32_t fb = smem_u32(&acc_full[a]);
          tc_commit_pair(cluster_addr(fb, 0));
          tc_commit_pair(cluster_addr(fb, 1));
        }
      }
      if (!ok) *abort_flag = 1;
      tc_commit_pair(cluster_addr(smem_u32(drain), 0));
      mbar_wait(drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- epilogue: warps 2..9 of both CTAs
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int et = threadIdx.x - 64;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int local = 0;
    for (int tile = cluster; tile < tiles; tile += clusters, ++local) {
      const int a = local & 1;
      const int m0 = (tile % num_m) * 2 * kBM + static_cast<int>(rank) * kBM, n0 = (tile / num_m) * BN;
      if (et == 0 && local > 0) bulk_wait_group_read0();
      float* psw = params + (local & 1) * 2 * BN;
      float* pbias = psw + BN;
      for (int c = et; c < BN; c += kEpiThreads) {
        const int n = n0 + c;
        psw[c] = n < e.N ? e.sw[n] : 0.f;
        pbias[c] = (e.bias && n < e.N) ? __uint_as_float(static_cast<uint32_t>(e.bias[n]) << 16) : 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[a], (local >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      const int r = quad * 32 + lane;
      const int m = m0 + r;
      const float sxm = m < e.M ? e.sx[m] : 0.f;
      const uint32_t taddr = tmem + lane_base + a * BN;
      uint8_t* stage_out = smem + C::kOffOut;
#pragma unroll 1
      for (int c = half * (BN / 64); c < (half + 1) * (BN / 64); ++c) {
        uint32_t acc[32];
        tmem_ld32(taddr + 32 * c, acc);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y[2];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int cc = 32 * c + 2 * j + t;
            float v = __fmul_rn(__int2float_rn(static_cast<int>(acc[2 * j + t])), sxm);
            v = __fmul_rn(v, psw[cc]);
            y[t] = __fadd_rn(v, pbias[cc]);
          }
          w[j] = pack_bf16x2(y[0], y[1]);
        }
        uint8_t* box = stage_out + (c >> 1) * (kBM * 128);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(box + sw128_offset(r, (c & 1) * 4 + j)) =
              make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        if (e.acc_out && m < e.M && n0 + 32 * c < e.N) {
          uint4* a4 = reinterpret_cast<uint4*>(e.acc_out + (size_t)m * e.ldacc + n0 + 32 * c);
#pragma unroll
          for (int j = 0; j < 8; ++j) a4[j] = make_uint4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(cluster_addr(smem_u32(&acc_empty[a]), 0));
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (et == 0) {
#pragma unroll 1
        for (int bx = 0; bx < BN / 64; ++bx)
          if (n0 + 64 * bx < e.N && m0 < e.M) tma_store_2d(&tmap_out, n0 + 64 * bx, m0, stage_out + bx * (kBM * 128));
        bulk_commit_group();
      }
    }
    if (et == 0) bulk_wait_group0();
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers or read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::kTmemCols);
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

// 2-D bf16 tensor map over the [M, N] output (leading dimension `ldo` elements): boxes of 64 columns x 128
// rows with 128-byte swizzle, matching the epilogue's staging layout.
bool make_tmap_out(CUtensorMap* map, void* base, int M, int N, int64_t ldo) {
  auto encode = get_encode_fn();
  if (!encode) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldo) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kBM)};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int BN, bool kGlu = false>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const GemmEpi& e,
                cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(w8a8_gemm_kernel<BN, kGlu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmCfg<BN>::kSmem) != cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((e.M + kBM - 1) / kBM) * ((e.N + BN - 1) / BN);
  w8a8_gemm_kernel<BN, kGlu><<<tiles < sms ? tiles : sms, kGemmThreads, GemmCfg<BN>::kSmem, stream>>>(ta, tb, to, e);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

template <int BN>
int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const GemmEpi& e,
                     cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(w8a8_gemm_pair_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PairCfg<BN>::kSmem) != cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((e.M + 2 * kBM - 1) / (2 * kBM)) * ((e.N + BN - 1) / BN);
  const int clusters = tiles < sms / 2 ? tiles : sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = PairCfg<BN>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, w8a8_gemm_pair_kernel<BN>, ta, tb, to, e) != cudaSuccess) return HB_ERR_LAUNCH;
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
  quant_rows_kernel<<<rows, kQuantThreads, 0, stream>>>(
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
  CUtensorMap ta, tb, to;
  if (!make_tmap_i8(&ta, qx, M, K, ldqx, kBM)) return HB_ERR_LAUNCH;
  if (!make_tmap_out(&to, out, M, N, ldo)) return HB_ERR_LAUNCH;
  // CTA pairs (256-row tiles, half the weight bytes per SM) pay off on long K: measured at 8192^3 2,911 vs
  // 2,557 TOPS; at the DiT / config-3 shapes (K <= 4096, two to nine waves) the one-CTA kernel is as fast
  // or faster (e.g. 5296 x 1024 x 8192: 53.2 vs 55.3 us), so it keeps those.
  if (M >= 8 * kBM && K >= 8192) {
    const bool wide = (N % 256 == 0) && ((long)((M + 2 * kBM - 1) / (2 * kBM)) * (N / 256) >= 74);
    if (!make_tmap_i8(&tb, qw, N, K, ldqw, wide ? 128 : 64)) return HB_ERR_LAUNCH;
    return wide ? launch_gemm_pair<256>(ta, tb, to, e, stream) : launch_gemm_pair<128>(ta, tb, to, e, stream);
  }
  // 256-column tiles whenever N allows, even with fewer tiles than SMs: MMAs of N = 128 followed by the stage
  // commits run at ~65 % of the tensor pipe's rate, N = 256 at the full rate (measured: config 3's second GEMM,
  // 84 tiles of 128 x 256 vs 168 of 128 x 128, 17.5 vs 27.0 us).
  const bool wide = (N % 256 == 0);
  if (!make_tmap_i8(&tb, qw, N, K, ldqw, wide ? 256 : 128)) return HB_ERR_LAUNCH;
  return wide ? launch_gemm<256>(ta, tb, to, e, stream) : launch_gemm<128>(ta, tb, to, e, stream);
}

extern "C" int hb_w8a8_gemm_glu(const void* qx, int64_t ldqx, const float* sx, const void* qw, int64_t ldqw,
                                const float* sw, const void* bias, void* z, int64_t ldz, int M, int F, int K,
                                cudaStream_t stream) {
  if (!qx || !sx || !qw || !sw || !z) return HB_ERR_NULL;
  if (M < 1 || F < 128 || F % 128 || K < 16 || K % 16 || ldqx < K || ldqw < K || ldz < F) return HB_ERR_SHAPE;
  if (!aligned16(qx) || ldqx % 16 || !aligned16(qw) || ldqw % 16 || !aligned16(z) || ldz % 8) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  GemmEpi e{sx, sw, static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(z), ldz, nullptr, 0, M, 2 * F, K};
  CUtensorMap ta, tb, to;
  if (!make_tmap_i8(&ta, qx, M, K, ldqx, kBM)) return HB_ERR_LAUNCH;
  if (!make_tmap_i8(&tb, qw, 2 * F, K, ldqw, 256)) return HB_ERR_LAUNCH;
  if (!make_tmap_out(&to, z, M, F, ldz)) return HB_ERR_LAUNCH;
  return launch_gemm<256, true>(ta, tb, to, e, stream);
}

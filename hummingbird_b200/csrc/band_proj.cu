// SAME-L attention front end in one tcgen05 GEMM: the block's DyT pre-norm, `to_qkv`, and the q / k DyT + RoPE
// of the band attention (same_l.py:157-160 and 191; band_attention.py:61-90).
//
//   x'  = bf16(gamma * tanh(alpha * x) + beta)      when a block pre-norm is given (`_dyt(x, pre_norm)` cast to
//                                                   the compute dtype, same_l.py:191), else x
//   qkv = bf16(x' W^T)                              `_linear(x, to_qkv)`: fp32 accumulation, one bf16 rounding
//   out = qkv                                       (prepare = 0), or (prepare = 1) with the q, k, q_diff, k_diff
//         columns of every head DyT'd (q_norm / k_norm) and rotated (half-half RoPE, angles fp32(position) *
//         inv_freq) in fp32 and rounded to bf16 once; v as is.
//
// The prepared columns use exactly the arithmetic the fused band kernel applies to raw tiles in shared memory
// (tanh.approx, the FMA order, `sincos_reduced`), so the band kernel reading them with its preparation stage
// skipped (hb_band_diff_attn_prepared) gives the output bit for bit of hb_band_diff_attn on the raw qkv.
//
// Layout: x [M, K] (M = batch * rows, 64 <= K <= 512, K % 64 == 0), W [N, K] (N = 5 H 64, the checkpoint's
// [out, in]), out [M, N]; bf16 row-major with row strides ldx, ldw, ldo.
//
// CTA pairs (clusters of two on neighbouring SMs, tcgen05 cta_group::2), one M256 N256 K16 pair MMA stream per
// pair. A unit is (256-row tile of x, group of 256-column tiles of W); CTA r of the pair owns rows
// [128 r, 128 r + 128) of the unit's x tile. That x tile lives in TMEM (the MMA's A operand: lane = row, 32-bit
// column i = bf16 pair of K elements 2i, 2i + 1; 256 columns for K = 512) for all the unit's column tiles, next
// to one 256-column fp32 accumulator, so only W streams through shared memory: CTA r loads W rows
// [128 r, 128 r + 128) of each 256 x 64 box into a 9-stage ring (144 KiB in flight per SM covers the L2 latency),
// and each stage is four MMAs (512 cycles), which hide the stage commits. The last column tile may reach past N:
// W rows there load as zeros and their head blocks are not stored. Units go to clusters round-robin, the column
// groups of one 256-row tile next to each other (its x tile is read from DRAM once, then from L2).
// x reaches TMEM through a two-slot shared-memory staging ring: the DyT warps read a landed 128 x 64 chunk (their
// rows), free the slot, apply the block DyT in registers, wait until the unit before has finished its MMAs on
// that chunk, and store it to TMEM with tcgen05.st; the next unit's DyT thus runs while the current unit's last
// tiles are multiplied, at about the MMA's pace.
// Roles (512 threads per CTA, registers rebalanced with setmaxnreg): warp 0 W producer; warp 1 TMEM allocation
// (both CTAs) and, in the even CTA, the pair MMA thread; warp 2 x producer; warp 3 idle; warps 4-7 the DyT warps
// (one TMEM lane quadrant each, one row per thread); warps 8-15 the epilogue of the CTA's 128 rows, one row per
// thread: warp w reads TMEM lane quadrant w % 4 and columns [128 g, 128 g + 128) (g = (w - 8) / 4) as packed
// bf16, releases the accumulator, then per 64-column head block: DyT / RoPE -> its group's swizzled staging box
// -> one TMA store. Barriers the MMA thread waits on live in the even CTA (x chunk in TMEM: the DyT warps of both
// CTAs; W stage full: both CTAs' TMA bytes; accumulator free: the epilogue warps of both CTAs); the MMA thread
// commits stage-free, chunk-free and accumulator-full to the barriers of both CTAs. No TMA load uses multicast.
//
// This file is compiled without relocatable device code (whole-program; see build.py): with -rdc ptxas ignores
// setmaxnreg. Its kernel records errors in its own status word (band_proj_take_status).
#define HB_WHOLE_PROGRAM 1
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "attn_internal.h"
#include "band_proj.h"
#include "hb_sm100.cuh"
#include "prep_common.cuh"

namespace hb {
namespace {

constexpr int kThreads = 512;
// Launched with 128 registers per thread; the control warpgroup gives up to 56, the DyT warpgroup to 120, the two
// epilogue warpgroups take 168: 56 + 120 + 2 * 168 = 4 * 128.
constexpr int kLaunchRegs = 128, kRegsCtl = 56, kRegsDyt = 120, kRegsEpi = 168;
static_assert(kRegsCtl + kRegsDyt + 2 * kRegsEpi == 4 * kLaunchRegs, "register split must equal the launch allocation");
constexpr int kEpiWarps = 8;                 // per CTA
constexpr int kBM = 128, kBN = 256;          // rows per CTA, columns per tile
constexpr int kChunkK = 64;                  // bf16 elements in one 128-byte swizzle row
constexpr int kMaxK = 512;
constexpr int kBoxBytes = kBM * 128;         // 128 x 64 bf16: an x chunk, an output staging box
constexpr int kWRows = kBN / 2;              // this CTA's half of a W box
constexpr int kWBytes = kWRows * 128;
constexpr int kStages = 9;
constexpr int kXSlots = 2;
constexpr uint32_t kColAcc = 0, kColX = 256;  // TMEM columns: accumulator [0, 256), x [256, 256 + K / 2)
constexpr int kNormStride = 132;             // alpha at [3], gamma at [4, 68), beta at [68, 132)
constexpr int kOffW = 0;
constexpr int kOffX = kOffW + kStages * kWBytes;
constexpr int kOffOut = kOffX + kXSlots * kBoxBytes;
constexpr int kOffPre = kOffOut + 2 * kBoxBytes;  // block pre-norm gamma[K], beta[K]
constexpr int kOffNorm = kOffPre + 2 * kMaxK * 4;
constexpr int kOffFreq = kOffNorm + 2 * kNormStride * 4;
constexpr int kOffBars = kOffFreq + 32 * 4;
constexpr int kNumBars = 2 * kStages + 2 * kXSlots + 2 * (kMaxK / kChunkK) + 3;
constexpr int kSmemBytes = kOffBars + kNumBars * 8 + 16 + 1024;
static_assert(kSmemBytes <= 232448, "shared memory per block");

struct ProjParams {
  int M, N, K;
  int rows;      // rows per batch element: the RoPE position of row m is pos0 + m % rows
  int64_t pos0;
  int sec;       // columns per section (H * 64)
  int half;
  int prepare;
  int has_pre;
  const float* pre_norm;  // [1 + 2K]: alpha, gamma[K], beta[K]
  const float* q_norm;    // [129]: alpha, gamma[64], beta[64]
  const float* k_norm;
  const float* inv_freq;  // [half]
  int num_m, groups, tiles_per_group, units;  // num_m: 256-row tiles; unit u: tile u / groups, group u % groups
};

template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// AND of `v` over the `count` threads that meet at named barrier `id` (the threads of an epilogue group decide
// together, so none of them is left waiting at a later barrier).
__device__ __forceinline__ bool bar_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r) : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(count) : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Rotate dims d < HALF with d + HALF (half-half RoPE) in the fused band kernel's order: y_d cos - y_{d+half} sin,
// y_{d+half} cos + y_d sin, products rounded, then one FMA each.
template <int HALF>
__device__ __forceinline__ void rope_head(float (&v)[64], float pos, const float* freqs) {
#pragma unroll
  for (int d = 0; d < HALF; ++d) {
    float sn, cs;
    sincos_reduced(__fmul_rn(pos, freqs[d]), sn, cs);
    const float y0 = v[d], y1 = v[d + HALF];
    v[d] = __fmaf_rn(y1, -sn, __fmul_rn(y0, cs));
    v[d + HALF] = __fmaf_rn(y0, sn, __fmul_rn(y1, cs));
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    band_proj_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_out, const ProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* w_full = bars;                        // [stage] (even CTA) TMA bytes of both halves of a W box
  uint64_t* w_empty = w_full + kStages;           // [stage] pair commit after the four MMAs on the box
  uint64_t* x_raw = w_empty + kStages;            // [slot] TMA bytes of a raw x chunk
  uint64_t* x_free = x_raw + kXSlots;             // [slot] 4 DyT warps: the chunk is in registers
  uint64_t* x_full = x_free + kXSlots;            // [chunk] (even CTA) 8 DyT warps of the pair: chunk in TMEM
  uint64_t* x_empty = x_full + kMaxK / kChunkK;   // [chunk] pair commit after the unit's last MMA on the chunk
  uint64_t* acc_full = x_empty + kMaxK / kChunkK;  // pair commit after a tile's last MMA
  uint64_t* acc_empty = acc_full + 1;             // (even CTA) 16 epilogue warps of the pair: accumulator read
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* pre = reinterpret_cast<float*>(smem + kOffPre);
  float* norms = reinterpret_cast<float*>(smem + kOffNorm);
  float* freqs = reinterpret_cast<float*>(smem + kOffFreq);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const int nkc = p.K / kChunkK;
  const int tpg = p.tiles_per_group;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int s = 0; s < kXSlots; ++s) {
      mbar_init(&x_raw[s], 1);
      mbar_init(&x_free[s], 4);
    }
    for (int c = 0; c < kMaxK / kChunkK; ++c) {
      mbar_init(&x_full[c], 8);
      mbar_init(&x_empty[c], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * kEpiWarps);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_out);
  }
  for (int i = threadIdx.x; i < 2 * kNormStride; i += kThreads) {
    const int which = i / kNormStride, k = i - which * kNormStride;
    norms[i] = (p.prepare && k >= 3) ? (which ? p.k_norm : p.q_norm)[k - 3] : 0.f;
  }
  if (threadIdx.x < 32) freqs[threadIdx.x] = (p.prepare && threadIdx.x < p.half) ? p.inv_freq[threadIdx.x] : 0.f;
  for (int i = threadIdx.x; i < 2 * p.K; i += kThreads) pre[i] = p.has_pre ? p.pre_norm[1 + i] : 0.f;
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    regs_dec<kRegsCtl>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------------- W producer (both CTAs)
      int w_issued = 0;
      bool ok = true;
      for (int u = cluster; ok && u < p.units; u += clusters) {
        const int g = u % p.groups;
        for (int t = 0; ok && t < tpg; ++t) {
          const int n0 = (g * tpg + t) * kBN + static_cast<int>(rank) * kWRows;
          for (int c = 0; c < nkc; ++c) {
            const int st = w_issued % kStages;
            if (w_issued >= kStages && !mbar_wait_sleep(&w_empty[st], ((w_issued / kStages) & 1) ^ 1, 100)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&w_full[st], 2 * kWBytes);
            tma_load_2d_pair(smem + kOffW + st * kWBytes, &tmap_w, c * kChunkK, n0,
                             cluster_addr(smem_u32(&w_full[st]), 0));
            ++w_issued;
          }
        }
      }
      if (!ok) *abort_flag = 1;
      // drain (bounded waits): in the even CTA the last stages of both CTAs have landed (the pair's final cluster
      // barrier holds the odd CTA until then)
      if (rank == 0)
        for (int i = max(0, w_issued - kStages); i < w_issued; ++i) mbar_wait(&w_full[i % kStages], (i / kStages) & 1);
    } else if (warp == 2 && lane == 0) {
      // ---------------------------------------------------------------- x producer (both CTAs): raw chunks
      int q = 0;
      bool ok = true;
      for (int u = cluster; ok && u < p.units; u += clusters) {
        const int m0 = (u / p.groups) * 2 * kBM + static_cast<int>(rank) * kBM;
        for (int c = 0; c < nkc; ++c, ++q) {
          const int slot = q % kXSlots;
          if (q >= kXSlots && !mbar_wait_sleep(&x_free[slot], ((q / kXSlots) & 1) ^ 1, 100)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_raw[slot], kBoxBytes);
          tma_load_2d(smem + kOffX + slot * kBoxBytes, &tmap_x, c * kChunkK, m0, &x_raw[slot]);
        }
      }
      if (!ok) *abort_flag = 1;
      for (int i = max(0, q - kXSlots); i < q; ++i) mbar_wait(&x_raw[i % kXSlots], (i / kXSlots) & 1);
    } else if (warp == 1 && lane == 0 && rank == 0) {
      // ---------------------------------------------------------------- pair MMA issuer (even CTA)
      constexpr uint32_t idesc = idesc_bf16_f32(2 * kBM, kBN, false);
      bool ok = true;
      int it = 0, tl = 0;
      for (int u = cluster, j = 0; ok && u < p.units; u += clusters, ++j) {
        for (int t = 0; ok && t < tpg; ++t, ++tl) {
          if (tl > 0 && !mbar_wait_cluster(acc_empty, (tl - 1) & 1)) {  // both epilogues have read the last tile
            ok = false;
            break;
          }
          tc_fence_after();
          for (int c = 0; c < nkc; ++c, ++it) {
            if (t == 0 && (!mbar_wait_cluster(&x_full[c], j & 1) || *abort_flag)) {
              ok = false;
              break;
            }
            const int st = it % kStages;
            if (!mbar_wait(&w_full[st], (it / kStages) & 1) || *abort_flag) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sb = smem_u32(smem + kOffW + st * kWBytes);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16_ts_pair(tmem + kColAcc, tmem + kColX + 32 * c + 8 * k, smem_desc_sw128(sb + 32 * k), idesc,
                               (c > 0 || k > 0));
            const uint32_t eb = smem_u32(&w_empty[st]);
            tc_commit_pair(cluster_addr(eb, 0));
            tc_commit_pair(cluster_addr(eb, 1));
            if (t == tpg - 1) {
              const uint32_t xb = smem_u32(&x_empty[c]);
              tc_commit_pair(cluster_addr(xb, 0));
              tc_commit_pair(cluster_addr(xb, 1));
            }
          }
          if (ok) {
            const uint32_t fb = smem_u32(acc_full);
            tc_commit_pair(cluster_addr(fb, 0));
            tc_commit_pair(cluster_addr(fb, 1));
          }
        }
      }
      if (!ok) *abort_flag = 1;
      tc_commit_pair(cluster_addr(smem_u32(drain), 0));
      mbar_wait(drain, 0);
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- DyT warps: raw x chunk -> TMEM
    regs_dec<kRegsDyt>();
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const float alpha = p.has_pre ? p.pre_norm[0] : 0.f;
    const uint32_t x_full0 = cluster_addr(smem_u32(x_full), 0);
    bool ok = true;
    int q = 0;
    for (int u = cluster, j = 0; ok && u < p.units; u += clusters, ++j) {
      for (int c = 0; c < nkc; ++c, ++q) {
        const int slot = q % kXSlots;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_sleep(&x_raw[slot], (q / kXSlots) & 1, 100) && !*abort_flag)))
          break;
        const uint8_t* buf = smem + kOffX + slot * kBoxBytes;
        uint32_t pk[32];  // the row's 64 elements of this chunk as bf16 pairs
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // two halves of 32 elements
          uint4 xr[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) xr[i] = *reinterpret_cast<const uint4*>(buf + sw128_offset(r, 4 * h + i));
          if (h == 1) {  // the whole row of the chunk is in registers: the producer may reload the slot
            __syncwarp();
            if (lane == 0) mbar_arrive(&x_free[slot]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t wv[4] = {xr[i].x, xr[i].y, xr[i].z, xr[i].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (p.has_pre) {
                const int col = c * kChunkK + 32 * h + 8 * i + 2 * e;
                const float y0 = __fmaf_rn(tanh_approx(__fmul_rn(alpha, bf16_lo(wv[e]))), pre[col], pre[p.K + col]);
                const float y1 =
                    __fmaf_rn(tanh_approx(__fmul_rn(alpha, bf16_hi(wv[e]))), pre[col + 1], pre[p.K + col + 1]);
                pk[16 * h + 4 * i + e] = pack_bf16x2(y0, y1);
              } else {
                pk[16 * h + 4 * i + e] = wv[e];
              }
            }
          }
        }
        // the unit before has finished its MMAs on this chunk of TMEM
        if (j > 0 && !(ok = __all_sync(0xffffffffu, mbar_wait_sleep(&x_empty[c], (j - 1) & 1, 100)))) break;
        tc_fence_after();
        tmem_st32(tmem + lane_base + kColX + 32 * c, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(x_full0 + 8u * c);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 8-15 of both CTAs)
    regs_inc<kRegsEpi>();
    const int quad = warp & 3;
    const int grp = (warp - 8) >> 2;               // columns [128 grp, 128 grp + 128): head blocks 2 grp, 2 grp + 1
    const int r = quad * 32 + lane;
    const int et = threadIdx.x - 256 - 128 * grp;  // 0..127 within the group
    const int bar_id = 1 + grp;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* stage = smem + kOffOut + grp * kBoxBytes;
    const uint32_t acc_empty0 = cluster_addr(smem_u32(acc_empty), 0);
    int tl = 0;
    bool ok = true;
    for (int u = cluster; ok && u < p.units; u += clusters) {
      const int m0 = (u / p.groups) * 2 * kBM + static_cast<int>(rank) * kBM, g = u % p.groups;
      const int m = m0 + r;
      const float pos = static_cast<float>(p.pos0 + (m % p.rows));
      for (int t = 0; t < tpg; ++t, ++tl) {
        // the MMA waits for this release, so the accumulator is polled without sleeping
        if (!(ok = bar_and(bar_id, 128, mbar_wait(acc_full, tl & 1)))) break;
        tc_fence_after();
        const int n0 = (g * tpg + t) * kBN;
        // the group's 128 columns as bf16 pairs (the projection's output rounding), two loads in flight per wait,
        // then release the accumulator
        uint32_t pk[64];
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          uint32_t a[32], b[32];
          tmem_ld32(tmem + lane_base + kColAcc + 128 * grp + 64 * q2, a);
          tmem_ld32(tmem + lane_base + kColAcc + 128 * grp + 64 * q2 + 32, b);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            pk[32 * q2 + i] = pack_bf16x2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
            pk[32 * q2 + 16 + i] = pack_bf16x2(__uint_as_float(b[2 * i]), __uint_as_float(b[2 * i + 1]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty0);
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {
          const int n = n0 + 128 * grp + 64 * h2, s = n / p.sec;
          if (n >= p.N) continue;  // past the last column (the last tile may reach beyond N): nothing to store
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = h2 ? pk[32 + i] : pk[i];
          if (p.prepare && s != 2) {  // q, k, q_diff, k_diff: DyT then RoPE in fp32, one bf16 rounding
            const float* nrm = norms + ((s == 1 || s == 4) ? kNormStride : 0);
            const float alpha = nrm[3];
            float v[64];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v[2 * i] = bf16_lo(w[i]);
              v[2 * i + 1] = bf16_hi(w[i]);
            }
#pragma unroll
            for (int d = 0; d < 64; ++d) v[d] = __fmaf_rn(tanh_approx(__fmul_rn(v[d], alpha)), nrm[4 + d], nrm[68 + d]);
            switch (p.half) {
              case 8: rope_head<8>(v, pos, freqs); break;
              case 16: rope_head<16>(v, pos, freqs); break;
              case 24: rope_head<24>(v, pos, freqs); break;
              default: rope_head<32>(v, pos, freqs); break;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
          }
          // the previous TMA store has read the staging box before it is overwritten
          if (et == 0) bulk_wait_group_read0();
          bar_sync(bar_id, 128);
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(stage + sw128_offset(r, ch)) =
                make_uint4(w[4 * ch], w[4 * ch + 1], w[4 * ch + 2], w[4 * ch + 3]);
          fence_proxy_async_smem();
          bar_sync(bar_id, 128);
          if (et == 0 && m0 < p.M) {  // rows past M are clipped by the tensor map
            tma_store_2d(&tmap_out, n, m0, stage);
            bulk_commit_group();
          }
        }
      }
    }
    if (et == 0) bulk_wait_group0();  // stores complete before the CTA's shared memory goes away
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers or read its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// bf16 [rows, cols] with row stride ld (elements), boxes of box_rows rows x 64 columns, 128-byte swizzle.
bool encode_box(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* base, int64_t cols,
                int64_t rows, int64_t ld, uint32_t box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Groups of column tiles per 256-row tile: the choice with the fewest tile-times over the CTA pairs, counting
// `overhead` tile-times per unit for its x chunks (and their DyT, which cannot start before the previous unit's
// last tile has released the chunks).
int choose_groups(int num_m, int ntn, int pairs, double overhead) {
  int best = 1;
  double best_cost = 1e30;
  for (int g = 1; g <= ntn; ++g) {
    if (ntn % g) continue;
    const long long units = (long long)num_m * g;
    const double cost = (double)((units + pairs - 1) / pairs) * (ntn / g + overhead);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = g;
    }
  }
  return best;
}

}  // namespace

int band_proj_take_status(unsigned int* status) {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status_local, sizeof(v)) != cudaSuccess) return HB_ERR_LAUNCH;
  if (v && cudaMemcpyToSymbol(g_device_status_local, &zero, sizeof(zero)) != cudaSuccess) return HB_ERR_LAUNCH;
  *status = v;
  return HB_OK;
}

}  // namespace hb

using namespace hb;

extern "C" int hb_band_qkv_project(const void* x, int64_t ldx, const float* pre_norm, const void* w, int64_t ldw,
                                   const float* q_norm, const float* k_norm, const float* inv_freq, int half,
                                   void* out, int64_t ldo, int batch, int rows, int64_t pos0, int d_model,
                                   int num_heads, int head_dim, int prepare, cudaStream_t stream) {
  if (!x || !w || !out) return HB_ERR_NULL;
  if (prepare && (!q_norm || !k_norm || !inv_freq)) return HB_ERR_NULL;
  if (head_dim != kHeadDim || num_heads < 2 || num_heads % 2 || batch < 1 || rows < 1) return HB_ERR_SHAPE;
  if (d_model < kChunkK || d_model > kMaxK || d_model % kChunkK) return HB_ERR_SHAPE;
  if (prepare && (half < 8 || half > 32 || half % 8)) return HB_ERR_SHAPE;
  if ((long long)batch * rows > 0x7fffffffLL || pos0 < 0 || pos0 + rows > (1 << 24)) return HB_ERR_SHAPE;
  const int N = kSections * num_heads * kHeadDim;
  if (ldx < d_model || ldw < d_model || ldo < N) return HB_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out) || ldx % 8 || ldw % 8 || ldo % 8) return HB_ERR_ALIGN;
  int st = check_device();
  if (st != HB_OK) return st;
  auto encode = encode_fn();
  if (!encode) return HB_ERR_LAUNCH;
  const int M = batch * rows;
  CUtensorMap tx, tw, to;
  if (!encode_box(encode, &tx, x, d_model, M, ldx, kBM) || !encode_box(encode, &tw, w, d_model, N, ldw, kWRows) ||
      !encode_box(encode, &to, out, N, M, ldo, kBM))
    return HB_ERR_LAUNCH;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    // The warpgroups' setmaxnreg split assumes the block is launched with exactly 128 registers per thread;
    // with any other count the register increase could never be granted, so refuse to launch.
    cudaFuncAttributes attr{};
    if (cudaFuncGetAttributes(&attr, band_proj_kernel) != cudaSuccess || attr.numRegs != kLaunchRegs)
      return HB_ERR_LAUNCH;
    if (cudaFuncSetAttribute(band_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  ProjParams p{};
  p.M = M;
  p.N = N;
  p.K = d_model;
  p.rows = rows;
  p.pos0 = pos0;
  p.sec = num_heads * kHeadDim;
  p.half = half;
  p.prepare = prepare ? 1 : 0;
  p.has_pre = pre_norm ? 1 : 0;
  p.pre_norm = pre_norm;
  p.q_norm = q_norm;
  p.k_norm = k_norm;
  p.inv_freq = inv_freq;
  p.num_m = (M + 2 * kBM - 1) / (2 * kBM);
  const int ntn = (N + kBN - 1) / kBN;
  const int pairs = sms / 2;
  const int groups = choose_groups(p.num_m, ntn, pairs, 0.5);
  p.groups = groups;
  p.tiles_per_group = ntn / groups;
  p.units = p.num_m * groups;
  const int clusters = p.units < pairs ? p.units : pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, band_proj_kernel, tx, tw, to, p) != cudaSuccess) return HB_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

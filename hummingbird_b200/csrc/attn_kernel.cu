// tcgen05 differential-attention kernel over prepared tiles, used for SAME-L band attention with windows
// wider than the fused band kernel handles (window > 128). It accepts the dense mode too (window < 0); the
// dense path runs attn_dense.cu.
//
// One CTA computes one 128-query tile of one head for BOTH differential branches:
//   A = softmax(Q  K^T  / 8) V,   B = softmax(Qd Kd^T / 8) V,   out = A - lambda * B   (fp32, one bf16 cast)
// which is the reference's per-tile body (dense_attention.py:79-94, band_attention.py:96-120) with an
// online softmax over 128-key tiles instead of whole-L scores.
//
// Roles (12 warps):
//   warp 0      producer: 1-D bulk copies (TMA engine) of the prepared Q/Qd tiles once and of K/Kd/V
//               tiles through a 3-stage ring, completion counted on mbarriers.
//   warp 1      allocates 512 TMEM columns; one thread issues every tcgen05.mma:
//                 S_X = Q_X K_X^T  (M128 N128 K16 x4, both operands K-major SW128 smem)
//                 O_X += P_X V     (M128 N64 K16 x8, P from TMEM, V MN-major SW128 smem)
//   warps 4-7   softmax of branch A, warps 8-11 softmax of branch B: one thread per query row reads its
//               128 scores with tcgen05.ld, keeps the running max / sum in fp32, writes bf16 P back into
//               the S columns with tcgen05.st and rescales its O row in TMEM when the max moves by > 2^8.
// TMEM columns: S_A [0,128) (P_A aliases [0,64)), S_B [128,256), O_A [256,320), O_B [320,384).
//
// MMAs from one thread complete in issue order, so "S_X(j) done" implies "PV_X(j-1) done": the softmax
// of tile j may rescale O_X as soon as it sees S_X(j). The MMA thread interleaves the branches
// (S_A(j), PV_B(j-1), S_B(j), PV_A(j)) so each softmax group overlaps the other branch's MMAs.
#include "attn_internal.h"
#include "hb_sm100.cuh"

namespace hb {

__device__ unsigned int g_device_status = 0;

namespace {

constexpr int kStages = 3;
constexpr int kThreads = 384;
constexpr int kOffQa = 0;
constexpr int kOffQb = kTileBytes;
constexpr int kOffStage = 2 * kTileBytes;
constexpr int kStageBytes = 3 * kTileBytes;  // K, Kd, V
constexpr int kOffBars = kOffStage + kStages * kStageBytes;
constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 1 + 1;
constexpr int kOffMisc = kOffBars + kNumBars * 8;
constexpr int kOffScaleB = kOffMisc + 16;
constexpr int kSmemBytes = kOffScaleB + kTileRows * 4 + 1024;  // + slack for 1024-B alignment
constexpr uint32_t kTmemCols = 512;
constexpr float kScoreScale = 1.4426950408889634f * 0.125f;  // log2(e) / sqrt(64)
constexpr float kRescaleThreshold = 8.0f;                     // log2 units

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) diff_attention_kernel(const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* bar_q = bars;
  uint64_t* bar_kv_full = bars + 1;
  uint64_t* bar_kv_empty = bars + 1 + kStages;
  uint64_t* bar_s = bars + 1 + 2 * kStages;  // [2]
  uint64_t* bar_p = bar_s + 2;                // [2]
  uint64_t* bar_o = bar_p + 2;
  uint64_t* bar_drain = bar_o + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* scale_b = reinterpret_cast<float*>(smem + kOffScaleB);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.q_begin / kTileRows + blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  int kt0 = 0, kt1 = p.ntiles - 1;
  if (p.window >= 0) {
    const int q_lo = qt * kTileRows, q_hi = min(qt * kTileRows + kTileRows - 1, p.rows - 1);
    kt0 = max(0, q_lo - p.window) / kTileRows;
    kt1 = min(p.ntiles - 1, (q_hi + p.window) / kTileRows);
  }
  const int nk = kt1 - kt0 + 1;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
    }
    mbar_init(&bar_s[0], 1);
    mbar_init(&bar_s[1], 1);
    mbar_init(&bar_p[0], 4);
    mbar_init(&bar_p[1], 4);
    mbar_init(bar_o, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint8_t* ws = p.ws;
      mbar_arrive_expect_tx(bar_q, 2 * kTileBytes);
      bulk_g2s(smem + kOffQa, ws + prep_tile_offset(b, h, 0, qt, p.heads, p.ntiles), kTileBytes, bar_q);
      bulk_g2s(smem + kOffQb, ws + prep_tile_offset(b, h, 3, qt, p.heads, p.ntiles), kTileBytes, bar_q);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int st = i % kStages;
        if (i >= kStages && !mbar_wait(&bar_kv_empty[st], ((i / kStages) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int kt = kt0 + i;
        uint8_t* stage = smem + kOffStage + st * kStageBytes;
        mbar_arrive_expect_tx(&bar_kv_full[st], 3 * kTileBytes);
        bulk_g2s(stage, ws + prep_tile_offset(b, h, 1, kt, p.heads, p.ntiles), kTileBytes, &bar_kv_full[st]);
        bulk_g2s(stage + kTileBytes, ws + prep_tile_offset(b, h, 4, kt, p.heads, p.ntiles), kTileBytes,
                 &bar_kv_full[st]);
        bulk_g2s(stage + 2 * kTileBytes, ws + prep_tile_offset(b, h, 2, kt, p.heads, p.ntiles), kTileBytes,
                 &bar_kv_full[st]);
        issued = i + 1;
      }
      // no copy into this CTA's shared memory may still be in flight when it exits
      mbar_wait(bar_q, 0);
      for (int i = max(0, issued - kStages); i < issued; ++i) mbar_wait(&bar_kv_full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idO = idesc_bf16_f32(128, 64, true);
      const uint32_t tSa = tmem, tSb = tmem + 128, tOa = tmem + 256, tOb = tmem + 320;
      const uint32_t qa = smem_u32(smem + kOffQa), qb = smem_u32(smem + kOffQb);
      bool ok = mbar_wait(bar_q, 0);
      tc_fence_after();
      for (int i = 0; ok && i < nk; ++i) {
        const int st = i % kStages;
        const uint32_t stage = smem_u32(smem + kOffStage + st * kStageBytes);
        if (!mbar_wait(&bar_kv_full[st], (i / kStages) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ss(tSa, smem_desc_sw128(qa + 32 * k), smem_desc_sw128(stage + 32 * k), idS, k > 0);
        tc_commit(&bar_s[0]);
        if (i > 0) {
          if (!mbar_wait(&bar_p[1], (i - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int pst = (i - 1) % kStages;
          const uint32_t vprev = smem_u32(smem + kOffStage + pst * kStageBytes + 2 * kTileBytes);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16_ts(tOb, tSb + 8 * k, smem_desc_sw128(vprev + 2048 * k), idO, (i > 1 || k > 0));
          tc_commit(&bar_kv_empty[pst]);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ss(tSb, smem_desc_sw128(qb + 32 * k), smem_desc_sw128(stage + kTileBytes + 32 * k), idS, k > 0);
        tc_commit(&bar_s[1]);
        if (!mbar_wait(&bar_p[0], i & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vcur = stage + 2 * kTileBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tOa, tSa + 8 * k, smem_desc_sw128(vcur + 2048 * k), idO, (i > 0 || k > 0));
      }
      if (ok) {
        const int i = nk - 1;
        if (mbar_wait(&bar_p[1], i & 1)) {
          tc_fence_after();
          const int pst = i % kStages;
          const uint32_t vlast = smem_u32(smem + kOffStage + pst * kStageBytes + 2 * kTileBytes);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16_ts(tOb, tSb + 8 * k, smem_desc_sw128(vlast + 2048 * k), idO, (i > 0 || k > 0));
          tc_commit(&bar_kv_empty[pst]);
          tc_commit(bar_o);
        } else {
          ok = false;
        }
      }
      if (!ok) *abort_flag = 1;
      tc_commit(bar_drain);  // every MMA this thread issued has finished before TMEM is freed
      mbar_wait(bar_drain, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax (one query row per thread)
    const int br = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + (br ? 128u : 0u);
    const uint32_t tO = tmem + lane_base + (br ? 320u : 256u);
    const int q = qt * kTileRows + row;
    const int q_lo_w = qt * kTileRows + quad * 32, q_hi_w = q_lo_w + 31;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_s[br], i & 1) && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      const int k0 = (kt0 + i) * kTileRows;
      // raw fp32 scores of this row's 128 keys: four loads in flight, one wait
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, r[c]);
      tmem_wait_ld();
      bool full = (k0 + kTileRows - 1) < p.rows;
      if (p.window >= 0) full = full && (k0 >= q_hi_w - p.window) && (k0 + kTileRows - 1 <= q_lo_w + p.window);
      if (!full) {
#pragma unroll
        for (int j = 0; j < 128; ++j) {
          const int k = k0 + j;
          const bool in = k < p.rows && (p.window < 0 || abs(k - q) <= p.window);
          if (!in) r[j >> 5][j & 31] = 0xff800000u;  // -inf
        }
      }
      // row max of the raw scores: four independent chains of three-input maxima (scale > 0 commutes)
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < 128; j += 8) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mx[u] = fmax3(mx[u], __uint_as_float(r[j >> 5][(j & 31) + 2 * u]),
                        __uint_as_float(r[j >> 5][(j & 31) + 2 * u + 1]));
      }
      const float rmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), mx[3]) * kScoreScale;
      const float m_new = fmaxf(m, rmax);
      const bool upd = m_new > m + kRescaleThreshold;
      float alpha = 1.f;
      if (upd) {
        alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - m_new);
        m = m_new;
      }
      const float nm = (m == -INFINITY) ? 0.f : -m;
      // P = exp2(s * scale - m): packed FMA per key pair, bf16 pairs into the first 64 columns of S;
      // the row sum in two packed accumulators (four partial sums)
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int e = 64 * c + 2 * j;
          float x0, x1;
          ffma2(x0, x1, __uint_as_float(r[e >> 5][e & 31]), __uint_as_float(r[e >> 5][(e & 31) + 1]), kScoreScale,
                kScoreScale, nm, nm);
          float p0, p1;
          if ((j & kPolyMask) == kPolyMask) {  // a share of the exponentials on the FMA pipe
            exp2_poly2(x0, x1, p0, p1);
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          const int a = (j & 1) * 2;
          fadd2(rs[a], rs[a + 1], rs[a], rs[a + 1], p0, p1);
          pk[j] = pack_bf16x2(p0, p1);
        }
        tmem_st32(tS + 32 * c, pk);
      }
      const float rsum = (rs[0] + rs[1]) + (rs[2] + rs[3]);
      l = l * alpha + rsum;
      if (i > 0 && __any_sync(0xffffffffu, upd)) {
        uint32_t o[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          tmem_st32(tO + 32 * c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p[br]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_o, 0));
    tc_fence_after();
    const float lam = p.lam ? p.lam[p.lam_pair0 + h / 2] : 1.f;
    if (br == 1) scale_b[row] = lam / l;
    named_bar_sync(1, 256);
    if (br == 0 && ok) {
      const float inv_a = 1.f / l;
      const float sb = scale_b[row];
      const bool store = q >= p.q_begin && q < p.q_begin + p.q_count;
      uint16_t* dst = p.out + ((size_t)b * p.q_count + (q - p.q_begin)) * p.out_row_stride + (size_t)h * kHeadDim;
      const uint32_t tOb = tmem + lane_base + 320u;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t oa[32], ob[32];
        tmem_ld32(tO + 32 * c, oa);
        tmem_ld32(tOb + 32 * c, ob);
        tmem_wait_ld();
        if (store) {
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // each branch normalised and rounded on its own, then one fp32 subtraction (no contraction)
            const float y0 = __fmul_rn(__uint_as_float(oa[2 * j]), inv_a) - __fmul_rn(__uint_as_float(ob[2 * j]), sb);
            const float y1 =
                __fmul_rn(__uint_as_float(oa[2 * j + 1]), inv_a) - __fmul_rn(__uint_as_float(ob[2 * j + 1]), sb);
            w[j] = pack_bf16x2(y0, y1);
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int launch_diff_attention(const AttnParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    e = cudaFuncSetAttribute(diff_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int qt_first = p.q_begin / kTileRows;
  const int qt_last = (p.q_begin + p.q_count - 1) / kTileRows;
  dim3 grid(qt_last - qt_first + 1, p.heads, p.B);
  diff_attention_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace hb

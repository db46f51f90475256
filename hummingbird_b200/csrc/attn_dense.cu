// Dense differential attention with the softmax probabilities in their own TMEM columns (the DiT
// self-attention, dense_attention.py:79-94: every key, no key mask).
//
// One CTA computes one 128-query tile of one head for both branches:
//   A = softmax(Q K^T / 8) V,   B = softmax(Qd Kd^T / 8) V,   out = A - lambda * B   (fp32, one bf16 cast)
// with an online softmax over 128-key tiles. Each branch has a score buffer S, a probability buffer P and an
// accumulator O in TMEM. The softmax releases S as soon as it has loaded the tile's 128 scores into registers,
// so S of tile i + 1 is computed while the softmax of tile i runs, and the softmax warps go from one tile to
// the next without waiting for P V and the next Q K^T (the chain S -> softmax -> P V -> S that a shared
// S / P buffer imposes).
//
// Roles (12 warps):
//   warp 0      producer: 1-D bulk copies of the prepared Q / Qd tiles once and of the K / Kd / V tiles
//               through a kStages ring
//   warp 1      allocates 512 TMEM columns; one thread issues every tcgen05.mma:
//                 S_X(i) = Q_X K_X(i)^T   (M128 N128 K16 x4, both operands K-major SW128 in shared memory)
//                 O_X += P_X(i) V(i)      (M128 N64 K16 x8, P from TMEM, V MN-major SW128 in shared memory)
//               per tile i: S_A(i+1), S_B(i+1) (each once the softmax has loaded S_X(i)), then PV_A(i), PV_B(i)
//   warps 4-7   softmax of branch A, warps 8-11 of branch B: one query row per thread; the tile's scores
//               with four tcgen05.ld and one wait, then S is released; P goes to P_X once the previous
//               P V has read it; O is rescaled in TMEM when the running maximum moves by more than 2^8
//   then both groups run the epilogue, each on half of the 64 output columns of its rows.
// TMEM columns: S_A [0,128), S_B [128,256), P_A [256,320), P_B [320,384), O_A [384,448), O_B [448,512).
#include "attn_internal.h"
#include "hb_sm100.cuh"

namespace hb {
namespace {

constexpr int kStages = 3;
constexpr int kThreads = 384;
constexpr int kOffQa = 0;
constexpr int kOffQb = kTileBytes;
constexpr int kOffStage = 2 * kTileBytes;
constexpr int kStageBytes = 3 * kTileBytes;  // K, Kd, V
constexpr int kOffBars = kOffStage + kStages * kStageBytes;
constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 2 + 2 + 1;
constexpr int kOffMisc = kOffBars + kNumBars * 8;
constexpr int kOffScale = kOffMisc + 16;  // [2][128]: 1 / l_A, lambda / l_B
constexpr int kSmemBytes = kOffScale + 2 * kTileRows * 4 + 1024;  // + slack for 1024-B alignment
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;
constexpr float kScoreScale = 1.4426950408889634f * 0.125f;  // log2(e) / sqrt(64)
constexpr float kRescaleThreshold = 8.0f;                     // log2 units
// Polls of the producer (it runs stages ahead) and of the softmax sleep between tries, so waiting warps leave
// issue slots to the working ones (measured: 0.2529 -> 0.2468 ms per 120 s block call); the MMA thread polls.
constexpr unsigned kSlackSleepNs = 200, kSoftSleepNs = 100;

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) dense_attention_kernel(const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* bar_q = bars;
  uint64_t* kv_full = bars + 1;                // [kStages]
  uint64_t* kv_empty = bars + 1 + kStages;     // [kStages]
  uint64_t* s_full = bars + 1 + 2 * kStages;   // [branch] commit
  uint64_t* s_free = s_full + 2;               // [branch] 4 softmax warps (scores loaded)
  uint64_t* p_ready = s_free + 2;              // [branch] 4 softmax warps
  uint64_t* o_done = p_ready + 2;              // [branch] commit after each P V of the branch
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* scale = reinterpret_cast<float*>(smem + kOffScale);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int nk = p.ntiles;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 4);
      mbar_init(&p_ready[x], 4);
      mbar_init(&o_done[x], 1);
    }
    mbar_init(drain, 1);
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
        if (i >= kStages && !mbar_wait_sleep(&kv_empty[st], ((i / kStages) & 1) ^ 1, kSlackSleepNs)) {
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        uint8_t* stage = smem + kOffStage + st * kStageBytes;
        mbar_arrive_expect_tx(&kv_full[st], 3 * kTileBytes);
        bulk_g2s(stage, ws + prep_tile_offset(b, h, 1, i, p.heads, p.ntiles), kTileBytes, &kv_full[st]);
        bulk_g2s(stage + kTileBytes, ws + prep_tile_offset(b, h, 4, i, p.heads, p.ntiles), kTileBytes, &kv_full[st]);
        bulk_g2s(stage + 2 * kTileBytes, ws + prep_tile_offset(b, h, 2, i, p.heads, p.ntiles), kTileBytes,
                 &kv_full[st]);
        issued = i + 1;
      }
      // no copy into this CTA's shared memory may still be in flight when it exits
      mbar_wait(bar_q, 0);
      for (int i = max(0, issued - kStages); i < issued; ++i) mbar_wait(&kv_full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idO = idesc_bf16_f32(128, 64, true);
      const uint32_t qa = smem_u32(smem + kOffQa), qb = smem_u32(smem + kOffQb);
      auto stage_addr = [&](int i) { return smem_u32(smem + kOffStage + (i % kStages) * kStageBytes); };
      // S_X(i) (X = 0: Q K^T, X = 1: Qd Kd^T); branch 0 first, so it waits for the tile's copies
      auto issue_s = [&](int x, int i) -> bool {
        if (x == 0 && (!mbar_wait(&kv_full[i % kStages], (i / kStages) & 1) || *abort_flag)) return false;
        if (i > 0 && !mbar_wait(&s_free[x], (i - 1) & 1)) return false;  // the softmax has loaded S_X(i - 1)
        tc_fence_after();
        const uint32_t kb = stage_addr(i) + (x ? kTileBytes : 0);
        const uint32_t qx = x ? qb : qa;
        const uint32_t tS = tmem + kColS + 128u * x;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ss(tS, smem_desc_sw128(qx + 32 * k), smem_desc_sw128(kb + 32 * k), idS, k > 0);
        tc_commit(&s_full[x]);
        return true;
      };
      auto issue_pv = [&](int x, int i) -> bool {
        if (!mbar_wait(&p_ready[x], i & 1)) return false;
        tc_fence_after();
        const uint32_t vb = stage_addr(i) + 2 * kTileBytes;
        const uint32_t tP = tmem + kColP + 64u * x;
        const uint32_t tO = tmem + kColO + 64u * x;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tO, tP + 8 * k, smem_desc_sw128(vb + 2048 * k), idO, (i > 0 || k > 0));
        tc_commit(&o_done[x]);
        return true;
      };
      bool ok = mbar_wait(bar_q, 0) && !*abort_flag;
      tc_fence_after();
      if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
      for (int i = 0; ok && i < nk; ++i) {
        if (i + 1 < nk) ok = issue_s(0, i + 1) && issue_s(1, i + 1);
        if (ok) ok = issue_pv(0, i) && issue_pv(1, i);
        if (ok) tc_commit(&kv_empty[i % kStages]);  // every MMA reading tile i's stage precedes this commit
      }
      if (!ok) *abort_flag = 1;
      tc_commit(drain);  // every MMA this thread issued has finished before TMEM is freed
      mbar_wait(drain, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax (one query row per thread)
    const int br = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + kColS + 128u * br;
    const uint32_t tP = tmem + lane_base + kColP + 64u * br;
    const uint32_t tO = tmem + lane_base + kColO + 64u * br;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      ok = __all_sync(0xffffffffu, mbar_wait_sleep(&s_full[br], i & 1, kSoftSleepNs) && !*abort_flag);
      if (!ok) break;
      tc_fence_after();
      const int k0 = i * kTileRows;
      // the tile's 128 raw fp32 scores: four loads in flight, one wait; then S may be overwritten
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, r[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[br]);
      if (k0 + kTileRows > p.rows) {  // keys past the sequence are not attended
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (k0 + e >= p.rows) r[e >> 5][e & 31] = 0xff800000u;  // -inf
      }
      // row max: four chains of three-input maxima (the scale is positive, so it commutes with the max)
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 128; e += 8) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mx[u] = fmax3(mx[u], __uint_as_float(r[e >> 5][(e & 31) + 2 * u]),
                        __uint_as_float(r[e >> 5][(e & 31) + 2 * u + 1]));
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
      // P = exp2(s * scale - m) as bf16 pairs: packed FMA per key pair, the row sum in two packed accumulators
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk0[32], pk1[32];
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const int e = 2 * j;
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
        if (j < 32)
          pk0[j] = pack_bf16x2(p0, p1);
        else
          pk1[j - 32] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
      if (i > 0) {
        // the previous P V has read P and landed in O
        ok = __all_sync(0xffffffffu, mbar_wait_sleep(&o_done[br], (i - 1) & 1, kSoftSleepNs));
        if (!ok) break;
        tc_fence_after();
      }
      tmem_st32(tP, pk0);
      tmem_st32(tP + 32, pk1);
      if (i > 0 && __any_sync(0xffffffffu, upd)) {
        uint32_t o[32];
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + 32 * c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[br]);
    }
    // the last P V of this group's branch has completed (each group waits only on its own branch's barrier,
    // whose phases it has followed tile by tile); the barrier below hands both results to both groups
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&o_done[br], (nk - 1) & 1));
    scale[br * kTileRows + row] = (br ? (p.lam ? p.lam[p.lam_pair0 + h / 2] : 1.f) : 1.f) / l;
    tc_fence_before();
    named_bar_sync(1, 256);
    tc_fence_after();
    const int q = qt * kTileRows + row;
    if (ok) {  // warp-uniform: the TMEM loads are .sync.aligned; only the stores depend on the row
      const float inv_a = scale[row], sb = scale[kTileRows + row];
      const uint32_t tOa = tmem + lane_base + kColO, tOb = tOa + 64u;
      // branch A's warps write output columns [0, 32), branch B's [32, 64)
      uint32_t oa[32], ob[32];
      tmem_ld32(tOa + 32 * br, oa);
      tmem_ld32(tOb + 32 * br, ob);
      tmem_wait_ld();
      const bool store = q >= p.q_begin && q < p.q_begin + p.q_count;
      uint16_t* dst = p.out + ((size_t)b * p.q_count + (store ? q - p.q_begin : 0)) * p.out_row_stride +
                      (size_t)h * kHeadDim;
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // each branch normalised and rounded on its own, then one fp32 subtraction (no contraction)
        const float y0 = __fmul_rn(__uint_as_float(oa[2 * j]), inv_a) - __fmul_rn(__uint_as_float(ob[2 * j]), sb);
        const float y1 = __fmul_rn(__uint_as_float(oa[2 * j + 1]), inv_a) - __fmul_rn(__uint_as_float(ob[2 * j + 1]), sb);
        w[j] = pack_bf16x2(y0, y1);
      }
      if (store) {
        uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * br);
#pragma unroll
        for (int j = 0; j < 4; ++j) d4[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
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

int launch_dense_attention(const AttnParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    e = cudaFuncSetAttribute(dense_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int qt_first = p.q_begin / kTileRows;
  const int qt_last = (p.q_begin + p.q_count - 1) / kTileRows;
  if (qt_first != 0 || p.window >= 0) return cudaErrorInvalidValue;  // dense only, every query row from row 0
  dim3 grid(qt_last + 1, p.heads, p.B);
  dense_attention_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace hb

// Fused differential cross-attention of the DiT (dit.py:203-215 through `_attend` / `_attend_out`,
// dit.py:131-176): for every 64-dim head,
//   A = softmax(rms(q) k^T / 8) v,   B = softmax(rms(q_diff) k_diff^T / 8) v,   out = A - lambda * B
// with q, q_diff the `to_q` output (dit.py:207-209) and k, k_diff, v the hoisted `to_kv` context keys
// (dit.py:274-284; at most 384 of them). No RoPE and no mask (dit.py:204-205). The q RMSNorm (and the k norm
// when the keys arrive raw) is applied in place in shared memory, so the `to_q` rows are read once and the
// merged `(B, Lq, H * 64)` output is written once.
//
// Work: the (batch, head, 128-row query tile) units, head-major, are split into contiguous runs, one run per
// CTA (grid = min(units, #SMs)). The K, K_diff, V tiles of one (batch, head) stay in shared memory for every
// query tile of the run that uses them.
//
// Roles (16 warps):
//   warp 0            3-D TMA (128B swizzle, rows past the end read as zero) of the raw q, q_diff tiles of each
//                     unit into a double buffer, and of the K, K_diff, V tiles at the start of each run
//   warp 1            TMEM allocation (512 columns) and the single MMA-issuing thread
//   warps 4-7         softmax of branch A, warps 8-11 softmax of branch B (one query row per thread); each
//                     hands its row's 1 / l (lambda / l for B) to the epilogue through shared memory
//   warps 2-3, 12-15  RMSNorm in place: x * rsqrt(mean(x^2) + eps) * w in fp32, then bf16 (dit.py:45-57), one
//                     unit ahead; warps 12-15 then run the epilogue of each unit: out = O_A / l_A - lambda O_B / l_B
//                     in fp32, bf16, staged in shared memory (SW128) and written by one TMA store per unit (full
//                     128-byte rows; rows past the end are not written)
// TMEM: S_A [0,128) (P_A in [0,64)), S_B [128,256), O_A/O_B double-buffered by unit parity at
// [256,320)/[320,384) and [384,448)/[448,512), so the epilogue of unit j overlaps unit j+1.
// MMA order per key tile i of a unit: S_A(i), PV_B(i-1), S_B(i), PV_A(i); PV_B of a unit's last key tile is
// issued after S_A of the next unit, or before the K/V of a new run are waited for.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "../../include/hb_b200.h"
#include "abi_common.h"
#include "attn_internal.h"
#include "hb_sm100.cuh"
#include "prep_common.cuh"

namespace hb {

#ifdef HB_TRACE
// Debug builds only (-DHB_TRACE): %clock cycles (since the CTA started) of pipeline events of CTA 0 and of the
// middle CTA, one slot per traced thread: producer, MMA issuer, softmax A, softmax B, RMSNorm.
__device__ unsigned int g_xtrace[2][5][512];
__device__ unsigned int g_xtrace_n[2][5];
#define XT(slot, id)                                                                                        \
  do {                                                                                                      \
    const int tc_ = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x / 2 ? 1 : -1);                            \
    if (tc_ >= 0 && xt_n < 256) {                                                                           \
      g_xtrace[tc_][slot][2 * xt_n] = (id);                                                                 \
      g_xtrace[tc_][slot][2 * xt_n + 1] = static_cast<unsigned>(clock64() - xt0);                          \
      g_xtrace_n[tc_][slot] = ++xt_n;                                                                       \
    }                                                                                                       \
  } while (0)
#else
#define XT(slot, id) \
  do {               \
  } while (0)
#endif

namespace {

constexpr int kThreads = 512;
constexpr int kPrepWarps = 6;  // warps 2, 3 and 12-15
constexpr int kPrepThreads = 32 * kPrepWarps;
constexpr int kMaxKvTiles = 3;                     // context length <= 384
constexpr int kKvTileBytes = 3 * kTileBytes;       // K, K_diff, V of one 128-key tile
constexpr int kQBytes = 2 * kTileBytes;            // Q, Q_diff
constexpr int kOffQ = kMaxKvTiles * kKvTileBytes;  // 144 KiB
constexpr int kOffStage = kOffQ + 2 * kQBytes;     // + 64 KiB: output staging tile (16 KiB)
constexpr int kOffBars = kOffStage + kTileBytes;
constexpr int kNumBars = 22;
constexpr int kOffMisc = kOffBars + kNumBars * 8;
constexpr int kOffW = kOffMisc + 16;               // q weight [64], k weight [64]
constexpr int kOffScale = kOffW + 128 * 4;  // [branch][row]: 1 / l_A and lambda / l_B of the unit in the epilogue
constexpr int kSmemBytes = kOffScale + 2 * kTileRows * 4 + 1024;  // + slack for 1024-B alignment
constexpr float kScoreScale = 1.4426950408889634f * 0.125f;         // log2(e) / sqrt(64)
constexpr float kRescaleThreshold = 8.0f;                            // log2 units
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct CrossParams {
  int B, Lq, Lkv, heads, nqt, nkt, units;
  const float* q_w;   // [64]
  const float* k_w;   // [64] or null (keys already normed)
  float eps;
  const float* lam;   // per pair (index h / 2), or null for 1
};

struct Unit {
  int b, h, qt;
};

__device__ __forceinline__ Unit decode(const CrossParams& p, int u) {
  Unit x;
  const int bh = u / p.nqt;
  x.qt = u - bh * p.nqt;
  x.b = bh / p.heads;
  x.h = bh - x.b * p.heads;
  return x;
}

__device__ __forceinline__ bool same_run(const Unit& a, const Unit& b) { return a.b == b.b && a.h == b.h; }

// Polls of the roles with slack (the TMA producer, the RMSNorm / epilogue warps) and of the softmax sleep between
// tries, so waiting warps leave issue slots to the working ones; the MMA thread polls without sleeping.
#ifndef HB_CROSS_SLACK_SLEEP_NS
#define HB_CROSS_SLACK_SLEEP_NS 200
#endif
#ifndef HB_CROSS_SOFT_SLEEP_NS
#define HB_CROSS_SOFT_SLEEP_NS 100
#endif
constexpr unsigned kSlackSleepNs = HB_CROSS_SLACK_SLEEP_NS, kSoftSleepNs = HB_CROSS_SOFT_SLEEP_NS;

__device__ __forceinline__ bool sleep_wait(uint64_t* bar, uint32_t parity, unsigned sleep_ns) {
  return sleep_ns ? mbar_wait_sleep(bar, parity, sleep_ns) : mbar_wait(bar, parity);
}
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned sleep_ns = kSlackSleepNs) {
  const bool ok = sleep_wait(bar, parity, sleep_ns) && !*abort_flag;
  return __all_sync(0xffffffffu, ok);
}

// RMSNorm of row `r` of two 128-row tiles in the SW128 image, in place, bf16 out (`dit._rms`, dit.py:45-57),
// for the two 16-byte chunks c0, c0 + 1 of the calling thread; four consecutive threads own a row and combine
// their sums of squares by shuffles (the caller keeps the calls warp-uniform). `rows` rows (1 or 2, at r and
// r + r2) are handled together, for independent chains.
template <int kRows>
__device__ __forceinline__ void rms_rows(uint8_t* buf0, uint8_t* buf1, int r, int r2, int c0, const float (&w0)[8],
                                         const float (&w1)[8], float eps) {
  constexpr int kChains = 2 * kRows;
  uint4* ptr[kChains][2];
  float x[kChains][16];
  float ss[kChains];
#pragma unroll
  for (int k = 0; k < kChains; ++k) {  // k: (row r or r2) x (tile 0 or 1)
    uint8_t* buf = (k & 1) ? buf1 : buf0;
    const int rr = (k >> 1) ? r2 : r;
    ptr[k][0] = reinterpret_cast<uint4*>(buf + sw128_offset(rr, c0));
    ptr[k][1] = reinterpret_cast<uint4*>(buf + sw128_offset(rr, c0 + 1));
    float lo[8], hi[8];
    unpack8(*ptr[k][0], lo);
    unpack8(*ptr[k][1], hi);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e += 2) ffma2(s0, s1, lo[e], lo[e + 1], lo[e], lo[e + 1], s0, s1);
#pragma unroll
    for (int e = 0; e < 8; e += 2) ffma2(s0, s1, hi[e], hi[e + 1], hi[e], hi[e + 1], s0, s1);
    ss[k] = s0 + s1;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      x[k][e] = lo[e];
      x[k][8 + e] = hi[e];
    }
  }
#pragma unroll
  for (int k = 0; k < kChains; ++k) {
    ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], 1);
    ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], 2);
  }
#pragma unroll
  for (int k = 0; k < kChains; ++k) {
    const float inv = rsqrtf(ss[k] * (1.f / kHeadDim) + eps);
    float lo[8], hi[8];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      fmul2(lo[e], lo[e + 1], x[k][e], x[k][e + 1], inv, inv);
      fmul2(lo[e], lo[e + 1], lo[e], lo[e + 1], w0[e], w0[e + 1]);
      fmul2(hi[e], hi[e + 1], x[k][8 + e], x[k][9 + e], inv, inv);
      fmul2(hi[e], hi[e + 1], hi[e], hi[e + 1], w1[e], w1[e + 1]);
    }
    *ptr[k][0] = pack8(lo);
    *ptr[k][1] = pack8(hi);
  }
}

// Every row of two 128-row tiles, by the kPrepThreads threads (pt = 0 .. kPrepThreads - 1): row group rg owns
// rows rg, rg + 48 and (for rg < 32) rg + 96; warps cover 8 row groups each, so every branch is warp-uniform.
__device__ __forceinline__ void rms_inplace(uint8_t* buf0, uint8_t* buf1, const float* w, float eps, int pt) {
  constexpr int kGroups = kPrepThreads / 4;
  static_assert(kGroups == 48 && kTileRows == 128, "row split");
  const int sub = pt & 3, rg = pt >> 2;
  const int c0 = 2 * sub;
  float w0[8], w1[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    w0[e] = w[c0 * 8 + e];
    w1[e] = w[c0 * 8 + 8 + e];
  }
  rms_rows<2>(buf0, buf1, rg, rg + kGroups, c0, w0, w1, eps);
  if (rg + 2 * kGroups < kTileRows) rms_rows<1>(buf0, buf1, rg + 2 * kGroups, 0, c0, w0, w1, eps);
}

__global__ void __launch_bounds__(kThreads, 1)
    cross_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                      const __grid_constant__ CUtensorMap tm_out, const CrossParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* q_raw = bars + 0;     // [2] TMA bytes of raw q, q_diff
  uint64_t* q_full = bars + 2;    // [2] prep-warp arrivals (normed q, q_diff)
  uint64_t* q_empty = bars + 4;   // [2] commit (last S MMA of the unit)
  uint64_t* kv_raw = bars + 6;    // TMA bytes of the run's K, K_diff, V
  uint64_t* kv_full = bars + 7;   // prep-warp arrivals (keys normed or passed through)
  uint64_t* kv_empty = bars + 8;  // commit (last PV_B of the run)
  uint64_t* s_full = bars + 9;    // [2] commit
  uint64_t* p_ready = bars + 11;  // [2] 4 softmax warps
  uint64_t* o_full = bars + 13;   // [2] commit
  uint64_t* o_empty = bars + 15;  // [2] 4 epilogue warps
  uint64_t* scale_full = bars + 17;  // 8 softmax warps wrote their rows' scales
  uint64_t* scale_free = bars + 18;  // 4 epilogue warps read them
  uint64_t* drain = bars + 19;
  uint64_t* stage_full = bars + 20;  // 4 epilogue warps wrote the staging tile
  uint64_t* stage_free = bars + 21;  // the previous unit's TMA store has read the staging tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* wq = reinterpret_cast<float*>(smem + kOffW);
  float* wk = wq + 64;
  float* scale = reinterpret_cast<float*>(smem + kOffScale);
  uint8_t* stage = smem + kOffStage;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef HB_TRACE
  const long long xt0 = clock64();
  int xt_n = 0;
#endif
  const int u0 = (int)(((long long)blockIdx.x * p.units) / gridDim.x);
  const int u1 = (int)(((long long)(blockIdx.x + 1) * p.units) / gridDim.x);
  const int nunits = u1 - u0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_raw[i], 1);
      mbar_init(&q_full[i], kPrepWarps);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(scale_full, 8);
    mbar_init(scale_free, 4);
    mbar_init(kv_raw, 1);
    mbar_init(kv_full, kPrepWarps);
    mbar_init(kv_empty, 1);
    mbar_init(drain, 1);
    mbar_init(stage_full, 4);
    mbar_init(stage_free, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_kv);
    prefetch_tmap(&tm_out);
  }
  if (threadIdx.x < 128) {
    const int i = threadIdx.x & 63;
    wq[threadIdx.x] = threadIdx.x < 64 ? p.q_w[i] : (p.k_w ? p.k_w[i] : 1.f);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int sec = p.heads * kHeadDim;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (raw tiles)
    if (lane == 0) {
      int run = -1, kv_issued = -1, prev_bh = -1, qissued = 0;
      for (int j = 0; j < nunits && !*abort_flag; ++j) {
        const Unit x = decode(p, u0 + j);
        const int bh = x.b * p.heads + x.h, col = x.h * kHeadDim;
        if (bh != prev_bh) {
          prev_bh = bh;
          ++run;
          if (run >= 1 && !sleep_wait(kv_empty, (run - 1) & 1, kSlackSleepNs)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(kv_raw, p.nkt * kKvTileBytes);
          for (int kt = 0; kt < p.nkt; ++kt) {
            uint8_t* dst = smem + kt * kKvTileBytes;
            tma_load_3d(dst, &tm_kv, col, kt * kTileRows, x.b, kv_raw);
            tma_load_3d(dst + kTileBytes, &tm_kv, sec + col, kt * kTileRows, x.b, kv_raw);
            tma_load_3d(dst + 2 * kTileBytes, &tm_kv, 2 * sec + col, kt * kTileRows, x.b, kv_raw);
          }
          kv_issued = run;
          XT(0, 200 + run);
        }
        const int qb = j & 1;
        if (j >= 2 && !sleep_wait(&q_empty[qb], ((j >> 1) & 1) ^ 1, kSlackSleepNs)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* qdst = smem + kOffQ + qb * kQBytes;
        mbar_arrive_expect_tx(&q_raw[qb], 2 * kTileBytes);
        tma_load_3d(qdst, &tm_q, col, x.qt * kTileRows, x.b, &q_raw[qb]);
        tma_load_3d(qdst + kTileBytes, &tm_q, sec + col, x.qt * kTileRows, x.b, &q_raw[qb]);
        qissued = j + 1;
        XT(0, 100 + j);
      }
      // drain: every copy issued into this CTA's shared memory lands before it exits
      if (kv_issued >= 0) mbar_wait(kv_raw, kv_issued & 1);
      for (int j = max(0, qissued - 2); j < qissued; ++j) mbar_wait(&q_raw[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idO = idesc_bf16_f32(128, 64, true);
      const uint32_t tSa = tmem, tSb = tmem + 128;
      const uint32_t qbase = smem_u32(smem + kOffQ), kbase = smem_u32(smem);
      bool ok = true;
      int t = 0, run = -1;
      // pending PV_B: step counter, key tile, O buffer, accumulate, last key tile of its unit, release K/V
      int pb_t = -1, pb_kt = 0, pb_ob = 0, pb_acc = 0, pb_last = 0, pb_rel = 0;
      auto issue_pv_b = [&]() -> bool {
        if (!mbar_wait(&p_ready[1], pb_t & 1)) return false;
        XT(1, 300 + pb_t);
        tc_fence_after();
        const uint32_t vb = kbase + pb_kt * kKvTileBytes + 2 * kTileBytes;
        const uint32_t tO = tmem + 320 + 128 * pb_ob;
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_bf16_ts(tO, tSb + 8 * k, smem_desc_sw128(vb + 2048 * k), idO, (pb_acc || k > 0));
        if (pb_last) tc_commit(&o_full[pb_ob]);
        if (pb_rel) tc_commit(kv_empty);
        pb_t = -1;
        return true;
      };
      Unit nx = nunits > 0 ? decode(p, u0) : Unit{};
      Unit prev = Unit{-1, -1, 0};
      for (int j = 0; ok && j < nunits; ++j) {
        const Unit x = nx;
        const bool has_next = j + 1 < nunits;
        if (has_next) nx = decode(p, u0 + j + 1);
        if (!same_run(prev, x)) {
          // the previous run's last PV_B releases its K/V before the new ones are waited for
          if (pb_t >= 0 && !issue_pv_b()) {
            ok = false;
            break;
          }
          ++run;
          if (!mbar_wait(kv_full, run & 1) || *abort_flag) {
            ok = false;
            break;
          }
          XT(1, 600 + run);
          tc_fence_after();
        }
        prev = x;
        const int qb = j & 1;
        if (!mbar_wait(&q_full[qb], (j >> 1) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        XT(1, 100 + j);
        tc_fence_after();
        const uint32_t qa = qbase + qb * kQBytes, qd = qa + kTileBytes;
        for (int kt = 0; kt < p.nkt; ++kt) {
          const uint32_t kb = kbase + kt * kKvTileBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_ss(tSa, smem_desc_sw128(qa + 32 * k), smem_desc_sw128(kb + 32 * k), idS, k > 0);
          tc_commit(&s_full[0]);
          if (pb_t >= 0 && !issue_pv_b()) {
            ok = false;
            break;
          }
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_ss(tSb, smem_desc_sw128(qd + 32 * k), smem_desc_sw128(kb + kTileBytes + 32 * k), idS, k > 0);
          tc_commit(&s_full[1]);
          if (kt == p.nkt - 1) tc_commit(&q_empty[qb]);
          if (kt == 0 && j >= 2 && !mbar_wait(&o_empty[qb], ((j >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          XT(1, 400 + j);
          if (!mbar_wait(&p_ready[0], t & 1)) {
            ok = false;
            break;
          }
          XT(1, 500 + j);
          tc_fence_after();
          const uint32_t vb = kb + 2 * kTileBytes;
          const uint32_t tOa = tmem + 256 + 128 * qb;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16_ts(tOa, tSa + 8 * k, smem_desc_sw128(vb + 2048 * k), idO, (kt > 0 || k > 0));
          pb_t = t;
          pb_kt = kt;
          pb_ob = qb;
          pb_acc = kt > 0;
          pb_last = kt == p.nkt - 1;
          pb_rel = pb_last && !(has_next && same_run(x, nx));
          ++t;
        }
      }
      if (ok && pb_t >= 0) ok = issue_pv_b();
      if (!ok) *abort_flag = 1;
      tc_commit(drain);  // every MMA this thread issued has finished before TMEM is freed
      mbar_wait(drain, 0);
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------------- softmax
    const int br = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + (br ? 128u : 0u);
    int t = 0;
    bool ok = true;
    for (int j = 0; ok && j < nunits; ++j) {
      const Unit x = decode(p, u0 + j);
      const uint32_t tO = tmem + lane_base + 256u + 128u * (j & 1) + (br ? 64u : 0u);
      float m = -INFINITY, l = 0.f;
      for (int kt = 0; kt < p.nkt; ++kt, ++t) {
        if (!(ok = warp_wait(&s_full[br], t & 1, abort_flag, kSoftSleepNs))) break;
        if (lane == 0 && quad == 0) XT(2 + br, 100 + t);
        tc_fence_after();
        const int k0 = kt * kTileRows;
        // pass 1: row max of the raw scores (keys past the context masked), 32 keys per TMEM load; two chains
        // of three-input maxima (the scale is positive, so it commutes with the max)
        float mx0 = -INFINITY, mx1 = -INFINITY;
        uint32_t r[32];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int kc = k0 + 32 * c;
          if (kc >= p.Lkv) break;
          tmem_ld32(tS + 32 * c, r);
          tmem_wait_ld();
          if (kc + 32 > p.Lkv) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (kc + e >= p.Lkv) r[e] = 0xff800000u;  // -inf
          }
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            mx0 = fmax3(mx0, __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
            mx1 = fmax3(mx1, __uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
          }
        }
        const float rmax = fmaxf(mx0, mx1) * kScoreScale;
        const float m_new = fmaxf(m, rmax);
        const bool upd = m_new > m + kRescaleThreshold;
        float alpha = 1.f;
        if (upd) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - m_new);
          m = m_new;
        }
        const float nm = (m == -INFINITY) ? 0.f : -m;
        // pass 2: P = exp2(s * scale - m) as bf16 pairs into the first 64 columns of S (in place); packed FMA
        // per key pair and two packed row-sum accumulators
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int kc = k0 + 32 * c;
          uint32_t pk[16];
          if (kc >= p.Lkv) {
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = 0u;
          } else {
            tmem_ld32(tS + 32 * c, r);
            tmem_wait_ld();
            if (kc + 32 > p.Lkv) {
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (kc + e >= p.Lkv) r[e] = 0xff800000u;
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float x0, x1;
              ffma2(x0, x1, __uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]), kScoreScale, kScoreScale, nm, nm);
              float p0, p1;
              if ((e & kPolyMask) == kPolyMask) {  // a share of the exponentials on the FMA pipe
                exp2_poly2(x0, x1, p0, p1);
              } else {
                p0 = ex2_approx(x0);
                p1 = ex2_approx(x1);
              }
              const int a2 = (e & 1) * 2;
              fadd2(rs[a2], rs[a2 + 1], rs[a2], rs[a2 + 1], p0, p1);
              pk[e] = pack_bf16x2(p0, p1);
            }
          }
          tmem_st16(tS + 16 * c, pk);
        }
        l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
        if (kt > 0 && __any_sync(0xffffffffu, upd)) {
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
        if (lane == 0 && quad == 0) XT(2 + br, 200 + t);
      }
      if (!ok) break;
      // this row's scale for the epilogue, once the epilogue of unit j - 1 has read the previous one
      if (j >= 1 && !(ok = warp_wait(scale_free, (j - 1) & 1, abort_flag))) break;
      if (lane == 0 && quad == 0) XT(2 + br, 300 + j);
      scale[br * kTileRows + row] = (br ? (p.lam ? p.lam[x.h / 2] : 1.f) : 1.f) / l;
      __syncwarp();
      if (lane == 0) mbar_arrive(scale_full);
    }
  } else {
    // ---------------------------------------------------------------- RMSNorm (warps 2, 3, 12-15) + epilogue (12-15)
    const int pt = warp >= 12 ? threadIdx.x - 10 * 32 : threadIdx.x - 2 * 32;
    const bool epi = warp >= 12;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int run = -1, prev_bh = -1;
    bool ok = true;
    // job n prepares unit n (its run's keys first when the run changes); the epilogue of unit n - 1 follows
    for (int n = 0; ok && n <= nunits; ++n) {
      if (n < nunits) {
        const Unit x = decode(p, u0 + n);
        const int bh = x.b * p.heads + x.h;
        if (bh != prev_bh) {
          prev_bh = bh;
          ++run;
          if (!(ok = warp_wait(kv_raw, run & 1, abort_flag))) break;
          if (pt == 0) XT(4, 300 + run);
          if (p.k_w) {
            for (int kt = 0; kt < p.nkt; ++kt) {
              uint8_t* kt_base = smem + kt * kKvTileBytes;
              rms_inplace(kt_base, kt_base + kTileBytes, wk, p.eps, pt);
            }
            fence_proxy_async_smem();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(kv_full);
        }
        const int qb = n & 1;
        if (!(ok = warp_wait(&q_raw[qb], (n >> 1) & 1, abort_flag))) break;
        if (pt == 0) XT(4, 100 + n);
        uint8_t* qbuf = smem + kOffQ + qb * kQBytes;
        rms_inplace(qbuf, qbuf + kTileBytes, wq, p.eps, pt);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[qb]);
        if (pt == 0) XT(4, 200 + n);
      }
      if (!epi || n == 0) continue;
      // ---- epilogue of unit j = n - 1
      const int j = n - 1, ob = j & 1;
      const Unit x = decode(p, u0 + j);
      if (!(ok = warp_wait(&o_full[ob], (j >> 1) & 1, abort_flag))) break;
      if (lane == 0 && quad == 0) XT(3, 300 + j);
      tc_fence_after();
      if (!(ok = warp_wait(scale_full, j & 1, abort_flag))) break;
      const float inv_a = scale[row], sb = scale[kTileRows + row];
      __syncwarp();
      if (lane == 0) mbar_arrive(scale_free);
      // the staging tile is free once the previous unit's store has read it
      if (j >= 1) {
        if (warp == 12 && lane == 0) {
          bulk_wait_group_read0();
          mbar_arrive(stage_free);
        }
        if (!(ok = warp_wait(stage_free, (j - 1) & 1, abort_flag))) break;
      }
      const uint32_t tOa = tmem + lane_base + 256u + 128u * ob, tOb = tOa + 64u;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t oa[32], obv[32];
        tmem_ld32(tOa + 32 * c, oa);
        tmem_ld32(tOb + 32 * c, obv);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          // each branch normalised and rounded on its own, then one fp32 subtraction (no contraction)
          const float y0 = __fmul_rn(__uint_as_float(oa[2 * e]), inv_a) - __fmul_rn(__uint_as_float(obv[2 * e]), sb);
          const float y1 =
              __fmul_rn(__uint_as_float(oa[2 * e + 1]), inv_a) - __fmul_rn(__uint_as_float(obv[2 * e + 1]), sb);
          w[e] = pack_bf16x2(y0, y1);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          *reinterpret_cast<uint4*>(stage + sw128_offset(row, 4 * c + e)) =
              make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&o_empty[ob]);  // both O buffers of unit j are read
        mbar_arrive(stage_full);
      }
      if (warp == 12 && lane == 0) {
        if (!mbar_wait(stage_full, j & 1)) {
          ok = false;
          *abort_flag = 1;
        } else {
          tma_store_3d(&tm_out, x.h * kHeadDim, x.qt * kTileRows, x.b, stage);
          bulk_commit_group();
        }
      }
      if (warp == 12) ok = __shfl_sync(0xffffffffu, ok, 0);
      if (lane == 0 && quad == 0) XT(3, 400 + j);
    }
    if (warp == 12 && lane == 0) bulk_wait_group0();  // the last stores complete before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
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

// 3-D map over a [batch, rows, row_stride] bf16 tensor, box 64 columns x 128 rows x 1, 128-byte swizzle:
// one head's 64 dims of 128 rows move as the SW128 image; loads read rows past `rows` as zero, stores skip them.
bool encode_rows(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* base, int64_t row_stride,
                 int rows, int batch) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_stride), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride) * 2, static_cast<cuuint64_t>(row_stride) * 2 * rows};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace hb

using namespace hb;

#ifdef HB_TRACE
extern "C" int hb_cross_debug_trace(unsigned int* out) {
  if (cudaMemcpyFromSymbol(out, g_xtrace, sizeof(g_xtrace)) != cudaSuccess) return 1;
  return cudaMemcpyFromSymbol(out + 2 * 5 * 512, g_xtrace_n, sizeof(g_xtrace_n)) != cudaSuccess;
}
#endif

extern "C" int hb_cross_diff_attn(const void* q, int64_t q_row_stride, const void* kv, int64_t kv_row_stride,
                                  const float* q_weight, const float* k_weight, const float* lam, void* out,
                                  int64_t out_row_stride, int batch, int q_len, int kv_len, int num_heads,
                                  int head_dim, float eps, cudaStream_t stream) {
  if (!q || !kv || !q_weight || !out) return HB_ERR_NULL;
  if (head_dim != kHeadDim || batch < 1 || q_len < 1 || kv_len < 1 || kv_len > kMaxKvTiles * kTileRows ||
      num_heads < 1 || (lam && num_heads % 2) || q_row_stride < 2LL * num_heads * kHeadDim ||
      kv_row_stride < 3LL * num_heads * kHeadDim || out_row_stride < (int64_t)num_heads * kHeadDim)
    return HB_ERR_SHAPE;
  const int nqt = (q_len + kTileRows - 1) / kTileRows;
  const long long units = (long long)batch * num_heads * nqt;
  if (units >= (1LL << 31) || (long long)batch * q_len * q_row_stride >= (1LL << 40)) return HB_ERR_SHAPE;
  if (!aligned16(q) || !aligned16(kv) || !aligned16(out) || q_row_stride % 8 || kv_row_stride % 8 ||
      out_row_stride % 8)
    return HB_ERR_ALIGN;
  const int st = check_device();
  if (st != HB_OK) return st;
  auto encode = encode_fn();
  if (!encode) return HB_ERR_LAUNCH;
  CUtensorMap tm_q, tm_kv, tm_out;
  if (!encode_rows(encode, &tm_q, q, q_row_stride, q_len, batch) ||
      !encode_rows(encode, &tm_kv, kv, kv_row_stride, kv_len, batch) ||
      !encode_rows(encode, &tm_out, out, out_row_stride, q_len, batch))
    return HB_ERR_LAUNCH;
  CrossParams p{};
  p.B = batch;
  p.Lq = q_len;
  p.Lkv = kv_len;
  p.heads = num_heads;
  p.nqt = nqt;
  p.nkt = (kv_len + kTileRows - 1) / kTileRows;
  p.units = static_cast<int>(units);
  p.q_w = q_weight;
  p.k_w = k_weight;
  p.eps = eps;
  p.lam = lam;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(cross_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
        cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  const int grid = p.units < sms ? p.units : sms;
  cross_attn_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tm_q, tm_kv, tm_out, p);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

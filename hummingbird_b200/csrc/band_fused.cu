// Fused, persistent SAME-L band differential attention (window <= 128): one kernel reads the raw
// `to_qkv` rows once and writes the merged output once (band_attention.py:61-120 in one pass).
//
// Work: the (batch, head, 128-row query tile) units, head-major, are split into contiguous runs, one run per
// CTA (grid = #SMs). Walking consecutive query tiles of one head, each key tile kt is used by query tiles
// kt-1, kt, kt+1, so it is prepared once and kept in a 3-slot ring (window <= 128 means a query tile needs
// at most the key tiles qt-1, qt, qt+1).
//
// Roles (16 warps):
//   warp 0       3-D TMA (128B swizzle, rows past the sequence read as zero) of the raw q, q_diff tile of
//                each unit into a double buffer and of each new k, k_diff, v tile into the ring slot
//   warp 1       TMEM allocation (512 columns) and the single MMA-issuing thread
//   warps 4-7    softmax of branch A (one query row per thread); writes 1/l_A per row for the epilogue
//   warps 8-11   softmax of branch B, then the per-tile epilogue: out = O_A / l_A - lambda O_B / l_B, bf16
//   warps 2-3, 12-15  preparation, in place in shared memory (DyT and RoPE only mix dims of one row):
//                DyT gamma * tanh(alpha x) + beta and RoPE in fp32 with angles fp32(pos) * inv_freq
//                reduced to [-pi, pi] (Cody-Waite) for the hardware sin/cos, then bf16 (q, k rounded once)
// TMEM: S_A [0,128) (P_A in [0,64)), S_B [128,256), O_A/O_B double-buffered by tile parity at
// [256,320)/[320,384) and [384,448)/[448,512), so the epilogue of tile j overlaps tile j+1.
//
// MMA order per key tile i of unit j: S_A(i), PV_B(i-1), S_B(i), PV_A(i), with PV_B(last) of unit j
// issued after S_A(0) of unit j+1. A key tile is released to the producers right after its last PV_B.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "attn_internal.h"
#include "band_fused.h"
#include "hb_sm100.cuh"
#include "prep_common.cuh"

namespace hb {

#ifdef HB_TRACE
// Debug builds only (-DHB_TRACE): %clock timestamps of pipeline events, one slot per traced thread, kept in
// shared memory while the kernel runs (no global traffic) and copied out by CTA 0 at the end.
__device__ unsigned int g_trace[8][2048];
__device__ unsigned int g_trace_n[8];
constexpr int kTraceSlots = 5, kTraceEvents = 240;
constexpr int kTraceBytes = kTraceSlots * kTraceEvents * 8 + 64;
#define TRACE(slot, id, t0)                                                         \
  do {                                                                              \
    trace_slot = (slot);                                                            \
    if (trace_n < kTraceEvents) {                                                   \
      trace_buf[((slot) * kTraceEvents + trace_n) * 2] = (id);                      \
      trace_buf[((slot) * kTraceEvents + trace_n) * 2 + 1] = (unsigned)clock();     \
      ++trace_n;                                                                    \
    }                                                                               \
  } while (0)
#else
constexpr int kTraceBytes = 0;
#define TRACE(slot, id, t0) \
  do {                      \
  } while (0)
#endif

namespace {

constexpr int kThreads = 512;
constexpr int kPrepWarps = 6;  // warps 2, 3 and 12-15
constexpr int kPrepThreads = 32 * kPrepWarps;
constexpr int kSlots = 3;
constexpr int kSlotBytes = 3 * kTileBytes;  // K, Kd, V
constexpr int kQBytes = 2 * kTileBytes;     // Q, Qd
constexpr int kOffQ = kSlots * kSlotBytes;
constexpr int kOffBars = kOffQ + 2 * kQBytes;
constexpr int kNumBars = 26;
constexpr int kOffMisc = kOffBars + kNumBars * 8;
constexpr int kOffNorm = kOffMisc + 16;
constexpr int kNormStride = 132;
constexpr int kOffScaleA = kOffNorm + 2 * kNormStride * 4;
constexpr int kOffFreq = kOffScaleA + 2 * kTileRows * 4;
constexpr int kOffTrace = kOffFreq + 32 * 4;
constexpr int kSmemBytes = kOffTrace + kTraceBytes + 1024;
// 2 pi = kTwoPi1 + kTwoPi2 + kTwoPi3 (fp32 parts of 2 pi taken to 60 digits) and fp32(1 / (2 pi))
constexpr float kTwoPi1 = 6.2831854820251465f, kTwoPi2 = -1.7484555314695172e-07f, kTwoPi3 = -6.8604980400235275e-15f;
constexpr float kInvTwoPi = 0.15915493667125702f;
constexpr float kScoreScale = 1.4426950408889634f * 0.125f;
constexpr float kRescaleThreshold = 8.0f;

struct Unit {
  int b, h, qt, klo, khi;
};

__device__ __forceinline__ Unit decode(const BandFusedParams& p, int u) {
  Unit x;
  const int bh = u / p.nqt;
  x.qt = p.qt_first + (u - bh * p.nqt);
  x.b = bh / p.heads;
  x.h = bh - x.b * p.heads;
  const int q_lo = x.qt * kTileRows, q_hi = min(q_lo + kTileRows - 1, p.rows - 1);
  x.klo = max(0, q_lo - p.window) / kTileRows;
  x.khi = min(p.ntiles - 1, (q_hi + p.window) / kTileRows);
  return x;
}

// Key-tile load sequence shared by every role: tiles get consecutive sequence numbers in the order first
// needed; tile seq s lives in slot s % 3 for its (s / 3)-th use of that slot.
struct Sched {
  int seq_next = 0, run_base = 0, run_klo = 0, prev_bh = -1, prev_khi = -1;
  int first_new = 0;  // first key tile of the current unit that is not yet loaded
  __device__ void advance(const Unit& x, int heads) {
    const int bh = x.b * heads + x.h;
    if (bh != prev_bh) {
      run_base = seq_next;
      run_klo = x.klo;
      first_new = x.klo;
    } else {
      first_new = prev_khi + 1;
    }
    if (x.khi >= first_new) seq_next += x.khi - first_new + 1;
    prev_khi = (bh != prev_bh) ? x.khi : max(prev_khi, x.khi);
    prev_bh = bh;
  }
  __device__ int seq(int kt) const { return run_base + kt - run_klo; }
};

// Bit e set iff key kc + e is inside the band of query q (|k - q| <= window) and inside the buffer.
__device__ __forceinline__ uint32_t band_bits(int kc, int q, int window, int rows) {
  const int lo = max(max(q - window, 0), kc) - kc;
  const int hi = min(min(q + window, rows - 1), kc + 31) - kc;
  if (hi < lo) return 0u;
  const uint32_t upto = hi >= 31 ? 0xffffffffu : ((1u << (hi + 1)) - 1u);
  return upto & (0xffffffffu << lo);
}

__device__ __forceinline__ bool same_run(const Unit& a, const Unit& b) { return a.b == b.b && a.h == b.h; }

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity) && !*abort_flag;
  return __all_sync(0xffffffffu, ok);
}

// cos / sin of an fp32 angle: Cody-Waite reduction by 2 pi (three-part constant, FMA) to |r| <= ~pi, then
// the hardware approximations on the reduced argument (absolute error ~2^-21 there).
__device__ __forceinline__ void sincos_reduced(float x, float& sn, float& cs) {
  const float k = rintf(x * kInvTwoPi);
  float r = fmaf(-k, kTwoPi1, x);
  r = fmaf(-k, kTwoPi2, r);
  r = fmaf(-k, kTwoPi3, r);
  sn = __sinf(r);
  cs = __cosf(r);
}

// Transform one 128-row tile of two raw sections (q/q_diff or k/k_diff, landed by TMA in the SW128 image)
// in place: DyT, RoPE, bf16. Four threads own a row; each owns two 8-dim chunks: for rotary dims a chunk
// and its rotate-half partner (so RoPE needs no exchange and each angle is evaluated once), the remaining
// chunks in pairs.
__device__ __forceinline__ void prep_inplace(const BandFusedParams& p, int tile, const float* norm,
                                             const float* freqs, uint8_t* buf0, uint8_t* buf1, int pt, int nthreads) {
  const int sub = pt & 3, rg = pt >> 2, ngroups = nthreads >> 2;
  const int hc8 = p.half >> 3;
  const bool rot = sub < hc8;
  const int c0 = rot ? sub : 2 * hc8 + 2 * (sub - hc8);
  const int c1 = rot ? sub + hc8 : c0 + 1;
  const float alpha = norm[0];
  float g0[8], b0[8], g1[8], b1[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    g0[e] = norm[1 + c0 * 8 + e];
    b0[e] = norm[65 + c0 * 8 + e];
    g1[e] = norm[1 + c1 * 8 + e];
    b1[e] = norm[65 + c1 * 8 + e];
  }
#pragma unroll 1
  for (int r = rg; r < kTileRows; r += ngroups) {
    const int row = tile * kTileRows + r;
    const bool valid = row < p.rows;
    float cs[8], sn[8];
    if (rot) {
      const float pos = static_cast<float>(p.pos0 + row);
#pragma unroll
      for (int e = 0; e < 8; ++e) sincos_reduced(pos * freqs[8 * sub + e], sn[e], cs[e]);  // fp32(pos) * inv_freq
    }
#pragma unroll
    for (int sec = 0; sec < 2; ++sec) {
      uint8_t* buf = sec ? buf1 : buf0;
      uint4* p0 = reinterpret_cast<uint4*>(buf + sw128_offset(r, c0));
      uint4* p1 = reinterpret_cast<uint4*>(buf + sw128_offset(r, c1));
      float x0[8], x1[8], y0[8], y1[8];
      unpack8(*p0, x0);
      unpack8(*p1, x1);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        y0[e] = fmaf(g0[e], tanh_approx(alpha * x0[e]), b0[e]);
        y1[e] = fmaf(g1[e], tanh_approx(alpha * x1[e]), b1[e]);
      }
      if (rot) {  // d < half pairs with d + half: y_d cos - y_{d+half} sin, y_{d+half} cos + y_d sin
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = y0[e], b = y1[e];
          y0[e] = a * cs[e] - b * sn[e];
          y1[e] = b * cs[e] + a * sn[e];
        }
      }
      *p0 = valid ? pack8(y0) : make_uint4(0, 0, 0, 0);
      *p1 = valid ? pack8(y1) : make_uint4(0, 0, 0, 0);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    band_fused_kernel(const __grid_constant__ CUtensorMap tmap, const BandFusedParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint64_t* q_full = bars + 0;    // [2] 4 prep-warp arrivals (prepared q, q_diff)
  uint64_t* q_empty = bars + 2;   // [2] commit (last S MMA of the unit)
  uint64_t* k_full = bars + 4;    // [3] 4 prep-warp arrivals (prepared k, k_diff; v landed)
  uint64_t* k_empty = bars + 7;   // [3] commit (last PV_B of the tile)
  uint64_t* s_full = bars + 10;   // [2] commit
  uint64_t* p_ready = bars + 12;  // [2] 4 softmax warps
  uint64_t* o_full = bars + 14;   // [2] commit
  uint64_t* o_empty = bars + 16;  // [2] 4 epilogue warps
  uint64_t* sa_full = bars + 18;  // [2] 4 branch-A warps
  uint64_t* drain = bars + 20;
  uint64_t* q_raw = bars + 21;    // [2] TMA bytes of raw q, q_diff
  uint64_t* k_raw = bars + 23;    // [3] TMA bytes of raw k, k_diff, v
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* norms = reinterpret_cast<float*>(smem + kOffNorm);
  float* scale_a = reinterpret_cast<float*>(smem + kOffScaleA);
  float* freqs = reinterpret_cast<float*>(smem + kOffFreq);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long t0 = clock64();
  (void)t0;
#ifdef HB_TRACE
  unsigned* trace_buf = reinterpret_cast<unsigned*>(smem + kOffTrace);
  int trace_n = 0, trace_slot = -1;
#endif
  const int u0 = (int)(((long long)blockIdx.x * p.units) / gridDim.x);
  const int u1 = (int)(((long long)(blockIdx.x + 1) * p.units) / gridDim.x);
  const int nunits = u1 - u0;

#ifdef HB_TRACE
  if (threadIdx.x < kTraceSlots) trace_buf[2 * kTraceSlots * kTraceEvents + threadIdx.x] = 0;
#endif
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], kPrepWarps);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
      mbar_init(&sa_full[i], 4);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&k_full[i], kPrepWarps);
      mbar_init(&k_empty[i], 1);
      mbar_init(&k_raw[i], 1);
    }
    mbar_init(&q_raw[0], 1);
    mbar_init(&q_raw[1], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap);
  }
  for (int i = threadIdx.x; i < 2 * kNormStride; i += kThreads) {
    const int which = i / kNormStride, k = i - which * kNormStride;
    norms[i] = k < 129 ? (which ? p.k_norm : p.q_norm)[k] : 0.f;
  }
  if (threadIdx.x < 32) freqs[threadIdx.x] = threadIdx.x < p.half ? p.inv_freq[threadIdx.x] : 0.f;
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (raw tiles)
    if (lane == 0) {
      Sched sch;
      int kissued = 0, qissued = 0;
      for (int j = 0; j < nunits && !*abort_flag; ++j) {
        const Unit x = decode(p, u0 + j);
        sch.advance(x, p.heads);
        const int col = (p.head0 + x.h) * kHeadDim, sec = p.H_total * kHeadDim;
        const int qb = j & 1;
        if (j >= 2 && !mbar_wait(&q_empty[qb], ((j >> 1) & 1) ^ 1)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* qdst = smem + kOffQ + qb * kQBytes;
        TRACE(0, 100 + j, t0);
        mbar_arrive_expect_tx(&q_raw[qb], 2 * kTileBytes);
        tma_load_3d(qdst, &tmap, col, x.qt * kTileRows, x.b, &q_raw[qb]);
        tma_load_3d(qdst + kTileBytes, &tmap, 3 * sec + col, x.qt * kTileRows, x.b, &q_raw[qb]);
        qissued = j + 1;
        for (int kt = sch.first_new; kt <= x.khi; ++kt) {
          const int s = sch.seq(kt), slot = s % kSlots;
          if (s >= kSlots && !mbar_wait(&k_empty[slot], ((s / kSlots) & 1) ^ 1)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* kdst = smem + slot * kSlotBytes;
          TRACE(0, 200 + kt, t0);
          mbar_arrive_expect_tx(&k_raw[slot], 3 * kTileBytes);
          tma_load_3d(kdst, &tmap, sec + col, kt * kTileRows, x.b, &k_raw[slot]);
          tma_load_3d(kdst + kTileBytes, &tmap, 4 * sec + col, kt * kTileRows, x.b, &k_raw[slot]);
          tma_load_3d(kdst + 2 * kTileBytes, &tmap, 2 * sec + col, kt * kTileRows, x.b, &k_raw[slot]);
          kissued = s + 1;
        }
      }
      // drain: every copy issued into this CTA's shared memory lands before it exits
      for (int s = max(0, kissued - kSlots); s < kissued; ++s) mbar_wait(&k_raw[s % kSlots], (s / kSlots) & 1);
      for (int j = max(0, qissued - 2); j < qissued; ++j) mbar_wait(&q_raw[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t idO = idesc_bf16_f32(128, 64, true);
      const uint32_t tSa = tmem, tSb = tmem + 128;
      const uint32_t qbase = smem_u32(smem + kOffQ), kbase = smem_u32(smem);
      Sched sch;
      bool ok = true;
      int t = 0;
      // pending PV_B: tile counter, slot, O buffer, accumulate, last tile of its unit, release its slot
      int pb_t = -1, pb_slot = 0, pb_ob = 0, pb_acc = 0, pb_last = 0, pb_rel = 0;
      auto issue_pv_b = [&]() -> bool {
        if (!mbar_wait(&p_ready[1], pb_t & 1)) return false;
        tc_fence_after();
        const uint32_t vb = kbase + pb_slot * kSlotBytes + 2 * kTileBytes;
        const uint32_t tO = tmem + 320 + 128 * pb_ob;
#pragma unroll
        for (int k = 0; k < 8; ++k) mma_bf16_ts(tO, tSb + 8 * k, smem_desc_sw128(vb + 2048 * k), idO, (pb_acc || k > 0));
        if (pb_last) tc_commit(&o_full[pb_ob]);
        if (pb_rel) tc_commit(&k_empty[pb_slot]);
        pb_t = -1;
        return true;
      };
      Unit nx = nunits > 0 ? decode(p, u0) : Unit{};
      for (int j = 0; ok && j < nunits; ++j) {
        const Unit x = nx;
        const bool has_next = j + 1 < nunits;
        if (has_next) nx = decode(p, u0 + j + 1);
        sch.advance(x, p.heads);
        const int qb = j & 1;
        if (!mbar_wait(&q_full[qb], (j >> 1) & 1) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        TRACE(1, 100 + j, t0);
        const uint32_t qa = qbase + qb * kQBytes, qd = qa + kTileBytes;
        for (int kt = x.klo; kt <= x.khi; ++kt) {
          const int i = kt - x.klo;
          const int s = sch.seq(kt), slot = s % kSlots;
          if (kt >= sch.first_new) {
            if (!mbar_wait(&k_full[slot], (s / kSlots) & 1) || *abort_flag) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          TRACE(1, 200 + kt, t0);
          const uint32_t kb = kbase + slot * kSlotBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_ss(tSa, smem_desc_sw128(qa + 32 * k), smem_desc_sw128(kb + 32 * k), idS, k > 0);
          tc_commit(&s_full[0]);
          TRACE(1, 500 + kt, t0);
          if (pb_t >= 0 && !issue_pv_b()) {
            ok = false;
            break;
          }
          TRACE(1, 600 + kt, t0);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16_ss(tSb, smem_desc_sw128(qd + 32 * k), smem_desc_sw128(kb + kTileBytes + 32 * k), idS, k > 0);
          tc_commit(&s_full[1]);
          if (kt == x.khi) tc_commit(&q_empty[qb]);
          if (i == 0 && j >= 2 && !mbar_wait(&o_empty[qb], ((j >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          TRACE(1, 300 + kt, t0);
          if (!mbar_wait(&p_ready[0], t & 1)) {
            ok = false;
            break;
          }
          TRACE(1, 400 + kt, t0);
          tc_fence_after();
          const uint32_t vb = kb + 2 * kTileBytes;
          const uint32_t tOa = tmem + 256 + 128 * qb;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16_ts(tOa, tSa + 8 * k, smem_desc_sw128(vb + 2048 * k), idO, (i > 0 || k > 0));
          pb_t = t;
          pb_slot = slot;
          pb_ob = qb;
          pb_acc = i > 0;
          pb_last = kt == x.khi;
          pb_rel = !(has_next && same_run(x, nx) && kt >= nx.klo);
          ++t;
        }
      }
      if (ok && pb_t >= 0) ok = issue_pv_b();
      if (!ok) *abort_flag = 1;
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------------- softmax (+ epilogue in branch B)
    const int br = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_base + (br ? 128u : 0u);
    int t = 0;
    bool ok = true;
    for (int j = 0; ok && j < nunits; ++j) {
      const Unit x = decode(p, u0 + j);
      const int ob = j & 1;
      const uint32_t tO = tmem + lane_base + 256u + 128u * ob + (br ? 64u : 0u);
      const int q = x.qt * kTileRows + row;
      const int qw_lo = x.qt * kTileRows + quad * 32, qw_hi = qw_lo + 31;
      float m = -INFINITY, l = 0.f;
      for (int kt = x.klo; kt <= x.khi; ++kt, ++t) {
        if (!(ok = warp_wait(&s_full[br], t & 1, abort_flag))) break;
        if (lane == 0 && quad == 0) TRACE(2 + br, 100 + kt, t0);
        tc_fence_after();
        const int k0 = kt * kTileRows;
        // pass 1: row max over in-band keys; 32-key chunks outside the band for the whole warp are skipped,
        // chunks inside it for every lane of the warp need no mask (two chains of three-input maxima)
        float mx0 = -INFINITY, mx1 = -INFINITY;
        uint32_t r[32];
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int kc = k0 + 32 * c;
          if (kc >= p.rows || kc > qw_hi + p.window || kc + 31 < qw_lo - p.window) continue;
          const uint32_t bits = band_bits(kc, q, p.window, p.rows);
          tmem_ld32(tS + 32 * c, r);
          tmem_wait_ld();
          if (!__all_sync(0xffffffffu, bits == 0xffffffffu)) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (!((bits >> e) & 1u)) r[e] = 0xff800000u;  // -inf
          }
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            mx0 = fmax3(mx0, __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
            mx1 = fmax3(mx1, __uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
          }
        }
        if (lane == 0 && quad == 0) TRACE(2 + br, 500 + kt, t0);
        const float rmax = fmaxf(mx0, mx1) * kScoreScale;
        const float m_new = fmaxf(m, rmax);
        const bool upd = m_new > m + kRescaleThreshold;
        float alpha = 1.f;
        if (upd) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - m_new);
          m = m_new;
        }
        const float nm = (m == -INFINITY) ? 0.f : -m;
        // pass 2: P = exp2(s * scale - m) as bf16 into the first 64 columns of S (in place); packed FMA per key
        // pair and two packed row-sum accumulators
        float rs0 = 0.f, rs1 = 0.f, rs2 = 0.f, rs3 = 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int kc = k0 + 32 * c;
          uint32_t pk[16];
          if (kc >= p.rows || kc > qw_hi + p.window || kc + 31 < qw_lo - p.window) {
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = 0u;
          } else {
            const uint32_t bits = band_bits(kc, q, p.window, p.rows);
            tmem_ld32(tS + 32 * c, r);
            tmem_wait_ld();
            if (!__all_sync(0xffffffffu, bits == 0xffffffffu)) {
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (!((bits >> e) & 1u)) r[e] = 0xff800000u;
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
              if (e & 1)
                fadd2(rs2, rs3, rs2, rs3, p0, p1);
              else
                fadd2(rs0, rs1, rs0, rs1, p0, p1);
              pk[e] = pack_bf16x2(p0, p1);
            }
          }
          tmem_st16(tS + 16 * c, pk);
        }
        const float rs = (rs0 + rs1) + (rs2 + rs3);
        l = l * alpha + rs;
        if (lane == 0 && quad == 0) TRACE(2 + br, 600 + kt, t0);
        if (kt > x.klo && __any_sync(0xffffffffu, upd)) {
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
        if (lane == 0 && quad == 0) TRACE(2 + br, 200 + kt, t0);
      }
      if (!ok) break;
      if (br == 0) {
        scale_a[ob * kTileRows + row] = 1.f / l;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sa_full[ob]);
        continue;
      }
      // branch B: epilogue of unit j once both O accumulators are final
      if (!(ok = warp_wait(&o_full[ob], (j >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      if (!(ok = warp_wait(&sa_full[ob], (j >> 1) & 1, abort_flag))) break;
      if (lane == 0 && quad == 0) TRACE(3, 300 + j, t0);
      const float inv_a = scale_a[ob * kTileRows + row];
      const float sb = (p.lam ? p.lam[p.lam_pair0 + x.h / 2] : 1.f) / l;
      const bool store = q >= p.q_begin && q < p.q_begin + p.q_count;
      uint16_t* dst = p.out + ((size_t)x.b * p.q_count + (q - p.q_begin)) * p.out_row_stride + (size_t)x.h * kHeadDim;
      const uint32_t tOa = tmem + lane_base + 256u + 128u * ob;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t oa[32], obv[32];
        tmem_ld32(tOa + 32 * c, oa);
        tmem_ld32(tO + 32 * c, obv);
        tmem_wait_ld();
        if (store) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float y0 = __fmul_rn(__uint_as_float(oa[2 * e]), inv_a) - __fmul_rn(__uint_as_float(obv[2 * e]), sb);
            const float y1 =
                __fmul_rn(__uint_as_float(oa[2 * e + 1]), inv_a) - __fmul_rn(__uint_as_float(obv[2 * e + 1]), sb);
            w[e] = pack_bf16x2(y0, y1);
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int e = 0; e < 4; ++e) d4[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
    }
  } else if (warp >= 12 || warp == 2 || warp == 3) {
    // ---------------------------------------------------------------- preparation (in place: DyT + RoPE -> bf16)
    const int pt = warp >= 12 ? threadIdx.x - 10 * 32 : threadIdx.x - 2 * 32;
    Sched sch;
    // one job list (q tile of unit j, then its new key tiles) so the transform is instantiated once
    int j = -1, kt = 0, khi = -1, qt = 0;
    bool q_job = false;
    while (true) {
      if (!q_job && kt > khi) {  // next unit
        if (++j >= nunits) break;
        const Unit x = decode(p, u0 + j);
        sch.advance(x, p.heads);
        kt = sch.first_new;
        khi = x.khi;
        qt = x.qt;
        q_job = true;
      }
      uint64_t* raw_bar;
      uint64_t* full_bar;
      uint32_t parity;
      uint8_t* dst;
      const float* nrm;
      int tile;
      if (q_job) {
        const int qb = j & 1;
        raw_bar = &q_raw[qb];
        full_bar = &q_full[qb];
        parity = (j >> 1) & 1;
        dst = smem + kOffQ + qb * kQBytes;
        nrm = norms;
        tile = qt;
        q_job = false;
      } else {
        const int s = sch.seq(kt), slot = s % kSlots;
        raw_bar = &k_raw[slot];
        full_bar = &k_full[slot];
        parity = (s / kSlots) & 1;
        dst = smem + slot * kSlotBytes;
        nrm = norms + kNormStride;
        tile = kt++;
      }
      if (!warp_wait(raw_bar, parity, abort_flag)) break;
      if (pt == 0) TRACE(4, 100 + tile, t0);
      prep_inplace(p, tile, nrm, freqs, dst, dst + kTileBytes, pt, kPrepThreads);
      if (pt == 0) TRACE(4, 200 + tile, t0);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(full_bar);
    }
  }
#ifdef HB_TRACE
  if (trace_slot >= 0) trace_buf[2 * kTraceSlots * kTraceEvents + trace_slot] = trace_n;
#endif
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#ifdef HB_TRACE
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < kTraceSlots * kTraceEvents; i += kThreads) {
      const int sl = i / kTraceEvents, e = i - sl * kTraceEvents;
      g_trace[sl][2 * e] = trace_buf[2 * i];
      g_trace[sl][2 * e + 1] = trace_buf[2 * i + 1];
    }
    if (threadIdx.x < kTraceSlots) g_trace_n[threadIdx.x] = trace_buf[2 * kTraceSlots * kTraceEvents + threadIdx.x];
  }
#endif
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

}  // namespace

#ifdef HB_TRACE
extern "C" int hb_debug_trace(unsigned int* out, int reset) {
  if (cudaMemcpyFromSymbol(out, g_trace, sizeof(g_trace)) != cudaSuccess) return 1;
  if (cudaMemcpyFromSymbol(out + 8 * 2048, g_trace_n, sizeof(g_trace_n)) != cudaSuccess) return 1;
  if (reset) {
    unsigned int z[8] = {};
    if (cudaMemcpyToSymbol(g_trace_n, z, sizeof(z)) != cudaSuccess) return 1;
  }
  return 0;
}
#endif

int band_fused_attend(const BandFusedParams& p, cudaStream_t stream) {
  auto encode = encode_fn();
  if (!encode) return HB_ERR_LAUNCH;
  CUtensorMap tmap;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.row_stride), static_cast<cuuint64_t>(p.rows),
                        static_cast<cuuint64_t>(p.B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.row_stride) * 2, static_cast<cuuint64_t>(p.row_stride) * 2 * p.rows};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  if (encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t*>(p.qkv), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return HB_ERR_LAUNCH;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return HB_ERR_LAUNCH;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(band_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
      return HB_ERR_LAUNCH;
    configured[dev] = true;
  }
  const int grid = p.units < sms ? p.units : sms;
  band_fused_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmap, p);
  return cudaGetLastError() == cudaSuccess ? HB_OK : HB_ERR_LAUNCH;
}

}  // namespace hb

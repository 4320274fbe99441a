// Prefill attention with log-sum-exp on the 5th-generation tensor cores (sm_100a).
//
// One CTA computes a 128-query tile of one (batch, query head) against every
// visible 128-key tile of its KV head:
//   warps 8, 10  TMA producers: Q once and the K ring (warp 8), the V ring (warp 10)
//   warp 9       MMA issuer (one thread, event driven): S(t) = Q K(t)^T into TMEM
//                buffer t&1, O_{t&1} += P(t) V(t); completion via tcgen05.commit
//   warps 0-3    softmax of the even key tiles, warps 4-7 of the odd ones:
//                one thread per query row (= TMEM lane) reads S from TMEM,
//                applies the position mask, keeps its own running max/sum in
//                fp32 (log2 domain), writes P (bf16/fp16) into shared memory in
//                the 128B-swizzled K-major operand layout and rescales its own O
//                accumulator in TMEM when its max grows by more than 2^8
//   warp 11      idle (it completes the third warpgroup for setmaxnreg)
// Two softmax warpgroups keep the MUFU pipe busy while the other one waits,
// reduces or stores; each owns an O accumulator (TMEM: S0, S1, O0, O1 = 512
// columns), and the epilogue merges the two partial results exactly, writes
// out/lse and, in accumulate mode, merges into the stored (out, lse).
//
// Tile skipping and masking follow per-tile position statistics computed by
// tile_stats_kernel, so any token layout (contiguous, zigzag, padded, uneven)
// takes the same path: fully invisible tiles are never loaded, fully visible
// ones skip the element mask.
#pragma once

#include <type_traits>

#include "cea_common.cuh"

namespace cea {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NUM_THREADS = 384;
constexpr int kSoftmaxWarps = 8;  // two warpgroups
constexpr int kProducerWarp = 8;   // Q and K tiles
constexpr int kMmaWarp = 9;
constexpr int kVProducerWarp = 10;  // V tiles
constexpr uint32_t kRegsSoftmax = 232;  // setmaxnreg split: 232 + 232 + 40 per SMSP (launch reserves 3 x 168)
constexpr uint32_t kRegsOther = 40;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: O is rescaled only when the max grows by > 256x

// 1: part of the exponentials of fully visible tiles run on the FMA pipe (exp2_poly3); off by
// default: measured slower here because the softmax is latency- rather than MUFU-bound
#ifndef CEA_POLY_EXP2
#define CEA_POLY_EXP2 0
#endif

template <int D>
struct Layout {
  static constexpr int KBOX = D / 64;              // 64-element (128-byte) swizzle boxes along D
  static constexpr int BOX = 128 * 128;            // 128 rows x 128 B
  static constexpr int TILE = KBOX * BOX;          // one Q, K or V tile
  static constexpr int NSTAGE = D == 128 ? 2 : 4;  // K/V ring depth
  static constexpr int PTILE = 2 * BOX;            // P: 128 rows x 128 keys (16-bit)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + TILE;
  static constexpr int OFF_V = OFF_K + NSTAGE * TILE;
  static constexpr int OFF_P = OFF_V + NSTAGE * TILE;
  static constexpr int OFF_BAR = OFF_P + 2 * PTILE;
  static constexpr int B_QFULL = 0;
  static constexpr int B_KFULL = 1;
  static constexpr int B_KEMPTY = B_KFULL + NSTAGE;
  static constexpr int B_VFULL = B_KEMPTY + NSTAGE;
  static constexpr int B_VEMPTY = B_VFULL + NSTAGE;
  static constexpr int B_SFULL = B_VEMPTY + NSTAGE;  // x2
  static constexpr int B_PFULL = B_SFULL + 2;        // x2
  static constexpr int B_PVDONE = B_PFULL + 2;       // x2
  static constexpr int NBAR = B_PVDONE + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // TMEM base address, abort flag
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = BYTES + 1024;      // slack to align the base to 1024 B
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct Params {
  const int64_t* q_pos;
  const int64_t* k_pos;
  int64_t qpos_sb, qpos_ss, kpos_sb, kpos_ss;
  void* out;
  int64_t o_sb, o_ss, o_sh;
  float* lse;
  int64_t l_sb, l_sh, l_ss;
  const int32_t* kv_map;
  const TileStat* qstat;  // [B][nqt]
  const TileStat* kstat;  // [B][nkt]
  const int2* qrange;     // [B][nqt]: first and last key tile each query tile can see
  int B, Sq, Sk, Hq, Hkv, group, nqt, nkt;
  float scale_log2;
  int causal, out_dtype, accumulate;
};

// warp-uniform bounded wait: every lane waits, the warp continues only if all succeeded
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort, int code) {
  const bool ok = mbar_wait(bar, parity, abort, code);
  return __all_sync(0xffffffffu, ok);
}

template <int D, bool kBF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const Params p) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + L::OFF_BAR + 8 * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // an earlier CTA gave up on a pipeline wait: fail fast instead of timing out again
  if (*reinterpret_cast<volatile int*>(&g_cea_status) != 0) return;

  // block -> (q tile, batch, head): heads of one q tile are adjacent (shared K/V stay in L2),
  // and the tiles with the most keys (last positions) start first
  int idx = blockIdx.x;
  const int h = idx % p.Hq;
  idx /= p.Hq;
  const int b = idx % p.B;
  idx /= p.B;
  const int qt = p.nqt - 1 - idx;
  const int kvh = p.kv_map ? p.kv_map[h] : h / p.group;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::B_QFULL), 1);
    for (int s = 0; s < L::NSTAGE; ++s) {
      mbar_init(bar(L::B_KFULL + s), 1);
      mbar_init(bar(L::B_KEMPTY + s), 1);
      mbar_init(bar(L::B_VFULL + s), 1);
      mbar_init(bar(L::B_VEMPTY + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(L::B_SFULL + s), 1);
      mbar_init(bar(L::B_PFULL + s), 4);  // one arrival per warp of the warpgroup that owns parity s
      mbar_init(bar(L::B_PVDONE + s), 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const TileStat qs = p.qstat[b * p.nqt + qt];
  const TileStat* kst = p.kstat + static_cast<size_t>(b) * p.nkt;
  const bool causal = p.causal != 0;
  const int2 krange = p.qrange[b * p.nqt + qt];

  if (warp >= kProducerWarp) {
    // ================================================================ warpgroup 2
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;");
    if ((warp == kProducerWarp || warp == kVProducerWarp) && lane == 0) {
      // ---------------------------------------------------------- TMA producers: Q and the K ring
      // (warp 8), the V ring (warp 10); independent, so a K tile never waits behind a V stage
      const bool is_k = warp == kProducerWarp;
      if (is_k) {
        mbar_arrive_expect_tx(bar(L::B_QFULL), L::TILE);
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb)
          tma_load_4d(sbase + L::OFF_Q + kb * L::BOX, &tmQ, bar(L::B_QFULL), kb * 64, qt * BM, h, b);
      }
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      const int off = is_k ? L::OFF_K : L::OFF_V;
      const int b_full = is_k ? L::B_KFULL : L::B_VFULL;
      const int b_empty = is_k ? L::B_KEMPTY : L::B_VEMPTY;
      int it = 0;
      for (int kt = krange.x; kt <= krange.y; ++kt) {
        if (classify(qs, kst[kt], causal) == kSkip) continue;
        const int st = it % L::NSTAGE;
        const uint32_t n = it / L::NSTAGE;
        if (n > 0 && !mbar_wait(bar(b_empty + st), (n - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(bar(b_full + st), L::TILE);
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb)
          tma_load_4d(sbase + off + st * L::TILE + kb * L::BOX, map, bar(b_full + st), kb * 64, kt * BN, kvh, b);
        ++it;
      }
    } else if (warp == kMmaWarp && lane == 0) {
      // ---------------------------------------------------------- MMA issuer (one thread)
      // Event driven: S(t) goes out as soon as K(t) has landed and softmax(t-2) has released
      // S buffer t&1; PV(t) as soon as P(t) and V(t) are ready.  p_full completions are observed
      // strictly in order per buffer (`seen`), so a parity test never aliases an older phase.
      constexpr uint32_t kIdescQK = idesc_f16(kBF16, false, BM, BN);
      constexpr uint32_t kIdescPV = idesc_f16(kBF16, true, BM, D);
      bool ok = mbar_wait(bar(L::B_QFULL), 0, abort_flag, CEA_DEV_TIMEOUT_MMA);
      int it_s = 0, it_pv = 0;  // next S and next PV, in processed-tile order
      int seen[2] = {0, 0};     // p_full completions observed, per buffer
      int kt = krange.x;        // key tile of S(it_s)
      while (kt <= krange.y && classify(qs, kst[kt], causal) == kSkip) ++kt;
      auto p_ready = [&](int t) -> bool {
        const int bb = t & 1, idx = t >> 1;
        if (seen[bb] > idx) return true;
        if (mbar_test(bar(L::B_PFULL + bb), idx & 1)) {
          seen[bb] = idx + 1;
          return true;
        }
        return false;
      };
      uint64_t t_prog = global_timer_ns();
      while (ok && (kt <= krange.y || it_pv < it_s)) {
        bool progress = false;
        if (kt <= krange.y) {
          const int st = it_s % L::NSTAGE;
          if ((it_s < 2 || p_ready(it_s - 2)) && mbar_test(bar(L::B_KFULL + st), (it_s / L::NSTAGE) & 1)) {
            tc_fence_after();
            const uint32_t tS = tmem + (it_s & 1) * BN;
            const uint32_t kbase = sbase + L::OFF_K + st * L::TILE;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * L::BOX + (kk & 3) * 32;
              umma_ss(tS, sw128_desc(sbase + L::OFF_Q + off, 16, 1024), sw128_desc(kbase + off, 16, 1024), kIdescQK,
                      kk > 0 ? 1u : 0u);
            }
            umma_commit(bar(L::B_SFULL + (it_s & 1)));
            umma_commit(bar(L::B_KEMPTY + st));
            ++it_s;
            ++kt;
            while (kt <= krange.y && classify(qs, kst[kt], causal) == kSkip) ++kt;
            progress = true;
          }
        }
        if (it_pv < it_s) {
          const int st = it_pv % L::NSTAGE;
          if (p_ready(it_pv) && mbar_test(bar(L::B_VFULL + st), (it_pv / L::NSTAGE) & 1)) {
            tc_fence_after();
            // O_{t&1} += P(t) V(t): P from shared memory (K-major over keys), V MN-major (D contiguous)
            const uint32_t pbase = sbase + L::OFF_P + (it_pv & 1) * L::PTILE;
            const uint32_t vbase = sbase + L::OFF_V + st * L::TILE;
            const uint32_t tO = tmem + 256 + (it_pv & 1) * 128;
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              const uint64_t a = sw128_desc(pbase + (kk >> 2) * L::BOX + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = sw128_desc(vbase + kk * 16 * 128, L::BOX, 1024);
              umma_ss(tO, a, bd, kIdescPV, (it_pv >= 2 || kk > 0) ? 1u : 0u);
            }
            umma_commit(bar(L::B_VEMPTY + st));
            umma_commit(bar(L::B_PVDONE + (it_pv & 1)));
            ++it_pv;
            progress = true;
          }
        }
        if (progress) {
          t_prog = global_timer_ns();
        } else if (*abort_flag) {
          ok = false;
        } else if (global_timer_ns() - t_prog > CEA_WAIT_LIMIT_NS) {
          record_error(CEA_DEV_TIMEOUT_MMA);
          *abort_flag = 1;
          ok = false;
        } else {
          __nanosleep(20);  // leave issue slots to the softmax warps sharing this SMSP
        }
      }
    }
  } else {
    // ================================================================ warpgroups 0, 1: softmax + epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;");
    const int wg = warp >> 2;        // owns the key tiles t with t % 2 == wg
    const int row = threadIdx.x & 127;  // TMEM lane == query row within the tile
    const int q_row = qt * BM + row;
    const bool row_in = q_row < p.Sq;
    const long long qpos = row_in ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(q_row) * p.qpos_ss] : -1ll;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + wg * BN + lane_base;
    const uint32_t tO = tmem + 256 + wg * 128 + lane_base;
    const int64_t* kpos_b = p.k_pos + b * p.kpos_sb;
    float m = -INFINITY;  // running max actually used as the exponent offset (log2 domain)
    float l = 0.f;        // running sum of exp2(s - m)
    int it = 0;           // key tiles processed by the CTA (both warpgroups)
    bool ok = true;
    for (int kt = krange.x; kt <= krange.y; ++kt) {
      const int cls = classify(qs, kst[kt], causal);
      if (cls == kSkip) continue;
      if ((it & 1) != wg) {
        ++it;
        continue;
      }
      if (!warp_wait(bar(L::B_SFULL + wg), (it >> 1) & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();

      // row max over the raw scores (the scale is positive, so it commutes with max); invisible keys
      // become -inf in place.  Eight independent accumulators keep the dependency chains short.
      float mx[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
      if (cls == kMasked) {
        // visibility of the tile's keys, 32 at a time (bounds the registers holding positions)
        uint32_t vis[BN / 32];
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t bits = 0u;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = kt * BN + c * 32 + e;
            const long long kp = key < p.Sk ? kpos_b[static_cast<int64_t>(key) * p.kpos_ss] : -1ll;
            bits |= (kp >= 0 && (!causal || kp <= qpos)) ? (1u << e) : 0u;
          }
          vis[c] = bits;
        }
#pragma unroll
        for (int j = 0; j < BN; ++j) {
          if (!((vis[j >> 5] >> (j & 31)) & 1u)) s[j] = __float_as_uint(-INFINITY);
          mx[j & 7] = fmaxf(mx[j & 7], __uint_as_float(s[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < BN; ++j) mx[j & 7] = fmaxf(mx[j & 7], __uint_as_float(s[j]));
      }
      const float tmax =
          fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
          p.scale_log2;
      const float m_new = fmaxf(m, tmax);
      const bool rescale = (m != -INFINITY) && (m_new > m + kRescaleThreshold);
      float alpha = 1.f;
      if (m == -INFINITY) {
        m = m_new;  // first visible key of this row for this warpgroup: its O and l are still zero
      } else if (rescale) {
        alpha = fast_exp2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;

      // P(it) goes into buffer wg, last read by PV(it-2); PV(it-2) is also the latest product in O_wg
      if (it >= 2 && !warp_wait(bar(L::B_PVDONE + wg), ((it - 2) >> 1) & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX)) {
        ok = false;
        break;
      }
      uint8_t* prow = smem + L::OFF_P + wg * L::PTILE + row * 128;
      float rs[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) rs[a] = 0.f;
      // P row = 2^(s*scale - m) as 16-bit pairs, stored 8 keys (16 B) at a time into the swizzled tile.
      // On fully visible tiles (no -inf arguments) elements 5, 6, 7 of every 8 may use the FMA pipe.
      auto emit = [&](auto use_poly) {
#pragma unroll
        for (int c = 0; c < BN / 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x0 = fmaf(__uint_as_float(s[c * 8 + 2 * e]), p.scale_log2, neg_m);
            const float x1 = fmaf(__uint_as_float(s[c * 8 + 2 * e + 1]), p.scale_log2, neg_m);
            const float p0 = (decltype(use_poly)::value && 2 * e >= 5) ? exp2_poly3(x0) : fast_exp2(x0);
            const float p1 = (decltype(use_poly)::value && 2 * e + 1 >= 5) ? exp2_poly3(x1) : fast_exp2(x1);
            rs[2 * e] += p0;
            rs[2 * e + 1] += p1;
            w[e] = pack2(p0, p1, kBF16);
          }
          const int chunk = (c & 7) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + (c >> 3) * L::BOX + chunk * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      };
      if (CEA_POLY_EXP2 && cls == kFull) {
        emit(std::true_type{});
      } else {
        emit(std::false_type{});
      }
      const float rowsum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      l += rowsum;

      if (__any_sync(0xffffffffu, rescale)) {
        // O_wg holds PV(wg), PV(wg+2), ..., PV(it-2), all complete (waited above)
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
        tmem_wait_st();
      }
      fence_async_smem();  // P stores -> visible to the tensor-core (async) proxy
      tc_fence_before();
      // one arrival per warp: 128 per-thread arrivals on one barrier are processed one by one and
      // delayed the MMA issuer by about a thousand cycles per tile
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L::B_PFULL + wg));
      ++it;
    }

    // --------------------------------------------------------------- epilogue
    // `it` is now the number of processed tiles N for both warpgroups.  Each warpgroup waits for
    // its own last PV on its own pv_done barrier: it has followed that barrier phase by phase, so
    // the parity wait cannot be satisfied by an older phase (the other warpgroup's barrier could be
    // two phases behind, where a parity wait returns at once).  After the named barrier both last
    // PVs, and with them every tcgen05 operation of the CTA (they complete in issue order), are done.
    const int N = it;
    const int n_mine = (N - wg + 1) / 2;  // tiles wg, wg+2, ... below N
    if (ok && n_mine > 0) {
      ok = warp_wait(bar(L::B_PVDONE + wg), (n_mine - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX);
      tc_fence_after();
    }
    float* lse_ptr = p.lse ? p.lse + b * p.l_sb + h * p.l_sh + static_cast<int64_t>(q_row) * p.l_ss : nullptr;
    const float lse_old = (ok && p.accumulate && row_in) ? *lse_ptr : -INFINITY;  // read before anyone writes
    asm volatile("bar.sync 1, 256;" ::: "memory");
    tc_fence_after();
    // the Q tile is dead now: the two warpgroups exchange (m, l) through it and merge exactly
    float2* ml = reinterpret_cast<float2*>(smem + L::OFF_Q);
    if (ok) ml[wg * 128 + row] = make_float2(m, l);
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const bool all_ok = ok && !*abort_flag;
    if (all_ok && !(N == 0 && p.accumulate)) {
      const float2 mine = ml[wg * 128 + row], other = ml[(wg ^ 1) * 128 + row];
      const float m0 = wg == 0 ? mine.x : other.x, l0 = wg == 0 ? mine.y : other.y;
      const float m1 = wg == 0 ? other.x : mine.x, l1 = wg == 0 ? other.y : mine.y;
      const float M = fmaxf(l0 > 0.f ? m0 : -INFINITY, l1 > 0.f ? m1 : -INFINITY);
      const float a0 = l0 > 0.f ? fast_exp2(m0 - M) : 0.f;
      const float a1 = l1 > 0.f ? fast_exp2(m1 - M) : 0.f;
      const float L = l0 * a0 + l1 * a1;
      const float inv_l = L > 0.f ? 1.f / L : 0.f;
      const float lse_row = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
      float w_old = 0.f, w_new = 1.f, lse_out = lse_row;
      if (p.accumulate && row_in) {
        const float mxl = fmaxf(lse_old, lse_row);
        if (mxl == -INFINITY) {
          lse_out = -INFINITY;
          w_old = 0.f;
          w_new = 0.f;
        } else {
          lse_out = mxl + log1pf(expf(-fabsf(lse_old - lse_row)));
          w_old = lse_old == -INFINITY ? 0.f : expf(lse_old - lse_out);
          w_new = lse_row == -INFINITY ? 0.f : expf(lse_row - lse_out);
        }
      }
      const float c0 = a0 * inv_l * w_new, c1 = a1 * inv_l * w_new;
      const bool has0 = N >= 1, has1 = N >= 2;  // accumulators that received at least one PV
      const uint32_t tO0 = tmem + 256 + lane_base, tO1 = tmem + 384 + lane_base;
      const int64_t obase = b * p.o_sb + static_cast<int64_t>(q_row) * p.o_ss + h * p.o_sh;
      // each warpgroup finishes half of the columns, 16 at a time
#pragma unroll 1
      for (int c = wg * (D / 32); c < (wg + 1) * (D / 32); ++c) {
        uint32_t o0[16], o1[16];
        if (has0) tmem_ld16(tO0 + c * 16, o0);
        if (has1) tmem_ld16(tO1 + c * 16, o1);
        tmem_wait_ld();
        float v[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          v[e] = (has0 ? __uint_as_float(o0[e]) * c0 : 0.f) + (has1 ? __uint_as_float(o1[e]) * c1 : 0.f);
        if (!row_in) continue;
        if (p.out_dtype == CEA_F32) {
          float* dst = reinterpret_cast<float*>(p.out) + obase + c * 16;
#pragma unroll
          for (int e = 0; e < 16; e += 4) {
            float4 x = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
            if (p.accumulate) {
              const float4 old = *reinterpret_cast<const float4*>(dst + e);
              x.x += old.x * w_old;
              x.y += old.y * w_old;
              x.z += old.z * w_old;
              x.w += old.w * w_old;
            }
            *reinterpret_cast<float4*>(dst + e) = x;
          }
        } else {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + obase + c * 16;
#pragma unroll
          for (int e = 0; e < 16; e += 8) {
            uint4 x;
            x.x = pack2(v[e], v[e + 1], kBF16);
            x.y = pack2(v[e + 2], v[e + 3], kBF16);
            x.z = pack2(v[e + 4], v[e + 5], kBF16);
            x.w = pack2(v[e + 6], v[e + 7], kBF16);
            *reinterpret_cast<uint4*>(dst + e) = x;
          }
        }
      }
      if (wg == 0 && row_in && lse_ptr) *lse_ptr = lse_out;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc
}  // namespace cea

// Prefill attention with log-sum-exp, two query tiles per CTA (sm_100a, tcgen05).
//
// A CTA owns two 128-row query tiles ("halves") that read the same KV head:
// two query heads of one GQA group at the same positions, or two adjacent
// query tiles of one head.  Every K/V tile is loaded once for both halves.
//   warps 0-3 / 4-7   softmax of half 0 / half 1 (one thread per row = TMEM lane)
//   warp 8            TMA producer (Q0, Q1, then a K ring and a V ring)
//   warps 10-11       idle (they complete the third warpgroup for setmaxnreg)
//   warp 9            MMA issuer, one thread:
//                       S_h = Q_h K^T           (SS form, fp32 into TMEM)
//                       O_h += P_h V            (TS form: P_h read from TMEM, V from smem)
// TMEM (512 columns): half h owns columns [256h, 256h+128) for S_h -- P_h
// (16-bit, two per column) is written over its first 64 columns once S_h has
// been read -- and [256h+128, 256h+128+D) for O_h.
//
// The MMA thread issues, per half, PV_h(previous tile) then S_h(this tile).
// tcgen05 operations of one thread complete in order, so when softmax h sees
// S_h(t) complete, PV_h(t-1) has completed too: O_h may be rescaled and the
// P_h columns rewritten without further waits.  The halves alternate, so one
// half's softmax overlaps the other half's MMAs.
//
// Registers: the softmax warpgroups raise their budget to 232 with setmaxnreg
// while the producer/MMA warpgroup drops to 40 (232 + 232 + 40 per SMSP stays
// within the 168 x 3 the launch reserves), so a softmax thread holds its whole
// S row in registers and reads TMEM with a single wait.
//
// Exponentials: ex2.approx on the MUFU pipe, except 3 of every 8 elements of
// fully visible tiles, which use exp2_poly3 on the FMA pipe (round-to-nearest
// range reduction, degree-3 least-squares fit of 2^f on [-0.5, 0.5], max
// relative error 7.5e-5 -- far below the bf16 rounding applied to P).
#pragma once

#include "attn_tc.cuh"

namespace cea {
namespace tc2 {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NUM_THREADS = 384;  // three warpgroups: softmax 0, softmax 1, producer + MMA (+2 idle)
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;

template <int D>
struct Layout {
  static constexpr int KBOX = D / 64;
  static constexpr int BOX = 128 * 128;
  static constexpr int TILE = KBOX * BOX;
  static constexpr int KST = D == 128 ? 2 : 4;
  static constexpr int VST = D == 128 ? 2 : 4;
  static constexpr int OFF_Q = 0;  // two tiles
  static constexpr int OFF_K = OFF_Q + 2 * TILE;
  static constexpr int OFF_V = OFF_K + KST * TILE;
  static constexpr int OFF_BAR = OFF_V + VST * TILE;
  static constexpr int B_QFULL = 0;
  static constexpr int B_KFULL = 1;
  static constexpr int B_KEMPTY = B_KFULL + KST;
  static constexpr int B_VFULL = B_KEMPTY + KST;
  static constexpr int B_VEMPTY = B_VFULL + VST;
  static constexpr int B_SFULL = B_VEMPTY + VST;  // x2 (per half)
  static constexpr int B_PFULL = B_SFULL + 2;     // x2
  static constexpr int B_PVDONE = B_PFULL + 2;    // x2
  static constexpr int NBAR = B_PVDONE + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = BYTES + 1024;
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct Params {
  tc::Params base;
  int pair_heads;  // 1: halves are query heads 2p, 2p+1 at one q tile; 0: q tiles 2i, 2i+1 of one head
  int nblk_q;      // CTAs along the query-tile axis
};

__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int D, bool kBF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const Params pp) {
  using L = Layout<D>;
  const tc::Params& p = pp.base;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + L::OFF_BAR + 8 * i; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (*reinterpret_cast<volatile int*>(&g_cea_status) != 0) return;

  // ---------------------------------------------------------------- work of this CTA
  int idx = blockIdx.x;
  int head[2], qt[2];
  bool active[2];
  if (pp.pair_heads) {
    const int hp = idx % (p.Hq / 2);
    idx /= (p.Hq / 2);
    head[0] = 2 * hp;
    head[1] = 2 * hp + 1;
    const int b_ = idx % p.B;
    (void)b_;
  } else {
    head[0] = head[1] = idx % p.Hq;
    idx /= p.Hq;
  }
  const int b = idx % p.B;
  idx /= p.B;
  const int blk = pp.nblk_q - 1 - idx;  // most work first
  if (pp.pair_heads) {
    qt[0] = qt[1] = blk;
  } else {
    qt[0] = 2 * blk;
    qt[1] = 2 * blk + 1;
  }
  active[0] = true;
  active[1] = qt[1] < p.nqt;
  const int kvh = p.kv_map ? p.kv_map[head[0]] : head[0] / p.group;
  const TileStat qs0 = p.qstat[b * p.nqt + qt[0]];
  const TileStat qs1 = active[1] ? p.qstat[b * p.nqt + qt[1]] : TileStat{LLONG_MAX, -1, 0, 0};
  const TileStat* kst = p.kstat + static_cast<size_t>(b) * p.nkt;
  const bool causal = p.causal != 0;
  int2 krange = p.qrange[b * p.nqt + qt[0]];
  if (active[1]) {
    const int2 r1 = p.qrange[b * p.nqt + qt[1]];
    krange = make_int2(min(krange.x, r1.x), max(krange.y, r1.y));
  }
  auto cls_of = [&](int h, int kt) -> int {
    if (!active[h]) return kSkip;
    return classify(h == 0 ? qs0 : qs1, kst[kt], causal);
  };

  if (threadIdx.x == 0) {
    mbar_init(bar(L::B_QFULL), 1);
    for (int s = 0; s < L::KST; ++s) {
      mbar_init(bar(L::B_KFULL + s), 1);
      mbar_init(bar(L::B_KEMPTY + s), 1);
    }
    for (int s = 0; s < L::VST; ++s) {
      mbar_init(bar(L::B_VFULL + s), 1);
      mbar_init(bar(L::B_VEMPTY + s), 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar(L::B_SFULL + h), 1);
      mbar_init(bar(L::B_PFULL + h), 128);
      mbar_init(bar(L::B_PVDONE + h), 1);
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
  if (warp >= 8) {
  // ==================================================================== warpgroup 2
  asm volatile("setmaxnreg.dec.sync.aligned.u32 40;");
  if (warp == kProducerWarp) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(bar(L::B_QFULL), (active[1] ? 2 : 1) * L::TILE);
      for (int h = 0; h < 2; ++h) {
        if (!active[h]) continue;
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb)
          tma_load_4d(sbase + L::OFF_Q + h * L::TILE + kb * L::BOX, &tmQ, bar(L::B_QFULL), kb * 64, qt[h] * BM,
                      head[h], b);
      }
      int u = 0;
      for (int kt = krange.x; kt <= krange.y; ++kt) {
        if (cls_of(0, kt) == kSkip && cls_of(1, kt) == kSkip) continue;
        const int ks = u % L::KST, vs = u % L::VST;
        const uint32_t kn = u / L::KST, vn = u / L::VST;
        if (kn > 0 && !mbar_wait(bar(L::B_KEMPTY + ks), (kn - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(bar(L::B_KFULL + ks), L::TILE);
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb)
          tma_load_4d(sbase + L::OFF_K + ks * L::TILE + kb * L::BOX, &tmK, bar(L::B_KFULL + ks), kb * 64, kt * BN,
                      kvh, b);
        if (vn > 0 && !mbar_wait(bar(L::B_VEMPTY + vs), (vn - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(bar(L::B_VFULL + vs), L::TILE);
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb)
          tma_load_4d(sbase + L::OFF_V + vs * L::TILE + kb * L::BOX, &tmV, bar(L::B_VFULL + vs), kb * 64, kt * BN,
                      kvh, b);
        ++u;
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescQK = idesc_f16(kBF16, false, BM, BN);
      constexpr uint32_t kIdescPV = idesc_f16(kBF16, true, BM, D);
      bool ok = mbar_wait(bar(L::B_QFULL), 0, abort_flag, CEA_DEV_TIMEOUT_MMA);
      int it[2] = {0, 0};          // S issued per half
      int pv[2] = {0, 0};          // PV issued per half
      int prev_u[2] = {-1, -1};    // union index of the tile whose PV is pending, per half
      int v_users[L::VST];         // halves still to read the V tile in each stage
#pragma unroll
      for (int s = 0; s < L::VST; ++s) v_users[s] = 0;
      auto issue_pv = [&](int h) -> bool {
        const int uu = prev_u[h];
        const int vs = uu % L::VST;
        if (!mbar_wait(bar(L::B_PFULL + h), (it[h] - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_MMA)) return false;
        if (!mbar_wait(bar(L::B_VFULL + vs), (uu / L::VST) & 1, abort_flag, CEA_DEV_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t tP = tmem + 256 * h;
        const uint32_t tO = tmem + 256 * h + 128;
        const uint32_t vbase = sbase + L::OFF_V + vs * L::TILE;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_ts(tO, tP + kk * 8, sw128_desc(vbase + kk * 16 * 128, L::BOX, 1024), kIdescPV,
                  (pv[h] > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar(L::B_PVDONE + h));
        ++pv[h];
        prev_u[h] = -1;
        if (--v_users[vs] == 0) umma_commit(bar(L::B_VEMPTY + vs));
        return true;
      };
      int u = 0;
      for (int kt = krange.x; ok && kt <= krange.y; ++kt) {
        const int c0 = cls_of(0, kt), c1 = cls_of(1, kt);
        if (c0 == kSkip && c1 == kSkip) continue;
        const int ks = u % L::KST;
        if (!mbar_wait(bar(L::B_KFULL + ks), (u / L::KST) & 1, abort_flag, CEA_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kbase = sbase + L::OFF_K + ks * L::TILE;
        for (int h = 0; h < 2; ++h) {
          // a pending PV is issued no later than the next union tile, even when this half skips
          // it: the V stage it holds is what the producer needs next
          if (prev_u[h] >= 0 && !issue_pv(h)) {
            ok = false;
            break;
          }
          if ((h == 0 ? c0 : c1) == kSkip) continue;
          const uint32_t tS = tmem + 256 * h;
          const uint32_t qbase = sbase + L::OFF_Q + h * L::TILE;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * L::BOX + (kk & 3) * 32;
            umma_ss(tS, sw128_desc(qbase + off, 16, 1024), sw128_desc(kbase + off, 16, 1024), kIdescQK,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(bar(L::B_SFULL + h));
          ++it[h];
          prev_u[h] = u;
          ++v_users[u % L::VST];
        }
        if (!ok) break;
        umma_commit(bar(L::B_KEMPTY + ks));
        ++u;
      }
      for (int h = 0; ok && h < 2; ++h)
        if (prev_u[h] >= 0) ok = issue_pv(h);
    }
  }
  } else {
    // ==================================================================== warpgroups 0, 1: softmax + epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;");
    const int h = warp >> 2;
    const int row = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + 256 * h + lane_base;
    const uint32_t tO = tmem + 256 * h + 128 + lane_base;
    const int q_row = qt[h] * BM + row;
    const bool row_in = active[h] && q_row < p.Sq;
    const long long qpos = row_in ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(q_row) * p.qpos_ss] : -1ll;
    const int64_t* kpos_b = p.k_pos + b * p.kpos_sb;
    float m = -INFINITY, l = 0.f;
    int it = 0;
    bool ok = true;
    if (active[h]) {
      for (int kt = krange.x; kt <= krange.y; ++kt) {
        const int cls = cls_of(h, kt);
        if (cls == kSkip) continue;
        if (!tc::warp_wait(bar(L::B_SFULL + h), it & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the whole S row in registers, one TMEM wait
        uint32_t r[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
        uint32_t vis_bits[BN / 32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) vis_bits[c] = 0xffffffffu;
        if (cls == kMasked) {  // overlaps the TMEM load
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t bits = 0u;
            const int kbase = kt * BN + c * 32;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int key = kbase + e;
              const long long kp = key < p.Sk ? kpos_b[static_cast<int64_t>(key) * p.kpos_ss] : -1ll;
              bits |= (kp >= 0 && (!causal || kp <= qpos)) ? (1u << e) : 0u;
            }
            vis_bits[c] = bits;
          }
        }
        tmem_wait_ld();
        // the scale is positive, so it commutes with max
        float rmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < BN; ++j)
          rmax = fmaxf(rmax, ((vis_bits[j >> 5] >> (j & 31)) & 1u) ? __uint_as_float(r[j]) : -INFINITY);
        const float tmax = rmax * p.scale_log2;
        const float m_new = fmaxf(m, tmax);
        const bool rescale = (m != -INFINITY) && (m_new > m + kRescaleThreshold);
        float alpha = 1.f;
        if (m == -INFINITY) {
          m = m_new;
        } else if (rescale) {
          alpha = fast_exp2(m - m_new);
          l *= alpha;
          m = m_new;
        }
        const float m_use = (m == -INFINITY) ? 0.f : m;
        // S_h(it) complete => PV_h(it-1) complete (in-order tcgen05): O_h is stable here
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
        }
        // P = 2^(s*scale - m) as 16-bit pairs over the first 64 S columns (already in registers)
        float rowsum = 0.f;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t pk[16];
          const uint32_t bits = vis_bits[c];
          if (cls == kFull) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float x0 = fmaf(__uint_as_float(r[c * 32 + 2 * e]), p.scale_log2, -m_use);
              const float x1 = fmaf(__uint_as_float(r[c * 32 + 2 * e + 1]), p.scale_log2, -m_use);
              // elements 5, 6, 7 of every 8 on the FMA pipe, the rest on MUFU
              const float p0 = ((2 * e) & 7) >= 5 ? exp2_poly3(x0) : fast_exp2(x0);
              const float p1 = ((2 * e + 1) & 7) >= 5 ? exp2_poly3(x1) : fast_exp2(x1);
              rowsum += p0 + p1;
              pk[e] = pack2(p0, p1, kBF16);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float x0 = ((bits >> (2 * e)) & 1u) ? fmaf(__uint_as_float(r[c * 32 + 2 * e]), p.scale_log2, -m_use)
                                                        : -INFINITY;
              const float x1 = ((bits >> (2 * e + 1)) & 1u)
                                   ? fmaf(__uint_as_float(r[c * 32 + 2 * e + 1]), p.scale_log2, -m_use)
                                   : -INFINITY;
              const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
              rowsum += p0 + p1;
              pk[e] = pack2(p0, p1, kBF16);
            }
          }
          tmem_st16(tS + c * 16, pk);
        }
        l += rowsum;
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(L::B_PFULL + h));
        ++it;
      }
    }

    // ---------------------------------------------------------------- epilogue
    if (ok && it > 0) {
      ok = tc::warp_wait(bar(L::B_PVDONE + h), (it - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX);
      tc_fence_after();
    }
    if (ok && active[h] && !(it == 0 && p.accumulate)) {
      const int hh = head[h];
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const float lse_row = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
      float w_old = 0.f, w_new = 1.f, lse_out = lse_row;
      float* lse_ptr = p.lse ? p.lse + b * p.l_sb + hh * p.l_sh + static_cast<int64_t>(q_row) * p.l_ss : nullptr;
      if (p.accumulate && row_in) {
        const float lse_old = *lse_ptr;
        const float mx = fmaxf(lse_old, lse_row);
        if (mx == -INFINITY) {
          lse_out = -INFINITY;
          w_new = 0.f;
        } else {
          lse_out = mx + log1pf(expf(-fabsf(lse_old - lse_row)));
          w_old = lse_old == -INFINITY ? 0.f : expf(lse_old - lse_out);
          w_new = lse_row == -INFINITY ? 0.f : expf(lse_row - lse_out);
        }
      }
      const float scale_new = inv_l * w_new;
      const int64_t obase = b * p.o_sb + static_cast<int64_t>(q_row) * p.o_ss + hh * p.o_sh;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (it > 0) {
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (!row_in) continue;
        if (p.out_dtype == CEA_F32) {
          float* dst = reinterpret_cast<float*>(p.out) + obase + c * 32;
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 v = make_float4(__uint_as_float(o[e]) * scale_new, __uint_as_float(o[e + 1]) * scale_new,
                                   __uint_as_float(o[e + 2]) * scale_new, __uint_as_float(o[e + 3]) * scale_new);
            if (p.accumulate) {
              const float4 old = *reinterpret_cast<const float4*>(dst + e);
              v.x += old.x * w_old;
              v.y += old.y * w_old;
              v.z += old.z * w_old;
              v.w += old.w * w_old;
            }
            *reinterpret_cast<float4*>(dst + e) = v;
          }
        } else {
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + obase + c * 32;
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 v;
            v.x = pack2(__uint_as_float(o[e]) * scale_new, __uint_as_float(o[e + 1]) * scale_new, kBF16);
            v.y = pack2(__uint_as_float(o[e + 2]) * scale_new, __uint_as_float(o[e + 3]) * scale_new, kBF16);
            v.z = pack2(__uint_as_float(o[e + 4]) * scale_new, __uint_as_float(o[e + 5]) * scale_new, kBF16);
            v.w = pack2(__uint_as_float(o[e + 6]) * scale_new, __uint_as_float(o[e + 7]) * scale_new, kBF16);
            *reinterpret_cast<uint4*>(dst + e) = v;
          }
        }
      }
      if (row_in && lse_ptr) *lse_ptr = lse_out;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace tc2
}  // namespace cea

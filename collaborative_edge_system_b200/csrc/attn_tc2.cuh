// Prefill attention with log-sum-exp, two query tiles per CTA sharing every K/V tile (sm_100a, tcgen05).
//
// A CTA owns two 128-row query tiles ("halves") that read the same KV head:
// two query heads of one GQA group at the same positions, or two adjacent
// query tiles of one head.  Each K/V tile is loaded once for both halves,
// which halves the L2-to-SM traffic of the one-tile kernel.
//   warps 0-3 / 4-7   softmax of half 0 / half 1: one thread per query row (=
//                     TMEM lane) reads S_h into registers, masks, keeps the
//                     running max/sum (log2 domain), writes P_h (16-bit pairs)
//                     into the upper 64 columns of S_h, rescales O_h in TMEM when
//                     its max grows by more than 2^8, and at the end normalises
//                     O_h and writes out/lse (merging into the stored result in
//                     accumulate mode)
//   warp 8            TMA: Q0, Q1, then the K ring
//   warp 10           TMA: the V ring
//   warps 9 / 11      MMA issuer of half 0 / half 1, one thread each:
//                       S_h(t) = Q_h K(t)^T      (SS form, fp32 into TMEM)
//                       O_h += P_h(t) V(t)       (TS form: P_h read from TMEM)
// Issuing a group of MMAs holds the issuing thread about as long as the group
// runs.  The issuers take turns, each pushing the pair PV_h(t-1), S_h(t) after
// the other half's previous pair: the tensor pipe then runs one half's pair
// while the other half's softmax runs, the softmaxes of the two halves do not
// compete, and each issuer's bookkeeping overlaps the other's MMAs.
// Both halves process every key tile that either half can see (a tile one half
// cannot see is processed as fully masked, P = 0), so both issuers release
// every K and V stage and the stage barriers count one arrival per half.
// TMEM (512 columns): half h owns [256h, 256h+128) for S_h / P_h and
// [256h+128, 256h+128+D) for O_h.  P_h(t) overlays S_h(t), so S_h(t+1) is
// issued only after PV_h(t).  tcgen05 operations of one thread execute in
// issue order, which gives both guarantees the softmax relies on: S_h(t+1)
// overwrites P_h(t) only after PV_h(t) has read it, and once S_h(t) is
// complete PV_h(t-1) is complete too, so O_h may be rescaled in place.
#pragma once

#include "cea_common.cuh"

namespace cea {
namespace tc2 {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int NUM_THREADS = 384;
constexpr int kKProducerWarp = 8;  // Q tiles and the K ring
constexpr int kMmaWarp = 9;         // MMA issuer of half 0; allocates TMEM
constexpr int kVProducerWarp = 10;  // the V ring
constexpr int kMmaWarp1 = 11;       // MMA issuer of half 1
// setmaxnreg split: softmax warpgroups 216, producers and issuers 72, drawn from the 168 registers per thread
// the launch gives (the most __launch_bounds__(384, 1) allows); the host checks the built count
constexpr int kLaunchRegs = 168;
constexpr int kRegsSoftmax = 216;
constexpr int kRegsOther = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsOther <= kLaunchRegs * NUM_THREADS, "register split");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kPCol = 64;  // P_h columns within S_h (128 keys x 16 bit = 64 columns)
constexpr float kRescaleThreshold = 8.0f;

// Instrumentation hook (no code unless a build defines it): CEA_TC2_MARK(half, event, tile).
#ifndef CEA_TC2_MARK
#define CEA_TC2_MARK(h, ev, t) ((void)0)
#endif

template <int D>
struct Layout {
  static constexpr int KBOX = D / 64;
  static constexpr int BOX = 128 * 128;
  static constexpr int TILE = KBOX * BOX;
  static constexpr int KST = D == 128 ? 3 : 5;  // K ring depth
  static constexpr int VST = D == 128 ? 2 : 5;  // V ring depth
  static constexpr int OFF_Q = 0;               // two tiles
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
  static constexpr int B_TURN = B_PVDONE + 2;     // x2: issuer h has pushed its next pair
  static constexpr int NBAR = B_TURN + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = BYTES + 1024;
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// Operands, strides and tile statistics of one launch (element strides; positions int64).
struct AttnArgs {
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
  // accumulate with a 16-bit out: the stored fp32 result is read from here instead of out (null: from out)
  const float* acc_in;
  int64_t a_sb, a_ss, a_sh;
};

// warp-uniform bounded wait: every lane waits, the warp continues only if all succeeded
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort, int code) {
  const bool ok = mbar_wait(bar, parity, abort, code);
  return __all_sync(0xffffffffu, ok);
}

struct Params {
  AttnArgs base;
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
  const AttnArgs& p = pp.base;
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
  // block -> (query block, head pair or head, batch), query blocks fastest and those with the most keys
  // first: the CTAs in flight then read the K/V of one or two KV heads, which stay in L2, instead of
  // streaming every KV head of the sequence through it at once
  // (scalars rather than 2-element arrays: a runtime index would put an array in local memory)
  int idx = blockIdx.x;
  const int blk = pp.nblk_q - 1 - idx % pp.nblk_q;
  idx /= pp.nblk_q;
  int head0, head1;
  if (pp.pair_heads) {
    const int hp = idx % (p.Hq / 2);
    idx /= (p.Hq / 2);
    head0 = 2 * hp;
    head1 = 2 * hp + 1;
  } else {
    head0 = head1 = idx % p.Hq;
    idx /= p.Hq;
  }
  const int b = idx;
  const int qt0 = pp.pair_heads ? blk : 2 * blk;
  const int qt1 = pp.pair_heads ? blk : 2 * blk + 1;
  const bool active1 = qt1 < p.nqt;  // an odd tile count leaves the last block with one half
  const int kvh = p.kv_map ? p.kv_map[head0] : head0 / p.group;
  const TileStat qs0 = p.qstat[b * p.nqt + qt0];
  const TileStat qs1 = active1 ? p.qstat[b * p.nqt + qt1] : qs0;
  const TileStat* kst = p.kstat + static_cast<size_t>(b) * p.nkt;
  const bool causal = p.causal != 0;
  int2 krange = p.qrange[b * p.nqt + qt0];
  if (active1) {
    const int2 r1 = p.qrange[b * p.nqt + qt1];
    krange = make_int2(min(krange.x, r1.x), max(krange.y, r1.y));
  }
  // class of key tile kt for half h (an inactive half skips everything)
  auto cls_of = [&](int h, int kt) -> int {
    if (h == 1 && !active1) return kSkip;
    return classify(h == 0 ? qs0 : qs1, kst[kt], causal);
  };
  auto union_needed = [&](int kt) -> bool { return cls_of(0, kt) != kSkip || cls_of(1, kt) != kSkip; };
  auto stat_needed = [&](const TileStat& ks) -> bool {
    return classify(qs0, ks, causal) != kSkip || (active1 && classify(qs1, ks, causal) != kSkip);
  };
  const uint32_t n_halves = active1 ? 2u : 1u;

  if (threadIdx.x == 0) {
    mbar_init(bar(L::B_QFULL), 1);
    for (int s = 0; s < L::KST; ++s) {
      mbar_init(bar(L::B_KFULL + s), 1);
      mbar_init(bar(L::B_KEMPTY + s), n_halves);  // released by each half's S
    }
    for (int s = 0; s < L::VST; ++s) {
      mbar_init(bar(L::B_VFULL + s), 1);
      mbar_init(bar(L::B_VEMPTY + s), n_halves);  // released by each half's PV
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar(L::B_SFULL + h), 1);
      mbar_init(bar(L::B_PFULL + h), 4);  // one arrival per softmax warp
      mbar_init(bar(L::B_PVDONE + h), 1);
      mbar_init(bar(L::B_TURN + h), 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kKProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kKProducerWarp) {
    // ================================================================ warpgroup 2
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
    if ((warp == kKProducerWarp || warp == kVProducerWarp) && lane == 0) {
      // ---------------------------------------------------------- TMA producers: Q + K ring, V ring
      const bool is_k = warp == kKProducerWarp;
      if (is_k) {
        mbar_arrive_expect_tx(bar(L::B_QFULL), (active1 ? 2 : 1) * L::TILE);
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb) {
          tma_load_4d(sbase + L::OFF_Q + kb * L::BOX, &tmQ, bar(L::B_QFULL), kb * 64, qt0 * BM, head0, b);
          if (active1)
            tma_load_4d(sbase + L::OFF_Q + L::TILE + kb * L::BOX, &tmQ, bar(L::B_QFULL), kb * 64, qt1 * BM, head1, b);
        }
      }
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      const int nst = is_k ? L::KST : L::VST;
      const int off = is_k ? L::OFF_K : L::OFF_V;
      const int b_full = is_k ? L::B_KFULL : L::B_VFULL;
      const int b_empty = is_k ? L::B_KEMPTY : L::B_VEMPTY;
      int u = 0;  // union tile: a key tile at least one half needs
      for (int kt = krange.x; kt <= krange.y; ++kt) {
        if (!union_needed(kt)) continue;
        const int st = u % nst;
        const uint32_t n = u / nst;
        if (n > 0 && !mbar_wait(bar(b_empty + st), (n - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(bar(b_full + st), L::TILE);
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb)
          tma_load_4d(sbase + off + st * L::TILE + kb * L::BOX, map, bar(b_full + st), kb * 64, kt * BN, kvh, b);
        ++u;
      }
    } else if ((warp == kMmaWarp || (warp == kMmaWarp1 && active1)) && lane == 0) {
      // ---------------------------------------------------------- MMA issuer of half h (one thread)
      // Pair j of half h is PV_h(j-1) (j >= 1) followed by S_h(j) (j < n); pairs j = 0..n.  Half 0 pushes
      // pair j after half 1 has pushed pair j-1, half 1 pushes pair j after half 0 has pushed pair j, so
      // turn_h completes once per pair and each wait below is one phase behind at most (unambiguous).
      // The statistics of the next key tile are loaded a tile ahead, so advancing never waits for an L2
      // round trip.
      const int h = warp == kMmaWarp ? 0 : 1;
      constexpr uint32_t kIdescQK = idesc_f16(kBF16, false, BM, BN);
      constexpr uint32_t kIdescPV = idesc_f16(kBF16, true, BM, D);
      const uint32_t tS = tmem + 256 * h;
      const uint32_t tP = tS + kPCol;
      const uint32_t tO = tS + 128;
      const uint64_t qdesc = sw128_desc(sbase + L::OFF_Q + h * L::TILE, 16, 1024);
      const uint64_t kdesc0 = sw128_desc(sbase + L::OFF_K, 16, 1024);
      const uint64_t vdesc0 = sw128_desc(sbase + L::OFF_V, L::BOX, 1024);
      bool ok = mbar_wait(bar(L::B_QFULL), 0, abort_flag, CEA_DEV_TIMEOUT_MMA);
      int kt = krange.x;
      TileStat cur = kt <= krange.y ? kst[kt] : qs0;
      while (kt <= krange.y && !stat_needed(cur)) {
        ++kt;
        if (kt <= krange.y) cur = kst[kt];
      }
      TileStat nxt = kt + 1 <= krange.y ? kst[kt + 1] : qs0;
      for (int j = 0; ok; ++j) {
        const bool has_s = kt <= krange.y;  // S_h(j) exists
        // what this pair needs: K(j) for S_h(j), P_h(j-1) and V(j-1) for PV_h(j-1), the other half's turn
        if (has_s && !mbar_wait(bar(L::B_KFULL + j % L::KST), (j / L::KST) & 1, abort_flag, CEA_DEV_TIMEOUT_MMA)) break;
        // P_h(j-1) and the other issuer's turn are on the critical path and usually short: poll them (a
        // thread woken from a suspended wait resumes a few hundred cycles after the phase completes)
        if (j > 0 && (!mbar_spin(bar(L::B_PFULL + h), (j - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_MMA) ||
                      !mbar_wait(bar(L::B_VFULL + (j - 1) % L::VST), ((j - 1) / L::VST) & 1, abort_flag,
                                 CEA_DEV_TIMEOUT_MMA)))
          break;
        if (active1) {
          const bool turn_ok =
              h == 0 ? (j == 0 || mbar_spin(bar(L::B_TURN + 1), (j - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_MMA))
                     : mbar_spin(bar(L::B_TURN + 0), j & 1, abort_flag, CEA_DEV_TIMEOUT_MMA);
          if (!turn_ok) break;
        }
        tc_fence_after();
        CEA_TC2_MARK(h, 4, j);
        if (j > 0) {
          const int vs = (j - 1) % L::VST;
          const uint64_t vdesc = vdesc0 + static_cast<uint64_t>((vs * L::TILE) >> 4);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_ts(tO, tP + kk * 8, vdesc + static_cast<uint64_t>((kk * 16 * 128) >> 4), kIdescPV,
                    (j > 1 || kk > 0) ? 1u : 0u);
          umma_commit(bar(L::B_PVDONE + h));
          umma_commit(bar(L::B_VEMPTY + vs));
          CEA_TC2_MARK(h, 6, j);
        }
        if (has_s) {
          const int ks = j % L::KST;
          // descriptors differ from the tile's by the start address field only (addresses stay < 256 KB)
          const uint64_t kdesc = kdesc0 + static_cast<uint64_t>((ks * L::TILE) >> 4);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * L::BOX + (kk & 3) * 32) >> 4;
            umma_ss(tS, qdesc + off, kdesc + off, kIdescQK, kk > 0 ? 1u : 0u);
          }
          umma_commit(bar(L::B_SFULL + h));
          umma_commit(bar(L::B_KEMPTY + ks));
        }
        CEA_TC2_MARK(h, 5, j);
        mbar_arrive(bar(L::B_TURN + h));
        if (!has_s) break;  // that was the last pair
        // next key tile any half can see, from the prefetched statistics
        ++kt;
        if (kt <= krange.y) {
          cur = nxt;
          while (kt <= krange.y && !stat_needed(cur)) {
            ++kt;
            if (kt <= krange.y) cur = kst[kt];
          }
          if (kt + 1 <= krange.y) nxt = kst[kt + 1];
        }
      }
    }
  } else {
    // ================================================================ warpgroups 0, 1: softmax + epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int h = warp >> 2;
    const bool active = h == 0 || active1;
    const int row = threadIdx.x & 127;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + 256 * h + lane_base;
    const uint32_t tO = tmem + 256 * h + 128 + lane_base;
    const int q_row = (h == 0 ? qt0 : qt1) * BM + row;
    const bool row_in = active && q_row < p.Sq;
    const long long qpos = row_in ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(q_row) * p.qpos_ss] : -1ll;
    const int64_t* kpos_b = p.k_pos + b * p.kpos_sb;
    float m = -INFINITY, l = 0.f;
    int it = 0;  // tiles processed by this half
    bool ok = true;
    if (active) {
      for (int kt = krange.x; kt <= krange.y; ++kt) {
        const int cls_own = cls_of(h, kt);
        const int cls_other = cls_of(h ^ 1, kt);
        if (cls_own == kSkip && cls_other == kSkip) continue;
        const int cls = cls_own == kSkip ? kMasked : cls_own;  // the other half's tile: every key masked here
        CEA_TC2_MARK(h, 3, it);
        if (!warp_wait(bar(L::B_SFULL + h), it & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX)) {
          ok = false;
          break;
        }
        tc_fence_after();
        CEA_TC2_MARK(h, 0, it);
        uint32_t s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
        tmem_wait_ld();
        float mx[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
        if (cls == kMasked) {
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
          m = m_new;
        } else if (rescale) {
          alpha = fast_exp2(m - m_new);
          l *= alpha;
          m = m_new;
        }
        const float neg_m = (m == -INFINITY) ? 0.f : -m;
        CEA_TC2_MARK(h, 1, it);
        // S_h(it) complete => PV_h(it-1) complete: O_h is stable until the first chunk of P_h(it) is
        // released, so a rescale goes first
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
        // P_h = 2^(s*scale - m) as 16-bit pairs into the upper half of S_h (S is in registers), scaled and
        // summed with packed pair arithmetic (one instruction per two keys)
        uint64_t rs2[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) rs2[a] = 0ull;
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t negm2 = f2_pack(neg_m, neg_m);
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(s[c * 32 + 2 * e]), __uint_as_float(s[c * 32 + 2 * e + 1])),
                             scale2, negm2),
                      x0, x1);
            const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
            rs2[e & 3] = f2_add(rs2[e & 3], f2_pack(p0, p1));
            pk[e] = pack2(p0, p1, kBF16);
          }
          tmem_st16(tS + kPCol + c * 16, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        // one arrival per warp: 128 per-thread arrivals on one barrier are processed one by one and
        // delayed the MMA issuer by about a thousand cycles per tile
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(L::B_PFULL + h));
        CEA_TC2_MARK(h, 2, it);
        {
          const uint64_t r = f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3]));
          float r0, r1;
          f2_unpack(r, r0, r1);
          l += r0 + r1;
        }
        ++it;
      }
    }

    // ---------------------------------------------------------------- epilogue
    // PV_h(it-1) is the last product in O_h.  S_h(it-1) completed, hence PV_h(it-2) did: pv_done_h has
    // completed it-1 or it phases, so the parity wait is unambiguous.
    if (ok && it > 0) {
      ok = warp_wait(bar(L::B_PVDONE + h), (it - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_SOFTMAX);
      tc_fence_after();
    }
    // a row that saw no key keeps its stored result, which with acc_in still has to reach out
    if (ok && active && !(it == 0 && p.accumulate && p.acc_in == nullptr)) {
      const int hh = h == 0 ? head0 : head1;
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const float lse_row = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
      float w_old = 0.f, w_new = 1.f, lse_out = lse_row;
      float* lse_ptr = p.lse ? p.lse + b * p.l_sb + hh * p.l_sh + static_cast<int64_t>(q_row) * p.l_ss : nullptr;
      if (p.accumulate && row_in) {
        const float lse_old = *lse_ptr;
        const float mxl = fmaxf(lse_old, lse_row);
        if (mxl == -INFINITY) {
          lse_out = -INFINITY;
          w_new = 0.f;
        } else {
          lse_out = mxl + log1pf(expf(-fabsf(lse_old - lse_row)));
          w_old = lse_old == -INFINITY ? 0.f : expf(lse_old - lse_out);
          w_new = lse_row == -INFINITY ? 0.f : expf(lse_row - lse_out);
        }
      }
      const float c_new = inv_l * w_new;
      const int64_t obase = b * p.o_sb + static_cast<int64_t>(q_row) * p.o_ss + hh * p.o_sh;
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t o[16];
        if (it > 0) {
          tmem_ld16(tO + c * 16, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = 0u;
        }
        if (!row_in) continue;
        if (p.out_dtype == CEA_F32) {
          float* dst = reinterpret_cast<float*>(p.out) + obase + c * 16;
#pragma unroll
          for (int e = 0; e < 16; e += 4) {
            float4 v = make_float4(__uint_as_float(o[e]) * c_new, __uint_as_float(o[e + 1]) * c_new,
                                   __uint_as_float(o[e + 2]) * c_new, __uint_as_float(o[e + 3]) * c_new);
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
          uint16_t* dst = reinterpret_cast<uint16_t*>(p.out) + obase + c * 16;
#pragma unroll
          for (int e = 0; e < 16; e += 8) {
            float f[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(o[e + j]) * c_new;
            if (p.acc_in != nullptr) {  // merge the running fp32 result and cast in one pass
              const float* src = p.acc_in + b * p.a_sb + static_cast<int64_t>(q_row) * p.a_ss + hh * p.a_sh + c * 16 + e;
              const float4 a0 = *reinterpret_cast<const float4*>(src);
              const float4 a1 = *reinterpret_cast<const float4*>(src + 4);
              f[0] += a0.x * w_old;
              f[1] += a0.y * w_old;
              f[2] += a0.z * w_old;
              f[3] += a0.w * w_old;
              f[4] += a1.x * w_old;
              f[5] += a1.y * w_old;
              f[6] += a1.z * w_old;
              f[7] += a1.w * w_old;
            }
            uint4 v;
            v.x = pack2(f[0], f[1], kBF16);
            v.y = pack2(f[2], f[3], kBF16);
            v.z = pack2(f[4], f[5], kBF16);
            v.w = pack2(f[6], f[7], kBF16);
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

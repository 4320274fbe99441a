// Split-KV decode: a few query rows per KV head against a long KV cache.
//
// The work is HBM-bound (about 4 FLOP per byte of K/V at GQA group 4), so the
// kernel is built to stream K and V once at full bandwidth:
//   * grid (split, kv head, batch); each split owns a contiguous key range;
//   * warp 4 streams 64-key K and V tiles with TMA (128B swizzle) into a
//     multi-stage shared-memory ring, so tens of KB per SM are in flight;
//   * warps 0-3 each take 16 keys of a tile: the Sq*G query rows of the KV
//     head (padded to 16) times the keys on mma.sync m16n8k16 (fp32
//     accumulate), online softmax in the log2 domain, P.V on mma.sync;
//   * the four warps merge in shared memory and write one normalised partial
//     (O, log2-sum-exp) per split; decode_combine_kernel merges the splits
//     exactly and writes out (+ natural-log lse), optionally merging into a
//     stored result.
// K/V may be strided views (e.g. token-major views of a head-major cache).
#pragma once

#include "cea_common.cuh"

namespace cea {
namespace dec {

constexpr int BKEYS = 64;
constexpr int NCW = 4;  // consumer warps, 16 keys each
constexpr int NTHREADS = (NCW + 1) * 32;
constexpr int MAX_ROWS = 16;

template <int D>
struct Layout {
  static constexpr int KBOX = D / 64;
  static constexpr int BOX = BKEYS * 128;  // 64 rows x 128 B
  static constexpr int TILE = KBOX * BOX;
  static constexpr int NSTAGE = D == 128 ? 3 : 4;
  static constexpr int STAGE = 2 * TILE;  // K tile then V tile
  static constexpr int OFF_BAR = NSTAGE * STAGE;
  static constexpr int OFF_MISC = OFF_BAR + 2 * NSTAGE * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = BYTES + 1024;
  // cross-warp merge scratch (reuses the stage ring once every tile is consumed)
  static constexpr int MERGE_BYTES = NCW * MAX_ROWS * (D + 2) * 4;
  static_assert(MERGE_BYTES <= OFF_BAR, "merge scratch fits in the ring");
};

struct Params {
  const void* q;
  int64_t q_sb, q_ss, q_sh;
  const int64_t* q_pos;
  int64_t qpos_sb, qpos_ss;
  const int64_t* k_pos;
  int64_t kpos_sb, kpos_ss;
  float* part_o;    // [B][Hq][Sq][nsplit][D], normalised
  float* part_lse;  // [B][Hq][Sq][nsplit], log2 domain
  int B, Sq, Sk, Hq, Hkv, G, nsplit, tiles_per_split;
  float scale_log2;
  int causal;
  // decode-step append: the last n_new keys come from new_k / new_v / new_pos and are written into the
  // cache views (k, v, k_pos_out) by the CTA whose key range holds them, before it reads that range
  int n_new;
  const uint16_t* new_k;
  const uint16_t* new_v;
  int64_t nk_sb, nk_ss, nk_sh, nv_sb, nv_ss, nv_sh;
  const int64_t* new_pos;
  int64_t np_sb, np_ss;
  uint16_t* k;
  uint16_t* v;
  int64_t k_sb, k_ss, k_sh, v_sb, v_ss, v_sh;
  int64_t* k_pos_out;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <bool kBF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kBF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// address of 16-byte chunk `chunk` (along D) of key row `key` inside a 128B-swizzled tile
__device__ __forceinline__ uint32_t swz(uint32_t tile, int key, int chunk) {
  return tile + (chunk >> 3) * (BKEYS * 128) + key * 128 + (((chunk & 7) ^ (key & 7)) << 4);
}

template <int D, bool kBF16>
__global__ void __launch_bounds__(NTHREADS)
    decode_partial_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const Params p) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC);
  auto full_bar = [&](int s) -> uint32_t { return sbase + L::OFF_BAR + 8 * s; };
  auto empty_bar = [&](int s) -> uint32_t { return sbase + L::OFF_BAR + 8 * (L::NSTAGE + s); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (*reinterpret_cast<volatile int*>(&g_cea_status) != 0) return;  // fail fast after a device-side timeout
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nkt = (p.Sk + BKEYS - 1) / BKEYS;
  const int t0 = split * p.tiles_per_split;
  const int t1 = min(nkt, t0 + p.tiles_per_split);
  const int k_end = min(p.Sk, t1 * BKEYS);
  const int R = p.Sq * p.G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::NSTAGE; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), NCW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // decode-step append: this CTA writes the new tokens of its key range for its KV head, and their positions,
  // into the cache, then orders those generic-proxy stores before its TMA reads of the range
  const int a0 = p.Sk - p.n_new;  // first new key
  if (p.n_new > 0 && max(a0, t0 * BKEYS) < k_end) {
    const int lo = max(a0, t0 * BKEYS);
    constexpr int CH = D / 8;  // 16-byte chunks of one K or V row
    const int units = (k_end - lo) * CH;
    for (int i = threadIdx.x; i < 2 * units; i += NTHREADS) {
      const bool is_v = i >= units;
      const int r = is_v ? i - units : i;
      const int key = lo + r / CH, c = r % CH;
      const int64_t j = key - a0;
      const uint16_t* src = is_v ? p.new_v + b * p.nv_sb + j * p.nv_ss + kvh * p.nv_sh
                                 : p.new_k + b * p.nk_sb + j * p.nk_ss + kvh * p.nk_sh;
      uint16_t* dst = is_v ? p.v + b * p.v_sb + static_cast<int64_t>(key) * p.v_ss + kvh * p.v_sh
                           : p.k + b * p.k_sb + static_cast<int64_t>(key) * p.k_ss + kvh * p.k_sh;
      reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
    }
    // every KV head's CTA stores the same positions: this CTA reads its own stores after the barrier below
    for (int key = lo + threadIdx.x; key < k_end; key += NTHREADS)
      p.k_pos_out[b * p.kpos_sb + static_cast<int64_t>(key) * p.kpos_ss] =
          p.new_pos[b * p.np_sb + static_cast<int64_t>(key - a0) * p.np_ss];
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __syncthreads();

  if (warp == NCW) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      for (int t = t0, it = 0; t < t1; ++t, ++it) {
        const int st = it % L::NSTAGE;
        const uint32_t n = it / L::NSTAGE;
        if (n > 0 && !mbar_wait(empty_bar(st), (n - 1) & 1, abort_flag, CEA_DEV_TIMEOUT_DECODE)) break;
        mbar_arrive_expect_tx(full_bar(st), 2 * L::TILE);
        const uint32_t kdst = sbase + st * L::STAGE;
#pragma unroll
        for (int kb = 0; kb < L::KBOX; ++kb) {
          tma_load_4d(kdst + kb * L::BOX, &tmK, full_bar(st), kb * 64, t * BKEYS, kvh, b);
          tma_load_4d(kdst + L::TILE + kb * L::BOX, &tmV, full_bar(st), kb * 64, t * BKEYS, kvh, b);
        }
      }
    }
    __syncthreads();  // matches the consumers' barrier before the cross-warp merge
    return;
  }

  // ------------------------------------------------------------------ consumers
  // query rows r = sq * G + g (head kvh * G + g), padded to 16; A fragments kept in registers
  const int rA = lane >> 2, rB = rA + 8;
  uint32_t qa[D / 16][4];
  {
    const uint16_t* qg = reinterpret_cast<const uint16_t*>(p.q);
    auto qword = [&](int r, int d) -> uint32_t {
      if (r >= R) return 0u;
      const int sq = r / p.G, h = kvh * p.G + r % p.G;
      const uint16_t* src = qg + b * p.q_sb + static_cast<int64_t>(sq) * p.q_ss + h * p.q_sh + d;
      return *reinterpret_cast<const uint32_t*>(src);
    };
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int d0 = kk * 16 + 2 * (lane & 3);
      qa[kk][0] = qword(rA, d0);
      qa[kk][1] = qword(rB, d0);
      qa[kk][2] = qword(rA, d0 + 8);
      qa[kk][3] = qword(rB, d0 + 8);
    }
  }
  const long long qposA = rA < R ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(rA / p.G) * p.qpos_ss] : -1ll;
  const long long qposB = rB < R ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(rB / p.G) * p.qpos_ss] : -1ll;
  const bool causal = p.causal != 0;
  const int64_t* kpos_b = p.k_pos + b * p.kpos_sb;

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

  for (int t = t0, it = 0; t < t1; ++t, ++it) {
    const int st = it % L::NSTAGE;
    const bool got = mbar_wait(full_bar(st), (it / L::NSTAGE) & 1, abort_flag, CEA_DEV_TIMEOUT_DECODE);
    if (!__all_sync(0xffffffffu, got)) break;
    const uint32_t kt = sbase + st * L::STAGE;
    const uint32_t vt = kt + L::TILE;
    const int key0 = warp * 16;  // this warp's 16 keys within the tile

    // S[16 rows x 16 keys] = Q K^T
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int key = key0 + ((mi >> 1) << 3) + ri;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(swz(kt, key, 2 * kk + (mi & 1)), b0, b1, b2, b3);
        mma16816<kBF16>(s[0], qa[kk], b0, b1);
        mma16816<kBF16>(s[1], qa[kk], b2, b3);
      }
    }
    // scale + position mask
    float tA = -INFINITY, tB = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = t * BKEYS + key0 + nt * 8 + 2 * (lane & 3) + e;
        const long long kp = key < k_end ? kpos_b[static_cast<int64_t>(key) * p.kpos_ss] : -1ll;
        const bool visA = kp >= 0 && (!causal || kp <= qposA) && rA < R;
        const bool visB = kp >= 0 && (!causal || kp <= qposB) && rB < R;
        s[nt][e] = visA ? s[nt][e] * p.scale_log2 : -INFINITY;
        s[nt][2 + e] = visB ? s[nt][2 + e] * p.scale_log2 : -INFINITY;
        tA = fmaxf(tA, s[nt][e]);
        tB = fmaxf(tB, s[nt][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, off));
      tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, off));
    }
    const float nA = fmaxf(mA, tA), nB = fmaxf(mB, tB);
    const float uA = nA == -INFINITY ? 0.f : nA, uB = nB == -INFINITY ? 0.f : nB;
    const float aA = fast_exp2(mA - uA), aB = fast_exp2(mB - uB);
    mA = nA;
    mB = nB;
    uint32_t pa[4];
    {
      float pv[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pv[nt][0] = fast_exp2(s[nt][0] - uA);
        pv[nt][1] = fast_exp2(s[nt][1] - uA);
        pv[nt][2] = fast_exp2(s[nt][2] - uB);
        pv[nt][3] = fast_exp2(s[nt][3] - uB);
      }
      lA = lA * aA + pv[0][0] + pv[0][1] + pv[1][0] + pv[1][1];
      lB = lB * aB + pv[0][2] + pv[0][3] + pv[1][2] + pv[1][3];
      pa[0] = pack2(pv[0][0], pv[0][1], kBF16);
      pa[1] = pack2(pv[0][2], pv[0][3], kBF16);
      pa[2] = pack2(pv[1][0], pv[1][1], kBF16);
      pa[3] = pack2(pv[1][2], pv[1][3], kBF16);
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= aA;
      o[i][1] *= aA;
      o[i][2] *= aB;
      o[i][3] *= aB;
    }
    // O[16 x D] += P[16 x 16 keys] V[16 keys x D]
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int key = key0 + ((mi & 1) << 3) + ri;
#pragma unroll
      for (int dn = 0; dn < D / 8; dn += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(swz(vt, key, dn + (mi >> 1)), b0, b1, b2, b3);
        mma16816<kBF16>(o[dn], pa, b0, b1);
        mma16816<kBF16>(o[dn + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(st));
  }

  // ------------------------------------------------- merge the four warps' partials
  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  __syncthreads();  // every tile consumed (and the producer idle): the ring becomes merge scratch
  float* ms = reinterpret_cast<float*>(smem);            // [NCW][16] max
  float* ls = ms + NCW * MAX_ROWS;                       // [NCW][16] sum
  float* os = ls + NCW * MAX_ROWS;                       // [NCW][16][D]
  if ((lane & 3) == 0) {
    ms[warp * MAX_ROWS + rA] = mA;
    ms[warp * MAX_ROWS + rB] = mB;
    ls[warp * MAX_ROWS + rA] = lA;
    ls[warp * MAX_ROWS + rB] = lB;
  }
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int d = i * 8 + 2 * (lane & 3);
    os[(warp * MAX_ROWS + rA) * D + d] = o[i][0];
    os[(warp * MAX_ROWS + rA) * D + d + 1] = o[i][1];
    os[(warp * MAX_ROWS + rB) * D + d] = o[i][2];
    os[(warp * MAX_ROWS + rB) * D + d + 1] = o[i][3];
  }
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));
  // thread -> (row, D/8 columns)
  const int row = threadIdx.x >> 3, part = threadIdx.x & 7;
  if (row < R) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCW; ++w) mx = fmaxf(mx, ms[w * MAX_ROWS + row]);
    const float mu = mx == -INFINITY ? 0.f : mx;
    float wsum = 0.f, wt[NCW];
#pragma unroll
    for (int w = 0; w < NCW; ++w) {
      wt[w] = fast_exp2(ms[w * MAX_ROWS + row] - mu);
      wsum += wt[w] * ls[w * MAX_ROWS + row];
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    const int sq = row / p.G, h = kvh * p.G + row % p.G;
    const int64_t prow = ((static_cast<int64_t>(b) * p.Hq + h) * p.Sq + sq) * p.nsplit + split;
    float* dst = p.part_o + prow * D;
    for (int d = part; d < D; d += 8) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) acc += wt[w] * os[(w * MAX_ROWS + row) * D + d];
      dst[d] = acc * inv;
    }
    if (part == 0) p.part_lse[prow] = wsum > 0.f ? mu + __log2f(wsum) : -INFINITY;
  }
}

struct CombineParams {
  const float* part_o;
  const float* part_lse;
  void* out;
  float* lse;
  int64_t o_sb, o_ss, o_sh, l_sb, l_sh, l_ss;
  int B, Sq, Hq, D, nsplit, out_dtype, accumulate;
};

// one warp per (b, h, sq) row: exact merge of the split partials
__global__ void decode_combine_kernel(const CombineParams c) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<int64_t>(c.B) * c.Hq * c.Sq) return;
  const int sq = wid % c.Sq;
  const int h = (wid / c.Sq) % c.Hq;
  const int b = wid / (static_cast<int64_t>(c.Sq) * c.Hq);
  const float* pl = c.part_lse + wid * c.nsplit;
  float mx = -INFINITY;
  for (int i = lane; i < c.nsplit; i += 32) mx = fmaxf(mx, pl[i]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const float mu = mx == -INFINITY ? 0.f : mx;
  float sum = 0.f;
  for (int i = lane; i < c.nsplit; i += 32) sum += exp2f(pl[i] - mu);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  const float lse_row = sum > 0.f ? (mu + log2f(sum)) * kLn2 : -INFINITY;
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  float w_old = 0.f, w_new = 1.f, lse_out = lse_row;
  float* lse_ptr = c.lse ? c.lse + b * c.l_sb + h * c.l_sh + static_cast<int64_t>(sq) * c.l_ss : nullptr;
  if (c.accumulate) {
    const float lse_old = *lse_ptr;
    const float m2 = fmaxf(lse_old, lse_row);
    if (m2 == -INFINITY) {
      lse_out = -INFINITY;
      w_new = 0.f;
    } else {
      lse_out = m2 + log1pf(expf(-fabsf(lse_old - lse_row)));
      w_old = lse_old == -INFINITY ? 0.f : expf(lse_old - lse_out);
      w_new = lse_row == -INFINITY ? 0.f : expf(lse_row - lse_out);
    }
  }
  const float* po = c.part_o + wid * c.nsplit * static_cast<int64_t>(c.D);
  const int64_t ooff = b * c.o_sb + static_cast<int64_t>(sq) * c.o_ss + h * c.o_sh;
  for (int d = lane; d < c.D; d += 32) {
    float acc = 0.f;
    for (int i = 0; i < c.nsplit; ++i) acc += exp2f(pl[i] - mu) * po[static_cast<int64_t>(i) * c.D + d];
    float v = acc * inv * w_new;
    if (c.out_dtype == CEA_F32) {
      float* dst = reinterpret_cast<float*>(c.out) + ooff + d;
      if (c.accumulate) v += *dst * w_old;
      *dst = v;
    } else if (c.out_dtype == CEA_BF16) {
      reinterpret_cast<__nv_bfloat16*>(c.out)[ooff + d] = __float2bfloat16_rn(v);
    } else {
      reinterpret_cast<__half*>(c.out)[ooff + d] = __float2half_rn(v);
    }
  }
  __syncwarp();
  if (lane == 0 && lse_ptr) *lse_ptr = lse_out;
}

}  // namespace dec
}  // namespace cea

// Attention with log-sum-exp on the CUDA cores, for the cases neither the tensor-core
// kernels nor the register-tiled fp32 kernel (attn_f32.cuh, fp32 at head dims 32/64)
// take: fp64 (the reference's own test precision), fp32 at other head dims (checked
// at 1e-4 / 1e-5), and 16-bit inputs at head dims other than 64/128.  Same masking, empty-row and accumulate semantics as the
// tcgen05 kernel; exp in the accumulation type (expf / exp).
//
// CTA = 128 threads = 16 query rows x 8 threads; keys in blocks of 32 staged
// in shared memory; each thread owns every 8th output column of its row.
#pragma once

#include "cea_common.cuh"

namespace cea {
namespace simt {

constexpr int BQ = 16;
constexpr int BK = 32;
constexpr int NT = 128;

struct Params {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  void* lse;
  const int64_t* q_pos;
  const int64_t* k_pos;
  const int32_t* kv_map;
  int64_t q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh, o_sb, o_ss, o_sh, l_sb, l_sh, l_ss;
  int64_t qpos_sb, qpos_ss, kpos_sb, kpos_ss;
  int B, Sq, Sk, Hq, Hkv, D, group;
  double scale;
  int causal, accumulate;
};

template <typename A> __device__ __forceinline__ A exp_acc(A x);
template <> __device__ __forceinline__ float exp_acc<float>(float x) { return expf(x); }
template <> __device__ __forceinline__ double exp_acc<double>(double x) { return exp(x); }
template <typename A> __device__ __forceinline__ A log_acc(A x);
template <> __device__ __forceinline__ float log_acc<float>(float x) { return logf(x); }
template <> __device__ __forceinline__ double log_acc<double>(double x) { return log(x); }
template <typename A> __device__ __forceinline__ A log1p_acc(A x);
template <> __device__ __forceinline__ float log1p_acc<float>(float x) { return log1pf(x); }
template <> __device__ __forceinline__ double log1p_acc<double>(double x) { return log1p(x); }

template <typename T, typename A> __device__ __forceinline__ A load_as(const T* p) { return static_cast<A>(to_f32<T>(*p)); }
template <> __device__ __forceinline__ double load_as<double, double>(const double* p) { return *p; }
template <> __device__ __forceinline__ float load_as<float, float>(const float* p) { return *p; }

template <typename O, typename A> __device__ __forceinline__ void store_as(O* p, A x) { *p = from_f32<O>(static_cast<float>(x)); }
template <> __device__ __forceinline__ void store_as<double, double>(double* p, double x) { *p = x; }
template <> __device__ __forceinline__ void store_as<float, float>(float* p, float x) { *p = x; }
template <> __device__ __forceinline__ void store_as<float, double>(float* p, double x) { *p = static_cast<float>(x); }

template <typename T, typename A, typename O, int DMAX>
__global__ void __launch_bounds__(NT) attn_simt_kernel(const Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  A* Qs = reinterpret_cast<A*>(smem_raw);                 // [BQ][DMAX]
  A* Ks = Qs + BQ * DMAX;                                  // [BK][DMAX + 1]
  A* Vs = Ks + BK * (DMAX + 1);                            // [BK][DMAX]
  A* Ps = Vs + BK * DMAX;                                  // [BQ][BK]
  long long* kpos_s = reinterpret_cast<long long*>(Ps + BQ * BK);  // [BK]

  const int t = threadIdx.x;
  const int r = t >> 3;  // row within the tile
  const int u = t & 7;
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int q0 = blockIdx.x * BQ;
  const int kvh = p.kv_map ? p.kv_map[h] : h / p.group;
  const int D = p.D;
  const bool causal = p.causal != 0;

  const T* qg = reinterpret_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
  const T* kg = reinterpret_cast<const T*>(p.k) + b * p.k_sb + kvh * p.k_sh;
  const T* vg = reinterpret_cast<const T*>(p.v) + b * p.v_sb + kvh * p.v_sh;

  for (int i = t; i < BQ * DMAX; i += NT) {
    const int rr = i / DMAX, d = i % DMAX;
    const int qi = q0 + rr;
    Qs[i] = (qi < p.Sq && d < D) ? load_as<T, A>(qg + static_cast<int64_t>(qi) * p.q_ss + d) : A(0);
  }
  const int qi = q0 + r;
  const bool row_in = qi < p.Sq;
  const long long qpos = row_in ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(qi) * p.qpos_ss] : -1ll;
  const A scale = static_cast<A>(p.scale);
  constexpr int NC = DMAX / 8;
  A acc[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) acc[i] = A(0);
  A m = -INFINITY, l = A(0);

  for (int k0 = 0; k0 < p.Sk; k0 += BK) {
    __syncthreads();
    for (int i = t; i < BK * DMAX; i += NT) {
      const int kk = i / DMAX, d = i % DMAX;
      const int kj = k0 + kk;
      const bool in = kj < p.Sk && d < D;
      Ks[kk * (DMAX + 1) + d] = in ? load_as<T, A>(kg + static_cast<int64_t>(kj) * p.k_ss + d) : A(0);
      Vs[kk * DMAX + d] = in ? load_as<T, A>(vg + static_cast<int64_t>(kj) * p.v_ss + d) : A(0);
    }
    if (t < BK) {
      const int kj = k0 + t;
      kpos_s[t] = kj < p.Sk ? p.k_pos[b * p.kpos_sb + static_cast<int64_t>(kj) * p.kpos_ss] : -1ll;
    }
    __syncthreads();

    A sc[BK / 8];
    A tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < BK / 8; ++j) {
      const int kk = u + 8 * j;
      A dot = A(0);
      for (int d = 0; d < D; ++d) dot += Qs[r * DMAX + d] * Ks[kk * (DMAX + 1) + d];
      const long long kp = kpos_s[kk];
      const bool vis = kp >= 0 && (!causal || kp <= qpos);
      sc[j] = vis ? dot * scale : A(-INFINITY);
      tmax = sc[j] > tmax ? sc[j] : tmax;
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      const A o = __shfl_xor_sync(0xffffffffu, tmax, off);
      tmax = o > tmax ? o : tmax;
    }
    const A m_new = tmax > m ? tmax : m;
    const A m_use = m_new == A(-INFINITY) ? A(0) : m_new;
    const A alpha = exp_acc<A>(m - m_use);  // 0 while the row has seen nothing
    A rowsum = A(0);
#pragma unroll
    for (int j = 0; j < BK / 8; ++j) {
      const A pj = exp_acc<A>(sc[j] - m_use);
      rowsum += pj;
      Ps[r * BK + u + 8 * j] = pj;
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) rowsum += __shfl_xor_sync(0xffffffffu, rowsum, off);
    l = l * alpha + rowsum;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < NC; ++i) acc[i] *= alpha;
    for (int kk = 0; kk < BK; ++kk) {
      const A pk = Ps[r * BK + kk];
#pragma unroll
      for (int i = 0; i < NC; ++i) acc[i] += pk * Vs[kk * DMAX + u + 8 * i];
    }
  }

  if (!row_in) return;
  const A lse_row = l > A(0) ? m + log_acc<A>(l) : A(-INFINITY);
  const A inv_l = l > A(0) ? A(1) / l : A(0);
  A w_old = A(0), w_new = A(1), lse_out = lse_row;
  A* lse_ptr = p.lse ? reinterpret_cast<A*>(p.lse) + b * p.l_sb + h * p.l_sh + static_cast<int64_t>(qi) * p.l_ss
                     : nullptr;
  if (p.accumulate) {
    const A lse_old = *lse_ptr;
    const A mx = lse_old > lse_row ? lse_old : lse_row;
    if (mx == A(-INFINITY)) {
      lse_out = -INFINITY;
      w_new = A(0);
    } else {
      const A diff = lse_old > lse_row ? lse_old - lse_row : lse_row - lse_old;
      lse_out = mx + log1p_acc<A>(exp_acc<A>(-diff));
      w_old = lse_old == A(-INFINITY) ? A(0) : exp_acc<A>(lse_old - lse_out);
      w_new = lse_row == A(-INFINITY) ? A(0) : exp_acc<A>(lse_row - lse_out);
    }
  }
  O* og = reinterpret_cast<O*>(p.out) + b * p.o_sb + static_cast<int64_t>(qi) * p.o_ss + h * p.o_sh;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int d = u + 8 * i;
    if (d < D) {
      A val = acc[i] * inv_l * w_new;
      if (p.accumulate) val += load_as<O, A>(og + d) * w_old;
      store_as<O, A>(og + d, val);
    }
  }
  if (u == 0 && lse_ptr) *lse_ptr = lse_out;
}

template <typename A, int DMAX>
constexpr size_t smem_bytes() {
  return sizeof(A) * (BQ * DMAX + BK * (DMAX + 1) + BK * DMAX + BQ * BK) + sizeof(long long) * BK;
}

}  // namespace simt

// ---------------------------------------------------------------------------
// per-tile position statistics (min/max valid position, padding) for the
// tcgen05 kernel's skip / full / masked decision; one warp per 128-token tile
// ---------------------------------------------------------------------------
__global__ void tile_stats_kernel(const int64_t* pos, int64_t sb, int64_t ss, int S, int ntiles, int B, int is_key,
                                  TileStat* out) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= B * ntiles) return;
  const int b = wid / ntiles, tile = wid % ntiles;
  long long lo = LLONG_MAX, hi = -1;
  int pad = 0, valid = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = tile * 128 + lane + 32 * i;
    if (s < S) {
      const long long v = pos[b * sb + static_cast<int64_t>(s) * ss];
      if (v >= 0) {
        valid = 1;
        lo = v < lo ? v : lo;
        hi = v > hi ? v : hi;
      } else {
        pad = 1;
      }
    } else if (is_key) {
      pad = 1;  // keys past the end are zero-filled by TMA and must be masked
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const long long olo = __shfl_xor_sync(0xffffffffu, lo, off);
    const long long ohi = __shfl_xor_sync(0xffffffffu, hi, off);
    lo = olo < lo ? olo : lo;
    hi = ohi > hi ? ohi : hi;
  }
  pad = __any_sync(0xffffffffu, pad);
  valid = __any_sync(0xffffffffu, valid);
  if (lane == 0) out[wid] = TileStat{lo, hi, pad, valid};
}

// ---------------------------------------------------------------------------
// per query tile, the first and last key tile it can see (one warp per tile), so
// the attention kernels do not scan the invisible causal future tile by tile
// ---------------------------------------------------------------------------
__global__ void tile_range_kernel(const TileStat* qstat, const TileStat* kstat, int nqt, int nkt, int B, int causal,
                                  int2* range) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= B * nqt) return;
  const int b = wid / nqt;
  const TileStat qs = qstat[wid];
  int first = nkt, last = -1;
  for (int kt = lane; kt < nkt; kt += 32) {
    if (classify(qs, kstat[static_cast<size_t>(b) * nkt + kt], causal != 0) != kSkip) {
      first = kt < first ? kt : first;
      last = kt > last ? kt : last;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    first = min(first, __shfl_xor_sync(0xffffffffu, first, off));
    last = max(last, __shfl_xor_sync(0xffffffffu, last, off));
  }
  if (lane == 0) range[wid] = make_int2(first, last);
}

// ---------------------------------------------------------------------------
// exact n-way merge of partial (out, lse) over disjoint key sets; one warp per row
// ---------------------------------------------------------------------------
struct MergeArgs {
  int n;
  const void* outs[CEA_MAX_MERGE];
  const void* lses[CEA_MAX_MERGE];
  void* out;
  void* lse;
  int64_t po_sb, po_ss, po_sh, pl_sb, pl_sh, pl_ss, o_sb, o_ss, o_sh, l_sb, l_sh, l_ss;
  int B, Sq, H, D;
};

constexpr int kMergeWarps = 8;  // merge_kernel is launched with 256 threads

template <typename P, typename O>
__global__ void __launch_bounds__(kMergeWarps * 32) merge_kernel(const MergeArgs a) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<int64_t>(a.B) * a.Sq * a.H) return;
  const int h = wid % a.H;
  const int s = (wid / a.H) % a.Sq;
  const int b = wid / (static_cast<int64_t>(a.H) * a.Sq);
  const int64_t loff = b * a.pl_sb + h * a.pl_sh + static_cast<int64_t>(s) * a.pl_ss;
  P li = lane < a.n ? reinterpret_cast<const P*>(a.lses[lane])[loff] : P(-INFINITY);
  P mx = li;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const P o = __shfl_xor_sync(0xffffffffu, mx, off);
    mx = o > mx ? o : mx;
  }
  P lse;
  if (mx == P(-INFINITY)) {
    lse = -INFINITY;
  } else {
    P e = lane < a.n ? simt::exp_acc<P>(li - mx) : P(0);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) e += __shfl_xor_sync(0xffffffffu, e, off);
    lse = mx + simt::log_acc<P>(e);
  }
  const P safe = lse == P(-INFINITY) ? P(0) : lse;
  // the weights go through shared memory: lanes past D leave the column loop early,
  // so no shuffle may sit inside it
  __shared__ P wsm[kMergeWarps][CEA_MAX_MERGE];
  const int wslot = threadIdx.x >> 5;
  if (lane < a.n) wsm[wslot][lane] = simt::exp_acc<P>(li - safe);
  __syncwarp();
  const int64_t ooff = b * a.po_sb + static_cast<int64_t>(s) * a.po_ss + h * a.po_sh;
  O* dst = reinterpret_cast<O*>(a.out) + b * a.o_sb + static_cast<int64_t>(s) * a.o_ss + h * a.o_sh;
  for (int d = lane; d < a.D; d += 32) {
    P acc = P(0);
    for (int i = 0; i < a.n; ++i) acc += reinterpret_cast<const P*>(a.outs[i])[ooff + d] * wsm[wslot][i];
    simt::store_as<O, P>(dst + d, acc);
  }
  // the partial lse values are all read (li) before any lane writes the merged one
  __syncwarp();
  if (lane == 0 && a.lse) reinterpret_cast<P*>(a.lse)[b * a.l_sb + h * a.l_sh + static_cast<int64_t>(s) * a.l_ss] = lse;
}

// ---------------------------------------------------------------------------
// segment copies for the Ulysses all-to-all pack / unpack
// ---------------------------------------------------------------------------
struct CopyArgs {
  int n, D, elem_bytes, vec;  // vec: 16-byte chunks are aligned everywhere
  cea_segment seg[CEA_MAX_SEGMENTS];
};

__global__ void copy_segments_kernel(const CopyArgs a) {
  const cea_segment& sg = a.seg[blockIdx.y];
  const int64_t rows = static_cast<int64_t>(sg.nb) * sg.ns * sg.nh;
  const int64_t row_bytes = static_cast<int64_t>(a.D) * a.elem_bytes;
  const int64_t units = a.vec ? row_bytes / 16 : row_bytes / a.elem_bytes;
  const int64_t total = rows * units;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / units, u = i % units;
    const int hh = row % sg.nh;
    const int ss = (row / sg.nh) % sg.ns;
    const int bb = row / (static_cast<int64_t>(sg.nh) * sg.ns);
    const int64_t so = (bb * sg.src_stride[0] + ss * sg.src_stride[1] + hh * sg.src_stride[2]) * a.elem_bytes;
    const int64_t dof = (bb * sg.dst_stride[0] + ss * sg.dst_stride[1] + hh * sg.dst_stride[2]) * a.elem_bytes;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(sg.src) + so;
    uint8_t* dst = reinterpret_cast<uint8_t*>(sg.dst) + dof;
    if (a.vec) {
      reinterpret_cast<uint4*>(dst)[u] = reinterpret_cast<const uint4*>(src)[u];
    } else if (a.elem_bytes == 2) {
      reinterpret_cast<uint16_t*>(dst)[u] = reinterpret_cast<const uint16_t*>(src)[u];
    } else if (a.elem_bytes == 4) {
      reinterpret_cast<uint32_t*>(dst)[u] = reinterpret_cast<const uint32_t*>(src)[u];
    } else {
      reinterpret_cast<uint64_t*>(dst)[u] = reinterpret_cast<const uint64_t*>(src)[u];
    }
  }
}

// out = 0 and lse = -inf for every row (attention over an empty key set)
template <typename O, typename LT>
__global__ void fill_empty_kernel(O* out, int64_t o_sb, int64_t o_ss, int64_t o_sh, LT* lse, int64_t l_sb, int64_t l_sh,
                                  int64_t l_ss, int B, int Sq, int H, int D) {
  const int64_t total = static_cast<int64_t>(B) * Sq * H;
  for (int64_t row = blockIdx.x; row < total; row += gridDim.x) {
    const int h = row % H;
    const int s = (row / H) % Sq;
    const int b = row / (static_cast<int64_t>(H) * Sq);
    O* o = out + b * o_sb + static_cast<int64_t>(s) * o_ss + h * o_sh;
    for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = O(0);
    if (threadIdx.x == 0 && lse) lse[b * l_sb + h * l_sh + static_cast<int64_t>(s) * l_ss] = LT(-INFINITY);
  }
}

}  // namespace cea

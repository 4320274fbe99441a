// fp32 attention with log-sum-exp for head dims 32 and 64 on the CUDA cores (collab_infer's config-1 precision: out
// within 1e-4 and lse within 1e-5 of the reference's fp32 computation, parallel/attention.py:163-181).
//
// Register-tiled like a CUDA-core GEMM: a CTA owns 64-row blocks of one head's queries and walks 64-key blocks
// staged in shared memory with two groups of 4 warps, the even blocks in one and the odd ones in the other (each
// group has its own K/V stages and its own online softmax; the two partial results of a row are merged exactly at
// the end).  Under a causal mask the row blocks see very different key counts, so a CTA takes two of them, the
// i-th from each end of the sequence, and every CTA has about the same work (the longest CTA otherwise sets the
// launch's duration).  In a group, thread (tr, tk) (tr = 0..15, tk = 0..7, the 8 tk of a tr in one warp) holds
// the scores of rows tr + 16i (i = 0..3) against keys tk + 8j (j = 0..7) and the output of the same rows at
// columns 4tk + 32c + e: each 16-byte shared-memory read then feeds 8 (scores) or 10.7 (output) FMAs on average
// instead of 4, which is what bounds an untiled kernel (shared-memory wavefronts).  Per block: S = Q K^T into
// registers, the position mask, the row max over the 8 threads of a row (shuffles), P = exp(S - m) into a
// transposed shared row buffer (rows of a thread contiguous), O = O alpha + P V.  Each thread keeps a partial row
// sum; the 8 parts share the row's max sequence and are added once at the end.  K/V blocks arrive by cp.async,
// two stages per group; only the key blocks a CTA can see are loaded (a pre-pass over the key positions gives the
// first and last one).
#pragma once

#include "cea_common.cuh"
#include "attn_simt.cuh"

namespace cea {
namespace f32k {

constexpr int ROWS = 64;   // query rows per CTA
constexpr int GT = 128;    // threads of a key group: 16 row groups x 8 key / column groups
constexpr int NT = 2 * GT; // two key groups: even and odd key blocks
constexpr int BK = 64;     // keys per staged block
constexpr int RI = 4;      // rows per thread (tr + 16 i)
constexpr int KJ = 8;      // keys per thread per block (tk + 8 j)
constexpr int STAGES = 2;
// CTAs along the query axis: under a causal mask two 64-row blocks each (the middle block alone when their count
// is odd), else one
__host__ __device__ constexpr int grid_x(int Sq, bool causal) {
  return causal ? ((Sq + ROWS - 1) / ROWS + 1) / 2 : (Sq + ROWS - 1) / ROWS;
}

template <int D>
struct Smem {
  static constexpr int STR = D + 4;               // padded row stride of Q, K, V (floats)
  static constexpr int PSTR = 4 * 16 + 4;         // transposed probabilities: [key][4 tr + i]
  static constexpr int Q = ROWS * STR;            // floats
  static constexpr int KV = STAGES * BK * STR;    // floats per tensor
  static constexpr int P = BK * PSTR;
  static constexpr int GROUP = 2 * KV + P;       // floats of one key group: K and V stages, probability rows
  static constexpr int X = RI * (D / 8) + 2 * RI;  // floats a thread hands over for the final merge
  static constexpr size_t BYTES = (Q + 2 * GROUP) * sizeof(float) + 2 * STAGES * BK * sizeof(long long);
  static_assert(GT * X <= KV, "the merge hand-over fits in a group's K stages");
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool in) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(in ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// simt::Params carries the same operands (element strides); p.D == D
template <int D>
__global__ void __launch_bounds__(NT, 1) attn_f32_kernel(const simt::Params p) {
  using S = Smem<D>;
  constexpr int STR = S::STR;
  constexpr int PSTR = S::PSTR;
  constexpr int DC = D / 32;  // 4-column groups per thread: columns 4 tk + 32 c + e
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int t = threadIdx.x;
  const int g = t / GT;  // key group: blocks kb0 + g, kb0 + g + 2, ...
  const int tg = t % GT;
  float* Qs = reinterpret_cast<float*>(smem_raw);  // [ROWS][STR], rows in query order
  float* Ks = Qs + S::Q + g * S::GROUP;
  float* Vs = Ks + S::KV;
  float* Pt = Vs + S::KV;  // [BK][PSTR]: probability of key j for row tr + 16 i at j * PSTR + 4 tr + i
  long long* kps = reinterpret_cast<long long*>(Qs + S::Q + 2 * S::GROUP) + g * STAGES * BK;
  float* handover = Qs + S::Q + S::GROUP;  // the odd group's K stages, once its loop is over
  __shared__ int s_range[2];
  __shared__ long long s_qmax;

  const int lane = tg & 31;
  const int tk = lane & 7;
  const int tr = (tg >> 5) * 4 + (lane >> 3);
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int kvh = p.kv_map ? p.kv_map[h] : h / p.group;
  const bool causal = p.causal != 0;
  const int nblk = (p.Sq + ROWS - 1) / ROWS;
  const int near = static_cast<int>(blockIdx.x);
  const int far = causal ? nblk - 1 - near : near;

  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && near == far) break;
    const int q0 = (pass == 0 ? far : near) * ROWS;

    // ---- this thread's rows and their positions
    long long qpos[RI];
#pragma unroll
    for (int i = 0; i < RI; ++i) {
      const int qi = q0 + tr + 16 * i;
      qpos[i] = qi < p.Sq ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(qi) * p.qpos_ss] : -1ll;
    }

    // ---- the CTA's visible key blocks: [first, last] over keys with 0 <= kpos (<= max q position when causal)
    __syncthreads();  // the previous row block's readers of the shared state are done
    if (t == 0) {
      s_range[0] = INT_MAX;
      s_range[1] = -1;
      s_qmax = -1;
    }
    __syncthreads();
    if (tk == 0) {
      long long mx = -1;
#pragma unroll
      for (int i = 0; i < RI; ++i)
        if (q0 + tr + 16 * i < p.Sq) mx = max(mx, qpos[i]);
      atomicMax(&s_qmax, mx);
    }
    __syncthreads();
    const long long qmax = s_qmax;
    {
      int first = INT_MAX, last = -1;
      const int64_t* kp = p.k_pos + b * p.kpos_sb;
      for (int j = t; j < p.Sk; j += NT) {
        const long long v = kp[static_cast<int64_t>(j) * p.kpos_ss];
        if (v >= 0 && (!causal || v <= qmax)) {
          first = min(first, j / BK);
          last = max(last, j / BK);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        first = min(first, __shfl_xor_sync(0xffffffffu, first, off));
        last = max(last, __shfl_xor_sync(0xffffffffu, last, off));
      }
      if (lane == 0) {
        atomicMin(&s_range[0], first);
        atomicMax(&s_range[1], last);
      }
    }

    // ---- the CTA's query rows into shared memory (zero past Sq)
    {
      const float* qg = reinterpret_cast<const float*>(p.q) + b * p.q_sb + h * p.q_sh;
      for (int e = t; e < ROWS * D; e += NT) {
        const int row = e / D, d = e % D;
        const int qi = q0 + row;
        Qs[row * STR + d] = qi < p.Sq ? qg[static_cast<int64_t>(qi) * p.q_ss + d] : 0.f;
      }
    }
    __syncthreads();
    const int kb0 = s_range[0], kb1 = s_range[1];

    float o[RI][4 * DC];  // o[i][4c + e]: row tr + 16 i, column 4 tk + 32 c + e
    float m[RI], l[RI];
#pragma unroll
    for (int i = 0; i < RI; ++i) {
      m[i] = -INFINITY;
      l[i] = 0.f;
#pragma unroll
      for (int d = 0; d < 4 * DC; ++d) o[i][d] = 0.f;
    }
    const float scale = static_cast<float>(p.scale);

    const float* kg = reinterpret_cast<const float*>(p.k) + b * p.k_sb + kvh * p.k_sh;
    const float* vg = reinterpret_cast<const float*>(p.v) + b * p.v_sb + kvh * p.v_sh;
    const int64_t* kpg = p.k_pos + b * p.kpos_sb;
    // block kb into stage st: BK rows x D/4 chunks of 16 bytes for K and for V; positions by BK threads
    auto load_block = [&](int kb, int st) {
      const uint32_t ks = smem_u32(Ks + st * BK * STR), vs = smem_u32(Vs + st * BK * STR);
#pragma unroll
      for (int it = 0; it < (BK * D / 4) / GT; ++it) {
        const int c = tg + it * GT;  // chunk: key row c / (D/4), 4-float column group c % (D/4)
        const int row = c / (D / 4), col = (c % (D / 4)) * 4;
        const int kj = kb * BK + row;
        const bool in = kj < p.Sk;
        const int64_t kjs = in ? kj : 0;
        const uint32_t so = static_cast<uint32_t>((row * STR + col) * sizeof(float));
        cp_async16(ks + so, kg + kjs * p.k_ss + col, in);
        cp_async16(vs + so, vg + kjs * p.v_ss + col, in);
      }
      if (tg < BK) {
        const int kj = kb * BK + tg;
        kps[st * BK + tg] = kj < p.Sk ? kpg[static_cast<int64_t>(kj) * p.kpos_ss] : -1ll;
      }
      cp_async_commit();
    };

    // this group's blocks: kb0 + g, kb0 + g + 2, ...; the group synchronises on its own named barrier
    auto group_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(GT) : "memory"); };
    // (kb0 is INT_MAX when no block is visible: no arithmetic on it then)
    const int kfirst = kb0 <= kb1 ? kb0 + g : 0, klast = kb0 <= kb1 ? kb1 : -1;
    if (kfirst <= klast) load_block(kfirst, 0);
    for (int kb = kfirst; kb <= klast; kb += 2) {
      const int st = ((kb - kfirst) >> 1) & 1;
      if (kb + 2 <= klast) {
        load_block(kb + 2, st ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      group_sync();
      const float* Kb = Ks + st * BK * STR;
      const float* Vb = Vs + st * BK * STR;
      const long long* kpb = kps + st * BK;

      // S tile: rows tr + 16 i, keys tk + 8 j
      float s[RI][KJ];
#pragma unroll
      for (int i = 0; i < RI; ++i)
#pragma unroll
        for (int j = 0; j < KJ; ++j) s[i][j] = 0.f;
#pragma unroll 4
      for (int d4 = 0; d4 < D / 4; ++d4) {
        float4 qv[RI], kv[KJ];
#pragma unroll
        for (int i = 0; i < RI; ++i) qv[i] = *reinterpret_cast<const float4*>(Qs + (tr + 16 * i) * STR + 4 * d4);
#pragma unroll
        for (int j = 0; j < KJ; ++j) kv[j] = *reinterpret_cast<const float4*>(Kb + (tk + 8 * j) * STR + 4 * d4);
#pragma unroll
        for (int i = 0; i < RI; ++i)
#pragma unroll
          for (int j = 0; j < KJ; ++j) {
            s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
            s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
            s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
            s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
          }
      }

      // mask, the row max over the row's 8 threads, probabilities into the transposed row buffer
      long long kp[KJ];
#pragma unroll
      for (int j = 0; j < KJ; ++j) kp[j] = kpb[tk + 8 * j];
#pragma unroll
      for (int i = 0; i < RI; ++i) {
        float mb = -INFINITY;
#pragma unroll
        for (int j = 0; j < KJ; ++j) {
          const bool vis = kp[j] >= 0 && (!causal || kp[j] <= qpos[i]);
          s[i][j] = vis ? s[i][j] * scale : -INFINITY;
          mb = fmaxf(mb, s[i][j]);
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        const float m_new = fmaxf(m[i], mb);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;  // a row that has seen nothing keeps p = 0
        const float alpha = expf(m[i] - m_use);                 // 0 while the row has seen nothing
        m[i] = m_new;
        float rs = 0.f;
#pragma unroll
        for (int j = 0; j < KJ; ++j) {
          const float pj = expf(s[i][j] - m_use);
          rs += pj;
          Pt[(tk + 8 * j) * PSTR + 4 * tr + i] = pj;
        }
        l[i] = l[i] * alpha + rs;  // this thread's part of the row sum
#pragma unroll
        for (int d = 0; d < 4 * DC; ++d) o[i][d] *= alpha;
      }
      __syncwarp();  // a row's probabilities come from the 8 threads of its row group, all in this warp

      // O += P V over the block's keys: 4 probabilities (one 16-byte read) x 4 DC columns per key
#pragma unroll 4
      for (int j = 0; j < BK; ++j) {
        const float4 pv = *reinterpret_cast<const float4*>(Pt + j * PSTR + 4 * tr);
        const float pr[RI] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
        for (int c = 0; c < DC; ++c) {
          const float4 vv = *reinterpret_cast<const float4*>(Vb + j * STR + 4 * tk + 32 * c);
#pragma unroll
          for (int i = 0; i < RI; ++i) {
            o[i][4 * c + 0] = fmaf(pr[i], vv.x, o[i][4 * c + 0]);
            o[i][4 * c + 1] = fmaf(pr[i], vv.y, o[i][4 * c + 1]);
            o[i][4 * c + 2] = fmaf(pr[i], vv.z, o[i][4 * c + 2]);
            o[i][4 * c + 3] = fmaf(pr[i], vv.w, o[i][4 * c + 3]);
          }
        }
      }
      group_sync();  // the stage and the row buffer are rewritten in the next iteration
    }

    // ---- the row sums (8 parts, same max sequence), then the odd group's rows merged into the even group's
#pragma unroll
    for (int i = 0; i < RI; ++i)
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], off);
    float* x = handover + tg * S::X;
    if (g == 1) {
#pragma unroll
      for (int i = 0; i < RI; ++i) {
#pragma unroll
        for (int d = 0; d < 4 * DC; ++d) x[i * 4 * DC + d] = o[i][d];
        x[RI * 4 * DC + i] = m[i];
        x[RI * 4 * DC + RI + i] = l[i];
      }
    }
    __syncthreads();
    if (g == 1) continue;  // the even group writes the rows
#pragma unroll
    for (int i = 0; i < RI; ++i) {
      const float m1 = x[RI * 4 * DC + i], l1 = x[RI * 4 * DC + RI + i];
      const float mm = fmaxf(m[i], m1);
      const float w0 = m[i] == -INFINITY ? 0.f : expf(m[i] - mm);
      const float w1 = m1 == -INFINITY ? 0.f : expf(m1 - mm);
      l[i] = l[i] * w0 + l1 * w1;
      m[i] = mm;
#pragma unroll
      for (int d = 0; d < 4 * DC; ++d) o[i][d] = o[i][d] * w0 + x[i * 4 * DC + d] * w1;
    }

    // ---- epilogue: normalisation, the optional exact merge into the stored result
#pragma unroll
    for (int i = 0; i < RI; ++i) {
      const int qi = q0 + tr + 16 * i;
      if (qi >= p.Sq) continue;
      const float lse_row = l[i] > 0.f ? m[i] + logf(l[i]) : -INFINITY;
      const float inv_l = l[i] > 0.f ? 1.f / l[i] : 0.f;
      float w_old = 0.f, w_new = 1.f, lse_out = lse_row;
      float* lse_ptr = p.lse ? reinterpret_cast<float*>(p.lse) + b * p.l_sb + h * p.l_sh +
                                   static_cast<int64_t>(qi) * p.l_ss
                             : nullptr;
      if (p.accumulate) {
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
      float* og = reinterpret_cast<float*>(p.out) + b * p.o_sb + static_cast<int64_t>(qi) * p.o_ss + h * p.o_sh;
#pragma unroll
      for (int c = 0; c < DC; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int d = 4 * tk + 32 * c + e;
          float val = o[i][4 * c + e] * inv_l * w_new;
          if (p.accumulate) val += og[d] * w_old;
          og[d] = val;
        }
      if (tk == 0 && lse_ptr) *lse_ptr = lse_out;
    }
  }  // row blocks
}

}  // namespace f32k
}  // namespace cea

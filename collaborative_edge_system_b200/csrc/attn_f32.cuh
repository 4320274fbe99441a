// fp32 attention with log-sum-exp for head dims 32 and 64 on the CUDA cores (collab_infer's config-1 precision: out
// within 1e-4 and lse within 1e-5 of the reference's fp32 computation, parallel/attention.py:163-181).
//
// CTA = 16 query rows of one head x 8 threads per row (128 threads).  Thread u of a row keeps the row of q in
// registers, scores keys u, u+8, ... of each 32-key block (whole dot products, no exchange), and owns D/8 of the
// row's output columns (32c + 4u + e): the eight threads share the row's running max (three shuffles per block),
// pass their probabilities through a small shared-memory row, and each updates only its output columns.  K/V
// blocks are staged in shared memory by cp.async, two stages, rows padded to D + 4 floats so that the 16-byte
// reads of a warp fall in distinct banks.  Only the key blocks a CTA can see are loaded: a pre-pass over the key
// positions gives the first and last block holding a visible key for any of the CTA's rows.
#pragma once

#include "cea_common.cuh"
#include "attn_simt.cuh"

namespace cea {
namespace f32k {

constexpr int ROWS = 16;         // query rows per CTA
constexpr int TPR = 8;           // threads per row
constexpr int NT = ROWS * TPR;   // 128
constexpr int BK = 32;           // keys per staged block
constexpr int KPT = BK / TPR;    // keys per thread per block
constexpr int STAGES = 2;
template <int D>
struct Smem {
  static constexpr int KSTR = D + 4;  // padded row stride of the staged K/V blocks (floats)
  static constexpr int KV = STAGES * BK * KSTR;  // floats per tensor
  static constexpr int PSTR = BK + 8;  // probability row stride (floats): the 4 rows of a warp in distinct banks
  static constexpr size_t BYTES = 2 * KV * sizeof(float) + ROWS * PSTR * sizeof(float) + STAGES * BK * sizeof(long long);
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
__global__ void __launch_bounds__(NT, 4) attn_f32_kernel(const simt::Params p) {
  constexpr int KSTR = Smem<D>::KSTR;
  constexpr int PSTR = Smem<D>::PSTR;
  constexpr int OC = D / TPR;  // output columns per thread
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* Ks = reinterpret_cast<float*>(smem_raw);
  float* Vs = Ks + Smem<D>::KV;
  float* Ps = Vs + Smem<D>::KV;  // [ROWS][PSTR]
  long long* kps = reinterpret_cast<long long*>(Ps + ROWS * PSTR);
  __shared__ int s_range[2];
  __shared__ long long s_qmax;

  const int t = threadIdx.x;
  const int r = t / TPR;
  const int u = t % TPR;
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int nblk = gridDim.x;
  const int q0 = (nblk - 1 - static_cast<int>(blockIdx.x)) * ROWS;  // the rows with the most keys start first
  const int kvh = p.kv_map ? p.kv_map[h] : h / p.group;
  const bool causal = p.causal != 0;

  const int qi = q0 + r;
  const bool row_in = qi < p.Sq;
  const long long qpos = row_in ? p.q_pos[b * p.qpos_sb + static_cast<int64_t>(qi) * p.qpos_ss] : -1ll;

  // ---- the CTA's visible key blocks: [first, last] over keys with 0 <= kpos (<= max q position when causal)
  if (t == 0) {
    s_range[0] = INT_MAX;
    s_range[1] = -1;
    s_qmax = -1;
  }
  __syncthreads();
  if (u == 0 && row_in) atomicMax(&s_qmax, qpos);
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
    if ((t & 31) == 0) {
      atomicMin(&s_range[0], first);
      atomicMax(&s_range[1], last);
    }
  }
  __syncthreads();
  const int kb0 = s_range[0], kb1 = s_range[1];

  // ---- q row into registers
  float q[D];
  {
    const float* qg = reinterpret_cast<const float*>(p.q) + b * p.q_sb + h * p.q_sh + static_cast<int64_t>(qi) * p.q_ss;
#pragma unroll
    for (int d = 0; d < D; ++d) q[d] = row_in ? qg[d] : 0.f;
  }
  float o[OC];  // o[4c + e] is output column 4 TPR c + 4u + e
#pragma unroll
  for (int d = 0; d < OC; ++d) o[d] = 0.f;
  float* prow = Ps + r * PSTR;
  float m = -INFINITY, l = 0.f;
  const float scale = static_cast<float>(p.scale);

  const float* kg = reinterpret_cast<const float*>(p.k) + b * p.k_sb + kvh * p.k_sh;
  const float* vg = reinterpret_cast<const float*>(p.v) + b * p.v_sb + kvh * p.v_sh;
  const int64_t* kpg = p.k_pos + b * p.kpos_sb;
  // block kb into stage st: 64 rows x D/4 chunks of 16 bytes for K and for V; positions by 64 threads
  auto load_block = [&](int kb, int st) {
    const uint32_t ks = smem_u32(Ks + st * BK * KSTR), vs = smem_u32(Vs + st * BK * KSTR);
#pragma unroll
    for (int i = 0; i < (BK * D / 4) / NT; ++i) {
      const int c = t + i * NT;  // chunk: key row c / (D/4), 4-float column group c % (D/4)
      const int row = c / (D / 4), col = (c % (D / 4)) * 4;
      const int kj = kb * BK + row;
      const bool in = kj < p.Sk;
      const int64_t kjs = in ? kj : 0;
      const uint32_t so = static_cast<uint32_t>((row * KSTR + col) * sizeof(float));
      cp_async16(ks + so, kg + kjs * p.k_ss + col, in);
      cp_async16(vs + so, vg + kjs * p.v_ss + col, in);
    }
    if (t < BK) {
      const int kj = kb * BK + t;
      kps[st * BK + t] = kj < p.Sk ? kpg[static_cast<int64_t>(kj) * p.kpos_ss] : -1ll;
    }
    cp_async_commit();
  };

  if (kb0 <= kb1) load_block(kb0, 0);
  for (int kb = kb0; kb <= kb1; ++kb) {
    const int st = (kb - kb0) & 1;
    if (kb < kb1) {
      load_block(kb + 1, st ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* Kb = Ks + st * BK * KSTR;
    const float* Vb = Vs + st * BK * KSTR;
    const long long* kpb = kps + st * BK;

    // scores of this thread's keys (u, u+4, ...), 16-byte reads of K rows
    float s[KPT];
#pragma unroll
    for (int i = 0; i < KPT; ++i) s[i] = 0.f;
#pragma unroll
    for (int d4 = 0; d4 < D / 4; ++d4) {
#pragma unroll
      for (int i = 0; i < KPT; ++i) {
        const float4 kv = *reinterpret_cast<const float4*>(Kb + (i * TPR + u) * KSTR + d4 * 4);
        s[i] = fmaf(q[d4 * 4 + 0], kv.x, s[i]);
        s[i] = fmaf(q[d4 * 4 + 1], kv.y, s[i]);
        s[i] = fmaf(q[d4 * 4 + 2], kv.z, s[i]);
        s[i] = fmaf(q[d4 * 4 + 3], kv.w, s[i]);
      }
    }
    float mb = -INFINITY;
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      const long long kp = kpb[i * TPR + u];
      const bool vis = kp >= 0 && (!causal || kp <= qpos);
      s[i] = vis ? s[i] * scale : -INFINITY;
      mb = fmaxf(mb, s[i]);
    }
    // the row's max over its four threads: the row's probabilities then share one reference
#pragma unroll
    for (int off = 1; off < TPR; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
    const float m_new = fmaxf(m, mb);
    const bool any = m_new != -INFINITY;  // the same for the four threads of a row
    if (any) {
      const float alpha = expf(m - m_new);  // 0 while nothing has been seen
      float rs = 0.f;
#pragma unroll
      for (int i = 0; i < KPT; ++i) {
        s[i] = expf(s[i] - m_new);
        rs += s[i];
        prow[i * TPR + u] = s[i];
      }
      l = l * alpha + rs;  // this thread's part of the row sum; the parts are added at the end
      m = m_new;
#pragma unroll
      for (int d = 0; d < OC; ++d) o[d] *= alpha;
    }
    __syncwarp();
    if (any) {
      // every key of the block, this thread's output columns 4 TPR c + 4u + e
#pragma unroll
      for (int j4 = 0; j4 < BK / 4; ++j4) {
        const float4 p4 = *reinterpret_cast<const float4*>(prow + 4 * j4);
        const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const float* vrow = Vb + (4 * j4 + jj) * KSTR + 4 * u;
#pragma unroll
          for (int c = 0; c < OC / 4; ++c) {
            const float4 vv = *reinterpret_cast<const float4*>(vrow + 4 * TPR * c);
            o[4 * c + 0] = fmaf(pj[jj], vv.x, o[4 * c + 0]);
            o[4 * c + 1] = fmaf(pj[jj], vv.y, o[4 * c + 1]);
            o[4 * c + 2] = fmaf(pj[jj], vv.z, o[4 * c + 2]);
            o[4 * c + 3] = fmaf(pj[jj], vv.w, o[4 * c + 3]);
          }
        }
      }
    }
    __syncthreads();  // the stage is overwritten by the load issued in the next iteration
  }

  // ---- the row sum: the four threads' parts, scaled alike
#pragma unroll
  for (int off = 1; off < TPR; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  const float M = m;
  if (!row_in) return;

  const float lse_row = l > 0.f ? M + logf(l) : -INFINITY;
  const float inv_l = l > 0.f ? 1.f / l : 0.f;
  float w_old = 0.f, w_new = 1.f, lse_out = lse_row;
  float* lse_ptr = p.lse ? reinterpret_cast<float*>(p.lse) + b * p.l_sb + h * p.l_sh + static_cast<int64_t>(qi) * p.l_ss
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
  for (int c = 0; c < OC / 4; ++c) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = 4 * TPR * c + 4 * u + e;
      float val = o[4 * c + e] * inv_l * w_new;
      if (p.accumulate) val += og[d] * w_old;
      og[d] = val;
    }
  }
  if (u == 0 && lse_ptr) *lse_ptr = lse_out;
}

}  // namespace f32k
}  // namespace cea

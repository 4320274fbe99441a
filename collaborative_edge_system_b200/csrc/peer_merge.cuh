// All-gather and exact merge of the distributed-KV decode partials in one kernel, over peer memory.
//
// Every rank owns a receive buffer of 2 parities x n slots x R rows x W floats (a row: the partial output in
// columns [0, D), its log-sum-exp in column D, padding to W) and n 64-bit counters, one per sending rank; each
// rank maps every peer's buffer and counters (CUDA IPC, NVLink P2P).  Call e (1, 2, ...) on these buffers uses
// parity e & 1.  The local decode kernel has already written this rank's partial into its own slot; this
// kernel then
//   1. stores that slot into the same slot of every peer's buffer (plain P2P stores, 16 bytes at a time),
//   2. after a system-scope fence, adds 1 to its counter in every peer's counter array (one add per CTA),
//   3. waits, with a bounded spin, until every peer's counter in its own array reaches grid * e, and
//   4. merges the n slots of every row exactly (log-sum-exp weights), writing the output in the caller's dtype.
// A wait that runs out (limit_ns) records CEA_DEV_TIMEOUT_PEER (device error word and the optional fault flag)
// and its CTA writes NaN into the output rows it owns, so a caller never reads stale or partial data.
// A slot of parity p is rewritten by call e + 2 only after the writer has merged call e + 1, which needed this
// rank's push of call e + 1, issued after this rank finished merging call e: no call overwrites data a peer
// may still read.  The grid is small enough to be resident at once on every GPU, so the CTAs waiting in step 3
// never keep this rank's other CTAs from pushing.
#pragma once

#include "attn_simt.cuh"

namespace cea {
namespace peer {

constexpr int kThreads = 256;
constexpr int kGrid = 64;  // CTAs per call: resident at once, one warp per row in the merge

struct Args {
  int n, rank, par;
  float* bufs[CEA_MAX_PEERS];                  // rank q's receive buffer, as mapped in this process
  unsigned long long* flags[CEA_MAX_PEERS];    // rank q's counters [n], as mapped in this process
  unsigned long long target;                   // kGrid * call number
  int64_t rows;                                // B * Sq * H
  int W, D, B, Sq, H;
  void* out;
  int64_t o_sb, o_ss, o_sh;
  int* fault_flag;               // optional, device-visible: CEA_DEV_TIMEOUT_PEER after a timeout
  unsigned long long limit_ns;   // bound of the wait for the peers
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename O>
__global__ void __launch_bounds__(kThreads) peer_merge_kernel(const Args a) {
  __shared__ int give_up;
  const int64_t slot_floats = a.rows * a.W;
  // ---- 1. push this rank's slot to every peer (float4: W is a multiple of 4, slots are 16-byte aligned)
  {
    const int64_t base = (static_cast<int64_t>(a.par) * a.n + a.rank) * slot_floats;
    const float4* src = reinterpret_cast<const float4*>(a.bufs[a.rank] + base);
    const int64_t nvec = slot_floats / 4;
    const int64_t lo = nvec * blockIdx.x / gridDim.x, hi = nvec * (blockIdx.x + 1) / gridDim.x;
    for (int q = 0; q < a.n; ++q) {
      if (q == a.rank) continue;
      float4* dst = reinterpret_cast<float4*>(a.bufs[q] + base);
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = src[i];
    }
  }
  __syncthreads();
  // ---- 2. signal: this CTA's part has landed in every peer
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < a.n; ++q)
      if (q != a.rank) atomicAdd_system(a.flags[q] + a.rank, 1ull);
    // ---- 3. wait for every peer's pushes into this rank's buffer (bounded)
    give_up = 0;
    const uint64_t t0 = global_timer_ns();
    for (int q = 0; q < a.n && !give_up; ++q) {
      if (q == a.rank) continue;
      uint32_t polls = 0;
      while (ld_acquire_sys(a.flags[a.rank] + q) < a.target) {
        if ((++polls & 255u) == 0 && global_timer_ns() - t0 > a.limit_ns) {
          record_error(CEA_DEV_TIMEOUT_PEER);
          if (a.fault_flag != nullptr) {
            atomicExch_system(a.fault_flag, CEA_DEV_TIMEOUT_PEER);
            __threadfence_system();
          }
          give_up = 1;
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  // ---- 4. exact merge of the n slots, one warp per row (after a timeout: NaN rows, never stale data)
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const float* mine = a.bufs[a.rank] + static_cast<int64_t>(a.par) * a.n * slot_floats;
  if (give_up) {
    for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; row < a.rows;
         row += warps) {
      const int h = row % a.H;
      const int s = (row / a.H) % a.Sq;
      const int b = row / (static_cast<int64_t>(a.H) * a.Sq);
      O* dst = reinterpret_cast<O*>(a.out) + b * a.o_sb + static_cast<int64_t>(s) * a.o_ss + h * a.o_sh;
      for (int d = lane; d < a.D; d += 32) simt::store_as<O, float>(dst + d, __int_as_float(0x7fc00000));
    }
    return;
  }
  for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; row < a.rows;
       row += warps) {
    const float li = lane < a.n ? mine[lane * slot_floats + row * a.W + a.D] : -INFINITY;
    float mx = li;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    // the weights follow merge_kernel's arithmetic exactly (lse = max + log sum, w = exp(l - lse)), so this
    // path and the all-gather + merge_kernel path give identical results
    float lse = -INFINITY;
    if (mx != -INFINITY) {
      float e = lane < a.n ? simt::exp_acc<float>(li - mx) : 0.f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) e += __shfl_xor_sync(0xffffffffu, e, off);
      lse = mx + simt::log_acc<float>(e);
    }
    const float safe = lse == -INFINITY ? 0.f : lse;
    const float wi = lane < a.n ? simt::exp_acc<float>(li - safe) : 0.f;
    // every lane takes all n weights while the warp is converged: lanes leave the column loop at different
    // times when D is not a multiple of 32, so no shuffle may sit inside it
    float w[CEA_MAX_PEERS];
#pragma unroll
    for (int q = 0; q < CEA_MAX_PEERS; ++q) w[q] = __shfl_sync(0xffffffffu, wi, q);
    const int h = row % a.H;
    const int s = (row / a.H) % a.Sq;
    const int b = row / (static_cast<int64_t>(a.H) * a.Sq);
    O* dst = reinterpret_cast<O*>(a.out) + b * a.o_sb + static_cast<int64_t>(s) * a.o_ss + h * a.o_sh;
    for (int d = lane; d < a.D; d += 32) {
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q < CEA_MAX_PEERS; ++q)
        if (q < a.n) acc += mine[q * slot_floats + row * a.W + d] * w[q];
      simt::store_as<O, float>(dst + d, acc);
    }
  }
}

}  // namespace peer
}  // namespace cea

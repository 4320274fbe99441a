// KV-cache append: token-major k/v [B, n, H, D] into head-major cache buffers [B, H, cap, D] at token slots
// offset .. offset + n - 1, and positions [B, n] into the cache's [B, cap], all in one launch.
//
// Pure data movement, HBM-bound: every (b, s, h) row of D elements is contiguous in the source and in the
// cache, so each thread moves 16-byte units (or the widest unit that divides every row start), consecutive
// threads walking along a source row, then along h, then s, then b.  blockIdx.y selects the tensor (0: k,
// 1: v, 2: positions), so the three copies share one launch.  Each thread issues kUnroll independent loads
// before its stores, and the flat unit index is split into (b, s, h, unit) with multiply-high divisions by
// the invariant row sizes (Granlund & Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994, section 4), so the per-unit index arithmetic stays a handful of instructions.
#pragma once

#include <cstdint>

namespace cea {
namespace kvc {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// n / d for any 32-bit n and a fixed divisor d >= 1: with l = ceil(log2 d) and
// m = floor(2^32 * (2^l - d) / d) + 1, t = mulhi(m, n) gives n / d = (t + ((n - t) >> 1)) >> (l - 1) when
// l >= 1; d = 1 (l = 0) returns n.
struct FastDiv {
  uint32_t d, m;
  int l;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f{d, 0u, 0};
  int l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  f.l = l;
  f.m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  if (f.l == 0) return n;  // d == 1
  const uint32_t t = __umulhi(f.m, n);
  return (t + ((n - t) >> 1)) >> (f.l - 1);
}

struct Tensor {
  const uint8_t* src;
  uint8_t* dst;
  int64_t src_stride[3];  // bytes: b, s, h
  int64_t dst_stride[3];  // bytes: b, t, h
  FastDiv units;          // units per row
  FastDiv H;              // heads
  FastDiv per_b;          // n * H * units: units per sequence
  uint32_t total;         // B * per_b (host guarantees < 2^31)
  int unit;               // bytes per unit: 16, 8, 4, 2 or 1
};

struct Args {
  Tensor t[2];
  const int64_t* pos_src;
  int64_t* pos_dst;
  int64_t ps_b, ps_s, pd_b, pd_t;  // elements
  int B, n;
  int64_t offset;
};

template <typename U>
__device__ __forceinline__ void unit_addrs(const Tensor& t, uint32_t i, int64_t offset, const U*& src, U*& dst) {
  const uint32_t b = fdiv(i, t.per_b);
  uint32_t r = i - b * t.per_b.d;
  const uint32_t row = fdiv(r, t.units);
  const uint32_t u = r - row * t.units.d;
  const uint32_t s = fdiv(row, t.H);
  const uint32_t h = row - s * t.H.d;
  src = reinterpret_cast<const U*>(t.src + b * t.src_stride[0] + s * t.src_stride[1] + h * t.src_stride[2]) + u;
  dst = reinterpret_cast<U*>(t.dst + b * t.dst_stride[0] + (offset + s) * t.dst_stride[1] + h * t.dst_stride[2]) + u;
}

template <typename U>
__device__ __forceinline__ void copy_rows(const Tensor& t, int64_t offset) {
  const uint32_t step = gridDim.x * kThreads * kUnroll;
  for (uint32_t base = blockIdx.x * kThreads * kUnroll + threadIdx.x; base < t.total; base += step) {
    U val[kUnroll];
    U* dst[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const uint32_t i = base + j * kThreads;
      dst[j] = nullptr;
      if (i < t.total) {
        const U* src;
        unit_addrs<U>(t, i, offset, src, dst[j]);
        val[j] = __ldg(src);
      }
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j)
      if (dst[j]) *dst[j] = val[j];
  }
}

__global__ void __launch_bounds__(kThreads) kv_append_kernel(const Args a) {
  if (blockIdx.y == 2) {
    const int64_t total = static_cast<int64_t>(a.B) * a.n;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t b = i / a.n, s = i % a.n;
      a.pos_dst[b * a.pd_b + (a.offset + s) * a.pd_t] = a.pos_src[b * a.ps_b + s * a.ps_s];
    }
    return;
  }
  const Tensor& t = a.t[blockIdx.y];
  switch (t.unit) {  // uniform over the block
    case 16: copy_rows<uint4>(t, a.offset); break;
    case 8: copy_rows<uint2>(t, a.offset); break;
    case 4: copy_rows<uint32_t>(t, a.offset); break;
    case 2: copy_rows<uint16_t>(t, a.offset); break;
    default: copy_rows<uint8_t>(t, a.offset); break;
  }
}

}  // namespace kvc
}  // namespace cea

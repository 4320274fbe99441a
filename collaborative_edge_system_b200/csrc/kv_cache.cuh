// KV-cache append: token-major k/v [B, n, H, D] into head-major cache buffers [B, H, cap, D] at token slots
// offset .. offset + n - 1, and positions [B, n] into the cache's [B, cap], all in one launch.
//
// Pure data movement, HBM-bound: every (b, s, h) row of D elements is contiguous in the source and in the
// cache, so each thread moves one 16-byte unit (or the widest unit that divides every row start) and a warp
// covers whole rows; consecutive threads walk along a source row, then along h, then s, then b.  blockIdx.y
// selects the tensor (0: k, 1: v, 2: positions), so the three copies share one launch.
#pragma once

#include <cstdint>

namespace cea {
namespace kvc {

struct Tensor {
  const uint8_t* src;
  uint8_t* dst;
  int64_t src_stride[3];  // bytes: b, s, h
  int64_t dst_stride[3];  // bytes: b, t, h
  int H;
  int units;  // units per row
  int unit;   // bytes per unit: 16, 8, 4, 2 or 1
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
__device__ __forceinline__ void copy_rows(const Tensor& t, int B, int n, int64_t offset) {
  const uint32_t units = static_cast<uint32_t>(t.units);
  const uint32_t per_b = static_cast<uint32_t>(n) * t.H * units;  // host guarantees < 2^31
  const uint32_t H = static_cast<uint32_t>(t.H);
  const int64_t total = static_cast<int64_t>(per_b) * B;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / per_b;
    uint32_t r = static_cast<uint32_t>(i - b * per_b);
    const uint32_t u = r % units;
    r /= units;
    const uint32_t h = r % H;
    const uint32_t s = r / H;
    const U* src = reinterpret_cast<const U*>(t.src + b * t.src_stride[0] + s * t.src_stride[1] + h * t.src_stride[2]);
    U* dst = reinterpret_cast<U*>(t.dst + b * t.dst_stride[0] + (offset + s) * t.dst_stride[1] + h * t.dst_stride[2]);
    dst[u] = src[u];
  }
}

__global__ void __launch_bounds__(256) kv_append_kernel(const Args a) {
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
    case 16: copy_rows<uint4>(t, a.B, a.n, a.offset); break;
    case 8: copy_rows<uint2>(t, a.B, a.n, a.offset); break;
    case 4: copy_rows<uint32_t>(t, a.B, a.n, a.offset); break;
    case 2: copy_rows<uint16_t>(t, a.B, a.n, a.offset); break;
    default: copy_rows<uint8_t>(t, a.B, a.n, a.offset); break;
  }
}

}  // namespace kvc
}  // namespace cea

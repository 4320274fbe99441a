// Ring wire pack / unpack: two [B, S, H, D] tensors (K and V, any b/s/h strides, D contiguous) copied into two
// destination tensors with a dtype conversion in the same pass.  Packing writes the K||V message of one ring step
// in the wire dtype (a narrower float when the communicator compresses), unpacking widens a received message
// back to the compute dtype.  Conversions follow torch's: float64 goes through float32 first, float32 to
// bfloat16 / float16 rounds to nearest even, and a float16 wire saturates at +-65504 instead of overflowing.
// HBM-bound; one thread per element group of kVec consecutive elements of a row.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace cea {
namespace wire {

constexpr int kThreads = 256;
constexpr int kVec = 4;

struct Args {
  const void* src[2];
  void* dst[2];
  int64_t src_stride[2][3];  // elements: b, s, h of each tensor
  int64_t dst_stride[2][3];
  int B, S, H, D;
};

template <typename T>
__device__ __forceinline__ float widen(T x);
template <>
__device__ __forceinline__ float widen<float>(float x) { return x; }
template <>
__device__ __forceinline__ float widen<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float widen<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename O>
__device__ __forceinline__ O narrow(float x);
template <>
__device__ __forceinline__ float narrow<float>(float x) { return x; }
// saturating: +-inf and out-of-range values become +-65504 (torch's clamp); NaN stays NaN
template <>
__device__ __forceinline__ __half narrow<__half>(float x) {
  return __float2half_rn(x > 65504.f ? 65504.f : (x < -65504.f ? -65504.f : x));
}
template <>
__device__ __forceinline__ __nv_bfloat16 narrow<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename I, typename O>
__device__ __forceinline__ O convert(I x) {
  return narrow<O>(widen<I>(x));
}
// same type: an exact copy (no saturation of a float16 infinity)
template <>
__device__ __forceinline__ __half convert<__half, __half>(__half x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 convert<__nv_bfloat16, __nv_bfloat16>(__nv_bfloat16 x) { return x; }
template <>
__device__ __forceinline__ float convert<float, float>(float x) { return x; }
// float64 sources: through float32 (torch's double -> half / bfloat16 path); float64 destinations: exact widening
template <>
__device__ __forceinline__ __half convert<double, __half>(double x) { return narrow<__half>(static_cast<float>(x)); }
template <>
__device__ __forceinline__ __nv_bfloat16 convert<double, __nv_bfloat16>(double x) {
  return narrow<__nv_bfloat16>(static_cast<float>(x));
}
template <>
__device__ __forceinline__ float convert<double, float>(double x) { return static_cast<float>(x); }
template <>
__device__ __forceinline__ double convert<double, double>(double x) { return x; }
template <>
__device__ __forceinline__ double convert<float, double>(float x) { return x; }
template <>
__device__ __forceinline__ double convert<__half, double>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ double convert<__nv_bfloat16, double>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename I, typename O>
__global__ void __launch_bounds__(kThreads) wire_cast_kernel(const Args a) {
  const int t = blockIdx.y;
  const I* src = reinterpret_cast<const I*>(a.src[t]);
  O* dst = reinterpret_cast<O*>(a.dst[t]);
  const int64_t* ss = a.src_stride[t];
  const int64_t* ds = a.dst_stride[t];
  const int groups = (a.D + kVec - 1) / kVec;
  const int64_t total = static_cast<int64_t>(a.B) * a.S * a.H * groups;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    int64_t row = i / groups;
    const int h = static_cast<int>(row % a.H);
    row /= a.H;
    const int s = static_cast<int>(row % a.S);
    const int b = static_cast<int>(row / a.S);
    const I* sp = src + b * ss[0] + s * ss[1] + h * ss[2];
    O* dp = dst + b * ds[0] + s * ds[1] + h * ds[2];
    const int d0 = g * kVec;
#pragma unroll
    for (int j = 0; j < kVec; ++j)
      if (d0 + j < a.D) dp[d0 + j] = convert<I, O>(sp[d0 + j]);
  }
}

}  // namespace wire
}  // namespace cea

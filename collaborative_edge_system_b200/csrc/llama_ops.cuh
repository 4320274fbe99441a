// The elementwise and row-wise steps of a LLaMA-family decoder layer around the attention (collab_infer
// models/llama.py): residual add + RMSNorm, rotary embedding applied in place to the q / k views of the fused
// QKV projection, and the SwiGLU activation.  All are HBM-bound; each rounds to the model dtype exactly where the
// reference's tensor expressions do (every torch op rounds its result to its dtype), so the fused kernels give
// the same values as the sequence of reference ops up to the last bit of the transcendental functions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace cea {
namespace llama {

constexpr int kNormThreads = 256;
constexpr int kEltThreads = 256;

template <typename T>
struct Acc {
  using type = float;
};
template <>
struct Acc<double> {
  using type = double;
};

template <typename T>
__device__ __forceinline__ typename Acc<T>::type up(T x) {
  return static_cast<typename Acc<T>::type>(x);
}
template <>
__device__ __forceinline__ float up<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float up<__half>(__half x) {
  return __half2float(x);
}

template <typename T>
__device__ __forceinline__ T down(typename Acc<T>::type x) {
  return static_cast<T>(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 down<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ __half down<__half>(float x) {
  return __float2half_rn(x);
}

// the value of x after a torch op rounds it to T
template <typename T>
__device__ __forceinline__ typename Acc<T>::type rnd(typename Acc<T>::type x) {
  return up<T>(down<T>(x));
}

__device__ __forceinline__ float rsqrt_acc(float x) { return rsqrtf(x); }
__device__ __forceinline__ double rsqrt_acc(double x) { return rsqrt(x); }
__device__ __forceinline__ float exp_acc(float x) { return expf(x); }
__device__ __forceinline__ double exp_acc(double x) { return exp(x); }
__device__ __forceinline__ void sincos_acc(float x, float* s, float* c) { sincosf(x, s, c); }
__device__ __forceinline__ void sincos_acc(double x, double* s, double* c) { sincos(x, s, c); }

// ---------------------------------------------------------------------------------------- residual + RMSNorm
// resid <- round(resid + delta) (when delta is given); y = round(w * round(r * resid)), r = rsqrt(mean(resid^2)
// + eps) in the accumulation type (models/llama.py:52-61 and the residual adds of DecoderLayer.forward, :337-339).
// One CTA per row; rows are contiguous in their last dimension.
struct NormArgs {
  void* resid;
  const void* delta;  // may be null
  const void* weight;
  void* y;
  int64_t rows, h;
  int64_t resid_stride, delta_stride, y_stride;  // elements between rows
  double eps;
};

template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(const NormArgs a) {
  using A = typename Acc<T>::type;
  __shared__ A red[kNormThreads / 32];
  __shared__ A total;
  T* resid = reinterpret_cast<T*>(a.resid);
  const T* delta = reinterpret_cast<const T*>(a.delta);
  const T* w = reinterpret_cast<const T*>(a.weight);
  T* y = reinterpret_cast<T*>(a.y);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    T* xr = resid + row * a.resid_stride;
    const T* dr = delta ? delta + row * a.delta_stride : nullptr;
    A ss = 0;
    for (int64_t i = threadIdx.x; i < a.h; i += blockDim.x) {
      A v = up<T>(xr[i]);
      if (dr) {
        v = rnd<T>(v + up<T>(dr[i]));
        xr[i] = down<T>(v);
      }
      ss += v * v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      A t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : A(0);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      if (threadIdx.x == 0) total = rsqrt_acc(t / static_cast<A>(a.h) + static_cast<A>(a.eps));
    }
    __syncthreads();
    const A r = total;
    T* yr = y + row * a.y_stride;
    for (int64_t i = threadIdx.x; i < a.h; i += blockDim.x) {
      const A hn = rnd<T>(up<T>(xr[i]) * r);
      yr[i] = down<T>(up<T>(w[i]) * hn);
    }
    __syncthreads();  // red / total are reused by the next row
  }
}

// ---------------------------------------------------------------------------------------------- rotary
// x <- x * cos + rotate_half(x) * sin for q [B, S, Hq, D] and k [B, S, Hk, D] (any b/s/h strides, D contiguous),
// with cos / sin of max(pos, 0) * inv_freq rounded to T (models/llama.py:64-88); rope_token_kernel below.
struct RopeArgs {
  void* x[2];
  int64_t stride[2][3];  // b, s, h
  int H[2];
  const int64_t* pos;
  int64_t pos_stride[2];
  const void* inv_freq;  // D/2 values, float (or double for a float64 model)
  int B, S, D;
};

// ---------------------------------------------------------------------------------------------- SwiGLU
// out = round(round(silu(gate)) * up), silu(g) = g / (1 + exp(-g)) in the accumulation type (models/llama.py:301-305);
// gate and up are the two halves of the fused gate_up projection, rows of gate_up_stride elements.
struct SiluArgs {
  const void* gate;
  const void* upv;
  void* out;
  int64_t rows, n;
  int64_t in_stride, out_stride;
};

template <typename T>
__global__ void __launch_bounds__(kEltThreads) silu_mul_kernel(const SiluArgs a) {
  using A = typename Acc<T>::type;
  const T* g = reinterpret_cast<const T*>(a.gate);
  const T* u = reinterpret_cast<const T*>(a.upv);
  T* o = reinterpret_cast<T*>(a.out);
  const int64_t total = a.rows * a.n;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / a.n, c = i % a.n;
    const A gv = up<T>(g[r * a.in_stride + c]);
    const A act = rnd<T>(gv / (A(1) + exp_acc(-gv)));
    o[r * a.out_stride + c] = down<T>(act * up<T>(u[r * a.in_stride + c]));
  }
}

// ------------------------------------------------------------------------------- vectorised forms
// The same arithmetic on 16-byte vectors (VecN<T> elements), used when every row start and stride is 16-byte
// aligned and the row length is a multiple of the vector; the kernels above serve the other shapes.
template <typename T>
struct VecN {
  static constexpr int N = 16 / static_cast<int>(sizeof(T));
};

template <typename T>
union Vec16 {
  uint4 raw;
  T e[VecN<T>::N];
};

constexpr int kNormMaxVecs = 4;  // vectors of a row held per thread: h <= kNormThreads * 4 * VecN<T>::N

// Residual add + RMSNorm with the row in registers: one read of resid (and delta), one write of resid and y.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_vec_kernel(const NormArgs a) {
  using A = typename Acc<T>::type;
  constexpr int N = VecN<T>::N;
  __shared__ A red[kNormThreads / 32];
  __shared__ A total;
  const int nv = static_cast<int>(a.h / N);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    T* xr = reinterpret_cast<T*>(a.resid) + row * a.resid_stride;
    const T* dr = a.delta ? reinterpret_cast<const T*>(a.delta) + row * a.delta_stride : nullptr;
    A v[kNormMaxVecs][N];
    A ss = 0;
#pragma unroll
    for (int k = 0; k < kNormMaxVecs; ++k) {
      const int vi = threadIdx.x + k * kNormThreads;
      if (vi < nv) {
        Vec16<T> x;
        x.raw = reinterpret_cast<const uint4*>(xr)[vi];
        if (dr) {
          Vec16<T> d;
          d.raw = reinterpret_cast<const uint4*>(dr)[vi];
#pragma unroll
          for (int e = 0; e < N; ++e) {
            v[k][e] = rnd<T>(up<T>(x.e[e]) + up<T>(d.e[e]));
            x.e[e] = down<T>(v[k][e]);
          }
          reinterpret_cast<uint4*>(xr)[vi] = x.raw;
        } else {
#pragma unroll
          for (int e = 0; e < N; ++e) v[k][e] = up<T>(x.e[e]);
        }
#pragma unroll
        for (int e = 0; e < N; ++e) ss += v[k][e] * v[k][e];
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      A t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : A(0);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
      if (threadIdx.x == 0) total = rsqrt_acc(t / static_cast<A>(a.h) + static_cast<A>(a.eps));
    }
    __syncthreads();
    const A r = total;
    T* yr = reinterpret_cast<T*>(a.y) + row * a.y_stride;
    const T* w = reinterpret_cast<const T*>(a.weight);
#pragma unroll
    for (int k = 0; k < kNormMaxVecs; ++k) {
      const int vi = threadIdx.x + k * kNormThreads;
      if (vi < nv) {
        Vec16<T> wv, out;
        wv.raw = reinterpret_cast<const uint4*>(w)[vi];
#pragma unroll
        for (int e = 0; e < N; ++e) out.e[e] = down<T>(up<T>(wv.e[e]) * rnd<T>(v[k][e] * r));
        reinterpret_cast<uint4*>(yr)[vi] = out.raw;
      }
    }
    __syncthreads();  // red / total are reused by the next row
  }
}

// Rotary embedding with one thread per (b, s, pair j): cos / sin of the token's angle once, applied to the pair
// (j, j + D/2) of every q and k head of the token (the angle does not depend on the head).
template <typename T>
__global__ void __launch_bounds__(kEltThreads) rope_token_kernel(const RopeArgs a) {
  using A = typename Acc<T>::type;
  const A* inv = reinterpret_cast<const A*>(a.inv_freq);
  const int half = a.D / 2;
  const int64_t total = static_cast<int64_t>(a.B) * a.S * half;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i % half);
    const int64_t bs = i / half;
    const int s = static_cast<int>(bs % a.S);
    const int b = static_cast<int>(bs / a.S);
    const int64_t p = a.pos[b * a.pos_stride[0] + s * a.pos_stride[1]];
    const A angle = static_cast<A>(p > 0 ? p : 0) * inv[j];
    A sn, cs;
    sincos_acc(angle, &sn, &cs);
    cs = rnd<T>(cs);
    sn = rnd<T>(sn);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      T* tok = reinterpret_cast<T*>(a.x[t]) + b * a.stride[t][0] + s * a.stride[t][1];
      for (int h = 0; h < a.H[t]; ++h) {
        T* row = tok + h * a.stride[t][2];
        const A x1 = up<T>(row[j]), x2 = up<T>(row[j + half]);
        row[j] = down<T>(rnd<T>(x1 * cs) + rnd<T>(-x2 * sn));
        row[j + half] = down<T>(rnd<T>(x2 * cs) + rnd<T>(x1 * sn));
      }
    }
  }
}

// SwiGLU on 16-byte vectors, one CTA per row at a time.
template <typename T>
__global__ void __launch_bounds__(kEltThreads) silu_mul_vec_kernel(const SiluArgs a) {
  using A = typename Acc<T>::type;
  constexpr int N = VecN<T>::N;
  const int64_t nv = a.n / N;
  for (int64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
    const uint4* g = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.gate) + r * a.in_stride);
    const uint4* u = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.upv) + r * a.in_stride);
    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.out) + r * a.out_stride);
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) {
      Vec16<T> gv, uv, ov;
      gv.raw = g[v];
      uv.raw = u[v];
#pragma unroll
      for (int e = 0; e < N; ++e) {
        const A x = up<T>(gv.e[e]);
        ov.e[e] = down<T>(rnd<T>(x / (A(1) + exp_acc(-x))) * up<T>(uv.e[e]));
      }
      o[v] = ov.raw;
    }
  }
}

}  // namespace llama
}  // namespace cea

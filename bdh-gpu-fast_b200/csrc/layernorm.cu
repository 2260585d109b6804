// Row LayerNorms of a BDH layer (affine-free, over the last dimension D, eps as F.layer_norm):
//
//   bdh_layernorm            y = LN(x)                   bdh.py:565-575 (BDH._ln), applied to the
//                                                        attention output at bdh.py:1044
//   bdh_residual_layernorm   out = LN(x + LN(y))         bdh.py:731-750 (BDH._residual_ln)
//
// One warp per row, 16-byte loads, fp32 statistics: mean, then the mean of squared deviations
// (the biased variance F.layer_norm normalises by), rstd = 1 / sqrt(var + eps). Under bf16
// autocast the reference runs each LN in fp32 on the bf16 tensor and the consumer casts the
// result back to bf16; here the cast is the store. The residual form also emits the bf16 copy
// of the new residual stream that the next layer's encoder projection reads.
#include <string>

#include "bdh_sm100.h"
#include "common.cuh"
#include "internal.h"
#include "tma_host.h"

namespace bdh {

namespace {

constexpr int kLnWarps = 8;       // rows per CTA
constexpr int kLnMaxPerLane = 32;  // D <= 1024

template <typename T>
__device__ __forceinline__ void load8v(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8v<uint16_t>(const uint16_t* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16x2_lo(w[i]);
    v[2 * i + 1] = bf16x2_hi(w[i]);
  }
}
template <>
__device__ __forceinline__ void load8v<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store8v(uint16_t* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(cvt_bf16x2(v[0], v[1]), cvt_bf16x2(v[2], v[3]),
                                            cvt_bf16x2(v[4], v[5]), cvt_bf16x2(v[6], v[7]));
}
__device__ __forceinline__ void store8v(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Normalise the NC = D/256 (rounded up) chunks of 8 values this lane holds in place.
template <int NC>
__device__ __forceinline__ void ln_inplace(float (&v)[NC][8], int D, int lane, float eps) {
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
    if (c * 256 + lane * 8 < D)
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[c][i];
  const float mean = warp_sum(s) / static_cast<float>(D);
  float q = 0.0f;
#pragma unroll
  for (int c = 0; c < NC; ++c)
    if (c * 256 + lane * 8 < D)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[c][i] - mean;
        q = fmaf(d, d, q);
      }
  const float var = warp_sum(q) / static_cast<float>(D);
  const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int c = 0; c < NC; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) v[c][i] = (v[c][i] - mean) * rstd;
}

template <typename TI, typename TO, int NC>
__global__ void __launch_bounds__(32 * kLnWarps) ln_rows_kernel(const TI* __restrict__ x,
                                                                int64_t xs, TO* __restrict__ y,
                                                                int64_t ys, int64_t rows, int D,
                                                                float eps) {
  pdl_wait();     // returns at once: these kernels launch plainly (internal.h, pdl_on)
  pdl_trigger();  // the next kernel's CTAs (the encode) may start setting up
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kLnWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  const TI* xr = x + r * xs;
  float v[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int n = c * 256 + lane * 8;
    if (n < D) load8v<TI>(xr + n, v[c]);
  }
  ln_inplace<NC>(v, D, lane, eps);
  TO* yr = y + r * ys;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int n = c * 256 + lane * 8;
    if (n < D) store8v(yr + n, v[c]);
  }
}

template <typename TY, int NC>
__global__ void __launch_bounds__(32 * kLnWarps) ln_residual_kernel(
    const float* __restrict__ x, int64_t xs, const TY* __restrict__ y, int64_t ys,
    float* __restrict__ out, int64_t os, uint16_t* __restrict__ out16, int64_t os16, int64_t rows,
    int D, float eps) {
  pdl_wait();     // returns at once: these kernels launch plainly (internal.h, pdl_on)
  pdl_trigger();  // the next kernel's CTAs (the encode) may start setting up
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kLnWarps + (threadIdx.x >> 5);
  if (r >= rows) return;
  float v[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int n = c * 256 + lane * 8;
    if (n < D) load8v<TY>(y + r * ys + n, v[c]);
  }
  ln_inplace<NC>(v, D, lane, eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int n = c * 256 + lane * 8;
    if (n < D) {
      float xv[8];
      load8v<float>(x + r * xs + n, xv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = __fadd_rn(v[c][i], xv[i]);
    }
  }
  ln_inplace<NC>(v, D, lane, eps);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int n = c * 256 + lane * 8;
    if (n < D) {
      store8v(out + r * os + n, v[c]);
      if (out16 != nullptr) store8v(out16 + r * os16 + n, v[c]);
    }
  }
}

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return 0;
}

}  // namespace

int launch_layernorm(const void* x, int x_dtype, int64_t xs, void* y, int y_dtype, int64_t ys,
                     int64_t rows, int D, float eps, cudaStream_t stream) {
  if (rows == 0) return 0;
  const unsigned grid = static_cast<unsigned>((rows + kLnWarps - 1) / kLnWarps);
  const int nc = (D + 255) / 256;
#define BDH_LN_LAUNCH(TI, TO, NC)                                                              \
  ln_rows_kernel<TI, TO, NC><<<grid, 32 * kLnWarps, 0, stream>>>(                              \
      static_cast<const TI*>(x), xs, static_cast<TO*>(y), ys, rows, D, eps)
#define BDH_LN_DISPATCH(TI, TO)            \
  switch (nc) {                            \
    case 1: BDH_LN_LAUNCH(TI, TO, 1); break; \
    case 2: BDH_LN_LAUNCH(TI, TO, 2); break; \
    default: BDH_LN_LAUNCH(TI, TO, 4); break; \
  }
  prof_start(kProfNorm, stream);
  if (x_dtype == BDH_DTYPE_BF16 && y_dtype == BDH_DTYPE_BF16) {
    BDH_LN_DISPATCH(uint16_t, uint16_t)
  } else if (x_dtype == BDH_DTYPE_BF16) {
    BDH_LN_DISPATCH(uint16_t, float)
  } else if (y_dtype == BDH_DTYPE_BF16) {
    BDH_LN_DISPATCH(float, uint16_t)
  } else {
    BDH_LN_DISPATCH(float, float)
  }
  prof_stop(kProfNorm, stream);
#undef BDH_LN_DISPATCH
#undef BDH_LN_LAUNCH
  return launch_check("layernorm launch");
}

int launch_residual_layernorm(const float* x, int64_t xs, const void* y, int y_dtype, int64_t ys,
                              float* out, int64_t os, uint16_t* out16, int64_t os16, int64_t rows,
                              int D, float eps, cudaStream_t stream) {
  if (rows == 0) return 0;
  const unsigned grid = static_cast<unsigned>((rows + kLnWarps - 1) / kLnWarps);
  const int nc = (D + 255) / 256;
#define BDH_RLN_LAUNCH(TY, NC)                                                                 \
  ln_residual_kernel<TY, NC><<<grid, 32 * kLnWarps, 0, stream>>>(                              \
      x, xs, static_cast<const TY*>(y), ys, out, os, out16, os16, rows, D, eps)
  prof_start(kProfNorm, stream);
  if (y_dtype == BDH_DTYPE_BF16) {
    switch (nc) {
      case 1: BDH_RLN_LAUNCH(uint16_t, 1); break;
      case 2: BDH_RLN_LAUNCH(uint16_t, 2); break;
      default: BDH_RLN_LAUNCH(uint16_t, 4); break;
    }
  } else {
    switch (nc) {
      case 1: BDH_RLN_LAUNCH(float, 1); break;
      case 2: BDH_RLN_LAUNCH(float, 2); break;
      default: BDH_RLN_LAUNCH(float, 4); break;
    }
  }
  prof_stop(kProfNorm, stream);
#undef BDH_RLN_LAUNCH
  return launch_check("residual layernorm launch");
}

}  // namespace bdh

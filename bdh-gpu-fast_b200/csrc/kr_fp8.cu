// fp8 wire format of the cached rotated keys: each cached row kr[b,h,t,:] (N values) is stored
// as e4m3 (1 byte per value) with one fp32 scale per row,
//
//   amax = max_n |x[n]|,  inv = 448 / amax (0 when amax == 0),  scale = amax / 448,
//   q8[n] = e4m3_rn_satfinite(x[n] * inv),   x[n] ~= q8[n] * scale,
//
// (448 = the largest finite e4m3 value), which halves the decode stream of a bf16 cache and
// quarters that of an fp32 one (the key history is most of the bytes a decode step reads). The
// reference stores its cache in fp32 / fp16 / bf16 only (bdh_cache.py:62-80,240-243); this
// storage kind is opt-in and lossy (e4m3 keeps 3 mantissa bits).
//
// One CTA per row: the row's absolute maximum by a warp-shuffle + shared-memory reduction, then
// a second pass (the row is in L2) converts pairs with the packed cvt.rn.satfinite.e4m3x2.f32
// and writes 16 values per 16-byte store.
#include <string>

#include "bdh_sm100.h"
#include "common.cuh"
#include "internal.h"
#include "tma_host.h"

namespace bdh {

namespace {

constexpr int kQThreads = 256;

template <typename T>
__device__ __forceinline__ float ldq(const T* p, int i);
template <>
__device__ __forceinline__ float ldq<float>(const float* p, int i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ldq<uint16_t>(const uint16_t* p, int i) {
  return bf16_bits_to_f32(p[i]);
}

// Two values to two e4m3 bytes (lo in bits 0-7), round to nearest even, saturating at +-448.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename TI>
__global__ void __launch_bounds__(kQThreads) quantize_rows_fp8_kernel(
    const TI* __restrict__ x, int64_t xsb, int64_t xsh, int64_t xst, uint8_t* __restrict__ out,
    int64_t osb, int64_t osh, int64_t ost, float* __restrict__ scale, int64_t ssb, int64_t ssh,
    int64_t sst, int H, int T, int N, bool vec) {
  __shared__ float red[kQThreads / 32];
  const int64_t row = blockIdx.x;
  const int t = static_cast<int>(row % T);
  const int64_t bh = row / T;
  const int h = static_cast<int>(bh % H);
  const int64_t b = bh / H;
  const TI* xr = x + b * xsb + h * xsh + t * xst;
  uint8_t* orow = out + b * osb + h * osh + t * ost;
  float m = 0.0f;
  for (int n = threadIdx.x; n < N; n += kQThreads) m = fmaxf(m, fabsf(ldq<TI>(xr, n)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = 0.0f;
#pragma unroll
  for (int w = 0; w < kQThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float inv = amax > 0.0f ? __fdiv_rn(448.0f, amax) : 0.0f;
  if (threadIdx.x == 0) scale[b * ssb + h * ssh + t * sst] = __fdiv_rn(amax, 448.0f);
  if (vec) {  // 16 values per thread and step, one 16-byte store
    for (int n = threadIdx.x * 16; n < N; n += kQThreads * 16) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t p0 = cvt_e4m3x2(__fmul_rn(ldq<TI>(xr, n + 4 * i), inv),
                                       __fmul_rn(ldq<TI>(xr, n + 4 * i + 1), inv));
        const uint32_t p1 = cvt_e4m3x2(__fmul_rn(ldq<TI>(xr, n + 4 * i + 2), inv),
                                       __fmul_rn(ldq<TI>(xr, n + 4 * i + 3), inv));
        w[i] = p0 | (p1 << 16);
      }
      *reinterpret_cast<uint4*>(orow + n) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {  // any even N: one pair per thread and step
    for (int n = threadIdx.x * 2; n < N; n += kQThreads * 2) {
      const uint32_t p = cvt_e4m3x2(__fmul_rn(ldq<TI>(xr, n), inv), __fmul_rn(ldq<TI>(xr, n + 1), inv));
      orow[n] = static_cast<uint8_t>(p & 0xFFu);
      orow[n + 1] = static_cast<uint8_t>(p >> 8);
    }
  }
}

}  // namespace

int launch_quantize_rows_fp8(const void* x, int x_dtype, const int64_t xs[4], int64_t B,
                             int64_t H, int64_t T, int64_t N, uint8_t* out, const int64_t os[4],
                             float* scale, const int64_t ss[3], cudaStream_t stream) {
  const int64_t rows = B * H * T;
  if (rows == 0 || N == 0) return BDH_OK;
  const bool vec = (N % 16) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                   os[0] % 16 == 0 && os[1] % 16 == 0 && os[2] % 16 == 0;
  const int Hi = static_cast<int>(H), Ti = static_cast<int>(T), Ni = static_cast<int>(N);
  if (x_dtype == BDH_DTYPE_F32)
    quantize_rows_fp8_kernel<float><<<static_cast<unsigned>(rows), kQThreads, 0, stream>>>(
        static_cast<const float*>(x), xs[0], xs[1], xs[2], out, os[0], os[1], os[2], scale, ss[0],
        ss[1], ss[2], Hi, Ti, Ni, vec);
  else
    quantize_rows_fp8_kernel<uint16_t><<<static_cast<unsigned>(rows), kQThreads, 0, stream>>>(
        static_cast<const uint16_t*>(x), xs[0], xs[1], xs[2], out, os[0], os[1], os[2], scale,
        ss[0], ss[1], ss[2], Hi, Ti, Ni, vec);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("quantize_rows_fp8 launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

}  // namespace bdh

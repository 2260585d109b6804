// fp32 decoder product of a decode step: out (M, D) = X (M, K) @ W (K, D), with M = B * T small
// (one token per sequence) and K = nh * N large (the reference's y_mlp = xy @ decoder in fp32,
// bdh.py:1050 outside autocast). A library GEMM launches a handful of CTAs for this shape
// (M = 64, D = 256 gives 8 tiles of 128 x 32); here K is split across the GPU instead.
//
// Slice kernel: CTA (s, mb, db) multiplies X rows [64 mb, 64 mb + 64) by W rows
// [kDecKS s, kDecKS (s + 1)) and columns [128 db, 128 db + 128) and writes the fp32 partial to
// part[s]. X's slice is staged transposed in shared memory; W's slice streams through a
// double-buffered shared-memory stage in chunks of kDecWK rows (16-byte asynchronous copies,
// the next chunk in flight while this one is multiplied). Each of the 256 threads keeps an
// 8-row x 4-column register tile: per k, two 16-byte shared loads of X (4 distinct addresses per
// warp), one of W (8 distinct per warp) and 32 FMAs. Reduce kernel: out = sum over s of part[s],
// in a fixed order (deterministic).
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "internal.h"
#include "tma_host.h"

namespace bdh {
namespace {

constexpr int kDecKS = 256;    // K rows per slice
constexpr int kDecRows = 64;   // X rows per CTA
constexpr int kDecCols = 128;  // output columns per CTA
constexpr int kDecPad = 68;    // floats per staged X k row (16-byte aligned, fewer bank conflicts)
constexpr int kDecThreads = 256;
constexpr int kDecWK = 32;     // W rows per shared-memory chunk
constexpr int kRedGroups = 4;  // slice groups summed side by side by the reduce kernel
constexpr int kDecSmem = (kDecKS * kDecPad + 2 * kDecWK * kDecCols) * static_cast<int>(sizeof(float));

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kDecThreads, 2) dec_f32_slice_kernel(
    const float* __restrict__ x, int64_t ldx, const float* __restrict__ w, int64_t ldw,
    float* __restrict__ part, int M, int K, int D) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                          // [kDecKS][kDecPad]
  float* wsm = smem + kDecKS * kDecPad;      // [2][kDecWK][kDecCols]
  const int k0 = blockIdx.x * kDecKS;
  const int m0 = blockIdx.y * kDecRows;
  const int d0 = blockIdx.z * kDecCols;
  const int ks = min(kDecKS, K - k0);
  const int nchunk = (ks + kDecWK - 1) / kDecWK;

  // W chunk c -> buffer c & 1: 32 rows x 128 columns, four 16-byte copies per thread (rows at or
  // beyond ks and columns at or beyond D are zero-filled)
  auto load_w = [&](int c) {
    float* dst = wsm + (c & 1) * (kDecWK * kDecCols);
#pragma unroll
    for (int i = 0; i < (kDecWK * kDecCols / 4) / kDecThreads; ++i) {
      const int e = i * kDecThreads + threadIdx.x;  // float4 index in the chunk
      const int r = e / (kDecCols / 4), c4 = e - r * (kDecCols / 4);
      const int k = c * kDecWK + r, d = d0 + 4 * c4;
      const bool ok = k < ks && d < D;
      const float* src = ok ? w + static_cast<int64_t>(k0 + k) * ldw + d : w;
      cp_async16(dst + r * kDecCols + 4 * c4, src, ok);
    }
    cp_async_commit();
  };
  load_w(0);
  if (nchunk > 1) load_w(1);
  for (int i = threadIdx.x; i < kDecKS * kDecRows; i += kDecThreads) {
    const int m = i / kDecKS, k = i - m * kDecKS;  // consecutive threads read consecutive k
    float v = 0.f;
    if (m0 + m < M && k < ks) v = __ldg(x + static_cast<int64_t>(m0 + m) * ldx + k0 + k);
    xs[k * kDecPad + m] = v;
  }

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cg = (warp & 3) * 8 + (lane >> 2);  // 4-column group, 0..31
  const int mg = (warp >> 2) * 4 + (lane & 3);  // 8-row group, 0..7
  float acc[8][4];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
  const float* xr = xs + mg * 8;
  for (int c = 0; c < nchunk; ++c) {
    if (c + 1 < nchunk) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncthreads();  // chunk c (and, at c = 0, the staged X) visible to every thread
    const float* wc = wsm + (c & 1) * (kDecWK * kDecCols) + cg * 4;
#pragma unroll 8
    for (int q = 0; q < kDecWK; ++q) {
      const int k = c * kDecWK + q;
      const float4 wv = *reinterpret_cast<const float4*>(wc + q * kDecCols);
      const float4 xa = *reinterpret_cast<const float4*>(xr + k * kDecPad);
      const float4 xb = *reinterpret_cast<const float4*>(xr + k * kDecPad + 4);
      const float xe[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc[e][0] = fmaf(xe[e], wv.x, acc[e][0]);
        acc[e][1] = fmaf(xe[e], wv.y, acc[e][1]);
        acc[e][2] = fmaf(xe[e], wv.z, acc[e][2]);
        acc[e][3] = fmaf(xe[e], wv.w, acc[e][3]);
      }
    }
    __syncthreads();  // every thread is done with buffer c & 1 before it is refilled
    if (c + 2 < nchunk) load_w(c + 2);
  }
  const int d = d0 + cg * 4;
  if (d >= D) return;  // D is a multiple of 4
  float* pp = part + static_cast<int64_t>(blockIdx.x) * M * D + d;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int m = m0 + mg * 8 + r;
    if (m < M)
      *reinterpret_cast<float4*>(pp + static_cast<int64_t>(m) * D) =
          make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
  }
}

// CTA m sums row m of the partials: thread (g, c) adds slices g, g + 4, ... of the 4-column
// group c; the four group sums are then added in order g = 0..3.
__global__ void __launch_bounds__(256) dec_f32_reduce_kernel(const float* __restrict__ part,
                                                             float* __restrict__ out,
                                                             int64_t ldo, int M, int D, int S) {
  __shared__ float4 red[kRedGroups][64];
  const int m = blockIdx.x;
  const int g = threadIdx.x >> 6, c = threadIdx.x & 63;
  for (int c4 = blockIdx.y * 64; c4 < D / 4; c4 += gridDim.y * 64) {
    const int col = c4 + c;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col < D / 4) {
      const float* p = part + static_cast<int64_t>(m) * D + 4 * col;
#pragma unroll 8
      for (int s = g; s < S; s += kRedGroups) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(p + static_cast<int64_t>(s) * M * D));
        a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      }
    }
    red[g][c] = a;
    __syncthreads();
    if (g == 0 && col < D / 4) {
      float4 t = red[0][c];
#pragma unroll
      for (int q = 1; q < kRedGroups; ++q) {
        const float4 v = red[q][c];
        t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
      }
      float* o = out + static_cast<int64_t>(m) * ldo + 4 * col;
      o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
    }
    __syncthreads();
  }
}

}  // namespace

int64_t decoder_f32_slices(int64_t K) { return (K + kDecKS - 1) / kDecKS; }

int launch_decoder_f32(const float* x, int64_t ldx, const float* w, int64_t ldw, float* out,
                       int64_t ldo, float* part, int64_t M, int64_t K, int64_t D,
                       cudaStream_t stream) {
  if (M == 0 || D == 0) return BDH_OK;
  const int64_t S = decoder_f32_slices(K);
  if (S == 0) {
    for (int64_t m = 0; m < M; ++m) {
      cudaError_t e = cudaMemsetAsync(out + m * ldo, 0, D * sizeof(float), stream);
      if (e != cudaSuccess) {
        set_error(std::string("decoder_f32 memset: ") + cudaGetErrorString(e));
        return BDH_ERR_CUDA;
      }
    }
    return BDH_OK;
  }
  const int smem = kDecSmem;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(dec_f32_slice_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error(std::string("decoder_f32 attribute: ") + cudaGetErrorString(e));
      return BDH_ERR_CUDA;
    }
    attr_set[dev] = true;
  }
  prof_start(kProfDecoder, stream);
  const dim3 grid(static_cast<unsigned>(S), static_cast<unsigned>((M + kDecRows - 1) / kDecRows),
                  static_cast<unsigned>((D + kDecCols - 1) / kDecCols));
  dec_f32_slice_kernel<<<grid, kDecThreads, smem, stream>>>(
      x, ldx, w, ldw, part, static_cast<int>(M), static_cast<int>(K), static_cast<int>(D));
  const dim3 rgrid(static_cast<unsigned>(M), static_cast<unsigned>((D / 4 + 63) / 64));
  dec_f32_reduce_kernel<<<rgrid, 256, 0, stream>>>(part, out, ldo, static_cast<int>(M),
                                                   static_cast<int>(D), static_cast<int>(S));
  prof_stop(kProfDecoder, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("decoder_f32 launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

}  // namespace bdh

// Cached decode step: out[b,h,tq] = sum_j (q[b,h,tq] . K_past[b,h,j]) V_past[b,hv,j]
// (reference: csrc/tril_attn_cuda.cu:431-542 tril_decode_*_kernel, kernels/attention.py:193-219
// _two_gemm_decode; every cached key precedes the query, so there is no mask).
//
// HBM-bound: the whole key history is streamed once per step. Grid = (split, b*h, tq); each
// CTA owns a run of consecutive cached rows of one (b, h) and one query:
//   1. the query (optionally RoPE-rotated in registers, and then also written to this step's
//      cache slot by split 0) is held as fp32: in registers, per warp column slice
//      (decode_slice_kernel, the default), or staged in shared memory (decode_partial_kernel,
//      for unaligned rows and very wide latents);
//   2. the key rows are streamed with 16-byte coalesced loads straight from the
//      capacity-strided cache view (no contiguous copy), widened in registers (bf16, e4m3),
//      and the dot products are reduced with warp shuffles;
//   3. the CTA forms its partial out = sum_j s_j V_j (one thread per output column);
//   4. a second small kernel sums the per-split partials in a fixed order (deterministic).
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <sstream>
#include <string>

#include <cuda_fp16.h>

#include "common.cuh"
#include "internal.h"
#include "tma_host.h"

namespace bdh {

namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecRowsMax = 128;  // cached rows per CTA at most (the plan picks 16..128)

__device__ __forceinline__ float bf16_round_d(float x) { return bf16_round_f32(x); }

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p, int64_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ld_elem<uint16_t>(const uint16_t* p, int64_t i) {
  return bf16_bits_to_f32(p[i]);
}
template <typename T>
__device__ __forceinline__ void st_elem(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st_elem<float>(float* p, int64_t i, float v) {
  p[i] = v;
}
template <>
__device__ __forceinline__ void st_elem<uint16_t>(uint16_t* p, int64_t i, float v) {
  p[i] = static_cast<uint16_t>(f32_to_bf16_bits(v));
}

// Dot products of q (shared, fp32) with two key rows; VEC = 16-byte loads along N.
template <typename TK, bool VEC>
__device__ __forceinline__ void dot2(const float* __restrict__ qs, const TK* __restrict__ k0,
                                     const TK* __restrict__ k1, int N, bool has1, float& d0,
                                     float& d1) {
  const int lane = threadIdx.x & 31;
  float a0 = 0.f, a1 = 0.f;
  if (VEC) {
    constexpr int E = 16 / sizeof(TK);  // elements per 16-byte load
#pragma unroll 4
    for (int n = lane * E; n < N; n += 32 * E) {
      float qv[E];
#pragma unroll
      for (int i = 0; i < E; i += 4) {
        const float4 t = *reinterpret_cast<const float4*>(qs + n + i);
        qv[i] = t.x; qv[i + 1] = t.y; qv[i + 2] = t.z; qv[i + 3] = t.w;
      }
      const uint4 u0 = __ldcs(reinterpret_cast<const uint4*>(k0 + n));
      uint4 u1 = make_uint4(0, 0, 0, 0);
      if (has1) u1 = __ldcs(reinterpret_cast<const uint4*>(k1 + n));
      const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w};
      const uint32_t w1[4] = {u1.x, u1.y, u1.z, u1.w};
      if (sizeof(TK) == 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a0 = fmaf(qv[i], __uint_as_float(w0[i]), a0);
          a1 = fmaf(qv[i], __uint_as_float(w1[i]), a1);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a0 = fmaf(qv[2 * i], bf16_bits_to_f32(w0[i] & 0xFFFFu), a0);
          a0 = fmaf(qv[2 * i + 1], bf16_bits_to_f32(w0[i] >> 16), a0);
          a1 = fmaf(qv[2 * i], bf16_bits_to_f32(w1[i] & 0xFFFFu), a1);
          a1 = fmaf(qv[2 * i + 1], bf16_bits_to_f32(w1[i] >> 16), a1);
        }
      }
    }
  } else {
    for (int n = lane; n < N; n += 32) {
      a0 = fmaf(qs[n], ld_elem(k0, n), a0);
      if (has1) a1 = fmaf(qs[n], ld_elem(k1, n), a1);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
  }
  d0 = a0;
  d1 = a1;
}

template <typename TQ, typename TK, bool VEC>
__global__ void __launch_bounds__(kDecThreads) decode_partial_kernel(
    const TQ* __restrict__ q, const TK* __restrict__ kp, const TK* __restrict__ vp,
    float* __restrict__ partial, TK* __restrict__ slot, const float* __restrict__ freqs,
    int H, int Hv, int Tq, int S, int N, int D, int64_t qsb, int64_t qsh, int64_t qst,
    int64_t ksb, int64_t ksh, int64_t kst, int64_t vsb, int64_t vsh, int64_t vst, int64_t ssb,
    int64_t ssh, int64_t sst, int64_t pos, int kDecRows) {
  extern __shared__ float dsm[];
  float* qs = dsm;              // N floats
  float* sc = dsm + N;          // kDecRows (<= kDecRowsMax) scores
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int tq = blockIdx.z;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int hv = Hv == 1 ? 0 : h;
  const int nsplit = gridDim.x;

  // 1. stage q (rotated when freqs is given).
  const TQ* qr = q + b * qsb + h * qsh + tq * qst;
  if (freqs != nullptr) {
    constexpr bool BF16 = sizeof(TQ) == 2;
    const float p = static_cast<float>(pos + tq);
    for (int n = threadIdx.x * 2; n < N; n += blockDim.x * 2) {
      float c0, s0, c1, s1;
      rope_cis(p, freqs[n], c0, s0);
      rope_cis(p, freqs[n + 1], c1, s1);
      const float x0 = ld_elem(qr, n), x1 = ld_elem(qr, n + 1);
      float y0, y1;
      if (BF16) {
        y0 = bf16_round_d(__fadd_rn(bf16_round_d(__fmul_rn(x0, c0)), bf16_round_d(__fmul_rn(-x1, s0))));
        y1 = bf16_round_d(__fadd_rn(bf16_round_d(__fmul_rn(x1, c1)), bf16_round_d(__fmul_rn(x0, s1))));
      } else {
        y0 = __fsub_rn(__fmul_rn(x0, c0), __fmul_rn(x1, s0));
        y1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1));
      }
      qs[n] = y0;
      qs[n + 1] = y1;
      if (slot != nullptr && split == 0) {
        TK* sr = slot + b * ssb + h * ssh + tq * sst;
        st_elem(sr, n, y0);
        st_elem(sr, n + 1, y1);
      }
    }
  } else if (sizeof(TQ) == 4 && (N & 3) == 0 && (reinterpret_cast<uintptr_t>(qr) & 15u) == 0) {
    // fp32 rows (the rotated queries): 16-byte loads, all of a thread's loads in flight at once
    const float4* q4 = reinterpret_cast<const float4*>(qr);
    float4* s4 = reinterpret_cast<float4*>(qs);
#pragma unroll 8
    for (int n = threadIdx.x; n < (N >> 2); n += kDecThreads) s4[n] = __ldg(q4 + n);
  } else {
    for (int n = threadIdx.x; n < N; n += blockDim.x) qs[n] = ld_elem(qr, n);
  }
  __syncthreads();

  // 2. scores for this split's rows.
  const int j0 = split * kDecRows;
  const int rows = max(0, min(kDecRows, S - j0));
  const int warp = threadIdx.x >> 5;
  const TK* kbase = kp + b * ksb + h * ksh;
  for (int r = warp * 2; r < rows; r += kDecWarps * 2) {
    const bool has1 = r + 1 < rows;
    float d0, d1;
    dot2<TK, VEC>(qs, kbase + (j0 + r) * kst, kbase + (j0 + r + (has1 ? 1 : 0)) * kst, N, has1,
                  d0, d1);
    if ((threadIdx.x & 31) == 0) {
      sc[r] = d0;
      if (has1) sc[r + 1] = d1;
    }
  }
  __syncthreads();

  // 3. partial out = sum_j s_j V_j.
  const TK* vbase = vp + b * vsb + hv * vsh;
  float* dst = partial + ((static_cast<int64_t>(split) * gridDim.y + bh) * Tq + tq) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) acc = fmaf(sc[r], ld_elem(vbase + (j0 + r) * vst, d), acc);
    dst[d] = acc;
  }
  (void)nsplit;
}

// ---------------------------------------------------------------- fp8 key history
// The e4m3 byte in bits 24-31 of `t` (lower bits arbitrary) to
// fp32, scaled by 2^-120, with integer operations only: shifting right arithmetically by 4
// puts s eeee mmm at bits 27-20 with the sign copied into bits 31-28, and the mask keeps the
// sign bit and the seven exponent/mantissa bits. An e4m3 value 2^(e-7) (1 + m/8) becomes the
// fp32 value 2^(e-127) (1 + m/8), and a subnormal 2^-6 (m/8) the fp32 denormal 2^-126 (m/8):
// both exactly 2^-120 times the e4m3 value. (The conversion instructions run on a narrow pipe
// that capped the fp8 stream at about half the HBM rate.)
__device__ __forceinline__ float e4m3_top_to_f32_2m120(uint32_t t) {
  return __int_as_float((static_cast<int32_t>(t) >> 4) & static_cast<int32_t>(0x87F00000u));
}
constexpr float kE4m3QScale = 18446744073709551616.0f;  // 2^64, folded into the staged query
constexpr float kE4m3RowScale = 72057594037927936.0f;   // 2^56 = 2^120 / 2^64, into each score

// Dot products of q (shared, fp32, pre-multiplied by 2^64) with two e4m3 key rows (unscaled,
// each value read as 2^-120 times itself); VEC = 16-byte loads.
template <bool VEC>
__device__ __forceinline__ void dot2_fp8(const float* __restrict__ qs, const uint8_t* __restrict__ k0,
                                         const uint8_t* __restrict__ k1, int N, bool has1,
                                         float& d0, float& d1) {
  const int lane = threadIdx.x & 31;
  float a0 = 0.f, a1 = 0.f;
  if (VEC) {
#pragma unroll 4
    for (int n = lane * 16; n < N; n += 32 * 16) {
      const uint4 u0 = __ldcs(reinterpret_cast<const uint4*>(k0 + n));
      uint4 u1 = make_uint4(0, 0, 0, 0);
      if (has1) u1 = __ldcs(reinterpret_cast<const uint4*>(k1 + n));
      const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w};
      const uint32_t w1[4] = {u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 qv = *reinterpret_cast<const float4*>(qs + n + 4 * i);
        a0 = fmaf(qv.x, e4m3_top_to_f32_2m120(w0[i] << 24), a0);
        a0 = fmaf(qv.y, e4m3_top_to_f32_2m120(w0[i] << 16), a0);
        a0 = fmaf(qv.z, e4m3_top_to_f32_2m120(w0[i] << 8), a0);
        a0 = fmaf(qv.w, e4m3_top_to_f32_2m120(w0[i]), a0);
        a1 = fmaf(qv.x, e4m3_top_to_f32_2m120(w1[i] << 24), a1);
        a1 = fmaf(qv.y, e4m3_top_to_f32_2m120(w1[i] << 16), a1);
        a1 = fmaf(qv.z, e4m3_top_to_f32_2m120(w1[i] << 8), a1);
        a1 = fmaf(qv.w, e4m3_top_to_f32_2m120(w1[i]), a1);
      }
    }
  } else {
    for (int n = lane; n < N; n += 32) {
      a0 = fmaf(qs[n], e4m3_top_to_f32_2m120(static_cast<uint32_t>(k0[n]) << 24), a0);
      if (has1) a1 = fmaf(qs[n], e4m3_top_to_f32_2m120(static_cast<uint32_t>(k1[n]) << 24), a1);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
  }
  d0 = a0;
  d1 = a1;
}

// Same split-S structure as decode_partial_kernel; the score of cached row j is
// scale_j * (q . e4m3_j).
template <typename TQ, typename TV, bool VEC>
__global__ void __launch_bounds__(kDecThreads) decode_partial_fp8_kernel(
    const TQ* __restrict__ q, const uint8_t* __restrict__ kp, const float* __restrict__ ksc,
    const TV* __restrict__ vp, float* __restrict__ partial, int H, int Hv, int Tq, int S, int N,
    int D, int64_t qsb, int64_t qsh, int64_t qst, int64_t ksb, int64_t ksh, int64_t kst,
    int64_t csb, int64_t csh, int64_t cst, int64_t vsb, int64_t vsh, int64_t vst, int kDecRows) {
  extern __shared__ float dsm[];
  float* qs = dsm;
  float* sc = dsm + N;
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int tq = blockIdx.z;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int hv = Hv == 1 ? 0 : h;
  const TQ* qr = q + b * qsb + h * qsh + tq * qst;
  // q * 2^64 (exact): with keys read as 2^-120 times their value, products of ordinary
  // magnitudes stay normal fp32 numbers
  if (sizeof(TQ) == 4 && (N & 3) == 0 && (reinterpret_cast<uintptr_t>(qr) & 15u) == 0) {
    const float4* q4 = reinterpret_cast<const float4*>(qr);
    float4* s4 = reinterpret_cast<float4*>(qs);
#pragma unroll 8
    for (int n = threadIdx.x; n < (N >> 2); n += kDecThreads) {
      float4 t = __ldg(q4 + n);
      t.x *= kE4m3QScale; t.y *= kE4m3QScale; t.z *= kE4m3QScale; t.w *= kE4m3QScale;
      s4[n] = t;
    }
  } else {
    for (int n = threadIdx.x; n < N; n += blockDim.x) qs[n] = ld_elem(qr, n) * kE4m3QScale;
  }
  __syncthreads();
  const int j0 = split * kDecRows;
  const int rows = max(0, min(kDecRows, S - j0));
  const int warp = threadIdx.x >> 5;
  const uint8_t* kbase = kp + b * ksb + h * ksh;
  const float* cbase = ksc + b * csb + h * csh;
  for (int r = warp * 2; r < rows; r += kDecWarps * 2) {
    const bool has1 = r + 1 < rows;
    float d0, d1;
    dot2_fp8<VEC>(qs, kbase + (j0 + r) * kst, kbase + (j0 + r + (has1 ? 1 : 0)) * kst, N, has1,
                  d0, d1);
    if ((threadIdx.x & 31) == 0) {
      sc[r] = (d0 * kE4m3RowScale) * cbase[(j0 + r) * cst];
      if (has1) sc[r + 1] = (d1 * kE4m3RowScale) * cbase[(j0 + r + 1) * cst];
    }
  }
  __syncthreads();
  const TV* vbase = vp + b * vsb + hv * vsh;
  float* dst = partial + ((static_cast<int64_t>(split) * gridDim.y + bh) * Tq + tq) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) acc = fmaf(sc[r], ld_elem(vbase + (j0 + r) * vst, d), acc);
    dst[d] = acc;
  }
}

// ------------------------------------------------------------ column-slice stream
// The same split-S decode with the query in registers and one continuous load pipeline per
// lane. Warp w of a CTA owns the column chunks c = w + 8 i (i < QC) of 32 x E elements
// (E = 16 / key size), keeps its q elements of those chunks in registers for the whole CTA,
// and streams all of the CTA's cached rows over those columns: each lane's 16-byte key loads
// form one sequence (row by row, QC loads per row) issued kSliceAhead loads before their use,
// so the stream does not drain between rows. The eight partial dots of a group of eight rows
// are reduced across the warp with nine shuffles, and the warps' partials are summed in shared
// memory. Measured on B200 at the config-4 shapes (B = 64, H = 4, S = 520, N = 8192): 7.2 /
// 7.1 / 6.0 TB/s for fp32 / bf16 / fp8 keys, against 5.8 / 5.0 / 3.6 TB/s for the row-per-warp
// kernels above (q staged in shared memory, loads drained at every row pair), which remain the
// path for unaligned rows and latent widths beyond the register budget.
constexpr int kSliceWarps = 8;
constexpr int kSliceAhead = 8;  // 16-byte key loads in flight per lane

template <typename TK>
__device__ __forceinline__ float dot16(const float* qv, const uint4 u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float a = 0.f;
  if (sizeof(TK) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) a = fmaf(qv[i], __uint_as_float(w[i]), a);
  } else if (sizeof(TK) == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a = fmaf(qv[2 * i], __uint_as_float(w[i] << 16), a);
      a = fmaf(qv[2 * i + 1], __uint_as_float(w[i] & 0xFFFF0000u), a);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a = fmaf(qv[4 * i], e4m3_top_to_f32_2m120(w[i] << 24), a);
      a = fmaf(qv[4 * i + 1], e4m3_top_to_f32_2m120(w[i] << 16), a);
      a = fmaf(qv[4 * i + 2], e4m3_top_to_f32_2m120(w[i] << 8), a);
      a = fmaf(qv[4 * i + 3], e4m3_top_to_f32_2m120(w[i]), a);
    }
  }
  return a;
}

// e4m3 keys widened by the conversion instructions: two bytes at a time to fp16
// (cvt.rn.f16x2.e4m3x2, exact: every e4m3 value is a normal fp16) and on to fp32, against
// unscaled query elements. In a probe at the config-4 shapes this streamed 6.0 TB/s, against
// 4.9 TB/s for the integer widening above (the decode is bound by the widening) and 5.5 TB/s
// for half of the bytes each way.
__device__ __forceinline__ float dot16_e4m3(const float* qv, const uint4 u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float a = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t h2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;"
          : "=r"(h2)
          : "h"(static_cast<uint16_t>(half ? (w[i] >> 16) : (w[i] & 0xFFFFu))));
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
      a = fmaf(qv[4 * i + 2 * half], f.x, a);
      a = fmaf(qv[4 * i + 2 * half + 1], f.y, a);
    }
  }
  return a;
}

// Four consecutive query elements; vec: one 16-byte (fp32) or 8-byte (bf16) load.
__device__ __forceinline__ void load_q4(const float* p, bool vec, float (&x)[4]) {
  if (vec) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = p[j];
  }
}
__device__ __forceinline__ void load_q4(const uint16_t* p, bool vec, float (&x)[4]) {
  if (vec) {
    const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    x[0] = __uint_as_float(t.x << 16); x[1] = __uint_as_float(t.x & 0xFFFF0000u);
    x[2] = __uint_as_float(t.y << 16); x[3] = __uint_as_float(t.y & 0xFFFF0000u);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = bf16_bits_to_f32(p[j]);
  }
}

// F8: TK = uint8_t e4m3 keys with one fp32 scale per row (ksc). ROT: the query is rotated
// here (freqs) and split 0 writes the cache slot; a separate instantiation, so that the kernels
// without it keep their registers for the load ring (F8 never rotates here).
template <typename TQ, typename TK, typename TV, int QC, bool F8, bool ROT>
__global__ void __launch_bounds__(kSliceWarps * 32, 2) decode_slice_kernel(
    const TQ* __restrict__ q, const TK* __restrict__ kp, const float* __restrict__ ksc,
    const TV* __restrict__ vp, float* __restrict__ partial, TK* __restrict__ slot,
    const float* __restrict__ freqs, int H, int Hv, int S, int N, int D, int64_t qsb,
    int64_t qsh, int64_t qst, int64_t ksb, int64_t ksh, int64_t kst, int64_t csb, int64_t csh,
    int64_t cst, int64_t vsb, int64_t vsh, int64_t vst, int64_t ssb, int64_t ssh, int64_t sst,
    int64_t pos, int rows_per_cta, bool qvec) {
  constexpr int E = 16 / sizeof(TK);
  constexpr int CS = kSliceWarps * 32 * E;  // elements of one chunk row across the CTA
  // rows per group: fewer when the lane holds many query elements (32 at N = 8192) or rotates
  // them here, so that the query slice, the load ring and the group's sums fit the 128
  // registers of two CTAs per SM (fp32 keys at N = 8192: two rows per group)
  constexpr int GR = (QC * E >= 32 && sizeof(TK) == 4) ? 2 : (QC * E >= 32 || (ROT && QC * E >= 16)) ? 4 : 8;
  constexpr int L = GR * QC;                // loads of a group of GR rows
  constexpr int DP = kSliceAhead;
  static_assert(DP % QC == 0 && L % DP == 0, "the prefetch distance covers whole rows");
  __shared__ float red[kSliceWarps][kDecRowsMax];
  __shared__ float sc[kDecRowsMax];
  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int tq = blockIdx.z;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int hv = Hv == 1 ? 0 : h;
  const int j0 = split * rows_per_cta;
  const int rows = max(0, min(rows_per_cta, S - j0));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int coff0 = (warp * 32 + lane) * E;  // this lane's chunk i starts at coff0 + i * CS
  const int nval = coff0 < N ? (N - coff0 + CS - 1) / CS : 0;

  // 1. the first kSliceAhead key loads
  const TK* lp = kp + b * ksb + h * ksh + static_cast<int64_t>(j0) * kst + coff0;
  int lr = 0;  // row of lp
  uint4 ring[DP];
#pragma unroll
  for (int t = 0; t < DP; ++t) {
    const int i = t % QC;
    ring[t] = make_uint4(0, 0, 0, 0);
    if (lr < rows && i < nval) ring[t] = __ldcs(reinterpret_cast<const uint4*>(lp + i * CS));
    if (i == QC - 1) {
      lp += kst;
      ++lr;
    }
  }

  // 2. this lane's query elements (rotated with freqs; split 0 then writes the cache slot)
  float qv[QC][E];
  const TQ* qr = q + b * qsb + h * qsh + tq * qst;
  const float ph = static_cast<float>(pos + tq);
#pragma unroll
  for (int i = 0; i < QC; ++i) {
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const int n = coff0 + i * CS + e;
      float x[4] = {0.f, 0.f, 0.f, 0.f};
      if (i < nval) {
        load_q4(qr + n, qvec, x);
        if constexpr (ROT && !F8) {
          {
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
              float c0, s0, c1, s1;
              rope_cis(ph, freqs[n + j], c0, s0);
              rope_cis(ph, freqs[n + j + 1], c1, s1);
              const float x0 = x[j], x1 = x[j + 1];
              if (sizeof(TQ) == 2) {
                x[j] = bf16_round_d(__fadd_rn(bf16_round_d(__fmul_rn(x0, c0)),
                                              bf16_round_d(__fmul_rn(-x1, s0))));
                x[j + 1] = bf16_round_d(__fadd_rn(bf16_round_d(__fmul_rn(x1, c1)),
                                                  bf16_round_d(__fmul_rn(x0, s1))));
              } else {
                x[j] = __fsub_rn(__fmul_rn(x0, c0), __fmul_rn(x1, s0));
                x[j + 1] = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1));
              }
            }
            if (slot != nullptr && split == 0) {
              TK* sr = slot + b * ssb + h * ssh + tq * sst;
#pragma unroll
              for (int j = 0; j < 4; ++j) st_elem(sr, n + j, x[j]);
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) qv[i][e + j] = x[j];
    }
  }

  // 3. the rows, GR at a time; loads run kSliceAhead ahead across group boundaries
  const int groups = (rows + GR - 1) / GR;
  for (int g = 0; g < groups; ++g) {
    float acc[GR];
#pragma unroll
    for (int k = 0; k < GR; ++k) acc[k] = 0.f;
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const uint4 u = ring[t % DP];
      const int i = t % QC;
      uint4 nx = make_uint4(0, 0, 0, 0);
      if (lr < rows && i < nval) nx = __ldcs(reinterpret_cast<const uint4*>(lp + i * CS));
      ring[t % DP] = nx;
      if (i == QC - 1) {
        lp += kst;
        ++lr;
      }
      if constexpr (F8)
        acc[t / QC] += dot16_e4m3(qv[i], u);
      else
        acc[t / QC] += dot16<TK>(qv[i], u);
    }
    const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
    if constexpr (GR == 2) {
      // two values per lane -> lane (b4) holds the warp's sum for row b4
      float u1 = (b4 ? acc[1] : acc[0]) + __shfl_xor_sync(0xffffffffu, b4 ? acc[0] : acc[1], 16);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 8);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 4);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 2);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 1);
      (void)b3;
      (void)b2;
      if ((lane & 15) == 0) red[warp][g * 2 + b4] = u1;
    } else if constexpr (GR == 8) {
      // eight values per lane -> lane (b4 b3 b2) holds the warp's sum for row 4 b4 + 2 b3 + b2
      float u4[4], u2[2];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float keep = b4 ? acc[k + 4] : acc[k], send = b4 ? acc[k] : acc[k + 4];
        u4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float keep = b3 ? u4[k + 2] : u4[k], send = b3 ? u4[k] : u4[k + 2];
        u2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      float u1 = (b2 ? u2[1] : u2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? u2[0] : u2[1], 4);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 2);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 1);
      if ((lane & 3) == 0) red[warp][g * 8 + 4 * b4 + 2 * b3 + b2] = u1;
    } else {
      // four values per lane -> lane (b4 b3) holds the warp's sum for row 2 b4 + b3
      float u2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float keep = b4 ? acc[k + 2] : acc[k], send = b4 ? acc[k] : acc[k + 2];
        u2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
      float u1 = (b3 ? u2[1] : u2[0]) + __shfl_xor_sync(0xffffffffu, b3 ? u2[0] : u2[1], 8);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 4);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 2);
      u1 += __shfl_xor_sync(0xffffffffu, u1, 1);
      (void)b2;
      if ((lane & 7) == 0) red[warp][g * 4 + 2 * b4 + b3] = u1;
    }
  }
  __syncthreads();

  // 4. scores, then partial out = sum_j s_j V_j
  const float* cbase = F8 ? ksc + b * csb + h * csh : nullptr;
  for (int r = threadIdx.x; r < rows; r += kSliceWarps * 32) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kSliceWarps; ++w) s += red[w][r];
    sc[r] = F8 ? s * cbase[(j0 + r) * cst] : s;
  }
  __syncthreads();
  const TV* vbase = vp + b * vsb + hv * vsh;
  float* dst = partial + ((static_cast<int64_t>(split) * gridDim.y + bh) * gridDim.z + tq) * D;
  for (int d = threadIdx.x; d < D; d += kSliceWarps * 32) {
    float acc = 0.f;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) acc = fmaf(sc[r], ld_elem(vbase + (j0 + r) * vst, d), acc);
    dst[d] = acc;
  }
}

// Chunks per warp for the column-slice kernel: the smallest of 1, 2, 4, 8 (fp8: 1, 2; bf16:
// up to 4) with QC * 8 warps * 32 lanes * E >= N, or 0 when N is wider (the row-per-warp kernel
// then runs). The caps keep the lane's query slice (QC * E floats) at 32 registers, N <= 8192.
int slice_qc(int64_t N, int key_bytes) {
  const int64_t per = static_cast<int64_t>(kSliceWarps) * 32 * (16 / key_bytes);
  const int qmax = key_bytes == 1 ? 2 : key_bytes == 2 ? 4 : 8;
  for (int qc = 1; qc <= qmax; qc *= 2)
    if (qc * per >= N) return qc;
  return 0;
}

template <typename TQ, typename TK, typename TV, bool F8, bool ROT>
void launch_slice(int qc, dim3 grid, cudaStream_t stream, const TQ* q, const TK* k,
                  const float* ksc, const TV* v, float* partial, TK* slot, const float* freqs,
                  int H, int Hv, int S, int N, int D, const int64_t qs[4], const int64_t ks[4],
                  const int64_t cs[3], const int64_t vs[4], const int64_t ss[4], int64_t pos,
                  int rows, bool qvec) {
#define BDH_SLICE(QC)                                                                             \
  decode_slice_kernel<TQ, TK, TV, QC, F8, ROT><<<grid, kSliceWarps * 32, 0, stream>>>(           \
      q, k, ksc, v, partial, slot, freqs, H, Hv, S, N, D, qs[0], qs[1], qs[2], ks[0], ks[1],      \
      ks[2], cs[0], cs[1], cs[2], vs[0], vs[1], vs[2], ss[0], ss[1], ss[2], pos, rows, qvec)
  constexpr int kB = sizeof(TK);  // key bytes: the widest QC instantiated follows slice_qc
  switch (qc) {
    case 1: BDH_SLICE(1); break;
    case 2: BDH_SLICE(2); break;
    case 4:
      if constexpr (kB >= 2) BDH_SLICE(4);
      break;
    default:
      if constexpr (kB == 4) BDH_SLICE(8);
      break;
  }
#undef BDH_SLICE
}

// 16-byte (fp32) / 8-byte (bf16) vector loads of the query rows.
bool q_vec_ok(const void* q, int q_dtype, const int64_t qs[4]) {
  const uintptr_t al = q_dtype == BDH_DTYPE_F32 ? 15u : 7u;
  return (reinterpret_cast<uintptr_t>(q) & al) == 0 && qs[0] % 4 == 0 && qs[1] % 4 == 0 &&
         qs[2] % 4 == 0;
}

template <typename TO>
__global__ void decode_reduce_kernel(const float* __restrict__ partial, TO* __restrict__ out,
                                     int nsplit, int H, int Tq, int D, int64_t BHT, int64_t osb,
                                     int64_t osh, int64_t ost) {
  const int64_t row = blockIdx.x;  // (b*H + h)*Tq + tq
  const int tq = static_cast<int>(row % Tq);
  const int64_t bh = row / Tq;
  const int h = static_cast<int>(bh % H);
  const int64_t b = bh / H;
  TO* o = out + b * osb + h * osh + tq * ost;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < nsplit; ++s) acc += partial[(s * BHT + row) * D + d];
    st_elem(o, d, acc);
  }
}

}  // namespace

// Rows per CTA and split count. Measured on B200 (config-4 model, S ~ 520, N = 8192): the
// split-S stream runs best with about four or more resident waves of CTAs, and small batches
// need short splits to fill the GPU at all (B = 4: 16 rows beat 8, 32 and more). Rule: the
// largest of 64, 32, 16 rows that still gives >= 4 x resident CTAs (resident = the column-slice
// kernel's occupancy, two CTAs per SM), else 16; at B = 64 that is 64 rows, which the
// column-slice kernel streams as fast as 32. `max_splits` caps the split count.
DecodePlan plan_decode(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N, int64_t max_splits) {
  DecodePlan pl;
  const int64_t units = std::max<int64_t>(1, B * H * Tq);
  if (S <= 0) {
    pl.splits = 1;
    pl.rows = 1;
    return pl;
  }
  static const int forced_rows = [] {
    const char* e = std::getenv("BDH_SM100_DECODE_ROWS");
    return e ? std::atoi(e) : 0;
  }();
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &occ, decode_slice_kernel<float, float, float, 8, false, false>, kSliceWarps * 32, 0) !=
          cudaSuccess ||
      occ <= 0) {
    cudaGetLastError();
    occ = 2;
  }
  const int64_t resident = static_cast<int64_t>(sm_count(dev)) * occ;
  int rows = 16;
  if (forced_rows >= 8 && forced_rows <= kDecRowsMax) {
    rows = forced_rows;
  } else {
    for (int r = 64; r >= 16; r /= 2) {
      if (units * ((S + r - 1) / r) >= 4 * resident) {
        rows = r;
        break;
      }
    }
  }
  if (max_splits > 0)
    while (rows < kDecRowsMax && (S + rows - 1) / rows > max_splits) rows *= 2;
  // a forced row count that is not a power of two can double past the kernels' score stages
  // (sc[kDecRowsMax], the N + kDecRowsMax shared-memory stage): never plan more rows than they hold
  rows = std::min(rows, kDecRowsMax);
  pl.rows = static_cast<int>(std::min<int64_t>(rows, S));
  pl.splits = static_cast<int>((S + rows - 1) / rows);
  return pl;
}

size_t decode_partial_bytes(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N, int64_t D,
                            int64_t max_splits) {
  const DecodePlan pl = plan_decode(B, H, Tq, S, N, max_splits);
  return (static_cast<size_t>(pl.splits) * static_cast<size_t>(B * H * Tq * D) * sizeof(float) + 255) &
         ~static_cast<size_t>(255);
}

// Partial sums, then (fused RoPE only) the rotated queries as fp32 (B*H*Tq*N).
size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N, int64_t D) {
  return decode_partial_bytes(B, H, Tq, S, N, D, 0) + static_cast<size_t>(B * H * Tq * N) * sizeof(float);
}

int launch_decode(const DecodeArgs& a_in, float* partial, float* qrot, int64_t max_splits,
                  cudaStream_t stream) {
  if (a_in.B * a_in.H * a_in.Tq == 0 || a_in.D == 0) {
    return BDH_OK;
  }
  DecodeArgs a = a_in;
  // the output keeps the caller's query dtype even when the kernel reads rotated fp32 queries
  const bool out_f32 = a_in.q_dtype == BDH_DTYPE_F32;
  if (a.freqs != nullptr && qrot != nullptr) {
    // RoPE of the new queries once, with each (position, column) phase shared by all B*H rows
    // (the elementwise RoPE kernel), instead of once per split CTA: an fp32 copy for the dot
    // products and the storage-dtype copy in this step's cache slot.
    const int64_t qs[4] = {a.H * a.Tq * a.N, a.Tq * a.N, a.N, 1};
    if (a.slot != nullptr && a.kv_dtype == BDH_DTYPE_F32) {
      // an fp32 slot holds exactly the fp32 rotated queries: one pass, and the kernel reads them
      // from the slot (the position after the past it streams)
      int rc = launch_rope(a.q, a.q_dtype, a.q_strides, a.slot, BDH_DTYPE_F32, a.slot_strides,
                           nullptr, a.freqs, a.B, a.H, a.Tq, a.N, a.pos, 0, stream);
      if (rc) return rc;
      a.q = a.slot;
      for (int i = 0; i < 4; ++i) a.q_strides[i] = a.slot_strides[i];
    } else {
      int rc = launch_rope(a.q, a.q_dtype, a.q_strides, qrot, BDH_DTYPE_F32, qs, nullptr, a.freqs,
                           a.B, a.H, a.Tq, a.N, a.pos, 0, stream);
      if (rc) return rc;
      if (a.slot != nullptr) {
        rc = launch_rope(a.q, a.q_dtype, a.q_strides, a.slot, a.kv_dtype, a.slot_strides, nullptr,
                         a.freqs, a.B, a.H, a.Tq, a.N, a.pos, 0, stream);
        if (rc) return rc;
      }
      a.q = qrot;
      for (int i = 0; i < 4; ++i) a.q_strides[i] = qs[i];
    }
    a.q_dtype = BDH_DTYPE_F32;
    a.freqs = nullptr;
    a.slot = nullptr;
  }
  const DecodePlan pl = plan_decode(a.B, a.H, a.Tq, a.S, a.N, max_splits);
  const int nsplit = pl.splits;
  const int ke = a.kv_dtype == BDH_DTYPE_F32 ? 4 : 2;
  bool vec = (a.N % (16 / ke) == 0) && ((reinterpret_cast<uintptr_t>(a.k) & 15u) == 0) &&
             (a.k_strides[0] * ke) % 16 == 0 && (a.k_strides[1] * ke) % 16 == 0 &&
             (a.k_strides[2] * ke) % 16 == 0;
  if (a.freqs != nullptr && (a.N % 2) != 0) {
    set_error("decode: fused RoPE needs an even latent width");
    return BDH_ERR_INVALID;
  }
  const dim3 grid(static_cast<unsigned>(nsplit), static_cast<unsigned>(a.B * a.H),
                  static_cast<unsigned>(a.Tq));
  const size_t smem = (static_cast<size_t>(a.N) + kDecRowsMax) * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("decode: latent width too large for the shared-memory q stage");
    return BDH_ERR_INVALID;
  }
  const int Hi = static_cast<int>(a.H), Hvi = static_cast<int>(a.Hv), Tqi = static_cast<int>(a.Tq);
  const int Si = static_cast<int>(a.S), Ni = static_cast<int>(a.N), Di = static_cast<int>(a.D);
#define BDH_DEC_LAUNCH(TQ, TK, V)                                                                 \
  do {                                                                                            \
    auto kern = decode_partial_kernel<TQ, TK, V>;                                                 \
    if (smem > 48 * 1024)                                                                         \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,                     \
                           static_cast<int>(smem));                                               \
    kern<<<grid, kDecThreads, smem, stream>>>(                                                    \
        static_cast<const TQ*>(a.q), static_cast<const TK*>(a.k), static_cast<const TK*>(a.v),    \
        partial, static_cast<TK*>(a.slot), a.freqs, Hi, Hvi, Tqi, Si, Ni, Di, a.q_strides[0],     \
        a.q_strides[1], a.q_strides[2], a.k_strides[0], a.k_strides[1], a.k_strides[2],           \
        a.v_strides[0], a.v_strides[1], a.v_strides[2], a.slot_strides[0], a.slot_strides[1],     \
        a.slot_strides[2], a.pos, pl.rows);                                                       \
  } while (0)
  const bool qf = a.q_dtype == BDH_DTYPE_F32, kf = a.kv_dtype == BDH_DTYPE_F32;
  const int qc = vec ? slice_qc(a.N, ke) : 0;
  prof_start(kProfDecode, stream);
  if (qc > 0) {
    const bool qv = q_vec_ok(a.q, a.q_dtype, a.q_strides);
    const int64_t cs[3] = {0, 0, 0};
#define BDH_SLICE_GO(TQ, TK)                                                                      \
  do {                                                                                            \
    if (a.freqs != nullptr)                                                                       \
      launch_slice<TQ, TK, TK, false, true>(                                                      \
          qc, grid, stream, static_cast<const TQ*>(a.q), static_cast<const TK*>(a.k), nullptr,    \
          static_cast<const TK*>(a.v), partial, static_cast<TK*>(a.slot), a.freqs, Hi, Hvi, Si,   \
          Ni, Di, a.q_strides, a.k_strides, cs, a.v_strides, a.slot_strides, a.pos, pl.rows, qv); \
    else                                                                                          \
      launch_slice<TQ, TK, TK, false, false>(                                                     \
          qc, grid, stream, static_cast<const TQ*>(a.q), static_cast<const TK*>(a.k), nullptr,    \
          static_cast<const TK*>(a.v), partial, nullptr, nullptr, Hi, Hvi, Si, Ni, Di,            \
          a.q_strides, a.k_strides, cs, a.v_strides, a.slot_strides, a.pos, pl.rows, qv);         \
  } while (0)
    if (qf && kf) BDH_SLICE_GO(float, float);
    else if (qf) BDH_SLICE_GO(float, uint16_t);
    else if (kf) BDH_SLICE_GO(uint16_t, float);
    else BDH_SLICE_GO(uint16_t, uint16_t);
#undef BDH_SLICE_GO
  } else if (qf && kf) {
    if (vec) BDH_DEC_LAUNCH(float, float, true); else BDH_DEC_LAUNCH(float, float, false);
  } else if (qf) {
    if (vec) BDH_DEC_LAUNCH(float, uint16_t, true); else BDH_DEC_LAUNCH(float, uint16_t, false);
  } else if (kf) {
    if (vec) BDH_DEC_LAUNCH(uint16_t, float, true); else BDH_DEC_LAUNCH(uint16_t, float, false);
  } else {
    if (vec) BDH_DEC_LAUNCH(uint16_t, uint16_t, true); else BDH_DEC_LAUNCH(uint16_t, uint16_t, false);
  }
#undef BDH_DEC_LAUNCH
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("decode_partial_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  const int64_t bht = a.B * a.H * a.Tq;
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, a.D)));
  if (out_f32)
    decode_reduce_kernel<float><<<static_cast<unsigned>(bht), threads, 0, stream>>>(
        partial, static_cast<float*>(a.out), nsplit, Hi, Tqi, Di, bht, a.out_strides[0],
        a.out_strides[1], a.out_strides[2]);
  else
    decode_reduce_kernel<uint16_t><<<static_cast<unsigned>(bht), threads, 0, stream>>>(
        partial, static_cast<uint16_t*>(a.out), nsplit, Hi, Tqi, Di, bht, a.out_strides[0],
        a.out_strides[1], a.out_strides[2]);
  prof_stop(kProfDecode, stream);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("decode_reduce_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

int launch_decode_fp8(const DecodeFp8Args& a_in, float* partial, float* qrot, cudaStream_t stream) {
  if (a_in.B * a_in.H * a_in.Tq == 0 || a_in.D == 0) return BDH_OK;
  DecodeFp8Args a = a_in;
  const bool out_f32 = a_in.q_dtype == BDH_DTYPE_F32;
  if (a.freqs != nullptr) {
    // the new queries rotated once (fp32), then quantized into this step's cache slot
    const int64_t qs[4] = {a.H * a.Tq * a.N, a.Tq * a.N, a.N, 1};
    int rc = launch_rope(a.q, a.q_dtype, a.q_strides, qrot, BDH_DTYPE_F32, qs, nullptr, a.freqs,
                         a.B, a.H, a.Tq, a.N, a.pos, 0, stream);
    if (rc) return rc;
    if (a.slot != nullptr) {
      rc = launch_quantize_rows_fp8(qrot, BDH_DTYPE_F32, qs, a.B, a.H, a.Tq, a.N, a.slot,
                                    a.slot_strides, a.slot_scale, a.slot_scale_strides, stream);
      if (rc) return rc;
    }
    a.q = qrot;
    a.q_dtype = BDH_DTYPE_F32;
    for (int i = 0; i < 4; ++i) a.q_strides[i] = qs[i];
  }
  const DecodePlan pl = plan_decode(a.B, a.H, a.Tq, a.S, a.N, 0);
  const bool vec = (a.N % 16) == 0 && (reinterpret_cast<uintptr_t>(a.k) & 15u) == 0 &&
                   a.k_strides[0] % 16 == 0 && a.k_strides[1] % 16 == 0 && a.k_strides[2] % 16 == 0;
  const dim3 grid(static_cast<unsigned>(pl.splits), static_cast<unsigned>(a.B * a.H),
                  static_cast<unsigned>(a.Tq));
  const size_t smem = (static_cast<size_t>(a.N) + kDecRowsMax) * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("decode: latent width too large for the shared-memory q stage");
    return BDH_ERR_INVALID;
  }
  const int Hi = static_cast<int>(a.H), Hvi = static_cast<int>(a.Hv), Tqi = static_cast<int>(a.Tq);
  const int Si = static_cast<int>(a.S), Ni = static_cast<int>(a.N), Di = static_cast<int>(a.D);
#define BDH_DEC8_LAUNCH(TQ, TV, V)                                                               \
  do {                                                                                           \
    auto kern = decode_partial_fp8_kernel<TQ, TV, V>;                                            \
    if (smem > 48 * 1024)                                                                        \
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,                    \
                           static_cast<int>(smem));                                              \
    kern<<<grid, kDecThreads, smem, stream>>>(                                                   \
        static_cast<const TQ*>(a.q), a.k, a.k_scale, static_cast<const TV*>(a.v), partial, Hi,   \
        Hvi, Tqi, Si, Ni, Di, a.q_strides[0], a.q_strides[1], a.q_strides[2], a.k_strides[0],    \
        a.k_strides[1], a.k_strides[2], a.ks_strides[0], a.ks_strides[1], a.ks_strides[2],       \
        a.v_strides[0], a.v_strides[1], a.v_strides[2], pl.rows);                                \
  } while (0)
#define BDH_DEC8_V(TQ, TV) \
  do {                      \
    if (vec)                \
      BDH_DEC8_LAUNCH(TQ, TV, true); \
    else                    \
      BDH_DEC8_LAUNCH(TQ, TV, false); \
  } while (0)
  const bool qf = a.q_dtype == BDH_DTYPE_F32, vf = a.v_dtype == BDH_DTYPE_F32;
  const int qc = vec ? slice_qc(a.N, 1) : 0;
  prof_start(kProfDecode, stream);
  if (qc > 0) {
    const bool qv = q_vec_ok(a.q, a.q_dtype, a.q_strides);
    const int64_t ss[4] = {0, 0, 0, 1};
#define BDH_SLICE8_GO(TQ, TV)                                                                    \
  launch_slice<TQ, uint8_t, TV, true, false>(qc, grid, stream, static_cast<const TQ*>(a.q), a.k,       \
                                      a.k_scale, static_cast<const TV*>(a.v), partial, nullptr,  \
                                      nullptr, Hi, Hvi, Si, Ni, Di, a.q_strides, a.k_strides,    \
                                      a.ks_strides, a.v_strides, ss, 0, pl.rows, qv)
    if (qf && vf) BDH_SLICE8_GO(float, float);
    else if (qf) BDH_SLICE8_GO(float, uint16_t);
    else if (vf) BDH_SLICE8_GO(uint16_t, float);
    else BDH_SLICE8_GO(uint16_t, uint16_t);
#undef BDH_SLICE8_GO
  } else if (qf && vf) BDH_DEC8_V(float, float);
  else if (qf) BDH_DEC8_V(float, uint16_t);
  else if (vf) BDH_DEC8_V(uint16_t, float);
  else BDH_DEC8_V(uint16_t, uint16_t);
#undef BDH_DEC8_V
#undef BDH_DEC8_LAUNCH
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    prof_stop(kProfDecode, stream);
    set_error(std::string("decode_partial_fp8_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  const int64_t bht = a.B * a.H * a.Tq;
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, a.D)));
  if (out_f32)
    decode_reduce_kernel<float><<<static_cast<unsigned>(bht), threads, 0, stream>>>(
        partial, static_cast<float*>(a.out), pl.splits, Hi, Tqi, Di, bht, a.out_strides[0],
        a.out_strides[1], a.out_strides[2]);
  else
    decode_reduce_kernel<uint16_t><<<static_cast<unsigned>(bht), threads, 0, stream>>>(
        partial, static_cast<uint16_t*>(a.out), pl.splits, Hi, Tqi, Di, bht, a.out_strides[0],
        a.out_strides[1], a.out_strides[2]);
  prof_stop(kProfDecode, stream);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("decode_reduce_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

}  // namespace bdh

// ------------------------------------------------------------- allocation-free decode
// Some callers cannot obtain device memory when they call in. Examples: a serving process that
// reserves its whole device-memory budget up front and forbids allocations afterwards; a
// foreign-language host binding that has no device allocator to hand; a latency-critical loop
// where an allocation's possible implicit device synchronisation is not acceptable. For them
// bdh_tril_decode_noalloc runs the same decode with its per-split partial sums placed in one
// fixed array compiled into this library, instead of a caller-provided workspace.
namespace bdh {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB, held by every device that loads the library

static __device__ __align__(256) float g_decode_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of the array on the current device. In host code the array's name only
// stands for it; the real address must be looked up once per device, with that device current.
// The cached address belongs to the CUDA context it was looked up in: after cudaDeviceReset, or
// under another context on the same device, the module is loaded again and the array can move,
// so each cache entry records its context and a different current context repeats the lookup.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {nullptr};
CUcontext g_noalloc_ctx[64] = {nullptr};

float* noalloc_scratch(int* rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("tril_decode_noalloc: no usable current CUDA device");
    *rc = BDH_ERR_CUDA;
    return nullptr;
  }
  const CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr) {
    set_error("tril_decode_noalloc: the driver has no cuCtxGetCurrent");
    *rc = BDH_ERR_CUDA;
    return nullptr;
  }
  // null before the runtime has bound a context on this thread; the lookup below binds one
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error(std::string("tril_decode_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
      *rc = BDH_ERR_CUDA;
      return nullptr;
    }
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
      set_error("tril_decode_noalloc: no current CUDA context after the address lookup");
      *rc = BDH_ERR_CUDA;
      return nullptr;
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
    g_noalloc_ctx[dev] = ctx;
  }
  *rc = BDH_OK;
  return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace bdh

extern "C" int bdh_tril_decode_noalloc(const void* q, const int64_t q_strides[4], int q_dtype,
                                       const void* k_past, const int64_t k_strides[4],
                                       const void* v_past, const int64_t v_strides[4],
                                       int kv_dtype, void* out, const int64_t out_strides[4],
                                       int64_t B, int64_t H, int64_t Hv, int64_t Tq, int64_t S,
                                       int64_t N, int64_t D, const float* freqs, int64_t pos,
                                       void* kr_slot, const int64_t slot_strides[4],
                                       void* stream) {
  if (B < 0 || H < 0 || Tq < 0 || S < 0 || D < 0) {
    bdh::set_error("tril_decode_noalloc: negative size");
    return BDH_ERR_INVALID;
  }
  const int64_t bhtd = std::max<int64_t>(1, B * H * Tq * D);
  const int64_t cap_splits = std::max<int64_t>(1, static_cast<int64_t>(bdh::kNoAllocScratchBytes / sizeof(float)) / bhtd);
  const size_t need = bdh::decode_partial_bytes(B, H, Tq, S, N, D, cap_splits);
  if (need > bdh::kNoAllocScratchBytes) {
    std::ostringstream os;
    os << "tril_decode_noalloc: this problem needs " << need << " bytes of scratch "
       << "(splits * B * H * Tq * D * 4, splits = ceil(S / rows) with 16..128 rows per split) "
       << "but the built-in array holds " << bdh::kNoAllocScratchBytes
       << " bytes; use bdh_tril_decode with a workspace";
    bdh::set_error(os.str());
    return BDH_ERR_INVALID;
  }
  int rc = BDH_OK;
  float* scratch = bdh::noalloc_scratch(&rc);
  if (scratch == nullptr) return rc;
  // the partial sums only: the new queries are rotated inside the decode kernel
  return bdh::decode_entry(q, q_strides, q_dtype, k_past, k_strides, v_past, v_strides, kv_dtype,
                           out, out_strides, B, H, Hv, Tq, S, N, D, freqs, pos, kr_slot,
                           slot_strides, scratch, nullptr, cap_splits, stream);
}


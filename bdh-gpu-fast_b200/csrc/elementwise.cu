// HBM-bound elementwise kernels of the path:
//   * RoPE apply with in-register phase and sincos (no cos/sin tables in HBM), reproducing
//     the reference arithmetic step by step:
//       bdh.py:142-150   positions (fp32 arange) * freqs            -> fp32 product
//       bdh.py:119-122   (phase mod 1) * 2pi, then cos / sin         -> fp32
//       kernels/rope.py:108-126 pair rotation; for bf16 inputs every product is rounded to
//       bf16 before the bf16 add (the `.to(v.dtype)` casts).
//   * tf32 split of fp32 operands (hi = tf32 round-to-nearest, lo = x - hi) feeding the
//     3-product tf32 tensor-core path.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "tma_host.h"

namespace bdh {

namespace {

__device__ __forceinline__ float bf16_round(float x) { return bf16_round_f32(x); }

__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Rotate one (x0, x1) pair. BF16 = the input dtype is bf16 (products rounded before the add).
template <bool BF16>
__device__ __forceinline__ void rotate_pair(float x0, float x1, float c0, float s0, float c1,
                                            float s1, float& y0, float& y1) {
  if (BF16) {
    y0 = bf16_round(__fadd_rn(bf16_round(__fmul_rn(x0, c0)), bf16_round(__fmul_rn(-x1, s0))));
    y1 = bf16_round(__fadd_rn(bf16_round(__fmul_rn(x1, c1)), bf16_round(__fmul_rn(x0, s1))));
  } else {
    y0 = __fsub_rn(__fmul_rn(x0, c0), __fmul_rn(x1, s0));
    y1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1));
  }
}

__device__ __forceinline__ float load1(const uint16_t* p) { return bf16_bits_to_f32(*p); }
__device__ __forceinline__ float load1(const float* p) { return *p; }
__device__ __forceinline__ void store1(uint16_t* p, float v) {
  *p = static_cast<uint16_t>(f32_to_bf16_bits(v));
}
__device__ __forceinline__ void store1(float* p, float v) { *p = v; }

// Grid: x = (position t, 2048-element chunk of N), y = group of (b, h) rows. The (cos, sin)
// of a (t, n) pair is computed once per thread and reused for every (b, h) row of the
// group, so the trigonometry is amortised over B*H rows and the kernel runs at HBM speed.
// Each thread keeps U rows of raw 16-byte vectors in flight (streaming loads/stores: the
// latent is read once and the rotated copy is not re-read by this kernel).
template <typename TX>
struct RawVec {  // 8 elements of TX as raw 16-byte words
  static constexpr int W = sizeof(TX) * 8 / 16;
  uint4 w[W];
};

__device__ __forceinline__ void raw_load(const uint16_t* p, RawVec<uint16_t>& r) {
  r.w[0] = __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void raw_load(const float* p, RawVec<float>& r) {
  r.w[0] = __ldcs(reinterpret_cast<const uint4*>(p));
  r.w[1] = __ldcs(reinterpret_cast<const uint4*>(p) + 1);
}
__device__ __forceinline__ void raw_unpack(const RawVec<uint16_t>& r, float (&v)[8]) {
  const uint32_t w[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16_bits_to_f32(w[i] & 0xFFFFu);
    v[2 * i + 1] = bf16_bits_to_f32(w[i] >> 16);
  }
}
__device__ __forceinline__ void raw_unpack(const RawVec<float>& r, float (&v)[8]) {
  v[0] = __uint_as_float(r.w[0].x); v[1] = __uint_as_float(r.w[0].y);
  v[2] = __uint_as_float(r.w[0].z); v[3] = __uint_as_float(r.w[0].w);
  v[4] = __uint_as_float(r.w[1].x); v[5] = __uint_as_float(r.w[1].y);
  v[6] = __uint_as_float(r.w[1].z); v[7] = __uint_as_float(r.w[1].w);
}
__device__ __forceinline__ void store8_cs(uint16_t* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  __stcs(reinterpret_cast<uint4*>(p), u);
}
__device__ __forceinline__ void store8_cs(float* p, const float (&v)[8]) {
  __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
  __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(v[4], v[5], v[6], v[7]));
}

template <typename TX, typename TY, bool VEC>
__global__ void __launch_bounds__(256) rope_kernel(const TX* __restrict__ x, TY* __restrict__ y,
                                                   float* __restrict__ y_lo,
                                                   const float* __restrict__ freqs, int H, int T,
                                                   int N, int BH, int rows_per_group,
                                                   int64_t xsb, int64_t xsh, int64_t xst,
                                                   int64_t ysb, int64_t ysh, int64_t yst,
                                                   int64_t pos0, int relu_in) {
  constexpr bool BF16_IN = sizeof(TX) == 2;
  constexpr int E = VEC ? 8 : 2;  // elements per thread
  const int chunks = (N + 256 * E - 1) / (256 * E);
  const int t = static_cast<int>(blockIdx.x / chunks);
  const int n0 = static_cast<int>(blockIdx.x % chunks) * 256 * E + threadIdx.x * E;
  if (n0 >= N) return;
  const float pos = static_cast<float>(pos0 + t);
  float c[E], s[E];
  {
    float f[E];
    if (VEC) {
      const float4 fa = __ldg(reinterpret_cast<const float4*>(freqs + n0));
      const float4 fb = __ldg(reinterpret_cast<const float4*>(freqs + n0 + 4));
      f[0] = fa.x; f[1] = fa.y; f[2] = fa.z; f[3] = fa.w;
      f[4 % E] = fb.x; f[5 % E] = fb.y; f[6 % E] = fb.z; f[7 % E] = fb.w;
    } else {
      f[0] = __ldg(freqs + n0);
      f[1] = __ldg(freqs + n0 + 1);
    }
#pragma unroll
    for (int p = 0; p < E / 2; ++p) {
      rope_cis(pos, f[2 * p], c[2 * p], s[2 * p]);
      if (f[2 * p + 1] == f[2 * p]) {
        c[2 * p + 1] = c[2 * p];
        s[2 * p + 1] = s[2 * p];
      } else {
        rope_cis(pos, f[2 * p + 1], c[2 * p + 1], s[2 * p + 1]);
      }
    }
  }
  const int bh0 = blockIdx.y * rows_per_group;
  const int bh1 = min(BH, bh0 + rows_per_group);
  if (VEC) {
    constexpr int U = 8;  // rows in flight per thread
    for (int bh = bh0; bh < bh1; bh += U) {
      RawVec<TX> raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (bh + u < bh1) {
          const int r = bh + u;
          const int b = r / H, h = r - (r / H) * H;
          raw_load(x + b * xsb + h * xsh + t * xst + n0, raw[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (bh + u >= bh1) break;
        const int r = bh + u;
        const int b = r / H, h = r - (r / H) * H;
        float v[8], o[8];
        raw_unpack(raw[u], v);
        if (relu_in) {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = fmaxf(v[i], 0.0f);
        }
        const int64_t yo = b * ysb + h * ysh + t * yst + n0;
        if (BF16_IN && sizeof(TY) == 2 && y_lo == nullptr) {
          uint4 w;
          w.x = rotate_pair_bf16x2(v[0], v[1], c[0], s[0], c[1], s[1]);
          w.y = rotate_pair_bf16x2(v[2], v[3], c[2], s[2], c[3], s[3]);
          w.z = rotate_pair_bf16x2(v[4], v[5], c[4], s[4], c[5], s[5]);
          w.w = rotate_pair_bf16x2(v[6], v[7], c[6], s[6], c[7], s[7]);
          __stcs(reinterpret_cast<uint4*>(y + yo), w);
          continue;
        }
        if (BF16_IN) {
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint32_t w = rotate_pair_bf16x2(v[2 * p], v[2 * p + 1], c[2 * p], s[2 * p],
                                                  c[2 * p + 1], s[2 * p + 1]);
            o[2 * p] = bf16x2_lo(w);
            o[2 * p + 1] = bf16x2_hi(w);
          }
        } else {
#pragma unroll
          for (int p = 0; p < 4; ++p)
            rotate_pair<false>(v[2 * p], v[2 * p + 1], c[2 * p], s[2 * p], c[2 * p + 1],
                               s[2 * p + 1], o[2 * p], o[2 * p + 1]);
        }
        if (y_lo != nullptr) {
          float lo[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float hi = tf32_round(o[i]);
            lo[i] = o[i] - hi;
            o[i] = hi;
          }
          store8_cs(y_lo + yo, lo);
        }
        store8_cs(y + yo, o);
      }
    }
  } else {
    for (int r = bh0; r < bh1; ++r) {
      const int b = r / H, h = r - (r / H) * H;
      const TX* xr = x + b * xsb + h * xsh + t * xst + n0;
      float o0, o1;
      float x0 = load1(xr), x1 = load1(xr + 1);
      if (relu_in) {
        x0 = fmaxf(x0, 0.0f);
        x1 = fmaxf(x1, 0.0f);
      }
      rotate_pair<BF16_IN>(x0, x1, c[0], s[0], c[1], s[1], o0, o1);
      const int64_t yo = b * ysb + h * ysh + t * yst + n0;
      if (y_lo != nullptr) {
        const float h0 = tf32_round(o0), h1 = tf32_round(o1);
        y_lo[yo] = o0 - h0;
        y_lo[yo + 1] = o1 - h1;
        o0 = h0;
        o1 = h1;
      }
      store1(y + yo, o0);
      store1(y + yo + 1, o1);
    }
  }
}

template <bool VEC>
__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ x,
                                                         float* __restrict__ hi,
                                                         float* __restrict__ lo, int H, int T,
                                                         int N, int64_t xsb, int64_t xsh,
                                                         int64_t xst) {
  const int64_t row = blockIdx.x;
  const int t = static_cast<int>(row % T);
  const int64_t bh = row / T;
  const int h = static_cast<int>(bh % H);
  const int64_t b = bh / H;
  const float* xr = x + b * xsb + h * xsh + t * xst;
  float* hr = hi + row * N;
  float* lr = lo + row * N;
  if (VEC) {
    for (int n0 = threadIdx.x * 4; n0 < N; n0 += blockDim.x * 4) {
      const float4 a = *reinterpret_cast<const float4*>(xr + n0);
      const float4 ha = make_float4(tf32_round(a.x), tf32_round(a.y), tf32_round(a.z), tf32_round(a.w));
      *reinterpret_cast<float4*>(hr + n0) = ha;
      *reinterpret_cast<float4*>(lr + n0) = make_float4(a.x - ha.x, a.y - ha.y, a.z - ha.z, a.w - ha.w);
    }
  } else {
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
      const float a = xr[n];
      const float ha = tf32_round(a);
      hr[n] = ha;
      lr[n] = a - ha;
    }
  }
}

// Transposing split: x (B, H, T, N) -> hi/lo [B*H][N][ldt] through a 32 x 32 shared tile.
__global__ void __launch_bounds__(256) split_tf32_t_kernel(const float* __restrict__ x,
                                                           float* __restrict__ hi,
                                                           float* __restrict__ lo, int H, int T,
                                                           int N, int64_t ldt, int64_t xsb,
                                                           int64_t xsh, int64_t xst) {
  __shared__ float tile[32][33];
  const int bh = blockIdx.z;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int n0 = blockIdx.x * 32, t0 = blockIdx.y * 32;
  const float* xb = x + b * xsb + h * xsh;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int t = t0 + r, n = n0 + threadIdx.x;
    tile[r][threadIdx.x] = (t < T && n < N) ? xb[t * xst + n] : 0.0f;
  }
  __syncthreads();
  float* hb = hi + static_cast<int64_t>(bh) * N * ldt;
  float* lb = lo + static_cast<int64_t>(bh) * N * ldt;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int n = n0 + r, t = t0 + threadIdx.x;
    if (n < N && t < T) {
      const float v = tile[threadIdx.x][r];
      const float hv = tf32_round(v);
      hb[n * ldt + t] = hv;
      lb[n * ldt + t] = v - hv;
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_rope(const void* x, int x_dtype, const int64_t xs[4], void* y, int y_dtype,
                const int64_t ys[4], float* y_lo, const float* freqs, int64_t B, int64_t H,
                int64_t T, int64_t N, int64_t pos0, int relu_in, cudaStream_t stream) {
  const int64_t rows = B * H * T;
  if (rows == 0 || N == 0) return BDH_OK;
  const int xe = x_dtype == BDH_DTYPE_F32 ? 4 : 2;
  const int ye = y_dtype == BDH_DTYPE_F32 ? 4 : 2;
  bool vec = (N % 8 == 0) && aligned16(x) && aligned16(y) && aligned16(freqs) &&
             (y_lo == nullptr || aligned16(y_lo));
  for (int i = 0; i < 3; ++i) vec = vec && (xs[i] * xe) % 16 == 0 && (ys[i] * ye) % 16 == 0;
  const int E = vec ? 8 : 2;
  const int64_t chunks = (N + 256 * E - 1) / (256 * E);
  const int64_t gx = T * chunks;
  const int64_t BH = B * H;
  // Enough (b, h) groups to give every SM several CTAs, fewer when T already does.
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t want = 16LL * sm_count(dev);
  int64_t groups = std::min<int64_t>(BH, std::max<int64_t>(1, (want + gx - 1) / gx));
  const int64_t rpg = (BH + groups - 1) / groups;
  groups = (BH + rpg - 1) / rpg;
  if (gx > 0x7FFFFFFFLL || groups > 65535) {
    set_error("rope: grid too large");
    return BDH_ERR_INVALID;
  }
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(groups));
  const int Hi = static_cast<int>(H), Ti = static_cast<int>(T), Ni = static_cast<int>(N);
  const int BHi = static_cast<int>(BH), R = static_cast<int>(rpg);
#define BDH_ROPE_LAUNCH(TX, TY)                                                                   \
  do {                                                                                            \
    if (vec)                                                                                      \
      rope_kernel<TX, TY, true><<<grid, 256, 0, stream>>>(                                        \
          static_cast<const TX*>(x), static_cast<TY*>(y), y_lo, freqs, Hi, Ti, Ni, BHi, R, xs[0], \
          xs[1], xs[2], ys[0], ys[1], ys[2], pos0, relu_in);                                      \
    else                                                                                          \
      rope_kernel<TX, TY, false><<<grid, 256, 0, stream>>>(                                       \
          static_cast<const TX*>(x), static_cast<TY*>(y), y_lo, freqs, Hi, Ti, Ni, BHi, R, xs[0], \
          xs[1], xs[2], ys[0], ys[1], ys[2], pos0, relu_in);                                      \
  } while (0)
  prof_start(kProfRope, stream);
  if (x_dtype == BDH_DTYPE_BF16 && y_dtype == BDH_DTYPE_BF16) BDH_ROPE_LAUNCH(uint16_t, uint16_t);
  else if (x_dtype == BDH_DTYPE_BF16) BDH_ROPE_LAUNCH(uint16_t, float);
  else if (y_dtype == BDH_DTYPE_BF16) BDH_ROPE_LAUNCH(float, uint16_t);
  else BDH_ROPE_LAUNCH(float, float);
#undef BDH_ROPE_LAUNCH
  prof_stop(kProfRope, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("rope_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

int launch_split_tf32(const float* x, const int64_t xs[4], float* hi, float* lo, int64_t B,
                      int64_t H, int64_t T, int64_t N, cudaStream_t stream) {
  const int64_t rows = B * H * T;
  if (rows == 0 || N == 0) return BDH_OK;
  bool vec = (N % 4 == 0) && aligned16(x) && aligned16(hi) && aligned16(lo);
  for (int i = 0; i < 3; ++i) vec = vec && (xs[i] * 4) % 16 == 0;
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, N / 4)));
  prof_start(kProfSplit, stream);
  if (vec)
    split_tf32_kernel<true><<<static_cast<unsigned>(rows), threads, 0, stream>>>(
        x, hi, lo, static_cast<int>(H), static_cast<int>(T), static_cast<int>(N), xs[0], xs[1], xs[2]);
  else
    split_tf32_kernel<false><<<static_cast<unsigned>(rows), threads, 0, stream>>>(
        x, hi, lo, static_cast<int>(H), static_cast<int>(T), static_cast<int>(N), xs[0], xs[1], xs[2]);
  prof_stop(kProfSplit, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("split_tf32_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

int launch_split_tf32_t(const float* x, const int64_t xs[4], float* hi, float* lo, int64_t B,
                        int64_t H, int64_t T, int64_t N, int64_t ldt, cudaStream_t stream) {
  if (B * H * T * N == 0) return BDH_OK;
  const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((T + 31) / 32),
                  static_cast<unsigned>(B * H));
  prof_start(kProfSplit, stream);
  split_tf32_t_kernel<<<grid, dim3(32, 8), 0, stream>>>(x, hi, lo, static_cast<int>(H),
                                                        static_cast<int>(T), static_cast<int>(N),
                                                        ldt, xs[0], xs[1], xs[2]);
  prof_stop(kProfSplit, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("split_tf32_t_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

// out = relu(x) * relu(y) over (B, H, T, N) tensors with a contiguous last dimension and
// arbitrary other strides (the model's gated product x_sparse * y_sparse, reference
// bdh_baseline.py:124-126 / bdh.py:927-945, with both ReLUs folded in). Products are rounded
// once to the output dtype, as the eager op does.
template <typename TE, bool VEC>
__global__ void __launch_bounds__(256) relu_mul_kernel(const TE* __restrict__ x,
                                                       const TE* __restrict__ y, TE* __restrict__ o,
                                                       int H, int T, int N, int64_t xsb,
                                                       int64_t xsh, int64_t xst, int64_t ysb,
                                                       int64_t ysh, int64_t yst, int64_t osb,
                                                       int64_t osh, int64_t ost) {
  const int64_t row = blockIdx.x;
  const int t = static_cast<int>(row % T);
  const int64_t bh = row / T;
  const int h = static_cast<int>(bh % H);
  const int64_t b = bh / H;
  const TE* xr = x + b * xsb + h * xsh + t * xst;
  const TE* yr = y + b * ysb + h * ysh + t * yst;
  TE* orow = o + b * osb + h * osh + t * ost;
  if (VEC) {
    for (int n0 = threadIdx.x * 8; n0 < N; n0 += blockDim.x * 8) {
      RawVec<TE> rx, ry;
      raw_load(xr + n0, rx);
      raw_load(yr + n0, ry);
      float vx[8], vy[8], vo[8];
      raw_unpack(rx, vx);
      raw_unpack(ry, vy);
#pragma unroll
      for (int i = 0; i < 8; ++i) vo[i] = __fmul_rn(fmaxf(vx[i], 0.0f), fmaxf(vy[i], 0.0f));
      store8_cs(orow + n0, vo);
    }
  } else {
    for (int n = threadIdx.x; n < N; n += blockDim.x)
      store1(orow + n, __fmul_rn(fmaxf(load1(xr + n), 0.0f), fmaxf(load1(yr + n), 0.0f)));
  }
}

int launch_relu_mul(const void* x, const int64_t xs[4], const void* y, const int64_t ys[4],
                    void* out, const int64_t os[4], int dtype, int64_t B, int64_t H, int64_t T,
                    int64_t N, cudaStream_t stream) {
  const int64_t rows = B * H * T;
  if (rows == 0 || N == 0) return BDH_OK;
  const int es = dtype == BDH_DTYPE_F32 ? 4 : 2;
  bool vec = (N % 8 == 0) && aligned16(x) && aligned16(y) && aligned16(out);
  for (int i = 0; i < 3; ++i)
    vec = vec && (xs[i] * es) % 16 == 0 && (ys[i] * es) % 16 == 0 && (os[i] * es) % 16 == 0;
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, N / 8)));
  const int Hi = static_cast<int>(H), Ti = static_cast<int>(T), Ni = static_cast<int>(N);
#define BDH_RM_LAUNCH(TE)                                                                         \
  do {                                                                                            \
    if (vec)                                                                                      \
      relu_mul_kernel<TE, true><<<static_cast<unsigned>(rows), threads, 0, stream>>>(             \
          static_cast<const TE*>(x), static_cast<const TE*>(y), static_cast<TE*>(out), Hi, Ti,   \
          Ni, xs[0], xs[1], xs[2], ys[0], ys[1], ys[2], os[0], os[1], os[2]);                    \
    else                                                                                          \
      relu_mul_kernel<TE, false><<<static_cast<unsigned>(rows), threads, 0, stream>>>(            \
          static_cast<const TE*>(x), static_cast<const TE*>(y), static_cast<TE*>(out), Hi, Ti,   \
          Ni, xs[0], xs[1], xs[2], ys[0], ys[1], ys[2], os[0], os[1], os[2]);                    \
  } while (0)
  prof_start(kProfOther, stream);
  if (dtype == BDH_DTYPE_F32) BDH_RM_LAUNCH(float); else BDH_RM_LAUNCH(uint16_t);
#undef BDH_RM_LAUNCH
  prof_stop(kProfOther, stream);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("relu_mul_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

}  // namespace bdh

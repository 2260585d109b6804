// Recurrent-state decode: the cached T = 1 step of the strictly causal linear attention kept as
// an N x D state per (b, h) instead of a key/value history,
//
//   S_t = sum_{j < t} k_j v_j^T          (k = the rotated query, K is Q in BDH)
//   out_t = q_t^T S_t,   then   S_{t+1} = S_t + q_t v_t^T,
//
// which equals the KV form out_t = sum_{j<t} (q_t . k_j) v_j (kernels/attention.py:193-219,
// bdh_cache.py:226-324 for the history it replaces) up to fp32 summation order. Each step reads
// and writes the state once, independent of the past length, and a latent row n whose rotated
// query is zero (both entries of its RoPE pair zero after the encoder's ReLU) neither contributes
// to out nor changes S, so it is skipped: no read, no write.
//
// Grid = (N / kRows chunks, B * H); one warp owns a row at a time, each lane 8 of the D = 256
// columns (16-byte loads and stores). Per-chunk partial outputs are summed in a fixed order by
// the decode reduce (deterministic).
#include <algorithm>
#include <string>

#include "bdh_sm100.h"
#include "common.cuh"
#include "internal.h"
#include "tma_host.h"

namespace bdh {

namespace {

constexpr int kStThreads = 256;
constexpr int kStWarps = kStThreads / 32;
constexpr int kStRows = 128;     // latent rows per CTA
constexpr int kStMaxD = 512;     // 16 columns per lane at most

template <typename TV>
__device__ __forceinline__ float ld_v(const TV* p, int i);
template <>
__device__ __forceinline__ float ld_v<float>(const float* p, int i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ld_v<uint16_t>(const uint16_t* p, int i) {
  return bf16_bits_to_f32(p[i]);
}

// CPL = columns per lane (D / 32, a multiple of 4).
template <typename TV, int CPL>
__global__ void __launch_bounds__(kStThreads) state_decode_kernel(
    const float* __restrict__ qrot, float* __restrict__ S, const TV* __restrict__ v,
    float* __restrict__ partial, int H, int Hv, int N, int D, int64_t qsb, int64_t qsh,
    int64_t ssb, int64_t ssh, int64_t ssn, int64_t vsb, int64_t vsh) {
  __shared__ float ys[kStWarps][kStMaxD];
  const int chunk = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh - (bh / H) * H;
  const int hv = Hv == 1 ? 0 : h;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d0 = lane * CPL;
  const bool active = d0 < D;
  float vv[CPL], acc[CPL];
  const TV* vr = v + b * vsb + hv * vsh;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    vv[i] = active ? ld_v<TV>(vr, d0 + i) : 0.0f;
    acc[i] = 0.0f;
  }
  const float* qr = qrot + b * qsb + h * qsh;
  float* Sb = S + b * ssb + h * ssh;
  const int n_lo = chunk * kStRows;
  const int n_hi = min(N, n_lo + kStRows);
  for (int n = n_lo + warp; n < n_hi; n += kStWarps) {
    const float qn = __ldg(qr + n);
    if (qn == 0.0f || !active) continue;  // warp-uniform: the row is neither read nor written
    float* row = Sb + n * ssn + d0;
    float s[CPL];
#pragma unroll
    for (int i = 0; i < CPL; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(row + i);
      s[i] = t.x; s[i + 1] = t.y; s[i + 2] = t.z; s[i + 3] = t.w;
    }
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      acc[i] = fmaf(qn, s[i], acc[i]);   // out uses the state before this step's update
      s[i] = fmaf(qn, vv[i], s[i]);      // S += q v^T
    }
#pragma unroll
    for (int i = 0; i < CPL; i += 4)
      *reinterpret_cast<float4*>(row + i) = make_float4(s[i], s[i + 1], s[i + 2], s[i + 3]);
  }
  if (active) {
#pragma unroll
    for (int i = 0; i < CPL; ++i) ys[warp][d0 + i] = acc[i];
  }
  __syncthreads();
  float* dst = partial + (static_cast<int64_t>(chunk) * gridDim.y + bh) * D;
  for (int d = threadIdx.x; d < D; d += kStThreads) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kStWarps; ++w) t += ys[w][d];
    dst[d] = t;
  }
}

template <typename TO>
__global__ void state_reduce_kernel(const float* __restrict__ partial, TO* __restrict__ out,
                                    int nchunk, int H, int D, int64_t BH, int64_t osb,
                                    int64_t osh) {
  const int64_t bh = blockIdx.x;
  const int h = static_cast<int>(bh % H);
  const int64_t b = bh / H;
  TO* o = out + b * osb + h * osh;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.0f;
    for (int c = 0; c < nchunk; ++c) acc += partial[(c * BH + bh) * D + d];
    if constexpr (sizeof(TO) == 4)
      o[d] = acc;
    else
      o[d] = static_cast<uint16_t>(f32_to_bf16_bits(acc));
  }
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

}  // namespace

size_t state_decode_partial_bytes(int64_t B, int64_t H, int64_t N, int64_t D) {
  const int64_t nchunk = (N + kStRows - 1) / kStRows;
  return (static_cast<size_t>(nchunk * B * H * D) * sizeof(float) + 255) & ~static_cast<size_t>(255);
}

size_t state_decode_workspace_bytes(int64_t B, int64_t H, int64_t N, int64_t D) {
  return state_decode_partial_bytes(B, H, N, D) + static_cast<size_t>(B * H * N) * sizeof(float);
}

int launch_state_decode(const StateDecodeArgs& a, float* partial, float* qrot, cudaStream_t stream) {
  if (a.B * a.H == 0 || a.D == 0) return BDH_OK;
  // 1. the rotated query, once per step (phases shared by all B*H rows)
  const int64_t qs[4] = {a.H * a.N, a.N, a.N, 1};
  int rc = launch_rope(a.q, a.q_dtype, a.q_strides, qrot, BDH_DTYPE_F32, qs, nullptr, a.freqs, a.B,
                       a.H, 1, a.N, a.pos, a.relu_input, stream);
  if (rc) return rc;
  // 2. out partials + in-place state update
  const int nchunk = static_cast<int>((a.N + kStRows - 1) / kStRows);
  const dim3 grid(static_cast<unsigned>(nchunk), static_cast<unsigned>(a.B * a.H));
  const int cpl = static_cast<int>((a.D + 31) / 32);
  const int Hi = static_cast<int>(a.H), Hvi = static_cast<int>(a.Hv), Ni = static_cast<int>(a.N),
            Di = static_cast<int>(a.D);
  prof_start(kProfDecode, stream);
#define BDH_ST_LAUNCH(TV, CPL)                                                                  \
  state_decode_kernel<TV, CPL><<<grid, kStThreads, 0, stream>>>(                                \
      qrot, a.state, static_cast<const TV*>(a.v), partial, Hi, Hvi, Ni, Di, qs[0], qs[1],       \
      a.state_strides[0], a.state_strides[1], a.state_strides[2], a.v_strides[0], a.v_strides[1])
#define BDH_ST_DISPATCH(TV)                      \
  switch (cpl <= 4 ? 4 : cpl <= 8 ? 8 : 16) {    \
    case 4: BDH_ST_LAUNCH(TV, 4); break;         \
    case 8: BDH_ST_LAUNCH(TV, 8); break;         \
    default: BDH_ST_LAUNCH(TV, 16); break;       \
  }
  if (a.v_dtype == BDH_DTYPE_F32) {
    BDH_ST_DISPATCH(float)
  } else {
    BDH_ST_DISPATCH(uint16_t)
  }
#undef BDH_ST_DISPATCH
#undef BDH_ST_LAUNCH
  rc = check_launch("state_decode_kernel launch");
  if (rc) {
    prof_stop(kProfDecode, stream);
    return rc;
  }
  // 3. fixed-order sum of the chunk partials
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, a.D)));
  if (a.q_dtype == BDH_DTYPE_F32)
    state_reduce_kernel<float><<<static_cast<unsigned>(a.B * a.H), threads, 0, stream>>>(
        partial, static_cast<float*>(a.out), nchunk, Hi, Di, a.B * a.H, a.out_strides[0],
        a.out_strides[1]);
  else
    state_reduce_kernel<uint16_t><<<static_cast<unsigned>(a.B * a.H), threads, 0, stream>>>(
        partial, static_cast<uint16_t*>(a.out), nchunk, Hi, Di, a.B * a.H, a.out_strides[0],
        a.out_strides[1]);
  prof_stop(kProfDecode, stream);
  return check_launch("state_reduce_kernel launch");
}

}  // namespace bdh

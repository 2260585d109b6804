// Forward strict-causal linear attention on tcgen05:
//   out[b,h] = tril(Q[b,h] K[b,h]^T, -1) V[b,hv]        (hv = h, or 0 when V is shared)
//
// Two persistent tensor-core passes over the (b,h) units:
//   1. score pass : P = tril(Q K^T, -1) over the lower-triangular 128 x BN tiles, K-loop
//                   over the latent width N. P is written once as an exact split pair
//                   (bf16 hi + bf16 lo, or tf32 hi + fp32 lo for fp32 inputs) so that the
//                   second pass keeps fp32-level accuracy on tensor cores.
//   2. value pass : out = P V with the K-loop over keys limited to the causal prefix of each
//                   128-row query block (longest blocks scheduled first).
// Semantics follow the reference kernels (csrc/tril_attn_cuda.cu:129-249) and eager path
// (kernels/attention.py:27-40): no softmax, no scale, diagonal excluded, V broadcast over
// heads when it has one head.
#include <algorithm>

#include "bdh_sm100.h"
#include "internal.h"
#include "tc_engine.cuh"
#include "tma_host.h"

namespace bdh {

__device__ __forceinline__ int ceil_div_d(int a, int b) { return (a + b - 1) / b; }

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// --------------------------------------------------------------- score pass ----
// ELEM 2: bf16 operands, one term each; output bf16 hi/lo.
// ELEM 4: tf32 operands, hi/lo terms each (3 products); output fp32 (tf32 hi, fp32 lo).
template <int ELEM, int BN, int STAGES>
struct ScoreProb {
  static constexpr int TERMS = ELEM == 2 ? 1 : 2;
  using S = TcShape<ELEM, BN, false, false, TERMS, TERMS, STAGES>;
  struct Params {
    CUtensorMap a_map[2];  // query rows of Q (hi, lo), box BK x 128
    CUtensorMap b_map[2];  // key rows of K (hi, lo), box BK x BN
    int H, T, K;           // heads, sequence length, contraction (latent) width
    int mt;                // 128-row query blocks per unit
    int tiles_per_unit;
    int units;
    void* p_hi;            // [units][T][ldp]
    void* p_lo;
    int64_t ldp;
    int* err;
  };
  struct Tile {
    int unit, mi, ni;
  };

  __device__ static int nt_for(const Params& p, int mi) {
    return ceil_div_d(min(p.T, (mi + 1) * S::BM), BN);
  }
  __device__ static int num_tiles(const Params& p) { return p.units * p.tiles_per_unit; }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    tl.unit = t / p.tiles_per_unit;
    int r = t - tl.unit * p.tiles_per_unit;
    int mi = 0;
    for (;; ++mi) {
      const int c = nt_for(p, mi);
      if (r < c) break;
      r -= c;
    }
    tl.mi = mi;
    tl.ni = r;
    return tl;
  }
  __device__ static int k_blocks(const Params& p, const Tile&) { return ceil_div_d(p.K, S::BK); }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x7u; }
  __device__ static void prefetch(const Params& p) {
    for (int i = 0; i < TERMS; ++i) {
      tma_prefetch_desc(&p.a_map[i]);
      tma_prefetch_desc(&p.b_map[i]);
    }
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    for (int i = 0; i < TERMS; ++i) {
      tma_load_4d(&p.a_map[i], bar, a_dst + i * S::A_TILE, kb * S::BK, tl.mi * S::BM, h, b);
      tma_load_4d(&p.b_map[i], bar, b_dst + i * S::B_TILE, kb * S::BK, tl.ni * BN, h, b);
    }
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int row, int c0,
                                  const uint32_t (&r)[32]) {
    const int gi = tl.mi * S::BM + row;
    if (gi >= p.T) return;
    const int gj_base = tl.ni * BN + c0;
    const size_t row_off = (static_cast<size_t>(tl.unit) * p.T + gi) * static_cast<size_t>(p.ldp);
    if (ELEM == 2) {
      uint16_t* hi = static_cast<uint16_t*>(p.p_hi) + row_off;
      uint16_t* lo = static_cast<uint16_t*>(p.p_lo) + row_off;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int gj0 = gj_base + 8 * v;
        if (gj0 + 8 > p.ldp) continue;
        uint32_t wh[4], wl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int gj = gj0 + 2 * e;
          const float x0 = gj < gi ? __uint_as_float(r[8 * v + 2 * e]) : 0.0f;
          const float x1 = gj + 1 < gi ? __uint_as_float(r[8 * v + 2 * e + 1]) : 0.0f;
          const uint32_t h0 = f32_to_bf16_bits(x0), h1 = f32_to_bf16_bits(x1);
          const float l0 = x0 - bf16_bits_to_f32(h0), l1 = x1 - bf16_bits_to_f32(h1);
          wh[e] = h0 | (h1 << 16);
          wl[e] = f32_to_bf16_bits(l0) | (f32_to_bf16_bits(l1) << 16);
        }
        *reinterpret_cast<uint4*>(hi + gj0) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
        *reinterpret_cast<uint4*>(lo + gj0) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
      }
    } else {
      float* hi = static_cast<float*>(p.p_hi) + row_off;
      float* lo = static_cast<float*>(p.p_lo) + row_off;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int gj0 = gj_base + 4 * v;
        if (gj0 + 4 > p.ldp) continue;
        float h4[4], l4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int gj = gj0 + e;
          const float x = gj < gi ? __uint_as_float(r[4 * v + e]) : 0.0f;
          h4[e] = tf32_rna(x);
          l4[e] = x - h4[e];
        }
        *reinterpret_cast<float4*>(hi + gj0) = make_float4(h4[0], h4[1], h4[2], h4[3]);
        *reinterpret_cast<float4*>(lo + gj0) = make_float4(l4[0], l4[1], l4[2], l4[3]);
      }
    }
  }
};

// --------------------------------------------------------------- value pass ----
// A = P (K-major over keys, hi/lo terms).
// ELEM 2: B = V as stored, MN-major (D contiguous); bf16 P hi/lo x bf16 V (2 products).
// ELEM 4: B = V^T hi/lo written by the tf32 split (K-major, keys contiguous); 3 products.
template <int ELEM, int STAGES>
struct ValueProb {
  static constexpr int BN = 256;
  static constexpr bool B_MN = ELEM == 2;
  static constexpr int B_TERMS = ELEM == 2 ? 1 : 2;
  using S = TcShape<ELEM, BN, false, B_MN, 2, B_TERMS, STAGES>;
  static constexpr int CHUNK = 128 / ELEM;  // MN elements per 128-byte chunk
  struct Params {
    CUtensorMap a_map[2];  // P hi / lo over [units][T][T], box BK x 128
    CUtensorMap b_map[2];  // bf16: V (B, Hv, T, D), box CHUNK x BK; tf32: V^T [B*Hv][D][T], box BK x 256
    int H, Hv, T, D;
    int mt, nd;            // query blocks, 256-wide D tiles
    int units;
    void* out;             // (B, H, T, D) strided, out_f32 ? float : bf16
    int64_t os_b, os_h, os_t;
    int out_f32;
    int vec_ok;
    int* err;
  };
  struct Tile {
    int unit, mi, ni;
  };
  __device__ static int num_tiles(const Params& p) { return p.units * p.mt * p.nd; }
  __device__ static Tile tile(const Params& p, int t) {
    // Longest (last) query blocks first for balance across the persistent CTAs.
    Tile tl;
    const int per_block = p.units * p.nd;
    const int rev = t / per_block;
    const int rem = t - rev * per_block;
    tl.mi = p.mt - 1 - rev;
    tl.unit = rem / p.nd;
    tl.ni = rem - tl.unit * p.nd;
    return tl;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) {
    return ceil_div_d(min(p.T, (tl.mi + 1) * S::BM), S::BK);
  }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x7u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map[0]);
    tma_prefetch_desc(&p.a_map[1]);
    for (int i = 0; i < B_TERMS; ++i) tma_prefetch_desc(&p.b_map[i]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int hv = p.Hv == 1 ? 0 : h;
    for (int i = 0; i < 2; ++i)
      tma_load_4d(&p.a_map[i], bar, a_dst + i * S::A_TILE, kb * S::BK, tl.mi * S::BM, tl.unit, 0);
    if (B_MN) {
#pragma unroll
      for (int c = 0; c < BN / CHUNK; ++c)
        tma_load_4d(&p.b_map[0], bar, b_dst + c * S::BK * 128, tl.ni * BN + c * CHUNK,
                    kb * S::BK, hv, b);
    } else {
      for (int i = 0; i < B_TERMS; ++i)
        tma_load_4d(&p.b_map[i], bar, b_dst + i * S::B_TILE, kb * S::BK, tl.ni * BN,
                    b * p.Hv + hv, 0);
    }
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int row, int c0,
                                  const uint32_t (&r)[32]) {
    const int gi = tl.mi * S::BM + row;
    if (gi >= p.T) return;
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int gd0 = tl.ni * BN + c0;
    const int64_t off = b * p.os_b + h * p.os_h + gi * p.os_t + gd0;
    if (p.out_f32) {
      float* o = static_cast<float*>(p.out) + off;
      if (p.vec_ok && gd0 + 32 <= p.D) {
#pragma unroll
        for (int v = 0; v < 8; ++v)
          *reinterpret_cast<float4*>(o + 4 * v) =
              make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                          __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
      } else {
        for (int e = 0; e < 32 && gd0 + e < p.D; ++e) o[e] = __uint_as_float(r[e]);
      }
    } else {
      uint16_t* o = static_cast<uint16_t*>(p.out) + off;
      if (p.vec_ok && gd0 + 32 <= p.D) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = pack_bf16x2(__uint_as_float(r[8 * v + 2 * e]),
                               __uint_as_float(r[8 * v + 2 * e + 1]));
          *reinterpret_cast<uint4*>(o + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        for (int e = 0; e < 32 && gd0 + e < p.D; ++e)
          o[e] = static_cast<uint16_t>(f32_to_bf16_bits(__uint_as_float(r[e])));
      }
    }
  }
};

// ----------------------------------------------------------------- launchers ----
template <class S, class P>
static int launch_tc(const typename P::Params& prm, int ntiles, cudaStream_t stream) {
  if (ntiles <= 0) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<S, P>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::SMEM_BYTES);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return BDH_ERR_CUDA;
    }
    attr_set[dev] = true;
  }
  const int grid = std::min(ntiles, sm_count(dev));
  tc_gemm_kernel<S, P><<<grid, kTcThreads, S::SMEM_BYTES, stream>>>(prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("tc_gemm_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return 0;
}

using ScoreBf16 = ScoreProb<2, 128, 6>;
using ScoreTf32 = ScoreProb<4, 128, 3>;
using ValueBf16 = ValueProb<2, 3>;
using ValueTf32 = ValueProb<4, 2>;

int64_t score_ld(int64_t T) { return (T + 7) / 8 * 8; }
int64_t vt_ld(int64_t T) { return (T + 3) / 4 * 4; }

// Score pass: P = tril(Q K^T, -1) written as a hi/lo pair into p_hi / p_lo ([B*H][T][ldp]).
int launch_score(const FwdArgs& a, void* p_hi, void* p_lo, cudaStream_t stream, int* err) {
  const int elem = a.dtype == BDH_DTYPE_F32 ? 4 : 2;
  const int64_t ldp = score_ld(a.T);
  const int64_t units = a.B * a.H;
  auto fill = [&](auto& prm, int bk, int bn) -> bool {
    const int terms = elem == 2 ? 1 : 2;
    for (int i = 0; i < terms; ++i) {
      const void* qb = i == 0 ? a.q : a.q_lo;
      const void* kb = i == 0 ? a.k : a.k_lo;
      int64_t qd[4] = {a.N, a.T, a.H, a.B};
      int64_t qs[3] = {a.q_strides[2] * elem, a.q_strides[1] * elem, a.q_strides[0] * elem};
      int64_t ks[3] = {a.k_strides[2] * elem, a.k_strides[1] * elem, a.k_strides[0] * elem};
      if (!make_map_4d(&prm.a_map[i], qb, elem, qd, qs, bk, 128, "score pass: q")) return false;
      if (!make_map_4d(&prm.b_map[i], kb, elem, qd, ks, bk, bn, "score pass: k")) return false;
    }
    prm.H = static_cast<int>(a.H);
    prm.T = static_cast<int>(a.T);
    prm.K = static_cast<int>(a.N);
    prm.mt = static_cast<int>((a.T + 127) / 128);
    int tpu = 0;
    for (int mi = 0; mi < prm.mt; ++mi) {
      const int64_t lim = std::min<int64_t>(a.T, int64_t(mi + 1) * 128);
      tpu += static_cast<int>((lim + bn - 1) / bn);
    }
    prm.tiles_per_unit = tpu;
    prm.units = static_cast<int>(units);
    prm.p_hi = p_hi;
    prm.p_lo = p_lo;
    prm.ldp = ldp;
    prm.err = err;
    return true;
  };
  if (elem == 2) {
    ScoreBf16::Params prm{};
    if (!fill(prm, ScoreBf16::S::BK, 128)) return BDH_ERR_INVALID;
    return launch_tc<ScoreBf16::S, ScoreBf16>(prm, prm.units * prm.tiles_per_unit, stream);
  } else {
    ScoreTf32::Params prm{};
    if (!fill(prm, ScoreTf32::S::BK, 128)) return BDH_ERR_INVALID;
    return launch_tc<ScoreTf32::S, ScoreTf32>(prm, prm.units * prm.tiles_per_unit, stream);
  }
}

// Value pass: out = P V from the hi/lo score pair.
int launch_value(const FwdArgs& a, const void* p_hi, const void* p_lo, cudaStream_t stream,
                 int* err) {
  const int elem = a.dtype == BDH_DTYPE_F32 ? 4 : 2;
  const int64_t ldp = score_ld(a.T);
  const int64_t units = a.B * a.H;
  auto fill = [&](auto& prm, int bk) -> bool {
    const int64_t pd[4] = {a.T, a.T, units, 1};
    const int64_t ps[3] = {ldp * elem, a.T * ldp * elem, units * a.T * ldp * elem};
    if (!make_map_4d(&prm.a_map[0], p_hi, elem, pd, ps, bk, 128, "value pass: P hi")) return false;
    if (!make_map_4d(&prm.a_map[1], p_lo, elem, pd, ps, bk, 128, "value pass: P lo")) return false;
    if (elem == 2) {
      int64_t vd[4] = {a.D, a.T, a.Hv, a.B};
      int64_t vs[3] = {a.v_strides[2] * elem, a.v_strides[1] * elem, a.v_strides[0] * elem};
      if (!make_map_4d(&prm.b_map[0], a.v, elem, vd, vs, 128 / elem, bk, "value pass: v"))
        return false;
    } else {
      // tf32: V^T hi/lo, [B*Hv][D][ldt] with keys contiguous (written by the split pass).
      const int64_t ldt = vt_ld(a.T);
      int64_t vd[4] = {a.T, a.D, a.B * a.Hv, 1};
      int64_t vs[3] = {ldt * 4, a.D * ldt * 4, a.B * a.Hv * a.D * ldt * 4};
      if (!make_map_4d(&prm.b_map[0], a.v, 4, vd, vs, bk, 256, "value pass: v^T hi")) return false;
      if (!make_map_4d(&prm.b_map[1], a.v_lo, 4, vd, vs, bk, 256, "value pass: v^T lo")) return false;
    }
    prm.H = static_cast<int>(a.H);
    prm.Hv = static_cast<int>(a.Hv);
    prm.T = static_cast<int>(a.T);
    prm.D = static_cast<int>(a.D);
    prm.mt = static_cast<int>((a.T + 127) / 128);
    prm.nd = static_cast<int>((a.D + 255) / 256);
    prm.units = static_cast<int>(units);
    prm.out = a.out;
    prm.os_b = a.out_strides[0];
    prm.os_h = a.out_strides[1];
    prm.os_t = a.out_strides[2];
    prm.out_f32 = a.out_dtype == BDH_DTYPE_F32 ? 1 : 0;
    const int oes = prm.out_f32 ? 4 : 2;
    prm.vec_ok = ((reinterpret_cast<uintptr_t>(a.out) & 15u) == 0 && (a.out_strides[0] * oes) % 16 == 0 &&
                  (a.out_strides[1] * oes) % 16 == 0 && (a.out_strides[2] * oes) % 16 == 0)
                     ? 1
                     : 0;
    prm.err = err;
    return true;
  };
  if (elem == 2) {
    ValueBf16::Params prm{};
    if (!fill(prm, ValueBf16::S::BK)) return BDH_ERR_INVALID;
    return launch_tc<ValueBf16::S, ValueBf16>(prm, prm.units * prm.mt * prm.nd, stream);
  } else {
    ValueTf32::Params prm{};
    if (!fill(prm, ValueTf32::S::BK)) return BDH_ERR_INVALID;
    return launch_tc<ValueTf32::S, ValueTf32>(prm, prm.units * prm.mt * prm.nd, stream);
  }
}

}  // namespace bdh

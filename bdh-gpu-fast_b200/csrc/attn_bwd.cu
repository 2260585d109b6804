// Backward of out = tril(Q K^T, -1) V on tcgen05 (reference math: kernels/attention_bwd.py:45-83;
// K-is-Q sum :284-291; RoPE adjoint kernels/rope.py:540-557).
//
//   dS = tril(dO V^T, -1)     M = tril(Q K^T, -1)
//   dQ = dS K                 dK = dS^T Q            dV = sum_{heads sharing V} M^T dO
//
// Passes (all persistent tcgen05 GEMMs of tc_engine.cuh):
//   1. score pass over (dO, V), K-loop over D -> G = dS + dS^T (K is Q) or dS / dS^T (else)
//   2. grad-Q pass: dQ_total = G QR over all keys (K is Q), or dS K / dS^T Q over the causal
//      key ranges; optional RoPE adjoint R(t)^T in the epilogue (gradient of the unrotated
//      latent), its phases computed in registers from freqs with the hardware sin / cos
//      (rope_cis_grad: the exact software sincos of the forward cost a third of the pass)
//   3. score pass over (Q, K) writing M^T (transposed store: the K-major A operand of dV)
//   4. grad-V pass: dV[j] = sum_h sum_{i > j} M^T_h[j][i] dO_h[i], longest key blocks first
// Score-like operands: bf16 inputs give one bf16 term (fp32 sums rounded once, as the
// reference's bf16 matmul chain rounds dM and M; BDH_SM100_SPLIT_SCORES=1 keeps an exact bf16
// hi + lo split), fp32 inputs an exact tf32 hi/lo split. bf16 Q/K/dO are used as stored
// (MN-major where needed); fp32 inputs use tf32 hi/lo copies laid out K-major.
#include <algorithm>
#include <cstdlib>

#include "bdh_sm100.h"
#include "internal.h"
#include "score_pass.cuh"
#include "tc_engine.cuh"
#include "tc_pair_engine.cuh"
#include "tma_host.h"

namespace bdh {

namespace {

// Store 32 consecutive fp32 values of one output row (bf16 or fp32, vectorised when aligned).
__device__ __forceinline__ void store_row32(void* base, int64_t off, bool f32, bool vec, int valid,
                                            const float (&v)[32]) {
  if (f32) {
    float* o = static_cast<float*>(base) + off;
    if (vec && valid >= 32) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4*>(o + 4 * i) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (e < valid) o[e] = v[e];
    }
  } else {
    uint16_t* o = static_cast<uint16_t*>(base) + off;
    if (vec && valid >= 32) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(o + 8 * i) =
            make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                       pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (e < valid) o[e] = static_cast<uint16_t>(f32_to_bf16_bits(v[e]));
    }
  }
}

// ------------------------------------------------------------------ grad-Q pass ----
// out[u][i][n] = sum_j Gs[u][i][j] X[u][j][n] with Gs a hi/lo score matrix ([u][T][ldp]).
// krange 0: all keys; 1: keys j < (i-block+1)*128 (dS K); 2: keys j >= i-block*128 (dS^T Q).
// AT = 1: Gs is a single bf16 term (the bf16 path's default, see launch_grad_q).
template <int ELEM, int STAGES, int AT = 2>
struct GradQProb {
  static constexpr int BN = ELEM == 2 ? 256 : 128;
  static constexpr bool B_MN = ELEM == 2;
  static constexpr int B_TERMS = ELEM == 2 ? 1 : 2;
  using S = TcShape<ELEM, BN, false, B_MN, AT, B_TERMS, STAGES, ELEM == 4 ? 8 : 0>;
  static constexpr int CHUNK = 128 / ELEM;
  struct Params {
    CUtensorMap a_map[2];  // Gs hi/lo over [units][T][T(ldp)], box BK x 128
    CUtensorMap b_map[2];  // bf16: X (B,H,T,N) box CHUNK x BK; tf32: X^T [units][N][ldt] box BK x 256
    int H, T, N;
    int mt, nn;            // query blocks, 256-wide N tiles
    int units;
    int krange;
    void* out;             // (B,H,T,N) strided
    int64_t os_b, os_h, os_t;
    int out_f32, vec_ok;
    const float* freqs;    // RoPE adjoint when non-null
    int64_t pos0;
    int* err;
  };
  struct Tile {
    int unit, mi, ni;
  };
  __device__ static int num_tiles(const Params& p) { return p.units * p.mt * p.nn; }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    // unit-major, then query block, then N tile: concurrent CTAs share Gs rows and X tiles.
    tl.unit = t / (p.mt * p.nn);
    const int r = t - tl.unit * p.mt * p.nn;
    tl.mi = r / p.nn;
    tl.ni = r - tl.mi * p.nn;
    return tl;
  }
  __device__ static int kb_begin(const Params& p, const Tile& tl) {
    return p.krange == 2 ? (tl.mi * S::BM) / S::BK : 0;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) {
    const int end = p.krange == 1 ? ceil_div_d(min(p.T, (tl.mi + 1) * S::BM), S::BK)
                                  : ceil_div_d(p.T, S::BK);
    return end - kb_begin(p, tl);
  }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x7u; }
  __device__ static void prefetch(const Params& p) {
    for (int i = 0; i < AT; ++i) tma_prefetch_desc(&p.a_map[i]);
    for (int i = 0; i < B_TERMS; ++i) tma_prefetch_desc(&p.b_map[i]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int j0 = (kb + kb_begin(p, tl)) * S::BK;
    for (int i = 0; i < AT; ++i)
      tma_load_4d(&p.a_map[i], bar, a_dst + i * S::A_TILE, j0, tl.mi * S::BM, tl.unit, 0);
    if (B_MN) {
      const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
#pragma unroll
      for (int c = 0; c < BN / CHUNK; ++c)
        tma_load_4d(&p.b_map[0], bar, b_dst + c * S::BK * 128, tl.ni * BN + c * CHUNK, j0, h, b);
    } else {
      for (int i = 0; i < B_TERMS; ++i)
        tma_load_4d(&p.b_map[i], bar, b_dst + i * S::B_TILE, j0, tl.ni * BN, tl.unit, 0);
    }
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int row, int c0,
                                  const uint32_t (&r)[32]) {
    const int gi = tl.mi * S::BM + row;
    if (gi >= p.T) return;
    const int gn0 = tl.ni * BN + c0;
    if (gn0 >= p.N) return;
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
    if (p.freqs != nullptr) {
      // gradient of the unrotated latent: dx0 = g0 c0 + g1 s1, dx1 = -g0 s0 + g1 c1
      const float pos = static_cast<float>(p.pos0 + gi);
      // fully unrolled so that v stays in registers (a partly unrolled loop indexes v at run
      // time and moves it to local memory)
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const int n = gn0 + e;
        if (n >= p.N) continue;
        float cc0, ss0, cc1, ss1;
        const float f0 = __ldg(p.freqs + n), f1 = __ldg(p.freqs + n + 1);
        rope_cis_grad(pos, f0, cc0, ss0);
        if (f1 == f0) {
          cc1 = cc0;
          ss1 = ss0;
        } else {
          rope_cis_grad(pos, f1, cc1, ss1);
        }
        const float g0 = v[e], g1 = v[e + 1];
        v[e] = fmaf(g0, cc0, g1 * ss1);
        v[e + 1] = fmaf(-g0, ss0, g1 * cc1);
      }
    }
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    store_row32(p.out, b * p.os_b + h * p.os_h + gi * p.os_t + gn0, p.out_f32 != 0,
                p.vec_ok != 0, p.N - gn0, v);
  }
};

// ------------------------------------------------------------------ grad-V pass ----
// dV[b,hv][j][d] = sum over heads h sharing (b,hv) of sum_{i} Mt_h[j][i] dO_h[i][d],
// Mt = M^T as a hi/lo pair ([units][T][ldp], rows j). Keys i < j-block start are all zero.
template <int ELEM, int STAGES, int AT = 2>
struct GradVProb {
  static constexpr int BN = ELEM == 2 ? 256 : 128;
  static constexpr bool B_MN = ELEM == 2;
  static constexpr int B_TERMS = ELEM == 2 ? 1 : 2;
  using S = TcShape<ELEM, BN, false, B_MN, AT, B_TERMS, STAGES, ELEM == 4 ? 8 : 0>;
  static constexpr int CHUNK = 128 / ELEM;
  struct Params {
    CUtensorMap a_map[2];  // Mt hi/lo over [units][T][T(ldp)], box BK x 128
    CUtensorMap b_map[2];  // bf16: dO (B,H,T,D) box CHUNK x BK; tf32: dO^T [units][D][ldt] box BK x 256
    int H, Hv, T, D;
    int mt, nd;
    int vunits;            // B * Hv
    void* out;             // dV (B,Hv,T,D) strided
    int64_t os_b, os_h, os_t;
    int out_f32, vec_ok;
    int* err;
  };
  struct Tile {
    int vunit, mi, ni;
  };
  __device__ static int num_tiles(const Params& p) { return p.vunits * p.mt * p.nd; }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;  // first key blocks have the longest K-loops: schedule them first
    const int per = p.vunits * p.nd;
    tl.mi = t / per;
    const int r = t - tl.mi * per;
    tl.vunit = r / p.nd;
    tl.ni = r - tl.vunit * p.nd;
    return tl;
  }
  __device__ static int heads(const Params& p) { return (p.Hv == 1 && p.H != 1) ? p.H : 1; }
  __device__ static int per_head(const Params& p, const Tile& tl) {
    return ceil_div_d(p.T, S::BK) - (tl.mi * S::BM) / S::BK;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) { return heads(p) * per_head(p, tl); }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x7u; }
  __device__ static void prefetch(const Params& p) {
    for (int i = 0; i < AT; ++i) tma_prefetch_desc(&p.a_map[i]);
    for (int i = 0; i < B_TERMS; ++i) tma_prefetch_desc(&p.b_map[i]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int ph = per_head(p, tl);
    const int hh = kb / ph;
    const int i0 = (kb - hh * ph + (tl.mi * S::BM) / S::BK) * S::BK;
    const int b = tl.vunit / p.Hv, hv = tl.vunit - (tl.vunit / p.Hv) * p.Hv;
    const int h = heads(p) > 1 ? hh : hv;
    const int unit = b * p.H + h;
    for (int i = 0; i < AT; ++i)
      tma_load_4d(&p.a_map[i], bar, a_dst + i * S::A_TILE, i0, tl.mi * S::BM, unit, 0);
    if (B_MN) {
#pragma unroll
      for (int c = 0; c < BN / CHUNK; ++c)
        tma_load_4d(&p.b_map[0], bar, b_dst + c * S::BK * 128, tl.ni * BN + c * CHUNK, i0, h, b);
    } else {
      for (int i = 0; i < B_TERMS; ++i)
        tma_load_4d(&p.b_map[i], bar, b_dst + i * S::B_TILE, i0, tl.ni * BN, unit, 0);
    }
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int row, int c0,
                                  const uint32_t (&r)[32]) {
    const int gj = tl.mi * S::BM + row;
    if (gj >= p.T) return;
    const int gd0 = tl.ni * BN + c0;
    if (gd0 >= p.D) return;
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
    const int b = tl.vunit / p.Hv, hv = tl.vunit - (tl.vunit / p.Hv) * p.Hv;
    store_row32(p.out, b * p.os_b + hv * p.os_h + gj * p.os_t + gd0, p.out_f32 != 0,
                p.vec_ok != 0, p.D - gd0, v);
  }
};

using GradQBf16 = GradQProb<2, 3>;

// CTA-pair grad-Q pass: 256 (query rows) x 256 (latent columns) tiles; each CTA stages its 128
// rows of the score matrix (AT terms: hi/lo, or the single bf16 term) and its 128 columns of X
// (MN-major), and stores its 128 rows with the single-CTA epilogue (including the RoPE adjoint).
template <int AT, int STG>
struct GradQPairT {
  using Base = GradQBf16;
  using Params = Base::Params;  // b_map box 64 x BK as in the single-CTA pass
  using S = PairShape<false, true, AT, 1, STG>;
  static constexpr int kEpiWarps = 8;  // the RoPE adjoint makes the epilogue long
  struct Tile {
    int unit, m, n;
  };
  __device__ static int mt2(const Params& p) { return ceil_div_d(p.T, 256); }
  __device__ static int num_tiles(const Params& p) { return p.units * mt2(p) * p.nn; }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    const int per = mt2(p) * p.nn;
    tl.unit = t / per;
    const int r = t - tl.unit * per;
    tl.m = r / p.nn;
    tl.n = r - tl.m * p.nn;
    return tl;
  }
  __device__ static int kb_begin(const Params& p, const Tile& tl) {
    return p.krange == 2 ? (tl.m * 256) / 64 : 0;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) {
    const int end = p.krange == 1 ? ceil_div_d(min(p.T, (tl.m + 1) * 256), 64) : ceil_div_d(p.T, 64);
    return end - kb_begin(p, tl);
  }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return AT == 2 ? 0x3u : 0x1u; }
  __device__ static uint32_t stage_tx(const Params&, const Tile&, int) { return 2 * S::STAGE_BYTES; }
  __device__ static void prefetch(const Params& p) {
    for (int i = 0; i < AT; ++i) tma_prefetch_desc(&p.a_map[i]);
    tma_prefetch_desc(&p.b_map[0]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint32_t rank,
                                    uint32_t bar, uint8_t* a_dst, uint8_t* b_dst) {
    const int j0 = (kb + kb_begin(p, tl)) * 64;
    const int r128 = static_cast<int>(rank) * 128;
    for (int i = 0; i < AT; ++i)
      tma_load_4d_pair(&p.a_map[i], bar, a_dst + i * S::A_TILE, j0, tl.m * 256 + r128, tl.unit, 0);
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d_pair(&p.b_map[0], bar, b_dst + c * 64 * 128, tl.n * 256 + r128 + c * 64, j0, h, b);
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int rank, int row, int c0,
                                  const uint32_t (&r)[32]) {
    Base::Tile t;
    t.unit = tl.unit;
    t.mi = 2 * tl.m + rank;
    t.ni = tl.n;
    Base::epilogue(p, t, row, c0, r);
  }
};
using GradQPair = GradQPairT<2, 4>;
using GradQPair1 = GradQPairT<1, 6>;

bool use_pairs_bwd() {
  static int on = [] {
    const char* e = std::getenv("BDH_SM100_PAIR");
    return (e != nullptr && std::atoi(e) == 0) ? 0 : 1;
  }();
  return on != 0;
}
using GradQTf32 = GradQProb<4, 3>;
using GradQBf16One = GradQProb<2, 4, 1>;
using GradVBf16 = GradVProb<2, 3>;
using GradVBf16One = GradVProb<2, 4, 1>;
using GradVTf32 = GradVProb<4, 3>;

bool out_vec_ok(const void* p, const int64_t s[4], int esz) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && (s[0] * esz) % 16 == 0 &&
         (s[1] * esz) % 16 == 0 && (s[2] * esz) % 16 == 0;
}

}  // namespace

int launch_grad_q(const GradQArgs& a, cudaStream_t stream, int* err) {
  const int elem = a.elem;
  const int64_t ldp = score_ld(a.T);
  const int64_t units = a.B * a.H;
  auto fill = [&](auto& prm, int bk, int bn) -> bool {
    const int64_t gd[4] = {a.T, a.T, units, 1};
    const int64_t gs[3] = {ldp * elem, a.T * ldp * elem, units * a.T * ldp * elem};
    if (!make_map_4d(&prm.a_map[0], a.g_hi, elem, gd, gs, bk, 128, "grad-q pass: score hi")) return false;
    if (a.g_lo != nullptr &&
        !make_map_4d(&prm.a_map[1], a.g_lo, elem, gd, gs, bk, 128, "grad-q pass: score lo"))
      return false;
    if (elem == 2) {
      int64_t xd[4] = {a.N, a.T, a.H, a.B};
      int64_t xs[3] = {a.x_strides[2] * 2, a.x_strides[1] * 2, a.x_strides[0] * 2};
      if (!make_map_4d(&prm.b_map[0], a.x[0], 2, xd, xs, 64, bk, "grad-q pass: X")) return false;
    } else {
      const int64_t ldt = vt_ld(a.T);
      int64_t xd[4] = {a.T, a.N, units, 1};
      int64_t xs[3] = {ldt * 4, a.N * ldt * 4, units * a.N * ldt * 4};
      for (int i = 0; i < 2; ++i)
        if (!make_map_4d(&prm.b_map[i], a.x[i], 4, xd, xs, bk, bn, "grad-q pass: X^T")) return false;
    }
    prm.H = static_cast<int>(a.H);
    prm.T = static_cast<int>(a.T);
    prm.N = static_cast<int>(a.N);
    prm.mt = static_cast<int>((a.T + 127) / 128);
    prm.nn = static_cast<int>((a.N + bn - 1) / bn);
    prm.units = static_cast<int>(units);
    prm.krange = a.krange;
    prm.out = a.out;
    prm.os_b = a.out_strides[0];
    prm.os_h = a.out_strides[1];
    prm.os_t = a.out_strides[2];
    prm.out_f32 = a.out_dtype == BDH_DTYPE_F32 ? 1 : 0;
    prm.vec_ok = out_vec_ok(a.out, a.out_strides, prm.out_f32 ? 4 : 2) ? 1 : 0;
    prm.freqs = a.freqs;
    prm.pos0 = a.pos0;
    prm.err = err;
    return true;
  };
  if (elem != 2 && a.g_lo == nullptr) {
    set_error("grad-q pass: the fp32 path needs the tf32 hi/lo score pair");
    return BDH_ERR_INVALID;
  }
  const bool one = a.g_lo == nullptr;  // bf16 path: Gs is one bf16 term
  if (elem == 2 && use_pairs_bwd()) {
    GradQPair::Params prm{};
    if (!fill(prm, GradQBf16::S::BK, GradQBf16::BN)) return BDH_ERR_INVALID;
    const int tiles = prm.units * static_cast<int>((a.T + 255) / 256) * prm.nn;
    return one ? launch_pair<GradQPair1::S, GradQPair1>(prm, tiles, stream, kProfGradQ)
               : launch_pair<GradQPair::S, GradQPair>(prm, tiles, stream, kProfGradQ);
  }
  if (elem == 2 && one) {
    GradQBf16One::Params prm{};
    if (!fill(prm, GradQBf16One::S::BK, GradQBf16One::BN)) return BDH_ERR_INVALID;
    return launch_tc<GradQBf16One::S, GradQBf16One>(prm, prm.units * prm.mt * prm.nn, stream,
                                                    kProfGradQ);
  }
  if (elem == 2) {
    GradQBf16::Params prm{};
    if (!fill(prm, GradQBf16::S::BK, GradQBf16::BN)) return BDH_ERR_INVALID;
    return launch_tc<GradQBf16::S, GradQBf16>(prm, prm.units * prm.mt * prm.nn, stream, kProfGradQ);
  }
  GradQTf32::Params prm{};
  if (!fill(prm, GradQTf32::S::BK, GradQTf32::BN)) return BDH_ERR_INVALID;
  return launch_tc<GradQTf32::S, GradQTf32>(prm, prm.units * prm.mt * prm.nn, stream, kProfGradQ);
}

int launch_grad_v(const GradVArgs& a, cudaStream_t stream, int* err) {
  const int elem = a.elem;
  const int64_t ldp = score_ld(a.T);
  const int64_t units = a.B * a.H;
  auto fill = [&](auto& prm, int bk, int bn) -> bool {
    const int64_t md[4] = {a.T, a.T, units, 1};
    const int64_t ms[3] = {ldp * elem, a.T * ldp * elem, units * a.T * ldp * elem};
    if (!make_map_4d(&prm.a_map[0], a.mt_hi, elem, md, ms, bk, 128, "grad-v pass: M^T hi")) return false;
    if (a.mt_lo != nullptr &&
        !make_map_4d(&prm.a_map[1], a.mt_lo, elem, md, ms, bk, 128, "grad-v pass: M^T lo"))
      return false;
    if (elem == 2) {
      int64_t dd[4] = {a.D, a.T, a.H, a.B};
      int64_t ds[3] = {a.do_strides[2] * 2, a.do_strides[1] * 2, a.do_strides[0] * 2};
      if (!make_map_4d(&prm.b_map[0], a.dout[0], 2, dd, ds, 64, bk, "grad-v pass: dO")) return false;
    } else {
      const int64_t ldt = vt_ld(a.T);
      int64_t dd[4] = {a.T, a.D, units, 1};
      int64_t ds[3] = {ldt * 4, a.D * ldt * 4, units * a.D * ldt * 4};
      for (int i = 0; i < 2; ++i)
        if (!make_map_4d(&prm.b_map[i], a.dout[i], 4, dd, ds, bk, bn, "grad-v pass: dO^T")) return false;
    }
    prm.H = static_cast<int>(a.H);
    prm.Hv = static_cast<int>(a.Hv);
    prm.T = static_cast<int>(a.T);
    prm.D = static_cast<int>(a.D);
    prm.mt = static_cast<int>((a.T + 127) / 128);
    prm.nd = static_cast<int>((a.D + bn - 1) / bn);
    prm.vunits = static_cast<int>(a.B * a.Hv);
    prm.out = a.out;
    prm.os_b = a.out_strides[0];
    prm.os_h = a.out_strides[1];
    prm.os_t = a.out_strides[2];
    prm.out_f32 = a.out_dtype == BDH_DTYPE_F32 ? 1 : 0;
    prm.vec_ok = out_vec_ok(a.out, a.out_strides, prm.out_f32 ? 4 : 2) ? 1 : 0;
    prm.err = err;
    return true;
  };
  if (elem != 2 && a.mt_lo == nullptr) {
    set_error("grad-v pass: the fp32 path needs the tf32 hi/lo score pair");
    return BDH_ERR_INVALID;
  }
  if (elem == 2 && a.mt_lo == nullptr) {
    GradVBf16One::Params prm{};
    if (!fill(prm, GradVBf16One::S::BK, GradVBf16One::BN)) return BDH_ERR_INVALID;
    return launch_tc<GradVBf16One::S, GradVBf16One>(prm, prm.vunits * prm.mt * prm.nd, stream,
                                                    kProfGradV);
  }
  if (elem == 2) {
    GradVBf16::Params prm{};
    if (!fill(prm, GradVBf16::S::BK, GradVBf16::BN)) return BDH_ERR_INVALID;
    return launch_tc<GradVBf16::S, GradVBf16>(prm, prm.vunits * prm.mt * prm.nd, stream, kProfGradV);
  }
  GradVTf32::Params prm{};
  if (!fill(prm, GradVTf32::S::BK, GradVTf32::BN)) return BDH_ERR_INVALID;
  return launch_tc<GradVTf32::S, GradVTf32>(prm, prm.vunits * prm.mt * prm.nd, stream, kProfGradV);
}

}  // namespace bdh

// Forward strict-causal linear attention on tcgen05:
//   out[b,h] = tril(Q[b,h] K[b,h]^T, -1) V[b,hv]        (hv = h, or 0 when V is shared)
//
// Two persistent tensor-core passes over the (b,h) units:
//   1. score pass : P = tril(Q K^T, -1) over the lower-triangular 128 x BN tiles, K-loop
//                   over the latent width N. P is written once as an exact split pair
//                   (bf16 hi + bf16 lo, or tf32 hi + fp32 lo for fp32 inputs) so that the
//                   second pass keeps fp32-level accuracy on tensor cores
//                   (BDH_SM100_SPLIT_SCORES=0: P as one bf16 term, the reference's rounding).
//   2. value pass : out = P V with the K-loop over keys limited to the causal prefix of each
//                   128-row query block (longest blocks scheduled first).
// Semantics follow the reference kernels (csrc/tril_attn_cuda.cu:129-249) and eager path
// (kernels/attention.py:27-40): no softmax, no scale, diagonal excluded, V broadcast over
// heads when it has one head.
#include <algorithm>
#include <cstdlib>

#include "bdh_sm100.h"
#include "internal.h"
#include "score_pass.cuh"
#include "tc_engine.cuh"
#include "tc_pair_engine.cuh"
#include "tma_host.h"

namespace bdh {

// --------------------------------------------------------------- value pass ----
// A = P (K-major over keys, hi/lo terms).
// ELEM 2: B = V as stored, MN-major (D contiguous); bf16 P hi/lo x bf16 V (2 products).
// ELEM 4: B = V^T hi/lo written by the tf32 split (K-major, keys contiguous); 3 products.
template <int ELEM, int STAGES, int AT = 2>  // AT = 1: P as one bf16 term
struct ValueProb {
  static constexpr int BN = ELEM == 2 ? 256 : 128;
  static constexpr bool B_MN = ELEM == 2;
  static constexpr int B_TERMS = ELEM == 2 ? 1 : 2;
  using S = TcShape<ELEM, BN, false, B_MN, AT, B_TERMS, STAGES, ELEM == 4 ? 8 : 0>;
  static constexpr int CHUNK = 128 / ELEM;  // MN elements per 128-byte chunk
  struct Params {
    CUtensorMap a_map[2];  // P hi / lo over [units][T][T], box BK x 128
    CUtensorMap b_map[2];  // bf16: V (B, Hv, T, D), box CHUNK x BK; tf32: V^T [B*Hv][D][T], box BK x 256
    int H, Hv, T, D;
    int mt, nd;            // query blocks, BN-wide D tiles
    int units;
    void* out;             // (B, H, T, D) strided, out_f32 ? float : bf16
    int64_t os_b, os_h, os_t;
    int out_f32;
    int vec_ok;
    float ln_eps;          // ValueLnProb: the LayerNorm's eps
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
    for (int i = 0; i < AT; ++i) tma_prefetch_desc(&p.a_map[i]);
    for (int i = 0; i < B_TERMS; ++i) tma_prefetch_desc(&p.b_map[i]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int hv = p.Hv == 1 ? 0 : h;
    for (int i = 0; i < AT; ++i)
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

// Value pass with the row LayerNorm of the attention output folded into the epilogue: the
// reference's y = LN(bf16(P V)) of a BDH layer (bdh.py:1044 after kernels/attention.py:27-40,
// the LayerNorm in fp32 under autocast, its result cast to bf16 by the next op). One thread owns
// one output row (all D <= 256 columns in its TMEM lane), so the un-normalised output
// never reaches HBM and no separate LayerNorm kernel runs. The row is read from TMEM three times
// (a compact loop each; keeping it in registers, fully unrolled, measured slower). Statistics as
// csrc/layernorm.cu computes them (fp32; mean, then the biased variance of the deviations;
// rstd = 1 / sqrt(var + eps)), each summed in four interleaved partial sums.
template <int STAGES, int AT>
struct ValueLnProb : ValueProb<2, STAGES, AT> {
  using Base = ValueProb<2, STAGES, AT>;
  using S = typename Base::S;
  using Params = typename Base::Params;
  using Tile = typename Base::Tile;
  static constexpr int kCustomEpilogue = 1;
  struct EpiState {};
  __device__ static void epilogue_begin(const Params&, int, int, uint8_t*, EpiState&, bool,
                                        const Tile&) {}
  __device__ static void epilogue_prefetch(const Params&, const Tile&, bool, const Tile&, int, int,
                                           uint8_t*, EpiState&) {}
  __device__ static bool epilogue_tile(const Params& p, const Tile& tl, int row, int,
                                       uint32_t taddr, uint8_t*, EpiState&, volatile int*) {
    const int D = p.D;  // <= S::BN (one D tile)
    // pass 1: mean; pass 2: variance of the deviations; pass 3: normalise and store. Each pass
    // reads the row from TMEM again (a compact loop); sums in four interleaved partial sums
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 1
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + static_cast<uint32_t>(c0), r);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const uint32_t p0 = cvt_bf16x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        const uint32_t p1 = cvt_bf16x2(__uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
        if (c0 + e < D) a0 += bf16x2_lo(p0);
        if (c0 + e + 1 < D) a1 += bf16x2_hi(p0);
        if (c0 + e + 2 < D) a2 += bf16x2_lo(p1);
        if (c0 + e + 3 < D) a3 += bf16x2_hi(p1);
      }
    }
    const float mean = ((a0 + a1) + (a2 + a3)) / static_cast<float>(D);
    a0 = a1 = a2 = a3 = 0.0f;
#pragma unroll 1
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + static_cast<uint32_t>(c0), r);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const uint32_t p0 = cvt_bf16x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        const uint32_t p1 = cvt_bf16x2(__uint_as_float(r[e + 2]), __uint_as_float(r[e + 3]));
        const float d0 = bf16x2_lo(p0) - mean, d1 = bf16x2_hi(p0) - mean;
        const float d2 = bf16x2_lo(p1) - mean, d3 = bf16x2_hi(p1) - mean;
        if (c0 + e < D) a0 = fmaf(d0, d0, a0);
        if (c0 + e + 1 < D) a1 = fmaf(d1, d1, a1);
        if (c0 + e + 2 < D) a2 = fmaf(d2, d2, a2);
        if (c0 + e + 3 < D) a3 = fmaf(d3, d3, a3);
      }
    }
    const float rstd = 1.0f / sqrtf(((a0 + a1) + (a2 + a3)) / static_cast<float>(D) + p.ln_eps);
    // every lane of the warp takes part in each TMEM load (tcgen05.ld is warp-aligned); rows at
    // or beyond T only skip the store
    const bool row_ok = tl.mi * S::BM + row < p.T;
    Tile t1 = tl;
    t1.ni = 0;
#pragma unroll 1
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + static_cast<uint32_t>(c0), r);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const uint32_t pr = cvt_bf16x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        r[e] = __float_as_uint((bf16x2_lo(pr) - mean) * rstd);
        r[e + 1] = __float_as_uint((bf16x2_hi(pr) - mean) * rstd);
      }
      if (row_ok) Base::epilogue(p, t1, row, c0, r);  // the output store of the plain value pass
    }
    return true;
  }
  __device__ static void epilogue_after(const Params&, const Tile&, int, int, uint8_t*, EpiState&) {}
  __device__ static void epilogue_end(const Params&, int, int, uint8_t*, EpiState&) {}
};

// ----------------------------------------------------------------- launchers ----
using ScoreBf16 = ScoreProb<2, 128, 6>;
using ScoreBf16Wide = ScoreProb<2, 256, 4>;  // 128 x 256 tiles: 25% fewer operand bytes per flop

// CTA-pair score pass: 256 x 256 tiles (each CTA 128 query rows x all 256 keys of the tile in
// TMEM, staging 128 query rows and 128 key rows per stage). Epilogue and parameters are those of
// the single-CTA 128 x 256 score pass, applied to each CTA's 128-row half.
// STAGES operand stages of 32 KB; SCRATCH bytes of shared memory per epilogue warp for the
// transposed stores of the backward's G and M^T (0: direct stores only, room for a seventh stage).
template <int STAGES, int SCRATCH>
struct ScorePairT {
  using Base = ScoreBf16Wide;
  using Params = Base::Params;  // b_map box is 64 x 128 (one CTA's key rows)
  using S = PairShape<false, false, 1, 1, STAGES>;
  struct Tile {
    int unit, m, n;  // 256-row query block, 256-key block
    int sub;         // -1: all 256 keys; else keys [sub * w, (sub + 1) * w), w = 256 / tail_sub
  };
  __device__ static int key0(const Params& p, int m) {
    return p.chunk > 0 ? (m * 256 / p.chunk) * p.chunk : 0;
  }
  __device__ static int nt_for(const Params& p, int m) {
    return ceil_div_d(min(p.T, (m + 1) * 256), 256) - key0(p, m) / 256;
  }
  __device__ static int num_tiles(const Params& p) {
    const int n = p.units * p.tiles_per_unit;
    return p.tail_sub > 1 ? p.tail_from + (n - p.tail_from) * p.tail_sub : n;
  }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    tl.sub = -1;
    if (p.tail_sub > 1 && t >= p.tail_from) {  // the narrow tiles of a tail tile are consecutive
      const int e = t - p.tail_from;
      const int q = e / p.tail_sub;
      tl.sub = e - q * p.tail_sub;
      t = p.tail_from + q;
    }
    tl.unit = t / p.tiles_per_unit;
    int r = t - tl.unit * p.tiles_per_unit;
    int m = 0;
    for (;; ++m) {
      const int c = nt_for(p, m);
      if (r < c) break;
      r -= c;
    }
    tl.m = m;
    tl.n = r + key0(p, m) / 256;
    return tl;
  }
  // narrow tail tiles: an M = 256, N = 256 / tail_sub MMA over all of K (pair-engine kVarN)
  static constexpr bool kVarN = true;
  __device__ static uint32_t tile_idesc(const Params& p, const Tile& tl) {
    return tl.sub < 0 ? S::IDESC : make_idesc(1u, 0u, 0u, 256u, static_cast<uint32_t>(256 / p.tail_sub));
  }
  __device__ static int tile_cols(const Params& p, const Tile& tl) {
    return tl.sub < 0 ? 256 : 256 / p.tail_sub;
  }
  __device__ static int k_blocks(const Params& p, const Tile&) { return ceil_div_d(p.K, 64); }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  // Diagonal tiles of Q Q^T (pair-engine kBFromA): each CTA's 128 query rows are also its 128
  // key rows, so a stage loads them once and the MMA reads both operands from that buffer
  // (two thirds of config 2's tiles, a third less operand traffic in all).
  static constexpr bool kBFromA = true;
  __device__ static bool b_is_a(const Params& p, const Tile& tl) {
    return p.self_ab && tl.sub < 0 && tl.n == tl.m;
  }
  __device__ static uint32_t stage_tx(const Params& p, const Tile& tl, int) {
    if (b_is_a(p, tl)) return 2 * S::A_TILE;
    return tl.sub < 0 ? 2 * S::STAGE_BYTES : 2 * (S::A_TILE + S::B_TILE / p.tail_sub);
  }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map[0]);
    tma_prefetch_desc(&p.b_map[0]);
    if (p.tail_sub > 1) tma_prefetch_desc(&p.b_nar);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint32_t rank,
                                    uint32_t bar, uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int hb = p.b_shared ? 0 : h;
    const int r128 = static_cast<int>(rank) * 128;
    tma_load_4d_pair(&p.a_map[0], bar, a_dst, kb * 64, tl.m * 256 + r128, h, b);
    if (b_is_a(p, tl)) {
      // B is the A rows just loaded
    } else if (tl.sub < 0) {
      tma_load_4d_pair(&p.b_map[0], bar, b_dst, kb * 64, tl.n * 256 + r128, hb, b);
    } else {  // this CTA's half of the narrow tile's keys
      const int w = 256 / p.tail_sub;
      tma_load_4d_pair(&p.b_nar, bar, b_dst, kb * 64,
                       tl.n * 256 + tl.sub * w + static_cast<int>(rank) * (w / 2), hb, b);
    }
  }
  // 4 KB per epilogue warp (SCRATCH): the transposed stores of the backward's G and M^T go
  // through shared memory (whole 64-byte column segments instead of two-byte element stores)
  static constexpr int kEpiScratch = SCRATCH;
  __device__ static void epilogue(const Params& p, const Tile& tl, int rank, int row, int c0,
                                  const uint32_t (&r)[32], uint8_t* scratch = nullptr) {
    Base::Tile t;
    t.unit = tl.unit;
    t.mi = 2 * tl.m + rank;
    t.ni = tl.n;
    // a narrow tile's accumulator columns are its keys: column c0 of the 256-key block below
    Base::epilogue(p, t, row, tl.sub < 0 ? c0 : tl.sub * (256 / p.tail_sub) + c0, r, scratch);
  }
};

using ScorePair = ScorePairT<6, 2 * 32 * 32 * 2>;
// Direct stores only (the forward's P): seven 32 KB stages, 224 KB of operands in flight.
using ScorePairDirect = ScorePairT<7, 0>;

// CTA pairs for the bf16 tensor passes (BDH_SM100_PAIR=0 selects single-CTA tiles instead).
bool use_pairs() {
  static int on = [] {
    const char* e = std::getenv("BDH_SM100_PAIR");
    return (e != nullptr && std::atoi(e) == 0) ? 0 : 1;
  }();
  return on != 0;
}

// Score-pass tile width for bf16: 128 or 256 keys (BDH_SM100_SCORE_BN, read once; default 128).
int score_tile_n() {
  static int bn = [] {
    const char* e = std::getenv("BDH_SM100_SCORE_BN");
    return (e != nullptr && std::atoi(e) == 256) ? 256 : 128;
  }();
  return bn;
}
using ScoreTf32 = ScoreProb<4, 128, 3>;
using ValueBf16 = ValueProb<2, 3>;
using ValueBf16One = ValueProb<2, 4, 1>;
using ValueLnBf16 = ValueLnProb<3, 2>;
using ValueLnBf16One = ValueLnProb<4, 1>;
using ValueTf32 = ValueProb<4, 3>;

// One row of the fp32 score pair from its K-split partials: columns of the row's stored tiles
// (up to the end of its diagonal 128-block), strictly lower part kept, tf32 hi + fp32 lo.
__global__ void score_split_reduce_kernel(const float* __restrict__ part, float* __restrict__ p_hi,
                                          float* __restrict__ p_lo, int ksplit, int T, int64_t ldp,
                                          int64_t rows) {
  const int64_t r = blockIdx.x;  // unit * T + i
  const int i = static_cast<int>(r % T);
  const int64_t cap = static_cast<int64_t>(i / 128 + 1) * 128;
  const int jend = static_cast<int>(ldp < cap ? ldp : cap);
  for (int j = threadIdx.x; j < jend; j += blockDim.x) {
    float x = 0.0f;
    if (j < i)
      for (int k = 0; k < ksplit; ++k) x += part[(k * rows + r) * ldp + j];
    const float h = tf32_rna(x);
    p_hi[r * ldp + j] = h;
    p_lo[r * ldp + j] = x - h;
  }
}

int64_t score_ld(int64_t T) { return (T + 7) / 8 * 8; }
int64_t vt_ld(int64_t T) { return (T + 3) / 4 * 4; }

int launch_score_pass(const ScoreArgs& a, cudaStream_t stream, int* err) {
  const int elem = a.elem;
  const int terms = elem == 2 ? 1 : 2;
  auto fill = [&](auto& prm, int bk, int bn) -> bool {
    for (int i = 0; i < terms; ++i) {
      int64_t ad[4] = {a.K, a.T, a.H, a.B};
      int64_t bd[4] = {a.K, a.T, a.Hb, a.B};
      int64_t as[3] = {a.a_strides[2] * elem, a.a_strides[1] * elem, a.a_strides[0] * elem};
      int64_t bs[3] = {a.b_strides[2] * elem, a.b_strides[1] * elem, a.b_strides[0] * elem};
      if (!make_map_4d(&prm.a_map[i], a.a[i], elem, ad, as, bk, 128, "score pass: A")) return false;
      if (!make_map_4d(&prm.b_map[i], a.b[i], elem, bd, bs, bk, bn, "score pass: B")) return false;
    }
    prm.H = static_cast<int>(a.H);
    prm.T = static_cast<int>(a.T);
    prm.K = static_cast<int>(a.K);
    prm.b_shared = (a.Hb == 1 && a.H != 1) ? 1 : 0;
    prm.mode = a.mode;
    prm.mt = static_cast<int>((a.T + 127) / 128);
    int tpu = 0;
    for (int mi = 0; mi < prm.mt; ++mi) {
      const int64_t lim = std::min<int64_t>(a.T, int64_t(mi + 1) * 128);
      const int64_t k0 = a.chunk > 0 ? (int64_t(mi) * 128 / a.chunk) * a.chunk : 0;
      tpu += static_cast<int>((lim + bn - 1) / bn - k0 / bn);
    }
    prm.tiles_per_unit = tpu;
    prm.units = static_cast<int>(a.B * a.H);
    prm.p_hi = a.p_hi;
    prm.p_lo = a.p_lo;
    prm.p2_hi = a.p2_hi;
    prm.p2_lo = a.p2_lo;
    prm.ldp = a.chunk > 0 ? a.chunk : score_ld(a.T);
    prm.chunk = a.chunk;
    prm.ksplit = 1;
    prm.kb_per_split = 0;
    prm.part = nullptr;
    if (elem == 4 && a.ksplit > 1 && a.mode == kStoreDirect && a.chunk == 0 && a.part != nullptr) {
      const int total = static_cast<int>((a.K + bk - 1) / bk);
      const int per = (total + a.ksplit - 1) / a.ksplit;
      prm.kb_per_split = (per + 7) / 8 * 8;  // whole 256-wide accumulation chunks
      prm.ksplit = (total + prm.kb_per_split - 1) / prm.kb_per_split;
      prm.part = a.part;
    }
    prm.err = err;
    return true;
  };
  if (elem == 2 && use_pairs()) {
    ScorePair::Params prm{};
    if (!fill(prm, 64, 128)) return BDH_ERR_INVALID;
    int tpu = 0;  // pair tiles per unit (256 x 256)
    for (int m = 0; m < (a.T + 255) / 256; ++m) {
      const int64_t lim = std::min<int64_t>(a.T, int64_t(m + 1) * 256);
      const int64_t k0 = a.chunk > 0 ? (int64_t(m) * 256 / a.chunk) * a.chunk : 0;
      tpu += static_cast<int>((lim + 255) / 256 - k0 / 256);
    }
    prm.tiles_per_unit = tpu;
    const int ntiles = prm.units * tpu;
    // Q K^T with K = Q (the self product): the diagonal tiles load their rows once
    prm.self_ab = (a.a[0] == a.b[0] && a.Hb == a.H && a.a_strides[0] == a.b_strides[0] &&
                   a.a_strides[1] == a.b_strides[1] && a.a_strides[2] == a.b_strides[2])
                      ? 1
                      : 0;
    // BDH_SM100_SCORE_TAIL=1: the last, partial wave of the persistent grid (ntiles mod pairs
    // tiles) runs as narrower tiles (64 or 128 keys) on the pairs the full waves leave idle, the
    // same MMAs over all of K for each output element (the same bits). Measured on B200 at
    // config 2's attention (384 tiles on 74 pairs, the last 14 as 56 narrow tiles): 0.306 ms per
    // launch against 0.289 ms with the wide last wave, so it is off by default.
    static const bool tail_on = [] {
      const char* e = std::getenv("BDH_SM100_SCORE_TAIL");
      return e != nullptr && std::atoi(e) == 1;
    }();
    const int cap = resident_pairs<ScorePair::S, ScorePair>();
    if (cap < 0) return -cap;
    const int tail = ntiles % cap;
    int sub = 0;
    if (tail_on && tail > 0 && a.mode == kStoreDirect) sub = tail * 4 <= cap ? 4 : tail * 2 <= cap ? 2 : 0;
    if (sub > 1) {
      int64_t bd[4] = {a.K, a.T, a.Hb, a.B};
      int64_t bs[3] = {a.b_strides[2] * elem, a.b_strides[1] * elem, a.b_strides[0] * elem};
      if (!make_map_4d(&prm.b_nar, a.b[0], elem, bd, bs, 64, 128 / sub, "score pass: B (tail)"))
        return BDH_ERR_INVALID;
      prm.tail_sub = sub;
      prm.tail_from = ntiles - tail;
      return launch_pair<ScorePair::S, ScorePair>(prm, prm.tail_from + tail * sub, stream, kProfScore);
    }
    // direct stores (the forward's P): the form with seven operand stages
    // (BDH_SM100_SCORE_STAGES=6 keeps six)
    static const bool seven = [] {
      const char* e = std::getenv("BDH_SM100_SCORE_STAGES");
      return !(e != nullptr && std::atoi(e) == 6);
    }();
    if (a.mode == kStoreDirect && seven)
      return launch_pair<ScorePairDirect::S, ScorePairDirect>(prm, ntiles, stream, kProfScore);
    return launch_pair<ScorePair::S, ScorePair>(prm, ntiles, stream, kProfScore);
  }
  if (elem == 2 && score_tile_n() == 256) {
    ScoreBf16Wide::Params prm{};
    if (!fill(prm, ScoreBf16Wide::S::BK, 256)) return BDH_ERR_INVALID;
    return launch_tc<ScoreBf16Wide::S, ScoreBf16Wide>(prm, prm.units * prm.tiles_per_unit, stream,
                                                      kProfScore);
  } else if (elem == 2) {
    ScoreBf16::Params prm{};
    if (!fill(prm, ScoreBf16::S::BK, 128)) return BDH_ERR_INVALID;
    return launch_tc<ScoreBf16::S, ScoreBf16>(prm, prm.units * prm.tiles_per_unit, stream, kProfScore);
  } else {
    ScoreTf32::Params prm{};
    if (!fill(prm, ScoreTf32::S::BK, 128)) return BDH_ERR_INVALID;
    const int rc = launch_tc<ScoreTf32::S, ScoreTf32>(
        prm, prm.units * prm.tiles_per_unit * std::max(1, prm.ksplit), stream, kProfScore);
    if (rc || prm.ksplit <= 1) return rc;
    // sum the K-split partials in order, mask j >= i, split into tf32 hi + fp32 lo
    const int64_t rows = a.B * a.H * a.T;
    prof_start(kProfScore, stream);
    score_split_reduce_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(
        prm.part, static_cast<float*>(a.p_hi), static_cast<float*>(a.p_lo), prm.ksplit,
        static_cast<int>(a.T), prm.ldp, rows);
    prof_stop(kProfScore, stream);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_error(std::string("score_split_reduce_kernel launch: ") + cudaGetErrorString(e));
      return BDH_ERR_CUDA;
    }
    return 0;
  }
}

// Wave-quantisation efficiency decides the split: ntiles * k tiles over the SMs, K / k >= 512.
int score_ksplit_f32(int64_t units, int64_t T, int64_t K) {
  const int64_t mt = (T + 127) / 128;
  const int64_t tiles = units * mt * (mt + 1) / 2;
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t sms = sm_count(dev);
  int best = 1;
  double best_eff = 0.0;
  for (int k = 1; k <= 16; k *= 2) {
    if (k > 1 && K / k < 512) break;
    const int64_t n = tiles * k;
    const int64_t waves = (n + sms - 1) / sms;
    const double eff = static_cast<double>(n) / static_cast<double>(waves * sms);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = k;
    }
  }
  return best;
}

// Score pass of the forward: P = tril(Q K^T, -1) as a hi/lo pair in p_hi / p_lo. fp32: `part`
// (null for none) holds the K-split partials.
int launch_score(const FwdArgs& a, void* p_hi, void* p_lo, float* part, cudaStream_t stream,
                 int* err) {
  ScoreArgs s;
  s.elem = a.dtype == BDH_DTYPE_F32 ? 4 : 2;
  s.a[0] = a.q;
  s.a[1] = a.q_lo;
  s.b[0] = a.k;
  s.b[1] = a.k_lo;
  for (int i = 0; i < 4; ++i) {
    s.a_strides[i] = a.q_strides[i];
    s.b_strides[i] = a.k_strides[i];
  }
  s.B = a.B;
  s.H = a.H;
  s.Hb = a.H;
  s.T = a.T;
  s.K = a.N;
  s.mode = kStoreDirect;
  s.p_hi = p_hi;
  s.p_lo = p_lo;
  if (s.elem == 4 && part != nullptr) {
    s.ksplit = score_ksplit_f32(a.B * a.H, a.T, a.N);
    s.part = part;
  }
  return launch_score_pass(s, stream, err);
}

// Value pass: out = P V from the hi/lo score pair (bf16: p_lo null = P as one bf16 term).
int launch_value(const FwdArgs& a, const void* p_hi, const void* p_lo, cudaStream_t stream,
                 int* err) {
  const int elem = a.dtype == BDH_DTYPE_F32 ? 4 : 2;
  const int64_t ldp = score_ld(a.T);
  const int64_t units = a.B * a.H;
  auto fill = [&](auto& prm, int bk, int bn) -> bool {
    const int64_t pd[4] = {a.T, a.T, units, 1};
    const int64_t ps[3] = {ldp * elem, a.T * ldp * elem, units * a.T * ldp * elem};
    if (!make_map_4d(&prm.a_map[0], p_hi, elem, pd, ps, bk, 128, "value pass: P hi")) return false;
    if (p_lo != nullptr && !make_map_4d(&prm.a_map[1], p_lo, elem, pd, ps, bk, 128, "value pass: P lo"))
      return false;
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
      if (!make_map_4d(&prm.b_map[0], a.v, 4, vd, vs, bk, 128, "value pass: v^T hi")) return false;
      if (!make_map_4d(&prm.b_map[1], a.v_lo, 4, vd, vs, bk, 128, "value pass: v^T lo")) return false;
    }
    prm.H = static_cast<int>(a.H);
    prm.Hv = static_cast<int>(a.Hv);
    prm.T = static_cast<int>(a.T);
    prm.D = static_cast<int>(a.D);
    prm.mt = static_cast<int>((a.T + 127) / 128);
    prm.nd = static_cast<int>((a.D + bn - 1) / bn);
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
  if (elem != 2 && p_lo == nullptr) {
    set_error("value pass: the fp32 path needs the tf32 hi/lo score pair");
    return BDH_ERR_INVALID;
  }
  if (elem == 2 && a.ln && a.D <= ValueLnBf16One::S::BN) {  // LayerNorm in the epilogue
    if (p_lo == nullptr) {
      ValueLnBf16One::Params prm{};
      if (!fill(prm, ValueLnBf16One::S::BK, ValueLnBf16One::BN)) return BDH_ERR_INVALID;
      prm.ln_eps = a.ln_eps;
      return launch_tc<ValueLnBf16One::S, ValueLnBf16One>(prm, prm.units * prm.mt * prm.nd,
                                                          stream, kProfValue);
    }
    ValueLnBf16::Params prm{};
    if (!fill(prm, ValueLnBf16::S::BK, ValueLnBf16::BN)) return BDH_ERR_INVALID;
    prm.ln_eps = a.ln_eps;
    return launch_tc<ValueLnBf16::S, ValueLnBf16>(prm, prm.units * prm.mt * prm.nd, stream,
                                                  kProfValue);
  }
  if (elem == 2 && p_lo == nullptr) {
    ValueBf16One::Params prm{};
    if (!fill(prm, ValueBf16One::S::BK, ValueBf16One::BN)) return BDH_ERR_INVALID;
    return launch_tc<ValueBf16One::S, ValueBf16One>(prm, prm.units * prm.mt * prm.nd, stream,
                                                    kProfValue);
  }
  if (elem == 2) {
    ValueBf16::Params prm{};
    if (!fill(prm, ValueBf16::S::BK, ValueBf16::BN)) return BDH_ERR_INVALID;
    return launch_tc<ValueBf16::S, ValueBf16>(prm, prm.units * prm.mt * prm.nd, stream, kProfValue);
  } else {
    ValueTf32::Params prm{};
    if (!fill(prm, ValueTf32::S::BK, ValueTf32::BN)) return BDH_ERR_INVALID;
    return launch_tc<ValueTf32::S, ValueTf32>(prm, prm.units * prm.mt * prm.nd, stream, kProfValue);
  }
}

}  // namespace bdh

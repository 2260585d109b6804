// Chunked long-sequence forward (bf16): the same strict-causal product computed as
//
//   out[c-th chunk rows] = tril(Q_c K_c^T, -1) V_c  +  Q_c S_{c-1},   S_c = sum_{c' <= c} K_c'^T V_c'
//
// with chunks of C keys. Work per (b,h) unit drops from T(T-1)(N+D) to about
// T(C-1)(N+D) + 2 T N D flops (for T = 8192, C = 256: 52 instead of 567 GFLOP), at the cost of
// streaming the N x D prefix states through HBM once written, once read (one bf16 term by
// default, 2 bytes per element; bf16 hi/lo with BDH_SM100_SPLIT_SCORES=1, which doubles the
// inter-chunk product and its bytes). C is 256 below T = 4096 and 512 from there on
// (chunk_len): the longer chunk doubles
// the intra-chunk score work but halves the prefix-state traffic, which bounds the state and
// value passes at long T (BDH_SM100_CHUNK=256|512 forces one).
//
// Three persistent tcgen05 passes (tc_engine.cuh):
//   1. score pass restricted to each 128-row block's own chunk (score_pass.cuh, chunk > 0),
//      P stored per row relative to the chunk start: [u][T][C] (bf16, or hi/lo);
//   2. state pass: S = K^T V accumulated over keys in chunk-sized accumulation rounds; after
//      each chunk the running fp32 sum (in registers) is written as the bf16 (or hi/lo) prefix
//      S_c ([u][chunk][N][D]) used by the next chunk; operands read MN-major straight from the
//      latents (keys are the contraction dimension);
//   3. chunk value pass: per 128-row block, K-segment 1 = intra-chunk P V, K-segment 2 = Q S_{c-1}
//      over the latent width, both accumulated into the same TMEM tile.
// The reference computes this path quadratically (kernels/attention.py:27-40, 676-777;
// csrc/tril_attn_cuda.cu:129-249); the chunked form is the north-star formulation.
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

int forced_chunk() {
  static int c = [] {
    const char* e = std::getenv("BDH_SM100_CHUNK");
    const int v = e ? std::atoi(e) : 0;
    return (v == 256 || v == 512) ? v : 0;
  }();
  return c;
}

// ------------------------------------------------------------------- state pass ----
// Each tile is a 128 (latent) x 128 (value) block of the N x D state; its epilogue emits one
// bf16 prefix per chunk (32 KB per tile per chunk, 64 KB as hi/lo), so the pass is bound by HBM
// writes.
// Every epilogue warp stages its 32 rows in shared memory in the 128B-swizzled layout of the
// store tensor map and writes them with four TMA bulk stores (whole 128-byte lines), then
// reuses the staging once the previous chunk's stores have read it.
// ST = 2: S as bf16 hi + lo; ST = 1: S as one bf16 term.
// BNS = 256 (D = 256 in one tile, eight epilogue warps, each 32 rows x 128 columns): every key
// row is staged once per latent block instead of once per 128-column value half, a quarter less
// operand traffic out of L2 (the latents once, V once per latent block) at three stages of
// 48 KB instead of four of 32 KB.
template <int STAGES, int CKB, int ST = 2, int BNS = 128>  // CKB = k-blocks (64 keys) per chunk
struct StateProb {
  using S = TcShape<2, BNS, true, true, 1, 1, STAGES, CKB>;
  static constexpr int kEmitEveryChunk = 1;
  static constexpr int kEpiWarps = BNS == 256 ? 8 : 4;
  static constexpr int kWarpStage = 2 * ST * 32 * 128;  // terms x two 64-column boxes x 32 rows
  static constexpr int kEpiSmemBytes = kEpiWarps * kWarpStage;
  struct Params {
    CUtensorMap a_map[1];  // K (B,H,T,N) read MN-major: box 64 (n) x 64 (t)
    CUtensorMap b_map[1];  // V (B,Hv,T,D) read MN-major: box 64 (d) x 64 (t)
    CUtensorMap s_map[2];  // S hi/lo over [units][nchunks][N][D], store box 64 (d) x 32 (n)
    int H, Hv, T, N, D;
    int nn, nd;            // 128-wide latent / value tiles
    int units, nchunks;
    int* err;
  };
  struct Tile {
    int unit, ni, di;
  };
  __device__ static int num_tiles(const Params& p) { return p.units * p.nn * p.nd; }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    tl.unit = t / (p.nn * p.nd);
    const int r = t - tl.unit * p.nn * p.nd;
    tl.ni = r / p.nd;
    tl.di = r - tl.ni * p.nd;
    return tl;
  }
  // the last chunk's total is never needed
  __device__ static int k_blocks(const Params& p, const Tile&) { return (p.nchunks - 1) * CKB; }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map[0]);
    tma_prefetch_desc(&p.b_map[0]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int hv = p.Hv == 1 ? 0 : h;
    const int t0 = kb * 64;
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d(&p.a_map[0], bar, a_dst + c * 64 * 128, tl.ni * 128 + c * 64, t0, h, b);
#pragma unroll
    for (int c = 0; c < BNS / 64; ++c)
      tma_load_4d(&p.b_map[0], bar, b_dst + c * 64 * 128, tl.di * BNS + c * 64, t0, hv, b);
  }
  __device__ static void epilogue(const Params&, const Tile&, int, int, const uint32_t (&)[32]) {}
  // After chunk ch the running sum is S_ch, the prefix state of chunk ch + 1.
  __device__ static void epilogue_chunk(const Params& p, const Tile& tl, int row, int ch, int,
                                        int c_tile, const uint32_t (&r)[32], uint8_t* epi) {
    const int quad = row >> 5, lr = row & 31;
    const bool leader = lr == 0;
    const int part = c_tile >> 7;  // this warp's 128 of the tile's columns
    const int c0 = c_tile & 127;
    uint8_t* st = epi + (part * 4 + quad) * kWarpStage;
    if (c0 == 0) {
      // the previous chunk's stores must have read the staging before it is overwritten
      if (leader) bulk_wait_read_all();
      __syncwarp();
    }
    const int half = c0 >> 6;
    const int j0 = (c0 & 63) >> 3;
    uint8_t* hi_row = st + half * 4096 + lr * 128;
    uint8_t* lo_row = hi_row + 2 * 4096;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint32_t wh[4], wl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0 = __uint_as_float(r[8 * v + 2 * e]), x1 = __uint_as_float(r[8 * v + 2 * e + 1]);
        wh[e] = cvt_bf16x2(x0, x1);
        if (ST == 2) wl[e] = cvt_bf16x2(x0 - bf16x2_lo(wh[e]), x1 - bf16x2_hi(wh[e]));
      }
      const int sw = ((j0 + v) ^ (lr & 7)) << 4;
      *reinterpret_cast<uint4*>(hi_row + sw) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
      if (ST == 2) *reinterpret_cast<uint4*>(lo_row + sw) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
    }
    if (c0 + 32 == 128) {
      fence_async_smem();
      __syncwarp();
      const int n0 = tl.ni * 128 + quad * 32;
      if (leader && n0 < p.N) {
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int x = tl.di * BNS + part * 128 + hb * 64;
          if (x < p.D) {
            tma_store_4d(&p.s_map[0], st + hb * 4096, x, n0, ch + 1, tl.unit);
            if (ST == 2) tma_store_4d(&p.s_map[1], st + (2 + hb) * 4096, x, n0, ch + 1, tl.unit);
          }
        }
        bulk_commit();
      }
    }
  }
  __device__ static void epilogue_end(const Params&, int row, uint8_t*) {
    if ((row & 31) == 0) bulk_wait_all();
    __syncwarp();
  }
};

// -------------------------------------------------------------- chunk value pass ----
// ONE: P and S as one bf16 term each (one product per k-block in both segments).
template <int STAGES, bool ONE = false>
struct ChunkValueProb {
  static constexpr int BN = 128;
  using S = TcShape<2, BN, false, true, ONE ? 1 : 2, ONE ? 1 : 2, STAGES>;
  static constexpr int kVarStageTx = 1;
  struct Params {
    CUtensorMap p_map[2];  // P hi/lo over [units][T][C], box 64 x 128
    CUtensorMap v_map;     // V (B,Hv,T,D), box 64 (d) x 64 (t)
    CUtensorMap q_map;     // Q (B,H,T,N), box 64 (n) x 128 (t)
    CUtensorMap s_map[2];  // S hi/lo over [units][nchunks][N][D], box 64 (d) x 64 (n)
    int H, Hv, T, N, D;
    int mt, nd, units, nchunks;
    int chunk;             // keys per chunk (256 or 512)
    void* out;             // (B,H,T,D) strided
    int64_t os_b, os_h, os_t;
    int out_f32, vec_ok;
    int* err;
  };
  struct Tile {
    int unit, mi, ni;
  };
  __device__ static int num_tiles(const Params& p) { return p.units * p.mt * p.nd; }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    tl.unit = t / (p.mt * p.nd);
    const int r = t - tl.unit * p.mt * p.nd;
    tl.mi = r / p.nd;
    tl.ni = r - tl.mi * p.nd;
    return tl;
  }
  __device__ static int cs(const Params& p, const Tile& tl) {
    return (tl.mi * 128 / p.chunk) * p.chunk;
  }
  __device__ static int n_intra(const Params& p, const Tile& tl) {
    return ceil_div_d(min(p.T, (tl.mi + 1) * 128) - cs(p, tl), 64);
  }
  __device__ static int n_inter(const Params& p, const Tile& tl) {
    return cs(p, tl) > 0 ? ceil_div_d(p.N, 64) : 0;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) { return n_intra(p, tl) + n_inter(p, tl); }
  // intra: A0 A1 (P hi, lo) x B0 (V); inter: A0 (Q) x B0 B1 (S hi, lo); ONE: A0 x B0 in both
  __device__ static uint32_t pair_mask(const Params& p, const Tile& tl, int kb) {
    if (ONE) return 0x1u;
    return kb < n_intra(p, tl) ? 0x3u : 0x5u;
  }
  __device__ static uint32_t stage_tx(const Params& p, const Tile& tl, int kb) {
    if (ONE) return S::A_TILE + S::B_TILE;
    return kb < n_intra(p, tl) ? 2 * S::A_TILE + S::B_TILE : S::A_TILE + 2 * S::B_TILE;
  }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.p_map[0]);
    if (!ONE) tma_prefetch_desc(&p.p_map[1]);
    tma_prefetch_desc(&p.v_map);
    tma_prefetch_desc(&p.q_map);
    tma_prefetch_desc(&p.s_map[0]);
    if (!ONE) tma_prefetch_desc(&p.s_map[1]);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int ni = n_intra(p, tl);
    if (kb < ni) {
      const int hv = p.Hv == 1 ? 0 : h;
      for (int i = 0; i < (ONE ? 1 : 2); ++i)
        tma_load_4d(&p.p_map[i], bar, a_dst + i * S::A_TILE, kb * 64, tl.mi * 128, tl.unit, 0);
#pragma unroll
      for (int c = 0; c < 2; ++c)
        tma_load_4d(&p.v_map, bar, b_dst + c * 64 * 128, tl.ni * BN + c * 64, cs(p, tl) + kb * 64, hv, b);
    } else {
      const int n0 = (kb - ni) * 64;
      const int chunk = cs(p, tl) / p.chunk;
      tma_load_4d(&p.q_map, bar, a_dst, n0, tl.mi * 128, h, b);
      for (int i = 0; i < (ONE ? 1 : 2); ++i)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tma_load_4d(&p.s_map[i], bar, b_dst + i * S::B_TILE + c * 64 * 128, tl.ni * BN + c * 64,
                      n0, chunk, tl.unit);
    }
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int row, int c0,
                                  const uint32_t (&r)[32]) {
    const int gi = tl.mi * 128 + row;
    if (gi >= p.T) return;
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int gd0 = tl.ni * BN + c0;
    if (gd0 >= p.D) return;
    const int64_t off = b * p.os_b + h * p.os_h + gi * p.os_t + gd0;
    if (p.out_f32) {
      float* o = static_cast<float*>(p.out) + off;
      for (int e = 0; e < 32 && gd0 + e < p.D; ++e) o[e] = __uint_as_float(r[e]);
      return;
    }
    uint16_t* o = static_cast<uint16_t*>(p.out) + off;
    if (p.vec_ok && gd0 + 32 <= p.D) {
#pragma unroll
      for (int v = 0; v < 4; ++v)
        *reinterpret_cast<uint4*>(o + 8 * v) = make_uint4(
            cvt_bf16x2(__uint_as_float(r[8 * v]), __uint_as_float(r[8 * v + 1])),
            cvt_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3])),
            cvt_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5])),
            cvt_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7])));
    } else {
      for (int e = 0; e < 32 && gd0 + e < p.D; ++e)
        o[e] = static_cast<uint16_t>(f32_to_bf16_bits(__uint_as_float(r[e])));
    }
  }
};

// CTA-pair form of the chunk value pass: one 256-row pair tile (a whole chunk at C = 256, half
// of one at C = 512), both row blocks at once (M = 256 across the pair), N = 256 value columns.
// Each CTA stages its own 128 rows of P / Q and its own 128 columns of V / S, so the operand
// bytes per SM per flop halve against the single-CTA form (whose inter-chunk Q S segment is
// bound by L2 -> shared memory ingress). The intra segment of a pair tile covers the keys from
// its chunk's start to the tile's last row; P holds zeros above the diagonal there (the pair
// score pass stores whole 256-key tiles).
template <bool ONE>
struct ChunkValuePairT {
  using Base = ChunkValueProb<ONE ? 4 : 3, ONE>;  // parameters and epilogue
  using Params = typename Base::Params;
  using S = PairShape<false, true, ONE ? 1 : 2, ONE ? 1 : 2, ONE ? 6 : 3>;
  struct Tile {
    int unit, c, n;  // c: 256-row pair tile of the unit
  };
  __device__ static int ntile(const Params& p) { return ceil_div_d(p.T, 256); }
  __device__ static int nd2(const Params& p) { return ceil_div_d(p.D, 256); }
  __device__ static int num_tiles(const Params& p) { return p.units * ntile(p) * nd2(p); }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    const int per = ntile(p) * nd2(p);
    tl.unit = t / per;
    const int r = t - tl.unit * per;
    tl.c = r / nd2(p);
    tl.n = r - tl.c * nd2(p);
    return tl;
  }
  __device__ static int chunk(const Params& p, const Tile& tl) { return tl.c * 256 / p.chunk; }
  __device__ static int n_intra(const Params& p, const Tile& tl) {
    return ceil_div_d(min(p.T, (tl.c + 1) * 256) - chunk(p, tl) * p.chunk, 64);
  }
  __device__ static int n_inter(const Params& p, const Tile& tl) {
    return chunk(p, tl) > 0 ? ceil_div_d(p.N, 64) : 0;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) { return n_intra(p, tl) + n_inter(p, tl); }
  __device__ static uint32_t pair_mask(const Params& p, const Tile& tl, int kb) {
    if (ONE) return 0x1u;
    return kb < n_intra(p, tl) ? 0x3u : 0x5u;
  }
  __device__ static uint32_t stage_tx(const Params& p, const Tile& tl, int kb) {
    if (ONE) return 2u * (S::A_TILE + S::B_TILE);
    return 2u * (kb < n_intra(p, tl) ? 2 * S::A_TILE + S::B_TILE : S::A_TILE + 2 * S::B_TILE);
  }
  __device__ static void prefetch(const Params& p) { Base::prefetch(p); }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint32_t rank,
                                    uint32_t bar, uint8_t* a_dst, uint8_t* b_dst) {
    const int b = tl.unit / p.H, h = tl.unit - (tl.unit / p.H) * p.H;
    const int r128 = static_cast<int>(rank) * 128;
    const int row0 = tl.c * 256 + r128;  // this CTA's 128 rows
    const int col0 = tl.n * 256 + r128;  // this CTA's 128 value columns
    const int ch = chunk(p, tl);
    const int ni = n_intra(p, tl);
    if (kb < ni) {
      const int hv = p.Hv == 1 ? 0 : h;
      for (int i = 0; i < (ONE ? 1 : 2); ++i)
        tma_load_4d_pair(&p.p_map[i], bar, a_dst + i * S::A_TILE, kb * 64, row0, tl.unit, 0);
#pragma unroll
      for (int c = 0; c < 2; ++c)
        tma_load_4d_pair(&p.v_map, bar, b_dst + c * 64 * 128, col0 + c * 64, ch * p.chunk + kb * 64,
                         hv, b);
    } else {
      const int n0 = (kb - ni) * 64;
      tma_load_4d_pair(&p.q_map, bar, a_dst, n0, row0, h, b);
      for (int i = 0; i < (ONE ? 1 : 2); ++i)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          tma_load_4d_pair(&p.s_map[i], bar, b_dst + i * S::B_TILE + c * 64 * 128, col0 + c * 64, n0,
                           ch, tl.unit);
    }
  }
  __device__ static void epilogue(const Params& p, const Tile& tl, int rank, int row, int c0,
                                  const uint32_t (&r)[32]) {
    typename Base::Tile t;
    t.unit = tl.unit;
    t.mi = 2 * tl.c + rank;
    t.ni = 2 * tl.n;  // Base columns: ni * 128 + c0 with c0 in [0, 256)
    Base::epilogue(p, t, row, c0, r);
  }
};
using ChunkValuePair = ChunkValuePairT<false>;
using ChunkValuePairOne = ChunkValuePairT<true>;

bool use_pairs_chunked() {
  static int on = [] {
    const char* e = std::getenv("BDH_SM100_PAIR");
    return (e != nullptr && std::atoi(e) == 0) ? 0 : 1;
  }();
  return on != 0;
}

using StateBf16C256 = StateProb<4, 4>;
using StateBf16C512 = StateProb<4, 8>;
using StateBf16C256One = StateProb<3, 4, 1, 256>;
using StateBf16C512One = StateProb<3, 8, 1, 256>;

}  // namespace

int chunk_len(int64_t T) {
  const int f = forced_chunk();
  if (f > 0) return f;
  return T >= 4096 ? 512 : 256;
}

size_t chunked_p_bytes(int64_t B, int64_t H, int64_t T) {
  return static_cast<size_t>(B * H * T * chunk_len(T)) * 2;
}
size_t chunked_s_bytes(int64_t B, int64_t H, int64_t T, int64_t N, int64_t D) {
  const int64_t C = chunk_len(T);
  const int64_t nch = (T + C - 1) / C;
  return static_cast<size_t>(B * H * nch * N * D) * 2;
}

namespace {
template <class SP>
int launch_state_pass(const FwdArgs& a, void* s_hi, void* s_lo, int nchunks, cudaStream_t stream,
                      int* err) {
  typename SP::Params prm{};
  const int64_t kd[4] = {a.N, a.T, a.H, a.B};
  const int64_t ks[3] = {a.k_strides[2] * 2, a.k_strides[1] * 2, a.k_strides[0] * 2};
  const int64_t vd[4] = {a.D, a.T, a.Hv, a.B};
  const int64_t vs[3] = {a.v_strides[2] * 2, a.v_strides[1] * 2, a.v_strides[0] * 2};
  if (!make_map_4d(&prm.a_map[0], a.k, 2, kd, ks, 64, 64, "state pass: K")) return BDH_ERR_INVALID;
  if (!make_map_4d(&prm.b_map[0], a.v, 2, vd, vs, 64, 64, "state pass: V")) return BDH_ERR_INVALID;
  prm.H = static_cast<int>(a.H);
  prm.Hv = static_cast<int>(a.Hv);
  prm.T = static_cast<int>(a.T);
  prm.N = static_cast<int>(a.N);
  prm.D = static_cast<int>(a.D);
  prm.nn = static_cast<int>((a.N + 127) / 128);
  prm.nd = static_cast<int>((a.D + SP::S::BN - 1) / SP::S::BN);
  prm.units = static_cast<int>(a.B * a.H);
  prm.nchunks = nchunks;
  const int64_t sd[4] = {a.D, a.N, nchunks, a.B * a.H};
  const int64_t ss[3] = {a.D * 2, a.N * a.D * 2, int64_t(nchunks) * a.N * a.D * 2};
  if (!make_map_4d(&prm.s_map[0], s_hi, 2, sd, ss, 64, 32, "state pass: S hi")) return BDH_ERR_INVALID;
  if (s_lo != nullptr && !make_map_4d(&prm.s_map[1], s_lo, 2, sd, ss, 64, 32, "state pass: S lo"))
    return BDH_ERR_INVALID;
  prm.err = err;
  return launch_tc<typename SP::S, SP>(prm, prm.units * prm.nn * prm.nd, stream, kProfState);
}

// 3. intra P V + inter Q S (ONE: P and S as one bf16 term each).
template <bool ONE>
int launch_chunk_value(const FwdArgs& a, void* p_hi, void* p_lo, void* s_hi, void* s_lo, int C,
                       int nchunks, cudaStream_t stream, int* err) {
  using CP = ChunkValuePairT<ONE>;
  using CV = typename CP::Base;
  const int64_t units = a.B * a.H;
  typename CP::Params prm{};
  const int64_t pd[4] = {C, a.T, units, 1};
  const int64_t ps[3] = {int64_t(C) * 2, a.T * C * 2, units * a.T * C * 2};
  if (!make_map_4d(&prm.p_map[0], p_hi, 2, pd, ps, 64, 128, "chunk value pass: P hi")) return BDH_ERR_INVALID;
  if (!ONE && !make_map_4d(&prm.p_map[1], p_lo, 2, pd, ps, 64, 128, "chunk value pass: P lo"))
    return BDH_ERR_INVALID;
  const int64_t vd[4] = {a.D, a.T, a.Hv, a.B};
  const int64_t vs[3] = {a.v_strides[2] * 2, a.v_strides[1] * 2, a.v_strides[0] * 2};
  if (!make_map_4d(&prm.v_map, a.v, 2, vd, vs, 64, 64, "chunk value pass: V")) return BDH_ERR_INVALID;
  const int64_t qd[4] = {a.N, a.T, a.H, a.B};
  const int64_t qs[3] = {a.q_strides[2] * 2, a.q_strides[1] * 2, a.q_strides[0] * 2};
  if (!make_map_4d(&prm.q_map, a.q, 2, qd, qs, 64, 128, "chunk value pass: Q")) return BDH_ERR_INVALID;
  const int64_t sd[4] = {a.D, a.N, nchunks, units};
  const int64_t ss[3] = {a.D * 2, a.N * a.D * 2, int64_t(nchunks) * a.N * a.D * 2};
  if (!make_map_4d(&prm.s_map[0], s_hi, 2, sd, ss, 64, 64, "chunk value pass: S hi")) return BDH_ERR_INVALID;
  if (!ONE && !make_map_4d(&prm.s_map[1], s_lo, 2, sd, ss, 64, 64, "chunk value pass: S lo"))
    return BDH_ERR_INVALID;
  prm.H = static_cast<int>(a.H);
  prm.Hv = static_cast<int>(a.Hv);
  prm.T = static_cast<int>(a.T);
  prm.N = static_cast<int>(a.N);
  prm.D = static_cast<int>(a.D);
  prm.mt = static_cast<int>((a.T + 127) / 128);
  prm.nd = static_cast<int>((a.D + CV::BN - 1) / CV::BN);
  prm.units = static_cast<int>(units);
  prm.nchunks = nchunks;
  prm.chunk = C;
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
  if (use_pairs_chunked()) {
    const int tiles = prm.units * static_cast<int>((a.T + 255) / 256) * static_cast<int>((a.D + 255) / 256);
    return launch_pair<typename CP::S, CP>(prm, tiles, stream, kProfValue);
  }
  return launch_tc<typename CV::S, CV>(prm, prm.units * prm.mt * prm.nd, stream, kProfValue);
}
}  // namespace

int launch_chunked_forward(const FwdArgs& a, void* p_hi, void* p_lo, void* s_hi, void* s_lo,
                           cudaStream_t stream, int* err) {
  if (a.dtype != BDH_DTYPE_BF16) {
    set_error("chunked forward: bf16 inputs only");
    return BDH_ERR_INVALID;
  }
  // p_lo / s_lo null: P and the prefix states as one bf16 term each
  const bool one = p_lo == nullptr || s_lo == nullptr;
  if (one && (p_lo != nullptr || s_lo != nullptr)) {
    set_error("chunked forward: P and S are both split or both single bf16 terms");
    return BDH_ERR_INVALID;
  }
  const int C = chunk_len(a.T);
  const int nchunks = static_cast<int>((a.T + C - 1) / C);
  // 1. intra-chunk scores
  ScoreArgs sa;
  sa.elem = 2;
  sa.a[0] = a.q;
  sa.b[0] = a.k;
  for (int i = 0; i < 4; ++i) {
    sa.a_strides[i] = a.q_strides[i];
    sa.b_strides[i] = a.k_strides[i];
  }
  sa.B = a.B; sa.H = a.H; sa.Hb = a.H; sa.T = a.T; sa.K = a.N;
  sa.mode = kStoreDirect;
  sa.chunk = C;
  sa.p_hi = p_hi;
  sa.p_lo = p_lo;
  int rc = launch_score_pass(sa, stream, err);
  if (rc) return rc;
  // 2. prefix states S_1 .. S_{nchunks-1}
  if (nchunks > 1) {
    if (one)
      rc = C == 512 ? launch_state_pass<StateBf16C512One>(a, s_hi, nullptr, nchunks, stream, err)
                    : launch_state_pass<StateBf16C256One>(a, s_hi, nullptr, nchunks, stream, err);
    else
      rc = C == 512 ? launch_state_pass<StateBf16C512>(a, s_hi, s_lo, nchunks, stream, err)
                    : launch_state_pass<StateBf16C256>(a, s_hi, s_lo, nchunks, stream, err);
    if (rc) return rc;
  }
  // 3. intra P V + inter Q S
  return one ? launch_chunk_value<true>(a, p_hi, p_lo, s_hi, s_lo, C, nchunks, stream, err)
             : launch_chunk_value<false>(a, p_hi, p_lo, s_hi, s_lo, C, nchunks, stream, err);
}

}  // namespace bdh

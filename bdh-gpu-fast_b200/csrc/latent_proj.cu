// The two latent projections that feed and follow the attention path in a BDH layer, each a
// K = D contraction (D = 256) whose epilogue carries the elementwise work the reference runs
// as separate passes over the (B, T, nh, N) latent:
//
//   encode: xs = relu(bf16(x enc_h))                      bdh.py:861-912 (_encoder_relu)
//           qr = R(xs) at positions pos0 + t              kernels/rope.py:108-126, bdh.py:396-412
//   gate:   xy = bf16(xs * relu(bf16(y_h encv_h)))        bdh.py:914-945 (_encoder_v_relu and
//                                                         the x * y product of _mlp_merge)
//
// x: (B, T, D) bf16; y: (B, H, T, D) bf16 (the LayerNormed attention output); enc / encv:
// (H, D, N) bf16; xs / xy: (B, T, H, N) bf16; qr: (B, H, T, N) bf16 (the attention operand or
// a cache slot). Both kernels move 2 x 128 x 128 x 2 bytes of latent per 128 x 128 tile and
// do only 8.4 MFLOP in it, so they are bound by HBM: each 32-row epilogue slice is staged in
// 128B-swizzled shared memory (double buffered) and leaves through TMA bulk stores; the gate
// kernel brings its xs slice in the same way with a TMA load issued one tile ahead.
//
// RoPE in the encode epilogue: BDH's frequencies come in equal pairs (bdh.py:41-49), so one
// (cos, sin) serves both elements of a pair. Tiles are walked in contiguous ranges ordered
// (t block, n block) outer and (b, h) inner, so a thread's 64 (cos, sin) pairs are computed
// once and reused across all B x H tiles that share its positions and columns.
#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include <string>

#include "bdh_sm100.h"
#include "common.cuh"
#include "internal.h"
#include "score_pass.cuh"
#include "tc_engine.cuh"
#include "tma_host.h"

namespace bdh {

namespace {

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Byte offset of the 16-byte chunk `j` (0..7) of row `r` inside a 128B-swizzled box.
__device__ __forceinline__ int sw128(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

struct LatentTile {
  int b, h, tb, nb;
};

// Tile order: group (tb, nb) outer, (b, h) inner.
__device__ __forceinline__ LatentTile latent_tile(int t, int B, int H, int nb_n) {
  LatentTile tl;
  const int bh = B * H;
  const int g = t / bh;
  const int w = t - g * bh;
  tl.b = w / H;
  tl.h = w - tl.b * H;
  tl.tb = g / nb_n;
  tl.nb = g - tl.tb * nb_n;
  return tl;
}

struct EncodeParams {
  CUtensorMap a_map;   // x (B,T,D): box 64 (k) x 128 (t)
  CUtensorMap b_map;   // enc (H,D,N): n-contiguous box 64 (n) x 64 (k), or d-contiguous 64 x 128
  CUtensorMap xs_map;  // xs (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1
  CUtensorMap qr_map;  // qr (B,H,T,N) as {N,T,H,B}: box 64 x 32 x 1 x 1
  const float* freqs;
  int B, T, H, D, N, pos0;
  int tb_n, nb_n;
  int walk_chunk;        // row blocks per chunk of the chunked walk (divides B * tb_n)
  int walk_rot;          // chunks start at rotated row blocks (latent_tile_chunked)
  FastDiv fd_chunk, fd_ncb, fd_b, fd_nb;  // by walk_chunk, H * nb_n, B, nb_n
  int* err;
};

struct GateParams {
  CUtensorMap a_map;   // y (B,H,T,D): box 64 (k) x 128 (t)
  CUtensorMap b_map;   // encv (H,D,N): n-contiguous box 64 (n) x 64 (k), or d-contiguous 64 x 128
  CUtensorMap xs_map;  // xs (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1 (load)
  CUtensorMap xy_map;  // xy (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1 (store)
  int B, T, H, D, N;
  int tb_n, nb_n;
  int walk_chunk;        // row blocks per chunk of the chunked walk (divides B * tb_n)
  int walk_rot;          // chunks start at rotated row blocks (latent_tile_chunked)
  FastDiv fd_chunk, fd_ncb, fd_b, fd_nb;  // by walk_chunk, H * nb_n, B, nb_n
  int* err;
};

// xy stores from registers: lane (g, j) of a warp that holds tile rows quadrant*32 + lane (64
// columns from n0 as eight 16-byte chunks) transposes them so that it stores chunk j of rows
// 8g..8g+7; every 8 lanes then write one contiguous 128-byte row segment.
__device__ __forceinline__ void store_xy_rows(uint16_t* xy, int64_t sb, int64_t st, int64_t sh,
                                              int T, int N, int b, int h, int t_quad, int n0,
                                              int lane, uint4 (&c)[8]) {
  transpose_chunks8(c, lane);
  const int n = n0 + (lane & 7) * 8;
  const int t0 = t_quad + (lane >> 3) * 8;
  uint16_t* base = xy + b * sb + h * sh + n;
  const uint64_t stream = l2_policy_evict_first();
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int t = t0 + k;
    if (t >= T || n >= N) continue;
    uint16_t* dst = base + static_cast<int64_t>(t) * st;
    if (n + 8 <= N) {
      st_global_v4_hint(dst, c[k], stream);
    } else {  // ragged last chunk (N even): whole bf16 pairs
      const uint32_t w[4] = {c[k].x, c[k].y, c[k].z, c[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (2 * e < N - n) reinterpret_cast<uint32_t*>(dst)[e] = w[e];
    }
  }
}

struct GateXParams {
  CUtensorMap a_map;   // y (B,H,T,D): box 64 (k) x 128 (t)
  CUtensorMap a2_map;  // x (B,T,D): box 64 (k) x 128 (t)
  CUtensorMap b_map;   // encv (H,D,N), as the gate's b_map
  CUtensorMap b2_map;  // enc (H,D,N), same layout as encv
  uint16_t* xy;        // xy (B,T,H,N) bf16, element strides below (n contiguous)
  int64_t xy_sb, xy_st, xy_sh;
  int B, T, H, D, N;
  int tb_n, nb_n;
  int kbs;               // k-blocks of one product, ceil(D / 64)
  int walk_chunk;
  int walk_rot;
  FastDiv fd_chunk, fd_ncb, fd_b, fd_nb;
  int* err;
};

// The epilogue uses eight warps: two per TMEM lane quadrant, each draining one 64-column half
// of the 128 x 128 tile (warp slot ew = quadrant + 4 * half owns its staging buffers).

struct ContiguousWalk {
  static constexpr int kContiguousTiles = 1;
};
struct StridedWalk {};
// Chunks of walk_chunk row blocks of one column block (h, nb), the column block fastest across
// chunks: a CTA keeps the column block's weights resident for the whole chunk, and the CTAs
// running at one time write neighbouring column blocks of the same row chunk.
template <int KBR>
struct ChunkedResidentWalkT {
  static constexpr int kChunkedWalk = 1;
  static constexpr int kResidentB = KBR;
};
using ChunkedResidentWalk = ChunkedResidentWalkT<4>;  // D <= 256

template <class Prm>
__device__ __forceinline__ LatentTile latent_tile_chunked(int t, const Prm& p) {
  LatentTile tl;
  int c, i, rc, cb, q, j;
  p.fd_chunk.divmod(t, c, i);
  p.fd_ncb.divmod(c, rc, cb);
  // walk_rot: each chunk starts at a different row block of the row chunk (the CTAs running at
  // one time read different activation tiles); else every chunk walks its row blocks in order
  // (the CTAs of a row chunk write the same rows at one time)
  if (p.walk_rot)
    p.fd_chunk.divmod(i + c - p.fd_chunk.div(c) * static_cast<int>(p.fd_chunk.d), q, j);
  else
    j = i;
  const int rb = rc * static_cast<int>(p.fd_chunk.d) + j;
  p.fd_b.divmod(rb, tl.tb, tl.b);
  p.fd_nb.divmod(cb, tl.h, tl.nb);
  return tl;
}

template <int ORDER>
using LatentWalk = std::conditional_t<
    ORDER == 0, ContiguousWalk, std::conditional_t<ORDER == 3, ChunkedResidentWalk, StridedWalk>>;

// Tile order across the grid: n block fastest, so the CTAs running at one time write adjacent
// column blocks of the same rows.
__device__ __forceinline__ LatentTile latent_tile_nfast(int t, int B, int H, int tb_n, int nb_n) {
  LatentTile tl;
  tl.nb = t % nb_n;
  int r = t / nb_n;
  tl.h = r % H;
  r /= H;
  tl.tb = r % tb_n;
  tl.b = r / tb_n;
  return tl;
}

// ------------------------------------------------------------------------ encode ----
// Tile order for a grid of G = k * nb_n CTAs walking with stride G: every CTA keeps one n block,
// the CTAs running at one time cover adjacent n blocks of the same rows, and the position
// block (slowest index) changes only every B*H*nb_n/G tiles of a CTA.
__device__ __forceinline__ LatentTile latent_tile_colfixed(int t, int B, int H, int nb_n) {
  LatentTile tl;
  tl.nb = t % nb_n;
  int r = t / nb_n;
  tl.h = r % H;
  r /= H;
  tl.b = r % B;
  tl.tb = r / B;
  return tl;
}

// WX = false: qr only (xs is recomputed by the fused gate, bdh_latent_gate_x).
template <int STAGES, int BUFS, int ORDER = 0, bool KW = false, bool WX = true>
struct EncodeProb : LatentWalk<ORDER> {
  using S = TcShape<2, 128, false, !KW, 1, 1, STAGES>;
  static constexpr int kCustomEpilogue = 1;
  static constexpr int kEpiWarps = 8;
  static constexpr int kAccBuffers = 4;
  static constexpr int kBox = 32 * 128;           // one 64-column x 32-row swizzled box
  static constexpr int kBuf = WX ? 2 * kBox : kBox;  // (xs box +) qr box
  static constexpr int kWarpStage = BUFS * kBuf;  // BUFS staging buffers per warp
  static constexpr int kEpiSmemBytes = 8 * kWarpStage;
  using Params = EncodeParams;
  using Tile = LatentTile;
  struct EpiState {
    float c[32], s[32];  // (cos, sin) of this thread's row for its 32 column pairs
    int key;             // tb * nb_n + nb of the cached phases
    int iter;            // tiles finished by this thread (selects the staging buffer)
  };
  __device__ static int num_tiles(const Params& p) { return p.B * p.H * p.tb_n * p.nb_n; }
  __device__ static Tile tile(const Params& p, int t) {
    return ORDER == 0   ? latent_tile(t, p.B, p.H, p.nb_n)
           : ORDER == 1 ? latent_tile_nfast(t, p.B, p.H, p.tb_n, p.nb_n)
           : ORDER == 2 ? latent_tile_colfixed(t, p.B, p.H, p.nb_n)
                        : latent_tile_chunked(t, p);
  }
  __device__ static const FastDiv& walk_chunk(const Params& p) { return p.fd_chunk; }
  __device__ static int b_key(const Params& p, const Tile& tl) { return tl.h * p.nb_n + tl.nb; }
  static int max_ctas(const Params& p, int sms) {
    if (ORDER != 2) return sms;
    return p.nb_n <= sms ? (sms / p.nb_n) * p.nb_n : sms;
  }
  __device__ static int k_blocks(const Params& p, const Tile&) { return (p.D + 63) / 64; }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map);
    tma_prefetch_desc(&p.b_map);
  }
  __device__ static void load_b(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                uint8_t* dst) {
    const uint64_t keep = l2_policy_evict_last();
    if (KW) {  // K-major weights: one 64 (k) x 128 (n) box
      tma_load_4d_hint(&p.b_map, bar, dst, kb * 64, tl.nb * 128, tl.h, 0, keep);
      return;
    }
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d_hint(&p.b_map, bar, dst + c * 64 * 128, tl.nb * 128 + c * 64, kb * 64, tl.h, 0,
                       keep);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const uint64_t keep = l2_policy_evict_last();
    tma_load_4d_hint(&p.a_map, bar, a_dst, kb * 64, tl.tb * 128, tl.b, 0, keep);
    if (ORDER != 3) load_b(p, tl, kb, bar, b_dst);
  }
  __device__ static uint8_t* stage(uint8_t* epi, int row, int part, int iter) {
    return epi + ((row >> 5) + 4 * part) * kWarpStage + (iter % BUFS) * kBuf;
  }

  __device__ static void epilogue_begin(const Params&, int, int, uint8_t*, EpiState& st, bool,
                                        const Tile&) {
    st.key = -1;
    st.iter = 0;
  }
  // (cos, sin) for the tile's positions and this warp's columns, when they changed.
  __device__ static void epilogue_prefetch(const Params& p, const Tile& tl, bool, const Tile&,
                                           int row, int part, uint8_t*, EpiState& st) {
    const int key = tl.tb * p.nb_n + tl.nb;
    if (key == st.key) return;
    st.key = key;
    const float pos = static_cast<float>(p.pos0 + tl.tb * 128 + row);
    const int n0 = tl.nb * 128 + part * 64;
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const int n = n0 + 2 * q;
      const float f = n < p.N ? __ldg(p.freqs + n) : 0.0f;
      rope_cis(pos, f, st.c[q], st.s[q]);
    }
  }
  __device__ static bool epilogue_tile(const Params&, const Tile&, int row, int part, uint32_t taddr,
                                       uint8_t* epi, EpiState& st, volatile int*) {
    const int lr = row & 31;
    uint8_t* xs_box = stage(epi, row, part, st.iter);
    uint8_t* qr_box = WX ? xs_box + kBox : xs_box;
    // the stores that last read this buffer were committed BUFS tiles ago
    if (lr == 0) bulk_wait_read<BUFS - 1>();
    __syncwarp();
    uint32_t r2[2][32];
    tmem_ld32(taddr + static_cast<uint32_t>(part * 64), r2[0]);
    tmem_ld32(taddr + static_cast<uint32_t>(part * 64 + 32), r2[1]);
    tmem_ld_wait();
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      const uint32_t(&r)[32] = r2[c0 >> 5];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint32_t xw[4], qw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * v + 2 * e;
          const int q = (c0 >> 1) + 4 * v + e;
          xw[e] = cvt_relu_bf16x2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]));
          qw[e] = rotate_pair_bf16x2(bf16x2_lo(xw[e]), bf16x2_hi(xw[e]), st.c[q], st.s[q], st.c[q],
                                     st.s[q]);
        }
        const int off = sw128(lr, (c0 >> 3) + v);
        if (WX) *reinterpret_cast<uint4*>(xs_box + off) = make_uint4(xw[0], xw[1], xw[2], xw[3]);
        *reinterpret_cast<uint4*>(qr_box + off) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
      }
    }
    return true;
  }
  __device__ static void epilogue_after(const Params& p, const Tile& tl, int row, int part,
                                        uint8_t* epi, EpiState& st) {
    uint8_t* xs_box = stage(epi, row, part, st.iter);
    fence_async_smem();
    __syncwarp();
    if ((row & 31) == 0) {
      const int t0 = tl.tb * 128 + (row & ~31);
      const int n = tl.nb * 128 + part * 64;
      if (t0 < p.T && n < p.N) {
        const uint64_t stream = l2_policy_evict_first();
        if (WX) tma_store_4d_hint(&p.xs_map, xs_box, n, tl.h, t0, tl.b, stream);
        tma_store_4d_hint(&p.qr_map, WX ? xs_box + kBox : xs_box, n, t0, tl.h, tl.b, stream);
      }
      bulk_commit();  // one group per tile (possibly empty)
    }
    ++st.iter;
  }
  __device__ static void epilogue_end(const Params&, int row, int, uint8_t*, EpiState&) {
    if ((row & 31) == 0) bulk_wait_all();
    __syncwarp();
  }
};

// -------------------------------------------------------------------------- gate ----
template <int STAGES, int SLOTS, int ORDER = 0, bool KW = false>
struct GateProb : LatentWalk<ORDER> {
  using S = TcShape<2, 128, false, !KW, 1, 1, STAGES>;
  static constexpr int kCustomEpilogue = 1;
  static constexpr int kEpiWarps = 8;
  static constexpr int kAccBuffers = 4;
  static constexpr int kBox = 32 * 128;           // one 32 x 64 slice: xs in, xy out in place
  static constexpr int kSlots = SLOTS;            // >= 2: the next tile's slice loads while
                                                  // this tile is drained
  static constexpr int kWarpStage = kSlots * kBox;
  static constexpr int kBarOff = 8 * kWarpStage;  // kSlots mbarriers per warp after the buffers
  static constexpr int kEpiSmemBytes = kBarOff + 1024;
  using Params = GateParams;
  using Tile = LatentTile;
  struct EpiState {
    int iter;     // tiles finished by this thread
    int loaded;   // tiles whose xs slice load was issued
  };
  __device__ static int num_tiles(const Params& p) { return p.B * p.H * p.tb_n * p.nb_n; }
  __device__ static Tile tile(const Params& p, int t) {
    return ORDER == 0   ? latent_tile(t, p.B, p.H, p.nb_n)
           : ORDER == 3 ? latent_tile_chunked(t, p)
                        : latent_tile_nfast(t, p.B, p.H, p.tb_n, p.nb_n);
  }
  __device__ static const FastDiv& walk_chunk(const Params& p) { return p.fd_chunk; }
  __device__ static int b_key(const Params& p, const Tile& tl) { return tl.h * p.nb_n + tl.nb; }
  __device__ static int k_blocks(const Params& p, const Tile&) { return (p.D + 63) / 64; }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map);
    tma_prefetch_desc(&p.b_map);
    tma_prefetch_desc(&p.xs_map);
  }
  __device__ static void load_b(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                uint8_t* dst) {
    const uint64_t keep = l2_policy_evict_last();
    if (KW) {  // K-major weights: one 64 (k) x 128 (n) box
      tma_load_4d_hint(&p.b_map, bar, dst, kb * 64, tl.nb * 128, tl.h, 0, keep);
      return;
    }
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d_hint(&p.b_map, bar, dst + c * 64 * 128, tl.nb * 128 + c * 64, kb * 64, tl.h, 0,
                       keep);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    const uint64_t keep = l2_policy_evict_last();
    tma_load_4d_hint(&p.a_map, bar, a_dst, kb * 64, tl.tb * 128, tl.h, tl.b, keep);
    if (ORDER != 3) load_b(p, tl, kb, bar, b_dst);
  }
  __device__ static int slot_warp(int row, int part) { return (row >> 5) + 4 * part; }
  __device__ static uint64_t* bar(uint8_t* epi, int w, int slot) {
    return reinterpret_cast<uint64_t*>(epi + kBarOff) + w * kSlots + slot;
  }
  // Load the xs slice of tile number `st.loaded` (of this CTA's walk) into its slot.
  __device__ static void load_xs(const Params& p, const Tile& tl, int row, int part, uint8_t* epi,
                                 EpiState& st) {
    const int w = slot_warp(row, part);
    const int slot = st.loaded % kSlots;
    if ((row & 31) == 0) {
      // the slot was last read by the stores of tile (loaded - kSlots); at most the
      // kSlots - 2 most recent store groups may still be reading
      bulk_wait_read<kSlots - 2>();
      uint64_t* b = bar(epi, w, slot);
      uint8_t* buf = epi + w * kWarpStage + slot * kBox;
      const int t0 = tl.tb * 128 + (row & ~31);
      const int n = tl.nb * 128 + part * 64;
      if (t0 < p.T && n < p.N) {
        mbar_arrive_expect_tx(b, kBox);
        tma_load_4d_hint(&p.xs_map, b, buf, n, tl.h, t0, tl.b, l2_policy_evict_first());
      } else {
        mbar_arrive(b);
      }
    }
    __syncwarp();
    ++st.loaded;
  }
  __device__ static void epilogue_begin(const Params& p, int row, int part, uint8_t* epi,
                                        EpiState& st, bool has_first, const Tile& first) {
    if ((row & 31) == 0) {
      for (int i = 0; i < kSlots; ++i) mbar_init(bar(epi, slot_warp(row, part), i), 1);
      fence_mbar_init();
    }
    __syncwarp();
    st.iter = 0;
    st.loaded = 0;
    if (has_first) load_xs(p, first, row, part, epi, st);
  }
  // One tile ahead: the next tile's xs slice is requested before this tile is drained.
  __device__ static void epilogue_prefetch(const Params& p, const Tile&, bool has_next,
                                           const Tile& next, int row, int part, uint8_t* epi,
                                           EpiState& st) {
    if (has_next) load_xs(p, next, row, part, epi, st);
  }
  __device__ static bool epilogue_tile(const Params& p, const Tile&, int row, int part,
                                       uint32_t taddr, uint8_t* epi, EpiState& st,
                                       volatile int* abort_flag) {
    const int lr = row & 31;
    const int w = slot_warp(row, part);
    const int slot = st.iter % kSlots;
    uint8_t* box = epi + w * kWarpStage + slot * kBox;
    const uint32_t parity = static_cast<uint32_t>(st.iter / kSlots) & 1u;
    // the whole warp leaves together on a timeout (the TMEM loads below are warp-aligned)
    const bool ok = wait_bounded(bar(epi, w, slot), parity, abort_flag, p.err, kErrTimeoutEpilogue);
    if (!__all_sync(0xffffffffu, ok)) return false;
    uint32_t rr[2][32];
    tmem_ld32(taddr + static_cast<uint32_t>(part * 64), rr[0]);
    tmem_ld32(taddr + static_cast<uint32_t>(part * 64 + 32), rr[1]);
    tmem_ld_wait();
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      const uint32_t(&r)[32] = rr[c0 >> 5];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int off = sw128(lr, (c0 >> 3) + v);
        const uint4 xsv = *reinterpret_cast<const uint4*>(box + off);
        const uint32_t xw[4] = {xsv.x, xsv.y, xsv.z, xsv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * v + 2 * e;
          o[e] = mul_bf16x2(xw[e], cvt_relu_bf16x2(__uint_as_float(r[i]), __uint_as_float(r[i + 1])));
        }
        *reinterpret_cast<uint4*>(box + off) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    return true;
  }
  __device__ static void epilogue_after(const Params& p, const Tile& tl, int row, int part,
                                        uint8_t* epi, EpiState& st) {
    uint8_t* box = epi + slot_warp(row, part) * kWarpStage + (st.iter % kSlots) * kBox;
    fence_async_smem();
    __syncwarp();
    if ((row & 31) == 0) {
      const int t0 = tl.tb * 128 + (row & ~31);
      const int n = tl.nb * 128 + part * 64;
      if (t0 < p.T && n < p.N)
        tma_store_4d_hint(&p.xy_map, box, n, tl.h, t0, tl.b, l2_policy_evict_first());
      bulk_commit();
    }
    ++st.iter;
  }
  __device__ static void epilogue_end(const Params&, int row, int, uint8_t*, EpiState&) {
    if ((row & 31) == 0) bulk_wait_all();
    __syncwarp();
  }
};

// ------------------------------------------------------------ gate, xs recomputed ----
// xy = bf16(relu(bf16(x enc_h)) * relu(bf16(y_h encv_h))) for one 128 x 128 tile: the tile's
// k-blocks [0, kbs) accumulate y encv into TMEM columns 0..127 and [kbs, 2 kbs) accumulate
// x enc into columns 128..255 (kSubAcc), both weight blocks resident for the chunk of row
// blocks. The x enc product repeats the encode kernel's MMAs on the same operands in the same
// order, so xs is bit-identical to the encoder's, and it never crosses HBM: the encode then
// writes qr only, halving its stores, and the gate reads no latent at all.
template <int STAGES, bool KW = false>
struct GateXProb : ChunkedResidentWalkT<8> {
  using S = TcShape<2, 128, false, !KW, 1, 1, STAGES>;
  static constexpr int kCustomEpilogue = 1;
  static constexpr int kEpiWarps = 8;
  static constexpr int kSubAcc = 2;
  using Params = GateXParams;
  using Tile = LatentTile;
  // The xy slice of this thread (its row, 64 columns as eight 16-byte chunks) between the
  // TMEM drain and the stores, which follow the accumulator's release.
  struct EpiState {
    uint4 c[8];
  };
  __device__ static int num_tiles(const Params& p) { return p.B * p.H * p.tb_n * p.nb_n; }
  __device__ static Tile tile(const Params& p, int t) { return latent_tile_chunked(t, p); }
  __device__ static const FastDiv& walk_chunk(const Params& p) { return p.fd_chunk; }
  __device__ static int b_key(const Params& p, const Tile& tl) { return tl.h * p.nb_n + tl.nb; }
  __device__ static int k_blocks(const Params& p, const Tile&) { return 2 * p.kbs; }
  __device__ static int sub_k_blocks(const Params& p, const Tile&) { return p.kbs; }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map);
    tma_prefetch_desc(&p.a2_map);
    tma_prefetch_desc(&p.b_map);
    tma_prefetch_desc(&p.b2_map);
  }
  __device__ static void load_b(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                uint8_t* dst) {
    const uint64_t keep = l2_policy_evict_last();
    const CUtensorMap* m = kb < p.kbs ? &p.b_map : &p.b2_map;
    const int k = (kb < p.kbs ? kb : kb - p.kbs) * 64;
    if (KW) {
      tma_load_4d_hint(m, bar, dst, k, tl.nb * 128, tl.h, 0, keep);
      return;
    }
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d_hint(m, bar, dst + c * 64 * 128, tl.nb * 128 + c * 64, k, tl.h, 0, keep);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t*) {
    const uint64_t keep = l2_policy_evict_last();
    if (kb < p.kbs)
      tma_load_4d_hint(&p.a_map, bar, a_dst, kb * 64, tl.tb * 128, tl.h, tl.b, keep);
    else
      tma_load_4d_hint(&p.a2_map, bar, a_dst, (kb - p.kbs) * 64, tl.tb * 128, tl.b, 0, keep);
  }
  __device__ static void epilogue_begin(const Params&, int, int, uint8_t*, EpiState&, bool,
                                        const Tile&) {}
  __device__ static void epilogue_prefetch(const Params&, const Tile&, bool, const Tile&, int, int,
                                           uint8_t*, EpiState&) {}
  __device__ static bool epilogue_tile(const Params&, const Tile&, int, int part, uint32_t taddr,
                                       uint8_t*, EpiState& st, volatile int*) {
    // all four loads in flight before the one wait
    uint32_t ry2[2][32], rx2[2][32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      tmem_ld32(taddr + static_cast<uint32_t>(part * 64 + 32 * h), ry2[h]);
      tmem_ld32(taddr + static_cast<uint32_t>(128 + part * 64 + 32 * h), rx2[h]);
    }
    tmem_ld_wait();
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      const uint32_t(&ry)[32] = ry2[c0 >> 5];
      const uint32_t(&rx)[32] = rx2[c0 >> 5];
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * v + 2 * e;
          o[e] = mul_bf16x2(cvt_relu_bf16x2(__uint_as_float(rx[i]), __uint_as_float(rx[i + 1])),
                            cvt_relu_bf16x2(__uint_as_float(ry[i]), __uint_as_float(ry[i + 1])));
        }
        st.c[(c0 >> 3) + v] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    return true;
  }
  // After the release: lane (g, j) of the warp stores chunk j of tile rows 8g..8g+7 of its
  // 32-row quadrant, so every 8 lanes write one contiguous 128-byte row segment.
  __device__ static void epilogue_after(const Params& p, const Tile& tl, int row, int part,
                                        uint8_t*, EpiState& st) {
    store_xy_rows(p.xy, p.xy_sb, p.xy_st, p.xy_sh, p.T, p.N, tl.b, tl.h,
                  tl.tb * 128 + (row & ~31), tl.nb * 128 + part * 64, row & 31, st.c);
  }
  __device__ static void epilogue_end(const Params&, int, int, uint8_t*, EpiState&) {}
};

// Pipeline forms. Default: weights resident per column block, chunked walk, six 16 KB
// activation stages (Encode / Gate; EncodeK / GateK read d-contiguous weights K-major).
// The streamed-operand forms (both operands through the stage ring; contiguous walk for
// encode, column-fastest strided walk for gate) serve D > 256, the encode of small batches
// (encode_streamed) and BDH_SM100_LATENT_VARIANT=1.
using Encode = EncodeProb<6, 1, 3>;
using EncodeK = EncodeProb<6, 1, 3, true>;
using EncodeS = EncodeProb<5, 1, 0>;
using EncodeSK = EncodeProb<5, 1, 0, true>;
using Gate = GateProb<6, 2, 3>;
using GateK = GateProb<6, 2, 3, true>;
using GateS = GateProb<5, 2, 1>;
using GateSK = GateProb<5, 2, 1, true>;
// qr-only encode (two staging buffers per warp in the room xs used) and the fused gate
using EncodeQ = EncodeProb<6, 2, 3, false, false>;
using EncodeQK = EncodeProb<6, 2, 3, true, false>;
using EncodeSQ = EncodeProb<5, 2, 0, false, false>;
using EncodeSQK = EncodeProb<5, 2, 0, true, false>;
using GateX = GateXProb<6>;
using GateXK = GateXProb<6, true>;

// Row blocks per chunk of the chunked walk: the largest divisor of the row-block count <= 32.
// Row blocks per chunk of the chunked walk: the largest divisor of row_blocks up to 32 that
// still leaves at least six chunks per SM (chunks = row_blocks / c x column blocks), so that the
// last round of chunks is a small share of a CTA's work; long chunks keep the resident weights
// of a column block for more tiles. Config 2 (128 row blocks, 256 column blocks): 32; B = 4:
// 4 instead of 16 (1024 chunks on 148 SMs instead of 256).
int walk_chunk_for(int64_t row_blocks, int64_t col_blocks) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t want = 6 * static_cast<int64_t>(sm_count(dev));
  for (int c = 32; c > 1; --c)
    if (row_blocks % c == 0 && (row_blocks / c) * col_blocks >= want) return c;
  return 1;
}

// Chunk starts rotated across the row chunk (BDH_SM100_WALK_ROT=1). Off by default: with every
// chunk walking its row blocks in order, the CTAs of one row chunk write the same rows at one
// time, and the config-2 encode measured 0.422 against 0.433 ms per launch alone (B200).
bool walk_rotate() {
  static const bool on = [] {
    const char* e = std::getenv("BDH_SM100_WALK_ROT");
    return e != nullptr && std::atoi(e) == 1;
  }();
  return on;
}

// BDH_SM100_LATENT_VARIANT: 1 forces the streamed-operand forms, 0 the resident-weight forms;
// unset (-1): the encode picks by shape (encode_streamed).
int latent_variant() {
  static int v = [] {
    const char* e = std::getenv("BDH_SM100_LATENT_VARIANT");
    return e ? std::atoi(e) : -1;
  }();
  return v;
}

// The encode streams both operands when the chunked walk would reload the resident weights
// every few tiles: with fewer than 16 row blocks per chunk (a small batch, e.g. one rank's share
// of a strongly scaled batch). Measured on B200 at config-2 layer shapes, per 6-layer step:
// B = 4 0.46 against 0.56 ms, B = 8 0.78 against 0.84 ms; at B = 32 (32-row-block chunks) the
// resident weights are faster.
bool encode_streamed(int walk_chunk) {
  const int v = latent_variant();
  if (v == 1) return true;
  if (v == 0) return false;
  return walk_chunk < 16;
}

bool map_x_btd(CUtensorMap* m, const void* x, const int64_t s[3], int64_t B, int64_t T, int64_t D,
               const char* what) {
  const int64_t dims[4] = {D, T, B, 1};
  const int64_t st[3] = {s[1] * 2, s[0] * 2, 16};
  return make_map_4d(m, x, 2, dims, st, 64, 128, what);
}
bool map_bhtd(CUtensorMap* m, const void* y, const int64_t s[4], int64_t B, int64_t H, int64_t T,
              int64_t D, const char* what) {
  const int64_t dims[4] = {D, T, H, B};
  const int64_t st[3] = {s[2] * 2, s[1] * 2, s[0] * 2};
  return make_map_4d(m, y, 2, dims, st, 64, 128, what);
}
// Weights (H, D, N) with either n contiguous (s[2] == 1, read MN-major in 64 x 64 boxes) or d
// contiguous (s[1] == 1, a transposed copy read K-major in 64 (k) x 128 (n) boxes).
bool weight_k_major(const int64_t s[3]) { return s[1] == 1 && s[2] != 1; }
bool map_weight(CUtensorMap* m, const void* w, const int64_t s[3], int64_t H, int64_t D, int64_t N,
                const char* what) {
  if (weight_k_major(s)) {
    const int64_t dims[4] = {D, N, H, 1};
    const int64_t st[3] = {s[2] * 2, s[0] * 2, 16};
    return make_map_4d(m, w, 2, dims, st, 64, 128, what);
  }
  const int64_t dims[4] = {N, D, H, 1};
  const int64_t st[3] = {s[1] * 2, s[0] * 2, 16};
  return make_map_4d(m, w, 2, dims, st, 64, 64, what);
}
// (B, T, H, N) latent viewed as {N, H, T, B}; box 64 columns x 32 positions of one head.
bool map_bthn(CUtensorMap* m, const void* p, const int64_t s[4], int64_t B, int64_t T, int64_t H,
              int64_t N, const char* what) {
  const int64_t dims[4] = {N, H, T, B};
  const int64_t st[3] = {s[2] * 2, s[1] * 2, s[0] * 2};
  const int box[4] = {64, 1, 32, 1};
  return make_map_4d_box(m, p, 2, dims, st, box, what);
}
// (B, H, T, N) viewed as {N, T, H, B}; box 64 columns x 32 positions.
bool map_bhtn_store(CUtensorMap* m, const void* p, const int64_t s[4], int64_t B, int64_t H,
                    int64_t T, int64_t N, const char* what) {
  const int64_t dims[4] = {N, T, H, B};
  const int64_t st[3] = {s[2] * 2, s[1] * 2, s[0] * 2};
  return make_map_4d(m, p, 2, dims, st, 64, 32, what);
}

}  // namespace

int launch_latent_encode(const LatentArgs& a, cudaStream_t stream, int* err) {
  EncodeParams prm{};
  if (!map_x_btd(&prm.a_map, a.x, a.x_strides, a.B, a.T, a.D, "latent_encode: x")) return BDH_ERR_INVALID;
  if (!map_weight(&prm.b_map, a.w, a.w_strides, a.H, a.D, a.N, "latent_encode: enc")) return BDH_ERR_INVALID;
  const bool wx = a.xs != nullptr;
  if (wx && !map_bthn(&prm.xs_map, a.xs, a.xs_strides, a.B, a.T, a.H, a.N, "latent_encode: xs"))
    return BDH_ERR_INVALID;
  if (!map_bhtn_store(&prm.qr_map, a.qr, a.qr_strides, a.B, a.H, a.T, a.N, "latent_encode: qr"))
    return BDH_ERR_INVALID;
  prm.freqs = a.freqs;
  prm.B = static_cast<int>(a.B);
  prm.T = static_cast<int>(a.T);
  prm.H = static_cast<int>(a.H);
  prm.D = static_cast<int>(a.D);
  prm.N = static_cast<int>(a.N);
  prm.pos0 = static_cast<int>(a.pos0);
  prm.tb_n = static_cast<int>((a.T + 127) / 128);
  prm.nb_n = static_cast<int>((a.N + 127) / 128);
  prm.walk_chunk = walk_chunk_for(a.B * int64_t(prm.tb_n), int64_t(prm.H) * prm.nb_n);
  prm.fd_chunk = FastDiv(static_cast<uint32_t>(prm.walk_chunk));
  prm.walk_rot = walk_rotate() ? 1 : 0;
  prm.fd_ncb = FastDiv(static_cast<uint32_t>(prm.H * prm.nb_n));
  prm.fd_b = FastDiv(static_cast<uint32_t>(prm.B));
  prm.fd_nb = FastDiv(static_cast<uint32_t>(prm.nb_n));
  prm.err = err;
  const int64_t ntiles = a.B * a.H * int64_t(prm.tb_n) * prm.nb_n;
  const bool kw = weight_k_major(a.w_strides);
  const int nt = static_cast<int>(ntiles);
  if (a.D > 256 || encode_streamed(prm.walk_chunk)) {  // resident weights hold D <= 256
    if (!wx)
      return kw ? launch_tc<EncodeSQK::S, EncodeSQK>(prm, nt, stream, kProfEncode)
                : launch_tc<EncodeSQ::S, EncodeSQ>(prm, nt, stream, kProfEncode);
    return kw ? launch_tc<EncodeSK::S, EncodeSK>(prm, nt, stream, kProfEncode)
              : launch_tc<EncodeS::S, EncodeS>(prm, nt, stream, kProfEncode);
  }
  if (!wx)
    return kw ? launch_tc<EncodeQK::S, EncodeQK>(prm, nt, stream, kProfEncode)
              : launch_tc<EncodeQ::S, EncodeQ>(prm, nt, stream, kProfEncode);
  if (kw) return launch_tc<EncodeK::S, EncodeK>(prm, nt, stream, kProfEncode);
  return launch_tc<Encode::S, Encode>(prm, nt, stream, kProfEncode);
}

int launch_latent_gate_x(const LatentArgs& a, cudaStream_t stream, int* err) {
  GateXParams prm{};
  if (a.D > 256) {
    set_error("latent_gate_x: D must be at most 256 (both weight blocks stay resident)");
    return BDH_ERR_INVALID;
  }
  if (weight_k_major(a.w_strides) != weight_k_major(a.w2_strides)) {
    set_error("latent_gate_x: enc and encv must have the same layout (n or d contiguous)");
    return BDH_ERR_INVALID;
  }
  if (!map_bhtd(&prm.a_map, a.y, a.y_strides, a.B, a.H, a.T, a.D, "latent_gate_x: y")) return BDH_ERR_INVALID;
  if (!map_x_btd(&prm.a2_map, a.x, a.x_strides, a.B, a.T, a.D, "latent_gate_x: x")) return BDH_ERR_INVALID;
  if (!map_weight(&prm.b_map, a.w, a.w_strides, a.H, a.D, a.N, "latent_gate_x: encv")) return BDH_ERR_INVALID;
  if (!map_weight(&prm.b2_map, a.w2, a.w2_strides, a.H, a.D, a.N, "latent_gate_x: enc")) return BDH_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a.xy) & 15u) != 0) {
    set_error("latent_gate_x: xy must be 16-byte aligned");
    return BDH_ERR_INVALID;
  }
  prm.xy = static_cast<uint16_t*>(a.xy);
  prm.xy_sb = a.xy_strides[0];
  prm.xy_st = a.xy_strides[1];
  prm.xy_sh = a.xy_strides[2];
  prm.B = static_cast<int>(a.B);
  prm.T = static_cast<int>(a.T);
  prm.H = static_cast<int>(a.H);
  prm.D = static_cast<int>(a.D);
  prm.N = static_cast<int>(a.N);
  prm.tb_n = static_cast<int>((a.T + 127) / 128);
  prm.nb_n = static_cast<int>((a.N + 127) / 128);
  prm.kbs = static_cast<int>((a.D + 63) / 64);
  prm.walk_chunk = walk_chunk_for(a.B * int64_t(prm.tb_n), int64_t(prm.H) * prm.nb_n);
  prm.fd_chunk = FastDiv(static_cast<uint32_t>(prm.walk_chunk));
  prm.walk_rot = walk_rotate() ? 1 : 0;
  prm.fd_ncb = FastDiv(static_cast<uint32_t>(prm.H * prm.nb_n));
  prm.fd_b = FastDiv(static_cast<uint32_t>(prm.B));
  prm.fd_nb = FastDiv(static_cast<uint32_t>(prm.nb_n));
  prm.err = err;
  const int nt = static_cast<int>(a.B * a.H * int64_t(prm.tb_n) * prm.nb_n);
  if (weight_k_major(a.w_strides)) return launch_tc<GateXK::S, GateXK>(prm, nt, stream, kProfGate);
  return launch_tc<GateX::S, GateX>(prm, nt, stream, kProfGate);
}

int launch_latent_gate(const LatentArgs& a, cudaStream_t stream, int* err) {
  GateParams prm{};
  if (!map_bhtd(&prm.a_map, a.y, a.y_strides, a.B, a.H, a.T, a.D, "latent_gate: y")) return BDH_ERR_INVALID;
  if (!map_weight(&prm.b_map, a.w, a.w_strides, a.H, a.D, a.N, "latent_gate: encv")) return BDH_ERR_INVALID;
  if (!map_bthn(&prm.xs_map, a.xs, a.xs_strides, a.B, a.T, a.H, a.N, "latent_gate: xs"))
    return BDH_ERR_INVALID;
  if (!map_bthn(&prm.xy_map, a.xy, a.xy_strides, a.B, a.T, a.H, a.N, "latent_gate: xy"))
    return BDH_ERR_INVALID;
  prm.B = static_cast<int>(a.B);
  prm.T = static_cast<int>(a.T);
  prm.H = static_cast<int>(a.H);
  prm.D = static_cast<int>(a.D);
  prm.N = static_cast<int>(a.N);
  prm.tb_n = static_cast<int>((a.T + 127) / 128);
  prm.nb_n = static_cast<int>((a.N + 127) / 128);
  prm.walk_chunk = walk_chunk_for(a.B * int64_t(prm.tb_n), int64_t(prm.H) * prm.nb_n);
  prm.fd_chunk = FastDiv(static_cast<uint32_t>(prm.walk_chunk));
  prm.walk_rot = walk_rotate() ? 1 : 0;
  prm.fd_ncb = FastDiv(static_cast<uint32_t>(prm.H * prm.nb_n));
  prm.fd_b = FastDiv(static_cast<uint32_t>(prm.B));
  prm.fd_nb = FastDiv(static_cast<uint32_t>(prm.nb_n));
  prm.err = err;
  const int64_t ntiles = a.B * a.H * int64_t(prm.tb_n) * prm.nb_n;
  const bool kw = weight_k_major(a.w_strides);
  if (a.D > 256 || latent_variant() == 1)
    return kw ? launch_tc<GateSK::S, GateSK>(prm, static_cast<int>(ntiles), stream, kProfGate)
              : launch_tc<GateS::S, GateS>(prm, static_cast<int>(ntiles), stream, kProfGate);
  if (kw)
    return launch_tc<GateK::S, GateK>(prm, static_cast<int>(ntiles), stream, kProfGate);
  return launch_tc<Gate::S, Gate>(prm, static_cast<int>(ntiles), stream, kProfGate);
}

}  // namespace bdh

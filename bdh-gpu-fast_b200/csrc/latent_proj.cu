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

// ------------------------------------------------------------------------ encode ----
struct EncodeProb {
  using S = TcShape<2, 128, false, true, 1, 1, 3>;
  static constexpr int kCustomEpilogue = 1;
  static constexpr int kContiguousTiles = 1;
  static constexpr int kBox = 32 * 128;           // one 64-column x 32-row swizzled box
  static constexpr int kBuf = 4 * kBox;           // xs (2 boxes) + qr (2 boxes)
  static constexpr int kWarpStage = 2 * kBuf;     // double buffered
  static constexpr int kEpiSmemBytes = 4 * kWarpStage;
  struct Params {
    CUtensorMap a_map;   // x (B,T,D): box 64 (k) x 128 (t)
    CUtensorMap b_map;   // enc (H,D,N) read MN-major: box 64 (n) x 64 (k)
    CUtensorMap xs_map;  // xs (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1
    CUtensorMap qr_map;  // qr (B,H,T,N) as {N,T,H,B}: box 64 x 32 x 1 x 1
    const float* freqs;
    int B, T, H, D, N, pos0;
    int tb_n, nb_n;
    int* err;
  };
  using Tile = LatentTile;
  struct EpiState {
    float c[64], s[64];
    int key;   // tb * nb_n + nb of the cached phases
    int iter;  // tiles finished by this thread (selects the staging buffer)
  };
  __device__ static int num_tiles(const Params& p) { return p.B * p.H * p.tb_n * p.nb_n; }
  __device__ static Tile tile(const Params& p, int t) { return latent_tile(t, p.B, p.H, p.nb_n); }
  __device__ static int k_blocks(const Params& p, const Tile&) { return (p.D + 63) / 64; }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map);
    tma_prefetch_desc(&p.b_map);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    tma_load_4d(&p.a_map, bar, a_dst, kb * 64, tl.tb * 128, tl.b, 0);
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d(&p.b_map, bar, b_dst + c * 64 * 128, tl.nb * 128 + c * 64, kb * 64, tl.h, 0);
  }

  __device__ static void epilogue_begin(const Params&, int, uint8_t*, EpiState& st, bool,
                                        const Tile&) {
    st.key = -1;
    st.iter = 0;
  }
  // (cos, sin) of this thread's row for the tile's 64 column pairs, when they changed.
  __device__ static void epilogue_prefetch(const Params& p, const Tile& tl, bool, const Tile&,
                                           int row, uint8_t*, EpiState& st) {
    const int key = tl.tb * p.nb_n + tl.nb;
    if (key == st.key) return;
    st.key = key;
    const float pos = static_cast<float>(p.pos0 + tl.tb * 128 + row);
    const int n0 = tl.nb * 128;
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      const int n = n0 + 2 * q;
      const float f = n < p.N ? __ldg(p.freqs + n) : 0.0f;
      rope_cis(pos, f, st.c[q], st.s[q]);
    }
  }
  __device__ static bool epilogue_tile(const Params&, const Tile&, int row, uint32_t taddr,
                                       uint8_t* epi, EpiState& st, volatile int*) {
    const int quad = row >> 5, lr = row & 31;
    uint8_t* buf = epi + quad * kWarpStage + (st.iter & 1) * kBuf;
    // the stores that last read this buffer were committed two tiles ago
    if (lr == 0) bulk_wait_read<1>();
    __syncwarp();
#pragma unroll
    for (int c0 = 0; c0 < 128; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + static_cast<uint32_t>(c0), r);
      tmem_ld_wait();
      uint8_t* xs_box = buf + (c0 >> 6) * kBox;
      uint8_t* qr_box = buf + (2 + (c0 >> 6)) * kBox;
      const int j0 = (c0 & 63) >> 3;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        uint32_t xw[4], qw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * v + 2 * e;
          const int q = (c0 >> 1) + 4 * v + e;
          xw[e] = cvt_bf16x2(fmaxf(__uint_as_float(r[i]), 0.0f), fmaxf(__uint_as_float(r[i + 1]), 0.0f));
          qw[e] = rotate_pair_bf16x2(bf16x2_lo(xw[e]), bf16x2_hi(xw[e]), st.c[q], st.s[q], st.c[q],
                                     st.s[q]);
        }
        const int off = sw128(lr, j0 + v);
        *reinterpret_cast<uint4*>(xs_box + off) = make_uint4(xw[0], xw[1], xw[2], xw[3]);
        *reinterpret_cast<uint4*>(qr_box + off) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
      }
    }
    return true;
  }
  __device__ static void epilogue_after(const Params& p, const Tile& tl, int row, uint8_t* epi,
                                        EpiState& st) {
    const int quad = row >> 5;
    uint8_t* buf = epi + quad * kWarpStage + (st.iter & 1) * kBuf;
    fence_async_smem();
    __syncwarp();
    const int t0 = tl.tb * 128 + quad * 32;
    if ((row & 31) == 0 && t0 < p.T) {
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int n = tl.nb * 128 + hb * 64;
        if (n < p.N) {
          tma_store_4d(&p.xs_map, buf + hb * kBox, n, tl.h, t0, tl.b);
          tma_store_4d(&p.qr_map, buf + (2 + hb) * kBox, n, t0, tl.h, tl.b);
        }
      }
    }
    if ((row & 31) == 0) bulk_commit();  // one group per tile (possibly empty)
    ++st.iter;
  }
  __device__ static void epilogue_end(const Params&, int row, uint8_t*, EpiState&) {
    if ((row & 31) == 0) bulk_wait_all();
    __syncwarp();
  }
};

// -------------------------------------------------------------------------- gate ----
struct GateProb {
  using S = TcShape<2, 128, false, true, 1, 1, 3>;
  static constexpr int kCustomEpilogue = 1;
  static constexpr int kContiguousTiles = 1;
  static constexpr int kBox = 32 * 128;
  static constexpr int kBuf = 2 * kBox;           // one 32 x 128 slice: xs in, xy out in place
  static constexpr int kSlots = 3;                // load one tile ahead while the previous
                                                  // tile's stores may still read their slot
  static constexpr int kWarpStage = kSlots * kBuf;
  static constexpr int kBarOff = 4 * kWarpStage;  // kSlots mbarriers per warp after the buffers
  static constexpr int kEpiSmemBytes = kBarOff + 1024;
  struct Params {
    CUtensorMap a_map;   // y (B,H,T,D): box 64 (k) x 128 (t)
    CUtensorMap b_map;   // encv (H,D,N) read MN-major: box 64 (n) x 64 (k)
    CUtensorMap xs_map;  // xs (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1 (load)
    CUtensorMap xy_map;  // xy (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1 (store)
    int B, T, H, D, N;
    int tb_n, nb_n;
    int* err;
  };
  using Tile = LatentTile;
  struct EpiState {
    int iter;     // tiles finished by this thread
    int loaded;   // tiles whose xs slice load was issued
  };
  __device__ static int num_tiles(const Params& p) { return p.B * p.H * p.tb_n * p.nb_n; }
  __device__ static Tile tile(const Params& p, int t) { return latent_tile(t, p.B, p.H, p.nb_n); }
  __device__ static int k_blocks(const Params& p, const Tile&) { return (p.D + 63) / 64; }
  __device__ static uint32_t pair_mask(const Params&, const Tile&, int) { return 0x1u; }
  __device__ static void prefetch(const Params& p) {
    tma_prefetch_desc(&p.a_map);
    tma_prefetch_desc(&p.b_map);
    tma_prefetch_desc(&p.xs_map);
  }
  __device__ static void load_stage(const Params& p, const Tile& tl, int kb, uint64_t* bar,
                                    uint8_t* a_dst, uint8_t* b_dst) {
    tma_load_4d(&p.a_map, bar, a_dst, kb * 64, tl.tb * 128, tl.h, tl.b);
#pragma unroll
    for (int c = 0; c < 2; ++c)
      tma_load_4d(&p.b_map, bar, b_dst + c * 64 * 128, tl.nb * 128 + c * 64, kb * 64, tl.h, 0);
  }

  __device__ static uint64_t* bar(uint8_t* epi, int quad, int slot) {
    return reinterpret_cast<uint64_t*>(epi + kBarOff) + quad * kSlots + slot;
  }
  // Load the xs slice of tile number `st.loaded` (of this CTA's walk) into its slot.
  __device__ static void load_xs(const Params& p, const Tile& tl, int row, uint8_t* epi,
                                 EpiState& st) {
    const int quad = row >> 5;
    const int slot = st.loaded % kSlots;
    if ((row & 31) == 0) {
      // the slot was last read by the stores of tile (loaded - kSlots); at most the
      // kSlots - 2 most recent store groups may still be reading
      bulk_wait_read<kSlots - 2>();
      uint64_t* b = bar(epi, quad, slot);
      uint8_t* buf = epi + quad * kWarpStage + slot * kBuf;
      const int t0 = tl.tb * 128 + quad * 32;
      if (t0 < p.T) {
        mbar_arrive_expect_tx(b, 2 * kBox);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb)
          tma_load_4d(&p.xs_map, b, buf + hb * kBox, tl.nb * 128 + hb * 64, tl.h, t0, tl.b);
      } else {
        mbar_arrive(b);
      }
    }
    __syncwarp();
    ++st.loaded;
  }
  __device__ static void epilogue_begin(const Params& p, int row, uint8_t* epi, EpiState& st,
                                        bool has_first, const Tile& first) {
    if ((row & 31) == 0) {
      for (int i = 0; i < kSlots; ++i) mbar_init(bar(epi, row >> 5, i), 1);
      fence_mbar_init();
    }
    __syncwarp();
    st.iter = 0;
    st.loaded = 0;
    if (has_first) load_xs(p, first, row, epi, st);
  }
  // One tile ahead: the next tile's xs slice is requested before this tile is drained.
  __device__ static void epilogue_prefetch(const Params& p, const Tile&, bool has_next,
                                           const Tile& next, int row, uint8_t* epi, EpiState& st) {
    if (has_next) load_xs(p, next, row, epi, st);
  }
  __device__ static bool epilogue_tile(const Params& p, const Tile&, int row, uint32_t taddr,
                                       uint8_t* epi, EpiState& st, volatile int* abort_flag) {
    const int quad = row >> 5, lr = row & 31;
    const int slot = st.iter % kSlots;
    uint8_t* buf = epi + quad * kWarpStage + slot * kBuf;
    const uint32_t parity = static_cast<uint32_t>(st.iter / kSlots) & 1u;
    if (!wait_bounded(bar(epi, quad, slot), parity, abort_flag, p.err, kErrTimeoutEpilogue))
      return false;
#pragma unroll
    for (int c0 = 0; c0 < 128; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + static_cast<uint32_t>(c0), r);
      tmem_ld_wait();
      uint8_t* box = buf + (c0 >> 6) * kBox;
      const int j0 = (c0 & 63) >> 3;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int off = sw128(lr, j0 + v);
        const uint4 xsv = *reinterpret_cast<const uint4*>(box + off);
        const uint32_t xw[4] = {xsv.x, xsv.y, xsv.z, xsv.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 8 * v + 2 * e;
          const uint32_t yw =
              cvt_bf16x2(fmaxf(__uint_as_float(r[i]), 0.0f), fmaxf(__uint_as_float(r[i + 1]), 0.0f));
          o[e] = cvt_bf16x2(__fmul_rn(bf16x2_lo(xw[e]), bf16x2_lo(yw)),
                            __fmul_rn(bf16x2_hi(xw[e]), bf16x2_hi(yw)));
        }
        *reinterpret_cast<uint4*>(box + off) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    return true;
  }
  __device__ static void epilogue_after(const Params& p, const Tile& tl, int row, uint8_t* epi,
                                        EpiState& st) {
    const int quad = row >> 5;
    uint8_t* buf = epi + quad * kWarpStage + (st.iter % kSlots) * kBuf;
    fence_async_smem();
    __syncwarp();
    const int t0 = tl.tb * 128 + quad * 32;
    if ((row & 31) == 0) {
      if (t0 < p.T) {
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int n = tl.nb * 128 + hb * 64;
          if (n < p.N) tma_store_4d(&p.xy_map, buf + hb * kBox, n, tl.h, t0, tl.b);
        }
      }
      bulk_commit();
    }
    ++st.iter;
  }
  __device__ static void epilogue_end(const Params&, int row, uint8_t*, EpiState&) {
    if ((row & 31) == 0) bulk_wait_all();
    __syncwarp();
  }
};

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
bool map_weight(CUtensorMap* m, const void* w, const int64_t s[3], int64_t H, int64_t D, int64_t N,
                const char* what) {
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
  EncodeProb::Params prm{};
  if (!map_x_btd(&prm.a_map, a.x, a.x_strides, a.B, a.T, a.D, "latent_encode: x")) return BDH_ERR_INVALID;
  if (!map_weight(&prm.b_map, a.w, a.w_strides, a.H, a.D, a.N, "latent_encode: enc")) return BDH_ERR_INVALID;
  if (!map_bthn(&prm.xs_map, a.xs, a.xs_strides, a.B, a.T, a.H, a.N, "latent_encode: xs"))
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
  prm.err = err;
  const int64_t ntiles = a.B * a.H * int64_t(prm.tb_n) * prm.nb_n;
  return launch_tc<EncodeProb::S, EncodeProb>(prm, static_cast<int>(ntiles), stream, kProfEncode);
}

int launch_latent_gate(const LatentArgs& a, cudaStream_t stream, int* err) {
  GateProb::Params prm{};
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
  prm.err = err;
  const int64_t ntiles = a.B * a.H * int64_t(prm.tb_n) * prm.nb_n;
  return launch_tc<GateProb::S, GateProb>(prm, static_cast<int>(ntiles), stream, kProfGate);
}

}  // namespace bdh

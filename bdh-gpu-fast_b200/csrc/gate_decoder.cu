// Fused post-attention MLP tail of a BDH layer (bdh.py:914-945 and the decoder product of
// bdh.py:1050):
//
//   y_mlp[b,t,:] = bf16( sum_{h,n} xy[b,t,h,n] dec[h N + n, :] ),
//   xy[b,t,h,n]  = bf16( xs[b,t,h,n] * relu(bf16( y[b,h,t,:] . encv[h,:,n] )) )
//
// with xy formed tile by tile in shared memory and consumed there by the decoder product, so
// the (B, T, H, N) xy latent never crosses HBM (the unfused path writes it once and reads it
// back: 2 x B T H N x 2 bytes per layer).
//
// One CTA pair (cta_group::2) owns 256 rows (two 128-row blocks of one batch) and walks every
// (head h, 128-column latent block nb) in order:
//   gate    : G = y[rows, h] (K = D = 256, resident per head) x encv[h, :, nb]  -> TMEM, M 256 N 128
//   epilogue: xy = bf16(xs * relu(bf16(G))), xs TMA-loaded two blocks ahead per 32-row x
//             64-column slice into one of three slots that then holds xy, in place: the K-major
//             128B-swizzled layout of the next product's A operand
//   decoder : Y += xy (K = 128) x decT[:, h N + nb]                            -> TMEM, M 256 N 256
// and at the end of its rows writes Y (each CTA its 128 rows x 256 columns) as bf16.
//
// Roles per CTA (cluster of 2, rank 0 = leader), as in tc_pair_engine.cuh:
//   warp 0     : TMA producer in both CTAs (y per head, encv and decT k-blocks in the order the
//                MMAs consume them); completions land on the leader's barriers.
//   warp 1     : TMEM allocation (512 columns: two gate accumulators + the decoder
//                accumulator); the leader's elected lane issues both MMA chains and commits to
//                the barriers of both CTAs.
//   warps 2..9 : epilogue in both CTAs, two warps per TMEM lane quadrant (64 gate columns and
//                128 output columns each); releases go to the leader with cluster-scope arrives.
// Every wait is bounded (an abort flag and the device error word as in the other engines).
//
// Few rows (B T / 256 row pairs well below the number of CTA pairs, e.g. a small batch, or one
// rank's share of a strongly scaled batch): with a workspace, each row pair's latent walk is cut
// into `split` equal ranges run by different pairs; each writes its fp32 decoder sums, and a
// second kernel adds the ranges in order and rounds once to bf16 (deterministic).
#include <algorithm>
#include <string>

#include "bdh_sm100.h"
#include "common.cuh"
#include "internal.h"
#include "tma_host.h"
#include "tc_pair_engine.cuh"

namespace bdh {

namespace {

constexpr int kGdEpiWarps = 8;
constexpr int kGdThreads = 64 + 32 * kGdEpiWarps;
constexpr int kGdD = 256;        // embedding width (gate K, decoder N)
constexpr int kGdYBytes = 4 * 128 * 128;  // y: four 64-wide k-blocks of this CTA's 128 rows
constexpr int kGdEvStage = 64 * 128;      // encv k-block: this CTA's 64 latent columns x 64 k
constexpr int kGdDtStage = 128 * 128;     // decT k-block: this CTA's 128 output columns x 64 k
constexpr int kGdXySlot = 2 * 128 * 128;  // xy: two 64-wide k-blocks of 128 rows
constexpr int kGdXySlots = 3;  // xs lands two blocks ahead of the one being formed
constexpr uint32_t kGdIdescGate = make_idesc(1u, 0u, 0u, 256, 128);
constexpr uint32_t kGdIdescDec = make_idesc(1u, 0u, 0u, 256, 256);

struct GateDecParams {
  CUtensorMap y_map;   // y (B,H,T,D) as {D,T,H,B}: box 64 (k) x 128 (t)
  CUtensorMap ev_map;  // encv, d contiguous, as {D,N,H,1}: box 64 (k) x 64 (n)
  CUtensorMap xs_map;  // xs (B,T,H,N) as {N,H,T,B}: box 64 x 1 x 32 x 1
  CUtensorMap dt_map;  // decoder^T, latent contiguous, as {H N, D, 1, 1}: box 64 (k) x 128 (d)
  uint16_t* out;       // y_mlp (B,T,D) bf16, element strides out_sb, out_st (d contiguous)
  int64_t out_sb, out_st;
  int B, T, H, N;
  int tb_n, tbp_n, nb_n;  // 128-row blocks, row-block pairs per batch; 128-column blocks per head
  int split, jper;        // latent ranges per row pair and blocks per range (split divides H nb_n)
  float* part;            // split > 1: fp32 sums [split][B][tbp_n * 256][256]
  int* err;
};

template <int ES, int DS>
struct GdLayout {
  static constexpr int Y = 0;
  static constexpr int EV = Y + kGdYBytes;
  static constexpr int DT = EV + ES * kGdEvStage;
  static constexpr int XY = DT + DS * kGdDtStage;
  static constexpr int BAR = XY + kGdXySlots * kGdXySlot;
  // barriers: y_full, y_empty, ev_full[ES], ev_empty[ES], dt_full[DS], dt_empty[DS], gfull[2],
  // gempty[2], xy_ready[3], xy_free[3], xs_full[3][8], dfull, dempty, drain
  static constexpr int NBAR = 2 + 2 * ES + 2 * DS + 4 + 2 * kGdXySlots + kGdXySlots * kGdEpiWarps + 3;
  static constexpr int BYTES = BAR + NBAR * 8 + 16;
  static constexpr int SMEM = BYTES + 1024;  // alignment slack
  static_assert(SMEM <= 232448, "shared memory budget");
};

struct GdBars {
  uint64_t *y_full, *y_empty, *ev_full, *ev_empty, *dt_full, *dt_empty, *gfull, *gempty, *xy_ready,
      *xy_free, *xs_full, *dfull, *dempty, *drain;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

template <int ES, int DS>
__device__ __forceinline__ GdBars gd_bars(uint8_t* smem) {
  using L = GdLayout<ES, DS>;
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + L::BAR);
  GdBars r;
  r.y_full = b;
  r.y_empty = b + 1;
  r.ev_full = b + 2;
  r.ev_empty = r.ev_full + ES;
  r.dt_full = r.ev_empty + ES;
  r.dt_empty = r.dt_full + DS;
  r.gfull = r.dt_empty + DS;
  r.gempty = r.gfull + 2;
  r.xy_ready = r.gempty + 2;
  r.xy_free = r.xy_ready + kGdXySlots;
  r.xs_full = r.xy_free + kGdXySlots;  // [slot][warp]
  r.dfull = r.xs_full + kGdXySlots * kGdEpiWarps;
  r.dempty = r.dfull + 1;
  r.drain = r.dempty + 1;
  r.tmem_slot = reinterpret_cast<uint32_t*>(r.drain + 1);
  r.abort_flag = reinterpret_cast<volatile int*>(r.tmem_slot + 1);
  return r;
}

// Work item = one row-block pair of one batch: (b, tbp), rows (2 tbp + rank) * 128 + [0, 128).
struct GdItem {
  int b, t0;  // this CTA's first row
};
__device__ __forceinline__ GdItem gd_item(const GateDecParams& p, int item, uint32_t rank) {
  GdItem it;
  it.b = item / p.tbp_n;
  const int tbp = item - it.b * p.tbp_n;
  it.t0 = (2 * tbp + static_cast<int>(rank)) * 128;
  return it;
}

// Named barrier 1 over the eight epilogue warps.
__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kGdEpiWarps) : "memory");
}

// Latent block (h * nb_n + nb) visited at step j of an item's walk: every item walks the blocks
// in order, so the decoder sums run over the latent index in ascending order, as a single-pass
// GEMM over K = H N does (measured: bit-identical to cuBLAS's bf16 GEMM on the config-2
// shapes). Starting the walks of different items at different blocks, so that concurrent pairs
// read different weight blocks, changes the summation order and was measured no faster inside
// the config-2 step (2.71-2.75 ms of gate + decoder per 6-layer step, against 2.68-2.70).
__device__ __forceinline__ int gd_walk(const GateDecParams&, int, int j, int) { return j; }

template <int ES, int DS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGdThreads, 1)
    gate_dec_kernel(const __grid_constant__ GateDecParams prm) {
  using L = GdLayout<ES, DS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const GdBars br = gd_bars<ES, DS>(smem);
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int nitems = prm.B * prm.tbp_n * prm.split;  // (row pair, latent range) items
  const int J = prm.H * prm.nb_n;  // latent blocks per row pair

  if (threadIdx.x == 0) {
    mbar_init(br.y_full, 1);
    mbar_init(br.y_empty, 1);
    for (int s = 0; s < ES; ++s) {
      mbar_init(br.ev_full + s, 1);
      mbar_init(br.ev_empty + s, 1);
    }
    for (int s = 0; s < DS; ++s) {
      mbar_init(br.dt_full + s, 1);
      mbar_init(br.dt_empty + s, 1);
    }
    // epilogue releases: gempty one arrive per epilogue warp of both CTAs, xy_ready one per CTA
    for (int a = 0; a < 2; ++a) {
      mbar_init(br.gfull + a, 1);
      mbar_init(br.gempty + a, 2 * kGdEpiWarps);
    }
    for (int a = 0; a < kGdXySlots; ++a) {
      mbar_init(br.xy_ready + a, 2);
      mbar_init(br.xy_free + a, 1);
      for (int w = 0; w < kGdEpiWarps; ++w) mbar_init(br.xs_full + a * kGdEpiWarps + w, 1);
    }
    mbar_init(br.dfull, 1);
    mbar_init(br.dempty, 2 * kGdEpiWarps);
    mbar_init(br.drain, 1);
    *br.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(br.tmem_slot, 512);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised and TMEM allocated before any use
  tc_fence_after();
  const uint32_t tmem = *br.tmem_slot;
  // the set-up above touches shared memory and TMEM only: with a programmatic launch it overlaps
  // the previous kernel's tail
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one()) {
      tma_prefetch_desc(&prm.y_map);
      tma_prefetch_desc(&prm.ev_map);
      tma_prefetch_desc(&prm.dt_map);
      const uint32_t yfull_l = mapa_shared(smem_u32(br.y_full), 0);
      const uint32_t evfull_l = mapa_shared(smem_u32(br.ev_full), 0);
      const uint32_t dtfull_l = mapa_shared(smem_u32(br.dt_full), 0);
      int es = 0, ds = 0, hc = 0;
      uint32_t eph = 0, dph = 0;
      bool ok = true;
      auto load_dt = [&](int item, int j) -> bool {
        const int jj = gd_walk(prm, item, j, J);
        const int h = jj / prm.nb_n, nb = jj - (jj / prm.nb_n) * prm.nb_n;
        for (int kb = 0; kb < 2; ++kb) {
          if (*br.abort_flag || !wait_bounded(br.dt_empty + ds, dph ^ 1u, br.abort_flag, prm.err,
                                              kErrTimeoutProducer))
            return false;
          if (leader) mbar_arrive_expect_tx(br.dt_full + ds, 2 * kGdDtStage);
          tma_load_4d_pair(&prm.dt_map, dtfull_l + ds * 8u, smem + L::DT + ds * kGdDtStage,
                           h * prm.N + nb * 128 + kb * 64, static_cast<int>(rank) * 128, 0, 0);
          if (++ds == DS) {
            ds = 0;
            dph ^= 1u;
          }
        }
        return true;
      };
      for (int item = pair; item < nitems && ok; item += npairs) {
        const int ri = item / prm.split;
        const int jlo = (item - ri * prm.split) * prm.jper, jhi = jlo + prm.jper;
        const GdItem it = gd_item(prm, ri, rank);
        for (int j = jlo; j < jhi && ok; ++j) {
          const int jj = gd_walk(prm, item, j, J);
          const int h = jj / prm.nb_n, nb = jj - (jj / prm.nb_n) * prm.nb_n;
          if (j == jlo || nb == 0) {  // a new head: its y rows (resident for its latent blocks)
            if (*br.abort_flag || !wait_bounded(br.y_empty, static_cast<uint32_t>(hc & 1) ^ 1u,
                                                br.abort_flag, prm.err, kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(br.y_full, 2 * kGdYBytes);
            for (int kb = 0; kb < 4; ++kb)
              tma_load_4d_pair(&prm.y_map, yfull_l, smem + L::Y + kb * 128 * 128, kb * 64, it.t0,
                               h, it.b);
            ++hc;
          }
          for (int kb = 0; kb < 4; ++kb) {
            if (*br.abort_flag || !wait_bounded(br.ev_empty + es, eph ^ 1u, br.abort_flag, prm.err,
                                                kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            if (leader) mbar_arrive_expect_tx(br.ev_full + es, 2 * kGdEvStage);
            tma_load_4d_pair(&prm.ev_map, evfull_l + es * 8u, smem + L::EV + es * kGdEvStage,
                             kb * 64, nb * 128 + static_cast<int>(rank) * 64, h, 0);
            if (++es == ES) {
              es = 0;
              eph ^= 1u;
            }
          }
          if (ok && j > jlo) ok = load_dt(item, j - 1);
        }
        if (ok) ok = load_dt(item, jhi - 1);
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer (leader)
    if (leader && elect_one()) {
      const uint32_t base = smem_u32(smem);
      const uint32_t own = 0, peer = 1;
      auto both = [&](uint64_t* bar) {
        umma_commit_pair(mapa_shared(smem_u32(bar), own));
        umma_commit_pair(mapa_shared(smem_u32(bar), peer));
      };
      int es = 0, ds = 0, hc = 0, ic = 0, g = 0;
      uint32_t eph = 0, dph = 0;
      bool ok = true;
      auto dec = [&](int gg, bool first) -> bool {
        const int s = gg % kGdXySlots;
        if (!wait_bounded(br.xy_ready + s, static_cast<uint32_t>(gg / kGdXySlots) & 1u,
                          br.abort_flag, prm.err, kErrTimeoutMma))
          return false;
        if (first && !wait_bounded(br.dempty, static_cast<uint32_t>(ic & 1) ^ 1u, br.abort_flag,
                                   prm.err, kErrTimeoutMma))
          return false;
        tc_fence_after();
        for (int kb = 0; kb < 2; ++kb) {
          if (!wait_bounded(br.dt_full + ds, dph, br.abort_flag, prm.err, kErrTimeoutMma))
            return false;
          tc_fence_after();
          const uint32_t a_addr = base + L::XY + s * kGdXySlot + kb * 128 * 128;
          const uint32_t b_addr = base + L::DT + ds * kGdDtStage;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_pair(tmem + 256u, smem_desc_sw128(a_addr + kk * 32, 16, 1024),
                          smem_desc_sw128(b_addr + kk * 32, 16, 1024), kGdIdescDec,
                          (first && kb == 0 && kk == 0) ? 0u : 1u);
          both(br.dt_empty + ds);
          if (++ds == DS) {
            ds = 0;
            dph ^= 1u;
          }
        }
        both(br.xy_free + s);
        return true;
      };
      for (int item = pair; item < nitems && ok; item += npairs) {
        const int jlo = (item - (item / prm.split) * prm.split) * prm.jper, jhi = jlo + prm.jper;
        for (int j = jlo; j < jhi && ok; ++j) {
          const int jj = gd_walk(prm, item, j, J);
          const int nb = jj - (jj / prm.nb_n) * prm.nb_n;
          if (j == jlo || nb == 0) {
            if (!wait_bounded(br.y_full, static_cast<uint32_t>(hc & 1), br.abort_flag, prm.err,
                              kErrTimeoutMma)) {
              ok = false;
              break;
            }
            ++hc;
          }
          const int s = g & 1;
          if (!wait_bounded(br.gempty + s, (static_cast<uint32_t>(g >> 1) & 1u) ^ 1u, br.abort_flag,
                            prm.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kb = 0; kb < 4 && ok; ++kb) {
            if (!wait_bounded(br.ev_full + es, eph, br.abort_flag, prm.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = base + L::Y + kb * 128 * 128;
            const uint32_t b_addr = base + L::EV + es * kGdEvStage;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_pair(tmem + static_cast<uint32_t>(s * 128),
                            smem_desc_sw128(a_addr + kk * 32, 16, 1024),
                            smem_desc_sw128(b_addr + kk * 32, 16, 1024), kGdIdescGate,
                            (kb > 0 || kk > 0) ? 1u : 0u);
            both(br.ev_empty + es);
            if (++es == ES) {
              es = 0;
              eph ^= 1u;
            }
          }
          if (!ok) break;
          both(br.gfull + s);
          if (nb == prm.nb_n - 1 || j == jhi - 1) both(br.y_empty);  // the head's gate MMAs issued
          if (j > jlo && !dec(g - 1, j == jlo + 1)) {
            ok = false;
            break;
          }
          ++g;
        }
        if (!ok) break;
        if (!dec(g - 1, prm.jper == 1)) break;
        both(br.dfull);
        ++ic;
      }
      umma_commit_pair(mapa_shared(smem_u32(br.drain), 0));
      wait_drain(br.drain, 0u, prm.err);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int w = warp - 2;
    const int quad = warp & 3;
    const int part = w >> 2;  // gate columns part*64.., output columns part*128..
    const int lr = static_cast<int>(lane_id());
    const int row = quad * 32 + lr;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t gempty_l = mapa_shared(smem_u32(br.gempty), 0);
    const uint32_t ready_l = mapa_shared(smem_u32(br.xy_ready), 0);
    const uint32_t dempty_l = mapa_shared(smem_u32(br.dempty), 0);
    const int my_items = pair < nitems ? (nitems - 1 - pair) / npairs + 1 : 0;
    const int total = my_items * prm.jper;
    // xs slice of latent block gg (this CTA's walk) into slot gg % 3 (lane 0 issues)
    auto issue_xs = [&](int gg) -> bool {
      bool ok = true;
      if (lr == 0) {
        const int s = gg % kGdXySlots;
        if (gg >= kGdXySlots)  // the decoder MMAs of block gg - 3 have read this slot
          ok = wait_bounded(br.xy_free + s,
                            (static_cast<uint32_t>(gg / kGdXySlots) & 1u) ^ 1u, br.abort_flag,
                            prm.err, kErrTimeoutEpilogue);
        if (ok) {
          const int item = pair + (gg / prm.jper) * npairs;
          const int ri = item / prm.split;
          const GdItem it = gd_item(prm, ri, rank);
          const int jj = gd_walk(prm, item,
                                 (item - ri * prm.split) * prm.jper + gg - (gg / prm.jper) * prm.jper, J);
          const int h = jj / prm.nb_n, nb = jj - (jj / prm.nb_n) * prm.nb_n;
          uint64_t* bar = br.xs_full + s * kGdEpiWarps + w;
          mbar_arrive_expect_tx(bar, 32 * 128);
          tma_load_4d_hint(&prm.xs_map, bar,
                           smem + L::XY + s * kGdXySlot + part * 128 * 128 + quad * 32 * 128,
                           nb * 128 + part * 64, h, it.t0 + quad * 32, it.b,
                           l2_policy_evict_first());
        }
      }
      return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    };
    bool ok = true;
    for (int gg = 0; gg < 2 && gg < total && ok; ++gg) ok = issue_xs(gg);
    int g = 0;
    for (int k = 0; k < my_items && ok; ++k) {
      const int item = pair + k * npairs;
      const int ri = item / prm.split;
      const int rs = item - ri * prm.split;  // latent range of a split row pair
      const GdItem it = gd_item(prm, ri, rank);
      for (int j = 0; j < prm.jper; ++j, ++g) {
        const int s = g % kGdXySlots;  // xs / xy slot
        const int a = g & 1;           // gate accumulator
        const bool okw = wait_bounded(br.xs_full + s * kGdEpiWarps + w,
                                      static_cast<uint32_t>(g / kGdXySlots) & 1u, br.abort_flag,
                                      prm.err, kErrTimeoutEpilogue) &&
                         wait_bounded(br.gfull + a, static_cast<uint32_t>(g >> 1) & 1u,
                                      br.abort_flag, prm.err, kErrTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, okw)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* box = smem + L::XY + s * kGdXySlot + part * 128 * 128 + quad * 32 * 128;
        uint32_t rr[2][32];
        tmem_ld32(lane_base + static_cast<uint32_t>(a * 128 + part * 64), rr[0]);
        tmem_ld32(lane_base + static_cast<uint32_t>(a * 128 + part * 64 + 32), rr[1]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        // a release at cluster scope here cost ~1 us per block; the CTA-scope form suffices
        if (lr == 0) mbar_arrive_remote(gempty_l + a * 8u);
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 32) {
          const uint32_t(&r)[32] = rr[c0 >> 5];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int off = lr * 128 + ((((c0 >> 3) + v) ^ (lr & 7)) << 4);
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
        fence_async_smem();  // xy is read by the tensor cores (async proxy)
        // all eight epilogue warps have written their xy slices; one release per CTA
        epi_bar_sync();
        if (w == 0 && lr == 0) mbar_arrive_remote(ready_l + s * 8u);
        // two blocks ahead: its slot held block g - 1, whose decoder MMAs are then in flight
        if (g + 2 < total && !issue_xs(g + 2)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      // the item's decoder sums: this thread's row, output columns part*128 .. +127
      const bool okd = wait_bounded(br.dfull, static_cast<uint32_t>(k & 1), br.abort_flag, prm.err,
                                    kErrTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, okd)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int t = it.t0 + row;
      uint16_t* orow = prm.out + it.b * prm.out_sb + static_cast<int64_t>(t) * prm.out_st + part * 128;
      float* prow = prm.split > 1
                        ? prm.part + ((static_cast<int64_t>(rs) * prm.B + it.b) * (prm.tbp_n * 256) + t) * kGdD +
                              part * 128
                        : nullptr;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + static_cast<uint32_t>(256 + part * 128 + c), r);
        tmem_ld_wait();
        if (prow != nullptr) {  // this range's fp32 sums (the reduce kernel adds the ranges)
          if (t < prm.T) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<uint4*>(prow + c + 4 * q) =
                  make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
        } else if (t < prm.T) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(orow + c + 8 * q) =
                make_uint4(cvt_bf16x2(__uint_as_float(r[8 * q]), __uint_as_float(r[8 * q + 1])),
                           cvt_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                           cvt_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                           cvt_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lr == 0) mbar_arrive_remote(dempty_l);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs (reading both CTAs' shared memory) have drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// out[b, t, :] = bf16(sum over the ranges s = 0 .. split-1 of part[s][b][t][:]), in that order:
// 32 threads per row, eight columns each.
__global__ void __launch_bounds__(256) gate_dec_reduce_kernel(const float* __restrict__ part,
                                                              uint16_t* __restrict__ out,
                                                              int64_t out_sb, int64_t out_st, int B,
                                                              int T, int tpad, int split) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(B) * T) return;
  const int b = static_cast<int>(row / T), t = static_cast<int>(row - static_cast<int64_t>(b) * T);
  const int c = (threadIdx.x & 31) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < split; ++s) {
    const float4* p = reinterpret_cast<const float4*>(
        part + ((static_cast<int64_t>(s) * B + b) * tpad + t) * kGdD + c);
    const float4 u = __ldcs(p), v = __ldcs(p + 1);
    acc[0] += u.x; acc[1] += u.y; acc[2] += u.z; acc[3] += u.w;
    acc[4] += v.x; acc[5] += v.y; acc[6] += v.z; acc[7] += v.w;
  }
  *reinterpret_cast<uint4*>(out + b * out_sb + static_cast<int64_t>(t) * out_st + c) =
      make_uint4(cvt_bf16x2(acc[0], acc[1]), cvt_bf16x2(acc[2], acc[3]), cvt_bf16x2(acc[4], acc[5]),
                 cvt_bf16x2(acc[6], acc[7]));
}

constexpr int kGdES = 4;
constexpr int kGdDS = 2;
constexpr int kGdSplitMax = 16;

// CTA pairs of the gate + decoder kernel that fit on the current device at once.
int gate_dec_pairs() {
  using L = GdLayout<kGdES, kGdDS>;
  auto kern = gate_dec_kernel<kGdES, kGdDS>;
  int dev = 0;
  cudaGetDevice(&dev);
  static int max_pairs[64] = {0};
  if (dev >= 0 && dev < 64 && max_pairs[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute (gate_dec): ") + cudaGetErrorString(e));
      return -BDH_ERR_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(kGdThreads);
    cfg.dynamicSmemBytes = L::SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count(dev) / 2;
    }
    max_pairs[dev] = n;
  }
  return max_pairs[(dev >= 0 && dev < 64) ? dev : 0];
}

// Latent ranges per row pair: 1, or the largest power of two (at most kGdSplitMax, dividing
// the H * N / 128 latent blocks) that keeps the split row pairs within one wave of CTA pairs,
// when the row pairs fill at most half of them.
int gate_dec_split(int64_t B, int64_t T, int64_t H, int64_t N, int pairs) {
  const int64_t rows = B * ((T + 255) / 256);
  const int64_t J = H * (N / 128);
  if (rows <= 0 || pairs <= 0 || 2 * rows > pairs) return 1;
  int split = 1;
  while (split * 2 <= kGdSplitMax && rows * split * 2 <= pairs && J % (split * 2) == 0) split *= 2;
  return split;
}

size_t gate_dec_part_bytes(int64_t B, int64_t T, int split) {
  return split > 1 ? static_cast<size_t>(split) * B * ((T + 255) / 256) * 256 * kGdD * sizeof(float) : 0;
}

}  // namespace

size_t latent_gate_dec_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D, int64_t N) {
  if (D != kGdD || N % 128 != 0 || B * T == 0 || H * N == 0) return 0;
  const int pairs = gate_dec_pairs();
  if (pairs <= 0) return 0;
  return gate_dec_part_bytes(B, T, gate_dec_split(B, T, H, N, pairs));
}

int launch_latent_gate_dec(const GateDecArgs& a, cudaStream_t stream, int* err) {
  if (a.D != kGdD || a.N % 128 != 0) {
    set_error("latent_gate_dec: needs D = 256 and N a multiple of 128");
    return BDH_ERR_INVALID;
  }
  GateDecParams prm{};
  {
    const int64_t dims[4] = {a.D, a.T, a.H, a.B};
    const int64_t st[3] = {a.y_strides[2] * 2, a.y_strides[1] * 2, a.y_strides[0] * 2};
    if (!make_map_4d(&prm.y_map, a.y, 2, dims, st, 64, 128, "latent_gate_dec: y")) return BDH_ERR_INVALID;
  }
  {
    const int64_t dims[4] = {a.D, a.N, a.H, 1};
    const int64_t st[3] = {a.encv_strides[2] * 2, a.encv_strides[0] * 2, 16};
    if (!make_map_4d(&prm.ev_map, a.encv, 2, dims, st, 64, 64, "latent_gate_dec: encv")) return BDH_ERR_INVALID;
  }
  {
    const int64_t dims[4] = {a.N, a.H, a.T, a.B};
    const int64_t st[3] = {a.xs_strides[2] * 2, a.xs_strides[1] * 2, a.xs_strides[0] * 2};
    const int box[4] = {64, 1, 32, 1};
    if (!make_map_4d_box(&prm.xs_map, a.xs, 2, dims, st, box, "latent_gate_dec: xs")) return BDH_ERR_INVALID;
  }
  {
    const int64_t dims[4] = {a.H * a.N, a.D, 1, 1};
    const int64_t st[3] = {a.dec_strides[1] * 2, 16, 16};
    if (!make_map_4d(&prm.dt_map, a.dec, 2, dims, st, 64, 128, "latent_gate_dec: decoder")) return BDH_ERR_INVALID;
  }
  prm.out = static_cast<uint16_t*>(a.out);
  prm.out_sb = a.out_strides[0];
  prm.out_st = a.out_strides[1];
  prm.B = static_cast<int>(a.B);
  prm.T = static_cast<int>(a.T);
  prm.H = static_cast<int>(a.H);
  prm.N = static_cast<int>(a.N);
  prm.tb_n = static_cast<int>((a.T + 127) / 128);
  prm.tbp_n = (prm.tb_n + 1) / 2;
  prm.nb_n = static_cast<int>(a.N / 128);
  prm.err = err;
  const int rows = prm.B * prm.tbp_n;
  if (rows == 0) return BDH_OK;
  using L = GdLayout<kGdES, kGdDS>;
  auto kern = gate_dec_kernel<kGdES, kGdDS>;
  const int cap = gate_dec_pairs();
  if (cap < 0) return -cap;
  int split = gate_dec_split(a.B, a.T, a.H, a.N, cap);
  if (split > 1 && (a.workspace == nullptr || a.workspace_bytes < gate_dec_part_bytes(a.B, a.T, split)))
    split = 1;  // no room for the range sums: one range per row pair
  prm.split = split;
  prm.jper = static_cast<int>(a.H) * prm.nb_n / split;
  prm.part = split > 1 ? static_cast<float*>(a.workspace) : nullptr;
  const int nitems = rows * split;
  const int pairs = std::min(nitems, cap);
  prof_start(kProfGate, stream);
  cudaError_t le = launch_pdl(kern, dim3(2 * pairs), dim3(kGdThreads), L::SMEM, stream, prm);
  if (le != cudaSuccess) {
    prof_stop(kProfGate, stream);
    set_error(std::string("gate_dec_kernel launch: ") + cudaGetErrorString(le));
    return BDH_ERR_CUDA;
  }
  if (split > 1) {
    const int64_t nrow = a.B * a.T;
    gate_dec_reduce_kernel<<<static_cast<unsigned>((nrow + 7) / 8), 256, 0, stream>>>(
        prm.part, prm.out, prm.out_sb, prm.out_st, prm.B, prm.T, prm.tbp_n * 256, split);
  }
  prof_stop(kProfGate, stream);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("gate_dec_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return BDH_OK;
}

}  // namespace bdh

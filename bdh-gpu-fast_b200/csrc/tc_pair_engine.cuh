// CTA-pair (tcgen05 cta_group::2) variant of the persistent GEMM engine.
//
// Why: a 128 x 128 single-CTA tile needs ~122 bytes of operands per SM per clock at full MMA
// rate (a 128 x 256 tile ~91), above what the L2 -> shared-memory path sustains per SM; the
// tensor pipe then idles ~45% (~30%) of the time. A CTA pair computes a 256 x 256 tile with
// one MMA stream: each CTA stages only its own 128 rows of A and 128 rows of B (~61 B/clk/SM),
// and each MMA instruction covers twice the tensor time, which also relaxes the issue loop.
//
// Roles per CTA (cluster of 2, rank 0 = leader):
//   warp 0     : TMA producer in both CTAs. Each loads its own halves into its own shared memory;
//                the transfers complete on the LEADER's full barrier (2-CTA TMA form). Only the
//                leader posts the expected byte count (both halves).
//   warp 1     : TMEM allocation (pair-wide) in both CTAs; the leader's elected lane issues the
//                MMAs (M = 256, N = 256) and commits to the barriers of both CTAs (one commit
//                per CTA; no multicast form is used).
//   warps 2..5 : epilogue in both CTAs: each drains its own TMEM (its 128 rows x 256 columns)
//                and releases the accumulator with one arrive per warp on the leader's barrier
//                (the CTA-scope remote form: a cluster-scope release measured ~1 us each).
// Every wait is bounded exactly as in tc_engine.cuh; both CTAs always meet at the final
// cluster barrier before TMEM is released and the CTAs retire.
#pragma once

#include "tc_engine.cuh"

namespace bdh {

// P::kEpiWarps = 8 -> two epilogue warps per TMEM lane quadrant, each draining one half of the
// tile's columns (more warps to hide the epilogue's latency); default four.
template <class P>
constexpr int pair_threads() {
  return 64 + 32 * EpiWarps<P>::value;
}

// P::kEpiScratch > 0: every epilogue warp gets that many bytes of shared memory after the
// barriers, passed to P::epilogue as a last argument (staging for stores that need a transpose).
template <class P, class = void>
struct EpiScratch {
  static constexpr int value = 0;
};
template <class P>
struct EpiScratch<P, std::void_t<decltype(P::kEpiScratch)>> {
  static constexpr int value = P::kEpiScratch;
};
template <class S, class P>
constexpr int pair_smem_bytes() {
  return S::SMEM_BYTES + EpiWarps<P>::value * EpiScratch<P>::value;
}

// P::kVarN: a tile may use fewer accumulator columns than S::BN (a narrower MMA):
// P::tile_idesc(prm, tile) is its instruction descriptor, P::tile_cols(prm, tile) the columns
// the epilogue drains (a multiple of 32, of 64 with eight epilogue warps).
template <class P, class = void>
struct HasVarN : std::false_type {};
template <class P>
struct HasVarN<P, std::void_t<decltype(P::kVarN)>> : std::true_type {};

// P::kBFromA: when P::b_is_a(prm, tile) holds, the tile's B operand is its A operand (a
// diagonal tile of a self product Q Q^T: each CTA's 128 rows of A are also its 128 rows of B),
// so the stages carry A only (P::load_stage loads no B) and the MMAs read B from A's buffer.
template <class P, class = void>
struct HasBFromA : std::false_type {};
template <class P>
struct HasBFromA<P, std::void_t<decltype(P::kBFromA)>> : std::true_type {};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the variable at local shared address `a` inside CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (possibly the peer CTA's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// The same with the default (CTA-scope) release, the form CUTLASS's cluster barriers use for
// their remote arrives; the cluster-scope release above measured ~1 us per arrive.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 4-D tiled TMA load into this CTA's shared memory completing on a barrier of either CTA of
// the pair (cta_group::2 form).
__device__ __forceinline__ void tma_load_4d_pair(const CUtensorMap* map, uint32_t bar_cluster,
                                                 void* dst, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the barrier at `bar_cluster` when all MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

// Shape of one pair tile: M = 256 (128 rows per CTA), N = 256 (128 B-rows per CTA), bf16.
template <bool A_MN_, bool B_MN_, int A_TERMS_, int B_TERMS_, int STAGES_>
struct PairShape {
  static constexpr int ELEM = 2;
  static constexpr int BM = 256;             // pair rows
  static constexpr int BN = 256;             // pair columns = TMEM columns per accumulator
  static constexpr int BK = 64;
  static constexpr int UK = 16;
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr int A_TERMS = A_TERMS_;
  static constexpr int B_TERMS = B_TERMS_;
  static constexpr int STAGES = STAGES_;
  static constexpr int A_TILE = 128 * 128;   // bytes of this CTA's A half, one term
  static constexpr int B_TILE = 128 * 128;   // bytes of this CTA's B half, one term
  static constexpr int STAGE_BYTES = A_TILE * A_TERMS + B_TILE * B_TERMS;  // per CTA
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 256 + 1024;
  static constexpr uint32_t IDESC = make_idesc(1u, A_MN ? 1u : 0u, B_MN ? 1u : 0u, BM, BN);
  static constexpr int NPAIRS = (A_TERMS == 1 && B_TERMS == 1) ? 1 : (A_TERMS == 2 && B_TERMS == 2 ? 3 : 2);
  static_assert(STAGES * STAGE_BYTES + 256 + 1024 <= 232448, "shared memory budget");

  __device__ static __forceinline__ uint32_t a_koff(int kk) {
    return A_MN ? static_cast<uint32_t>(kk * UK * 128) : static_cast<uint32_t>(kk * 32);
  }
  __device__ static __forceinline__ uint32_t b_koff(int kk) {
    return B_MN ? static_cast<uint32_t>(kk * UK * 128) : static_cast<uint32_t>(kk * 32);
  }
  __device__ static __forceinline__ uint64_t a_desc(uint32_t addr) {
    return smem_desc_sw128(addr, A_MN ? BK * 128 : 16, 1024);
  }
  __device__ static __forceinline__ uint64_t b_desc(uint32_t addr) {
    return smem_desc_sw128(addr, B_MN ? BK * 128 : 16, 1024);
  }
};

template <class S, class P>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads<P>(), 1)
    tc_pair_kernel(const __grid_constant__ typename P::Params prm) {
  constexpr int EW = EpiWarps<P>::value;
  static_assert(EW == 4 || EW == 8, "four or eight epilogue warps");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::STAGES * S::STAGE_BYTES);
  uint64_t* empty = full + S::STAGES;
  uint64_t* tfull = empty + S::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int ntiles = P::num_tiles(prm);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 2 * EW);  // one arrive per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised and TMEM allocated before any use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the set-up above touches shared memory and TMEM only: with a programmatic launch it overlaps
  // the previous kernel's tail
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one()) {
      P::prefetch(prm);
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      const uint32_t full_leader0 = mapa_shared(smem_u32(full), 0);
      for (int t = pair; t < ntiles && ok; t += npairs) {
        typename P::Tile tile = P::tile(prm, t);
        const int nkb = P::k_blocks(prm, tile);
        for (int kb = 0; kb < nkb; ++kb) {
          if (*abort_flag ||
              !wait_bounded(empty + stage, ph ^ 1u, abort_flag, prm.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(full + stage, P::stage_tx(prm, tile, kb));
          uint8_t* a_dst = smem + stage * S::STAGE_BYTES;
          uint8_t* b_dst = a_dst + S::A_TERMS * S::A_TILE;
          P::load_stage(prm, tile, kb, rank, full_leader0 + stage * 8u, a_dst, b_dst);
          if (++stage == S::STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer (leader)
    if (leader && elect_one()) {
      const uint32_t base = smem_u32(smem);
      const uint64_t a0 = S::a_desc(base);
      const uint64_t b0_own = S::b_desc(base + S::A_TERMS * S::A_TILE);
      const uint64_t b0_a = S::b_desc(base);  // B read from A's buffer (kBFromA)
      const uint32_t empty_peer = mapa_shared(smem_u32(empty), 1);
      const uint32_t tfull_peer = mapa_shared(smem_u32(tfull), 1);
      const uint32_t empty_own = mapa_shared(smem_u32(empty), 0);
      const uint32_t tfull_own = mapa_shared(smem_u32(tfull), 0);
      int stage = 0;
      uint32_t soff16 = 0;
      uint32_t ph = 0;
      int lt = 0;
      bool ok = true;
      for (int t = pair; t < ntiles && ok; t += npairs, ++lt) {
        typename P::Tile tile = P::tile(prm, t);
        const int nkb = P::k_blocks(prm, tile);
        const int acc = lt & 1;
        const uint32_t aph = static_cast<uint32_t>(lt >> 1) & 1u;
        if (!wait_bounded(tempty + acc, aph ^ 1u, abort_flag, prm.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * S::BN);
        uint32_t idesc = S::IDESC;
        if constexpr (HasVarN<P>::value) idesc = P::tile_idesc(prm, tile);
        uint64_t b0 = b0_own;
        if constexpr (HasBFromA<P>::value) {
          if (P::b_is_a(prm, tile)) b0 = b0_a;
        }
        for (int kb = 0; kb < nkb; ++kb) {
          if (!wait_bounded(full + stage, ph, abort_flag, prm.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pair_mask = P::pair_mask(prm, tile, kb);
#pragma unroll
          for (int kk = 0; kk < S::BK / S::UK; ++kk) {
#pragma unroll
            for (int pr = 0; pr < S::NPAIRS; ++pr) {
              if (!((pair_mask >> pr) & 1u)) continue;
              const int ta = (pr == 1 && S::A_TERMS == 2) ? 1 : 0;
              const int tb = (pr == 2 || (pr == 1 && S::A_TERMS == 1)) ? 1 : 0;
              const uint64_t ad = a0 + (soff16 + ((ta * S::A_TILE + S::a_koff(kk)) >> 4));
              const uint64_t bd = b0 + (soff16 + ((tb * S::B_TILE + S::b_koff(kk)) >> 4));
              umma_f16_pair(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0 || pr > 0) ? 1u : 0u);
            }
          }
          umma_commit_pair(empty_own + stage * 8u);
          umma_commit_pair(empty_peer + stage * 8u);
          if (++stage == S::STAGES) {
            stage = 0;
            soff16 = 0;
            ph ^= 1u;
          } else {
            soff16 += S::STAGE_BYTES >> 4;
          }
        }
        if (!ok) break;
        umma_commit_pair(tfull_own + acc * 8u);
        umma_commit_pair(tfull_peer + acc * 8u);
      }
      umma_commit_pair(mapa_shared(smem_u32(drain), 0));
      wait_drain(drain, 0u, prm.err);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int row = quad * 32 + static_cast<int>(lane_id());
    const int part = (warp - 2) >> 2;  // column half (eight epilogue warps) or 0
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    int lt = 0;
    for (int t = pair; t < ntiles; t += npairs, ++lt) {
      typename P::Tile tile = P::tile(prm, t);
      const int acc = lt & 1;
      const uint32_t aph = static_cast<uint32_t>(lt >> 1) & 1u;
      bool ok = wait_bounded(tfull + acc, aph, abort_flag, prm.err, kErrTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t tbase =
          tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * S::BN);
      int cols = S::BN;
      if constexpr (HasVarN<P>::value) cols = P::tile_cols(prm, tile);
      const int c_begin = EW == 8 ? part * (cols / 2) : 0;
      const int c_end = EW == 8 ? c_begin + cols / 2 : cols;
#pragma unroll 1
      for (int c0 = c_begin; c0 < c_end; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tbase + static_cast<uint32_t>(c0), r);
        tmem_ld_wait();
        if constexpr (EpiScratch<P>::value > 0)
          P::epilogue(prm, tile, static_cast<int>(rank), row, c0, r,
                      smem + S::STAGES * S::STAGE_BYTES + 256 + (warp - 2) * EpiScratch<P>::value);
        else
          P::epilogue(prm, tile, static_cast<int>(rank), row, c0, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane_id() == 0) mbar_arrive_remote(tempty_leader + acc * 8u);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs (reading both CTAs' shared memory) have drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, S::TMEM_COLS);
  }
}

// CTA pairs of this kernel that fit on the current device at once (the persistent grid), or a
// negative BDH error code. Looked up once per device.
template <class S, class P>
static int resident_pairs() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int max_pairs[64] = {0};
  if (dev >= 0 && dev < 64 && max_pairs[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(tc_pair_kernel<S, P>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pair_smem_bytes<S, P>());
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute (pair): ") + cudaGetErrorString(e));
      return -BDH_ERR_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(pair_threads<P>());
    cfg.dynamicSmemBytes = pair_smem_bytes<S, P>();
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, tc_pair_kernel<S, P>, &cfg);
    if (e != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count(dev) / 2;
    }
    max_pairs[dev] = n;
  }
  return max_pairs[(dev >= 0 && dev < 64) ? dev : 0];
}

template <class S, class P>
static int launch_pair(const typename P::Params& prm, int ntiles, cudaStream_t stream, int kind) {
  if (ntiles <= 0) return 0;
  const int cap = resident_pairs<S, P>();
  if (cap < 0) return -cap;
  const int pairs = std::min(ntiles, cap);
  prof_start(kind, stream);
  cudaError_t e = launch_pdl(tc_pair_kernel<S, P>, dim3(2 * pairs), dim3(pair_threads<P>()),
                             pair_smem_bytes<S, P>(), stream, prm);
  prof_stop(kind, stream);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("tc_pair_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return 0;
}

}  // namespace bdh

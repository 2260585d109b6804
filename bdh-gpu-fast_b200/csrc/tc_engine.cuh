// Persistent, warp-specialised tcgen05 GEMM engine for the tril-attention contractions.
//
// One CTA per SM (192 threads) walks a strided list of output tiles:
//   warp 0      : TMA producer (one elected lane) filling a ring of STAGES shared-memory
//                 stages; each stage holds one 128-byte-wide K slice of every operand term.
//   warp 1      : TMEM allocator + MMA issuer (one elected lane); accumulates a 128 x BN
//                 fp32 tile into one of two TMEM buffers (double buffered across tiles).
//   warps 2..5  : epilogue (128 threads = 128 TMEM lanes = 128 tile rows); drains the
//                 accumulator with tcgen05.ld and hands 32-column chunks to the problem's
//                 epilogue (masking, hi/lo splitting, RoPE adjoint, stores).
//
// The problem policy `P` supplies the tile list, the K-block count of each tile, the TMA
// loads of one stage and the epilogue. Operands are 128B-swizzled, either K-major (rows of
// 128 bytes along K) or MN-major (128-byte chunks along M/N, K rows of 128 bytes).
// "Terms" implement split precision: A = sum of A_TERMS tiles, B = sum of B_TERMS tiles, and
// the MMA issues hi*hi (+ hi*lo + lo*hi) products; the lo*lo product is dropped.
#pragma once

#include <type_traits>
#include <utility>

#include "common.cuh"

namespace bdh {

// Optional policy hooks (detected at compile time):
//   P::stage_tx(prm, tile, kb) -> bytes the TMA loads of k-block kb deliver (default: all terms)
//   P::epilogue_chunk(prm, tile, row, ch, nch, c0, r) -> called with the running fp32 sums
//       after every accumulation chunk (KCHUNK > 0), instead of the final P::epilogue.
template <class P, class = void>
struct HasStageTx : std::false_type {};
template <class P>
struct HasStageTx<P, std::void_t<decltype(P::kVarStageTx)>> : std::true_type {};
template <class P, class = void>
struct HasChunkEmit : std::false_type {};
template <class P>
struct HasChunkEmit<P, std::void_t<decltype(P::kEmitEveryChunk)>> : std::true_type {};
//   P::kEpiSmemBytes -> shared memory reserved for the epilogue warps (1024-aligned), passed to
//       P::epilogue_chunk(..., epi) and P::epilogue_end(prm, row, epi) (called once per thread
//       after the tile loop, e.g. to drain bulk stores reading that memory).
//   P::kCustomEpilogue -> the policy drains the accumulator itself (no KCHUNK):
//       P::EpiState st (per epilogue thread, lives across tiles),
//       P::epilogue_begin(prm, row, part, epi, st, has_first, first_tile)  once, before the tiles;
//       P::epilogue_prefetch(prm, tile, has_next, next_tile, row, part, epi, st)
//                                                         before the accumulator is ready;
//       P::epilogue_tile(prm, tile, row, part, taddr, epi, st, abort_flag) -> bool
//                                                         tcgen05.ld of the tile (lane quadrant
//                                                         base `taddr`), all loads waited;
//       P::epilogue_after(prm, tile, row, part, epi, st)  after the TMEM buffer is released;
//       P::epilogue_end(prm, row, part, epi, st)          once, after the last tile.
//   (`row` is the tile row = TMEM lane of the thread, `part` its column half, see kEpiWarps.)
//   P::kContiguousTiles -> CTA i walks the contiguous tile range [i n / G, (i+1) n / G) instead
//       of the strided list i, i + G, ... (consecutive tiles of a CTA then share operands or
//       epilogue state).
template <class P, class = void>
struct HasCustomEpi : std::false_type {};
template <class P>
struct HasCustomEpi<P, std::void_t<decltype(P::kCustomEpilogue)>> : std::true_type {};
template <class P, class = void>
struct HasContigTiles : std::false_type {};
template <class P>
struct HasContigTiles<P, std::void_t<decltype(P::kContiguousTiles)>> : std::true_type {};

//   P::kChunkedWalk + P::walk_chunk(prm) (a FastDiv by the chunk length) -> the tile list is cut
//       into chunks of walk_chunk
//       consecutive tiles; CTA i takes chunks i, i + G, ... and walks each chunk in order (the
//       CTAs running at one time hold neighbouring chunks, each CTA keeps a chunk's operands).
template <class P, class = void>
struct HasChunkedWalk : std::false_type {};
template <class P>
struct HasChunkedWalk<P, std::void_t<decltype(P::kChunkedWalk)>> : std::true_type {};

// Tile walk of this CTA: t = first, next(first), ... while t < end.
struct TileWalk {
  int first, end, step, chunk;  // chunk > 0: chunked walk
  FastDiv fd;                    // division by chunk
  __device__ __forceinline__ int next(int t) const {
    if (chunk > 0) {
      const int u = t + 1;
      return (u - fd.div(u) * chunk != 0) ? u : u + (step - 1) * chunk;
    }
    return t + step;
  }
};
template <class P>
__device__ __forceinline__ TileWalk tile_walk(const typename P::Params& prm, int ntiles) {
  TileWalk w;
  if constexpr (HasChunkedWalk<P>::value) {
    w.fd = P::walk_chunk(prm);
    w.chunk = static_cast<int>(w.fd.d);
    w.first = static_cast<int>(blockIdx.x) * w.chunk;
    w.end = ntiles;
    w.step = static_cast<int>(gridDim.x);
  } else if constexpr (HasContigTiles<P>::value) {
    w.chunk = 0;
    w.first = static_cast<int>(static_cast<long long>(blockIdx.x) * ntiles / gridDim.x);
    w.end = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * ntiles / gridDim.x);
    w.step = 1;
  } else {
    w.chunk = 0;
    w.first = static_cast<int>(blockIdx.x);
    w.end = ntiles;
    w.step = static_cast<int>(gridDim.x);
  }
  return w;
}

//   P::kResidentB = KBR -> the B operand of a tile (all its k-blocks, at most KBR) is kept in a
//       dedicated shared-memory region while consecutive tiles of the CTA share it:
//       P::b_key(prm, tile) identifies it, P::load_b(prm, tile, kb, bar, dst) loads k-block kb;
//       the stage ring then carries only A. Needs B_TERMS == 1.
template <class P, class = void>
struct ResidentB {
  static constexpr int value = 0;
};
template <class P>
struct ResidentB<P, std::void_t<decltype(P::kResidentB)>> {
  static constexpr int value = P::kResidentB;
};

//   P::max_ctas(prm, sm_count) (host) -> cap on the persistent grid (e.g. a multiple of the
//       column-block count, so every CTA of a strided walk keeps one column block).
template <class P, class = void>
struct HasMaxCtas : std::false_type {};
template <class P>
struct HasMaxCtas<P, std::void_t<decltype(P::max_ctas(std::declval<const typename P::Params&>(), 0))>>
    : std::true_type {};

//   P::kAccBuffers = 4 (BN <= 128) -> four TMEM accumulators instead of two, so the MMA issuer
//       can run up to three tiles ahead of the epilogue (short-K tiles otherwise stall on the
//       accumulator hand-back of the tile before last).
template <class P, class = void>
struct AccBufs {
  static constexpr int value = 2;
};
template <class P>
struct AccBufs<P, std::void_t<decltype(P::kAccBuffers)>> {
  static constexpr int value = P::kAccBuffers;
};

//   P::kSubAcc = 2 (no KCHUNK) -> a tile accumulates kSubAcc independent products side by side:
//       k-blocks [i * P::sub_k_blocks(prm, tile), (i + 1) * ...) form product i, accumulated from
//       zero into TMEM columns [i * BN, (i + 1) * BN) of the tile's buffer, so the epilogue sees
//       kSubAcc * BN columns (e.g. two projections of the same rows that it multiplies
//       elementwise).
template <class P, class = void>
struct SubAcc {
  static constexpr int value = 1;
};
template <class P>
struct SubAcc<P, std::void_t<decltype(P::kSubAcc)>> {
  static constexpr int value = P::kSubAcc;
};

template <class P, class = void>
struct EpiSmem {
  static constexpr int value = 0;
};
template <class P>
struct EpiSmem<P, std::void_t<decltype(P::kEpiSmemBytes)>> {
  static constexpr int value = P::kEpiSmemBytes;
};

constexpr int kTcThreads = 192;
constexpr int kEpiThreads = 128;

//   P::kEpiWarps = 8 (custom epilogues, or chunked accumulation) -> two epilogue warps per TMEM
//       lane quadrant, each draining half of the tile's columns (`part` 0 / 1 in the custom
//       hooks; with KCHUNK each keeps BN / 2 running sums and passes its columns' c0 offsets,
//       part * BN / 2 + ..., to P::epilogue_chunk); the CTA then has 64 + 256 threads.
template <class P, class = void>
struct EpiWarps {
  static constexpr int value = 4;
};
template <class P>
struct EpiWarps<P, std::void_t<decltype(P::kEpiWarps)>> {
  static constexpr int value = P::kEpiWarps;
};
template <class P>
constexpr int tc_threads() {
  return 64 + 32 * EpiWarps<P>::value;
}

// KCHUNK_ > 0: the K-loop of a tile is cut into chunks of KCHUNK_ k-blocks, each accumulated in
// its own TMEM buffer and summed by the epilogue in fp32 registers (round-to-nearest). This
// bounds the length of every tensor-core accumulation chain, which matters for the fp32 path:
// one accumulator fed by thousands of MMAs drifted to ~5e-5 relative error at K = 8192 with
// the 3-product tf32 split, above the 1e-5 fp32 tolerance).
template <int ELEM_, int BN_, bool A_MN_, bool B_MN_, int A_TERMS_, int B_TERMS_, int STAGES_,
          int KCHUNK_ = 0>
struct TcShape {
  static constexpr int ELEM = ELEM_;               // operand element bytes: 2 (bf16) or 4 (tf32)
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int BK = 128 / ELEM;            // K elements per stage
  static constexpr int UK = 32 / ELEM;             // K elements per tcgen05.mma
  static constexpr bool A_MN = A_MN_;
  static constexpr bool B_MN = B_MN_;
  static constexpr int A_TERMS = A_TERMS_;
  static constexpr int B_TERMS = B_TERMS_;
  static constexpr int STAGES = STAGES_;
  static constexpr int KCHUNK = KCHUNK_;
  static constexpr int A_TILE = BM * 128;          // bytes of one A term in one stage
  static constexpr int B_TILE = BN * 128;
  static constexpr int STAGE_BYTES = A_TILE * A_TERMS + B_TILE * B_TERMS;
  static constexpr int TMEM_COLS = 2 * BN;         // two fp32 accumulators
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC =
      make_idesc(ELEM == 2 ? 1u : 2u, A_MN ? 1u : 0u, B_MN ? 1u : 0u, BM, BN);
  static constexpr int NPAIRS = (A_TERMS == 1 && B_TERMS == 1) ? 1 : (A_TERMS == 2 && B_TERMS == 2 ? 3 : 2);

  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");
  static_assert(KCHUNK == 0 || BN <= 256, "chunked accumulation keeps the tile's fp32 sums in registers");

  __host__ __device__ static int chunks(int nkb) {
    return KCHUNK == 0 ? 1 : (nkb + KCHUNK - 1) / KCHUNK;
  }

  // Byte offset of the kk-th MMA's K slice inside one term tile.
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

// Bytes of one ring stage (A only when B is resident), of the ring, and of the resident B.
template <class S, class P>
constexpr int tc_stage_bytes() {
  return ResidentB<P>::value > 0 ? S::A_TILE * S::A_TERMS : S::STAGE_BYTES;
}
template <class S, class P>
constexpr int tc_ring_bytes() {
  return S::STAGES * tc_stage_bytes<S, P>() + ResidentB<P>::value * S::B_TILE;
}
// Dynamic shared memory of one CTA: the stage ring (+ resident B), a barrier block, the
// epilogue's own region (if any) and 1 KB of alignment slack.
template <class S, class P>
constexpr int tc_smem_bytes() {
  return EpiSmem<P>::value == 0 && ResidentB<P>::value == 0
             ? S::SMEM_BYTES
             : tc_ring_bytes<S, P>() + 1024 + EpiSmem<P>::value + 1024;
}

// Spin on `bar` ignoring the abort flag (used to drain in-flight async work before exit).
__device__ __forceinline__ bool wait_drain(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u && globaltimer_ns() - t0 > BDH_WAIT_TIMEOUT_NS) {
      if (err != nullptr) atomicCAS(err, 0, kErrTimeoutDrain);
      return false;
    }
  }
}

template <class S, class P>
__global__ void __launch_bounds__(tc_threads<P>(), 1)
    tc_gemm_kernel(const __grid_constant__ typename P::Params prm) {
  static_assert(EpiWarps<P>::value == 4 ||
                    (EpiWarps<P>::value == 8 && (HasCustomEpi<P>::value || S::KCHUNK > 0)),
                "eight epilogue warps need a custom epilogue or chunked accumulation");
  static_assert(S::KCHUNK == 0 || S::BN / (EpiWarps<P>::value / 4) <= 128,
                "at most 128 running sums per epilogue thread");
  static_assert(tc_smem_bytes<S, P>() <= 232448, "shared memory budget");
  static_assert(ResidentB<P>::value == 0 || S::B_TERMS == 1, "resident B holds one term");
  static_assert(S::STAGES <= 8, "barrier block layout (2 x 8 stages + 2 x 4 accumulators + 5)");
  constexpr bool kRes = ResidentB<P>::value > 0;
  constexpr int NACC = AccBufs<P>::value;
  constexpr int NSUB = SubAcc<P>::value;
  constexpr int ACC_COLS = NSUB * S::BN;  // TMEM columns of one tile's accumulator buffer
  static_assert(NACC == 2 || NACC == 4, "two or four accumulator buffers");
  static_assert(NACC * ACC_COLS <= 512, "accumulator buffers exceed the 512 TMEM columns");
  static_assert(NSUB == 1 || S::KCHUNK == 0, "side-by-side products need unchunked accumulation");
  constexpr uint32_t kTmemCols = static_cast<uint32_t>(NACC * ACC_COLS);
  constexpr int SB = tc_stage_bytes<S, P>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* bres = smem + S::STAGES * SB;  // resident B (kRes)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + tc_ring_bytes<S, P>());
  uint64_t* empty = full + S::STAGES;
  uint64_t* tfull = empty + S::STAGES;
  uint64_t* tempty = tfull + NACC;
  uint64_t* drain = tempty + NACC;
  uint64_t* full_b = drain + 1;
  uint64_t* empty_b = full_b + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(empty_b + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int ntiles = P::num_tiles(prm);
  const TileWalk walk = tile_walk<P>(prm, ntiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, 32 * EpiWarps<P>::value);
    }
    mbar_init(drain, 1);
    mbar_init(full_b, 1);
    mbar_init(empty_b, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the set-up above touches shared memory and TMEM only: with a programmatic launch it overlaps
  // the previous kernel's tail
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      P::prefetch(prm);
      int stage = 0;
      uint32_t ph = 0;
      uint32_t n_issued = 0;
      int b_loads = 0;
      int b_key = 0;
      bool ok = true;
      for (int t = walk.first; t < walk.end && ok; t = walk.next(t)) {
        typename P::Tile tile = P::tile(prm, t);
        const int nkb = P::k_blocks(prm, tile);
        if constexpr (kRes) {
          const int key = P::b_key(prm, tile);
          if (b_loads == 0 || key != b_key) {
            // the MMAs that read the previous B must have completed
            if (b_loads > 0 &&
                !wait_bounded(empty_b, static_cast<uint32_t>(b_loads - 1) & 1u, abort_flag, prm.err,
                              kErrTimeoutProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full_b, static_cast<uint32_t>(nkb * S::B_TILE));
            for (int kb = 0; kb < nkb; ++kb) P::load_b(prm, tile, kb, full_b, bres + kb * S::B_TILE);
            ++b_loads;
            b_key = key;
          }
        }
        for (int kb = 0; kb < nkb; ++kb) {
          if (*abort_flag ||
              !wait_bounded(empty + stage, ph ^ 1u, abort_flag, prm.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          uint32_t tx = SB;
          if constexpr (HasStageTx<P>::value) tx = P::stage_tx(prm, tile, kb);
          mbar_arrive_expect_tx(full + stage, tx);
          uint8_t* a_dst = smem + stage * SB;
          uint8_t* b_dst = kRes ? nullptr : a_dst + S::A_TERMS * S::A_TILE;
          P::load_stage(prm, tile, kb, full + stage, a_dst, b_dst);
          ++n_issued;
          if (++stage == S::STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      // Every issued TMA load must land before this CTA may retire its shared memory.
      for (int s = 0; s < S::STAGES; ++s) {
        if (n_issued > static_cast<uint32_t>(s)) {
          const uint32_t k_last = (n_issued - 1u - static_cast<uint32_t>(s)) / S::STAGES;
          wait_drain(full + s, k_last & 1u, prm.err);
        }
      }
      if (kRes && b_loads > 0) wait_drain(full_b, static_cast<uint32_t>(b_loads - 1) & 1u, prm.err);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    // The issue loop is kept lean: at N = 128 one MMA covers only 64 tensor cycles, so every
    // scalar instruction of this thread is on the critical path. Descriptors are built once
    // and advanced by adding the 16-byte-unit offset of each stage / K slice to their low field.
    if (elect_one()) {
      const uint32_t base = smem_u32(smem);
      const uint64_t a0 = S::a_desc(base);
      // ring-relative B (stage offset added) or the resident region (k-block offset added)
      const uint64_t b0 = kRes ? S::b_desc(smem_u32(bres)) : S::b_desc(base + S::A_TERMS * S::A_TILE);
      int stage = 0;
      uint32_t soff16 = 0;  // stage * SB / 16
      uint32_t ph = 0;
      int lc = 0;  // accumulation chunks issued by this CTA (selects the TMEM buffer)
      int b_uses = 0;
      int b_key = 0;
      bool ok = true;
      for (int t = walk.first; t < walk.end && ok; t = walk.next(t)) {
        typename P::Tile tile = P::tile(prm, t);
        const int nkb = P::k_blocks(prm, tile);
        const int nch = S::chunks(nkb);
        if constexpr (kRes) {
          const int key = P::b_key(prm, tile);
          if (b_uses == 0 || key != b_key) {
            if (b_uses > 0) umma_commit(empty_b);  // arrives once the old B's MMAs complete
            if (!wait_bounded(full_b, static_cast<uint32_t>(b_uses) & 1u, abort_flag, prm.err,
                              kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            ++b_uses;
            b_key = key;
          }
        }
        for (int ch = 0; ch < nch && ok; ++ch, ++lc) {
          const int acc = lc % NACC;
          const uint32_t aph = static_cast<uint32_t>(lc / NACC) & 1u;
          if (!wait_bounded(tempty + acc, aph ^ 1u, abort_flag, prm.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * ACC_COLS);
          const int kb0 = S::KCHUNK == 0 ? 0 : ch * S::KCHUNK;
          const int kb1 = S::KCHUNK == 0 ? nkb : min(nkb, kb0 + S::KCHUNK);
          int sub_kbs = 0;  // k-blocks per side-by-side product (NSUB > 1)
          if constexpr (NSUB > 1) sub_kbs = P::sub_k_blocks(prm, tile);
          int in_sub = 0;   // k-blocks already accumulated into the current product
          for (int kb = kb0; kb < kb1; ++kb) {
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
                // pair 0: A0*B0; pair 1: A1*B0 (or A0*B1 when only B is split); pair 2: A0*B1
                const int ta = (pr == 1 && S::A_TERMS == 2) ? 1 : 0;
                const int tb = (pr == 2 || (pr == 1 && S::A_TERMS == 1)) ? 1 : 0;
                const uint64_t ad = a0 + (soff16 + ((ta * S::A_TILE + S::a_koff(kk)) >> 4));
                const uint64_t bd =
                    kRes ? b0 + static_cast<uint32_t>((kb * S::B_TILE + S::b_koff(kk)) >> 4)
                         : b0 + (soff16 + ((tb * S::B_TILE + S::b_koff(kk)) >> 4));
                const bool first_kb = NSUB > 1 ? in_sub == 0 : kb == kb0;
                const uint32_t accumulate = (!first_kb || kk > 0 || pr > 0) ? 1u : 0u;
                if (S::ELEM == 2)
                  umma_f16(d_tmem, ad, bd, S::IDESC, accumulate);
                else
                  umma_tf32(d_tmem, ad, bd, S::IDESC, accumulate);
              }
            }
            umma_commit(empty + stage);
            if constexpr (NSUB > 1) {
              if (++in_sub == sub_kbs) {
                in_sub = 0;
                d_tmem += static_cast<uint32_t>(S::BN);
              }
            }
            if (++stage == S::STAGES) {
              stage = 0;
              soff16 = 0;
              ph ^= 1u;
            } else {
              soff16 += SB >> 4;
            }
          }
          if (!ok) break;
          umma_commit(tfull + acc);
        }
      }
      // All MMAs issued by this thread must finish before TMEM is released.
      umma_commit(drain);
      wait_drain(drain, 0u, prm.err);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + static_cast<int>(lane_id());
    const int part = (warp - 2) >> 2;  // column half (eight epilogue warps) or 0
    uint8_t* epi = smem + tc_ring_bytes<S, P>() + 1024;
    (void)epi;
    int lc = 0;
    bool ok = true;
    if constexpr (HasCustomEpi<P>::value) {
      typename P::EpiState st{};
      P::epilogue_begin(prm, row, part, epi, st, walk.first < walk.end,
                        P::tile(prm, walk.first < walk.end ? walk.first : 0));
      for (int t = walk.first; t < walk.end && ok; t = walk.next(t)) {
        typename P::Tile tile = P::tile(prm, t);
        const int tn = walk.next(t);
        const bool has_next = tn < walk.end;
        P::epilogue_prefetch(prm, tile, has_next, P::tile(prm, has_next ? tn : t), row, part, epi,
                             st);
        const int acc = lc % NACC;
        const uint32_t aph = static_cast<uint32_t>(lc / NACC) & 1u;
        ok = wait_bounded(tfull + acc, aph, abort_flag, prm.err, kErrTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase =
            tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * ACC_COLS);
        ok = P::epilogue_tile(prm, tile, row, part, tbase, epi, st, abort_flag);
        tc_fence_before();
        mbar_arrive(tempty + acc);
        ++lc;
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        P::epilogue_after(prm, tile, row, part, epi, st);
      }
      P::epilogue_end(prm, row, part, epi, st);
    } else {
    for (int t = walk.first; t < walk.end && ok; t = walk.next(t)) {
      typename P::Tile tile = P::tile(prm, t);
      if (S::KCHUNK == 0) {
        const int acc = lc % NACC;
        const uint32_t aph = static_cast<uint32_t>(lc / NACC) & 1u;
        ok = wait_bounded(tfull + acc, aph, abort_flag, prm.err, kErrTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tbase =
            tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * ACC_COLS);
#pragma unroll 1
        for (int c0 = 0; c0 < S::BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + static_cast<uint32_t>(c0), r);
          tmem_ld_wait();
          P::epilogue(prm, tile, row, c0, r);
        }
        tc_fence_before();
        mbar_arrive(tempty + acc);
        ++lc;
      } else {
        // this thread's columns: all BN (four epilogue warps) or one half (eight)
        constexpr int BNC = S::KCHUNK == 0 ? 32 : S::BN / (EpiWarps<P>::value / 4);
        const int col0 = part * BNC;
        float sum[BNC];
#pragma unroll
        for (int i = 0; i < BNC; ++i) sum[i] = 0.0f;
        const int nch = S::chunks(P::k_blocks(prm, tile));
        for (int ch = 0; ch < nch; ++ch, ++lc) {
          const int acc = lc % NACC;
          const uint32_t aph = static_cast<uint32_t>(lc / NACC) & 1u;
          ok = wait_bounded(tfull + acc, aph, abort_flag, prm.err, kErrTimeoutEpilogue);
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tbase =
              tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * ACC_COLS);
          // 16 columns at a time when a thread keeps 128 running sums (register budget)
          constexpr int LDC = BNC > 64 ? 16 : 32;
#pragma unroll
          for (int c0 = 0; c0 < BNC; c0 += LDC) {
            uint32_t r[LDC];
            if constexpr (LDC == 16)
              tmem_ld16(tbase + static_cast<uint32_t>(col0 + c0), r);
            else
              tmem_ld32(tbase + static_cast<uint32_t>(col0 + c0), r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < LDC; ++e) sum[c0 + e] = __fadd_rn(sum[c0 + e], __uint_as_float(r[e]));
          }
          tc_fence_before();
          mbar_arrive(tempty + acc);
          if constexpr (HasChunkEmit<P>::value) {
#pragma unroll
            for (int c0 = 0; c0 < BNC; c0 += 32) {
              uint32_t r[32];
#pragma unroll
              for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(sum[c0 + e]);
              P::epilogue_chunk(prm, tile, row, ch, nch, col0 + c0, r, epi);
            }
          }
        }
        if (!ok) break;
        if constexpr (!HasChunkEmit<P>::value) {
#pragma unroll
          for (int c0 = 0; c0 < BNC; c0 += 32) {
            uint32_t r[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(sum[c0 + e]);
            P::epilogue(prm, tile, row, col0 + c0, r);
          }
        }
      }
    }
    if constexpr (HasChunkEmit<P>::value) P::epilogue_end(prm, row, epi);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace bdh

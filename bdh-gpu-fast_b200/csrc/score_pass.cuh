// The masked score pass shared by forward and backward, and the persistent launcher.
//
//   S[u] = tril(A[u] B[u]^T, -1)   over the lower-triangular 128 x BN tiles of each unit u=(b,h)
//
// with the K-loop over the contraction width (N for Q K^T, D for dO V^T). S is written as an
// exact split pair (bf16 hi + bf16 lo, or tf32 hi + fp32 lo) in one of four layouts:
//   kStoreDirect : S at [u][i][j]                       (forward P)
//   kStoreTrans  : S^T at [u][j][i]                     (backward M^T, the K-major A of dV)
//   kStoreSym    : S + S^T at [u][i][j]                 (backward G = dS + dS^T, K is Q)
//   kStoreLU     : S at out1[u][i][j], S^T at out2      (backward dS / dS^T, K distinct)
// Transposed stores are coalesced across the warp: lanes own consecutive rows i, so for a
// fixed column j the 32 lanes write 32 consecutive elements of row j of the transpose. A null
// lo destination (bf16 only) stores the bf16-rounded scores alone.
#pragma once

#include <algorithm>
#include <string>

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

// fp32 inputs (ELEM 4) accumulate in 256-wide K chunks (see TcShape::KCHUNK).
template <int ELEM, int BN, int STAGES>
struct ScoreProb {
  static constexpr int TERMS = ELEM == 2 ? 1 : 2;
  using S = TcShape<ELEM, BN, false, false, TERMS, TERMS, STAGES, ELEM == 4 ? 8 : 0>;
  struct Params {
    CUtensorMap a_map[2];  // rows i of A (hi, lo), box BK x 128
    CUtensorMap b_map[2];  // rows j of B (hi, lo), box BK x BN
    // CTA-pair pass: the tiles from tail_from on (the last, partial wave of the persistent
    // grid) run as tail_sub narrower tiles of 256 / tail_sub keys each (tail_sub > 1), their
    // B rows loaded through b_nar (box BK x 128 / tail_sub)
    CUtensorMap b_nar;
    int tail_from, tail_sub;
    int self_ab;           // CTA-pair pass: B is A (one tensor, one set of strides, per head)
    int H, T, K;           // heads, sequence length, contraction width
    int b_shared;          // B has a single head shared by all H heads of A
    int mode;              // ScoreStore
    int mt;                // 128-row blocks per unit
    int tiles_per_unit;
    int units;
    void* p_hi;            // [units][T][ldp]
    void* p_lo;
    void* p2_hi;           // kStoreLU: transposed destination
    void* p2_lo;
    int64_t ldp;
    int chunk;             // > 0: keys restricted to the query block's chunk, stored relative
    int ksplit;            // > 1: K-split partial tiles (fp32, direct mode) into part
    int kb_per_split;      // k-blocks per split (a multiple of the accumulation chunk)
    float* part;           // [ksplit][units][T][ldp]
    int* err;
  };
  struct Tile {
    int unit, mi, ni, ks;
  };

  // First key column of row block mi: 0, or the start of its chunk (chunked forward).
  __device__ static int key0(const Params& p, int mi) {
    return p.chunk > 0 ? (mi * S::BM / p.chunk) * p.chunk : 0;
  }
  __device__ static int nt_for(const Params& p, int mi) {
    return ceil_div_d(min(p.T, (mi + 1) * S::BM), BN) - key0(p, mi) / BN;
  }
  __device__ static int num_tiles(const Params& p) { return p.units * p.tiles_per_unit * max(1, p.ksplit); }
  __device__ static Tile tile(const Params& p, int t) {
    Tile tl;
    tl.ks = 0;
    if (p.ksplit > 1) {  // the split index fastest: the splits of a tile run side by side
      tl.ks = t % p.ksplit;
      t /= p.ksplit;
    }
    tl.unit = t / p.tiles_per_unit;
    int r = t - tl.unit * p.tiles_per_unit;
    int mi = 0;
    for (;; ++mi) {
      const int c = nt_for(p, mi);
      if (r < c) break;
      r -= c;
    }
    tl.mi = mi;
    tl.ni = r + key0(p, mi) / BN;
    return tl;
  }
  __device__ static int k_blocks(const Params& p, const Tile& tl) {
    const int total = ceil_div_d(p.K, S::BK);
    if (p.ksplit <= 1) return total;
    return max(0, min(total, (tl.ks + 1) * p.kb_per_split) - tl.ks * p.kb_per_split);
  }
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
    const int hb = p.b_shared ? 0 : h;
    const int kg = kb + (p.ksplit > 1 ? tl.ks * p.kb_per_split : 0);
    for (int i = 0; i < TERMS; ++i) {
      tma_load_4d(&p.a_map[i], bar, a_dst + i * S::A_TILE, kg * S::BK, tl.mi * S::BM, h, b);
      tma_load_4d(&p.b_map[i], bar, b_dst + i * S::B_TILE, kg * S::BK, tl.ni * BN, hb, b);
    }
  }

  // Split x into the stored pair (hi, lo): bf16 bits or tf32/fp32 values.
  __device__ static __forceinline__ void split(float x, uint32_t& hi, uint32_t& lo) {
    if (ELEM == 2) {
      hi = f32_to_bf16_bits(x);
      lo = f32_to_bf16_bits(x - bf16_bits_to_f32(hi));
    } else {
      const float h = tf32_rna(x);
      hi = __float_as_uint(h);
      lo = __float_as_uint(x - h);
    }
  }
  __device__ static __forceinline__ void store1(void* base, size_t idx, uint32_t bits) {
    if (ELEM == 2)
      static_cast<uint16_t*>(base)[idx] = static_cast<uint16_t>(bits);
    else
      static_cast<uint32_t*>(base)[idx] = bits;
  }

  // Transposed store S^T[j][i] of one warp's 32 consecutive rows x 32 columns staged through
  // `scratch` (4 KB: hi and lo, 32 x 32 bf16 each): the warp writes the values column by column,
  // then every column's 32 rows leave as 64 contiguous bytes in four 16-byte stores, instead of
  // one two-byte store per element and lane. All 32 lanes take part (rows at or beyond T are
  // not written). bf16 only.
  __device__ static void store_trans_staged(const Params& p, void* th, void* tlo, size_t unit_off,
                                            int gi, int gj_base, const uint32_t (&hi)[32],
                                            const uint32_t (&lo)[32], uint8_t* scratch) {
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint16_t* sh = reinterpret_cast<uint16_t*>(scratch);
    uint16_t* sl = sh + 32 * 32;
    __syncwarp();  // the previous chunk's reads of the staging are done
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      sh[e * 32 + lane] = static_cast<uint16_t>(hi[e]);
      if (tlo != nullptr) sl[e * 32 + lane] = static_cast<uint16_t>(lo[e]);
    }
    __syncwarp();
    const int gi0 = gi - lane;  // the warp's first row
    const int q = lane & 3;     // 16-byte quarter of a column: rows gi0 + 8q .. + 7
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = (lane >> 2) + 8 * k;
      const int gj = gj_base + e;
      if (gj >= p.T) continue;
      const int r0 = gi0 + 8 * q;
      const size_t idx = (unit_off + gj) * static_cast<size_t>(p.ldp) + r0;
      for (int t = 0; t < (tlo != nullptr ? 2 : 1); ++t) {
        const uint16_t* src = (t == 0 ? sh : sl) + e * 32 + 8 * q;
        uint16_t* dst = static_cast<uint16_t*>(t == 0 ? th : tlo) + idx;
        if (r0 + 8 <= p.T) {
          *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
        } else {
          for (int u = 0; u < 8 && r0 + u < p.T; ++u) dst[u] = src[u];
        }
      }
    }
  }

  // scratch (pair engine only): 4 KB of this warp's shared memory for the staged transposed
  // store; with it all lanes stay in the call, rows at or beyond T write nothing.
  __device__ static void epilogue(const Params& p, const Tile& tl, int row, int c0,
                                  const uint32_t (&r)[32], uint8_t* scratch = nullptr) {
    const int gi = tl.mi * S::BM + row;
    const bool row_ok = gi < p.T;
    if (!row_ok && scratch == nullptr) return;
    const int gj_base = tl.ni * BN + c0;
    if (ELEM == 4 && p.ksplit > 1) {
      if (!row_ok) return;
      // K-split partial: raw fp32 sums, masked and split by the reduce pass
      float* dst = p.part + ((static_cast<size_t>(tl.ks) * p.units + tl.unit) * p.T + gi) *
                                static_cast<size_t>(p.ldp);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int gj0 = gj_base + 4 * v;
        if (gj0 + 4 > p.ldp) continue;
        *reinterpret_cast<uint4*>(dst + gj0) = make_uint4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
      }
      return;
    }
    const bool diag = tl.ni * BN < (tl.mi + 1) * S::BM && (tl.ni + 1) * BN > tl.mi * S::BM;
    uint32_t hi[32], lo[32];
    if (ELEM == 2) {
      // packed conversions: one cvt per pair for hi, one for lo
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const float x0 = gj_base + e < gi ? __uint_as_float(r[e]) : 0.0f;
        const float x1 = gj_base + e + 1 < gi ? __uint_as_float(r[e + 1]) : 0.0f;
        const uint32_t wh = cvt_bf16x2(x0, x1);
        const uint32_t wl = cvt_bf16x2(x0 - bf16x2_lo(wh), x1 - bf16x2_hi(wh));
        hi[e] = wh & 0xFFFFu;
        hi[e + 1] = wh >> 16;
        lo[e] = wl & 0xFFFFu;
        lo[e + 1] = wl >> 16;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float x = gj_base + e < gi ? __uint_as_float(r[e]) : 0.0f;
        split(x, hi[e], lo[e]);
      }
    }
    const size_t unit_off = static_cast<size_t>(tl.unit) * p.T;
    // ---- direct store S[i][j] (vectorised unless it must skip the upper part of a diagonal tile)
    // On a diagonal tile of G only chunks that cross the diagonal need element stores: a chunk
    // wholly below row i is stored whole, one wholly above it is the other orientation's.
    const bool below = gj_base + 31 < gi;
    if (!row_ok || (p.mode == kStoreSym && diag && gj_base > gi)) {
      // nothing of this row and chunk is stored here (staged transposed store below only)
    } else if (p.mode == kStoreDirect || p.mode == kStoreLU || (p.mode == kStoreSym && (!diag || below))) {
      // chunked forward: columns are stored relative to the chunk's first key
      const int cb = key0(p, tl.mi);
      const size_t row_off = (unit_off + gi) * static_cast<size_t>(p.ldp) - static_cast<size_t>(cb);
      if (ELEM == 2) {
        uint16_t* dh = static_cast<uint16_t*>(p.p_hi) + row_off;
        uint16_t* dl = static_cast<uint16_t*>(p.p_lo) + row_off;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int gj0 = gj_base + 8 * v;
          if (gj0 - cb + 8 > p.ldp) continue;
          *reinterpret_cast<uint4*>(dh + gj0) =
              make_uint4(hi[8 * v] | (hi[8 * v + 1] << 16), hi[8 * v + 2] | (hi[8 * v + 3] << 16),
                         hi[8 * v + 4] | (hi[8 * v + 5] << 16), hi[8 * v + 6] | (hi[8 * v + 7] << 16));
          if (p.p_lo != nullptr)
            *reinterpret_cast<uint4*>(dl + gj0) =
                make_uint4(lo[8 * v] | (lo[8 * v + 1] << 16), lo[8 * v + 2] | (lo[8 * v + 3] << 16),
                           lo[8 * v + 4] | (lo[8 * v + 5] << 16), lo[8 * v + 6] | (lo[8 * v + 7] << 16));
        }
      } else {
        uint32_t* dh = static_cast<uint32_t*>(p.p_hi) + row_off;
        uint32_t* dl = static_cast<uint32_t*>(p.p_lo) + row_off;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const int gj0 = gj_base + 4 * v;
          if (gj0 - cb + 4 > p.ldp) continue;
          *reinterpret_cast<uint4*>(dh + gj0) = make_uint4(hi[4 * v], hi[4 * v + 1], hi[4 * v + 2], hi[4 * v + 3]);
          *reinterpret_cast<uint4*>(dl + gj0) = make_uint4(lo[4 * v], lo[4 * v + 1], lo[4 * v + 2], lo[4 * v + 3]);
        }
      }
    } else if (p.mode == kStoreSym) {
      // diagonal tile: this orientation owns j <= i (the diagonal itself is zero)
      const size_t row_off = (unit_off + gi) * static_cast<size_t>(p.ldp);
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int gj = gj_base + e;
        if (gj <= gi) {
          store1(p.p_hi, row_off + gj, hi[e]);
          if (p.p_lo != nullptr) store1(p.p_lo, row_off + gj, lo[e]);
        }
      }
    }
    // ---- transposed store S^T[j][i]
    if (p.mode == kStoreTrans || p.mode == kStoreLU || p.mode == kStoreSym) {
      void* th = p.mode == kStoreLU ? p.p2_hi : p.p_hi;
      void* tlo = p.mode == kStoreLU ? p.p2_lo : p.p_lo;
      const bool strict = p.mode == kStoreSym && diag;  // Sym diagonal: only j < i here
      if (ELEM == 2 && scratch != nullptr) {
        // warp-uniform: the warp's rows are gi0 .. gi0 + 31
        const int gi0 = gi - static_cast<int>(threadIdx.x & 31);
        if (!strict || gj_base + 31 < gi0) {  // every (i, j) of the chunk has j < i
          store_trans_staged(p, th, tlo, unit_off, gi, gj_base, hi, lo, scratch);
          return;
        }
        if (gj_base >= gi0 + 31) return;  // no (i, j) of the chunk has j < i
      }
      if (!row_ok) return;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int gj = gj_base + e;
        if (gj >= p.T || (strict && gj >= gi)) continue;
        const size_t idx = (unit_off + gj) * static_cast<size_t>(p.ldp) + gi;
        store1(th, idx, hi[e]);
        if (tlo != nullptr) store1(tlo, idx, lo[e]);
      }
    }
  }
};

template <class S, class P>
static int launch_tc(const typename P::Params& prm, int ntiles, cudaStream_t stream, int kind) {
  if (ntiles <= 0) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<S, P>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tc_smem_bytes<S, P>());
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return BDH_ERR_CUDA;
    }
    attr_set[dev] = true;
  }
  int grid = std::min(ntiles, sm_count(dev));
  if constexpr (HasMaxCtas<P>::value) grid = std::max(1, std::min(grid, P::max_ctas(prm, sm_count(dev))));
  prof_start(kind, stream);
  cudaError_t e = launch_pdl(tc_gemm_kernel<S, P>, dim3(grid), dim3(tc_threads<P>()),
                             tc_smem_bytes<S, P>(), stream, prm);
  prof_stop(kind, stream);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string("tc_gemm_kernel launch: ") + cudaGetErrorString(e));
    return BDH_ERR_CUDA;
  }
  return 0;
}

}  // namespace bdh

// Internal launch descriptors shared between the C-ABI layer (capi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "bdh_sm100.h"

namespace bdh {

// One forward problem. For fp32 inputs q/k/v point at tf32 "hi" operands and *_lo at the
// matching residuals (x - hi); for bf16 the *_lo pointers are unused.
struct FwdArgs {
  const void* q = nullptr;
  const void* q_lo = nullptr;
  int64_t q_strides[4] = {0, 0, 0, 1};
  const void* k = nullptr;
  const void* k_lo = nullptr;
  int64_t k_strides[4] = {0, 0, 0, 1};
  const void* v = nullptr;
  const void* v_lo = nullptr;
  int64_t v_strides[4] = {0, 0, 0, 1};
  int dtype = BDH_DTYPE_BF16;
  void* out = nullptr;
  int64_t out_strides[4] = {0, 0, 0, 1};
  int out_dtype = BDH_DTYPE_BF16;
  int64_t B = 0, H = 0, Hv = 0, T = 0, N = 0, D = 0;
};

int64_t score_ld(int64_t T);
// Row length (keys) of the transposed tf32 V operand: [B*Hv][D][vt_ld(T)].
int64_t vt_ld(int64_t T);
int launch_score(const FwdArgs& a, void* p_hi, void* p_lo, cudaStream_t stream, int* err);
int launch_value(const FwdArgs& a, const void* p_hi, const void* p_lo, cudaStream_t stream,
                 int* err);

// Elementwise kernels (elementwise.cu).
int launch_rope(const void* x, int x_dtype, const int64_t xs[4], void* y, int y_dtype,
                const int64_t ys[4], float* y_lo, const float* freqs, int64_t B, int64_t H,
                int64_t T, int64_t N, int64_t pos0, cudaStream_t stream);
// x (strided, fp32) -> contiguous hi = tf32(x), lo = x - hi.
int launch_split_tf32(const float* x, const int64_t xs[4], float* hi, float* lo, int64_t B,
                      int64_t H, int64_t T, int64_t N, cudaStream_t stream);
// x (B, H, T, N) strided fp32 -> transposed hi/lo [B*H][N][ldt] (T contiguous, ldt >= T).
int launch_split_tf32_t(const float* x, const int64_t xs[4], float* hi, float* lo, int64_t B,
                        int64_t H, int64_t T, int64_t N, int64_t ldt, cudaStream_t stream);

// Decode (decode.cu).
struct DecodeArgs {
  const void* q = nullptr;
  int64_t q_strides[4] = {0, 0, 0, 1};
  int q_dtype = BDH_DTYPE_F32;
  const void* k = nullptr;
  int64_t k_strides[4] = {0, 0, 0, 1};
  const void* v = nullptr;
  int64_t v_strides[4] = {0, 0, 0, 1};
  int kv_dtype = BDH_DTYPE_F32;
  void* out = nullptr;
  int64_t out_strides[4] = {0, 0, 0, 1};
  int64_t B = 0, H = 0, Hv = 0, Tq = 0, S = 0, N = 0, D = 0;
  const float* freqs = nullptr;
  int64_t pos = 0;
  void* slot = nullptr;
  int64_t slot_strides[4] = {0, 0, 0, 1};
};
int decode_splits(int64_t S);
size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t D);
int launch_decode(const DecodeArgs& a, float* partial, cudaStream_t stream);

}  // namespace bdh

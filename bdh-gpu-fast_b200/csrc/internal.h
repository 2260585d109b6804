// Internal launch descriptors shared between the C-ABI layer (capi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <utility>

#include "bdh_sm100.h"

namespace bdh {

// Programmatic dependent launch of the persistent tensor-core kernels (BDH_SM100_PDL=0 turns it
// off; read once). Such a launch lets the kernel's CTAs start, set up their barriers and TMEM and
// wait on the device (griddepcontrol.wait, before their first global-memory access) on the SMs
// that the previous kernel of the stream has already left, instead of starting only after it
// completes. Results are the same either way. The row LayerNorms launch plainly: launched early,
// their small CTAs fit beside the running gate + decoder's and waited there for its whole run,
// and the config-2 step measured slower.
inline bool pdl_on() {
  static const bool on = [] {
    const char* e = std::getenv("BDH_SM100_PDL");
    return !(e != nullptr && std::atoi(e) == 0);
  }();
  return on;
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_on() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Launch timing hooks (prof.cpp); kinds as documented at bdh_profile_end.
enum ProfKind : int { kProfScore = 0, kProfValue = 1, kProfRope = 2, kProfDecode = 3,
                      kProfGradQ = 4, kProfGradV = 5, kProfSplit = 6, kProfOther = 7,
                      kProfState = 8, kProfEncode = 9, kProfGate = 10, kProfNorm = 11,
                      kProfDecoder = 12 };
void prof_start(int kind, cudaStream_t s);
void prof_stop(int kind, cudaStream_t s);

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
  // > 0: each output row (over D) is LayerNormed (affine-free, eps = ln_eps) before the store
  int ln = 0;
  float ln_eps = 1e-5f;
};

// Layouts of the masked score pass output (see score_pass.cuh).
enum ScoreStore : int { kStoreDirect = 0, kStoreTrans = 1, kStoreSym = 2, kStoreLU = 3 };

// One masked score pass S = tril(A B^T, -1) per unit; A: (B,H,T,K), B: (B,Hb,T,K) with
// Hb in {1,H}. elem 2: bf16 operands (a[0], b[0]); elem 4: tf32 hi/lo pairs (a[0..1], b[0..1]).
struct ScoreArgs {
  int elem = 2;
  const void* a[2] = {nullptr, nullptr};
  int64_t a_strides[4] = {0, 0, 0, 1};
  const void* b[2] = {nullptr, nullptr};
  int64_t b_strides[4] = {0, 0, 0, 1};
  int64_t B = 0, H = 0, Hb = 0, T = 0, K = 0;
  int mode = kStoreDirect;
  int chunk = 0;  // > 0 (kStoreDirect only): keys limited to each row block's chunk, [u][T][chunk]
  void* p_hi = nullptr;
  void* p_lo = nullptr;
  void* p2_hi = nullptr;
  void* p2_lo = nullptr;
  // split-K (fp32 direct forward only): ksplit > 1 partial tiles in part [ksplit][u][T][ldp]
  // fp32, then summed in order and split into (p_hi, p_lo) by a reduce pass
  int ksplit = 1;
  float* part = nullptr;
};
int launch_score_pass(const ScoreArgs& a, cudaStream_t stream, int* err);
// K-split count of the fp32 forward score pass (1 = none) for units x T x K.
int score_ksplit_f32(int64_t units, int64_t T, int64_t K);

int64_t score_ld(int64_t T);
// Row length (keys) of the transposed tf32 V operand: [B*Hv][D][vt_ld(T)].
int64_t vt_ld(int64_t T);
int launch_score(const FwdArgs& a, void* p_hi, void* p_lo, float* part, cudaStream_t stream,
                 int* err);
int launch_value(const FwdArgs& a, const void* p_hi, const void* p_lo, cudaStream_t stream,
                 int* err);

// Chunked long-sequence forward (attn_chunked.cu), bf16 only.
int chunk_len(int64_t T);  // keys per chunk of the chunked forward at sequence length T
size_t chunked_p_bytes(int64_t B, int64_t H, int64_t T);
size_t chunked_s_bytes(int64_t B, int64_t H, int64_t T, int64_t N, int64_t D);
int launch_chunked_forward(const FwdArgs& a, void* p_hi, void* p_lo, void* s_hi, void* s_lo,
                           cudaStream_t stream, int* err);

// Backward passes (attn_bwd.cu).
// out[u] = Gs[u] X[u] with Gs a hi/lo score pair ([B*H][T][score_ld(T)]); krange 0: all keys,
// 1: keys below the end of each 128-row block, 2: keys from the start of each block.
// elem 2: X is (B,H,T,N) bf16 (x[0], x_strides); elem 4: X^T tf32 hi/lo [B*H][N][vt_ld(T)].
struct GradQArgs {
  int elem = 2;
  const void* g_hi = nullptr;
  const void* g_lo = nullptr;
  const void* x[2] = {nullptr, nullptr};
  int64_t x_strides[4] = {0, 0, 0, 1};
  int64_t B = 0, H = 0, T = 0, N = 0;
  int krange = 0;
  void* out = nullptr;
  int64_t out_strides[4] = {0, 0, 0, 1};
  int out_dtype = BDH_DTYPE_BF16;
  const float* freqs = nullptr;
  int64_t pos0 = 0;
};
int launch_grad_q(const GradQArgs& a, cudaStream_t stream, int* err);

// dV[b,hv] = sum over heads sharing hv of Mt_h dO_h with Mt = M^T as a hi/lo score pair.
// elem 2: dO is (B,H,T,D) bf16; elem 4: dO^T tf32 hi/lo [B*H][D][vt_ld(T)].
struct GradVArgs {
  int elem = 2;
  const void* mt_hi = nullptr;
  const void* mt_lo = nullptr;
  const void* dout[2] = {nullptr, nullptr};
  int64_t do_strides[4] = {0, 0, 0, 1};
  int64_t B = 0, H = 0, Hv = 0, T = 0, D = 0;
  void* out = nullptr;
  int64_t out_strides[4] = {0, 0, 0, 1};
  int out_dtype = BDH_DTYPE_BF16;
};
int launch_grad_v(const GradVArgs& a, cudaStream_t stream, int* err);

// Elementwise kernels (elementwise.cu).
int launch_rope(const void* x, int x_dtype, const int64_t xs[4], void* y, int y_dtype,
                const int64_t ys[4], float* y_lo, const float* freqs, int64_t B, int64_t H,
                int64_t T, int64_t N, int64_t pos0, int relu_in, cudaStream_t stream);
// out = relu(x) * relu(y), all (B,H,T,N) with a contiguous last dimension.
// fp32 decoder product of a decode step (decoder_f32.cu): out (M, D) = X (M, K) @ W (K, D),
// K split into decoder_f32_slices(K) slices whose fp32 partials go to part (slices x M x D).
int64_t decoder_f32_slices(int64_t K);
int launch_decoder_f32(const float* x, int64_t ldx, const float* w, int64_t ldw, float* out,
                       int64_t ldo, float* part, int64_t M, int64_t K, int64_t D,
                       cudaStream_t stream);
int launch_relu_mul(const void* x, const int64_t xs[4], const void* y, const int64_t ys[4],
                    void* out, const int64_t os[4], int dtype, int64_t B, int64_t H, int64_t T,
                    int64_t N, cudaStream_t stream);
// x (strided, fp32) -> contiguous hi = tf32(x), lo = x - hi.
int launch_split_tf32(const float* x, const int64_t xs[4], float* hi, float* lo, int64_t B,
                      int64_t H, int64_t T, int64_t N, cudaStream_t stream);
// x (B, H, T, N) strided fp32 -> transposed hi/lo [B*H][N][ldt] (T contiguous, ldt >= T).
int launch_split_tf32_t(const float* x, const int64_t xs[4], float* hi, float* lo, int64_t B,
                        int64_t H, int64_t T, int64_t N, int64_t ldt, cudaStream_t stream);

// Fused latent projections (latent_proj.cu), bf16; strides in elements.
struct LatentArgs {
  const void* x = nullptr;       // encode: (B,T,D) {b,t,d}
  int64_t x_strides[3] = {0, 0, 1};
  const void* y = nullptr;       // gate: (B,H,T,D) {b,h,t,d}
  int64_t y_strides[4] = {0, 0, 0, 1};
  const void* w = nullptr;       // enc / encv (H,D,N) {h,d,n}
  int64_t w_strides[3] = {0, 0, 1};
  const void* w2 = nullptr;      // gate_x: enc (H,D,N) {h,d,n}
  int64_t w2_strides[3] = {0, 0, 1};
  void* xs = nullptr;            // (B,T,H,N) {b,t,h,n}: written by encode, read by gate
  int64_t xs_strides[4] = {0, 0, 0, 1};
  void* qr = nullptr;            // (B,H,T,N) {b,h,t,n}
  int64_t qr_strides[4] = {0, 0, 0, 1};
  void* xy = nullptr;            // (B,T,H,N) {b,t,h,n}
  int64_t xy_strides[4] = {0, 0, 0, 1};
  const float* freqs = nullptr;
  int64_t B = 0, T = 0, H = 0, D = 0, N = 0, pos0 = 0;
};
// Fused gate + decoder (gate_decoder.cu): y_mlp = bf16(sum_{h,n} bf16(xs * relu(bf16(y encv)))
// dec), D = 256, N a multiple of 128; encv (H,D,N) with d contiguous, dec (H*N, D) with the
// latent index contiguous (a transposed copy), out (B,T,D) bf16.
struct GateDecArgs {
  const void* y = nullptr;       // (B,H,T,D) {b,h,t,d}
  int64_t y_strides[4] = {0, 0, 0, 1};
  const void* encv = nullptr;    // (H,D,N) {h,d,n}, d contiguous
  int64_t encv_strides[3] = {0, 1, 0};
  const void* xs = nullptr;      // (B,T,H,N) {b,t,h,n}
  int64_t xs_strides[4] = {0, 0, 0, 1};
  const void* dec = nullptr;     // (H*N, D) {k,d}, k contiguous
  int64_t dec_strides[2] = {1, 0};
  void* out = nullptr;           // (B,T,D) {b,t,d}
  int64_t out_strides[3] = {0, 0, 1};
  int64_t B = 0, T = 0, H = 0, D = 0, N = 0;
  void* workspace = nullptr;     // optional: the latent-range sums of few-row problems
  size_t workspace_bytes = 0;
};
int launch_latent_gate_dec(const GateDecArgs& a, cudaStream_t stream, int* err);
// Workspace bytes with which launch_latent_gate_dec splits the latent walk of these sizes on
// the current device (0: no split).
size_t latent_gate_dec_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D, int64_t N);
int launch_latent_encode(const LatentArgs& a, cudaStream_t stream, int* err);
int launch_latent_gate_x(const LatentArgs& a, cudaStream_t stream, int* err);
int launch_latent_gate(const LatentArgs& a, cudaStream_t stream, int* err);

// Row LayerNorms (layernorm.cu); strides in elements.
int launch_layernorm(const void* x, int x_dtype, int64_t xs, void* y, int y_dtype, int64_t ys,
                     int64_t rows, int D, float eps, cudaStream_t stream);
int launch_residual_layernorm(const float* x, int64_t xs, const void* y, int y_dtype, int64_t ys,
                              float* out, int64_t os, uint16_t* out16, int64_t os16, int64_t rows,
                              int D, float eps, cudaStream_t stream);

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
// Decode against an fp8 key history (e4m3 rows with one fp32 scale each, kr_fp8.cu); values
// in f32 or bf16. With freqs the new queries are rotated first and, with slot, quantized into
// this step's cache slot (row + scale).
struct DecodeFp8Args {
  const void* q = nullptr;
  int64_t q_strides[4] = {0, 0, 0, 1};
  int q_dtype = BDH_DTYPE_F32;
  const uint8_t* k = nullptr;
  int64_t k_strides[4] = {0, 0, 0, 1};
  const float* k_scale = nullptr;
  int64_t ks_strides[3] = {0, 0, 1};
  const void* v = nullptr;
  int64_t v_strides[4] = {0, 0, 0, 1};
  int v_dtype = BDH_DTYPE_F32;
  void* out = nullptr;
  int64_t out_strides[4] = {0, 0, 0, 1};
  int64_t B = 0, H = 0, Hv = 0, Tq = 0, S = 0, N = 0, D = 0;
  const float* freqs = nullptr;
  int64_t pos = 0;
  uint8_t* slot = nullptr;
  int64_t slot_strides[4] = {0, 0, 0, 1};
  float* slot_scale = nullptr;
  int64_t slot_scale_strides[3] = {0, 0, 1};
};
int launch_decode_fp8(const DecodeFp8Args& a, float* partial, float* qrot, cudaStream_t stream);
int launch_quantize_rows_fp8(const void* x, int x_dtype, const int64_t xs[4], int64_t B,
                             int64_t H, int64_t T, int64_t N, uint8_t* out, const int64_t os[4],
                             float* scale, const int64_t ss[3], cudaStream_t stream);
struct DecodePlan {
  int splits = 1;  // CTAs per (b, h, tq)
  int rows = 1;    // cached rows per CTA (<= 128)
};
// max_splits > 0 caps the split count (longer splits), e.g. to fit a fixed scratch.
DecodePlan plan_decode(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N, int64_t max_splits = 0);
size_t decode_partial_bytes(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N, int64_t D,
                            int64_t max_splits = 0);
size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N, int64_t D);
// partial: split partial sums; qrot: rotated fp32 queries (null: rotate inside the kernel).
int launch_decode(const DecodeArgs& a, float* partial, float* qrot, int64_t max_splits,
                  cudaStream_t stream);
int decode_entry(const void* q, const int64_t q_strides[4], int q_dtype, const void* k_past,
                 const int64_t k_strides[4], const void* v_past, const int64_t v_strides[4],
                 int kv_dtype, void* out, const int64_t out_strides[4], int64_t B, int64_t H,
                 int64_t Hv, int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                 int64_t pos, void* kr_slot, const int64_t slot_strides[4], float* partial,
                 float* qrot, int64_t max_splits, void* stream);

// Recurrent-state decode (state_decode.cu). state: (B,H,N,D) fp32 strides {b,h,n,1}.
struct StateDecodeArgs {
  const void* q = nullptr;
  int64_t q_strides[4] = {0, 0, 0, 1};
  int q_dtype = BDH_DTYPE_F32;
  float* state = nullptr;
  int64_t state_strides[4] = {0, 0, 0, 1};
  const void* v = nullptr;
  int64_t v_strides[4] = {0, 0, 0, 1};
  int v_dtype = BDH_DTYPE_F32;
  void* out = nullptr;
  int64_t out_strides[4] = {0, 0, 0, 1};
  int64_t B = 0, H = 0, Hv = 0, N = 0, D = 0;
  const float* freqs = nullptr;
  int64_t pos = 0;
  int relu_input = 0;
};
size_t state_decode_partial_bytes(int64_t B, int64_t H, int64_t N, int64_t D);
size_t state_decode_workspace_bytes(int64_t B, int64_t H, int64_t N, int64_t D);
int launch_state_decode(const StateDecodeArgs& a, float* partial, float* qrot, cudaStream_t stream);

}  // namespace bdh

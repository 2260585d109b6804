/*
 * bdh_sm100.h — C ABI of the B200 (sm_100a) strict-causal linear "tril" attention of BDH.
 *
 *   forward : out = tril((R.Q)(R.Q)^T, -1) . V        (no softmax, no scale, diagonal excluded)
 *   decode  : out = (q . K_past^T) . V_past             (every cached key precedes the query)
 *   backward: dQ_total = (dS + dS^T) . QR,  dV = sum_h M^T . dO,
 *             with M = tril(QR QR^T, -1) and dS = tril(dO V^T, -1)
 *
 * Every entry point takes plain device pointers, element strides and sizes, and a CUDA
 * stream (cudaStream_t passed as void*). Tensors are 4-D (B, H, T, X) with the last
 * dimension contiguous (stride 1); any other strides are accepted as long as each
 * row/head/batch stride is a multiple of 16 bytes (TMA rule) — so permuted views and
 * capacity-strided cache views are read in place, never copied. V may have one head
 * (shared by all query heads) or H heads. Outputs are written, never accumulated into.
 *
 * Scratch memory is always provided by the caller (`workspace`, sized by the matching
 * *_workspace_size function); the library itself never allocates device memory.
 *
 * Return value: BDH_OK (0) or an error code; bdh_last_error() gives the message of the
 * calling thread's last failure. Kernels never trap: a pipeline wait that exceeds its
 * time limit records a code in the device error word (bdh_device_error) and returns.
 */
#ifndef BDH_SM100_H_
#define BDH_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BDH_ABI_VERSION 9

#define BDH_DTYPE_F32 0
#define BDH_DTYPE_BF16 1

#define BDH_OK 0
#define BDH_ERR_INVALID 1   /* bad shape / dtype / stride / alignment (nothing launched) */
#define BDH_ERR_CUDA 2      /* CUDA runtime error at launch */
#define BDH_ERR_WORKSPACE 3 /* workspace missing or too small */

/* ABI version of the loaded library (BDH_ABI_VERSION); bindings refuse a library of another
 * version. No counterpart in the reference (its module is built together with its callers). */
int bdh_abi_version(void);

/* Message of the calling thread's last failing call ("" if none). The reference reports the
 * same failures as C++ exceptions through pybind (TORCH_CHECK, csrc/tril_attn_cuda.cu:252,
 * csrc/tril_attn_bind.cpp:8); a C-ABI returns a code and keeps the message here. */
const char* bdh_last_error(void);

/* Read (and optionally clear) the device error word of `device`: 0 = no kernel has
 * reported a failure; otherwise one of the codes of csrc/common.cuh (pipeline timeouts).
 * Synchronises the device. No counterpart in the reference (its kernels have no waits that
 * can time out). */
int bdh_device_error(int device, int* code, int reset);

/*
 * RoPE apply: y = R(pos0 + t) x, pairwise on (x[2p], x[2p+1]) with
 *   phase[t,n] = ((pos0 + t) * freqs[n] mod 1) * 2pi   (fp32, as the reference computes it)
 *   y0 = x0*cos - x1*sin,  y1 = x1*cos + x0*sin
 * For bf16 x each product is rounded to bf16 before the add, as the reference does.
 * x: (B,H,T,N) in x_dtype; y: (B,H,T,N) in y_dtype (may differ: a cache slot in another
 * dtype). `y_lo` (optional, only with y_dtype F32) receives y - tf32(y) and y then holds
 * tf32(y): the split operand of the fp32 tensor-core path.
 * Replaces: kernels/rope.py:220-240 (eager_rope_rotate) behind kernels/rope_dispatch.py:64-99
 * (bdh_rope_rotate / bdh_rope_rotate_paired) and bdh.py:119-150 (phase / cos / sin tables).
 */
#define BDH_ROPE_RELU_INPUT 1 /* flags bit: rotate relu(x) (the ReLU of the BDH encoder, bdh.py:994) */
int bdh_rope_rotate(const void* x, int x_dtype, const int64_t x_strides[4], void* y, int y_dtype,
                    const int64_t y_strides[4], void* y_lo, const float* freqs, int64_t B,
                    int64_t H, int64_t T, int64_t N, int64_t pos0, int flags, void* stream);

/*
 * Gated product of the BDH layer: out = relu(x) * relu(y), all (B,H,T,N) with a contiguous last
 * dimension and any other strides (the einsum outputs are read in place), rounded once to dtype.
 * Replaces the eager `x_sparse * y_sparse` of bdh.py:927-945 / bdh_baseline.py:124-126 together
 * with the two F.relu passes before it (bdh.py:861-925).
 */
int bdh_relu_mul(const void* x, const int64_t x_strides[4], const void* y,
                 const int64_t y_strides[4], void* out, const int64_t out_strides[4], int dtype,
                 int64_t B, int64_t H, int64_t T, int64_t N, void* stream);

/*
 * Forward algorithm selection (process-wide): BDH_FWD_AUTO picks the chunked form for bf16
 * inputs when T >= 1536 (fewer flops: about T*C*(N+D) + 4*T*N*D per unit with C = 256 instead of
 * T*T*(N+D)), else the quadratic form; the other values force one form (the chunked form needs
 * bf16 inputs and falls back to quadratic for fp32). Returns the previous setting.
 * No counterpart in the reference (its forward is always quadratic).
 */
#define BDH_FWD_AUTO 0
#define BDH_FWD_QUADRATIC 1
#define BDH_FWD_CHUNKED 2
int bdh_set_forward_algo(int algo);

/*
 * bf16 score-like operands (P of the forward, the chunked prefix states, G and M^T of the
 * backward) for the calling thread only: BDH_SCORES_ONE rounds each fp32 sum once to bf16
 * before the next tensor-core product, as the reference's bf16 matmul chain does
 * (kernels/attention.py:27-40: (q @ k.mT).tril_(-1) @ v returns bf16 scores under autocast);
 * BDH_SCORES_SPLIT keeps it exact as a bf16 hi + lo pair (twice the work of the consuming
 * product); BDH_SCORES_DEFAULT returns to the process default (BDH_SM100_SPLIT_SCORES, else the
 * quadratic forward's P split and every other operand one term). The workspace-size queries
 * follow the same setting, so set it before querying. fp32 inputs are unaffected (always the
 * exact tf32 split). Returns the previous setting of the thread, or -2 for an unknown mode.
 * No counterpart in the reference (a knob of this build's kernels).
 */
#define BDH_SCORES_DEFAULT (-1)
#define BDH_SCORES_ONE 0
#define BDH_SCORES_SPLIT 1
int bdh_set_score_terms(int mode);

/* Scratch bytes bdh_tril_score_v needs for these sizes (dtype of q/k/v). */
size_t bdh_tril_score_v_workspace_size(int dtype, int64_t B, int64_t H, int64_t Hv, int64_t T,
                                       int64_t N, int64_t D, int k_is_q);

/*
 * Forward: out[b,h] = tril(q[b,h] k[b,h]^T, -1) v[b,hv], fp32 accumulation.
 * q, k: (B,H,T,N); v: (B,Hv,T,D) with Hv in {1,H}; out: (B,H,T,D) in out_dtype.
 * dtype is the element type of q, k and v (all the same). k may equal q (BDH: K is Q).
 * Replaces: csrc/tril_attn.h:20 tril_score_v(q,k,v) as bound at csrc/tril_attn_bind.cpp:3-12
 * and :27 (pybind "tril_score_v"), called from kernels/cuda_attn.py:391-414.
 */
int bdh_tril_score_v(const void* q, const int64_t q_strides[4], const void* k,
                     const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                     int dtype, void* out, const int64_t out_strides[4], int out_dtype,
                     int64_t B, int64_t H, int64_t Hv, int64_t T, int64_t N, int64_t D,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * The forward followed by the affine-free LayerNorm of every output row over D (eps as
 * F.layer_norm): out = LN(tril(q k^T, -1) v), the attention output of a BDH layer as its
 * encoder_v projection reads it (bdh.py:1044; under bf16 autocast the LayerNorm runs in fp32 on
 * the bf16 attention output and its consumer casts the result to bf16). For the quadratic bf16
 * forward with D <= 256 the normalisation is done in the value pass's epilogue (the
 * un-normalised output never reaches HBM); other forms normalise the output rows in place
 * afterwards and then need rows of one stride. Arguments and workspace (the
 * bdh_tril_score_v_workspace_size figure) as bdh_tril_score_v. No counterpart in the
 * reference (a model-level fusion).
 */
int bdh_tril_score_v_layernorm(const void* q, const int64_t q_strides[4], const void* k,
                               const int64_t k_strides[4], const void* v,
                               const int64_t v_strides[4], int dtype, void* out,
                               const int64_t out_strides[4], int out_dtype, int64_t B, int64_t H,
                               int64_t Hv, int64_t T, int64_t N, int64_t D, float eps,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes bdh_tril_decode needs: the split partial sums, plus B*H*Tq*N*4 for the rotated
 * queries (used when freqs is given). */
size_t bdh_tril_decode_workspace_size(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N,
                                      int64_t D);

/*
 * Decode against a packed past: out[b,h] = (q[b,h] k_past[b,h]^T) v_past[b,hv].
 * q: (B,H,Tq,N) in q_dtype; k_past: (B,H,S,N) and v_past: (B,Hv,S,D) in kv_dtype (the cache
 * storage type; read as stored, widened in registers); out: (B,H,Tq,D) in q_dtype.
 * S == 0 gives zeros. Optional fused RoPE: when freqs != NULL, q is first rotated to
 * position `pos` (all Tq rows at pos .. pos+Tq-1) and, when kr_slot != NULL, the rotated
 * rows are also written to kr_slot (B,H,Tq,N) in kv_dtype (the cache write of this step).
 * Replaces: csrc/tril_attn.h:21 tril_decode(q,k_past,v_past) bound at
 * csrc/tril_attn_bind.cpp:14-23 and :31, called from kernels/cuda_attn.py:490-502; the fused
 * form replaces bdh.py:396-401 (RoPE into the cache slot) + bdh.py:431-437 (decode call).
 */
int bdh_tril_decode(const void* q, const int64_t q_strides[4], int q_dtype, const void* k_past,
                    const int64_t k_strides[4], const void* v_past, const int64_t v_strides[4],
                    int kv_dtype, void* out, const int64_t out_strides[4], int64_t B, int64_t H,
                    int64_t Hv, int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                    int64_t pos, void* kr_slot, const int64_t slot_strides[4], void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * Decode without any device allocation: the same computation as bdh_tril_decode, for callers
 * that cannot provide a workspace (a process with a fixed device-memory budget reserved up
 * front, a host binding without a device allocator, a loop that must not risk the implicit
 * synchronisation of an allocation). The per-split partial sums live in one 8 MiB array
 * compiled into the library, which every device that loads the library keeps until exit.
 * Limit: splits * B * H * Tq * D * 4 bytes must not exceed 8 MiB, where splits = ceil(S / rows)
 * and rows (16..128 cached rows per CTA, longer when needed to fit) is chosen to fill the GPU
 * (e.g. B*H = 256, Tq = 1, D = 256 allows S <= 32 * 128 = 4096); larger problems return
 * BDH_ERR_INVALID with a message.
 * The new queries are rotated inside the decode kernel here (the workspace form rotates them
 * once in a separate pass).
 * The first call on each device looks the array's device address up (cudaGetSymbolAddress)
 * with that device current: make that first call before any stream capture begins. The address
 * is remembered per device together with the CUDA context it was found in; a call under another
 * current context (after cudaDeviceReset, or a context the caller created) looks it up again,
 * so such a call, too, must not be the first one inside a stream capture.
 * All calls on a device share the array and it keeps the last call's contents; every
 * element a call reads is written by the same call first, so nothing needs clearing, but
 * calls whose work overlaps on the GPU (different streams, no ordering) race on it.
 * No counterpart in the reference: it has no allocation-free entry point.
 */
int bdh_tril_decode_noalloc(const void* q, const int64_t q_strides[4], int q_dtype,
                            const void* k_past, const int64_t k_strides[4], const void* v_past,
                            const int64_t v_strides[4], int kv_dtype, void* out,
                            const int64_t out_strides[4], int64_t B, int64_t H, int64_t Hv,
                            int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                            int64_t pos, void* kr_slot, const int64_t slot_strides[4],
                            void* stream);

/*
 * Recurrent-state decode step, the N x D state form of the cached T = 1 attention (an opt-in
 * alternative to the key/value history of bdh_cache.py:38-111,226-324 and the decode of
 * kernels/attention.py:193-219; no counterpart function in the reference):
 *   qr        = RoPE(relu_input ? relu(q) : q) at position pos          (freqs required)
 *   out[b,h]  = qr[b,h] . S[b,h]                 S = sum over the past of k_j v_j^T (k = qr)
 *   S[b,h]   += qr[b,h]^T v[b,hv]                in place, after out is formed
 * q (B,H,1,N) f32/bf16; state (B,H,N,D) fp32 (strides {b,h,n,1}, n stride a multiple of 4);
 * v (B,Hv,1,D) f32/bf16 with Hv in {1,H}; out (B,H,1,D) in q's dtype. D must be 128, 256 or
 * 512. Latent rows whose rotated query is zero are neither read nor written. One step costs
 * 2 * B * H * nnz(qr) * D * 4 bytes of state traffic, independent of the past length.
 */
size_t bdh_state_decode_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D);
int bdh_state_decode(const void* q, const int64_t q_strides[4], int q_dtype, float* state,
                     const int64_t state_strides[4], const void* v, const int64_t v_strides[4],
                     int v_dtype, void* out, const int64_t out_strides[4], int64_t B, int64_t H,
                     int64_t Hv, int64_t N, int64_t D, const float* freqs, int64_t pos,
                     int relu_input, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes bdh_tril_score_v_bwd needs. */
size_t bdh_tril_score_v_bwd_workspace_size(int dtype, int64_t B, int64_t H, int64_t Hv, int64_t T,
                                           int64_t N, int64_t D, int k_is_q);

/*
 * Backward of the forward above for upstream gradient dout (B,H,T,D):
 *   dS = tril(dout v^T, -1), M = tril(q k^T, -1)
 *   dq = dS k,  dk = dS^T q,  dv = sum over heads sharing v of M^T dout.
 * When k == q (k_is_q = 1) dq receives dq + dk (the self-attention gradient) and dk is unused.
 * When freqs != NULL (requires k_is_q) q is the ROTATED input QR and dq receives the gradient
 * with respect to the UNROTATED latent: R(pos0+t)^T (dS + dS^T) QR (RoPE adjoint fused).
 * Outputs dq (B,H,T,N), dk (B,H,T,N), dv (B,Hv,T,D) are written in `dtype`.
 * Replaces: kernels/attention_bwd.py:45-83 / :86-181 (analytic_tril_attn_backward[_blocked])
 * as used by StrictTrilAttnFn / StrictTrilSelfAttnFn (kernels/attention_bwd.py:218-291) and,
 * with freqs, the RoPE backward of kernels/rope.py:540-557.
 */
int bdh_tril_score_v_bwd(const void* q, const int64_t q_strides[4], const void* k,
                         const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                         const void* dout, const int64_t dout_strides[4], int dtype, void* dq,
                         const int64_t dq_strides[4], void* dk, const int64_t dk_strides[4],
                         void* dv, const int64_t dv_strides[4], int64_t B, int64_t H, int64_t Hv,
                         int64_t T, int64_t N, int64_t D, const float* freqs, int64_t pos0,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused latent projections around the attention path (bf16 only; the step before and the
 * step after it in a BDH layer). Both are K = D tensor-core contractions with their
 * elementwise work in the epilogue, so the (B, T, nh, N) latent crosses HBM once per output.
 *
 * bdh_latent_encode replaces the encoder projection + ReLU of bdh.py:861-912
 * (BDH._encoder_relu / _encoder_relu_fwd) and the RoPE apply of the attention input,
 * bdh.py:396-412 with kernels/rope.py:220-240 (bdh_rope_rotate into Attention.forward's
 * out_kr):
 *   xs[b,t,h,n] = relu(bf16(sum_k x[b,t,k] enc[h,k,n]))          x (B,T,D), enc (H,D,N)
 *   qr[b,h,t,n] = RoPE(xs[b,t,h,:])[n] at position pos0 + t       qr (B,H,T,N) strided
 * freqs must come in equal pairs (freqs[2p] == freqs[2p+1], as bdh.py:41-49 builds them).
 * Strides are in elements: x_strides {b,t,d}, enc_strides {h,d,n}, xs_strides {b,t,h,n},
 * qr_strides {b,h,t,n}; xs may be NULL (not written); the last stride of each must be 1, the
 * others multiples of 8 — except
 * the weights, which may instead have d contiguous (a transposed (H,N,D) copy seen as (H,D,N),
 * enc_strides {N*D, 1, D}); that layout is read K-major and is the faster one.
 *
 * bdh_latent_gate replaces the encoder_v projection + ReLU and the sparse product of
 * bdh.py:914-945 (BDH._encoder_v_relu and the x * y of _mlp_merge):
 *   xy[b,t,h,n] = bf16(xs[b,t,h,n] * relu(bf16(sum_k y[b,h,t,k] encv[h,k,n])))
 * y (B,H,T,D) strides {b,h,t,d}; encv (H,D,N); xs and xy (B,T,H,N) strides {b,t,h,n}.
 *
 * bdh_latent_gate_x is bdh_latent_gate with xs recomputed from x and enc in the same kernel
 * (the encoder's MMAs on the same operands, so xs is bit-identical) instead of read back:
 *   xy[b,t,h,n] = bf16(relu(bf16(sum_k x[b,t,k] enc[h,k,n])) * relu(bf16(sum_k y[b,h,t,k] encv[h,k,n])))
 * With it, bdh_latent_encode may be called with xs == NULL (qr only) and the (B,T,nh,N) xs
 * latent never exists. D <= 256; enc and encv must share one weight layout.
 *
 * bdh_latent_gate_dec is bdh_latent_gate followed by the decoder product of bdh.py:1050
 * ((x_sparse * y_sparse) @ decoder under bf16 autocast), in one kernel that keeps each xy tile
 * in shared memory as the decoder's operand, so xy never reaches HBM:
 *   out[b,t,d] = bf16(sum_{h,n} xy[b,t,h,n] dec[h*N + n, d])     xy as in bdh_latent_gate
 * D = 256 and N a multiple of 128; encv (H,D,N) must have d contiguous (encv_strides {N*D, 1, D});
 * dec (H*N, D) must have the latent index contiguous (a transposed copy, dec_strides {1, H*N});
 * out (B,T,D) bf16 strides {b,t,d}.
 * None of these calls allocates; all are stream-ordered and graph-capturable.
 */
int bdh_latent_encode(const void* x, const int64_t x_strides[3], const void* enc,
                      const int64_t enc_strides[3], void* xs, const int64_t xs_strides[4],
                      void* qr, const int64_t qr_strides[4], const float* freqs, int64_t B,
                      int64_t T, int64_t H, int64_t D, int64_t N, int64_t pos0, void* stream);
int bdh_latent_gate(const void* y, const int64_t y_strides[4], const void* encv,
                    const int64_t encv_strides[3], const void* xs, const int64_t xs_strides[4],
                    void* xy, const int64_t xy_strides[4], int64_t B, int64_t T, int64_t H,
                    int64_t D, int64_t N, void* stream);
int bdh_latent_gate_x(const void* y, const int64_t y_strides[4], const void* encv,
                      const int64_t encv_strides[3], const void* x, const int64_t x_strides[3],
                      const void* enc, const int64_t enc_strides[3], void* xy,
                      const int64_t xy_strides[4], int64_t B, int64_t T, int64_t H, int64_t D,
                      int64_t N, void* stream);
int bdh_latent_gate_dec(const void* y, const int64_t y_strides[4], const void* encv,
                        const int64_t encv_strides[3], const void* xs, const int64_t xs_strides[4],
                        const void* dec, const int64_t dec_strides[2], void* out,
                        const int64_t out_strides[3], int64_t B, int64_t T, int64_t H, int64_t D,
                        int64_t N, void* stream);
/*
 * bdh_latent_gate_dec with a workspace (same computation, same reference lines). When the
 * problem has few rows (B * ceil(T / 256) row pairs filling at most half the GPU's CTA pairs: a
 * small batch, or one rank's share of a strongly scaled batch), each row pair's walk over the
 * H * N latent columns is cut into up to 16 ranges run side by side, and the ranges' fp32 sums
 * are added in range order before the single rounding to bf16 (deterministic). The workspace
 * holds those sums: bdh_latent_gate_dec_workspace_size bytes (0 when no split is made; a smaller
 * workspace than asked for runs unsplit), 16-byte aligned. No counterpart in the reference.
 */
size_t bdh_latent_gate_dec_workspace_size(int64_t B, int64_t T, int64_t H, int64_t D, int64_t N);
int bdh_latent_gate_dec_ws(const void* y, const int64_t y_strides[4], const void* encv,
                           const int64_t encv_strides[3], const void* xs, const int64_t xs_strides[4],
                           const void* dec, const int64_t dec_strides[2], void* out,
                           const int64_t out_strides[3], int64_t B, int64_t T, int64_t H, int64_t D,
                           int64_t N, void* workspace, size_t workspace_bytes, void* stream);

/*
 * fp8 wire format of the cached rotated keys (opt-in cache storage; the reference keeps its
 * cache in fp32 / fp16 / bf16, bdh_cache.py:62-80,240-243, so this has no reference entry and
 * is lossy). Every row x[b,h,t,:] of N values becomes e4m3 bytes plus one fp32 scale:
 *   amax = max |x|,  q8 = e4m3_rn_satfinite(x * (448 / amax)),  scale = amax / 448
 * (all-zero rows: q8 = 0, scale = 0), so that x ~= q8 * scale.
 *
 * bdh_quantize_rows_fp8: x (B,H,T,N) f32 or bf16 (x_strides {b,h,t,n}, last 1) into out
 * (B,H,T,N) bytes (out_strides, last 1) and scale (B,H,T) fp32 (scale_strides {b,h,t}). N even.
 *
 * bdh_tril_decode_fp8 is bdh_tril_decode (same shapes, workspace from
 * bdh_tril_decode_workspace_size, same RoPE / slot semantics) against such a key history:
 *   out[b,h,tq] = sum_j k_scale[b,h,j] (q[b,h,tq] . k8[b,h,j]) v_past[b,hv,j]
 * k_past (B,H,S,N) bytes with k_strides, k_scale (B,H,S) fp32 with ks_strides; v_past f32 or
 * bf16 (v_dtype). With kr_slot, the rotated queries are quantized into the slot's bytes and
 * slot_scale (B,H,Tq) with slot_scale_strides.
 */
int bdh_quantize_rows_fp8(const void* x, const int64_t x_strides[4], int x_dtype, int64_t B,
                          int64_t H, int64_t T, int64_t N, void* out,
                          const int64_t out_strides[4], float* scale,
                          const int64_t scale_strides[3], void* stream);
int bdh_tril_decode_fp8(const void* q, const int64_t q_strides[4], int q_dtype,
                        const void* k_past, const int64_t k_strides[4], const float* k_scale,
                        const int64_t ks_strides[3], const void* v_past,
                        const int64_t v_strides[4], int v_dtype, void* out,
                        const int64_t out_strides[4], int64_t B, int64_t H, int64_t Hv,
                        int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                        int64_t pos, void* kr_slot, const int64_t slot_strides[4],
                        float* slot_scale, const int64_t slot_scale_strides[3],
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Affine-free LayerNorm over the last dimension, as the BDH layer applies it with F.layer_norm
 * (BDH._ln, bdh.py:565-575; on the attention output at bdh.py:1044):
 *   y[r, :] = (x[r, :] - mean_r) / sqrt(var_r + eps),  r < rows, biased variance, fp32 math.
 * x and y are f32 or bf16 (BDH_DTYPE_*), rows of D elements at the given row strides (elements).
 * D must be a multiple of 8 and at most 1024; strides multiples of 8; bases 16-byte aligned.
 */
int bdh_layernorm(const void* x, int x_dtype, int64_t x_row_stride, void* y, int y_dtype,
                  int64_t y_row_stride, int64_t rows, int64_t D, float eps, void* stream);
/*
 * Residual double LayerNorm of the BDH layer, out = LN(x + LN(y)) (BDH._residual_ln,
 * bdh.py:731-750): x and out f32, y f32 or bf16 (the decoder output). out_bf16 (may be NULL)
 * receives bf16(out), the copy the next layer's encoder projection reads.
 */
int bdh_residual_layernorm(const float* x, int64_t x_row_stride, const void* y, int y_dtype,
                           int64_t y_row_stride, float* out, int64_t out_row_stride,
                           void* out_bf16, int64_t out_bf16_row_stride, int64_t rows, int64_t D,
                           float eps, void* stream);

/*
 * fp32 decoder product of a decode step: out (M, D) = x (M, K) @ w (K, D), all fp32, with M =
 * B * T small and K = nh * N large. Replaces, for the fp32 model's decode steps, the reference's
 * y_mlp = xy @ decoder (bdh.py:1050, torch.matmul / F.linear outside autocast). K is split into
 * bdh_decoder_f32_slices(K) slices of 256 rows summed in fp32 in a fixed order, so results are
 * deterministic; they differ from a library GEMM's only by summation order.
 * x: row stride ldx (elements), unit column stride; w: row-major with row stride ldw (a multiple
 * of 4, 16-byte aligned); out: row stride ldo; D a multiple of 4. partial: caller-provided
 * fp32 workspace of bdh_decoder_f32_slices(K) * M * D elements, 16-byte aligned.
 */
int64_t bdh_decoder_f32_slices(int64_t K);
int bdh_decoder_f32(const float* x, int64_t ldx, const float* w, int64_t ldw, float* out,
                    int64_t ldo, float* partial, int64_t M, int64_t K, int64_t D, void* stream);

/*
 * Launch timing for benchmarks (no counterpart in the reference, which timed whole calls with
 * perf_counter, benchmarks/bench_gpu_attn.py:263-280). Between begin and end, every kernel of
 * this library is bracketed by CUDA events on its own stream; end synchronises them and
 * returns the summed device milliseconds and launch counts per kernel kind:
 *   0 score pass, 1 value pass, 2 RoPE, 3 decode, 4 grad-Q pass, 5 grad-V pass, 6 split/transpose,
 *   7 gated product (bdh_relu_mul), 8 state pass of the chunked forward,
 *   9 latent encode (bdh_latent_encode), 10 latent gate (bdh_latent_gate), 11 LayerNorms,
 *   12 fp32 decoder product of a decode step (bdh_decoder_f32).
 */
#define BDH_PROF_KINDS 13
int bdh_profile_begin(void);
int bdh_profile_end(double ms[BDH_PROF_KINDS], int launches[BDH_PROF_KINDS]);

#ifdef __cplusplus
}
#endif

#endif /* BDH_SM100_H_ */

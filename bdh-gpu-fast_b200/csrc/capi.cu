// extern "C" boundary of libbdh_sm100.so: argument validation, workspace carving and kernel
// sequencing. No torch types cross this boundary and nothing here allocates device memory.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <sstream>
#include <string>

#include "bdh_sm100.h"
#include "internal.h"
#include "tma_host.h"

namespace bdh {
__device__ int g_device_error = 0;  // first pipeline failure code of any kernel on this device

namespace {

int* device_error_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

bool dtype_ok(int d) { return d == BDH_DTYPE_F32 || d == BDH_DTYPE_BF16; }
int esize(int d) { return d == BDH_DTYPE_F32 ? 4 : 2; }

size_t align_up(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

std::atomic<int> g_fwd_algo{BDH_FWD_AUTO};

bool use_chunked(int dtype, int64_t T) {
  if (dtype != BDH_DTYPE_BF16) return false;
  const int algo = g_fwd_algo.load();
  if (algo == BDH_FWD_CHUNKED) return T > chunk_len(T);
  if (algo == BDH_FWD_QUADRATIC) return false;
  return T >= 1536;
}

// bf16 inputs: which score-like operands enter their tensor-core passes as one bf16 term (fp32
// sums rounded once to bf16, as the reference's bf16 matmul chain rounds P = Q K^T and
// dM = dO V^T before the next product: kernels/attention.py:27-40,
// kernels/attention_bwd.py:72-78) instead of an exact bf16 hi + lo split (twice the tensor work
// of the products that consume them, and twice their bytes). Default: the chunked forward's P
// and prefix states S and the backward's dS / G and M^T are one term; the quadratic forward's P
// stays split (its product is a small share of the forward). BDH_SM100_SPLIT_SCORES=1 splits
// every one of them, =0 none. The fp32 path always uses the tf32 hi/lo split.
// bdh_set_score_terms overrides both for the calling thread (the model's bf16 prefill asks for
// one term, the reference's autocast rounding of its eager scores).
enum ScoreTerms { kTermsDefault = -1, kTermsOne = 0, kTermsSplit = 1 };
thread_local int g_score_terms_thread = kTermsDefault;
int bf16_score_terms_env() {
  if (g_score_terms_thread != kTermsDefault) return g_score_terms_thread;
  static const int v = [] {
    const char* e = std::getenv("BDH_SM100_SPLIT_SCORES");
    if (e == nullptr || *e == 0) return static_cast<int>(kTermsDefault);
    return std::atoi(e) == 1 ? static_cast<int>(kTermsSplit) : static_cast<int>(kTermsOne);
  }();
  return v;
}
// One bf16 term for this operand? `split_by_default`: the operand is split unless forced.
bool bf16_one_term(bool split_by_default) {
  const int v = bf16_score_terms_env();
  if (v == kTermsDefault) return !split_by_default;
  return v == kTermsOne;
}

// Workspace layout of the forward (byte offsets), shared by the size query and the call.
struct FwdLayout {
  size_t q_hi = 0, q_lo = 0, k_hi = 0, k_lo = 0, v_hi = 0, v_lo = 0, p_hi = 0, p_lo = 0;
  size_t s_hi = 0, s_lo = 0;
  size_t part = 0;  // fp32 K-split partials of the score pass (0 when not split)
  bool chunked = false;
  bool one = false;  // bf16: P (and S) as one bf16 term, no lo buffers
  size_t total = 0;
};

FwdLayout fwd_layout(int dtype, int64_t B, int64_t H, int64_t Hv, int64_t T, int64_t N, int64_t D,
                     bool k_is_q) {
  FwdLayout L;
  size_t off = 0;
  const int e = esize(dtype);
  const bool chunked = use_chunked(dtype, T);
  const bool one = dtype == BDH_DTYPE_BF16 && bf16_one_term(/*split_by_default=*/!chunked);
  L.one = one;
  if (chunked) {
    L.chunked = true;
    const size_t pb = align_up(chunked_p_bytes(B, H, T));
    const size_t sb = align_up(chunked_s_bytes(B, H, T, N, D));
    L.p_hi = off; off += pb;
    L.p_lo = off; off += one ? 0 : pb;
    L.s_hi = off; off += sb;
    L.s_lo = off; off += one ? 0 : sb;
    L.total = off;
    return L;
  }
  if (dtype == BDH_DTYPE_F32) {
    const size_t qbytes = align_up(static_cast<size_t>(B * H * T * N) * 4);
    const size_t vbytes = align_up(static_cast<size_t>(B * Hv * D * vt_ld(T)) * 4);
    L.q_hi = off; off += qbytes;
    L.q_lo = off; off += qbytes;
    if (!k_is_q) {
      L.k_hi = off; off += qbytes;
      L.k_lo = off; off += qbytes;
    }
    L.v_hi = off; off += vbytes;
    L.v_lo = off; off += vbytes;
  }
  const size_t pbytes = align_up(static_cast<size_t>(B * H * T * score_ld(T)) * e);
  L.p_hi = off; off += pbytes;
  L.p_lo = off; off += one ? 0 : pbytes;
  if (dtype == BDH_DTYPE_F32) {
    const int ks = score_ksplit_f32(B * H, T, N);
    if (ks > 1) {
      L.part = off;
      off += align_up(static_cast<size_t>(ks) * static_cast<size_t>(B * H * T * score_ld(T)) * 4);
    }
  }
  L.total = off;
  return L;
}

// Workspace layout of the backward (byte offsets).
struct BwdLayout {
  size_t s1_hi = 0, s1_lo = 0, s2_hi = 0, s2_lo = 0;
  size_t do_hi = 0, do_lo = 0, v_hi = 0, v_lo = 0, q_hi = 0, q_lo = 0, k_hi = 0, k_lo = 0;
  size_t qt_hi = 0, qt_lo = 0, kt_hi = 0, kt_lo = 0, dot_hi = 0, dot_lo = 0;
  size_t total = 0;
};

BwdLayout bwd_layout(int dtype, int64_t B, int64_t H, int64_t Hv, int64_t T, int64_t N, int64_t D,
                     bool k_is_q) {
  BwdLayout L;
  size_t off = 0;
  const int e = esize(dtype);
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align_up(bytes);
    return o;
  };
  const size_t pbytes = static_cast<size_t>(B * H * T * score_ld(T)) * e;
  const size_t lobytes = dtype == BDH_DTYPE_BF16 && bf16_one_term(false) ? 0 : pbytes;
  L.s1_hi = take(pbytes);
  L.s1_lo = take(lobytes);
  if (!k_is_q) {
    L.s2_hi = take(pbytes);
    L.s2_lo = take(lobytes);
  }
  if (dtype == BDH_DTYPE_F32) {
    const int64_t ldt = vt_ld(T);
    const size_t dob = static_cast<size_t>(B * H * T * D) * 4;
    const size_t vb = static_cast<size_t>(B * Hv * T * D) * 4;
    const size_t qb = static_cast<size_t>(B * H * T * N) * 4;
    const size_t qtb = static_cast<size_t>(B * H * N * ldt) * 4;
    const size_t dotb = static_cast<size_t>(B * H * D * ldt) * 4;
    L.do_hi = take(dob); L.do_lo = take(dob);
    L.v_hi = take(vb); L.v_lo = take(vb);
    L.q_hi = take(qb); L.q_lo = take(qb);
    L.qt_hi = take(qtb); L.qt_lo = take(qtb);
    L.dot_hi = take(dotb); L.dot_lo = take(dotb);
    if (!k_is_q) {
      L.k_hi = take(qb); L.k_lo = take(qb);
      L.kt_hi = take(qtb); L.kt_lo = take(qtb);
    }
  }
  L.total = off;
  return L;
}

bool check_rows(const char* what, const int64_t s[4], int elem, std::string* msg) {
  if (s[3] != 1) {
    *msg = std::string(what) + ": the last dimension must be contiguous (stride 1)";
    return false;
  }
  return true;
}

bool strides_ok(const int64_t* s, int n) {
  if (s[n - 1] != 1) return false;
  for (int i = 0; i < n - 1; ++i)
    if (s[i] <= 0 || (s[i] % 8) != 0) return false;
  return true;
}
// (H, D, N) weights: n contiguous, or d contiguous (a transposed copy); other strides multiples of 8.
bool weight_strides_ok(const int64_t* s) {
  if (s[2] == 1) return strides_ok(s, 3);
  if (s[1] != 1) return false;
  return s[0] > 0 && s[0] % 8 == 0 && s[2] > 0 && s[2] % 8 == 0;
}
bool latent_sizes_ok(int64_t B, int64_t T, int64_t H, int64_t D, int64_t N, std::string* msg) {
  if (B < 0 || T < 0 || H < 0 || D < 0 || N < 0) {
    *msg = "negative size";
    return false;
  }
  if ((N % 2) != 0) {
    *msg = "latent width N must be even (RoPE pairs)";
    return false;
  }
  if (B * H * ((T + 127) / 128) * ((N + 127) / 128) >= (int64_t(1) << 31) || T >= (int64_t(1) << 24)) {
    *msg = "sizes beyond the supported range";
    return false;
  }
  return true;
}
}  // namespace

// Validated decode of the C entry points (bdh_tril_decode, bdh_tril_decode_noalloc); `qrot`
// (B*H*Tq*N fp32) receives the rotated queries when freqs is given, or is null to rotate them
// inside the decode kernel.
int decode_entry(const void* q, const int64_t q_strides[4], int q_dtype, const void* k_past,
                 const int64_t k_strides[4], const void* v_past, const int64_t v_strides[4],
                 int kv_dtype, void* out, const int64_t out_strides[4], int64_t B, int64_t H,
                 int64_t Hv, int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                 int64_t pos, void* kr_slot, const int64_t slot_strides[4], float* partial,
                 float* qrot, int64_t max_splits, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(kv_dtype)) return fail(BDH_ERR_INVALID, "tril_decode: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || Tq < 0 || S < 0 || N < 0 || D < 0) return fail(BDH_ERR_INVALID, "tril_decode: negative size");
  if (Hv != 1 && Hv != H) return fail(BDH_ERR_INVALID, "tril_decode: v_past heads must equal q heads or 1");
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || out_strides[3] != 1)
    return fail(BDH_ERR_INVALID, "tril_decode: last dimension must be contiguous");
  if (kr_slot != nullptr && (freqs == nullptr || slot_strides == nullptr || slot_strides[3] != 1))
    return fail(BDH_ERR_INVALID, "tril_decode: kr_slot needs freqs and contiguous slot rows");
  if (B * H * Tq == 0) return BDH_OK;
  if (S > (int64_t(1) << 30) || N > 48 * 1024) return fail(BDH_ERR_INVALID, "tril_decode: sizes beyond the supported range");
  if (freqs != nullptr && (N % 2) != 0) return fail(BDH_ERR_INVALID, "tril_decode: fused RoPE needs an even latent width");
  DecodeArgs a;
  a.q = q; a.q_dtype = q_dtype; a.k = k_past; a.v = v_past; a.kv_dtype = kv_dtype; a.out = out;
  std::memcpy(a.q_strides, q_strides, sizeof(a.q_strides));
  std::memcpy(a.k_strides, k_strides, sizeof(a.k_strides));
  std::memcpy(a.v_strides, v_strides, sizeof(a.v_strides));
  std::memcpy(a.out_strides, out_strides, sizeof(a.out_strides));
  a.B = B; a.H = H; a.Hv = Hv; a.Tq = Tq; a.S = S; a.N = N; a.D = D;
  a.freqs = freqs; a.pos = pos; a.slot = kr_slot;
  if (slot_strides != nullptr) std::memcpy(a.slot_strides, slot_strides, sizeof(a.slot_strides));
  return launch_decode(a, partial, qrot, max_splits, static_cast<cudaStream_t>(stream));
}
}  // namespace bdh

using namespace bdh;

extern "C" {

int bdh_abi_version(void) { return BDH_ABI_VERSION; }

const char* bdh_last_error(void) { return last_error(); }

int bdh_device_error(int device, int* code, int reset) {
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return fail(BDH_ERR_CUDA, "bdh_device_error: bad device");
  int* p = device_error_ptr();
  int v = 0;
  cudaError_t e = p ? cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) : cudaErrorInvalidSymbol;
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(BDH_ERR_CUDA, std::string("bdh_device_error: ") + cudaGetErrorString(e));
  if (code) *code = v;
  return BDH_OK;
}

int bdh_rope_rotate(const void* x, int x_dtype, const int64_t x_strides[4], void* y, int y_dtype,
                    const int64_t y_strides[4], void* y_lo, const float* freqs, int64_t B,
                    int64_t H, int64_t T, int64_t N, int64_t pos0, int flags, void* stream) {
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(BDH_ERR_INVALID, "rope: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || T < 0 || N < 0) return fail(BDH_ERR_INVALID, "rope: negative size");
  if (N % 2 != 0) return fail(BDH_ERR_INVALID, "rope: RoPE last dim must be even");
  if (x_strides[3] != 1 || y_strides[3] != 1) return fail(BDH_ERR_INVALID, "rope: last dim must be contiguous");
  if (y_lo != nullptr && y_dtype != BDH_DTYPE_F32) return fail(BDH_ERR_INVALID, "rope: y_lo requires f32 output");
  if (B * H * T * N > 0 && (x == nullptr || y == nullptr || freqs == nullptr))
    return fail(BDH_ERR_INVALID, "rope: null pointer");
  if ((flags & ~BDH_ROPE_RELU_INPUT) != 0) return fail(BDH_ERR_INVALID, "rope: unknown flags");
  return launch_rope(x, x_dtype, x_strides, y, y_dtype, y_strides, static_cast<float*>(y_lo), freqs,
                     B, H, T, N, pos0, (flags & BDH_ROPE_RELU_INPUT) ? 1 : 0,
                     static_cast<cudaStream_t>(stream));
}

int bdh_relu_mul(const void* x, const int64_t x_strides[4], const void* y,
                 const int64_t y_strides[4], void* out, const int64_t out_strides[4], int dtype,
                 int64_t B, int64_t H, int64_t T, int64_t N, void* stream) {
  if (!dtype_ok(dtype)) return fail(BDH_ERR_INVALID, "relu_mul: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || T < 0 || N < 0) return fail(BDH_ERR_INVALID, "relu_mul: negative size");
  if (x_strides[3] != 1 || y_strides[3] != 1 || out_strides[3] != 1)
    return fail(BDH_ERR_INVALID, "relu_mul: last dimension must be contiguous");
  return launch_relu_mul(x, x_strides, y, y_strides, out, out_strides, dtype, B, H, T, N,
                         static_cast<cudaStream_t>(stream));
}

int64_t bdh_decoder_f32_slices(int64_t K) { return K > 0 ? bdh::decoder_f32_slices(K) : 0; }

int bdh_decoder_f32(const float* x, int64_t ldx, const float* w, int64_t ldw, float* out,
                    int64_t ldo, float* partial, int64_t M, int64_t K, int64_t D, void* stream) {
  if (M < 0 || K < 0 || D < 0) return fail(BDH_ERR_INVALID, "decoder_f32: negative size");
  if (M == 0 || D == 0) return BDH_OK;
  if (M > 65535) return fail(BDH_ERR_INVALID, "decoder_f32: more than 65535 rows");
  if (D % 4 != 0 || ldw % 4 != 0 || ldw < D || ldo < D || (K > 0 && ldx < K))
    return fail(BDH_ERR_INVALID,
                "decoder_f32: D and ldw must be multiples of 4, and ldx >= K, ldw >= D, ldo >= D");
  if (out == nullptr || (K > 0 && (x == nullptr || w == nullptr || partial == nullptr)))
    return fail(BDH_ERR_INVALID, "decoder_f32: null pointer");
  if (K > 0 && ((reinterpret_cast<uintptr_t>(w) & 15u) != 0 ||
                (reinterpret_cast<uintptr_t>(partial) & 15u) != 0))
    return fail(BDH_ERR_INVALID, "decoder_f32: w and partial must be 16-byte aligned");
  return bdh::launch_decoder_f32(x, ldx, w, ldw, out, ldo, partial, M, K, D,
                                 static_cast<cudaStream_t>(stream));
}

int bdh_latent_encode(const void* x, const int64_t x_strides[3], const void* enc,
                      const int64_t enc_strides[3], void* xs, const int64_t xs_strides[4],
                      void* qr, const int64_t qr_strides[4], const float* freqs, int64_t B,
                      int64_t T, int64_t H, int64_t D, int64_t N, int64_t pos0, void* stream) {
  std::string msg;
  if (!latent_sizes_ok(B, T, H, D, N, &msg)) return fail(BDH_ERR_INVALID, "latent_encode: " + msg);
  if (B * T * H * N == 0) return BDH_OK;
  if (D == 0) return fail(BDH_ERR_INVALID, "latent_encode: D must be positive");
  if (!strides_ok(x_strides, 3) || !weight_strides_ok(enc_strides) ||
      (xs != nullptr && !strides_ok(xs_strides, 4)) || !strides_ok(qr_strides, 4))
    return fail(BDH_ERR_INVALID,
                "latent_encode: last stride must be 1 and the others positive multiples of 8");
  if (freqs == nullptr) return fail(BDH_ERR_INVALID, "latent_encode: freqs is null");
  if (pos0 < 0 || pos0 + T > (int64_t(1) << 24))
    return fail(BDH_ERR_INVALID, "latent_encode: positions beyond the supported range");
  LatentArgs a;
  a.x = x;
  std::memcpy(a.x_strides, x_strides, sizeof(a.x_strides));
  a.w = enc;
  std::memcpy(a.w_strides, enc_strides, sizeof(a.w_strides));
  a.xs = xs;
  if (xs != nullptr) std::memcpy(a.xs_strides, xs_strides, sizeof(a.xs_strides));
  a.qr = qr;
  std::memcpy(a.qr_strides, qr_strides, sizeof(a.qr_strides));
  a.freqs = freqs;
  a.B = B; a.T = T; a.H = H; a.D = D; a.N = N; a.pos0 = pos0;
  return launch_latent_encode(a, static_cast<cudaStream_t>(stream), device_error_ptr());
}

int bdh_latent_gate(const void* y, const int64_t y_strides[4], const void* encv,
                    const int64_t encv_strides[3], const void* xs, const int64_t xs_strides[4],
                    void* xy, const int64_t xy_strides[4], int64_t B, int64_t T, int64_t H,
                    int64_t D, int64_t N, void* stream) {
  std::string msg;
  if (!latent_sizes_ok(B, T, H, D, N, &msg)) return fail(BDH_ERR_INVALID, "latent_gate: " + msg);
  if (B * T * H * N == 0) return BDH_OK;
  if (D == 0) return fail(BDH_ERR_INVALID, "latent_gate: D must be positive");
  if (!strides_ok(y_strides, 4) || !weight_strides_ok(encv_strides) || !strides_ok(xs_strides, 4) ||
      !strides_ok(xy_strides, 4))
    return fail(BDH_ERR_INVALID,
                "latent_gate: last stride must be 1 and the others positive multiples of 8");
  LatentArgs a;
  a.y = y;
  std::memcpy(a.y_strides, y_strides, sizeof(a.y_strides));
  a.w = encv;
  std::memcpy(a.w_strides, encv_strides, sizeof(a.w_strides));
  a.xs = const_cast<void*>(xs);
  std::memcpy(a.xs_strides, xs_strides, sizeof(a.xs_strides));
  a.xy = xy;
  std::memcpy(a.xy_strides, xy_strides, sizeof(a.xy_strides));
  a.B = B; a.T = T; a.H = H; a.D = D; a.N = N;
  return launch_latent_gate(a, static_cast<cudaStream_t>(stream), device_error_ptr());
}

int bdh_latent_gate_x(const void* y, const int64_t y_strides[4], const void* encv,
                      const int64_t encv_strides[3], const void* x, const int64_t x_strides[3],
                      const void* enc, const int64_t enc_strides[3], void* xy,
                      const int64_t xy_strides[4], int64_t B, int64_t T, int64_t H, int64_t D,
                      int64_t N, void* stream) {
  std::string msg;
  if (!latent_sizes_ok(B, T, H, D, N, &msg)) return fail(BDH_ERR_INVALID, "latent_gate_x: " + msg);
  if (B * T * H * N == 0) return BDH_OK;
  if (D <= 0 || D > 256) return fail(BDH_ERR_INVALID, "latent_gate_x: D must be in 1..256");
  if (!strides_ok(y_strides, 4) || !weight_strides_ok(encv_strides) || !strides_ok(x_strides, 3) ||
      !weight_strides_ok(enc_strides) || !strides_ok(xy_strides, 4))
    return fail(BDH_ERR_INVALID,
                "latent_gate_x: last stride must be 1 and the others positive multiples of 8");
  LatentArgs a;
  a.y = y;
  std::memcpy(a.y_strides, y_strides, sizeof(a.y_strides));
  a.w = encv;
  std::memcpy(a.w_strides, encv_strides, sizeof(a.w_strides));
  a.x = x;
  std::memcpy(a.x_strides, x_strides, sizeof(a.x_strides));
  a.w2 = enc;
  std::memcpy(a.w2_strides, enc_strides, sizeof(a.w2_strides));
  a.xy = xy;
  std::memcpy(a.xy_strides, xy_strides, sizeof(a.xy_strides));
  a.B = B; a.T = T; a.H = H; a.D = D; a.N = N;
  return launch_latent_gate_x(a, static_cast<cudaStream_t>(stream), device_error_ptr());
}

size_t bdh_latent_gate_dec_workspace_size(int64_t B, int64_t T, int64_t H, int64_t D, int64_t N) {
  if (B < 0 || T < 0 || H < 0 || D < 0 || N < 0) return 0;
  return latent_gate_dec_workspace_bytes(B, T, H, D, N);
}

int bdh_latent_gate_dec_ws(const void* y, const int64_t y_strides[4], const void* encv,
                           const int64_t encv_strides[3], const void* xs, const int64_t xs_strides[4],
                           const void* dec, const int64_t dec_strides[2], void* out,
                           const int64_t out_strides[3], int64_t B, int64_t T, int64_t H, int64_t D,
                           int64_t N, void* workspace, size_t workspace_bytes, void* stream) {
  std::string msg;
  if (!latent_sizes_ok(B, T, H, D, N, &msg)) return fail(BDH_ERR_INVALID, "latent_gate_dec: " + msg);
  if (D != 256 || N % 128 != 0)
    return fail(BDH_ERR_INVALID, "latent_gate_dec: needs D = 256 and N a multiple of 128");
  if (B * T == 0) return BDH_OK;
  if (H == 0 || N == 0) return fail(BDH_ERR_INVALID, "latent_gate_dec: H and N must be positive");
  if (!strides_ok(y_strides, 4) || !strides_ok(xs_strides, 4) || !strides_ok(out_strides, 3))
    return fail(BDH_ERR_INVALID,
                "latent_gate_dec: last stride must be 1 and the others positive multiples of 8");
  if (!(encv_strides[1] == 1 && encv_strides[2] > 0 && encv_strides[2] % 8 == 0 &&
        encv_strides[0] > 0 && encv_strides[0] % 8 == 0))
    return fail(BDH_ERR_INVALID,
                "latent_gate_dec: encv must have d contiguous (a transposed (H,N,D) copy seen as (H,D,N))");
  if (!(dec_strides[0] == 1 && dec_strides[1] > 0 && dec_strides[1] % 8 == 0))
    return fail(BDH_ERR_INVALID,
                "latent_gate_dec: the decoder must have the latent index contiguous (a transposed "
                "(D, H*N) copy seen as (H*N, D))");
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return fail(BDH_ERR_INVALID, "latent_gate_dec: out must be 16-byte aligned");
  GateDecArgs a;
  a.y = y;
  std::memcpy(a.y_strides, y_strides, sizeof(a.y_strides));
  a.encv = encv;
  std::memcpy(a.encv_strides, encv_strides, sizeof(a.encv_strides));
  a.xs = xs;
  std::memcpy(a.xs_strides, xs_strides, sizeof(a.xs_strides));
  a.dec = dec;
  std::memcpy(a.dec_strides, dec_strides, sizeof(a.dec_strides));
  a.out = out;
  std::memcpy(a.out_strides, out_strides, sizeof(a.out_strides));
  a.B = B; a.T = T; a.H = H; a.D = D; a.N = N;
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return fail(BDH_ERR_INVALID, "latent_gate_dec: the workspace must be 16-byte aligned");
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  return launch_latent_gate_dec(a, static_cast<cudaStream_t>(stream), device_error_ptr());
}

int bdh_latent_gate_dec(const void* y, const int64_t y_strides[4], const void* encv,
                        const int64_t encv_strides[3], const void* xs, const int64_t xs_strides[4],
                        const void* dec, const int64_t dec_strides[2], void* out,
                        const int64_t out_strides[3], int64_t B, int64_t T, int64_t H, int64_t D,
                        int64_t N, void* stream) {
  return bdh_latent_gate_dec_ws(y, y_strides, encv, encv_strides, xs, xs_strides, dec, dec_strides,
                                out, out_strides, B, T, H, D, N, nullptr, 0, stream);
}

int bdh_quantize_rows_fp8(const void* x, const int64_t x_strides[4], int x_dtype, int64_t B,
                          int64_t H, int64_t T, int64_t N, void* out,
                          const int64_t out_strides[4], float* scale,
                          const int64_t scale_strides[3], void* stream) {
  if (!dtype_ok(x_dtype)) return fail(BDH_ERR_INVALID, "quantize_rows_fp8: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || T < 0 || N < 0) return fail(BDH_ERR_INVALID, "quantize_rows_fp8: negative size");
  if (N % 2 != 0) return fail(BDH_ERR_INVALID, "quantize_rows_fp8: N must be even");
  if (x_strides[3] != 1 || out_strides[3] != 1)
    return fail(BDH_ERR_INVALID, "quantize_rows_fp8: last dimension must be contiguous");
  if (B * H * T * N == 0) return BDH_OK;
  if (x == nullptr || out == nullptr || scale == nullptr)
    return fail(BDH_ERR_INVALID, "quantize_rows_fp8: null pointer");
  if (B * H * T >= (int64_t(1) << 31) || N > (int64_t(1) << 30))
    return fail(BDH_ERR_INVALID, "quantize_rows_fp8: sizes beyond the supported range");
  return launch_quantize_rows_fp8(x, x_dtype, x_strides, B, H, T, N, static_cast<uint8_t*>(out),
                                  out_strides, scale, scale_strides,
                                  static_cast<cudaStream_t>(stream));
}

int bdh_tril_decode_fp8(const void* q, const int64_t q_strides[4], int q_dtype,
                        const void* k_past, const int64_t k_strides[4], const float* k_scale,
                        const int64_t ks_strides[3], const void* v_past,
                        const int64_t v_strides[4], int v_dtype, void* out,
                        const int64_t out_strides[4], int64_t B, int64_t H, int64_t Hv,
                        int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                        int64_t pos, void* kr_slot, const int64_t slot_strides[4],
                        float* slot_scale, const int64_t slot_scale_strides[3],
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(v_dtype))
    return fail(BDH_ERR_INVALID, "tril_decode_fp8: q and v dtypes must be f32 or bf16");
  if (B < 0 || H < 0 || Tq < 0 || S < 0 || N < 0 || D < 0)
    return fail(BDH_ERR_INVALID, "tril_decode_fp8: negative size");
  if (Hv != 1 && Hv != H) return fail(BDH_ERR_INVALID, "tril_decode_fp8: v_past heads must equal q heads or 1");
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || out_strides[3] != 1)
    return fail(BDH_ERR_INVALID, "tril_decode_fp8: last dimension must be contiguous");
  if (kr_slot != nullptr && (freqs == nullptr || slot_strides == nullptr || slot_strides[3] != 1 ||
                             slot_scale == nullptr || slot_scale_strides == nullptr))
    return fail(BDH_ERR_INVALID, "tril_decode_fp8: kr_slot needs freqs, contiguous slot rows and a slot scale");
  if (S > 0 && (k_scale == nullptr || ks_strides == nullptr))
    return fail(BDH_ERR_INVALID, "tril_decode_fp8: k_scale is required");
  if (B * H * Tq == 0) return BDH_OK;
  if (S > (int64_t(1) << 30) || N > 48 * 1024) return fail(BDH_ERR_INVALID, "tril_decode_fp8: sizes beyond the supported range");
  if (freqs != nullptr && (N % 2) != 0) return fail(BDH_ERR_INVALID, "tril_decode_fp8: fused RoPE needs an even latent width");
  const size_t need = decode_workspace_bytes(B, H, Tq, S, N, D);
  if (workspace == nullptr || workspace_bytes < need) {
    std::ostringstream os;
    os << "tril_decode_fp8: workspace of " << need << " bytes required, got " << workspace_bytes;
    return fail(BDH_ERR_WORKSPACE, os.str());
  }
  DecodeFp8Args a;
  a.q = q; a.q_dtype = q_dtype; a.k = static_cast<const uint8_t*>(k_past); a.k_scale = k_scale;
  a.v = v_past; a.v_dtype = v_dtype; a.out = out;
  std::memcpy(a.q_strides, q_strides, sizeof(a.q_strides));
  std::memcpy(a.k_strides, k_strides, sizeof(a.k_strides));
  if (ks_strides != nullptr) std::memcpy(a.ks_strides, ks_strides, sizeof(a.ks_strides));
  std::memcpy(a.v_strides, v_strides, sizeof(a.v_strides));
  std::memcpy(a.out_strides, out_strides, sizeof(a.out_strides));
  a.B = B; a.H = H; a.Hv = Hv; a.Tq = Tq; a.S = S; a.N = N; a.D = D;
  a.freqs = freqs; a.pos = pos;
  a.slot = static_cast<uint8_t*>(kr_slot);
  if (slot_strides != nullptr) std::memcpy(a.slot_strides, slot_strides, sizeof(a.slot_strides));
  a.slot_scale = slot_scale;
  if (slot_scale_strides != nullptr)
    std::memcpy(a.slot_scale_strides, slot_scale_strides, sizeof(a.slot_scale_strides));
  float* partial = static_cast<float*>(workspace);
  float* qrot = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         decode_partial_bytes(B, H, Tq, S, N, D));
  return launch_decode_fp8(a, partial, qrot, static_cast<cudaStream_t>(stream));
}

int bdh_layernorm(const void* x, int x_dtype, int64_t x_row_stride, void* y, int y_dtype,
                  int64_t y_row_stride, int64_t rows, int64_t D, float eps, void* stream) {
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype))
    return fail(BDH_ERR_INVALID, "layernorm: dtype must be f32 or bf16");
  if (rows < 0 || D <= 0 || D > 1024 || (D % 8) != 0)
    return fail(BDH_ERR_INVALID, "layernorm: D must be a positive multiple of 8, at most 1024");
  if ((rows > 1 && (x_row_stride % 8 != 0 || y_row_stride % 8 != 0 || x_row_stride < D ||
                    y_row_stride < D)) ||
      (reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (reinterpret_cast<uintptr_t>(y) & 15u) != 0)
    return fail(BDH_ERR_INVALID, "layernorm: row strides must be multiples of 8 >= D, bases 16-byte aligned");
  if (!(eps >= 0.0f)) return fail(BDH_ERR_INVALID, "layernorm: eps must be >= 0");
  return launch_layernorm(x, x_dtype, x_row_stride, y, y_dtype, y_row_stride, rows,
                          static_cast<int>(D), eps, static_cast<cudaStream_t>(stream));
}

int bdh_residual_layernorm(const float* x, int64_t x_row_stride, const void* y, int y_dtype,
                           int64_t y_row_stride, float* out, int64_t out_row_stride,
                           void* out_bf16, int64_t out_bf16_row_stride, int64_t rows, int64_t D,
                           float eps, void* stream) {
  if (!dtype_ok(y_dtype)) return fail(BDH_ERR_INVALID, "residual_layernorm: dtype must be f32 or bf16");
  if (rows < 0 || D <= 0 || D > 1024 || (D % 8) != 0)
    return fail(BDH_ERR_INVALID, "residual_layernorm: D must be a positive multiple of 8, at most 1024");
  const bool strides =
      rows <= 1 || (x_row_stride % 8 == 0 && y_row_stride % 8 == 0 && out_row_stride % 8 == 0 &&
                    x_row_stride >= D && y_row_stride >= D && out_row_stride >= D &&
                    (out_bf16 == nullptr || (out_bf16_row_stride % 8 == 0 && out_bf16_row_stride >= D)));
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(out_bf16)) &
                        15u) == 0;
  if (!strides || !aligned)
    return fail(BDH_ERR_INVALID,
                "residual_layernorm: row strides must be multiples of 8 >= D, bases 16-byte aligned");
  if (!(eps >= 0.0f)) return fail(BDH_ERR_INVALID, "residual_layernorm: eps must be >= 0");
  return launch_residual_layernorm(x, x_row_stride, y, y_dtype, y_row_stride, out, out_row_stride,
                                   static_cast<uint16_t*>(out_bf16), out_bf16_row_stride, rows,
                                   static_cast<int>(D), eps, static_cast<cudaStream_t>(stream));
}

size_t bdh_tril_score_v_workspace_size(int dtype, int64_t B, int64_t H, int64_t Hv, int64_t T,
                                       int64_t N, int64_t D, int k_is_q) {
  if (!dtype_ok(dtype)) return 0;
  return fwd_layout(dtype, B, H, Hv, T, N, D, k_is_q != 0).total;
}

namespace {
// The forward; ln: each output row LayerNormed (eps) before the store (bdh_tril_score_v_layernorm).
int score_v_impl(const void* q, const int64_t q_strides[4], const void* k,
                 const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                 int dtype, void* out, const int64_t out_strides[4], int out_dtype,
                 int64_t B, int64_t H, int64_t Hv, int64_t T, int64_t N, int64_t D,
                 void* workspace, size_t workspace_bytes, void* stream, bool ln, float eps) {
  if (!dtype_ok(dtype) || !dtype_ok(out_dtype))
    return fail(BDH_ERR_INVALID, "tril_score_v: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || T < 0 || N < 0 || D < 0)
    return fail(BDH_ERR_INVALID, "tril_score_v: negative size");
  if (Hv != 1 && Hv != H) return fail(BDH_ERR_INVALID, "tril_score_v: v heads must equal q heads or 1");
  if (B * H * T * D == 0) return BDH_OK;
  if (N == 0) return fail(BDH_ERR_INVALID, "tril_score_v: latent width N must be positive");
  std::string msg;
  if (!check_rows("q", q_strides, esize(dtype), &msg) || !check_rows("k", k_strides, esize(dtype), &msg) ||
      !check_rows("v", v_strides, esize(dtype), &msg) ||
      !check_rows("out", out_strides, esize(out_dtype), &msg))
    return fail(BDH_ERR_INVALID, "tril_score_v: " + msg);
  if (T > (int64_t(1) << 24) || B * H > (int64_t(1) << 30))
    return fail(BDH_ERR_INVALID, "tril_score_v: sizes beyond the supported range");
  const bool k_is_q = (k == q) && std::memcmp(q_strides, k_strides, 4 * sizeof(int64_t)) == 0;
  const FwdLayout L = fwd_layout(dtype, B, H, Hv, T, N, D, k_is_q);
  if (workspace == nullptr || workspace_bytes < L.total) {
    std::ostringstream os;
    os << "tril_score_v: workspace of " << L.total << " bytes required, got " << workspace_bytes;
    return fail(BDH_ERR_WORKSPACE, os.str());
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = device_error_ptr();
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  FwdArgs a;
  a.dtype = dtype;
  a.out = out;
  a.out_dtype = out_dtype;
  std::memcpy(a.out_strides, out_strides, sizeof(a.out_strides));
  a.B = B; a.H = H; a.Hv = Hv; a.T = T; a.N = N; a.D = D;
  if (dtype == BDH_DTYPE_F32) {
    // fp32 operands become exact tf32 hi/lo pairs (contiguous) for the 3-product path.
    const int64_t qcs[4] = {H * T * N, T * N, N, 1};
    float* qh = reinterpret_cast<float*>(ws + L.q_hi);
    float* ql = reinterpret_cast<float*>(ws + L.q_lo);
    int rc = launch_split_tf32(static_cast<const float*>(q), q_strides, qh, ql, B, H, T, N, st);
    if (rc) return rc;
    a.q = qh; a.q_lo = ql;
    std::memcpy(a.q_strides, qcs, sizeof(qcs));
    if (k_is_q) {
      a.k = qh; a.k_lo = ql;
    } else {
      float* kh = reinterpret_cast<float*>(ws + L.k_hi);
      float* kl = reinterpret_cast<float*>(ws + L.k_lo);
      rc = launch_split_tf32(static_cast<const float*>(k), k_strides, kh, kl, B, H, T, N, st);
      if (rc) return rc;
      a.k = kh; a.k_lo = kl;
    }
    std::memcpy(a.k_strides, qcs, sizeof(qcs));
    float* vh = reinterpret_cast<float*>(ws + L.v_hi);
    float* vl = reinterpret_cast<float*>(ws + L.v_lo);
    // V is consumed transposed ([B*Hv][D][keys]) so that both tf32 operands are K-major.
    rc = launch_split_tf32_t(static_cast<const float*>(v), v_strides, vh, vl, B, Hv, T, D,
                             vt_ld(T), st);
    if (rc) return rc;
    a.v = vh; a.v_lo = vl;
  } else {
    a.q = q; a.k = k; a.v = v;
    std::memcpy(a.q_strides, q_strides, sizeof(a.q_strides));
    std::memcpy(a.k_strides, k_strides, sizeof(a.k_strides));
    std::memcpy(a.v_strides, v_strides, sizeof(a.v_strides));
  }
  void* p_lo = L.one ? nullptr : ws + L.p_lo;
  // the LayerNorm folds into the quadratic bf16 value pass; other forms normalise the output
  // rows in place afterwards (rows of one stride)
  const bool ln_fused = ln && !L.chunked && dtype == BDH_DTYPE_BF16 && D <= 256;
  const bool ln_after = ln && !ln_fused;
  if (ln_after) {
    const bool rows_flat = (H <= 1 || out_strides[1] == T * out_strides[2]) &&
                           (B <= 1 || out_strides[0] == H * T * out_strides[2]);
    if (!rows_flat || D > 1024 || D % 8 != 0 || (out_strides[2] % 8) != 0 ||
        (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
      return fail(BDH_ERR_INVALID,
                  "tril_score_v_layernorm: this form needs output rows of one stride (a multiple "
                  "of 8), D a multiple of 8 up to 1024 and a 16-byte aligned output");
  }
  a.ln = ln_fused ? 1 : 0;
  a.ln_eps = eps;
  int rc;
  if (L.chunked) {
    rc = launch_chunked_forward(a, ws + L.p_hi, p_lo, ws + L.s_hi,
                                L.one ? nullptr : ws + L.s_lo, st, err);
  } else {
    rc = launch_score(a, ws + L.p_hi, p_lo,
                      L.part ? reinterpret_cast<float*>(ws + L.part) : nullptr, st, err);
    if (!rc) rc = launch_value(a, ws + L.p_hi, p_lo, st, err);
  }
  if (rc || !ln_after) return rc;
  return launch_layernorm(out, out_dtype, out_strides[2], out, out_dtype, out_strides[2],
                          B * H * T, static_cast<int>(D), eps, st);
}
}  // namespace

int bdh_tril_score_v(const void* q, const int64_t q_strides[4], const void* k,
                     const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                     int dtype, void* out, const int64_t out_strides[4], int out_dtype,
                     int64_t B, int64_t H, int64_t Hv, int64_t T, int64_t N, int64_t D,
                     void* workspace, size_t workspace_bytes, void* stream) {
  return score_v_impl(q, q_strides, k, k_strides, v, v_strides, dtype, out, out_strides,
                      out_dtype, B, H, Hv, T, N, D, workspace, workspace_bytes, stream, false,
                      0.0f);
}

int bdh_tril_score_v_layernorm(const void* q, const int64_t q_strides[4], const void* k,
                               const int64_t k_strides[4], const void* v,
                               const int64_t v_strides[4], int dtype, void* out,
                               const int64_t out_strides[4], int out_dtype, int64_t B, int64_t H,
                               int64_t Hv, int64_t T, int64_t N, int64_t D, float eps,
                               void* workspace, size_t workspace_bytes, void* stream) {
  if (!(eps >= 0.0f)) return fail(BDH_ERR_INVALID, "tril_score_v_layernorm: eps must be >= 0");
  return score_v_impl(q, q_strides, k, k_strides, v, v_strides, dtype, out, out_strides,
                      out_dtype, B, H, Hv, T, N, D, workspace, workspace_bytes, stream, true, eps);
}

int bdh_set_forward_algo(int algo) {
  if (algo != BDH_FWD_AUTO && algo != BDH_FWD_QUADRATIC && algo != BDH_FWD_CHUNKED)
    return -1;
  return g_fwd_algo.exchange(algo);
}

int bdh_set_score_terms(int mode) {
  if (mode != BDH_SCORES_DEFAULT && mode != BDH_SCORES_ONE && mode != BDH_SCORES_SPLIT) return -2;
  const int prev = g_score_terms_thread;
  g_score_terms_thread = mode;
  return prev;
}

size_t bdh_tril_decode_workspace_size(int64_t B, int64_t H, int64_t Tq, int64_t S, int64_t N,
                                      int64_t D) {
  if (B < 0 || H < 0 || Tq < 0 || S < 0 || N < 0 || D < 0) return 0;
  return decode_workspace_bytes(B, H, Tq, S, N, D);
}

int bdh_tril_decode(const void* q, const int64_t q_strides[4], int q_dtype, const void* k_past,
                    const int64_t k_strides[4], const void* v_past, const int64_t v_strides[4],
                    int kv_dtype, void* out, const int64_t out_strides[4], int64_t B, int64_t H,
                    int64_t Hv, int64_t Tq, int64_t S, int64_t N, int64_t D, const float* freqs,
                    int64_t pos, void* kr_slot, const int64_t slot_strides[4], void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (B < 0 || H < 0 || Tq < 0 || S < 0 || N < 0 || D < 0)
    return fail(BDH_ERR_INVALID, "tril_decode: negative size");
  if (B * H * Tq == 0) return BDH_OK;
  const size_t need = decode_workspace_bytes(B, H, Tq, S, N, D);
  if (workspace == nullptr || workspace_bytes < need) {
    std::ostringstream os;
    os << "tril_decode: workspace of " << need << " bytes required, got " << workspace_bytes;
    return fail(BDH_ERR_WORKSPACE, os.str());
  }
  float* partial = static_cast<float*>(workspace);
  float* qrot = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         decode_partial_bytes(B, H, Tq, S, N, D));
  return decode_entry(q, q_strides, q_dtype, k_past, k_strides, v_past, v_strides, kv_dtype, out,
                      out_strides, B, H, Hv, Tq, S, N, D, freqs, pos, kr_slot, slot_strides, partial,
                      qrot, 0, stream);
}

size_t bdh_state_decode_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D) {
  if (B < 0 || H < 0 || N < 0 || D < 0) return 0;
  return state_decode_workspace_bytes(B, H, N, D);
}

int bdh_state_decode(const void* q, const int64_t q_strides[4], int q_dtype, float* state,
                     const int64_t state_strides[4], const void* v, const int64_t v_strides[4],
                     int v_dtype, void* out, const int64_t out_strides[4], int64_t B, int64_t H,
                     int64_t Hv, int64_t N, int64_t D, const float* freqs, int64_t pos,
                     int relu_input, void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(q_dtype) || !dtype_ok(v_dtype)) return fail(BDH_ERR_INVALID, "state_decode: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || N < 0 || D < 0) return fail(BDH_ERR_INVALID, "state_decode: negative size");
  if (Hv != 1 && Hv != H) return fail(BDH_ERR_INVALID, "state_decode: v heads must equal q heads or 1");
  if (B * H == 0 || D == 0) return BDH_OK;
  if (D != 128 && D != 256 && D != 512) return fail(BDH_ERR_INVALID, "state_decode: D must be 128, 256 or 512");
  if (N <= 0 || (N % 2) != 0 || N > (int64_t(1) << 24))
    return fail(BDH_ERR_INVALID, "state_decode: latent width N must be even and positive");
  if (freqs == nullptr) return fail(BDH_ERR_INVALID, "state_decode: freqs is required (the step rotates q)");
  if (q_strides[3] != 1 || v_strides[3] != 1 || out_strides[3] != 1 || state_strides[3] != 1)
    return fail(BDH_ERR_INVALID, "state_decode: last dimension must be contiguous");
  if ((reinterpret_cast<uintptr_t>(state) & 15u) != 0 || state_strides[0] % 4 != 0 ||
      state_strides[1] % 4 != 0 || state_strides[2] % 4 != 0)
    return fail(BDH_ERR_INVALID, "state_decode: state base and strides must be 16-byte aligned");
  if (pos < 0 || pos >= (int64_t(1) << 24)) return fail(BDH_ERR_INVALID, "state_decode: position out of range");
  const size_t need = state_decode_workspace_bytes(B, H, N, D);
  if (workspace == nullptr || workspace_bytes < need) {
    std::ostringstream os;
    os << "state_decode: workspace of " << need << " bytes required, got " << workspace_bytes;
    return fail(BDH_ERR_WORKSPACE, os.str());
  }
  StateDecodeArgs a;
  a.q = q; a.q_dtype = q_dtype; a.state = state; a.v = v; a.v_dtype = v_dtype; a.out = out;
  std::memcpy(a.q_strides, q_strides, sizeof(a.q_strides));
  std::memcpy(a.state_strides, state_strides, sizeof(a.state_strides));
  std::memcpy(a.v_strides, v_strides, sizeof(a.v_strides));
  std::memcpy(a.out_strides, out_strides, sizeof(a.out_strides));
  a.B = B; a.H = H; a.Hv = Hv; a.N = N; a.D = D; a.freqs = freqs; a.pos = pos;
  a.relu_input = relu_input ? 1 : 0;
  float* partial = static_cast<float*>(workspace);
  float* qrot = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         state_decode_partial_bytes(B, H, N, D));
  return launch_state_decode(a, partial, qrot, static_cast<cudaStream_t>(stream));
}

size_t bdh_tril_score_v_bwd_workspace_size(int dtype, int64_t B, int64_t H, int64_t Hv, int64_t T,
                                           int64_t N, int64_t D, int k_is_q) {
  if (!dtype_ok(dtype)) return 0;
  return bwd_layout(dtype, B, H, Hv, T, N, D, k_is_q != 0).total;
}

int bdh_tril_score_v_bwd(const void* q, const int64_t q_strides[4], const void* k,
                         const int64_t k_strides[4], const void* v, const int64_t v_strides[4],
                         const void* dout, const int64_t dout_strides[4], int dtype, void* dq,
                         const int64_t dq_strides[4], void* dk, const int64_t dk_strides[4],
                         void* dv, const int64_t dv_strides[4], int64_t B, int64_t H, int64_t Hv,
                         int64_t T, int64_t N, int64_t D, const float* freqs, int64_t pos0,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(dtype)) return fail(BDH_ERR_INVALID, "tril_score_v_bwd: dtype must be f32 or bf16");
  if (B < 0 || H < 0 || T < 0 || N < 0 || D < 0)
    return fail(BDH_ERR_INVALID, "tril_score_v_bwd: negative size");
  if (Hv != 1 && Hv != H) return fail(BDH_ERR_INVALID, "tril_score_v_bwd: v heads must equal q heads or 1");
  const bool k_is_q = (k == q) && std::memcmp(q_strides, k_strides, 4 * sizeof(int64_t)) == 0;
  if (!k_is_q && (dk == nullptr || dk_strides == nullptr))
    return fail(BDH_ERR_INVALID, "tril_score_v_bwd: dk is required when k is not q");
  if (freqs != nullptr && !k_is_q)
    return fail(BDH_ERR_INVALID, "tril_score_v_bwd: the fused RoPE adjoint needs k == q");
  if (freqs != nullptr && (N % 2) != 0)
    return fail(BDH_ERR_INVALID, "tril_score_v_bwd: RoPE last dim must be even");
  for (const int64_t* st : {q_strides, k_strides, v_strides, dout_strides, dq_strides, dv_strides})
    if (st[3] != 1) return fail(BDH_ERR_INVALID, "tril_score_v_bwd: last dimension must be contiguous");
  if (!k_is_q && dk_strides[3] != 1)
    return fail(BDH_ERR_INVALID, "tril_score_v_bwd: last dimension must be contiguous");
  if (T > (int64_t(1) << 24) || B * H > (int64_t(1) << 30))
    return fail(BDH_ERR_INVALID, "tril_score_v_bwd: sizes beyond the supported range");
  if (B * H * T == 0) return BDH_OK;
  const BwdLayout L = bwd_layout(dtype, B, H, Hv, T, N, D, k_is_q);
  if (workspace == nullptr || workspace_bytes < L.total) {
    std::ostringstream os;
    os << "tril_score_v_bwd: workspace of " << L.total << " bytes required, got " << workspace_bytes;
    return fail(BDH_ERR_WORKSPACE, os.str());
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* err = device_error_ptr();
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int elem = esize(dtype);
  const bool f32 = dtype == BDH_DTYPE_F32;
  int rc = 0;
  // Operands as the tensor-core passes consume them.
  const void* q_op[2] = {q, nullptr};
  const void* k_op[2] = {k, nullptr};
  const void* v_op[2] = {v, nullptr};
  const void* do_op[2] = {dout, nullptr};
  int64_t qs[4], ks[4], vs[4], dos[4];
  std::memcpy(qs, q_strides, sizeof(qs));
  std::memcpy(ks, k_strides, sizeof(ks));
  std::memcpy(vs, v_strides, sizeof(vs));
  std::memcpy(dos, dout_strides, sizeof(dos));
  const void* qT[2] = {q, nullptr};   // grad-q B operand for dS^T Q / G Q
  const void* kT[2] = {k, nullptr};   // grad-q B operand for dS K
  const void* doT[2] = {dout, nullptr};
  if (f32) {
    const int64_t ldt = vt_ld(T);
    auto split = [&](const void* x, const int64_t* xs, int64_t h, int64_t w, size_t hi_off,
                     size_t lo_off, const void** dst, int64_t* dst_strides) -> int {
      float* hi = reinterpret_cast<float*>(ws + hi_off);
      float* lo = reinterpret_cast<float*>(ws + lo_off);
      int r = launch_split_tf32(static_cast<const float*>(x), xs, hi, lo, B, h, T, w, st);
      dst[0] = hi;
      dst[1] = lo;
      const int64_t cs[4] = {h * T * w, T * w, w, 1};
      std::memcpy(dst_strides, cs, sizeof(cs));
      return r;
    };
    auto split_t = [&](const void* x, const int64_t* xs, int64_t h, int64_t w, size_t hi_off,
                       size_t lo_off, const void** dst) -> int {
      float* hi = reinterpret_cast<float*>(ws + hi_off);
      float* lo = reinterpret_cast<float*>(ws + lo_off);
      dst[0] = hi;
      dst[1] = lo;
      return launch_split_tf32_t(static_cast<const float*>(x), xs, hi, lo, B, h, T, w, ldt, st);
    };
    if ((rc = split(dout, dout_strides, H, D, L.do_hi, L.do_lo, do_op, dos))) return rc;
    if ((rc = split(v, v_strides, Hv, D, L.v_hi, L.v_lo, v_op, vs))) return rc;
    if ((rc = split(q, q_strides, H, N, L.q_hi, L.q_lo, q_op, qs))) return rc;
    if ((rc = split_t(q, q_strides, H, N, L.qt_hi, L.qt_lo, qT))) return rc;
    if ((rc = split_t(dout, dout_strides, H, D, L.dot_hi, L.dot_lo, doT))) return rc;
    if (k_is_q) {
      k_op[0] = q_op[0]; k_op[1] = q_op[1];
      std::memcpy(ks, qs, sizeof(ks));
    } else {
      if ((rc = split(k, k_strides, H, N, L.k_hi, L.k_lo, k_op, ks))) return rc;
      if ((rc = split_t(k, k_strides, H, N, L.kt_hi, L.kt_lo, kT))) return rc;
    }
  }
  const bool one = !f32 && bf16_one_term(false);
  void* g_hi = ws + L.s1_hi;
  void* g_lo = one ? nullptr : ws + L.s1_lo;
  void* g2_lo = one ? nullptr : ws + L.s2_lo;
  // 1. dS = tril(dO V^T, -1) -> G (K is Q) or L / U.
  ScoreArgs sa;
  sa.elem = elem;
  sa.a[0] = do_op[0]; sa.a[1] = do_op[1];
  sa.b[0] = v_op[0]; sa.b[1] = v_op[1];
  std::memcpy(sa.a_strides, dos, sizeof(dos));
  std::memcpy(sa.b_strides, vs, sizeof(vs));
  sa.B = B; sa.H = H; sa.Hb = Hv; sa.T = T; sa.K = D;
  sa.mode = k_is_q ? kStoreSym : kStoreLU;
  sa.p_hi = g_hi; sa.p_lo = g_lo;
  sa.p2_hi = ws + L.s2_hi; sa.p2_lo = g2_lo;
  if ((rc = launch_score_pass(sa, st, err))) return rc;
  // 2. dQ (and dK).
  GradQArgs ga;
  ga.elem = elem;
  ga.B = B; ga.H = H; ga.T = T; ga.N = N;
  ga.out_dtype = dtype;
  ga.g_hi = g_hi; ga.g_lo = g_lo;
  ga.out = dq;
  std::memcpy(ga.out_strides, dq_strides, sizeof(ga.out_strides));
  if (k_is_q) {
    ga.krange = 0;
    ga.x[0] = qT[0]; ga.x[1] = qT[1];
    std::memcpy(ga.x_strides, q_strides, sizeof(ga.x_strides));
    ga.freqs = freqs;
    ga.pos0 = pos0;
    if ((rc = launch_grad_q(ga, st, err))) return rc;
  } else {
    ga.krange = 1;
    ga.x[0] = kT[0]; ga.x[1] = kT[1];
    std::memcpy(ga.x_strides, k_strides, sizeof(ga.x_strides));
    if ((rc = launch_grad_q(ga, st, err))) return rc;
    ga.krange = 2;
    ga.g_hi = ws + L.s2_hi; ga.g_lo = g2_lo;
    ga.x[0] = qT[0]; ga.x[1] = qT[1];
    std::memcpy(ga.x_strides, q_strides, sizeof(ga.x_strides));
    ga.out = dk;
    std::memcpy(ga.out_strides, dk_strides, sizeof(ga.out_strides));
    if ((rc = launch_grad_q(ga, st, err))) return rc;
  }
  // 3. M^T = tril(Q K^T, -1)^T into the first score pair (its G / L contents are consumed).
  ScoreArgs sm;
  sm.elem = elem;
  sm.a[0] = q_op[0]; sm.a[1] = q_op[1];
  sm.b[0] = k_op[0]; sm.b[1] = k_op[1];
  std::memcpy(sm.a_strides, qs, sizeof(qs));
  std::memcpy(sm.b_strides, ks, sizeof(ks));
  sm.B = B; sm.H = H; sm.Hb = H; sm.T = T; sm.K = N;
  sm.mode = kStoreTrans;
  sm.p_hi = g_hi; sm.p_lo = g_lo;
  if ((rc = launch_score_pass(sm, st, err))) return rc;
  // 4. dV = sum_h M^T dO.
  GradVArgs va;
  va.elem = elem;
  va.mt_hi = g_hi; va.mt_lo = g_lo;
  va.dout[0] = doT[0]; va.dout[1] = doT[1];
  std::memcpy(va.do_strides, dout_strides, sizeof(va.do_strides));
  va.B = B; va.H = H; va.Hv = Hv; va.T = T; va.D = D;
  va.out = dv;
  std::memcpy(va.out_strides, dv_strides, sizeof(va.out_strides));
  va.out_dtype = dtype;
  return launch_grad_v(va, st, err);
}

}  // extern "C"

// bdh_sm100_ext: the reference's native attention module for the sm_100a library.
//
// The reference binds its CUDA / CPU kernels as the PyTorch extension `bdh_cuda_ext`
// (csrc/tril_attn_bind.cpp:25-40: tril_score_v(q, k, v), tril_decode(q, k_past, v_past),
// attribute has_cuda; declarations csrc/tril_attn.h:14-23) and kernels/cuda_attn.py calls it
// (:391-414, :490-502). This module exports the same names with the same arguments, results
// and error type (RuntimeError from TORCH_CHECK) on top of the C-ABI of libbdh_sm100.so
// (include/bdh_sm100.h), plus the ops of the fused path: the analytic backward, RoPE and the
// RoPE-fused forms of the forward and the decode step.
//
// Semantics kept from the reference module: inputs are borrowed (any strides with a contiguous
// last dimension; no .contiguous() copies of the operands), outputs are fresh tensors in q's
// dtype, the launch goes to the current CUDA stream of q's device with no host sync (so the ops
// can be captured in CUDA graphs). Differences on purpose: CUDA tensors only (no CPU path: a CPU
// tensor raises), fp32 and bf16 only, and scratch memory comes from the PyTorch caching
// allocator (the library itself never allocates).
#include <ATen/MemoryOverlap.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <cstdint>
#include <mutex>
#include <optional>
#include <string>
#include <tuple>
#include <vector>

#include "bdh_sm100.h"

namespace {

// Messages are put together as std::string: streaming integers through TORCH_CHECK's message
// builder crashed this build (torch 2.11 headers, the image's g++), strings do not.
void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, std::string("cuda_sm100 ") + what + " failed (code " + std::to_string(rc) +
                           "): " + bdh_last_error());
}

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kFloat) return BDH_DTYPE_F32;
  if (t.scalar_type() == at::kBFloat16) return BDH_DTYPE_BF16;
  TORCH_CHECK(false, std::string("cuda_sm100 supports float32 and bfloat16 tensors, got ") +
                         c10::toString(t.scalar_type()));
  return -1;
}

struct Strides4 {
  int64_t s[4];
  explicit Strides4(const at::Tensor& t) {
    for (int i = 0; i < 4; ++i) s[i] = t.stride(i);
  }
};

void require_cuda(std::initializer_list<const at::Tensor*> ts) {
  const at::Device dev = (*ts.begin())->device();
  for (const at::Tensor* t : ts) {
    TORCH_CHECK(t->is_cuda(), "cuda_sm100 requires CUDA tensors (no CPU fallback)");
    TORCH_CHECK(t->device() == dev, "cuda_sm100: all tensors must be on the same device");
  }
}

void* stream_of(const at::Tensor& t) {
  return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// The operand itself when TMA can read it in place (16-byte aligned base, 16-byte multiple
// strides, contiguous last dimension), else a contiguous copy zero-padded on the last dimension
// to a 16-byte multiple (zeros change no dot product over that dimension).
at::Tensor tma_ready(const at::Tensor& x) {
  const int64_t esz = x.element_size();
  bool ok = x.stride(-1) == 1 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0;
  for (int64_t d = 0; ok && d + 1 < x.dim(); ++d)
    if (x.size(d) > 1 && (x.stride(d) * esz) % 16 != 0) ok = false;
  if (ok) return x;
  const int64_t mult = 16 / esz;
  const int64_t n = x.size(-1);
  const int64_t npad = (n + mult - 1) / mult * mult;
  std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
  shape.back() = npad;
  at::Tensor y = at::zeros(shape, x.options());
  y.narrow(-1, 0, n).copy_(x);
  return y;
}

// "(d0, d1, ...)" of a tensor's shape, for error messages.
std::string shape_str(const at::Tensor& t) {
  std::string s = "(";
  for (int64_t d = 0; d < t.dim(); ++d) s += (d ? ", " : "") + std::to_string(t.size(d));
  return s + ")";
}

bool same_operand(const at::Tensor& a, const at::Tensor& b) {
  return a.data_ptr() == b.data_ptr() && a.sizes() == b.sizes() && a.strides() == b.strides() &&
         a.scalar_type() == b.scalar_type();
}

void check_cold_shapes(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "q, k, v must be 4D (B, H, T, D)");
  TORCH_CHECK(q.sizes() == k.sizes(), "q and k shapes must match, got ", shape_str(q), " vs ", shape_str(k));
  TORCH_CHECK(v.size(0) == q.size(0) && v.size(2) == q.size(2), "v batch/seq must match q");
  TORCH_CHECK(v.size(1) == 1 || v.size(1) == q.size(1), "v heads must equal q heads or 1");
  TORCH_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(),
              "cuda_sm100: q, k, v dtypes must match");
}

at::Tensor freqs_vector(const at::Tensor& freqs, int64_t n) {
  at::Tensor f = freqs.reshape({-1});
  TORCH_CHECK(f.scalar_type() == at::kFloat && f.numel() == n,
              "freqs must be float32 with one entry per latent dimension");
  return f.contiguous();
}

// ------------------------------------------------------------------------ forward
// ln_eps >= 0: each output row LayerNormed over D (bdh_tril_score_v_layernorm).
at::Tensor score_v(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double ln_eps) {
  check_cold_shapes(q, k, v);
  require_cuda({&q, &k, &v});
  const c10::cuda::CUDAGuard guard(q.device());
  const int dt = dtype_code(q);
  const int64_t B = q.size(0), H = q.size(1), T = q.size(2), Hv = v.size(1), D = v.size(3);
  at::Tensor out = at::empty({B, H, T, D}, q.options());
  if (out.numel() == 0) return out;
  const bool same = same_operand(q, k);
  at::Tensor qq = tma_ready(q);
  at::Tensor kk = same ? qq : tma_ready(k);
  at::Tensor vv = tma_ready(v);
  const int64_t Np = qq.size(3), Dp = vv.size(3);
  at::Tensor out_full = Dp != D ? at::empty({B, H, T, Dp}, q.options()) : out;
  const int k_is_q = same_operand(qq, kk) ? 1 : 0;
  const size_t wsz = bdh_tril_score_v_workspace_size(dt, B, H, Hv, T, Np, Dp, k_is_q);
  at::Tensor ws = at::empty({static_cast<int64_t>(std::max<size_t>(wsz, 1))},
                            q.options().dtype(at::kByte));
  const Strides4 sq(qq), sk(kk), sv(vv), so(out_full);
  if (ln_eps < 0) {
    check_rc(bdh_tril_score_v(qq.data_ptr(), sq.s, kk.data_ptr(), sk.s, vv.data_ptr(), sv.s, dt,
                              out_full.data_ptr(), so.s, dt, B, H, Hv, T, Np, Dp, ws.data_ptr(),
                              wsz, stream_of(q)),
             "tril_score_v");
  } else {
    TORCH_CHECK(Dp == D, "tril_score_v: the fused LayerNorm needs D a multiple of 16 bytes");
    check_rc(bdh_tril_score_v_layernorm(qq.data_ptr(), sq.s, kk.data_ptr(), sk.s, vv.data_ptr(),
                                        sv.s, dt, out_full.data_ptr(), so.s, dt, B, H, Hv, T, Np,
                                        Dp, static_cast<float>(ln_eps), ws.data_ptr(), wsz,
                                        stream_of(q)),
             "tril_score_v_layernorm");
  }
  if (Dp != D) out.copy_(out_full.narrow(3, 0, D));
  return out;
}

at::Tensor tril_score_v(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                        std::optional<double> ln_eps) {
  if (ln_eps.has_value()) TORCH_CHECK(*ln_eps >= 0.0, "ln_eps must be >= 0");
  return score_v(q, k, v, ln_eps.has_value() ? *ln_eps : -1.0);
}

// RoPE of x (B,H,T,N) at positions pos0 .. pos0 + T - 1 (phases from freqs in registers);
// relu_input rotates relu(x). out may be a strided view of another dtype (e.g. a cache slot).
at::Tensor rope_rotate(const at::Tensor& x_in, const at::Tensor& freqs, int64_t pos0,
                       std::optional<at::Tensor> out_opt, bool relu_input) {
  TORCH_CHECK(x_in.dim() == 4, "rope_rotate expects a 4-D (B, H, T, N) tensor");
  TORCH_CHECK(x_in.size(3) % 2 == 0, "RoPE last dim must be even, got " + std::to_string(x_in.size(3)));
  require_cuda({&x_in, &freqs});
  const c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor f = freqs_vector(freqs, x_in.size(3));
  at::Tensor out;
  if (out_opt.has_value()) {
    out = *out_opt;
    TORCH_CHECK(out.sizes() == x_in.sizes() && out.device() == x_in.device(),
                "rope out= must match x shape/device");
    const at::MemOverlapStatus ov = at::get_overlap_status(out, x_in);
    TORCH_CHECK(ov != at::MemOverlapStatus::Full && ov != at::MemOverlapStatus::Partial,
                "rope out= must not alias x");
    TORCH_CHECK(out.stride(3) == 1, "rope out= must have a contiguous last dimension");
  } else {
    out = at::empty(x_in.sizes(), x_in.options());
  }
  const at::Tensor x = x_in.stride(3) == 1 ? x_in : x_in.contiguous();
  if (x.numel() == 0) return out;
  const Strides4 sx(x), so(out);
  check_rc(bdh_rope_rotate(x.data_ptr(), dtype_code(x), sx.s, out.data_ptr(), dtype_code(out), so.s,
                           nullptr, f.data_ptr<float>(), x.size(0), x.size(1), x.size(2), x.size(3),
                           pos0, relu_input ? 1 : 0, stream_of(x)),
           "rope_rotate");
  return out;
}

// RoPE then the forward, as the attention module runs them (bdh.py:396-412 with the
// reference's RoPE, kernels/rope.py:108-126): QR = R(q) at positions rope_start.. (one pass),
// out = tril(QR QR^T, -1) v. Returns (out, QR); QR goes to qr_out when given (e.g. the cache
// slot of a prefill).
std::tuple<at::Tensor, at::Tensor> rope_tril_score_v(const at::Tensor& q, const at::Tensor& v,
                                                     const at::Tensor& freqs, int64_t rope_start,
                                                     std::optional<at::Tensor> qr_out) {
  at::Tensor qr = rope_rotate(q, freqs, rope_start, qr_out, false);
  at::Tensor qq = qr.scalar_type() == q.scalar_type() ? qr : qr.to(q.scalar_type());
  return {score_v(qq, qq, v, -1.0), qr};
}

// ------------------------------------------------------------------------- decode
at::Tensor decode_impl(const at::Tensor& q_in, const at::Tensor& k_past, const at::Tensor& v_past,
                       const at::Tensor* freqs, int64_t pos, std::optional<at::Tensor> kr_slot) {
  TORCH_CHECK(q_in.dim() == 4 && k_past.dim() == 4 && v_past.dim() == 4,
              "q, k_past, v_past must be 4D");
  const int64_t B = q_in.size(0), H = q_in.size(1), Tq = q_in.size(2), N = q_in.size(3);
  const int64_t S = k_past.size(2), Hv = v_past.size(1), D = v_past.size(3);
  TORCH_CHECK(k_past.size(0) == B && k_past.size(1) == H && k_past.size(3) == N,
              "k_past shape ", shape_str(k_past), " incompatible with q ", shape_str(q_in));
  TORCH_CHECK(v_past.size(0) == B && v_past.size(2) == S, "v_past shape ", shape_str(v_past),
              " incompatible with k_past S=" + std::to_string(S));
  TORCH_CHECK(Hv == 1 || Hv == H, "v_past heads must equal q heads or 1");
  require_cuda({&q_in, &k_past, &v_past});
  TORCH_CHECK(k_past.scalar_type() == v_past.scalar_type(),
              "k_past and v_past must share the cache storage dtype");
  const c10::cuda::CUDAGuard guard(q_in.device());
  const int qd = dtype_code(q_in), kd = dtype_code(k_past);
  at::Tensor out = at::empty({B, H, Tq, D}, q_in.options());
  if (out.numel() == 0) {
    if (kr_slot.has_value() && freqs != nullptr && Tq > 0) rope_rotate(q_in, *freqs, pos, kr_slot, false);
    return out;
  }
  const at::Tensor q = q_in.stride(3) == 1 ? q_in : q_in.contiguous();
  TORCH_CHECK(k_past.stride(3) == 1 && v_past.stride(3) == 1,
              "cache views must have a contiguous last dimension");
  at::Tensor f;
  const float* fptr = nullptr;
  if (freqs != nullptr) {
    f = freqs_vector(*freqs, N);
    fptr = f.data_ptr<float>();
  }
  void* slot_ptr = nullptr;
  int64_t slot_strides[4] = {0, 0, 0, 1};
  if (kr_slot.has_value()) {
    TORCH_CHECK(freqs != nullptr, "kr_slot requires freqs (the slot receives the rotated query)");
    const at::Tensor& s = *kr_slot;
    TORCH_CHECK(s.sizes() == q.sizes() && s.scalar_type() == k_past.scalar_type() && s.stride(3) == 1,
                "kr_slot must match q's shape, the cache dtype and have unit last stride");
    slot_ptr = s.data_ptr();
    for (int i = 0; i < 4; ++i) slot_strides[i] = s.stride(i);
  }
  const size_t wsz = bdh_tril_decode_workspace_size(B, H, Tq, S, N, D);
  at::Tensor ws = at::empty({static_cast<int64_t>(std::max<size_t>(wsz, 4))},
                            q.options().dtype(at::kByte));
  const Strides4 sq(q), sk(k_past), sv(v_past), so(out);
  check_rc(bdh_tril_decode(q.data_ptr(), sq.s, qd, k_past.data_ptr(), sk.s, v_past.data_ptr(), sv.s,
                           kd, out.data_ptr(), so.s, B, H, Hv, Tq, S, N, D, fptr, pos, slot_ptr,
                           slot_ptr != nullptr ? slot_strides : nullptr, ws.data_ptr(), wsz,
                           stream_of(q)),
           "tril_decode");
  return out;
}

// out = (q k_past^T) v_past over the packed past only (no self term); S = 0 gives zeros.
at::Tensor tril_decode(const at::Tensor& q, const at::Tensor& k_past, const at::Tensor& v_past) {
  return decode_impl(q, k_past, v_past, nullptr, 0, std::nullopt);
}

// The decode step with the new query rotated to positions pos.. inside the kernel and, with
// kr_slot, the rotated rows written there (the cache append of this step).
at::Tensor rope_tril_decode(const at::Tensor& q_new, const at::Tensor& freqs, int64_t pos,
                            const at::Tensor& kr_past, const at::Tensor& v_past,
                            std::optional<at::Tensor> kr_slot) {
  return decode_impl(q_new, kr_past, v_past, &freqs, pos, kr_slot);
}

// ----------------------------------------------------------------------- backward
// Analytic gradients of tril(q k^T, -1) v (kernels/attention_bwd.py:45-83): (dq, dk, dv).
// When k is q the returned dq holds dq + dk and dk is None (StrictTrilSelfAttnFn's form); with
// freqs (self form only) q is the rotated QR and dq is the gradient of the unrotated latent.
std::tuple<at::Tensor, std::optional<at::Tensor>, at::Tensor> tril_score_v_bwd(
    const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
    std::optional<at::Tensor> freqs, int64_t pos0) {
  check_cold_shapes(q, k, v);
  require_cuda({&q, &k, &v, &dout});
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t B = q.size(0), H = q.size(1), T = q.size(2), N = q.size(3);
  const int64_t Hv = v.size(1), D = v.size(3);
  TORCH_CHECK(dout.dim() == 4 && dout.size(0) == B && dout.size(1) == H && dout.size(2) == T &&
                  dout.size(3) == D,
              "dout shape " + shape_str(dout) + " must be (" + std::to_string(B) + ", " +
                  std::to_string(H) + ", " + std::to_string(T) + ", " + std::to_string(D) + ")");
  const int dt = dtype_code(q);
  const bool same = same_operand(q, k);
  TORCH_CHECK(!freqs.has_value() || same,
              "the fused RoPE adjoint needs the self-attention form (k is q)");
  at::Tensor qq = tma_ready(q);
  at::Tensor kk = same ? qq : tma_ready(k);
  at::Tensor vv = tma_ready(v);
  at::Tensor dd = tma_ready(dout.to(q.scalar_type()));
  const int64_t Np = qq.size(3), Dp = vv.size(3);
  if (dd.size(3) != Dp) dd = at::constant_pad_nd(dd, {0, Dp - dd.size(3)});
  at::Tensor dq = at::empty({B, H, T, Np}, q.options());
  std::optional<at::Tensor> dk;
  if (!same) dk = at::empty({B, H, T, Np}, q.options());
  at::Tensor dv = at::empty({B, Hv, T, Dp}, q.options());
  at::Tensor f;
  const float* fptr = nullptr;
  if (freqs.has_value()) {
    f = freqs_vector(*freqs, N);
    TORCH_CHECK(Np == N, "the fused RoPE adjoint needs an aligned latent width");
    fptr = f.data_ptr<float>();
  }
  const size_t wsz = bdh_tril_score_v_bwd_workspace_size(dt, B, H, Hv, T, Np, Dp, same ? 1 : 0);
  at::Tensor ws = at::empty({static_cast<int64_t>(std::max<size_t>(wsz, 1))},
                            q.options().dtype(at::kByte));
  const Strides4 sq(qq), sk(kk), sv(vv), sd(dd), sdq(dq), sdv(dv);
  const Strides4 sdk(dk.has_value() ? *dk : dq);
  if (B * H * T > 0)
    check_rc(bdh_tril_score_v_bwd(qq.data_ptr(), sq.s, kk.data_ptr(), sk.s, vv.data_ptr(), sv.s,
                                  dd.data_ptr(), sd.s, dt, dq.data_ptr(), sdq.s,
                                  dk.has_value() ? dk->data_ptr() : nullptr, sdk.s, dv.data_ptr(),
                                  sdv.s, B, H, Hv, T, Np, Dp, fptr, pos0, ws.data_ptr(), wsz,
                                  stream_of(q)),
             "tril_score_v_bwd");
  if (Np != N) {
    dq = dq.narrow(3, 0, N).contiguous();
    if (dk.has_value()) dk = dk->narrow(3, 0, N).contiguous();
  }
  if (Dp != D) dv = dv.narrow(3, 0, D).contiguous();
  return {dq, dk, dv};
}

// ------------------------------------------------------------ fused layer (model path)
// The same checks and C-ABI calls as kernels/sm100_attn.py's latent_encode, latent_gate_dec,
// layer_norm and residual_layer_norm (bf16 latents with a contiguous last dimension, 16-byte
// aligned bases, strides in multiples of 8 elements; weights d-contiguous or n-contiguous).
void check_latent(const char* name, std::initializer_list<const at::Tensor*> ts) {
  for (const at::Tensor* t : ts) {
    TORCH_CHECK(t->scalar_type() == at::kBFloat16,
                std::string(name) + ": bf16 tensors required, got " + c10::toString(t->scalar_type()));
    bool ok = t->stride(-1) == 1 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0;
    for (int64_t d = 0; ok && d + 1 < t->dim(); ++d)
      if (t->size(d) > 1 && t->stride(d) % 8 != 0) ok = false;
    TORCH_CHECK(ok, std::string(name) +
                        ": tensors need a contiguous last dim, 16-byte aligned base and strides "
                        "that are multiples of 8 elements");
  }
}

void check_weight(const char* name, const at::Tensor& w) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16,
              std::string(name) + ": bf16 weights required, got " + c10::toString(w.scalar_type()));
  const bool k_major = w.stride(1) == 1 && w.stride(2) != 1 && w.stride(0) % 8 == 0 && w.stride(2) % 8 == 0;
  if (!k_major) {
    check_latent(name, {&w});
  } else {
    TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
                std::string(name) + ": weights need a 16-byte aligned base");
  }
}

// Element strides for the C-ABI: a size-1 dimension is never stepped, so an odd stride there
// becomes a legal 8.
template <int R>
struct StridesN {
  int64_t s[R];
  explicit StridesN(const at::Tensor& t) {
    for (int i = 0; i < R; ++i) {
      const int64_t st = t.stride(i);
      s[i] = (t.size(i) > 1 || st % 8 == 0 || st == 1) ? st : 8;
    }
    s[R - 1] = t.stride(R - 1);
  }
};

// freqs[2p] == freqs[2p + 1] (BDH's get_freqs): the fused encode shares one (cos, sin) per
// pair. Checked once per freqs tensor version (the check reads the tensor back).
bool paired_freqs(const at::Tensor& f) {
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int64_t, int64_t, bool>> seen;
  const auto key = std::make_tuple(f.data_ptr(), static_cast<int64_t>(f._version()), f.numel());
  {
    std::lock_guard<std::mutex> g(mu);
    for (const auto& e : seen)
      if (std::get<0>(e) == std::get<0>(key) && std::get<1>(e) == std::get<1>(key) &&
          std::get<2>(e) == std::get<2>(key))
        return std::get<3>(e);
  }
  const bool ok = at::equal(f.slice(0, 0, f.numel(), 2), f.slice(0, 1, f.numel(), 2));
  std::lock_guard<std::mutex> g(mu);
  if (seen.size() > 64) seen.clear();
  seen.emplace_back(std::get<0>(key), std::get<1>(key), std::get<2>(key), ok);
  return ok;
}

// xs = relu(x enc) (B,T,H,N) and qr = RoPE(xs) (B,H,T,N) at positions pos0.., bf16.
std::tuple<std::optional<at::Tensor>, at::Tensor> latent_encode(
    const at::Tensor& x, const at::Tensor& enc, const at::Tensor& freqs, int64_t pos0,
    std::optional<at::Tensor> xs_out, std::optional<at::Tensor> qr_out, bool want_xs) {
  TORCH_CHECK(x.dim() == 3 && enc.dim() == 3 && x.size(2) == enc.size(1),
              "latent_encode expects x (B,T,D) and enc (H,D,N)");
  require_cuda({&x, &enc, &freqs});
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.size(0), T = x.size(1), D = x.size(2), H = enc.size(0), N = enc.size(2);
  const at::Tensor f = freqs_vector(freqs, N);
  TORCH_CHECK(paired_freqs(f), "latent_encode requires paired frequencies (freqs[2p] == freqs[2p+1])");
  std::optional<at::Tensor> xs = xs_out;
  if (!xs.has_value() && want_xs) xs = at::empty({B, T, H, N}, x.options().dtype(at::kBFloat16));
  at::Tensor qr = qr_out.has_value() ? *qr_out : at::empty({B, H, T, N}, x.options().dtype(at::kBFloat16));
  TORCH_CHECK((!xs.has_value() || xs->sizes() == at::IntArrayRef({B, T, H, N})) &&
                  qr.sizes() == at::IntArrayRef({B, H, T, N}),
              "latent_encode: xs_out must be (B,T,H,N) and qr_out (B,H,T,N)");
  if (xs.has_value())
    check_latent("latent_encode", {&x, &*xs, &qr});
  else
    check_latent("latent_encode", {&x, &qr});
  check_weight("latent_encode", enc);
  const StridesN<3> sx(x), se(enc);
  const StridesN<4> sq(qr);
  std::optional<StridesN<4>> sxs;
  if (xs.has_value()) sxs.emplace(*xs);
  check_rc(bdh_latent_encode(x.data_ptr(), sx.s, enc.data_ptr(), se.s,
                             xs.has_value() ? xs->data_ptr() : nullptr, sxs ? sxs->s : nullptr,
                             qr.data_ptr(), sq.s, f.data_ptr<float>(), B, T, H, D, N, pos0,
                             stream_of(x)),
           "latent_encode");
  return {xs, qr};
}

// (xs * relu(y encv)) dec in one kernel: y (B,H,T,D), encv (H,D,N) d-contiguous, xs (B,T,H,N),
// dec (H*N, D) latent-contiguous; D = 256, N a multiple of 128. Returns (B,T,D) bf16.
at::Tensor latent_gate_dec(const at::Tensor& y, const at::Tensor& encv, const at::Tensor& xs,
                           const at::Tensor& dec, std::optional<at::Tensor> out_opt) {
  TORCH_CHECK(y.dim() == 4 && encv.dim() == 3 && xs.dim() == 4 && dec.dim() == 2,
              "latent_gate_dec expects y (B,H,T,D), encv (H,D,N), xs (B,T,H,N), dec (H*N,D)");
  require_cuda({&y, &encv, &xs, &dec});
  const c10::cuda::CUDAGuard guard(y.device());
  const int64_t B = y.size(0), H = y.size(1), T = y.size(2), D = y.size(3), N = encv.size(2);
  TORCH_CHECK(xs.sizes() == at::IntArrayRef({B, T, H, N}) && encv.sizes() == at::IntArrayRef({H, D, N}) &&
                  dec.sizes() == at::IntArrayRef({H * N, D}),
              "latent_gate_dec: shapes of y, encv, xs and dec disagree");
  TORCH_CHECK(D == 256 && N % 128 == 0, "latent_gate_dec: needs D = 256 and N a multiple of 128");
  TORCH_CHECK(dec.scalar_type() == at::kBFloat16 && encv.scalar_type() == at::kBFloat16,
              "latent_gate_dec: bf16 weights required");
  at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({B, T, D}, y.options().dtype(at::kBFloat16));
  TORCH_CHECK(out.sizes() == at::IntArrayRef({B, T, D}), "latent_gate_dec: out must be (B,T,D)");
  check_latent("latent_gate_dec", {&y, &xs, &out});
  check_weight("latent_gate_dec", encv);
  const size_t wsz = bdh_latent_gate_dec_workspace_size(B, T, H, D, N);
  at::Tensor ws;
  if (wsz > 0) ws = at::empty({static_cast<int64_t>(wsz)}, y.options().dtype(at::kByte));
  const StridesN<4> sy(y), sxs(xs);
  const StridesN<3> sev(encv), so(out);
  const StridesN<2> sd(dec);
  check_rc(bdh_latent_gate_dec_ws(y.data_ptr(), sy.s, encv.data_ptr(), sev.s, xs.data_ptr(), sxs.s,
                                  dec.data_ptr(), sd.s, out.data_ptr(), so.s, B, T, H, D, N,
                                  wsz > 0 ? ws.data_ptr() : nullptr, wsz, stream_of(y)),
           "latent_gate_dec");
  return out;
}

// (rows, D) with one row stride for the LayerNorm entries: a view when the leading dimensions
// flatten to one, else nullopt.
std::optional<at::Tensor> rows_view(const at::Tensor& t) {
  if (t.stride(-1) != 1) return std::nullopt;
  try {
    return t.view({-1, t.size(-1)});
  } catch (const c10::Error&) {
    return std::nullopt;
  }
}

int64_t row_stride(const at::Tensor& v) { return v.size(0) > 1 ? v.stride(0) : v.size(1); }

// Affine-free LayerNorm over the last dim, fp32 math, stored in out_dtype (default x's dtype).
at::Tensor layer_norm(const at::Tensor& x, double eps, std::optional<at::ScalarType> out_dtype,
                      std::optional<at::Tensor> out_opt) {
  require_cuda({&x});
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t D = x.size(-1);
  std::optional<at::Tensor> xv = rows_view(x);
  if (!xv.has_value()) xv = x.contiguous().view({-1, D});
  at::Tensor out = out_opt.has_value() ? *out_opt
                                       : at::empty(x.sizes(), x.options().dtype(out_dtype.value_or(x.scalar_type())));
  std::optional<at::Tensor> ov = rows_view(out);
  TORCH_CHECK(ov.has_value() && ov->size(0) == xv->size(0),
              "layer_norm: out must be row-contiguous with x's shape");
  check_rc(bdh_layernorm(xv->data_ptr(), dtype_code(*xv), row_stride(*xv), ov->data_ptr(),
                         dtype_code(*ov), row_stride(*ov), xv->size(0), D, static_cast<float>(eps),
                         stream_of(x)),
           "layer_norm");
  return out;
}

// LN(x + LN(y)) over the last dim (BDH._residual_ln): x fp32, y fp32 or bf16. Returns the
// fp32 result and, with want_bf16, its bf16 copy.
std::tuple<at::Tensor, std::optional<at::Tensor>> residual_layer_norm(const at::Tensor& x,
                                                                      const at::Tensor& y,
                                                                      double eps, bool want_bf16) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.sizes() == y.sizes(),
              "residual_layer_norm: x must be fp32 and y of x's shape");
  require_cuda({&x, &y});
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t D = x.size(-1);
  std::optional<at::Tensor> xv = rows_view(x);
  if (!xv.has_value()) xv = x.contiguous().view({-1, D});
  std::optional<at::Tensor> yv = rows_view(y);
  if (!yv.has_value()) yv = y.contiguous().view({-1, D});
  at::Tensor out = at::empty(x.sizes(), x.options());
  std::optional<at::Tensor> out16;
  if (want_bf16) out16 = at::empty(x.sizes(), x.options().dtype(at::kBFloat16));
  check_rc(bdh_residual_layernorm(xv->data_ptr<float>(), row_stride(*xv), yv->data_ptr(),
                                  dtype_code(*yv), row_stride(*yv), out.data_ptr<float>(), D,
                                  out16.has_value() ? out16->data_ptr() : nullptr, D, xv->size(0), D,
                                  static_cast<float>(eps), stream_of(x)),
           "residual_layer_norm");
  return {out, out16};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "BDH strict lower-triangular score x V, decode and backward on sm_100a (no softmax)";
  m.def("tril_score_v", &tril_score_v,
        "out = tril(Q@K.T, diagonal=-1) @ V  (no softmax, no scale); with ln_eps each output row "
        "is LayerNormed over D before the store",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("ln_eps") = py::none());
  m.def("tril_decode", &tril_decode,
        "out = (Q @ K_past.T) @ V_past  (packed past; no self-attend)", py::arg("q"),
        py::arg("k_past"), py::arg("v_past"));
  m.def("tril_score_v_bwd", &tril_score_v_bwd,
        "(dq, dk, dv) of tril(Q@K.T, -1) @ V; dq = dq + dk and dk = None when k is q; with freqs "
        "q is the rotated QR and dq the gradient of the unrotated latent",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("dout"), py::arg("freqs") = py::none(),
        py::arg("pos0") = 0);
  m.def("rope_rotate", &rope_rotate, "BDH RoPE at positions pos0.. (phases in registers)",
        py::arg("x"), py::arg("freqs"), py::arg("pos0") = 0, py::arg("out") = py::none(),
        py::arg("relu_input") = false);
  m.def("rope_tril_score_v", &rope_tril_score_v,
        "(out, QR): QR = RoPE(q) at positions rope_start.., out = tril(QR@QR.T, -1) @ V",
        py::arg("q"), py::arg("v"), py::arg("freqs"), py::arg("rope_start") = 0,
        py::arg("qr_out") = py::none());
  m.def("rope_tril_decode", &rope_tril_decode,
        "decode step with the new query RoPE-rotated to positions pos.. (and written to kr_slot)",
        py::arg("q_new"), py::arg("freqs"), py::arg("pos"), py::arg("kr_past"), py::arg("v_past"),
        py::arg("kr_slot") = py::none());
  m.def("latent_encode", &latent_encode,
        "(xs, qr): xs = relu(x @ enc) (B,T,H,N), qr = RoPE(xs) (B,H,T,N) at positions pos0.., bf16",
        py::arg("x"), py::arg("enc"), py::arg("freqs"), py::arg("pos0") = 0,
        py::arg("xs_out") = py::none(), py::arg("qr_out") = py::none(), py::arg("want_xs") = true);
  m.def("latent_gate_dec", &latent_gate_dec, "(xs * relu(y @ encv)) @ dec in one kernel, (B,T,D) bf16",
        py::arg("y"), py::arg("encv"), py::arg("xs"), py::arg("dec"), py::arg("out") = py::none());
  m.def("layer_norm", &layer_norm, "affine-free LayerNorm over the last dim (fp32 math)",
        py::arg("x"), py::arg("eps") = 1e-5, py::arg("out_dtype") = py::none(),
        py::arg("out") = py::none());
  m.def("residual_layer_norm", &residual_layer_norm,
        "(LN(x + LN(y)), its bf16 copy or None): the BDH layer's residual double LayerNorm",
        py::arg("x"), py::arg("y"), py::arg("eps") = 1e-5, py::arg("want_bf16") = false);
  m.def("abi_version", &bdh_abi_version, "ABI version of the loaded libbdh_sm100.so");
  m.attr("has_cuda") = true;
}

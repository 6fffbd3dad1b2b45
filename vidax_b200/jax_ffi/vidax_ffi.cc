// vidax_ffi.cc -- XLA FFI handlers over the C ABI of libvidax_cuda.so, so
// that vidax's JAX code (jit / shard_map) calls the sm_100a kernels as XLA
// custom calls.
//
// Built by vidax_b200.jax_ffi.build() only where jaxlib's FFI headers exist
// (jax.ffi.include_dir()); registered with jax.ffi.register_ffi_target by
// vidax_b200.jax_ffi.register(). Each handler adapts XLA's row-major buffers
// to the library's strided arguments and maps VX_* return codes to
// ffi::Error codes (VX_EINVAL -> InvalidArgument, VX_EUNSUPPORTED ->
// Unimplemented, VX_ETIMEOUT -> DeadlineExceeded, else Internal).
//
// Handlers (the vidax function each one serves):
//   VidaxAttnFwd       dot_product_attention / local_attention
//                      (src/vidax/core/attention.py:321-338, 467-533)
//   VidaxNa3dFwd       neighborhood_attention_3d
//                      (src/vidax/models/ltx2_5/diffusion_vae.py:179-234)
//   VidaxUlyssesPack   the tokens->heads layout half of the tiled all_to_all
//   VidaxUlyssesUnpack the heads->tokens layout half
//                      (src/vidax/core/attention.py:379-381, 388)
#include <cstdint>

#include "vidax_cuda.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error to_error(int rc) {
  if (rc == VX_OK) return ffi::Error::Success();
  ffi::ErrorCode code = ffi::ErrorCode::kInternal;
  if (rc == VX_EINVAL) code = ffi::ErrorCode::kInvalidArgument;
  if (rc == VX_EUNSUPPORTED) code = ffi::ErrorCode::kUnimplemented;
  if (rc == VX_ETIMEOUT) code = ffi::ErrorCode::kDeadlineExceeded;
  return ffi::Error(code, vx_last_error());
}

// Row-major (B, S, H, D): element strides of (b, s, h).
void bshd_strides(int64_t S, int64_t H, int64_t D, int64_t (&st)[3]) {
  st[2] = D;
  st[1] = H * D;
  st[0] = S * H * D;
}

ffi::Error AttnImpl(cudaStream_t stream, ffi::Buffer<ffi::BF16> q, ffi::Buffer<ffi::BF16> k,
                    ffi::Buffer<ffi::BF16> v, ffi::ResultBuffer<ffi::BF16> o, float scale) {
  auto dq = q.dimensions();
  auto dk = k.dimensions();
  if (dq.size() != 4 || dk.size() != 4)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "q, k, v must be (B, S, H, D)");
  vx_attn_args a = {};
  a.q = q.untyped_data();
  a.k = k.untyped_data();
  a.v = v.untyped_data();
  a.o = o->untyped_data();
  bshd_strides(dq[1], dq[2], dq[3], a.q_stride);
  bshd_strides(dq[1], dq[2], dq[3], a.o_stride);
  bshd_strides(dk[1], dk[2], dk[3], a.k_stride);
  bshd_strides(dk[1], dk[2], dk[3], a.v_stride);
  a.batch = static_cast<int32_t>(dq[0]);
  a.seq_q = static_cast<int32_t>(dq[1]);
  a.seq_k = static_cast<int32_t>(dk[1]);
  a.heads_q = static_cast<int32_t>(dq[2]);
  a.heads_kv = static_cast<int32_t>(dk[2]);
  a.head_dim = static_cast<int32_t>(dq[3]);
  a.scale = scale;
  a.schedule = VX_SCHED_STATIC;
  return to_error(vx_attn_fwd(&a, reinterpret_cast<vx_stream_t>(stream)));
}

ffi::Error Na3dImpl(cudaStream_t stream, ffi::Buffer<ffi::BF16> q, ffi::Buffer<ffi::BF16> k,
                    ffi::Buffer<ffi::BF16> v, ffi::ResultBuffer<ffi::BF16> o, int32_t kt,
                    int32_t kh, int32_t kw, int32_t round_logits) {
  auto d = q.dimensions();  // (B, T, H, W, NH, HD)
  if (d.size() != 6 || k.dimensions().size() != 6)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "q, k, v must be (B, T, H, W, NH, HD)");
  vx_na3d_args a = {};
  a.q = q.untyped_data();
  a.k = k.untyped_data();
  a.v = v.untyped_data();
  a.o = o->untyped_data();
  a.batch = static_cast<int32_t>(d[0]);
  a.T = static_cast<int32_t>(d[1]);
  a.H = static_cast<int32_t>(d[2]);
  a.W = static_cast<int32_t>(d[3]);
  a.heads = static_cast<int32_t>(d[4]);
  a.head_dim = static_cast<int32_t>(d[5]);
  a.heads_kv = static_cast<int32_t>(k.dimensions()[4]);
  auto strides = [&](int64_t nh, int64_t (&s)[5]) {  // (b, t, h, w, head)
    s[4] = d[5];
    s[3] = nh * d[5];
    s[2] = d[3] * s[3];
    s[1] = d[2] * s[2];
    s[0] = d[1] * s[1];
  };
  strides(a.heads, a.q_stride);
  strides(a.heads, a.o_stride);
  strides(a.heads_kv, a.k_stride);
  strides(a.heads_kv, a.v_stride);
  a.kernel_t = kt;
  a.kernel_h = kh;
  a.kernel_w = kw;
  a.scale = 1.0f;  // vidax pre-scales q (diffusion_vae.py:265)
  a.round_logits = round_logits;
  return to_error(vx_na3d_fwd(&a, reinterpret_cast<vx_stream_t>(stream)));
}

// x (S_loc, H, D) <-> packed (groups, S_loc, ceil(H / groups), D).
ffi::Error SlabImpl(bool pack, cudaStream_t stream, ffi::Buffer<ffi::BF16> in,
                    ffi::ResultBuffer<ffi::BF16> out, int32_t groups, int32_t heads) {
  auto di = in.dimensions();
  auto dd = out->dimensions();
  const auto& strided = pack ? di : dd;
  if (di.size() != (pack ? 3u : 4u) || dd.size() != (pack ? 4u : 3u))
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "strided side (S, H, D), packed side (P, S, Hg, D)");
  vx_head_slab_args a = {};
  a.num_tensors = 1;
  a.src[0] = in.untyped_data();
  a.dst[0] = out->untyped_data();
  a.stride[0][0] = strided[1] * strided[2];
  a.stride[0][1] = strided[2];
  a.seq = static_cast<int32_t>(strided[0]);
  a.heads = heads;
  a.head_dim = static_cast<int32_t>(strided[2]);
  a.groups = groups;
  const vx_stream_t s = reinterpret_cast<vx_stream_t>(stream);
  return to_error(pack ? vx_ulysses_pack(&a, s) : vx_ulysses_unpack(&a, s));
}

ffi::Error PackImpl(cudaStream_t stream, ffi::Buffer<ffi::BF16> in, ffi::ResultBuffer<ffi::BF16> out,
                    int32_t groups, int32_t heads) {
  return SlabImpl(true, stream, in, out, groups, heads);
}
ffi::Error UnpackImpl(cudaStream_t stream, ffi::Buffer<ffi::BF16> in,
                      ffi::ResultBuffer<ffi::BF16> out, int32_t groups, int32_t heads) {
  return SlabImpl(false, stream, in, out, groups, heads);
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(VidaxAttnFwd, AttnImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Attr<float>("scale"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(VidaxNa3dFwd, Na3dImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Attr<int32_t>("kt")
                                  .Attr<int32_t>("kh")
                                  .Attr<int32_t>("kw")
                                  .Attr<int32_t>("round_logits"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(VidaxUlyssesPack, PackImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Attr<int32_t>("groups")
                                  .Attr<int32_t>("heads"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(VidaxUlyssesUnpack, UnpackImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Attr<int32_t>("groups")
                                  .Attr<int32_t>("heads"));
